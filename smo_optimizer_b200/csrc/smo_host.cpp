// smo_host.cpp -- the per-step host work of SMO8bit.step() / SMO.step() in C++.
//
// The Python optimizer builds a step plan once its state exists (after the
// first step of a parameter set): one entry per parameter with the finished
// smo_tensor descriptor for each moment-buffer parity.  Every later step is
// one call, plan_step(), which
//   1. checks that nothing the plan relies on has changed: the param groups
//      and their parameter lists (identity), each parameter's data pointer
//      and layout, its gradient (defined, strided, same dtype and device, the
//      layout the descriptor assumes), the state's moment tensors (one of the two buffer
//      sets), its integer "step", and no change to the optimizer's state
//      mapping (a dict watcher);
//   2. increments each state's "step", writes the gradient pointer and the
//      step's fp32 scalars into the descriptor table, and calls smo_step()
//      on the parameters' device and its current CUDA stream;
//   3. points the state at the buffers the step wrote (the double-buffered
//      pooled kinds), as the Python path does.
// When a check fails nothing has been modified and plan_step() returns -1;
// the Python path then steps and builds a new plan.  A positive return is an
// smo_status from smo_step().
//
// The scalars follow the reference's Python expressions (spatial_8bit.py:
// 210-297, the same as _host.step_scalars): formed in double, rounded once.

#include <Python.h>

#include <climits>
#include <cmath>
#include <cstring>
#include <vector>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>

#include "smo_b200.h"

namespace {

using StepFn = int (*)(const smo_tensor *, int32_t, void *, size_t, void *);

PyObject *s_params, *s_step, *s_lr, *s_betas, *s_eps, *s_weight_decay;
int g_watcher = -1;
unsigned long long g_state_generation = 0;  // bumped on any change to a watched state mapping

int on_state_change(PyDict_WatchEvent, PyObject *, PyObject *, PyObject *) {
    g_state_generation++;
    return 0;
}

struct Entry {
    PyObject *param = nullptr;  // owned
    PyObject *state = nullptr;  // owned; null: the parameter had no gradient when the plan was made
    int group = 0;
    int nkeys = 0;              // moment keys checked each step
    bool swap = false;          // double-buffered: the state moves to the other set after a step
    PyObject *keys[4] = {};     // owned
    PyObject *set[2][4] = {};   // owned: buffer set 0 (the state's at plan time) and set 1
    smo_tensor row[2];          // descriptor while the state holds set 0 / set 1
    void *param_ptr = nullptr;
    std::vector<int64_t> sizes, strides;  // the parameter's layout the rows were made for
    bool dense = false;         // gradient must have the parameter's sizes and strides (else contiguous)
};

struct Group {
    PyObject *dict = nullptr;    // owned
    PyObject *params = nullptr;  // owned
    Py_ssize_t n = 0;
};

struct Plan {
    PyObject *groups_list = nullptr;  // owned: the optimizer's param_groups
    std::vector<Group> groups;
    std::vector<Entry> entries;
    int device = 0;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    StepFn step_fn = nullptr;
    unsigned long long generation = 0;
    // per step
    std::vector<smo_tensor> table;
    std::vector<void *> grad_ptr;
    std::vector<int> parity;
    std::vector<long long> next_step;
    std::vector<double> hp_in;  // per group: lr, beta1, beta2, eps, weight_decay

    ~Plan() {
        for (Entry &e : entries) {
            Py_XDECREF(e.param);
            Py_XDECREF(e.state);
            for (int k = 0; k < 4; k++) {
                Py_XDECREF(e.keys[k]);
                Py_XDECREF(e.set[0][k]);
                Py_XDECREF(e.set[1][k]);
            }
        }
        for (Group &g : groups) {
            Py_XDECREF(g.dict);
            Py_XDECREF(g.params);
        }
        Py_XDECREF(groups_list);
    }
};

smo_hyper make_hyper(const double *in, long long step) {
    const double lr = in[0], b1 = in[1], b2 = in[2], eps = in[3], wd = in[4];
    const double bc1 = 1.0 - std::pow(b1, (double)step);
    const double bc2 = 1.0 - std::pow(b2, (double)step);
    const double step_size = lr / bc1;
    smo_hyper h;
    std::memset(&h, 0, sizeof(h));
    h.beta1 = (float)b1;
    h.omb1 = (float)(1.0 - b1);
    h.beta2 = (float)b2;
    h.omb2 = (float)(1.0 - b2);
    h.weight_decay = (float)wd;
    h.wd_on = wd != 0.0;
    h.neg_step = (float)(-step_size);
    h.sqrt_bc2 = (float)std::sqrt(bc2);
    h.eps = (float)eps;
    return h;
}

// a group's lr, betas, eps and weight_decay as doubles (false: not numbers)
bool read_group(PyObject *g, double *out) {
    PyObject *lr = PyDict_GetItemWithError(g, s_lr);
    PyObject *betas = PyDict_GetItemWithError(g, s_betas);
    PyObject *eps = PyDict_GetItemWithError(g, s_eps);
    PyObject *wd = PyDict_GetItemWithError(g, s_weight_decay);
    if (!lr || !betas || !eps || !wd) return false;
    PyObject *b0, *b1;
    if (PyTuple_Check(betas) && PyTuple_GET_SIZE(betas) == 2) {
        b0 = PyTuple_GET_ITEM(betas, 0);
        b1 = PyTuple_GET_ITEM(betas, 1);
    } else if (PyList_Check(betas) && PyList_GET_SIZE(betas) == 2) {
        b0 = PyList_GET_ITEM(betas, 0);
        b1 = PyList_GET_ITEM(betas, 1);
    } else {
        return false;
    }
    // plain numbers only (a tensor-valued hyperparameter takes the Python path)
    if (!PyFloat_Check(lr) && !PyLong_Check(lr)) return false;
    if (!PyFloat_Check(b0) && !PyLong_Check(b0)) return false;
    if (!PyFloat_Check(b1) && !PyLong_Check(b1)) return false;
    if (!PyFloat_Check(eps) && !PyLong_Check(eps)) return false;
    if (!PyFloat_Check(wd) && !PyLong_Check(wd)) return false;
    out[0] = PyFloat_AsDouble(lr);
    out[1] = PyFloat_AsDouble(b0);
    out[2] = PyFloat_AsDouble(b1);
    out[3] = PyFloat_AsDouble(eps);
    out[4] = PyFloat_AsDouble(wd);
    return !PyErr_Occurred();
}

// -1: the plan does not apply (nothing modified); 0: stepped; > 0: smo_status
int run_plan(Plan &pl) {
    // the param groups and their parameter lists
    if (pl.generation != g_state_generation) return -1;
    if (!PyList_CheckExact(pl.groups_list) || PyList_GET_SIZE(pl.groups_list) != (Py_ssize_t)pl.groups.size())
        return -1;
    size_t k = 0;
    for (size_t gi = 0; gi < pl.groups.size(); gi++) {
        const Group &g = pl.groups[gi];
        if (PyList_GET_ITEM(pl.groups_list, gi) != g.dict) return -1;
        PyObject *ps = PyDict_GetItemWithError(g.dict, s_params);
        if (ps != g.params || !PyList_CheckExact(ps) || PyList_GET_SIZE(ps) != g.n) return -1;
        for (Py_ssize_t j = 0; j < g.n; j++, k++)
            if (PyList_GET_ITEM(ps, j) != pl.entries[k].param) return -1;
        if (!read_group(g.dict, &pl.hp_in[5 * gi])) {
            PyErr_Clear();
            return -1;
        }
    }
    // pass 1: every check, no modification
    const size_t n = pl.entries.size();
    for (size_t i = 0; i < n; i++) {
        const Entry &e = pl.entries[i];
        if (!THPVariable_Check(e.param)) return -1;
        const at::Tensor &pt = THPVariable_Unpack(e.param);
        const at::Tensor &g = pt.grad();
        if (!e.state) {
            if (g.defined()) return -1;
            continue;
        }
        if (!g.defined() || pt.data_ptr() != e.param_ptr) return -1;
        if (pt.sizes() != c10::IntArrayRef(e.sizes) || pt.strides() != c10::IntArrayRef(e.strides)) return -1;
        if (g.layout() != c10::kStrided || g.scalar_type() != pt.scalar_type() || g.device() != pt.device())
            return -1;
        if (g.sizes() != pt.sizes()) return -1;
        if (e.dense ? g.strides() != pt.strides() : !g.is_contiguous()) return -1;
        PyObject *cur = PyDict_GetItemWithError(e.state, e.keys[0]);
        const int par = cur == e.set[0][0] ? 0 : (cur == e.set[1][0] ? 1 : -1);
        if (par < 0) return -1;
        for (int q = 1; q < e.nkeys; q++)
            if (PyDict_GetItemWithError(e.state, e.keys[q]) != e.set[par][q]) return -1;
        PyObject *st = PyDict_GetItemWithError(e.state, s_step);
        if (!st || !PyLong_CheckExact(st)) return -1;
        int overflow = 0;
        const long long s = PyLong_AsLongLongAndOverflow(st, &overflow);
        if (overflow || s < 0 || s == LLONG_MAX || PyErr_Occurred()) {
            PyErr_Clear();
            return -1;
        }
        pl.grad_ptr[i] = g.data_ptr();
        pl.parity[i] = par;
        pl.next_step[i] = s + 1;
    }
    if (PyErr_Occurred()) {
        PyErr_Clear();
        return -1;
    }
    // pass 2: step counters and the descriptor table
    size_t m = 0;
    int last_group = -1;
    long long last_step = -1;
    smo_hyper hp{};
    for (size_t i = 0; i < n; i++) {
        const Entry &e = pl.entries[i];
        if (!e.state) continue;
        PyObject *ns = PyLong_FromLongLong(pl.next_step[i]);
        if (!ns || PyDict_SetItem(e.state, s_step, ns) < 0) {
            Py_XDECREF(ns);
            return -2;  // a Python error is set
        }
        Py_DECREF(ns);
        smo_tensor &r = pl.table[m++];
        r = e.row[pl.parity[i]];
        r.grad = (const float *)pl.grad_ptr[i];
        if (e.group != last_group || pl.next_step[i] != last_step) {
            hp = make_hyper(&pl.hp_in[5 * e.group], pl.next_step[i]);
            last_group = e.group;
            last_step = pl.next_step[i];
        }
        r.hp = hp;
    }
    int rc;
    {
        c10::cuda::CUDAGuard guard((c10::DeviceIndex)pl.device);
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream((c10::DeviceIndex)pl.device).stream();
        rc = pl.step_fn(pl.table.data(), (int32_t)m, pl.ws, pl.ws_bytes, (void *)stream);
    }
    if (rc != SMO_OK) return rc;
    // pass 3: the state now holds the buffers this step wrote
    for (size_t i = 0; i < n; i++) {
        const Entry &e = pl.entries[i];
        if (!e.state || !e.swap) continue;
        const int other = 1 - pl.parity[i];
        for (int q = 0; q < e.nkeys; q++)
            if (PyDict_SetItem(e.state, e.keys[q], e.set[other][q]) < 0) return -2;
    }
    return 0;
}

void plan_free(PyObject *cap) {
    delete (Plan *)PyCapsule_GetPointer(cap, "smo_plan");
}

bool fill_row(PyObject *bytes, smo_tensor &row) {
    if (!PyBytes_Check(bytes) || PyBytes_GET_SIZE(bytes) != (Py_ssize_t)sizeof(smo_tensor)) {
        PyErr_SetString(PyExc_ValueError, "descriptor rows must be sizeof(smo_tensor) bytes");
        return false;
    }
    std::memcpy(&row, PyBytes_AS_STRING(bytes), sizeof(smo_tensor));
    return true;
}

// plan_new(param_groups, state_mapping, entries, device, ws_ptr, ws_bytes, step_fn_addr) -> capsule
// entries: one per parameter of every group, in group order:
//   (param, None)                                     no gradient at plan time
//   (param, state, group, swap, keys, set0, set1, row0, row1, dense)
PyObject *plan_new(PyObject *, PyObject *args) {
    PyObject *groups_list, *state_map, *entries;
    int device;
    unsigned long long ws_ptr, ws_bytes, fn;
    if (!PyArg_ParseTuple(args, "O!O!O!iKKK", &PyList_Type, &groups_list, &PyDict_Type, &state_map, &PyList_Type,
                          &entries, &device, &ws_ptr, &ws_bytes, &fn))
        return nullptr;
    if (g_watcher < 0) {
        PyErr_SetString(PyExc_RuntimeError, "no dict watcher available");
        return nullptr;
    }
    Plan *pl = new Plan();
    PyObject *cap = PyCapsule_New(pl, "smo_plan", plan_free);
    if (!cap) {
        delete pl;
        return nullptr;
    }
    Py_INCREF(groups_list);
    pl->groups_list = groups_list;
    pl->device = device;
    pl->ws = (void *)(uintptr_t)ws_ptr;
    pl->ws_bytes = (size_t)ws_bytes;
    pl->step_fn = (StepFn)(uintptr_t)fn;
    const Py_ssize_t ng = PyList_GET_SIZE(groups_list);
    pl->groups.resize(ng);
    Py_ssize_t total = 0;
    for (Py_ssize_t gi = 0; gi < ng; gi++) {
        Group &g = pl->groups[gi];
        g.dict = PyList_GET_ITEM(groups_list, gi);
        Py_INCREF(g.dict);
        if (!PyDict_Check(g.dict)) goto bad_structure;
        g.params = PyDict_GetItemWithError(g.dict, s_params);
        if (!g.params || !PyList_CheckExact(g.params)) goto bad_structure;
        Py_INCREF(g.params);
        g.n = PyList_GET_SIZE(g.params);
        total += g.n;
    }
    if (PyList_GET_SIZE(entries) != total) goto bad_structure;
    pl->entries.resize(total);
    for (Py_ssize_t i = 0; i < total; i++) {
        Entry &e = pl->entries[i];
        PyObject *t = PyList_GET_ITEM(entries, i);
        if (!PyTuple_Check(t) || PyTuple_GET_SIZE(t) < 2) goto bad_structure;
        e.param = PyTuple_GET_ITEM(t, 0);
        Py_INCREF(e.param);
        if (!THPVariable_Check(e.param)) goto bad_structure;
        {
            const at::Tensor &pt = THPVariable_Unpack(e.param);
            e.param_ptr = pt.data_ptr();
            e.sizes.assign(pt.sizes().begin(), pt.sizes().end());
            e.strides.assign(pt.strides().begin(), pt.strides().end());
        }
        PyObject *state = PyTuple_GET_ITEM(t, 1);
        if (state == Py_None) continue;
        if (PyTuple_GET_SIZE(t) != 10 || !PyDict_Check(state)) goto bad_structure;
        Py_INCREF(state);
        e.state = state;
        e.group = (int)PyLong_AsLong(PyTuple_GET_ITEM(t, 2));
        e.swap = PyObject_IsTrue(PyTuple_GET_ITEM(t, 3)) == 1;
        PyObject *keys = PyTuple_GET_ITEM(t, 4), *s0 = PyTuple_GET_ITEM(t, 5), *s1 = PyTuple_GET_ITEM(t, 6);
        if (!PyTuple_Check(keys) || !PyTuple_Check(s0) || !PyTuple_Check(s1)) goto bad_structure;
        e.nkeys = (int)PyTuple_GET_SIZE(keys);
        if (e.nkeys < 1 || e.nkeys > 4 || PyTuple_GET_SIZE(s0) != e.nkeys || PyTuple_GET_SIZE(s1) != e.nkeys)
            goto bad_structure;
        for (int q = 0; q < e.nkeys; q++) {
            e.keys[q] = PyTuple_GET_ITEM(keys, q);
            e.set[0][q] = PyTuple_GET_ITEM(s0, q);
            e.set[1][q] = PyTuple_GET_ITEM(s1, q);
            Py_INCREF(e.keys[q]);
            Py_INCREF(e.set[0][q]);
            Py_INCREF(e.set[1][q]);
        }
        if (e.group < 0 || e.group >= ng) goto bad_structure;
        if (!fill_row(PyTuple_GET_ITEM(t, 7), e.row[0]) || !fill_row(PyTuple_GET_ITEM(t, 8), e.row[1])) {
            Py_DECREF(cap);
            return nullptr;
        }
        e.dense = PyObject_IsTrue(PyTuple_GET_ITEM(t, 9)) == 1;
    }
    if (PyErr_Occurred()) {
        Py_DECREF(cap);
        return nullptr;
    }
    if (PyDict_Watch(g_watcher, state_map) < 0) {
        Py_DECREF(cap);
        return nullptr;
    }
    pl->generation = g_state_generation;
    pl->table.resize(total);
    pl->grad_ptr.resize(total);
    pl->parity.resize(total);
    pl->next_step.resize(total);
    pl->hp_in.resize(5 * ng);
    return cap;

bad_structure:
    Py_DECREF(cap);
    if (!PyErr_Occurred()) PyErr_SetString(PyExc_ValueError, "malformed step plan");
    return nullptr;
}

PyObject *plan_step(PyObject *, PyObject *cap) {
    Plan *pl = (Plan *)PyCapsule_GetPointer(cap, "smo_plan");
    if (!pl) return nullptr;
    const int rc = run_plan(*pl);
    if (rc == -2) return nullptr;
    return PyLong_FromLong(rc);
}

// the fp32 scalars of one step as the plan forms them (smo_hyper's 40 bytes)
PyObject *hyper_bytes(PyObject *, PyObject *args) {
    double in[5];
    long long step;
    if (!PyArg_ParseTuple(args, "dddddL", &in[0], &in[1], &in[2], &in[3], &in[4], &step)) return nullptr;
    const smo_hyper h = make_hyper(in, step);
    return PyBytes_FromStringAndSize((const char *)&h, sizeof(h));
}

PyMethodDef methods[] = {
    {"plan_new", plan_new, METH_VARARGS, "Build a step plan (see smo_host.cpp)."},
    {"plan_step", plan_step, METH_O, "Run one step of a plan: 0, -1 (plan does not apply) or an smo_status."},
    {"hyper_bytes", hyper_bytes, METH_VARARGS, "smo_hyper bytes of (lr, beta1, beta2, eps, weight_decay, step)."},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef module = {PyModuleDef_HEAD_INIT, "_smo_host", "Host fast path of the SMO optimizer step.", -1, methods};

}  // namespace

PyMODINIT_FUNC PyInit__smo_host(void) {
    s_params = PyUnicode_InternFromString("params");
    s_step = PyUnicode_InternFromString("step");
    s_lr = PyUnicode_InternFromString("lr");
    s_betas = PyUnicode_InternFromString("betas");
    s_eps = PyUnicode_InternFromString("eps");
    s_weight_decay = PyUnicode_InternFromString("weight_decay");
    if (!s_params || !s_step || !s_lr || !s_betas || !s_eps || !s_weight_decay) return nullptr;
    g_watcher = PyDict_AddWatcher(on_state_change);
    if (g_watcher < 0) PyErr_Clear();  // none free: plan_new refuses, the Python path stays
    PyObject *m = PyModule_Create(&module);
    if (m) PyModule_AddIntConstant(m, "sizeof_smo_tensor", (long)sizeof(smo_tensor));
    return m;
}
