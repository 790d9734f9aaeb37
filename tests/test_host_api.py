"""CPU-only checks: the C ABI library loads and exports what the header
declares, the ctypes layout matches the C struct, the host-side shape rules
match the reference's state metadata, and the drop-in classes keep the
reference's constructor/step errors (tests/test_spatial_optimizers.py:50-58,
:269-274, :400-402 of the reference)."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import cases as C
from _golden import load
from smo_optimizer_b200 import SMO, SMO8bit, _host, _lib, compression_view, protected_param_groups

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "smo_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SMO_API\s+[\w\s\*]+?\b(smo_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.lib_path())
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), f"{name} declared in smo_b200.h but not exported"


def test_binding_layout_matches_library():
    lib = _lib.load()
    assert lib.smo_abi_version() == _lib.ABI_VERSION
    assert lib.smo_tensor_struct_size() == _lib.TENSOR_DTYPE.itemsize == 248


def test_status_strings_and_host_side_validation():
    lib = _lib.load()
    assert lib.smo_status_string(0) == b"ok"
    assert lib.smo_status_string(5).startswith(b"bounded")
    # descriptors are validated before anything is launched (no GPU needed)
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    t["kind"] = 99
    t["param"] = t["grad"] = 256
    ws = (ctypes.c_uint8 * 4096)()
    addr = (ctypes.addressof(ws) + 255) // 256 * 256
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 1           # SMO_ERR_INVALID
    t["kind"] = _lib.SMO_KIND_DENSE
    t["cols"] = 1
    t["param"] = 258                                                          # misaligned fp32 pointer
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 2           # SMO_ERR_ALIGNMENT
    t["param"] = 256
    assert lib.smo_step(t.ctypes.data, 1, None, 0, None) == 1              # dense: no pointers for m/v
    assert lib.smo_step(t.ctypes.data, 0, addr, 2048, None) == 0           # empty step is a no-op


def test_dtype_field_rules():
    """smo_tensor.dtype: 0 fp32, 1 bf16, 2 fp16, anything else is invalid;
    half-precision pointers need 2-byte alignment, fp32 ones 4."""
    lib = _lib.load()
    ws = (ctypes.c_uint8 * 4096)()
    addr = (ctypes.addressof(ws) + 255) // 256 * 256
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    t["kind"], t["rows"], t["cols"] = _lib.SMO_KIND_DENSE, 16, 1
    t["param"] = 258                                                          # 2-byte aligned only
    t["grad"] = 512
    t["dtype"] = 3
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 1           # unknown dtype
    t["dtype"] = _lib.SMO_DTYPE_F32
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 2           # fp32 needs 4 bytes
    for dt in (_lib.SMO_DTYPE_BF16, _lib.SMO_DTYPE_F16):
        t["dtype"] = dt
        # alignment accepted; the missing moment pointers are what is reported
        assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 1
        t["m_in"], t["v_in"], t["m_out"] = 1024, 2048, 4096
        t["v_out"] = 8193                                                     # odd: misaligned half
        assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 2
        t["m_in"] = t["v_in"] = t["m_out"] = t["v_out"] = 0


def test_no_alloc_validates_before_touching_its_scratch():
    """smo_step_no_alloc checks the descriptors first (a bad one returns its
    own error without any CUDA call, so this runs without a GPU), then the
    size against its fixed scratch."""
    lib = _lib.load()
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    t["kind"] = 99
    t["param"] = t["grad"] = 256
    assert lib.smo_step_no_alloc(t.ctypes.data, 1, None, None) == 1        # SMO_ERR_INVALID
    t["kind"] = _lib.SMO_KIND_DENSE
    t["cols"] = 1
    t["param"] = 258
    assert lib.smo_step_no_alloc(t.ctypes.data, 1, None, None) == 2        # SMO_ERR_ALIGNMENT
    assert lib.smo_step_no_alloc(t.ctypes.data, 0, None, None) == 0        # empty step
    # an oversize descriptor that is also invalid reports the invalid field, not the size
    big = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    big["kind"] = _lib.SMO_KIND_POOLED8
    big["rows"], big["cols"], big["comp_rows"], big["comp_cols"], big["q_block"] = 8000, 6000, 2400, 1800, 64
    big["param"] = big["grad"] = 1 << 32                                     # state pointers missing
    assert lib.smo_step_no_alloc(big.ctypes.data, 1, None, None) == 1


def test_wait_limit_setting_round_trips():
    lib = _lib.load()
    prev = lib.smo_set_wait_limit(5)
    try:
        assert lib.smo_set_wait_limit(0) == 5
        assert lib.smo_set_wait_limit(-7) == 0
        assert lib.smo_set_wait_limit(-1) == -1                                # negative = default
    finally:
        lib.smo_set_wait_limit(prev)
    assert lib.smo_inject_wait_timeout(1) == 0
    assert lib.smo_inject_wait_timeout(0) == 1


def test_permutation_descriptor_rules():
    """permute_basis index arrays: all four or none, pooled kinds only, no bands."""
    lib = _lib.load()
    ws = (ctypes.c_uint8 * 4096)()
    addr = (ctypes.addressof(ws) + 255) // 256 * 256
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    t["kind"] = _lib.SMO_KIND_POOLED8
    t["rows"], t["cols"], t["comp_rows"], t["comp_cols"], t["q_block"] = 64, 64, 16, 16, 64
    base = 1 << 32
    for k in ("param", "grad", "m_q_in", "m_s_in", "v_q_in", "v_s_in", "m_q_out", "m_s_out", "v_q_out", "v_s_out"):
        t[k] = base
        base += 1 << 20
    t["row_perm"] = base                                                     # one of four
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 1
    t["col_perm"], t["row_perm_inv"], t["col_perm_inv"] = base + 1024, base + 2048, base + 3072
    t["interp_band"] = 4                                                     # bands + permutation
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 1
    t["interp_band"] = 0
    t["col_perm"] = base + 1028                                              # misaligned int64 array
    assert lib.smo_step(t.ctypes.data, 1, addr, 2048, None) == 2
    d = np.zeros(1, dtype=_lib.TENSOR_DTYPE)                                 # dense kind with a permutation
    d["kind"], d["rows"], d["cols"] = _lib.SMO_KIND_DENSE, 16, 1
    d["param"] = d["grad"] = d["m_in"] = d["v_in"] = d["m_out"] = d["v_out"] = 1 << 32
    d["row_perm"] = d["col_perm"] = d["row_perm_inv"] = d["col_perm_inv"] = 1 << 33
    assert lib.smo_step(d.ctypes.data, 1, addr, 2048, None) == 1


@pytest.mark.parametrize("name", list(C.CASES))
def test_host_rules_match_reference_metadata(name):
    """compression_view / comp_shape / q_block / quant_only layout agree with the
    state metadata the reference produced for each golden case."""
    case = C.CASES[name]
    _, meta = load(name)
    kw = case["kwargs"]
    specs = case.get("groups") or [{}]
    for i, ((shape, gi), tm) in enumerate(zip(case["tensors"], meta["tensors"])):
        raw = specs[gi].get("compress", True)
        if raw == "quant_only":
            assert tm["is_quant_only"] and tm["q_block"] == _host.quant_only_q_block(shape, kw.get("block_size", 64))
            continue
        view = compression_view(shape, kw.get("compress_conv", False)) if raw else None
        assert tm["is_compressed"] == (view is not None)
        if view is None:
            continue
        vshape, pshape = view
        assert tm["orig_shape"] == list(vshape) and tm["param_shape"] == list(pshape)
        cs = _host.comp_shape(vshape, kw["k_ratio"])
        if case["opt"] == "SMO8bit":
            assert tm["comp_shape"] == list(cs)
            assert tm["q_block"] == _host.pooled_q_block(pshape, cs, kw.get("block_size", 64))


def test_compression_view_rules():
    # reference tests/test_spatial_optimizers.py:119-130
    assert compression_view((64, 64)) == ((64, 64), (64, 64))
    assert compression_view((16, 16)) is None
    assert compression_view((256, 128, 3, 3)) is None
    assert compression_view((256, 128, 3, 3), include_conv=True) == ((256, 1152), (256, 128, 3, 3))
    assert compression_view((16, 3, 3, 3), include_conv=True) is None
    assert compression_view((8, 16, 32), include_conv=True) is None


def test_band_rows_formula():
    # spatial_8bit.py:359 with band_mb = 0.05 on a (128, 256) view at k=0.25
    assert _host.band_comp_rows((128, 256), (32, 64), 0.05) == max(2, int(0.05 * 1024 ** 2 / (2 * 256 * 4 * 4)))
    assert _host.band_comp_rows((1536, 6144), (384, 1536), 64.0) == 341


def test_step_scalars_follow_python_double_arithmetic():
    s = _host.step_scalars(1e-3, (0.9, 0.999), 1e-8, 0.01, 3)
    assert s.neg_step == np.float32(-(1e-3 / (1 - 0.9 ** 3)))
    assert s.sqrt_bc2 == np.float32((1 - 0.999 ** 3) ** 0.5)
    assert s.omb1 == np.float32(1 - 0.9) and s.wd_on == 1
    assert _host.step_scalars(1e-3, (0.9, 0.999), 1e-8, 0, 1).wd_on == 0


def test_host_extension_forms_the_scalars_as_the_python_path():
    """The C++ host path (_smo_host) forms each step's fp32 scalars from the
    group's Python numbers exactly as _host.step_scalars does (double
    arithmetic, one rounding), for steps 1 .. 10^6 and assorted values."""
    from smo_optimizer_b200 import optimizers
    ext = optimizers._host_ext()
    assert ext.sizeof_smo_tensor == _lib.TENSOR_DTYPE.itemsize
    rng = np.random.default_rng(0)
    cases = [(1e-3, 0.9, 0.999, 1e-8, 0.01), (3e-4, 0.8, 0.99, 1e-6, 0), (1, 0.5, 0.5, 1e-12, 1e-5),
             (2e-3, 0.0, 0.0, 0.0, 0.1)]
    cases += [tuple(float(x) for x in (10 ** rng.uniform(-6, -1), rng.uniform(0, 0.999), rng.uniform(0.9, 0.99999),
                                       10 ** rng.uniform(-12, -4), rng.uniform(0, 0.2))) for _ in range(40)]
    steps = [1, 2, 3, 7, 10, 100, 1000, 12345, 10 ** 6]
    for lr, b1, b2, eps, wd in cases:
        for step in steps:
            s = _host.step_scalars(lr, (b1, b2), eps, wd, step)
            want = np.array([(s.beta1, s.omb1, s.beta2, s.omb2, s.wd, s.wd_on, s.neg_step, s.sqrt_bc2, s.eps, 0)],
                            dtype=_lib.HYPER_DTYPE).tobytes()
            assert ext.hyper_bytes(lr, b1, b2, eps, wd, step) == want, (lr, b1, b2, eps, wd, step)


@pytest.mark.parametrize("cls", [SMO, SMO8bit])
def test_constructor_errors(cls):
    p = [torch.nn.Parameter(torch.zeros(32, 32))]
    for kw in (dict(lr=-1.0), dict(eps=-1.0), dict(betas=(1.0, 0.9)), dict(betas=(0.9, 1.0)), dict(k_ratio=0.0),
               dict(k_ratio=1.5)):
        with pytest.raises(ValueError):
            cls(p, **kw)
    if cls is SMO8bit:
        with pytest.raises(ValueError):
            cls(p, block_size=0)
        with pytest.raises(ValueError):
            cls(p, low_peak=True, permute_basis=True)


def test_k_alias_and_defaults():
    p = [torch.nn.Parameter(torch.zeros(32, 32))]
    opt = SMO8bit(p, k=0.5)
    g = opt.param_groups[0]
    assert g["k_ratio"] == 0.5 and g["block_size"] == 64 and g["lr"] == 1e-3
    assert SMO(p).param_groups[0]["k_ratio"] == 0.25
    assert SMO(p)._param_buffers == {}


def test_sparse_gradient_rejected():
    dense = torch.nn.Parameter(torch.zeros(8, 8))
    opt = SMO8bit([dense], lr=1e-3)
    dense.grad = torch.sparse_coo_tensor(torch.tensor([[0, 1], [2, 3]]), torch.tensor([1.0, -1.0]), dense.shape)
    with pytest.raises(RuntimeError):
        opt.step()


def test_smo_rejects_quant_only_group():
    p = torch.nn.Parameter(torch.zeros(64, 64))
    opt = SMO([{"params": [p], "compress": "quant_only"}], lr=1e-3)
    p.grad = torch.randn_like(p)
    with pytest.raises(ValueError):
        opt.step()


def test_cpu_tensors_fail_loudly():
    p = torch.nn.Parameter(torch.zeros(64, 64))
    opt = SMO8bit([p])
    p.grad = torch.zeros_like(p)
    with pytest.raises(RuntimeError, match="CUDA"):
        opt.step()


def test_protect_output_groups():
    named = [("tok_emb.weight", torch.nn.Parameter(torch.zeros(4, 4))),
             ("blocks.0.attn.in_proj_weight", torch.nn.Parameter(torch.zeros(4, 4))),
             ("head.weight", torch.nn.Parameter(torch.zeros(4, 4)))]
    groups = protected_param_groups(named, True)
    assert [len(g["params"]) for g in groups] == [1, 2]
    assert groups[0]["compress"] is True and groups[1]["compress"] is False
    assert protected_param_groups(named, "quant")[1]["compress"] == "quant_only"
    assert protected_param_groups(named, "quant", quant_capable=False)[1]["compress"] is False
    opt = SMO8bit(named, protect_output="dense")
    assert len(opt.param_groups) == 2 and opt.param_groups[1]["compress"] is False
    with pytest.raises(ValueError):
        SMO8bit([p for _, p in named], protect_output=True)


def test_single_shape_workload_names():
    """bench.py's RxCxN[@mode] sets: N tensors of R x C with the decoder's
    settings; the modes pick the group's compress setting or pin the general
    kernels, and the algorithmic bytes follow the mode."""
    from smo_optimizer_b200 import workloads, zero
    wl = workloads.get("64x128x3")
    assert wl.tensors == (("w0", (64, 128)), ("w1", (64, 128)), ("w2", (64, 128)))
    assert wl.compress is True and not wl.general_path and wl.kwargs["low_peak"]
    assert workloads.get("64x128x3@dense").compress is False
    assert workloads.get("64x128x3@quant_only").compress == "quant_only"
    assert workloads.get("64x128x3@general").general_path
    for bad in ("64x128", "64x128x0", "64x128x3@fast", "nope"):
        with pytest.raises(KeyError):
            workloads.get(bad)
    n = 64 * 128
    assert zero.step_bytes((64, 128), "SMO8bit", compress=False) == 28 * n
    assert zero.step_bytes((64, 128), "SMO8bit", compress="quant_only") == 16 * n + 16 * (n // 64)
    assert zero.step_bytes((64, 128), "SMO8bit", elem=2) == 6 * n + 4 * (16 * 32) + 8 * (16 * 32 // 64)
