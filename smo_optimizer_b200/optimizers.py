"""Drop-in ``SMO8bit`` and ``SMO`` optimizers running the step on the B200.

Same constructor arguments, errors, per-group ``compress`` contract and
``state_dict`` layout as the reference classes
(smo/optimizers/spatial_8bit.py:27-374, smo/optimizers/spatial.py:35-208);
the per-tensor arithmetic runs in the CUDA library (include/smo_b200.h), one
``smo_step`` call per device per step, on the current CUDA stream.

Differences a user can observe:
  * Tensors must live on a CUDA device; there is no CPU path.  Parameters
    are fp32, bf16 or fp16 with gradients of the same dtype; as in the
    reference, the state's block scales and float moments take the
    parameter's dtype and every op rounds to it.
  * Pooled moments are double-buffered: after a step ``state[p]['m_q']`` (and
    the other moment tensors) refer to the buffer the step wrote, and the
    previous buffer is reused two steps later.  ``state_dict()`` returns live
    references (as torch.optim.Adam does); deep-copy a snapshot to keep it.
  * ``SMO`` needs no full-resolution reconstruction buffers: the kernels
    reconstruct the moments in registers.  ``_param_buffers`` stays empty.
  * Extra constructor arguments: ``k`` (alias of ``k_ratio``) and
    ``protect_output`` (the grouping rule of the reference's benchmark
    harness, which needs named parameters).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch
from torch.optim.optimizer import Optimizer

from . import _host, _lib

__all__ = ["SMO", "SMO8bit", "protected_param_groups"]


def protected_param_groups(named_params, protect_output, quant_capable: bool = True):
    """Param groups of the reference harness's ``protect_output`` rule.

    benchmarks/suites/comparison/t4_memory_benchmark.py:117-133: parameters
    whose name contains ``"emb"`` or ``"head"`` are protected: dense fp32
    moments (``True`` / ``"dense"``) or full-resolution int8 moments
    (``"quant"``, SMO8bit only; SMO falls back to dense).
    """
    named_params = list(named_params)
    if not protect_output:
        return [{"params": [p for _, p in named_params]}]
    mode = protect_output if protect_output in ("dense", "quant") else "dense"
    if mode == "quant" and not quant_capable:
        mode = "dense"
    flag = "quant_only" if mode == "quant" else False
    protected, regular = [], []
    for name, p in named_params:
        (protected if ("emb" in name or "head" in name) else regular).append(p)
    groups = []
    if regular:
        groups.append({"params": regular, "compress": True})
    if protected:
        groups.append({"params": protected, "compress": flag})
    return groups


def _same_dense_layout(*tensors) -> bool:
    """True when the tensors share shape and strides and each covers one
    gap-free span of memory (any dimension order).  An elementwise step can
    then treat them as flat arrays: the element at memory position k of one is
    the element at position k of the others."""
    t0 = tensors[0]
    if any(t.shape != t0.shape or t.stride() != t0.stride() for t in tensors[1:]):
        return False
    expect = 1
    for stride, size in sorted((st, n) for st, n in zip(t0.stride(), t0.shape) if n != 1):
        if stride != expect:
            return False
        expect *= size
    return True


# torch dtype -> smo_dtype code of the descriptor
_DTYPE_CODES = {torch.float32: _lib.SMO_DTYPE_F32, torch.bfloat16: _lib.SMO_DTYPE_BF16,
                torch.float16: _lib.SMO_DTYPE_F16}


def _check_state(p, state, expected):
    """Raise TypeError unless each present state tensor has its expected dtype
    and lives on the parameter's device; codes, scales and permutations must
    also be contiguous (full-resolution moments follow the parameter's layout,
    which the step checks itself)."""
    for key, dtype in expected:
        t = state.get(key)
        if not torch.is_tensor(t):
            continue
        contiguous = t.is_contiguous() or key in ("exp_avg", "exp_avg_sq")
        if t.dtype != dtype or t.device != p.device or not contiguous:
            raise TypeError(f"state['{key}'] must be a contiguous {dtype} tensor on {p.device}; "
                            f"got {t.dtype} on {t.device}")


# descriptor fields a step reads (in) and writes (out) for the double-buffered kinds
_IN_OUT = {
    _lib.SMO_KIND_POOLED8: (("m_q_in", "m_q_out"), ("m_s_in", "m_s_out"), ("v_q_in", "v_q_out"),
                            ("v_s_in", "v_s_out")),
    _lib.SMO_KIND_POOLED32: (("m_in", "m_out"), ("v_in", "v_out")),
}


class _StepPlan:
    """The C++ host path of one optimizer's parameter set (csrc/smo_host.cpp).

    Built after a step of the Python path, when every parameter with a
    gradient lives on one CUDA device, needs no staged copies and has no
    basis permutation: one entry per parameter of every group with the
    descriptor for each moment-buffer parity.  ``run`` does the whole step in
    one C++ call and returns 0, -1 when the plan no longer applies (nothing
    was modified; the caller steps through the Python path) or an smo_status.
    """

    __slots__ = ("ext", "cap", "flags", "state", "ws")

    @staticmethod
    def build(opt):
        if type(opt)._launch is not _SpatialBase._launch:
            return None  # a subclass that launches its own way keeps the Python path
        entries, dev = [], None
        for gi, group in enumerate(opt.param_groups):
            for p in group["params"]:
                grad = p.grad
                if grad is None:
                    entries.append((p, None))
                    continue
                state = opt.state.get(p)
                if not state or "step" not in state or "row_perm" in state or p.device.type != "cuda":
                    return None
                if dev is None:
                    dev = p.device
                elif p.device != dev:
                    return None
                kp, kg, kst, back = opt._stage(p, grad, state)
                if back is not None or kp is not p or kg is not grad or kst is not state:
                    return None
                rec = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
                opt._fill(rec[0], p, grad, state, group)
                keys, double = opt._moment_keys(state)
                cur = tuple(state[k] for k in keys)
                other = opt._other(p, state, keys) if double else cur
                row0 = rec.tobytes()
                if double:
                    for a, b in _IN_OUT[int(rec["kind"][0])]:
                        rec[a], rec[b] = rec[b].copy(), rec[a].copy()
                dense = not state.get("is_compressed") and not state.get("is_quant_only")
                entries.append((p, state, gi, double, keys, cur, other, row0, rec.tobytes(), dense))
        ws = opt._workspace.get(dev.index) if dev is not None else None
        if ws is None:
            return None
        ext = _host_ext()
        fn = ctypes.cast(_lib.load().smo_step, ctypes.c_void_p).value
        try:
            cap = ext.plan_new(opt.param_groups, opt.state, entries, dev.index, ws.data_ptr(), ws.numel(), fn)
        except (RuntimeError, ValueError):
            return None
        plan = _StepPlan()
        plan.ext, plan.cap, plan.flags, plan.state, plan.ws = ext, cap, opt._kernel_flags, opt.state, ws
        return plan

    def run(self, opt) -> int:
        if opt._kernel_flags != self.flags or opt.state is not self.state:
            return -1
        return self.ext.plan_step(self.cap)


_HOST_EXT = None
_PLAN_MAX_MISSES = 8


def _host_ext():
    """The _smo_host extension (built in-tree by smo_optimizer_b200.build)."""
    global _HOST_EXT
    if _HOST_EXT is None:
        try:
            from . import _smo_host
        except ImportError as e:
            raise _lib.SmoError("host extension _smo_host not built (run `python -m smo_optimizer_b200.build`)") \
                from e
        if _smo_host.sizeof_smo_tensor != _lib.TENSOR_DTYPE.itemsize:
            raise _lib.SmoError("_smo_host was built against another smo_tensor layout")
        _HOST_EXT = _smo_host
    return _HOST_EXT


def _named(params):
    params = list(params)
    if params and isinstance(params[0], tuple) and len(params[0]) == 2 and isinstance(params[0][0], str):
        return params
    raise ValueError("protect_output needs named parameters: pass model.named_parameters()")


class _SpatialBase(Optimizer):
    _name = "SMO"
    _quant = False

    def __init__(self, params, defaults, compress_conv, protect_output):
        if protect_output:
            params = protected_param_groups(_named(params), protect_output, quant_capable=self._quant)
        super().__init__(params, defaults)
        self.compress_conv = bool(compress_conv)
        self._spare = {}        # param -> (buffer set A, buffer set B) of double-buffered moments
        self._workspace = {}    # device index -> uint8 workspace tensor
        self._hyper_cache = {}
        self._inv_perm = {}     # param -> (row_perm, col_perm, their inverses) for permute_basis
        self._rows = {}         # param -> {row key: finished descriptor row (uint64 words)}
        # smo_tensor.flags for every tensor (SMO_FLAG_GENERAL_PATH pins the
        # general two-launch kernels; used to cross-check the fused kernel)
        self._kernel_flags = 0
        # step plan of the C++ host path (_smo_host); built after a step of the
        # Python path, dropped when it stops applying (_PLAN_MAX_MISSES misses
        # with no plan step in between turn it off until the state is loaded)
        self._plan = None
        self._plan_misses = 0

    # ---------------------------------------------------------------- state

    # dtypes of the state tensors that are not the parameter's dtype (block
    # scales and fp32-kind moments have the parameter's dtype)
    _STATE_DTYPES = (("m_q", torch.int8), ("v_q", torch.int8), ("row_perm", torch.int64), ("col_perm", torch.int64))
    _PARAM_DTYPE_STATE = ("m_s", "v_s", "exp_avg", "exp_avg_sq")

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        # torch.optim.Optimizer.load_state_dict casts every state tensor of a
        # floating-point parameter (except "step") to the parameter's dtype,
        # which turns the int8 codes and int64 permutations into float
        # tensors; the values are exact integers, so cast them back
        for st in self.state.values():
            for key, dtype in self._STATE_DTYPES:
                t = st.get(key)
                if torch.is_tensor(t) and t.dtype != dtype:
                    st[key] = t.to(dtype).contiguous()
        self._spare.clear()
        self._inv_perm.clear()
        self._rows.clear()
        self._plan = None
        self._plan_misses = 0

    def _hyper(self, group, step):
        return self._hyper_words(group, step)[0]

    def _hyper_words(self, group, step):
        """(smo_hyper tuple, the same 40 bytes as five uint64 words) of a group at a step."""
        betas = group["betas"]
        key = (group["lr"], betas[0], betas[1], group["eps"], group["weight_decay"], step)
        hp = self._hyper_cache.get(key)
        if hp is None:
            s = _host.step_scalars(group["lr"], betas, group["eps"], group["weight_decay"], step)
            tup = (s.beta1, s.omb1, s.beta2, s.omb2, s.wd, s.wd_on, s.neg_step, s.sqrt_bc2, s.eps, 0)
            words = np.array([tup], dtype=_lib.HYPER_DTYPE).view(np.uint64).reshape(-1).copy()
            hp = (tup, words)
            if len(self._hyper_cache) > 4096:
                self._hyper_cache.clear()
            self._hyper_cache[key] = hp
        return hp

    def _init_state(self, p, grad, group):
        raise NotImplementedError

    def _fill(self, rec, p, grad, state, group):
        raise NotImplementedError

    # ---------------------------------------------------------------- step

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()

        plan = self._plan
        if plan is not None:
            rc = plan.run(self)
            if rc == 0:
                self._plan_misses = 0
                return loss
            if rc > 0:
                _lib.check(rc, "smo_step")
            self._plan = None
            self._plan_misses += 1

        per_dev = {}
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                grad = p.grad
                if grad.is_sparse:
                    raise RuntimeError(f"{self._name} does not support sparse gradients.")
                self._check_compress(group)
                if p.device.type != "cuda":
                    raise RuntimeError(f"{self._name} (B200 build) steps CUDA tensors only; "
                                       f"got a parameter on {p.device}")
                if p.dtype not in _DTYPE_CODES or grad.dtype != p.dtype:
                    raise TypeError(f"{self._name} (B200 build) steps fp32, bf16 or fp16 parameters with "
                                    f"gradients of the same dtype; got {p.dtype} / {grad.dtype}")
                state = self.state[p]
                if "step" not in state:
                    self._init_state(p, grad, group)
                state["step"] += 1
                per_dev.setdefault(p.device, []).append((p, grad, state, group))

        for dev, items in per_dev.items():
            self._launch(dev, items)
        if self._plan_misses < _PLAN_MAX_MISSES:
            self._plan = _StepPlan.build(self)
        return loss

    # ---------------------------------------------------------------- buffers

    # (state keys of the moments, double-buffered?) of a tensor's state
    def _moment_keys(self, state):
        if "m_q" in state:
            return ("m_q", "m_s", "v_q", "v_s"), bool(state.get("is_compressed"))
        return ("exp_avg", "exp_avg_sq"), bool(state.get("is_compressed"))

    def _other(self, p, state, keys):
        """The buffer set a step of a double-buffered tensor writes: the one of
        its pair that the state does not hold (a pair is made, with fresh
        buffers, when the state holds neither)."""
        cur = tuple(state[k] for k in keys)
        pair = self._spare.get(p)
        if pair is not None:
            a, b = pair
            if all(x is y for x, y in zip(cur, a)):
                return b
            if all(x is y for x, y in zip(cur, b)):
                return a
        spare = tuple(torch.empty_like(t) for t in cur)
        self._spare[p] = (cur, spare)
        return spare

    def _swap(self, p, state):
        keys, double = self._moment_keys(state)
        if double:
            state.update(zip(keys, self._other(p, state, keys)))

    def _check_compress(self, group):
        pass

    # Descriptor rows: the first time a tensor is seen with a given set of
    # buffers, _fill writes its row field by field; the finished row is kept
    # (keyed by every address it holds, the group and the kernel flags, so the
    # two ping-pong parities get one row each) and later steps only patch the
    # gradient address and the step's scalars.
    _ROW_WORDS = _lib.TENSOR_DTYPE.itemsize // 8
    _GRAD_WORD = _lib.TENSOR_DTYPE.fields["grad"][1] // 8
    _HP_WORD = _lib.TENSOR_DTYPE.fields["hp"][1] // 8
    _HP_WORDS = _lib.HYPER_DTYPE.itemsize // 8

    def _row(self, p, grad, state, group):
        # every address the row encodes is part of its key: the parameter, the
        # moment buffers read and written, the basis permutations
        keys, double = self._moment_keys(state)
        ptrs = tuple(state[k].data_ptr() for k in keys)
        if double:
            ptrs += tuple(t.data_ptr() for t in self._other(p, state, keys))
        perm = (state["row_perm"].data_ptr(), state["col_perm"].data_ptr()) if "row_perm" in state else ()
        key = (p.data_ptr(), ptrs, perm, id(group), self._kernel_flags, getattr(self, "low_peak", False),
               getattr(self, "band_mb", 0.0))
        rows = self._rows.get(p)
        if rows is None:
            rows = self._rows[p] = {}
        row = rows.get(key)
        if row is None:
            rec = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
            self._fill(rec[0], p, grad, state, group)
            row = rec.view(np.uint64).reshape(-1).copy()
            if len(rows) >= 4:
                rows.clear()
            rows[key] = row
        return row

    @staticmethod
    def _stage(p, grad, state):
        """The tensors a step hands to the kernels, and the copies back to make
        after it (None when the kernels work on the real tensors).

        Pooled tensors are contiguous by their init rule.  A dense tensor whose
        parameter and moments share one gap-free layout (a transposed view, for
        instance) is stepped in place as flat arrays, its gradient first brought
        to that layout; any other strided parameter (and a strided quant_only
        parameter, whose codes follow the logical order) is stepped on
        contiguous copies that are written back in stream order, so the
        parameter and its moments are still updated in place as the
        reference's in-place ops update them (spatial_8bit.py:205-208, 280-283,
        297)."""
        if state.get("is_compressed"):
            return p, (grad if grad.is_contiguous() else grad.contiguous()), state, None
        if state.get("is_quant_only"):
            if p.is_contiguous():
                return p, (grad if grad.is_contiguous() else grad.contiguous()), state, None
            pc = p.contiguous()
            return pc, grad.contiguous(), state, [(p, pc)]
        m, v = state["exp_avg"], state["exp_avg_sq"]
        if _same_dense_layout(p, m, v):
            if grad.shape != p.shape or grad.stride() != p.stride():
                grad = torch.empty_like(p).copy_(grad)  # empty_like keeps the dense layout of p
            return p, grad, state, None
        pc, mc, vc = p.contiguous(), m.contiguous(), v.contiguous()
        st = dict(state)
        st["exp_avg"], st["exp_avg_sq"] = mc, vc
        back = [(p, pc)] + [(dst, src) for dst, src in ((m, mc), (v, vc)) if src is not dst]
        return pc, grad.contiguous(), st, back

    def _launch(self, dev, items):
        words = np.empty((len(items), self._ROW_WORDS), dtype=np.uint64)
        keep, writeback = [], []
        g0, h0, h1 = self._GRAD_WORD, self._HP_WORD, self._HP_WORD + self._HP_WORDS
        for i, (p, grad, state, group) in enumerate(items):
            kp, kg, kst, back = self._stage(p, grad, state)
            if kg is not grad:
                keep.append(kg)
            if back is None:
                words[i] = self._row(kp, kg, kst, group)
            else:
                # staged copies change every step: a fresh row, not a cached one
                rec = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
                self._fill(rec[0], kp, kg, kst, group)
                words[i] = rec.view(np.uint64).reshape(-1)
                keep.append((kp, kst))
                writeback += back
            words[i, g0] = kg.data_ptr()
            words[i, h0:h1] = self._hyper_words(group, state["step"])[1]
        table = words.view(_lib.TENSOR_DTYPE).reshape(-1)
        with torch.cuda.device(dev):
            nbytes = _lib.workspace_size(table)
            ws = self._workspace.get(dev.index)
            if ws is None or ws.numel() < nbytes:
                ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
                self._workspace[dev.index] = ws
            stream = torch.cuda.current_stream(dev).cuda_stream
            _lib.step(table, ws.data_ptr(), ws.numel(), stream)
            for dst, src in writeback:
                dst.copy_(src)
        for p, grad, state, group in items:
            self._swap(p, state)

    def workspace_status(self) -> int:
        """Device-side status of the steps since the last check, on every device
        (synchronises; a non-zero status is cleared by reading it)."""
        worst = 0
        lib = _lib.load()
        for idx, ws in self._workspace.items():
            with torch.cuda.device(idx):
                st = lib.smo_workspace_status(ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
            worst = worst or st
        return worst

    def check_device_status(self) -> None:
        """Raise ``SmoError`` if a step since the last check reported a
        device-side failure (a bounded inter-CTA wait that ran out); the
        parameters of that step are then not valid.  Synchronises."""
        _lib.check(self.workspace_status(), f"{self._name}.step (device status)")


class SMO8bit(_SpatialBase):
    """SMO-8bit: spatially pooled, block-wise int8 moments (spatial_8bit.py:27-79).

    Args are those of the reference; ``k`` is an alias of ``k_ratio`` and
    ``protect_output`` builds the reference harness's param groups.
    """
    _name = "SMO8bit"
    _quant = True

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0, k_ratio=0.25,
                 block_size=64, low_peak=False, band_mb=64.0, permute_basis=False, compress_conv=False,
                 k=None, protect_output=False):
        if k is not None:
            k_ratio = k
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not 0.0 < k_ratio <= 1.0:
            raise ValueError(f"Invalid k_ratio: {k_ratio}")
        if block_size <= 0:
            raise ValueError(f"Invalid block_size: {block_size}")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, k_ratio=k_ratio,
                        block_size=block_size)
        super().__init__(params, defaults, compress_conv, protect_output)
        self.low_peak = low_peak
        self.band_mb = float(band_mb)
        if low_peak and permute_basis:
            raise ValueError("permute_basis is not supported with low_peak")
        self.permute_basis = permute_basis

    # reference helpers (spatial_8bit.py:81-122), on CUDA tensors
    @staticmethod
    def _compress_2d(tensor, target_shape):
        from . import ops
        return ops.compress_2d(tensor, target_shape)

    def _quantize_blockwise(self, data, block_size):
        from . import ops
        q, s = ops.quantize_blockwise(data, block_size)
        return q, s, data.shape

    def _dequantize_blockwise(self, q_blocks, scales, orig_shape, numel=None, dtype=None):
        from . import ops
        if numel is None:
            numel = math.prod(orig_shape)
        out = ops.dequantize_blockwise(q_blocks, scales, numel, q_blocks.shape[-1])
        if dtype is not None:
            out = out.to(dtype)
        return out.view(orig_shape)

    def _check_compress(self, group):
        pass

    def _init_state(self, p, grad, group):
        state = self.state[p]
        state["step"] = 0
        raw = group.get("compress", True)
        dev = grad.device
        if raw == "quant_only":
            state["is_quant_only"] = True
            state["is_compressed"] = False
            state["q_shape"] = tuple(grad.shape)
            state["q_numel"] = grad.numel()
            qb = _host.quant_only_q_block(grad.shape, group["block_size"])
            state["q_block"] = qb
            nb = _host.num_blocks(grad.numel(), qb)
            state["m_q"] = torch.zeros((nb, qb), dtype=torch.int8, device=dev)
            state["m_s"] = torch.full((nb, 1), 1e-12, dtype=grad.dtype, device=dev)
            state["v_q"] = torch.zeros((nb, qb), dtype=torch.int8, device=dev)
            state["v_s"] = torch.full((nb, 1), 1e-12, dtype=grad.dtype, device=dev)
            return
        view = _host.compression_view(grad.shape, self.compress_conv) if raw else None
        if view is not None and p.is_contiguous():
            vshape, pshape = view
            state["is_compressed"] = True
            state["orig_shape"] = vshape
            state["param_shape"] = pshape
            cs = _host.comp_shape(vshape, group["k_ratio"])
            state["comp_numel"] = cs[0] * cs[1]
            qb = _host.pooled_q_block(pshape, cs, group["block_size"])
            state["q_block"] = qb
            nb = _host.num_blocks(cs[0] * cs[1], qb)
            # quantising zeros gives zero codes and 1e-12 scales in the gradient's
            # dtype (spatial_8bit.py:195-200; 0 in fp16, which has no 1e-12)
            state["m_q"] = torch.zeros((nb, qb), dtype=torch.int8, device=dev)
            state["m_s"] = torch.full((nb, 1), 1e-12, dtype=grad.dtype, device=dev)
            state["v_q"] = torch.zeros((nb, qb), dtype=torch.int8, device=dev)
            state["v_s"] = torch.full((nb, 1), 1e-12, dtype=grad.dtype, device=dev)
            state["comp_shape"] = cs
            if self.permute_basis:
                # random basis permutations drawn as the reference does
                # (spatial_8bit.py:202-204); permutations already placed in the
                # state before the first step are kept
                for key, n in (("row_perm", vshape[0]), ("col_perm", vshape[1])):
                    if key in state:
                        perm = state[key]
                        if perm.dtype != torch.int64 or tuple(perm.shape) != (n,):
                            raise ValueError(f"state['{key}'] must be an int64 permutation of {n} indices")
                        state[key] = perm.to(dev).contiguous()
                    else:
                        state[key] = torch.randperm(n, device=dev)
        else:
            state["is_compressed"] = False
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)

    def _perms(self, p, state):
        """(row_perm, col_perm, row_perm_inv, col_perm_inv) of a permuted-basis tensor."""
        rp, cp = state["row_perm"], state["col_perm"]
        cached = self._inv_perm.get(p)
        if cached is None or cached[0] is not rp or cached[1] is not cp:
            if rp.device != p.device or cp.device != p.device:
                rp = state["row_perm"] = rp.to(p.device).contiguous()
                cp = state["col_perm"] = cp.to(p.device).contiguous()
            cached = (rp, cp, torch.argsort(rp), torch.argsort(cp))
            self._inv_perm[p] = cached
        return cached


    def _fill(self, rec, p, grad, state, group):
        _check_state(p, state, self._STATE_DTYPES + tuple((k, p.dtype) for k in self._PARAM_DTYPE_STATE))
        rec["dtype"] = _DTYPE_CODES[p.dtype]
        rec["param"] = p.data_ptr()
        rec["grad"] = grad.data_ptr()
        rec["flags"] = self._kernel_flags
        rec["hp"] = self._hyper(group, state["step"])
        if state.get("is_quant_only"):
            rec["kind"] = _lib.SMO_KIND_QUANT_ONLY
            rec["rows"], rec["cols"] = p.numel(), 1
            rec["q_block"] = state["q_block"]
            for k in ("m_q", "m_s", "v_q", "v_s"):
                rec[k + "_in"] = rec[k + "_out"] = state[k].data_ptr()
        elif state["is_compressed"]:
            if not p.is_contiguous():
                raise RuntimeError("a pooled parameter must stay contiguous (it was at init)")
            rec["kind"] = _lib.SMO_KIND_POOLED8
            rec["rows"], rec["cols"] = state["orig_shape"]
            rec["comp_rows"], rec["comp_cols"] = state["comp_shape"]
            rec["q_block"] = state["q_block"]
            if self.low_peak and _host.can_band(state["orig_shape"], state["comp_shape"]):
                rec["interp_band"] = _host.band_comp_rows(state["orig_shape"], state["comp_shape"],
                                                          self.band_mb, grad.element_size())
            if "row_perm" in state:
                for k, t in zip(("row_perm", "col_perm", "row_perm_inv", "col_perm_inv"), self._perms(p, state)):
                    rec[k] = t.data_ptr()
            sp = self._other(p, state, ("m_q", "m_s", "v_q", "v_s"))
            for k, s in zip(("m_q", "m_s", "v_q", "v_s"), sp):
                rec[k + "_in"] = state[k].data_ptr()
                rec[k + "_out"] = s.data_ptr()
        else:
            if not _same_dense_layout(p, grad, state["exp_avg"], state["exp_avg_sq"]):
                raise RuntimeError("dense step: parameter, gradient and moments must share one memory layout")
            rec["kind"] = _lib.SMO_KIND_DENSE
            rec["rows"], rec["cols"] = p.numel(), 1
            rec["m_in"] = rec["m_out"] = state["exp_avg"].data_ptr()
            rec["v_in"] = rec["v_out"] = state["exp_avg_sq"].data_ptr()


class SMO(_SpatialBase):
    """SMO-Spatial: spatially pooled fp32 moments (spatial.py:35-75)."""
    _name = "SMO"
    _quant = False

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0, k_ratio=0.25,
                 compress_conv=False, k=None, protect_output=False):
        if k is not None:
            k_ratio = k
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not 0.0 < k_ratio <= 1.0:
            raise ValueError(f"Invalid k_ratio: {k_ratio}. Must be in (0, 1]")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, k_ratio=k_ratio)
        super().__init__(params, defaults, compress_conv, protect_output)
        # The reference caches full-resolution reconstruction buffers here
        # (spatial.py:73-75); the fused kernels need none, so it stays empty.
        self._param_buffers = {}

    @staticmethod
    def _compress_2d(tensor, target_shape):
        from . import ops
        return ops.compress_2d(tensor, target_shape)

    def _check_compress(self, group):
        if group.get("compress", True) == "quant_only":
            raise ValueError("SMO (fp32) has no int8 storage; 'quant_only' groups require SMO8bit")

    def _init_state(self, p, grad, group):
        state = self.state[p]
        state["step"] = 0
        use = group.get("compress", True)
        view = _host.compression_view(grad.shape, self.compress_conv) if use else None
        if view is not None and p.is_contiguous():
            vshape, pshape = view
            state["is_compressed"] = True
            cs = _host.comp_shape(vshape, group["k_ratio"])
            state["exp_avg"] = torch.zeros(cs, dtype=grad.dtype, device=grad.device)
            state["exp_avg_sq"] = torch.zeros(cs, dtype=grad.dtype, device=grad.device)
            state["orig_shape"] = vshape
            state["param_shape"] = pshape
        else:
            state["is_compressed"] = False
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)

    def _fill(self, rec, p, grad, state, group):
        _check_state(p, state, tuple((k, p.dtype) for k in ("exp_avg", "exp_avg_sq")))
        rec["dtype"] = _DTYPE_CODES[p.dtype]
        rec["param"] = p.data_ptr()
        rec["grad"] = grad.data_ptr()
        rec["flags"] = self._kernel_flags
        rec["hp"] = self._hyper(group, state["step"])
        if state["is_compressed"]:
            if not p.is_contiguous():
                raise RuntimeError("a pooled parameter must stay contiguous (it was at init)")
            if not (state["exp_avg"].is_contiguous() and state["exp_avg_sq"].is_contiguous()):
                raise TypeError("pooled moments state['exp_avg'] / state['exp_avg_sq'] must be contiguous")
            rec["kind"] = _lib.SMO_KIND_POOLED32
            rec["rows"], rec["cols"] = state["orig_shape"]
            rec["comp_rows"], rec["comp_cols"] = state["exp_avg"].shape
            sp = self._other(p, state, ("exp_avg", "exp_avg_sq"))
            rec["m_in"], rec["v_in"] = state["exp_avg"].data_ptr(), state["exp_avg_sq"].data_ptr()
            rec["m_out"], rec["v_out"] = sp[0].data_ptr(), sp[1].data_ptr()
        else:
            if not _same_dense_layout(p, grad, state["exp_avg"], state["exp_avg_sq"]):
                raise RuntimeError("dense step: parameter, gradient and moments must share one memory layout")
            rec["kind"] = _lib.SMO_KIND_DENSE
            rec["rows"], rec["cols"] = p.numel(), 1
            rec["m_in"] = rec["m_out"] = state["exp_avg"].data_ptr()
            rec["v_in"] = rec["v_out"] = state["exp_avg_sq"].data_ptr()

