"""ctypes front-end of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs use this module, and only as the checker or the CPU timing arm.
It never runs on the product path.

``OracleOptimizer`` replays the reference's per-tensor state logic
(lazy init, per-group ``compress`` contract, compression view, q_block,
low_peak bands) from smo/optimizers/spatial_8bit.py:124-374 and
smo/optimizers/spatial.py:82-208 on numpy arrays, and calls the C restatement
in smo_oracle.c for the arithmetic.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from smo_optimizer_b200 import _host

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libsmo_oracle.so")
_lib = None


class _Hyper(ctypes.Structure):
    _fields_ = [
        ("beta1", ctypes.c_float), ("omb1", ctypes.c_float),
        ("beta2", ctypes.c_float), ("omb2", ctypes.c_float),
        ("wd", ctypes.c_float), ("wd_on", ctypes.c_int32),
        ("neg_step", ctypes.c_float), ("sqrt_bc2", ctypes.c_float),
        ("eps", ctypes.c_float), ("dtype", ctypes.c_int32),
    ]


# parameter dtypes (the reference computes in the parameter's dtype)
DTYPES = {"float32": 0, "bfloat16": 1, "float16": 2}


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 values rounded to ``dtype`` (nearest even) and widened back to fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "bfloat16":
        from smo_optimizer_b200 import synthetic
        return synthetic.round_to_bf16(x)
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    return x


def build(force: bool = False) -> str:
    """Compile libsmo_oracle.so with oracle/Makefile (gcc, no GPU needed)."""
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "smo_oracle.c"))):
        subprocess.run(["make", "-s", "-C", _HERE, "libsmo_oracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        i64, P = ctypes.c_int64, ctypes.c_void_p
        hp = ctypes.POINTER(_Hyper)
        _lib.oracle_smo8bit_pooled_step.argtypes = [P, P, P, P, P, P, i64, i64, i64, i64, i64, i64, hp]
        _lib.oracle_smo_pooled_step.argtypes = [P, P, P, P, i64, i64, i64, i64, hp]
        _lib.oracle_dense_step.argtypes = [P, P, P, P, i64, hp]
        _lib.oracle_quant_only_step.argtypes = [P, P, P, P, P, P, i64, i64, hp]
        _lib.oracle_pool_pair.argtypes = [P, P, i64, i64, i64, i64, hp, P, P]
        _lib.oracle_quantize_dt.argtypes = [P, i64, i64, P, P, ctypes.c_int]
        _lib.oracle_dequantize_dt.argtypes = [P, P, i64, i64, P, ctypes.c_int]
        _lib.oracle_upsample.argtypes = [P, i64, i64, i64, i64, i64, P]
        _lib.oracle_num_threads.restype = ctypes.c_int
        _lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def hyper(s: _host.StepScalars, dtype: str = "float32") -> _Hyper:
    return _Hyper(float(s.beta1), float(s.omb1), float(s.beta2), float(s.omb2), float(s.wd),
                  int(s.wd_on), float(s.neg_step), float(s.sqrt_bc2), float(s.eps), DTYPES[dtype])


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


# ---------------------------------------------------------------- primitives

def quantize(x: np.ndarray, block: int, dtype: str = "float32"):
    """_quantize_blockwise (spatial_8bit.py:85-107): codes (nb, block), scales (nb, 1) in ``dtype``."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    nb = _host.num_blocks(x.size, block)
    q = np.zeros((nb, block), np.int8)
    s = np.zeros((nb, 1), np.float32)
    lib().oracle_quantize_dt(_ptr(x), x.size, block, _ptr(q), _ptr(s), DTYPES[dtype])
    return q, s


def dequantize(q: np.ndarray, s: np.ndarray, n: int, block: int, dtype: str = "float32") -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oracle_dequantize_dt(_ptr(np.ascontiguousarray(q)), _ptr(np.ascontiguousarray(s)), n, block, _ptr(out),
                               DTYPES[dtype])
    return out


def pool_pair(g, p, cshape, scalars):
    g = np.ascontiguousarray(g, np.float32)
    p = np.ascontiguousarray(p, np.float32)
    H, W = g.shape
    h, w = cshape
    og = np.empty((h, w), np.float32)
    og2 = np.empty((h, w), np.float32)
    lib().oracle_pool_pair(_ptr(g), _ptr(p), H, W, h, w, ctypes.byref(hyper(scalars)), _ptr(og), _ptr(og2))
    return og, og2


def upsample(src, out_shape, interp_band: int = 0):
    src = np.ascontiguousarray(src, np.float32)
    h, w = src.shape
    H, W = out_shape
    out = np.empty((H, W), np.float32)
    lib().oracle_upsample(_ptr(src), h, w, H, W, interp_band, _ptr(out))
    return out


# ---------------------------------------------------------------- per-tensor steps

def smo8bit_pooled_step(p2d, g2d, st, scalars, interp_band=0, dtype="float32"):
    H, W = p2d.shape
    h, w = st["comp_shape"]
    rc = lib().oracle_smo8bit_pooled_step(
        _ptr(p2d), _ptr(g2d), _ptr(st["m_q"]), _ptr(st["m_s"]), _ptr(st["v_q"]), _ptr(st["v_s"]),
        H, W, h, w, st["q_block"], interp_band, ctypes.byref(hyper(scalars, dtype)))
    assert rc == 0, "oracle allocation failed"


def smo_pooled_step(p2d, g2d, st, scalars, dtype="float32"):
    H, W = p2d.shape
    h, w = st["exp_avg"].shape
    rc = lib().oracle_smo_pooled_step(_ptr(p2d), _ptr(g2d), _ptr(st["exp_avg"]), _ptr(st["exp_avg_sq"]),
                                      H, W, h, w, ctypes.byref(hyper(scalars, dtype)))
    assert rc == 0, "oracle allocation failed"


def dense_step(p, g, st, scalars, dtype="float32"):
    lib().oracle_dense_step(_ptr(p), _ptr(g), _ptr(st["exp_avg"]), _ptr(st["exp_avg_sq"]), p.size,
                            ctypes.byref(hyper(scalars, dtype)))


def quant_only_step(p, g, st, scalars, dtype="float32"):
    rc = lib().oracle_quant_only_step(_ptr(p), _ptr(g), _ptr(st["m_q"]), _ptr(st["m_s"]), _ptr(st["v_q"]),
                                      _ptr(st["v_s"]), p.size, st["q_block"], ctypes.byref(hyper(scalars, dtype)))
    assert rc == 0, "oracle allocation failed"


# ---------------------------------------------------------------- optimizer replay

class OracleOptimizer:
    """The reference's SMO8bit / SMO step logic over numpy fp32 arrays.

    ``groups`` is a list of dicts ``{"params": [np.ndarray, ...], ...}`` with
    optional per-group overrides and ``compress`` (True / False / "quant_only").
    Arrays are updated in place.  ``state`` is keyed by (group, index).
    ``param_dtype`` ("float32", "bfloat16", "float16") is the dtype the
    reference's parameters, gradients and state would have: arrays stay fp32
    numpy arrays holding values of that dtype, and every op rounds to it.
    """

    def __init__(self, kind, groups, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                 k_ratio=0.25, block_size=64, low_peak=False, band_mb=64.0, compress_conv=False,
                 permute_basis=False, param_dtype="float32"):
        assert kind in ("SMO8bit", "SMO")
        if low_peak and permute_basis:
            raise ValueError("permute_basis is not supported with low_peak")
        self.kind = kind
        self.defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, k_ratio=k_ratio,
                             block_size=block_size)
        self.groups = []
        for g in groups:
            d = dict(self.defaults)
            d.update(g)
            self.groups.append(d)
        self.low_peak = low_peak
        self.band_mb = float(band_mb)
        self.compress_conv = bool(compress_conv)
        self.permute_basis = bool(permute_basis) and kind == "SMO8bit"
        if param_dtype not in DTYPES:
            raise ValueError(f"param_dtype must be one of {sorted(DTYPES)}")
        self.dtype = param_dtype
        # permute_basis: (row_perm, col_perm) per state key, placed before the
        # first step (the reference draws them with torch.randperm,
        # spatial_8bit.py:202-204); absent keys get a seeded numpy permutation
        self.preset_perms = {}
        self.state = {}

    def params(self):
        for gi, g in enumerate(self.groups):
            for pi, p in enumerate(g["params"]):
                yield (gi, pi), g, p

    def _init(self, p, group, key=None):
        raw = group.get("compress", True)
        quant_only = (raw == "quant_only")
        st = {"step": 0}
        if quant_only:
            if self.kind == "SMO":
                raise ValueError("quant_only groups require SMO8bit")
            st.update(is_quant_only=True, is_compressed=False, q_shape=tuple(p.shape), q_numel=p.size,
                      q_block=_host.quant_only_q_block(p.shape, group["block_size"]))
            z = np.zeros(p.size, np.float32)
            st["m_q"], st["m_s"] = quantize(z, st["q_block"], self.dtype)
            st["v_q"], st["v_s"] = quantize(z, st["q_block"], self.dtype)
            return st
        view = _host.compression_view(p.shape, self.compress_conv) if raw else None
        if view is not None:
            vshape, pshape = view
            cs = _host.comp_shape(vshape, group["k_ratio"])
            st.update(is_compressed=True, orig_shape=vshape, param_shape=pshape)
            if self.kind == "SMO8bit":
                st["comp_numel"] = cs[0] * cs[1]
                st["q_block"] = _host.pooled_q_block(pshape, cs, group["block_size"])
                z = np.zeros(cs[0] * cs[1], np.float32)
                st["m_q"], st["m_s"] = quantize(z, st["q_block"], self.dtype)
                st["v_q"], st["v_s"] = quantize(z, st["q_block"], self.dtype)
                st["comp_shape"] = cs
                if self.permute_basis:
                    rp, cp = self.preset_perms.get(key) or (np.random.default_rng(0).permutation(vshape[0]),
                                                             np.random.default_rng(1).permutation(vshape[1]))
                    st["row_perm"] = np.asarray(rp, np.int64)
                    st["col_perm"] = np.asarray(cp, np.int64)
            else:
                st["exp_avg"] = np.zeros(cs, np.float32)
                st["exp_avg_sq"] = np.zeros(cs, np.float32)
        else:
            st["is_compressed"] = False
            st["exp_avg"] = np.zeros(p.shape, np.float32)
            st["exp_avg_sq"] = np.zeros(p.shape, np.float32)
        return st

    def step(self, grads):
        """``grads``: list of arrays in ``params()`` order (None skips a tensor)."""
        for (key, group, p), g in zip(list(self.params()), grads):
            if g is None:
                continue
            st = self.state.get(key)
            if st is None:
                st = self.state[key] = self._init(p, group, key)
            st["step"] += 1
            sc = _host.step_scalars(group["lr"], group["betas"], group["eps"], group["weight_decay"],
                                    st["step"])
            g = np.ascontiguousarray(g, np.float32)
            dt = self.dtype
            if st.get("is_quant_only"):
                quant_only_step(p.reshape(-1), g.reshape(-1), st, sc, dt)
            elif st["is_compressed"]:
                p2 = p.reshape(st["orig_shape"])
                g2 = g.reshape(st["orig_shape"])
                if self.kind == "SMO8bit":
                    band = 0
                    if self.low_peak and _host.can_band(st["orig_shape"], st["comp_shape"]):
                        band = _host.band_comp_rows(st["orig_shape"], st["comp_shape"], self.band_mb,
                                                    4 if dt == "float32" else 2)
                    if "row_perm" in st:
                        # the step in the permuted basis (spatial_8bit.py:231-253): pool
                        # g[rp][:, cp], reconstruct there, map the update back
                        ix = np.ix_(st["row_perm"], st["col_perm"])
                        pp = np.ascontiguousarray(p2[ix])
                        smo8bit_pooled_step(pp, np.ascontiguousarray(g2[ix]), st, sc, band, dt)
                        p2[ix] = pp
                    else:
                        smo8bit_pooled_step(p2, g2, st, sc, band, dt)
                else:
                    smo_pooled_step(p2, g2, st, sc, dt)
            else:
                dense_step(p.reshape(-1), g.reshape(-1),
                           {"exp_avg": st["exp_avg"].reshape(-1), "exp_avg_sq": st["exp_avg_sq"].reshape(-1)},
                           sc, dt)
