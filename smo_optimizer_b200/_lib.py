"""ctypes binding of the CUDA library (include/smo_b200.h).

The library is built in-tree (``python -m smo_optimizer_b200.build``) as
``smo_optimizer_b200/libsmo_b200.so``.  There is no fallback: if the library
is missing or cannot be loaded, every call raises.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np


SMO_OK = 0
SMO_KIND_POOLED8 = 1
SMO_KIND_POOLED32 = 2
SMO_KIND_DENSE = 3
SMO_KIND_QUANT_ONLY = 4
SMO_ERR_TIMEOUT = 5
SMO_DTYPE_F32 = 0
SMO_DTYPE_BF16 = 1
SMO_DTYPE_F16 = 2
SMO_FLAG_GENERAL_PATH = 1
ABI_VERSION = 3

# Field layout of struct smo_hyper / smo_tensor, as a numpy structured dtype so
# that descriptor tables are filled column-wise without per-field Python calls.
HYPER_DTYPE = np.dtype([
    ("beta1", np.float32), ("omb1", np.float32), ("beta2", np.float32), ("omb2", np.float32),
    ("weight_decay", np.float32), ("wd_on", np.int32), ("neg_step", np.float32),
    ("sqrt_bc2", np.float32), ("eps", np.float32), ("reserved", np.int32),
])

TENSOR_DTYPE = np.dtype([
    ("param", np.uint64), ("grad", np.uint64),
    ("m_q_in", np.uint64), ("m_s_in", np.uint64), ("v_q_in", np.uint64), ("v_s_in", np.uint64),
    ("m_q_out", np.uint64), ("m_s_out", np.uint64), ("v_q_out", np.uint64), ("v_s_out", np.uint64),
    ("m_in", np.uint64), ("v_in", np.uint64), ("m_out", np.uint64), ("v_out", np.uint64),
    ("rows", np.int64), ("cols", np.int64), ("comp_rows", np.int64), ("comp_cols", np.int64),
    ("q_block", np.int64), ("interp_band", np.int64),
    ("kind", np.int32), ("flags", np.int32),
    ("hp", HYPER_DTYPE),
    ("row_perm", np.uint64), ("col_perm", np.uint64), ("row_perm_inv", np.uint64), ("col_perm_inv", np.uint64),
    ("dtype", np.int32), ("reserved", np.int32),
])

HYPER_FIELDS = HYPER_DTYPE.names


class SmoError(RuntimeError):
    """A call into the CUDA library failed."""


_lib = None


def lib_path() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsmo_b200.so")


def load():
    """Load libsmo_b200.so (raising if it is absent or has the wrong ABI)."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise SmoError(f"CUDA library not built: {path} is missing "
                       "(run `python -m smo_optimizer_b200.build`)")
    lib = ctypes.CDLL(path)
    P, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t
    sigs = {
        "smo_workspace_size": (sz, [P, i32]),
        "smo_step": (ctypes.c_int, [P, i32, P, sz, P]),
        "smo_workspace_status": (ctypes.c_int, [P, P]),
        "smo_quantize_blockwise": (ctypes.c_int, [P, i64, i64, P, P, P]),
        "smo_dequantize_blockwise": (ctypes.c_int, [P, P, i64, i64, P, P]),
        "smo_pool2d_pair": (ctypes.c_int, [P, P, i64, i64, i64, i64, ctypes.c_float, i32, P, P, P]),
        "smo_upsample2d": (ctypes.c_int, [P, i64, i64, i64, i64, i64, P, P]),
        "smo_synth_normal": (ctypes.c_int, [P, i64, ctypes.c_uint64, ctypes.c_float, i64, P]),
        "smo_selftest_wait_timeout": (ctypes.c_int, [P, sz, i64, ctypes.POINTER(ctypes.c_int32), P]),
        "smo_selftest_fastmath": (ctypes.c_int, [P, sz, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64), P]),
        "smo_status_string": (ctypes.c_char_p, [ctypes.c_int]),
        "smo_last_cuda_error": (ctypes.c_int, []),
        "smo_abi_version": (ctypes.c_int, []),
        "smo_tensor_struct_size": (sz, []),
        "smo_launch_count": (ctypes.c_uint64, []),
        "smo_step_no_alloc": (ctypes.c_int, [P, i32, P, P]),
        "smo_set_wait_limit": (i64, [i64]),
        "smo_inject_wait_timeout": (ctypes.c_int, [ctypes.c_int]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.smo_abi_version() != ABI_VERSION:
        raise SmoError(f"libsmo_b200 ABI {lib.smo_abi_version()} != binding ABI {ABI_VERSION}")
    if lib.smo_tensor_struct_size() != TENSOR_DTYPE.itemsize:
        raise SmoError(f"smo_tensor is {lib.smo_tensor_struct_size()} bytes in the library, "
                       f"{TENSOR_DTYPE.itemsize} in the binding")
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != SMO_OK:
        lib = load()
        msg = lib.smo_status_string(status).decode()
        if status == 4:
            msg += f" (cudaError {lib.smo_last_cuda_error()})"
        raise SmoError(f"{what} failed: {msg} [{status}]")


def workspace_size(table: np.ndarray) -> int:
    return int(load().smo_workspace_size(table.ctypes.data, len(table)))


def step(table: np.ndarray, workspace_ptr: int, workspace_bytes: int, stream: int) -> None:
    assert table.dtype == TENSOR_DTYPE and table.flags["C_CONTIGUOUS"]
    check(load().smo_step(table.ctypes.data, len(table), workspace_ptr, workspace_bytes, stream), "smo_step")
