"""Loading of the golden vectors written by tests/golden/make_golden.py."""

import json
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as z:
        data = {k: z[k] for k in z.files}
    meta = json.loads(bytes(data.pop("meta")).decode())
    return data, meta


def golden_perms(name, n_tensors):
    """The reference's permute_basis draws of a case: (row_perm, col_perm) or None per tensor."""
    try:
        data, _ = load(name)
    except FileNotFoundError:
        return [None] * n_tensors
    return [(data[f"{i}.row_perm"], data[f"{i}.col_perm"]) if f"{i}.row_perm" in data else None
            for i in range(n_tensors)]


def code_mismatch_fraction(a, b):
    a = np.asarray(a).reshape(-1)
    b = np.asarray(b).reshape(-1)
    assert a.shape == b.shape
    diff = a.astype(np.int32) - b.astype(np.int32)
    assert np.abs(diff).max(initial=0) <= 1, "codes differ by more than one LSB"
    return float(np.count_nonzero(diff)) / max(1, a.size)


# Half-precision cases (bf16 / fp16 parameters): torch's CPU kernels run the
# last n mod 32 elements of each elementwise op (and the tail of each thread's
# chunk) through a scalar loop that rounds the product in add(alpha=) and the
# scalar of add_(scalar) to the dtype, where the vectorised loop -- which the
# oracle and the CUDA kernels follow -- keeps them in fp32.  Those elements of
# the reference can differ by a rounding of the dtype.  The contract: at most
# HALF_FRAC of an array's elements differ, codes by one LSB, values by at most
# HALF_TOL of the array's largest finite magnitude; NaN and infinities match.
HALF_TOL = {"bfloat16": 2.0 ** -6, "float16": 2.0 ** -8}
HALF_FRAC = 0.02


def half_close(got, ref, dtype, what):
    got = np.asarray(got).reshape(-1)
    ref = np.asarray(ref).reshape(-1)
    assert got.shape == ref.shape, what
    if ref.dtype == np.int8:
        d = np.abs(got.astype(np.int32) - ref.astype(np.int32))
        assert d.max(initial=0) <= 1, f"{what}: codes differ by more than one LSB"
        assert np.count_nonzero(d) <= HALF_FRAC * d.size, f"{what}: {np.count_nonzero(d)} codes differ"
        return
    g, r = got.astype(np.float64), ref.astype(np.float64)
    same = (g == r) | (np.isnan(g) & np.isnan(r))
    bad = ~same
    assert np.count_nonzero(bad) <= HALF_FRAC * bad.size, f"{what}: {np.count_nonzero(bad)} of {bad.size} differ"
    if bad.any():
        fin = np.isfinite(r)
        scale = np.max(np.abs(r[fin])) if fin.any() else 1.0
        assert np.all(np.isfinite(g[bad]) & np.isfinite(r[bad])), f"{what}: non-finite values differ"
        worst = np.max(np.abs(g[bad] - r[bad]))
        assert worst <= HALF_TOL[dtype] * scale, f"{what}: difference {worst:.3g} vs magnitude {scale:.3g}"
