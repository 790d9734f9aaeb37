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
