"""Pin the CPU oracle to the reference: the oracle replays every golden case and
must reproduce the reference's own outputs (written by make_golden.py).

Tolerances are the parity contract of the step:
  * int8 codes bit-identical, except at most 1e-5 of them off by one LSB;
  * scales and params within rtol 1e-5 / atol 1e-7 (fp32).

Half-precision parameters (bf16 / fp16 cases): the oracle computes every op
as torch's vectorised CPU loop does (fp32 arithmetic, one rounding to the
dtype per op); the elements torch's scalar tail loop rounds differently are
covered by _golden.half_close (at most 2 % of an array's elements differ,
codes by one LSB, values by at most 2^-6 (bf16) / 2^-8 (fp16) of the
array's largest finite magnitude; NaN and infinities match).
"""

import numpy as np
import pytest

import cases as C
from _golden import code_mismatch_fraction, golden_perms, half_close, load
from oracle import oracle

CODE_FRAC = 1e-5
RTOL, ATOL = 1e-5, 1e-7


def run_oracle(name):
    case = C.CASES[name]
    params = C.case_params(case)
    groups = C.case_groups(case, params)
    assert [gi for _, gi in case["tensors"]] == sorted(gi for _, gi in case["tensors"])
    kw = dict(case["kwargs"])
    opt = oracle.OracleOptimizer(case["opt"], groups, param_dtype=C.case_dtype(case), **kw)
    keys = [k for k, _, _ in opt.params()]
    for k, pr in zip(keys, golden_perms(name, len(keys))):
        if pr is not None:
            opt.preset_perms[k] = pr
    for step in range(1, case["steps"] + 1):
        opt.step(C.case_grads(case, step))
    return case, params, [opt.state[k] for k in keys]


def compare_to_golden(name, params, states, code_frac=CODE_FRAC, rtol=RTOL, atol=ATOL):
    case = C.CASES[name]
    dtype = C.case_dtype(case)
    gold, meta = load(name)
    stride = case.get("sample_stride")
    for i, (p, st) in enumerate(zip(params, states)):
        tm = meta["tensors"][i]
        for k, v in tm.items():
            got = st.get(k)
            got = list(got) if isinstance(got, tuple) else got
            assert got == v, f"{name}[{i}] state[{k!r}] = {got!r}, reference has {v!r}"
        for k in C.STATE_ARRAY_KEYS:
            gk = f"{i}.{k}"
            assert (gk in gold) == (k in st), f"{name}[{i}] state key {k} presence differs"
            if gk not in gold:
                continue
            ref = gold[gk]
            got = np.asarray(st[k]).reshape(ref.shape)
            if dtype != "float32":
                half_close(got, ref, dtype, f"{name}[{i}] {k}")
            elif ref.dtype == np.int8:
                frac = code_mismatch_fraction(got, ref)
                assert frac <= code_frac, f"{name}[{i}] {k}: {frac:.2e} of codes differ"
            else:
                np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol, err_msg=f"{name}[{i}] {k}")
        flat = np.asarray(p).reshape(-1)
        if dtype != "float32":
            half_close(flat[C.sample_indices(flat.size, stride)] if stride else flat,
                       gold[f"{i}.param_sample"] if stride else gold[f"{i}.param"], dtype, f"{name}[{i}] param")
        elif stride:
            np.testing.assert_allclose(flat[C.sample_indices(flat.size, stride)], gold[f"{i}.param_sample"],
                                       rtol=rtol, atol=atol, err_msg=f"{name}[{i}] param")
        else:
            np.testing.assert_allclose(flat, gold[f"{i}.param"], rtol=rtol, atol=atol,
                                       err_msg=f"{name}[{i}] param")


@pytest.mark.parametrize("name", [n for n in C.CASES if n != "single1024"])
def test_oracle_matches_reference(name):
    _, params, states = run_oracle(name)
    compare_to_golden(name, params, states)


def test_oracle_matches_reference_single1024_100_steps():
    _, params, states = run_oracle("single1024")
    compare_to_golden("single1024", params, states)


def test_oracle_codes_exact_on_small_cases():
    """On the short cases the codes must be bit-identical (no tie slips at all)."""
    for name in ("s8_64x64", "s8_128x256_band_wd", "s8_multi", "s8_groups", "s8_808x96_band"):
        _, params, states = run_oracle(name)
        compare_to_golden(name, params, states, code_frac=0.0)
