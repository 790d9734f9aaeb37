"""Drop-in behaviour on the GPU beyond the step arithmetic.

* A ``state_dict()`` written by the reference optimizer itself (saved with
  ``torch.save`` by tests/golden/make_golden.py at the end of a golden case)
  loads into the drop-in optimizer, which then continues the run for three
  more steps bit-identically to the CPU oracle continuing from the same state.
"""

import os

import numpy as np
import pytest
import torch

import cases as C
from _golden import GOLDEN_DIR, load
from oracle import oracle
from smo_optimizer_b200 import SMO, SMO8bit, _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    _lib.load()


def host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("name", ["s8_groups", "s8_128x256_band_wd", "smo_groups"])
def test_reference_state_dict_loads_and_continues(name):
    case = C.CASES[name]
    sd = torch.load(os.path.join(GOLDEN_DIR, f"{name}.state.pt"))
    gold, _ = load(name)
    shapes = [s for s, _ in case["tensors"]]
    # the reference's parameters at the end of the case (full, not sampled)
    p_end = [gold[f"{i}.param"].reshape(s).astype(np.float32) for i, s in enumerate(shapes)]
    params = [torch.nn.Parameter(torch.from_numpy(a.copy()).cuda()) for a in p_end]
    cls = SMO8bit if case["opt"] == "SMO8bit" else SMO
    opt = cls(C.case_groups(case, params), **case["kwargs"])
    opt.load_state_dict(sd)

    ref_p = [a.copy() for a in p_end]
    ref = oracle.OracleOptimizer(case["opt"], C.case_groups(case, ref_p), **case["kwargs"])
    keys = [k for k, _, _ in ref.params()]
    for idx, k in enumerate(keys):
        ref.state[k] = {key: (v.numpy().copy() if torch.is_tensor(v) else v) for key, v in sd["state"][idx].items()}

    first = case["steps"] + 1
    for step in range(first, first + 3):
        grads = C.case_grads(case, step)
        for p, g in zip(params, grads):
            p.grad = torch.from_numpy(g).cuda()
        opt.step()
        ref.step(grads)
    torch.cuda.synchronize()
    opt.check_device_status()
    for i, (p, k) in enumerate(zip(params, keys)):
        st, rst = opt.state[p], ref.state[k]
        assert st["step"] == rst["step"] == case["steps"] + 3
        for key in C.STATE_ARRAY_KEYS:
            if key in rst:
                got = host(st[key])
                assert got.dtype == np.asarray(rst[key]).dtype, f"{name}[{i}] {key} dtype"
                assert np.array_equal(got.reshape(-1), np.asarray(rst[key]).reshape(-1)), f"{name}[{i}] {key}"
        assert np.array_equal(host(p).view(np.uint32), ref_p[i].view(np.uint32)), f"{name}[{i}] param"


@pytest.mark.parametrize("cls", [SMO8bit, SMO])
def test_non_contiguous_dense_parameters_step_in_place(cls):
    """Strided parameters take the dense path (the reference pools only
    contiguous tensors, spatial_8bit.py:172) and are updated in place, as the
    reference's in-place ops update them: a transposed view (one gap-free
    layout: stepped as flat arrays), a column slice and a strided 1-D view
    (stepped on contiguous copies written back).  Bit-identical to the oracle
    in logical element order; the base tensors see the updates."""
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25)
    bases = [torch.from_numpy(np.random.default_rng(i).standard_normal(s).astype(np.float32) * 0.02).cuda()
             for i, s in enumerate([(64, 48), (64, 100), (600,)])]
    views = [bases[0].t(), bases[1][:, :50], bases[2][::2]]
    assert not any(v.is_contiguous() for v in views)
    params = [torch.nn.Parameter(v) for v in views]
    assert all(p.data_ptr() == v.data_ptr() and p.stride() == v.stride() for p, v in zip(params, views))
    opt = cls(params, **kw)
    ref_p = [host(v).copy() for v in views]  # logical order, contiguous
    # the oracle's arrays are contiguous copies: its group takes the dense path
    # that the reference's contiguity rule picks for the strided parameters
    ref = oracle.OracleOptimizer(cls.__name__, [{"params": ref_p, "compress": False}], **kw)
    for step in range(1, 4):
        gs = [np.random.default_rng(100 * step + i).standard_normal(r.shape).astype(np.float32) * 1e-3
              for i, r in enumerate(ref_p)]
        for p, g in zip(params, gs):
            p.grad = torch.from_numpy(g).cuda()
        opt.step()
        ref.step(gs)
    torch.cuda.synchronize()
    opt.check_device_status()
    keys = [k for k, _, _ in ref.params()]
    for i, (p, v, k) in enumerate(zip(params, views, keys)):
        st = opt.state[p]
        assert st["is_compressed"] is False
        assert np.array_equal(host(p).view(np.uint32), ref_p[i].view(np.uint32)), f"param {i}"
        assert np.array_equal(host(v).view(np.uint32), ref_p[i].view(np.uint32)), f"base view {i}"
        for key in ("exp_avg", "exp_avg_sq"):
            assert np.array_equal(host(st[key]), ref.state[k][key]), f"{key} {i}"
