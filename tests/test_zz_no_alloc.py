"""smo_step_no_alloc: the optimizer step for callers that cannot allocate
device memory (its scratch is a fixed array inside the library).

It must give exactly what smo_step with a caller workspace gives, call after
call (the shared array keeps the previous call's contents), and refuse a step
that needs more scratch than the array holds.  Collected last on purpose."""

import numpy as np
import pytest
import torch

from smo_optimizer_b200 import SMO8bit, _lib, synthetic

pytestmark = pytest.mark.gpu

SHAPES = [(1024, 1024), (384, 1152), (50, 30), (384, 10), (300,)]
KW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25, block_size=64,
          low_peak=True, band_mb=0.5)


class NoAllocSMO8bit(SMO8bit):
    """SMO8bit whose launches go through smo_step_no_alloc (no workspace)."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.statuses = []

    def _launch(self, dev, items):
        table = np.zeros(len(items), dtype=_lib.TENSOR_DTYPE)
        for i, (p, grad, state, group) in enumerate(items):
            self._fill(table[i], p, grad, state, group)
        status = torch.full((1,), -1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            rc = _lib.load().smo_step_no_alloc(table.ctypes.data, len(table), status.data_ptr(),
                                               torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "smo_step_no_alloc")
        self.statuses.append(status)
        for p, grad, state, group in items:
            self._swap(p, state)


def _make(cls):
    params = [torch.nn.Parameter(torch.from_numpy(synthetic.synth_param(21, i, s)).cuda())
              for i, s in enumerate(SHAPES)]
    return params, cls(params, **KW)


def test_no_alloc_step_matches_workspace_step_twice():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    pa, oa = _make(SMO8bit)
    pb, ob = _make(NoAllocSMO8bit)
    for step in (1, 2):
        for i, s in enumerate(SHAPES):
            g = torch.from_numpy(synthetic.synth_grad(21, step, i, s)).cuda()
            pa[i].grad = g
            pb[i].grad = g.clone()
        oa.step()
        ob.step()
        torch.cuda.synchronize()
        # bit-identical (the tests' tolerance for the library against itself is zero)
        for i, (a, b) in enumerate(zip(pa, pb)):
            assert torch.equal(a, b), f"step {step}: param {i} differs"
            sa, sb = oa.state[a], ob.state[b]
            for k in ("m_q", "m_s", "v_q", "v_s", "exp_avg", "exp_avg_sq"):
                if k in sa:
                    assert torch.equal(sa[k], sb[k]), f"step {step}: state {k} of param {i} differs"
        assert int(ob.statuses[-1].item()) == 0


def test_no_alloc_rejects_a_step_larger_than_its_scratch():
    # an adaptive-window tensor whose general-path scratch (8 B per compact cell)
    # exceeds the fixed array; rejected on the host before anything is enqueued
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    H, W, h, w = 8000, 6000, 2400, 1800
    nb = (h * w + 63) // 64
    t["kind"] = _lib.SMO_KIND_POOLED8
    t["rows"], t["cols"], t["comp_rows"], t["comp_cols"], t["q_block"] = H, W, h, w, 64
    base = 1 << 32
    for k_ in ("param", "grad", "m_q_in", "m_s_in", "v_q_in", "v_s_in", "m_q_out", "m_s_out", "v_q_out", "v_s_out"):
        t[k_] = base
        base += 1 << 28
    lib = _lib.load()
    assert nb > 0 and _lib.workspace_size(t) > (32 << 20)
    assert lib.smo_step_no_alloc(t.ctypes.data, 1, None, None) == 3  # SMO_ERR_WORKSPACE
