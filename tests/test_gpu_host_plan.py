"""The C++ host path of the optimizer step (one call per step,
csrc/smo_host.cpp) gives exactly what the Python path gives, and hands the
step back to the Python path whenever something it relies on has changed."""

import copy

import pytest
import torch

from smo_optimizer_b200 import SMO, SMO8bit, synthetic

pytestmark = pytest.mark.gpu

SHAPES = [(512, 1536), (384, 1152), (50, 30), (384, 10), (300,), (64, 48), (96, 192)]
KW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25)
KW8 = dict(KW, block_size=64, low_peak=True, band_mb=0.5)
STATE_KEYS = ("m_q", "m_s", "v_q", "v_s", "exp_avg", "exp_avg_sq")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")


def _make(cls, dtype, python_only):
    params = [torch.nn.Parameter(torch.from_numpy(synthetic.synth_param(40, i, s)).cuda().to(dtype))
              for i, s in enumerate(SHAPES)]
    if cls is SMO8bit:
        groups = [{"params": params[:5]}, {"params": params[5:6], "compress": "quant_only"},
                  {"params": params[6:], "lr": 2e-3}]
        opt = cls(groups, **KW8)
    else:
        groups = [{"params": params[:6]}, {"params": params[6:], "lr": 2e-3}]
        opt = cls(groups, **KW)
    if python_only:
        opt._plan_misses = 1 << 30  # the plan stays off: every step takes the Python path
    return params, opt


def _set_grads(params, step, dtype):
    for i, (p, s) in enumerate(zip(params, SHAPES)):
        p.grad = torch.from_numpy(synthetic.synth_grad(40, step, i, s)).cuda().to(dtype)


def _bits(t):
    """The tensor's bit patterns (NaN compares equal to the same NaN)."""
    t = t.detach()
    return t.view({4: torch.int32, 2: torch.int16, 1: torch.int8}[t.element_size()])


def _assert_same(pa, oa, pb, ob, what):
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(pa, pb)):
        assert torch.equal(_bits(a), _bits(b)), f"{what}: param {i}"
        sa, sb = oa.state[a], ob.state[b]
        assert sa["step"] == sb["step"], f"{what}: step of param {i}"
        for k in STATE_KEYS:
            if k in sa:
                assert torch.equal(_bits(sa[k]), _bits(sb[k])), f"{what}: state {k} of param {i}"


def _fast_step(opt):
    """One step that must go through the plan (it exists before and after)."""
    plan = opt._plan
    assert plan is not None
    opt.step()
    assert opt._plan is plan and opt._plan_misses == 0


@pytest.mark.parametrize("cls,dtype", [(SMO8bit, torch.float32), (SMO, torch.float32),
                                       (SMO8bit, torch.bfloat16), (SMO, torch.float16)])
def test_plan_matches_python_path(cls, dtype):
    pa, oa = _make(cls, dtype, python_only=False)
    pb, ob = _make(cls, dtype, python_only=True)
    for step in range(1, 7):
        _set_grads(pa, step, dtype)
        _set_grads(pb, step, dtype)
        if step == 4:  # a schedule changes the learning rate between steps
            for o in (oa, ob):
                o.param_groups[0]["lr"] = 5e-4
                o.param_groups[-1]["betas"] = [0.85, 0.995]
        if step == 1:
            oa.step()
        else:
            _fast_step(oa)
        ob.step()
        _assert_same(pa, oa, pb, ob, f"step {step}")
    assert ob._plan is None
    oa.check_device_status()


def test_plan_hands_back_when_its_assumptions_change():
    dt = torch.float32
    pa, oa = _make(SMO8bit, dt, python_only=False)
    pb, ob = _make(SMO8bit, dt, python_only=True)

    def both(fn):
        fn(pa, oa)
        fn(pb, ob)

    for step in range(1, 11):
        _set_grads(pa, step, dt)
        _set_grads(pb, step, dt)
        if step == 3:    # a parameter without a gradient is skipped
            pa[2].grad = pb[2].grad = None
        if step == 5:    # a strided gradient of a dense parameter is copied to the parameter's layout
            both(lambda ps, o: setattr(ps[4], "grad", ps[4].grad.repeat(2)[::2]))
        if step == 7:    # a state restored from a snapshot
            snap_a, snap_b = copy.deepcopy(oa.state_dict()), copy.deepcopy(ob.state_dict())
            oa.load_state_dict(snap_a)
            ob.load_state_dict(snap_b)
            assert oa._plan is None
        if step == 9:    # a moment buffer replaced by the user
            both(lambda ps, o: o.state[ps[0]].__setitem__("m_s", o.state[ps[0]]["m_s"].clone()))
        plan = oa._plan
        oa.step()
        ob.step()
        fast = plan is not None and oa._plan is plan
        # the plan runs where its assumptions hold; steps 3-5 and 9 change one,
        # steps 1, 6 and 7 start without a plan (first step, a strided
        # gradient at step 5 builds none, a loaded state drops it)
        assert fast == (step in (2, 8, 10)), f"step {step}: plan taken = {fast}"
        _assert_same(pa, oa, pb, ob, f"step {step}")
    oa.check_device_status()


def test_subclass_with_its_own_launch_keeps_the_python_path():
    class Own(SMO8bit):
        calls = 0

        def _launch(self, dev, items):
            Own.calls += 1
            super()._launch(dev, items)

    params = [torch.nn.Parameter(torch.from_numpy(synthetic.synth_param(41, i, s)).cuda())
              for i, s in enumerate(SHAPES[:3])]
    opt = Own(params, **KW8)
    for step in range(1, 4):
        for i, p in enumerate(params):
            p.grad = torch.from_numpy(synthetic.synth_grad(41, step, i, SHAPES[i])).cuda()
        opt.step()
    assert Own.calls == 3 and opt._plan is None
