"""GPU parity at the benchmarked configurations, and the step's failure paths.

* Every benchmark workload (the TinyViT SMO8bit and SMO sets, the char-LM set
  with protected embedding/head and bf16-drawn gradients, and the whole ~700M
  decoder set in low_peak mode) is stepped three times through the drop-in
  optimizer and compared with the CPU oracle bit for bit: every parameter and
  every state tensor.  Inputs are drawn on the device with the library's
  synthetic generator and copied to the host for the oracle, so both sides see
  the same bits.
* The fused kernel's strip-ready flags live in a region nothing else writes:
  general-path scratch holding float bit patterns equal to the next launch
  epoch does not disturb the next step.
* The fused kernel's own bounded wait, made to wait for a flag value that no
  strip publishes, with a short poll limit, on a many-strip tensor: the launch
  returns, the device status reports SMO_ERR_TIMEOUT, the optimizer raises,
  and a step after normal operation is restored is correct again.
"""

import copy
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from smo_optimizer_b200 import SMO, SMO8bit, _lib, ops, protected_param_groups, synthetic, workloads

pytestmark = pytest.mark.gpu

STATE_KEYS = ("m_q", "m_s", "v_q", "v_s", "exp_avg", "exp_avg_sq")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    _lib.load()
    oracle.set_num_threads(os.cpu_count() or 1)


def host(t):
    return t.detach().cpu().numpy()


def _device_grad(seed, step, i, shape, bf16):
    g = torch.empty(shape, dtype=torch.float32, device="cuda")
    ops.synth_normal_(g, seed, synthetic.stream_id(synthetic.STREAM_GRAD, step, i), 1e-3)
    if bf16:
        g = g.to(torch.bfloat16).to(torch.float32)  # round to nearest even, as synthetic.round_to_bf16
    return g


@pytest.mark.parametrize("name", ["tinyvit_8bit", "tinyvit_spatial", "charlm40m", "decoder700m"])
def test_workload_bit_exact_vs_oracle(name):
    wl = workloads.WORKLOADS[name]
    seed, steps = 3, 3
    named = []
    for i, (pname, shape) in enumerate(wl.tensors):
        p = torch.empty(shape, dtype=torch.float32, device="cuda")
        ops.synth_normal_(p, seed, synthetic.stream_id(synthetic.STREAM_PARAM, 0, i), 0.02)
        named.append((pname, torch.nn.Parameter(p)))
    ref_named = [(n, host(p).copy()) for n, p in named]
    cls = SMO8bit if wl.optimizer == "SMO8bit" else SMO
    if wl.protect_output:
        opt = cls(named, protect_output=wl.protect_output, **wl.kwargs)
        groups = protected_param_groups(ref_named, wl.protect_output, quant_capable=wl.optimizer == "SMO8bit")
    else:
        opt = cls([p for _, p in named], **wl.kwargs)
        groups = [{"params": [a for _, a in ref_named]}]
    ref = oracle.OracleOptimizer(wl.optimizer, groups, **wl.kwargs)
    # oracle order: group by group; map each oracle slot to its tensor index
    index_of = {id(a): i for i, (_, a) in enumerate(ref_named)}
    order = [index_of[id(a)] for _, _, a in ref.params()]
    keys = [k for k, _, _ in ref.params()]
    for step in range(1, steps + 1):
        grads = [_device_grad(seed, step, i, shape, wl.bf16_grads) for i, (_, shape) in enumerate(wl.tensors)]
        for (_, p), g in zip(named, grads):
            p.grad = g
        opt.step()
        ref.step([host(grads[i]) for i in order])
        del grads
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    for k, i in zip(keys, order):
        p = named[i][1]
        st, rst = opt.state[p], ref.state[k]
        for key in STATE_KEYS:
            if key in rst:
                assert np.array_equal(host(st[key]).reshape(-1), np.asarray(rst[key]).reshape(-1)), \
                    f"{name}: {named[i][0]} {tuple(p.shape)} state {key} differs from the oracle"
        assert np.array_equal(host(p).view(np.uint32).reshape(-1), ref_named[i][1].view(np.uint32).reshape(-1)), \
            f"{name}: {named[i][0]} {tuple(p.shape)} param differs from the oracle"


def test_flag_words_survive_general_scratch():
    """A step that mixes a fused tensor with a general-path int8 tensor whose
    post-EMA moments are the float bit patterns of small integers (denormals
    equal to the next launch epochs): the next steps stay bit-exact, because
    the flag words the fused kernel waits on are never written by the general
    path's scratch."""
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, k_ratio=0.25, block_size=64)
    # fused (300 compact rows in many strips) and general (W <= 128: 100 x 32 compact cells)
    shapes = [(4 * 300, 4 * 384), (400, 128)]
    p0 = [synthetic.synth_param(40, i, s) for i, s in enumerate(shapes)]
    ps = [torch.nn.Parameter(torch.from_numpy(a.copy()).cuda()) for a in p0]
    opt = SMO8bit(ps, **kw)
    ref_p = [a.copy() for a in p0]
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": ref_p}], **kw)
    denorm = np.float32(np.ldexp(1.0, -149))
    for step in range(1, 5):
        gs = [synthetic.synth_grad(40, step, i, s) for i, s in enumerate(shapes)]
        if step == 1:
            # compact cell c of the general tensor gets a uniform 4x4 window of
            # 10k * 2^-149, so its first post-EMA m is RN(0.1 * 10k * 2^-149)
            # = k * 2^-149: the bit pattern k = 1..8 (the epoch of the second
            # step's fused launch is 2)
            for c in range(128):
                k = c % 8 + 1
                r, q = (c // 32) * 4, (c % 32) * 4
                gs[1][r:r + 4, q:q + 4] = np.float32(10 * k) * denorm
        for p, g in zip(ps, gs):
            p.grad = torch.from_numpy(g).cuda()
        opt.step()
        ref.step(gs)
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    keys = [k for k, _, _ in ref.params()]
    for i, (p, k) in enumerate(zip(ps, keys)):
        for key in ("m_q", "m_s", "v_q", "v_s"):
            assert np.array_equal(host(opt.state[p][key]).reshape(-1), ref.state[k][key].reshape(-1)), (i, key)
        assert np.array_equal(host(p).view(np.uint32), ref_p[i].view(np.uint32)), f"param {i}"


def test_fused_wait_timeout_reports_and_recovers():
    lib = _lib.load()
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25, block_size=64,
              low_peak=True)
    shape = (4 * 2048, 4 * 384)  # 2048 compact rows: hundreds of strips, each waiting on its predecessor
    p0 = synthetic.synth_param(41, 0, shape)
    p = torch.nn.Parameter(torch.from_numpy(p0.copy()).cuda())
    opt = SMO8bit([p], **kw)
    ref_p = p0.copy()
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": [ref_p]}], **kw)
    g1 = synthetic.synth_grad(41, 1, 0, shape)
    p.grad = torch.from_numpy(g1).cuda()
    opt.step()
    ref.step([g1])
    opt.check_device_status()
    snap_p = p.detach().clone()
    snap_s = copy.deepcopy(opt.state_dict())

    g2 = synthetic.synth_grad(41, 2, 0, shape)
    p.grad = torch.from_numpy(g2).cuda()
    prev = lib.smo_set_wait_limit(1000)
    prev_inject = lib.smo_inject_wait_timeout(1)
    try:
        opt.step()                      # every strip after the first waits for a flag nothing sets
        torch.cuda.synchronize()        # the launch returns
    finally:
        lib.smo_inject_wait_timeout(prev_inject)
        lib.smo_set_wait_limit(prev)
    with pytest.raises(_lib.SmoError, match="bounded device wait timed out"):
        opt.check_device_status()
    assert opt.workspace_status() == 0  # read and cleared

    # restore the state of step 1 and redo step 2 with the default limit
    with torch.no_grad():
        p.copy_(snap_p)
    opt.load_state_dict(snap_s)
    p.grad = torch.from_numpy(g2).cuda()
    opt.step()
    ref.step([g2])
    opt.check_device_status()
    st, rst = opt.state[p], ref.state[(0, 0)]
    for key in ("m_q", "m_s", "v_q", "v_s"):
        assert np.array_equal(host(st[key]).reshape(-1), rst[key].reshape(-1)), key
    assert np.array_equal(host(p).view(np.uint32), ref_p.view(np.uint32))
