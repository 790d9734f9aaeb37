"""ZeRO-1 over NCCL on two GPUs (one process per GPU): after three steps the
sharded step leaves every rank's parameters, and the owner's optimizer state
of each tensor, bit-identical to SMO8bit stepping every tensor on one GPU.

Run both without gradient exchange (every rank holds the same gradients, as a
replicated backward after an all-reduce would leave them) and with the
ZeRO-2 communication pattern (each rank holds its own gradients; one
reduce-scatter averages them into the owner's slot), against one GPU stepping
the averaged gradients.  Needs two GPUs; skipped otherwise."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(512, 1536), (1536, 512), (384, 1152), (1024, 1024), (1536,), (256, 256)]
KW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25, block_size=64, low_peak=True)
STATE_KEYS = ("m_q", "m_s", "v_q", "v_s", "exp_avg", "exp_avg_sq")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads(step, rank):
    """Gradients of rank `rank` at `step`: shared part plus a rank-dependent
    part that the reduce-scatter averages away."""
    from smo_optimizer_b200 import synthetic
    out = []
    for i, s in enumerate(SHAPES):
        g = synthetic.synth_grad(50, step, i, s)
        if rank is not None:
            g = g + np.float32(rank) * synthetic.synth_grad(51, step, i, s)
        out.append(g)
    return out


def _worker(rank, world, port, reduce_grads, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from smo_optimizer_b200 import SMO8bit, synthetic, zero
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        init = [synthetic.synth_param(50, i, s) for i, s in enumerate(SHAPES)]
        params = [torch.nn.Parameter(torch.from_numpy(a.copy()).to(dev)) for a in init]
        z = zero.Zero1(params, SMO8bit, reduce_grads=reduce_grads, **KW)
        for step in range(1, 4):
            gs = _grads(step, rank if reduce_grads else None)
            for p, g in zip(params, gs):
                if reduce_grads:
                    p.grad.copy_(torch.from_numpy(g).to(dev))  # the gradient views of the flat buffer
                else:
                    p.grad = torch.from_numpy(g).to(dev)
            z.step()
        torch.cuda.synchronize(dev)
        if z.optimizer is not None:
            z.optimizer.check_device_status()

        # the same steps on this GPU alone, every tensor, averaged gradients
        ref = [torch.nn.Parameter(torch.from_numpy(a.copy()).to(dev)) for a in init]
        opt = SMO8bit(ref, **KW)
        for step in range(1, 4):
            if reduce_grads:
                # what the reduce-scatter computes: the two ranks' sum, then / 2
                g0, g1 = _grads(step, 0), _grads(step, 1)
                gs = [(torch.from_numpy(a).to(dev) + torch.from_numpy(b).to(dev)) / world for a, b in zip(g0, g1)]
            else:
                gs = [torch.from_numpy(g).to(dev) for g in _grads(step, None)]
            for p, g in zip(ref, gs):
                p.grad = g
            opt.step()
        torch.cuda.synchronize(dev)
        opt.check_device_status()

        bad = []
        for i, (p, r) in enumerate(zip(params, ref)):
            if not torch.equal(p.detach(), r.detach()):
                bad.append(f"param {i}")
            if z.owner[i] == rank:
                for k in STATE_KEYS:
                    if k in opt.state[r] and not torch.equal(z.optimizer.state[p][k], opt.state[r][k]):
                        bad.append(f"state {k} of {i}")
        out[rank] = ("ok", bad, list(z.owner))
    except Exception as e:  # pragma: no cover - reported to the parent
        out[rank] = ("error", repr(e), None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("reduce_grads", [False, True])
def test_zero1_two_gpus_bit_identical_to_one_gpu(reduce_grads):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, reduce_grads, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    assert [p.exitcode for p in procs] == [0, 0]
    r0, r1 = out[0], out[1]
    assert r0[0] == "ok" and r1[0] == "ok", (r0, r1)
    assert r0[2] == r1[2] and set(r0[2]) == {0, 1}
    assert r0[1] == [] and r1[1] == [], (r0[1], r1[1])
