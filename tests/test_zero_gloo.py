"""ZeRO-1 host logic on CPU ranks (gloo, world_size 2): the partition, the
flat all-gather and the per-tensor broadcast exchanges, and a rank failing
before the exchange.

The CUDA step cannot run on the CPU, so the ranks use a stand-in optimizer
(plain SGD on their owned tensors); what is under test is the sharding and the
collective plumbing around the step."""

import copy
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from smo_optimizer_b200 import zero


class StandIn(torch.optim.Optimizer):
    def __init__(self, params, lr=0.1, **_):
        super().__init__(params, dict(lr=lr))

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                p.add_(p.grad, alpha=-g["lr"])


class StandInMomentum(torch.optim.Optimizer):
    """Stand-in with per-parameter state (a step count and a moment tensor), so
    that the sharded state_dict paths have state to gather and scatter."""

    def __init__(self, params, lr=0.1, **_):
        super().__init__(params, dict(lr=lr))

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p)
                st["step"] += 1
                st["exp_avg"].mul_(0.9).add_(p.grad)
                p.add_(st["exp_avg"], alpha=-g["lr"])


SHAPES = [(64, 256), (128, 128), (32, 32), (300,), (256, 64), (96, 96), (1024,)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(s, generator=g) for s in SHAPES]


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        params = [torch.nn.Parameter(t) for t in _params(0)]
        grads = _params(1)
        for p, g in zip(params, grads):
            p.grad = g.clone() * (rank + 1 if mode == "rs" else 1)
        z = zero.Zero1(params, StandIn, lr=0.5, flat=(mode != "bcast"), reduce_grads=(mode == "rs"))
        if mode != "bcast":
            # every parameter is a 256-byte aligned view of the one flat buffer
            base = z.flat.buffer.data_ptr()
            assert all(p.data_ptr() % 256 == base % 256 and
                       base <= p.data_ptr() < base + z.flat.buffer.numel() * 4 for p in params)
        else:
            assert z.flat is None
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # this rank dies before the broadcast
        t0 = time.time()
        try:
            z.step()
            result = [p.detach().clone() for p in params]
            if mode == "rs":
                # zero_grad keeps every gradient a view of the flat buffer, zeroed
                z.zero_grad()
                base = z.flat.grad_buffer.data_ptr()
                end = base + z.flat.grad_buffer.numel() * 4
                assert all(p.grad is not None and base <= p.grad.data_ptr() < end for p in params)
                assert float(z.flat.grad_buffer.abs().sum()) == 0.0
            out[rank] = ("ok", result, z.owner)
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            out[rank] = ("error", type(e).__name__, time.time() - t0)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _state_worker(rank, world, port, full_in, out):
    """Three sharded steps, the full state gathered to rank 0; then a fresh
    Zero1 loads a single-process state dict and takes one more step."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        params = [torch.nn.Parameter(t) for t in _params(0)]
        z = zero.Zero1(params, StandInMomentum, lr=0.5)
        for step in range(3):
            for p, g in zip(params, _params(10 + step)):
                p.grad = g
            z.step()
        full = z.full_state_dict()
        params2 = [torch.nn.Parameter(t.clone()) for t in full_in["params"]]
        z2 = zero.Zero1(params2, StandInMomentum, lr=0.5)
        # tensors handed to a spawned process share the parent's storage; the
        # loaded state is stepped in place, so load a private copy
        z2.load_full_state_dict(copy.deepcopy(full_in["sd"]))
        for p, g in zip(params2, _params(13)):
            p.grad = g
        z2.step()
        out[rank] = ("ok", full, [p.detach().clone() for p in params2])
    except Exception as e:
        out[rank] = ("error", repr(e), None)
    finally:
        dist.destroy_process_group()


def _run(mode, target=None, args=()):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    target = target or _worker
    procs = [ctx.Process(target=target, args=(r, 2, port) + (args or (mode,)) + (out,)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return dict(out), [p.exitcode for p in procs]


def test_lpt_partition_is_deterministic_and_balanced():
    costs = [zero.step_bytes(s, "SMO8bit") for s in SHAPES * 5]
    owner = zero.lpt_partition(costs, 4)
    assert owner == zero.lpt_partition(costs, 4)
    loads = zero.rank_loads(costs, owner, 4)
    assert max(loads) <= min(loads) + max(costs)
    assert zero.lpt_partition(costs, 1) == [0] * len(costs)


def test_flat_layout_is_rank_contiguous_and_padded():
    params = [torch.nn.Parameter(t) for t in _params(0)]
    owner = [0, 1, 1, 0, 1, 0, 0]
    f = zero.FlatParams(params, owner, 2, 1)
    ref = [t.clone() for t in _params(0)]
    f.bind()
    sizes = [0, 0]
    for p, r, off, e in zip(params, owner, f.offsets, ref):
        assert off == sizes[r] and off % 64 == 0
        sizes[r] += (p.numel() + 63) // 64 * 64
        assert torch.equal(p.data, e)
        assert p.data.data_ptr() == f.buffer.data_ptr() + 4 * (r * f.shard + off)
    assert f.shard == max(sizes) and f.local_slot().numel() == f.shard
    assert f.bytes_per_rank == 4 * f.shard
    with pytest.raises(ValueError):
        zero.FlatParams([torch.zeros(4), torch.zeros(4, dtype=torch.float64)], [0, 1], 2, 0)


def test_step_bytes_formula():
    # pooled int8, 1024x1024 at k=0.25: 12 B/param + 4 B/cell + 16 B/block
    assert zero.step_bytes((1024, 1024), "SMO8bit") == 12 * 1024 * 1024 + 4 * 65536 + 16 * 1024
    assert zero.step_bytes((300,), "SMO8bit") == 28 * 300
    assert zero.step_bytes((1024, 1024), "SMO", k_ratio=0.5) == 12 * 1024 * 1024 + 16 * 512 * 512


@pytest.mark.parametrize("mode", ["ok", "bcast", "rs"])
def test_zero1_exchange_makes_replicas_identical(mode):
    out, codes = _run(mode)
    assert codes == [0, 0]
    (s0, p0, own0), (s1, p1, own1) = out[0], out[1]
    assert s0 == s1 == "ok" and own0 == own1 and set(own0) == {0, 1}
    # "rs": rank r's gradients are (r + 1) g; the reduce-scatter averages them to 1.5 g
    scale = 1.5 if mode == "rs" else 1.0
    expected = [p - 0.5 * scale * g for p, g in zip(_params(0), _params(1))]
    for a, b, e in zip(p0, p1, expected):
        assert torch.equal(a, b)
        assert torch.allclose(a, e)


def test_rank_failure_before_broadcast_surfaces_as_error():
    out, codes = _run("fail")
    assert codes[1] == 3
    status = out[0]
    assert status[0] == "error", status
    assert status[2] < 60.0


def test_full_state_dict_gathers_and_reloads_across_world_sizes():
    """full_state_dict() on two ranks equals the state dict of one process
    stepping every tensor; a single-process state dict loaded into a sharded
    Zero1 continues exactly as the single process does."""
    params = [torch.nn.Parameter(t) for t in _params(0)]
    single = StandInMomentum(params, lr=0.5)
    for step in range(3):
        for p, g in zip(params, _params(10 + step)):
            p.grad = g
        single.step()
    sd = copy.deepcopy(single.state_dict())  # state_dict() holds live references
    snap = [p.detach().clone() for p in params]
    for p, g in zip(params, _params(13)):
        p.grad = g
    single.step()
    out, codes = _run(None, _state_worker, ({"sd": sd, "params": snap},))
    assert codes == [0, 0]
    assert out[0][0] == out[1][0] == "ok", (out[0][1], out[1][1])
    full = out[0][1]
    assert out[1][1] is None
    assert sorted(full["state"]) == list(range(len(SHAPES)))
    assert full["param_groups"][0]["params"] == list(range(len(SHAPES)))
    assert full["param_groups"][0]["lr"] == 0.5
    for i in range(len(SHAPES)):
        assert full["state"][i]["step"] == sd["state"][i]["step"] == 3
        assert torch.equal(full["state"][i]["exp_avg"], sd["state"][i]["exp_avg"])
    for rank in (0, 1):
        for a, b in zip(out[rank][2], params):
            assert torch.equal(a, b)
