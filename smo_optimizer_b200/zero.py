"""ZeRO-1 sharding of the optimizer step across the ranks of one node.

Each rank owns a subset of the parameter tensors (chosen by a greedy
longest-processing-time partition on the step's algorithmic bytes), keeps the
optimizer state for those tensors only, steps them locally, and then the
updated parameters are broadcast from their owners so every replica holds the
same weights.  The reference has no distributed code; this is the build's own
multi-GPU layer.  Tensors are independent, so the step itself needs no
exchange: the only collective is the parameter broadcast/all-gather after it.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

from . import _host


def step_bytes(shape, kind: str, k_ratio: float = 0.25, block: int = 64, compress_conv: bool = False) -> int:
    """Algorithmic HBM bytes of one tensor's step (what the kernels must move).

    pooled int8: p r+w, g r (12 B/elem) + codes r+w (4 B/cell) + scales r+w (16 B/block);
    pooled fp32: 12 B/elem + 16 B/cell; dense fp32 Adam: 28 B/elem.
    """
    n = 1
    for s in shape:
        n *= int(s)
    view = _host.compression_view(shape, compress_conv)
    if view is None:
        return 28 * n
    h, w = _host.comp_shape(view[0], k_ratio)
    c = h * w
    if kind == "SMO8bit":
        qb = _host.pooled_q_block(view[1], (h, w), block)
        return 12 * n + 4 * c + 16 * _host.num_blocks(c, qb)
    return 12 * n + 16 * c


def lpt_partition(costs, world: int):
    """Owner rank of each item: greedy LPT (largest cost to the least-loaded rank).

    Deterministic: ties break on the lower rank and the lower item index.
    """
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + costs[i], r))
    return owner


def rank_loads(costs, owner, world: int):
    loads = [0] * world
    for c, r in zip(costs, owner):
        loads[r] += c
    return loads


class Zero1:
    """ZeRO-1 wrapper around ``SMO`` / ``SMO8bit``.

    ``Zero1(params, SMO8bit, lr=..., ...)`` builds the inner optimizer over the
    tensors this rank owns.  ``step()`` steps them and then broadcasts every
    tensor from its owner (NCCL over NVLink for CUDA tensors), so all ranks end
    the step with identical parameters.  ``state_dict()`` is this rank's shard.
    """

    def __init__(self, params, optimizer_cls, process_group=None, **kwargs):
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.params = [p for p in params]
        kind = optimizer_cls.__name__
        costs = [step_bytes(p.shape, kind, kwargs.get("k_ratio", kwargs.get("k") or 0.25),
                            kwargs.get("block_size", 64), kwargs.get("compress_conv", False)) for p in self.params]
        self.owner = lpt_partition(costs, self.world)
        self.costs = costs
        self.owned = [p for p, r in zip(self.params, self.owner) if r == self.rank]
        self.optimizer = optimizer_cls(self.owned, **kwargs) if self.owned else None

    @property
    def param_groups(self):
        return self.optimizer.param_groups if self.optimizer else []

    def local_step(self):
        if self.optimizer is not None:
            self.optimizer.step()

    def broadcast_params(self):
        """Every tensor from its owner to all ranks (one async broadcast each)."""
        if self.world == 1:
            return
        works = []
        for p, r in zip(self.params, self.owner):
            src = dist.get_global_rank(self.group, r) if self.group is not None else r
            works.append(dist.broadcast(p.data, src=src, group=self.group, async_op=True))
        for w in works:
            w.wait()

    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.local_step()
        self.broadcast_params()
        return loss

    def zero_grad(self, set_to_none: bool = True):
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def state_dict(self):
        return self.optimizer.state_dict() if self.optimizer else {"state": {}, "param_groups": []}
