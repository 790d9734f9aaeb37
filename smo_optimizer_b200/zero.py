"""ZeRO-1 sharding of the optimizer step across the ranks of one node.

Each rank owns a subset of the parameter tensors (chosen by a greedy
longest-processing-time partition on the step's algorithmic bytes), keeps the
optimizer state for those tensors only, steps them locally, and then the
updated parameters are exchanged so every replica holds the same weights.
The reference has no distributed code; this is the build's own multi-GPU
layer.  Tensors are independent, so the step itself needs no exchange: the
only collective is the parameter exchange after it.

Two exchanges:
  * flat (default when every parameter has the same device and dtype): the
    parameters are rebound to views of one rank-contiguous buffer (rank r's
    tensors in slot r, slots padded to the largest rank's size), so one
    in-place all-gather completes the step, with every link busy in both
    directions;
  * per tensor: an async broadcast of each tensor from its owner.

With ``reduce_grads=True`` the gradients live in a second flat buffer of the
same layout (``p.grad`` are views of it) and one reduce-scatter before the
local step leaves every rank the summed (by default averaged) gradients of the
tensors it owns: the communication pattern of ZeRO-2 (reduce-scatter of
gradients, local step, all-gather of parameters) in place of a full
all-reduce.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

from . import _host


def step_bytes(shape, kind: str, k_ratio: float = 0.25, block: int = 64, compress_conv: bool = False,
               elem: int = 4, compress=True) -> int:
    """Algorithmic HBM bytes of one tensor's step (what the kernels must move),
    for parameters of ``elem`` bytes (the state's floats have the same size)
    in a group with the given ``compress`` setting.

    pooled int8: p r+w, g r (3 elem B/elem) + codes r+w (4 B/cell) + scales r+w (4 elem B/block);
    pooled float: 3 elem B/elem + 4 elem B/cell; dense Adam: 7 elem B/elem;
    quant_only: 3 elem B/elem + codes r+w (4 B/elem) + scales r+w (4 elem B/block).
    """
    n = 1
    for s in shape:
        n *= int(s)
    if compress == "quant_only":
        qb = _host.quant_only_q_block(shape, block)
        return 3 * elem * n + 4 * n + 4 * elem * _host.num_blocks(n, qb)
    view = _host.compression_view(shape, compress_conv) if compress else None
    if view is None:
        return 7 * elem * n
    h, w = _host.comp_shape(view[0], k_ratio)
    c = h * w
    if kind == "SMO8bit":
        qb = _host.pooled_q_block(view[1], (h, w), block)
        return 3 * elem * n + 4 * c + 4 * elem * _host.num_blocks(c, qb)
    return 3 * elem * n + 4 * elem * c


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


class FlatParams:
    """Rank-contiguous flat parameter buffer for the one-collective exchange.

    Rank r's owned tensors sit one after another in slot r of ``buffer``
    (``shard`` elements per slot, the largest rank's total rounded up); each
    tensor starts on a 64-element (256-byte) boundary, which keeps the fused
    kernel's 16-byte vector loads aligned.  ``bind()`` copies every parameter
    into its place and rebinds ``p.data`` to that view.
    """

    ALIGN = 64

    def __init__(self, params, owner, world: int, rank: int):
        params = list(params)
        if not params:
            raise ValueError("no parameters")
        dev, dtype = params[0].device, params[0].dtype
        if any(p.device != dev or p.dtype != dtype for p in params):
            raise ValueError("flat exchange needs one device and one dtype for every parameter")
        self.params, self.owner, self.world, self.rank = params, list(owner), world, rank
        fill = [0] * world
        self.offsets = []
        for p, r in zip(params, self.owner):
            self.offsets.append(fill[r])
            fill[r] += (p.numel() + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        self.shard = max(max(fill), self.ALIGN)
        self.buffer = torch.zeros(world * self.shard, dtype=dtype, device=dev)
        self.grad_buffer = None

    def bind(self):
        with torch.no_grad():
            for p, r, off in zip(self.params, self.owner, self.offsets):
                view = self.buffer.narrow(0, r * self.shard + off, p.numel()).view(p.shape)
                view.copy_(p.data)
                p.data = view
        return self

    def local_slot(self):
        return self.buffer.narrow(0, self.rank * self.shard, self.shard)

    def bind_grads(self):
        """Gradients as views of one flat buffer of the parameter layout (existing
        gradients are copied in); backward accumulates into the views."""
        self.grad_buffer = torch.zeros_like(self.buffer)
        with torch.no_grad():
            for p, r, off in zip(self.params, self.owner, self.offsets):
                view = self.grad_buffer.narrow(0, r * self.shard + off, p.numel()).view(p.shape)
                if p.grad is not None:
                    view.copy_(p.grad)
                p.grad = view
        return self

    def reduce_scatter_grads(self, group=None, average: bool = True, async_op: bool = False):
        """Sum every rank's gradients into the owner's slot, in place (this
        rank's slot of the gradient buffer), divided by the world size when
        ``average``; the other slots keep this rank's own gradients."""
        slot = self.grad_buffer.narrow(0, self.rank * self.shard, self.shard)
        work = dist.reduce_scatter_tensor(slot, self.grad_buffer, op=dist.ReduceOp.SUM, group=group,
                                          async_op=async_op)
        if average:
            if work is not None:
                work.wait()
                work = None
            slot.div_(self.world)
        return work

    def all_gather(self, group=None, async_op: bool = False):
        """Every rank's slot to every rank, in place (input = this rank's slot)."""
        return dist.all_gather_into_tensor(self.buffer, self.local_slot(), group=group, async_op=async_op)

    @property
    def bytes_per_rank(self) -> int:
        return (self.world - 1) * self.shard * self.buffer.element_size()


class Zero1:
    """ZeRO-1 wrapper around ``SMO`` / ``SMO8bit``.

    ``Zero1(params, SMO8bit, lr=..., ...)`` builds the inner optimizer over the
    tensors this rank owns.  ``step()`` steps them and then exchanges the
    updated tensors (NCCL over NVLink for CUDA tensors), so all ranks end the
    step with identical parameters.  ``state_dict()`` is this rank's shard.

    ``flat=True`` (default) rebinds the parameters to views of one flat
    buffer (see ``FlatParams``) and exchanges with a single all-gather; it
    falls back to per-tensor broadcasts when the parameters differ in device
    or dtype.  ``flat=False`` always broadcasts per tensor.
    """

    def __init__(self, params, optimizer_cls, process_group=None, flat: bool = True, reduce_grads: bool = False,
                 average_grads: bool = True, **kwargs):
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.params = [p for p in params]
        kind = optimizer_cls.__name__
        costs = [step_bytes(p.shape, kind, kwargs.get("k_ratio", kwargs.get("k") or 0.25),
                            kwargs.get("block_size", 64), kwargs.get("compress_conv", False)) for p in self.params]
        self.owner = lpt_partition(costs, self.world)
        self.costs = costs
        self.flat = None
        if flat and self.world > 1 and len({(p.device, p.dtype) for p in self.params}) == 1:
            self.flat = FlatParams(self.params, self.owner, self.world, self.rank).bind()
        self.reduce_grads = bool(reduce_grads)
        self.average_grads = bool(average_grads)
        if self.reduce_grads:
            if self.world > 1 and self.flat is None:
                raise ValueError("reduce_grads needs the flat layout (one device and dtype for every parameter)")
            if self.flat is not None:
                self.flat.bind_grads()
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

    def exchange_params(self):
        """Bring every rank's updated tensors to all ranks."""
        if self.world == 1:
            return
        if self.flat is not None:
            self.flat.all_gather(self.group)
        else:
            self.broadcast_params()

    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self.reduce_grads and self.flat is not None:
            self.flat.reduce_scatter_grads(self.group, average=self.average_grads)
        self.local_step()
        self.exchange_params()
        return loss

    def step_async(self):
        """``step()`` with the parameter exchange left in flight: the gradient
        reduce-scatter (``reduce_grads=True``) and the local step are enqueued,
        the flat all-gather is issued asynchronously, and its work handle is
        returned (None on one rank, or when the per-tensor broadcast exchange
        is in use, which completes before returning).  Call ``wait()`` on it
        before anything reads the parameters (the next forward); host work in
        between overlaps the exchange."""
        if self.reduce_grads and self.flat is not None:
            self.flat.reduce_scatter_grads(self.group, average=self.average_grads)
        self.local_step()
        if self.world == 1:
            return None
        if self.flat is not None:
            return self.flat.all_gather(self.group, async_op=True)
        self.broadcast_params()
        return None

    def zero_grad(self, set_to_none: bool = True):
        if self.reduce_grads and self.flat is not None:
            self.flat.grad_buffer.zero_()  # the gradient views stay bound
            return
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def state_dict(self):
        return self.optimizer.state_dict() if self.optimizer else {"state": {}, "param_groups": []}

    def load_state_dict(self, state_dict):
        """Load this rank's shard (what ``state_dict()`` returned on the same rank)."""
        if self.optimizer is not None:
            self.optimizer.load_state_dict(state_dict)

    def _local_params(self):
        if self.optimizer is None:
            return []
        return [p for g in self.optimizer.param_groups for p in g["params"]]

    def full_state_dict(self, dst: int = 0):
        """The whole optimizer state in the single-process layout, on rank
        ``dst`` of the process group (None on the other ranks): ``state`` keyed
        by each parameter's position in the list given to the constructor and
        one param group holding all of them, i.e. what the wrapped class returns
        when one process steps every parameter (for SMO8bit / SMO the
        reference's layout, smo/optimizers/spatial_8bit.py:155-208).  State
        tensors are moved to the CPU.  Every rank must call it (one gather)."""
        index = {id(p): i for i, p in enumerate(self.params)}
        local = self.state_dict()
        shard = {}
        for li, p in enumerate(self._local_params()):
            st = local["state"].get(li)
            if st is not None:
                shard[index[id(p)]] = {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in st.items()}
        hyper = [{k: v for k, v in g.items() if k != "params"} for g in local["param_groups"]]
        if len(hyper) > 1:
            raise ValueError("full_state_dict supports a wrapped optimizer with one param group")
        if self.world == 1:
            gathered = [(shard, hyper)]
        else:
            root = dist.get_global_rank(self.group, dst) if self.group is not None else dst
            gathered = [None] * self.world if self.rank == dst else None
            dist.gather_object((shard, hyper), gathered, dst=root, group=self.group)
            if self.rank != dst:
                return None
        state = {}
        for sh, _ in gathered:
            state.update(sh)
        group = next((h[0] for _, h in gathered if h), {})
        return {"state": dict(sorted(state.items())),
                "param_groups": [dict(group, params=list(range(len(self.params))))]}

    def load_full_state_dict(self, state_dict):
        """Load a single-process state dict (from ``full_state_dict()`` at any
        world size, or saved by one process stepping every parameter with the
        wrapped class) into this rank's shard: the entries of the parameters
        this rank owns under the current partition.  Every rank passes the
        same dict."""
        if self.optimizer is None:
            return
        index = {id(p): i for i, p in enumerate(self.params)}
        local = self._local_params()
        full = state_dict["state"]
        state = {}
        for li, p in enumerate(local):
            gi = index[id(p)]
            if gi in full:
                state[li] = full[gi]
        group = {k: v for k, v in state_dict["param_groups"][0].items() if k != "params"}
        self.optimizer.load_state_dict({"state": state, "param_groups": [dict(group, params=list(range(len(local))))]})
