"""Parameter sets of the benchmark workloads (synthetic weights, no checkpoints).

Each workload is a list of ``(name, shape)`` pairs.  Names follow the
reference's models so that the ``protect_output`` grouping rule (a name that
contains ``"emb"`` or ``"head"`` is protected) selects the same tensors as
``make_optimizer`` in benchmarks/suites/comparison/t4_memory_benchmark.py:88-134.
Matrix shapes are written rows x cols of the 2-D row view the optimizer pools.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class Workload:
    name: str
    tensors: tuple  # ((name, shape), ...)
    optimizer: str  # "SMO8bit" | "SMO"
    kwargs: dict = field(default_factory=dict)
    protect_output: object = False
    bf16_grads: bool = False
    compress: object = True      # the group's compress setting (True, False = dense, "quant_only")
    general_path: bool = False   # pin the general two-launch kernels (SMO_FLAG_GENERAL_PATH)

    @property
    def numel(self) -> int:
        total = 0
        for _, shape in self.tensors:
            n = 1
            for s in shape:
                n *= s
            total += n
        return total


def _vit_tensors(width=384, depth=8, mlp=1536, patch_in=192, classes=10):
    t = [("patch_embed.weight", (patch_in, width)), ("patch_embed.bias", (width,))]
    for i in range(depth):
        p = f"blocks.{i}."
        t += [
            (p + "ln1.weight", (width,)), (p + "ln1.bias", (width,)),
            (p + "attn.in_proj_weight", (width, 3 * width)), (p + "attn.in_proj_bias", (3 * width,)),
            (p + "attn.out_proj.weight", (width, width)), (p + "attn.out_proj.bias", (width,)),
            (p + "ln2.weight", (width,)), (p + "ln2.bias", (width,)),
            (p + "mlp.fc1.weight", (width, mlp)), (p + "mlp.fc1.bias", (mlp,)),
            (p + "mlp.fc2.weight", (mlp, width)), (p + "mlp.fc2.bias", (width,)),
        ]
    t += [("ln_f.weight", (width,)), ("ln_f.bias", (width,)),
          ("head.weight", (width, classes)), ("head.bias", (classes,))]
    return tuple(t)


def _charlm_tensors(vocab=256, d=512, layers=12):
    t = [("tok_emb.weight", (vocab, d))]
    for i in range(layers):
        p = f"blocks.{i}."
        t += [
            (p + "ln1.weight", (d,)), (p + "ln1.bias", (d,)),
            (p + "attn.in_proj_weight", (d, 3 * d)), (p + "attn.in_proj_bias", (3 * d,)),
            (p + "attn.out_proj.weight", (d, d)), (p + "attn.out_proj.bias", (d,)),
            (p + "ln2.weight", (d,)), (p + "ln2.bias", (d,)),
            (p + "mlp.fc1.weight", (d, 4 * d)), (p + "mlp.fc1.bias", (4 * d,)),
            (p + "mlp.fc2.weight", (4 * d, d)), (p + "mlp.fc2.bias", (d,)),
        ]
    t += [("ln_f.weight", (d,)), ("ln_f.bias", (d,)), ("head.weight", (d, vocab))]
    return tuple(t)


def _decoder700m_tensors(d=1536, layers=24, vocab=50304):
    t = []
    for i in range(layers):
        p = f"blocks.{i}."
        t += [
            (p + "attn.qkv.weight", (d, 3 * d)),
            (p + "attn.proj.weight", (d, d)),
            (p + "mlp.fc1.weight", (d, 4 * d)),
            (p + "mlp.fc2.weight", (4 * d, d)),
        ]
    t.append(("tok_emb.weight", (vocab, d)))
    return tuple(t)


_HP = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)

WORKLOADS = {
    # single 1024x1024 weight, SMO8bit k=0.25, 100 steps (parity case)
    "single1024": Workload("single1024", (("weight", (1024, 1024)),), "SMO8bit",
                           dict(_HP, k_ratio=0.25, block_size=64)),
    # TinyViT-like ~14M, SMO8bit k=0.25
    "tinyvit_8bit": Workload("tinyvit_8bit", _vit_tensors(), "SMO8bit",
                             dict(_HP, k_ratio=0.25, block_size=64)),
    # same set, SMO-Spatial fp32 pooled moments k=0.5
    "tinyvit_spatial": Workload("tinyvit_spatial", _vit_tensors(), "SMO",
                                dict(_HP, k_ratio=0.5)),
    # char-LM ~40M, emb/head protected (dense moments), bf16 grads upcast
    "charlm40m": Workload("charlm40m", _charlm_tensors(), "SMO8bit",
                          dict(_HP, k_ratio=0.25, block_size=64),
                          protect_output=True, bf16_grads=True),
    # ~700M decoder, SMO8bit k=0.25 low_peak (row-banded)
    "decoder700m": Workload("decoder700m", _decoder700m_tensors(), "SMO8bit",
                            dict(_HP, k_ratio=0.25, block_size=64, low_peak=True)),
    # the first 4 layers of the ~700M decoder (113M params, ~1.4 GB of params and
    # grads: larger than L2, small enough for profiler captures)
    "decoder700m_4layers": Workload("decoder700m_4layers", _decoder700m_tensors()[:16], "SMO8bit",
                                    dict(_HP, k_ratio=0.25, block_size=64, low_peak=True)),
}


_MODES = {"": {}, "dense": dict(compress=False), "quant_only": dict(compress="quant_only"),
          "general": dict(general_path=True)}


def get(name: str) -> Workload:
    """A named workload, or ``RxCxN[@mode]``: N tensors of R x C with the 700M
    decoder's optimizer settings (a single-shape set, for per-shape
    measurements); ``@dense`` / ``@quant_only`` put them in a group with that
    ``compress`` setting, ``@general`` pins the general two-launch kernels."""
    if name in WORKLOADS:
        return WORKLOADS[name]
    shape, _, mode = name.partition("@")
    parts = shape.split("x")
    if len(parts) == 3 and all(x.isdigit() and int(x) > 0 for x in parts) and mode in _MODES:
        r, c, n = map(int, parts)
        base = WORKLOADS["decoder700m"]
        kwargs = dict(base.kwargs)
        if mode in ("dense", "quant_only"):
            kwargs.pop("low_peak", None)
        return Workload(name, tuple((f"w{i}", (r, c)) for i in range(n)), base.optimizer, kwargs, **_MODES[mode])
    raise KeyError(f"unknown workload {name!r}: one of {sorted(WORKLOADS)} or RxCxN[@dense|@quant_only|@general]")
