"""Parity cases shared by the golden-vector generator and the tests.

Each case is a list of parameter tensors (synthetic, seeded), an optimizer
class name with constructor kwargs, optional param groups, and a step count.
The cases mirror the reference's own hot-path tests
(tests/test_spatial_optimizers.py) plus the shapes of the benchmark workloads.
"""

from __future__ import annotations

import numpy as np

from smo_optimizer_b200 import synthetic

HP = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8)

# name -> dict(opt, kwargs, tensors=[(shape, group_index)], groups=[{...}], steps, seed, bf16,
#              param_dtype ("bfloat16" / "float16": params, grads and state in that dtype), grad_std)
CASES = {
    # the single-weight parity workload: 1024x1024, k=0.25, 100 steps
    "single1024": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                       tensors=[((1024, 1024), 0)], steps=100, seed=0, sample_stride=17),
    # H+W <= 128: torch's channels-last bilinear kernel
    "s8_64x64": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25),
                     tensors=[((64, 64), 0)], steps=5, seed=1),
    # tests/test_spatial_optimizers.py:80-110 shapes, monolithic and banded
    "s8_128x256_mono": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25, block_size=64),
                            tensors=[((128, 256), 0)], steps=3, seed=2),
    "s8_128x256_band": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25, block_size=64,
                                                       low_peak=True, band_mb=0.05),
                            tensors=[((128, 256), 0)], steps=3, seed=2),
    "s8_128x256_band_wd": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                                          low_peak=True, band_mb=0.05),
                               tensors=[((128, 256), 0)], steps=4, seed=3),
    # adaptive pooling, low_peak falls back to monolithic (spatial_8bit.py:112-115)
    "s8_50x30_adaptive": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, low_peak=True,
                                                         band_mb=0.05),
                              tensors=[((50, 30), 0)], steps=3, seed=4),
    "s8_100x200_adaptive": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.3),
                                tensors=[((100, 200), 0)], steps=3, seed=5),
    # conv views with row-aligned quant blocks (q_block = comp_w = 18)
    "s8_conv_64x8x3x3": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                                        compress_conv=True),
                             tensors=[((64, 8, 3, 3), 0)], steps=4, seed=6),
    "s8_conv_band_128x8x4x4": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25, block_size=64,
                                                              low_peak=True, band_mb=0.05, compress_conv=True),
                                   tensors=[((128, 8, 4, 4), 0)], steps=3, seed=7),
    "s8_block1_32x32": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25, block_size=1),
                            tensors=[((32, 32), 0)], steps=3, seed=8),
    "s8_k1_64x64": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=1.0, block_size=1),
                        tensors=[((64, 64), 0)], steps=3, seed=9),
    # a multi-tensor step: row-straddling blocks (w=96, 288), a dense head and a 1-D bias
    "s8_multi": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                     tensors=[((192, 384), 0), ((384, 1152), 0), ((384, 10), 0), ((384,), 0), ((1536, 384), 0)],
                     steps=3, seed=10, sample_stride=7),
    # per-group compress contract: dense and quant_only groups (spatial_8bit.py:142-169)
    "s8_groups": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                      tensors=[((256, 128), 0), ((64, 64), 1), ((48, 32), 2), ((300,), 2)],
                      groups=[{"compress": True}, {"compress": False}, {"compress": "quant_only"}],
                      steps=4, seed=11),
    # a tall low_peak tensor with many bands and a short last band
    "s8_808x96_band": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                                      low_peak=True, band_mb=0.02),
                           tensors=[((808, 96), 0)], steps=3, seed=12),
    # fused-kernel shapes: strips of 16, 16 and 1 compact rows, wide rows, low_peak bands
    "s8_132x2048_band": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                                        low_peak=True, band_mb=0.2),
                             tensors=[((132, 2048), 0)], steps=3, seed=18, sample_stride=3),
    # 8x8 windows (k = 0.125)
    "s8_256x512_k0125": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.125, block_size=64),
                             tensors=[((256, 512), 0)], steps=3, seed=19),
    # permute_basis (spatial_8bit.py:202-204, 231-253): an exact-window and an
    # adaptive tensor pooled in a randomly permuted basis (the reference's
    # torch.randperm draws, seeded, are stored with the golden state)
    "s8_perm": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                               permute_basis=True),
                    tensors=[((96, 160), 0), ((50, 70), 0)], steps=3, seed=20),
    # char-LM shapes with bf16-drawn gradients upcast to fp32, the embedding
    # protected (dense moments) as protect_output=True makes it
    "s8_bf16_grads": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                          tensors=[((512, 1536), 0), ((2048, 512), 0), ((512,), 0), ((256, 256), 1)],
                          groups=[{"compress": True}, {"compress": False}], steps=3, seed=22, bf16=True,
                          sample_stride=17),
    # half-precision parameters: the reference computes in the parameter's
    # dtype, its moments and block scales included
    "bf16_s8_mono": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                         tensors=[((128, 256), 0), ((300,), 0), ((64, 40), 0)], steps=3, seed=23,
                         param_dtype="bfloat16"),
    "bf16_s8_band_groups": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64,
                                                           low_peak=True, band_mb=0.03),
                                tensors=[((256, 512), 0), ((50, 30), 0), ((64, 64), 1), ((48, 32), 2), ((100,), 2)],
                                groups=[{"compress": True}, {"compress": False}, {"compress": "quant_only"}],
                                steps=3, seed=24, param_dtype="bfloat16"),
    "bf16_smo": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.5),
                     tensors=[((96, 192), 0), ((192,), 0), ((100, 200), 0)], steps=3, seed=25, param_dtype="bfloat16"),
    "fp16_s8_groups": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, block_size=64),
                           tensors=[((128, 256), 0), ((300,), 0), ((64, 64), 1), ((48, 32), 2)],
                           groups=[{"compress": True}, {"compress": False}, {"compress": "quant_only"}],
                           steps=3, seed=26, param_dtype="float16", grad_std=0.05),
    "fp16_s8_band": dict(opt="SMO8bit", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25, block_size=64,
                                                    low_peak=True, band_mb=0.03),
                         tensors=[((256, 512), 0)], steps=3, seed=27, param_dtype="float16", grad_std=0.05),
    "fp16_smo": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.5),
                     tensors=[((96, 192), 0), ((192,), 0)], steps=3, seed=28, param_dtype="float16", grad_std=0.05),
    # SMO-Spatial fp32 pooled moments
    "smo_96x192_k05": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.5),
                           tensors=[((96, 192), 0), ((192,), 0)], steps=5, seed=13),
    "smo_64x64_k025": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.0, k_ratio=0.25),
                           tensors=[((64, 64), 0)], steps=3, seed=14),
    "smo_conv": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.25, compress_conv=True),
                     tensors=[((64, 8, 3, 3), 0)], steps=3, seed=15),
    "smo_groups": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.5),
                       tensors=[((128, 256), 0), ((64, 64), 1)],
                       groups=[{"compress": True}, {"compress": False}], steps=3, seed=16),
    "smo_100x200_adaptive": dict(opt="SMO", kwargs=dict(HP, weight_decay=0.01, k_ratio=0.3),
                                 tensors=[((100, 200), 0)], steps=3, seed=17),
}

STATE_ARRAY_KEYS = ("m_q", "m_s", "v_q", "v_s", "exp_avg", "exp_avg_sq", "row_perm", "col_perm")
STATE_META_KEYS = ("step", "is_compressed", "is_quant_only", "orig_shape", "param_shape", "comp_numel",
                   "q_block", "comp_shape", "q_shape", "q_numel")


def round_to_dtype(x, dtype):
    """fp32 values rounded to ``dtype`` ("float32", "bfloat16", "float16"), as fp32."""
    if dtype == "bfloat16":
        return synthetic.round_to_bf16(x)
    if dtype == "float16":
        return np.ascontiguousarray(x, np.float32).astype(np.float16).astype(np.float32)
    return x


def case_dtype(case):
    return case.get("param_dtype", "float32")


def case_params(case):
    """Initial parameter arrays (~N(0, 0.02), values of the case's parameter dtype, as fp32)."""
    return [round_to_dtype(synthetic.synth_param(case["seed"], i, shape), case_dtype(case))
            for i, (shape, _) in enumerate(case["tensors"])]


def case_grads(case, step):
    """Gradients for 1-based ``step`` (~N(0, grad_std = 1e-3), values of the parameter dtype)."""
    std = case.get("grad_std", 1e-3)
    return [round_to_dtype(synthetic.synth_grad(case["seed"], step, i, shape, std=std, bf16=case.get("bf16", False)),
                           case_dtype(case))
            for i, (shape, _) in enumerate(case["tensors"])]


def case_groups(case, params):
    """Param-group list for the optimizer constructor."""
    specs = case.get("groups") or [{}]
    groups = [dict(spec, params=[]) for spec in specs]
    for p, (_, gi) in zip(params, case["tensors"]):
        groups[gi]["params"].append(p)
    return groups


def sample_indices(n, stride):
    return np.arange(0, n, stride, dtype=np.int64)
