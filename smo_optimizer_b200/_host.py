"""Host-side shape rules and scalar hyper-parameters of the SMO step.

Pure Python, no device work.  Mirrors the reference's eligibility and layout
rules so that state shapes, quantisation blocks and low_peak bands come out the
same as in smo/optimizers/_spatial_utils.py and smo/optimizers/spatial_8bit.py.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# _spatial_utils.py:10 -- a pooled view needs both dims >= 32
MIN_SPATIAL_DIM = 32


def compression_view(shape, include_conv: bool = False):
    """``((rows, cols), param_shape)`` when a tensor is pooled, else ``None``.

    Same rule as _spatial_utils.py:13-42: a 2-D tensor with both dims >= 32,
    or (only with ``include_conv``) a 4-D conv weight viewed as
    ``(out_c, in_c*kh*kw)`` with both view dims >= 32.
    """
    shape = tuple(int(s) for s in shape)
    if len(shape) == 2:
        if shape[0] >= MIN_SPATIAL_DIM and shape[1] >= MIN_SPATIAL_DIM:
            return shape, shape
        return None
    if len(shape) == 4 and include_conv:
        flat_cols = shape[1] * shape[2] * shape[3]
        if shape[0] >= MIN_SPATIAL_DIM and flat_cols >= MIN_SPATIAL_DIM:
            return (shape[0], flat_cols), shape
    return None


def comp_shape(view_shape, k_ratio: float):
    """Compact moment grid, spatial_8bit.py:179-181 / spatial.py:112-114."""
    return (max(1, int(view_shape[0] * k_ratio)), max(1, int(view_shape[1] * k_ratio)))


def exact_pool(view_shape, cshape) -> bool:
    """_spatial_utils.py:45-53: whole windows tile the view."""
    (H, W), (h, w) = view_shape, cshape
    return h > 0 and w > 0 and H % h == 0 and W % w == 0


def can_band(view_shape, cshape) -> bool:
    """spatial_8bit.py:301-305 (low_peak needs the exact-pool path)."""
    return view_shape[0] % cshape[0] == 0 and view_shape[1] % cshape[1] == 0


def band_comp_rows(view_shape, cshape, band_mb: float, elem_size: int = 4) -> int:
    """Compact rows per low_peak interpolation band, spatial_8bit.py:359."""
    H, W = view_shape
    kh = H // cshape[0]
    return max(2, int(band_mb * 1024 ** 2 / (2 * W * elem_size * kh)))


def pooled_q_block(param_shape, cshape, block_size: int) -> int:
    """spatial_8bit.py:192: conv views quantise one compact row per block."""
    return min(block_size, cshape[1]) if len(param_shape) == 4 else block_size


def quant_only_q_block(shape, block_size: int) -> int:
    """spatial_8bit.py:165-166: matrix-like tensors get one scale per row."""
    if len(shape) >= 2:
        return min(block_size, int(shape[-1]))
    return block_size


def num_blocks(n: int, block: int) -> int:
    return (n + block - 1) // block


@dataclass(frozen=True)
class StepScalars:
    """fp32 scalars of one tensor's step, rounded from double as torch does."""
    beta1: np.float32
    omb1: np.float32
    beta2: np.float32
    omb2: np.float32
    wd: np.float32
    wd_on: int
    neg_step: np.float32
    sqrt_bc2: np.float32
    eps: np.float32


def step_scalars(lr, betas, eps, weight_decay, step: int) -> StepScalars:
    """Scalars of spatial_8bit.py:210-297 for 1-based ``step``.

    Every value is formed in double precision exactly as the reference's Python
    expressions form it, then rounded once to fp32 (torch casts a Python scalar
    to the tensor dtype when it meets an fp32 tensor).
    """
    beta1, beta2 = float(betas[0]), float(betas[1])
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    step_size = float(lr) / bc1
    return StepScalars(
        beta1=np.float32(beta1), omb1=np.float32(1 - beta1),
        beta2=np.float32(beta2), omb2=np.float32(1 - beta2),
        wd=np.float32(weight_decay), wd_on=int(weight_decay != 0),
        neg_step=np.float32(-step_size), sqrt_bc2=np.float32(math.sqrt(bc2)),
        eps=np.float32(eps),
    )
