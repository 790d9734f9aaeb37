"""torch-facing wrappers of the stage entry points of the CUDA library.

Each takes CUDA fp32 tensors and launches on the current stream.  They mirror
the reference helpers the optimizer classes expose (``_quantize_blockwise``,
``_dequantize_blockwise``, ``_compress_2d``, ``upsample_2d_pair``) and are used
by the tests to check each stage on its own.
"""

from __future__ import annotations

import torch

from . import _host, _lib, synthetic


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda_f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.device.type != "cuda":
        raise RuntimeError(f"{name}: CUDA tensor required (got {t.device})")
    if t.dtype != torch.float32:
        raise TypeError(f"{name}: fp32 tensor required (got {t.dtype})")
    return t.contiguous()


def quantize_blockwise(data: torch.Tensor, block: int):
    """codes (nb, block) int8 and scales (nb, 1) fp32 (spatial_8bit.py:85-107)."""
    x = _cuda_f32(data, "quantize_blockwise").reshape(-1)
    nb = _host.num_blocks(x.numel(), block)
    q = torch.empty((nb, block), dtype=torch.int8, device=x.device)
    s = torch.empty((nb, 1), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().smo_quantize_blockwise(x.data_ptr(), x.numel(), block, q.data_ptr(), s.data_ptr(),
                                                      _stream(x)), "smo_quantize_blockwise")
    return q, s


def dequantize_blockwise(codes: torch.Tensor, scales: torch.Tensor, numel: int, block: int) -> torch.Tensor:
    """flat fp32 moments from codes and scales (spatial_8bit.py:109-122)."""
    if codes.device.type != "cuda":
        raise RuntimeError("dequantize_blockwise: CUDA tensors required")
    q = codes.contiguous()
    s = scales.to(torch.float32).contiguous()
    out = torch.empty(numel, dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().smo_dequantize_blockwise(q.data_ptr(), s.data_ptr(), numel, block, out.data_ptr(),
                                                        _stream(q)), "smo_dequantize_blockwise")
    return out


def pool2d_pair(grad: torch.Tensor, target_shape, param: torch.Tensor = None, weight_decay: float = 0.0):
    """Window means of x and x*x, x = grad + wd*param (_spatial_utils.py:72-91)."""
    g = _cuda_f32(grad, "pool2d_pair")
    H, W = g.shape
    h, w = int(target_shape[0]), int(target_shape[1])
    wd_on = int(weight_decay != 0 and param is not None)
    p = _cuda_f32(param, "pool2d_pair") if wd_on else g
    om = torch.empty((h, w), dtype=torch.float32, device=g.device)
    o2 = torch.empty((h, w), dtype=torch.float32, device=g.device)
    with torch.cuda.device(g.device):
        _lib.check(_lib.load().smo_pool2d_pair(g.data_ptr(), p.data_ptr(), H, W, h, w, float(weight_decay), wd_on,
                                               om.data_ptr(), o2.data_ptr(), _stream(g)), "smo_pool2d_pair")
    return om, o2


def compress_2d(tensor: torch.Tensor, target_shape) -> torch.Tensor:
    """Window mean of a 2-D tensor onto ``target_shape`` (_spatial_utils.py:56-69)."""
    return pool2d_pair(tensor, target_shape)[0]


def upsample2d(src: torch.Tensor, target_shape, interp_band: int = 0) -> torch.Tensor:
    """Bilinear (align_corners=False) reconstruction onto ``target_shape`` (_spatial_utils.py:128-146)."""
    s = _cuda_f32(src, "upsample2d")
    h, w = s.shape
    H, W = int(target_shape[0]), int(target_shape[1])
    out = torch.empty((H, W), dtype=torch.float32, device=s.device)
    with torch.cuda.device(s.device):
        _lib.check(_lib.load().smo_upsample2d(s.data_ptr(), h, w, H, W, interp_band, out.data_ptr(), _stream(s)),
                   "smo_upsample2d")
    return out


def synth_normal_(out: torch.Tensor, seed: int, stream_id: int, std: float, offset: int = 0) -> torch.Tensor:
    """Fill a CUDA fp32 tensor with the synthetic N(0, std) stream (same bits as synthetic.synth_normal)."""
    t = out
    if t.device.type != "cuda" or t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError("synth_normal_: contiguous CUDA fp32 tensor required")
    base = synthetic.stream_base(seed, stream_id)
    scale = float(synthetic.normal_scale(std))
    with torch.cuda.device(t.device):
        _lib.check(_lib.load().smo_synth_normal(t.data_ptr(), t.numel(), base, scale, offset, _stream(t)),
                   "smo_synth_normal")
    return t
