"""Deterministic synthetic parameters and gradients.

The workloads are quoted on seeded synthetic data: fp32 params ~N(0, 0.02) and
grads ~N(0, 1e-3) redrawn every step.  ``torch.randn`` on the CPU is not a safe
source for bit-identical inputs across machines (its vectorised Box-Muller path
depends on the host's ISA), so the inputs here come from a counter-based
integer hash that numpy (host) and the CUDA library (device,
``smo_synth_normal``) evaluate identically:

* ``base = splitmix64(splitmix64(seed) ^ stream)``
* for element ``i``: ``ha = splitmix64(base + 2i)``, ``hb = splitmix64(base + 2i + 1)``
* ``S`` = sum of the eight 16-bit lanes of ``ha`` and ``hb`` (an Irwin-Hall(8)
  variate), ``c = 2*S - 8*65535`` (an exact integer, |c| <= 524280)
* ``value = float32(c) * float32(std / (2 * 65536 * sqrt(8/12)))``

The only floating-point operation is one correctly rounded fp32 multiply, so
every platform produces the same bits.  The distribution has mean 0, standard
deviation ``std`` (to within 1e-5 relative) and tails bounded at 3.46 std.
"""

from __future__ import annotations

import math

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
_GOLD = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)

# stream namespaces (top byte of the 64-bit stream id)
STREAM_PARAM = 1
STREAM_GRAD = 2


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLD
        z = (z ^ (z >> np.uint64(30))) * _C1
        z = (z ^ (z >> np.uint64(27))) * _C2
        return z ^ (z >> np.uint64(31))


def _splitmix64_int(x: int) -> int:
    x &= 0xFFFFFFFFFFFFFFFF
    z = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def stream_id(kind: int, step: int, index: int) -> int:
    """64-bit stream id: kind in the top byte, step in bits 24..55, tensor index below."""
    return ((kind & 0xFF) << 56) | ((step & 0xFFFFFFFF) << 24) | (index & 0xFFFFFF)


def stream_base(seed: int, stream: int) -> int:
    """Per-stream key shared by the host and device generators."""
    return _splitmix64_int(_splitmix64_int(seed) ^ (stream & 0xFFFFFFFFFFFFFFFF))


def normal_scale(std: float) -> np.float32:
    """fp32 multiplier that maps the centred Irwin-Hall(8) integer to N(0, std)."""
    return np.float32(std / (2.0 * 65536.0 * math.sqrt(8.0 / 12.0)))


def synth_normal(seed: int, stream: int, n: int, std: float, offset: int = 0) -> np.ndarray:
    """``n`` fp32 values of the synthetic N(0, std) stream, starting at element ``offset``."""
    base = np.uint64(stream_base(seed, stream))
    out = np.empty(n, dtype=np.float32)
    scale = normal_scale(std)
    chunk = 1 << 20
    mask = np.uint64(0xFFFF)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        idx = np.arange(offset + s, offset + e, dtype=np.uint64)
        with np.errstate(over="ignore"):
            ha = _splitmix64(base + idx * np.uint64(2))
            hb = _splitmix64(base + idx * np.uint64(2) + np.uint64(1))
        tot = np.zeros(e - s, dtype=np.int64)
        for h in (ha, hb):
            for k in range(4):
                tot += ((h >> np.uint64(16 * k)) & mask).astype(np.int64)
        c = (2 * tot - 8 * 65535).astype(np.float32)
        out[s:e] = c * scale
    return out


def synth_param(seed: int, index: int, shape, std: float = 0.02) -> np.ndarray:
    n = int(np.prod(shape)) if len(shape) else 1
    return synth_normal(seed, stream_id(STREAM_PARAM, 0, index), n, std).reshape(shape)


def synth_grad(seed: int, step: int, index: int, shape, std: float = 1e-3,
               bf16: bool = False) -> np.ndarray:
    """Gradient of tensor ``index`` at 1-based ``step``; ``bf16`` rounds it to bf16 and back."""
    n = int(np.prod(shape)) if len(shape) else 1
    g = synth_normal(seed, stream_id(STREAM_GRAD, step, index), n, std).reshape(shape)
    if bf16:
        g = round_to_bf16(g)
    return g


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and widen back to fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) << np.uint64(16)
    return (r & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32).reshape(x.shape)
