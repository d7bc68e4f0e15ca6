"""bfloat16 helpers for numpy (which has no bf16 dtype) — oracle only.

Values that live in bf16 in the reference (the KV pool when it is bf16, the
Quest bounds, the grouped query) are held here as float32 arrays whose
values are exactly representable in bf16.  ``round_bf16`` is IEEE
round-to-nearest-even, the rounding ``torch.Tensor.to(torch.bfloat16)``
applies (used e.g. at ``src/qwenquest/quest.py:260-275``, ``:298``).
"""

from __future__ import annotations

import numpy as np

#: ``torch.finfo(torch.bfloat16).max`` / ``.min`` — the sentinels of
#: ``src/qwenquest/quest.py:57-58``.
BF16_MAX = float(np.uint32(0x7F7F0000).view(np.float32))
BF16_MIN = -BF16_MAX


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern (uint16), round-to-nearest-even; NaN -> 0x7FC0."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit pattern (uint16) -> float32 (exact)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return bf16_from_bits(bf16_bits(x))
