"""``ForwardMode`` / ``ForwardBatch`` with the fields of ``src/qwenquest/batch.py:27-64``.

The backends only read attributes, so a reference ``ForwardBatch`` works
unchanged; this mirror lets the package run where the reference is not
installed (the GPU benchmark box).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Any

import torch


class ForwardMode(enum.Enum):
    EXTEND = "extend"
    DECODE = "decode"

    def is_extend(self) -> bool:
        return self is ForwardMode.EXTEND

    def is_decode(self) -> bool:
        return self is ForwardMode.DECODE


@dataclass
class ForwardBatch:
    forward_mode: ForwardMode
    input_ids: torch.Tensor
    positions: torch.Tensor
    req_pool_indices: torch.Tensor  # [bs] int64
    seq_lens: torch.Tensor  # [bs] int64, counts the token being decoded
    out_cache_loc: torch.Tensor | None
    req_to_token_pool: Any
    token_to_kv_pool: Any
    attn_backend: Any
    extend_prefix_lens: torch.Tensor | None = None
    extend_seq_lens: torch.Tensor | None = None

    @property
    def batch_size(self) -> int:
        return int(self.req_pool_indices.shape[0])

    def extend_token_offsets(self) -> list[int]:
        assert self.extend_seq_lens is not None
        offsets = [0]
        for n in self.extend_seq_lens.tolist():
            offsets.append(offsets[-1] + int(n))
        return offsets
