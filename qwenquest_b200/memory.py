"""KV pools with the layouts of ``src/qwenquest/memory.py:28-120``.

The kernels read these layouts directly: ``req_to_token`` int32
``[max_reqs, max_context_len]`` and one ``[size + 1, kv_heads, head_dim]`` K
and V tensor per layer (row 0 is padding).  The backends accept the
reference's own pool objects as well (same attributes); these mirrors let the
package run without the reference installed.
"""

from __future__ import annotations

import torch


class ReqToTokenPool:
    """``req_to_token[req_pool_idx, position] -> physical token index`` (memory.py:28-50)."""

    def __init__(self, size: int, max_context_len: int, device):
        self.size = size
        self.max_context_len = max_context_len
        self.device = torch.device(device)
        self.req_to_token = torch.zeros((size, max_context_len), dtype=torch.int32, device=self.device)
        self._free_slots = list(range(size))

    def available_size(self) -> int:
        return len(self._free_slots)

    def alloc(self) -> int:
        if not self._free_slots:
            raise RuntimeError("ReqToTokenPool is full; lower the number of concurrent requests")
        return self._free_slots.pop(0)

    def free(self, req_pool_idx: int) -> None:
        self.req_to_token[req_pool_idx].zero_()
        self._free_slots.append(req_pool_idx)


class TokenToKVPoolAllocator:
    """Free list over physical token indices ``[1, size]`` (memory.py:53-76)."""

    def __init__(self, size: int, device="cpu"):
        self.size = size
        self.device = torch.device(device)
        self._free = torch.arange(1, size + 1, dtype=torch.int64, device=self.device)

    def available_size(self) -> int:
        return int(self._free.numel())

    def alloc(self, n: int) -> torch.Tensor:
        if n > self._free.numel():
            raise RuntimeError(f"KV pool out of memory: need {n} token slots, {self._free.numel()} free")
        out, self._free = self._free[:n], self._free[n:]
        return out

    def free(self, indices: torch.Tensor) -> None:
        indices = indices.to(device=self.device, dtype=torch.int64).flatten()
        indices = indices[indices > 0]
        if indices.numel():
            self._free = torch.cat([self._free, indices])


class MHATokenToKVPool:
    """Per-layer K / V buffers ``[size + 1, kv_heads, head_dim]`` (memory.py:79-120)."""

    def __init__(self, size: int, num_layers: int, kv_heads: int, head_dim: int, dtype, device):
        self.size = size
        self.num_layers = num_layers
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (size + 1, kv_heads, head_dim)
        self.k_buffer = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(num_layers)]
        self.v_buffer = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(num_layers)]

    def get_key_buffer(self, layer_id: int) -> torch.Tensor:
        return self.k_buffer[layer_id]

    def get_value_buffer(self, layer_id: int) -> torch.Tensor:
        return self.v_buffer[layer_id]

    def get_kv_buffer(self, layer_id: int):
        return self.k_buffer[layer_id], self.v_buffer[layer_id]

    def set_kv_buffer(self, layer_id: int, loc: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        loc = loc.to(torch.int64)
        self.k_buffer[layer_id][loc] = k.to(self.dtype)
        self.v_buffer[layer_id][loc] = v.to(self.dtype)
