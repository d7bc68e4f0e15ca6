"""numpy restatement of ``HiSparseCoordinator`` (``src/qwenquest/hisparse/coordinator.py``) — oracle only."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.quest import OracleQuest


@dataclass
class OracleSwapInStats:
    """``SwapInStats`` of ``coordinator.py:48-59``."""

    hits: int = 0
    misses: int = 0
    fast_path_calls: int = 0


class OracleHostAllocator:
    """``TokenToKVPoolAllocator`` (``src/qwenquest/memory.py:53-76``): free list over ``[1, size]``."""

    def __init__(self, size: int):
        self.size = size
        self._free = np.arange(1, size + 1, dtype=np.int64)

    def available_size(self) -> int:
        return int(self._free.shape[0])

    def alloc(self, n: int) -> np.ndarray:
        if n > self._free.shape[0]:
            raise RuntimeError(f"KV pool out of memory: need {n}, {self._free.shape[0]} free")
        out, self._free = self._free[:n], self._free[n:]
        return out

    def free(self, indices) -> None:
        idx = np.asarray(indices, dtype=np.int64).reshape(-1)
        idx = idx[idx > 0]
        if idx.size:
            self._free = np.concatenate([self._free, idx])


def unique_first_occurrence(x: np.ndarray) -> np.ndarray:
    """``_unique_first_occurrence`` (``coordinator.py:62-71``): unique values in first-seen order."""
    if x.size == 0:
        return x
    _, first = np.unique(x, return_index=True)
    return x[np.sort(first)]


class OracleHiSparse:
    """Follows ``HiSparseCoordinator`` (``coordinator.py:74-324``)."""

    def __init__(
        self,
        *,
        quest: OracleQuest,
        num_layers: int,
        kv_heads: int,
        head_dim: int,
        max_reqs: int,
        max_context_len: int,
        top_k: int,
        device_buffer_size: int,
        host_pool_size: int,
    ):
        # coordinator.py:91-134
        if device_buffer_size < top_k:
            raise ValueError("device_buffer_size must be >= top_k")
        if quest.top_k != top_k:
            raise ValueError("QuestAlgorithm.top_k != top_k")
        self.quest = quest
        self.num_layers = num_layers
        self.top_k = top_k
        self.device_buffer_size = buf = device_buffer_size
        self.host_allocator = OracleHostAllocator(host_pool_size)
        hshape = (host_pool_size + 1, kv_heads, head_dim)
        self.host_k = [np.zeros(hshape, np.float32) for _ in range(num_layers)]
        self.host_v = [np.zeros(hshape, np.float32) for _ in range(num_layers)]
        self.req_to_host_pool = np.full((max_reqs, max_context_len), -1, dtype=np.int64)
        dshape = (max_reqs * (buf + 1), kv_heads, head_dim)
        self.device_k = [np.zeros(dshape, np.float32) for _ in range(num_layers)]
        self.device_v = [np.zeros(dshape, np.float32) for _ in range(num_layers)]
        self.req_to_device_buffer = np.arange(max_reqs * (buf + 1), dtype=np.int64).reshape(
            max_reqs, buf + 1
        )
        self.buffer_tokens = np.full((num_layers, max_reqs, buf), -1, dtype=np.int64)
        self._lru_init = np.arange(buf, dtype=np.int64)
        self.lru_slots = np.tile(self._lru_init, (num_layers, max_reqs, 1))
        self._skip_first_backup = [False] * max_reqs
        self.stats = OracleSwapInStats()

    # coordinator.py:138-174  [H1]
    def admit_request(self, req, prefill_len, k_buffers, v_buffers, prefill_indices):
        idx = np.asarray(prefill_indices, dtype=np.int64)
        host_idx = self.host_allocator.alloc(prefill_len)
        self.req_to_host_pool[req, :prefill_len] = host_idx
        n_dev = min(prefill_len, self.device_buffer_size)
        dev = self.req_to_device_buffer[req, :n_dev]
        for layer in range(self.num_layers):
            k_rows, v_rows = k_buffers[layer][idx], v_buffers[layer][idx]
            self.host_k[layer][host_idx] = k_rows
            self.host_v[layer][host_idx] = v_rows
            self.device_k[layer][dev] = k_rows[:n_dev]
            self.device_v[layer][dev] = v_rows[:n_dev]
        self.buffer_tokens[:, req, :] = self._lru_init
        self.lru_slots[:, req, :] = self._lru_init
        for layer in range(self.quest.start_layer, self.quest.end_layer):
            self.quest.update_prefill_representations(layer, req, k_buffers[layer], idx)
        self._skip_first_backup[req] = True

    # coordinator.py:178-181
    def newest_slot(self, seq_lens) -> np.ndarray:
        return np.minimum(np.asarray(seq_lens, dtype=np.int64) - 1, self.device_buffer_size)

    # coordinator.py:183-215  [H2]
    def prepare_decode_step(self, req_pool_indices, seq_lens) -> None:
        reqs_l, pos_l = [], []
        for req, sl in zip(np.asarray(req_pool_indices).tolist(), np.asarray(seq_lens).tolist()):
            if self._skip_first_backup[req]:
                self._skip_first_backup[req] = False
                continue
            reqs_l.append(req)
            pos_l.append(sl - 2)
        if not reqs_l:
            return
        reqs = np.asarray(reqs_l, dtype=np.int64)
        prev = np.asarray(pos_l, dtype=np.int64)
        dev = self.req_to_device_buffer[reqs, np.minimum(prev, self.device_buffer_size)]
        for layer in range(self.quest.start_layer, self.quest.end_layer):
            self.quest.update_decode_representations(layer, reqs, self.device_k[layer], dev)
        self.quest.maybe_finalize_decode_representations(reqs)
        host_idx = self.host_allocator.alloc(len(reqs_l))
        self.req_to_host_pool[reqs, prev] = host_idx
        for layer in range(self.num_layers):
            self.host_k[layer][host_idx] = self.device_k[layer][dev]
            self.host_v[layer][host_idx] = self.device_v[layer][dev]

    # coordinator.py:217-228
    def write_new_token(self, layer, req_pool_indices, seq_lens, k, v) -> None:
        reqs = np.asarray(req_pool_indices, dtype=np.int64)
        locs = self.req_to_device_buffer[reqs, self.newest_slot(seq_lens)]
        self.device_k[layer][locs] = k
        self.device_v[layer][locs] = v

    # coordinator.py:232-257  [H3]
    def swap_in_selected_pages(self, req_pool_indices, seq_lens, top_k_result, layer) -> np.ndarray:
        reqs = np.asarray(req_pool_indices, dtype=np.int64)
        sls = np.asarray(seq_lens, dtype=np.int64)
        bs = reqs.shape[0]
        out = np.full((bs, self.top_k), -1, dtype=np.int64)
        for i in range(bs):
            req, sl = int(reqs[i]), int(sls[i])
            n = min(sl, self.top_k)
            pos = np.asarray(top_k_result[i, :n], dtype=np.int64)
            if sl <= self.device_buffer_size:
                self.stats.fast_path_calls += 1
                out[i, :n] = self.req_to_device_buffer[req, pos]
            else:
                out[i, :n] = self._swap_in_long(layer, req, sl, pos)
        return out

    # coordinator.py:259-304
    def _swap_in_long(self, layer, req, seq_len, positions) -> np.ndarray:
        buf = self.device_buffer_size
        locs = np.empty_like(positions)
        newest = positions == seq_len - 1
        locs[newest] = self.req_to_device_buffer[req, buf]
        wanted = positions[~newest]
        uniq = unique_first_occurrence(wanted)
        tokens = self.buffer_tokens[layer, req]  # view: writes go through
        lru = self.lru_slots[layer, req].copy()
        hit_in_lru = np.isin(tokens[lru], uniq)
        hit_slots = lru[hit_in_lru]
        evictable = lru[~hit_in_lru]
        misses = uniq[~np.isin(uniq, tokens)]
        num_miss = int(misses.shape[0])
        if num_miss > evictable.shape[0]:
            raise RuntimeError("device_buffer_size too small for this top-k")
        victims = evictable[:num_miss]
        if num_miss:
            host_idx = self.req_to_host_pool[req, misses]
            if bool((host_idx < 0).any()):
                raise AssertionError(f"req {req}: positions without host backup were selected")
            dst = self.req_to_device_buffer[req, victims]
            self.device_k[layer][dst] = self.host_k[layer][host_idx]
            self.device_v[layer][dst] = self.host_v[layer][host_idx]
            tokens[victims] = misses
        self.lru_slots[layer, req] = np.concatenate([evictable[num_miss:], victims, hit_slots])
        slot_of = {int(t): s for s, t in enumerate(tokens.tolist()) if t >= 0}
        slots = np.asarray([slot_of[int(p)] for p in wanted.tolist()], dtype=np.int64)
        locs[~newest] = self.req_to_device_buffer[req, slots] if slots.size else slots
        self.stats.hits += int(uniq.shape[0]) - num_miss
        self.stats.misses += num_miss
        return locs

    # coordinator.py:308-316  [H4]
    def request_finished(self, req) -> None:
        host_idx = self.req_to_host_pool[req]
        self.host_allocator.free(host_idx[host_idx >= 0])
        self.req_to_host_pool[req] = -1
        self.buffer_tokens[:, req, :] = -1
        self.lru_slots[:, req, :] = self._lru_init
        self._skip_first_backup[req] = False
        self.quest.invalidate_request(req)
