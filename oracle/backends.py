"""numpy restatement of the Quest attention backends — oracle only.

* :class:`OracleKVPools` — ``ReqToTokenPool`` + ``MHATokenToKVPool`` +
  ``TokenToKVPoolAllocator`` (``src/qwenquest/memory.py:28-120``).
* :class:`OracleQuestOnlyBackend` — ``QuestOnlyBackend``
  (``src/qwenquest/attention/quest_only.py:39-167``).
* :class:`OracleQuestHiSparseBackend` — ``QuestHiSparseBackend``
  (``src/qwenquest/attention/quest_hisparse.py:44-138``).

The backends take numpy arrays where the reference takes a ``ForwardBatch``:
``req_pool_indices`` / ``seq_lens`` (``batch.py:38-64``) and, for Mode 2,
``out_cache_loc``.  The KV pool dtype is bf16 when ``kv_bf16`` (values held as
bf16-exact float32) and float32 otherwise.
"""

from __future__ import annotations

import numpy as np

from oracle.attention import decode_attention
from oracle.bf16 import round_bf16
from oracle.hisparse import OracleHiSparse, OracleHostAllocator
from oracle.quest import OracleQuest


class OracleKVPools:
    """The token pools of ``memory.py``: slot 0 of the KV pool is padding."""

    def __init__(self, size, max_reqs, max_context_len, num_layers, kv_heads, head_dim, *, kv_bf16):
        self.size = size
        self.max_reqs = max_reqs
        self.max_context_len = max_context_len
        self.num_layers = num_layers
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.kv_bf16 = kv_bf16
        self.req_to_token = np.zeros((max_reqs, max_context_len), dtype=np.int32)  # memory.py:35-37
        shape = (size + 1, kv_heads, head_dim)
        self.k_buffer = [np.zeros(shape, np.float32) for _ in range(num_layers)]  # memory.py:98-103
        self.v_buffer = [np.zeros(shape, np.float32) for _ in range(num_layers)]
        self.allocator = OracleHostAllocator(size)

    def cast(self, x) -> np.ndarray:
        x = np.asarray(x, dtype=np.float32)
        return round_bf16(x) if self.kv_bf16 else x

    # memory.py:114-120
    def set_kv_buffer(self, layer, loc, k, v) -> None:
        loc = np.asarray(loc, dtype=np.int64)
        self.k_buffer[layer][loc] = self.cast(k)
        self.v_buffer[layer][loc] = self.cast(v)


class OracleQuestOnlyBackend:
    """Mode 2 (``quest_only.py``)."""

    def __init__(self, pools: OracleKVPools, top_k, page_size, *, avoid_recent_overlap=False,
                 start_layer=0, end_layer=None):
        # quest_only.py:42-75
        self.pools = pools
        self.quest = OracleQuest(top_k, page_size, avoid_recent_overlap=avoid_recent_overlap)
        self.quest.init_storage(
            start_layer, pools.num_layers if end_layer is None else end_layer,
            pools.max_reqs, pools.max_context_len, pools.kv_heads, pools.head_dim,
        )
        self._skip_first_decode_update = np.zeros(pools.max_reqs, dtype=bool)

    # quest_only.py:79-82
    def init_forward_metadata_decode(self, req_pool_indices, seq_lens) -> None:
        self._do_quest_decode_step_update(req_pool_indices, seq_lens)
        self.quest.prepare_step(seq_lens)

    # quest_only.py:84-97
    def _do_quest_decode_step_update(self, req_pool_indices, seq_lens) -> None:
        reqs = np.asarray(req_pool_indices, dtype=np.int64)
        sls = np.asarray(seq_lens, dtype=np.int64)
        skip = self._skip_first_decode_update[reqs]
        self._skip_first_decode_update[reqs] = False
        active = reqs[~skip]
        prev = np.maximum(sls[~skip] - 2, 0)
        locs = self.pools.req_to_token[active, prev]
        for layer in range(self.quest.start_layer, self.quest.end_layer):
            self.quest.update_decode_representations(layer, active, self.pools.k_buffer[layer], locs)
        self.quest.maybe_finalize_decode_representations(active)

    # quest_only.py:115-128  [Q2], called after the last layer's extend
    def update_quest_for_extend(self, req_pool_indices, seq_lens) -> None:
        for req, sl in zip(np.asarray(req_pool_indices).tolist(), np.asarray(seq_lens).tolist()):
            idx = self.pools.req_to_token[req, :sl]
            for layer in range(self.quest.start_layer, self.quest.end_layer):
                self.quest.update_prefill_representations(layer, req, self.pools.k_buffer[layer], idx)
            self._skip_first_decode_update[req] = True

    # quest_only.py:132-159  [Q6][Q7]
    def forward_decode(self, q, k, v, layer, req_pool_indices, seq_lens, out_cache_loc, scaling,
                       *, q_bf16: bool):
        self.pools.set_kv_buffer(layer, out_cache_loc, k, v)
        positions, actual = self.quest.retrieve_topk(q, layer, req_pool_indices, query_is_bf16=q_bf16)
        kb, vb = self.pools.k_buffer[layer], self.pools.v_buffer[layer]
        out = []
        for i, req in enumerate(np.asarray(req_pool_indices).tolist()):
            n = int(actual[i])
            locs = self.pools.req_to_token[req, positions[i, :n]].astype(np.int64)
            out.append(decode_attention(q[i], kb[locs], vb[locs], scaling, out_bf16=q_bf16))
        return np.stack(out), positions, actual

    # quest_only.py:163-167  [Q8]
    def on_request_finished(self, req) -> None:
        self.quest.invalidate_request(req)
        self._skip_first_decode_update[req] = False


class OracleQuestHiSparseBackend:
    """Mode 3 (``quest_hisparse.py``)."""

    def __init__(self, pools: OracleKVPools, top_k, page_size, *, device_buffer_size,
                 host_pool_size, avoid_recent_overlap=False, start_layer=0, end_layer=None):
        # quest_hisparse.py:49-94
        self.pools = pools
        self.quest = OracleQuest(top_k, page_size, avoid_recent_overlap=avoid_recent_overlap)
        self.quest.init_storage(
            start_layer, pools.num_layers if end_layer is None else end_layer,
            pools.max_reqs, pools.max_context_len, pools.kv_heads, pools.head_dim,
        )
        self.coord = OracleHiSparse(
            quest=self.quest, num_layers=pools.num_layers, kv_heads=pools.kv_heads,
            head_dim=pools.head_dim, max_reqs=pools.max_reqs,
            max_context_len=pools.max_context_len, top_k=top_k,
            device_buffer_size=device_buffer_size, host_pool_size=host_pool_size,
        )

    # quest_hisparse.py:98-101
    def init_forward_metadata_decode(self, req_pool_indices, seq_lens) -> None:
        self.coord.prepare_decode_step(req_pool_indices, seq_lens)
        self.quest.prepare_step(seq_lens)

    # quest_hisparse.py:103-108
    def on_extend_finished(self, req_pool_indices, seq_lens) -> None:
        for req, sl in zip(np.asarray(req_pool_indices).tolist(), np.asarray(seq_lens).tolist()):
            idx = self.pools.req_to_token[req, :sl]
            self.coord.admit_request(req, sl, self.pools.k_buffer, self.pools.v_buffer, idx)

    # quest_hisparse.py:112-133
    def forward_decode(self, q, k, v, layer, req_pool_indices, seq_lens, scaling, *, q_bf16: bool):
        self.coord.write_new_token(layer, req_pool_indices, seq_lens, self.pools.cast(k),
                                   self.pools.cast(v))
        positions, actual = self.quest.retrieve_topk(q, layer, req_pool_indices, query_is_bf16=q_bf16)
        rows = self.coord.swap_in_selected_pages(req_pool_indices, seq_lens, positions, layer)
        kd, vd = self.coord.device_k[layer], self.coord.device_v[layer]
        out = []
        for i in range(len(rows)):
            r = rows[i, : int(actual[i])]
            out.append(decode_attention(q[i], kd[r], vd[r], scaling, out_bf16=q_bf16))
        return np.stack(out), positions, actual, rows

    # quest_hisparse.py:136-138
    def on_request_finished(self, req) -> None:
        self.coord.request_finished(req)
