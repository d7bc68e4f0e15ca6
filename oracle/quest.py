"""numpy restatement of ``QuestAlgorithm`` (``src/qwenquest/quest.py``) — oracle only.

Storage mirrors ``quest.py:171-209``: page bounds
``[layers, reqs, pages, kv_heads, head_dim, 2]`` (``[..., 0]`` = min,
``[..., 1]`` = max) with the ``+bf16max / -bf16max`` sentinels, running
bounds ``[layers, reqs, kv_heads, head_dim]`` and two int32 counters per
request.  Bounds are float32 arrays holding bf16-exact values.

Top-k tie order: ``torch.topk`` on CPU orders equal scores in an
implementation-defined way; this oracle (like the CUDA kernels) ranks equal
scores by lower page index first.  Parity checks therefore compare selections
through :func:`oracle.parity.compare_selection`, which excuses only
differences among near-tied pages.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.bf16 import BF16_MAX, BF16_MIN, round_bf16


@dataclass
class OracleStepLayout:
    """``StepLayout`` of ``quest.py:61-75``."""

    seq_lens: np.ndarray  # [bs] int64
    recent_positions: np.ndarray  # [bs, P] int64
    short_layout: np.ndarray  # [bs, top_k] int64
    is_short: np.ndarray  # [bs] bool
    actual_lens: np.ndarray  # [bs] int32
    candidate_limit: np.ndarray  # [bs] int64


class OracleQuest:
    """Follows ``QuestAlgorithm`` (``quest.py:107-480``)."""

    def __init__(self, top_k: int, page_size: int, *, avoid_recent_overlap: bool = False):
        # quest.py:138-149
        if page_size <= 0:
            raise ValueError(f"quest page_size must be > 0, got {page_size}")
        if top_k % page_size != 0:
            raise ValueError(f"top_k ({top_k}) must be divisible by quest_page_size ({page_size})")
        self.top_k = top_k
        self.page_size = page_size
        self.top_k_pages = top_k // page_size
        self.avoid_recent_overlap = avoid_recent_overlap
        self._step: OracleStepLayout | None = None
        #: diagnostics of the last retrieve_topk call
        self.last_scores: np.ndarray | None = None
        self.last_topk_pages: np.ndarray | None = None

    # quest.py:171-209
    def init_storage(self, start_layer, end_layer, max_reqs, max_context_len, kv_heads, head_dim):
        self.start_layer = start_layer
        self.end_layer = end_layer
        self.num_layers = end_layer - start_layer
        self.max_reqs = max_reqs
        self.max_pages_per_req = (max_context_len + self.page_size - 1) // self.page_size
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        shape = (self.num_layers, max_reqs, self.max_pages_per_req, kv_heads, head_dim, 2)
        self.page_k_bounds = np.empty(shape, dtype=np.float32)
        self.page_k_bounds[..., 0] = BF16_MAX
        self.page_k_bounds[..., 1] = BF16_MIN
        rshape = (self.num_layers, max_reqs, kv_heads, head_dim)
        self.running_k_min = np.full(rshape, BF16_MAX, dtype=np.float32)
        self.running_k_max = np.full(rshape, BF16_MIN, dtype=np.float32)
        self.running_token_count = np.zeros(max_reqs, dtype=np.int32)
        self.running_page_idx = np.zeros(max_reqs, dtype=np.int32)

    @property
    def page_valid(self) -> np.ndarray:
        # quest.py:220-223
        return (self.page_k_bounds[..., 1] > BF16_MIN).any(axis=(-1, -2))

    # quest.py:231-280  [Q2]
    def update_prefill_representations(self, layer_id, req_pool_idx, k_buffer, prefill_indices):
        lo = layer_id - self.start_layer
        idx = np.asarray(prefill_indices, dtype=np.int64)
        n = int(idx.shape[0])
        P = self.page_size
        full = n // P
        if full > 0:
            paged = k_buffer[idx[: full * P]].reshape(full, P, self.kv_heads, self.head_dim)
            self.page_k_bounds[lo, req_pool_idx, :full, :, :, 0] = round_bf16(paged.min(axis=1))
            self.page_k_bounds[lo, req_pool_idx, :full, :, :, 1] = round_bf16(paged.max(axis=1))
        partial = n - full * P
        if partial > 0:
            part = k_buffer[idx[full * P :]]
            self.running_k_min[lo, req_pool_idx] = round_bf16(part.min(axis=0))
            self.running_k_max[lo, req_pool_idx] = round_bf16(part.max(axis=0))
        if layer_id == self.end_layer - 1:
            self.running_token_count[req_pool_idx] = partial
            self.running_page_idx[req_pool_idx] = full

    # quest.py:284-302  [Q3]
    def update_decode_representations(self, layer_id, req_indices, k_buffer, device_locs):
        lo = layer_id - self.start_layer
        reqs = np.asarray(req_indices, dtype=np.int64)
        new_k = round_bf16(k_buffer[np.asarray(device_locs, dtype=np.int64)])
        self.running_k_min[lo, reqs] = np.minimum(self.running_k_min[lo, reqs], new_k)
        self.running_k_max[lo, reqs] = np.maximum(self.running_k_max[lo, reqs], new_k)

    # quest.py:304-321  [Q3]
    def maybe_finalize_decode_representations(self, req_indices):
        reqs = np.asarray(req_indices, dtype=np.int64)
        counts = self.running_token_count[reqs]
        completing = reqs[counts == (self.page_size - 1)]
        pages = self.running_page_idx[completing].astype(np.int64)
        for r, p in zip(completing.tolist(), pages.tolist(), strict=True):
            self.page_k_bounds[:, r, p, :, :, 0] = self.running_k_min[:, r]
            self.page_k_bounds[:, r, p, :, :, 1] = self.running_k_max[:, r]
        self.running_k_min[:, completing] = BF16_MAX
        self.running_k_max[:, completing] = BF16_MIN
        self.running_page_idx[completing] += 1
        self.running_token_count[reqs] = (counts + 1) % self.page_size

    # quest.py:325-362  [Q4]
    def prepare_step(self, seq_lens) -> OracleStepLayout:
        P = self.page_size
        seq = np.asarray(seq_lens, dtype=np.int64)
        last_valid = np.maximum(seq - 1, 0)[:, None]
        recent_start = np.maximum(seq - P, 0)[:, None]
        recent = np.minimum(recent_start + np.arange(P)[None, :], last_valid)
        short = np.minimum(np.arange(self.top_k)[None, :], last_valid)
        is_short = seq <= self.top_k
        actual = np.minimum(seq, self.top_k).astype(np.int32)
        full = seq // P
        limit = np.maximum(full - 1, 0) if self.avoid_recent_overlap else full
        self._step = OracleStepLayout(seq, recent, short, is_short, actual, limit)
        return self._step

    # quest.py:366-391  [Q5]
    def group_queries(self, queries: np.ndarray, *, query_is_bf16: bool) -> np.ndarray:
        """Mean over each KV head's query heads, in the query dtype.

        bf16 queries: ``bf16(fp32 sum / group)``; the fp32 sum runs over the
        group in head order.  fp32 queries: the same fp32 sum / group.
        """
        q = np.asarray(queries, dtype=np.float32)
        bs = q.shape[0]
        if q.ndim == 2:
            if q.shape[1] % self.head_dim != 0:
                raise ValueError("query hidden not divisible by head_dim")
            q = q.reshape(bs, q.shape[1] // self.head_dim, self.head_dim)
        elif q.ndim != 3:
            raise ValueError(f"Unsupported query shape {q.shape}")
        heads = q.shape[1]
        if heads == self.kv_heads:
            return q.copy()
        if heads % self.kv_heads != 0:
            raise ValueError(f"q_heads {heads} not divisible by kv_heads {self.kv_heads}")
        group = heads // self.kv_heads
        g = q.reshape(bs, self.kv_heads, group, self.head_dim)
        acc = np.zeros((bs, self.kv_heads, self.head_dim), dtype=np.float32)
        for j in range(group):
            acc = (acc + g[:, :, j]).astype(np.float32)
        mean = (acc / np.float32(group)).astype(np.float32)
        return round_bf16(mean) if query_is_bf16 else mean

    # quest.py:393-405  [Q5]
    def page_scores(self, grouped_q, layer_id, req_pool_indices, num_pages=None) -> np.ndarray:
        """``sum_{h,d} q * (q >= 0 ? kmax : kmin)`` in float32, pages ``[0, num_pages)``."""
        lo = layer_id - self.start_layer
        reqs = np.asarray(req_pool_indices, dtype=np.int64)
        npages = self.max_pages_per_req if num_pages is None else num_pages
        ch = self.kv_heads * self.head_dim
        out = np.empty((reqs.shape[0], npages), dtype=np.float32)
        for i, r in enumerate(reqs.tolist()):
            q = np.asarray(grouped_q[i], dtype=np.float32).reshape(ch)
            b = self.page_k_bounds[lo, r, :npages].reshape(npages, ch, 2)
            chosen = b[:, np.arange(ch), (q >= 0).astype(np.int64)]
            # sentinel pages overflow to -inf, as in the reference (quest.py:399-400)
            with np.errstate(over="ignore"):
                out[i] = (chosen * q[None, :]).sum(axis=1, dtype=np.float32)
        return out

    # quest.py:409-464  [Q6]
    def retrieve_topk(self, queries, layer_id, req_pool_indices, *, query_is_bf16: bool):
        step = self._step
        if step is None:
            raise RuntimeError("prepare_step() must be called once per decode step first")
        bs = np.asarray(queries).shape[0]
        if step.seq_lens.shape[0] != bs:
            raise ValueError("batch size differs from the one given to prepare_step()")
        P = self.page_size
        self.last_scores = None
        self.last_topk_pages = None
        if bool(step.is_short.all()):
            return step.short_layout.astype(np.int32), step.actual_lens.copy()
        q = self.group_queries(queries, query_is_bf16=query_is_bf16)
        scores = self.page_scores(q, layer_id, req_pool_indices)
        sel = self.top_k_pages - 1
        if sel > 0:
            page_idx = np.arange(scores.shape[1])[None, :]
            scores = np.where(page_idx >= step.candidate_limit[:, None], -np.inf, scores)
            scores = scores.astype(np.float32)
            # descending, ties -> lower page index first
            order = np.argsort(-scores, axis=1, kind="stable")[:, :sel]
            select = (order[:, :, None] * P + np.arange(P)[None, None, :]).reshape(bs, sel * P)
            self.last_topk_pages = order
        else:
            select = np.empty((bs, 0), dtype=np.int64)
        self.last_scores = scores
        long_layout = np.concatenate([select, step.recent_positions], axis=1)
        positions = np.where(step.is_short[:, None], step.short_layout, long_layout)
        return positions.astype(np.int32), step.actual_lens.copy()

    # quest.py:468-479  [Q8]
    def invalidate_request(self, req_pool_idx: int) -> None:
        self.page_k_bounds[:, req_pool_idx, :, :, :, 0] = BF16_MAX
        self.page_k_bounds[:, req_pool_idx, :, :, :, 1] = BF16_MIN
        self.running_k_min[:, req_pool_idx] = BF16_MAX
        self.running_k_max[:, req_pool_idx] = BF16_MIN
        self.running_token_count[req_pool_idx] = 0
        self.running_page_idx[req_pool_idx] = 0
