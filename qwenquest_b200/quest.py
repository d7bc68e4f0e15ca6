"""``QuestAlgorithm`` on B200: the API of ``src/qwenquest/quest.py:107-515``, every step a CUDA kernel.

Storage and semantics follow the reference exactly (bounds layout, sentinels,
counters, the per-step layout, the top-k layout); the work is done by
``libqquest.so``:

==========================================  ==========================================
reference                                   here
==========================================  ==========================================
``init_storage`` fills (quest.py:196-208)   ``qq_quest_init_storage``
``update_prefill_representations`` [Q2]     ``qq_quest_bounds_prefill`` (one or all layers)
``update_decode_representations`` +         ``qq_quest_decode_step`` (fold / finalize,
``maybe_finalize_...`` [Q3]                 all layers in one launch)
``group_queries`` / ``page_scores`` [Q5]    ``qq_quest_group_queries`` / ``qq_quest_page_scores``
``retrieve_topk`` [Q6]                      ``qq_quest_retrieve_topk`` (fused, one launch)
``invalidate_request`` [Q8]                 ``qq_quest_invalidate``
==========================================  ==========================================

Top-k ties (equal fp32 scores) are ranked lower page index first; the
reference leaves their order to ``torch.topk``.  Traces are the reference's
own ``QuestTrace`` / ``QuestSelection`` records (``quest.py:78-104``).
"""

from __future__ import annotations

import torch
from qwenquest.quest import QuestSelection, QuestTrace  # the reference's own records

from qwenquest_b200 import _lib
from qwenquest_b200._lib import QQ_BF16, QQ_F32, QQ_STEP_FINALIZE, QQ_STEP_FOLD, check

__all__ = ["QuestAlgorithm", "QuestSelection", "QuestTrace", "StepLayout"]

_BF16_POS_INF = torch.finfo(torch.bfloat16).max
_BF16_NEG_INF = torch.finfo(torch.bfloat16).min


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return QQ_BF16
    if dtype == torch.float32:
        return QQ_F32
    raise ValueError(f"unsupported dtype {dtype}: the kernels take bfloat16 or float32")


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class StepLayout:
    """``StepLayout`` (``quest.py:61-75``).  The kernels derive the layout from
    ``seq_lens`` themselves; the other fields are computed on first access."""

    def __init__(self, seq_lens: torch.Tensor, top_k: int, page_size: int, avoid_recent_overlap: bool):
        self.seq_lens = seq_lens
        self._top_k, self._P, self._avoid = top_k, page_size, avoid_recent_overlap

    @property
    def recent_positions(self) -> torch.Tensor:
        seq = self.seq_lens
        last = (seq - 1).clamp(min=0).unsqueeze(1)
        start = (seq - self._P).clamp(min=0).unsqueeze(1)
        offs = torch.arange(self._P, device=seq.device, dtype=torch.int64).unsqueeze(0)
        return torch.minimum(start + offs, last)

    @property
    def short_layout(self) -> torch.Tensor:
        last = (self.seq_lens - 1).clamp(min=0).unsqueeze(1)
        return torch.minimum(torch.arange(self._top_k, device=last.device).unsqueeze(0), last)

    @property
    def is_short(self) -> torch.Tensor:
        return (self.seq_lens <= self._top_k).unsqueeze(1)

    @property
    def actual_lens(self) -> torch.Tensor:
        return self.seq_lens.clamp(max=self._top_k).to(torch.int32)

    @property
    def candidate_limit(self) -> torch.Tensor:
        full = self.seq_lens // self._P
        lim = (full - 1).clamp(min=0) if self._avoid else full
        return lim.unsqueeze(1)


class QuestAlgorithm:
    """Quest page-wise sparse attention, bounds indexed by ``(layer, req_pool_idx, page)``."""

    def __init__(self, top_k: int, page_size: int, device, *, avoid_recent_overlap: bool = False):
        if page_size <= 0:
            raise ValueError(f"quest page_size must be > 0, got {page_size}")
        if top_k % page_size != 0:
            raise ValueError(
                f"top_k ({top_k}) must be divisible by quest_page_size ({page_size}); "
                "Quest emits whole pages worth of token positions."
            )
        self.top_k = top_k
        self.page_size = page_size
        self.top_k_pages = top_k // page_size
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("qwenquest_b200.QuestAlgorithm runs on a CUDA device only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.avoid_recent_overlap = avoid_recent_overlap
        self.lib = _lib.load()
        self.start_layer = self.end_layer = self.num_layers = 0
        self.max_reqs = self.max_pages_per_req = self.kv_heads = self.head_dim = 0
        self._initialized = False
        self._step: StepLayout | None = None
        self.trace: QuestTrace | None = None
        self._scores: torch.Tensor | None = None

    # ------------------------------------------------------------------ setup

    def init_storage(self, start_layer, end_layer, max_reqs, max_context_len, kv_heads, head_dim) -> None:
        self.start_layer = start_layer
        self.end_layer = end_layer
        self.num_layers = end_layer - start_layer
        if not 0 < self.num_layers <= _lib.QQ_MAX_LAYERS:
            raise ValueError(f"num_layers must be in [1, {_lib.QQ_MAX_LAYERS}]")
        self.max_reqs = max_reqs
        self.max_pages_per_req = (max_context_len + self.page_size - 1) // self.page_size
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        dev = self.device
        shape = (self.num_layers, max_reqs, self.max_pages_per_req, kv_heads, head_dim, 2)
        self.page_k_bounds = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        rshape = (self.num_layers, max_reqs, kv_heads, head_dim)
        self.running_k_min = torch.empty(rshape, dtype=torch.bfloat16, device=dev)
        self.running_k_max = torch.empty(rshape, dtype=torch.bfloat16, device=dev)
        self.running_token_count = torch.empty(max_reqs, dtype=torch.int32, device=dev)
        self.running_page_idx = torch.empty(max_reqs, dtype=torch.int32, device=dev)
        self._state = _lib.QQQuestState(
            self.page_k_bounds.data_ptr(), self.running_k_min.data_ptr(), self.running_k_max.data_ptr(),
            self.running_token_count.data_ptr(), self.running_page_idx.data_ptr(),
            self.num_layers, max_reqs, self.max_pages_per_req, kv_heads, head_dim, self.page_size,
            self.top_k, int(self.avoid_recent_overlap),
        )
        ws_bytes = int(self.lib.qq_workspace_bytes(0, self.top_k, 0, 0))
        self._workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        self._scores = torch.empty((max_reqs, self.max_pages_per_req), dtype=torch.float32, device=dev)
        check(self.lib.qq_quest_init_storage(self._state, self._stream()), "init_storage")
        self._initialized = True

    def _stream(self) -> int:
        return stream_of(self.device)

    @property
    def page_k_min(self) -> torch.Tensor:
        return self.page_k_bounds[..., 0]

    @property
    def page_k_max(self) -> torch.Tensor:
        return self.page_k_bounds[..., 1]

    @property
    def page_valid(self) -> torch.Tensor:
        return (self.page_k_max > _BF16_NEG_INF).any(dim=(-1, -2))

    def storage_bytes(self) -> int:
        n = self.page_k_bounds.numel() + self.running_k_min.numel() + self.running_k_max.numel()
        return n * 2

    # ------------------------------------------------------------------ helpers

    def _i64(self, x) -> torch.Tensor:
        if not isinstance(x, torch.Tensor):
            x = torch.as_tensor(x)
        return x.to(device=self.device, dtype=torch.int64).contiguous()

    def _scores_buf(self, bs: int) -> torch.Tensor:
        if self._scores is None or self._scores.shape[0] < bs:
            self._scores = torch.empty((bs, self.max_pages_per_req), dtype=torch.float32, device=self.device)
        return self._scores

    def _queries(self, queries: torch.Tensor) -> torch.Tensor:
        """``[bs, H*D]`` or ``[bs, H, D]`` -> contiguous ``[bs, H, D]`` (validation of quest.py:374-390)."""
        bs = queries.shape[0]
        if queries.dim() == 2:
            if queries.shape[1] % self.head_dim != 0:
                raise ValueError(f"Query hidden {queries.shape[1]} not divisible by head_dim {self.head_dim}")
            q = queries.view(bs, queries.shape[1] // self.head_dim, self.head_dim)
        elif queries.dim() == 3:
            q = queries
        else:
            raise ValueError(f"Unsupported query shape {tuple(queries.shape)}")
        if q.shape[1] % self.kv_heads != 0:
            raise ValueError(f"q_heads {q.shape[1]} not divisible by kv_heads {self.kv_heads}")
        if q.shape[2] != self.head_dim:
            raise ValueError(f"query head_dim {q.shape[2]} != {self.head_dim}")
        if q.dtype not in (torch.bfloat16, torch.float32):
            q = q.float()
        return q.to(self.device).contiguous()

    def _layers(self, k_buffers) -> tuple:
        return _lib.ptr_array([t.data_ptr() for t in k_buffers])

    # ------------------------------------------------------ [Q2] prefill bounds

    def update_prefill_representations(self, layer_id, req_pool_idx, k_buffer, prefill_indices) -> None:
        """[Q2] Bounds of one request's prefill keys at one layer (quest.py:231-280)."""
        self._prefill(layer_id, layer_id + 1, [k_buffer], req_pool_idx, prefill_indices)

    def update_prefill_representations_all_layers(self, req_pool_idx, k_buffers, prefill_indices) -> None:
        """[Q2] for every layer ``[start_layer, end_layer)`` in one launch.

        ``k_buffers[i]`` is the K buffer of layer ``start_layer + i``.
        """
        self._prefill(self.start_layer, self.end_layer, list(k_buffers), req_pool_idx, prefill_indices)

    def _prefill(self, layer_begin, layer_end, k_buffers, req, prefill_indices) -> None:
        idx = prefill_indices.to(device=self.device, dtype=torch.int32).contiguous()
        k0 = k_buffers[0]
        arr, keep = self._layers(k_buffers)
        rc = self.lib.qq_quest_bounds_prefill(
            self._state, layer_begin - self.start_layer, layer_end - self.start_layer, arr,
            dtype_code(k0.dtype), k0.stride(0), idx.data_ptr(), int(idx.numel()), int(req),
            int(layer_end == self.end_layer), self._stream(),
        )
        check(rc, "update_prefill_representations")
        del keep

    # ------------------------------------------------------- [Q3] decode bounds

    def update_decode_representations(self, layer_id, req_indices, k_buffer, device_locs) -> None:
        """[Q3] Fold the previous token's key into the running bounds of one layer."""
        reqs = self._i64(req_indices)
        rows = self._i64(device_locs)
        self.decode_step(QQ_STEP_FOLD, reqs, None, [k_buffer], rows=rows,
                         layer_begin=layer_id, layer_end=layer_id + 1)

    def maybe_finalize_decode_representations(self, req_indices) -> None:
        """[Q3] Advance counters; finalize pages whose last token just arrived (all layers)."""
        reqs = self._i64(req_indices)
        self.decode_step(QQ_STEP_FINALIZE, reqs, None, None)

    def decode_step(self, flags, reqs, seq_lens, k_buffers, *, rows=None, skip_flags=None,
                    req_to_token=None, device_buffer_size=0, layer_begin=None, layer_end=None,
                    k_ptrs=None, kv_dtype=None, k_row_stride=None) -> None:
        """One launch of ``qq_quest_decode_step`` over layers ``[layer_begin, layer_end)``."""
        lb = self.start_layer if layer_begin is None else layer_begin
        le = self.end_layer if layer_end is None else layer_end
        bs = int(reqs.shape[0])
        if bs == 0:
            return
        batch = _lib.QQBatch(reqs.data_ptr(), seq_lens.data_ptr() if seq_lens is not None else None, bs)
        keep = None
        if k_ptrs is not None:
            arr = k_ptrs
        elif k_buffers is not None:
            arr, keep = self._layers(k_buffers)
            kv_dtype, k_row_stride = dtype_code(k_buffers[0].dtype), k_buffers[0].stride(0)
        else:
            arr, kv_dtype, k_row_stride = None, QQ_BF16, 0
        table = None
        if req_to_token is not None:
            table = _lib.QQTokenTable(req_to_token.data_ptr(), req_to_token.stride(0), req_to_token.shape[0])
        rc = self.lib.qq_quest_decode_step(
            self._state, flags, lb - self.start_layer, le - self.start_layer, arr, kv_dtype,
            k_row_stride or 0, batch, skip_flags.data_ptr() if skip_flags is not None else None,
            rows.data_ptr() if rows is not None else None, table, int(device_buffer_size),
            self._workspace.data_ptr(), self._workspace.numel(), self._stream(),
        )
        check(rc, "decode bounds step")
        del keep

    # ----------------------------------------------------- [Q4] per-step layout

    def prepare_step(self, seq_lens: torch.Tensor) -> StepLayout:
        """[Q4] Remember this step's ``seq_lens``; the kernels derive the layout from them."""
        seq = self._i64(seq_lens)
        self._step = StepLayout(seq, self.top_k, self.page_size, self.avoid_recent_overlap)
        return self._step

    # ---------------------------------------------------- [Q5] page criticality

    def group_queries(self, queries: torch.Tensor) -> torch.Tensor:
        q = self._queries(queries)
        bs, heads = q.shape[0], q.shape[1]
        if heads == self.kv_heads:
            return q
        out = torch.empty((bs, self.kv_heads, self.head_dim), dtype=q.dtype, device=self.device)
        rc = self.lib.qq_quest_group_queries(q.data_ptr(), dtype_code(q.dtype), bs, heads, self.kv_heads,
                                             self.head_dim, q.stride(0), out.data_ptr(), self._stream())
        check(rc, "group_queries")
        return out

    def page_scores(self, grouped_q: torch.Tensor, layer_id: int, req_pool_indices) -> torch.Tensor:
        """[Q5] ``[bs, max_pages_per_req]`` float32 scores of every page slot."""
        q = self._queries(grouped_q)
        if q.shape[1] != self.kv_heads:
            raise ValueError("page_scores takes grouped queries [bs, kv_heads, head_dim]")
        reqs = self._i64(req_pool_indices)
        bs = int(reqs.shape[0])
        out = torch.empty((bs, self.max_pages_per_req), dtype=torch.float32, device=self.device)
        batch = _lib.QQBatch(reqs.data_ptr(), None, bs)
        rc = self.lib.qq_quest_page_scores(self._state, layer_id - self.start_layer, batch, q.data_ptr(),
                                           dtype_code(q.dtype), q.stride(0), self.max_pages_per_req,
                                           out.data_ptr(), self._stream())
        check(rc, "page_scores")
        return out

    # ----------------------------------------------------------- [Q6] top-k

    def retrieve_topk(self, queries, layer_id, req_pool_indices, seq_lens):
        """[Q6] ``(token_positions [bs, top_k] int32, actual_lens [bs] int32)`` (quest.py:409-464)."""
        step = self._step
        if step is None:
            raise RuntimeError("prepare_step() must be called once per decode step first")
        bs = queries.shape[0]
        if step.seq_lens.shape[0] != bs or seq_lens.shape[0] != bs:
            raise ValueError("batch size differs from the one given to prepare_step()")
        q = self._queries(queries)
        reqs = self._i64(req_pool_indices)
        positions = torch.empty((bs, self.top_k), dtype=torch.int32, device=self.device)
        actual = torch.empty(bs, dtype=torch.int32, device=self.device)
        self.select(q, layer_id, reqs, step.seq_lens, positions, actual)
        return positions, actual

    def select(self, q, layer_id, reqs, seq_lens, positions, actual_lens, *, translate=None,
               rows=None, new_token=None, scores=None) -> torch.Tensor:
        """One launch of ``qq_quest_retrieve_topk``; returns the scores buffer it wrote."""
        bs = int(reqs.shape[0])
        scores = self._scores_buf(bs) if scores is None else scores
        batch = _lib.QQBatch(reqs.data_ptr(), seq_lens.data_ptr(), bs)
        rc = self.lib.qq_quest_retrieve_topk(
            self._state, layer_id - self.start_layer, batch, q.data_ptr(), dtype_code(q.dtype), q.shape[1],
            q.stride(0), positions.data_ptr(), actual_lens.data_ptr() if actual_lens is not None else None,
            scores.data_ptr(), translate, rows.data_ptr() if rows is not None else None, new_token,
            self._workspace.data_ptr(), self._workspace.numel(), self._stream(),
        )
        check(rc, "retrieve_topk")
        if self.trace is not None:
            self._record(layer_id, reqs, seq_lens, positions, scores)
        return scores

    def select_attend(self, q, layer_id, reqs, seq_lens, positions, actual_lens, *, translate, rows,
                      new_token, k_pool, v_pool, scaling, out, err_ptr, scores=None, batch=None) -> None:
        """One ``qq_quest_decode_attention`` call: ``select`` (with ``rows``) and the sparse
        decode attention over those rows into ``out``, the attention kernel starting on each
        request as soon as its rows are written.  Not traced (use ``select`` for traces)."""
        bs = int(reqs.shape[0])
        scores = self._scores_buf(bs) if scores is None else scores
        if batch is None:
            batch = _lib.QQBatch(reqs.data_ptr(), seq_lens.data_ptr(), bs)
        rc = self.lib.qq_quest_decode_attention(
            self._state, layer_id - self.start_layer, batch, q.data_ptr(), dtype_code(q.dtype), q.shape[1],
            q.stride(0), positions.data_ptr(), actual_lens.data_ptr() if actual_lens is not None else None,
            scores.data_ptr(), translate, rows.data_ptr(), new_token, k_pool.data_ptr(), v_pool.data_ptr(),
            k_pool.stride(0), k_pool.shape[0], float(scaling), out.data_ptr(), out.stride(0), err_ptr,
            self._workspace.data_ptr(), self._workspace.numel(), self._stream(),
        )
        check(rc, "decode attention")

    # ------------------------------------------------------ [Q8] request end

    def invalidate_request(self, req_pool_idx: int) -> None:
        check(self.lib.qq_quest_invalidate(self._state, int(req_pool_idx), self._stream()), "invalidate_request")

    # ----------------------------------------------------------- tracing

    def _record(self, layer_id, reqs, seq_lens, positions, scores) -> None:
        """``QuestTrace`` records (quest.py:483-515); copies to the host, so only when tracing."""
        assert self.trace is not None
        P = self.page_size
        sel = self.top_k_pages - 1
        seq = seq_lens.cpu().tolist()
        rq = reqs.cpu().tolist()
        pos = positions.cpu()
        all_short = all(s <= self.top_k for s in seq)
        sc = None if all_short else scores.cpu()
        for i, (seq_len, req) in enumerate(zip(seq, rq)):
            dense = seq_len <= self.top_k
            n = min(seq_len, self.top_k)
            full_pages = seq_len // P
            pages = [] if dense or sel <= 0 else sorted(int(p) // P for p in pos[i, : sel * P : P].tolist())
            self.trace.add(
                QuestSelection(
                    layer_id=layer_id,
                    req_pool_idx=int(req),
                    seq_len=int(seq_len),
                    dense=dense,
                    selected_pages=pages,
                    recent_window=(max(seq_len - P, 0), seq_len),
                    page_scores=None if dense or sc is None else sc[i, :full_pages].clone(),
                    positions=pos[i, :n].to(torch.int64),
                )
            )

    _ = (QQ_F32,)
