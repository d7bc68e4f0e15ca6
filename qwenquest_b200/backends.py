"""The Quest attention backends on B200 — drop-ins for the reference's
``QuestOnlyBackend`` (``src/qwenquest/attention/quest_only.py``) and
``QuestHiSparseBackend`` (``src/qwenquest/attention/quest_hisparse.py``).

Same constructor arguments, class flags, lifecycle hooks and public
attributes (``.quest``, ``.coord``, ``.sparse_config``); ``Engine.generate``
runs unchanged once the engine holds one of these as ``attn_backend``.

Per decode step and layer the work is a fixed, small number of launches on
the current stream with no host synchronisation:

* ``init_forward_metadata``: one ``qq_quest_decode_step`` launch folds the
  previous token's key into the running bounds of **all** layers and
  finalizes completed pages (Mode 3 adds the eager host backup launch);
* ``forward_decode``: one ``qq_quest_retrieve_topk`` launch (new K/V write +
  GQA mean + page scores + top-k + layout + ``req_to_token`` translation),
  Mode 3 one ``qq_hisparse_swap_in`` launch, and one
  ``qq_sparse_decode_attention`` launch.

Prefill attention stays dense, as in the reference (``attention/base.py:65-93``);
per prefill layer one ``qq_quest_extend_kv`` launch writes the new K/V rows
and builds that layer's Quest bounds from them (Mode 3 also fills the hot
buffer and backs the layer up to the host tier on a side stream), where the
reference writes the pool and re-reads every key for the bounds after the
last layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from qwenquest.attention.base import AttentionBackend
from qwenquest.attention.ops import extend_attention
from qwenquest.config import parse_hisparse_config

from qwenquest_b200 import _lib
from qwenquest_b200._lib import QQ_STEP_FINALIZE, QQ_STEP_FOLD, check
from qwenquest_b200.hisparse import HiSparseCoordinator, _DeviceError
from qwenquest_b200.kernels import EXTEND_TILE, extend_tiles
from qwenquest_b200.quest import QuestAlgorithm, dtype_code, stream_of

__all__ = ["B200QuestHiSparseBackend", "B200QuestOnlyBackend"]


def _parse_quest_config(sparse_config):
    """The reference's own parsing and check (``quest_only.py:52-54``)."""
    cfg = parse_hisparse_config(sparse_config)
    if cfg.algorithm != "quest" or cfg.quest_page_size is None:
        raise ValueError("Quest backends require hisparse_config with algorithm='quest'")
    return cfg


@dataclass
class _ExtendPlan:
    """The per-batch constants of every prefill layer's ``qq_quest_extend_kv`` launch."""

    batch: object
    reqs: list[int]
    seq_lens: list[int]
    reqs_dev: torch.Tensor  # device int64 [bs]
    tensors: tuple  # every device tensor the struct points into (kept alive with it)
    qq: _lib.QQExtendBatch
    prefix: list[int] = None
    unfused: bool = False
    admission: object = None
    tiles: torch.Tensor | None = None

    @property
    def num_tiles(self) -> int:
        return sum(-(-(s - p) // EXTEND_TILE) for s, p in zip(self.seq_lens, self.prefix, strict=True))

    def tiles_dev(self) -> torch.Tensor:
        """The tile list of ``qq_extend_attention`` (heaviest first), built once per batch."""
        if self.tiles is None:
            self.tiles = torch.tensor(extend_tiles(self.seq_lens, self.prefix), dtype=torch.int32,
                                      device=self.reqs_dev.device)
        return self.tiles


class _QuestDecodeMixin:
    """Shared decode plumbing: step tensors, persistent buffers, the attention launch."""

    quest: QuestAlgorithm
    device: torch.device

    def _extend_attention(self, q, layer, batch) -> torch.Tensor:
        """The attention half of the reference's ``forward_extend`` (``base.py:71-93``), over the K/V rows
        already in the pool.  bf16 pools of head_dim 128 with an even number of query heads per KV head:
        one ``qq_extend_attention`` launch for the whole batch (tcgen05 tensor cores, rows read in place
        through ``req_to_token``).  Other geometries (the reference's fp32 test models) keep the
        reference's own per-request ``extend_attention`` loop on the GPU."""
        k_buf, v_buf = self.token_to_kv_pool.get_kv_buffer(layer.layer_id)
        plan = self._extend_plan(batch)
        if self._prefill_kernel_fits(q, k_buf, plan):
            return self._extend_attention_kernel(q, k_buf, v_buf, layer, plan)
        offsets = batch.extend_token_offsets()
        outputs = []
        for i in range(batch.batch_size):
            req = int(batch.req_pool_indices[i])
            locs = self.req_to_token[req, :int(batch.seq_lens[i])].long()
            outputs.append(extend_attention(q[offsets[i]:offsets[i + 1]], k_buf[locs], v_buf[locs],
                                            prefix_len=int(batch.extend_prefix_lens[i]), scaling=layer.scaling))
        return torch.cat(outputs, dim=0)

    def _prefill_kernel_fits(self, q, k_buf, plan) -> bool:
        if not self.fused_prefill_attention or q.dim() != 3 or k_buf.dim() != 3:
            return False
        heads, dim = q.shape[1], q.shape[2]
        kv = k_buf.shape[1]
        return (q.dtype == torch.bfloat16 and k_buf.dtype == torch.bfloat16 and dim == 128
                and k_buf.shape[2] == dim and heads % kv == 0 and (heads // kv) % 2 == 0
                and k_buf.stride(2) == 1 and k_buf.stride(1) == dim and (k_buf.stride(0) * 2) % 16 == 0
                and k_buf.data_ptr() % 16 == 0 and plan.num_tiles <= 65535 and len(plan.reqs) < 32768)

    def _extend_attention_kernel(self, q, k_buf, v_buf, layer, plan) -> torch.Tensor:
        tokens, heads, dim = q.shape
        if q.stride(2) != 1 or q.stride(1) != dim or (q.stride(0) * 2) % 16 or q.data_ptr() % 16:
            q = q.contiguous()
        out = torch.empty((tokens, heads * dim), dtype=q.dtype, device=self.device)
        tiles = plan.tiles_dev()
        rc = self.lib.qq_extend_attention(
            plan.qq, self._token_table(), tiles.data_ptr(), tiles.numel(), q.data_ptr(), dtype_code(q.dtype),
            heads, k_buf.shape[1], dim, q.stride(0), k_buf.data_ptr(), v_buf.data_ptr(), k_buf.stride(0),
            k_buf.shape[0], float(layer.scaling), out.data_ptr(), out.stride(0), self._xerr.ptr(),
            stream_of(self.device),
        )
        check(rc, "prefill attention")
        return out

    def _setup_decode(self, max_reqs: int) -> None:
        dev = self.device
        top_k = self.quest.top_k
        self._positions = torch.empty((max_reqs, top_k), dtype=torch.int32, device=dev)
        self._rows = torch.empty((max_reqs, top_k), dtype=torch.int32, device=dev)
        self._actual = torch.empty(max_reqs, dtype=torch.int32, device=dev)
        self._attn_ws: torch.Tensor | None = None
        self._attn_err = _DeviceError(torch.zeros(1, dtype=torch.int32).pin_memory())
        self._step_reqs: torch.Tensor | None = None
        self._step_seq: torch.Tensor | None = None
        self._step_dst: torch.Tensor | None = None
        self._step_loc_src = None
        self._step_batch = None
        self._r2t_table = None
        self._max_reqs = max_reqs
        self.lib = _lib.load()
        #: when a dict, every launch of the decode path records a (start, end)
        #: CUDA event pair under its kernel name (benchmark instrumentation)
        self.kernel_events: dict[str, list] | None = None
        #: selection and attention in one call (qq_quest_decode_attention) when
        #: nothing traces the selection or times the kernels one by one
        self.fused = True
        #: prefill K/V write, bounds (and Mode 3 hot buffer) in one launch per
        #: layer (qq_quest_extend_kv); False keeps the reference's order:
        #: set_kv_buffer per layer, bounds from the pool after the last layer
        self.fused_extend = True
        #: dense prefill attention as one qq_extend_attention launch per layer
        #: (bf16, head_dim 128); False keeps the reference's per-request loop
        self.fused_prefill_attention = True
        self._xplan: _ExtendPlan | None = None
        self._xerr = _DeviceError(torch.zeros(1, dtype=torch.int32).pin_memory())

    def _ev_begin(self):
        if self.kernel_events is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(self.device))
        return ev

    def _ev_end(self, name: str, start) -> None:
        if start is None:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(self.device))
        self.kernel_events.setdefault(name, []).append((start, ev))

    def _begin_step(self, batch) -> None:
        self._step_reqs = batch.req_pool_indices.to(device=self.device, dtype=torch.int64).contiguous()
        self._step_seq = batch.seq_lens.to(device=self.device, dtype=torch.int64).contiguous()
        self.quest.prepare_step(self._step_seq)
        # per-step constants of every layer's launch, built once
        loc = getattr(batch, "out_cache_loc", None)
        self._step_dst = None if loc is None else loc.to(device=self.device, dtype=torch.int64).contiguous()
        self._step_loc_src = loc
        self._step_batch = _lib.QQBatch(self._step_reqs.data_ptr(), self._step_seq.data_ptr(),
                                        int(self._step_reqs.shape[0]))

    def _token_table(self) -> _lib.QQTokenTable:
        r2t = self.req_to_token
        t = self._r2t_table
        if t is None or t.req_to_token != r2t.data_ptr() or t.stride != r2t.stride(0):
            t = self._r2t_table = _lib.QQTokenTable(r2t.data_ptr(), r2t.stride(0), r2t.shape[0])
        return t

    def check_errors(self) -> None:
        """Raise for device errors reported by earlier launches (no synchronisation)."""
        _lib.raise_device_error(self._attn_err.take(), "(attention)")
        _lib.raise_device_error(self._xerr.take(), "(prefill K/V write or attention)")

    # ----------------------------------------------------------------- prefill

    def _extend_plan(self, batch) -> _ExtendPlan:
        """Device copies of the batch's request, length, prefix and offset arrays (once per batch)."""
        plan = self._xplan
        if plan is not None and plan.batch is batch:
            return plan
        dev = self.device
        reqs = batch.req_pool_indices.to(device=dev, dtype=torch.int64).contiguous()
        seq = batch.seq_lens.to(device=dev, dtype=torch.int64).contiguous()
        if batch.extend_prefix_lens is None:
            prefix = torch.zeros_like(seq)
        else:
            prefix = batch.extend_prefix_lens.to(device=dev, dtype=torch.int64).contiguous()
        seq_h = [int(x) for x in seq.tolist()]
        if batch.extend_seq_lens is None:
            new_h = [n - p for n, p in zip(seq_h, prefix.tolist(), strict=True)]
        else:
            new_h = [int(x) for x in batch.extend_seq_lens.tolist()]
        if any(n < 0 for n in new_h) or any(
                s - p != n for s, p, n in zip(seq_h, prefix.tolist(), new_h, strict=True)):
            raise ValueError("extend batch: seq_lens must equal extend_prefix_lens + extend_seq_lens")
        offsets_h = [0]
        for n in new_h[:-1]:
            offsets_h.append(offsets_h[-1] + n)
        offsets = torch.tensor(offsets_h, dtype=torch.int64, device=dev)
        loc = batch.out_cache_loc.to(device=dev, dtype=torch.int64).contiguous()
        if loc.numel() != sum(new_h):
            raise ValueError(f"extend batch: {loc.numel()} out_cache_loc rows for {sum(new_h)} new tokens")
        qq = _lib.QQExtendBatch(reqs.data_ptr(), seq.data_ptr(), prefix.data_ptr(), offsets.data_ptr(),
                                loc.data_ptr(), loc.numel(), len(seq_h), max(seq_h, default=0))
        plan = _ExtendPlan(batch, [int(x) for x in reqs.tolist()], seq_h, reqs, (reqs, seq, prefix, offsets, loc), qq,
                           prefix=[int(x) for x in prefix.tolist()])
        self._xplan = plan
        return plan

    def _extend_write(self, k, v, layer_id: int, plan: _ExtendPlan, hot=None) -> None:
        """[Q2] one prefill layer: new K/V rows into the pool and this layer's bounds, one launch."""
        k_buf, v_buf = self.token_to_kv_pool.get_kv_buffer(layer_id)
        q = self.quest
        dim = q.kv_heads * q.head_dim
        n = k.shape[0]
        kk = k.to(k_buf.dtype).reshape(n, dim)
        vv = v.to(v_buf.dtype).reshape(n, dim)
        esize = kk.element_size()
        if (kk.stride(1) != 1 or vv.stride(1) != 1 or kk.stride(0) != vv.stride(0)
                or (kk.stride(0) * esize) % 4 or kk.data_ptr() % 4 or vv.data_ptr() % 4):
            # the kernel moves 4- or 16-byte words: fresh contiguous copies are aligned
            kk, vv = kk.contiguous().clone(), vv.contiguous().clone()
        in_quest = q.start_layer <= layer_id < q.end_layer
        rc = self.lib.qq_quest_extend_kv(
            q._state if in_quest else None, layer_id - q.start_layer, int(layer_id == q.end_layer - 1),
            plan.qq, self._token_table(), kk.data_ptr(), vv.data_ptr(), dtype_code(k_buf.dtype), dim,
            kk.stride(0), k_buf.data_ptr(), v_buf.data_ptr(), k_buf.stride(0), k_buf.shape[0], hot,
            self._xerr.ptr(), stream_of(self.device),
        )
        check(rc, "prefill K/V write")

    def _extend_fusable(self) -> bool:
        """The one-launch prefill write takes bf16 / fp32 pools whose rows are a multiple of 4 bytes."""
        pool = self.token_to_kv_pool
        if not self.fused_extend or pool.dtype not in (torch.bfloat16, torch.float32):
            return False
        k_buf = pool.get_key_buffer(self.quest.start_layer)
        row_bytes = self.quest.kv_heads * self.quest.head_dim * k_buf.element_size()
        return row_bytes % 4 == 0 and (k_buf.stride(0) * k_buf.element_size()) % 4 == 0

    def synchronize(self) -> None:
        """Wait for this backend's work and raise any device error it reported."""
        torch.cuda.current_stream(self.device).synchronize()
        self.check_errors()

    def _workspace(self, q_heads: int, head_dim: int) -> torch.Tensor:
        need = int(self.lib.qq_workspace_bytes(self._max_reqs, self.quest.top_k, q_heads, head_dim))
        if self._attn_ws is None or self._attn_ws.numel() < need:
            self._attn_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._attn_ws

    def _attend(self, q3, layer, reqs, seq, rows, k_pool, v_pool) -> torch.Tensor:
        bs, heads, dim = q3.shape
        out = torch.empty((bs, heads * dim), dtype=q3.dtype, device=self.device)
        ws = self._workspace(heads, dim)
        batch = _lib.QQBatch(reqs.data_ptr(), seq.data_ptr(), bs)
        ev = self._ev_begin()
        rc = self.lib.qq_sparse_decode_attention(
            batch, self.quest.top_k, q3.data_ptr(), dtype_code(q3.dtype), heads, self.quest.kv_heads, dim,
            q3.stride(0), rows.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.stride(0),
            k_pool.shape[0], float(layer.scaling), out.data_ptr(), out.stride(0), self._attn_err.ptr(),
            ws.data_ptr(), ws.numel(), stream_of(self.device),
        )
        check(rc, "sparse decode attention")
        self._ev_end("sparse_decode_attention", ev)
        return out

    def _new_token(self, k, v, k_dst, v_dst, dst_rows, buf) -> _lib.QQNewToken:
        dim = self.quest.kv_heads * self.quest.head_dim
        return _lib.QQNewToken(
            k.data_ptr(), v.data_ptr(), dim, k_dst.data_ptr(), v_dst.data_ptr(), k_dst.stride(0),
            dst_rows.data_ptr() if dst_rows is not None else None, int(buf), int(k_dst.shape[0]),
            dtype_code(k_dst.dtype),
        )

    def _q3(self, q, bs) -> torch.Tensor:
        q3 = q.reshape(bs, -1, self.quest.head_dim)
        if q3.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"unsupported query dtype {q3.dtype}")
        return q3.contiguous()


class B200QuestOnlyBackend(_QuestDecodeMixin, AttentionBackend):
    """Mode 2: Quest top-k with the full KV pool on the device (quest_only.py:39-167)."""

    name = "flashinfer_quest"

    def __init__(self, req_to_token_pool, token_to_kv_pool, sparse_config, *, start_layer: int = 0,
                 end_layer: int | None = None):
        AttentionBackend.__init__(self, req_to_token_pool, token_to_kv_pool)
        cfg = _parse_quest_config(sparse_config)
        self.sparse_config = cfg
        self.device = torch.device(token_to_kv_pool.device)
        if self.device.type != "cuda":
            raise ValueError("B200QuestOnlyBackend needs the KV pool on a CUDA device")
        self.quest = QuestAlgorithm(top_k=cfg.top_k, page_size=cfg.quest_page_size, device=self.device,
                                    avoid_recent_overlap=cfg.avoid_recent_overlap)
        self.device = self.quest.device
        self.quest.init_storage(
            start_layer=start_layer,
            end_layer=token_to_kv_pool.num_layers if end_layer is None else end_layer,
            max_reqs=req_to_token_pool.size,
            max_context_len=req_to_token_pool.max_context_len,
            kv_heads=token_to_kv_pool.kv_heads,
            head_dim=token_to_kv_pool.head_dim,
        )
        self._skip_first_decode_update = torch.zeros(req_to_token_pool.size, dtype=torch.uint8, device=self.device)
        q = self.quest
        self._k_layers = _lib.ptr_array(
            [token_to_kv_pool.get_key_buffer(layer).data_ptr() for layer in range(q.start_layer, q.end_layer)]
        )
        kb0 = token_to_kv_pool.get_key_buffer(q.start_layer)
        self._kv_dtype, self._k_row_stride = dtype_code(kb0.dtype), kb0.stride(0)
        self._setup_decode(req_to_token_pool.size)

    # ---------------------------------------------------------------- per step

    def init_forward_metadata(self, batch) -> None:
        if batch.forward_mode.is_decode():
            self.check_errors()
            self._begin_step(batch)
            # [Q3] fold the previous token (seq_len - 2) into all layers' running bounds (quest_only.py:84-97)
            ev = self._ev_begin()
            self.quest.decode_step(
                QQ_STEP_FOLD | QQ_STEP_FINALIZE, self._step_reqs, self._step_seq, None,
                skip_flags=self._skip_first_decode_update, req_to_token=self.req_to_token,
                k_ptrs=self._k_layers[0], kv_dtype=self._kv_dtype, k_row_stride=self._k_row_stride,
            )
            self._ev_end("quest_decode_step", ev)

    # ----------------------------------------------------------------- prefill

    def forward_extend(self, q, k, v, layer, batch) -> torch.Tensor:
        li = layer.layer_id
        plan = self._extend_plan(batch)
        if self._extend_fusable() and not plan.unfused:
            # [Q2] K/V write + this layer's bounds in one launch
            assert batch.out_cache_loc is not None
            self._extend_write(k, v, li, plan)
            out = self._extend_attention(q, layer, batch)
            if li == self.quest.end_layer - 1:
                self._skip_first_decode_update.index_fill_(0, plan.reqs_dev, 1)
            return out
        plan.unfused = True
        out = super().forward_extend(q, k, v, layer, batch)
        if li == self.quest.end_layer - 1:
            self._update_quest_for_extend(batch)
        return out

    def on_extend_finished(self, batch) -> None:
        if self._xplan is not None and self._xplan.batch is batch:
            self._xplan = None  # the prefill's device index arrays

    def _update_quest_for_extend(self, batch) -> None:
        """[Q2] bounds of positions ``0 .. seq_len-1`` of every layer (quest_only.py:101-128)."""
        q = self.quest
        kb = [self.token_to_kv_pool.get_key_buffer(layer) for layer in range(q.start_layer, q.end_layer)]
        for req_idx, seq_len in zip(batch.req_pool_indices.tolist(), batch.seq_lens.tolist(), strict=True):
            prefill_indices = self.req_to_token[req_idx, :seq_len]
            q.update_prefill_representations_all_layers(req_idx, kb, prefill_indices)
            self._skip_first_decode_update[req_idx] = 1

    # ------------------------------------------------------------------ decode

    def forward_decode(self, q, k, v, layer, batch) -> torch.Tensor:
        assert batch.out_cache_loc is not None
        li = layer.layer_id
        if self._step_reqs is None or self._step_reqs.shape[0] != batch.batch_size:
            self._begin_step(batch)
        reqs, seq = self._step_reqs, self._step_seq
        bs = reqs.shape[0]
        k_buf, v_buf = self.token_to_kv_pool.get_kv_buffer(li)
        q3 = self._q3(q, bs)
        kk = k.to(k_buf.dtype).reshape(bs, -1).contiguous()
        vv = v.to(v_buf.dtype).reshape(bs, -1).contiguous()
        dst = self._step_dst
        if dst is None or dst.shape[0] != bs or batch.out_cache_loc is not getattr(self, "_step_loc_src", None):
            dst = batch.out_cache_loc.to(device=self.device, dtype=torch.int64).contiguous()
        nt = self._new_token(kk, vv, k_buf, v_buf, dst, 0)
        table = self._token_table()
        if self.fused and self.kernel_events is None and self.quest.trace is None:
            # [Q6] + [Q7] selection, translation, new K/V write and attention in one call:
            # the attention starts on each request as soon as its rows are written
            out = torch.empty((bs, q3.shape[1] * q3.shape[2]), dtype=q3.dtype, device=self.device)
            self.quest.select_attend(q3, li, reqs, seq, self._positions, self._actual, translate=table,
                                     rows=self._rows, new_token=nt, k_pool=k_buf, v_pool=v_buf,
                                     scaling=layer.scaling, out=out, err_ptr=self._attn_err.ptr(),
                                     batch=self._step_batch)
            return out
        # [Q6] + [Q7] translation + new K/V write, one launch
        ev = self._ev_begin()
        self.quest.select(q3, li, reqs, seq, self._positions, self._actual, translate=table,
                          rows=self._rows, new_token=nt)
        self._ev_end("quest_retrieve_topk", ev)
        # [Q7] attention over exactly those rows (duplicates kept)
        return self._attend(q3, layer, reqs, seq, self._rows, k_buf, v_buf)

    # --------------------------------------------------------------- lifecycle

    def on_request_finished(self, req_pool_idx: int) -> None:
        self.quest.invalidate_request(req_pool_idx)
        self._skip_first_decode_update[req_pool_idx] = 0


class B200QuestHiSparseBackend(_QuestDecodeMixin, AttentionBackend):
    """Mode 3: Quest top-k + HiSparse host tier / LRU hot buffer (quest_hisparse.py:44-138)."""

    name = "flashinfer_hisparse"
    uses_token_pool_for_decode = False
    frees_prefill_kv_after_admission = True

    def __init__(self, req_to_token_pool, token_to_kv_pool, sparse_config, *, host_pool_size: int,
                 start_layer: int = 0, end_layer: int | None = None, host_device="cpu",
                 host_layers: int | None = None):
        AttentionBackend.__init__(self, req_to_token_pool, token_to_kv_pool)
        cfg = _parse_quest_config(sparse_config)
        self.sparse_config = cfg
        self.device = torch.device(token_to_kv_pool.device)
        if self.device.type != "cuda":
            raise ValueError("B200QuestHiSparseBackend needs the KV pool on a CUDA device")
        num_layers = token_to_kv_pool.num_layers
        self.quest = QuestAlgorithm(top_k=cfg.top_k, page_size=cfg.quest_page_size, device=self.device,
                                    avoid_recent_overlap=cfg.avoid_recent_overlap)
        self.device = self.quest.device
        self.quest.init_storage(
            start_layer=start_layer,
            end_layer=num_layers if end_layer is None else end_layer,
            max_reqs=req_to_token_pool.size,
            max_context_len=req_to_token_pool.max_context_len,
            kv_heads=token_to_kv_pool.kv_heads,
            head_dim=token_to_kv_pool.head_dim,
        )
        self.coord = HiSparseCoordinator(
            quest=self.quest,
            num_layers=num_layers,
            kv_heads=token_to_kv_pool.kv_heads,
            head_dim=token_to_kv_pool.head_dim,
            max_reqs=req_to_token_pool.size,
            max_context_len=req_to_token_pool.max_context_len,
            top_k=cfg.top_k,
            device_buffer_size=cfg.device_buffer_size,
            host_pool_size=host_pool_size,
            dtype=token_to_kv_pool.dtype,
            device=self.device,
            host_device=host_device,
            host_layers=host_layers,
        )
        self._setup_decode(req_to_token_pool.size)

    def check_errors(self) -> None:
        super().check_errors()
        self.coord.check_errors("(swap-in)")

    def init_forward_metadata(self, batch) -> None:
        if batch.forward_mode.is_decode():
            self.check_errors()
            self.coord.prepare_decode_step(batch.req_pool_indices, batch.seq_lens)
            self._begin_step(batch)

    def forward_extend(self, q, k, v, layer, batch) -> torch.Tensor:
        li = layer.layer_id
        plan = self._extend_plan(batch)
        if self._extend_fusable() and not plan.unfused:
            # [H1] + [Q2] K/V write, hot buffer and this layer's bounds in one
            # launch; the layer's host backup follows on a side stream
            assert batch.out_cache_loc is not None
            if plan.admission is None:
                plan.admission = self.coord.begin_admission(plan.reqs, plan.seq_lens, self.req_to_token)
            self._extend_write(k, v, li, plan, hot=self.coord.hot_buffer(li))
            self.coord.backup_layer(plan.admission, li, self.token_to_kv_pool)
            return self._extend_attention(q, layer, batch)
        if plan.admission is not None:
            raise RuntimeError("a prefill batch switched from the fused K/V write to set_kv_buffer")
        plan.unfused = True
        return super().forward_extend(q, k, v, layer, batch)

    def on_extend_finished(self, batch) -> None:
        plan = self._xplan
        if plan is not None and plan.batch is batch and plan.admission is not None:
            self.coord.finish_admission(plan.admission)
            self._xplan = None
            return
        for req_idx, seq_len in zip(batch.req_pool_indices.tolist(), batch.seq_lens.tolist(), strict=True):
            prefill_indices = self.req_to_token[req_idx, :seq_len]
            self.coord.admit_request(req_idx, seq_len, self.token_to_kv_pool, prefill_indices)

    def forward_decode(self, q, k, v, layer, batch) -> torch.Tensor:
        li = layer.layer_id
        if self._step_reqs is None or self._step_reqs.shape[0] != batch.batch_size:
            self._begin_step(batch)
        reqs, seq = self._step_reqs, self._step_seq
        bs = reqs.shape[0]
        coord = self.coord
        k_dev, v_dev = coord.device_k[li], coord.device_v[li]
        q3 = self._q3(q, bs)
        kk = k.to(k_dev.dtype).reshape(bs, -1).contiguous()
        vv = v.to(v_dev.dtype).reshape(bs, -1).contiguous()
        # 1. new K/V into the newest slot, 2. [Q6] selection — one launch
        nt = self._new_token(kk, vv, k_dev, v_dev, None, coord.device_buffer_size)
        ev = self._ev_begin()
        self.quest.select(q3, li, reqs, seq, self._positions, self._actual, new_token=nt)
        self._ev_end("quest_retrieve_topk", ev)
        # 3. [H3] positions -> hot-buffer rows (misses copied from the host tier)
        ev = self._ev_begin()
        coord.swap_in(reqs, seq, self._positions, li, self._rows)
        self._ev_end("hisparse_swap_in", ev)
        # 4. [Q7] attention over the hot buffer
        return self._attend(q3, layer, reqs, seq, self._rows, k_dev, v_dev)

    def on_request_finished(self, req_pool_idx: int) -> None:
        self.check_errors()
        self.coord.request_finished(req_pool_idx)

