"""A model-free serving loop that drives an ``AttentionBackend`` through its lifecycle.

:class:`LifecycleDriver` plays ``Engine.generate`` (``src/qwenquest/engine.py:143-256``)
with the model replaced by seeded ``q/k/v`` (:func:`tests.workloads.scenario_tensors`):
slot and token-pool allocation, prefill forwards, ``on_extend_finished``,
batched decode forwards with ``init_forward_metadata`` once per step, and
``on_request_finished`` before a slot is reused.  It only touches the backend
through the public interface the Engine uses, so the same driver runs the
reference backends (given the reference's classes) and this package's CUDA
backends (given :func:`b200_api`), and records what both decided.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Any

import numpy as np
import torch

from tests._reference import ensure_importable
from tests.workloads import Scenario, scenario_tensors

ensure_importable()


@dataclass
class LifecycleAPI:
    """The classes a driver needs: the reference's pools and batch with either backend family."""

    ForwardBatch: Any
    ForwardMode: Any
    ReqToTokenPool: Any
    MHATokenToKVPool: Any
    TokenToKVPoolAllocator: Any
    QuestOnlyBackend: Any
    QuestHiSparseBackend: Any
    QuestTrace: Any


def reference_api() -> LifecycleAPI:
    """The reference's own backends, pools, batch and trace (``src/qwenquest``)."""
    from qwenquest.attention import QuestHiSparseBackend, QuestOnlyBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool, TokenToKVPoolAllocator
    from qwenquest.quest import QuestTrace

    return LifecycleAPI(
        ForwardBatch, ForwardMode, ReqToTokenPool, MHATokenToKVPool, TokenToKVPoolAllocator,
        QuestOnlyBackend, QuestHiSparseBackend, QuestTrace,
    )


def b200_api() -> LifecycleAPI:
    """The B200 backends and trace with the reference's pools and batch."""
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool, TokenToKVPoolAllocator

    from qwenquest_b200.backends import B200QuestHiSparseBackend, B200QuestOnlyBackend
    from qwenquest_b200.quest import QuestTrace

    return LifecycleAPI(
        ForwardBatch, ForwardMode, ReqToTokenPool, MHATokenToKVPool, TokenToKVPoolAllocator,
        B200QuestOnlyBackend, B200QuestHiSparseBackend, QuestTrace,
    )


@dataclass
class DecodeRecord:
    step: int
    layer: int
    req: int  # admission-order request index
    slot: int  # req_pool_idx
    seq_len: int
    positions: np.ndarray  # [n] int64, attention order
    out: np.ndarray  # [H*D] float32
    buffer_tokens: np.ndarray | None = None
    lru_slots: np.ndarray | None = None
    #: float64 Quest scores of the candidate pages (oracle runs only)
    scores64: np.ndarray | None = None


class LifecycleDriver:
    """Runs one :class:`Scenario` through a backend, recording every decode decision."""

    def __init__(
        self,
        sc: Scenario,
        mode: str,
        api: LifecycleAPI,
        device: str | torch.device,
        *,
        prefill: str = "forward",
        record_hisparse: bool = True,
        trace: bool = True,
    ):
        if mode not in ("quest", "quest_hisparse"):
            raise ValueError(mode)
        if prefill not in ("forward", "direct"):
            raise ValueError(prefill)
        self.sc, self.mode, self.api = sc, mode, api
        self.device = torch.device(device)
        self.prefill_mode = prefill
        self.record_hisparse = record_hisparse and mode == "quest_hisparse"
        self.dtype = torch.bfloat16 if sc.bf16 else torch.float32
        max_ctx = sc.max_context_len
        # engine.py:96-111
        pool_size = max_ctx if mode == "quest_hisparse" else sc.max_running * max_ctx
        self.req_to_token_pool = api.ReqToTokenPool(sc.max_running, max_ctx, self.device)
        self.token_to_kv_pool = api.MHATokenToKVPool(
            pool_size, sc.layers, sc.kv_heads, sc.head_dim, self.dtype, self.device
        )
        self.allocator = api.TokenToKVPoolAllocator(pool_size, self.device)
        # engine.py:115-135
        if mode == "quest":
            self.backend = api.QuestOnlyBackend(
                self.req_to_token_pool, self.token_to_kv_pool, sc.sparse_config()
            )
        else:
            self.backend = api.QuestHiSparseBackend(
                self.req_to_token_pool,
                self.token_to_kv_pool,
                sc.sparse_config(),
                host_pool_size=sc.max_running * max_ctx,
                host_device="cpu",
            )
        if trace:
            self.backend.quest.trace = api.QuestTrace()
        self.layers = [
            SimpleNamespace(
                layer_id=i, num_heads=sc.q_heads, num_kv_heads=sc.kv_heads,
                head_dim=sc.head_dim, scaling=sc.scaling,
            )
            for i in range(sc.layers)
        ]
        self.inputs = [scenario_tensors(sc, r) for r in range(len(sc.prompt_lens))]
        self.records: list[DecodeRecord] = []
        self._slot: dict[int, int] = {}
        self._seq: dict[int, int] = {}
        self._emitted: dict[int, int] = {}
        self._step = 0

    # ------------------------------------------------------------------ helpers

    def _t(self, x: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(x)).to(self.device, self.dtype)

    def _i64(self, xs) -> torch.Tensor:
        return torch.tensor(list(xs), dtype=torch.int64, device=self.device)

    def _finished(self, r: int) -> bool:
        return self._emitted[r] >= self.sc.new_tokens[r] or self._seq[r] >= self.sc.max_context_len

    # ------------------------------------------------------------------ lifecycle

    def run(self) -> list[DecodeRecord]:
        waiting = deque(range(len(self.sc.prompt_lens)))
        running: list[int] = []
        while waiting or running:
            while waiting and len(running) < self.sc.max_running:
                r = waiting.popleft()
                self._prefill(r)
                self._emitted[r] = 1
                if self._finished(r):
                    self._finish(r)
                else:
                    running.append(r)
            if running:
                self._decode(running)
                for r in running:
                    self._emitted[r] += 1
                for r in [x for x in running if self._finished(x)]:
                    running.remove(r)
                    self._finish(r)
        return self.records

    def _prefill(self, r: int) -> None:
        api, sc = self.api, self.sc
        n = sc.prompt_lens[r]
        slot = self.req_to_token_pool.alloc()
        locs = self.allocator.alloc(n)
        self.req_to_token_pool.req_to_token[slot, :n] = locs.to(torch.int32)
        dev = self.device
        batch = api.ForwardBatch(
            forward_mode=api.ForwardMode.EXTEND,
            input_ids=torch.zeros(n, dtype=torch.int64, device=dev),
            positions=torch.arange(n, dtype=torch.int64, device=dev),
            req_pool_indices=self._i64([slot]),
            seq_lens=self._i64([n]),
            out_cache_loc=locs,
            req_to_token_pool=self.req_to_token_pool,
            token_to_kv_pool=self.token_to_kv_pool,
            attn_backend=self.backend,
            extend_prefix_lens=torch.zeros(1, dtype=torch.int64, device=dev),
            extend_seq_lens=self._i64([n]),
        )
        self.backend.init_forward_metadata(batch)
        x = self.inputs[r]
        if self.prefill_mode == "forward":
            for layer in self.layers:
                li = layer.layer_id
                self.backend.forward(
                    self._t(x["q"][li, :n]), self._t(x["k"][li, :n]), self._t(x["v"][li, :n]),
                    layer, batch,
                )
        else:
            for layer in self.layers:
                li = layer.layer_id
                self.token_to_kv_pool.set_kv_buffer(
                    li, locs, self._t(x["k"][li, :n]), self._t(x["v"][li, :n])
                )
            if self.mode == "quest":
                self.backend._update_quest_for_extend(batch)
        self.backend.on_extend_finished(batch)
        if self.backend.frees_prefill_kv_after_admission:
            self.allocator.free(locs)
            self.req_to_token_pool.req_to_token[slot, :n] = 0
        self._slot[r] = slot
        self._seq[r] = n

    def _decode(self, running: list[int]) -> None:
        api = self.api
        slots = [self._slot[r] for r in running]
        pos = [self._seq[r] for r in running]
        req_idx, positions = self._i64(slots), self._i64(pos)
        out_cache_loc = None
        if self.backend.uses_token_pool_for_decode:
            out_cache_loc = self.allocator.alloc(len(running))
            self.req_to_token_pool.req_to_token[req_idx, positions] = out_cache_loc.to(torch.int32)
        batch = api.ForwardBatch(
            forward_mode=api.ForwardMode.DECODE,
            input_ids=torch.zeros(len(running), dtype=torch.int64, device=self.device),
            positions=positions,
            req_pool_indices=req_idx,
            seq_lens=positions + 1,
            out_cache_loc=out_cache_loc,
            req_to_token_pool=self.req_to_token_pool,
            token_to_kv_pool=self.token_to_kv_pool,
            attn_backend=self.backend,
        )
        self.backend.init_forward_metadata(batch)
        trace = self.backend.quest.trace
        for layer in self.layers:
            li = layer.layer_id
            q = self._t(np.stack([self.inputs[r]["q"][li, p] for r, p in zip(running, pos)]))
            k = self._t(np.stack([self.inputs[r]["k"][li, p] for r, p in zip(running, pos)]))
            v = self._t(np.stack([self.inputs[r]["v"][li, p] for r, p in zip(running, pos)]))
            n_before = len(trace.records) if trace is not None else 0
            out = self.backend.forward(q, k, v, layer, batch)
            out_np = out.float().cpu().numpy()
            recs = trace.records[n_before:] if trace is not None else [None] * len(running)
            # without a trace, a B200 backend's positions are read back from its position buffer
            pos_buf = (self.backend._positions[:len(running)].cpu().numpy()
                       if trace is None and hasattr(self.backend, "_positions") else None)
            for i, r in enumerate(running):
                rec = recs[i]
                bt = lru = None
                if self.record_hisparse:
                    coord = self.backend.coord
                    bt = coord.buffer_tokens[li, slots[i]].cpu().numpy().astype(np.int64)
                    lru = coord.lru_slots[li, slots[i]].cpu().numpy().astype(np.int64)
                self.records.append(
                    DecodeRecord(
                        step=self._step, layer=li, req=r, slot=slots[i], seq_len=pos[i] + 1,
                        positions=(rec.positions.numpy().astype(np.int64) if rec is not None
                                   else pos_buf[i, :min(pos[i] + 1, self.sc.top_k)].astype(np.int64)
                                   if pos_buf is not None else np.zeros(0, np.int64)),
                        out=out_np[i], buffer_tokens=bt, lru_slots=lru,
                    )
                )
        for r in running:
            self._seq[r] += 1
        self._step += 1

    def _finish(self, r: int) -> None:
        slot = self._slot[r]
        self.backend.on_request_finished(slot)
        self.allocator.free(self.req_to_token_pool.req_to_token[slot, : self._seq[r]])
        self.req_to_token_pool.free(slot)

    # ------------------------------------------------------------------ export

    def stats(self) -> dict[str, int]:
        if self.mode != "quest_hisparse":
            return {}
        s = self.backend.coord.stats
        return {"hits": int(s.hits), "misses": int(s.misses), "fast_path_calls": int(s.fast_path_calls)}


def records_to_arrays(records: list[DecodeRecord], top_k: int) -> dict[str, np.ndarray]:
    """Pack decode records into fixed-shape arrays (positions padded with -1)."""
    R = len(records)
    out: dict[str, np.ndarray] = {
        "step": np.array([r.step for r in records], np.int32),
        "layer": np.array([r.layer for r in records], np.int32),
        "req": np.array([r.req for r in records], np.int32),
        "slot": np.array([r.slot for r in records], np.int32),
        "seq_len": np.array([r.seq_len for r in records], np.int64),
        "n": np.array([len(r.positions) for r in records], np.int32),
        "out": np.stack([r.out for r in records]).astype(np.float32) if R else np.zeros((0, 0)),
    }
    pos = np.full((R, top_k), -1, np.int32)
    for i, r in enumerate(records):
        pos[i, : len(r.positions)] = r.positions
    out["positions"] = pos
    if R and records[0].buffer_tokens is not None:
        out["buffer_tokens"] = np.stack([r.buffer_tokens for r in records]).astype(np.int32)
        out["lru_slots"] = np.stack([r.lru_slots for r in records]).astype(np.int32)
    return out
