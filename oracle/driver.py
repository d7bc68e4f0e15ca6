"""Runs a :class:`tests.workloads.Scenario` through the numpy oracle — test infrastructure only.

Same schedule as ``Engine.generate`` (``src/qwenquest/engine.py:143-256``) and
as :class:`tests.harness.LifecycleDriver`: slot allocation from a
free list (``memory.py:39-50``), token-pool allocation (``memory.py:53-76``),
prefill writes + bounds / admission, batched decode, finish.
"""

from __future__ import annotations

from collections import deque

import numpy as np

from oracle.backends import OracleKVPools, OracleQuestHiSparseBackend, OracleQuestOnlyBackend
from oracle.parity import score_pages_f64
from tests.harness import DecodeRecord
from tests.workloads import Scenario, scenario_tensors


class OracleLifecycleDriver:
    def __init__(self, sc: Scenario, mode: str):
        self.sc, self.mode = sc, mode
        max_ctx = sc.max_context_len
        pool_size = max_ctx if mode == "quest_hisparse" else sc.max_running * max_ctx
        self.pools = OracleKVPools(
            pool_size, sc.max_running, max_ctx, sc.layers, sc.kv_heads, sc.head_dim, kv_bf16=sc.bf16
        )
        self._free_slots = list(range(sc.max_running))
        if mode == "quest":
            self.backend = OracleQuestOnlyBackend(
                self.pools, sc.top_k, sc.page_size, avoid_recent_overlap=sc.avoid_recent_overlap
            )
        else:
            self.backend = OracleQuestHiSparseBackend(
                self.pools, sc.top_k, sc.page_size, device_buffer_size=sc.device_buffer_size,
                host_pool_size=sc.max_running * max_ctx,
                avoid_recent_overlap=sc.avoid_recent_overlap,
            )
        self.inputs = [scenario_tensors(sc, r) for r in range(len(sc.prompt_lens))]
        self.records: list[DecodeRecord] = []
        self._slot: dict[int, int] = {}
        self._seq: dict[int, int] = {}
        self._emitted: dict[int, int] = {}
        self._step = 0

    def _finished(self, r):
        return self._emitted[r] >= self.sc.new_tokens[r] or self._seq[r] >= self.sc.max_context_len

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

    def _prefill(self, r):
        n = self.sc.prompt_lens[r]
        slot = self._free_slots.pop(0)
        locs = self.pools.allocator.alloc(n)
        self.pools.req_to_token[slot, :n] = locs.astype(np.int32)
        x = self.inputs[r]
        for layer in range(self.sc.layers):
            self.pools.set_kv_buffer(layer, locs, x["k"][layer, :n], x["v"][layer, :n])
        if self.mode == "quest":
            self.backend.update_quest_for_extend([slot], [n])
        else:
            self.backend.on_extend_finished([slot], [n])
            self.pools.allocator.free(locs)
            self.pools.req_to_token[slot, :n] = 0
        self._slot[r] = slot
        self._seq[r] = n

    def _decode(self, running):
        sc = self.sc
        slots = np.array([self._slot[r] for r in running], np.int64)
        pos = np.array([self._seq[r] for r in running], np.int64)
        seq_lens = pos + 1
        out_cache_loc = None
        if self.mode == "quest":
            out_cache_loc = self.pools.allocator.alloc(len(running))
            self.pools.req_to_token[slots, pos] = out_cache_loc.astype(np.int32)
        self.backend.init_forward_metadata_decode(slots, seq_lens)
        for layer in range(sc.layers):
            q = np.stack([self.inputs[r]["q"][layer, p] for r, p in zip(running, pos)])
            k = np.stack([self.inputs[r]["k"][layer, p] for r, p in zip(running, pos)])
            v = np.stack([self.inputs[r]["v"][layer, p] for r, p in zip(running, pos)])
            if self.mode == "quest":
                out, positions, actual = self.backend.forward_decode(
                    q, k, v, layer, slots, seq_lens, out_cache_loc, sc.scaling, q_bf16=sc.bf16
                )
            else:
                out, positions, actual, _ = self.backend.forward_decode(
                    q, k, v, layer, slots, seq_lens, sc.scaling, q_bf16=sc.bf16
                )
            quest = self.backend.quest
            qbar = quest.group_queries(q, query_is_bf16=sc.bf16)
            for i, r in enumerate(running):
                bt = lru = None
                if self.mode == "quest_hisparse":
                    bt = self.backend.coord.buffer_tokens[layer, slots[i]].copy()
                    lru = self.backend.coord.lru_slots[layer, slots[i]].copy()
                s64 = None
                if seq_lens[i] > sc.top_k:
                    c = int(quest._step.candidate_limit[i])
                    s64 = score_pages_f64(quest.page_k_bounds[layer, slots[i], :c], qbar[i])
                self.records.append(
                    DecodeRecord(
                        step=self._step, layer=layer, req=r, slot=int(slots[i]),
                        seq_len=int(seq_lens[i]),
                        positions=positions[i, : int(actual[i])].astype(np.int64),
                        out=out[i].astype(np.float32), buffer_tokens=bt, lru_slots=lru,
                        scores64=s64,
                    )
                )
        for r in running:
            self._seq[r] += 1
        self._step += 1

    def _finish(self, r):
        slot = self._slot[r]
        self.backend.on_request_finished(slot)
        self.pools.allocator.free(self.pools.req_to_token[slot, : self._seq[r]])
        self.pools.req_to_token[slot] = 0
        self._free_slots.append(slot)

    def stats(self):
        if self.mode != "quest_hisparse":
            return {}
        s = self.backend.coord.stats
        return {"hits": s.hits, "misses": s.misses, "fast_path_calls": s.fast_path_calls}
