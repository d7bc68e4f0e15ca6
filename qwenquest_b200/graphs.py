"""A Quest decode step captured in a CUDA graph and replayed.

Per decode step ``B200QuestOnlyBackend`` makes 1 + 2 x layers launches (the
step's bounds fold, then per layer the selection and the attention) and per
layer some Python and ctypes work to set each launch up (~35 us of host time
per layer, more than the GPU needs for a small batch).  Captured once in a
CUDA graph, a step becomes one graph launch: the host cost of a 48-layer step
falls from ~1.8 ms to a few tens of microseconds, and the launches keep their
programmatic (early-launch) dependencies.

Inputs are static: ``q``, ``k``, ``v`` (``[layers, bs, heads, head_dim]``) and
the batch's ``req_pool_indices``, ``seq_lens`` and ``out_cache_loc`` are copied
into buffers the graph owns before each replay; the outputs are the graph's own
``[bs, heads * head_dim]`` tensors per layer, overwritten by the next replay
(with ``stack_outputs`` also gathered into one ``[layers, bs, heads *
head_dim]`` tensor inside the graph, for a single device-to-host copy).

Inside the graph the backend makes the same call per layer as eagerly: the
fused ``qq_quest_decode_attention`` (selection and attention, the attention
starting on each request as soon as its rows are written), whose per-call
epoch is kept on the device and so is renewed on every replay; with
``backend.fused = False`` the two calls.  A HiSparse (Mode 3) step is
captured the same way: its per-step plan, bounds fold and host backup, and
per layer the selection, the swap-in and the attention, all on the device.
"""

from __future__ import annotations

import torch
from qwenquest.batch import ForwardBatch, ForwardMode

from .backends import B200QuestHiSparseBackend, B200QuestOnlyBackend

__all__ = ["DecodeStepGraph"]


class DecodeStepGraph:
    """One decode step of ``backend`` over ``layers``, captured for a fixed batch size.

    The backend must have run at least one eager decode step (its kernels'
    one-time set-up and its workspace happen then); capturing runs nothing, so
    the backend's state advances only on ``replay``.
    """

    def __init__(self, backend: B200QuestOnlyBackend | B200QuestHiSparseBackend, layers, batch: ForwardBatch,
                 q, k, v, *, stack_outputs: bool = False):
        if not isinstance(backend, (B200QuestOnlyBackend, B200QuestHiSparseBackend)):
            raise TypeError("DecodeStepGraph captures B200QuestOnlyBackend / B200QuestHiSparseBackend decode steps")
        if backend.quest.trace is not None or backend.kernel_events is not None:
            raise ValueError("a traced or per-kernel-timed backend copies to the host every layer")
        dev = backend.device
        self.backend = backend
        self.layers = list(layers)
        self.q = q.detach().clone()
        self.k = k.detach().clone()
        self.v = v.detach().clone()
        self.req_pool_indices = batch.req_pool_indices.to(device=dev, dtype=torch.int64).clone()
        self.seq_lens = batch.seq_lens.to(device=dev, dtype=torch.int64).clone()
        self.out_cache_loc = (None if batch.out_cache_loc is None else
                              batch.out_cache_loc.to(device=dev, dtype=torch.int64).clone())
        bs = int(self.req_pool_indices.shape[0])
        self.batch = ForwardBatch(
            forward_mode=ForwardMode.DECODE,
            input_ids=torch.zeros(bs, dtype=torch.int64, device=dev),
            positions=self.seq_lens - 1,
            req_pool_indices=self.req_pool_indices,
            seq_lens=self.seq_lens,
            out_cache_loc=self.out_cache_loc,
            req_to_token_pool=batch.req_to_token_pool,
            token_to_kv_pool=batch.token_to_kv_pool,
            attn_backend=backend,
        )
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            backend.init_forward_metadata(self.batch)
            self.out = [backend.forward(self.q[layer.layer_id], self.k[layer.layer_id],
                                        self.v[layer.layer_id], layer, self.batch)
                        for layer in self.layers]
            self.out_stacked = torch.stack(self.out) if stack_outputs else None

    def replay(self, batch: ForwardBatch | None = None, q=None, k=None, v=None) -> list[torch.Tensor]:
        """Copy this step's inputs into the graph's buffers (those given), then run the step."""
        if batch is not None:
            self.req_pool_indices.copy_(batch.req_pool_indices, non_blocking=True)
            self.seq_lens.copy_(batch.seq_lens, non_blocking=True)
            if self.out_cache_loc is not None:
                self.out_cache_loc.copy_(batch.out_cache_loc, non_blocking=True)
        for dst, src in ((self.q, q), (self.k, k), (self.v, v)):
            if src is not None:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out
