"""Seeded synthetic workloads for the Quest decode path.

Two kinds of workload live here:

* :class:`Scenario` — a small, complete serving lifecycle (admission,
  prefill, batched decode, request finish and slot reuse) described by its
  geometry and prompt lengths.  :func:`scenario_tensors` turns it into seeded
  per-request ``q/k/v`` arrays (numpy, float32; bf16-exact when the model
  dtype is bf16).  The same arrays drive the reference (when it is
  importable), the numpy oracle and the CUDA backends.
* The benchmark configurations (``config0`` … ``config3``): the value
  distributions of the benchmark specification — K, V ~ N(0,1) scaled per
  channel by LogNormal(0, 0.5), q ~ N(0,1), a few planted pages, a random-walk
  drift for long contexts.  They are generated on the target device with
  ``torch`` so that multi-GB pools never pass through host memory.

There is no public dataset for this path: these seeded inputs are the whole
workload.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def _round_bf16_np(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value (round-to-nearest-even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


@dataclass(frozen=True)
class Scenario:
    """A seeded serving lifecycle without a model.

    Requests are admitted in order while fewer than ``max_running`` run, each
    is prefilled alone, then all running requests decode together; request
    ``r`` stops after ``new_tokens[r]`` emitted tokens (the prefill emits the
    first), exactly like ``Engine.generate`` (``src/qwenquest/engine.py:143-192``).
    """

    name: str
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    bf16: bool
    top_k: int
    page_size: int
    device_buffer_size: int
    prompt_lens: tuple[int, ...]
    new_tokens: tuple[int, ...]
    max_running: int
    max_context_len: int
    avoid_recent_overlap: bool = False
    seed: int = 0
    #: number of pages whose keys are pulled towards the request's query mean
    planted_pages: int = 2
    #: > 0: K = scale * (W + N(0,1)) with W a per-(layer, head, channel)
    #: random walk along the positions, steps N(0, k_walk^2) (benchmark config 2)
    k_walk: float = 0.0
    #: > 0: decode queries follow q[t+1] = q_ar * q[t] + N(0,1) (benchmark config 3)
    q_ar: float = 0.0
    #: generate q only for decode positions (>= prompt length); prefill must be "direct"
    q_decode_only: bool = False
    extra: dict = field(default_factory=dict, hash=False, compare=False)

    @property
    def scaling(self) -> float:
        return float(self.head_dim) ** -0.5

    def sparse_config(self) -> dict:
        d = {
            "algorithm": "quest",
            "top_k": self.top_k,
            "quest_page_size": self.page_size,
            "device_buffer_size": self.device_buffer_size,
        }
        if self.avoid_recent_overlap:
            d["avoid_recent_overlap"] = True
        return d


class OffsetRows:
    """``[layers, positions, ...]`` rows that start at position ``start``: ``x[layer, p]`` is position ``p``."""

    def __init__(self, rows: np.ndarray, start: int):
        self.rows, self.start = rows, start

    def __getitem__(self, key):
        layer, pos = key
        if isinstance(pos, slice):
            if self.start and (pos.start or 0) < self.start:
                raise IndexError("rows before the first generated position")
            return self.rows[layer, slice((pos.start or 0) - self.start,
                                          None if pos.stop is None else pos.stop - self.start)]
        return self.rows[layer, pos - self.start]


def scenario_tensors(sc: Scenario, req: int) -> dict[str, np.ndarray]:
    """Seeded ``q/k/v`` of request ``req`` (admission-order index) for every position.

    Returns float32 arrays ``k, v: [layers, total, kv_heads, head_dim]`` and
    ``q: [layers, total, q_heads, head_dim]`` with ``total = prompt + new
    tokens``; bf16-exact when ``sc.bf16``.  Row ``t`` is the token at
    position ``t``; ``q`` rows of prompt positions feed prefill.  With
    ``sc.q_decode_only`` ``q`` is an :class:`OffsetRows` of the decode
    positions only.
    """
    if sc.k_walk or sc.q_ar or sc.q_decode_only:
        return _scenario_tensors_v2(sc, req)
    total = sc.prompt_lens[req] + sc.new_tokens[req]
    rng = np.random.default_rng([sc.seed, req])
    L, H, KV, D = sc.layers, sc.q_heads, sc.kv_heads, sc.head_dim
    scale = rng.lognormal(0.0, 0.5, size=(L, 1, KV, D)).astype(np.float32)
    k = rng.standard_normal((L, total, KV, D), dtype=np.float32) * scale
    v = rng.standard_normal((L, total, KV, D), dtype=np.float32) * scale
    q = rng.standard_normal((L, total, H, D), dtype=np.float32)
    if sc.planted_pages and sc.prompt_lens[req] >= 2 * sc.page_size:
        group = H // KV
        # the query of the first decode step (position = prompt length)
        qd = q[:, sc.prompt_lens[req]]
        if sc.bf16:
            qd = _round_bf16_np(qd)
        qbar = qd.reshape(L, KV, group, D).mean(axis=2)  # [L, KV, D]
        full = sc.prompt_lens[req] // sc.page_size
        pages = rng.choice(full, size=min(sc.planted_pages, full), replace=False)
        for p in pages.tolist():
            sl = slice(p * sc.page_size, (p + 1) * sc.page_size)
            k[:, sl] += 0.5 * qbar[:, None]
    if sc.bf16:
        q, k, v = _round_bf16_np(q), _round_bf16_np(k), _round_bf16_np(v)
    return {"q": q, "k": k, "v": v}


def _scenario_tensors_v2(sc: Scenario, req: int) -> dict:
    """The benchmark's config-2 / config-3 distributions (see :class:`Scenario`)."""
    prompt = sc.prompt_lens[req]
    total = prompt + sc.new_tokens[req]
    rng = np.random.default_rng([sc.seed, req, 2])
    L, H, KV, D = sc.layers, sc.q_heads, sc.kv_heads, sc.head_dim
    scale = rng.lognormal(0.0, 0.5, size=(L, 1, KV, D)).astype(np.float32)
    k = rng.standard_normal((L, total, KV, D), dtype=np.float32)
    if sc.k_walk:
        walk = rng.standard_normal((L, total, KV, D), dtype=np.float32)
        walk *= np.float32(sc.k_walk)
        np.cumsum(walk, axis=1, out=walk)
        k += walk
        del walk
    k *= scale
    v = rng.standard_normal((L, total, KV, D), dtype=np.float32) * scale
    q0 = prompt if sc.q_decode_only else 0
    q = rng.standard_normal((L, total - q0, H, D), dtype=np.float32)
    if sc.q_ar:
        first = prompt - q0  # the first decode query keeps its N(0,1) draw
        for t in range(first + 1, total - q0):
            q[:, t] += np.float32(sc.q_ar) * q[:, t - 1]
    if sc.planted_pages and prompt >= 2 * sc.page_size:
        group = H // KV
        qd = q[:, prompt - q0]
        if sc.bf16:
            qd = _round_bf16_np(qd)
        qbar = qd.reshape(L, KV, group, D).mean(axis=2)
        full = prompt // sc.page_size
        pages = rng.choice(full, size=min(sc.planted_pages, full), replace=False)
        for p in pages.tolist():
            k[:, p * sc.page_size:(p + 1) * sc.page_size] += 0.5 * qbar[:, None]
    if sc.bf16:
        q, k, v = _round_bf16_np(q), _round_bf16_np(k), _round_bf16_np(v)
    return {"q": OffsetRows(q, q0) if q0 else q, "k": k, "v": v}


# --------------------------------------------------------------------------- #
# Benchmark configurations (generated on the device with torch)
# --------------------------------------------------------------------------- #

#: Qwen3-30B-A3B attention geometry
Q_HEADS, KV_HEADS, HEAD_DIM = 32, 4, 128
TOP_K, PAGE = 2048, 64


def torch_generator(device, seed: int):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def channel_scale(device, seed: int, layers: int = 1):
    """Per-(layer, kv head, channel) scale ~ LogNormal(0, 0.5), float32 ``[layers, KV, D]``."""
    import torch

    g = torch_generator(device, seed)
    return torch.exp(0.5 * torch.randn(layers, KV_HEADS, HEAD_DIM, generator=g, device=device))


def fill_rows_normal_(dst, scale, gen, chunk_rows: int = 1 << 18) -> None:
    """``dst[rows, KV, D] = bf16(N(0,1) * scale)``, generated in chunks on ``dst.device``."""
    import torch

    n = dst.shape[0]
    for s in range(0, n, chunk_rows):
        e = min(n, s + chunk_rows)
        x = torch.randn((e - s,) + tuple(dst.shape[1:]), generator=gen, device=dst.device)
        dst[s:e].copy_(x.mul_(scale))
