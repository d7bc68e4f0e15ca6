"""numpy restatement of ``Qwen3MoeSparseMoeBlock.forward`` (``src/qwenquest/model/qwen3_moe.py:121-147``) — oracle only.

The reference computes in the input dtype; in bf16 every tensor it makes is
rounded to bf16: the gate logits (``:133``), each projection's output, the
SiLU, the product (``Qwen3MoeMLP.forward``, ``:116-117``), the weighted
expert output and every ``index_add_`` into the bf16 output (``:144-146``).
The restatement rounds at the same places (``round_bf16``) and sums in
float32; the top-k takes the larger probability first, ties to the lower
expert.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import round_bf16


def _silu(v: np.ndarray) -> np.ndarray:
    return (v / (np.float32(1.0) + np.exp(-v, dtype=np.float32))).astype(np.float32)


def sparse_moe_block(x, gate_w, w_gate, w_up, w_down, top_k: int, norm_topk_prob: bool, *, bf16: bool):
    """``x`` ``[T, H]``; ``gate_w`` ``[E, H]``; ``w_gate``/``w_up`` ``[E, I, H]``; ``w_down`` ``[E, H, I]``.
    Returns ``[T, H]`` float32 (bf16-exact when ``bf16``)."""
    rnd = round_bf16 if bf16 else (lambda a: np.asarray(a, dtype=np.float32))
    x = np.asarray(x, dtype=np.float32)
    logits = rnd(x @ np.asarray(gate_w, np.float32).T)                       # :133
    z = logits - logits.max(axis=-1, keepdims=True)
    probs = np.exp(z, dtype=np.float32)
    probs = probs / probs.sum(axis=-1, keepdims=True, dtype=np.float32)     # :134 (fp32)
    experts = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k]          # :135
    weights = np.take_along_axis(probs, experts, axis=-1)
    if norm_topk_prob:
        weights = weights / weights.sum(axis=-1, keepdims=True, dtype=np.float32)  # :136-137
    weights = rnd(weights)                                                   # :138
    out = np.zeros_like(x)
    for e in np.unique(experts):                                             # :141
        token_idx, slot = np.nonzero(experts == e)                           # :142
        xe = x[token_idx]
        g = rnd(xe @ np.asarray(w_gate[e], np.float32).T)
        u = rnd(xe @ np.asarray(w_up[e], np.float32).T)
        h = rnd(rnd(_silu(g)) * u)                                           # :116-117
        y = rnd(h @ np.asarray(w_down[e], np.float32).T)
        y = rnd(y * weights[token_idx, slot, None])                          # :143
        out[token_idx] = rnd(out[token_idx] + y)                             # :144 index_add_
    return out
