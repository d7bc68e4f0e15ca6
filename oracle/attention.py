"""numpy restatement of ``decode_attention`` (``src/qwenquest/attention/ops.py:48-66``) — oracle only."""

from __future__ import annotations

import numpy as np

from oracle.bf16 import round_bf16


def decode_attention(q, k, v, scaling: float, *, out_bf16: bool) -> np.ndarray:
    """One query token against an explicit list of KV rows (duplicates counted).

    ``q``: ``[H, D]``; ``k``/``v``: ``[n, KV, D]``.  Query head ``h`` reads KV
    head ``h // (H // KV)``; scores, softmax and the weighted sum are float32
    (``ops.py:60-65``); the result is cast to the query dtype (``ops.py:66``).
    Returns ``[H * D]`` float32 (bf16-exact when ``out_bf16``).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    heads, dim = q.shape
    kv = k.shape[1]
    qg = q.reshape(kv, heads // kv, dim)
    s = np.matmul(qg, k.transpose(1, 2, 0)).astype(np.float32) * np.float32(scaling)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s, dtype=np.float32)
    p = p / p.sum(axis=-1, keepdims=True, dtype=np.float32)
    out = np.matmul(p, v.transpose(1, 0, 2)).astype(np.float32).reshape(heads * dim)
    return round_bf16(out) if out_bf16 else out
