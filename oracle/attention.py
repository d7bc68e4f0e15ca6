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


def extend_attention(q, k, v, prefix_len: int, scaling: float, *, out_bf16: bool) -> np.ndarray:
    """Causal attention of one request's new tokens (``src/qwenquest/attention/ops.py:18-45``).

    ``q``: ``[n, H, D]`` queries of positions ``prefix_len .. prefix_len + n - 1``;
    ``k``/``v``: ``[prefix_len + n, KV, D]`` keys / values of positions ``0 ..``.
    Query head ``h`` reads KV head ``h // (H // KV)`` (the reference's
    ``repeat_interleave``, ``ops.py:36-37``); query ``t`` sees keys ``0 ..
    prefix_len + t`` (the causal mask of ``ops.py:38-43``); scores, softmax and
    the weighted sum in float32.  Returns ``[n, H * D]`` float32 (bf16-exact
    when ``out_bf16``, the cast SDPA's bf16 output carries).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    n, heads, dim = q.shape
    kv_len, kv, _ = k.shape
    group = heads // kv
    qh = q.transpose(1, 0, 2).reshape(kv, group * n, dim)  # [KV, G*n, D], row g*n + t
    s = np.matmul(qh, k.transpose(1, 2, 0)).astype(np.float32) * np.float32(scaling)  # [KV, G*n, L]
    s = s.reshape(kv, group, n, kv_len)
    qpos = prefix_len + np.arange(n)
    visible = np.arange(kv_len)[None, :] <= qpos[:, None]  # [n, L]
    s = np.where(visible[None, None], s, -np.inf).astype(np.float32)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s, dtype=np.float32)
    p = p / p.sum(axis=-1, keepdims=True, dtype=np.float32)
    out = np.matmul(p.reshape(kv, group * n, kv_len), v.transpose(1, 0, 2)).astype(np.float32)  # [KV, G*n, D]
    out = out.reshape(heads, n, dim).transpose(1, 0, 2).reshape(n, heads * dim)
    return round_bf16(out) if out_bf16 else out
