"""Functional wrappers over single C-ABI entry points (torch tensors in, torch tensors out).

* :func:`sparse_decode_attention` — ``qq_sparse_decode_attention``: the
  reference's ``decode_attention`` (``attention/ops.py:48-66``) for a whole
  batch, gathering the listed rows of a KV pool itself.
"""

from __future__ import annotations

import torch

from qwenquest_b200 import _lib
from qwenquest_b200._lib import check
from qwenquest_b200.quest import dtype_code, stream_of

__all__ = ["sparse_decode_attention"]


def sparse_decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, rows: torch.Tensor,
                            seq_lens: torch.Tensor, top_k: int, scaling: float,
                            *, check_errors: bool = True) -> torch.Tensor:
    """``out[b] = decode_attention(q[b], k_pool[rows[b, :n]], v_pool[rows[b, :n]])``, ``n = min(seq_len, top_k)``.

    ``q``: ``[bs, H, D]``; ``k_pool``/``v_pool``: ``[rows, KV, D]`` (same dtype
    as ``q``); ``rows``: ``[bs, top_k]`` int32; returns ``[bs, H*D]`` in ``q``'s dtype.
    """
    lib = _lib.load()
    dev = q.device
    bs, heads, dim = q.shape
    q = q.contiguous()
    rows = rows.to(device=dev, dtype=torch.int32).contiguous()
    seq = seq_lens.to(device=dev, dtype=torch.int64).contiguous()
    if rows.shape != (bs, top_k):
        raise ValueError(f"rows must be [bs, top_k] = {(bs, top_k)}, got {tuple(rows.shape)}")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("q, k_pool and v_pool must share a dtype")
    if k_pool.stride() != v_pool.stride() or k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must have the same layout")
    out = torch.empty((bs, heads * dim), dtype=q.dtype, device=dev)
    ws = torch.zeros(int(lib.qq_workspace_bytes(bs, top_k, heads, dim)), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32).pin_memory()
    from qwenquest_b200.hisparse import host_device_pointer

    batch = _lib.QQBatch(0, seq.data_ptr(), bs)
    rc = lib.qq_sparse_decode_attention(
        batch, top_k, q.data_ptr(), dtype_code(q.dtype), heads, k_pool.shape[1], dim, q.stride(0),
        rows.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.stride(0), k_pool.shape[0],
        float(scaling), out.data_ptr(), out.stride(0), host_device_pointer(err), ws.data_ptr(), ws.numel(),
        stream_of(dev),
    )
    check(rc, "sparse_decode_attention")
    if check_errors:
        torch.cuda.current_stream(dev).synchronize()
        _lib.raise_device_error(int(err[0]), "(attention)")
    return out
