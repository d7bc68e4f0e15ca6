"""Functional wrappers over single C-ABI entry points (torch tensors in, torch tensors out).

* :func:`sparse_decode_attention` — ``qq_sparse_decode_attention``: the
  reference's ``decode_attention`` (``attention/ops.py:48-66``) for a whole
  batch, gathering the listed rows of a KV pool itself.
* :func:`extend_attention` — ``qq_extend_attention``: the reference's dense
  causal prefill (``attention/base.py:71-93`` over ``attention/ops.py:18-45``)
  for a whole extend batch, reading the K/V rows in place through
  ``req_to_token`` (tcgen05 tensor cores).
"""

from __future__ import annotations

import torch

from qwenquest_b200 import _lib
from qwenquest_b200._lib import check
from qwenquest_b200.quest import dtype_code, stream_of

__all__ = ["extend_attention", "extend_tiles", "sparse_decode_attention", "EXTEND_TILE"]

#: new tokens per tile of qq_extend_attention
EXTEND_TILE = 128


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


def extend_tiles(seq_lens: list[int], prefix_lens: list[int]) -> list[int]:
    """The tile list of ``qq_extend_attention``: ``(entry << 16) | t`` for every tile of
    ``EXTEND_TILE`` new tokens of every request, the tiles with the most key tiles
    (the most work under the causal mask) first, so the longest CTAs start first."""
    T = EXTEND_TILE
    if len(seq_lens) >= 32768:
        raise ValueError("extend attention: at most 32767 requests per batch")
    items = []
    for i, (L, p) in enumerate(zip(seq_lens, prefix_lens, strict=True)):
        n = int(L) - int(p)
        if n < 0 or p < 0:
            raise ValueError(f"extend attention: request {i} has seq_len {L} < prefix {p}")
        for t in range((n + T - 1) // T):
            work = (min(int(L), int(p) + (t + 1) * T) + T - 1) // T
            items.append((-work, i, t))
    items.sort()
    if len(items) > 65535:
        raise ValueError(f"extend attention: {len(items)} tiles, at most 65535 per call")
    return [(i << 16) | t for _, i, t in items]


def extend_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, req_to_token: torch.Tensor,
                     req_pool_indices, seq_lens, prefix_lens, scaling: float,
                     *, check_errors: bool = True) -> torch.Tensor:
    """Causal prefill attention of an extend batch over the KV pool.

    Request ``i`` contributes ``seq_lens[i] - prefix_lens[i]`` new tokens (rows
    of ``q`` in batch order, ``q``: ``[tokens, H, D]`` bf16); new token ``t``
    (position ``prefix_lens[i] + t``) attends to the keys of positions
    ``0 .. prefix_lens[i] + t``, read from ``k_pool``/``v_pool`` (``[rows, KV, D]``)
    at rows ``req_to_token[req_pool_indices[i], pos]``.  Returns ``[tokens, H*D]``,
    what ``AttentionBackend.forward_extend`` (``base.py:71-93``) concatenates.
    """
    lib = _lib.load()
    dev = q.device
    tokens, heads, dim = q.shape
    reqs_h = [int(x) for x in torch.as_tensor(req_pool_indices).tolist()]
    seq_h = [int(x) for x in torch.as_tensor(seq_lens).tolist()]
    pre_h = [int(x) for x in torch.as_tensor(prefix_lens).tolist()]
    new_h = [s - p for s, p in zip(seq_h, pre_h, strict=True)]
    if sum(new_h) != tokens:
        raise ValueError(f"extend attention: {tokens} query rows for {sum(new_h)} new tokens")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("q, k_pool and v_pool must share a dtype")
    if k_pool.stride() != v_pool.stride() or k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must have the same layout")
    offsets_h = [0]
    for n in new_h[:-1]:
        offsets_h.append(offsets_h[-1] + n)
    i64 = dict(dtype=torch.int64, device=dev)
    reqs = torch.tensor(reqs_h, **i64)
    seq = torch.tensor(seq_h, **i64)
    pre = torch.tensor(pre_h, **i64)
    offs = torch.tensor(offsets_h, **i64)
    tiles = torch.tensor(extend_tiles(seq_h, pre_h), dtype=torch.int32, device=dev)
    r2t = req_to_token.to(device=dev, dtype=torch.int32)
    if r2t.stride(1) != 1:
        r2t = r2t.contiguous()
    q = q.contiguous()
    out = torch.empty((tokens, heads * dim), dtype=q.dtype, device=dev)
    err = torch.zeros(1, dtype=torch.int32).pin_memory()
    from qwenquest_b200.hisparse import host_device_pointer

    batch = _lib.QQExtendBatch(reqs.data_ptr(), seq.data_ptr(), pre.data_ptr(), offs.data_ptr(), 0, tokens,
                               len(seq_h), max(seq_h, default=0))
    table = _lib.QQTokenTable(r2t.data_ptr(), r2t.stride(0), r2t.shape[0])
    rc = lib.qq_extend_attention(
        batch, table, tiles.data_ptr(), tiles.numel(), q.data_ptr(), dtype_code(q.dtype), heads, k_pool.shape[1],
        dim, q.stride(0), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.stride(0), k_pool.shape[0], float(scaling),
        out.data_ptr(), out.stride(0), host_device_pointer(err), stream_of(dev),
    )
    check(rc, "extend_attention")
    if check_errors:
        torch.cuda.current_stream(dev).synchronize()
        _lib.raise_device_error(int(err[0]), "(extend attention)")
    return out
