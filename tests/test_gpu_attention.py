"""Sparse decode attention kernel against the oracle's ``decode_attention`` (GPU).

Tolerances: the kernel's bf16 output must be within 2e-2 absolute of the
oracle's fp32 attention result (the value the reference computes before its
final cast to bf16, ``attention/ops.py:60-66``); fp32 outputs within 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention
from qwenquest_b200.kernels import sparse_decode_attention

pytestmark = pytest.mark.gpu


def _case(bs, heads, kv, d, top_k, lens, dtype, seed=0, pool_rows=6000):
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(0.5 * torch.randn(1, kv, d, generator=g))
    k = (torch.randn(pool_rows, kv, d, generator=g) * scale).to(dtype)
    v = (torch.randn(pool_rows, kv, d, generator=g) * scale).to(dtype)
    q = torch.randn(bs, heads, d, generator=g).to(dtype)
    rows = torch.randint(1, pool_rows, (bs, top_k), generator=g, dtype=torch.int32)
    rows[:, 1::7] = rows[:, 0:1]  # duplicates are attended twice
    seq = torch.tensor(lens, dtype=torch.int64)
    return q, k, v, rows, seq


def _check(q, k, v, rows, seq, top_k, atol):
    scaling = q.shape[-1] ** -0.5
    out = sparse_decode_attention(q.cuda(), k.cuda(), v.cuda(), rows.cuda(), seq.cuda(), top_k, scaling)
    out = out.float().cpu().numpy()
    kn, vn, qn = k.float().numpy(), v.float().numpy(), q.float().numpy()
    worst = 0.0
    for b in range(q.shape[0]):
        n = int(min(seq[b], top_k))
        r = rows[b, :n].long().numpy()
        ref = decode_attention(qn[b], kn[r], vn[r], scaling, out_bf16=False)
        worst = max(worst, float(np.abs(out[b] - ref).max()))
    assert worst <= atol, worst
    return worst


@pytest.mark.parametrize("lens", [
    [2049, 5000, 70000, 2100],           # full 2048-row selections (16 chunks)
    [1, 31, 32, 33],                     # single partial stages
    [127, 128, 129, 255],                # chunk boundaries
    [2048, 1000, 64, 1537],              # dense-fallback lengths
])
def test_fast_path_bf16_matches_oracle(lens):
    q, k, v, rows, seq = _case(len(lens), 32, 4, 128, 2048, lens, torch.bfloat16, seed=len(lens) + sum(lens) % 97)
    _check(q, k, v, rows, seq, 2048, 2e-2)


def test_fast_path_many_requests_balances_items():
    bs = 80  # more work items than SMs in flight per wave; chunk merges across blocks
    lens = [2049 + 37 * i for i in range(bs)]
    q, k, v, rows, seq = _case(bs, 32, 4, 128, 2048, lens, torch.bfloat16, seed=5, pool_rows=40000)
    _check(q, k, v, rows, seq, 2048, 2e-2)


def test_fast_path_is_deterministic_across_calls():
    q, k, v, rows, seq = _case(8, 32, 4, 128, 2048, [3000] * 8, torch.bfloat16, seed=9)
    args = (q.cuda(), k.cuda(), v.cuda(), rows.cuda(), seq.cuda(), 2048, 128 ** -0.5)
    a = sparse_decode_attention(*args)
    b = sparse_decode_attention(*args)
    assert torch.equal(a, b)


@pytest.mark.parametrize(("heads", "kv", "d"), [(8, 2, 16), (16, 4, 32), (8, 2, 8), (32, 4, 128)])
def test_generic_path_fp32_matches_oracle(heads, kv, d):
    lens = [40, 1, 300, 257]
    q, k, v, rows, seq = _case(4, heads, kv, d, 256, lens, torch.float32, seed=heads + d)
    _check(q, k, v, rows, seq, 256, 1e-5)


@pytest.mark.parametrize(("heads", "kv", "d"), [(8, 2, 16), (16, 4, 64)])
def test_generic_path_bf16_matches_oracle(heads, kv, d):
    lens = [33, 90, 2, 64]
    q, k, v, rows, seq = _case(4, heads, kv, d, 64, lens, torch.bfloat16, seed=3)
    _check(q, k, v, rows, seq, 64, 2e-2)


def test_out_of_range_row_is_reported_not_read():
    """A row index past the pool is skipped by the kernel's bounds check and reported."""
    q, k, v, rows, seq = _case(2, 32, 4, 128, 2048, [3000, 3000], torch.bfloat16, seed=1, pool_rows=4000)
    rows[1, 5] = 4000  # one past the end
    with pytest.raises(RuntimeError):
        sparse_decode_attention(q.cuda(), k.cuda(), v.cuda(), rows.cuda(), seq.cuda(), 2048, 128 ** -0.5)
