"""The oracle's prefill attention pinned to the reference's own ``extend_attention`` (CPU).

``oracle.attention.extend_attention`` restates ``attention/ops.py:18-45``; here
both run on the same seeded fp32 inputs (prefix 0, which takes the reference's
``is_causal`` branch, and a cached prefix, which takes its explicit-mask
branch) and must agree within 1e-5.  Also checks the host-side tile list of
``qq_extend_attention``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import extend_attention as oracle_extend
from qwenquest_b200.kernels import EXTEND_TILE, extend_tiles


@pytest.mark.parametrize("prefix,n,heads,kv", [(0, 37, 8, 2), (19, 23, 8, 2), (0, 130, 32, 4), (200, 5, 32, 4)])
def test_oracle_matches_reference_extend_attention(prefix, n, heads, kv):
    from qwenquest.attention.ops import extend_attention as ref_extend

    g = torch.Generator().manual_seed(prefix * 31 + n)
    d = 64
    q = torch.randn(n, heads, d, generator=g)
    k = torch.randn(prefix + n, kv, d, generator=g)
    v = torch.randn(prefix + n, kv, d, generator=g)
    ref = ref_extend(q, k, v, prefix_len=prefix, scaling=d ** -0.5).numpy()
    ora = oracle_extend(q.numpy(), k.numpy(), v.numpy(), prefix, d ** -0.5, out_bf16=False)
    assert ora.shape == ref.shape
    assert float(np.abs(ora - ref).max()) <= 1e-5


def test_tile_list_covers_every_tile_heaviest_first():
    seq, pre = [1, 300, 1300, 128], [0, 0, 1000, 0]
    tiles = extend_tiles(seq, pre)
    want = {(i, t) for i in range(4) for t in range(-(-(seq[i] - pre[i]) // EXTEND_TILE))}
    got = [(c >> 16, c & 0xFFFF) for c in tiles]
    assert sorted(got) == sorted(want) and len(got) == len(want)
    work = [-(-min(seq[i], pre[i] + (t + 1) * EXTEND_TILE) // EXTEND_TILE) for i, t in got]
    assert work == sorted(work, reverse=True)


def test_tile_list_rejects_bad_lengths():
    with pytest.raises(ValueError):
        extend_tiles([10], [11])
    with pytest.raises(ValueError):
        extend_tiles([128 * 70000], [0])
