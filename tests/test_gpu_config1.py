"""Benchmark config 1 at full size against the oracle (GPU).

The benchmark's own workload — 64 requests with 32768-token prefixes, top_k
2048 / page 64, 32 query heads over 4 KV heads x 128, bf16 — for one layer
and one decode step through the fused selection + attention call (the path
``bench.py`` times), on the full 148-block grid.  For a sample of requests
the check is done in numpy from the device's own inputs: the float64 Quest
scores of every candidate page from the bounds and the bf16 GQA mean of the
queries, the top-31 pages (lower page on ties) and the recent window as the
reference lays them out (near-ties excused), the rows as ``req_to_token`` of
those positions, and the attention over those rows in float32 (2e-2 on the
bf16 output).  Every request's output must be finite.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle.attention import decode_attention
from oracle.bf16 import round_bf16
from oracle.parity import compare_selection, score_pages_f64
from tests.parity_helpers import bf16_output_tolerance

pytestmark = pytest.mark.gpu

SAMPLE = (0, 17, 42, 63)


def _bf16_mean(q: np.ndarray, kv: int) -> np.ndarray:
    """GQA mean of ``q [H, D]`` (bf16 values): fp32 sum in head order, / G, rounded to bf16."""
    heads, dim = q.shape
    g = heads // kv
    qg = q.reshape(kv, g, dim).astype(np.float32)
    acc = np.zeros((kv, dim), dtype=np.float32)
    for j in range(g):
        acc = (acc + qg[:, j]).astype(np.float32)
    return round_bf16((acc / np.float32(g)).astype(np.float32))


def _reference_positions(scores: np.ndarray, seq_len: int, top_k: int, page: int) -> np.ndarray:
    sel = top_k // page - 1
    order = sorted(range(len(scores)), key=lambda p: (-scores[p], p))[:sel]
    pos = [p * page + t for p in order for t in range(page)]
    start = max(seq_len - page, 0)
    pos += [min(start + t, seq_len - 1) for t in range(page)]
    return np.asarray(pos, dtype=np.int64)


def test_config1_step_matches_oracle(cuda_device):
    dev = torch.device(cuda_device)
    backend, pool, r2t, max_ctx, (qs, ks, vs) = bench.build_config1(dev, 2, 5, layers=1, resident=1)
    batches, layers = bench.make_batches(dev, backend, pool, r2t, max_ctx, 2)
    assert backend.fused
    b = batches[0]
    backend.init_forward_metadata(b)
    out = backend.forward(qs[0], ks[0], vs[0], layers[0], b)
    backend.synchronize()
    out_np = out.float().cpu().numpy()
    assert np.isfinite(out_np).all()
    bs = bench.N_REQ
    positions = backend._positions[:bs].cpu().numpy().astype(np.int64)
    rows = backend._rows[:bs].cpu().numpy().astype(np.int64)
    seq = b.seq_lens.cpu().numpy()
    top_k, page = bench.TOP_K, bench.PAGE
    exact = excused = 0
    for i in SAMPLE:
        L = int(seq[i])
        F = L // page
        bounds = backend.quest.page_k_bounds[0, i, :F].float().cpu().numpy()  # [F, kv, d, 2]
        q = qs[0, i].float().cpu().numpy()
        scores = score_pages_f64(bounds, _bf16_mean(q, bench.KV))
        ref = _reference_positions(scores, L, top_k, page)
        m = compare_selection(positions[i], ref, seq_len=L, top_k=top_k, page_size=page, scores_f64=scores)
        assert m.exact or m.excused, (i, m.detail)
        exact += m.exact
        excused += m.excused
        r2t_row = r2t.req_to_token[i].cpu().numpy().astype(np.int64)
        assert np.array_equal(rows[i], r2t_row[positions[i]])
        kr = pool.k_buffer[0][torch.from_numpy(rows[i]).to(dev)].float().cpu().numpy()
        vr = pool.v_buffer[0][torch.from_numpy(rows[i]).to(dev)].float().cpu().numpy()
        want = decode_attention(q, kr, vr, layers[0].scaling, out_bf16=True)
        assert np.all(np.abs(out_np[i] - want) <= bf16_output_tolerance(want)), i
    assert exact >= len(SAMPLE) - 1, (exact, excused)
