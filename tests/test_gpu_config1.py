"""Benchmark config 1 at full size against the oracle (GPU).

The benchmark's own workload — 64 requests with 32768-token prefixes, top_k
2048 / page 64, 32 query heads over 4 KV heads x 128, bf16 — through the
fused selection + attention call (the path ``bench.py`` times), on the full
148-block grid.  The check is done in numpy from the device's own inputs:
the float64 Quest scores of every candidate page from the bounds and the
bf16 GQA mean of the queries, the top-31 pages (lower page on ties) and the
recent window as the reference lays them out (near-ties excused), the rows
as ``req_to_token`` of those positions, and the attention over those rows in
float32 (2e-2 on the bf16 output, one bf16 step above |x| = 4).

``test_config1_step_matches_oracle``: one layer, one step, a sample of four
requests.  ``test_config1_every_request_over_four_steps``: every request,
two layers, four consecutive decode steps from prefixes that end three
tokens short of a page, so that the step folds complete page 511 (its bounds
checked bit for bit against the min / max of its 64 keys) and the last step
scores 512 candidate pages instead of 511.
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


def test_config1_every_request_over_four_steps(cuda_device):
    dev = torch.device(cuda_device)
    prefix, layers_n, steps = bench.PREFIX - 3, 2, 4
    backend, pool, r2t, max_ctx, (qs, ks, vs) = bench.build_config1(dev, steps + 1, 11, prefix=prefix,
                                                                     layers=layers_n, resident=1)
    batches, layers = bench.make_batches(dev, backend, pool, r2t, max_ctx, steps + 1, prefix=prefix)
    assert backend.fused and backend.kernel_events is None and backend.quest.trace is None
    bs, top_k, page = bench.N_REQ, bench.TOP_K, bench.PAGE
    kbuf, vbuf = pool.k_buffer[0], pool.v_buffer[0]
    r2t_np = r2t.req_to_token[:bs].cpu().numpy().astype(np.int64)
    exact = excused = checked = 0
    for s in range(steps):
        b = batches[s]
        backend.init_forward_metadata(b)
        seq = b.seq_lens.cpu().numpy()
        L = int(seq[0])
        assert (seq == L).all() and L == prefix + 1 + s
        if s == steps - 1:
            # the folds of steps 1-3 completed page 511 (positions 32704-32767): its bounds are
            # the min / max of its keys, bit for bit, in every layer
            done = L // page - 1
            assert done == 511
            rows = torch.from_numpy(r2t_np[:, done * page:(done + 1) * page]).to(dev)
            keys = kbuf[rows]  # [bs, 64, kv, d]
            for li in range(layers_n):
                got = backend.quest.page_k_bounds[li, :bs, done]  # [bs, kv, d, 2]
                assert torch.equal(got[..., 0], keys.amin(dim=1)), li
                assert torch.equal(got[..., 1], keys.amax(dim=1)), li
        for layer in layers:
            li = layer.layer_id
            out = backend.forward(qs[li], ks[li], vs[li], layer, b)
            backend.synchronize()
            out_np = out.float().cpu().numpy()
            assert np.isfinite(out_np).all()
            positions = backend._positions[:bs].cpu().numpy().astype(np.int64)
            rows = backend._rows[:bs].cpu().numpy().astype(np.int64)
            F = L // page
            bounds = backend.quest.page_k_bounds[li, :bs, :F].float().cpu().numpy()  # [bs, F, kv, d, 2]
            q_np = qs[li].float().cpu().numpy()
            kr_all = kbuf[backend._rows[:bs].long()].float().cpu().numpy()  # [bs, top_k, kv, d]
            vr_all = vbuf[backend._rows[:bs].long()].float().cpu().numpy()
            for i in range(bs):
                scores = score_pages_f64(bounds[i], _bf16_mean(q_np[i], bench.KV))
                ref = _reference_positions(scores, L, top_k, page)
                m = compare_selection(positions[i], ref, seq_len=L, top_k=top_k, page_size=page,
                                      scores_f64=scores)
                assert m.exact or m.excused, (s, li, i, m.detail)
                exact += m.exact
                excused += m.excused
                assert np.array_equal(rows[i], r2t_np[i][positions[i]]), (s, li, i)
                want = decode_attention(q_np[i], kr_all[i], vr_all[i], layer.scaling, out_bf16=True)
                assert np.all(np.abs(out_np[i] - want) <= bf16_output_tolerance(want)), (s, li, i)
                checked += 1
    backend.check_errors()
    assert checked == steps * layers_n * bs
    assert exact >= checked - 4, (exact, excused, checked)
