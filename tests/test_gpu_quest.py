"""B200 ``QuestAlgorithm`` against the reference's QuestAlgorithm contract (GPU).

The cases restate the known answers and invariants that the reference pins
for its ``QuestAlgorithm`` (``tests/test_quest_algorithm.py``: geometry
top_k 256 / page 64 / 4 KV heads / head_dim 32 / 2 layers / 8 requests /
context 2048), run on the CUDA implementation, plus checks of the fused
all-layer entry points against the per-layer ones and of scores / selections
against the CPU oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.parity import compare_selection, score_pages_f64
from oracle.quest import OracleQuest
from qwenquest_b200.quest import QuestAlgorithm, QuestTrace

pytestmark = pytest.mark.gpu

TOP_K, PAGE, KV, D, LAYERS, MAX_REQS, MAX_CTX = 256, 64, 4, 32, 2, 8, 2048
BMAX = torch.finfo(torch.bfloat16).max
BMIN = torch.finfo(torch.bfloat16).min


def make_quest(top_k=TOP_K, page=PAGE, kv=KV, d=D, **kw) -> QuestAlgorithm:
    q = QuestAlgorithm(top_k=top_k, page_size=page, device="cuda", **kw)
    q.init_storage(0, LAYERS, MAX_REQS, MAX_CTX, kv, d)
    return q


def keys(n, seed=0, dtype=torch.bfloat16, kv=KV, d=D) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, kv, d, generator=g).to(dtype).cuda()


def prefill(q: QuestAlgorithm, req: int, pool: torch.Tensor, n: int) -> None:
    idx = torch.arange(n, dtype=torch.int32, device="cuda")
    for layer in range(LAYERS):
        q.update_prefill_representations(layer, req, pool, idx)


def decode(q: QuestAlgorithm, req: int, pool: torch.Tensor, locs) -> None:
    reqs = torch.tensor([req], device="cuda")
    for loc in locs:
        for layer in range(LAYERS):
            q.update_decode_representations(layer, reqs, pool, torch.tensor([loc], device="cuda"))
        q.maybe_finalize_decode_representations(reqs)


def retrieve(q: QuestAlgorithm, queries, reqs, seq_lens, layer=0):
    reqs = torch.as_tensor(reqs, dtype=torch.int64, device="cuda")
    seq = torch.as_tensor(seq_lens, dtype=torch.int64, device="cuda")
    q.prepare_step(seq)
    return q.retrieve_topk(queries.cuda(), layer, reqs, seq)


# --------------------------------------------------------------- configuration


def test_rejects_bad_top_k_page_combinations():
    with pytest.raises(ValueError):
        QuestAlgorithm(top_k=100, page_size=64, device="cuda")
    with pytest.raises(ValueError):
        QuestAlgorithm(top_k=64, page_size=0, device="cuda")


def test_storage_shapes_and_sentinels():
    q = make_quest()
    assert q.page_k_min.shape == (LAYERS, MAX_REQS, MAX_CTX // PAGE, KV, D)
    assert q.page_k_bounds.dtype == torch.bfloat16
    assert q.page_valid.shape == (LAYERS, MAX_REQS, MAX_CTX // PAGE) and not q.page_valid.any()
    assert bool((q.page_k_min == BMAX).all()) and bool((q.page_k_max == BMIN).all())
    assert bool((q.running_k_min == BMAX).all()) and bool((q.running_k_max == BMIN).all())
    assert int(q.running_token_count.abs().sum()) == 0 and int(q.running_page_idx.abs().sum()) == 0


# --------------------------------------------------------------- [Q2] prefill


def test_prefill_writes_full_pages_only():
    q, pool = make_quest(), keys(512)
    prefill(q, 2, pool, 192)
    assert q.page_valid[:, 2, :3].all() and not q.page_valid[:, 2, 3:].any()
    for layer in range(LAYERS):
        for p in range(3):
            slab = pool[p * PAGE : (p + 1) * PAGE]
            assert torch.equal(q.page_k_min[layer, 2, p], slab.amin(0))
            assert torch.equal(q.page_k_max[layer, 2, p], slab.amax(0))
    assert int(q.running_token_count[2]) == 0 and int(q.running_page_idx[2]) == 3


def test_prefill_partial_tail_seeds_running_bounds():
    q, pool = make_quest(), keys(512)
    prefill(q, 1, pool, 200)
    assert q.page_valid[:, 1, :3].all() and not q.page_valid[:, 1, 3:].any()
    for layer in range(LAYERS):
        assert torch.equal(q.running_k_min[layer, 1], pool[192:200].amin(0))
        assert torch.equal(q.running_k_max[layer, 1], pool[192:200].amax(0))
    assert int(q.running_token_count[1]) == 8 and int(q.running_page_idx[1]) == 3


def test_prefill_shorter_than_a_page():
    q, pool = make_quest(), keys(128)
    prefill(q, 0, pool, 30)
    assert not q.page_valid[:, 0].any()
    assert int(q.running_token_count[0]) == 30 and int(q.running_page_idx[0]) == 0


def test_prefill_float32_keys_round_to_bf16():
    q, pool = make_quest(), keys(256, seed=4, dtype=torch.float32)
    prefill(q, 3, pool, 130)
    for layer in range(LAYERS):
        assert torch.equal(q.page_k_min[layer, 3, 1], pool[64:128].amin(0).to(torch.bfloat16))
        assert torch.equal(q.running_k_max[layer, 3], pool[128:130].amax(0).to(torch.bfloat16))


def test_all_layer_prefill_equals_per_layer_calls():
    a, b = make_quest(), make_quest()
    pools = [keys(700, seed=s) for s in (1, 2)]
    idx = torch.randperm(700, generator=torch.Generator().manual_seed(0))[:650].to(torch.int32).cuda()
    for layer in range(LAYERS):
        a.update_prefill_representations(layer, 5, pools[layer], idx)
    b.update_prefill_representations_all_layers(5, pools, idx)
    assert torch.equal(a.page_k_bounds, b.page_k_bounds)
    assert torch.equal(a.running_k_min, b.running_k_min) and torch.equal(a.running_k_max, b.running_k_max)
    assert torch.equal(a.running_token_count, b.running_token_count)
    assert torch.equal(a.running_page_idx, b.running_page_idx)


# --------------------------------------------------------------- [Q3] decode


def test_decode_finalizes_a_completed_page():
    q, pool = make_quest(), keys(512, seed=11)
    prefill(q, 3, pool, 64)
    decode(q, 3, pool, range(64, 128))
    assert q.page_valid[:, 3, :2].all()
    for layer in range(LAYERS):
        assert torch.equal(q.page_k_min[layer, 3, 1], pool[64:128].amin(0))
        assert torch.equal(q.page_k_max[layer, 3, 1], pool[64:128].amax(0))
    assert int(q.running_token_count[3]) == 0 and int(q.running_page_idx[3]) == 2
    assert bool((q.running_k_min[:, 3] == BMAX).all()) and bool((q.running_k_max[:, 3] == BMIN).all())


def test_decode_continues_a_partial_prefill_page():
    q, pool = make_quest(), keys(256, seed=22)
    prefill(q, 4, pool, 50)
    decode(q, 4, pool, range(50, 64))
    assert q.page_valid[:, 4, 0].all()
    assert torch.equal(q.page_k_min[0, 4, 0], pool[:64].amin(0))
    assert int(q.running_page_idx[4]) == 1 and int(q.running_token_count[4]) == 0


def test_page_becomes_valid_only_with_its_last_token():
    q, pool = make_quest(), keys(256)
    prefill(q, 0, pool, 64)
    decode(q, 0, pool, range(64, 127))
    assert not q.page_valid[:, 0, 1].any()
    decode(q, 0, pool, [127])
    assert q.page_valid[:, 0, 1].all()


def test_fused_fold_and_finalize_equals_separate_calls():
    a, b = make_quest(), make_quest()
    pool = keys(1024, seed=3)
    for q in (a, b):
        for r, n in ((0, 63), (1, 100), (2, 64)):
            prefill(q, r, pool, n)
    reqs = torch.tensor([0, 1, 2], device="cuda")
    for step in range(70):
        locs = torch.tensor([63 + step, 100 + step, 64 + step], device="cuda")
        for layer in range(LAYERS):
            a.update_decode_representations(layer, reqs, pool, locs)
        a.maybe_finalize_decode_representations(reqs)
        b.decode_step(3, reqs, None, [pool] * LAYERS, rows=locs)
    assert torch.equal(a.page_k_bounds, b.page_k_bounds)
    assert torch.equal(a.running_k_min, b.running_k_min) and torch.equal(a.running_k_max, b.running_k_max)
    assert torch.equal(a.running_token_count, b.running_token_count)
    assert torch.equal(a.running_page_idx, b.running_page_idx)


# --------------------------------------------------------------- [Q8] invalidate


def test_invalidate_resets_one_slot_only():
    q, pool = make_quest(), keys(512)
    for r in (1, 2, 3, 5):
        prefill(q, r, pool, 150 if r == 5 else 128)
    q.invalidate_request(5)
    assert not q.page_valid[:, 5].any()
    assert int(q.running_token_count[5]) == 0 and int(q.running_page_idx[5]) == 0
    assert bool((q.running_k_min[:, 5] == BMAX).all()) and bool((q.running_k_max[:, 5] == BMIN).all())
    q.invalidate_request(2)
    assert q.page_valid[:, 1, :2].all() and q.page_valid[:, 3, :2].all() and not q.page_valid[:, 2].any()


# --------------------------------------------------------------- [Q4][Q6] selection


def test_retrieve_topk_return_contract():
    q, pool = make_quest(), keys(2048, seed=99)
    prefill(q, 0, pool, 800)
    pos, actual = retrieve(q, torch.randn(1, KV, D, dtype=torch.bfloat16), [0], [800])
    assert pos.shape == (1, TOP_K) and pos.dtype == torch.int32 and pos.is_cuda
    assert actual.shape == (1,) and actual.dtype == torch.int32 and int(actual[0]) == TOP_K
    assert int(pos.min()) >= 0 and int(pos.max()) < 800


def test_long_request_ends_with_the_recent_window():
    q, pool = make_quest(), keys(2048, seed=99)
    prefill(q, 0, pool, 800)
    pos, _ = retrieve(q, torch.randn(1, KV, D), [0], [800])
    assert pos[0, -PAGE:].tolist() == list(range(800 - PAGE, 800))


def test_short_request_is_dense_and_padded():
    q, pool = make_quest(), keys(256, seed=77)
    prefill(q, 0, pool, 128)
    pos, actual = retrieve(q, torch.randn(1, KV, D), [0], [128])
    assert int(actual[0]) == 128 and pos[0, :128].tolist() == list(range(128))
    assert int(pos[0, 128:].max()) == 127 and int(pos[0, 128:].min()) == 127


def test_high_scoring_page_is_selected():
    q = make_quest()
    pool = torch.zeros(2048, KV, D, dtype=torch.bfloat16, device="cuda")
    pool[320:384] = 5.0
    prefill(q, 0, pool, 640)
    pos, _ = retrieve(q, torch.ones(1, KV, D), [0], [640])
    assert set(range(320, 384)) <= set(pos[0].tolist())


def test_score_upper_bounds_every_token_of_its_page():
    q = make_quest(top_k=128, page=16)
    pool = keys(512, seed=5)
    prefill(q, 0, pool, 512)
    for seed in range(5):
        query = torch.randn(1, KV, D, generator=torch.Generator().manual_seed(seed)).cuda()
        scores = q.page_scores(query, 0, torch.tensor([0]))[0, :32]
        per_token = torch.einsum("hd,thd->t", query[0], pool.float())
        assert bool((scores >= per_token.view(32, 16).amax(1) - 1e-3).all())


def test_scores_match_a_naive_loop():
    q = make_quest(top_k=128, page=16)
    pool = keys(256, seed=6)
    prefill(q, 0, pool, 256)
    query = torch.randn(1, KV, D, generator=torch.Generator().manual_seed(1))
    fast = q.page_scores(query.cuda(), 1, torch.tensor([0]))[0, :16].cpu()
    kmin, kmax = q.page_k_min[1, 0].float().cpu(), q.page_k_max[1, 0].float().cpu()
    for p in range(16):
        naive = sum(max(float(query[0, h, d] * kmin[p, h, d]), float(query[0, h, d] * kmax[p, h, d]))
                    for h in range(KV) for d in range(D))
        assert abs(float(fast[p]) - naive) < 1e-3


def test_gqa_mean_per_kv_group():
    q = make_quest()
    queries = torch.randn(3, 4 * KV, D).cuda()
    grouped = q.group_queries(queries.view(3, -1))
    for h in range(KV):
        assert torch.allclose(grouped[:, h], queries[:, 4 * h : 4 * h + 4].mean(1), atol=1e-6)
    with pytest.raises(ValueError):
        q.group_queries(torch.randn(3, 6, D).cuda())


def test_gqa_mean_bf16_is_bf16_of_fp32_mean():
    q = make_quest()
    queries = torch.randn(16, 8 * KV, D).to(torch.bfloat16).cuda()
    grouped = q.group_queries(queries)
    expect = queries.float().view(16, KV, 8, D).sum(2).div(8).to(torch.bfloat16)
    assert torch.equal(grouped, expect)
    assert torch.equal(grouped, queries.view(16, KV, 8, D).mean(2))


def test_incomplete_and_stale_pages_never_win():
    q = make_quest(top_k=128, page=16)
    pool = keys(1024, seed=3)
    big = 100 * torch.randn(1, KV, D, generator=torch.Generator().manual_seed(0))
    prefill(q, 0, pool, 176)
    decode(q, 0, pool, range(176, 191))
    pos, _ = retrieve(q, big, [0], [192])
    assert int(pos[0, : 128 - 16].max()) < 176
    prefill(q, 1, pool, 1000)
    pos, _ = retrieve(q, big, [1], [300])
    assert int(pos[0, : 128 - 16].max()) < (300 // 16) * 16


def test_recent_window_overlap_default_vs_avoid():
    pool = torch.zeros(2048, KV, D, dtype=torch.bfloat16, device="cuda")
    pool[48:64] = 3.0
    queries = torch.ones(1, KV, D)
    up = make_quest(top_k=32, page=16)
    prefill(up, 0, pool, 70)
    pos, _ = retrieve(up, queries, [0], [70])
    lst = pos[0].tolist()
    assert len(lst) != len(set(lst)) and set(range(54, 64)) <= set(lst[:16])
    fixed = make_quest(top_k=32, page=16, avoid_recent_overlap=True)
    prefill(fixed, 0, pool, 70)
    pos, actual = retrieve(fixed, queries, [0], [70])
    assert len(set(pos[0].tolist())) == int(actual[0]) == 32
    assert pos[0, -16:].tolist() == list(range(54, 70))


def test_mixed_short_and_long_batch():
    q, pool = make_quest(top_k=64, page=16), keys(1024, seed=8)
    prefill(q, 0, pool, 40)
    prefill(q, 1, pool, 300)
    pos, actual = retrieve(q, torch.randn(2, KV, D), [0, 1], [40, 300])
    assert actual.tolist() == [40, 64]
    assert pos[0, :40].tolist() == list(range(40))
    assert pos[1, -16:].tolist() == list(range(284, 300))
    assert int(pos[1, :48].max()) < 288


def test_retrieve_without_prepare_step_raises():
    q = make_quest()
    with pytest.raises(RuntimeError):
        q.retrieve_topk(torch.randn(1, KV, D).cuda(), 0, torch.tensor([0]), torch.tensor([5]))


def test_retrieve_rejects_batch_size_mismatch():
    q = make_quest()
    q.prepare_step(torch.tensor([300, 300], device="cuda"))
    with pytest.raises(ValueError):
        q.retrieve_topk(torch.randn(1, KV, D).cuda(), 0, torch.tensor([0]), torch.tensor([300]))


def test_trace_records_each_decision():
    q, pool = make_quest(top_k=64, page=16), keys(1024, seed=9)
    q.trace = QuestTrace()
    prefill(q, 0, pool, 500)
    pos, _ = retrieve(q, torch.randn(1, KV, D), [0], [500], layer=1)
    (rec,) = q.trace.records
    assert rec.layer_id == 1 and not rec.dense and len(rec.selected_pages) == 3
    assert rec.page_scores is not None and rec.page_scores.shape == (500 // 16,)
    assert rec.recent_window == (484, 500)
    assert torch.equal(rec.positions, pos[0].cpu().long())


# --------------------------------------------------------------- against the oracle


def _oracle_from(q: QuestAlgorithm, top_k, page, avoid=False) -> OracleQuest:
    o = OracleQuest(top_k, page, avoid_recent_overlap=avoid)
    o.init_storage(0, q.num_layers, q.max_reqs, q.max_pages_per_req * page, q.kv_heads, q.head_dim)
    o.page_k_bounds = q.page_k_bounds.float().cpu().numpy()
    return o


@pytest.mark.parametrize("avoid", [False, True])
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float32])
def test_selection_matches_oracle_on_random_batches(avoid, qdtype):
    top_k, page, kv, d, heads = 256, 16, 4, 32, 16
    q = QuestAlgorithm(top_k=top_k, page_size=page, device="cuda", avoid_recent_overlap=avoid)
    q.init_storage(0, LAYERS, MAX_REQS, MAX_CTX, kv, d)
    rng = np.random.default_rng(7)
    lens = [int(x) for x in rng.integers(1, MAX_CTX - 1, size=MAX_REQS)] + [257, 272, 256]
    lens = lens[:MAX_REQS]
    for r, n in enumerate(lens):
        pool = keys(MAX_CTX, seed=100 + r, kv=kv, d=d)
        prefill(q, r, pool, n)
    reqs = list(range(MAX_REQS))
    seq = [n + 1 for n in lens]
    queries = torch.randn(MAX_REQS, heads, d, generator=torch.Generator().manual_seed(3)).to(qdtype)
    pos, actual = retrieve(q, queries, reqs, seq, layer=1)
    o = _oracle_from(q, top_k, page, avoid)
    o.prepare_step(np.array(seq))
    qn = queries.float().numpy()
    opos, oact = o.retrieve_topk(qn, 1, np.array(reqs), query_is_bf16=qdtype == torch.bfloat16)
    assert actual.cpu().tolist() == oact.tolist()
    qbar = o.group_queries(qn, query_is_bf16=qdtype == torch.bfloat16)
    for i in range(MAX_REQS):
        c = int(o._step.candidate_limit[i])
        s64 = score_pages_f64(o.page_k_bounds[1, i, :c], qbar[i])
        m = compare_selection(pos[i].cpu().numpy(), opos[i], seq_len=seq[i], top_k=top_k, page_size=page,
                              scores_f64=s64)
        assert m.exact or m.excused, (i, m.detail)
