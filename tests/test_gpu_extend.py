"""One prefill layer in one launch (``qq_quest_extend_kv``) against the reference's order (GPU).

With ``fused_extend`` (the default) a backend writes each prefill layer's new
K/V rows and builds that layer's Quest bounds in one launch (Mode 3 also
fills the hot buffer there and backs the layer up to the host tier on a side
stream).  With ``fused_extend = False`` it follows the reference:
``set_kv_buffer`` per layer, then the bounds re-read from the pool after the
last layer (``quest_only.py:101-128``) or, in Mode 3, the admission copies in
``on_extend_finished`` (``coordinator.py:138-174``).  Both must leave
bit-identical pools, bounds, running bounds, counters, skip flags, hot
buffers, host tiers and slot layouts, and give the same prefill outputs:
bit-identical where both take the reference's ``extend_attention``, within
max(2e-2, one bf16 step) where the fused backend's dense prefill attention is
the tcgen05 kernel (bf16, head_dim 128) and the other is torch SDPA; the
bounds must also equal the numpy oracle's, computed from the pool's keys.

Cases: ragged lengths (1 token, below / at / above a page, several pages),
a chunked prefill whose cached prefix ends inside a page, layers outside the
Quest range (no bounds; counters written at the last Quest layer), bf16 and
fp32 pools, and a row width (2 x 34 bf16, 136 bytes) that takes the 4-byte path.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle.quest import OracleQuest
from qwenquest_b200.backends import B200QuestHiSparseBackend, B200QuestOnlyBackend
from qwenquest.batch import ForwardBatch, ForwardMode
from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool

pytestmark = pytest.mark.gpu

LAYERS, START, END = 4, 1, 3
PAGE, TOP_K, BUF = 16, 64, 128
MAX_REQS, MAX_CTX = 8, 1024
Q_PER_KV = 2

GEOMS = [(torch.bfloat16, 4, 128), (torch.float32, 2, 64), (torch.bfloat16, 2, 34)]
GEOM_IDS = ["bf16_4x128", "f32_2x64", "bf16_2x34_4byte"]


def _backend(mode, dtype, kv, d, fused, dev):
    r2t = ReqToTokenPool(MAX_REQS, MAX_CTX, dev)
    pool = MHATokenToKVPool(MAX_REQS * MAX_CTX, LAYERS, kv, d, dtype, dev)
    cfg = {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE, "device_buffer_size": BUF}
    if mode == "quest":
        be = B200QuestOnlyBackend(r2t, pool, cfg, start_layer=START, end_layer=END)
    else:
        be = B200QuestHiSparseBackend(r2t, pool, cfg, host_pool_size=MAX_REQS * MAX_CTX, start_layer=START,
                                      end_layer=END)
    be.fused_extend = fused
    return be, r2t, pool


class _Run:
    """Drives prefill batches through a backend; the same seed gives the same inputs and rows."""

    def __init__(self, mode, dtype, kv, d, fused, dev, seed=0):
        self.be, self.r2t, self.pool = _backend(mode, dtype, kv, d, fused, dev)
        self.dev, self.dtype, self.kv, self.d = dev, dtype, kv, d
        self.gen = torch.Generator().manual_seed(seed)
        # pool rows handed out in a scattered order
        self.free = (torch.randperm(MAX_REQS * MAX_CTX, generator=self.gen) + 1).tolist()
        self.layers = [SimpleNamespace(layer_id=i, num_heads=kv * Q_PER_KV, num_kv_heads=kv, head_dim=d,
                                       scaling=d ** -0.5) for i in range(LAYERS)]

    def extend(self, reqs, prefix, new):
        """One prefill forward of requests ``reqs`` with ``prefix`` cached and ``new`` new tokens each."""
        dev, kv, d = self.dev, self.kv, self.d
        locs = []
        for r, p, n in zip(reqs, prefix, new, strict=True):
            rows = [self.free.pop() for _ in range(n)]
            self.r2t.req_to_token[r, p:p + n] = torch.tensor(rows, dtype=torch.int32, device=dev)
            locs += rows
        t = sum(new)
        k = torch.randn(LAYERS, t, kv, d, generator=self.gen).to(dev, self.dtype)
        v = torch.randn(LAYERS, t, kv, d, generator=self.gen).to(dev, self.dtype)
        q = torch.randn(LAYERS, t, kv * Q_PER_KV, d, generator=self.gen).to(dev, self.dtype)

        def i64(xs):
            return torch.tensor(xs, dtype=torch.int64, device=dev)

        batch = ForwardBatch(
            forward_mode=ForwardMode.EXTEND, input_ids=torch.zeros(t, dtype=torch.int64, device=dev),
            positions=torch.cat([torch.arange(p, p + n) for p, n in zip(prefix, new, strict=True)]).to(dev),
            req_pool_indices=i64(reqs), seq_lens=i64([p + n for p, n in zip(prefix, new, strict=True)]),
            out_cache_loc=i64(locs), req_to_token_pool=self.r2t, token_to_kv_pool=self.pool,
            attn_backend=self.be, extend_prefix_lens=i64(prefix), extend_seq_lens=i64(new),
        )
        self.be.init_forward_metadata(batch)
        outs = [self.be.forward(q[li], k[li], v[li], layer, batch) for li, layer in enumerate(self.layers)]
        self.be.on_extend_finished(batch)
        return outs


def _assert_same_outputs(outs_a, outs_b, dtype, d) -> None:
    """Prefill outputs of the fused and the reference-order backend (layer by layer)."""
    kernel = dtype == torch.bfloat16 and d == 128  # qq_extend_attention on the fused side
    for oa, ob in zip(outs_a, outs_b, strict=True):
        if not kernel:
            assert torch.equal(oa, ob)
            continue
        a, b = oa.float(), ob.float()
        step = torch.exp2(torch.floor(torch.log2(b.abs().clamp_min(1e-30))) - 7)
        assert bool(((a - b).abs() <= torch.clamp(step, min=2e-2)).all()), float((a - b).abs().max())


def _assert_same_state(a: _Run, b: _Run) -> None:
    for li in range(LAYERS):
        assert torch.equal(a.pool.k_buffer[li], b.pool.k_buffer[li]), li
        assert torch.equal(a.pool.v_buffer[li], b.pool.v_buffer[li]), li
    qa, qb = a.be.quest, b.be.quest
    for name in ("page_k_bounds", "running_k_min", "running_k_max", "running_token_count", "running_page_idx"):
        assert torch.equal(getattr(qa, name), getattr(qb, name)), name


def _assert_oracle_bounds(run: _Run, reqs, seq_lens) -> None:
    """The bounds of every Quest layer equal the numpy restatement's, from the pool's keys."""
    q = run.be.quest
    orc = OracleQuest(TOP_K, PAGE)
    orc.init_storage(START, END, MAX_REQS, MAX_CTX, run.kv, run.d)
    for layer in range(START, END):
        kbuf = run.pool.k_buffer[layer].float().cpu().numpy()
        for r, n in zip(reqs, seq_lens, strict=True):
            idx = run.r2t.req_to_token[r, :n].cpu().numpy()
            orc.update_prefill_representations(layer, r, kbuf, idx)
    for r, n in zip(reqs, seq_lens, strict=True):
        full = n // PAGE
        got = q.page_k_bounds[:, r, :full].float().cpu().numpy()
        assert np.array_equal(got, orc.page_k_bounds[:, r, :full]), r
        if n % PAGE:
            assert np.array_equal(q.running_k_min[:, r].float().cpu().numpy(), orc.running_k_min[:, r]), r
            assert np.array_equal(q.running_k_max[:, r].float().cpu().numpy(), orc.running_k_max[:, r]), r
        assert int(q.running_token_count[r]) == n % PAGE
        assert int(q.running_page_idx[r]) == full


@pytest.mark.parametrize(("dtype", "kv", "d"), GEOMS, ids=GEOM_IDS)
def test_quest_extend_fused_equals_reference_order(dtype, kv, d, cuda_device):
    runs = [_Run("quest", dtype, kv, d, fused, cuda_device) for fused in (True, False)]
    # first prefill: ragged, no prefix
    reqs1, new1 = [0, 1, 2, 3, 4, 5], [1, 15, 16, 17, 100, 333]
    outs = [r.extend(reqs1, [0] * 6, new1) for r in runs]
    _assert_same_outputs(*outs, dtype, d)
    _assert_same_state(*runs)
    _assert_oracle_bounds(runs[0], reqs1, new1)
    # second prefill: two requests continue after a prefix ending inside a page, one new request
    reqs2, prefix2, new2 = [3, 4, 6], [17, 100, 0], [40, 7, 64]
    outs = [r.extend(reqs2, prefix2, new2) for r in runs]
    _assert_same_outputs(*outs, dtype, d)
    torch.cuda.synchronize(cuda_device)
    for r in runs:
        r.be.check_errors()
    _assert_same_state(*runs)
    assert torch.equal(runs[0].be._skip_first_decode_update, runs[1].be._skip_first_decode_update)
    assert int(runs[0].be._skip_first_decode_update[:7].sum()) == 7
    lens = dict(zip(reqs1, new1, strict=True))
    lens.update({r: p + n for r, p, n in zip(reqs2, prefix2, new2, strict=True)})
    _assert_oracle_bounds(runs[0], list(lens), list(lens.values()))


@pytest.mark.parametrize(("dtype", "kv", "d"), GEOMS[:2], ids=GEOM_IDS[:2])
def test_hisparse_admission_fused_equals_reference_order(dtype, kv, d, cuda_device):
    runs = [_Run("quest_hisparse", dtype, kv, d, fused, cuda_device) for fused in (True, False)]
    # lengths below, at and above the hot buffer (128 slots)
    reqs, new = [0, 1, 2, 3], [5, 128, 129, 300]
    outs = [r.extend(reqs, [0] * 4, new) for r in runs]
    _assert_same_outputs(*outs, dtype, d)
    torch.cuda.synchronize(cuda_device)
    for r in runs:
        r.be.check_errors()
    _assert_same_state(*runs)
    _assert_oracle_bounds(runs[0], reqs, new)
    ca, cb = runs[0].be.coord, runs[1].be.coord
    assert torch.equal(ca.req_to_host_pool, cb.req_to_host_pool)
    for li in range(LAYERS):
        for name in ("device_k", "device_v", "host_k", "host_v"):
            assert torch.equal(getattr(ca, name)[li], getattr(cb, name)[li]), (name, li)
    assert torch.equal(ca.buffer_tokens, cb.buffer_tokens)
    assert torch.equal(ca.lru_slots, cb.lru_slots)
    assert torch.equal(ca._skip_first_backup, cb._skip_first_backup)
    # the host tier holds every prefill position's K/V, the hot buffer positions [0, BUF)
    pool = runs[0].pool
    for r, n in zip(reqs, new, strict=True):
        rows = runs[0].r2t.req_to_token[r, :n].long()
        host = ca.req_to_host_pool[r, :n].long().cpu()
        hot = min(n, BUF)
        for li in range(LAYERS):
            assert torch.equal(ca.host_k[li][host], pool.k_buffer[li][rows].cpu())
            assert torch.equal(ca.host_v[li][host], pool.v_buffer[li][rows].cpu())
            assert torch.equal(ca.device_k[li][r * (BUF + 1): r * (BUF + 1) + hot], pool.k_buffer[li][rows[:hot]])
            assert torch.equal(ca.device_v[li][r * (BUF + 1): r * (BUF + 1) + hot], pool.v_buffer[li][rows[:hot]])


def test_quest_extend_large_batch(cuda_device):
    """Enough pages that a launch covers half rows (32 words) per block instead of quarter rows."""
    runs = [_Run("quest", torch.bfloat16, 4, 128, fused, cuda_device, seed=3) for fused in (True, False)]
    reqs, new = list(range(MAX_REQS)), [1000, 999, 1001 - 64, 640, 1017, 1008, 961, 1023]
    outs = [r.extend(reqs, [0] * MAX_REQS, new) for r in runs]
    _assert_same_outputs(*outs, torch.bfloat16, 128)
    torch.cuda.synchronize(cuda_device)
    for r in runs:
        r.be.check_errors()
    _assert_same_state(*runs)
    _assert_oracle_bounds(runs[0], reqs, new)
