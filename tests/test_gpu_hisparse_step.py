"""A HiSparse (Mode 3) decode step runs on the device alone (GPU).

``prepare_decode_step`` (``coordinator.py:183-215``) takes a new host row per
request from the free list, records it in ``req_to_host_pool``, folds the
previous token into the bounds and backs it up to the host tier.  Here the
free list lives on the device, so a whole step (step plan, fold, backup,
then per layer selection, swap-in and attention) must run with no host
synchronisation, checked under ``torch.cuda.set_sync_debug_mode("error")``,
and can be captured in a CUDA graph: replayed steps equal eager ones bit for
bit (outputs, ``buffer_tokens``, ``lru_slots``, ``req_to_host_pool``, hit and
miss counts).  The host rows come out of the free list in the reference's
order (front first, a finished request's rows appended in position order).
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch
from qwenquest.batch import ForwardBatch, ForwardMode
from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool

from qwenquest_b200.backends import B200QuestHiSparseBackend
from qwenquest_b200.graphs import DecodeStepGraph

pytestmark = pytest.mark.gpu

H, KV, D = 32, 4, 128
PREFIXES = (5000, 6100, 7300, 3000)
LAYERS, STEPS, BUF, MAX_CTX = 3, 5, 2560, 8192


def _setup(dev, seed=0):
    gen = torch.Generator(device=dev).manual_seed(seed)
    n_req = len(PREFIXES)
    r2t = ReqToTokenPool(n_req, MAX_CTX, dev)
    pool = MHATokenToKVPool(sum(PREFIXES), LAYERS, KV, D, torch.bfloat16, dev)
    backend = B200QuestHiSparseBackend(
        r2t, pool, {"algorithm": "quest", "top_k": 2048, "quest_page_size": 64, "device_buffer_size": BUF},
        host_pool_size=n_req * MAX_CTX)
    start = 1
    for n in PREFIXES:
        slot = r2t.alloc()
        locs = torch.arange(start, start + n, dtype=torch.int64, device=dev)
        start += n
        r2t.req_to_token[slot, :n] = locs.to(torch.int32)
        for li in range(LAYERS):
            pool.k_buffer[li][locs] = torch.randn((n, KV, D), generator=gen, device=dev).to(torch.bfloat16)
            pool.v_buffer[li][locs] = torch.randn((n, KV, D), generator=gen, device=dev).to(torch.bfloat16)
        one = torch.ones(1, dtype=torch.int64, device=dev)
        backend.on_extend_finished(ForwardBatch(
            forward_mode=ForwardMode.EXTEND, input_ids=torch.zeros(n, dtype=torch.int64, device=dev),
            positions=locs - locs[0], req_pool_indices=one * slot, seq_lens=one * n, out_cache_loc=locs,
            req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend,
            extend_prefix_lens=one * 0, extend_seq_lens=one * n))
    pre = torch.tensor(PREFIXES, dtype=torch.int64, device=dev)
    reqs = torch.arange(n_req, dtype=torch.int64, device=dev)
    batches = [ForwardBatch(
        forward_mode=ForwardMode.DECODE, input_ids=torch.zeros(n_req, dtype=torch.int64, device=dev),
        positions=pre + s, req_pool_indices=reqs, seq_lens=pre + s + 1, out_cache_loc=None,
        req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend) for s in range(STEPS)]
    q = torch.randn((STEPS, LAYERS, n_req, H, D), generator=gen, device=dev).to(torch.bfloat16)
    k = torch.randn((STEPS, LAYERS, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn((STEPS, LAYERS, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    layers = [SimpleNamespace(layer_id=i, scaling=D ** -0.5, num_heads=H, num_kv_heads=KV, head_dim=D)
              for i in range(LAYERS)]
    torch.cuda.synchronize(dev)
    return backend, batches, layers, (q, k, v)


def _eager_step(backend, batch, layers, q, k, v):
    backend.init_forward_metadata(batch)
    return [backend.forward(q[lay.layer_id], k[lay.layer_id], v[lay.layer_id], lay, batch) for lay in layers]


def _state(backend):
    c = backend.coord
    return [t.clone() for t in (c.buffer_tokens, c.lru_slots, c.req_to_host_pool, c._stats)]


def test_mode3_steps_make_no_host_sync(cuda_device):
    dev = torch.device(cuda_device)
    backend, batches, layers, (q, k, v) = _setup(dev)
    _eager_step(backend, batches[0], layers, q[0], k[0], v[0])  # the first step skips the backup
    torch.cuda.synchronize(dev)
    torch.cuda.set_sync_debug_mode("error")
    try:
        for s in range(1, STEPS):
            _eager_step(backend, batches[s], layers, q[s], k[s], v[s])
    finally:
        torch.cuda.set_sync_debug_mode("default")
    backend.synchronize()
    stats = backend.coord.stats
    assert stats.misses > 0 and stats.hits > 0
    # one host row per request and step after the first, handed out in order after the prefills
    h2p = backend.coord.req_to_host_pool.cpu()
    first = sum(PREFIXES) + 1
    got = sorted(int(h2p[i, p]) for s in range(1, STEPS) for i, p in enumerate(t + s - 1 for t in PREFIXES))
    assert got == list(range(first, first + (STEPS - 1) * len(PREFIXES)))


def test_mode3_graph_replay_equals_eager_steps(cuda_device):
    dev = torch.device(cuda_device)
    eager, batches, layers, (q, k, v) = _setup(dev, seed=3)
    ref = [[o.clone() for o in _eager_step(eager, batches[s], layers, q[s], k[s], v[s])] for s in range(STEPS)]
    torch.cuda.synchronize(dev)
    ref_state = _state(eager)

    graphed, gbatches, glayers, (gq, gk, gv) = _setup(dev, seed=3)
    first = _eager_step(graphed, gbatches[0], glayers, gq[0], gk[0], gv[0])
    for a, b in zip(ref[0], first, strict=True):
        assert torch.equal(a, b)
    g = DecodeStepGraph(graphed, glayers, gbatches[1], gq[1], gk[1], gv[1])
    for s in range(1, STEPS):
        outs = [o.clone() for o in g.replay(gbatches[s], gq[s], gk[s], gv[s])]
        for li, (a, b) in enumerate(zip(ref[s], outs, strict=True)):
            assert torch.equal(a, b), (s, li)
    torch.cuda.synchronize(dev)
    for a, b in zip(ref_state, _state(graphed), strict=True):
        assert torch.equal(a, b)
    graphed.check_errors()
    eager.check_errors()


def test_finished_requests_return_their_host_rows_in_order(cuda_device):
    dev = torch.device(cuda_device)
    backend, batches, layers, (q, k, v) = _setup(dev, seed=5)
    for s in range(3):
        _eager_step(backend, batches[s], layers, q[s], k[s], v[s])
    alloc = backend.coord.host_allocator
    free_before = alloc.available_size()
    rows1 = backend.coord.req_to_host_pool[1].cpu()
    kept = rows1[rows1 >= 0].tolist()
    backend.on_request_finished(1)
    assert alloc.available_size() == free_before + len(kept)
    assert bool((backend.coord.req_to_host_pool[1] == -1).all())
    # the freed rows come back at the end of the free list, in position order
    got = alloc.alloc(free_before + len(kept))[free_before:].cpu().tolist()
    assert got == kept
