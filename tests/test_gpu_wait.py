"""The bounded wait of the attention's early start (GPU).

``qq_sparse_decode_attention_ready`` reads a request's rows once its ready
word holds the call's epoch.  With words that nothing sets, every wait must
give up after the caller's limit, report ``QQ_DEV_ERR_TIMEOUT`` (raised as
``RuntimeError`` on the host, like the reference's runtime failures), and the
call must return; the GPU stays usable, and a following call whose words are
set gives exactly the output of ``qq_sparse_decode_attention`` (the same
kernel over the same rows).  The failure is made by the test on the host: a
word that nothing sets; no GPU fault is involved.
"""

from __future__ import annotations

import time

import pytest
import torch

from qwenquest_b200 import _lib
from qwenquest_b200.hisparse import host_device_pointer
from qwenquest_b200.quest import stream_of

pytestmark = pytest.mark.gpu

H, KV, D, TOP_K = 32, 4, 128, 2048
LIMIT_NS = 200_000  # 0.2 ms per wait


def _case(lens, seed=3, pool_rows=9000):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(pool_rows, KV, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(pool_rows, KV, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(len(lens), H, D, generator=g).to(torch.bfloat16).cuda()
    rows = torch.randint(1, pool_rows, (len(lens), TOP_K), generator=g, dtype=torch.int32).cuda()
    seq = torch.tensor(lens, dtype=torch.int64).cuda()
    return q, k, v, rows, seq


def _call(q, k, v, rows, seq, ready=None, epoch=0):
    """One attention call; returns (output, device error bits)."""
    lib = _lib.load()
    bs = q.shape[0]
    out = torch.empty((bs, H * D), dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(int(lib.qq_workspace_bytes(bs, TOP_K, H, D)), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32).pin_memory()
    batch = _lib.QQBatch(0, seq.data_ptr(), bs)
    common = (batch, TOP_K, q.data_ptr(), _lib.QQ_BF16, H, KV, D, q.stride(0), rows.data_ptr(), k.data_ptr(),
              v.data_ptr(), k.stride(0), k.shape[0], D ** -0.5, out.data_ptr(), out.stride(0),
              host_device_pointer(err))
    if ready is None:
        rc = lib.qq_sparse_decode_attention(*common, ws.data_ptr(), ws.numel(), stream_of(q.device))
    else:
        rc = lib.qq_sparse_decode_attention_ready(*common, ready.data_ptr(), epoch, LIMIT_NS, ws.data_ptr(),
                                                  ws.numel(), stream_of(q.device))
    _lib.check(rc, "attention")
    torch.cuda.synchronize()
    return out, int(err[0])


@pytest.mark.parametrize("lens", [[2049, 3000, 100, 2048], [40000] * 16])
def test_unpublished_ready_words_time_out_and_the_next_call_is_exact(lens):
    q, k, v, rows, seq = _case(lens)
    ref, err = _call(q, k, v, rows, seq)
    assert err == 0
    ready = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _, err = _call(q, k, v, rows, seq, ready, epoch=7)
    elapsed = time.perf_counter() - t0
    assert err & _lib.QQ_DEV_ERR_TIMEOUT, err
    assert elapsed < 1.0, f"the waits took {elapsed:.3f} s, not the caller's limit"
    with pytest.raises(RuntimeError):
        _lib.raise_device_error(err, "(attention)")
    # the GPU is still usable and the words, once set, release the same work
    ready.fill_(7)
    out, err = _call(q, k, v, rows, seq, ready, epoch=7)
    assert err == 0
    assert torch.equal(out, ref)


def test_partly_published_words_time_out_only_for_the_rest():
    lens = [2049] * 8
    q, k, v, rows, seq = _case(lens, seed=5)
    ref, _ = _call(q, k, v, rows, seq)
    ready = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
    ready[:4] = 9
    _, err = _call(q, k, v, rows, seq, ready, epoch=9)
    assert err & _lib.QQ_DEV_ERR_TIMEOUT
    ready[4:] = 9
    out, err = _call(q, k, v, rows, seq, ready, epoch=9)
    assert err == 0 and torch.equal(out, ref)
