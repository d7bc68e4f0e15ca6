"""``qq_sparse_decode_attention_noalloc``, the attention entry point that allocates nothing (GPU).

Called through the C-ABI, it must match ``qq_sparse_decode_attention`` (the
same attention given a workspace) within the attention tests' bf16
tolerance, on two calls in a row: the second call reuses the library's fixed
scratch array right after the first.  Both are also checked against the CPU
oracle's ``decode_attention`` (the reference's ``attention/ops.py:48-66``
restated in numpy) on a sample of requests, so an error the two entry points
shared would not pass.  The file name sorts last, so the full
suite runs it after every other GPU test; it also passes alone in a fresh
process, where its first call does the per-device set-up.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention
from qwenquest_b200 import _lib
from qwenquest_b200.hisparse import host_device_pointer

pytestmark = pytest.mark.gpu

ATOL = 2e-2  # bf16 output, as in the attention tests
HEADS, KV, DIM = 32, 4, 128


def _inputs(lens, top_k, pool_rows=30000, seed=0):
    g = torch.Generator().manual_seed(seed)
    bs = len(lens)
    k = torch.randn(pool_rows, KV, DIM, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(pool_rows, KV, DIM, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(bs, HEADS, DIM, generator=g).to(torch.bfloat16).cuda()
    rows = torch.randint(0, pool_rows, (bs, top_k), generator=g, dtype=torch.int32).cuda()
    seq = torch.tensor(lens, dtype=torch.int64).cuda()
    return q, k, v, rows, seq


def _args(q, k, v, rows, seq, top_k, out, err_ptr, dtype=_lib.QQ_BF16, bs=None):
    batch = _lib.QQBatch(0, seq.data_ptr(), q.shape[0] if bs is None else bs)
    return [batch, top_k, q.data_ptr(), dtype, HEADS, KV, DIM, q.stride(0), rows.data_ptr(), k.data_ptr(),
            v.data_ptr(), k.stride(0), k.shape[0], DIM ** -0.5, out.data_ptr(), out.stride(0), err_ptr]


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("lens, top_k", [
    ([2049 + 37 * i for i in range(48)] + [5, 64, 1000, 2048] * 4, 2048),  # split segments, dense fallbacks
    ([1, 17, 300, 4096], 256),
    ([40 + (i * 7) % 300 for i in range(_lib.QQ_NOALLOC_MAX_BS)], 64),      # the largest batch accepted
])
def test_noalloc_matches_the_workspace_entry_twice_in_a_row(lens, top_k):
    lib = _lib.load()
    q, k, v, rows, seq = _inputs(lens, top_k)
    bs = len(lens)
    err = torch.zeros(1, dtype=torch.int32).pin_memory()
    err_ptr = host_device_pointer(err)

    ref = torch.empty(bs, HEADS * DIM, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(int(lib.qq_workspace_bytes(bs, top_k, HEADS, DIM)), dtype=torch.uint8, device="cuda")
    rc = lib.qq_sparse_decode_attention(*_args(q, k, v, rows, seq, top_k, ref, err_ptr), ws.data_ptr(),
                                        ws.numel(), _stream())
    assert rc == _lib.QQ_OK, lib.qq_status_string(rc)

    outs = [torch.full((bs, HEADS * DIM), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    for out in outs:  # back to back on one stream, no synchronisation between them
        rc = lib.qq_sparse_decode_attention_noalloc(*_args(q, k, v, rows, seq, top_k, out, err_ptr), _stream())
        assert rc == _lib.QQ_OK, lib.qq_status_string(rc)
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    for out in outs:
        worst = (out.float() - ref.float()).abs().max().item()
        assert worst <= ATOL, worst
    # the oracle, over the same rows, for requests spread over the batch
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    rn, lens_n = rows.cpu().numpy(), seq.cpu().numpy()
    for b in sorted({0, 1, bs // 3, bs // 2, bs - 2, bs - 1}):
        r = rn[b, :min(int(lens_n[b]), top_k)].astype(np.int64)
        want = decode_attention(qn[b], kn[r], vn[r], DIM ** -0.5, out_bf16=False)
        for out in outs:
            worst = float(np.abs(out[b].float().cpu().numpy() - want).max())
            assert worst <= ATOL, (b, worst)


def test_noalloc_rejects_what_its_fixed_scratch_cannot_hold():
    lib = _lib.load()
    top_k = 64
    q, k, v, rows, seq = _inputs([100, 200], top_k)
    out = torch.empty(2, HEADS * DIM, dtype=torch.bfloat16, device="cuda")
    too_many = _args(q, k, v, rows, seq, top_k, out, None, bs=_lib.QQ_NOALLOC_MAX_BS + 1)
    assert lib.qq_sparse_decode_attention_noalloc(*too_many, _stream()) == _lib.QQ_ERR_UNSUPPORTED
    fp32 = _args(q, k, v, rows, seq, top_k, out, None, dtype=_lib.QQ_F32)
    assert lib.qq_sparse_decode_attention_noalloc(*fp32, _stream()) == _lib.QQ_ERR_UNSUPPORTED
    ragged = _args(q, k, v, rows, seq, 60, out, None)  # top_k not a multiple of 16
    assert lib.qq_sparse_decode_attention_noalloc(*ragged, _stream()) == _lib.QQ_ERR_UNSUPPORTED
    assert lib.qq_sparse_decode_attention_noalloc(*_args(q, k, v, rows, seq, top_k, out, None), _stream()) == 0
    torch.cuda.synchronize()
