"""Dense causal prefill attention (``qq_extend_attention``, tcgen05) against the oracle and the reference (GPU).

The oracle is ``oracle.attention.extend_attention``, a numpy restatement of
the reference's ``extend_attention`` (``attention/ops.py:18-45``) over the
rows ``forward_extend`` gathers (``attention/base.py:71-93``).  Tolerance,
against the oracle's fp32 result and against the reference's own bf16 output
(torch SDPA on the same GPU) alike: max(2e-2, one bf16 step of the value).
The early queries of a prefill see few keys, so their outputs are close to
single value rows, which reach |x| > 4 here; there one correct rounding to
bf16 alone moves the value by up to half a step (0.016-0.031), and two
independent roundings by up to a step.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import extend_attention as oracle_extend
from qwenquest_b200 import _lib
from qwenquest_b200.kernels import extend_attention, extend_tiles

pytestmark = pytest.mark.gpu

H, KV, D = 32, 4, 128
SCALING = D ** -0.5


def _bf16_step(x: np.ndarray) -> np.ndarray:
    """One bf16 ulp of |x| (8 mantissa bits)."""
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-30)))
    return np.exp2(e - 7)


def _case(reqs, pool_rows, seed, *, k_drift=0.0):
    """reqs: list of (slot, prefix, new).  The pool rows of each request are a random
    permutation (paged), row 0 stays padding.  Returns host tensors."""
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(0.5 * torch.randn(1, KV, D, generator=g))
    k = torch.randn(pool_rows, KV, D, generator=g) * scale
    if k_drift:
        # a slow drift along the rows, so later keys score higher (running maximum raised often)
        k = k + k_drift * torch.linspace(0, 1, pool_rows)[:, None, None] * torch.randn(1, KV, D, generator=g)
    k = k.to(torch.bfloat16)
    v = (torch.randn(pool_rows, KV, D, generator=g) * scale).to(torch.bfloat16)
    max_ctx = max(p + n for _, p, n in reqs) + 7
    slots = max(s for s, _, _ in reqs) + 2
    r2t = torch.zeros(slots, max_ctx, dtype=torch.int32)
    perm = torch.randperm(pool_rows - 1, generator=g) + 1
    used = 0
    for slot, p, n in reqs:
        r2t[slot, : p + n] = perm[used: used + p + n].to(torch.int32)
        used += p + n
    assert used <= pool_rows - 1
    tokens = sum(n for _, _, n in reqs)
    q = torch.randn(tokens, H, D, generator=g).to(torch.bfloat16)
    return q, k, v, r2t


def _run(reqs, q, k, v, r2t):
    dev = torch.device("cuda", 0)
    slots = [s for s, _, _ in reqs]
    seq = [p + n for _, p, n in reqs]
    pre = [p for _, p, _ in reqs]
    out = extend_attention(q.to(dev), k.to(dev), v.to(dev), r2t.to(dev), slots, seq, pre, SCALING)
    return out.float().cpu().numpy()


def _oracle(reqs, q, k, v, r2t):
    outs, off = [], 0
    kn, vn, qn = k.float().numpy(), v.float().numpy(), q.float().numpy()
    for slot, p, n in reqs:
        locs = r2t[slot, : p + n].long().numpy()
        outs.append(oracle_extend(qn[off: off + n], kn[locs], vn[locs], p, SCALING, out_bf16=False))
        off += n
    return np.concatenate(outs, axis=0)


def _reference(reqs, q, k, v, r2t):
    """The reference's own per-request loop (base.py:78-93) on the GPU, bf16 SDPA."""
    from qwenquest.attention.ops import extend_attention as ref_extend

    dev = torch.device("cuda", 0)
    kd, vd, qd, rd = k.to(dev), v.to(dev), q.to(dev), r2t.to(dev)
    outs, off = [], 0
    for slot, p, n in reqs:
        locs = rd[slot, : p + n].long()
        outs.append(ref_extend(qd[off: off + n], kd[locs], vd[locs], prefix_len=p, scaling=SCALING))
        off += n
    return torch.cat(outs, 0).float().cpu().numpy()


def _within(out: np.ndarray, ref: np.ndarray) -> None:
    tol = np.maximum(2e-2, _bf16_step(ref))
    bad = np.abs(out - ref) > tol
    assert not bad.any(), (f"{int(bad.sum())} elements off; max |diff| {float(np.abs(out - ref).max())} "
                           f"at |ref| {float(np.abs(ref).flat[int(np.argmax(np.abs(out - ref)))])}")


@pytest.mark.parametrize("reqs", [
    [(0, 0, 300)],                          # three query tiles, the last partial; prefix 0 (is_causal)
    [(3, 200, 260)],                        # chunked prefill: a cached prefix not on a tile boundary
    [(1, 0, 129), (4, 64, 1), (2, 1000, 333)],  # ragged batch: one-token extend, long prefix
    [(0, 0, 1)],                            # a single token
])
def test_matches_oracle_and_reference(reqs):
    q, k, v, r2t = _case(reqs, 4096, seed=sum(p * 7 + n for _, p, n in reqs))
    out = _run(reqs, q, k, v, r2t)
    _within(out, _oracle(reqs, q, k, v, r2t))
    _within(out, _reference(reqs, q, k, v, r2t))


def test_running_maximum_raises():
    """Keys that drift so later tiles score higher: the running maximum is raised
    (and O rescaled in tensor memory) many times along a row."""
    reqs = [(0, 0, 1024)]
    q, k, v, r2t = _case(reqs, 2048, seed=5, k_drift=6.0)
    _within(_run(reqs, q, k, v, r2t), _oracle(reqs, q, k, v, r2t))


def test_long_prefill_against_fp32_torch():
    """4096 new tokens after a 1000-token prefix, against a plain PyTorch fp32 causal
    attention of the same rows on the GPU (the oracle would take minutes)."""
    reqs = [(2, 1000, 4096)]
    q, k, v, r2t = _case(reqs, 6000, seed=11)
    out = _run(reqs, q, k, v, r2t)
    dev = torch.device("cuda", 0)
    locs = r2t[2, :5096].long().to(dev)
    kk = k.to(dev)[locs].float().repeat_interleave(H // KV, dim=1).transpose(0, 1)  # [H, L, D]
    vv = v.to(dev)[locs].float().repeat_interleave(H // KV, dim=1).transpose(0, 1)
    qq = q.to(dev).float().transpose(0, 1)  # [H, n, D]
    s = torch.matmul(qq, kk.transpose(1, 2)) * SCALING
    qpos = 1000 + torch.arange(4096, device=dev)
    s = s.masked_fill(torch.arange(5096, device=dev)[None, :] > qpos[:, None], float("-inf"))
    ref = torch.matmul(torch.softmax(s, dim=-1), vv).transpose(0, 1).reshape(4096, H * D)
    _within(out, ref.cpu().numpy())


def test_tiles_heaviest_first():
    t = extend_tiles([300, 1300], [0, 1000])
    work = []
    for code in t:
        i, tile = code >> 16, code & 0xFFFF
        L, p = [300, 1300][i], [0, 1000][i]
        work.append(-(-min(L, p + (tile + 1) * 128) // 128))
    assert work == sorted(work, reverse=True)
    assert sorted(t) == sorted([(0 << 16) | i for i in range(3)] + [(1 << 16) | i for i in range(3)])


def test_bad_row_reported():
    """A req_to_token entry outside the pool is read as row 0 and reported (QQ_DEV_ERR_BOUNDS)."""
    reqs = [(0, 0, 200)]
    q, k, v, r2t = _case(reqs, 1024, seed=3)
    r2t[0, 17] = 1 << 20  # checked on the host: far outside the 1024-row pool
    dev = torch.device("cuda", 0)
    with pytest.raises(_lib.QQError):
        extend_attention(q.to(dev), k.to(dev), v.to(dev), r2t.to(dev), [0], [200], [0], SCALING)
    # the context stays usable: a clean call right after is exact again
    r2t[0, 17] = 5
    _within(_run(reqs, q, k, v, r2t), _oracle(reqs, q, k, v, r2t))


def test_unsupported_geometry_is_a_value_error():
    dev = torch.device("cuda", 0)
    q = torch.zeros(4, 32, 128, dtype=torch.float32, device=dev)
    kv = torch.zeros(16, 4, 128, dtype=torch.float32, device=dev)
    r2t = torch.arange(16, dtype=torch.int32, device=dev)[None]
    with pytest.raises(ValueError):
        extend_attention(q, kv, kv, r2t, [0], [4], [0], SCALING)
