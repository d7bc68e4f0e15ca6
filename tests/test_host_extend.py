"""Host side of the prefill K/V write (CPU): the per-batch plan behind ``qq_quest_extend_kv``.

``forward_extend`` builds, once per extend batch, the device arrays the
launch reads (request slots, lengths, cached prefixes, each request's first
row in ``k`` / ``v`` / ``out_cache_loc``) and reuses them for every layer.
The plan is pure host logic over tensors, so it is checked here on CPU
tensors without a device: offsets follow ``extend_seq_lens``, the struct
sizes the grid by the longest request, the plan is cached per batch and
dropped by ``on_extend_finished``, and inconsistent batches raise
``ValueError`` before anything is launched.
"""

from __future__ import annotations

import pytest
import torch

from qwenquest_b200.backends import B200QuestOnlyBackend
from qwenquest.batch import ForwardBatch, ForwardMode


def _bare_backend() -> B200QuestOnlyBackend:
    """A backend object with only the attributes the plan uses (no pools, no device)."""
    be = object.__new__(B200QuestOnlyBackend)
    be.device = torch.device("cpu")
    be._xplan = None
    return be


def _batch(reqs, prefix, new, seq=None, n_loc=None) -> ForwardBatch:
    i64 = lambda xs: torch.tensor(xs, dtype=torch.int64)  # noqa: E731
    seq = [p + n for p, n in zip(prefix, new, strict=True)] if seq is None else seq
    t = sum(new) if n_loc is None else n_loc
    return ForwardBatch(
        forward_mode=ForwardMode.EXTEND, input_ids=torch.zeros(t, dtype=torch.int64),
        positions=torch.zeros(t, dtype=torch.int64), req_pool_indices=i64(reqs), seq_lens=i64(seq),
        out_cache_loc=torch.arange(1, t + 1), req_to_token_pool=None, token_to_kv_pool=None, attn_backend=None,
        extend_prefix_lens=i64(prefix), extend_seq_lens=i64(new),
    )


def test_plan_offsets_lengths_and_grid_size():
    be = _bare_backend()
    batch = _batch([3, 5, 1], prefix=[0, 40, 0], new=[10, 30, 5])
    plan = be._extend_plan(batch)
    assert plan.reqs == [3, 5, 1]
    assert plan.seq_lens == [10, 70, 5]
    reqs, seq, prefix, offsets, loc = plan.tensors
    assert offsets.tolist() == [0, 10, 40]
    assert prefix.tolist() == [0, 40, 0]
    assert loc.dtype == torch.int64 and loc.numel() == 45
    assert (plan.qq.bs, plan.qq.max_seq_len, plan.qq.num_tokens) == (3, 70, 45)
    assert plan.qq.token_offsets == offsets.data_ptr() and plan.qq.out_cache_loc == loc.data_ptr()
    assert plan.reqs_dev is reqs


def test_plan_is_cached_per_batch_and_dropped_after_the_prefill():
    be = _bare_backend()
    batch = _batch([0], prefix=[0], new=[7])
    plan = be._extend_plan(batch)
    assert be._extend_plan(batch) is plan
    other = _batch([0], prefix=[0], new=[7])
    assert be._extend_plan(other) is not plan
    be.on_extend_finished(other)
    assert be._xplan is None


def test_missing_prefix_lens_mean_no_cached_prefix():
    be = _bare_backend()
    batch = _batch([2], prefix=[0], new=[9])
    batch.extend_prefix_lens = None
    plan = be._extend_plan(batch)
    assert plan.tensors[2].tolist() == [0]


@pytest.mark.parametrize("case", ["seq_mismatch", "loc_count", "negative"])
def test_inconsistent_batches_raise_before_any_launch(case):
    be = _bare_backend()
    if case == "seq_mismatch":
        batch = _batch([0, 1], prefix=[0, 4], new=[8, 8], seq=[8, 11])
    elif case == "loc_count":
        batch = _batch([0], prefix=[0], new=[8], n_loc=7)
    else:
        batch = _batch([0], prefix=[5], new=[-1], seq=[4], n_loc=0)
    with pytest.raises(ValueError):
        be._extend_plan(batch)


class _FakePool:
    def __init__(self, dtype, kv, d):
        self.dtype = dtype
        self._k = torch.zeros((4, kv, d), dtype=dtype)

    def get_key_buffer(self, layer):
        return self._k


@pytest.mark.parametrize(("dtype", "kv", "d", "fusable"), [
    (torch.bfloat16, 4, 128, True),
    (torch.float32, 1, 33, True),      # 132-byte rows: the 4-byte path
    (torch.bfloat16, 2, 34, True),     # 136-byte rows: the 4-byte path
    (torch.bfloat16, 1, 33, False),    # 66-byte rows: the reference's order
    (torch.float16, 4, 128, False),    # a pool dtype the kernel does not take
])
def test_fused_prefill_write_only_for_geometries_the_kernel_takes(dtype, kv, d, fusable):
    from types import SimpleNamespace

    be = _bare_backend()
    be.fused_extend = True
    be.token_to_kv_pool = _FakePool(dtype, kv, d)
    be.quest = SimpleNamespace(start_layer=0, kv_heads=kv, head_dim=d)
    assert be._extend_fusable() is fusable
    be.fused_extend = False
    assert be._extend_fusable() is False


def test_prefill_attention_kernel_gate():
    """Only bf16 pools of head_dim 128 with query heads in pairs of one KV group take
    qq_extend_attention; other geometries (the reference's fp32 test models) keep its loop."""
    be = _bare_backend()
    be.fused_prefill_attention = True
    plan = be._extend_plan(_batch([0, 1], [0, 64], [300, 5]))
    assert plan.num_tiles == 3 + 1
    # most key tiles first (3, 2, 1, 1); ties to the lower batch entry
    assert plan.tiles_dev().tolist() == [(0 << 16) | 2, (0 << 16) | 1, (0 << 16) | 0, (1 << 16) | 0]

    def fits(q_shape, q_dtype, kv_shape, kv_dtype):
        q = torch.zeros(q_shape, dtype=q_dtype)
        kv = torch.zeros(kv_shape, dtype=kv_dtype)
        return be._prefill_kernel_fits(q, kv, plan)

    assert fits((8, 32, 128), torch.bfloat16, (100, 4, 128), torch.bfloat16)
    assert not fits((8, 32, 128), torch.float32, (100, 4, 128), torch.float32)   # fp32
    assert not fits((8, 8, 64), torch.bfloat16, (100, 2, 64), torch.bfloat16)    # head_dim 64
    assert not fits((8, 12, 128), torch.bfloat16, (100, 4, 128), torch.bfloat16)  # 3 query heads per KV head
    be.fused_prefill_attention = False
    assert not fits((8, 32, 128), torch.bfloat16, (100, 4, 128), torch.bfloat16)
