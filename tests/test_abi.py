"""The C-ABI library loads without a GPU and exports exactly what include/qquest.h declares (CPU)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from qwenquest_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "qquest.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(qq_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        import __graft_entry__

        __graft_entry__.build()
    return _lib.load()


def test_header_declares_the_bound_functions():
    assert declared_functions() == set(_lib.SIGNATURES), (
        declared_functions() ^ set(_lib.SIGNATURES)
    )


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_introspection_calls_need_no_gpu(lib):
    assert b"sm_100a" in lib.qq_version()
    assert lib.qq_status_string(_lib.QQ_ERR_INVALID) == b"invalid argument"
    ws = lib.qq_workspace_bytes(64, 2048, 32, 128)
    # arrival counters (6 x QQ_MAX_BS int32) + two (m, l, O) records of 8 x 128 floats per
    # streaming warp (8 warps per SM; the SM count defaults to 148 without a device)
    assert ws >= 6 * 4 * _lib.QQ_MAX_BS + 148 * 8 * 2 * (8 * 128 + 16) * 4


def test_argument_errors_are_reported_without_touching_a_device(lib):
    st = _lib.QQQuestState()
    assert lib.qq_quest_init_storage(st, None) == _lib.QQ_ERR_INVALID
    assert lib.qq_quest_invalidate(None, 0, None) == _lib.QQ_ERR_INVALID
    assert lib.qq_copy_rows(None, None, 0, 0, 0, 0, None, 0, None, 0, 0, None) == _lib.QQ_ERR_INVALID
    # the ready-word attention needs words and a nonzero epoch (0 is a cleared word)
    b = _lib.QQBatch(0x10000, 0x10000, 1)
    args = (b, 2048, 0x10000, _lib.QQ_BF16, 32, 4, 128, 4096, 0x10000, 0x10000, 0x10000, 512, 100, 0.1,
            0x10000, 4096, None)
    assert lib.qq_sparse_decode_attention_ready(*args, None, 1, 0, 0x10000, 1 << 30, None) == _lib.QQ_ERR_INVALID
    assert lib.qq_sparse_decode_attention_ready(*args, 0x10000, 0, 0, 0x10000, 1 << 30, None) == _lib.QQ_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(_lib.QQ_ERR_INVALID, "probe")


def test_extend_argument_errors_are_reported_without_touching_a_device(lib):
    """qq_quest_extend_kv checks its arguments before any CUDA call (fake, never dereferenced pointers)."""
    ok, inv, uns = _lib.QQ_OK, _lib.QQ_ERR_INVALID, _lib.QQ_ERR_UNSUPPORTED
    table = _lib.QQTokenTable(0x10000, 64)

    def call(st, eb, k=0x20000, v=0x30000, dtype=_lib.QQ_BF16, row=512, src_stride=512, pool_rows=100,
             tbl=table, hot=None):
        return lib.qq_quest_extend_kv(st, 0, 0, eb, tbl, k, v, dtype, row, src_stride, 0x40000, 0x50000,
                                      row, pool_rows, hot, None, None)

    eb = _lib.QQExtendBatch(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 8, 1, 8)
    assert call(None, None) == inv                                   # no batch
    assert call(None, _lib.QQExtendBatch()) == ok                    # empty batch: nothing to do
    assert call(None, eb, dtype=7) == inv                            # unknown dtype
    assert call(None, eb, tbl=None) == inv                           # prefix rows need req_to_token
    assert call(None, eb, tbl=_lib.QQTokenTable(0x10000, 4)) == inv  # table narrower than max_seq_len
    assert call(None, eb, src_stride=256) == inv                     # rows overlap
    assert call(None, eb, pool_rows=0) == inv
    assert call(None, eb, k=0x20002, v=0x30002) == uns               # rows neither 16- nor 4-byte aligned
    st = _lib.QQQuestState(0x1, 0x2, 0x3, 0x4, 0x5, 2, 4, 8, 2, 64, 16, 64, 0)
    assert call(st, eb) == inv                                       # 2 x 64 channels, rows of 512
    hot = _lib.QQHotBuffer(0x60000, None, 512, 128, 100)
    assert call(None, eb, hot=hot) == inv                            # hot buffer without V


def test_prefill_attention_and_moe_argument_errors_without_a_device(lib):
    """qq_extend_attention and qq_moe_experts check their arguments before any CUDA call."""
    ok, inv, uns = _lib.QQ_OK, _lib.QQ_ERR_INVALID, _lib.QQ_ERR_UNSUPPORTED
    eb = _lib.QQExtendBatch(0x1000, 0x2000, 0x3000, 0x4000, 0, 8, 1, 8)
    table = _lib.QQTokenTable(0x10000, 64, 4)

    def attn(batch=eb, tbl=table, tiles=0x5000, n_tiles=1, q=0x20000, dtype=_lib.QQ_BF16, heads=32, kv=4, d=128,
             q_stride=4096, k=0x30000, v=0x40000, row=512, rows=100, out=0x50000, out_stride=4096):
        return lib.qq_extend_attention(batch, tbl, tiles, n_tiles, q, dtype, heads, kv, d, q_stride, k, v, row, rows,
                                       0.088, out, out_stride, None, None)

    assert attn(batch=None) == inv
    assert attn(tbl=_lib.QQTokenTable()) == inv                   # no req_to_token
    assert attn(q=0) == inv
    assert attn(heads=30, kv=4) == inv                             # heads not a multiple of KV heads
    assert attn(n_tiles=0) == ok                                   # nothing to do
    assert attn(tiles=0) == inv
    assert attn(dtype=_lib.QQ_F32) == uns                          # the tcgen05 kernel is bf16 only
    assert attn(d=64) == uns                                       # head_dim 128 only
    assert attn(heads=12, kv=4) == uns                             # 3 query heads per KV head: not in pairs
    assert attn(q=0x20008) == uns                                  # rows must be 16-byte aligned
    assert attn(n_tiles=70000) == uns

    plan = _lib.QQMoePlan(0x1000, 0x2000, 0x3000, 0x4000, 8, 64, 8, 128)

    def moe(p=plan, x=0x10000, hidden=2048, inter=768, wg=0x20000, out=0x30000):
        return lib.qq_moe_experts(p, x, hidden, hidden, inter, wg, 0x21000, 0x22000, 0x40000, 0x50000, out, hidden,
                                  None, None)

    assert moe(p=None) == inv
    assert moe(wg=0) == inv
    assert moe(p=_lib.QQMoePlan(0x1000, 0x2000, 0x3000, 0x4000, 0, 0, 8, 128)) == ok   # no tokens
    assert moe(hidden=2000) == uns                                  # hidden a multiple of 256
    assert moe(inter=700) == uns                                    # intermediate a multiple of 128
    assert moe(p=_lib.QQMoePlan(0x1000, 0x2000, 0x3000, 0x4000, 8, 64, 17, 128)) == uns  # top_k <= 16
    assert moe(x=0x10008) == uns
    route = lib.qq_moe_route_plan
    assert route(None, 0x1000, 8, 8, 128, 0x2000, 0x3000, 0x4000, 0x5000, None, None) == inv
    assert route(0x1000, 0x1000, 8, 0, 128, 0x2000, 0x3000, 0x4000, 0x5000, None, None) == inv
    assert route(0x1000, 0x1000, 257, 8, 128, 0x2000, 0x3000, 0x4000, 0x5000, None, None) == uns  # > 2048 pairs
    assert route(0x1000, 0x1000, 8, 8, 2000, 0x2000, 0x3000, 0x4000, 0x5000, None, None) == uns  # > 1024 experts


def test_device_error_bits_map_to_reference_exceptions():
    with pytest.raises(RuntimeError):
        _lib.raise_device_error(_lib.QQ_DEV_ERR_CAPACITY)
    with pytest.raises(AssertionError):
        _lib.raise_device_error(_lib.QQ_DEV_ERR_NO_HOST_BACKUP)
    with pytest.raises(RuntimeError):
        _lib.raise_device_error(_lib.QQ_DEV_ERR_TIMEOUT)
    _lib.raise_device_error(0)


def test_no_cpu_fallback():
    """The product refuses to run without a CUDA device instead of computing on the CPU."""
    import torch

    from qwenquest_b200.quest import QuestAlgorithm

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(ValueError):
        QuestAlgorithm(top_k=64, page_size=16, device="cpu")


def test_package_does_not_import_the_oracle():
    root = Path(__file__).resolve().parents[1] / "qwenquest_b200"
    for p in root.rglob("*.py"):
        assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", p.read_text(), flags=re.M), p
