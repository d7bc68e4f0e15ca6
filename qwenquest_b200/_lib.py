"""ctypes binding of ``libqquest.so`` (the C ABI declared in ``include/qquest.h``).

The library is built in-tree by ``__graft_entry__.build()`` (``nvcc`` for
``sm_100a``) into ``qwenquest_b200/_lib/libqquest.so``.  There is no fallback:
importing a backend without the library, or without a CUDA device, raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "libqquest.so"

QQ_OK = 0
QQ_ERR_INVALID = -1
QQ_ERR_UNSUPPORTED = -2
QQ_ERR_CUDA = -3
QQ_ERR_WORKSPACE = -4

QQ_DEV_ERR_CAPACITY = 1
QQ_DEV_ERR_NO_HOST_BACKUP = 2
QQ_DEV_ERR_BOUNDS = 4
QQ_DEV_ERR_TIMEOUT = 8

QQ_BF16 = 0
QQ_F32 = 1

QQ_STEP_FOLD = 1
QQ_STEP_FINALIZE = 2

QQ_MAX_LAYERS = 128
QQ_MAX_BS = 4096
QQ_NOALLOC_MAX_BS = 1024


class QQQuestState(ctypes.Structure):
    _fields_ = [
        ("page_bounds", c_void_p),
        ("running_min", c_void_p),
        ("running_max", c_void_p),
        ("running_token_count", c_void_p),
        ("running_page_idx", c_void_p),
        ("num_layers", c_int32),
        ("max_reqs", c_int32),
        ("max_pages", c_int32),
        ("kv_heads", c_int32),
        ("head_dim", c_int32),
        ("page_size", c_int32),
        ("top_k", c_int32),
        ("avoid_recent_overlap", c_int32),
    ]


class QQBatch(ctypes.Structure):
    _fields_ = [("req_pool_indices", c_void_p), ("seq_lens", c_void_p), ("bs", c_int32)]


class QQTokenTable(ctypes.Structure):
    _fields_ = [("req_to_token", c_void_p), ("stride", c_int64), ("rows", c_int64)]


class QQNewToken(ctypes.Structure):
    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("src_stride", c_int64),
        ("k_dst", c_void_p),
        ("v_dst", c_void_p),
        ("dst_row_stride", c_int64),
        ("dst_rows", c_void_p),
        ("device_buffer_size", c_int64),
        ("dst_num_rows", c_int64),
        ("dtype", c_int32),
    ]


class QQExtendBatch(ctypes.Structure):
    _fields_ = [
        ("req_pool_indices", c_void_p),
        ("seq_lens", c_void_p),
        ("prefix_lens", c_void_p),
        ("token_offsets", c_void_p),
        ("out_cache_loc", c_void_p),
        ("num_tokens", c_int64),
        ("bs", c_int32),
        ("max_seq_len", c_int32),
    ]


class QQHotBuffer(ctypes.Structure):
    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("row_stride", c_int64),
        ("device_buffer_size", c_int64),
        ("num_rows", c_int64),
    ]


class QQMoePlan(ctypes.Structure):
    _fields_ = [
        ("pair_token", c_void_p),
        ("expert_offsets", c_void_p),
        ("pair_weight", c_void_p),
        ("token_pairs", c_void_p),
        ("num_tokens", c_int64),
        ("num_pairs", c_int64),
        ("top_k", c_int32),
        ("num_experts", c_int32),
    ]


class QQHostRing(ctypes.Structure):
    _fields_ = [("rows", c_void_p), ("state", c_void_p), ("capacity", c_int64)]


class QQHiSparseState(ctypes.Structure):
    _fields_ = [
        ("buffer_tokens", c_void_p),
        ("lru_slots", c_void_p),
        ("req_to_host_pool", c_void_p),
        ("stats", c_void_p),
        ("num_layers", c_int32),
        ("max_reqs", c_int32),
        ("max_context_len", c_int32),
        ("device_buffer_size", c_int32),
        ("top_k", c_int32),
    ]


_S = POINTER(QQQuestState)
_B = POINTER(QQBatch)
_T = POINTER(QQTokenTable)
_N = POINTER(QQNewToken)
_H = POINTER(QQHiSparseState)
_E = POINTER(QQExtendBatch)
_HB = POINTER(QQHotBuffer)
_PP = POINTER(c_void_p)

#: every exported symbol with its (restype, argtypes); tests check the list
#: against include/qquest.h
SIGNATURES: dict[str, tuple] = {
    "qq_host_device_pointer": (c_int, [c_void_p, POINTER(c_void_p)]),
    "qq_version": (c_char_p, []),
    "qq_status_string": (c_char_p, [c_int]),
    "qq_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "qq_quest_init_storage": (c_int, [_S, c_void_p]),
    "qq_quest_invalidate": (c_int, [_S, c_int, c_void_p]),
    "qq_quest_bounds_prefill": (
        c_int, [_S, c_int, c_int, _PP, c_int, c_int64, c_void_p, c_int, c_int, c_int, c_void_p]),
    "qq_quest_extend_kv": (
        c_int, [_S, c_int, c_int, _E, _T, c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p,
                c_int64, c_int64, _HB, c_void_p, c_void_p]),
    "qq_extend_attention": (
        c_int, [_E, _T, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p, c_void_p,
                c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qq_moe_route_plan": (
        c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_void_p]),
    "qq_moe_experts": (
        c_int, [POINTER(QQMoePlan), c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "qq_quest_decode_step": (
        c_int, [_S, c_int, c_int, c_int, _PP, c_int, c_int64, _B, c_void_p, c_void_p, _T, c_int64,
                c_void_p, c_size_t, c_void_p]),
    "qq_quest_group_queries": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int64, c_void_p, c_void_p]),
    "qq_quest_page_scores": (c_int, [_S, c_int, _B, c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p]),
    "qq_quest_retrieve_topk": (
        c_int, [_S, c_int, _B, c_void_p, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p, _T, c_void_p,
                _N, c_void_p, c_size_t, c_void_p]),
    "qq_sparse_decode_attention": (
        c_int, [_B, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p,
                c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "qq_sparse_decode_attention_ready": (
        c_int, [_B, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p,
                c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p, c_uint32, c_uint64, c_void_p,
                c_size_t, c_void_p]),
    "qq_quest_decode_attention": (
        c_int, [_S, c_int, _B, c_void_p, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p, _T, c_void_p,
                _N, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p,
                c_size_t, c_void_p]),
    "qq_sparse_decode_attention_noalloc": (
        c_int, [_B, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p,
                c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qq_hisparse_swap_in": (
        c_int, [_H, c_int, _B, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                c_void_p]),
    "qq_hisparse_reset": (c_int, [_H, c_int, c_void_p]),
    "qq_hisparse_admit_layout": (c_int, [_H, c_int, c_void_p]),
    "qq_host_ring_init": (c_int, [POINTER(QQHostRing), c_void_p]),
    "qq_host_ring_alloc": (c_int, [POINTER(QQHostRing), c_int64, c_void_p, c_void_p, c_void_p]),
    "qq_host_ring_free_request": (c_int, [_H, c_int, POINTER(QQHostRing), c_void_p]),
    "qq_hisparse_plan_step": (
        c_int, [_H, _B, c_void_p, POINTER(QQHostRing), c_void_p, c_void_p, c_void_p, c_void_p]),
    "qq_copy_rows": (
        c_int, [_PP, _PP, c_int, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int, c_int64, c_void_p]),
}

_lib: ctypes.CDLL | None = None


class QQError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("QQUEST_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} not found: the CUDA extension is not built (run __graft_entry__.build()); "
            "qwenquest_b200 has no CPU fallback"
        )
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    """Map a C-ABI status to the exception type the reference raises."""
    if rc == QQ_OK:
        return
    msg = load().qq_status_string(rc).decode()
    if rc in (QQ_ERR_INVALID, QQ_ERR_UNSUPPORTED, QQ_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    raise QQError(f"{what}: {msg}")


def raise_device_error(bits: int, what: str = "") -> None:
    """Raise the reference's exception for device error bits (``coordinator.py:278-286``)."""
    if bits == 0:
        return
    if bits & QQ_DEV_ERR_CAPACITY:
        raise RuntimeError(f"device_buffer_size too small for this top-k {what}".strip())
    if bits & QQ_DEV_ERR_NO_HOST_BACKUP:
        raise AssertionError(f"positions without host backup were selected {what}".strip())
    if bits & QQ_DEV_ERR_BOUNDS:
        raise QQError(f"an index out of range was skipped on the device {what}".strip())
    if bits & QQ_DEV_ERR_TIMEOUT:
        raise QQError(f"a bounded device wait ran out {what}".strip())
    raise QQError(f"device error bits {bits:#x} {what}".strip())


def ptr_array(ptrs: list[int]):
    """A host array of device pointers (``const void* const*``)."""
    arr = (c_void_p * len(ptrs))(*ptrs)
    return ctypes.cast(arr, _PP), arr


__all__ = [
    "QQBatch",
    "QQError",
    "QQExtendBatch",
    "QQHiSparseState",
    "QQMoePlan",
    "QQHotBuffer",
    "QQNewToken",
    "QQQuestState",
    "QQTokenTable",
    "QQHostRing",
    "check",
    "load",
    "ptr_array",
    "raise_device_error",
]

_ = (c_uint32,)
