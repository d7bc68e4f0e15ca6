"""``HiSparseCoordinator`` on B200: the API of ``src/qwenquest/hisparse/coordinator.py:74-324``.

Two tiers, as in the reference:

* host: every request's full KV history in **pinned** host memory
  (``host_k/v[layer]``, ``[host_pool_size + 1, kv_heads, head_dim]``), mapped
  into the device address space so kernels read misses and write backups
  directly (zero-copy over the host link, no staging copies);
* device: per request a hot buffer of ``device_buffer_size`` LRU slots plus
  the reserved newest-token slot (``device_k/v[layer]``), with
  ``buffer_tokens`` / ``lru_slots`` (int32) describing it.

The swap-in (dedupe, hit detection, eviction, host->device copy, LRU
rewrite, row lookup) is one kernel launch per layer (``qq_hisparse_swap_in``);
the eager host backup of the previous token and admission copies are
``qq_copy_rows`` launches.  The host tier's free rows are a ring in device
memory (:class:`DeviceHostRows`, the reference's ``TokenToKVPoolAllocator``
API), so ``prepare_decode_step`` is three launches (the step plan, the bounds
fold, the backup copy) with no host round trip, and a whole decode step can
be captured in a CUDA graph.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from qwenquest_b200 import _lib
from qwenquest_b200._lib import QQ_STEP_FINALIZE, QQ_STEP_FOLD, check
from qwenquest_b200.quest import QuestAlgorithm, dtype_code, stream_of

__all__ = ["DeviceHostRows", "HiSparseCoordinator", "SwapInStats"]


class SwapInStats:
    """``SwapInStats`` (coordinator.py:48-59), counted on the device; reading syncs."""

    def __init__(self, counters: torch.Tensor):
        self._c = counters  # int64 [3]: hits, misses, fast_path_calls

    @property
    def hits(self) -> int:
        return int(self._c[0])

    @property
    def misses(self) -> int:
        return int(self._c[1])

    @property
    def fast_path_calls(self) -> int:
        return int(self._c[2])

    @property
    def hit_rate(self) -> float:
        total = self.hits + self.misses
        return self.hits / total if total else float("nan")

    def __repr__(self) -> str:
        return f"SwapInStats(hits={self.hits}, misses={self.misses}, fast_path_calls={self.fast_path_calls})"


def host_device_pointer(t: torch.Tensor) -> int:
    """Device address of a pinned host tensor (``cudaHostGetDevicePointer``)."""
    if not t.is_pinned():
        raise ValueError("the host tier must be pinned memory")
    out = ctypes.c_void_p()
    check(_lib.load().qq_host_device_pointer(t.data_ptr(), ctypes.byref(out)), "host_device_pointer")
    return int(out.value)


_DeviceErrorLike = "_DeviceError"


class DeviceHostRows:
    """The host tier's free rows (1 .. size) as a ring in device memory.

    The API of the reference's ``TokenToKVPoolAllocator`` over host indices
    (``memory.py:53-76``, used at ``coordinator.py:117``): ``alloc`` hands out
    rows from the front of the free list and freed rows go to its back, in
    the same order, but the list lives on the device, so allocating in a
    decode step needs no host round trip.  ``alloc`` returns a device tensor
    at once; running out is reported through the coordinator's device error
    word (``RuntimeError`` at its next check) instead of raising here.
    ``available_size`` reads the device and so synchronizes.
    """

    def __init__(self, size: int, device: torch.device, err: _DeviceErrorLike):
        self.size = size
        self.device = device
        self.lib = _lib.load()
        self._err = err
        self.rows = torch.empty(max(size, 1), dtype=torch.int64, device=device)
        self.state = torch.zeros(2, dtype=torch.int64, device=device)  # head, tail
        self.ring = _lib.QQHostRing(self.rows.data_ptr(), self.state.data_ptr(), size)
        if size > 0:
            check(self.lib.qq_host_ring_init(ctypes.byref(self.ring), stream_of(device)), "host ring init")

    def available_size(self) -> int:
        head, tail = self.state.tolist()
        return int(tail - head)

    def alloc(self, n: int) -> torch.Tensor:
        out = torch.empty(int(n), dtype=torch.int64, device=self.device)
        check(self.lib.qq_host_ring_alloc(ctypes.byref(self.ring), int(n), out.data_ptr(), self._err.ptr(),
                                          stream_of(self.device)), "host rows alloc")
        return out

    def free(self, indices: torch.Tensor) -> None:
        """Rows back to the end of the free list (synchronizes; the decode path frees per request on the device)."""
        idx = indices.to(device=self.device, dtype=torch.int64).flatten()
        idx = idx[idx > 0]
        n = int(idx.numel())
        if not n:
            return
        tail = int(self.state[1])
        pos = (tail + torch.arange(n, device=self.device)) % self.size
        self.rows[pos] = idx
        self.state[1] = tail + n


@dataclass
class _DeviceError:
    word: torch.Tensor  # pinned host int32 [1]; kernels OR error bits into it
    dev_ptr: int = 0

    def ptr(self) -> int:
        if not self.dev_ptr:
            self.dev_ptr = host_device_pointer(self.word)
        return self.dev_ptr

    def take(self) -> int:
        bits = int(self.word[0])
        if bits:
            self.word.zero_()
        return bits


@dataclass
class _Admission:
    """A prefill batch being admitted layer by layer."""

    reqs: list[int]
    src_rows: torch.Tensor  # device int32: pool row of every prefill position, requests in order
    host_rows: torch.Tensor  # device int64: the host-tier row it is backed up to
    layers: int = 0


class HiSparseCoordinator:
    def __init__(
        self,
        *,
        quest: QuestAlgorithm,
        num_layers: int,
        kv_heads: int,
        head_dim: int,
        max_reqs: int,
        max_context_len: int,
        top_k: int,
        device_buffer_size: int,
        host_pool_size: int,
        dtype: torch.dtype,
        device,
        host_device="cpu",
        host_layers: int | None = None,
    ):
        # coordinator.py:91-94
        if device_buffer_size < top_k:
            raise ValueError("device_buffer_size must be >= top_k")
        if quest.top_k != top_k:
            raise ValueError(f"QuestAlgorithm.top_k ({quest.top_k}) != top_k ({top_k})")
        if torch.device(host_device).type != "cpu":
            raise ValueError("the HiSparse host tier lives in pinned CPU memory")
        if not 0 < num_layers <= _lib.QQ_MAX_LAYERS:
            raise ValueError(f"num_layers must be in [1, {_lib.QQ_MAX_LAYERS}]")
        self.lib = _lib.load()
        self.quest = quest
        self.num_layers = num_layers
        self.top_k = top_k
        self.device_buffer_size = buf = device_buffer_size
        self.device = quest.device
        self.host_device = torch.device("cpu")
        self.kv_heads, self.head_dim, self.dtype = kv_heads, head_dim, dtype
        self.max_reqs, self.max_context_len = max_reqs, max_context_len
        dev = self.device

        # ---- host tier (pinned, device-mapped); its free rows on the device
        self._err = _DeviceError(torch.zeros(1, dtype=torch.int32).pin_memory())
        self.host_allocator = DeviceHostRows(host_pool_size, dev, self._err)
        hshape = (host_pool_size + 1, kv_heads, head_dim)
        # host_layers < num_layers aliases layer l onto host buffer l % host_layers
        # (benchmarks whose full host history would not fit in host RAM)
        nh = num_layers if host_layers is None else host_layers
        hk = [torch.zeros(hshape, dtype=dtype).pin_memory() for _ in range(nh)]
        hv = [torch.zeros(hshape, dtype=dtype).pin_memory() for _ in range(nh)]
        self.host_k = [hk[i % nh] for i in range(num_layers)]
        self.host_v = [hv[i % nh] for i in range(num_layers)]
        self.req_to_host_pool = torch.full((max_reqs, max_context_len), -1, dtype=torch.int32, device=dev)

        # ---- device tier
        dshape = (max_reqs * (buf + 1), kv_heads, head_dim)
        self.device_k = [torch.zeros(dshape, dtype=dtype, device=dev) for _ in range(num_layers)]
        self.device_v = [torch.zeros(dshape, dtype=dtype, device=dev) for _ in range(num_layers)]
        self.req_to_device_buffer = torch.arange(max_reqs * (buf + 1), dtype=torch.int64, device=dev).view(
            max_reqs, buf + 1
        )
        self.buffer_tokens = torch.full((num_layers, max_reqs, buf), -1, dtype=torch.int32, device=dev)
        self._lru_init = torch.arange(buf, dtype=torch.int32, device=dev)
        self.lru_slots = self._lru_init.repeat(num_layers, max_reqs, 1).contiguous()
        # set at admission, cleared by the first decode step (no previous token to back up yet)
        self._skip_first_backup = torch.zeros(max_reqs, dtype=torch.uint8, device=dev)
        self._plan_dev = torch.empty(max_reqs, dtype=torch.int64, device=dev)
        self._plan_host = torch.empty(max_reqs, dtype=torch.int64, device=dev)
        self._backup_stream: torch.cuda.Stream | None = None
        self._stats = torch.zeros(3, dtype=torch.int64, device=dev)
        self.stats = SwapInStats(self._stats)
        self._hs = _lib.QQHiSparseState(
            self.buffer_tokens.data_ptr(), self.lru_slots.data_ptr(), self.req_to_host_pool.data_ptr(),
            self._stats.data_ptr(), num_layers, max_reqs, max_context_len, buf, top_k,
        )
        self.row_bytes = kv_heads * head_dim * torch.empty(0, dtype=dtype).element_size()
        # per-layer pointer arrays (K layers then V layers)
        self._dev_ptrs = _lib.ptr_array([t.data_ptr() for t in self.device_k + self.device_v])
        self._host_dev = [host_device_pointer(t) for t in self.host_k + self.host_v]
        self._host_ptrs = _lib.ptr_array(self._host_dev)
        self._dev_k_ptrs = _lib.ptr_array([t.data_ptr() for t in self.device_k[quest.start_layer:quest.end_layer]])

    def _stream(self) -> int:
        return stream_of(self.device)

    def check_errors(self, what: str = "") -> None:
        _lib.raise_device_error(self._err.take(), what)

    # -------------------------------------------------- [H1] admission

    def admit_request(self, req_pool_idx, prefill_len, token_to_kv_pool, prefill_indices) -> None:
        """[H1] (coordinator.py:138-174): host backup of the prefill, hot buffer, bounds."""
        req = int(req_pool_idx)
        n = int(prefill_len)
        idx = prefill_indices.to(device=self.device, dtype=torch.int32).contiguous()
        host_idx_dev = self.host_allocator.alloc(n)
        self.req_to_host_pool[req, :n] = host_idx_dev.to(torch.int32)
        n_dev = min(n, self.device_buffer_size)
        kb = [token_to_kv_pool.get_key_buffer(layer) for layer in range(self.num_layers)]
        vb = [token_to_kv_pool.get_value_buffer(layer) for layer in range(self.num_layers)]
        src_arr, keep = _lib.ptr_array([t.data_ptr() for t in kb + vb])
        stride = kb[0].stride(0) * kb[0].element_size()
        s = self._stream()
        # all prefill rows -> host tier
        check(self.lib.qq_copy_rows(src_arr, self._host_ptrs[0], 2 * self.num_layers, stride, self.row_bytes,
                                    self.row_bytes, idx.data_ptr(), 0, host_idx_dev.data_ptr(), 1, n, s),
              "admit_request host copy")
        # positions [0, n_dev) -> slots [0, n_dev) of the hot buffer
        dev_rows = self.req_to_device_buffer[req, :n_dev].contiguous()
        check(self.lib.qq_copy_rows(src_arr, self._dev_ptrs[0], 2 * self.num_layers, stride, self.row_bytes,
                                    self.row_bytes, idx.data_ptr(), 0, dev_rows.data_ptr(), 1, n_dev, s),
              "admit_request device copy")
        check(self.lib.qq_hisparse_admit_layout(self._hs, req, s), "admit_request layout")
        q = self.quest
        q.update_prefill_representations_all_layers(req, kb[q.start_layer:q.end_layer], idx)
        self._skip_first_backup[req] = 1
        del keep

    # ------------------------------------ [H1] admission fused with the prefill

    def begin_admission(self, reqs: list[int], seq_lens: list[int], req_to_token: torch.Tensor) -> _Admission:
        """Host rows for a prefill batch, taken before its first layer so each layer backs up as it goes.

        The layers' K/V writes (``qq_quest_extend_kv`` with this coordinator's
        hot buffer) fill the device tier and the bounds; :meth:`backup_layer`
        copies each layer's rows to the host tier on a side stream, overlapped
        with the following layers; :meth:`finish_admission` joins it and lays
        out the slots.  Together the same state as :meth:`admit_request`
        (``coordinator.py:138-174``).
        """
        src, dst = [], []
        for req, n in zip(reqs, seq_lens, strict=True):
            host_idx_dev = self.host_allocator.alloc(n)
            self.req_to_host_pool[req, :n] = host_idx_dev.to(torch.int32)
            src.append(req_to_token[req, :n].to(torch.int32))
            dst.append(host_idx_dev.to(torch.int64))
        if self._backup_stream is None:
            self._backup_stream = torch.cuda.Stream(device=self.device)
        return _Admission(list(reqs), torch.cat(src).contiguous(), torch.cat(dst).contiguous())

    def hot_buffer(self, layer_id: int) -> _lib.QQHotBuffer:
        kd, vd = self.device_k[layer_id], self.device_v[layer_id]
        return _lib.QQHotBuffer(kd.data_ptr(), vd.data_ptr(), kd.stride(0), self.device_buffer_size, kd.shape[0])

    def backup_layer(self, adm: _Admission, layer_id: int, token_to_kv_pool) -> None:
        """Copy layer ``layer_id``'s prefill rows to the host tier, behind that layer's K/V write."""
        kb, vb = token_to_kv_pool.get_kv_buffer(layer_id)
        side = self._backup_stream
        side.wait_stream(torch.cuda.current_stream(self.device))
        src, keep_s = _lib.ptr_array([kb.data_ptr(), vb.data_ptr()])
        dst, keep_d = _lib.ptr_array([self._host_dev[layer_id], self._host_dev[self.num_layers + layer_id]])
        check(self.lib.qq_copy_rows(src, dst, 2, kb.stride(0) * kb.element_size(), self.row_bytes,
                                    self.row_bytes, adm.src_rows.data_ptr(), 0, adm.host_rows.data_ptr(), 1,
                                    adm.host_rows.numel(), side.cuda_stream),
              "admission host backup")
        del keep_s, keep_d
        adm.layers += 1

    def finish_admission(self, adm: _Admission) -> None:
        """Join the host backups and set each request's slot layout (the end of ``admit_request``)."""
        if adm.layers != self.num_layers:
            raise RuntimeError(f"admission backed up {adm.layers} of {self.num_layers} layers")
        torch.cuda.current_stream(self.device).wait_stream(self._backup_stream)
        s = self._stream()
        for req in adm.reqs:
            check(self.lib.qq_hisparse_admit_layout(self._hs, req, s), "admit_request layout")
        self._skip_first_backup[torch.tensor(adm.reqs, dtype=torch.int64).to(self.device, non_blocking=True)] = 1

    # -------------------------------------------------- [H2] per decode step

    def newest_slot(self, seq_lens: torch.Tensor) -> torch.Tensor:
        return (seq_lens.long() - 1).clamp(max=self.device_buffer_size)

    def prepare_decode_step(self, req_pool_indices: torch.Tensor, seq_lens: torch.Tensor) -> None:
        """[H2] (coordinator.py:183-215): fold the previous token's key into the bounds, back it up.

        Three launches and no host round trip: the step plan (skip flags, a
        new host row per request from the device free list, in batch order,
        ``req_to_host_pool``), the bounds fold of the previous token (all
        layers) and its K/V copy from the hot buffer to the host tier.
        """
        dev = self.device
        reqs = req_pool_indices.to(device=dev, dtype=torch.int64).contiguous()
        seq = seq_lens.to(device=dev, dtype=torch.int64).contiguous()
        bs = int(reqs.shape[0])
        if bs == 0:
            return
        if bs > self.max_reqs:
            raise ValueError(f"batch of {bs} requests exceeds max_reqs ({self.max_reqs})")
        s = self._stream()
        batch = _lib.QQBatch(reqs.data_ptr(), seq.data_ptr(), bs)
        check(self.lib.qq_hisparse_plan_step(self._hs, batch, self._skip_first_backup.data_ptr(),
                                             ctypes.byref(self.host_allocator.ring), self._plan_dev.data_ptr(),
                                             self._plan_host.data_ptr(), self._err.ptr(), s),
              "decode step plan")
        q = self.quest
        q.decode_step(QQ_STEP_FOLD | QQ_STEP_FINALIZE, reqs, None, None, rows=self._plan_dev,
                      k_ptrs=self._dev_k_ptrs[0], kv_dtype=dtype_code(self.dtype),
                      k_row_stride=self.kv_heads * self.head_dim)
        check(self.lib.qq_copy_rows(self._dev_ptrs[0], self._host_ptrs[0], 2 * self.num_layers, self.row_bytes,
                                    self.row_bytes, self.row_bytes, self._plan_dev.data_ptr(), 1,
                                    self._plan_host.data_ptr(), 1, bs, s),
              "eager host backup")

    def write_new_token(self, layer_id, req_pool_indices, seq_lens, k, v) -> None:
        """``set_kv_buffer`` redirected into the hot buffer (coordinator.py:217-228)."""
        locs = self.req_to_device_buffer[req_pool_indices.long(), self.newest_slot(seq_lens)]
        self.device_k[layer_id][locs] = k.to(self.device_k[layer_id].dtype)
        self.device_v[layer_id][locs] = v.to(self.device_v[layer_id].dtype)

    # -------------------------------------------------- [H3] swap-in

    def swap_in(self, reqs, seq_lens, positions, layer_id, rows_out) -> None:
        """One ``qq_hisparse_swap_in`` launch writing int32 rows into ``rows_out``."""
        bs = int(reqs.shape[0])
        batch = _lib.QQBatch(reqs.data_ptr(), seq_lens.data_ptr(), bs)
        rc = self.lib.qq_hisparse_swap_in(
            self._hs, int(layer_id), batch, positions.data_ptr(), rows_out.data_ptr(),
            self._host_dev[layer_id], self._host_dev[self.num_layers + layer_id],
            self.device_k[layer_id].data_ptr(), self.device_v[layer_id].data_ptr(), self.row_bytes,
            self._err.ptr(), self._stream(),
        )
        check(rc, "swap_in_selected_pages")

    def swap_in_selected_pages(self, req_pool_indices, seq_lens, top_k_result, layer_id) -> torch.Tensor:
        """[H3] (coordinator.py:232-257): ``[bs, top_k]`` int64 device rows, ``-1`` padded.

        Errors (buffer too small, missing host backup) raise here, as in the
        reference; this synchronizes the stream.
        """
        dev = self.device
        reqs = req_pool_indices.to(device=dev, dtype=torch.int64).contiguous()
        seq = seq_lens.to(device=dev, dtype=torch.int64).contiguous()
        pos = top_k_result.to(device=dev, dtype=torch.int32).contiguous()
        if pos.shape[1] != self.top_k:
            full = torch.zeros((pos.shape[0], self.top_k), dtype=torch.int32, device=dev)
            full[:, : pos.shape[1]] = pos
            pos = full
        rows = torch.empty((reqs.shape[0], self.top_k), dtype=torch.int32, device=dev)
        self.swap_in(reqs, seq, pos, layer_id, rows)
        torch.cuda.current_stream(dev).synchronize()
        self.check_errors(f"(layer {layer_id})")
        return rows.to(torch.int64)

    # -------------------------------------------------- [H4] release

    def request_finished(self, req_pool_idx: int) -> None:
        """[H4] (coordinator.py:308-316), on the device: the host rows go back to the free list."""
        req = int(req_pool_idx)
        s = self._stream()
        check(self.lib.qq_host_ring_free_request(self._hs, req, ctypes.byref(self.host_allocator.ring), s),
              "request_finished host rows")
        check(self.lib.qq_hisparse_reset(self._hs, req, s), "request_finished")
        self._skip_first_backup[req] = 0
        self.quest.invalidate_request(req)

    # -------------------------------------------------- introspection

    def device_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (*self.device_k, *self.device_v))

    def host_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in {id(t): t for t in self.host_k + self.host_v}.values())

