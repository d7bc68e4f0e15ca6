// Shared device helpers for the Quest kernels (sm_100a).
#pragma once

#include <atomic>
#include <cstdlib>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qquest.h"

namespace qq {

// ---------------------------------------------------------------- numbers

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// +bf16max / -bf16max, the sentinels of an empty page (quest.py:57-58).
constexpr uint16_t kBf16MaxBits = 0x7F7F;
constexpr uint16_t kBf16MinBits = 0xFF7F;

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};
template <>
struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float round(float x) { return x; }
  static __device__ __forceinline__ void store(float* p, float x) { *p = x; }
};

// float -> uint32 key whose unsigned order is the float order (-inf lowest).
__device__ __forceinline__ uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------- errors

// The error word may live in mapped pinned host memory, where device atomics
// are not guaranteed; a plain read-modify-write is enough to leave it nonzero.
__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t bits) {
  if (err != nullptr) {
    volatile uint32_t* e = err;
    *e = *e | bits;
    __threadfence_system();
  }
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every spin-wait in these kernels gives up after this long and reports
// QQ_DEV_ERR_TIMEOUT instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------- shared memory

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- loads

// 16-byte async copy global -> shared (L2 only).
__device__ __forceinline__ void cp_async_16(uint32_t smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_dst), "l"(gmem_src) : "memory");
}
// The same with a source size: the bytes past src_bytes (all 16 for 0) are written as zeros.
__device__ __forceinline__ void cp_async_16_zfill(uint32_t smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_dst), "l"(gmem_src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}


// Read-only streaming 128-bit load (not volatile: the compiler may batch them).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// ---------------------------------------------------------------- programmatic dependent launch
//
// The decode-step kernels are launched with programmatic stream
// serialization: a kernel's blocks may be dispatched while the previous
// kernel in the stream finishes, and each block waits in wait_prior_grid()
// (griddepcontrol.wait: the previous grid has completed and its writes are
// visible) before it reads anything.  Without the launch attribute the wait
// returns at once.

__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream be dispatched once every block of this
// one has started (or exited); its blocks still wait for this grid to finish.
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- host helpers

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// QQ_PDL=0 in the environment launches without the attribute (for comparisons).
inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("QQ_PDL");
    on = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) == cudaSuccess ? QQ_OK : QQ_ERR_CUDA;
}

// ---------------------------------------------------------------- per-device state
//
// Values and kernel attributes are per device: a process may drive several
// GPUs, from several host threads.

constexpr int kMaxDevices = 64;

inline int current_device() {
  int d = -1;
  return cudaGetDevice(&d) == cudaSuccess ? d : -1;
}

// The current device's SM count, queried once per device.
inline int device_sm_count() {
  static std::atomic<int> cache[kMaxDevices];
  const int d = current_device();
  const bool cached = d >= 0 && d < kMaxDevices;
  if (cached) {
    const int v = cache[d].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d < 0 ? 0 : d) != cudaSuccess || n <= 0) n = 148;
  if (cached) cache[d].store(n, std::memory_order_relaxed);
  return n;
}

// A kernel's dynamic shared-memory limit on the current device, raised (never
// lowered) to what a launch needs, once per size and device, under a lock.
class SmemLimit {
 public:
  int ensure(const void* kernel, size_t bytes) {
    const int need = (int)bytes;
    if (need <= 48 * 1024) return QQ_OK;  // within the default limit
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return set(kernel, need);
    if (limit_[d].load(std::memory_order_acquire) >= need) return QQ_OK;
    std::lock_guard<std::mutex> lock(mutex_);
    if (limit_[d].load(std::memory_order_relaxed) >= need) return QQ_OK;
    const int rc = set(kernel, need);
    if (rc == QQ_OK) limit_[d].store(need, std::memory_order_release);
    return rc;
  }

 private:
  static int set(const void* kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess
               ? QQ_OK
               : QQ_ERR_CUDA;
  }
  std::atomic<int> limit_[kMaxDevices] = {};
  std::mutex mutex_;
};

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QQ_OK : QQ_ERR_CUDA;
}

// Workspace layout: arrival counters (int32, kept at zero between launches) —
// QQ_MAX_BS for the selection, QQ_MAX_BS for the bounds step, 4 * QQ_MAX_BS
// for the attention's (request, KV head) segments — then the selection's
// per-part top-32 lists (QQ_MAX_BS lists of 32 uint64 keys), then the
// attention partials.
constexpr size_t kCounterBytes = sizeof(int32_t) * QQ_MAX_BS;
enum CounterSlot { kCounterSelect = 0, kCounterStep = 1, kCounterAttn = 2 };
inline int32_t* ws_counters(void* ws, CounterSlot slot) {
  return reinterpret_cast<int32_t*>(static_cast<char*>(ws) + slot * kCounterBytes);
}
constexpr size_t kSelectListOffset = 6 * kCounterBytes;
constexpr int kSelectListLen = 32;
constexpr size_t kSelectListBytes = sizeof(uint64_t) * kSelectListLen * QQ_MAX_BS;
inline uint64_t* ws_select_lists(void* ws) {
  return reinterpret_cast<uint64_t*>(static_cast<char*>(ws) + kSelectListOffset);
}
constexpr size_t kPartialOffset = kSelectListOffset + kSelectListBytes;

// Attention partials: two (m, l, O) records of 8 query heads x 128 channels
// per warp of the streaming grid (8 warps per SM), then two per block.
constexpr int kAttnWarpsPerSm = 8;  // warps per block of the streaming kernel
constexpr size_t kAttnPartialFloats = 2 * (8 * 128 + 2 * 8);
inline size_t attn_warp_partial_floats(int sm_count) {
  return (size_t)sm_count * kAttnWarpsPerSm * kAttnPartialFloats;
}
inline size_t attn_partial_floats(int sm_count) {
  return attn_warp_partial_floats(sm_count) + (size_t)sm_count * kAttnPartialFloats;
}
// Then one ready word per request (uint32) for the fused selection +
// attention call: the selection stores the call's epoch once the request's
// rows are written, the attention spins on it.  Then the epoch state: the
// call counter (the current call's epoch is counter + 1, never 0) and the
// attention blocks' exit counter; the attention's last block to exit
// advances the call counter, so epochs live on the device and a captured
// call renews them on every replay.
inline size_t ready_offset(int sm_count) { return kPartialOffset + sizeof(float) * attn_partial_floats(sm_count); }
inline size_t epoch_offset(int sm_count) { return ready_offset(sm_count) + sizeof(uint32_t) * QQ_MAX_BS; }
inline size_t workspace_end(int sm_count) { return epoch_offset(sm_count) + 2 * sizeof(uint32_t); }

// The epoch that follows counter value c (0 and 0xFFFFFFFF are never epochs: ready words start at 0).
__host__ __device__ __forceinline__ uint32_t next_call_counter(uint32_t c) { return c + 2 == 0 ? 0u : c + 1; }

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace qq
