// [H3] HiSparse swap-in, [H1]/[H4] slot layout resets, and row copies
// between the device pools and the pinned host tier.
//
// Swap-in: one 1024-thread block per request.  In shared memory it holds the
// slot -> position table of the request's hot buffer (buffer_tokens), its LRU
// order, and two open-addressing hash tables (cached position -> slot, and
// wanted position -> first index).  Every step that the reference performs
// with unique / isin / cat / sort is a block-wide stable compaction (prefix
// sum) here, so the results — first-occurrence order of the unique positions,
// LRU scan order of the hits, victims taken from the least recently used end
// — are the same bit for bit.  Misses are read straight from the host tier
// (mapped pinned memory) by the block's warps, one 1 KiB row per warp at a
// time, and written into the victim slots.  Integer/byte work, latency- and
// host-link-bound.

#include <climits>

#include <algorithm>

#include "common.cuh"

namespace qq {
namespace {

constexpr int kSwapThreads = 1024;

struct SwapArgs {
  qq_hisparse_state hs;
  int layer;
  const int64_t* reqs;
  const int64_t* seq_lens;
  const int32_t* positions;
  int32_t* rows_out;
  const char* host_k;
  const char* host_v;
  char* dev_k;
  char* dev_v;
  int64_t row_bytes;
  uint32_t* err;
  int ht1_log2;  // cached-position table: 2^ht1_log2 entries
  int ht2_log2;  // wanted-position table
};

__device__ __forceinline__ uint32_t hash_slot(int32_t key, int log2n) {
  return ((uint32_t)key * 2654435761u) >> (32 - log2n);
}

__device__ __forceinline__ void ht_insert(int32_t* keys, int32_t* vals, int log2n, int32_t key, int32_t val,
                                          bool keep_min) {
  const uint32_t mask = (1u << log2n) - 1;
  uint32_t h = hash_slot(key, log2n);
  while (true) {
    const int32_t prev = atomicCAS(&keys[h], -1, key);
    if (prev == -1 || prev == key) {
      if (keep_min)
        atomicMin(&vals[h], val);
      else
        vals[h] = val;
      return;
    }
    h = (h + 1) & mask;
  }
}

// Entry index of `key`, or -1.  Tables are never more than half full, so the
// probe always reaches an empty entry.
__device__ __forceinline__ int ht_index(const int32_t* keys, int log2n, int32_t key) {
  const uint32_t mask = (1u << log2n) - 1;
  uint32_t h = hash_slot(key, log2n);
  while (true) {
    const int32_t k = keys[h];
    if (k == key) return (int)h;
    if (k == -1) return -1;
    h = (h + 1) & mask;
  }
}

__device__ __forceinline__ int32_t ht_find(const int32_t* keys, const int32_t* vals, int log2n, int32_t key) {
  const int e = ht_index(keys, log2n, key);
  return e < 0 ? -1 : vals[e];
}

// Exclusive prefix sum of one flag per thread over the block; returns the
// prefix, writes the block total to *total.  `scratch`: 32 ints.
__device__ __forceinline__ int block_scan(int flag, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned ballot = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(ballot & ((1u << lane) - 1));
  if (lane == 0) scratch[warp] = __popc(ballot);
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int v = lane < nw ? scratch[lane] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane < nw) scratch[lane] = incl - v;
    if (lane == 31) scratch[32] = incl;
  }
  __syncthreads();
  const int res = scratch[warp] + in_warp;
  *total = scratch[32];
  __syncthreads();
  return res;
}

__device__ __forceinline__ void copy_row(char* dst, const char* src, int64_t bytes, int lane) {
  if ((bytes & 15) == 0 && ((uintptr_t)dst & 15) == 0 && ((uintptr_t)src & 15) == 0) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int64_t w = lane; w < bytes / 16; w += 32) d[w] = s[w];
  } else {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (int64_t w = lane; w < bytes / 4; w += 32) d[w] = s[w];
  }
}

__global__ void __launch_bounds__(kSwapThreads) swap_in_kernel(SwapArgs a) {
  extern __shared__ int32_t sm[];
  const qq_hisparse_state& hs = a.hs;
  const int buf = hs.device_buffer_size;
  const int top_k = hs.top_k;
  const int n1 = 1 << a.ht1_log2, n2 = 1 << a.ht2_log2;
  int32_t* s_tok = sm;                // [buf]
  int32_t* s_lru = s_tok + buf;       // [buf]
  int32_t* s_hit = s_lru + buf;       // [buf] slot is wanted
  int32_t* s_pos = s_hit + buf;       // [top_k]
  int32_t* s_uniq = s_pos + top_k;    // [top_k]
  int32_t* s_miss = s_uniq + top_k;   // [top_k]
  int32_t* s_vict = s_miss + top_k;   // [top_k]
  int32_t* h1k = s_vict + top_k;      // [n1] cached position -> slot
  int32_t* h1v = h1k + n1;
  int32_t* h2k = h1v + n1;            // [n2] wanted position -> first index
  int32_t* h2v = h2k + n2;
  __shared__ int s_scan[33];

  const int i = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t req = a.reqs[i];
  const int64_t L = a.seq_lens[i];
  const int n = (int)(L < top_k ? L : top_k);
  const int32_t* pos_in = a.positions + (int64_t)i * top_k;
  int32_t* rows = a.rows_out + (int64_t)i * top_k;
  const int64_t base_row = req * (int64_t)(buf + 1);
  for (int j = n + tid; j < top_k; j += kSwapThreads) rows[j] = -1;

  if (L <= buf) {  // fast path: slot == position (coordinator.py:251-254)
    for (int j = tid; j < n; j += kSwapThreads) rows[j] = (int32_t)(base_row + pos_in[j]);
    if (tid == 0) atomicAdd(&hs.stats[2], 1ull);
    return;
  }

  const size_t lr = ((size_t)a.layer * hs.max_reqs + req) * buf;
  int32_t* g_tok = hs.buffer_tokens + lr;
  int32_t* g_lru = hs.lru_slots + lr;
  const int32_t* h2p = hs.req_to_host_pool + req * (int64_t)hs.max_context_len;
  const int32_t newest = (int32_t)(L - 1);

  // 1. load state, build the cached-position table and the wanted-position table
  for (int e = tid; e < n1; e += kSwapThreads) h1k[e] = -1;
  for (int e = tid; e < n2; e += kSwapThreads) {
    h2k[e] = -1;
    h2v[e] = INT_MAX;
  }
  for (int s = tid; s < buf; s += kSwapThreads) {
    s_tok[s] = g_tok[s];
    s_lru[s] = g_lru[s];
    s_hit[s] = 0;
  }
  int bad_pos = 0;
  for (int j = tid; j < n; j += kSwapThreads) {
    const int32_t p = pos_in[j];
    s_pos[j] = p;
    bad_pos |= p < 0 || p >= L;
  }
  if (__syncthreads_or(bad_pos)) {  // positions come from the selection; never index with bad ones
    if (tid == 0) raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    return;
  }
  for (int s = tid; s < buf; s += kSwapThreads)
    if (s_tok[s] >= 0) ht_insert(h1k, h1v, a.ht1_log2, s_tok[s], s, false);
  for (int j = tid; j < n; j += kSwapThreads)
    if (s_pos[j] != newest) ht_insert(h2k, h2v, a.ht2_log2, s_pos[j], j, true);
  __syncthreads();

  // 2. unique wanted positions in first-occurrence order (coordinator.py:62-71, 267-268)
  int n_uniq = 0;
  for (int j0 = 0; j0 < n; j0 += kSwapThreads) {
    const int j = j0 + tid;
    int first = 0;
    if (j < n) {
      const int32_t p = s_pos[j];
      first = p != newest && ht_find(h2k, h2v, a.ht2_log2, p) == j;
    }
    int tot;
    const int pre = block_scan(first, s_scan, &tot);
    if (first) s_uniq[n_uniq + pre] = s_pos[j];
    n_uniq += tot;
  }
  __syncthreads();

  // 3. hit detection: misses in unique order, hit slots marked (coordinator.py:273-276).
  // From here on the wanted-position table maps a position to its slot.
  int n_miss = 0;
  for (int u0 = 0; u0 < n_uniq; u0 += kSwapThreads) {
    const int u = u0 + tid;
    int miss = 0;
    if (u < n_uniq) {
      const int32_t slot = ht_find(h1k, h1v, a.ht1_log2, s_uniq[u]);
      if (slot >= 0) {
        s_hit[slot] = 1;
        h2v[ht_index(h2k, a.ht2_log2, s_uniq[u])] = slot;
      } else {
        miss = 1;
      }
    }
    int tot;
    const int pre = block_scan(miss, s_scan, &tot);
    if (miss) s_miss[n_miss + pre] = s_uniq[u];
    n_miss += tot;
  }
  __syncthreads();

  // 4. LRU scan: hits keep scan order, evictables are least recently used first
  int n_hit = 0;
  for (int k0 = 0; k0 < buf; k0 += kSwapThreads) {
    const int k = k0 + tid;
    const int hit = k < buf ? s_hit[s_lru[k]] : 0;
    int tot;
    const int pre = block_scan(hit, s_scan, &tot);
    if (k < buf && !hit) {
      const int e = k - (n_hit + pre);  // rank among evictables
      if (e < n_miss) s_vict[e] = s_lru[k];
    }
    n_hit += tot;
  }
  const int n_evict = buf - n_hit;
  // capacity and host-backup checks before any state changes (coordinator.py:278-286)
  if (n_miss > n_evict) {
    if (tid == 0) raise_error(a.err, QQ_DEV_ERR_CAPACITY);
    return;
  }
  int bad = 0;
  for (int m = tid; m < n_miss; m += kSwapThreads) {
    const int32_t p = s_miss[m];
    if (p < 0 || p >= hs.max_context_len || h2p[p] < 0) bad = 1;
  }
  if (__syncthreads_or(bad)) {
    if (tid == 0) raise_error(a.err, QQ_DEV_ERR_NO_HOST_BACKUP);
    return;
  }

  // 5. new LRU order [evictable[n_miss:] | victims | hits] (coordinator.py:295)
  {
    int hits_before = 0;
    for (int k0 = 0; k0 < buf; k0 += kSwapThreads) {
      const int k = k0 + tid;
      const int hit = k < buf ? s_hit[s_lru[k]] : 0;
      int tot;
      const int pre = block_scan(hit, s_scan, &tot);
      if (k < buf) {
        int dst;
        if (hit) {
          dst = n_evict + hits_before + pre;
        } else {
          const int e = k - (hits_before + pre);
          dst = e >= n_miss ? e - n_miss : (n_evict - n_miss) + e;
        }
        g_lru[dst] = s_lru[k];
      }
      hits_before += tot;
    }
  }
  // 6. load the misses into the victim slots: host tier -> hot buffer
  for (int m = tid; m < n_miss; m += kSwapThreads) {
    const int32_t v = s_vict[m];
    g_tok[v] = s_miss[m];
    h2v[ht_index(h2k, a.ht2_log2, s_miss[m])] = v;
  }
  for (int m = warp; m < n_miss; m += kSwapThreads / 32) {
    const int64_t host_row = h2p[s_miss[m]];
    const int64_t dev_row = base_row + s_vict[m];
    copy_row(a.dev_k + dev_row * a.row_bytes, a.host_k + host_row * a.row_bytes, a.row_bytes, lane);
    copy_row(a.dev_v + dev_row * a.row_bytes, a.host_v + host_row * a.row_bytes, a.row_bytes, lane);
  }
  __syncthreads();

  // 7. row of every requested entry, duplicates included (coordinator.py:298-300)
  for (int j = tid; j < n; j += kSwapThreads) {
    const int32_t p = s_pos[j];
    int32_t slot = p == newest ? buf : ht_find(h2k, h2v, a.ht2_log2, p);
    if (slot < 0) {  // cannot happen: every wanted position is cached now
      raise_error(a.err, QQ_DEV_ERR_BOUNDS);
      slot = buf;
    }
    rows[j] = (int32_t)(base_row + slot);
  }
  if (tid == 0) {
    atomicAdd(&hs.stats[0], (unsigned long long)(n_uniq - n_miss));
    atomicAdd(&hs.stats[1], (unsigned long long)n_miss);
  }
}

__global__ void hisparse_layout_kernel(qq_hisparse_state hs, int req, int mode) {
  // mode 0: reset (tokens -1, lru 0..buf-1, host table -1); mode 1: admission (tokens = lru = 0..buf-1)
  const int layer = blockIdx.y;
  const int buf = hs.device_buffer_size;
  const size_t off = ((size_t)layer * hs.max_reqs + req) * buf;
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < buf; s += gridDim.x * blockDim.x) {
    hs.buffer_tokens[off + s] = mode == 0 ? -1 : s;
    hs.lru_slots[off + s] = s;
  }
  if (mode == 0 && layer == 0) {
    int32_t* t = hs.req_to_host_pool + (int64_t)req * hs.max_context_len;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < hs.max_context_len; p += gridDim.x * blockDim.x)
      t[p] = -1;
  }
}

constexpr int kCopyMaxPtrs = 2 * QQ_MAX_LAYERS;
struct CopyArgs {
  const char* src[kCopyMaxPtrs];
  char* dst[kCopyMaxPtrs];
  int64_t src_stride;
  int64_t dst_stride;
  int64_t row_bytes;
  const void* src_idx;
  const void* dst_idx;
  int src64;
  int dst64;
  int64_t n;
};

__global__ void copy_rows_kernel(CopyArgs a) {
  const int layer = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= a.n) return;
  const int64_t si = a.src64 ? static_cast<const int64_t*>(a.src_idx)[r] : static_cast<const int32_t*>(a.src_idx)[r];
  const int64_t di = a.dst64 ? static_cast<const int64_t*>(a.dst_idx)[r] : static_cast<const int32_t*>(a.dst_idx)[r];
  if (si < 0 || di < 0) return;  // an entry with nothing to copy
  copy_row(a.dst[layer] + di * a.dst_stride, a.src[layer] + si * a.src_stride, a.row_bytes, lane);
}

// ------------------------------------------------------------------ host-tier rows on the device
//
// The host tier's free rows are a ring in device memory (the role of the
// reference's TokenToKVPoolAllocator over host indices, memory.py:53-76):
// rows[(c) % capacity] for allocation count c in [head, tail); allocation
// takes from the head in ring order, a finished request's rows go back at
// the tail in position order, so the order of rows handed out is the
// reference's (its free list pops from the front and appends at the back).
// head and tail only grow; everything runs on the device, in stream order.

// Exclusive prefix sum of `v` over the block (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < nw) s_warp[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int before = warp > 0 ? s_warp[warp - 1] : 0;
  total = s_warp[nw - 1];
  __syncthreads();
  return before + incl - v;
}

__global__ void ring_init_kernel(qq_host_ring r) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < r.capacity; k += (int64_t)gridDim.x * blockDim.x)
    r.rows[k] = k + 1;  // rows 1 .. capacity (row 0 is padding)
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    r.state[0] = 0;
    r.state[1] = r.capacity;
  }
}

// n rows from the head into out (-1 and QQ_DEV_ERR_CAPACITY when fewer are free).
__global__ void ring_alloc_kernel(qq_host_ring r, int64_t n, int64_t* out, uint32_t* err) {
  const int64_t head = r.state[0], avail = r.state[1] - head;
  for (int64_t k = threadIdx.x; k < n; k += blockDim.x) out[k] = k < avail ? r.rows[(head + k) % r.capacity] : -1;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (n > avail) raise_error(err, QQ_DEV_ERR_CAPACITY);
    r.state[0] = head + (n < avail ? n : avail);
  }
}

// A finished request's host rows (req_to_host_pool[req][p] >= 0, in position
// order) go back to the ring's tail; the entries become -1.
__global__ void ring_free_request_kernel(qq_hisparse_state hs, int req, qq_host_ring r) {
  __shared__ int s_warp[32];
  __shared__ int64_t s_tail;
  int32_t* row = hs.req_to_host_pool + (int64_t)req * hs.max_context_len;
  if (threadIdx.x == 0) s_tail = r.state[1];
  __syncthreads();
  for (int p0 = 0; p0 < hs.max_context_len; p0 += blockDim.x) {
    const int p = p0 + threadIdx.x;
    const int32_t h = p < hs.max_context_len ? row[p] : -1;
    int total = 0;
    const int rank = block_exclusive_scan(h >= 0 ? 1 : 0, s_warp, total);
    if (h >= 0) {
      r.rows[(s_tail + rank) % r.capacity] = h;
      row[p] = -1;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_tail += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) r.state[1] = s_tail;
}

// [H2] The per-step plan of HiSparseCoordinator.prepare_decode_step
// (coordinator.py:183-215) without the host: for every batch entry whose
// request is not on its first decode step (skip flag, cleared here), the
// previous token (position seq_len - 2) is backed up from its hot-buffer row
// req * (buf + 1) + min(seq_len - 2, buf) to a new host row taken from the
// ring in batch order; req_to_host_pool records it.  plan_dev / plan_host
// get those rows (-1 for a skipped entry) for the bounds fold and the copy.
__global__ void plan_step_kernel(qq_hisparse_state hs, const int64_t* reqs, const int64_t* seq_lens, int bs,
                                 uint8_t* skip, qq_host_ring r, int64_t* plan_dev, int64_t* plan_host,
                                 uint32_t* err) {
  __shared__ int s_warp[32];
  __shared__ int64_t s_head, s_avail;
  if (threadIdx.x == 0) {
    s_head = r.state[0];
    s_avail = r.state[1] - s_head;
  }
  __syncthreads();
  const int64_t buf = hs.device_buffer_size;
  int64_t taken = 0;
  for (int i0 = 0; i0 < bs; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    bool need = false;
    int64_t req = -1, prev = 0;
    if (i < bs) {
      req = reqs[i];
      if (req < 0 || req >= hs.max_reqs) {
        raise_error(err, QQ_DEV_ERR_BOUNDS);
      } else if (skip[req]) {
        skip[req] = 0;
      } else {
        prev = seq_lens[i] - 2;
        need = prev >= 0 && prev < hs.max_context_len;
      }
    }
    int total = 0;
    const int64_t rank = taken + block_exclusive_scan(need ? 1 : 0, s_warp, total);
    if (i < bs) {
      int64_t dev = -1, host = -1;
      if (need) {
        if (rank < s_avail) {
          dev = req * (buf + 1) + (prev < buf ? prev : buf);
          host = r.rows[(s_head + rank) % r.capacity];
          hs.req_to_host_pool[req * hs.max_context_len + prev] = (int32_t)host;
        } else {
          raise_error(err, QQ_DEV_ERR_CAPACITY);
        }
      }
      plan_dev[i] = dev;
      plan_host[i] = host;
    }
    taken += total;
  }
  if (threadIdx.x == 0) r.state[0] = s_head + (taken < s_avail ? taken : s_avail);
}

bool valid_hs(const qq_hisparse_state* hs) {
  return hs != nullptr && hs->buffer_tokens && hs->lru_slots && hs->req_to_host_pool && hs->stats &&
         hs->num_layers > 0 && hs->max_reqs > 0 && hs->max_context_len > 0 && hs->device_buffer_size > 0 &&
         hs->top_k > 0 && hs->top_k <= hs->device_buffer_size;
}

int ceil_log2(int x) {
  int l = 0;
  while ((1 << l) < x) ++l;
  return l;
}

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" int qq_hisparse_swap_in(const qq_hisparse_state* hs, int layer, const qq_batch* batch,
                                   const int32_t* positions, int32_t* rows_out, const void* host_k,
                                   const void* host_v, void* dev_k, void* dev_v, int64_t row_bytes,
                                   uint32_t* err, void* stream) {
  if (!valid_hs(hs) || batch == nullptr || layer < 0 || layer >= hs->num_layers || positions == nullptr ||
      rows_out == nullptr || !host_k || !host_v || !dev_k || !dev_v || row_bytes <= 0 || row_bytes % 4)
    return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || !batch->req_pool_indices || !batch->seq_lens)
    return QQ_ERR_INVALID;
  SwapArgs a{};
  a.hs = *hs;
  a.layer = layer;
  a.reqs = batch->req_pool_indices;
  a.seq_lens = batch->seq_lens;
  a.positions = positions;
  a.rows_out = rows_out;
  a.host_k = static_cast<const char*>(host_k);
  a.host_v = static_cast<const char*>(host_v);
  a.dev_k = static_cast<char*>(dev_k);
  a.dev_v = static_cast<char*>(dev_v);
  a.row_bytes = row_bytes;
  a.err = err;
  a.ht1_log2 = std::max(5, ceil_log2(2 * hs->device_buffer_size));
  a.ht2_log2 = std::max(5, ceil_log2(2 * hs->top_k));
  const size_t smem = sizeof(int32_t) * (3 * (size_t)hs->device_buffer_size + 4 * (size_t)hs->top_k +
                                         2 * ((size_t)1 << a.ht1_log2) + 2 * ((size_t)1 << a.ht2_log2));
  int dev = 0, max_optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem > (size_t)max_optin) return QQ_ERR_UNSUPPORTED;
  static SmemLimit limit;  // per device
  const int rc = limit.ensure((const void*)swap_in_kernel, smem);
  if (rc != QQ_OK) return rc;
  swap_in_kernel<<<batch->bs, kSwapThreads, smem, as_stream(stream)>>>(a);
  return launch_status();
}

extern "C" int qq_hisparse_reset(const qq_hisparse_state* hs, int req, void* stream) {
  if (!valid_hs(hs) || req < 0 || req >= hs->max_reqs) return QQ_ERR_INVALID;
  hisparse_layout_kernel<<<dim3(8, hs->num_layers), 256, 0, as_stream(stream)>>>(*hs, req, 0);
  return launch_status();
}

extern "C" int qq_hisparse_admit_layout(const qq_hisparse_state* hs, int req, void* stream) {
  if (!valid_hs(hs) || req < 0 || req >= hs->max_reqs) return QQ_ERR_INVALID;
  hisparse_layout_kernel<<<dim3(8, hs->num_layers), 256, 0, as_stream(stream)>>>(*hs, req, 1);
  return launch_status();
}

extern "C" int qq_copy_rows(const void* const* src_layers, void* const* dst_layers, int num_layers,
                            int64_t src_row_stride, int64_t dst_row_stride, int64_t row_bytes,
                            const void* src_idx, int src_idx_is64, const void* dst_idx, int dst_idx_is64,
                            int64_t n, void* stream) {
  if (src_layers == nullptr || dst_layers == nullptr || num_layers <= 0 || num_layers > kCopyMaxPtrs ||
      row_bytes <= 0 || row_bytes % 4 || n < 0 || src_row_stride < row_bytes || dst_row_stride < row_bytes)
    return QQ_ERR_INVALID;
  if (n == 0) return QQ_OK;
  if (src_idx == nullptr || dst_idx == nullptr) return QQ_ERR_INVALID;
  CopyArgs a{};
  for (int l = 0; l < num_layers; ++l) {
    if (!src_layers[l] || !dst_layers[l]) return QQ_ERR_INVALID;
    a.src[l] = static_cast<const char*>(src_layers[l]);
    a.dst[l] = static_cast<char*>(dst_layers[l]);
  }
  a.src_stride = src_row_stride;
  a.dst_stride = dst_row_stride;
  a.row_bytes = row_bytes;
  a.src_idx = src_idx;
  a.dst_idx = dst_idx;
  a.src64 = src_idx_is64;
  a.dst64 = dst_idx_is64;
  a.n = n;
  const int warps = 8;
  dim3 grid((unsigned)((n + warps - 1) / warps), num_layers);
  copy_rows_kernel<<<grid, warps * 32, 0, as_stream(stream)>>>(a);
  return launch_status();
}


static bool valid_ring(const qq_host_ring* r) {
  return r != nullptr && r->rows != nullptr && r->state != nullptr && r->capacity > 0;
}

extern "C" int qq_host_ring_init(const qq_host_ring* ring, void* stream) {
  if (!valid_ring(ring)) return QQ_ERR_INVALID;
  const int64_t blocks = std::min<int64_t>((ring->capacity + 255) / 256, 4096);
  ring_init_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(*ring);
  return launch_status();
}

extern "C" int qq_host_ring_alloc(const qq_host_ring* ring, int64_t n, int64_t* out, uint32_t* err, void* stream) {
  if (!valid_ring(ring) || n < 0 || (n > 0 && out == nullptr)) return QQ_ERR_INVALID;
  if (n == 0) return QQ_OK;
  ring_alloc_kernel<<<1, 1024, 0, as_stream(stream)>>>(*ring, n, out, err);
  return launch_status();
}

extern "C" int qq_host_ring_free_request(const qq_hisparse_state* hs, int req, const qq_host_ring* ring,
                                         void* stream) {
  if (!valid_hs(hs) || !valid_ring(ring) || req < 0 || req >= hs->max_reqs) return QQ_ERR_INVALID;
  ring_free_request_kernel<<<1, 1024, 0, as_stream(stream)>>>(*hs, req, *ring);
  return launch_status();
}

extern "C" int qq_hisparse_plan_step(const qq_hisparse_state* hs, const qq_batch* batch, uint8_t* skip_flags,
                                     const qq_host_ring* ring, int64_t* plan_dev, int64_t* plan_host, uint32_t* err,
                                     void* stream) {
  if (!valid_hs(hs) || !valid_ring(ring) || batch == nullptr || skip_flags == nullptr || plan_dev == nullptr ||
      plan_host == nullptr)
    return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || !batch->req_pool_indices || !batch->seq_lens) return QQ_ERR_INVALID;
  plan_step_kernel<<<1, 1024, 0, as_stream(stream)>>>(*hs, batch->req_pool_indices, batch->seq_lens, batch->bs,
                                                      skip_flags, *ring, plan_dev, plan_host, err);
  return launch_status();
}

extern "C" int qq_host_device_pointer(const void* host_ptr, void** device_ptr) {
  if (host_ptr == nullptr || device_ptr == nullptr) return QQ_ERR_INVALID;
  return cudaHostGetDevicePointer(device_ptr, const_cast<void*>(host_ptr), 0) == cudaSuccess ? QQ_OK
                                                                                             : QQ_ERR_INVALID;
}

extern "C" const char* qq_version(void) { return "qquest-b200 0.1.0 (sm_100a)"; }

extern "C" const char* qq_status_string(int status) {
  switch (status) {
    case QQ_OK:
      return "ok";
    case QQ_ERR_INVALID:
      return "invalid argument";
    case QQ_ERR_UNSUPPORTED:
      return "unsupported geometry (beyond a documented limit)";
    case QQ_ERR_CUDA:
      return "CUDA launch failed";
    case QQ_ERR_WORKSPACE:
      return "workspace missing or too small";
    default:
      return "unknown status";
  }
}
