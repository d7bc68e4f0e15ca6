// Quest page bounds: storage init, invalidation, prefill bounds [Q2] and the
// per-step fold + finalize of the previous token's key [Q3].
//
// Bounds are bf16 (min, max) pairs per channel; one 32-bit word holds the
// pair of one channel (low half = min, high half = max), so every kernel here
// moves whole words.  All of them are HBM/latency-bound byte work.

#include "common.cuh"

namespace qq {
namespace {

constexpr uint32_t kEmptyPair = (uint32_t(kBf16MinBits) << 16) | kBf16MaxBits;

struct LayerPtrs {
  const void* k[QQ_MAX_LAYERS];
};

__global__ void fill_u32_kernel(uint32_t* dst, size_t n, uint32_t value) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) dst[i] = value;
}

__global__ void fill_u16_kernel(uint16_t* dst, size_t n, uint16_t value) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) dst[i] = value;
}

int fill_u32(uint32_t* dst, size_t n, uint32_t value, cudaStream_t s) {
  if (n == 0) return QQ_OK;
  const int threads = 256;
  const size_t blocks = std::min<size_t>((n + threads - 1) / threads, 148 * 16);
  fill_u32_kernel<<<(unsigned)blocks, threads, 0, s>>>(dst, n, value);
  return launch_status();
}

int fill_u16(uint16_t* dst, size_t n, uint16_t value, cudaStream_t s) {
  if (n == 0) return QQ_OK;
  const int threads = 256;
  const size_t blocks = std::min<size_t>((n + threads - 1) / threads, 148 * 16);
  fill_u16_kernel<<<(unsigned)blocks, threads, 0, s>>>(dst, n, value);
  return launch_status();
}

// One request slot of every layer back to the empty state (quest.py:474-479).
__global__ void invalidate_kernel(qq_quest_state st, int req) {
  const int layer = blockIdx.y;
  const size_t nch = (size_t)st.kv_heads * st.head_dim;
  uint32_t* pages = reinterpret_cast<uint32_t*>(st.page_bounds) +
                    ((size_t)layer * st.max_reqs + req) * st.max_pages * nch;
  const size_t n = (size_t)st.max_pages * nch;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    pages[i] = kEmptyPair;
  if (blockIdx.x == 0) {
    uint16_t* rmin = st.running_min + ((size_t)layer * st.max_reqs + req) * nch;
    uint16_t* rmax = st.running_max + ((size_t)layer * st.max_reqs + req) * nch;
    for (size_t c = threadIdx.x; c < nch; c += blockDim.x) {
      rmin[c] = kBf16MaxBits;
      rmax[c] = kBf16MinBits;
    }
    if (layer == 0 && threadIdx.x == 0) {
      st.running_token_count[req] = 0;
      st.running_page_idx[req] = 0;
    }
  }
}

// [Q2] bounds of one request's prefill keys (quest.py:252-280).  Block
// (page, layer); the threads stride over channels, the page's rows are
// walked in order.  Keys are loaded as fp32 and rounded to bf16 once, after
// the min/max (rounding is monotone, so this equals min/max of the rounded keys).
template <typename T>
__global__ void prefill_bounds_kernel(qq_quest_state st, LayerPtrs kp, int layer_begin,
                                      int64_t row_stride, const int32_t* __restrict__ idx, int n,
                                      int req, int write_counters) {
  extern __shared__ int32_t s_rows[];
  const int P = st.page_size;
  const int page = blockIdx.x;
  const int lo = blockIdx.y;  // index into kp
  const int layer = layer_begin + lo;
  const int full = n / P;
  const int r0 = page * P;
  const int r1 = min(n, r0 + P);
  for (int t = threadIdx.x; t < r1 - r0; t += blockDim.x) s_rows[t] = idx[r0 + t];
  __syncthreads();
  const int nch = st.kv_heads * st.head_dim;
  const T* K = static_cast<const T*>(kp.k[lo]);
  for (int c = threadIdx.x; c < nch; c += blockDim.x) {
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
    for (int t = 0; t < r1 - r0; ++t) {
      const float x = Elem<T>::load(K + (int64_t)s_rows[t] * row_stride + c);
      mn = fminf(mn, x);
      mx = fmaxf(mx, x);
    }
    const uint32_t lo16 = f32_to_bf16_bits(mn), hi16 = f32_to_bf16_bits(mx);
    if (page < full) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(st.page_bounds) +
                      (((size_t)layer * st.max_reqs + req) * st.max_pages + page) * nch;
      dst[c] = (hi16 << 16) | lo16;
    } else {
      const size_t off = ((size_t)layer * st.max_reqs + req) * nch + c;
      st.running_min[off] = (uint16_t)lo16;
      st.running_max[off] = (uint16_t)hi16;
    }
  }
  if (write_counters && page == 0 && lo == 0 && threadIdx.x == 0) {
    st.running_token_count[req] = n - full * P;
    st.running_page_idx[req] = full;
  }
}

struct StepArgs {
  qq_quest_state st;
  LayerPtrs kp;
  int flags;
  int layer_begin;
  int nlayers;
  int groups;
  int64_t row_stride;
  const int64_t* reqs;
  const int64_t* seq_lens;
  uint8_t* skip;
  const int64_t* rows;
  const int32_t* r2t;
  int64_t r2t_stride;
  int64_t r2t_rows;  // 0: not checked
  int64_t buf;
  int32_t* counters;
};

// [Q3] Block (request i, layer group g).  Every block reads the request's
// counters before doing its layers; the last block of the request (by an
// arrival counter) advances the counters and clears the skip flag, so no
// block can observe the advanced values (quest.py:304-321).
template <typename T>
__global__ void decode_step_kernel(StepArgs a) {
  wait_prior_grid();
  // The next kernel (a selection) may read the bounds before its own grid
  // wait, so this kernel lets it launch only from its end, after its writes
  // (allow_next_grid below).
  const int i = blockIdx.x;
  const int g = blockIdx.y;
  const qq_quest_state& st = a.st;
  const int64_t req = a.reqs[i];
  // a request index outside the state (or the table) is skipped: nothing of it is read or written
  if (req < 0 || req >= st.max_reqs || (a.r2t != nullptr && a.r2t_rows > 0 && req >= a.r2t_rows)) {
    allow_next_grid();
    return;
  }
  const int P = st.page_size;
  // a batch entry whose row is -1 (a HiSparse request on its first decode step) takes no part
  if (a.rows != nullptr && a.rows[i] < 0) {
    allow_next_grid();
    return;
  }
  const bool skip = a.skip != nullptr && a.skip[req] != 0;
  const int count = st.running_token_count[req];
  const int page = st.running_page_idx[req];
  const bool finalize = (a.flags & QQ_STEP_FINALIZE) != 0;
  const bool completing = finalize && count == P - 1;
  const bool fold = (a.flags & QQ_STEP_FOLD) != 0;
  const int nch = st.kv_heads * st.head_dim;

  if (!skip) {
    int64_t row = 0;
    if (fold) {
      if (a.rows != nullptr) {
        row = a.rows[i];
      } else {
        const int64_t prev = a.seq_lens[i] - 2;
        if (a.r2t != nullptr)
          row = a.r2t[req * a.r2t_stride + (prev < 0 ? 0 : prev)];
        else
          row = req * (a.buf + 1) + (prev < a.buf ? prev : a.buf);
      }
    }
    const int per = (a.nlayers + a.groups - 1) / a.groups;
    const int l0 = g * per, l1 = min(a.nlayers, l0 + per);
    for (int lo = l0; lo < l1; ++lo) {
      const int layer = a.layer_begin + lo;
      const size_t roff = ((size_t)layer * st.max_reqs + req) * nch;
      uint32_t* pdst = reinterpret_cast<uint32_t*>(st.page_bounds) +
                       (((size_t)layer * st.max_reqs + req) * st.max_pages + page) * nch;
      const T* K = fold ? static_cast<const T*>(a.kp.k[lo]) + row * a.row_stride : nullptr;
      for (int c = threadIdx.x; c < nch; c += blockDim.x) {
        uint32_t mn = st.running_min[roff + c], mx = st.running_max[roff + c];
        if (fold) {
          const uint32_t kb = f32_to_bf16_bits(Elem<T>::load(K + c));
          const float kf = bf16_bits_to_f32(kb);
          if (kf < bf16_bits_to_f32(mn)) mn = kb;
          if (kf > bf16_bits_to_f32(mx)) mx = kb;
        }
        if (completing) {
          pdst[c] = (mx << 16) | mn;
          st.running_min[roff + c] = kBf16MaxBits;
          st.running_max[roff + c] = kBf16MinBits;
        } else if (fold) {
          st.running_min[roff + c] = (uint16_t)mn;
          st.running_max[roff + c] = (uint16_t)mx;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(&a.counters[i], 1);
    if (old == a.groups - 1) {
      __threadfence();
      if (skip) {
        a.skip[req] = 0;
      } else if (finalize) {
        st.running_token_count[req] = (count + 1) % P;
        if (completing) st.running_page_idx[req] = page + 1;
      }
      if (a.skip != nullptr && !skip) a.skip[req] = 0;
      a.counters[i] = 0;
    }
  }
  __threadfence();
  allow_next_grid();
}

bool valid_state(const qq_quest_state* st) {
  return st != nullptr && st->page_bounds && st->running_min && st->running_max &&
         st->running_token_count && st->running_page_idx && st->num_layers > 0 &&
         st->num_layers <= QQ_MAX_LAYERS && st->max_reqs > 0 && st->max_pages > 0 &&
         st->kv_heads > 0 && st->head_dim > 0 && st->page_size > 0 &&
         st->kv_heads * st->head_dim <= QQ_MAX_CHANNELS;
}

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" int qq_quest_init_storage(const qq_quest_state* st, void* stream) {
  if (!valid_state(st)) return QQ_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  const size_t nch = (size_t)st->kv_heads * st->head_dim;
  const size_t pages = (size_t)st->num_layers * st->max_reqs * st->max_pages * nch;
  const size_t run = (size_t)st->num_layers * st->max_reqs * nch;
  int rc = fill_u32(reinterpret_cast<uint32_t*>(st->page_bounds), pages, kEmptyPair, s);
  if (rc == QQ_OK) rc = fill_u16(st->running_min, run, kBf16MaxBits, s);
  if (rc == QQ_OK) rc = fill_u16(st->running_max, run, kBf16MinBits, s);
  if (rc == QQ_OK) rc = fill_u32(reinterpret_cast<uint32_t*>(st->running_token_count), st->max_reqs, 0, s);
  if (rc == QQ_OK) rc = fill_u32(reinterpret_cast<uint32_t*>(st->running_page_idx), st->max_reqs, 0, s);
  return rc;
}

extern "C" int qq_quest_invalidate(const qq_quest_state* st, int req, void* stream) {
  if (!valid_state(st) || req < 0 || req >= st->max_reqs) return QQ_ERR_INVALID;
  const size_t n = (size_t)st->max_pages * st->kv_heads * st->head_dim;
  const unsigned bx = (unsigned)std::min<size_t>((n + 255) / 256, 64);
  invalidate_kernel<<<dim3(bx, st->num_layers), 256, 0, as_stream(stream)>>>(*st, req);
  return launch_status();
}

extern "C" int qq_quest_bounds_prefill(const qq_quest_state* st, int layer_begin, int layer_end,
                                       const void* const* k_layers, int kv_dtype,
                                       int64_t k_row_stride, const int32_t* prefill_indices,
                                       int prefill_len, int req, int write_counters, void* stream) {
  if (!valid_state(st) || k_layers == nullptr || layer_begin < 0 || layer_end > st->num_layers ||
      layer_end <= layer_begin || req < 0 || req >= st->max_reqs || prefill_len < 0)
    return QQ_ERR_INVALID;
  if (kv_dtype != QQ_BF16 && kv_dtype != QQ_F32) return QQ_ERR_INVALID;
  if (prefill_len == 0) return QQ_OK;
  if (prefill_indices == nullptr) return QQ_ERR_INVALID;
  const int P = st->page_size;
  const int full = prefill_len / P;
  if (full > st->max_pages) return QQ_ERR_INVALID;
  const int blocks_x = full + (prefill_len % P ? 1 : 0);
  LayerPtrs kp{};
  for (int l = 0; l < layer_end - layer_begin; ++l) kp.k[l] = k_layers[l];
  const size_t smem = sizeof(int32_t) * (size_t)P;
  if (smem > 48 * 1024) return QQ_ERR_UNSUPPORTED;
  dim3 grid(blocks_x, layer_end - layer_begin);
  cudaStream_t s = as_stream(stream);
  if (kv_dtype == QQ_BF16)
    prefill_bounds_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(
        *st, kp, layer_begin, k_row_stride, prefill_indices, prefill_len, req, write_counters);
  else
    prefill_bounds_kernel<float><<<grid, 256, smem, s>>>(*st, kp, layer_begin, k_row_stride,
                                                         prefill_indices, prefill_len, req,
                                                         write_counters);
  return launch_status();
}

extern "C" int qq_quest_decode_step(const qq_quest_state* st, int flags, int layer_begin,
                                    int layer_end, const void* const* k_layers, int kv_dtype,
                                    int64_t k_row_stride, const qq_batch* batch, uint8_t* skip_flags,
                                    const int64_t* rows, const qq_token_table* table,
                                    int64_t device_buffer_size, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!valid_state(st) || batch == nullptr || layer_begin < 0 || layer_end > st->num_layers ||
      layer_end <= layer_begin || (flags & ~(QQ_STEP_FOLD | QQ_STEP_FINALIZE)) != 0)
    return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || batch->req_pool_indices == nullptr)
    return QQ_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < kPartialOffset) return QQ_ERR_WORKSPACE;
  const bool fold = (flags & QQ_STEP_FOLD) != 0;
  if (fold) {
    if (k_layers == nullptr || (kv_dtype != QQ_BF16 && kv_dtype != QQ_F32)) return QQ_ERR_INVALID;
    if (rows == nullptr && batch->seq_lens == nullptr) return QQ_ERR_INVALID;
    if (rows == nullptr && table == nullptr && device_buffer_size <= 0) return QQ_ERR_INVALID;
  }
  StepArgs a{};
  a.st = *st;
  a.flags = flags;
  a.layer_begin = layer_begin;
  a.nlayers = layer_end - layer_begin;
  a.groups = a.nlayers;  // one block per (request, layer): every load of the step in flight at once
  a.row_stride = k_row_stride;
  if (fold)
    for (int l = 0; l < a.nlayers; ++l) a.kp.k[l] = k_layers[l];
  a.reqs = batch->req_pool_indices;
  a.seq_lens = batch->seq_lens;
  a.skip = skip_flags;
  a.rows = rows;
  a.r2t = table ? table->req_to_token : nullptr;
  a.r2t_stride = table ? table->stride : 0;
  a.r2t_rows = table ? table->rows : 0;
  a.buf = device_buffer_size;
  a.counters = ws_counters(workspace, kCounterStep);
  dim3 grid(batch->bs, a.groups);
  cudaStream_t s = as_stream(stream);
  if (kv_dtype == QQ_F32) return launch_pdl(decode_step_kernel<float>, grid, dim3(128), 0, s, a);
  return launch_pdl(decode_step_kernel<__nv_bfloat16>, grid, dim3(128), 0, s, a);
}
