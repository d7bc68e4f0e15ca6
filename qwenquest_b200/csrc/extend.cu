// One layer of a prefill (extend) batch in one launch [Q2][H1]: the new
// tokens' K/V rows are written to the token pool (set_kv_buffer,
// memory.py:114-120), this layer's Quest page bounds of positions
// [0, seq_len) are built from the same registers (quest.py:231-280, which
// the reference runs after the last layer and which re-reads every key from
// the pool), and in Mode 3 positions [0, device_buffer_size) are copied into
// the request's hot-buffer slots (coordinator.py:154-162).  Keys and values
// of positions below a request's cached prefix are read from the pool
// through req_to_token.
//
// Block (page, request, row chunk), 256 threads: the threads of a row group
// cover 16-64 of a row's 16-byte words (4-byte words when the rows or pointers
// are not 16-byte aligned) and the 4-16 row groups walk the page's positions; each
// thread keeps the min / max of its channels (bf16 pairs packed, fp32 as
// is), the row groups are folded in shared memory and fp32 is rounded to bf16
// once (rounding is monotone).  Loads
// of four positions are issued before their stores.  HBM-bound byte work:
// per new token and layer 2 x row bytes read and written (+ 2 x row bytes
// into the hot buffer in Mode 3), per page 2 x channels x 2 bytes of bounds.

#include "common.cuh"

namespace qq {
namespace {

constexpr int kExtendThreads = 256;
constexpr int kExtendUnroll = 4;
// Words of a row one block covers: at most 64 (a whole 1 KiB bf16 row), halved
// (down to 16) while the launch would give fewer than 4 blocks per SM — 4 is
// the residency at this kernel's register count.  Measured on a 32K-token
// layer: 64 or 32 words per block 1.376 / 1.379 ms per 48 layers, 16 words
// 1.475, 8 words 1.77 (more, smaller blocks add per-block latency).
constexpr int kExtendMaxWordsPerBlock = 64;
constexpr int kExtendMinWordsPerBlock = 16;
constexpr int kExtendBlocksPerSm = 4;

int extend_sm_count() { return device_sm_count(); }

struct ExtendArgs {
  qq_quest_state st;
  int bounds;  // build this layer's bounds into st
  int layer;   // index into st
  int write_counters;
  int page_size;
  const int64_t* reqs;
  const int64_t* seq_lens;
  const int64_t* prefix_lens;
  const int64_t* offsets;
  const int64_t* out_loc;
  int64_t num_tokens;
  const int32_t* r2t;
  int64_t r2t_stride;
  int64_t r2t_rows;  // 0: not checked
  const char* k_src;
  const char* v_src;
  int64_t src_stride;  // bytes between new tokens
  char* k_pool;
  char* v_pool;
  int64_t pool_stride;  // bytes between pool rows
  int64_t pool_rows;
  char* hot_k;  // nullptr outside Mode 3
  char* hot_v;
  int64_t hot_stride;
  int64_t hot_buf;  // device_buffer_size
  int64_t hot_rows;
  int words;       // vector words per row
  int wpb;         // words per block (one row chunk)
  int row_groups;  // kExtendThreads / wpb
  uint32_t* err;
};

template <int VB>
struct VecOf;
template <>
struct VecOf<16> {
  using type = uint4;
};
template <>
struct VecOf<4> {
  using type = uint32_t;
};

// 32-bit word j of a vector word.
template <int VB>
__device__ __forceinline__ uint32_t word32(const typename VecOf<VB>::type& v, int j) {
  if constexpr (VB == 16)
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
  else
    return v;
}

// Running min / max of one 32-bit word: two bf16 channels (packed, exact for
// bf16 inputs) or one fp32 channel.  A NaN operand yields the other operand.
template <typename T>
__device__ __forceinline__ uint32_t word_min(uint32_t a, uint32_t b) {
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat162 r = __hmin2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                     *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    return __float_as_uint(fminf(__uint_as_float(a), __uint_as_float(b)));
  }
}
template <typename T>
__device__ __forceinline__ uint32_t word_max(uint32_t a, uint32_t b) {
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                     *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    return __float_as_uint(fmaxf(__uint_as_float(a), __uint_as_float(b)));
  }
}

// bf16 bits of channel e of the accumulated words (fp32 rounded to nearest even).
template <typename T, int NW>
__device__ __forceinline__ uint16_t channel_bits(const uint32_t (&w)[NW], int e) {
  if constexpr (sizeof(T) == 2)
    return (uint16_t)((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu));
  else
    return f32_to_bf16_bits(__uint_as_float(w[e]));
}

template <typename T, int VB>
__global__ void __launch_bounds__(kExtendThreads, kExtendBlocksPerSm) extend_kv_kernel(ExtendArgs a) {
  using Vec = typename VecOf<VB>::type;
  constexpr int NW = VB / 4;                        // 32-bit words per vector word
  constexpr int CH = VB / (int)sizeof(T);           // channels per vector word
  constexpr uint32_t kPosInf = sizeof(T) == 2 ? 0x7f807f80u : 0x7f800000u;
  constexpr uint32_t kNegInf = sizeof(T) == 2 ? 0xff80ff80u : 0xff800000u;
  __shared__ uint32_t s_min[kExtendThreads * NW], s_max[kExtendThreads * NW];

  const int i = blockIdx.y;
  const int page = blockIdx.x;
  const int P = a.page_size;
  // the request's four words are loaded together
  const int64_t seq = a.seq_lens[i];
  const int64_t prefix = a.prefix_lens[i];
  const int64_t req = a.reqs[i];
  const int64_t off = a.offsets[i];
  const int64_t p0 = (int64_t)page * P;
  // a request index outside the table (or the Quest state) is reported once and its request skipped
  if (req < 0 || (a.r2t_rows > 0 && req >= a.r2t_rows) || (a.bounds && req >= a.st.max_reqs)) {
    if (page == 0 && blockIdx.z == 0 && threadIdx.x == 0) raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    return;
  }
  if (p0 >= seq) return;
  const int64_t p1 = seq < p0 + P ? seq : p0 + P;
  const bool hot_page = a.hot_k != nullptr && p0 < a.hot_buf;
  // a page wholly inside the cached prefix only feeds the bounds and the hot buffer
  if (p1 <= prefix && !a.bounds && !hot_page) return;

  const int tid = threadIdx.x;
  const int rg = tid / a.wpb;
  const int w = blockIdx.z * a.wpb + (tid - rg * a.wpb);
  const bool active = rg < a.row_groups && w < a.words;
  const int64_t wbytes = (int64_t)w * VB;

  uint32_t mn[NW], mx[NW];
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    mn[j] = kPosInf;
    mx[j] = kNegInf;
  }

  if (active) {
    const int64_t stride = (int64_t)a.row_groups;
    for (int64_t base = p0 + rg; base < p1; base += kExtendUnroll * stride) {
      Vec kv[kExtendUnroll], vv[kExtendUnroll];
      int32_t pool_dst[kExtendUnroll], hot_dst[kExtendUnroll];  // rows < 2^31 (checked on the host)
      bool ok[kExtendUnroll];
#pragma unroll
      for (int u = 0; u < kExtendUnroll; ++u) {
        const int64_t pos = base + u * stride;
        ok[u] = pos < p1;
        pool_dst[u] = -1;
        hot_dst[u] = -1;
        if (!ok[u]) continue;
        const char* ks;
        const char* vs;
        if (pos >= prefix) {
          const int64_t j = off + (pos - prefix);
          if (j < 0 || j >= a.num_tokens) {
            raise_error(a.err, QQ_DEV_ERR_BOUNDS);
            ok[u] = false;
            continue;
          }
          ks = a.k_src + j * a.src_stride + wbytes;
          vs = a.v_src + j * a.src_stride + wbytes;
          const int64_t dst = a.out_loc[j];
          if (dst >= 0 && dst < a.pool_rows)
            pool_dst[u] = (int32_t)dst;
          else
            raise_error(a.err, QQ_DEV_ERR_BOUNDS);
        } else {
          const int64_t row = a.r2t[req * a.r2t_stride + pos];
          if (row < 0 || row >= a.pool_rows) {
            raise_error(a.err, QQ_DEV_ERR_BOUNDS);
            ok[u] = false;
            continue;
          }
          ks = a.k_pool + row * a.pool_stride + wbytes;
          vs = a.v_pool + row * a.pool_stride + wbytes;
        }
        if (a.hot_k != nullptr && pos < a.hot_buf) {
          const int64_t h = req * (a.hot_buf + 1) + pos;
          if (h < a.hot_rows)
            hot_dst[u] = (int32_t)h;
          else
            raise_error(a.err, QQ_DEV_ERR_BOUNDS);
        }
        kv[u] = *reinterpret_cast<const Vec*>(ks);
        if (pool_dst[u] >= 0 || hot_dst[u] >= 0) vv[u] = *reinterpret_cast<const Vec*>(vs);
      }
#pragma unroll
      for (int u = 0; u < kExtendUnroll; ++u) {
        if (!ok[u]) continue;
        if (pool_dst[u] >= 0) {
          *reinterpret_cast<Vec*>(a.k_pool + (int64_t)pool_dst[u] * a.pool_stride + wbytes) = kv[u];
          *reinterpret_cast<Vec*>(a.v_pool + (int64_t)pool_dst[u] * a.pool_stride + wbytes) = vv[u];
        }
        if (hot_dst[u] >= 0) {
          *reinterpret_cast<Vec*>(a.hot_k + (int64_t)hot_dst[u] * a.hot_stride + wbytes) = kv[u];
          *reinterpret_cast<Vec*>(a.hot_v + (int64_t)hot_dst[u] * a.hot_stride + wbytes) = vv[u];
        }
        if (a.bounds) {
#pragma unroll
          for (int j = 0; j < NW; ++j) {
            mn[j] = word_min<T>(mn[j], word32<VB>(kv[u], j));
            mx[j] = word_max<T>(mx[j], word32<VB>(kv[u], j));
          }
        }
      }
    }
  }
  if (!a.bounds) return;

  const qq_quest_state& st = a.st;
  if (a.write_counters && page == 0 && blockIdx.z == 0 && tid == 0) {
    if (req >= 0 && req < st.max_reqs) {
      st.running_token_count[req] = (int32_t)(seq % P);
      st.running_page_idx[req] = (int32_t)(seq / P);
    } else {
      raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    }
  }
  if (a.row_groups > 1) {
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      s_min[tid * NW + j] = mn[j];
      s_max[tid * NW + j] = mx[j];
    }
    __syncthreads();
    if (rg == 0 && active) {
      for (int r = 1; r < a.row_groups; ++r) {
        const int t = r * a.wpb + tid;
#pragma unroll
        for (int j = 0; j < NW; ++j) {
          mn[j] = word_min<T>(mn[j], s_min[t * NW + j]);
          mx[j] = word_max<T>(mx[j], s_max[t * NW + j]);
        }
      }
    }
  }
  if (rg != 0 || !active) return;
  if (req < 0 || req >= st.max_reqs) return;  // reported with the counters or by block 0
  const int nch = st.kv_heads * st.head_dim;
  const int64_t c0 = (int64_t)w * CH;
  if (p1 - p0 == P) {
    if (page >= st.max_pages) {
      raise_error(a.err, QQ_DEV_ERR_BOUNDS);
      return;
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(st.page_bounds) +
                    (((size_t)a.layer * st.max_reqs + req) * st.max_pages + page) * nch + c0;
#pragma unroll
    for (int e = 0; e < CH; ++e)
      dst[e] = (uint32_t(channel_bits<T>(mx, e)) << 16) | channel_bits<T>(mn, e);
  } else {
    const size_t roff = ((size_t)a.layer * st.max_reqs + req) * nch + c0;
#pragma unroll
    for (int e = 0; e < CH; ++e) {
      st.running_min[roff + e] = channel_bits<T>(mn, e);
      st.running_max[roff + e] = channel_bits<T>(mx, e);
    }
  }
}

bool quest_state_ok(const qq_quest_state* st) {
  return st->page_bounds && st->running_min && st->running_max && st->running_token_count &&
         st->running_page_idx && st->num_layers > 0 && st->max_reqs > 0 && st->max_pages > 0 &&
         st->kv_heads > 0 && st->head_dim > 0 && st->page_size > 0 &&
         st->kv_heads * st->head_dim <= QQ_MAX_CHANNELS;
}

bool aligned(const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

template <typename T, int VB>
int launch_extend(const ExtendArgs& a, dim3 grid, cudaStream_t s) {
  extend_kv_kernel<T, VB><<<grid, kExtendThreads, 0, s>>>(a);
  return launch_status();
}

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" int qq_quest_extend_kv(const qq_quest_state* st, int layer, int write_counters,
                                  const qq_extend_batch* eb, const qq_token_table* table, const void* k,
                                  const void* v, int dtype, int64_t row_elems, int64_t src_stride,
                                  void* k_pool, void* v_pool, int64_t pool_row_stride, int64_t pool_rows,
                                  const qq_hot_buffer* hot, uint32_t* err, void* stream) {
  if (eb == nullptr || eb->bs < 0 || eb->bs > QQ_MAX_BS || eb->max_seq_len < 0 || eb->num_tokens < 0)
    return QQ_ERR_INVALID;
  if (eb->bs == 0 || eb->max_seq_len == 0) return QQ_OK;
  if (!eb->req_pool_indices || !eb->seq_lens || !eb->prefix_lens || !eb->token_offsets || !eb->out_cache_loc)
    return QQ_ERR_INVALID;
  if (table == nullptr || table->req_to_token == nullptr || table->stride < eb->max_seq_len)
    return QQ_ERR_INVALID;
  if (dtype != QQ_BF16 && dtype != QQ_F32) return QQ_ERR_INVALID;
  if (!k || !v || !k_pool || !v_pool || row_elems <= 0 || row_elems > QQ_MAX_CHANNELS ||
      src_stride < row_elems || pool_row_stride < row_elems || pool_rows <= 0 || pool_rows > INT32_MAX)
    return QQ_ERR_INVALID;
  int page_size = 64;
  if (st != nullptr) {
    if (!quest_state_ok(st) || layer < 0 || layer >= st->num_layers ||
        (int64_t)st->kv_heads * st->head_dim != row_elems)
      return QQ_ERR_INVALID;
    if (eb->max_seq_len / st->page_size > st->max_pages) return QQ_ERR_INVALID;
    page_size = st->page_size;
  }
  if (hot != nullptr && (!hot->k || !hot->v || hot->device_buffer_size <= 0 || hot->num_rows <= 0 ||
                         hot->num_rows > INT32_MAX || hot->row_stride < row_elems))
    return QQ_ERR_INVALID;

  const int esize = dtype == QQ_BF16 ? 2 : 4;
  const int64_t row_bytes = row_elems * esize;
  auto fits = [&](int n) {
    bool ok = row_bytes % n == 0 && (src_stride * esize) % n == 0 && (pool_row_stride * esize) % n == 0 &&
              aligned(k, n) && aligned(v, n) && aligned(k_pool, n) && aligned(v_pool, n);
    if (hot != nullptr) ok = ok && (hot->row_stride * esize) % n == 0 && aligned(hot->k, n) && aligned(hot->v, n);
    return ok;
  };
  const int vb = fits(16) ? 16 : fits(4) ? 4 : 0;
  if (vb == 0) return QQ_ERR_UNSUPPORTED;

  ExtendArgs a{};
  if (st != nullptr) a.st = *st;
  a.bounds = st != nullptr;
  a.layer = layer;
  a.write_counters = st != nullptr && write_counters != 0;
  a.page_size = page_size;
  a.reqs = eb->req_pool_indices;
  a.seq_lens = eb->seq_lens;
  a.prefix_lens = eb->prefix_lens;
  a.offsets = eb->token_offsets;
  a.out_loc = eb->out_cache_loc;
  a.num_tokens = eb->num_tokens;
  a.r2t = table->req_to_token;
  a.r2t_stride = table->stride;
  a.r2t_rows = table->rows;
  a.k_src = static_cast<const char*>(k);
  a.v_src = static_cast<const char*>(v);
  a.src_stride = src_stride * esize;
  a.k_pool = static_cast<char*>(k_pool);
  a.v_pool = static_cast<char*>(v_pool);
  a.pool_stride = pool_row_stride * esize;
  a.pool_rows = pool_rows;
  if (hot != nullptr) {
    a.hot_k = static_cast<char*>(hot->k);
    a.hot_v = static_cast<char*>(hot->v);
    a.hot_stride = hot->row_stride * esize;
    a.hot_buf = hot->device_buffer_size;
    a.hot_rows = hot->num_rows;
  }
  a.words = (int)(row_bytes / vb);
  const unsigned pages = (unsigned)((eb->max_seq_len + page_size - 1) / page_size);
  int wpb = a.words < kExtendMaxWordsPerBlock ? a.words : kExtendMaxWordsPerBlock;
  const int64_t want = (int64_t)extend_sm_count() * kExtendBlocksPerSm;
  while (wpb > kExtendMinWordsPerBlock && wpb % 2 == 0 &&
         (int64_t)pages * eb->bs * ((a.words + wpb - 1) / wpb) < want)
    wpb /= 2;
  a.wpb = wpb;
  a.row_groups = kExtendThreads / a.wpb;
  a.err = err;
  const unsigned chunks = (unsigned)((a.words + a.wpb - 1) / a.wpb);
  dim3 grid(pages, (unsigned)eb->bs, chunks);
  cudaStream_t s = as_stream(stream);
  if (dtype == QQ_BF16)
    return vb == 16 ? launch_extend<__nv_bfloat16, 16>(a, grid, s) : launch_extend<__nv_bfloat16, 4>(a, grid, s);
  return vb == 16 ? launch_extend<float, 16>(a, grid, s) : launch_extend<float, 4>(a, grid, s);
}
