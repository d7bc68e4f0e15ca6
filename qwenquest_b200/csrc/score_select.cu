// [Q5][Q6][Q7] Quest page scoring, top-k page selection and the position
// layout, fused into one launch per layer.
//
// Grid (page chunk, request).  Each block averages the request's GQA query
// groups into q̄ (shared memory), then every warp scores whole pages: a page's
// bounds are 4*nch bytes (2 KiB at 4 KV heads x 128 channels) read as
// coalesced 128-bit loads, lane l taking 16-byte words l, l+32, ... so that
// its q̄ values stay in registers.  The last block of a request to finish (an
// arrival counter in the workspace) selects the top pages from the fp32 scores
// (L2-resident by then) and writes the position layout, the req_to_token
// translation and actual_lens.  Scoring is HBM-bound; selection is a short
// latency-bound tail that overlaps other requests' scoring.

#include "common.cuh"

namespace qq {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPagesPerBlock = 64;

struct SelectArgs {
  qq_quest_state st;
  int layer;
  const int64_t* reqs;
  const int64_t* seq_lens;
  const void* q;
  int q_heads;
  int64_t q_stride;
  int32_t* positions;
  int32_t* actual_lens;
  float* scores;
  const int32_t* r2t;
  int64_t r2t_stride;
  int32_t* rows;
  // fused new-token K/V write
  const uint32_t* nt_k;
  const uint32_t* nt_v;
  int64_t nt_src_stride_words;
  uint32_t* nt_k_dst;
  uint32_t* nt_v_dst;
  int64_t nt_dst_stride_words;
  int nt_row_words;
  const int64_t* nt_dst_rows;
  int64_t nt_buf;
  int64_t nt_dst_num_rows;
  int32_t* counters;
  int score_all;  // page_scores API: score pages [0, num_pages) of every request, no selection
  int num_pages;
};

__device__ __forceinline__ float bound_term(uint32_t pair, float q) {
  // pair: low half = min, high half = max (bf16); where(q >= 0, max, min)
  const float b = q >= 0.f ? __uint_as_float(pair & 0xFFFF0000u) : __uint_as_float(pair << 16);
  return __fmul_rn(q, b);
}

__device__ __forceinline__ uint64_t composite(float score, uint32_t page) {
  return ((uint64_t)float_order_key(score) << 32) | (uint64_t)(0xFFFFFFFFu - page);
}

template <typename QT, int KITER>
__global__ void __launch_bounds__(kThreads) score_select_kernel(SelectArgs a) {
  __shared__ float s_qbar[QQ_MAX_CHANNELS];
  __shared__ uint64_t s_gm[64];
  __shared__ uint64_t s_T;
  __shared__ int s_M;
  __shared__ int s_last;
  extern __shared__ uint64_t s_dyn[];  // [max_pages] candidates, then [sel] selected pages

  const qq_quest_state& st = a.st;
  const int i = blockIdx.y;
  const int chunk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t req = a.reqs[i];
  const int P = st.page_size;
  const int nch = st.kv_heads * st.head_dim;
  const int64_t L = a.score_all ? 0 : a.seq_lens[i];

  int64_t F, C;
  bool is_long;
  if (a.score_all) {
    F = C = a.num_pages;
    is_long = true;
  } else {
    F = L / P;
    if (F > st.max_pages) F = st.max_pages;  // seq_len beyond max_context_len: never index past the slot
    C = st.avoid_recent_overlap ? (F > 0 ? F - 1 : 0) : F;
    is_long = L > st.top_k;
  }

  // (a) the new token's K/V into its pool row (quest_only.py:136-137, coordinator.py:226-228)
  if (a.nt_k != nullptr && chunk == 0) {
    const int64_t buf = a.nt_buf;
    const int64_t dst = a.nt_dst_rows != nullptr ? a.nt_dst_rows[i]
                                                 : req * (buf + 1) + (L - 1 < buf ? L - 1 : buf);
    for (int w = tid; dst >= 0 && dst < a.nt_dst_num_rows && w < a.nt_row_words; w += kThreads) {
      a.nt_k_dst[dst * a.nt_dst_stride_words + w] = a.nt_k[i * a.nt_src_stride_words + w];
      a.nt_v_dst[dst * a.nt_dst_stride_words + w] = a.nt_v[i * a.nt_src_stride_words + w];
    }
  }

  // (b) scores of candidate pages [p0, p1)
  const int64_t p0 = (int64_t)chunk * kPagesPerBlock;
  const int64_t p1 = min(C, p0 + kPagesPerBlock);
  float* scores = a.scores + (int64_t)i * st.max_pages;
  if (is_long && p0 < p1) {
    const QT* q = static_cast<const QT*>(a.q) + (int64_t)i * a.q_stride;
    const int G = a.q_heads / st.kv_heads;
    const int D = st.head_dim;
    for (int c = tid; c < nch; c += kThreads) {
      const int h = c / D, d = c - h * D;
      float acc = 0.f;
      for (int g = 0; g < G; ++g) acc = __fadd_rn(acc, Elem<QT>::load(q + (int64_t)(h * G + g) * D + d));
      // mean in the query dtype (quest.py:390): fp32 sum / G rounded to QT
      s_qbar[c] = G == 1 ? acc : Elem<QT>::round(__fdiv_rn(acc, (float)G));
    }
    __syncthreads();
    float qv[KITER][4];
    const int nvec = nch >> 2;
#pragma unroll
    for (int it = 0; it < KITER; ++it) {
      const int j = lane + 32 * it;
#pragma unroll
      for (int e = 0; e < 4; ++e) qv[it][e] = j < nvec ? s_qbar[4 * j + e] : 0.f;
    }
    const uint16_t* breq = st.page_bounds +
                           (((size_t)a.layer * st.max_reqs + req) * st.max_pages) * (size_t)nch * 2;
    // two pages per warp iteration: 2 * KITER independent 128-bit loads in flight per lane
    for (int64_t p = p0 + warp; p < p1; p += 2 * kWarps) {
      const int64_t pp[2] = {p, p + kWarps};
      uint4 w[2][KITER];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint4* pb = reinterpret_cast<const uint4*>(breq + (size_t)pp[u] * nch * 2);
#pragma unroll
        for (int it = 0; it < KITER; ++it) {
          const int j = lane + 32 * it;
          w[u][it] = (j < nvec && pp[u] < p1) ? ld_stream_u4(pb + j) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float acc = 0.f;
#pragma unroll
        for (int it = 0; it < KITER; ++it) {
          if (lane + 32 * it < nvec) {
            acc = __fadd_rn(acc, bound_term(w[u][it].x, qv[it][0]));
            acc = __fadd_rn(acc, bound_term(w[u][it].y, qv[it][1]));
            acc = __fadd_rn(acc, bound_term(w[u][it].z, qv[it][2]));
            acc = __fadd_rn(acc, bound_term(w[u][it].w, qv[it][3]));
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0 && pp[u] < p1) scores[pp[u]] = acc;
      }
    }
  }
  if (a.score_all) return;
  // pages that are complete but not candidates read -inf (quest.py:450-451)
  if (is_long) {
    const int64_t m0 = max(p0, C), m1 = min(F, p0 + kPagesPerBlock);
    for (int64_t p = m0 + tid; p < m1; p += kThreads) scores[p] = -__int_as_float(0x7f800000);
  }

  // (c) the last block of this request does the selection; every writer
  // fences before the arrival so that block sees all scores
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&a.counters[i], 1);
    s_last = old == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) a.counters[i] = 0;

  const int top_k = st.top_k;
  const int n = (int)(L < top_k ? L : top_k);
  if (a.actual_lens != nullptr && tid == 0) a.actual_lens[i] = n;
  int32_t* pos_out = a.positions + (int64_t)i * top_k;
  int32_t* rows_out = a.rows != nullptr ? a.rows + (int64_t)i * top_k : nullptr;
  const int32_t* r2t = a.r2t != nullptr ? a.r2t + req * a.r2t_stride : nullptr;
  const int64_t last = L > 0 ? L - 1 : 0;

  if (!is_long) {  // dense: 0 .. L-1, padded with L-1 (quest.py:339-340)
    for (int s = tid; s < top_k; s += kThreads) {
      const int32_t pos = (int32_t)(s < last ? s : last);
      pos_out[s] = pos;
      if (rows_out != nullptr && s < n) rows_out[s] = pos < a.r2t_stride ? r2t[pos] : 0;
    }
    return;
  }

  const int sel = top_k / P - 1;
  uint64_t* s_cand = s_dyn;
  int32_t* s_sel = reinterpret_cast<int32_t*>(s_dyn + st.max_pages);
  if (sel > 0) {
    // threshold: the sel-th largest of 64 group maxima bounds the sel-th largest score
    uint64_t T = 0;
    if (sel <= 64) {
      uint64_t m = 0;
      for (int64_t p = tid; p < C; p += kThreads) m = max(m, composite(__ldcg(scores + p), (uint32_t)p));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      if ((tid & 3) == 0) s_gm[tid >> 2] = m;
      __syncthreads();
      if (tid < 64) {
        const uint64_t me = s_gm[tid];
        int rank = 0;
        for (int j = 0; j < 64; ++j) {
          const uint64_t o = s_gm[j];
          rank += (o > me) || (o == me && j < tid);
        }
        if (rank == sel - 1) s_T = me;
      }
      __syncthreads();
      T = s_T;
    }
    if (tid == 0) s_M = 0;
    __syncthreads();
    for (int64_t p = tid; p < C; p += kThreads) {
      const uint64_t key = composite(__ldcg(scores + p), (uint32_t)p);
      if (key >= T) s_cand[atomicAdd(&s_M, 1)] = key;
    }
    __syncthreads();
    const int M = s_M;
    for (int c = tid; c < M; c += kThreads) {
      const uint64_t kc = s_cand[c];
      int rank = 0;
      for (int j = 0; j < M; ++j) rank += s_cand[j] > kc;
      if (rank < sel) s_sel[rank] = (int32_t)(0xFFFFFFFFu - (uint32_t)(kc & 0xFFFFFFFFu));
    }
    __syncthreads();
  }
  // layout: selected pages in score order, then the recent window (quest.py:453-459)
  const int64_t rp0 = L - P > 0 ? L - P : 0;
  const int sp = sel * P;
  for (int s = tid; s < top_k; s += kThreads) {
    int64_t pos;
    if (s < sp) {
      const int b = s / P;
      pos = (int64_t)s_sel[b] * P + (s - b * P);
    } else {
      const int64_t r = rp0 + (s - sp);
      pos = r < last ? r : last;
    }
    pos_out[s] = (int32_t)pos;
    if (rows_out != nullptr) rows_out[s] = pos < a.r2t_stride ? r2t[pos] : 0;
  }
}

template <typename QT>
__global__ void group_queries_kernel(const QT* __restrict__ q, int q_heads, int kv_heads, int D,
                                     int64_t q_stride, QT* __restrict__ out) {
  const int b = blockIdx.x;
  const int G = q_heads / kv_heads;
  const int nch = kv_heads * D;
  for (int c = threadIdx.x; c < nch; c += blockDim.x) {
    const int h = c / D, d = c - h * D;
    float acc = 0.f;
    for (int g = 0; g < G; ++g) acc = __fadd_rn(acc, Elem<QT>::load(q + b * q_stride + (int64_t)(h * G + g) * D + d));
    Elem<QT>::store(out + (int64_t)b * nch + c, G == 1 ? acc : __fdiv_rn(acc, (float)G));
  }
}

template <typename QT>
int launch_select(const SelectArgs& a, dim3 grid, size_t smem, int kiter, cudaStream_t s) {
  switch (kiter) {
    case 1:
      score_select_kernel<QT, 1><<<grid, kThreads, smem, s>>>(a);
      break;
    case 2:
      score_select_kernel<QT, 2><<<grid, kThreads, smem, s>>>(a);
      break;
    case 4:
      score_select_kernel<QT, 4><<<grid, kThreads, smem, s>>>(a);
      break;
    case 8:
      score_select_kernel<QT, 8><<<grid, kThreads, smem, s>>>(a);
      break;
    default:
      return QQ_ERR_UNSUPPORTED;
  }
  return launch_status();
}

int kiter_for(int nch) {
  const int k = (nch + 127) / 128;
  return k <= 1 ? 1 : k <= 2 ? 2 : k <= 4 ? 4 : 8;
}

bool valid_state(const qq_quest_state* st) {
  return st != nullptr && st->page_bounds && st->num_layers > 0 && st->max_reqs > 0 &&
         st->max_pages > 0 && st->kv_heads > 0 && st->head_dim > 0 && st->page_size > 0 &&
         st->kv_heads * st->head_dim <= QQ_MAX_CHANNELS && (st->kv_heads * st->head_dim) % 4 == 0;
}

size_t select_smem(const qq_quest_state* st) {
  const int sel = st->top_k / st->page_size;
  return sizeof(uint64_t) * (size_t)st->max_pages + sizeof(int32_t) * (size_t)sel;
}

template <typename QT>
int set_smem_attr(size_t smem) {
  const void* fns[4] = {(const void*)score_select_kernel<QT, 1>, (const void*)score_select_kernel<QT, 2>,
                        (const void*)score_select_kernel<QT, 4>, (const void*)score_select_kernel<QT, 8>};
  for (const void* f : fns)
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return QQ_ERR_CUDA;
  return QQ_OK;
}

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" int qq_quest_retrieve_topk(const qq_quest_state* st, int layer, const qq_batch* batch,
                                      const void* q, int q_dtype, int q_heads, int64_t q_stride,
                                      int32_t* positions, int32_t* actual_lens, float* scores,
                                      const qq_token_table* translate, int32_t* rows,
                                      const qq_new_token* nt, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (!valid_state(st) || batch == nullptr || layer < 0 || layer >= st->num_layers) return QQ_ERR_INVALID;
  if (st->top_k <= 0 || st->top_k % st->page_size != 0) return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || !batch->req_pool_indices || !batch->seq_lens)
    return QQ_ERR_INVALID;
  if (q == nullptr || positions == nullptr || scores == nullptr) return QQ_ERR_INVALID;
  if (q_heads <= 0 || q_heads % st->kv_heads != 0) return QQ_ERR_INVALID;
  if (q_dtype != QQ_BF16 && q_dtype != QQ_F32) return QQ_ERR_INVALID;
  if ((rows != nullptr) != (translate != nullptr && translate->req_to_token != nullptr))
    return QQ_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < kPartialOffset) return QQ_ERR_WORKSPACE;
  SelectArgs a{};
  a.st = *st;
  a.layer = layer;
  a.reqs = batch->req_pool_indices;
  a.seq_lens = batch->seq_lens;
  a.q = q;
  a.q_heads = q_heads;
  a.q_stride = q_stride;
  a.positions = positions;
  a.actual_lens = actual_lens;
  a.scores = scores;
  a.r2t = translate ? translate->req_to_token : nullptr;
  a.r2t_stride = translate ? translate->stride : 0;
  a.rows = rows;
  a.counters = ws_counters(workspace, kCounterSelect);
  if (nt != nullptr && nt->k != nullptr) {
    const int esz = nt->dtype == QQ_F32 ? 4 : 2;
    const int64_t row_bytes = (int64_t)st->kv_heads * st->head_dim * esz;
    if (row_bytes % 4 || (nt->src_stride * esz) % 4 || (nt->dst_row_stride * esz) % 4 || !nt->v ||
        !nt->k_dst || !nt->v_dst || nt->dst_num_rows <= 0 ||
        (nt->dst_rows == nullptr && nt->device_buffer_size <= 0))
      return QQ_ERR_INVALID;
    a.nt_k = static_cast<const uint32_t*>(nt->k);
    a.nt_v = static_cast<const uint32_t*>(nt->v);
    a.nt_src_stride_words = nt->src_stride * esz / 4;
    a.nt_k_dst = static_cast<uint32_t*>(nt->k_dst);
    a.nt_v_dst = static_cast<uint32_t*>(nt->v_dst);
    a.nt_dst_stride_words = nt->dst_row_stride * esz / 4;
    a.nt_row_words = (int)(row_bytes / 4);
    a.nt_dst_rows = nt->dst_rows;
    a.nt_buf = nt->device_buffer_size;
    a.nt_dst_num_rows = nt->dst_num_rows;
  }
  const size_t smem = select_smem(st);
  if (smem > 200 * 1024) return QQ_ERR_UNSUPPORTED;
  const int chunks = (st->max_pages + kPagesPerBlock - 1) / kPagesPerBlock;
  dim3 grid(chunks, batch->bs);
  cudaStream_t s = as_stream(stream);
  const int kiter = kiter_for(st->kv_heads * st->head_dim);
  if (q_dtype == QQ_BF16) {
    if (smem > 48 * 1024 && set_smem_attr<__nv_bfloat16>(smem) != QQ_OK) return QQ_ERR_CUDA;
    return launch_select<__nv_bfloat16>(a, grid, smem, kiter, s);
  }
  if (smem > 48 * 1024 && set_smem_attr<float>(smem) != QQ_OK) return QQ_ERR_CUDA;
  return launch_select<float>(a, grid, smem, kiter, s);
}

extern "C" int qq_quest_group_queries(const void* q, int dtype, int bs, int q_heads, int kv_heads,
                                      int head_dim, int64_t q_stride, void* out, void* stream) {
  if (q == nullptr || out == nullptr || bs < 0 || kv_heads <= 0 || head_dim <= 0 ||
      q_heads % kv_heads != 0)
    return QQ_ERR_INVALID;
  if (bs == 0) return QQ_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == QQ_BF16)
    group_queries_kernel<__nv_bfloat16><<<bs, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(q), q_heads,
                                                          kv_heads, head_dim, q_stride,
                                                          static_cast<__nv_bfloat16*>(out));
  else if (dtype == QQ_F32)
    group_queries_kernel<float><<<bs, 256, 0, s>>>(static_cast<const float*>(q), q_heads, kv_heads,
                                                  head_dim, q_stride, static_cast<float*>(out));
  else
    return QQ_ERR_INVALID;
  return launch_status();
}

extern "C" int qq_quest_page_scores(const qq_quest_state* st, int layer, const qq_batch* batch,
                                    const void* grouped_q, int q_dtype, int64_t q_stride,
                                    int num_pages, float* scores, void* stream) {
  if (!valid_state(st) || batch == nullptr || layer < 0 || layer >= st->num_layers ||
      grouped_q == nullptr || scores == nullptr || num_pages < 0 || num_pages > st->max_pages)
    return QQ_ERR_INVALID;
  if (batch->bs == 0 || num_pages == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || !batch->req_pool_indices) return QQ_ERR_INVALID;
  SelectArgs a{};
  a.st = *st;
  a.layer = layer;
  a.reqs = batch->req_pool_indices;
  a.q = grouped_q;
  a.q_heads = st->kv_heads;  // already grouped: the mean is the identity
  a.q_stride = q_stride;
  a.scores = scores;
  a.score_all = 1;
  a.num_pages = num_pages;
  dim3 grid((num_pages + kPagesPerBlock - 1) / kPagesPerBlock, batch->bs);
  const int kiter = kiter_for(st->kv_heads * st->head_dim);
  cudaStream_t s = as_stream(stream);
  if (q_dtype == QQ_BF16) return launch_select<__nv_bfloat16>(a, grid, 0, kiter, s);
  if (q_dtype == QQ_F32) return launch_select<float>(a, grid, 0, kiter, s);
  return QQ_ERR_INVALID;
}
