// [Q7] Split-K sparse decode attention over an explicit row list.
//
// Fast path (bf16, 4 KV heads, head_dim 128, 8 query heads per KV head),
// two launches:
//
// 1. attn_stream_kernel — one 256-thread block per SM, and every warp is an
//    independent pipeline.  Work unit = (request, KV head, chunk of 64 rows
//    of the request's row list); units go round-robin to the warps of the
//    grid, so the four warps of a block that share a chunk read the four
//    256-byte head slices of the same rows.  A warp gathers only its own
//    head's K and V slices: per 16-row stage each lane issues 16 16-byte
//    cp.async.cg copies (one instruction = 256 B of K + 256 B of V of a row),
//    into a private 3-slot ring at a 272-byte row pitch (ldmatrix reads are
//    bank-conflict free), with an L2 evict-first policy (every K/V byte is
//    read once).  Waits are per warp (cp.async.wait_group + __syncwarp): no
//    block barrier, atomic or fence in the streaming loop, so one warp's slow
//    request never stalls the others.  Per stage:
//      S^T[16 rows x 8 heads] = K[16 x 128] . Q^T[128 x 8]   (8 x mma m16n8k16)
//      online softmax in fp32 (exp2 domain), P^T via movmatrix.trans
//      O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8]          (P as bf16 hi + lo: 16 mma)
//    At the end of a unit the warp writes its fp32 partial (m, l, O) to the
//    workspace.
// 2. attn_merge_kernel — block (request, KV head) combines the partials of
//    the request's chunks into the bf16 output.
//
// Generic path (any head_dim / group / fp32): one block per (request, KV
// head), scores in shared memory, two-pass softmax, fp32 FMA.

#include <cfloat>

#include "common.cuh"

namespace qq {
namespace {

// ------------------------------------------------------------------ fast path constants
constexpr int kD = 128;
constexpr int kKV = 4;
constexpr int kG = 8;
constexpr int kH = kKV * kG;
constexpr int kSlice = kD * 2;          // 256 bytes: one KV head of one row
constexpr int kPitch = kSlice + 16;     // 272
constexpr int kToks = 16;               // rows per stage (the MMA's M)
constexpr int kSlots = 3;               // stages in a warp's ring
constexpr int kUnitRows = kAttnChunk;   // 64 rows per work unit
constexpr int kWarpsFast = 8;
constexpr int kThreadsFast = kWarpsFast * 32;
constexpr int kSlotBytes = 2 * kToks * kPitch;  // K slice tile + V slice tile: 8704
constexpr int kWarpSmem = kSlots * kSlotBytes;  // 26112
constexpr size_t kSmemFast = (size_t)kWarpsFast * kWarpSmem;  // 208896
constexpr int kMaxChunksFast = 64;      // top_k <= 4096 on the fast path
constexpr int kMergeThreads = 256;

struct AttnArgs {
  const int64_t* seq_lens;
  int bs;
  int top_k;
  int max_chunks;  // 64-row chunks per request at top_k
  const void* q;
  int64_t q_stride;
  const int32_t* rows;
  const char* k_pool;
  const char* v_pool;
  int64_t row_stride_bytes;
  int64_t num_rows;
  float scale_log2;  // scaling * log2(e)
  float scaling;
  void* out;
  int64_t out_stride;
  uint32_t* err;
  float* part_o;   // [bs][max_chunks][kKV][kG][kD]
  float* part_ml;  // [bs][max_chunks][kKV][kG][2]
  int32_t* counters;
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t l = f32_to_bf16_bits(lo), h = f32_to_bf16_bits(hi);
  return (h << 16) | l;
}

// Packs bf16(lo), bf16(hi) and returns the rounded values as floats.
__device__ __forceinline__ uint32_t pack_bf16x2_split(float lo, float hi, float& lo_r, float& hi_r) {
  const uint32_t l = f32_to_bf16_bits(lo), h = f32_to_bf16_bits(hi);
  lo_r = bf16_bits_to_f32(l);
  hi_r = bf16_bits_to_f32(h);
  return (h << 16) | l;
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 16-byte async copy global -> shared with an L2 cache policy; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src, uint32_t src_bytes,
                                            uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src), "r"(src_bytes), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

#define kNegInf (-__int_as_float(0x7f800000))

// A position in a warp's stream of stages: stage `sub` of work unit `unit`.
struct Cursor {
  int unit;  // -1 before the first stage, >= total when exhausted
  int sub;
  int cnt;   // rows of the unit
  int req;   // batch index
  int head;  // KV head
  int chunk; // 64-row chunk of the request's row list
};

// Advance to the next stage of the warp's stream (units W, W + NW, ...).
__device__ __forceinline__ bool next_stage(const AttnArgs& a, Cursor& c, int W, int NW, int total_units) {
  if (c.unit >= 0 && c.unit < total_units && (c.sub + 1) * kToks < c.cnt) {
    ++c.sub;
    return true;
  }
  for (int u = c.unit < 0 ? W : c.unit + NW; u < total_units; u += NW) {
    const int head = u & (kKV - 1);
    const int rest = u >> 2;
    const int req = rest / a.max_chunks;
    const int chunk = rest - req * a.max_chunks;
    const int64_t L = __ldg(a.seq_lens + req);
    const int n = (int)(L < a.top_k ? L : a.top_k);
    const int cnt = min(kUnitRows, n - chunk * kUnitRows);
    if (cnt > 0) {
      c.unit = u;
      c.sub = 0;
      c.cnt = cnt;
      c.req = req;
      c.head = head;
      c.chunk = chunk;
      return true;
    }
  }
  c.unit = total_units;
  return false;
}

// Lane l's pool row for row l of stage `c` (lanes >= 16 and rows past the end: 0).
__device__ __forceinline__ int32_t load_stage_row(const AttnArgs& a, const Cursor& c, int lane) {
  const int ntok = min(kToks, c.cnt - c.sub * kToks);
  return lane < ntok
             ? __ldg(a.rows + (int64_t)c.req * a.top_k + c.chunk * kUnitRows + c.sub * kToks + lane)
             : 0;
}

// Gather the head slices of the stage's 16 K and V rows into `slot`: per row
// one warp instruction, lanes 0-15 K bytes [16 l, 16 l + 16), lanes 16-31 V.
__device__ __forceinline__ void issue_stage(const AttnArgs& a, const Cursor& c, int32_t row_l, char* slot, int lane,
                                            uint64_t policy) {
  const int ntok = min(kToks, c.cnt - c.sub * kToks);
  int64_t my_row = row_l;
  if (lane < ntok && (my_row < 0 || my_row >= a.num_rows)) {
    raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    my_row = 0;
  }
  const bool is_v = lane >= 16;
  const int off = (lane & 15) * 16;
  const char* src0 = (is_v ? a.v_pool : a.k_pool) + c.head * kSlice + off;
  char* dst0 = slot + (is_v ? kToks * kPitch : 0) + off;
#pragma unroll
  for (int k = 0; k < kToks; ++k) {
    const int64_t row = __shfl_sync(0xffffffffu, my_row, k);
    cp_async_16(dst0 + k * kPitch, src0 + row * a.row_stride_bytes, k < ntok ? 16u : 0u, policy);
  }
}

__global__ void __launch_bounds__(kThreadsFast, 1) attn_stream_kernel(AttnArgs a) {
  extern __shared__ __align__(128) char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  char* ring = smem + (size_t)warp * kWarpSmem;
  const int W = blockIdx.x * kWarpsFast + warp;
  const int NW = gridDim.x * kWarpsFast;
  const int total_units = a.bs * a.max_chunks * kKV;
  const uint64_t policy = evict_first_policy();
  const __nv_bfloat16* qbase = static_cast<const __nv_bfloat16*>(a.q);

  // prologue: kSlots - 1 stages in flight; row indices always one stage ahead
  Cursor fc{-1, 0, 0, 0, 0, 0}, cc{-1, 0, 0, 0, 0, 0};
  bool have_f = next_stage(a, fc, W, NW, total_units);
  int32_t row_f = have_f ? load_stage_row(a, fc, lane) : 0;
#pragma unroll
  for (int s = 0; s < kSlots - 1; ++s) {
    if (have_f) {
      issue_stage(a, fc, row_f, ring + s * kSlotBytes, lane, policy);
      have_f = next_stage(a, fc, W, NW, total_units);
      if (have_f) row_f = load_stage_row(a, fc, lane);
    }
    cp_async_commit();
  }

  uint32_t qb[8][2];
  float acc[8][4];
  float m_a = kNegInf, m_b = kNegInf, l_a = 0.f, l_b = 0.f;
  int g = 0;
  while (next_stage(a, cc, W, NW, total_units)) {
    if (cc.sub == 0) {
      // Q^T fragments of this KV head: B[k = d][n = query head]; loaded before
      // the wait so their latency hides behind it
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbase + (int64_t)cc.req * a.q_stride +
                                                               (int64_t)(cc.head * kG + gid) * kD);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[kk][0] = __ldg(qrow + (kk * 16 + 2 * tig) / 2);
        qb[kk][1] = __ldg(qrow + (kk * 16 + 8 + 2 * tig) / 2);
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
      m_a = m_b = kNegInf;
      l_a = l_b = 0.f;
    }
    cp_async_wait<kSlots - 2>();
    __syncwarp();  // stage g visible to every lane; slot of stage g - 1 free
    if (have_f) {
      issue_stage(a, fc, row_f, ring + ((g + kSlots - 1) % kSlots) * kSlotBytes, lane, policy);
      have_f = next_stage(a, fc, W, NW, total_units);
      if (have_f) row_f = load_stage_row(a, fc, lane);
    }
    cp_async_commit();

    const int ntok = min(kToks, cc.cnt - cc.sub * kToks);
    const char* sk = ring + (g % kSlots) * kSlotBytes;
    const char* sv = sk + kToks * kPitch;
    // ---- S^T = K . Q^T
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kaddr = smem_u32(sk + (lane & 15) * kPitch + (lane >> 4) * 16);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, kaddr + kk * 32);
      mma_bf16_16816(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
    }
    // ---- online softmax (exp2 domain); rows >= ntok are masked
    const bool v0 = gid < ntok, v1 = gid + 8 < ntok;
    const float s00 = v0 ? c[0] * a.scale_log2 : kNegInf;  // row gid, head 2tig
    const float s01 = v0 ? c[1] * a.scale_log2 : kNegInf;  // row gid, head 2tig+1
    const float s10 = v1 ? c[2] * a.scale_log2 : kNegInf;  // row gid+8, head 2tig
    const float s11 = v1 ? c[3] * a.scale_log2 : kNegInf;  // row gid+8, head 2tig+1
    float mx_a = fmaxf(s00, s10), mx_b = fmaxf(s01, s11);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = mn_a == kNegInf ? 1.f : fast_exp2(m_a - mn_a);
    const float al_b = mn_b == kNegInf ? 1.f : fast_exp2(m_b - mn_b);
    const float p00 = mn_a == kNegInf ? 0.f : fast_exp2(s00 - mn_a);
    const float p10 = mn_a == kNegInf ? 0.f : fast_exp2(s10 - mn_a);
    const float p01 = mn_b == kNegInf ? 0.f : fast_exp2(s01 - mn_b);
    const float p11 = mn_b == kNegInf ? 0.f : fast_exp2(s11 - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a = l_a * al_a + p00 + p10;
    l_b = l_b * al_b + p01 + p11;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      acc[mt][0] *= al_a;
      acc[mt][1] *= al_b;
      acc[mt][2] *= al_a;
      acc[mt][3] *= al_b;
    }
    // ---- P^T fragments (rows x heads -> heads x rows) and O^T += V^T . P^T,
    // P split into bf16 hi + lo parts (two MMAs per tile): the weights carry
    // ~16 mantissa bits and the fp32 result tracks an fp32 softmax-weighted sum
    float h00, h01, h10, h11;
    const uint32_t pb0 = movmatrix_trans(pack_bf16x2_split(p00, p01, h00, h01));
    const uint32_t pb1 = movmatrix_trans(pack_bf16x2_split(p10, p11, h10, h11));
    const uint32_t pl0 = movmatrix_trans(pack_bf16x2(p00 - h00, p01 - h01));
    const uint32_t pl1 = movmatrix_trans(pack_bf16x2(p10 - h10, p11 - h11));
    const int j = lane >> 3, r = lane & 7;
    const uint32_t vaddr = smem_u32(sv + ((j >> 1) * 8 + r) * kPitch + (j & 1) * 16);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4_trans(a0, a1, a2, a3, vaddr + mt * 32);
      mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
      mma_bf16_16816(acc[mt], a0, a1, a2, a3, pl0, pl1);
    }
    ++g;
    if ((cc.sub + 1) * kToks < cc.cnt) continue;

    // ---- end of the unit: fp32 partial (m, l, O) of (request, chunk, KV head)
    float la = l_a, lb = l_b;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, o);
      lb += __shfl_xor_sync(0xffffffffu, lb, o);
    }
    const int64_t pu = ((int64_t)cc.req * a.max_chunks + cc.chunk) * kKV + cc.head;
    float* po = a.part_o + pu * (kG * kD);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d0 = mt * 16 + gid;
      po[(2 * tig) * kD + d0] = acc[mt][0];
      po[(2 * tig + 1) * kD + d0] = acc[mt][1];
      po[(2 * tig) * kD + d0 + 8] = acc[mt][2];
      po[(2 * tig + 1) * kD + d0 + 8] = acc[mt][3];
    }
    if (gid == 0) {
      float* pml = a.part_ml + pu * (kG * 2);
      pml[(2 * tig) * 2] = m_a;
      pml[(2 * tig) * 2 + 1] = la;
      pml[(2 * tig + 1) * 2] = m_b;
      pml[(2 * tig + 1) * 2 + 1] = lb;
    }
  }
  cp_async_wait<0>();
}

// Block (request, KV head): out = sum_c w_c O_c with w_c = 2^(m_c - M) / sum_c l_c 2^(m_c - M).
__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(AttnArgs a) {
  __shared__ float s_w[kMaxChunksFast][kG];
  const int req = blockIdx.x, head = blockIdx.y, tid = threadIdx.x;
  const int64_t L = a.seq_lens[req];
  const int n = (int)(L < a.top_k ? L : a.top_k);
  const int nch = (n + kUnitRows - 1) / kUnitRows;
  const int64_t base = (int64_t)req * a.max_chunks * kKV + head;  // unit index of chunk 0
  if (tid < kG) {
    float M = kNegInf;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, a.part_ml[(base + (int64_t)c * kKV) * (kG * 2) + tid * 2]);
    float S = 0.f;
    for (int c = 0; c < nch; ++c) {
      const float* ml = a.part_ml + (base + (int64_t)c * kKV) * (kG * 2) + tid * 2;
      S += ml[1] * fast_exp2(ml[0] - M);
    }
    const float inv = 1.f / S;
    for (int c = 0; c < nch; ++c)
      s_w[c][tid] = fast_exp2(a.part_ml[(base + (int64_t)c * kKV) * (kG * 2) + tid * 2] - M) * inv;
  }
  __syncthreads();
  constexpr int kPer = kG * kD / kMergeThreads;  // 4 consecutive outputs per thread
  const int e0 = tid * kPer;
  const int g = e0 / kD;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int c = 0; c < nch; ++c) {
    const float w = s_w[c][g];
    const float4 x = *reinterpret_cast<const float4*>(a.part_o + (base + (int64_t)c * kKV) * (kG * kD) + e0);
    o.x += w * x.x;
    o.y += w * x.y;
    o.z += w * x.z;
    o.w += w * x.w;
  }
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)req * a.out_stride + head * (kG * kD) + e0;
  __nv_bfloat162 p0, p1;
  p0.x = __float2bfloat16_rn(o.x);
  p0.y = __float2bfloat16_rn(o.y);
  p1.x = __float2bfloat16_rn(o.z);
  p1.y = __float2bfloat16_rn(o.w);
  reinterpret_cast<__nv_bfloat162*>(out)[0] = p0;
  reinterpret_cast<__nv_bfloat162*>(out)[1] = p1;
}

// ------------------------------------------------------------------ generic path

template <typename T>
__global__ void attn_generic_kernel(AttnArgs a, int q_heads, int kv_heads, int D) {
  extern __shared__ float gsm[];
  const int i = blockIdx.x, h = blockIdx.y;
  const int G = q_heads / kv_heads;
  const int64_t L = a.seq_lens[i];
  const int n = (int)(L < a.top_k ? L : a.top_k);
  float* q_s = gsm;                 // [G][D]
  float* s_s = gsm + G * D;         // [G][top_k]
  float* red = s_s + G * a.top_k;   // [G][2]
  const T* q = static_cast<const T*>(a.q) + (int64_t)i * a.q_stride + (int64_t)h * G * D;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) q_s[e] = Elem<T>::load(q + e);
  __syncthreads();
  const int32_t* rows = a.rows + (int64_t)i * a.top_k;
  const int64_t rs = a.row_stride_bytes / (int64_t)sizeof(T);
  const T* K = reinterpret_cast<const T*>(a.k_pool);
  const T* V = reinterpret_cast<const T*>(a.v_pool);
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    int64_t row = rows[t];
    if (row < 0 || row >= a.num_rows) {
      raise_error(a.err, QQ_DEV_ERR_BOUNDS);
      row = 0;
    }
    const T* kr = K + row * rs + (int64_t)h * D;
    for (int g = 0; g < G; ++g) {
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(q_s[g * D + d], Elem<T>::load(kr + d), dot);
      s_s[g * a.top_k + t] = dot * a.scaling;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int g = warp; g < G; g += nw) {
    float m = -FLT_MAX;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, s_s[g * a.top_k + t]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float p = expf(s_s[g * a.top_k + t] - m);
      s_s[g * a.top_k + t] = p;
      sum += p;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[g] = sum;
  }
  __syncthreads();
  T* out = static_cast<T*>(a.out) + (int64_t)i * a.out_stride + (int64_t)h * G * D;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    float acc = 0.f;
    for (int t = 0; t < n; ++t) {
      int64_t row = rows[t];
      if (row < 0 || row >= a.num_rows) row = 0;
      acc = fmaf(s_s[g * a.top_k + t], Elem<T>::load(V + row * rs + (int64_t)h * D + d), acc);
    }
    Elem<T>::store(out + e, acc / red[g]);
  }
}

int g_sm_count = 0;

int sm_count() {
  if (g_sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  return g_sm_count;
}

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" size_t qq_workspace_bytes(int max_bs, int top_k, int q_heads, int head_dim) {
  if (max_bs < 0 || top_k < 0 || q_heads < 0 || head_dim < 0) return 0;
  return kPartialOffset + sizeof(float) * attn_partial_floats(max_bs, top_k, q_heads, head_dim) + 256;
}

extern "C" int qq_sparse_decode_attention(const qq_batch* batch, int top_k, const void* q, int dtype,
                                          int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                                          const int32_t* rows, const void* k_pool, const void* v_pool,
                                          int64_t kv_row_stride, int64_t num_rows, float scaling,
                                          void* out, int64_t out_stride, uint32_t* err, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (batch == nullptr || q == nullptr || rows == nullptr || k_pool == nullptr || v_pool == nullptr ||
      out == nullptr || top_k <= 0 || kv_heads <= 0 || head_dim <= 0 || q_heads % kv_heads != 0 ||
      num_rows <= 0)
    return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->bs > QQ_MAX_BS || batch->seq_lens == nullptr) return QQ_ERR_INVALID;
  if (dtype != QQ_BF16 && dtype != QQ_F32) return QQ_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < qq_workspace_bytes(batch->bs, top_k, q_heads, head_dim))
    return QQ_ERR_WORKSPACE;
  const int esz = dtype == QQ_BF16 ? 2 : 4;
  AttnArgs a{};
  a.seq_lens = batch->seq_lens;
  a.bs = batch->bs;
  a.top_k = top_k;
  a.max_chunks = (top_k + kAttnChunk - 1) / kAttnChunk;
  a.q = q;
  a.q_stride = q_stride;
  a.rows = rows;
  a.k_pool = static_cast<const char*>(k_pool);
  a.v_pool = static_cast<const char*>(v_pool);
  a.row_stride_bytes = kv_row_stride * esz;
  a.num_rows = num_rows;
  a.scaling = scaling;
  a.scale_log2 = scaling * 1.4426950408889634f;
  a.out = out;
  a.out_stride = out_stride;
  a.err = err;
  char* ws = static_cast<char*>(workspace);
  a.part_o = reinterpret_cast<float*>(ws + kPartialOffset);
  a.part_ml = a.part_o + (size_t)batch->bs * a.max_chunks * q_heads * head_dim;
  a.counters = ws_counters(workspace, kCounterAttn);
  cudaStream_t s = as_stream(stream);

  const bool fast = dtype == QQ_BF16 && kv_heads == kKV && head_dim == kD && q_heads == kH &&
                    (kv_row_stride * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(k_pool) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(v_pool) % 16) == 0 && (q_stride % 2) == 0 &&
                    (out_stride % 4) == 0 && (reinterpret_cast<uintptr_t>(out) % 8) == 0 &&
                    a.max_chunks <= kMaxChunksFast;
  if (fast) {
    static bool attr_set = false;
    if (!attr_set) {
      if (cudaFuncSetAttribute(attn_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemFast) !=
          cudaSuccess)
        return QQ_ERR_CUDA;
      attr_set = true;
    }
    const int units = batch->bs * a.max_chunks * kKV;
    const int grid = std::max(1, std::min((units + kWarpsFast - 1) / kWarpsFast, sm_count()));
    attn_stream_kernel<<<grid, kThreadsFast, kSmemFast, s>>>(a);
    const int rc = launch_status();
    if (rc != QQ_OK) return rc;
    attn_merge_kernel<<<dim3(batch->bs, kKV), kMergeThreads, 0, s>>>(a);
    return launch_status();
  }
  const int G = q_heads / kv_heads;
  const size_t smem = sizeof(float) * ((size_t)G * head_dim + (size_t)G * top_k + 2 * (size_t)G);
  if (smem > 200 * 1024) return QQ_ERR_UNSUPPORTED;
  dim3 grid(batch->bs, kv_heads);
  if (dtype == QQ_BF16) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(attn_generic_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return QQ_ERR_CUDA;
    attn_generic_kernel<__nv_bfloat16><<<grid, 128, smem, s>>>(a, q_heads, kv_heads, head_dim);
  } else {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(attn_generic_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
      return QQ_ERR_CUDA;
    attn_generic_kernel<float><<<grid, 128, smem, s>>>(a, q_heads, kv_heads, head_dim);
  }
  return launch_status();
}
