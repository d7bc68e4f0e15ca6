// [Q7] Split-K sparse decode attention over an explicit row list.
//
// Fast path (bf16, 4 KV heads, head_dim 128, 8 query heads per KV head):
// a persistent kernel, one 256-thread block per SM.  Work items are
// (request, chunk of 128 rows), assigned round-robin; a block walks the
// 32-row stages of its items as one stream through a 3-slot shared-memory
// ring, so the gather of stage g+2 is in flight while stage g is computed,
// across item boundaries.  The gather is done by all 8 warps with 16-byte
// cp.async.cg copies (a warp moves 512 contiguous bytes of one row per
// instruction; rows past the end are zero-filled by the copy), 4096 copies
// per 64 KiB stage, so every SM keeps ~128 KiB of independent requests in
// flight.  Rows land at a 1040-byte pitch: ldmatrix reads are bank-conflict
// free.  Warp w computes KV head w%4 on half w/4 of every stage:
//   S^T[16 rows x 8 heads] = K[16 x 128] . Q^T[128 x 8]   (8 x mma m16n8k16)
//   online softmax in fp32 (exp2 domain), P^T via movmatrix.trans
//   O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8]          (P as bf16 hi + lo: 16 mma)
// The two halves of a head merge through shared memory at the end of the
// item; chunks of one request merge in the last block to finish (arrival
// counter in the workspace).  Per row the kernel reads 2 KiB, so it is
// HBM-bound.
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
constexpr int kRowBytes = kKV * kD * 2;    // 1024: one K (or V) row, all KV heads
constexpr int kPitch = kRowBytes + 16;     // 1040
constexpr int kToks = 32;                  // rows per stage
constexpr int kSlots = 3;                  // stages resident in shared memory
constexpr int kChunk = kAttnChunk;         // 128 rows per work item
constexpr int kWarpsFast = 8;
constexpr int kThreadsFast = kWarpsFast * 32;
constexpr int kSlotBytes = 2 * kToks * kPitch;  // K tile + V tile
constexpr int kMergeFloats = kKV * kG * kD;     // 4096
constexpr int kCopiesPerThread = kToks * 2 * kRowBytes / 16 / kThreadsFast;  // 16
// chunks per request the in-kernel merge handles (its staging lives in the
// 4096-float merge buffer: chunks x 32 heads x 3 floats); top_k <= 32 * 128
constexpr int kMaxChunksFast = 32;
constexpr size_t kSmemFast = (size_t)kSlots * kSlotBytes + sizeof(float) * (kMergeFloats + 2 * kKV * kG) + 16;

struct AttnArgs {
  const int64_t* seq_lens;
  int bs;
  int top_k;
  int max_chunks;
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
  float* part_o;   // [bs * max_chunks][kH][kD]
  float* part_ml;  // [bs * max_chunks][kH][2]
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

// 16-byte async copy global -> shared; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

#define kNegInf (-__int_as_float(0x7f800000))

// A position in a block's stream of stages: stage `sub` of work item `item`.
struct Cursor {
  int item;  // -1 before the first stage, >= total when exhausted
  int sub;
  int cnt;   // rows of the item
  int base;  // first row (within the request's list) of the item
  int req;   // batch index
};

__device__ __forceinline__ int item_rows(const AttnArgs& a, int item, int& req, int& base) {
  req = item / a.max_chunks;
  const int c = item - req * a.max_chunks;
  const int64_t L = __ldg(a.seq_lens + req);
  const int n = (int)(L < a.top_k ? L : a.top_k);
  base = c * kChunk;
  const int cnt = n - base;
  return cnt <= 0 ? 0 : (cnt < kChunk ? cnt : kChunk);
}

// Advance to the next stage of this block's stream; false when exhausted.
__device__ __forceinline__ bool next_stage(const AttnArgs& a, Cursor& c, int total_items) {
  if (c.item >= 0 && c.item < total_items && (c.sub + 1) * kToks < c.cnt) {
    ++c.sub;
    return true;
  }
  int item = c.item < 0 ? (int)blockIdx.x : c.item + (int)gridDim.x;
  for (; item < total_items; item += gridDim.x) {
    int req, base;
    const int cnt = item_rows(a, item, req, base);
    if (cnt > 0) {
      c.item = item;
      c.sub = 0;
      c.cnt = cnt;
      c.base = base;
      c.req = req;
      return true;
    }
  }
  c.item = total_items;
  return false;
}

// Lane l's pool row for row l of stage `c` (loaded one iteration before use).
__device__ __forceinline__ int32_t load_stage_row(const AttnArgs& a, const Cursor& c, int lane) {
  const int ntok = min(kToks, c.cnt - c.sub * kToks);
  return lane < ntok ? __ldg(a.rows + (int64_t)c.req * a.top_k + c.base + c.sub * kToks + lane) : 0;
}

// Gather the 32 K and V rows of stage `c` into `slot` (all 256 threads,
// kCopiesPerThread 16-byte copies each; a warp copies 512 contiguous bytes).
// `row_l` is this lane's value from load_stage_row.
__device__ __forceinline__ void issue_stage(const AttnArgs& a, const Cursor& c, int32_t row_l, char* slot, int warp,
                                            int lane) {
  const int ntok = min(kToks, c.cnt - c.sub * kToks);
  int64_t my_row = row_l;  // lane l holds the pool row of stage row l
  if (lane < ntok && (my_row < 0 || my_row >= a.num_rows)) {
    raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    my_row = 0;
  }
  const int sub_row = warp >> 2;           // 0/1: which of the two rows this warp copies per round
  const int chunk = (warp & 3) * 32 + lane;  // 16-byte chunk within the 2 KiB (K | V) row
  const bool is_v = chunk >= 64;
  const int off = (chunk & 63) * 16;
  const char* pool = is_v ? a.v_pool : a.k_pool;
  char* dst0 = slot + (is_v ? kToks * kPitch : 0) + off;
#pragma unroll
  for (int k = 0; k < kCopiesPerThread; ++k) {
    const int r = 2 * k + sub_row;
    const int64_t row = __shfl_sync(0xffffffffu, my_row, r);
    const bool valid = r < ntok;
    cp_async_16(dst0 + r * kPitch, pool + row * a.row_stride_bytes + off, valid ? 16u : 0u);
  }
}

__global__ void __launch_bounds__(kThreadsFast, 1) attn_fast_kernel(AttnArgs a) {
  extern __shared__ __align__(128) char smem[];
  float* s_merge = reinterpret_cast<float*>(smem + (size_t)kSlots * kSlotBytes);
  float* s_mm = s_merge + kMergeFloats;  // [kKV][kG] m of the second half
  float* s_ml = s_mm + kKV * kG;         // [kKV][kG] l of the second half
  int* s_flag = reinterpret_cast<int*>(s_ml + kKV * kG);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = warp & 3;      // KV head
  const int half = warp >> 2;  // which 16 rows of each stage
  const int gid = lane >> 2, tig = lane & 3;
  const int total_items = a.bs * a.max_chunks;
  const __nv_bfloat16* qbase = static_cast<const __nv_bfloat16*>(a.q);

  // prologue: put kSlots - 1 stages in flight; the fetch cursor's row
  // indices are always loaded one stage ahead of their use
  Cursor fc{-1, 0, 0, 0, 0}, cc{-1, 0, 0, 0, 0};
  bool have_f = next_stage(a, fc, total_items);
  int32_t row_f = have_f ? load_stage_row(a, fc, lane) : 0;
#pragma unroll
  for (int s = 0; s < kSlots - 1; ++s) {
    if (have_f) {
      issue_stage(a, fc, row_f, smem + (size_t)s * kSlotBytes, warp, lane);
      have_f = next_stage(a, fc, total_items);
      if (have_f) row_f = load_stage_row(a, fc, lane);
    }
    cp_async_commit();
  }

  uint32_t qb[8][2];
  float acc[8][4];
  float m_a = kNegInf, m_b = kNegInf, l_a = 0.f, l_b = 0.f;
  int g = 0;
  while (next_stage(a, cc, total_items)) {
    cp_async_wait<kSlots - 2>();
    __syncthreads();  // stage g visible to all; slot (g - 1) % kSlots free
    if (have_f) {
      issue_stage(a, fc, row_f, smem + (size_t)((g + kSlots - 1) % kSlots) * kSlotBytes, warp, lane);
      have_f = next_stage(a, fc, total_items);
      if (have_f) row_f = load_stage_row(a, fc, lane);
    }
    cp_async_commit();

    if (cc.sub == 0) {
      // Q^T fragments of KV head h: B[k = d][n = query head g]
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbase + (int64_t)cc.req * a.q_stride +
                                                               (int64_t)(h * kG + gid) * kD);
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

    const int ntok = min(kToks, cc.cnt - cc.sub * kToks);
    const char* sk = smem + (size_t)(g % kSlots) * kSlotBytes;
    const char* sv = sk + kToks * kPitch;
    const int t0 = half * 16 + gid, t1 = t0 + 8;
    if (half * 16 < ntok) {
      // ---- S^T = K . Q^T
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t kaddr = smem_u32(sk + (half * 16 + (lane & 15)) * kPitch + h * (kD * 2) + (lane >> 4) * 16);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, kaddr + kk * 32);
        mma_bf16_16816(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      // ---- online softmax (exp2 domain); rows >= ntok are masked
      const bool v0 = t0 < ntok, v1 = t1 < ntok;
      const float s00 = v0 ? c[0] * a.scale_log2 : kNegInf;  // row t0, head 2tig
      const float s01 = v0 ? c[1] * a.scale_log2 : kNegInf;  // row t0, head 2tig+1
      const float s10 = v1 ? c[2] * a.scale_log2 : kNegInf;  // row t1, head 2tig
      const float s11 = v1 ? c[3] * a.scale_log2 : kNegInf;  // row t1, head 2tig+1
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
      // ---- P^T fragments (rows x heads -> heads x rows) and O^T += V^T . P^T.
      // P is split into bf16 hi + lo parts (two MMAs per tile), so the
      // weights carry ~16 mantissa bits and the fp32 result tracks an fp32
      // softmax-weighted sum to ~1e-5 relative.
      float h00, h01, h10, h11;
      const uint32_t pb0 = movmatrix_trans(pack_bf16x2_split(p00, p01, h00, h01));
      const uint32_t pb1 = movmatrix_trans(pack_bf16x2_split(p10, p11, h10, h11));
      const uint32_t pl0 = movmatrix_trans(pack_bf16x2(p00 - h00, p01 - h01));
      const uint32_t pl1 = movmatrix_trans(pack_bf16x2(p10 - h10, p11 - h11));
      const int j = lane >> 3, r = lane & 7;
      const uint32_t vaddr =
          smem_u32(sv + (half * 16 + (j >> 1) * 8 + r) * kPitch + h * (kD * 2) + (j & 1) * 16);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, vaddr + mt * 32);
        mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
        mma_bf16_16816(acc[mt], a0, a1, a2, a3, pl0, pl1);
      }
    }
    ++g;
    if ((cc.sub + 1) * kToks < cc.cnt) continue;

    // ------------------------------------------------------------ item epilogue
    const int req = cc.req;
    const int chunk = cc.base / kChunk;
    const int64_t Lr = __ldg(a.seq_lens + req);
    const int nchunks = (int)(((Lr < a.top_k ? Lr : a.top_k) + kChunk - 1) / kChunk);
    float la = l_a, lb = l_b;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, o);
      lb += __shfl_xor_sync(0xffffffffu, lb, o);
    }
    float* mo = s_merge + h * (kG * kD);
    if (half == 1) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d0 = mt * 16 + gid;
        mo[(2 * tig) * kD + d0] = acc[mt][0];
        mo[(2 * tig + 1) * kD + d0] = acc[mt][1];
        mo[(2 * tig) * kD + d0 + 8] = acc[mt][2];
        mo[(2 * tig + 1) * kD + d0 + 8] = acc[mt][3];
      }
      if (gid == 0) {
        s_mm[h * kG + 2 * tig] = m_a;
        s_mm[h * kG + 2 * tig + 1] = m_b;
        s_ml[h * kG + 2 * tig] = la;
        s_ml[h * kG + 2 * tig + 1] = lb;
      }
    }
    __syncthreads();
    if (half == 0) {
      const float mo_a = s_mm[h * kG + 2 * tig], mo_b = s_mm[h * kG + 2 * tig + 1];
      const float lo_a = s_ml[h * kG + 2 * tig], lo_b = s_ml[h * kG + 2 * tig + 1];
      const float M_a = fmaxf(m_a, mo_a), M_b = fmaxf(m_b, mo_b);
      const float fa_a = m_a == kNegInf ? 0.f : fast_exp2(m_a - M_a);
      const float fo_a = mo_a == kNegInf ? 0.f : fast_exp2(mo_a - M_a);
      const float fa_b = m_b == kNegInf ? 0.f : fast_exp2(m_b - M_b);
      const float fo_b = mo_b == kNegInf ? 0.f : fast_exp2(mo_b - M_b);
      const float L_a = la * fa_a + lo_a * fo_a, L_b = lb * fa_b + lo_b * fo_b;
      const int qh_a = h * kG + 2 * tig, qh_b = qh_a + 1;  // query heads of this thread
      if (nchunks == 1) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)req * a.out_stride;
        const float inv_a = 1.f / L_a, inv_b = 1.f / L_b;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + gid;
          out[qh_a * kD + d0] = __float2bfloat16_rn((acc[mt][0] * fa_a + mo[(2 * tig) * kD + d0] * fo_a) * inv_a);
          out[qh_b * kD + d0] =
              __float2bfloat16_rn((acc[mt][1] * fa_b + mo[(2 * tig + 1) * kD + d0] * fo_b) * inv_b);
          out[qh_a * kD + d0 + 8] =
              __float2bfloat16_rn((acc[mt][2] * fa_a + mo[(2 * tig) * kD + d0 + 8] * fo_a) * inv_a);
          out[qh_b * kD + d0 + 8] =
              __float2bfloat16_rn((acc[mt][3] * fa_b + mo[(2 * tig + 1) * kD + d0 + 8] * fo_b) * inv_b);
        }
      } else {
        const int64_t pidx = (int64_t)req * a.max_chunks + chunk;
        float* po = a.part_o + pidx * (kH * kD);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + gid;
          po[qh_a * kD + d0] = acc[mt][0] * fa_a + mo[(2 * tig) * kD + d0] * fo_a;
          po[qh_b * kD + d0] = acc[mt][1] * fa_b + mo[(2 * tig + 1) * kD + d0] * fo_b;
          po[qh_a * kD + d0 + 8] = acc[mt][2] * fa_a + mo[(2 * tig) * kD + d0 + 8] * fo_a;
          po[qh_b * kD + d0 + 8] = acc[mt][3] * fa_b + mo[(2 * tig + 1) * kD + d0 + 8] * fo_b;
        }
        if (gid == 0) {
          float* pml = a.part_ml + pidx * (kH * 2);
          pml[qh_a * 2] = M_a;
          pml[qh_a * 2 + 1] = L_a;
          pml[qh_b * 2] = M_b;
          pml[qh_b * 2 + 1] = L_b;
        }
        __threadfence();
      }
    }
    __syncthreads();
    if (nchunks > 1) {
      // ---- the last chunk of the request to finish merges all chunks
      if (tid == 0) {
        const int old = atomicAdd(&a.counters[req], 1);
        *s_flag = old == nchunks - 1;
      }
      __syncthreads();
      if (*s_flag) {
        // merge the request's chunks: (m, l) of every (chunk, head) staged in
        // shared memory with one batch of loads, per-head weights computed
        // once, then each thread combines 16 outputs with independent float4 loads
        __threadfence();
        const float* pml = a.part_ml + (int64_t)req * a.max_chunks * (kH * 2);
        const float* po = a.part_o + (int64_t)req * a.max_chunks * (kH * kD);
        float* s_pml = s_merge;                      // [nchunks][kH][2]
        float* s_w = s_merge + kMaxChunksFast * kH * 2;  // [nchunks][kH]
        for (int t = tid; t < nchunks * kH * 2; t += kThreadsFast) s_pml[t] = __ldcg(pml + t);
        __syncthreads();
        if (tid < kH) {
          float M = kNegInf;
          for (int c = 0; c < nchunks; ++c) M = fmaxf(M, s_pml[(c * kH + tid) * 2]);
          float S = 0.f;
          for (int c = 0; c < nchunks; ++c) S += s_pml[(c * kH + tid) * 2 + 1] * fast_exp2(s_pml[(c * kH + tid) * 2] - M);
          const float inv = 1.f / S;
          for (int c = 0; c < nchunks; ++c) s_w[c * kH + tid] = fast_exp2(s_pml[(c * kH + tid) * 2] - M) * inv;
        }
        __syncthreads();
        constexpr int kPer = kH * kD / kThreadsFast;  // 16 consecutive outputs per thread
        const int e0 = tid * kPer;
        const int qh = e0 / kD;
        float o[kPer];
#pragma unroll
        for (int v = 0; v < kPer; ++v) o[v] = 0.f;
#pragma unroll 4
        for (int c = 0; c < nchunks; ++c) {
          const float w = s_w[c * kH + qh];
          const float4* src = reinterpret_cast<const float4*>(po + (int64_t)c * (kH * kD) + e0);
#pragma unroll
          for (int v = 0; v < kPer / 4; ++v) {
            const float4 x = __ldcg(src + v);
            o[4 * v] += w * x.x;
            o[4 * v + 1] += w * x.y;
            o[4 * v + 2] += w * x.z;
            o[4 * v + 3] += w * x.w;
          }
        }
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)req * a.out_stride + e0;
#pragma unroll
        for (int v = 0; v < kPer; v += 2) {
          __nv_bfloat162 pair;
          pair.x = __float2bfloat16_rn(o[v]);
          pair.y = __float2bfloat16_rn(o[v + 1]);
          *reinterpret_cast<__nv_bfloat162*>(out + v) = pair;
        }
        if (tid == 0) a.counters[req] = 0;
      }
      __syncthreads();
    }
  }
  cp_async_wait<0>();
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
                    kv_row_stride == kKV * kD && (reinterpret_cast<uintptr_t>(k_pool) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(v_pool) % 16) == 0 && (q_stride % 2) == 0 &&
                    (out_stride % 2) == 0 && a.max_chunks <= kMaxChunksFast;
  if (fast) {
    static bool attr_set = false;
    if (!attr_set) {
      if (cudaFuncSetAttribute(attn_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemFast) !=
          cudaSuccess)
        return QQ_ERR_CUDA;
      attr_set = true;
    }
    const int items = batch->bs * a.max_chunks;
    const int grid = std::min(items, sm_count());
    attn_fast_kernel<<<grid, kThreadsFast, kSmemFast, s>>>(a);
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
