// Qwen3-MoE expert block as two grouped GEMMs on the fifth-generation tensor
// cores (tcgen05.mma, accumulators in tensor memory) and a combine kernel.
//
// Replaces the per-expert loop of Qwen3MoeSparseMoeBlock.forward
// (model/qwen3_moe.py:121-147): for every expert e that any token picked,
//   y = down_e(silu(gate_e(x[tokens])) * up_e(x[tokens])) * weight
//   out.index_add_(0, tokens, y)
// Here the routing's (token, slot) pairs are grouped by expert (ascending,
// tokens ascending within an expert, as torch.where returns them) and
//   GEMM 1: H[p] = bf16(bf16(silu(bf16(X[tok p] . Wg_e^T))) * bf16(X[tok p] . Wu_e^T))
//   GEMM 2: Y[p] = bf16(bf16(H[p] . Wd_e^T) * w_p)
//   combine: out[t] = ((Y[p1] + Y[p2]) + ...) in ascending expert order,
//            rounded to bf16 after every add (index_add_ into a bf16 tensor)
// with the roundings where the reference's bf16 tensors round.
//
// Grouped GEMM CTA: 128 pairs of one expert (M) x 256 weight rows (N: GEMM 1
// the 128 gate rows and the 128 up rows of the same intermediate columns,
// GEMM 2 256 hidden columns), K in blocks of 64 through a 4-stage ring.
// The grid's M slots are an upper bound (ceil(pairs / 128) + experts); each
// CTA finds its expert and pair tile from the expert offsets on the device,
// so no host round trip is needed, and slots past the last tile exit.
// Warp roles: warps 0-3 epilogue (thread = pair row = TMEM lane), warps 4-7
// loaders (16-byte cp.async; pair rows gathered through their token index,
// rows past the expert's pairs zero-filled without a read; each thread's
// copies of a stage arrive on its barrier asynchronously), warp 8 TMEM
// allocation and MMA issue (one thread).  Every mbarrier wait is bounded.

#include <cmath>

#include "tcgen05.cuh"

namespace qq {
namespace {

using namespace tc;

constexpr int kMM = 128;                    // pairs per tile
constexpr int kMN = 256;                    // weight rows per tile
constexpr int kMK = 64;                     // K elements per stage (128-byte rows)
constexpr int kStages = 4;
constexpr int kABytes = kMM * kMK * 2;      // 16 KiB
constexpr int kBBytes = kMN * kMK * 2;      // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 4, kLoadWarps = 4;
constexpr int kMmaWarp = kEpiWarps + kLoadWarps;  // 8
constexpr int kThreads = (kMmaWarp + 1) * 32;     // 288
constexpr int kDynSmem = kStages * kStageBytes + 1024;
constexpr uint32_t kTmemCols = 256;
constexpr int kMaxExperts = 1024;

enum : int { kBarFull = 0, kBarEmpty = kStages, kBarDone = 2 * kStages, kNumBars = kBarDone + 1 };

struct MoeArgs {
  const int32_t* pair_token;      // [pairs]
  const int64_t* offsets;         // [E + 1]
  const uint16_t* pair_weight;    // [pairs] bf16 (GEMM 2)
  int num_experts;
  int64_t num_pairs;
  int64_t num_tokens;
  const char* a;                  // GEMM 1: x rows (by token); GEMM 2: H rows (by pair)
  int64_t a_stride;               // bytes between rows of a
  const void* const* w0;          // GEMM 1: gate; GEMM 2: down   (device array of E pointers)
  const void* const* w1;          // GEMM 1: up
  int64_t w_stride;               // bytes between weight rows
  int K;                          // hidden (GEMM 1) or intermediate (GEMM 2)
  int n_cols;                     // intermediate (GEMM 1) or hidden (GEMM 2)
  char* c;                        // GEMM 1: H [pairs][inter]; GEMM 2: Y [pairs][hidden]
  int64_t c_stride;               // bytes between rows of c
  uint32_t* err;
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// MODE 0: gate/up + SiLU * up -> H.  MODE 1: down x routing weight -> Y.
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) moe_gemm_kernel(MoeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_expert;
  __shared__ int64_t s_row0, s_rows;  // the tile's first pair and its valid rows
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  volatile int* abort_flag = &s_abort;

  // ---- which expert and pair tile: M slot blockIdx.y in the experts' tile prefix
  if (threadIdx.x == 0) s_expert = -1;
  __syncthreads();
  {
    const int E = a.num_experts;
    int64_t run = 0;  // tiles of experts before this thread's chunk
    for (int e0 = 0; e0 < E; e0 += kThreads) {
      const int e = e0 + threadIdx.x;
      int64_t t = 0, n = 0;
      if (e < E) {
        n = a.offsets[e + 1] - a.offsets[e];
        t = n > 0 ? (n + kMM - 1) / kMM : 0;
      }
      // block-wide inclusive scan of t (the thread count is small: a simple smem scan)
      __shared__ int64_t scan[kThreads];
      scan[threadIdx.x] = t;
      __syncthreads();
      for (int o = 1; o < kThreads; o <<= 1) {
        const int64_t v = threadIdx.x >= o ? scan[threadIdx.x - o] : 0;
        __syncthreads();
        scan[threadIdx.x] += v;
        __syncthreads();
      }
      const int64_t incl = run + scan[threadIdx.x], excl = incl - t;
      if (e < E && t > 0 && (int64_t)blockIdx.y >= excl && (int64_t)blockIdx.y < incl) {
        s_expert = e;
        const int64_t m0 = ((int64_t)blockIdx.y - excl) * kMM;
        s_row0 = a.offsets[e] + m0;
        s_rows = min((int64_t)kMM, n - m0);
      }
      run += scan[kThreads - 1];
      __syncthreads();
    }
  }
  const int e = s_expert;
  if (e < 0) return;  // past the last tile (uniform over the CTA)
  const int64_t row0 = s_row0, rows = s_rows;
  const int c0 = blockIdx.x * (MODE == 0 ? kMM : kMN);  // first output column of the tile
  const int KB = a.K / kMK;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(kBarFull + i), kLoadWarps * 32);
      mbar_init(bar(kBarEmpty + i), 1);
    }
    mbar_init(bar(kBarDone), 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&s_tmem), kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp >= kEpiWarps && warp < kMmaWarp) {
    // ================================================================ loaders
    // lane l: 16-byte chunk l & 7 of rows (l >> 3) + 4 i; warp lw: A rows
    // 32 lw .. 32 lw + 31, B rows 64 lw .. 64 lw + 63
    const int lw = warp - kEpiWarps;
    const int ch = lane & 7, rs = lane >> 3;
    const char* arow[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = lw * 32 + rs + 4 * i;
      const int64_t p = row0 + r;
      const char* src = nullptr;
      if (r < rows) {
        int64_t ar = p;  // GEMM 2 reads H by pair
        if (MODE == 0) {
          ar = a.pair_token[p];
          if (ar < 0 || ar >= a.num_tokens) {
            raise_error(a.err, QQ_DEV_ERR_BOUNDS);
            ar = 0;
          }
        }
        src = a.a + ar * a.a_stride + ch * 16;
      }
      arow[i] = src;
    }
    const char* w0 = static_cast<const char*>(a.w0[e]);
    const char* w1 = MODE == 0 ? static_cast<const char*>(a.w1[e]) : nullptr;
#pragma unroll 1
    for (int t = 0; t < KB; ++t) {
      const int st = t % kStages;
      if (t >= kStages &&
          !__all_sync(0xffffffffu, mbar_wait(bar(kBarEmpty + st), ((t / kStages) - 1) & 1, abort_flag, a.err)))
        break;
      const uint32_t sa = base + st * kStageBytes, sb = sa + kABytes;
      const int64_t koff = (int64_t)t * (kMK * 2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = lw * 32 + rs + 4 * i;
        const uint32_t dst = sa + r * 128 + (((ch ^ (r & 7))) << 4);
        if (arow[i] != nullptr) cp_async_16(dst, arow[i] + koff);
        else cp_async_16_zfill(dst, a.a, 0u);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = lw * 64 + rs + 4 * i;  // weight row of the tile, 0..255
        const char* src;
        if (MODE == 0) src = (r < kMM ? w0 + (int64_t)(c0 + r) * a.w_stride : w1 + (int64_t)(c0 + r - kMM) * a.w_stride);
        else src = w0 + (int64_t)(c0 + r) * a.w_stride;
        cp_async_16(sb + r * 128 + (((ch ^ (r & 7))) << 4), src + koff + ch * 16);
      }
      cp_async_arrive(bar(kBarFull + st));
    }
    cp_async_wait<0>();
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issue
    if (lane == 0) {
      constexpr uint32_t kId = instr_desc(0, kMM, kMN);
      bool ok = true;
#pragma unroll 1
      for (int t = 0; t < KB && ok; ++t) {
        const int st = t % kStages;
        ok = mbar_wait(bar(kBarFull + st), (t / kStages) & 1, abort_flag, a.err);
        if (!ok) break;
        tc_fence_after();
        const uint64_t da = desc_k(base + st * kStageBytes), db = desc_k(base + st * kStageBytes + kABytes);
        umma_bf16_x4(tmem, da, db, 2, 2, kId, t > 0 ? 1u : 0u);  // four 32-byte k-steps
        umma_commit(bar(kBarEmpty + st));
      }
      umma_commit(bar(kBarDone));
      mbar_wait(bar(kBarDone), 0, abort_flag, a.err, true);
    }
    __syncwarp();
  } else {
    // ================================================================ epilogue (warps 0-3)
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarDone), 0, abort_flag, a.err));
    tc_fence_after();
    const int r = warp * 32 + lane;
    const bool valid = ok && r < rows;
    const int64_t p = row0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    char* dst = a.c + (valid ? p : 0) * a.c_stride + (int64_t)c0 * 2;
    uint32_t v[32];
    if (MODE == 0) {
      uint32_t u[32];
#pragma unroll 1
      for (int cc = 0; cc < kMM / 32; ++cc) {
        tmem_ld32(lane_base + cc * 32, v);
        tmem_ld32(lane_base + kMM + cc * 32, u);
        tmem_ld_wait();
        if (valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float h2[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const float g = bf16r(__uint_as_float(v[i + k]));
              const float up = bf16r(__uint_as_float(u[i + k]));
              const float s = bf16r(g / (1.0f + expf(-g)));
              h2[k] = s * up;
            }
            pk[i >> 1] = pack_bf16(h2[0], h2[1]);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + cc * 64 + q * 16) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
    } else {
      const float w = valid ? __uint_as_float((uint32_t)a.pair_weight[p] << 16) : 0.f;
#pragma unroll 1
      for (int cc = 0; cc < kMN / 32; ++cc) {
        tmem_ld32(lane_base + cc * 32, v);
        tmem_ld_wait();
        if (valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            pk[i >> 1] = pack_bf16(bf16r(__uint_as_float(v[i])) * w, bf16r(__uint_as_float(v[i + 1])) * w);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + cc * 64 + q * 16) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// out[t] = Y[p_1] + Y[p_2] + ... over token t's pairs in ascending pair order
// (= ascending expert), rounded to bf16 after every add.  One 256-thread CTA
// per token, 8 columns (16 bytes) per thread per step.
__global__ void __launch_bounds__(256) moe_combine_kernel(const int32_t* token_pairs, int top_k, const char* y,
                                                          int64_t y_stride, int hidden, int64_t num_pairs, char* out,
                                                          int64_t out_stride, uint32_t* err) {
  const int64_t t = blockIdx.x;
  int32_t pr[16];
  int n = 0;
  for (int s = 0; s < top_k && s < 16; ++s) {
    const int32_t p = token_pairs[t * top_k + s];
    if (p < 0 || p >= num_pairs) {
      if (threadIdx.x == 0) raise_error(err, QQ_DEV_ERR_BOUNDS);
      continue;
    }
    int k = n++;
    while (k > 0 && pr[k - 1] > p) {  // insertion sort: ascending pair index
      pr[k] = pr[k - 1];
      --k;
    }
    pr[k] = p;
  }
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < n; ++i) {
      const uint4 w = *reinterpret_cast<const uint4*>(y + pr[i] * y_stride + (int64_t)c * 2);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[2 * k] = bf16r(acc[2 * k] + __uint_as_float(ws[k] << 16));
        acc[2 * k + 1] = bf16r(acc[2 * k + 1] + __uint_as_float(ws[k] & 0xFFFF0000u));
      }
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]);
    o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]);
    o.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * out_stride + (int64_t)c * 2) = o;
  }
}

// The routing's pairs grouped by expert in one CTA (small batches): thread e
// counts expert e's pairs, a block scan gives the offsets, then thread e
// walks the pairs in (token, slot) order and places its own, so the order
// within an expert is ascending token (the reference loop's torch.where
// order) with no atomics.  An expert index out of range is skipped and
// reported.
constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxPairs = 2048;

__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(const int64_t* experts, const uint16_t* weights,
                                                                int num_pairs, int top_k, int num_experts,
                                                                int32_t* pair_token, uint16_t* pair_weight,
                                                                int64_t* offsets, int32_t* token_pairs, uint32_t* err) {
  __shared__ int16_t s_ex[kPlanMaxPairs];
  __shared__ int32_t s_off[kMaxExperts + 1];
  for (int i = threadIdx.x; i < num_pairs; i += blockDim.x) {
    const int64_t e = experts[i];
    if (e < 0 || e >= num_experts) {
      raise_error(err, QQ_DEV_ERR_BOUNDS);
      s_ex[i] = -1;
      token_pairs[i] = 0;
    } else {
      s_ex[i] = (int16_t)e;
    }
  }
  __syncthreads();
  const int e = threadIdx.x;
  int cnt = 0;
  if (e < num_experts)
    for (int i = 0; i < num_pairs; ++i) cnt += s_ex[i] == e;
  // exclusive scan of the counts over the block (experts <= blockDim)
  s_off[threadIdx.x + 1] = cnt;
  if (threadIdx.x == 0) s_off[0] = 0;
  __syncthreads();
  for (int o = 1; o < kPlanThreads; o <<= 1) {
    const int t = threadIdx.x + 1;
    const int val = t > o ? s_off[t - o] : 0;
    __syncthreads();
    s_off[t] += val;
    __syncthreads();
  }
  if (e < num_experts) {
    const int base = s_off[e];
    offsets[e] = base;
    if (e == num_experts - 1) offsets[num_experts] = s_off[num_experts];
    int run = 0;
    for (int i = 0; i < num_pairs; ++i) {
      if (s_ex[i] != e) continue;
      const int p = base + run++;
      pair_token[p] = i / top_k;
      pair_weight[p] = weights[i];
      token_pairs[i] = p;
    }
  }
}

}  // namespace
}  // namespace qq

extern "C" int qq_moe_experts(const qq_moe_plan* plan, const void* x, int64_t x_stride, int hidden, int inter,
                              const void* const* w_gate, const void* const* w_up, const void* const* w_down,
                              void* h_buf, void* y_buf, void* out, int64_t out_stride, uint32_t* err, void* stream) {
  using namespace qq;
  if (plan == nullptr || x == nullptr || w_gate == nullptr || w_up == nullptr || w_down == nullptr ||
      h_buf == nullptr || y_buf == nullptr || out == nullptr || plan->pair_token == nullptr ||
      plan->expert_offsets == nullptr || plan->pair_weight == nullptr || plan->token_pairs == nullptr ||
      plan->num_tokens < 0 || plan->num_pairs < 0 || plan->top_k <= 0 || plan->num_experts <= 0)
    return QQ_ERR_INVALID;
  if (plan->num_tokens == 0) return QQ_OK;
  if (hidden % kMN != 0 || inter % kMM != 0 || hidden % kMK != 0 || inter % kMK != 0 ||
      plan->num_experts > kMaxExperts || plan->top_k > 16 || (x_stride * 2) % 16 != 0 ||
      (out_stride * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0 || reinterpret_cast<uintptr_t>(h_buf) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(y_buf) % 16 != 0)
    return QQ_ERR_UNSUPPORTED;
  const int64_t m_slots = (plan->num_pairs + kMM - 1) / kMM + plan->num_experts;
  if (m_slots > 65535) return QQ_ERR_UNSUPPORTED;
  cudaStream_t s = as_stream(stream);
  MoeArgs g{};
  g.pair_token = plan->pair_token;
  g.offsets = plan->expert_offsets;
  g.pair_weight = plan->pair_weight;
  g.num_experts = plan->num_experts;
  g.num_pairs = plan->num_pairs;
  g.num_tokens = plan->num_tokens;
  g.err = err;
  if (plan->num_pairs > 0) {
    static SmemLimit lim0, lim1;
    int rc = lim0.ensure((const void*)moe_gemm_kernel<0>, kDynSmem);
    if (rc != QQ_OK) return rc;
    rc = lim1.ensure((const void*)moe_gemm_kernel<1>, kDynSmem);
    if (rc != QQ_OK) return rc;
    // GEMM 1: H = silu(X Wg^T) * (X Wu^T), tiles of 128 intermediate columns (gate and up rows)
    g.a = static_cast<const char*>(x);
    g.a_stride = x_stride * 2;
    g.w0 = w_gate;
    g.w1 = w_up;
    g.w_stride = (int64_t)hidden * 2;
    g.K = hidden;
    g.n_cols = inter;
    g.c = static_cast<char*>(h_buf);
    g.c_stride = (int64_t)inter * 2;
    moe_gemm_kernel<0><<<dim3(inter / kMM, (unsigned)m_slots), kThreads, kDynSmem, s>>>(g);
    rc = launch_status();
    if (rc != QQ_OK) return rc;
    // GEMM 2: Y = (H Wd^T) * w, tiles of 256 hidden columns
    g.a = static_cast<const char*>(h_buf);
    g.a_stride = (int64_t)inter * 2;
    g.w0 = w_down;
    g.w1 = nullptr;
    g.w_stride = (int64_t)inter * 2;
    g.K = inter;
    g.n_cols = hidden;
    g.c = static_cast<char*>(y_buf);
    g.c_stride = (int64_t)hidden * 2;
    moe_gemm_kernel<1><<<dim3(hidden / kMN, (unsigned)m_slots), kThreads, kDynSmem, s>>>(g);
    rc = launch_status();
    if (rc != QQ_OK) return rc;
  }
  moe_combine_kernel<<<(unsigned)plan->num_tokens, 256, 0, s>>>(
      plan->token_pairs, plan->top_k, static_cast<const char*>(y_buf), (int64_t)hidden * 2, hidden, plan->num_pairs,
      static_cast<char*>(out), out_stride * 2, err);
  return launch_status();
}

extern "C" int qq_moe_route_plan(const int64_t* experts, const uint16_t* weights, int64_t num_tokens, int top_k,
                           int num_experts, int32_t* pair_token, uint16_t* pair_weight, int64_t* expert_offsets,
                           int32_t* token_pairs, uint32_t* err, void* stream) {
  using namespace qq;
  if (experts == nullptr || weights == nullptr || pair_token == nullptr || pair_weight == nullptr ||
      expert_offsets == nullptr || token_pairs == nullptr || num_tokens < 0 || top_k <= 0 || num_experts <= 0)
    return QQ_ERR_INVALID;
  if (num_experts > kMaxExperts || num_tokens * top_k > kPlanMaxPairs) return QQ_ERR_UNSUPPORTED;
  moe_plan_kernel<<<1, kPlanThreads, 0, as_stream(stream)>>>(experts, weights, (int)(num_tokens * top_k), top_k,
                                                             num_experts, pair_token, pair_weight, expert_offsets,
                                                             token_pairs, err);
  return launch_status();
}
