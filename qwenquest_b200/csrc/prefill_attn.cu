// Dense causal prefill attention over the paged KV pool, on the
// fifth-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// Replaces the per-request loop of AttentionBackend.forward_extend
// (attention/base.py:71-93) over extend_attention (attention/ops.py:18-45):
// the reference gathers every request's K/V rows (k_buf[locs]), repeats them
// for the query heads of a group and calls SDPA with a causal mask.  Here one
// launch covers the whole extend batch and reads the rows in place through
// req_to_token; query t of request i (position prefix_i + t) attends to the
// keys of positions 0 .. prefix_i + t.
//
// Work unit (one CTA): a tile of 128 new tokens of one request x a pair of
// query heads of the same KV head group (32 / 4 heads: 16 pairs), so every
// K/V tile brought into shared memory serves two products.  Keys go in
// tiles of 64.
// Warp roles, 14 warps:
//   warps 0-3  softmax of head 0 of the pair (thread = query row = TMEM lane)
//   warps 4-7  softmax of head 1
//   warps 8-11 loaders: Q tiles once, then K_0 V_0 K_1 V_1 ... through a ring
//              of ten 16 KiB slots, 16-byte cp.async row gathers into the
//              128-byte-swizzled layouts the MMA descriptors name; each
//              thread's copies of a tile arrive on its barrier asynchronously
//              (cp.async.mbarrier.arrive), so the loaders never wait for data
//   warps 12-13 one per head: lane 0 issues that head's tcgen05.mma (one
//              issuing thread for both heads measured 0.76x as fast: the
//              issue of the small MMAs, not the tensor pipe, set the pace);
//              warp 12 also allocates the tensor memory
// Tensor memory (512 columns): per head h two score buffers S_h[0], S_h[1]
// (fp32 128 x 64) and the output O_h (fp32 128 x 128).
// MMA issue order of head h per key tile j (b = j mod 2): PV_h(j) S_h(j+2),
// with S_h(j+2) into the buffer the softmax of tile j just released, so the
// scores of the next tile are ready while a head's softmax of tile j runs.
// P_h(j) (bf16 pairs) replaces the first 32 columns of its score buffer and
// is the A operand of PV_h(j) straight from tensor memory; the MMAs run in
// issue order, so S_h(j+2) overwrites it only after PV_h(j) has read it.
// Shared memory holds Q and the K/V ring only.
// Softmax (exp2 domain, fp32): a row's running maximum is only raised when a
// tile's maximum exceeds it by more than 8 (a factor of 256); only then is
// O rescaled in TMEM (after PV_h(j-1) has completed: its commit barrier).
// Between raises the unscaled weights stay below 256, which bf16 P and the
// fp32 sums carry as well as any others.  A quarter of the exponentials are
// evaluated on the FMA pipe (exp2_fma) to relieve the MUFU pipe.
// Every wait on an mbarrier is bounded (kWaitLimitNs of %globaltimer); on
// expiry the CTA sets QQ_DEV_ERR_TIMEOUT, stops issuing work, waits for its
// own copies and MMAs, frees its tensor memory and returns.

#include <cmath>

#include "tcgen05.cuh"

namespace qq {
namespace {

using namespace tc;

constexpr int kPD = 128;                     // head_dim
constexpr int kPM = 128;                     // query rows per tile (MMA M)
constexpr int kPN = 64;                      // keys per tile (N of S, K of P.V)
constexpr int kQBytes = kPM * kPD * 2;       // 32 KiB: 128 rows x 256 bytes
constexpr int kQHalf = kQBytes / 2;          // one 64-column block of Q (128-byte rows)
constexpr int kKVBytes = kPN * kPD * 2;      // 16 KiB: 64 key rows x 256 bytes
constexpr int kKVHalf = kKVBytes / 2;        // one 64-column block of K or V
constexpr int kRing = 10;                    // K / V slots
constexpr int kSoftWarps = 8;
constexpr int kLoadWarps = 4;
constexpr int kMmaWarp = kSoftWarps + kLoadWarps;  // 12: the first of two MMA warps
constexpr int kThreads = (kMmaWarp + 2) * 32;      // 448: one MMA warp per head
constexpr int kOffQ = 0;
constexpr int kOffKV = 2 * kQBytes;
constexpr int kDynSmem = kOffKV + kRing * kKVBytes + 1024;  // + slack to align the base to 1024
constexpr uint32_t kTmemCols = 512;
constexpr float kRaise = 8.0f;  // log2 of the largest unscaled weight
constexpr int32_t kPastEnd = INT32_MIN;  // pool row of a key past the request's keys

// mbarrier slots: Q; ring full / empty (a slot is free once both heads'
// MMAs that read it are done: two commits); per head and buffer S full,
// P full; per head one arrival per finished P.V; per head the final commit
enum : int { kBarQ = 0, kBarFull = 1, kBarEmpty = kBarFull + kRing, kBarS = kBarEmpty + kRing,
             kBarP = kBarS + 4, kBarODone = kBarP + 4, kBarO = kBarODone + 2, kNumBars = kBarO + 2 };

struct PrefillArgs {
  const int64_t* req_idx;
  const int64_t* seq_lens;
  const int64_t* prefix_lens;
  const int64_t* tok_off;
  int bs;
  int64_t num_tokens;
  const int32_t* tiles;  // (batch entry << 16) | query tile, heaviest first
  const int32_t* r2t;
  int64_t r2t_stride;
  int64_t r2t_rows;      // 0: not checked
  const char* q;
  int64_t q_stride_bytes;
  const char* k_pool;
  const char* v_pool;
  int64_t row_bytes;
  int64_t num_rows;
  char* out;
  int64_t out_stride_bytes;
  int group;             // query heads per KV head (even)
  float scale_log2;      // scaling * log2(e)
  uint32_t* err;
};

// ------------------------------------------------------------------ PTX helpers

// 2^x on the FMA pipe, for x <= 8 (x below -125 gives ~2^-125 instead of 0,
// far below any row sum, which is >= 1): x = r + f with r = round(x), f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted here (relative error
// 7.5e-5, against bf16's 2^-9), 2^r added to the exponent bits.  The
// round-to-integer is the 1.5 * 2^23 shift: its low mantissa bits hold r,
// which (times 2^23) is the exponent increment.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  float p = fmaf(0.05517166f, f, 0.24261113f);
  p = fmaf(p, f, 0.69326097f);
  p = fmaf(p, f, 0.99992806f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// ------------------------------------------------------------------ the kernel

__global__ void __launch_bounds__(kThreads, 1) prefill_attn_kernel(PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  volatile int* abort_flag = &s_abort;

  // ---- the CTA's work: query tile `tile` of batch entry `entry`, heads h0, h0 + 1
  const int32_t code = a.tiles[blockIdx.y];
  const int entry = code >> 16, tile = code & 0xFFFF;
  const int h0 = 2 * (int)blockIdx.x;
  const int kvh = h0 / a.group;
  if (entry < 0 || entry >= a.bs) {
    if (threadIdx.x == 0) raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    return;
  }
  const int64_t L = a.seq_lens[entry], prefix = a.prefix_lens[entry];
  const int64_t n = L - prefix, t0 = (int64_t)tile * kPM;
  const int64_t req = a.req_idx[entry], tok0 = a.tok_off[entry];
  if (prefix < 0 || n <= 0 || t0 >= n || L > a.r2t_stride || req < 0 || (a.r2t_rows > 0 && req >= a.r2t_rows) ||
      tok0 < 0 || tok0 + n > a.num_tokens) {
    if (threadIdx.x == 0) raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    return;  // uniform over the CTA: nothing set up yet
  }
  const int64_t kv_end = min(L, prefix + t0 + kPM);  // keys [0, kv_end)
  const int nkv = (int)((kv_end + kPN - 1) / kPN);

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bar(kBarQ), kLoadWarps * 32);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(bar(kBarFull + i), kLoadWarps * 32);
      mbar_init(bar(kBarEmpty + i), 2);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar(kBarS + i), 1);
      mbar_init(bar(kBarP + i), 4 * 32);
    }
    mbar_init(bar(kBarODone + 0), 1);
    mbar_init(bar(kBarODone + 1), 1);
    mbar_init(bar(kBarO), 1);
    mbar_init(bar(kBarO + 1), 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&s_tmem), kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp >= kSoftWarps && warp < kMmaWarp) {
    // ================================================================ loaders
    const int lw = warp - kSoftWarps;
    const int chunk = lane & 15, half = lane >> 4;
    const uint32_t qdst = base + kOffQ;
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int r = lw * 32 + 2 * i + half;
        const bool ok = t0 + r < n;
        const char* src = a.q + (ok ? tok0 + t0 + r : 0) * a.q_stride_bytes + (int64_t)(h0 + hh) * (kPD * 2) + chunk * 16;
        cp_async_16_zfill(qdst + hh * kQBytes + sw128(r, chunk, kQHalf), src, ok ? 16u : 0u);
      }
    }
    cp_async_arrive(bar(kBarQ));

    // each warp moves 16 key rows of a tile: rows lw * 16 + 2 i + half, i < 8.
    // Keys past kv_end carry kPastEnd and are zero-filled.
    // Lanes 0-15 (and 16-31, the same) hold the pool rows of the warp's 16
    // keys of the current key tile; the next tile's are loaded one tile ahead.
    // Each thread's copies of a tile count on the tile's full barrier by an
    // asynchronous arrival (cp.async.mbarrier.arrive), so tiles are in flight
    // as deep as the ring allows, with no wait on the loaders' side.
    auto key_row = [&](int j) -> int32_t {
      const int64_t kp = (int64_t)j * kPN + lw * 16 + (lane & 15);
      return kp < kv_end ? __ldg(a.r2t + req * a.r2t_stride + kp) : kPastEnd;
    };
    int32_t row_next = key_row(0);
    int32_t myrow = kPastEnd;
    const int T = 2 * nkv;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      const int slot = t % kRing;
      if (t >= kRing &&
          !__all_sync(0xffffffffu, mbar_wait(bar(kBarEmpty + slot), ((t / kRing) - 1) & 1, abort_flag, a.err)))
        break;
      const bool is_v = (t & 1) != 0;
      if (!is_v) {
        const int j = t >> 1;
        myrow = row_next;
        row_next = j + 1 < nkv ? key_row(j + 1) : kPastEnd;
        if (myrow != kPastEnd && (myrow < 0 || myrow >= a.num_rows)) {
          raise_error(a.err, QQ_DEV_ERR_BOUNDS);
          myrow = 0;
        }
      }
      const char* pool = (is_v ? a.v_pool : a.k_pool) + (int64_t)kvh * (kPD * 2) + chunk * 16;
      const uint32_t dst = base + kOffKV + slot * kKVBytes;
#pragma unroll
      for (int i = 0; i < kPN / 8; ++i) {
        const int r = lw * 16 + 2 * i + half;
        const int32_t row = __shfl_sync(0xffffffffu, myrow, 2 * i + half);
        cp_async_16_zfill(dst + sw128(r, chunk, kKVHalf), pool + (int64_t)(row < 0 ? 0 : row) * a.row_bytes,
                          row >= 0 ? 16u : 0u);
      }
      cp_async_arrive(bar(kBarFull + slot));
    }
    cp_async_wait<0>();
  } else if (warp >= kMmaWarp) {
    // ================================================================ MMA issue
    if (lane == 0) {
      const int h = warp - kMmaWarp;  // this warp issues head h's MMAs
      constexpr uint32_t kIdQK = instr_desc(0, kPM, kPN);
      constexpr uint32_t kIdPV = instr_desc(1, kPM, kPD);
      auto tS = [&](int b) { return tmem + h * 256 + b * 64; };
      const uint32_t tO = tmem + h * 256 + 128;
      const uint64_t dq = desc_k(base + kOffQ + h * kQBytes);
      auto slot_addr = [&](int t) { return base + kOffKV + (uint32_t)(t % kRing) * kKVBytes; };
      auto qk = [&](int b, uint32_t ks) {
        const uint64_t dk = desc_k(ks);
        umma_bf16_x4(tS(b), dq, dk, 2, 2, kIdQK, 0u);
        umma_bf16_x4(tS(b), dq + (uint64_t)(kQHalf >> 4), dk + (uint64_t)(kKVHalf >> 4), 2, 2, kIdQK, 1u);
      };
      auto pv = [&](int b, uint32_t vs, bool acc) {
        umma_bf16_ts_x4(tO, tS(b), desc_mn(vs, kKVHalf), 8, (16 * 128) >> 4, kIdPV, acc ? 1u : 0u);
      };
      auto wait_full = [&](int t) {
        return mbar_wait(bar(kBarFull + t % kRing), (t / kRing) & 1, abort_flag, a.err);
      };
      bool ok = mbar_wait(bar(kBarQ), 0, abort_flag, a.err);
#pragma unroll 1
      for (int jj = 0; jj < 2 && jj < nkv && ok; ++jj) {
        ok = wait_full(2 * jj);
        if (!ok) break;
        tc_fence_after();
        qk(jj, slot_addr(2 * jj));
        umma_commit(bar(kBarS + 2 * h + jj));
        umma_commit(bar(kBarEmpty + (2 * jj) % kRing));
      }
#pragma unroll 1
      for (int j = 0; j < nkv && ok; ++j) {
        const int b = j & 1;
        const int tv = 2 * j + 1, tk = 2 * j + 4;
        const bool more = j + 2 < nkv;
        ok = wait_full(tv) && mbar_wait(bar(kBarP + 2 * h + b), (j >> 1) & 1, abort_flag, a.err);
        if (!ok) break;
        tc_fence_after();
        pv(b, slot_addr(tv), j > 0);
        umma_commit(bar(kBarODone + h));
        umma_commit(bar(kBarEmpty + tv % kRing));
        if (more) {
          ok = wait_full(tk);
          if (!ok) break;
          tc_fence_after();
          qk(b, slot_addr(tk));
          umma_commit(bar(kBarS + 2 * h + b));
          umma_commit(bar(kBarEmpty + tk % kRing));
        }
      }
      umma_commit(bar(kBarO + h));
      mbar_wait(bar(kBarO + h), 0, abort_flag, a.err, true);
    }
    __syncwarp();
  } else {
    // ================================================================ softmax (warps 0-7)
    const int hh = warp >> 2;  // head h0 + hh
    const int q4 = warp & 3;   // TMEM lanes 32 q4 .. 32 q4 + 31
    const int r = q4 * 32 + lane;
    const int64_t qpos = prefix + t0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16) + hh * 256;
    const uint32_t tO = lane_base + 128;
    const float sl2 = a.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    uint32_t v[64];
#pragma unroll 1
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarS + 2 * hh + b), (j >> 1) & 1, abort_flag, a.err));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = lane_base + b * 64;
      tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      const int64_t lim64 = qpos - (int64_t)j * kPN;  // columns c <= lim are visible to this row
      const int lim = lim64 > kPN - 1 ? kPN - 1 : (lim64 < -1 ? -1 : (int)lim64);
      const bool full = __all_sync(0xffffffffu, lim == kPN - 1);
      if (!full) {
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = e <= lim ? v[e] : __float_as_uint(-INFINITY);
      }
      float mx0 = __uint_as_float(v[0]), mx1 = __uint_as_float(v[1]);
#pragma unroll
      for (int e = 2; e < 64; e += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(v[e]));
        mx1 = fmaxf(mx1, __uint_as_float(v[e + 1]));
      }
      // raise the running maximum only past a factor of 2^8; tcgen05.ld / st
      // are warp-wide, so a warp rescales O when any of its rows needs it
      // (alpha = 1 for the others), once P.V of the previous tile is done
      const float mb = fmaxf(mx0, mx1) * sl2;
      const bool raise = mb > m_used + kRaise;
      float alpha = 1.f;
      if (raise) {
        if (j > 0) alpha = ex2(m_used - mb);
        m_used = mb;
      }
      l *= alpha;
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarODone + hh), (j - 1) & 1, abort_flag, a.err));
        if (!ok) break;
        tc_fence_after();
        uint32_t o[32];
#pragma unroll 1
        for (int c = 0; c < kPD / 32; ++c) {
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_st_wait();
      }
      // P = 2^(s * scale_log2 - m_used) as bf16 pairs over the first 32
      // columns of the score buffer; the row sum in fp32
      const float neg = -m_used;
      float l0 = 0.f, l1 = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int e2 = 0; e2 < 32; ++e2) {
        const float x0 = fmaf(__uint_as_float(v[2 * e2]), sl2, neg);
        const float x1 = fmaf(__uint_as_float(v[2 * e2 + 1]), sl2, neg);
        // one pair in four on the FMA pipe; masked (-inf) scores only through ex2
        const float p0 = ((e2 & 3) == 0 && full) ? exp2_fma(x0) : ex2(x0);
        const float p1 = ((e2 & 3) == 0 && full) ? exp2_fma(x1) : ex2(x1);
        l0 += p0;
        l1 += p1;
        pk[e2] = pack_bf16(p0, p1);
      }
      l += l0 + l1;
      tmem_st32(tS, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(kBarP + 2 * hh + b));
    }
    // ---- epilogue: O / l in the query dtype
    ok = __all_sync(0xffffffffu, ok && mbar_wait(bar(kBarO + hh), 0, abort_flag, a.err));
    tc_fence_after();
    const bool valid = ok && t0 + r < n;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    char* dst = a.out + (tok0 + t0 + r) * a.out_stride_bytes + (int64_t)(h0 + hh) * (kPD * 2);
#pragma unroll 1
    for (int c = 0; c < kPD / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tO + c * 32, o);
      tmem_ld_wait();
      if (valid) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 w;
          w.x = pack_bf16(__uint_as_float(o[8 * u + 0]) * inv, __uint_as_float(o[8 * u + 1]) * inv);
          w.y = pack_bf16(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv);
          w.z = pack_bf16(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv);
          w.w = pack_bf16(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 64 + u * 16) = w;
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

}  // namespace
}  // namespace qq

extern "C" int qq_extend_attention(const qq_extend_batch* batch, const qq_token_table* table,
                                   const int32_t* tiles, int num_tiles, const void* q, int dtype, int q_heads,
                                   int kv_heads, int head_dim, int64_t q_stride, const void* k_pool,
                                   const void* v_pool, int64_t kv_row_stride, int64_t num_rows, float scaling,
                                   void* out, int64_t out_stride, uint32_t* err, void* stream) {
  using namespace qq;
  if (batch == nullptr || table == nullptr || table->req_to_token == nullptr || q == nullptr ||
      k_pool == nullptr || v_pool == nullptr || out == nullptr || num_tiles < 0 || kv_heads <= 0 ||
      q_heads <= 0 || q_heads % kv_heads != 0 || num_rows <= 0 || table->stride <= 0)
    return QQ_ERR_INVALID;
  if (num_tiles == 0 || batch->bs == 0) return QQ_OK;
  if (tiles == nullptr || batch->bs < 0 || batch->req_pool_indices == nullptr || batch->seq_lens == nullptr ||
      batch->prefix_lens == nullptr || batch->token_offsets == nullptr)
    return QQ_ERR_INVALID;
  const int group = q_heads / kv_heads;
  // the tcgen05 kernel's geometry: bf16, head_dim 128, heads in pairs of one group
  if (dtype != QQ_BF16 || head_dim != kPD || group % 2 != 0 || q_heads / 2 > 65535 || num_tiles > 65535 ||
      batch->bs >= 32768 || (q_stride * 2) % 16 != 0 || (out_stride * 2) % 16 != 0 ||
      (kv_row_stride * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(q) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0 || reinterpret_cast<uintptr_t>(k_pool) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16 != 0)
    return QQ_ERR_UNSUPPORTED;
  PrefillArgs a{};
  a.req_idx = batch->req_pool_indices;
  a.seq_lens = batch->seq_lens;
  a.prefix_lens = batch->prefix_lens;
  a.tok_off = batch->token_offsets;
  a.bs = batch->bs;
  a.num_tokens = batch->num_tokens;
  a.tiles = tiles;
  a.r2t = table->req_to_token;
  a.r2t_stride = table->stride;
  a.r2t_rows = table->rows;
  a.q = static_cast<const char*>(q);
  a.q_stride_bytes = q_stride * 2;
  a.k_pool = static_cast<const char*>(k_pool);
  a.v_pool = static_cast<const char*>(v_pool);
  a.row_bytes = kv_row_stride * 2;
  a.num_rows = num_rows;
  a.out = static_cast<char*>(out);
  a.out_stride_bytes = out_stride * 2;
  a.group = group;
  a.scale_log2 = scaling * 1.4426950408889634f;
  a.err = err;
  static SmemLimit limit;
  const int rc = limit.ensure((const void*)prefill_attn_kernel, kDynSmem);
  if (rc != QQ_OK) return rc;
  dim3 grid(q_heads / 2, num_tiles);
  prefill_attn_kernel<<<grid, kThreads, kDynSmem, as_stream(stream)>>>(a);
  return launch_status();
}
