// [Q7] Split-K sparse decode attention over an explicit row list.
//
// Fast path (bf16, 4 KV heads, head_dim 128, 8 query heads per KV head):
// one launch, one 256-thread block per SM, every warp an independent
// pipeline over a stream-K split of the work.
//
// * Work space: the (request, KV head) segments in order, segment (i, h)
//   holding the n_i = min(seq_len_i, top_k) rows of request i; each warp of
//   the grid takes one contiguous, equal share of the flattened rows.  A
//   segment that lies inside one warp's share is finished by that warp and
//   written straight to the output; only the first and last segment of a
//   share can be split, so a warp writes at most two fp32 partials
//   (m, l, O), and the last warp to finish a split segment (an arrival
//   counter in the workspace) merges it.  Behind a fused selection the
//   kernel starts early and reads a request's rows once its ready word holds
//   the call's epoch.
// * Data movement: a warp gathers only its own KV head's 256-byte K and V
//   slices.  Per 16-row stage every lane reads the stage's 16 row indices
//   (four broadcast int4 loads) and issues 16 16-byte cp.async copies (one
//   commit group per stage) into a private ring of slots at a 272-byte row
//   pitch (ldmatrix reads are bank-conflict free).  Waits are per warp
//   (cp.async.wait_group): no block barrier in the loop.  Warps per block x
//   slots per warp are template parameters (8 x 3).
// * Math per stage:
//     S^T[16 rows x 8 heads] = K[16 x 128] . Q^T[128 x 8]   (8 x mma m16n8k16)
//     online softmax in fp32 (exp2 domain), P^T via movmatrix.trans
//     O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8]          (P as bf16 hi + lo: 16 mma)
//
// Generic path (any head_dim / group / fp32): one block per (request, KV
// head), scores in shared memory, two-pass softmax, fp32 FMA.

#include <cfloat>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace qq {
namespace {

// QQ_ATTN_FMA=1 builds the streaming kernel's per-stage contraction with fp32
// FMA instead of mma.sync (for the measured comparison of the two; the
// library ships the MMA build).
#ifndef QQ_ATTN_FMA
#define QQ_ATTN_FMA 0
#endif

// ------------------------------------------------------------------ fast path constants
constexpr int kD = 128;
constexpr int kKV = 4;
constexpr int kG = 8;
constexpr int kH = kKV * kG;
constexpr int kSlice = kD * 2;          // 256 bytes: one KV head of one row
constexpr int kPitch = kSlice + 16;     // 272
constexpr int kToks = 16;               // rows per stage (the MMA's M)

constexpr int kMinShare = 64;           // rows per warp at least
constexpr int kSlotBytes = 2 * kToks * kPitch;  // K slice tile + V slice tile: 8704
constexpr int kPartFloats = kG * kD + 2 * kG;   // one partial record: O [8][128], (m, l) [8]

struct AttnArgs {
  const int64_t* seq_lens;
  int bs;
  int top_k;
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
  float* part;        // [warps][2][kPartFloats]: the warps' records of split segments
  float* bpart;       // [blocks][2][kPartFloats]: the blocks' records of segments split across blocks
  int32_t* seg_count; // [bs * kKV] arrival counters (blocks) of segments split across blocks
  // fused selection + attention: rows of request i may be read once
  // ready[i] == epoch (the selection kernel runs ahead); null: the rows
  // were written before this launch.  The epoch is *call_counter + 1 (the
  // last block to exit advances the counter; exit_count: arrivals), or
  // fixed_epoch without a counter.  A wait gives up after wait_limit_ns.
  const uint32_t* ready;
  uint32_t* call_counter;
  int32_t* exit_count;
  uint32_t fixed_epoch;
  uint64_t wait_limit_ns;
};

// Request r's rows are written: lane 0 spins on its ready word (acquire,
// bounded), the warp barrier orders every lane's later reads after it.
// `known` is the last request this warp saw ready (warps visit requests in
// increasing order).
__device__ __forceinline__ void ensure_ready(const AttnArgs& a, uint32_t epoch, int r, int& known) {
  if (a.ready == nullptr || r == known) return;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.ready + r) : "memory");
      if (v == epoch) break;
      if (globaltimer_ns() - t0 > a.wait_limit_ns) {
        raise_error(a.err, QQ_DEV_ERR_TIMEOUT);
        break;
      }
      __nanosleep(100);
    }
  }
  __syncwarp();
  known = r;
}

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

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 x) {
  return *reinterpret_cast<const uint32_t*>(&x);
}

// 2^x by the hardware approximation (ex2.approx.ftz: relative error ~2^-22,
// results below 2^-126 flush to 0, 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

#define kNegInf (-__int_as_float(0x7f800000))

// ------------------------------------------------------------------ stream-K walk
//
// Flattened position p in [0, T), T = 4 * sum_i n_i: segment (i, h) covers
// [4 P_i + h n_i, 4 P_i + (h + 1) n_i) with P_i = sum_{j<i} n_j.  Warp w of
// NW owns [B(w), B(w + 1)), B(w) = floor(w T / NW) moved down to a 16-row
// stage boundary of its segment, so every stage starts at a multiple of 16
// rows into its segment (its row indices are four aligned int4 loads).  The
// fast path requires T < 2^31 (positions are int32).

struct Split {
  const int32_t* prefix4;  // shared: 4 * P_i, i = 0..bs
  int bs;
  int T;
  int NW;
  // segment containing p: largest i with prefix4[i] <= p, then the head
  __device__ __forceinline__ void seek(int p, int& req, int& head, int& n, int& seg_start) const {
    int lo = 0, hi = bs;  // prefix4[lo] <= p < prefix4[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix4[mid] <= p) lo = mid; else hi = mid;
    }
    req = lo;
    n = (prefix4[lo + 1] - prefix4[lo]) >> 2;
    head = (p - prefix4[lo]) / n;
    seg_start = prefix4[lo] + head * n;
  }
  __device__ __forceinline__ int begin(int w) const {
    if (w >= NW) return T;
    const int raw = (int)((int64_t)w * T / NW);
    if (raw == 0) return 0;
    int req, head, n, s0;
    seek(raw, req, head, n, s0);
    return s0 + ((raw - s0) & ~(kToks - 1));
  }
  // warp owning position p.  Shares are >= 64 rows before alignment, so the
  // aligned owner is the unaligned one or the next warp.
  __device__ __forceinline__ int owner(int p) const {
    int w = (int)(((int64_t)(p + 1) * NW - 1) / T);
    if (w + 1 < NW && begin(w + 1) <= p) ++w;
    return w;
  }
};

struct Walk {
  int begin;               // start of the share
  int pos, end;            // next position to issue, end of the share
  int req, head, n;        // current segment
  int seg_start;
  // the stage last produced by next():
  int r0, cnt;             // rows [r0, r0 + cnt) of segment (req, head); r0 % 16 == 0
  int stage_seg_start;
  int s_req, s_head, s_n;
  bool s_first, s_last;    // stage opens / closes this warp's portion of the segment
};

__device__ __forceinline__ void walk_init(const Split& sp, Walk& w, int warp_id) {
  w.begin = w.pos = sp.begin(warp_id);
  w.end = sp.begin(warp_id + 1);
  if (w.pos < w.end) sp.seek(w.pos, w.req, w.head, w.n, w.seg_start);
}

__device__ __forceinline__ bool walk_next(const Split& sp, Walk& w) {
  if (w.pos >= w.end) return false;
  const int seg_end = w.seg_start + w.n;
  const int stop = min(min(w.pos + kToks, seg_end), w.end);
  w.r0 = w.pos - w.seg_start;
  w.cnt = stop - w.pos;
  w.stage_seg_start = w.seg_start;
  w.s_req = w.req;
  w.s_head = w.head;
  w.s_n = w.n;
  w.s_first = w.r0 == 0 || w.pos == w.begin;
  w.s_last = stop == seg_end || stop == w.end;
  w.pos = stop;
  if (stop == seg_end && stop < w.end) {
    if (++w.head == kKV) {
      w.head = 0;
      ++w.req;
      // skip empty requests (seq_len 0 cannot occur in decode, kept for safety)
      while (w.req < sp.bs && sp.prefix4[w.req + 1] == sp.prefix4[w.req]) ++w.req;
      w.n = (sp.prefix4[w.req + 1] - sp.prefix4[w.req]) >> 2;
      w.seg_start = sp.prefix4[w.req];
    } else {
      w.seg_start += w.n;
    }
  }
  return true;
}

// Gather the head slices of the stage's rows into a ring slot: per row one
// warp instruction of 16-byte cp.async.cg copies, lanes 0-15 K bytes
// [16 l, 16 l + 16), lanes 16-31 V.  Every lane reads the stage's 16 row
// indices with four broadcast int4 loads; a row outside [0, num_rows) raises
// QQ_DEV_ERR_BOUNDS and is replaced by row 0.  Rows past the end of a short
// stage are zero-filled by the copy (0 * V stays 0).
// (256-byte bulk copies on an mbarrier measured slower for this gather.)
struct StageRows {
  uint32_t r[kToks];  // the stage's 16 row indices (every lane)
  uint32_t own;       // row threadIdx % 16 of the stage, 0 past cnt
};

__device__ __forceinline__ void load_stage_rows(const AttnArgs& a, const Walk& w, StageRows& s) {
  const int4* rp = reinterpret_cast<const int4*>(a.rows + (int64_t)w.s_req * a.top_k + w.r0);
#pragma unroll
  for (int i = 0; i < kToks / 4; ++i) {
    const int4 x = __ldg(rp + i);
    s.r[4 * i] = (uint32_t)x.x;
    s.r[4 * i + 1] = (uint32_t)x.y;
    s.r[4 * i + 2] = (uint32_t)x.z;
    s.r[4 * i + 3] = (uint32_t)x.w;
  }
  const int own = threadIdx.x & 15;
  s.own = own < w.cnt ? (uint32_t)__ldg(a.rows + (int64_t)w.s_req * a.top_k + w.r0 + own) : 0u;
}

__device__ __forceinline__ void copy_stage(const AttnArgs& a, const Walk& w, StageRows& s, const char* lane_pool,
                                           uint32_t lane_dst, uint32_t stride, uint32_t max_row) {
  const bool full = w.cnt == kToks;
  if (!full) {
#pragma unroll
    for (int k = 0; k < kToks; ++k) s.r[k] = k < w.cnt ? s.r[k] : 0u;
  }
  // lane l (< cnt) checks row l; the broadcast loads give every lane all 16
  if (__any_sync(0xffffffffu, s.own > max_row)) {
    raise_error(a.err, QQ_DEV_ERR_BOUNDS);
#pragma unroll
    for (int k = 0; k < kToks; ++k) s.r[k] = s.r[k] > max_row ? 0u : s.r[k];
  }
  const char* src = lane_pool + w.s_head * kSlice;
  if (full) {
#pragma unroll
    for (int k = 0; k < kToks; ++k) cp_async_16(lane_dst + k * kPitch, src + (size_t)s.r[k] * stride);
  } else {
#pragma unroll
    for (int k = 0; k < kToks; ++k)
      cp_async_16_zfill(lane_dst + k * kPitch, src + (size_t)s.r[k] * stride, k < w.cnt ? 16u : 0u);
  }
}

__device__ __forceinline__ void issue_stage(const AttnArgs& a, uint32_t epoch, const Walk& w, const char* lane_pool,
                                            uint32_t lane_dst, uint32_t stride, uint32_t max_row, int& known) {
  ensure_ready(a, epoch, w.s_req, known);
  StageRows s;
  load_stage_rows(a, w, s);
  copy_stage(a, w, s, lane_pool, lane_dst, stride, max_row);
}

template <int WARPS, int SLOTS>
struct StreamCfg {
  static_assert(SLOTS >= 2, "the ring overlaps the copy of one stage with the math of another");
  static constexpr int kThreads = WARPS * 32;
  static constexpr size_t kRing = (size_t)WARPS * SLOTS * kSlotBytes;
  static constexpr size_t kSmem = kRing + sizeof(int32_t) * (QQ_MAX_BS + 1);
};

// A segment split across warps, as the block's merge sees it.  A warp's (a
// block's) record of a segment is in slot 0 when the segment is the first
// of its share (range), else in slot 1: only the first warp (block) holding
// a record can have it in slot 1, the others' shares start inside it.
struct SegTask {
  int req, head;
  int wa, wb;     // this block's warps holding records of it
  int ba, bb;     // blocks holding records of it (ba < bb: it continues beyond this block)
  int slot_wa;    // slot of warp wa's record
  int slot_ba;    // slot of block ba's record
  int slot_here;  // slot of this block's record
};

// The block's list of split segments to merge, filled while the warps
// stream: the first of the block's warps that holds a record of a segment
// adds it when it finishes its portion (at most two per warp).
constexpr int kMaxTasks = 2 * kAttnWarpsPerSm;
struct BlockTasks {
  SegTask task[kMaxTasks];
  int n;
};

// One warp's share of the stream-K split: its stages through the warp's ring,
// whole segments written to the output, split ones as (m, l, O) records.
template <int WARPS, int SLOTS>
__device__ __forceinline__ void stream_share(const AttnArgs& a, uint32_t epoch, const Split& sp, int W, char* ring,
                                             BlockTasks& bt) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const __nv_bfloat16* qbase = static_cast<const __nv_bfloat16*>(a.q);

  // per-lane copy constants
  const char* lane_pool = (lane < 16 ? a.k_pool : a.v_pool) + (lane & 15) * 16;
  const uint32_t ring_dst = smem_u32(ring) + (lane < 16 ? 0 : kToks * kPitch) + (lane & 15) * 16;
  const uint32_t stride = (uint32_t)a.row_stride_bytes;
  const uint32_t max_row = (uint32_t)min(a.num_rows - 1, (int64_t)INT32_MAX);

  // cursors: fc copies into the ring, cc computes
  Walk fc, cc;
  walk_init(sp, fc, W);
  cc = fc;
  const int share_begin = fc.pos;
  bool have_f = walk_next(sp, fc);
  int fslot = 0;
  int known = -1;  // the last request seen ready
  {
    // the first stages' row indices are loaded together, then copied
    Walk pw[SLOTS - 1];
    StageRows pr[SLOTS - 1];
    bool ph[SLOTS - 1];
#pragma unroll
    for (int s = 0; s < SLOTS - 1; ++s) {
      ph[s] = have_f;
      if (have_f) {
        pw[s] = fc;
        ensure_ready(a, epoch, fc.s_req, known);
        load_stage_rows(a, fc, pr[s]);
        have_f = walk_next(sp, fc);
      }
    }
#pragma unroll
    for (int s = 0; s < SLOTS - 1; ++s) {
      if (ph[s]) copy_stage(a, pw[s], pr[s], lane_pool, ring_dst + fslot * kSlotBytes, stride, max_row);
      cp_async_commit();
      fslot = fslot + 1 == SLOTS ? 0 : fslot + 1;
    }
  }

  uint32_t qb[8][2];
  float acc[8][4];
  float m_a = kNegInf, m_b = kNegInf, l_a = 0.f, l_b = 0.f;
  int slot = 0;
  while (walk_next(sp, cc)) {
    if (cc.s_first) {
      // a new portion of a segment: Q^T fragments of this KV head, loaded
      // before the wait so their latency hides behind it
#if QQ_ATTN_FMA
      // query head gid, channels [32 tig, 32 tig + 32) as bf16 pairs
      const uint4* q4 = reinterpret_cast<const uint4*>(qbase + (int64_t)cc.s_req * a.q_stride +
                                                       (cc.s_head * kG + gid) * kD + 32 * tig);
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        const uint4 w = __ldg(q4 + c4);
        qb[2 * c4][0] = w.x;
        qb[2 * c4][1] = w.y;
        qb[2 * c4 + 1][0] = w.z;
        qb[2 * c4 + 1][1] = w.w;
      }
#else
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbase + (int64_t)cc.s_req * a.q_stride +
                                                               (cc.s_head * kG + gid) * kD);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[kk][0] = __ldg(qrow + (kk * 16 + 2 * tig) / 2);
        qb[kk][1] = __ldg(qrow + (kk * 16 + 8 + 2 * tig) / 2);
      }
#endif
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
      m_a = m_b = kNegInf;
      l_a = l_b = 0.f;
    }
    cp_async_wait<SLOTS - 2>();
    __syncwarp();  // the current stage is visible to every lane; the previous stage's slot is free
    if (have_f) {
      issue_stage(a, epoch, fc, lane_pool, ring_dst + fslot * kSlotBytes, stride, max_row, known);
      have_f = walk_next(sp, fc);
    }
    cp_async_commit();
    fslot = fslot + 1 == SLOTS ? 0 : fslot + 1;

    const int ntok = cc.cnt;
    const char* sk = ring + slot * kSlotBytes;
    const char* sv = sk + kToks * kPitch;
    slot = slot + 1 == SLOTS ? 0 : slot + 1;
#if QQ_ATTN_FMA
    // ---- the same stage with fp32 FMA instead of tensor-core MMA: lane ->
    // query head gid, channels [32 tig, 32 tig + 32); scores of the 16 rows
    // summed over the four lanes of a head, softmax per lane (the four
    // lanes of a head hold the same values), O^T in acc as 32 channels.
    {
      float sc[kToks];
#pragma unroll
      for (int r = 0; r < kToks; ++r) {
        const uint4* kr = reinterpret_cast<const uint4*>(sk + r * kPitch + tig * 64);
        float t = 0.f;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const uint4 w = kr[c4];
          const uint32_t kw[4] = {w.x, w.y, w.z, w.w};
          const uint32_t qw[4] = {qb[2 * c4][0], qb[2 * c4][1], qb[2 * c4 + 1][0], qb[2 * c4 + 1][1]};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            t = fmaf(__uint_as_float(kw[e] << 16), __uint_as_float(qw[e] << 16), t);
            t = fmaf(__uint_as_float(kw[e] & 0xFFFF0000u), __uint_as_float(qw[e] & 0xFFFF0000u), t);
          }
        }
        sc[r] = t;
      }
      float mx = kNegInf;
#pragma unroll
      for (int r = 0; r < kToks; ++r) {
        sc[r] += __shfl_xor_sync(0xffffffffu, sc[r], 1);
        sc[r] += __shfl_xor_sync(0xffffffffu, sc[r], 2);
        sc[r] = r < ntok ? sc[r] * a.scale_log2 : kNegInf;
        mx = fmaxf(mx, sc[r]);
      }
      const float mn = fmaxf(m_a, mx);
      const float base = mn == kNegInf ? 0.f : mn;
      if (mn != m_a) {
        const float al = fast_exp2(m_a - base);
        l_a *= al;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          acc[mt][0] *= al;
          acc[mt][1] *= al;
          acc[mt][2] *= al;
          acc[mt][3] *= al;
        }
      }
      m_a = mn;
#pragma unroll
      for (int r = 0; r < kToks; ++r) {
        const float pr = fast_exp2(sc[r] - base);
        l_a += pr;
        const uint4* vr = reinterpret_cast<const uint4*>(sv + r * kPitch + tig * 64);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const uint4 w = vr[c4];
          const uint32_t vw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float* o = &acc[2 * c4 + (e >> 1)][(e & 1) * 2];
            o[0] = fmaf(pr, __uint_as_float(vw[e] << 16), o[0]);
            o[1] = fmaf(pr, __uint_as_float(vw[e] & 0xFFFF0000u), o[1]);
          }
        }
      }
    }
#else
    // ---- S^T = K . Q^T
    // two accumulators (even / odd k-steps) halve the dependent MMA chain
    float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kaddr = smem_u32(sk + (lane & 15) * kPitch + (lane >> 4) * 16);
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldmatrix_x4(a0, a1, a2, a3, kaddr + kk * 32);
      ldmatrix_x4(b0, b1, b2, b3, kaddr + (kk + 1) * 32);
      mma_bf16_16816(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      mma_bf16_16816(c2, b0, b1, b2, b3, qb[kk + 1][0], qb[kk + 1][1]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] += c2[e];
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
    // a head whose running max is still -inf has seen only masked rows: its
    // weights are 0 and its (zero) accumulator needs no rescale
    const float base_a = mn_a == kNegInf ? 0.f : mn_a;
    const float base_b = mn_b == kNegInf ? 0.f : mn_b;
    const float p00 = fast_exp2(s00 - base_a), p10 = fast_exp2(s10 - base_a);
    const float p01 = fast_exp2(s01 - base_b), p11 = fast_exp2(s11 - base_b);
    if (__any_sync(0xffffffffu, mn_a != m_a || mn_b != m_b)) {
      const float al_a = fast_exp2(m_a - base_a), al_b = fast_exp2(m_b - base_b);
      l_a *= al_a;
      l_b *= al_b;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        acc[mt][0] *= al_a;
        acc[mt][1] *= al_b;
        acc[mt][2] *= al_a;
        acc[mt][3] *= al_b;
      }
    }
    m_a = mn_a;
    m_b = mn_b;
    l_a += p00 + p10;
    l_b += p01 + p11;
    // ---- P^T fragments (rows x heads -> heads x rows) and O^T += V^T . P^T,
    // P split into bf16 hi + lo parts (two MMAs per tile): the weights carry
    // ~16 mantissa bits and the fp32 result tracks an fp32 softmax-weighted sum
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(p00, p01);
    const __nv_bfloat162 h1 = __floats2bfloat162_rn(p10, p11);
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    const __nv_bfloat162 lo0 = __floats2bfloat162_rn(p00 - f0.x, p01 - f0.y);
    const __nv_bfloat162 lo1 = __floats2bfloat162_rn(p10 - f1.x, p11 - f1.y);
    const uint32_t pb0 = movmatrix_trans(bf162_bits(h0));
    const uint32_t pb1 = movmatrix_trans(bf162_bits(h1));
    const uint32_t pl0 = movmatrix_trans(bf162_bits(lo0));
    const uint32_t pl1 = movmatrix_trans(bf162_bits(lo1));
    const int j = lane >> 3, r = lane & 7;
    const uint32_t vaddr = smem_u32(sv + ((j >> 1) * 8 + r) * kPitch + (j & 1) * 16);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4_trans(a0, a1, a2, a3, vaddr + mt * 32);
      mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
      mma_bf16_16816(acc[mt], a0, a1, a2, a3, pl0, pl1);
    }
#endif
    if (!cc.s_last) continue;

    // ---- end of this warp's portion of segment (req, head)
    float la = l_a, lb = l_b;
#if !QQ_ATTN_FMA
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, o);
      lb += __shfl_xor_sync(0xffffffffu, lb, o);
    }
#endif
    const int seg0 = cc.stage_seg_start;
    const int seg1 = seg0 + cc.s_n;
    const int w_first = sp.owner(seg0), w_last = sp.owner(seg1 - 1);
    const int qh_a = cc.s_head * kG + 2 * tig, qh_b = qh_a + 1;  // this thread's query heads
    if (w_first == w_last) {
      // the whole segment is this warp's: normalize and write bf16
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)cc.s_req * a.out_stride;
#if QQ_ATTN_FMA
      const float inv = 1.f / la;
      __nv_bfloat16* oh = out + (cc.s_head * kG + gid) * kD + 32 * tig;
#pragma unroll
      for (int j = 0; j < 32; ++j) oh[j] = __float2bfloat16_rn(acc[j >> 2][j & 3] * inv);
#else
      const float inv_a = 1.f / la, inv_b = 1.f / lb;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d0 = mt * 16 + gid;
        out[qh_a * kD + d0] = __float2bfloat16_rn(acc[mt][0] * inv_a);
        out[qh_b * kD + d0] = __float2bfloat16_rn(acc[mt][1] * inv_b);
        out[qh_a * kD + d0 + 8] = __float2bfloat16_rn(acc[mt][2] * inv_a);
        out[qh_b * kD + d0 + 8] = __float2bfloat16_rn(acc[mt][3] * inv_b);
      }
#endif
      continue;
    }
    // split segment: record (m, l, O) in slot 0 (the share's first segment)
    // or 1; the block merges the records of its warps once they are all done
    const int rslot = seg0 <= share_begin ? 0 : 1;
    const int W0 = blockIdx.x * WARPS;
    if (lane == 0 && W == max(w_first, W0)) {
      // the first of this block's warps holding a record lists the segment
      const int ba = w_first / WARPS, bb = w_last / WARPS;
      const int slot_here = seg0 <= sp.begin(W0) ? 0 : 1;
      const int slot_ba = ba == (int)blockIdx.x ? slot_here : (seg0 <= sp.begin(ba * WARPS) ? 0 : 1);
      const int t = atomicAdd(&bt.n, 1);
      bt.task[t] = SegTask{cc.s_req, cc.s_head, W, min(w_last, W0 + WARPS - 1), ba, bb, rslot, slot_ba, slot_here};
    }
    float* rec = a.part + ((int64_t)W * 2 + rslot) * kPartFloats;
#if QQ_ATTN_FMA
#pragma unroll
    for (int j = 0; j < 32; ++j) rec[gid * kD + 32 * tig + j] = acc[j >> 2][j & 3];
    if (tig == 0) *reinterpret_cast<float2*>(rec + kG * kD + gid * 2) = make_float2(m_a, la);
#else
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d0 = mt * 16 + gid;
      rec[(2 * tig) * kD + d0] = acc[mt][0];
      rec[(2 * tig + 1) * kD + d0] = acc[mt][1];
      rec[(2 * tig) * kD + d0 + 8] = acc[mt][2];
      rec[(2 * tig + 1) * kD + d0 + 8] = acc[mt][3];
    }
    if (gid == 0) {
      float* ml = rec + kG * kD;
      ml[(2 * tig) * 2] = m_a;
      ml[(2 * tig) * 2 + 1] = la;
      ml[(2 * tig + 1) * 2] = m_b;
      ml[(2 * tig + 1) * 2 + 1] = lb;
    }
#endif
  }
}

// ------------------------------------------------------------------ merging split segments
//
// Once every warp of a block has finished its share (one block barrier),
// the block merges the records its warps wrote for each split segment, all
// 256 threads at once (two segments at a time, 128 threads each: thread
// -> query head (t % 128) / 16, channels 8 ((t % 128) % 16) .. + 8), so a
// merge is one round of loads.  A segment whose warps all belong to this
// block is finished here and written to the output.  One that continues
// into other blocks becomes a block record (the same (m, l, O) form) and
// the block arrives on the segment's counter (acq_rel atomic); the last
// block to arrive merges the block records the same way.  Merge order is
// fixed (records in warp / block order), so results do not depend on
// arrival order.

// Records r = 0 .. nr - 1 (rec(r) -> the record) merged for one query head
// and 8 channels: running max M, sum S = sum_r 2^(m_r - M) l_r, O likewise.
template <typename RecFn>
__device__ __forceinline__ void merge_records(int nr, int h, int c, RecFn rec, float& M, float& S, float (&o)[8]) {
  M = kNegInf;
  S = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = 0.f;
  for (int r0 = 0; r0 < nr; r0 += 8) {
    float2 ml[8];
    float4 x[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (r0 + j < nr) {
        const float* rw = rec(r0 + j);
        ml[j] = __ldcg(reinterpret_cast<const float2*>(rw + kG * kD + h * 2));
        const float4* src = reinterpret_cast<const float4*>(rw + h * kD + c);
        x[j][0] = __ldcg(src);
        x[j][1] = __ldcg(src + 1);
      } else {
        ml[j] = make_float2(kNegInf, 0.f);
        x[j][0] = x[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float Mb = M;
#pragma unroll
    for (int j = 0; j < 8; ++j) Mb = fmaxf(Mb, ml[j].x);
    if (Mb == kNegInf) continue;
    const float sc = fast_exp2(M - Mb);  // 0 while M is -inf (S and o are 0 then)
    S *= sc;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] *= sc;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = ml[j].x == kNegInf ? 0.f : fast_exp2(ml[j].x - Mb);
      S += f * ml[j].y;
      o[0] += f * x[j][0].x;
      o[1] += f * x[j][0].y;
      o[2] += f * x[j][0].z;
      o[3] += f * x[j][0].w;
      o[4] += f * x[j][1].x;
      o[5] += f * x[j][1].y;
      o[6] += f * x[j][1].z;
      o[7] += f * x[j][1].w;
    }
    M = Mb;
  }
}

// Final output of (request, KV head) = (req, head): O / S in bf16.
__device__ __forceinline__ void store_output(const AttnArgs& a, int req, int head, int h, int c, float S,
                                             const float (&o)[8]) {
  const float inv = 1.f / S;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)req * a.out_stride + (head * kG + h) * kD + c;
  uint4 v;
  __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
  __nv_bfloat162 p1 = __floats2bfloat162_rn(o[2] * inv, o[3] * inv);
  __nv_bfloat162 p2 = __floats2bfloat162_rn(o[4] * inv, o[5] * inv);
  __nv_bfloat162 p3 = __floats2bfloat162_rn(o[6] * inv, o[7] * inv);
  v.x = bf162_bits(p0);
  v.y = bf162_bits(p1);
  v.z = bf162_bits(p2);
  v.w = bf162_bits(p3);
  if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    *reinterpret_cast<uint4*>(out) = v;
  } else {  // the output row stride keeps 4-byte alignment only
    uint32_t* o32 = reinterpret_cast<uint32_t*>(out);
    o32[0] = v.x;
    o32[1] = v.y;
    o32[2] = v.z;
    o32[3] = v.w;
  }
}

__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <int WARPS>
__device__ void merge_block(const AttnArgs& a, const BlockTasks& bt) {
  static_assert(WARPS == kAttnWarpsPerSm, "two segments at a time, 128 threads x 8 channels each");
  __shared__ int s_last[2];
  const int tid = threadIdx.x;
  const int ntask = bt.n;
  const int half = tid >> 7, t7 = tid & 127;
  const int h = t7 >> 4, c = (t7 & 15) * 8;
  for (int t0 = 0; t0 < ntask; t0 += 2) {
    const int ti = t0 + half;
    const bool mine = ti < ntask;
    SegTask tk{};
    float M = kNegInf, S = 0.f, o[8];
    if (mine) {
      tk = bt.task[ti];
      // record of warp w for this segment: slot 0 when it is the warp's first segment
      merge_records(tk.wb - tk.wa + 1, h, c,
                    [&](int r) {
                      return a.part + ((int64_t)(tk.wa + r) * 2 + (r == 0 ? tk.slot_wa : 0)) * kPartFloats;
                    },
                    M, S, o);
      if (tk.ba == tk.bb) {
        store_output(a, tk.req, tk.head, h, c, S, o);
      } else {
        // the block record: slot 0 when the segment starts at or before this block's range
        float* rec = a.bpart + ((int64_t)blockIdx.x * 2 + tk.slot_here) * kPartFloats;
        float4* dst = reinterpret_cast<float4*>(rec + h * kD + c);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        if ((t7 & 15) == 0) *reinterpret_cast<float2*>(rec + kG * kD + h * 2) = make_float2(M, S);
      }
    }
    __syncthreads();  // the block records are written
    if (mine && t7 == 0 && tk.ba != tk.bb) {
      const int seg_id = tk.req * kKV + tk.head;
      const bool last = atom_add_acq_rel_gpu(&a.seg_count[seg_id], 1) == tk.bb - tk.ba;
      if (last) a.seg_count[seg_id] = 0;  // ready for the next launch
      s_last[half] = last;
    }
    __syncthreads();
    if (mine && tk.ba != tk.bb && s_last[half]) {
      merge_records(tk.bb - tk.ba + 1, h, c,
                    [&](int r) {
                      return a.bpart + ((int64_t)(tk.ba + r) * 2 + (r == 0 ? tk.slot_ba : 0)) * kPartFloats;
                    },
                    M, S, o);
      store_output(a, tk.req, tk.head, h, c, S, o);
    }
  }
}

// Every block read the call's epoch at its start; the last of the grid's
// blocks to exit (idle ones included) advances the call counter for the next call.
__device__ __forceinline__ void exit_arrival(const AttnArgs& a, uint32_t epoch) {
  if (a.call_counter == nullptr) return;  // a caller-given epoch
  if (atom_add_acq_rel_gpu(a.exit_count, 1) == (int)gridDim.x - 1) {
    *a.exit_count = 0;
    *a.call_counter = next_call_counter(epoch - 1);
  }
}

template <int WARPS, int SLOTS>
__global__ void __launch_bounds__(WARPS * 32, 1) attn_stream_kernel(AttnArgs a) {
  using Cfg = StreamCfg<WARPS, SLOTS>;
  // behind a fused selection the ready words order the reads instead of the
  // grid dependency; the selection's own wait keeps earlier grids ahead
  if (a.ready == nullptr) wait_prior_grid();
  allow_next_grid();
  extern __shared__ __align__(128) char smem[];
  __shared__ BlockTasks s_tasks;
  __shared__ uint32_t s_epoch;
  int32_t* s_prefix4 = reinterpret_cast<int32_t*>(smem + Cfg::kRing);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  char* ring = smem + (size_t)warp * SLOTS * kSlotBytes;
  if (threadIdx.x == 0) s_tasks.n = 0;
  // this call's epoch (the selection read the same counter value), by a
  // thread outside warp 0, whose prefix loads come first
  if (threadIdx.x == 32)
    s_epoch = a.ready == nullptr ? 0u : a.call_counter != nullptr ? ld_volatile_u32(a.call_counter) + 1 : a.fixed_epoch;

  // segment prefix 4 * P_i over the batch (warp 0, 32 requests at a time)
  if (warp == 0) {
    int32_t run = 0;
    for (int b0 = 0; b0 < a.bs; b0 += 32) {
      const int b = b0 + lane;
      int32_t n = 0;
      if (b < a.bs) {
        const int64_t L = a.seq_lens[b];
        n = (int32_t)(L < a.top_k ? (L < 0 ? 0 : L) : a.top_k);
      }
      int32_t incl = 4 * n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (b < a.bs) s_prefix4[b + 1] = run + incl;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_prefix4[0] = 0;
  }
  __syncthreads();

  Split sp;
  sp.prefix4 = s_prefix4;
  sp.bs = a.bs;
  sp.T = s_prefix4[a.bs];
  const uint32_t epoch = s_epoch;
  if (sp.T == 0) {
    if (a.ready != nullptr && threadIdx.x == 0) exit_arrival(a, epoch);
    return;
  }
  const int grid_warps = gridDim.x * WARPS;
  sp.NW = min(grid_warps, max(1, sp.T / kMinShare));
  const int W = blockIdx.x * WARPS + warp;
  if (blockIdx.x * WARPS >= sp.NW) {
    // the whole block is idle; it still counts as exited
    if (a.ready != nullptr && threadIdx.x == 0) exit_arrival(a, epoch);
    return;
  }
  if (W < sp.NW) stream_share<WARPS, SLOTS>(a, epoch, sp, W, ring, s_tasks);
  cp_async_wait<0>();
  __syncthreads();  // every warp's records are written and its segments listed
  merge_block<WARPS>(a, s_tasks);
  if (a.ready != nullptr && threadIdx.x == 0) exit_arrival(a, epoch);
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

int sm_count() { return device_sm_count(); }

}  // namespace
}  // namespace qq

namespace qq {
namespace {

template <int WARPS, int SLOTS>
int launch_stream_variant(const AttnArgs& a, cudaStream_t s) {
  static_assert(WARPS <= kAttnWarpsPerSm, "the workspace holds partial records for kAttnWarpsPerSm warps per SM");
  using Cfg = StreamCfg<WARPS, SLOTS>;
  static SmemLimit limit;  // per device
  const int rc = limit.ensure((const void*)attn_stream_kernel<WARPS, SLOTS>, Cfg::kSmem);
  if (rc != QQ_OK) return rc;
  return launch_pdl(attn_stream_kernel<WARPS, SLOTS>, dim3(sm_count()), dim3(Cfg::kThreads), Cfg::kSmem, s, a);
}

// 8 warps per block x 3 ring slots per warp: the measured best of the
// variants tried (6 x 4, 12 x 2, 16 x 1).
int launch_stream(const AttnArgs& a, cudaStream_t s) { return launch_stream_variant<8, 3>(a, s); }

}  // namespace
}  // namespace qq

using namespace qq;

extern "C" size_t qq_workspace_bytes(int max_bs, int top_k, int q_heads, int head_dim) {
  if (max_bs < 0 || top_k < 0 || q_heads < 0 || head_dim < 0) return 0;
  return workspace_end(sm_count()) + 256;
}

namespace qq {

// The geometry and alignment the streaming kernel handles (else the generic kernel runs).
bool stream_fast_path(int bs, int top_k, int dtype, int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                      const int32_t* rows, const void* k_pool, const void* v_pool, int64_t kv_row_stride,
                      const void* out, int64_t out_stride) {
  const int esz = dtype == QQ_BF16 ? 2 : 4;
  return dtype == QQ_BF16 && kv_heads == kKV && head_dim == kD && q_heads == kH &&
         (kv_row_stride * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(k_pool) % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(v_pool) % 16) == 0 && (q_stride % 2) == 0 && (out_stride % 2) == 0 &&
         (reinterpret_cast<uintptr_t>(out) % 4) == 0 && (int64_t)bs * top_k * kKV < (1ll << 31) &&
         top_k % kToks == 0 && (reinterpret_cast<uintptr_t>(rows) % 16) == 0 && kv_row_stride * esz < (1ll << 32);
}

// qq_sparse_decode_attention; with `ready` the streaming kernel reads a
// request's rows once ready[i] holds the call's epoch (see ensure_ready).
int sparse_decode_attention(const qq_batch* batch, int top_k, const void* q, int dtype, int q_heads,
                            int kv_heads, int head_dim, int64_t q_stride, const int32_t* rows,
                            const void* k_pool, const void* v_pool, int64_t kv_row_stride, int64_t num_rows,
                            float scaling, void* out, int64_t out_stride, uint32_t* err, void* workspace,
                            size_t workspace_bytes, void* stream, const uint32_t* ready, uint32_t* call_counter,
                            uint32_t fixed_epoch = 0, uint64_t wait_limit_ns = kWaitLimitNs) {
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
  a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kPartialOffset);
  a.bpart = a.part + attn_warp_partial_floats(sm_count());
  a.seg_count = ws_counters(workspace, kCounterAttn);
  cudaStream_t s = as_stream(stream);

  if (stream_fast_path(batch->bs, top_k, dtype, q_heads, kv_heads, head_dim, q_stride, rows, k_pool, v_pool,
                       kv_row_stride, out, out_stride)) {
    a.ready = ready;
    a.call_counter = call_counter;
    a.exit_count = call_counter != nullptr ? reinterpret_cast<int32_t*>(call_counter + 1) : nullptr;
    a.fixed_epoch = fixed_epoch;
    a.wait_limit_ns = wait_limit_ns;
    return launch_stream(a, s);
  }
  const int G = q_heads / kv_heads;
  const size_t smem = sizeof(float) * ((size_t)G * head_dim + (size_t)G * top_k + 2 * (size_t)G);
  if (smem > 200 * 1024) return QQ_ERR_UNSUPPORTED;
  dim3 grid(batch->bs, kv_heads);
  static SmemLimit limit_bf16, limit_f32;  // per device
  if (dtype == QQ_BF16) {
    const int rc = limit_bf16.ensure((const void*)attn_generic_kernel<__nv_bfloat16>, smem);
    if (rc != QQ_OK) return rc;
    attn_generic_kernel<__nv_bfloat16><<<grid, 128, smem, s>>>(a, q_heads, kv_heads, head_dim);
  } else {
    const int rc = limit_f32.ensure((const void*)attn_generic_kernel<float>, smem);
    if (rc != QQ_OK) return rc;
    attn_generic_kernel<float><<<grid, 128, smem, s>>>(a, q_heads, kv_heads, head_dim);
  }
  return launch_status();
}

int retrieve_topk(const qq_quest_state* st, int layer, const qq_batch* batch, const void* q, int q_dtype,
                  int q_heads, int64_t q_stride, int32_t* positions, int32_t* actual_lens, float* scores,
                  const qq_token_table* translate, int32_t* rows, const qq_new_token* nt, void* workspace,
                  size_t workspace_bytes, void* stream, uint32_t* ready, const uint32_t* call_counter,
                  uint32_t* err);

}  // namespace qq

extern "C" int qq_sparse_decode_attention(const qq_batch* batch, int top_k, const void* q, int dtype,
                                          int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                                          const int32_t* rows, const void* k_pool, const void* v_pool,
                                          int64_t kv_row_stride, int64_t num_rows, float scaling,
                                          void* out, int64_t out_stride, uint32_t* err, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return qq::sparse_decode_attention(batch, top_k, q, dtype, q_heads, kv_heads, head_dim, q_stride, rows, k_pool,
                                     v_pool, kv_row_stride, num_rows, scaling, out, out_stride, err, workspace,
                                     workspace_bytes, stream, nullptr, nullptr);
}

extern "C" int qq_sparse_decode_attention_ready(const qq_batch* batch, int top_k, const void* q, int dtype,
                                                int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                                                const int32_t* rows, const void* k_pool, const void* v_pool,
                                                int64_t kv_row_stride, int64_t num_rows, float scaling, void* out,
                                                int64_t out_stride, uint32_t* err, const uint32_t* ready,
                                                uint32_t epoch, uint64_t wait_limit_ns, void* workspace,
                                                size_t workspace_bytes, void* stream) {
  if (ready == nullptr || epoch == 0) return QQ_ERR_INVALID;
  return qq::sparse_decode_attention(batch, top_k, q, dtype, q_heads, kv_heads, head_dim, q_stride, rows, k_pool,
                                     v_pool, kv_row_stride, num_rows, scaling, out, out_stride, err, workspace,
                                     workspace_bytes, stream, ready, nullptr, epoch,
                                     wait_limit_ns == 0 ? kWaitLimitNs : wait_limit_ns);
}

extern "C" int qq_quest_decode_attention(const qq_quest_state* st, int layer, const qq_batch* batch,
                                         const void* q, int q_dtype, int q_heads, int64_t q_stride,
                                         int32_t* positions, int32_t* actual_lens, float* scores,
                                         const qq_token_table* translate, int32_t* rows,
                                         const qq_new_token* new_token, const void* k_pool,
                                         const void* v_pool, int64_t kv_row_stride, int64_t num_rows,
                                         float scaling, void* out, int64_t out_stride, uint32_t* err,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  if (st == nullptr || batch == nullptr || rows == nullptr || translate == nullptr) return QQ_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < qq_workspace_bytes(batch->bs, st->top_k, q_heads, st->head_dim))
    return QQ_ERR_WORKSPACE;
  // ready words only when the streaming kernel follows (the generic one is stream-ordered)
  const bool early = stream_fast_path(batch->bs, st->top_k, q_dtype, q_heads, st->kv_heads, st->head_dim, q_stride,
                                      rows, k_pool, v_pool, kv_row_stride, out, out_stride);
  char* ws = static_cast<char*>(workspace);
  uint32_t* ready = early ? reinterpret_cast<uint32_t*>(ws + ready_offset(sm_count())) : nullptr;
  uint32_t* counter = early ? reinterpret_cast<uint32_t*>(ws + epoch_offset(sm_count())) : nullptr;
  int rc = retrieve_topk(st, layer, batch, q, q_dtype, q_heads, q_stride, positions, actual_lens, scores,
                         translate, rows, new_token, workspace, workspace_bytes, stream, ready, counter, err);
  if (rc != QQ_OK) return rc;
  rc = sparse_decode_attention(batch, st->top_k, q, q_dtype, q_heads, st->kv_heads, st->head_dim, q_stride, rows,
                               k_pool, v_pool, kv_row_stride, num_rows, scaling, out, out_stride, err, workspace,
                               workspace_bytes, stream, ready, counter);
  if (rc != QQ_OK && early) {
    // the selection published this call's epoch but no attention will
    // advance the counter: clear the words so the next call cannot match them
    cudaMemsetAsync(ready, 0, sizeof(uint32_t) * QQ_MAX_BS, as_stream(stream));
  }
  return rc;
}

// ------------------------------------------------------------------ attention without a workspace
//
// Some callers cannot hand the library a workspace: an engine that reserves
// all device memory for its KV pool and activation arena before serving and
// allows no allocation on the decode path (an allocation there can block on
// the device or fragment the reserved region), or a host program that binds
// this C-ABI directly (cgo, JNI, ctypes) and has no device allocator of its
// own.  qq_sparse_decode_attention_noalloc serves them: the streaming
// kernel's scratch (arrival counters and split partials) lives in one
// fixed-size array compiled into this library, so a call allocates nothing.
//
// * Limits: at most QQ_NOALLOC_MAX_BS requests and the fast-path geometry
//   only (bf16, 32 query heads over 4 KV heads, head_dim 128, top_k a
//   multiple of 16); anything else returns QQ_ERR_UNSUPPORTED.  The grid is
//   capped at kNoAllocBlocks blocks, the number of blocks the partial
//   records are sized for.
// * Set-up: the first call on each device, made with that device current,
//   looks up the array's device address (cudaGetSymbolAddress) and sets the
//   kernel's shared-memory limit.  Make that first call before any stream
//   capture begins.
// * Each call clears the arrival counters it uses (an async memset on the
//   caller's stream) before the kernel runs; the partial records need no
//   clearing.
// * One array per device: calls that overlap on the same device (two
//   streams, or two host threads, with both kernels in flight) race on it
//   and give wrong results.  Order them on one stream.

namespace qq {

constexpr int kNoAllocBlocks = 148;
constexpr int kNoAllocWarps = 8;  // warps per block of the instantiation below
constexpr int kNoAllocSlots = 3;
constexpr size_t kNoAllocCounterBytes = sizeof(int32_t) * kKV * QQ_NOALLOC_MAX_BS;
constexpr size_t kNoAllocWarpPartialBytes = sizeof(float) * (size_t)kNoAllocBlocks * kNoAllocWarps * 2 * kPartFloats;
constexpr size_t kNoAllocPartialBytes = kNoAllocWarpPartialBytes + sizeof(float) * (size_t)kNoAllocBlocks * 2 * kPartFloats;
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;
static_assert(kNoAllocCounterBytes % 256 == 0, "partials start 256-byte aligned");
static_assert(kNoAllocScratchBytes == 11098624, "the size the header documents");

// 16 KiB of counters + 10.6 MiB of partial records, per warp and per block (11,098,624 bytes).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices];  // device address of the array, per device once set up

// Device address of the scratch array on the current device; the first call
// per device does the set-up.
int noalloc_setup(void** scratch) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return QQ_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return QQ_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return QQ_ERR_CUDA;
    using Cfg = StreamCfg<kNoAllocWarps, kNoAllocSlots>;
    if (cudaFuncSetAttribute(attn_stream_kernel<kNoAllocWarps, kNoAllocSlots>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem) != cudaSuccess)
      return QQ_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *scratch = g_noalloc_ptr[dev];
  return QQ_OK;
}

}  // namespace
}  // namespace qq

extern "C" int qq_sparse_decode_attention_noalloc(const qq_batch* batch, int top_k, const void* q, int dtype,
                                                  int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                                                  const int32_t* rows, const void* k_pool, const void* v_pool,
                                                  int64_t kv_row_stride, int64_t num_rows, float scaling,
                                                  void* out, int64_t out_stride, uint32_t* err, void* stream) {
  if (batch == nullptr || q == nullptr || rows == nullptr || k_pool == nullptr || v_pool == nullptr ||
      out == nullptr || top_k <= 0 || kv_heads <= 0 || head_dim <= 0 || q_heads % kv_heads != 0 ||
      num_rows <= 0)
    return QQ_ERR_INVALID;
  if (batch->bs == 0) return QQ_OK;
  if (batch->bs < 0 || batch->seq_lens == nullptr) return QQ_ERR_INVALID;
  if (batch->bs > QQ_NOALLOC_MAX_BS) return QQ_ERR_UNSUPPORTED;
  const int64_t row_bytes = kv_row_stride * 2;
  const bool geometry = dtype == QQ_BF16 && kv_heads == kKV && head_dim == kD && q_heads == kH &&
                        top_k % kToks == 0 && (int64_t)batch->bs * top_k * kKV < (1ll << 31) &&
                        row_bytes > 0 && row_bytes % 16 == 0 && row_bytes < (1ll << 32) &&
                        (reinterpret_cast<uintptr_t>(k_pool) % 16) == 0 &&
                        (reinterpret_cast<uintptr_t>(v_pool) % 16) == 0 &&
                        (reinterpret_cast<uintptr_t>(rows) % 16) == 0 && (q_stride % 2) == 0 &&
                        (out_stride % 2) == 0 && (reinterpret_cast<uintptr_t>(out) % 4) == 0;
  if (!geometry) return QQ_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  const int rc = noalloc_setup(&scratch);
  if (rc != QQ_OK) return rc;
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t) * kKV * (size_t)batch->bs, s) != cudaSuccess)
    return QQ_ERR_CUDA;
  AttnArgs a{};
  a.seq_lens = batch->seq_lens;
  a.bs = batch->bs;
  a.top_k = top_k;
  a.q = q;
  a.q_stride = q_stride;
  a.rows = rows;
  a.k_pool = static_cast<const char*>(k_pool);
  a.v_pool = static_cast<const char*>(v_pool);
  a.row_stride_bytes = row_bytes;
  a.num_rows = num_rows;
  a.scaling = scaling;
  a.scale_log2 = scaling * 1.4426950408889634f;
  a.out = out;
  a.out_stride = out_stride;
  a.err = err;
  a.seg_count = static_cast<int32_t*>(scratch);
  a.part = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoAllocCounterBytes);
  a.bpart = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoAllocCounterBytes + kNoAllocWarpPartialBytes);
  using Cfg = StreamCfg<kNoAllocWarps, kNoAllocSlots>;
  const int blocks = sm_count() < kNoAllocBlocks ? sm_count() : kNoAllocBlocks;
  attn_stream_kernel<kNoAllocWarps, kNoAllocSlots><<<blocks, Cfg::kThreads, Cfg::kSmem, s>>>(a);
  return launch_status();
}
