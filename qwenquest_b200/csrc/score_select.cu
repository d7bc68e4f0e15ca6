// [Q5][Q6][Q7] Quest page scoring, top-k page selection and the position
// layout, fused into one launch per layer.
//
// Persistent: one 512-thread block per SM (at most), walking work units with
// a stride of the grid.  A unit is one part of one request's pages: with a
// small batch a request's candidate pages are split evenly into `parts`
// ranges so that every SM streams bounds.  Within a unit each warp streams its own pages (page
// pg0 + warp + 16 m): lane l takes 16-byte words l, l + 32, ... of a page
// (four channels' (min, max) pairs each) so that its q̄ values stay in
// registers, and the sign of q̄ picks max or min by a byte permute.  For
// 512 channels the pages pass through a per-warp ring of RING slots in
// shared memory (cp.async, RING - 1 pages in flight); other widths load
// DEPTH pages per warp into registers.  There is no block barrier inside a
// unit: the only ones are around q̄ (computed once per unit, while the first
// pages are in flight) and the unit's end, where each warp's running top 32
// joins a merge tree and the block arrives on the request's counter in the
// workspace.  The last part of a request to arrive merges the parts' lists
// (or, beyond 32 selected pages, runs an 8-bit-per-pass radix select over
// the fp32 scores), then writes the position layout with the req_to_token
// reads in flight together; in a fused selection + attention call it then
// marks the request ready.

#include <type_traits>

#include "common.cuh"

namespace qq {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

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
  int64_t r2t_rows;  // 0: not checked
  int32_t* rows;
  uint32_t* err;     // optional: QQ_DEV_ERR_BOUNDS for a request index outside the state / table
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
  uint64_t* lists;  // per-part top-32 lists (workspace)
  int pages;      // page slots per request (max_pages, or num_pages): bounds the number of parts
  int parts;      // units per request: part j takes pages [j * pages / parts, (j + 1) * pages / parts)
  int units;      // bs * parts
  int score_all;  // page_scores API: score pages [0, num_pages) of every request, no selection
  int num_pages;
  uint32_t* ready;  // optional: ready[i] = epoch once request i's positions and rows are written
  const uint32_t* call_counter;  // with ready: this call's epoch is *call_counter + 1
};

// Request i's layout is written (by the whole block, before a barrier): its
// ready word takes this launch's epoch for a consumer that spins on it
// instead of waiting for the whole grid.  The barrier orders the block's
// writes before this thread's release store, which is cumulative over them.
__device__ __forceinline__ void publish_ready(const SelectArgs& a, int i, uint32_t epoch) {
  if (a.ready == nullptr) return;
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.ready + i), "r"(epoch) : "memory");
}

// Arrival of a part on request i's counter (acq_rel: the block's writes,
// ordered by the preceding barrier, are released; the last arriver's later
// reads of the other parts' writes are acquired).  True for the last part,
// which resets the counter for the next launch.
__device__ __forceinline__ bool arrive_last(int32_t* counter, int parts) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  const bool last = old == parts - 1;
  if (last) *counter = 0;
  return last;
}

// Dynamic shared memory of the selection: order keys of the candidate
// pages, then the selected pages, their keys and their score order.
inline size_t selection_smem(int max_pages, int sel) {
  return sizeof(uint32_t) * (size_t)max_pages +
         (sizeof(uint64_t) + 2 * sizeof(int32_t)) * (size_t)(sel > 0 ? sel : 0) + 16;
}

__device__ __forceinline__ uint32_t lane_mask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// q * bound + acc: for a bf16 query mean the product of two bf16 values is
// exact in fp32, so one fused multiply-add rounds exactly like the
// reference's product-then-sum; an fp32 mean keeps the separate rounding.
template <typename QT>
__device__ __forceinline__ float bound_fma(float q, float b, float acc) {
  if constexpr (std::is_same<QT, float>::value) return __fadd_rn(acc, __fmul_rn(q, b));
  else return __fmaf_rn(q, b, acc);
}

__device__ __forceinline__ uint64_t composite_key(float score, int64_t page) {
  return ((uint64_t)float_order_key(score) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)page);
}

__device__ __forceinline__ uint64_t shfl64(uint64_t v, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src), hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
  return ((uint64_t)hi << 32) | lo;
}

// A warp's running top-32 of distinct 64-bit keys, one per lane, descending
// (lane 0 the largest; 0 = empty).  Insert x, known to beat the smallest.
__device__ __forceinline__ void top32_insert(uint64_t& mine, uint64_t x, int lane) {
  const int pos = __popc(__ballot_sync(0xffffffffu, mine > x));  // keys that stay ahead of x
  const uint64_t up = shfl64(mine, lane > 0 ? lane - 1 : 0);
  mine = lane < pos ? mine : (lane == pos ? x : up);
}

// Top 32 of the union of two descending lists, descending: the element-wise
// max of a and reversed b is bitonic and holds the top 32; a bitonic
// half-cleaner cascade sorts it.
__device__ __forceinline__ uint64_t top32_merge(uint64_t a, uint64_t b, int lane) {
  const uint64_t br = shfl64(b, 31 - lane);
  uint64_t c = a > br ? a : br;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const uint64_t o = shfl64(c, lane ^ d);
    c = (lane & d) == 0 ? (c > o ? c : o) : (c < o ? c : o);
  }
  return c;
}

// Position layout of request i from the selected pages in score order
// (quest.py:453-459), or the dense layout 0 .. L-1 padded with L-1
// (quest.py:339-340); four positions per thread in flight so the
// req_to_token reads overlap.
__device__ void write_layout(const SelectArgs& a, int i, int64_t req, int64_t L, bool is_long, int sel,
                             const int32_t* s_order) {
  const qq_quest_state& st = a.st;
  const int tid = threadIdx.x;
  const int P = st.page_size;
  const int top_k = st.top_k;
  const int n = (int)(L < top_k ? L : top_k);
  if (a.actual_lens != nullptr && tid == 0) a.actual_lens[i] = n;
  int32_t* pos_out = a.positions + (int64_t)i * top_k;
  int32_t* rows_out = a.rows != nullptr ? a.rows + (int64_t)i * top_k : nullptr;
  const int32_t* r2t = a.r2t != nullptr ? a.r2t + req * a.r2t_stride : nullptr;
  const int64_t last = L > 0 ? L - 1 : 0;
  const int sel_req = top_k / P - 1;
  const int64_t rp0 = L - P > 0 ? L - P : 0;
  const int sp = sel_req * P;
  constexpr int kU = 4;
  for (int s0 = 0; s0 < top_k; s0 += kThreads * kU) {
    int64_t pos[kU];
    int32_t rv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int s = s0 + u * kThreads + tid;
      if (!is_long) {
        pos[u] = s < last ? s : last;
      } else if (s < sp) {
        const int b = s / P;
        const int32_t page = b < sel ? s_order[b] : (sel > 0 ? s_order[sel - 1] : 0);
        pos[u] = (int64_t)page * P + (s - b * P);
      } else {
        const int64_t r = rp0 + (s - sp);
        pos[u] = r < last ? r : last;
      }
    }
    if (rows_out != nullptr) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int s = s0 + u * kThreads + tid;
        rv[u] = (s < top_k && (is_long || s < n) && pos[u] < a.r2t_stride) ? __ldg(r2t + pos[u]) : 0;
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int s = s0 + u * kThreads + tid;
      if (s < top_k) {
        pos_out[s] = (int32_t)pos[u];
        if (rows_out != nullptr && (is_long || s < n)) rows_out[s] = rv[u];
      }
    }
  }
}

// The request's selection (any sel, by radix select) and position layout, by the whole block.
__device__ void select_request(const SelectArgs& a, int i, int64_t req, int64_t L, int64_t C, bool is_long,
                               unsigned char* smem, int* s_hist, int& s_digit, int& s_above, int& s_ngt) {
  const qq_quest_state& st = a.st;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P = st.page_size;
  const int top_k = st.top_k;
  const float* scores = a.scores + (int64_t)i * st.max_pages;
  const int sel_req = top_k / P - 1;
  const int sel = is_long ? (int)min((int64_t)sel_req, C) : 0;
  uint32_t* s_okey = reinterpret_cast<uint32_t*>(smem);
  int32_t* s_selp = reinterpret_cast<int32_t*>(s_okey + st.max_pages);
  uint64_t* s_selk = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uintptr_t>(s_selp + (sel_req > 0 ? sel_req : 0) + 1) & ~(uintptr_t)7);
  int32_t* s_order = reinterpret_cast<int32_t*>(s_selk + (sel_req > 0 ? sel_req : 0));

  if (sel > 0) {
    for (int64_t p = tid; p < C; p += kThreads) s_okey[p] = float_order_key(__ldcg(scores + p));
    // radix select, 8 bits a pass from the top: t = the sel-th largest order
    // key, `above` = keys greater than t
    uint32_t prefix = 0, mask = 0;
    int k = sel, above = 0;
    const int64_t c_round = (C + 31) / 32 * 32;  // whole warps for __match_any_sync
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) s_hist[tid] = 0;
      __syncthreads();
      for (int64_t p = tid; p < c_round; p += kThreads) {
        const bool in = p < C && (s_okey[p] & mask) == prefix;
        const uint32_t digit = in ? (s_okey[p] >> shift) & 255u : 256u;
        const uint32_t peers = __match_any_sync(0xffffffffu, digit);
        if (in && (__ffs(peers) - 1) == lane) atomicAdd(&s_hist[digit], __popc(peers));
      }
      __syncthreads();
      if (warp == 0) {
        int c8[8], tot = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          c8[e] = s_hist[255 - 8 * lane - e];
          tot += c8[e];
        }
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        int run = incl - tot;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run < k && k <= run + c8[e]) {
            s_digit = 255 - 8 * lane - e;
            s_above = run;
          }
          run += c8[e];
        }
      }
      __syncthreads();
      prefix |= (uint32_t)s_digit << shift;
      mask |= 255u << shift;
      above += s_above;
      k -= s_above;
    }
    // selected: every key above t, and the k lowest pages among keys equal to t
    if (tid == 0) s_ngt = 0;
    __syncthreads();
    for (int64_t p = tid; p < C; p += kThreads)
      if (s_okey[p] > prefix) s_selp[atomicAdd(&s_ngt, 1)] = (int32_t)p;
    if (warp == kWarps - 1) {
      int taken = 0;
      for (int64_t b = 0; b < C && taken < k; b += 32) {
        const int64_t p = b + lane;
        const bool eq = p < C && s_okey[p] == prefix;
        const uint32_t bal = __ballot_sync(0xffffffffu, eq);
        const int r = taken + __popc(bal & lane_mask_lt());
        if (eq && r < k) s_selp[above + r] = (int32_t)p;
        taken += __popc(bal);
      }
    }
    __syncthreads();
    // descending score, ties -> lower page (quest.py:452 topk order, stable)
    for (int c = tid; c < sel; c += kThreads) {
      const int32_t p = s_selp[c];
      s_selk[c] = ((uint64_t)s_okey[p] << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)p);
    }
    __syncthreads();
    for (int c = tid; c < sel; c += kThreads) {
      const uint64_t kc = s_selk[c];
      int rank = 0;
#pragma unroll 8
      for (int j = 0; j < sel; ++j) rank += s_selk[j] > kc;
      s_order[rank] = s_selp[c];
    }
    __syncthreads();
  }
  write_layout(a, i, req, L, is_long, sel, s_order);
}

// KW 16-byte words per lane and page; pages in flight per warp: DEPTH in
// registers, or with RING > 0 RING - 1 in a per-warp ring of RING page slots
// in shared memory filled by cp.async (each lane copies and reads only its
// own words, so the waits are per thread and no barrier is needed).
template <typename QT, int KW, int DEPTH, int RING = 0>
__global__ void __launch_bounds__(kThreads, 1) score_select_kernel(SelectArgs a) {
  constexpr int kQPerThread = QQ_MAX_CHANNELS / kThreads;  // query-mean channels per thread
  __shared__ float s_qbar[QQ_MAX_CHANNELS];
  __shared__ int s_hist[256];
  __shared__ uint64_t s_lists[2][kWarps][kSelectListLen];
  __shared__ int32_t s_top[kSelectListLen];
  __shared__ int s_digit, s_above, s_last, s_ngt;
  extern __shared__ __align__(16) unsigned char s_dyn[];  // the radix selection's keys and pages

  const qq_quest_state& st = a.st;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = st.kv_heads * st.head_dim;
  const int nvec = nch >> 2;
  const size_t page_words = (size_t)nvec;  // 16-byte words per page
  constexpr uint32_t kSlot = KW * 32 * 16;  // bytes of one page
  const uint32_t ring = smem_u32(s_dyn) + (uint32_t)warp * (RING > 0 ? RING : 1) * kSlot + lane * 16;

  // Before the grid wait: the block's first unit puts its warps' first
  // RING - 1 pages in flight into the ring.  The bounds do not depend on
  // the previous kernel (a fused attention, or the model's layers in an
  // engine): the step's bounds fold wrote them, and it completed before
  // that kernel started.  The previous attention's last blocks leave HBM
  // partly idle, so these copies cost its tail little.
  int pre_unit = -1;
  if constexpr (RING > 0) {
    if (!a.score_all && (int)blockIdx.x < a.units) {
      const int u = blockIdx.x, i = u / a.parts, j = u - (u / a.parts) * a.parts;
      const int64_t req = a.reqs[i], L = a.seq_lens[i];
      if (req >= 0 && req < st.max_reqs && !(a.r2t != nullptr && a.r2t_rows > 0 && req >= a.r2t_rows) &&
          L > st.top_k) {
        int64_t F = L / st.page_size;
        if (F > st.max_pages) F = st.max_pages;
        const int64_t C = st.avoid_recent_overlap ? (F > 0 ? F - 1 : 0) : F;
        const int64_t pg0 = (int64_t)j * C / a.parts, p_end = (int64_t)(j + 1) * C / a.parts;
        const uint4* bounds = reinterpret_cast<const uint4*>(st.page_bounds) +
                              ((size_t)a.layer * st.max_reqs + req) * st.max_pages * page_words;
        const int64_t pw0 = pg0 + warp;
        const int npages = p_end > pw0 ? (int)((p_end - pw0 + kWarps - 1) / kWarps) : 0;
#pragma unroll
        for (int d = 0; d < (RING > 0 ? RING - 1 : 0); ++d) {
          if (d < npages) {
            const uint4* src = bounds + (size_t)(pw0 + (int64_t)d * kWarps) * page_words;
#pragma unroll
            for (int it = 0; it < KW; ++it)
              if (lane + 32 * it < nvec) cp_async_16(ring + d * kSlot + it * 512, src + lane + 32 * it);
          }
          cp_async_commit();
        }
        pre_unit = u;
      }
    }
  }

  wait_prior_grid();
  // the call's epoch (thread 0 publishes): the counter is advanced only by
  // the previous call's attention (complete by now) and read by this call's
  // attention; the value is used only once a request is ready
  const uint32_t epoch = a.ready != nullptr && threadIdx.x == 0 ? ld_volatile_u32(a.call_counter) + 1 : 0u;
  allow_next_grid();
  const int G = a.q_heads / st.kv_heads;
  const int D = st.head_dim;
  const int sel_req = st.top_k / st.page_size - 1;
  // sel <= 32: every warp keeps the top 32 of its pages while it scores them
  const bool lists = !a.score_all && sel_req <= kSelectListLen;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const int i = u / a.parts, j = u - (u / a.parts) * a.parts;
    // request row, length and the query rows all in flight at once; a
    // request index outside the state (or the table) is reported and read
    // as slot 0, so every address stays inside its buffer
    const int64_t req_in = a.reqs[i];
    const bool req_bad = req_in < 0 || req_in >= st.max_reqs ||
                         (a.r2t != nullptr && a.r2t_rows > 0 && req_in >= a.r2t_rows);
    const int64_t req = req_bad ? 0 : req_in;
    if (req_bad && tid == 0 && j == 0) raise_error(a.err, QQ_DEV_ERR_BOUNDS);
    const int64_t L = a.score_all ? 0 : a.seq_lens[i];
    const QT* q = static_cast<const QT*>(a.q) + (int64_t)i * a.q_stride;
    // the new token's K/V words (part 0 writes them to the pool row below):
    // loaded here, with the query rows, so that their latency overlaps
    const bool nt_here = a.nt_k != nullptr && j == 0;
    const int64_t nt_dst_row = nt_here && a.nt_dst_rows != nullptr ? a.nt_dst_rows[i] : -1;
    uint32_t nt_kw = 0, nt_vw = 0;
    if (nt_here && tid < a.nt_row_words) {
      nt_kw = a.nt_k[i * a.nt_src_stride_words + tid];
      nt_vw = a.nt_v[i * a.nt_src_stride_words + tid];
    }
    float qsum[kQPerThread];
#pragma unroll
    for (int ci = 0; ci < kQPerThread; ++ci) {
      // q̄: the GQA mean in the query dtype (quest.py:390), fp32 sum over the
      // group in head order, eight loads in flight at a time
      const int c = tid + ci * kThreads;
      qsum[ci] = 0.f;
      if (c < nch) {
        const int h = c / D, d = c - h * D;
        const QT* qc = q + (int64_t)h * G * D + d;
        int g = 0;
        for (; g + 8 <= G; g += 8) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = Elem<QT>::load(qc + (int64_t)(g + e) * D);
#pragma unroll
          for (int e = 0; e < 8; ++e) qsum[ci] = __fadd_rn(qsum[ci], v[e]);
        }
        for (; g < G; ++g) qsum[ci] = __fadd_rn(qsum[ci], Elem<QT>::load(qc + (int64_t)g * D));
      }
    }
    int64_t F, C;
    bool is_long;
    if (a.score_all) {
      F = C = a.num_pages;
      is_long = true;
    } else {
      F = L / st.page_size;
      if (F > st.max_pages) F = st.max_pages;  // seq_len beyond max_context_len: never index past the slot
      C = st.avoid_recent_overlap ? (F > 0 ? F - 1 : 0) : F;
      is_long = L > st.top_k;
    }
    // candidate pages of this part: [pg0, p_end), an even split of the request's own candidates
    // (not of its page slots, which a long context limit would leave mostly to part 0)
    const int64_t pg0 = is_long ? (int64_t)j * C / a.parts : 0;
    const int64_t p_end = is_long ? (int64_t)(j + 1) * C / a.parts : 0;
    float* scores = a.scores + (int64_t)i * st.max_pages;
    const uint4* bounds = reinterpret_cast<const uint4*>(st.page_bounds) +
                          ((size_t)a.layer * st.max_reqs + req) * st.max_pages * page_words;

    // the first DEPTH (RING - 1) pages of this warp in flight
    uint4 buf[RING > 0 ? 1 : DEPTH][KW];
    auto load_page = [&](uint4 (&w)[KW], int64_t p) {
      const uint4* src = bounds + (size_t)p * page_words;
#pragma unroll
      for (int it = 0; it < KW; ++it) {
        const int wi = lane + 32 * it;
        w[it] = wi < nvec ? ld_stream_u4(src + wi) : make_uint4(0, 0, 0, 0);
      }
    };
    const int64_t pw0 = pg0 + warp;
    const int npages = p_end > pw0 ? (int)((p_end - pw0 + kWarps - 1) / kWarps) : 0;  // this warp's pages
    const bool prefetched = u == pre_unit;  // its first RING - 1 pages are in flight already
    auto copy_page = [&](int slot, int64_t p) {
      const uint4* src = bounds + (size_t)p * page_words;
#pragma unroll
      for (int it = 0; it < KW; ++it)
        if (lane + 32 * it < nvec) cp_async_16(ring + slot * kSlot + it * 512, src + lane + 32 * it);
    };
    // With the ring one page per warp goes in flight before the query
    // loads are used, the others once q̄ is in registers: a deeper start
    // queues the query loads of every block behind the pages and delays the
    // first scores (measured).
    constexpr int kPre = 1;
    if constexpr (RING > 0) {
      if (!prefetched) {
#pragma unroll
        for (int d = 0; d < kPre; ++d) {
          if (d < npages) copy_page(d, pw0 + (int64_t)d * kWarps);
          cp_async_commit();
        }
      }
    } else {
#pragma unroll
      for (int d = 0; d < DEPTH; ++d)
        if (pw0 + d * kWarps < p_end) load_page(buf[d], pw0 + d * kWarps);
    }

    // (a) the new token's K/V into its pool row (quest_only.py:136-137, coordinator.py:226-228)
    if (nt_here) {
      const int64_t b = a.nt_buf;
      const int64_t dst = a.nt_dst_rows != nullptr ? nt_dst_row : req * (b + 1) + (L - 1 < b ? L - 1 : b);
      if (dst >= 0 && dst < a.nt_dst_num_rows) {
        if (tid < a.nt_row_words) {
          a.nt_k_dst[dst * a.nt_dst_stride_words + tid] = nt_kw;
          a.nt_v_dst[dst * a.nt_dst_stride_words + tid] = nt_vw;
        }
        for (int w = tid + kThreads; w < a.nt_row_words; w += kThreads) {
          a.nt_k_dst[dst * a.nt_dst_stride_words + w] = a.nt_k[i * a.nt_src_stride_words + w];
          a.nt_v_dst[dst * a.nt_dst_stride_words + w] = a.nt_v[i * a.nt_src_stride_words + w];
        }
      }
    }

    // (b) scores of the part's candidate pages
    uint64_t top = 0, top_min = 0;  // this warp's top 32 (lists), and its smallest
    if (pg0 < p_end) {
#pragma unroll
      for (int ci = 0; ci < kQPerThread; ++ci) {
        const int c = tid + ci * kThreads;
        if (c < nch) s_qbar[c] = G == 1 ? qsum[ci] : Elem<QT>::round(__fdiv_rn(qsum[ci], (float)G));
      }
      if constexpr (RING > 0) {
        if (!prefetched) {
#pragma unroll
          for (int d = kPre; d < RING - 1; ++d) {
            if (d < npages) copy_page(d, pw0 + (int64_t)d * kWarps);
            cp_async_commit();
          }
        }
      }
      __syncthreads();
      float qv[KW][4];
      uint32_t pick[KW][4];
#pragma unroll
      for (int it = 0; it < KW; ++it) {
        const int wi = lane + 32 * it;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          qv[it][e] = wi < nvec ? s_qbar[4 * wi + e] : 0.f;
          pick[it][e] = qv[it][e] >= 0.f ? 0x3244u : 0x1044u;  // high half (max) or low half (min)
        }
      }
      // one page's score: every lane ends with the same value
      auto page_score = [&](const uint4 (&w)[KW]) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int it = 0; it < KW; ++it) {
          acc[0] = bound_fma<QT>(qv[it][0], __uint_as_float(__byte_perm(w[it].x, 0u, pick[it][0])), acc[0]);
          acc[1] = bound_fma<QT>(qv[it][1], __uint_as_float(__byte_perm(w[it].y, 0u, pick[it][1])), acc[1]);
          acc[2] = bound_fma<QT>(qv[it][2], __uint_as_float(__byte_perm(w[it].z, 0u, pick[it][2])), acc[2]);
          acc[3] = bound_fma<QT>(qv[it][3], __uint_as_float(__byte_perm(w[it].w, 0u, pick[it][3])), acc[3]);
        }
        return __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
      };
      auto take_score = [&](float sum, int64_t p) {
        // butterfly sum over the lanes
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        if (lane == 0) scores[p] = sum;
        if (lists) {
          const uint64_t key = composite_key(sum, p);
          if (key > top_min) {
            top32_insert(top, key, lane);
            top_min = shfl64(top, 31);
          }
        }
      };
      if constexpr (RING > 0) {
        for (int k = 0; k < npages; ++k) {
          cp_async_wait<RING - 2>();  // page k is in its slot
          const int kn = k + RING - 1;
          if (kn < npages) copy_page(kn % RING, pw0 + (int64_t)kn * kWarps);
          cp_async_commit();
          uint4 w[KW];
#pragma unroll
          for (int it = 0; it < KW; ++it) {
            const uint32_t addr = ring + (k % RING) * kSlot + it * 512;
            if (lane + 32 * it < nvec)
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(w[it].x), "=r"(w[it].y), "=r"(w[it].z), "=r"(w[it].w)
                           : "r"(addr));
            else
              w[it] = make_uint4(0, 0, 0, 0);
          }
          take_score(page_score(w), pw0 + (int64_t)k * kWarps);
        }
      } else {
        for (int64_t pc = pw0; pc < p_end; pc += DEPTH * kWarps) {
#pragma unroll
          for (int d = 0; d < DEPTH; ++d) {
            const int64_t p = pc + d * kWarps;
            if (p < p_end) {
              const float sum = page_score(buf[d]);
              // the next page of this slot goes in flight before the reduction
              const int64_t pn = p + DEPTH * kWarps;
              if (pn < p_end) load_page(buf[d], pn);
              take_score(sum, p);
            }
          }
        }
      }
    }
    if (a.score_all) continue;
    // pages that are complete but not candidates read -inf (quest.py:450-451)
    if (is_long && j == a.parts - 1)
      for (int64_t p = C + tid; p < F; p += kThreads) scores[p] = -__int_as_float(0x7f800000);

    const int sel = is_long ? (int)min((int64_t)sel_req, C) : 0;
    if (lists) {
      // the block's top 32 of the warps' lists (a merge tree in shared memory)
      auto block_top32 = [&](uint64_t mine) {
        s_lists[0][warp][lane] = mine;
        __syncthreads();
        int cur = 0;
        for (int n = kWarps; n > 1; n >>= 1) {
          if (warp < n / 2)
            s_lists[cur ^ 1][warp][lane] =
                top32_merge(s_lists[cur][2 * warp][lane], s_lists[cur][2 * warp + 1][lane], lane);
          cur ^= 1;
          __syncthreads();
        }
        return s_lists[cur][0][lane];
      };
      top = block_top32(top);
      if (a.parts > 1) {
        // the req_to_token entries of this part's top pages go to L2 while
        // the parts arrive, for the last one's translation
        if (warp == 0 && a.r2t != nullptr && is_long && top != 0) {
          const int64_t page = (int64_t)(0xFFFFFFFFu - (uint32_t)(top & 0xFFFFFFFFu));
          const char* src = reinterpret_cast<const char*>(a.r2t + req * a.r2t_stride + page * st.page_size);
          for (int off = 0; off < 4 * st.page_size; off += 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(src + off));
        }
        // publish the part's list; the barrier and thread 0's acq_rel
        // arrival order every thread's writes before it, and the last
        // arriver's reads of the other lists after it
        if (warp == 0) a.lists[(size_t)u * kSelectListLen + lane] = top;
        __syncthreads();
        if (tid == 0) s_last = arrive_last(a.counters + i, a.parts);
        __syncthreads();
        if (!s_last) continue;
        const uint64_t* plist = a.lists + (size_t)i * a.parts * kSelectListLen + lane;
        if (a.parts <= 4) {
          // warp 0 merges its own list with the other parts' (loaded
          // together); with four parts the two merges that do not depend on
          // each other run side by side
          if (warp == 0) {
            uint64_t x[3];
#pragma unroll
            for (int e = 0; e < 3; ++e) {
              const int jj = e < j ? e : e + 1;  // the other parts
              x[e] = jj < a.parts ? __ldcg(plist + (size_t)jj * kSelectListLen) : 0ull;
            }
            uint64_t y = x[0];
            if (a.parts > 2) y = top32_merge(x[0], x[1], lane);
            if (a.parts > 3) top = top32_merge(top, x[2], lane);
            top = top32_merge(top, y, lane);
          }
        } else {
          // warp w takes lists w, w + 16, ... (four loads in flight at a
          // time; only real lists are merged, the first one taken as it is),
          // then the merge tree joins the warps
          uint64_t mine = 0;
          bool have = false;
          for (int j0 = warp; j0 < a.parts; j0 += 4 * kWarps) {
            uint64_t x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int jj = j0 + e * kWarps;
              x[e] = jj < a.parts ? __ldcg(plist + (size_t)jj * kSelectListLen) : 0ull;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (j0 + e * kWarps < a.parts) {
                mine = have ? top32_merge(mine, x[e], lane) : x[e];
                have = true;
              }
            }
          }
          top = block_top32(mine);
        }
      }
      if (warp == 0 && lane < sel) s_top[lane] = (int32_t)(0xFFFFFFFFu - (uint32_t)(top & 0xFFFFFFFFu));
      __syncthreads();
      write_layout(a, i, req, L, is_long, sel, s_top);
      __syncthreads();  // s_lists and s_top are free again
      if (tid == 0) publish_ready(a, i, epoch);
      continue;
    }

    // (c) sel > 32: the block arrives on the request's counter; the last
    // part to arrive does the radix selection.
    __syncthreads();
    if (tid == 0) s_last = arrive_last(a.counters + i, a.parts);
    __syncthreads();
    if (s_last) select_request(a, i, req, L, C, is_long, s_dyn, s_hist, s_digit, s_above, s_ngt);
    __syncthreads();  // the selection's shared memory is free again
    if (s_last && tid == 0) publish_ready(a, i, epoch);
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

// Words per lane for nch channels (nch / 4 16-byte words per page).
int words_for(int nch) {
  const int nvec = nch / 4;
  return nvec <= 32 ? 1 : nvec <= 64 ? 2 : nvec <= 128 ? 4 : 8;  // nch <= QQ_MAX_CHANNELS = 1024
}

// Page slots of the shared-memory ring of the 4-word (512-channel) kernel:
// 5 pages (10 KiB) in flight per warp, 160 KiB per block.
constexpr int kRing4 = 6;

template <typename QT>
const void* kernel_for(int kw) {
  switch (kw) {
    case 1: return (const void*)score_select_kernel<QT, 1, 4>;
    case 2: return (const void*)score_select_kernel<QT, 2, 4>;
    case 4: return (const void*)score_select_kernel<QT, 4, 1, kRing4>;
    default: return (const void*)score_select_kernel<QT, 8, 1>;
  }
}

// Dynamic shared memory of the kernel for kw words per lane: the selection's
// buffers, or the ring (they are never in use together).
inline size_t select_dyn_smem(int kw, size_t selection) {
  const size_t ring = kw == 4 ? (size_t)kWarps * kRing4 * 4 * 32 * 16 : 0;
  return selection > ring ? selection : ring;
}

template <typename QT>
int launch_select(const SelectArgs& a, int grid, int kw, size_t smem, cudaStream_t s) {
  static SmemLimit limit[4];  // per kernel variant, per device
  const int ki = kw == 1 ? 0 : kw == 2 ? 1 : kw == 4 ? 2 : 3;
  smem = select_dyn_smem(kw, smem);
  const int rc = limit[ki].ensure(kernel_for<QT>(kw), smem);
  if (rc != QQ_OK) return rc;
  switch (kw) {
    case 1: return launch_pdl(score_select_kernel<QT, 1, 4>, dim3(grid), dim3(kThreads), smem, s, a);
    case 2: return launch_pdl(score_select_kernel<QT, 2, 4>, dim3(grid), dim3(kThreads), smem, s, a);
    case 4: return launch_pdl(score_select_kernel<QT, 4, 1, kRing4>, dim3(grid), dim3(kThreads), smem, s, a);
    default: return launch_pdl(score_select_kernel<QT, 8, 1>, dim3(grid), dim3(kThreads), smem, s, a);
  }
}

bool valid_state(const qq_quest_state* st) {
  return st != nullptr && st->page_bounds && st->num_layers > 0 && st->max_reqs > 0 &&
         st->max_pages > 0 && st->kv_heads > 0 && st->head_dim > 0 && st->page_size > 0 &&
         st->kv_heads * st->head_dim <= QQ_MAX_CHANNELS && (st->kv_heads * st->head_dim) % 4 == 0 &&
         reinterpret_cast<uintptr_t>(st->page_bounds) % 16 == 0;
}

int sm_count() { return device_sm_count(); }

// Units and grid of one launch over `pages` page slots per request: with a
// small batch every request is split into parts so that each SM streams
// bounds, and no block does two selections.
void plan_units(SelectArgs& a, int pages, int bs, int* grid) {
  int parts = sm_count() / (bs > 0 ? bs : 1);
  const int max_parts = pages / (2 * kWarps);  // at least two pages per warp and part
  if (parts > max_parts) parts = max_parts;
  if (parts < 1) parts = 1;
  a.pages = pages;
  a.parts = parts;
  a.units = parts * bs;
  *grid = a.units < sm_count() ? a.units : sm_count();
}

}  // namespace
}  // namespace qq

using namespace qq;

namespace qq {

// qq_quest_retrieve_topk, optionally publishing per-request ready words
// (ready[i] = epoch) for a consumer launched behind it.
int retrieve_topk(const qq_quest_state* st, int layer, const qq_batch* batch, const void* q, int q_dtype,
                  int q_heads, int64_t q_stride, int32_t* positions, int32_t* actual_lens, float* scores,
                  const qq_token_table* translate, int32_t* rows, const qq_new_token* nt, void* workspace,
                  size_t workspace_bytes, void* stream, uint32_t* ready, const uint32_t* call_counter,
                  uint32_t* err) {
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
  a.r2t_rows = translate ? translate->rows : 0;
  a.err = err;
  a.rows = rows;
  a.counters = ws_counters(workspace, kCounterSelect);
  a.lists = ws_select_lists(workspace);
  a.ready = ready;
  a.call_counter = call_counter;
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
  const size_t smem = selection_smem(st->max_pages, st->top_k / st->page_size - 1);
  if (smem > 200 * 1024) return QQ_ERR_UNSUPPORTED;
  int grid = 0;
  plan_units(a, st->max_pages, batch->bs, &grid);
  cudaStream_t s = as_stream(stream);
  const int kw = words_for(st->kv_heads * st->head_dim);
  if (q_dtype == QQ_BF16) return launch_select<__nv_bfloat16>(a, grid, kw, smem, s);
  return launch_select<float>(a, grid, kw, smem, s);
}

}  // namespace qq

extern "C" int qq_quest_retrieve_topk(const qq_quest_state* st, int layer, const qq_batch* batch,
                                      const void* q, int q_dtype, int q_heads, int64_t q_stride,
                                      int32_t* positions, int32_t* actual_lens, float* scores,
                                      const qq_token_table* translate, int32_t* rows,
                                      const qq_new_token* nt, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  return qq::retrieve_topk(st, layer, batch, q, q_dtype, q_heads, q_stride, positions, actual_lens, scores,
                           translate, rows, nt, workspace, workspace_bytes, stream, nullptr, nullptr, nullptr);
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
  if (q_dtype != QQ_BF16 && q_dtype != QQ_F32) return QQ_ERR_INVALID;
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
  int grid = 0;
  plan_units(a, num_pages, batch->bs, &grid);
  const int kw = words_for(st->kv_heads * st->head_dim);
  cudaStream_t s = as_stream(stream);
  if (q_dtype == QQ_BF16) return launch_select<__nv_bfloat16>(a, grid, kw, 0, s);
  return launch_select<float>(a, grid, kw, 0, s);
}
