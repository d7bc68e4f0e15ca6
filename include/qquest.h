/*
 * qquest.h — C ABI of the B200 Quest sparse-decode kernels (libqquest.so).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void*`, allocates nothing, and returns a status code
 * (QQ_OK = 0, negative on argument errors).  Errors detected on the device
 * (hot buffer too small, a selected position without host backup, an index
 * out of range, a bounded wait that ran out) are OR-ed into a caller-owned
 * 32-bit error word (`err`, device or mapped pinned host memory) and the
 * offending request is left unmodified; the host maps them to the same
 * exception types the reference raises.
 *
 * Layouts are those of the reference (wengyinqi/QwenQuest, src/qwenquest):
 *   page bounds   bf16 [num_layers][max_reqs][max_pages][kv_heads][head_dim][2]
 *                 ([...][0] = min, [...][1] = max; sentinels +-bf16max)   quest.py:194-198
 *   running min/max bf16 [num_layers][max_reqs][kv_heads][head_dim]       quest.py:200-206
 *   counters      int32 [max_reqs]                                        quest.py:207-208
 *   req_to_token  int32 [max_reqs][max_context_len]                       memory.py:35-37
 *   K / V pool    [rows][kv_heads][head_dim] per layer, row 0 = padding   memory.py:96-103
 *   hot buffer    [max_reqs * (buf + 1)][kv_heads][head_dim] per layer    coordinator.py:116-126
 *   buffer_tokens / lru_slots int32 [num_layers][max_reqs][buf]           coordinator.py:127-131
 *
 * Workspace: entry points that take `workspace` need qq_workspace_bytes()
 * bytes of device memory, zero-filled once when allocated; the kernels leave
 * its counters at zero again when they finish.  Calls that share one
 * workspace must be ordered on one stream.
 */
#ifndef QQUEST_H
#define QQUEST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host) ---------------------------------------------- */
#define QQ_OK 0
#define QQ_ERR_INVALID (-1)     /* bad argument -> ValueError                     */
#define QQ_ERR_UNSUPPORTED (-2) /* geometry beyond a documented limit -> ValueError */
#define QQ_ERR_CUDA (-3)        /* a CUDA launch failed -> RuntimeError             */
#define QQ_ERR_WORKSPACE (-4)   /* workspace too small -> ValueError                */

/* ---- device error bits (OR-ed into *err) ------------------------------ */
#define QQ_DEV_ERR_CAPACITY 1u       /* device_buffer_size too small for this top-k -> RuntimeError */
#define QQ_DEV_ERR_NO_HOST_BACKUP 2u /* selected position without host backup -> AssertionError     */
#define QQ_DEV_ERR_BOUNDS 4u         /* an index out of range was skipped -> RuntimeError            */
#define QQ_DEV_ERR_TIMEOUT 8u        /* a bounded wait ran out -> RuntimeError                       */

/* ---- dtypes ----------------------------------------------------------- */
#define QQ_BF16 0
#define QQ_F32 1

/* ---- limits ----------------------------------------------------------- */
#define QQ_MAX_LAYERS 128  /* per-layer pointers travel inside the kernel parameters */
#define QQ_MAX_BS 4096     /* requests per call                                       */
#define QQ_MAX_CHANNELS 1024 /* kv_heads * head_dim                                   */

/* Quest state of QuestAlgorithm.init_storage (quest.py:171-209). */
typedef struct qq_quest_state {
  uint16_t* page_bounds;
  uint16_t* running_min;
  uint16_t* running_max;
  int32_t* running_token_count;
  int32_t* running_page_idx;
  int32_t num_layers;
  int32_t max_reqs;
  int32_t max_pages;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t page_size;
  int32_t top_k;
  int32_t avoid_recent_overlap;
} qq_quest_state;

/* The decode batch of ForwardBatch (batch.py:38-64). */
typedef struct qq_batch {
  const int64_t* req_pool_indices; /* device [bs] */
  const int64_t* seq_lens;         /* device [bs]; counts the token being decoded */
  int32_t bs;
} qq_batch;

/* Where a row of the attended pool comes from. */
typedef struct qq_token_table {
  const int32_t* req_to_token; /* device [rows][stride] */
  int64_t stride;
  int64_t rows;                /* request rows of the table; a request index outside [0, rows)
                                  is reported as QQ_DEV_ERR_BOUNDS (0: not checked) */
} qq_token_table;

/* The new token's K/V write fused into qq_quest_retrieve_topk.
 * Destination row of request i: dst_rows[i] (Mode 2, out_cache_loc) or,
 * when dst_rows is NULL, req * (buf + 1) + min(seq_len - 1, buf)
 * (Mode 3 newest slot, coordinator.py:178-181). */
typedef struct qq_new_token {
  const void* k;          /* device [bs][kv_heads*head_dim], pool dtype */
  const void* v;
  int64_t src_stride;     /* elements between requests */
  void* k_dst;            /* layer base of the destination pool */
  void* v_dst;
  int64_t dst_row_stride; /* elements between rows */
  const int64_t* dst_rows;
  int64_t device_buffer_size;
  int64_t dst_num_rows;   /* rows of the destination pool; rows outside are skipped */
  int32_t dtype;
} qq_new_token;

/* HiSparse state of HiSparseCoordinator (coordinator.py:74-134). */
typedef struct qq_hisparse_state {
  int32_t* buffer_tokens;
  int32_t* lru_slots;
  int32_t* req_to_host_pool; /* device [max_reqs][max_context_len], -1 = no backup */
  unsigned long long* stats; /* device [3]: hits, misses, fast_path_calls */
  int32_t num_layers;
  int32_t max_reqs;
  int32_t max_context_len;
  int32_t device_buffer_size;
  int32_t top_k;
} qq_hisparse_state;

/* ---- introspection ---------------------------------------------------- */
/* Device address of pinned host memory (cudaHostGetDevicePointer); the
 * HiSparse host tier is read and written by kernels through it. */
int qq_host_device_pointer(const void* host_ptr, void** device_ptr);
const char* qq_version(void);
const char* qq_status_string(int status);
/* Workspace bytes for calls with up to max_bs requests (any of the calls
 * below that take a workspace; one workspace may serve all of them when
 * the calls are ordered on one stream). */
size_t qq_workspace_bytes(int max_bs, int top_k, int q_heads, int head_dim);

/* ---- storage initialisation ------------------------------------------ */
/* Fill bounds and running bounds with the +-bf16max sentinels and zero the
 * counters.  Replaces QuestAlgorithm.init_storage fills (quest.py:196-208). */
int qq_quest_init_storage(const qq_quest_state* st, void* stream);

/* Reset one request slot.  Replaces QuestAlgorithm.invalidate_request
 * (quest.py:468-479). */
int qq_quest_invalidate(const qq_quest_state* st, int req_pool_idx, void* stream);

/* ---- [Q2] prefill bounds ---------------------------------------------- */
/* Page bounds of one request's prefill keys for layers [layer_begin,
 * layer_end): full pages into page_bounds, a partial tail into the running
 * bounds, counters written when write_counters != 0.  k_layers is a HOST
 * array of (layer_end - layer_begin) device pointers.  Replaces
 * QuestAlgorithm.update_prefill_representations (quest.py:231-280), called
 * per layer by QuestOnlyBackend._update_quest_for_extend (quest_only.py:101-128)
 * and HiSparseCoordinator.admit_request (coordinator.py:169-172). */
int qq_quest_bounds_prefill(const qq_quest_state* st, int layer_begin, int layer_end,
                            const void* const* k_layers, int kv_dtype, int64_t k_row_stride,
                            const int32_t* prefill_indices, int prefill_len, int req_pool_idx,
                            int write_counters, void* stream);

/* ---- [Q2] + [H1] one prefill layer: K/V write, bounds, hot buffer ------ */
/* An extend batch (ForwardBatch in EXTEND mode, batch.py:38-64): request i
 * adds seq_lens[i] - prefix_lens[i] new tokens after prefix_lens[i] tokens
 * already in the pool; its new tokens are rows token_offsets[i] .. of k, v
 * and out_cache_loc. */
typedef struct qq_extend_batch {
  const int64_t* req_pool_indices; /* device [bs] */
  const int64_t* seq_lens;         /* device [bs]: prefix + new tokens */
  const int64_t* prefix_lens;      /* device [bs] (extend_prefix_lens) */
  const int64_t* token_offsets;    /* device [bs]: first new-token row of request i */
  const int64_t* out_cache_loc;    /* device [tokens]: pool row of each new token */
  int64_t num_tokens;              /* rows of k, v and out_cache_loc; rows past it are skipped */
  int32_t bs;
  int32_t max_seq_len;             /* >= every seq_lens[i]; sizes the grid */
} qq_extend_batch;

/* The HiSparse device tier of one layer (coordinator.py:120-128): position
 * pos < device_buffer_size of request req lives in row req * (buf + 1) + pos. */
typedef struct qq_hot_buffer {
  void* k;
  void* v;
  int64_t row_stride;         /* elements between rows */
  int64_t device_buffer_size; /* buf */
  int64_t num_rows;           /* rows of k / v; rows outside are skipped and reported */
} qq_hot_buffer;

/* One layer of an extend batch in one launch: the new tokens' K/V rows go
 * to k_pool / v_pool at out_cache_loc (set_kv_buffer, memory.py:114-120);
 * when st is given, layer `layer` of st gets the page bounds of positions
 * [0, seq_len) of every request (full pages into page_bounds, a partial tail
 * into the running bounds, counters written when write_counters != 0), as
 * QuestAlgorithm.update_prefill_representations (quest.py:231-280) computes
 * them after the last layer (QuestOnlyBackend._update_quest_for_extend,
 * quest_only.py:101-128); when hot is given, positions [0, buf) are copied
 * into the hot buffer, the device half of HiSparseCoordinator.admit_request
 * (coordinator.py:154-162).  Keys and values of positions below a request's
 * prefix come from the pool through table.  k / v: device
 * [tokens][row_elems] rows src_stride elements apart, in the pool dtype.
 * Rows and pointers 16-byte aligned use 16-byte moves, 4-byte aligned ones
 * 4-byte moves, anything else returns QQ_ERR_UNSUPPORTED.  Out-of-range rows
 * are skipped and set QQ_DEV_ERR_BOUNDS in err (nullable). */
int qq_quest_extend_kv(const qq_quest_state* st, int layer, int write_counters,
                       const qq_extend_batch* batch, const qq_token_table* table, const void* k,
                       const void* v, int dtype, int64_t row_elems, int64_t src_stride, void* k_pool,
                       void* v_pool, int64_t pool_row_stride, int64_t pool_rows, const qq_hot_buffer* hot,
                       uint32_t* err, void* stream);

/* ---- dense causal prefill attention (tcgen05) ------------------------- */
/* For every request i of an extend batch: out[token_offsets[i] + t] (t <
 * seq_lens[i] - prefix_lens[i]) = causal attention of q[token_offsets[i] + t]
 * (position prefix_lens[i] + t, q_heads x head_dim) over the keys and values
 * of positions 0 .. prefix_lens[i] + t, read in place from k_pool / v_pool
 * at rows table->req_to_token[req][pos]; query head h reads KV head
 * h / (q_heads / kv_heads); fp32 scores, softmax and accumulation, bf16
 * result.  tiles (device int32 [num_tiles]) lists the work as
 * (batch entry << 16) | t-tile (128 new tokens each), one entry per tile of
 * every request, heaviest first (qwenquest_b200.kernels.extend_tiles builds
 * it); each tile runs on one CTA per pair of query heads.  bf16, head_dim
 * 128, an even number of query heads per KV head, 16-byte aligned rows and
 * pointers, num_tiles <= 65535; anything else returns QQ_ERR_UNSUPPORTED.
 * Rows outside [0, num_rows) are read as row 0 and a batch entry whose
 * lengths do not fit the table or the token count is skipped, both reported
 * as QQ_DEV_ERR_BOUNDS in err (nullable).  Replaces the per-request loop of
 * AttentionBackend.forward_extend (attention/base.py:71-93) over
 * extend_attention (attention/ops.py:18-45). */
int qq_extend_attention(const qq_extend_batch* batch, const qq_token_table* table, const int32_t* tiles,
                        int num_tiles, const void* q, int dtype, int q_heads, int kv_heads, int head_dim,
                        int64_t q_stride, const void* k_pool, const void* v_pool, int64_t kv_row_stride,
                        int64_t num_rows, float scaling, void* out, int64_t out_stride, uint32_t* err,
                        void* stream);

/* ---- Qwen3-MoE expert block (tcgen05) ---------------------------------- */
/* The routing of a token batch as (token, slot) pairs grouped by expert:
 * pairs [expert_offsets[e], expert_offsets[e + 1]) belong to expert e, their
 * tokens ascending (the order torch.where gives the reference's loop);
 * pair_weight is each pair's routing weight in bf16; token_pairs[t][s] is the
 * pair of token t's slot s. */
typedef struct qq_moe_plan {
  const int32_t* pair_token;     /* device [num_pairs] */
  const int64_t* expert_offsets; /* device [num_experts + 1] */
  const uint16_t* pair_weight;   /* device [num_pairs], bf16 bits */
  const int32_t* token_pairs;    /* device [num_tokens][top_k] */
  int64_t num_tokens;
  int64_t num_pairs;
  int32_t top_k;
  int32_t num_experts;
} qq_moe_plan;

/* The plan of a small routing in one launch: experts and weights (bf16 bits)
 * are device [num_tokens][top_k] (torch.topk's indices and the cast
 * weights); writes pair_token, pair_weight, expert_offsets ([num_experts + 1])
 * and token_pairs as the qq_moe_plan struct describes them, pairs ascending by expert
 * and by token within an expert.  num_tokens * top_k <= 2048 and
 * num_experts <= 1024, else QQ_ERR_UNSUPPORTED (larger batches sort with a
 * library routine).  Replaces the grouping the reference's loop makes with
 * torch.unique / torch.where (model/qwen3_moe.py:141-142). */
int qq_moe_route_plan(const int64_t* experts, const uint16_t* weights, int64_t num_tokens, int top_k, int num_experts,
                      int32_t* pair_token, uint16_t* pair_weight, int64_t* expert_offsets, int32_t* token_pairs,
                      uint32_t* err, void* stream);

/* out[t] = sum over token t's pairs p (ascending expert) of
 * down_e(silu(gate_e(x[t])) * up_e(x[t])) * pair_weight[p], with the bf16
 * roundings of the reference's tensors (each projection's output, silu, the
 * product, the weighted output, and every add into out).  x, out: bf16
 * [tokens][hidden] rows x_stride / out_stride elements apart; w_gate / w_up
 * (each [inter][hidden]) and w_down ([hidden][inter]) are device arrays of
 * num_experts device pointers to row-major bf16 weights; h_buf (>= num_pairs x
 * inter bf16) and y_buf (>= num_pairs x hidden bf16) are caller-owned
 * scratch.  Three launches, no host synchronisation: the grouped GEMMs find
 * each tile's expert on the device.  hidden a multiple of 256, inter of 128,
 * top_k <= 16, num_experts <= 1024, 16-byte aligned rows; anything else
 * returns QQ_ERR_UNSUPPORTED.  A pair token or pair index out of range is
 * read as 0 / skipped and reported as QQ_DEV_ERR_BOUNDS in err (nullable).
 * Replaces the expert loop of Qwen3MoeSparseMoeBlock.forward
 * (model/qwen3_moe.py:139-147); the routing (qwen3_moe.py:133-138) is the
 * caller's. */
int qq_moe_experts(const qq_moe_plan* plan, const void* x, int64_t x_stride, int hidden, int inter,
                   const void* const* w_gate, const void* const* w_up, const void* const* w_down, void* h_buf,
                   void* y_buf, void* out, int64_t out_stride, uint32_t* err, void* stream);

/* ---- [Q3] per-step bounds fold + finalize ----------------------------- */
#define QQ_STEP_FOLD 1     /* running min/max <- key of the previous token */
#define QQ_STEP_FINALIZE 2 /* finalize pages whose 64th token arrived, advance counters */
/* For every request i of the batch whose skip flag is clear: fold the key of
 * its previous token into the running bounds of layers [layer_begin,
 * layer_end) and/or finalize.  The previous token's row is rows[i] when rows
 * is given (an entry of -1 takes no part: no fold, no finalize), else
 * req_to_token[req][max(seq_len-2,0)] when table is given,
 * else req * (buf + 1) + min(seq_len - 2, buf).  skip_flags (device [max_reqs],
 * nullable) are read and cleared.  Replaces
 * QuestOnlyBackend._do_quest_decode_step_update (quest_only.py:84-97),
 * QuestAlgorithm.update_decode_representations and
 * maybe_finalize_decode_representations (quest.py:284-321) and the bounds
 * part of HiSparseCoordinator.prepare_decode_step (coordinator.py:199-209). */
int qq_quest_decode_step(const qq_quest_state* st, int flags, int layer_begin, int layer_end,
                         const void* const* k_layers, int kv_dtype, int64_t k_row_stride,
                         const qq_batch* batch, uint8_t* skip_flags, const int64_t* rows,
                         const qq_token_table* table, int64_t device_buffer_size,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---- [Q5] GQA grouping + page scores ---------------------------------- */
/* out[b][h][d] = mean over the group of q[b][h*G + g][d], in the query dtype.
 * Replaces QuestAlgorithm.group_queries (quest.py:366-391). */
int qq_quest_group_queries(const void* q, int dtype, int bs, int q_heads, int kv_heads,
                           int head_dim, int64_t q_stride, void* out, void* stream);

/* scores[b][p] = sum_{h,d} qg * (qg >= 0 ? kmax : kmin) in fp32 for pages
 * [0, num_pages) of layer `layer`, with qg the already grouped query
 * [bs][kv_heads][head_dim].  Replaces QuestAlgorithm.page_scores (quest.py:393-405). */
int qq_quest_page_scores(const qq_quest_state* st, int layer, const qq_batch* batch,
                         const void* grouped_q, int q_dtype, int64_t q_stride, int num_pages,
                         float* scores, void* stream);

/* ---- [Q5][Q6][Q7] fused score + top-k + layout + translation ---------- */
/* One launch per layer: GQA-mean of q, page scores of the candidate pages,
 * the top (top_k/page - 1) pages (descending score, ties -> lower page),
 * their positions followed by the recent window, or the dense layout when
 * seq_len <= top_k; optional req_to_token translation into rows and the
 * optional new-token K/V write.  scores (device [bs][max_pages]) receives
 * the fp32 scores of pages [0, seq_len/page) with -inf for pages that are
 * not candidates.  Replaces QuestAlgorithm.prepare_step + retrieve_topk
 * (quest.py:325-464), the req_to_token gather of QuestOnlyBackend.forward_decode
 * (quest_only.py:153-158) and set_kv_buffer / write_new_token
 * (memory.py:114-120, coordinator.py:217-228). */
int qq_quest_retrieve_topk(const qq_quest_state* st, int layer, const qq_batch* batch,
                           const void* q, int q_dtype, int q_heads, int64_t q_stride,
                           int32_t* positions, int32_t* actual_lens, float* scores,
                           const qq_token_table* translate, int32_t* rows,
                           const qq_new_token* new_token, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ---- [Q7] sparse decode attention ------------------------------------ */
/* out[b] = attention of q[b] ([q_heads][head_dim]) over the rows
 * rows[b][0 .. min(seq_len, top_k)) of k_pool / v_pool (duplicates counted),
 * fp32 softmax and accumulation, result in the query dtype.  The rows of
 * all requests are split into equal per-warp shares; segments cut by a
 * share boundary are merged in-kernel.  Replaces decode_attention
 * (attention/ops.py:48-66) as called by QuestOnlyBackend.forward_decode
 * (quest_only.py:153-158) and QuestHiSparseBackend.forward_decode
 * (quest_hisparse.py:128-132). */
int qq_sparse_decode_attention(const qq_batch* batch, int top_k, const void* q, int dtype,
                               int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                               const int32_t* rows, const void* k_pool, const void* v_pool,
                               int64_t kv_row_stride, int64_t num_rows, float scaling,
                               void* out, int64_t out_stride, uint32_t* err, void* workspace,
                               size_t workspace_bytes, void* stream);

/* The same attention with no workspace argument; it allocates nothing.  No
 * reference counterpart: the reference gets its attention scratch from
 * torch on every call.  This entry exists for callers that cannot allocate
 * device memory at call time — an engine that reserves all memory before it
 * serves and forbids allocations on its decode path, or a host program that
 * binds this C-ABI without a device allocator of its own.  Its scratch is a
 * fixed array inside the library (11,098,624 bytes per device: arrival
 * counters for QQ_NOALLOC_MAX_BS requests and partial records of the warps
 * and blocks of a grid of at most 148 blocks).  Fast-path geometry only (bf16, 32 query heads over
 * 4 KV heads, head_dim 128, top_k a multiple of 16, 16-byte aligned rows
 * and pools) and bs <= QQ_NOALLOC_MAX_BS; anything else returns
 * QQ_ERR_UNSUPPORTED.  The first call on a device, made with that device
 * current, does the set-up (looks up the array's address, sets the kernel's
 * shared-memory limit) and must come before any stream capture.  Every call
 * clears the counters it uses on `stream` first.  Calls that overlap on one
 * device share the array and race: keep them on one stream. */
#define QQ_NOALLOC_MAX_BS 1024
int qq_sparse_decode_attention_noalloc(const qq_batch* batch, int top_k, const void* q, int dtype,
                                       int q_heads, int kv_heads, int head_dim, int64_t q_stride,
                                       const int32_t* rows, const void* k_pool, const void* v_pool,
                                       int64_t kv_row_stride, int64_t num_rows, float scaling,
                                       void* out, int64_t out_stride, uint32_t* err, void* stream);

/* ---- [Q7] attention behind a caller's own producer ------------------- */
/* qq_sparse_decode_attention that may start before the rows are written: on
 * the fast path it reads request i's rows once ready[i] == epoch (an acquire
 * load), for a producer kernel launched just before it on `stream` that
 * writes the rows and then stores the word with release semantics (as the
 * selection of qq_quest_decode_attention does).  Each wait gives up after
 * wait_limit_ns of %globaltimer (0: 2 s), reports QQ_DEV_ERR_TIMEOUT in
 * `err` and reads the rows as they are; no wait can hang the GPU.  epoch
 * must not be 0 (a cleared word).  Other geometries run the generic kernel
 * after the producer, stream-ordered.  No reference counterpart: the
 * reference attends only after its selection has returned
 * (quest_only.py:153-158). */
int qq_sparse_decode_attention_ready(const qq_batch* batch, int top_k, const void* q, int dtype, int q_heads,
                                     int kv_heads, int head_dim, int64_t q_stride, const int32_t* rows,
                                     const void* k_pool, const void* v_pool, int64_t kv_row_stride,
                                     int64_t num_rows, float scaling, void* out, int64_t out_stride,
                                     uint32_t* err, const uint32_t* ready, uint32_t epoch,
                                     uint64_t wait_limit_ns, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* ---- [Q5][Q6][Q7] + [Q7] selection and attention in one call ---------- */
/* qq_quest_retrieve_topk (with the req_to_token translation into rows)
 * followed by qq_sparse_decode_attention over those rows, q_heads x
 * st->head_dim queries over st->kv_heads KV heads, both kernels sharing
 * `workspace`.  The results are those of the two calls.  On the attention
 * fast path the attention kernel starts while the selection still runs and
 * reads a request's rows as soon as that request's ready word in the
 * workspace holds this call's epoch, so its set-up and the selection's tail
 * overlap.  The epoch is a call counter kept in the workspace on the device
 * (the attention's last block advances it), so a call captured in a CUDA
 * graph gets a fresh epoch on every replay.  A request index outside the
 * state or the table is reported in `err` (QQ_DEV_ERR_BOUNDS).  No reference
 * counterpart: QuestOnlyBackend.forward_decode makes the two calls in turn
 * (quest_only.py:153-158). */
int qq_quest_decode_attention(const qq_quest_state* st, int layer, const qq_batch* batch,
                              const void* q, int q_dtype, int q_heads, int64_t q_stride,
                              int32_t* positions, int32_t* actual_lens, float* scores,
                              const qq_token_table* translate, int32_t* rows,
                              const qq_new_token* new_token, const void* k_pool, const void* v_pool,
                              int64_t kv_row_stride, int64_t num_rows, float scaling, void* out,
                              int64_t out_stride, uint32_t* err, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ---- [H3] HiSparse swap-in -------------------------------------------- */
/* For every request of the batch: fast path (seq_len <= buf: row = slot =
 * position) or first-occurrence dedupe, hit detection in LRU order,
 * eviction of the least recently used slots, copy of the misses from the
 * host tier (mapped pinned memory, read by the kernel), LRU rewrite
 * [stale evictables | loaded misses | hits] and rows_out[b][j] =
 * req * (buf + 1) + slot of positions[b][j].  Replaces
 * HiSparseCoordinator.swap_in_selected_pages / _swap_in_long
 * (coordinator.py:232-304). */
int qq_hisparse_swap_in(const qq_hisparse_state* hs, int layer, const qq_batch* batch,
                        const int32_t* positions, int32_t* rows_out, const void* host_k,
                        const void* host_v, void* dev_k, void* dev_v, int64_t row_bytes,
                        uint32_t* err, void* stream);

/* Reset one request slot: buffer_tokens = -1, lru_slots = 0..buf-1,
 * req_to_host_pool = -1.  Replaces the device part of
 * HiSparseCoordinator.request_finished (coordinator.py:312-314). */
int qq_hisparse_reset(const qq_hisparse_state* hs, int req_pool_idx, void* stream);

/* Admission layout: buffer_tokens[:, req, :] = lru_slots[:, req, :] = 0..buf-1
 * (coordinator.py:166-167). */
int qq_hisparse_admit_layout(const qq_hisparse_state* hs, int req_pool_idx, void* stream);

/* ---- [H1][H2][H4] host-tier rows handed out on the device ------------- */
/* The host tier's free rows as a ring in device memory, the role of the
 * reference's TokenToKVPoolAllocator over host indices (memory.py:53-76,
 * coordinator.py:117): allocation takes rows from the head in ring order,
 * freed rows go back at the tail, so rows come out in the reference's order
 * and no host round trip is needed.  state[0] = head, state[1] = tail
 * (allocation counts; free rows = tail - head). */
typedef struct qq_host_ring {
  int64_t* rows;     /* device [capacity] */
  int64_t* state;    /* device [2]: head, tail */
  int64_t capacity;  /* host rows 1 .. capacity */
} qq_host_ring;
/* All rows free, in order 1 .. capacity. */
int qq_host_ring_init(const qq_host_ring* ring, void* stream);
/* out[0 .. n) <- the next n free rows (TokenToKVPoolAllocator.alloc,
 * memory.py:64-70); fewer free: the rest are -1 and err gets
 * QQ_DEV_ERR_CAPACITY (the reference raises RuntimeError). */
int qq_host_ring_alloc(const qq_host_ring* ring, int64_t n, int64_t* out, uint32_t* err, void* stream);
/* Request req's host rows (req_to_host_pool[req] >= 0, in position order)
 * back to the ring, entries reset to -1 (coordinator.py:310-312). */
int qq_host_ring_free_request(const qq_hisparse_state* hs, int req_pool_idx, const qq_host_ring* ring,
                              void* stream);
/* [H2] The plan of HiSparseCoordinator.prepare_decode_step
 * (coordinator.py:183-215) on the device: for each batch entry i whose
 * request's skip flag (device [max_reqs], set at admission) is clear, the
 * previous token (position seq_len - 2) gets a new host row from the ring,
 * in batch order, recorded in req_to_host_pool; plan_dev[i] = its hot-buffer
 * row req * (buf + 1) + min(seq_len - 2, buf), plan_host[i] = the host row
 * (both -1 for an entry whose flag was set; the flag is cleared).  The bounds
 * fold (qq_quest_decode_step with rows = plan_dev) and the backup
 * (qq_copy_rows plan_dev -> plan_host, -1 entries skipped) follow. */
int qq_hisparse_plan_step(const qq_hisparse_state* hs, const qq_batch* batch, uint8_t* skip_flags,
                          const qq_host_ring* ring, int64_t* plan_dev, int64_t* plan_host, uint32_t* err,
                          void* stream);

/* ---- row copies (admission, eager backup) ----------------------------- */
/* For every (layer, i < n): dst_layers[layer][dst_idx[i]] <- src_layers[layer][src_idx[i]],
 * row_bytes bytes per row; strides in bytes; index arrays int32 or int64
 * (idx_is64 != 0); an entry with a negative index is skipped.  src/dst may
 * be device memory or mapped pinned host memory.  Used for HiSparse admission (coordinator.py:154-164) and the
 * eager host backup of the previous token (coordinator.py:211-215). */
int qq_copy_rows(const void* const* src_layers, void* const* dst_layers, int num_layers,
                 int64_t src_row_stride, int64_t dst_row_stride, int64_t row_bytes,
                 const void* src_idx, int src_idx_is64, const void* dst_idx, int dst_idx_is64,
                 int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QQUEST_H */
