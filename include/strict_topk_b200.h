/*
 * strict_topk_b200.h — C ABI of libstk_sm100.so, the sm_100a (B200) kernels
 * behind the `strict_topk` speculative block-sparse decode API.
 *
 * Every entry point:
 *   - takes raw device pointers, explicit sizes, dtype enums and a CUDA stream
 *     (passed as `void*`, i.e. a cudaStream_t), never a framework type;
 *   - is asynchronous and stream-ordered: it only enqueues kernels, never
 *     synchronises the device, never allocates (scratch is caller-provided),
 *     and is capturable into a CUDA graph;
 *   - returns 0 on success, a negative STK_E* code for an invalid argument
 *     found on the host (message in stk_last_error()), or a positive
 *     cudaError_t from a launch.
 * Device-detected data faults (an out-of-range block ID, a bounded wait that
 * ran out) are written to the optional `status` word (first code wins) and
 * never trap.
 *
 * The reference (6Mikao9/strict-topk-overlap) is Python + Triton with no FFI
 * of its own; each entry point names the reference function(s) whose device
 * work it replaces (file:line within that project).
 */
#ifndef STRICT_TOPK_B200_H_
#define STRICT_TOPK_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STK_ABI_VERSION 1

#if defined(__GNUC__)
#define STK_API __attribute__((visibility("default")))
#else
#define STK_API
#endif

/* dtypes */
#define STK_F32 0
#define STK_F16 1
#define STK_BF16 2

/* host-side error codes */
#define STK_EINVAL (-1)   /* bad shape / argument */
#define STK_ESMEM (-2)    /* per-row sizes exceed the kernel's shared-memory plan */
#define STK_EDIM (-3)     /* head dimension unsupported (> 1024) */
#define STK_EWS (-4)      /* workspace too small */

/* device status codes (written to *status) */
#define STK_STATUS_OK 0
#define STK_STATUS_WAIT_TIMEOUT 1
#define STK_STATUS_BAD_BLOCK_ID 2
#define STK_STATUS_SHAPE_OVERFLOW 3

/* block-state job modes */
#define STK_MODE_FULL 0   /* (m, l, u) per block */
#define STK_MODE_MASS 1   /* (m, l) only, K read only */
#define STK_MODE_FIXED 2  /* l, u (and |w v| envelope) at a caller-given logit frame */

/* prediction modes */
#define STK_PRED_SAVED 0
#define STK_PRED_HYBRID 1
#define STK_PRED_COMPACT 2
#define STK_PRED_NONE 3

/* repair variants */
#define STK_VAR_SPLIT 0         /* kernels.py:504-550  repair()              */
#define STK_VAR_FUSED 1         /* fused.py:176-220    repair_fused()        */
#define STK_VAR_SIGNED 2        /* signed_repair.py:175-232 repair_signed()  */
#define STK_VAR_SIGNED_FUSED 3  /* signed_fused.py:148-193 repair_signed_fused() */
#define STK_VAR_SAVED 4         /* gqa.py:186-188, gqa_light.py:63-77, gqa_hierarchical.py:137-144 */
#define STK_VAR_UNION 5         /* gqa.py:191-193      repair_union()        */

/* KV cache description. Dense: k/v are [hkv, n, b, d] (per request, requests
 * `kv_request_stride` elements apart). Paged: k/v are page pools
 * [pages, hkv, page_size, d] and block `j` of request `r` is made of pages
 * page_table[(block_offsets[r] + j) * (b / page_size) + i]. */
typedef struct stk_kv {
  const void* k;
  const void* v;
  int kv_dtype;
  int hkv, n, b, d;
  const int32_t* page_table;    /* NULL = dense */
  const int32_t* block_offsets; /* [R + 1] per-request block offsets, or NULL (one request) */
  int page_size;
  long long kv_request_stride;  /* dense batched layouts; 0 for one request */
} stk_kv;

/* Speculative prediction state (strict_topk.kernels.Prediction, kernels.py:13-39). */
typedef struct stk_prediction {
  int mode;                 /* STK_PRED_* */
  int sc;                   /* state slots: sp (saved/hybrid) or capacity (compact) */
  const float* m;           /* [rows, sc] */
  const float* l;           /* [rows, sc] */
  const float* u;           /* [rows, sc, d] */
  const uint8_t* high;      /* [rows, sp] (hybrid, compact) */
  const void* retained_ids; /* [rows, sc] (compact) */
  int retained_ids64;
  const float* low_m;       /* [rows] */
  const float* low_l;       /* [rows] */
  const float* low_u;       /* [rows, d] */
  const float* low_abs;     /* [rows, d] */
  const float* mass_m;      /* [rows, sp] (keep_mass) */
  const float* mass_l;      /* [rows, sp] */
} stk_prediction;

/* Repair outputs (RepairResult / SignedRepairResult, kernels.py:33-39,
 * signed_repair.py:12-15). Optional pointers may be NULL. */
typedef struct stk_repair_out {
  float* out;            /* [rows, d] FP32 */
  uint8_t* fallback;     /* [rows] */
  float* remaining;      /* [rows] */
  uint8_t* approx;       /* [rows] or NULL */
  float* extra;          /* [rows] or NULL */
  int32_t* positive_jobs;/* [rows] or NULL */
  int32_t* total_jobs;   /* [rows] or NULL */
} stk_repair_out;

STK_API int stk_abi_version(void);
STK_API const char* stk_last_error(void);
STK_API int stk_device_sm_count(int device);

/* Limit of every bounded device wait in this library's kernels (a wait on a
 * bulk copy's mbarrier), in nanoseconds of the GPU's global timer, for the
 * current device; the default is 2 s, far above any legal copy time. A wait
 * that runs out writes STK_STATUS_WAIT_TIMEOUT to the call's status word,
 * waits once more (same limit) for copies still in flight on that barrier,
 * and its kernel returns without its results; treat the outputs of that call
 * (and of calls ordered after it on the stream) as invalid. New: no
 * counterpart in the reference, whose Triton kernels have no bounded waits.
 * Synchronous (it writes a device constant): call it outside stream capture
 * and while no kernel of this library runs on the device. */
STK_API int stk_set_wait_limit_ns(unsigned long long ns);

/* Exercises the bounded-wait path without a fault: one CTA arms an mbarrier
 * for 16 bytes that no copy will deliver and waits on it with the current
 * limit, so the wait runs out, STK_STATUS_WAIT_TIMEOUT is written to *status
 * and the kernel returns (after about twice the limit). It issues no copy and
 * touches no other memory. New: a test hook with no reference counterpart. */
STK_API int stk_check_wait_timeout(int32_t* status, void* stream);

/* Fused min/max query-sign bound scores, FP64 fixed-order sum rounded to FP32.
 * Replaces selector.py:23-38 block_scores() (_score, selector.py:8-20) and the
 * scoring half of gqa.py:145-161 (_bound_score, gqa.py:15-26).
 * q [hq, d] (q_dtype); lo/hi [hmeta, n, d] FP32 with hq % hmeta == 0;
 * scores [hq, n] FP32. */
STK_API int stk_bound_scores(const void* q, int q_dtype, const float* lo, const float* hi, int hq, int hmeta, int n, int d,
                     float* scores, void* stream);

/* Workspace (bytes) for stk_select_topk: one 8-byte slot per (selection row,
 * block) — an FP32 score interval, or an FP64 score where no interval
 * scorer applies. */
STK_API size_t stk_select_workspace_bytes(int sel_heads, int total_blocks);

/* Score + strict Top-K, ties to the lower block ID, IDs ascending per row.
 * Replaces selector.py:41-43 select_blocks() and gqa.py:145-161
 * select_blocks() (torch.topk at selector.py:43 / gqa.py:161).
 * q [R, hq, d]; lo/hi [hmeta, total_blocks, d]; requests own block ranges
 * block_offsets[r]..block_offsets[r+1] (or [0, n) when NULL, R == 1).
 * group_select = 0: one row per query head; 1: one row per KV head, scored by
 * the sum of its query heads' scores (shared per-group selection).
 * ids_out [R, rows_per_request, topk] int32 (+ id_base); keys_out optional
 * [.., topk] order keys (for cross-shard merges). */
STK_API int stk_select_topk(const void* q, int q_dtype, const float* lo, const float* hi, int R, int hq, int hmeta, int n,
                    const int32_t* block_offsets, int total_blocks, int max_blocks, int d, int topk, int group_select,
                    int id_base, int32_t* ids_out, unsigned long long* keys_out, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream);

/* Capacity of the library's own score scratch, in scores (rows x blocks). */
#define STK_SELECT_STATIC_MAX_SCORES (1 << 20)

/* stk_select_topk for callers that cannot allocate device memory: a decode
 * loop that must not call cudaMalloc (it may synchronise the device, and it
 * is not allowed while the stream is being captured), or a plugin host that
 * passes only inputs and outputs. No counterpart in the reference (whose
 * selector allocates its scores with torch). Same arguments and results as
 * stk_select_topk, without workspace / workspace_bytes: the 8-byte score
 * slots go to one static device array of STK_SELECT_STATIC_MAX_SCORES slots (8 MiB,
 * held by every GPU that loads the library until the process exits).
 * Selections needing more than that ((group_select ? hmeta : hq) x
 * total_blocks scores) return STK_EWS. Allocates nothing: no cudaMalloc,
 * cudaFree or allocating library call. The first call on each device (and
 * the first after that device's context is re-created, e.g. by
 * cudaDeviceReset) looks up the array's device address
 * (cudaGetSymbolAddress) with that device current, so make it before any
 * stream capture. Every call on a device
 * shares the one array and leaves its scores in it: calls whose kernels
 * overlap on the GPU (other streams, other threads) race and must be
 * ordered by the caller. */
STK_API int stk_select_topk_static(const void* q, int q_dtype, const float* lo, const float* hi, int R, int hq,
                                   int hmeta, int n, const int32_t* block_offsets, int total_blocks, int max_blocks,
                                   int d, int topk, int group_select, int id_base, int32_t* ids_out,
                                   unsigned long long* keys_out, int32_t* status, void* stream);

/* Merge shard-local Top-K candidates (ascending IDs per row) into the global
 * strict Top-K. New: the context-parallel exchange of the decode path. */
STK_API int stk_merge_candidates(const unsigned long long* keys, const int32_t* ids, int rows, int ncand, int topk,
                         int32_t* ids_out, int32_t* status, void* stream);

/* Per-block softmax states for ids [rows, s] (row = r * hq + h, kv = h / (hq / hkv)).
 * Replaces kernels.py:425-434 block_partials() (_partial, kernels.py:42-71),
 * gqa.py:128-137 partials() and its REPAIR slot search (gqa.py:29-59),
 * gqa_hierarchical.py:55-61 partials(), kernels.py:263-278 (_mass_only),
 * kernels.py:312-356 (_compact_values, fixed-frame low aggregation) and
 * kernels.py:384-407 (_wrong_aggregate).
 * active: NULL, per-row [rows] (active_mode 1) or per-slot [rows, s] (2).
 * pred != NULL: search each id in pred[row, :sp], write slot_out, skip hits. */
STK_API int stk_block_states(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* ids, int ids64,
                     int s, const uint8_t* active, int active_mode, int active_invert, const void* pred, int pred64,
                     int sp, int32_t* slot_out, int mode, const float* frame, float* m, float* l, float* u,
                     float* uabs, int32_t* status, void* stream);

/* LSE merge of per-slot states with an optional include mask.
 * Replaces kernels.py:437-442 merge_partials() (_merge, kernels.py:74-91). */
STK_API int stk_merge_states(const float* m, const float* l, const float* u, const uint8_t* include, int rows, int s, int d,
                     float* out, void* stream);

/* LSE reduction of per-slot states to one unnormalised state per row:
 * m_out = max over included slots of m (-inf when none), l_out = sum exp(m - m_out) l,
 * u_out = sum exp(m - m_out) u. New: the per-shard reduction of the
 * context-parallel path, whose rows' states are then exchanged between
 * shards and merged with stk_merge_states (kernels.py:74-91 semantics). */
STK_API int stk_reduce_states(const float* m, const float* l, const float* u, const uint8_t* include, int rows, int s,
                      int d, float* m_out, float* l_out, float* u_out, void* stream);

/* Full speculation for one prediction mode.
 * Replaces kernels.py:450-501 speculate() incl. _group (kernels.py:94-117) and
 * the compact pipeline (_mass_only, _compact_group, _compact_values).
 * Outputs follow stk_prediction: state m/l/u [rows, sc]; high [rows, sp];
 * retained_ids [rows, sc]; low m/l [rows], low u/abs [rows, d];
 * overflow [rows]; mass_m/mass_l [rows, sp] (compact: pass-1 statistics).
 * workspace: stk_speculate_workspace_bytes(). */
STK_API size_t stk_speculate_workspace_bytes(int rows, int sp, int d, int mode);
STK_API int stk_speculate(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* pred, int pred64, int sp,
                  int mode, float mass_threshold, int sc, float* state_m, float* state_l, float* state_u,
                  uint8_t* high, void* retained_ids, float* low_m, float* low_l, float* low_u, float* low_abs,
                  uint8_t* overflow, float* mass_m, float* mass_l, void* workspace, size_t workspace_bytes,
                  int32_t* status, void* stream);

/* One-launch repair: set difference, signed recompute of misses and
 * wrong-low blocks, guarded LSE merge, in-launch strict fallback.
 * Replaces kernels.py:504-550 repair(), fused.py:176-220 repair_fused(),
 * signed_repair.py:175-232 repair_signed(), signed_fused.py:148-193
 * repair_signed_fused(), gqa.py:164-193 repair_saved()/repair_union(),
 * gqa_light.py:63-92 repair_saved_light()/auto, gqa_hierarchical.py:111-144
 * repair_saved()/repair_saved_shared(); with pred_state->mode ==
 * STK_PRED_NONE it is kernels.py:445-447 exact_attention() / gqa.py:140-142. */
STK_API int stk_repair(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* sel, int sel64, int sa,
               const void* pred, int pred64, int sp, const stk_prediction* pred_state, int variant,
               float min_remaining, float cancellation_tol, float max_extra_mass, int max_blocks,
               const stk_repair_out* out, int32_t* status, void* stream);

/* Workspace (bytes) for stk_speculative_step: selection scratch plus the
 * predicted blocks' FP32 states. */
STK_API size_t stk_speculative_step_workspace_bytes(int hq, int n, int sp, int d);

/* One speculative decode step of one dense request ([hkv, n, b, d] K/V,
 * [hkv, n, d] lo/hi, per-head selection) on one stream: bound scores ->
 * strict Top-K (selected [hq, topk], ascending) -> FP32 states of the
 * predicted blocks pred [hq, sp] -> saved repair into out [hq, d] FP32.
 * The predicted-block states are launched as the programmatic dependent of
 * the Top-K kernel, so their K/V traffic overlaps the selection instead of
 * running on a second stream, and the repair follows without a stream join.
 * Results equal stk_select_topk + stk_block_states + stk_repair(SAVED) in
 * sequence. Replaces the two-stream harness of
 * benchmarks/run_benchmark.py:99-118 (selector || gqa.partials, then
 * gqa.repair_saved, gqa.py:128-137 / 164-188) for the saved method. */
STK_API int stk_speculative_step(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int hq,
                                 int topk, const void* pred, int pred64, int sp, int32_t* selected, float* out,
                                 void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Workspace (bytes) for stk_decode_step: a control block of
 * (hkv + 2 hq + 1) 32-bit counters, then one 8-byte score slot per (query
 * head, block), the block states of `slots` blocks per query head
 * (slots = sp for a speculative step, topk for a serial one) and one 32-bit
 * tag per (query head, slot). */
STK_API size_t stk_decode_step_workspace_bytes(int hq, int hkv, int n, int slots, int d);

/* The whole decode step in one persistent, cooperative launch (one CTA per
 * SM; CTAs wait for one another through the workspace's counters, every wait
 * bounded by the library's wait limit).
 * With pred (sp > 0): the speculative saved step — the strict Top-K
 * selection, the states of the predicted blocks computed while the selection
 * runs, and the saved repair (hits reused, misses computed) — equal to
 * stk_speculative_step. Replaces the reference's overlapped step
 * (benchmarks/run_benchmark.py:99-118: selector.py:41-43 / gqa.py:145-161
 * select_blocks || gqa.py:128-137 partials, then gqa.py:186-188
 * repair_saved).
 * With pred == NULL (sp == 0): the serial step — selection, then exact
 * attention over the selected blocks (run_benchmark.py:139,
 * critical_path.py:110: gqa.py:140-142 exact(select_blocks(...))).
 * One dense request; D = 128, 32-token blocks, 16-bit K/V, at most 16 query
 * heads per KV head and 4096 query values (hq * d), topk <= n <= 4096,
 * topk and sp <= 256, fewer than half as many query heads as SMs; other
 * shapes return STK_ESMEM and take stk_speculative_step / stk_select_topk +
 * stk_repair. The workspace must be zero before its first use (e.g. one
 * cudaMemset after allocation); every call leaves its control block, score
 * slots and tags zero again (a call whose status word reports
 * STK_STATUS_WAIT_TIMEOUT may not: zero the workspace before reusing it).
 * Calls sharing a workspace must be ordered on one stream. */
STK_API int stk_decode_step(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int hq,
                            int topk, const void* pred, int pred64, int sp, int32_t* selected, float* out,
                            void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Workspace (bytes) for stk_speculative_step_batched: selection scratch for
 * total_blocks blocks of hq query heads, the predicted blocks' states of the
 * R * hq rows and, with hybrid != 0, the hybrid grouping's mask and low
 * aggregate. */
STK_API size_t stk_speculative_step_batched_workspace_bytes(int R, int hq, int total_blocks, int sp, int d, int hybrid);

/* The chained speculative step (stk_speculative_step, stk_speculative_step_hybrid)
 * for a batch of R requests of hq query heads each, dense (R == 1) or paged /
 * batched (kv->block_offsets [R + 1], total_blocks, max_blocks as in
 * stk_select_topk); rows = R * hq, request-local block IDs. One stream, one
 * chain of dependent launches: bound scores -> strict Top-K (selected
 * [rows, topk]) -> predicted blocks' states -> variant STK_VAR_SAVED: saved
 * repair (out->out only); STK_VAR_FUSED / STK_VAR_SIGNED_FUSED: hybrid
 * grouping with mass_threshold, then the guarded repair relaxed by
 * max_extra_mass (every field of out as in stk_repair). Replaces, per
 * request, the reference's overlapped step (benchmarks/run_benchmark.py:99-118
 * with gqa.py:128-137,186-188, or kernels.py:450-501 + fused.py:174-220 /
 * signed_fused.py:144-193) run over a batch. */
STK_API int stk_speculative_step_batched(const stk_kv* kv, const void* q, int q_dtype, const float* lo,
                                         const float* hi, int R, int hq, int total_blocks, int max_blocks, int topk,
                                         const void* pred, int pred64, int sp, float mass_threshold, int variant,
                                         float min_remaining, float cancellation_tol, float max_extra_mass,
                                         int32_t* selected, const stk_repair_out* out, void* workspace,
                                         size_t workspace_bytes, int32_t* status, void* stream);

/* Workspace (bytes) for stk_speculative_step_hybrid: the saved step's
 * workspace plus the hybrid grouping's high mask and low aggregate. */
STK_API size_t stk_speculative_step_hybrid_workspace_bytes(int hq, int n, int sp, int d);

/* The hybrid methods' speculative step of one dense request on one stream:
 * bound scores -> strict Top-K (selected [hq, topk]) -> FP32 states of the
 * predicted blocks (the Top-K kernel's programmatic dependent, as in
 * stk_speculative_step) -> hybrid grouping with threshold mass_threshold ->
 * repair with variant STK_VAR_FUSED (fused.py:176-220 repair_fused) or
 * STK_VAR_SIGNED_FUSED (signed_fused.py:148-193 repair_signed_fused) into
 * out. The prediction keeps its mass (keep_mass=True aliases the states'
 * m and l, kernels.py:450-477), so max_extra_mass > 0 is accepted. Results
 * equal stk_select_topk + stk_speculate(STK_PRED_HYBRID) + stk_repair in
 * sequence. Replaces the two-stream harness of
 * benchmarks/run_benchmark.py:99-118 for the repair_fused / signed_fused
 * methods. */
STK_API int stk_speculative_step_hybrid(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi,
                                        int hq, int topk, const void* pred, int pred64, int sp, float mass_threshold,
                                        int variant, float min_remaining, float cancellation_tol,
                                        float max_extra_mass, int32_t* selected, const stk_repair_out* out,
                                        void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Per-block K bounds: lo/hi [hkv, total, d] FP32 = min / max over each
 * block's tokens (NaN propagates). total = n for one dense request (R == 1,
 * block_offsets NULL) or total_blocks for block_offsets layouts (paged or
 * batched dense). Replaces the prefill-time k.amin(dim=2).float(),
 * k.amax(dim=2).float() of benchmarks/run_benchmark.py:42-43 and
 * experiments/trace_replay.py:68. */
STK_API int stk_build_metadata(const stk_kv* kv, int R, int total_blocks, float* lo, float* hi, int32_t* status,
                               void* stream);

/* Decode-loop append: for each request r, write k_new / v_new [R, hkv, d]
 * (the cache's dtype) as token positions[r] of the request (block
 * positions[r] / b, slot positions[r] % b) and fold the key into that
 * block's lo/hi (the block's first token resets them), so metadata never has
 * to be rebuilt. The cache described by kv must be writable. New: the
 * reference builds metadata once, outside its timed region. */
STK_API int stk_append_token(const stk_kv* kv, int R, int total_blocks, const void* k_new, const void* v_new,
                             const int32_t* positions, float* lo, float* hi, int32_t* status, void* stream);

#define STK_PREDICT_PREVIOUS_STEP 0
#define STK_PREDICT_PREVIOUS_LAYER 1
#define STK_PREDICT_RANK_INTERLEAVE 2

/* Predicted block IDs for the next decode step, on the device. Replaces the
 * policies of experiments/hisparse_cache_trace.py:40-57 predict() and
 * experiments/predictor_rank_trace.py:37-48 interleave() (previous step's
 * ranking; previous layer's ranking; alternating unique IDs, the step's
 * first). step_ids [rows, ks] / layer_ids [rows, kl] are selection rows;
 * with keys (stk_select_topk keys_out) they are ranked best first, ties to
 * the lower position, else taken in their given order. out [rows, budget];
 * a slot that no list can fill is -1 (the reference raises when an
 * interleave source runs out; here the other source fills the slot). */
STK_API int stk_predict(int policy, const int32_t* step_ids, const unsigned long long* step_keys, int ks,
                        const int32_t* layer_ids, const unsigned long long* layer_keys, int kl, int rows,
                        int n_blocks, int budget, int32_t* out, int32_t* status, void* stream);

/* Workspace (bytes) for stk_group_repair_saved. */
STK_API size_t stk_group_repair_saved_workspace_bytes(int hq, int hkv, int sa, int sp, int b, int d);

/* The saved repair for shared lists on the tensor cores: every query head of
 * a KV group has the same selected IDs (selected [hq, sa] int32, ascending)
 * and the same predicted IDs (pred [hq, sp] int32), so the misses (A not in
 * P, from each group's first row) are attended on the group's MMA tile (each
 * missed block read once per group) and each head folds its own saved
 * states (pm, pl [hq, sp], pu [hq, sp, d]) of the hits (P slots in A); out
 * [hq, d] FP32. One dense request, q and K/V both bf16 or both f16, d 64 or
 * 128, b dividing 64, hq / hkv <= 16. Replaces gqa_hierarchical.py:137-144
 * repair_saved_shared (its _match_ids, _packed_partials and _groups passes). */
STK_API int stk_group_repair_saved(const stk_kv* kv, const void* q, int q_dtype, int hq, const int32_t* selected,
                                   int sa, const int32_t* pred, int sp, const float* pm, const float* pl,
                                   const float* pu, float* out, void* workspace, size_t workspace_bytes,
                                   int32_t* status, void* stream);

/* Workspace (bytes) for stk_group_attention. */
STK_API size_t stk_group_attention_workspace_bytes(int hq, int sa, int b, int d);

/* Attention of every query head over its KV group's shared block list, on
 * the tensor cores: the hq / hkv (<= 16) query heads of a KV head form one
 * MMA tile, so each listed K/V block is read once per group. One dense
 * request, q and K/V both bf16 or both f16, d 64 or 128, b dividing 64;
 * group_ids [hkv, sa] int32; out [hq, d] FP32 (normalised). Replaces, for
 * shared lists (select_blocks_shared), the per-head partials and merge of
 * gqa_hierarchical.py:55-112 and gqa.py:140-142. */
STK_API int stk_group_attention(const stk_kv* kv, const void* q, int q_dtype, int hq, const int32_t* group_ids,
                                int sa, float* out, void* workspace, size_t workspace_bytes, int32_t* status,
                                void* stream);

/* Prefetch baseline: read predicted K/V, write per-tile checksums.
 * Replaces kernels.py:553-560 touch_kv() (_touch, kernels.py:250-260).
 * out [rows, s, ceil(b * d / 1024)] FP32. */
STK_API int stk_touch_kv(const stk_kv* kv, int rows, int hq, const void* ids, int ids64, int s, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* STRICT_TOPK_B200_H_ */
