// Internal argument structs and launchers shared by the library's translation units.
#pragma once
#include <utility>

#include "common.cuh"

namespace stk {

enum JobMode : int { kModeFull = 0, kModeMass = 1, kModeFixed = 2 };

enum PredMode : int { kPredSaved = 0, kPredHybrid = 1, kPredCompact = 2, kPredNone = 3 };

enum PredictPolicy : int { kPredictPreviousStep = 0, kPredictPreviousLayer = 1, kPredictRankInterleave = 2 };

enum Variant : int {
  kVarSplit = 0,        // kernels.repair: guards in the common frame
  kVarFused = 1,        // fused.repair_fused: negatives per token at low_m
  kVarSigned = 2,       // signed_repair.repair_signed: negatives block-local, rescaled to low_m
  kVarSignedFused = 3,  // signed_fused: hybrid block-local rescaled, compact per token
  kVarSaved = 4,        // gqa.repair_saved / gqa_light / hierarchical: output only
  kVarUnion = 5,        // gqa.repair_union: all predicted states + misses
};

struct ScoreArgs {
  const void* q;  // [R * hq, d]
  int q_dtype;
  const float* lo;  // [hmeta, total_blocks, d]
  const float* hi;
  int R, hq, hmeta, d;
  int n;                     // blocks per request when block_offsets is null
  const int* block_offsets;  // [R + 1] or null
  int total_blocks;
  int group_select;   // 1: write per-KV-group sums instead of per-head scores
  float* scores_f32;  // optional [hq, total_blocks]
  double* scores_f64; // optional [hq or hmeta (group), total_blocks]
  int* status;
};

struct SelectArgs {
  const double* scores;  // [hsel, total_blocks]
  int R, hsel, topk;
  int n;                     // blocks per request when block_offsets is null
  const int* block_offsets;  // [R + 1] or null
  int total_blocks;
  int id_base;               // added to every written ID (shard offset)
  int* ids_out;              // [R * hsel, topk], ascending
  unsigned long long* keys_out;  // optional: [R * hsel, topk] ordered keys of the chosen IDs
  int* status;
  // Two-stage selection (bounds != null): FP32 score intervals from the
  // interval scorer, exact FP64 scores recomputed for boundary blocks only.
  float2* bounds;  // [hsel, total_blocks] (lower, upper); reused as key scratch
  const void* q;
  int q_dtype;
  const float* lo;
  const float* hi;
  int hq, hmeta, d, group_select;
};

struct MergeArgs {
  const unsigned long long* keys;  // [rows, ncand]
  const int* ids;                  // [rows, ncand], ascending per row
  int rows, ncand, topk;
  int* ids_out;                    // [rows, topk] ascending
  int* status;
};

struct JobArgs {
  KVLayout L;
  const void* q;  // [rows, d]
  int q_dtype;
  int rows, hq, g, d;
  float scale;  // D^-0.5 as FP32
  const void* ids;  // [rows, s] block ids (per request)
  int ids64, s;
  const unsigned char* active;  // optional mask
  int active_mode;              // 0 none, 1 per row [rows], 2 per slot [rows, s], 3 per slot: int [rows, s] < 0
  int active_invert;            // 1: a set mask entry means "skip"
  const void* pred;             // optional: search ids in pred[row, :sp]; hits are skipped
  int pred64, sp;
  int* slot_out;                // optional [rows, s]: matching pred slot or -1
  int mode;                     // JobMode
  const float* frame;           // kModeFixed: [rows] fixed logit frame
  float* m;                     // [rows, s]   (full, mass)
  float* l;                     // [rows, s]
  float* u;                     // [rows, s, d] (full, fixed)
  float* uabs;                  // [rows, s, d] (fixed, optional)
  int* status;
  // 1: launched as the programmatic dependent of a kernel whose outputs it
  // does not read (the Top-K of the same decode step): lets its own
  // dependent launch at once and waits for that kernel before exiting, so
  // that its completion implies the predecessor's.
  int chain;
  // Chained launches: SMs left to the predecessor (one per Top-K row); the
  // persistent grid takes the others (a CTA of this kernel and a 512-thread
  // Top-K CTA together exceed an SM's registers, so they could not share an
  // SM anyway, and a static job range waiting for one would hold the grid).
  int sm_skip;
  // 1: no L2 prefetch beyond the copy ring. In the chained step the Top-K
  // kernel runs beside this one, and its latency-bound phases slow down under
  // a deeper flood of outstanding requests.
  int l2_lean;
};

struct RepairArgs {
  KVLayout L;
  const void* q;
  int q_dtype;
  int rows, hq, g, d;
  float scale;
  const void* sel;  // A [rows, sa]
  int sel64, sa;
  const void* pred;  // P [rows, sp] (null for kPredNone)
  int pred64, sp;
  int pmode, sc;
  const float* pm;  // [rows, sc]
  const float* pl;
  const float* pu;  // [rows, sc, d]
  const unsigned char* high;  // [rows, sp]
  const void* rids;           // [rows, sc] compact retained ids
  int rids64;
  const float* low_m;  // [rows]
  const float* low_l;
  const float* low_u;    // [rows, d]
  const float* low_abs;  // [rows, d]
  const float* mass_m;   // [rows, sp]
  const float* mass_l;
  int variant;
  float min_remaining, cancel_tol, eps;
  int max_n;  // upper bound of blocks per request (bitmap size)
  int stage_pred;  // set by the launcher: the row's prediction numerators fit in shared memory
  int cluster;     // set by the launcher: CTAs per row (the launch's cluster size)
  float* out;                // [rows, d]
  unsigned char* fallback;   // [rows]
  float* remaining;          // [rows]
  unsigned char* approx;     // [rows] or null
  float* extra;              // [rows] or null
  int* pos_out;              // [rows] or null
  int* total_out;            // [rows] or null
  int* status;
  // 1: the prediction states (pm, pl, pu) come from the immediately
  // preceding kernel on the stream, so they are read after pdl_wait(); the
  // cluster repair kernel is then launched as a programmatic dependent and
  // waits before its first load.
  int chain;
};

// The fused decode step (step.cu): one dense request, D = 128, 32-token
// blocks, 16-bit K/V. sp = 0 runs the serial step (selection, then
// attention over the selected blocks).
struct StepArgs {
  const void* q;  // [hq, D]
  int q_dtype;
  const float* lo;  // [hkv, n, D]
  const float* hi;
  const void* k;  // [hkv, n, B, D]
  const void* v;
  int hq, hkv, n, topk;
  const void* pred;  // [hq, sp] predicted IDs; null (sp = 0) for the serial step
  int pred64, sp;
  int* selected;   // [hq, topk] out, ascending
  float* out;      // [hq, D] out
  float2* bounds;  // [hq, n] score intervals
  float* sm;       // [hq, S] block states, S = sp (speculative) or topk (serial)
  float* sl;
  float* su;       // [hq, S, D]
  unsigned* ctrl;  // [hkv + 2 hq + 1]
  int* sel_tag;    // [hq, topk] serial step: selected ID + 1 (0 = not yet published)
  int* status;
  float scale;
};

// Launch `kern` with programmatic stream serialization: it may begin while
// the previous kernel on `stream` finishes (it must call pdl_wait() before
// reading that kernel's outputs). Optional cluster size (x) when cluster > 0.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

// Ask for the largest shared-memory carveout for `kern`. The kernels of one
// decode step share SMs (a dependent launch starts while its predecessor
// runs), and an SM whose L1/shared split was set for small-smem CTAs cannot
// take a large-smem CTA until it has drained.
template <typename... KArgs>
inline void prefer_shared(void (*kern)(KArgs...)) {
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

// Each translation unit's copy of the bounded-wait limit (common.cuh
// c_wait_ns), written for the current device.
int set_wait_limit_select(unsigned long long ns);
int set_wait_limit_states(unsigned long long ns);
int set_wait_limit_repair(unsigned long long ns);
int set_wait_limit_attend(unsigned long long ns);
int set_wait_limit_group_mma(unsigned long long ns);
int set_wait_limit_step(unsigned long long ns);

int launch_score(const ScoreArgs& a, cudaStream_t stream);
int launch_select(const SelectArgs& a, int max_n, cudaStream_t stream);
// Two-stage selection: returns 1 (nothing launched) when the shape has no
// interval-scorer kernel (d not in {64, 128, 256}, unaligned metadata, or
// more than 16 query heads per KV head).
int launch_bounds(const ScoreArgs& a, float2* bounds, cudaStream_t stream);
int launch_select_bounded(const SelectArgs& a, int max_n, cudaStream_t stream);
int launch_merge_candidates(const MergeArgs& a, cudaStream_t stream);
size_t group_mma_smem(int d, int esize);
int group_mma_splits(int sa, int b);
int launch_group_repair(const KVLayout& L, int kv_dtype, const void* q, int G, float scale, const int* sel, int sa,
                        const int* pred, int sp, const float* pm, const float* pl, const float* pu, int* miss, int* count,
                        unsigned char* hit, float* sm, float* sl, float* su, float* out, int* status,
                        cudaStream_t stream);
int launch_group_mma(const KVLayout& L, int kv_dtype, const void* q, int G, const int* ids, int sa, float scale,
                     float* m, float* l, float* u, int* status, cudaStream_t stream);
int launch_build_metadata(const KVLayout& L, int R, int total, int kv_dtype, float* lo, float* hi, cudaStream_t stream);
int launch_append_token(const KVLayout& L, int R, int total, int kv_dtype, const void* k_new, const void* v_new,
                        const int* pos, float* lo, float* hi, int* status, cudaStream_t stream);
int launch_predict(int policy, const int* step_ids, const unsigned long long* step_keys, int ks, const int* layer_ids,
                   const unsigned long long* layer_keys, int kl, int rows, int n_blocks, int budget, int* out,
                   int* status, cudaStream_t stream);
int launch_jobs(const JobArgs& a, int kv_dtype, int num_sms, cudaStream_t stream);
int launch_merge(const float* m, const float* l, const float* u, const unsigned char* include, int rows, int s, int d,
                 float* out, cudaStream_t stream);
int launch_reduce_states(const float* m, const float* l, const float* u, const unsigned char* include, int rows,
                         int s, int d, float* m_out, float* l_out, float* u_out, cudaStream_t stream);
// chain: launched as the programmatic dependent of the preceding kernel
// (the kernel waits for it before reading the states).
int launch_hybrid_group(const float* m, const float* l, const float* u, int rows, int s, int d, float tau,
                        unsigned char* high, float* low_m, float* low_l, float* low_u, float* low_abs,
                        cudaStream_t stream, bool chain = false);
int launch_compact_group(const float* pm, const float* pl, const void* pred, int pred64, int rows, int s, int c,
                         float tau, unsigned char* high, void* rids, float* low_m, float* low_l,
                         unsigned char* overflow, cudaStream_t stream);
int launch_slot_sum(const float* x, const float* y, int rows, int s, int d, float* out_x, float* out_y,
                    cudaStream_t stream);
int launch_touch(const KVLayout& L, int rows, int hq, int g, const void* ids, int ids64, int s, float* out,
                 int kv_dtype, cudaStream_t stream);
int launch_repair(const RepairArgs& a, int kv_dtype, cudaStream_t stream);
// Exact / saved / union (plain LSE merge) fast path; returns 1 when it does not apply.
int launch_attend(const RepairArgs& a, int kv_dtype, cudaStream_t stream);
// The fused decode step: dynamic shared memory per CTA, the reason a shape
// is outside its plan (null when it fits), and the cooperative launch (one
// CTA per SM).
size_t decode_step_smem(int hq);
const char* decode_step_unsupported(int hq, int hkv, int n, int b, int d, int kv_dtype, int topk, int sp,
                                    int num_sms);
int launch_decode_step(const StepArgs& a, int kv_dtype, int num_sms, cudaStream_t stream);

}  // namespace stk
