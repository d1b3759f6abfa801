// extern "C" entry points of libstk_sm100.so (declared in include/strict_topk_b200.h).
// Host-side validation, argument packing and launch orchestration only; all
// arithmetic lives in select.cu, states.cu and repair.cu.
#include <cuda.h>
#include <math.h>
#include <stdarg.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.cuh"
#include "../../include/strict_topk_b200.h"


using namespace stk;

namespace {
thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_status(int rc, const char* what) {
  if (rc > 0) {
    g_err = std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(rc));
  } else if (rc < 0) {
    g_err = std::string(what) + ": per-row sizes exceed the kernel plan";
  }
  return rc;
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

int sm_count_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sm_count[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sm_count[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

std::atomic<int> g_smem_optin[kMaxDevices];

// Largest dynamic shared memory a CTA may opt in to on the current device.
int smem_optin_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 227 * 1024;
  int v = g_smem_optin[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
      v = 227 * 1024;
    g_smem_optin[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// The hybrid grouping stages a row's (m, l, weight) per predicted slot.
bool hybrid_group_fits(int sp) {
  return static_cast<size_t>(sp) * 3 * sizeof(float) <= static_cast<size_t>(smem_optin_current());
}

bool valid_dtype(int t) { return t == STK_F32 || t == STK_F16 || t == STK_BF16; }

KVLayout make_layout(const stk_kv* kv) {
  KVLayout L;
  L.k = kv->k;
  L.v = kv->v;
  L.hkv = kv->hkv;
  L.n = kv->n;
  L.b = kv->b;
  L.d = kv->d;
  L.page_table = kv->page_table;
  L.block_offsets = kv->block_offsets;
  L.page_size = kv->page_size > 0 ? kv->page_size : kv->b;
  L.kv_request_stride = kv->kv_request_stride;
  return L;
}

int check_kv(const stk_kv* kv, int hq) {
  if (kv == nullptr || kv->k == nullptr || kv->v == nullptr) return fail(STK_EINVAL, "kv description is null");
  if (!valid_dtype(kv->kv_dtype)) return fail(STK_EINVAL, "unsupported KV dtype %d", kv->kv_dtype);
  if (kv->hkv <= 0 || kv->b <= 0 || kv->d <= 0 || (kv->n <= 0 && kv->block_offsets == nullptr))
    return fail(STK_EINVAL, "KV shape must be nonempty (hkv=%d n=%d b=%d d=%d)", kv->hkv, kv->n, kv->b, kv->d);
  if (hq <= 0 || hq % kv->hkv != 0) return fail(STK_EINVAL, "query heads %d not divisible by KV heads %d", hq, kv->hkv);
  if (kv->d > 1024) return fail(STK_EDIM, "head dim %d > 1024 unsupported", kv->d);
  if (kv->page_table != nullptr) {
    if (kv->page_size <= 0 || kv->b % kv->page_size != 0)
      return fail(STK_EINVAL, "page size %d must divide the block size %d", kv->page_size, kv->b);
    if (kv->block_offsets == nullptr) return fail(STK_EINVAL, "paged KV needs block_offsets");
  }
  return 0;
}

float attn_scale(int d) { return static_cast<float>(1.0 / sqrt(static_cast<double>(d))); }

// Test hook of the bounded-wait path: arm a barrier for bytes no copy will
// bring and wait on it; mbar_wait gives up after the current limit, records
// kStatusWaitTimeout and returns. No copy is issued, so nothing is in flight
// when the CTA exits.
__global__ void wait_probe_kernel(int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bar, 16);
    (void)mbar_wait(&bar, 0, status);
  }
}
}  // namespace

extern "C" {

int stk_abi_version(void) { return STK_ABI_VERSION; }

const char* stk_last_error(void) { return g_err.c_str(); }

int stk_device_sm_count(int device) {
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return v;
}

int stk_set_wait_limit_ns(unsigned long long ns) {
  if (ns == 0) return fail(STK_EINVAL, "the wait limit must be positive");
  int (*const setters[])(unsigned long long) = {set_wait_limit_select, set_wait_limit_states, set_wait_limit_repair,
                                                set_wait_limit_attend, set_wait_limit_group_mma, set_wait_limit_step};
  for (auto set : setters) {
    const int rc = set(ns);
    if (rc) return cuda_status(rc, "set wait limit");
  }
  return cuda_status(set_wait_limit_this_unit(ns), "set wait limit");
}

int stk_check_wait_timeout(int32_t* status, void* stream) {
  if (!status) return fail(STK_EINVAL, "status word required");
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status);
  return cuda_status(static_cast<int>(cudaGetLastError()), "wait probe");
}

int stk_bound_scores(const void* q, int q_dtype, const float* lo, const float* hi, int hq, int hmeta, int n, int d,
                     float* scores, void* stream) {
  if (!q || !lo || !hi || !scores) return fail(STK_EINVAL, "null pointer");
  if (!valid_dtype(q_dtype)) return fail(STK_EINVAL, "unsupported q dtype");
  if (hq <= 0 || hmeta <= 0 || n <= 0 || d <= 0 || hq % hmeta) return fail(STK_EINVAL, "bad score shape");
  ScoreArgs a{};
  a.q = q; a.q_dtype = q_dtype; a.lo = lo; a.hi = hi;
  a.R = 1; a.hq = hq; a.hmeta = hmeta; a.d = d; a.n = n;
  a.block_offsets = nullptr; a.total_blocks = n; a.group_select = 0;
  a.scores_f32 = scores; a.scores_f64 = nullptr;
  if ((reinterpret_cast<uintptr_t>(lo) | reinterpret_cast<uintptr_t>(hi)) & 15) {
    // The vectorised path needs 16-byte rows; misaligned metadata uses scalar loads.
  }
  return cuda_status(launch_score(a, static_cast<cudaStream_t>(stream)), "bound_scores");
}

size_t stk_select_workspace_bytes(int sel_heads, int total_blocks) {
  return static_cast<size_t>(sel_heads) * static_cast<size_t>(total_blocks) * sizeof(double);
}

int stk_select_topk(const void* q, int q_dtype, const float* lo, const float* hi, int R, int hq, int hmeta, int n,
                    const int32_t* block_offsets, int total_blocks, int max_blocks, int d, int topk, int group_select,
                    int id_base, int32_t* ids_out, unsigned long long* keys_out, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream) {
  if (!q || !lo || !hi || !ids_out || !workspace) return fail(STK_EINVAL, "null pointer");
  if (!valid_dtype(q_dtype)) return fail(STK_EINVAL, "unsupported q dtype");
  if (R <= 0 || hq <= 0 || hmeta <= 0 || d <= 0 || hq % hmeta) return fail(STK_EINVAL, "bad select shape");
  if (block_offsets == nullptr) {
    if (R != 1 || n <= 0) return fail(STK_EINVAL, "one request with n > 0 expected without block_offsets");
    total_blocks = n;
    max_blocks = n;
  }
  if (topk <= 0 || topk > max_blocks) return fail(STK_EINVAL, "topk %d outside [1, %d]", topk, max_blocks);
  const int hsel = group_select ? hmeta : hq;
  if (workspace_bytes < stk_select_workspace_bytes(hsel, total_blocks)) return fail(STK_EWS, "select workspace too small");
  if (static_cast<size_t>(max_blocks) * 8 > 200 * 1024)
    return fail(STK_ESMEM, "%d blocks per row exceed the single-pass selection plan (max 25600); "
                "split the row into segments and merge candidates", max_blocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ScoreArgs a{};
  a.q = q; a.q_dtype = q_dtype; a.lo = lo; a.hi = hi;
  a.R = R; a.hq = hq; a.hmeta = hmeta; a.d = d; a.n = n;
  a.block_offsets = block_offsets; a.total_blocks = total_blocks;
  a.group_select = group_select; a.scores_f32 = nullptr;
  a.scores_f64 = static_cast<double*>(workspace);
  a.status = status;
  SelectArgs b{};
  b.scores = static_cast<const double*>(workspace);
  b.R = R; b.hsel = hsel; b.topk = topk; b.n = n;
  b.block_offsets = block_offsets; b.total_blocks = total_blocks;
  b.id_base = id_base; b.ids_out = ids_out; b.keys_out = keys_out; b.status = status;
  // Two-stage selection (FP32 score intervals, exact FP64 only at the
  // boundary) where an interval scorer exists; the FP64 scorer otherwise.
  // Both give the strict Top-K of the same FP64 fixed-order scores.
  int rc = launch_bounds(a, static_cast<float2*>(workspace), s);
  if (rc == 0) {
    b.bounds = static_cast<float2*>(workspace);
    b.q = q; b.q_dtype = q_dtype; b.lo = lo; b.hi = hi;
    b.hq = hq; b.hmeta = hmeta; b.d = d; b.group_select = group_select;
    return cuda_status(launch_select_bounded(b, max_blocks, s), "select");
  }
  if (rc != 1) return cuda_status(rc, "bound scores");
  rc = launch_score(a, s);
  if (rc) return cuda_status(rc, "score");
  return cuda_status(launch_select(b, max_blocks, s), "select");
}

int stk_merge_candidates(const unsigned long long* keys, const int32_t* ids, int rows, int ncand, int topk,
                         int32_t* ids_out, int32_t* status, void* stream) {
  if (!keys || !ids || !ids_out) return fail(STK_EINVAL, "null pointer");
  if (rows <= 0 || ncand <= 0 || topk <= 0 || topk > ncand) return fail(STK_EINVAL, "bad candidate shape");
  MergeArgs a{keys, ids, rows, ncand, topk, ids_out, status};
  return cuda_status(launch_merge_candidates(a, static_cast<cudaStream_t>(stream)), "merge_candidates");
}

int stk_block_states(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* ids, int ids64,
                     int s, const uint8_t* active, int active_mode, int active_invert, const void* pred, int pred64,
                     int sp, int32_t* slot_out, int mode, const float* frame, float* m, float* l, float* u,
                     float* uabs, int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!q || !ids || !valid_dtype(q_dtype)) return fail(STK_EINVAL, "bad q / ids");
  if (rows <= 0 || rows % hq != 0 || s <= 0) return fail(STK_EINVAL, "bad job shape rows=%d s=%d", rows, s);
  if (mode < 0 || mode > 2) return fail(STK_EINVAL, "bad mode");
  if (mode != STK_MODE_FIXED && (!m || !l)) return fail(STK_EINVAL, "m/l outputs required");
  if (mode != STK_MODE_MASS && !u) return fail(STK_EINVAL, "u output required");
  if (mode == STK_MODE_FIXED && !frame) return fail(STK_EINVAL, "frame required");
  if (pred && sp <= 0) return fail(STK_EINVAL, "pred needs sp > 0");
  JobArgs a{};
  a.L = make_layout(kv);
  a.q = q; a.q_dtype = q_dtype;
  a.rows = rows; a.hq = hq; a.g = hq / kv->hkv; a.d = kv->d; a.scale = attn_scale(kv->d);
  a.ids = ids; a.ids64 = ids64; a.s = s;
  a.active = active; a.active_mode = active ? active_mode : 0; a.active_invert = active_invert;
  a.pred = pred; a.pred64 = pred64; a.sp = sp; a.slot_out = slot_out;
  a.mode = mode; a.frame = frame; a.m = m; a.l = l; a.u = u; a.uabs = uabs; a.status = status;
  return cuda_status(launch_jobs(a, kv->kv_dtype, sm_count_current(), static_cast<cudaStream_t>(stream)), "block_states");
}

int stk_merge_states(const float* m, const float* l, const float* u, const uint8_t* include, int rows, int s, int d,
                     float* out, void* stream) {
  if (!m || !l || !u || !out || rows <= 0 || s <= 0 || d <= 0) return fail(STK_EINVAL, "bad merge arguments");
  return cuda_status(launch_merge(m, l, u, include, rows, s, d, out, static_cast<cudaStream_t>(stream)), "merge");
}

int stk_reduce_states(const float* m, const float* l, const float* u, const uint8_t* include, int rows, int s, int d,
                      float* m_out, float* l_out, float* u_out, void* stream) {
  if (!m || !l || !u || !m_out || !l_out || !u_out || rows <= 0 || s <= 0 || d <= 0)
    return fail(STK_EINVAL, "bad reduce arguments");
  return cuda_status(launch_reduce_states(m, l, u, include, rows, s, d, m_out, l_out, u_out,
                                          static_cast<cudaStream_t>(stream)),
                     "reduce_states");
}

size_t stk_speculate_workspace_bytes(int rows, int sp, int d, int mode) {
  if (mode != STK_PRED_COMPACT) return 0;
  // Fixed-frame low aggregation: per-slot u and |w v| rows.
  return static_cast<size_t>(rows) * sp * d * sizeof(float) * 2;
}

int stk_speculate(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* pred, int pred64, int sp,
                  int mode, float mass_threshold, int sc, float* state_m, float* state_l, float* state_u,
                  uint8_t* high, void* retained_ids, float* low_m, float* low_l, float* low_u, float* low_abs,
                  uint8_t* overflow, float* mass_m, float* mass_l, void* workspace, size_t workspace_bytes,
                  int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!(mass_threshold >= 0.f && mass_threshold <= 1.f)) return fail(STK_EINVAL, "mass_threshold must be in [0,1]");
  if (rows <= 0 || rows % hq || sp <= 0) return fail(STK_EINVAL, "bad speculate shape");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int d = kv->d;
  if (mode == STK_PRED_HYBRID && !hybrid_group_fits(sp))
    return fail(STK_ESMEM, "hybrid grouping of %d predicted blocks per row exceeds the shared-memory plan", sp);
  if (mode == STK_PRED_SAVED || mode == STK_PRED_HYBRID) {
    rc = stk_block_states(kv, q, q_dtype, rows, hq, pred, pred64, sp, nullptr, 0, 0, nullptr, 0, 0, nullptr,
                          STK_MODE_FULL, nullptr, state_m, state_l, state_u, nullptr, status, stream);
    if (rc || mode == STK_PRED_SAVED) return rc;
    if (!high || !low_m || !low_l || !low_u || !low_abs) return fail(STK_EINVAL, "hybrid outputs required");
    return cuda_status(launch_hybrid_group(state_m, state_l, state_u, rows, sp, d, mass_threshold, high, low_m, low_l,
                                           low_u, low_abs, st),
                       "hybrid_group");
  }
  if (mode != STK_PRED_COMPACT) return fail(STK_EINVAL, "bad prediction mode %d", mode);
  if (!mass_m || !mass_l || !high || !retained_ids || !overflow || !low_m || !low_l || !low_u || !low_abs)
    return fail(STK_EINVAL, "compact outputs required");
  if (sc <= 0 || sc > sp) return fail(STK_EINVAL, "compact capacity %d outside [1, %d]", sc, sp);
  if (workspace_bytes < stk_speculate_workspace_bytes(rows, sp, d, mode)) return fail(STK_EWS, "compact workspace too small");
  // Pass 1: per-block (m, l) from K only (kernels.py:263-278).
  rc = stk_block_states(kv, q, q_dtype, rows, hq, pred, pred64, sp, nullptr, 0, 0, nullptr, 0, 0, nullptr,
                        STK_MODE_MASS, nullptr, mass_m, mass_l, nullptr, nullptr, status, stream);
  if (rc) return rc;
  // Grouping with capacity-C packing (kernels.py:281-309).
  rc = launch_compact_group(mass_m, mass_l, pred, pred64, rows, sp, sc, mass_threshold, high, retained_ids, low_m,
                            low_l, overflow, st);
  if (rc) return cuda_status(rc, "compact_group");
  // Pass 2a: retained high blocks, full states (kernels.py:337-356).
  rc = stk_block_states(kv, q, q_dtype, rows, hq, retained_ids, pred64, sc, nullptr, 0, 0, nullptr, 0, 0, nullptr,
                        STK_MODE_FULL, nullptr, state_m, state_l, state_u, nullptr, status, stream);
  if (rc) return rc;
  // Pass 2b: low blocks per token at low_m, then per-row sums (kernels.py:320-336).
  float* su = static_cast<float*>(workspace);
  float* sa = su + static_cast<size_t>(rows) * sp * d;
  rc = stk_block_states(kv, q, q_dtype, rows, hq, pred, pred64, sp, high, 2, 1, nullptr, 0, 0, nullptr,
                        STK_MODE_FIXED, low_m, nullptr, nullptr, su, sa, status, stream);
  if (rc) return rc;
  return cuda_status(launch_slot_sum(su, sa, rows, sp, d, low_u, low_abs, st), "slot_sum");
}

// stk_repair's body; chain = 1 launches the repair as the programmatic
// dependent of the preceding kernel (the chained hybrid step).
static int repair_entry(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* sel, int sel64,
                        int sa, const void* pred, int pred64, int sp, const stk_prediction* ps, int variant,
                        float min_remaining, float cancellation_tol, float max_extra_mass, int max_blocks,
                        const stk_repair_out* out, int32_t* status, void* stream, int chain) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!q || !sel || !out || !out->out || !valid_dtype(q_dtype)) return fail(STK_EINVAL, "bad repair pointers");
  if (rows <= 0 || rows % hq || sa <= 0) return fail(STK_EINVAL, "bad repair shape");
  if (variant < 0 || variant > 5) return fail(STK_EINVAL, "bad variant");
  if (!(max_extra_mass >= 0.f && max_extra_mass <= 1.f)) return fail(STK_EINVAL, "max_extra_mass must be in [0, 1]");
  const int pmode = ps ? ps->mode : STK_PRED_NONE;
  if (pmode != STK_PRED_NONE) {
    if (!pred || sp <= 0 || !ps->m || !ps->l || !ps->u) return fail(STK_EINVAL, "prediction state required");
    if ((pmode == STK_PRED_HYBRID || pmode == STK_PRED_COMPACT) &&
        (!ps->high || !ps->low_m || !ps->low_l || !ps->low_u || !ps->low_abs))
      return fail(STK_EINVAL, "hybrid/compact prediction needs high mask and low aggregate");
    if (pmode == STK_PRED_COMPACT && !ps->retained_ids) return fail(STK_EINVAL, "compact prediction needs retained ids");
    if (max_extra_mass > 0.f && (pmode == STK_PRED_HYBRID || pmode == STK_PRED_COMPACT) && (!ps->mass_m || !ps->mass_l))
      return fail(STK_EINVAL, "positive max_extra_mass requires speculate(..., keep_mass=True)");
  }
  const int max_n = kv->block_offsets ? max_blocks : kv->n;
  if (max_n <= 0) return fail(STK_EINVAL, "max_blocks required for batched layouts");
  RepairArgs a{};
  a.L = make_layout(kv);
  a.q = q; a.q_dtype = q_dtype;
  a.rows = rows; a.hq = hq; a.g = hq / kv->hkv; a.d = kv->d; a.scale = attn_scale(kv->d);
  a.sel = sel; a.sel64 = sel64; a.sa = sa;
  a.pred = pmode == STK_PRED_NONE ? nullptr : pred; a.pred64 = pred64; a.sp = pmode == STK_PRED_NONE ? 0 : sp;
  a.pmode = pmode; a.sc = pmode == STK_PRED_NONE ? 0 : ps->sc;
  if (ps) {
    a.pm = ps->m; a.pl = ps->l; a.pu = ps->u; a.high = ps->high;
    a.rids = ps->retained_ids; a.rids64 = ps->retained_ids64;
    a.low_m = ps->low_m; a.low_l = ps->low_l; a.low_u = ps->low_u; a.low_abs = ps->low_abs;
    a.mass_m = ps->mass_m; a.mass_l = ps->mass_l;
  }
  a.variant = variant;
  a.min_remaining = min_remaining; a.cancel_tol = cancellation_tol; a.eps = max_extra_mass;
  a.max_n = max_n;
  a.out = out->out; a.fallback = out->fallback; a.remaining = out->remaining; a.approx = out->approx;
  a.extra = out->extra; a.pos_out = out->positive_jobs; a.total_out = out->total_jobs;
  a.status = status;
  a.chain = chain;
  return cuda_status(launch_repair(a, kv->kv_dtype, static_cast<cudaStream_t>(stream)), "repair");
}

int stk_repair(const stk_kv* kv, const void* q, int q_dtype, int rows, int hq, const void* sel, int sel64, int sa,
               const void* pred, int pred64, int sp, const stk_prediction* ps, int variant, float min_remaining,
               float cancellation_tol, float max_extra_mass, int max_blocks, const stk_repair_out* out,
               int32_t* status, void* stream) {
  return repair_entry(kv, q, q_dtype, rows, hq, sel, sel64, sa, pred, pred64, sp, ps, variant, min_remaining,
                      cancellation_tol, max_extra_mass, max_blocks, out, status, stream, 0);
}

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// ------------------------------------------------------------------ chained steps
// One speculative step as one chain of dependent launches on one stream, for
// R requests of hq query heads each (rows = R hq): bound scores -> strict
// Top-K -> states of the predicted blocks (the Top-K kernel's programmatic
// dependent: it streams the predicted K/V while the selection finishes) ->
// [hybrid grouping ->] repair. Dense single requests (R = 1, no block
// offsets) and batched or paged layouts take the same path.
struct ChainShape {
  int R, hq, rows, total, max_n;
  const int32_t* block_offsets;
};

static int chain_shape(const stk_kv* kv, int R, int hq, const int32_t* block_offsets, int total_blocks,
                       int max_blocks, ChainShape* c) {
  if (R <= 0 || hq <= 0) return fail(STK_EINVAL, "R and hq must be positive");
  if (kv->page_table && !block_offsets) return fail(STK_EINVAL, "a paged layout needs block offsets");
  c->R = R; c->hq = hq; c->rows = R * hq; c->block_offsets = block_offsets;
  if (block_offsets) {
    if (total_blocks <= 0 || max_blocks <= 0) return fail(STK_EINVAL, "total_blocks and max_blocks required");
    c->total = total_blocks; c->max_n = max_blocks;
  } else {
    if (R != 1) return fail(STK_EINVAL, "batched dense requests need block offsets");
    c->total = kv->n; c->max_n = kv->n;
  }
  return 0;
}

static size_t chain_ws_saved(int rows_sel_hq, int total, int rows, int sp, int d) {
  const size_t slots = static_cast<size_t>(rows) * sp;
  return align256(stk_select_workspace_bytes(rows_sel_hq, total)) + 2 * align256(slots * sizeof(float)) +
         align256(slots * d * sizeof(float));
}
static size_t chain_ws_hybrid(int rows_sel_hq, int total, int rows, int sp, int d) {
  const size_t slots = static_cast<size_t>(rows) * sp;
  return chain_ws_saved(rows_sel_hq, total, rows, sp, d) + align256(slots) + 2 * align256(rows * sizeof(float)) +
         2 * align256(static_cast<size_t>(rows) * d * sizeof(float));
}

// variant STK_VAR_SAVED: saved speculation + saved repair (gqa.py:128-137,
// 186-188); STK_VAR_FUSED / STK_VAR_SIGNED_FUSED: hybrid speculation with
// threshold mass_threshold, then the guarded repair (fused.py:176-220,
// signed_fused.py:144-193) relaxed by max_extra_mass.
static int chain_step(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi,
                      const ChainShape& c, int topk, const void* pred, int pred64, int sp, float mass_threshold,
                      int variant, float min_remaining, float cancellation_tol, float max_extra_mass,
                      int32_t* selected, const stk_repair_out* out, void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream) {
  int rc = check_kv(kv, c.hq);
  if (rc) return rc;
  if (!q || !lo || !hi || !pred || !selected || !out || !out->out || !workspace || !valid_dtype(q_dtype))
    return fail(STK_EINVAL, "null pointer or unsupported q dtype");
  if (sp <= 0) return fail(STK_EINVAL, "empty prediction");
  const bool hybrid = variant != STK_VAR_SAVED;
  if (hybrid && variant != STK_VAR_FUSED && variant != STK_VAR_SIGNED_FUSED)
    return fail(STK_EINVAL, "the hybrid chained step repairs with STK_VAR_FUSED or STK_VAR_SIGNED_FUSED");
  if (!(mass_threshold >= 0.f && mass_threshold <= 1.f)) return fail(STK_EINVAL, "mass_threshold must be in [0,1]");
  if (!(max_extra_mass >= 0.f && max_extra_mass <= 1.f)) return fail(STK_EINVAL, "max_extra_mass must be in [0, 1]");
  if (hybrid && !hybrid_group_fits(sp))
    return fail(STK_ESMEM, "hybrid grouping of %d predicted blocks per row exceeds the shared-memory plan", sp);
  const int d = kv->d, rows = c.rows;
  const size_t need = hybrid ? chain_ws_hybrid(c.hq, c.total, rows, sp, d) : chain_ws_saved(c.hq, c.total, rows, sp, d);
  if (workspace_bytes < need) return fail(STK_EWS, "chained step workspace too small");
  unsigned char* w = static_cast<unsigned char*>(workspace);
  const size_t sel_bytes = stk_select_workspace_bytes(c.hq, c.total);
  const size_t slots = static_cast<size_t>(rows) * sp;
  float* pm = reinterpret_cast<float*>(w + align256(sel_bytes));
  float* pl = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(pm) + align256(slots * sizeof(float)));
  float* pu = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(pl) + align256(slots * sizeof(float)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 1. Bound scores and strict Top-K (the scorer, then the Top-K kernel as its dependent).
  rc = stk_select_topk(q, q_dtype, lo, hi, c.R, c.hq, kv->hkv, c.block_offsets ? 0 : kv->n, c.block_offsets, c.total,
                       c.max_n, d, topk, 0, 0, selected, nullptr, w, sel_bytes, status, stream);
  if (rc) return rc;
  // 2. States of the predicted blocks, launched as the Top-K kernel's
  //    dependent: it starts as soon as every Top-K CTA is running and streams
  //    the predicted K/V while the selection finishes, then holds its own
  //    completion until the Top-K grid's. With few rows it leaves one SM per
  //    Top-K CTA and skips the L2 prefetch window (the Top-K kernel beside it
  //    is latency-bound); with many rows the Top-K grid runs in waves and the
  //    states kernel takes every SM with its window.
  const int nsm = sm_count_current();
  JobArgs a{};
  a.L = make_layout(kv);
  a.q = q; a.q_dtype = q_dtype;
  a.rows = rows; a.hq = c.hq; a.g = c.hq / kv->hkv; a.d = d; a.scale = attn_scale(d);
  a.ids = pred; a.ids64 = pred64; a.s = sp;
  a.mode = STK_MODE_FULL; a.m = pm; a.l = pl; a.u = pu; a.status = status;
  a.chain = 1;
  const bool few = rows <= nsm / 2;
  a.sm_skip = few ? rows : 0;
  a.l2_lean = few ? 1 : 0;
  rc = launch_jobs(a, kv->kv_dtype, nsm, st);
  if (rc) return cuda_status(rc, "block_states (chained)");
  if (!hybrid) {
    // 3. Saved repair (reuse predicted hits, compute selected misses, merge),
    //    the states' dependent: its wait covers both the states and Top-K.
    RepairArgs r{};
    r.L = a.L;
    r.q = q; r.q_dtype = q_dtype;
    r.rows = rows; r.hq = c.hq; r.g = a.g; r.d = d; r.scale = a.scale;
    r.sel = selected; r.sel64 = 0; r.sa = topk;
    r.pred = pred; r.pred64 = pred64; r.sp = sp;
    r.pmode = STK_PRED_SAVED; r.sc = sp;
    r.pm = pm; r.pl = pl; r.pu = pu;
    r.variant = STK_VAR_SAVED;
    r.max_n = c.max_n;
    r.out = out->out;
    r.status = status;
    r.chain = 1;
    return cuda_status(launch_repair(r, kv->kv_dtype, st), "repair (chained)");
  }
  uint8_t* high = reinterpret_cast<uint8_t*>(w + chain_ws_saved(c.hq, c.total, rows, sp, d));
  float* low_m = reinterpret_cast<float*>(high + align256(slots));
  float* low_l = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(low_m) + align256(rows * sizeof(float)));
  float* low_u = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(low_l) + align256(rows * sizeof(float)));
  float* low_abs = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(low_u) +
                                            align256(static_cast<size_t>(rows) * d * sizeof(float)));
  // 3. Hybrid grouping (kernels.py:94-117) as the states' programmatic
  //    dependent: it waits for their grid, whose completion follows Top-K's.
  rc = launch_hybrid_group(pm, pl, pu, rows, sp, d, mass_threshold, high, low_m, low_l, low_u, low_abs, st, true);
  if (rc) return cuda_status(rc, "hybrid_group");
  // 4. Fused or signed-fused repair, the grouping's programmatic dependent
  //    (it also reads A, written before the states completed). keep_mass
  //    aliases the states' (m, l) (kernels.py:450-477), which the extra-mass
  //    budget reads.
  stk_prediction ps{};
  ps.mode = STK_PRED_HYBRID; ps.sc = sp;
  ps.m = pm; ps.l = pl; ps.u = pu; ps.high = high;
  ps.low_m = low_m; ps.low_l = low_l; ps.low_u = low_u; ps.low_abs = low_abs;
  ps.mass_m = pm; ps.mass_l = pl;
  return repair_entry(kv, q, q_dtype, rows, c.hq, selected, 0, topk, pred, pred64, sp, &ps, variant, min_remaining,
                      cancellation_tol, max_extra_mass, c.max_n, out, status, stream, 1);
}

size_t stk_speculative_step_workspace_bytes(int hq, int n, int sp, int d) {
  if (hq <= 0 || n <= 0 || sp <= 0 || d <= 0) return 0;
  return chain_ws_saved(hq, n, hq, sp, d);
}

int stk_speculative_step(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int hq,
                         int topk, const void* pred, int pred64, int sp, int32_t* selected, float* out,
                         void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (kv->page_table || kv->block_offsets) return fail(STK_EINVAL, "speculative_step takes one dense request");
  ChainShape c{};
  rc = chain_shape(kv, 1, hq, nullptr, 0, 0, &c);
  if (rc) return rc;
  stk_repair_out ro{};
  ro.out = out;
  return chain_step(kv, q, q_dtype, lo, hi, c, topk, pred, pred64, sp, 0.f, STK_VAR_SAVED, 0.f, 0.f, 0.f, selected,
                    &ro, workspace, workspace_bytes, status, stream);
}

size_t stk_speculative_step_batched_workspace_bytes(int R, int hq, int total_blocks, int sp, int d, int hybrid) {
  if (R <= 0 || hq <= 0 || total_blocks <= 0 || sp <= 0 || d <= 0) return 0;
  return hybrid ? chain_ws_hybrid(hq, total_blocks, R * hq, sp, d) : chain_ws_saved(hq, total_blocks, R * hq, sp, d);
}

int stk_speculative_step_batched(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int R,
                                 int hq, int total_blocks, int max_blocks, int topk, const void* pred, int pred64,
                                 int sp, float mass_threshold, int variant, float min_remaining,
                                 float cancellation_tol, float max_extra_mass, int32_t* selected,
                                 const stk_repair_out* out, void* workspace, size_t workspace_bytes, int32_t* status,
                                 void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  ChainShape c{};
  rc = chain_shape(kv, R, hq, kv->block_offsets, total_blocks, max_blocks, &c);
  if (rc) return rc;
  return chain_step(kv, q, q_dtype, lo, hi, c, topk, pred, pred64, sp, mass_threshold, variant, min_remaining,
                    cancellation_tol, max_extra_mass, selected, out, workspace, workspace_bytes, status, stream);
}

static size_t decode_step_ctrl_bytes(int hq, int hkv) {
  return align256(static_cast<size_t>(hkv + 2 * hq + 1) * sizeof(unsigned));
}

size_t stk_decode_step_workspace_bytes(int hq, int hkv, int n, int slots, int d) {
  if (hq <= 0 || hkv <= 0 || n <= 0 || slots <= 0 || d <= 0) return 0;
  const size_t s = static_cast<size_t>(hq) * slots;
  return decode_step_ctrl_bytes(hq, hkv) + align256(stk_select_workspace_bytes(hq, n)) +
         2 * align256(s * sizeof(float)) + align256(s * d * sizeof(float)) + align256(s * sizeof(int32_t));
}

int stk_decode_step(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int hq, int topk,
                    const void* pred, int pred64, int sp, int32_t* selected, float* out, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (kv->page_table || kv->block_offsets || kv->kv_request_stride) return fail(STK_EINVAL, "decode_step takes one dense request");
  if (!q || !lo || !hi || !selected || !out || !workspace || !valid_dtype(q_dtype))
    return fail(STK_EINVAL, "null pointer or unsupported q dtype");
  if ((pred == nullptr) != (sp == 0) || sp < 0) return fail(STK_EINVAL, "pred and sp > 0 go together (sp = 0: serial)");
  const int n = kv->n, d = kv->d;
  if (topk <= 0 || topk > n) return fail(STK_EINVAL, "topk %d outside [1, %d]", topk, n);
  const int nsm = sm_count_current();
  if (const char* why = decode_step_unsupported(hq, kv->hkv, n, kv->b, d, kv->kv_dtype, topk, sp, nsm))
    return fail(STK_ESMEM, "%s", why);
  const uintptr_t align = reinterpret_cast<uintptr_t>(lo) | reinterpret_cast<uintptr_t>(hi) |
                          reinterpret_cast<uintptr_t>(kv->k) | reinterpret_cast<uintptr_t>(kv->v) |
                          reinterpret_cast<uintptr_t>(q);
  if (align & 15) return fail(STK_EINVAL, "q, lo, hi, K and V must be 16-byte aligned");
  const int slots = sp > 0 ? sp : topk;
  if (workspace_bytes < stk_decode_step_workspace_bytes(hq, kv->hkv, n, slots, d))
    return fail(STK_EWS, "decode_step workspace too small");
  unsigned char* w = static_cast<unsigned char*>(workspace);
  StepArgs a{};
  a.q = q; a.q_dtype = q_dtype; a.lo = lo; a.hi = hi; a.k = kv->k; a.v = kv->v;
  a.hq = hq; a.hkv = kv->hkv; a.n = n; a.topk = topk;
  a.pred = pred; a.pred64 = pred64; a.sp = sp;
  a.selected = selected; a.out = out;
  a.ctrl = reinterpret_cast<unsigned*>(w);
  w += decode_step_ctrl_bytes(hq, kv->hkv);
  a.bounds = reinterpret_cast<float2*>(w);
  w += align256(stk_select_workspace_bytes(hq, n));
  const size_t s = static_cast<size_t>(hq) * slots;
  a.sm = reinterpret_cast<float*>(w);
  w += align256(s * sizeof(float));
  a.sl = reinterpret_cast<float*>(w);
  w += align256(s * sizeof(float));
  a.su = reinterpret_cast<float*>(w);
  w += align256(s * d * sizeof(float));
  a.sel_tag = reinterpret_cast<int*>(w);
  a.status = status;
  a.scale = attn_scale(d);
  rc = launch_decode_step(a, kv->kv_dtype, nsm, static_cast<cudaStream_t>(stream));
  if (rc < 0) return fail(STK_ESMEM, "the fused step's shared memory exceeds this device's limit");
  return cuda_status(rc, "decode_step");
}

size_t stk_speculative_step_hybrid_workspace_bytes(int hq, int n, int sp, int d) {
  if (hq <= 0 || n <= 0 || sp <= 0 || d <= 0) return 0;
  return chain_ws_hybrid(hq, n, hq, sp, d);
}

int stk_speculative_step_hybrid(const stk_kv* kv, const void* q, int q_dtype, const float* lo, const float* hi, int hq,
                                int topk, const void* pred, int pred64, int sp, float mass_threshold, int variant,
                                float min_remaining, float cancellation_tol, float max_extra_mass, int32_t* selected,
                                const stk_repair_out* out, void* workspace, size_t workspace_bytes, int32_t* status,
                                void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (kv->page_table || kv->block_offsets) return fail(STK_EINVAL, "speculative_step_hybrid takes one dense request");
  if (variant != STK_VAR_FUSED && variant != STK_VAR_SIGNED_FUSED)
    return fail(STK_EINVAL, "speculative_step_hybrid repairs with STK_VAR_FUSED or STK_VAR_SIGNED_FUSED");
  ChainShape c{};
  rc = chain_shape(kv, 1, hq, nullptr, 0, 0, &c);
  if (rc) return rc;
  return chain_step(kv, q, q_dtype, lo, hi, c, topk, pred, pred64, sp, mass_threshold, variant, min_remaining,
                    cancellation_tol, max_extra_mass, selected, out, workspace, workspace_bytes, status, stream);
}

static int metadata_rows(const stk_kv* kv, int R, int total) {
  if (kv->block_offsets == nullptr) return R == 1 ? kv->n : -1;
  return total;
}

int stk_build_metadata(const stk_kv* kv, int R, int total_blocks, float* lo, float* hi, int32_t* status,
                       void* stream) {
  int rc = check_kv(kv, kv ? kv->hkv : 1);
  if (rc) return rc;
  if (!lo || !hi) return fail(STK_EINVAL, "null metadata output");
  if (R <= 0) return fail(STK_EINVAL, "R must be positive");
  const int total = metadata_rows(kv, R, total_blocks);
  if (total <= 0) return fail(STK_EINVAL, "one dense request (R == 1) or block_offsets with total_blocks > 0 expected");
  (void)status;
  return cuda_status(launch_build_metadata(make_layout(kv), R, total, kv->kv_dtype, lo, hi,
                                           static_cast<cudaStream_t>(stream)),
                     "build_metadata");
}

int stk_append_token(const stk_kv* kv, int R, int total_blocks, const void* k_new, const void* v_new,
                     const int32_t* positions, float* lo, float* hi, int32_t* status, void* stream) {
  int rc = check_kv(kv, kv ? kv->hkv : 1);
  if (rc) return rc;
  if (!k_new || !v_new || !positions || !lo || !hi) return fail(STK_EINVAL, "null pointer");
  if (R <= 0) return fail(STK_EINVAL, "R must be positive");
  const int total = metadata_rows(kv, R, total_blocks);
  if (total <= 0) return fail(STK_EINVAL, "one dense request (R == 1) or block_offsets with total_blocks > 0 expected");
  return cuda_status(launch_append_token(make_layout(kv), R, total, kv->kv_dtype, k_new, v_new, positions, lo, hi,
                                         status, static_cast<cudaStream_t>(stream)),
                     "append_token");
}

int stk_predict(int policy, const int32_t* step_ids, const unsigned long long* step_keys, int ks,
                const int32_t* layer_ids, const unsigned long long* layer_keys, int kl, int rows, int n_blocks,
                int budget, int32_t* out, int32_t* status, void* stream) {
  if (policy < STK_PREDICT_PREVIOUS_STEP || policy > STK_PREDICT_RANK_INTERLEAVE) return fail(STK_EINVAL, "bad policy");
  if (rows <= 0 || budget <= 0 || n_blocks <= 0 || !out) return fail(STK_EINVAL, "bad predict shape");
  const bool need_step = policy != STK_PREDICT_PREVIOUS_LAYER, need_layer = policy != STK_PREDICT_PREVIOUS_STEP;
  if (need_step && (!step_ids || ks <= 0)) return fail(STK_EINVAL, "previous-step IDs required");
  if (need_layer && (!layer_ids || kl <= 0)) return fail(STK_EINVAL, "previous-layer IDs required");
  return cuda_status(launch_predict(policy, need_step ? step_ids : nullptr, need_step ? step_keys : nullptr,
                                    need_step ? ks : 0, need_layer ? layer_ids : nullptr,
                                    need_layer ? layer_keys : nullptr, need_layer ? kl : 0, rows, n_blocks, budget,
                                    out, status, static_cast<cudaStream_t>(stream)),
                     "predict");
}

size_t stk_group_attention_workspace_bytes(int hq, int sa, int b, int d) {
  if (hq <= 0 || sa <= 0 || b <= 0 || d <= 0) return 0;
  const size_t slots = static_cast<size_t>(hq) * group_mma_splits(sa, b);
  return align256(slots * sizeof(float)) * 2 + align256(slots * d * sizeof(float));
}

int stk_group_attention(const stk_kv* kv, const void* q, int q_dtype, int hq, const int32_t* group_ids, int sa,
                        float* out, void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!q || !group_ids || !out || !workspace) return fail(STK_EINVAL, "null pointer");
  if (kv->page_table || kv->block_offsets) return fail(STK_EINVAL, "group attention takes one dense request");
  if (q_dtype != kv->kv_dtype || (q_dtype != STK_BF16 && q_dtype != STK_F16))
    return fail(STK_EINVAL, "group attention needs q and K/V in the same 16-bit type (bf16 or f16)");
  if (kv->d != 64 && kv->d != 128) return fail(STK_EDIM, "group attention supports head dim 64 or 128, not %d", kv->d);
  const int G = hq / kv->hkv;
  if (G > 16) return fail(STK_EINVAL, "group attention tiles at most 16 query heads per KV head, not %d", G);
  if (64 % kv->b) return fail(STK_EINVAL, "block size %d must divide 64", kv->b);
  if (sa <= 0) return fail(STK_EINVAL, "empty block list");
  if ((reinterpret_cast<uintptr_t>(kv->k) | reinterpret_cast<uintptr_t>(kv->v)) & 15)
    return fail(STK_EINVAL, "K/V must be 16-byte aligned");
  if (workspace_bytes < stk_group_attention_workspace_bytes(hq, sa, kv->b, kv->d))
    return fail(STK_EWS, "group attention workspace too small");
  const int splits = group_mma_splits(sa, kv->b);
  const size_t slots = static_cast<size_t>(hq) * splits;
  float* m = static_cast<float*>(workspace);
  float* l = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(m) + align256(slots * sizeof(float)));
  float* u = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(l) + align256(slots * sizeof(float)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = launch_group_mma(make_layout(kv), kv->kv_dtype, q, G, group_ids, sa, attn_scale(kv->d), m, l, u, status, st);
  if (rc) return cuda_status(rc, "group attention");
  return cuda_status(launch_merge(m, l, u, nullptr, hq, splits, kv->d, out, st), "group attention merge");
}

size_t stk_group_repair_saved_workspace_bytes(int hq, int hkv, int sa, int sp, int b, int d) {
  if (hq <= 0 || hkv <= 0 || sa <= 0 || sp <= 0 || b <= 0 || d <= 0) return 0;
  const size_t slots = static_cast<size_t>(hq) * group_mma_splits(sa, b);
  return align256(static_cast<size_t>(hkv) * sa * 4) + align256(static_cast<size_t>(hkv) * 4) +
         align256(static_cast<size_t>(hkv) * sp) + 2 * align256(slots * sizeof(float)) +
         align256(slots * d * sizeof(float));
}

int stk_group_repair_saved(const stk_kv* kv, const void* q, int q_dtype, int hq, const int32_t* selected, int sa,
                           const int32_t* pred, int sp, const float* pm, const float* pl, const float* pu, float* out,
                           void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!q || !selected || !pred || !pm || !pl || !pu || !out || !workspace) return fail(STK_EINVAL, "null pointer");
  if (kv->page_table || kv->block_offsets) return fail(STK_EINVAL, "group repair takes one dense request");
  if (q_dtype != kv->kv_dtype || (q_dtype != STK_BF16 && q_dtype != STK_F16))
    return fail(STK_EINVAL, "group repair needs q and K/V in the same 16-bit type (bf16 or f16)");
  if (kv->d != 64 && kv->d != 128) return fail(STK_EDIM, "group repair supports head dim 64 or 128, not %d", kv->d);
  const int G = hq / kv->hkv;
  if (G > 16) return fail(STK_EINVAL, "group repair tiles at most 16 query heads per KV head, not %d", G);
  if (64 % kv->b) return fail(STK_EINVAL, "block size %d must divide 64", kv->b);
  if (sa <= 0 || sp <= 0) return fail(STK_EINVAL, "empty block list");
  if ((reinterpret_cast<uintptr_t>(kv->k) | reinterpret_cast<uintptr_t>(kv->v)) & 15)
    return fail(STK_EINVAL, "K/V must be 16-byte aligned");
  if (workspace_bytes < stk_group_repair_saved_workspace_bytes(hq, kv->hkv, sa, sp, kv->b, kv->d))
    return fail(STK_EWS, "group repair workspace too small");
  const int splits = group_mma_splits(sa, kv->b);
  const size_t slots = static_cast<size_t>(hq) * splits;
  unsigned char* w = static_cast<unsigned char*>(workspace);
  int* miss = reinterpret_cast<int*>(w);
  w += align256(static_cast<size_t>(kv->hkv) * sa * 4);
  int* count = reinterpret_cast<int*>(w);
  w += align256(static_cast<size_t>(kv->hkv) * 4);
  unsigned char* hit = w;
  w += align256(static_cast<size_t>(kv->hkv) * sp);
  float* sm = reinterpret_cast<float*>(w);
  w += align256(slots * sizeof(float));
  float* sl = reinterpret_cast<float*>(w);
  w += align256(slots * sizeof(float));
  float* su = reinterpret_cast<float*>(w);
  return cuda_status(launch_group_repair(make_layout(kv), kv->kv_dtype, q, G, attn_scale(kv->d), selected, sa, pred, sp, pm, pl, pu, miss,
                                         count, hit, sm, sl, su, out, status, static_cast<cudaStream_t>(stream)),
                     "group repair");
}

int stk_touch_kv(const stk_kv* kv, int rows, int hq, const void* ids, int ids64, int s, float* out, void* stream) {
  int rc = check_kv(kv, hq);
  if (rc) return rc;
  if (!ids || !out || rows <= 0 || s <= 0) return fail(STK_EINVAL, "bad touch arguments");
  return cuda_status(launch_touch(make_layout(kv), rows, hq, hq / kv->hkv, ids, ids64, s, out, kv->kv_dtype,
                                  static_cast<cudaStream_t>(stream)),
                     "touch_kv");
}

}  // extern "C"

// ------------------------------------------------------------------ selection without a caller workspace
//
// Some callers cannot hand this library a device workspace: a host whose
// decode loop must not call cudaMalloc (it can synchronise the whole device
// and stall the other streams of the step, and it is not allowed while the
// stream is being captured), or a plugin interface that passes only input and
// output buffers. For them the score scratch of stk_select_topk (one 8-byte
// slot per row and block: an FP32 score interval, an exact order key, or an
// FP64 score) lives in one file-scope device array instead. Every GPU that
// loads this library holds the array (STK_SELECT_STATIC_MAX_SCORES slots,
// 8 MiB) until the process exits.
//
// In host code `g_select_scores` names a host-side stand-in, not device
// memory, so it is never passed to a kernel. Its device address is looked up
// with cudaGetSymbolAddress on the first call made while a device is current
// and cached together with the identity of that device's context; when the
// context differs (after cudaDeviceReset, the module is loaded again), the
// address is looked up again.
namespace {
static __device__ __align__(256) double g_select_scores[STK_SELECT_STATIC_MAX_SCORES];

std::mutex g_static_setup;
void* g_select_scores_addr[kMaxDevices];
unsigned long long g_select_scores_ctx[kMaxDevices];

// Identity of the calling thread's current context (0 when none is current
// yet), through the driver entry points the runtime hands out.
int current_context_id(unsigned long long* id) {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(f);
  });
  *id = 0;
  if (!get_current || !get_id) return fail(STK_EINVAL, "driver context queries unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return fail(STK_EINVAL, "cuCtxGetCurrent failed");
  if (ctx == nullptr) return 0;
  if (get_id(ctx, id) != CUDA_SUCCESS) return fail(STK_EINVAL, "cuCtxGetId failed");
  return 0;
}

int static_scores_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(STK_EINVAL, "device %d beyond the %d this library tracks", dev, kMaxDevices);
  unsigned long long ctx = 0;
  int rc = current_context_id(&ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_static_setup);
  if (ctx == 0 || g_select_scores_addr[dev] == nullptr || g_select_scores_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_select_scores);  // initialises the context when none is current
    if (e != cudaSuccess || p == nullptr)
      return fail(e != cudaSuccess ? static_cast<int>(e) : STK_EINVAL, "cudaGetSymbolAddress(select scratch): %s",
                  cudaGetErrorString(e));
    rc = current_context_id(&ctx);
    if (rc) return rc;
    g_select_scores_addr[dev] = p;
    g_select_scores_ctx[dev] = ctx;
  }
  *out = g_select_scores_addr[dev];
  return 0;
}
}  // namespace

extern "C" int stk_select_topk_static(const void* q, int q_dtype, const float* lo, const float* hi, int R, int hq,
                                      int hmeta, int n, const int32_t* block_offsets, int total_blocks,
                                      int max_blocks, int d, int topk, int group_select, int id_base,
                                      int32_t* ids_out, unsigned long long* keys_out, int32_t* status,
                                      void* stream) {
  if (R <= 0 || hq <= 0 || hmeta <= 0 || hq % hmeta) return fail(STK_EINVAL, "bad select shape");
  if (block_offsets == nullptr) total_blocks = n;
  if (total_blocks <= 0) return fail(STK_EINVAL, "bad select shape");
  const int hsel = group_select ? hmeta : hq;
  const size_t need = stk_select_workspace_bytes(hsel, total_blocks);
  const size_t have = sizeof(double) * static_cast<size_t>(STK_SELECT_STATIC_MAX_SCORES);
  if (need > have)
    return fail(STK_EWS,
                "selection of %d rows x %d blocks needs %zu bytes of score scratch; the static scratch holds %zu "
                "(STK_SELECT_STATIC_MAX_SCORES = %d scores); use stk_select_topk with a workspace",
                hsel, total_blocks, need, have, STK_SELECT_STATIC_MAX_SCORES);
  void* scratch = nullptr;
  const int rc = static_scores_address(&scratch);
  if (rc) return rc;
  // The score pass writes every slot the Top-K pass reads, so nothing in the
  // shared array has to start at zero.
  return stk_select_topk(q, q_dtype, lo, hi, R, hq, hmeta, n, block_offsets, total_blocks, max_blocks, d, topk,
                         group_select, id_base, ids_out, keys_out, scratch, have, status, stream);
}
