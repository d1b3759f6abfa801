// K3: one repair kernel for every strict / relaxed repair entry point.
//
// Replaces, with one launch per call:
//   kernels.py:120-247,359-407 + repair()       (split repair, 3-5 launches)
//   fused.py:10-173          (_accumulate, _repair)
//   signed_repair.py:18-172  (_schedule, _signed_partials, _merge) + _fallback
//   signed_fused.py:14-145   (_kv_tile, _corrections, _finalize)
//   gqa.py:29-104            (REPAIR _partial + _merge_repair, saved and union)
//   gqa_light.py:10-60       (_repair_light)
//   gqa_hierarchical.py:99-130 (_match_ids, REPAIR packed partials, _groups)
//   kernels.py:437-447       (exact_attention = repair with no prediction)
//
// One thread-block cluster of CS CTAs (kNW warps each, CS <= 8 chosen on the
// host) serves one (request, query head) row. Phases:
//   1. every CTA of the cluster takes the row's set difference A vs P through
//      shared-memory bitmaps over block IDs — hit / miss / high / wrong-low
//      flags, the optional extra-mass budget (EPS) and the job queue (misses
//      in A order, then wrong-low blocks in P order) — so every CTA holds the
//      same queue without talking to the others;
//   2. CTA c takes queue entries c, c + CS, c + 2 CS, ...: it asks L2 for all
//      of their blocks at once (cp.async.bulk.prefetch.L2), then each warp
//      streams its entries through a private shared-memory stage with bulk
//      copies and reduces them — misses are added (+) to a per-warp LSE
//      state, wrong-low blocks subtracted (-) from the low group in its own
//      exponent frame — while the CTA's threads merge retained prediction
//      slots c, c + CS, ... (weights relative to the row's retained maximum);
//   3. per-warp states merge into one CTA partial; after a cluster barrier
//      every CTA reads all CS partials through distributed shared memory in
//      rank order, so every CTA holds bit-identical row totals and takes the
//      same guard decision (remaining low mass, cancellation envelope,
//      non-finite output); rank 0 writes the outputs;
//   4. a flagged row recomputes the strict selected set across the cluster,
//      in this launch.
// Waits on bulk copies are bounded; a warp whose wait ran out records the
// status, stops issuing work and its CTA still takes part in every cluster
// barrier.
#include <cooperative_groups.h>

#include "block_state.cuh"

namespace cg = cooperative_groups;

namespace stk {

constexpr int kNW = 4;          // warps per CTA
constexpr int kMaxCluster = 8;  // CTAs per row (portable cluster size)

#ifdef STK_TRACE
// [cta][8] timeline of the repair kernel (profiling builds only).
static __device__ unsigned long long g_repair_trace[4096 * 8];
extern "C" __attribute__((visibility("default"))) void* stk_trace_repair() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_repair_trace);
  return p;
}
#define RT(ev) do { if (blockIdx.x < 4096 && threadIdx.x == 0) STK_TRACE_AT(g_repair_trace, blockIdx.x * 8 + (ev)); } while (0)
#else
#define RT(ev) ((void)0)
#endif

// Negative-job frame rules.
enum NegRule : int { kNegPerToken = 0, kNegBlockRescale = 1 };

struct RowScalars {
  int miss_count, wrong_count, queue_len;
  int low_hit;
  int skip;
  float extra;
  float lm;
};

__device__ __forceinline__ bool bit_test(const unsigned* bits, long long i) {
  return (bits[i >> 5] >> (i & 31)) & 1u;
}

// Merge a block state into a warp's positive aggregate (shared memory).
__device__ __forceinline__ void agg_pos_merge(float* S, float* U, int d, float mb, float lb, const float* ub_lane,
                                              int dpl, int lane, bool lane_contig) {
  if (mb == neg_inf()) return;
  const float M = S[0];
  const float Mn = fmaxf(M, mb);
  const float a1 = expf(M - Mn), a2 = expf(mb - Mn);
  __syncwarp();
  if (lane_contig) {
    // Half-warp layout: lanes 16h + i hold dims [i*dpl, (i+1)*dpl) (halves agree).
    if (lane < 16)
      for (int j = 0; j < dpl; ++j) {
        const int dd = lane * dpl + j;
        if (dd < d) U[dd] = U[dd] * a1 + ub_lane[j] * a2;
      }
  } else {
    for (int j = 0, dd = lane; dd < d; ++j, dd += 32) U[dd] = U[dd] * a1 + ub_lane[j] * a2;
  }
  __syncwarp();
  if (lane == 0) {
    S[1] = S[1] * a1 + lb * a2;
    S[0] = Mn;
  }
  __syncwarp();
}

struct RepairSmem {
  float* pw;      // [sc] retained weights exp(pm - M_keep) (0 when not kept)
  unsigned* bitA;
  unsigned* bitP;
  long long* a_ids;
  long long* p_ids;
  int* queue;
  float* aggU;    // [kNW + 1][d]: per-warp positive numerators, then the retained share
  float* aggN;    // [kNW][d]: per-warp negative numerators (low frame)
  float* aggS;    // [kNW + 1][4]: M, Z, Zneg, -
  float* vecA;    // [d] CTA partial: positive numerator (read by the cluster)
  float* vecB;    // [d] CTA partial: negative numerator (read by the cluster)
  float* cS;      // [4] CTA partial scalars: M, Z, Zneg, - (read by the cluster)
  float* gU;      // [d] row total positive numerator
  float* gN;      // [d] row total negative numerator
  float* pm_s;    // [sc] retained maxima
  float* pl_s;    // [sc] retained normalisers
  float* mm_s;    // [sp] keep_mass maxima (budget)
  float* ml_s;    // [sp] keep_mass normalisers (budget)
  float* lu_s;    // [d] low-group numerator
  float* la_s;    // [d] low-group absolute envelope
  float* qv;      // [d] q as FP32
  unsigned char* high_s;  // [sp]
  unsigned char* a_miss;
  unsigned char* p_flag;  // bit0 hit, bit1 high, bit2 wrong
  unsigned char* keep;
};

template <int DPH, int NST, typename T>
__host__ __device__ inline size_t repair_layout(const RepairArgs& a, RepairSmem* S, unsigned char* base) {
  const int D = a.d;
  size_t off = 0;
  auto take = [&](size_t bytes, size_t align) {
    off = (off + align - 1) & ~(align - 1);
    const size_t at = off;
    off += bytes;
    return at;
  };
  const size_t stages = DPH > 0 ? static_cast<size_t>(kNW) * NST * 2 * 32 * D * sizeof(T) : 0;
  take(stages, 128);
  const size_t pw_at = take(static_cast<size_t>(a.sc) * 4, 16);
  const int nwords = (a.max_n + 31) / 32;
  const size_t ba = take(nwords * 4, 16), bp = take(nwords * 4, 16);
  const size_t ai = take(static_cast<size_t>(a.sa) * 8, 16), pi = take(static_cast<size_t>(a.sp) * 8, 16);
  const size_t qu = take(static_cast<size_t>(a.sa + a.sp) * 4, 16);
  const size_t au = take(static_cast<size_t>(kNW + 1) * D * 4, 16);
  const size_t an = take(static_cast<size_t>(kNW) * D * 4, 16);
  const size_t as = take(static_cast<size_t>(kNW + 1) * 16, 16);
  const size_t va = take(D * 4, 16), vb = take(D * 4, 16), cs = take(16, 16);
  const size_t gu = take(D * 4, 16), gn = take(D * 4, 16);
  const size_t pms = take(static_cast<size_t>(a.sc) * 4, 16), pls = take(static_cast<size_t>(a.sc) * 4, 16);
  const size_t mms = take(static_cast<size_t>(a.sp) * 4, 16), mls = take(static_cast<size_t>(a.sp) * 4, 16);
  const size_t lus = take(D * 4, 16), las = take(D * 4, 16), qs = take(D * 4, 16);
  const size_t hs = take(a.sp, 1);
  const size_t am = take(a.sa, 1), pf = take(a.sp, 1), kp = take(a.sc, 1);
  if (S != nullptr) {
    S->pw = reinterpret_cast<float*>(base + pw_at);
    S->bitA = reinterpret_cast<unsigned*>(base + ba);
    S->bitP = reinterpret_cast<unsigned*>(base + bp);
    S->a_ids = reinterpret_cast<long long*>(base + ai);
    S->p_ids = reinterpret_cast<long long*>(base + pi);
    S->queue = reinterpret_cast<int*>(base + qu);
    S->aggU = reinterpret_cast<float*>(base + au);
    S->aggN = reinterpret_cast<float*>(base + an);
    S->aggS = reinterpret_cast<float*>(base + as);
    S->vecA = reinterpret_cast<float*>(base + va);
    S->vecB = reinterpret_cast<float*>(base + vb);
    S->cS = reinterpret_cast<float*>(base + cs);
    S->gU = reinterpret_cast<float*>(base + gu);
    S->gN = reinterpret_cast<float*>(base + gn);
    S->pm_s = reinterpret_cast<float*>(base + pms);
    S->pl_s = reinterpret_cast<float*>(base + pls);
    S->mm_s = reinterpret_cast<float*>(base + mms);
    S->ml_s = reinterpret_cast<float*>(base + mls);
    S->lu_s = reinterpret_cast<float*>(base + lus);
    S->la_s = reinterpret_cast<float*>(base + las);
    S->qv = reinterpret_cast<float*>(base + qs);
    S->high_s = base + hs;
    S->a_miss = base + am;
    S->p_flag = base + pf;
    S->keep = base + kp;
  }
  return off;
}

// ------------------------------------------------------------------ kernel

template <typename T, int DPH, int NST, bool FULL32>
__global__ void __launch_bounds__(kNW * 32) repair_kernel(RepairArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bars[kNW * NST];
  __shared__ RowScalars rs;
  __shared__ int sh_count[4];
  __shared__ float sh_f[8];
  __shared__ int sh_failed;

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());

  // A launch whose cluster shape differs from the host's plan (rows x CS
  // CTAs in clusters of CS) would map CTAs to the wrong rows: refuse it.
  if (CS != a.cluster || gridDim.x != static_cast<unsigned>(a.rows) * a.cluster) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  constexpr bool kFast = DPH > 0;
  const int D = kFast ? 16 * DPH : a.d;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x / CS;
  const int r = row / a.hq;
  const int kv = (row - r * a.hq) / a.g;
  const int nblocks = request_blocks(a.L, r);
  const bool hybrid = a.pmode == kPredHybrid || a.pmode == kPredCompact;
  const bool has_pred = a.pmode != kPredNone;

  RT(0);
  if (a.chain) pdl_wait();  // programmatic dependent: inputs come from the preceding kernel
  RepairSmem S;
  repair_layout<DPH, NST, T>(a, &S, smem);
  T* stages = reinterpret_cast<T*>(smem);
  const int nwords = (a.max_n + 31) / 32;

  // ---- phase 0: barriers.
  if (lane == 0) {
    if (kFast)
      for (int st = 0; st < NST; ++st) mbar_init(&bars[warp * NST + st], 1);
    fence_barrier_init();
  }
  if (tid == 0) sh_failed = 0;

  // ---- phase 1: every per-row global load in one independent pass.
  const bool want_mass = hybrid && a.eps > 0.f && a.mass_m != nullptr;
  for (int i = tid; i < nwords; i += blockDim.x) { S.bitA[i] = 0; S.bitP[i] = 0; }
  for (int i = tid; i < a.sa; i += blockDim.x) S.a_ids[i] = load_id(a.sel, a.sel64, static_cast<long long>(row) * a.sa + i);
  if (has_pred) {
    const long long pr = static_cast<long long>(row) * a.sp, sr = static_cast<long long>(row) * a.sc;
    for (int i = tid; i < a.sp; i += blockDim.x) {
      S.p_ids[i] = load_id(a.pred, a.pred64, pr + i);
      S.high_s[i] = hybrid ? a.high[pr + i] : 0;
      if (want_mass) { S.mm_s[i] = a.mass_m[pr + i]; S.ml_s[i] = a.mass_l[pr + i]; }
    }
    for (int c = tid; c < a.sc; c += blockDim.x) {
      S.pm_s[c] = a.pm[sr + c];
      S.pl_s[c] = a.pl[sr + c];
      if (a.pmode == kPredCompact) S.keep[c] = 0, S.pw[c] = 0.f;
    }
    if (a.pmode == kPredCompact)
      for (int c = tid; c < a.sc; c += blockDim.x) {
        // Compact retained IDs are checked against A after the bitmaps exist.
        const long long id = load_id(a.rids, a.rids64, sr + c);
        S.pw[c] = __int_as_float(static_cast<int>(id));  // staged temporarily
      }
    if (hybrid)
      for (int dd = tid; dd < D; dd += blockDim.x) {
        S.lu_s[dd] = a.low_u[static_cast<long long>(row) * D + dd];
        S.la_s[dd] = a.low_abs[static_cast<long long>(row) * D + dd];
      }
  }
  for (int dd = tid; dd < D; dd += blockDim.x) S.qv[dd] = load_any(a.q, a.q_dtype, static_cast<long long>(row) * D + dd);
  __syncthreads();
  RT(1);
  for (int i = tid; i < a.sa; i += blockDim.x) {
    long long id = S.a_ids[i];
    if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); id = -1; S.a_ids[i] = -1; }
    if (id >= 0) atomicOr(&S.bitA[id >> 5], 1u << (id & 31));
  }
  if (has_pred) {
    for (int i = tid; i < a.sp; i += blockDim.x) {
      long long id = S.p_ids[i];
      if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); id = -1; S.p_ids[i] = -1; }
      if (id >= 0) atomicOr(&S.bitP[id >> 5], 1u << (id & 31));
    }
  }
  __syncthreads();
  for (int i = tid; i < a.sa; i += blockDim.x) {
    const long long id = S.a_ids[i];
    S.a_miss[i] = id >= 0 && !(has_pred && bit_test(S.bitP, id));
  }
  for (int i = tid; i < a.sp && has_pred; i += blockDim.x) {
    const long long id = S.p_ids[i];
    const bool hit = id >= 0 && bit_test(S.bitA, id);
    S.p_flag[i] = (hit ? 1 : 0) | (S.high_s[i] ? 2 : 0);
  }
  for (int c = tid; c < a.sc && has_pred; c += blockDim.x) {
    bool kp;
    if (a.variant == kVarUnion) {
      kp = true;
    } else if (a.pmode == kPredCompact) {
      const long long id = static_cast<long long>(__float_as_int(S.pw[c]));
      kp = id >= 0 && id < nblocks && bit_test(S.bitA, id);
    } else {
      // saved: every hit; hybrid: hits that were kept high.
      const long long id = S.p_ids[c];
      const bool hit = id >= 0 && bit_test(S.bitA, id);
      kp = hit && (a.pmode == kPredSaved || S.high_s[c] != 0);
    }
    S.keep[c] = kp;
    S.pw[c] = kp ? S.pm_s[c] : neg_inf();
  }
  __syncthreads();

  // ---- phase 1b (warp 0): counts, low_hit, extra-mass budget, queue;
  //      (warp 1): retained-state weights and this CTA's share of their mass.
  if (warp == 0) {
    int low_hit = 0;
    if (hybrid) {
      for (int i = lane; i < a.sp; i += 32) low_hit |= ((S.p_flag[i] & 3) == 1);
      low_hit = __any_sync(kFull, low_hit);
    }
    int wrong_count = 0;
    if (hybrid && low_hit) {
      for (int i = lane; i < a.sp; i += 32) {
        const bool w = (S.p_flag[i] & 3) == 0 && S.p_ids[i] >= 0;
        if (w) S.p_flag[i] |= 4;
        wrong_count += w;
      }
      wrong_count = warp_sum_int(wrong_count);
    }
    __syncwarp();
    float lm = neg_inf();
    int skip = 0;
    float extra = 0.f;
    if (hybrid && low_hit) lm = a.low_m[row];
    const bool eps_variant = a.variant == kVarFused || a.variant == kVarSigned || a.variant == kVarSignedFused;
    if (eps_variant && a.eps > 0.f && hybrid && low_hit && wrong_count > 0) {
      // Reference: fused.py:104-112, signed_repair.py:60-73.
      float rm = neg_inf();
      for (int c = lane; c < a.sc; c += 32)
        if (S.keep[c]) rm = fmaxf(rm, S.pm_s[c]);
      rm = warp_max(rm);
      const float ref = fmaxf(rm, lm);
      float wm = 0.f, den = 0.f;
      for (int i = lane; i < a.sp; i += 32)
        if (S.p_flag[i] & 4) wm += expf(S.mm_s[i] - ref) * S.ml_s[i];
      for (int c = lane; c < a.sc; c += 32)
        if (S.keep[c]) den += expf(S.pm_s[c] - ref) * S.pl_s[c];
      wm = warp_sum(wm);
      den = warp_sum(den);
      den += expf(lm - ref) * a.low_l[row];
      extra = wm / den;
      skip = extra <= a.eps;
    }
    int n = 0;
    for (int base = 0; base < a.sa; base += 32) {
      const int i = base + lane;
      const bool m = i < a.sa && S.a_miss[i];
      const unsigned bal = __ballot_sync(kFull, m);
      if (m) S.queue[n + __popc(bal & ((1u << lane) - 1))] = i;
      n += __popc(bal);
    }
    const int miss_count = n;
    if (hybrid && low_hit && !skip) {
      for (int base = 0; base < a.sp; base += 32) {
        const int i = base + lane;
        const bool w = i < a.sp && (S.p_flag[i] & 4);
        const unsigned bal = __ballot_sync(kFull, w);
        if (w) S.queue[n + __popc(bal & ((1u << lane) - 1))] = a.sa + i;
        n += __popc(bal);
      }
    }
    if (lane == 0) {
      rs.miss_count = miss_count;
      rs.wrong_count = n - miss_count;
      rs.queue_len = n;
      rs.low_hit = low_hit;
      rs.skip = skip;
      rs.extra = extra;
      rs.lm = lm;
    }
  } else if (warp == 1 && has_pred) {
    // Retained weights relative to the row's retained maximum M (the same in
    // every CTA); this CTA's share of Z covers slots rank, rank + CS, ...
    float M = neg_inf();
    for (int c = lane; c < a.sc; c += 32) M = fmaxf(M, S.pw[c]);
    M = warp_max(M);
    float Z = 0.f;
    for (int c = lane; c < a.sc; c += 32) {
      const float w = S.keep[c] ? expf(S.pw[c] - M) : 0.f;
      S.pw[c] = w;
      if (S.keep[c] && c % CS == rank) Z += w * S.pl_s[c];
    }
    Z = warp_sum(Z);
    if (lane == 0) {
      S.aggS[kNW * 4 + 0] = M;
      S.aggS[kNW * 4 + 1] = Z;
    }
  }
  for (int i = tid; i < (kNW + 1) * D; i += blockDim.x) S.aggU[i] = 0.f;
  for (int i = tid; i < kNW * D; i += blockDim.x) S.aggN[i] = 0.f;
  if (lane == 0 && warp < kNW) {
    S.aggS[warp * 4 + 0] = neg_inf();
    S.aggS[warp * 4 + 1] = 0.f;
    S.aggS[warp * 4 + 2] = 0.f;
    S.aggS[warp * 4 + 3] = 0.f;
  }
  if (tid == 0 && !has_pred) {
    S.aggS[kNW * 4 + 0] = neg_inf();
    S.aggS[kNW * 4 + 1] = 0.f;
  }
  __syncthreads();

  const int neg_rule =
      (a.variant == kVarFused || (a.variant == kVarSignedFused && a.pmode == kPredCompact) ||
       (a.variant == kVarSplit && a.pmode == kPredCompact))
          ? kNegPerToken
          : kNegBlockRescale;
  const float lm = rs.lm;
  float* myU = S.aggU + warp * D;
  float* myN = S.aggN + warp * D;
  float* myS = S.aggS + warp * 4;

  constexpr int kQ = kFast ? DPH : 1;
  float qf[kQ];
  if constexpr (kFast) {
#pragma unroll
    for (int j = 0; j < DPH; ++j) qf[j] = S.qv[(lane & 15) * DPH + j];
  }

  // ---- per-warp block pipeline. Queue entry k belongs to CTA k % CS and,
  // within it, to warp (k / CS) % kNW; items = (entry, 32-token chunk).
  const int kfirst = rank + CS * warp, kstep = CS * kNW;
  unsigned phase_bits = 0;
  const int nchunks = (a.L.b + 31) / 32;
  constexpr int kChunkElems = 32 * 16 * (DPH > 0 ? DPH : 1);
  T* wst = stages + static_cast<size_t>(warp) * NST * (2 * kChunkElems);
  uint64_t* wbar = bars + warp * NST;
  int ik = kfirst, ic = 0;  // issue cursor
  bool fallback_pass = false;
  bool warp_failed = false;
  int count = 0;
  auto job_entry = [&](int k, long long& bid, bool& negative) {
    const int e = fallback_pass ? k : S.queue[k];
    negative = !fallback_pass && e >= a.sa;
    bid = negative ? S.p_ids[e - a.sa] : S.a_ids[e];
  };
  auto job_valid = [&](int k) { return fallback_pass ? S.a_ids[k] >= 0 : true; };
  auto issue = [&](int st) {
    if (ik >= count) return;
    if (lane == 0) {
      long long bid; bool neg;
      job_entry(ik, bid, neg);
      const int t0 = ic * 32, ntok = min(32, a.L.b - t0);
      T* ks = wst + static_cast<size_t>(st) * 2 * kChunkElems;
      T* vs = ks + kChunkElems;
      const unsigned bytes = static_cast<unsigned>(ntok * D * sizeof(T));
      mbar_arrive_expect_tx(&wbar[st], 2 * bytes);
      const T* K = static_cast<const T*>(a.L.k);
      const T* V = static_cast<const T*>(a.L.v);
      if (a.L.page_table == nullptr) {
        const long long o = block_seg(a.L, r, kv, bid, 0).elem_off + static_cast<long long>(t0) * D;
        bulk_g2s(ks, K + o, bytes, &wbar[st]);
        bulk_g2s(vs, V + o, bytes, &wbar[st]);
      } else {
        for (int t = t0; t < t0 + ntok;) {
          const int pg = t / a.L.page_size, po = t - pg * a.L.page_size;
          const int cnt = min(a.L.page_size - po, t0 + ntok - t);
          const long long o = block_seg(a.L, r, kv, bid, pg).elem_off + static_cast<long long>(po) * D;
          const unsigned sb = static_cast<unsigned>(cnt * D * sizeof(T));
          bulk_g2s(ks + (t - t0) * D, K + o, sb, &wbar[st]);
          bulk_g2s(vs + (t - t0) * D, V + o, sb, &wbar[st]);
          t += cnt;
        }
      }
    }
    if (++ic == nchunks) {
      ic = 0;
      ik += kstep;
      while (ik < count && !job_valid(ik)) ik += kstep;
    }
  };
  // Start a pass over `cnt` entries: every thread asks L2 for one of this
  // CTA's blocks, then each warp issues its first chunk copies.
  auto prefill = [&](int cnt, bool fb) {
    fallback_pass = fb;
    count = cnt;
    if constexpr (kFast) {
      for (int i = tid;; i += blockDim.x) {
        const int k = rank + CS * i;
        if (k >= cnt) break;
        if (!job_valid(k)) continue;
        long long bid; bool neg;
        job_entry(k, bid, neg);
        prefetch_block<T>(a.L, r, kv, bid, true);
      }
    }
    ik = kfirst;
    ic = 0;
    while (ik < count && !job_valid(ik)) ik += kstep;
    if constexpr (kFast) {
      for (int st = 0; st < NST; ++st) issue(st);
      __syncwarp();
    }
  };

  auto consume = [&]() {
    if constexpr (kFast) {
      int item = 0;
      float m, l, u[DPH], ua[DPH];
      for (int k = kfirst; k < count; k += kstep) {
        if (!job_valid(k)) continue;
        long long bid; bool neg;
        job_entry(k, bid, neg);
        const bool per_token = neg && neg_rule == kNegPerToken;
        m = neg_inf(); l = 0.f;
#pragma unroll
        for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
        for (int c = 0; c < nchunks; ++c, ++item) {
          const int st = item % NST;
          if (!mbar_wait(&wbar[st], (phase_bits >> st) & 1u, a.status)) return false;
          phase_bits ^= 1u << st;
          const int t0 = c * 32, ntok = min(32, a.L.b - t0);
          const T* ks = wst + static_cast<size_t>(st) * 2 * kChunkElems;
          if (per_token)
            warp_block_state<T, DPH, kModeFixed, FULL32>(ks, ks + kChunkElems, ntok, qf, a.scale, lm, m, l, u, ua, lane);
          else
            warp_block_state<T, DPH, kModeFull, FULL32>(ks, ks + kChunkElems, ntok, qf, a.scale, 0.f, m, l, u, ua, lane);
          (void)t0;
          __syncwarp();
          issue(st);
        }
        if (!neg) {
          agg_pos_merge(myS, myU, D, m, l, u, DPH, lane, true);
        } else {
          const float f = per_token ? 1.f : expf(m - lm);
          if (lane < 16) {
#pragma unroll
            for (int j = 0; j < DPH; ++j) myN[lane * DPH + j] += u[j] * f;
          }
          __syncwarp();
          if (lane == 0) myS[2] += l * f;
          __syncwarp();
        }
      }
    } else {
      // Generic: lane = token for QK (q from qv), lane = dim for PV.
      const T* K = static_cast<const T*>(a.L.k);
      const T* V = static_cast<const T*>(a.L.v);
      __shared__ float gw[kNW][32];
      __shared__ long long go[kNW][32];
      const int per = (D + 31) / 32;
      for (int k = kfirst; k < count; k += kstep) {
        if (!job_valid(k)) continue;
        long long bid; bool neg;
        job_entry(k, bid, neg);
        const bool per_token = neg && neg_rule == kNegPerToken;
        float m = neg_inf(), l = 0.f;
        float u[32];
        for (int t = 0; t < 32; ++t) u[t] = 0.f;
        for (int t0 = 0; t0 < a.L.b; t0 += 32) {
          const int t = t0 + lane, ntok = min(32, a.L.b - t0);
          long long toff = 0;
          float s = neg_inf();
          if (t < a.L.b) {
            int seg = 0, within = t;
            if (a.L.page_table != nullptr) { seg = t / a.L.page_size; within = t - seg * a.L.page_size; }
            toff = block_seg(a.L, r, kv, bid, seg).elem_off + static_cast<long long>(within) * D;
            float acc = 0.f;
            for (int dd = 0; dd < D; ++dd) acc = fmaf(to_f32(K[toff + dd]), S.qv[dd], acc);
            s = acc * a.scale;
          }
          float w, al = 1.f;
          if (per_token) {
            w = t < a.L.b ? expf(s - lm) : 0.f;
            l += warp_sum(w);
          } else {
            const float mn = fmaxf(m, warp_max(s));
            al = expf(m - mn);
            w = t < a.L.b ? expf(s - mn) : 0.f;
            l = l * al + warp_sum(w);
            m = mn;
          }
          gw[warp][lane] = w;
          go[warp][lane] = toff;
          __syncwarp();
          for (int i = 0, dd = lane; i < per && i < 32; ++i, dd += 32) {
            if (dd >= D) break;
            float acc = u[i] * al;
            for (int tt = 0; tt < ntok; ++tt) acc += gw[warp][tt] * to_f32(V[go[warp][tt] + dd]);
            u[i] = acc;
          }
          __syncwarp();
        }
        if (!neg) {
          agg_pos_merge(myS, myU, D, m, l, u, per, lane, false);
        } else {
          const float f = per_token ? 1.f : expf(m - lm);
          for (int i = 0, dd = lane; i < per && dd < D; ++i, dd += 32) myN[dd] += u[i] * f;
          __syncwarp();
          if (lane == 0) myS[2] += l * f;
          __syncwarp();
        }
      }
    }
    return true;
  };

  // Per-warp aggregates (+ the retained share) -> this CTA's partial.
  auto cta_partial = [&](bool with_retained) {
    const int nagg = with_retained ? kNW + 1 : kNW;
    if (tid == 0) {
      float M = neg_inf();
      for (int w = 0; w < nagg; ++w) M = fmaxf(M, S.aggS[w * 4]);
      float Z = 0.f, Zn = 0.f;
      for (int w = 0; w < nagg; ++w) {
        if (S.aggS[w * 4] != neg_inf()) Z += expf(S.aggS[w * 4] - M) * S.aggS[w * 4 + 1];
        if (w < kNW) Zn += S.aggS[w * 4 + 2];
      }
      S.cS[0] = M;
      S.cS[1] = Z;
      S.cS[2] = Zn;
      sh_f[4] = M;
    }
    __syncthreads();
    const float M = sh_f[4];
    for (int dd = tid; dd < D; dd += blockDim.x) {
      float U = 0.f, N = 0.f;
      for (int w = 0; w < nagg; ++w) {
        const float Mw = S.aggS[w * 4];
        if (Mw != neg_inf()) U += expf(Mw - M) * S.aggU[w * D + dd];
        if (w < kNW) N += S.aggN[w * D + dd];
      }
      S.vecA[dd] = U;
      S.vecB[dd] = N;
    }
  };
  // Row totals from every CTA's partial, in rank order (distributed shared
  // memory), into sh_f[0..2] and gU / gN. Ends with a cluster barrier, after
  // which no CTA reads another's partial any more.
  auto cluster_totals = [&]() {
    cluster.sync();
    if (tid == 0) {
      float M = neg_inf();
      for (int c = 0; c < CS; ++c) M = fmaxf(M, cluster.map_shared_rank(S.cS, c)[0]);
      float Z = 0.f, Zn = 0.f;
      for (int c = 0; c < CS; ++c) {
        const float* cs = cluster.map_shared_rank(S.cS, c);
        if (cs[0] != neg_inf()) Z += expf(cs[0] - M) * cs[1];
        Zn += cs[2];
      }
      sh_f[0] = M;
      sh_f[1] = Z;
      sh_f[2] = Zn;
    }
    __syncthreads();
    const float M = sh_f[0];
    for (int dd = tid; dd < D; dd += blockDim.x) {
      float U = 0.f, N = 0.f;
      for (int c = 0; c < CS; ++c) {
        const float Mc = cluster.map_shared_rank(S.cS, c)[0];
        if (Mc != neg_inf()) U += expf(Mc - M) * cluster.map_shared_rank(S.vecA, c)[dd];
        N += cluster.map_shared_rank(S.vecB, c)[dd];
      }
      S.gU[dd] = U;
      S.gN[dd] = N;
    }
    cluster.sync();
  };

  // ---- phase 2: prefetch + first copies, retained share, then queued blocks.
  RT(2);
  prefill(rs.queue_len, false);
  RT(3);
  if (has_pred) {
    float* keepU = S.aggU + kNW * D;
    const float* pu = a.pu + static_cast<long long>(row) * a.sc * D;
    // The CTA's slots are loaded kKeepBatch at a time (in bounds whatever
    // the weight) and folded in slot order, skipping zero weights as before:
    // one round trip to the states per batch instead of one per slot.
    constexpr int kKeepBatch = 8;
    for (int dd = tid; dd < D; dd += blockDim.x) {
      float acc = 0.f;
      for (int c0 = rank; c0 < a.sc; c0 += CS * kKeepBatch) {
        float x[kKeepBatch];
#pragma unroll
        for (int t = 0; t < kKeepBatch; ++t) {
          const int c = c0 + t * CS;
          x[t] = c < a.sc ? pu[static_cast<long long>(c) * D + dd] : 0.f;
        }
#pragma unroll
        for (int t = 0; t < kKeepBatch; ++t) {
          const int c = c0 + t * CS;
          if (c < a.sc) {
            const float w = S.pw[c];
            if (w != 0.f) acc = fmaf(w, x[t], acc);
          }
        }
      }
      keepU[dd] = acc;
    }
  }
  if (!consume()) warp_failed = true;
  RT(4);
  __syncthreads();

  // ---- phase 3: CTA partial, cluster totals, guards (identical in every CTA).
  cta_partial(true);
  RT(5);
  cluster_totals();
  RT(6);
  if (tid < 4) sh_count[tid] = 0;
  __syncthreads();
  const float Mp = sh_f[0], Zp = sh_f[1], Zn = sh_f[2];

  const bool low_hit = rs.low_hit != 0;
  float fraction = 1.f;
  bool bad = false;
  float z_final, cp, cl_scale;
  if (a.variant == kVarSplit && hybrid) {
    // kernels.py:172-221: everything in the common frame m.
    const float m = fmaxf(Mp, low_hit ? lm : neg_inf());
    const float lowalpha = low_hit ? expf(lm - m) : 0.f;
    const float ll = low_hit ? a.low_l[row] * lowalpha : 0.f;
    const float removed = Zn * lowalpha;
    const float remaining_mass = ll - removed;
    fraction = ll > 0.f ? remaining_mass / fmaxf(ll, 1e-30f) : 1.f;
    cp = Mp == neg_inf() ? 0.f : expf(Mp - m);
    const float z = remaining_mass + cp * Zp;
    int cancel = 0, invalid = 0;
    for (int dd = tid; dd < D; dd += blockDim.x) {
      const float lu = low_hit ? S.lu_s[dd] * lowalpha : 0.f;
      const float ru = S.gN[dd] * lowalpha;
      const float residual = lu - ru;
      const float labs = low_hit ? S.la_s[dd] * lowalpha : 0.f;
      const float sc = labs + fabsf(ru);
      cancel |= low_hit && (fabsf(residual) < a.cancel_tol * sc) && (sc > 0.f);
      const float o = (residual + cp * S.gU[dd]) / fmaxf(z, 1e-30f);
      invalid |= !isfinite(o);
    }
    if (cancel) atomicOr(&sh_count[0], 1);
    if (invalid) atomicOr(&sh_count[1], 1);
    __syncthreads();
    bad = (z <= 0.f) || (fraction < a.min_remaining) || (fraction != fraction) || isinf(z) || sh_count[0] ||
          sh_count[1];
    z_final = fmaxf(z, 1e-30f);
    cl_scale = lowalpha;
  } else if (hybrid && a.variant != kVarSaved && a.variant != kVarUnion) {
    // fused.py:94-166 / signed_repair.py:139-165 / signed_fused.py:90-125: low frame.
    float mass = 0.f;
    if (low_hit) {
      const float ll = a.low_l[row];
      mass = ll - Zn;
      fraction = mass / ll;
      int cancel = 0;
      for (int dd = tid; dd < D; dd += blockDim.x) {
        const float residual = S.lu_s[dd] - S.gN[dd];
        const float sc = S.la_s[dd] + fabsf(S.gN[dd]);
        cancel |= (fabsf(residual) < a.cancel_tol * sc) && (sc > 0.f);
      }
      if (cancel) atomicOr(&sh_count[0], 1);
    }
    const float m = fmaxf(Mp, low_hit ? lm : neg_inf());
    const float ref = m == neg_inf() ? 0.f : m;
    cp = Mp == neg_inf() ? 0.f : expf(Mp - ref);
    const float lw = low_hit ? expf(lm - ref) : 0.f;
    const float z = cp * Zp + lw * mass;
    int invalid = 0;
    for (int dd = tid; dd < D; dd += blockDim.x) {
      const float resid = low_hit ? S.lu_s[dd] - S.gN[dd] : 0.f;
      const float o = (cp * S.gU[dd] + lw * resid) / z;
      invalid |= !isfinite(o);
    }
    if (invalid) atomicOr(&sh_count[1], 1);
    __syncthreads();
    bad = (low_hit && ((fraction < a.min_remaining) || (fraction != fraction) || sh_count[0])) || (z <= 0.f) ||
          isinf(z) || sh_count[1];
    z_final = z;
    cl_scale = lw;
  } else {
    // Saved / union / exact: plain LSE merge of retained states and misses.
    cp = 1.f;
    cl_scale = 0.f;
    z_final = Zp;
  }

  if (bad) {
    // ---- phase 4: strict fallback over A, spread over the cluster (every
    // CTA took the same decision, so every CTA reaches the same barriers).
    for (int i = tid; i < (kNW + 1) * D; i += blockDim.x) S.aggU[i] = 0.f;
    if (lane == 0) { S.aggS[warp * 4] = neg_inf(); S.aggS[warp * 4 + 1] = 0.f; S.aggS[warp * 4 + 2] = 0.f; }
    __syncthreads();
    if (!warp_failed) {
      prefill(a.sa, true);
      if (!consume()) warp_failed = true;
    }
    __syncthreads();
    cta_partial(false);
    cluster_totals();
    if (rank == 0) {
      const float Z = sh_f[1];
      for (int dd = tid; dd < D; dd += blockDim.x) a.out[static_cast<long long>(row) * D + dd] = S.gU[dd] / Z;
    }
  } else if (rank == 0) {
    for (int dd = tid; dd < D; dd += blockDim.x) {
      float lowv = 0.f;
      if (cl_scale != 0.f) lowv = S.lu_s[dd] - S.gN[dd];
      a.out[static_cast<long long>(row) * D + dd] = (cp * S.gU[dd] + cl_scale * lowv) / z_final;
    }
  }
  RT(7);
  if (rank == 0 && tid == 0) {
    if (a.fallback) a.fallback[row] = bad;
    if (a.remaining) a.remaining[row] = fraction;
    if (a.approx) a.approx[row] = rs.skip && !bad;
    if (a.extra) a.extra[row] = (rs.skip && !bad) ? rs.extra : 0.f;
    if (a.pos_out) a.pos_out[row] = rs.miss_count;
    if (a.total_out) a.total_out[row] = rs.queue_len;
  }
  (void)sh_failed;
}

// ------------------------------------------------------------------ host side

// CTAs per row: enough warps for the row's largest pass (A for a strict
// fallback or exact attention, P for wrong-low blocks) at one block per warp,
// up to the portable cluster size.
static int repair_cluster_size(const RepairArgs& a) {
  const int jobs = a.sa > a.sp ? a.sa : a.sp;
  int cs = (jobs + kNW - 1) / kNW;
  if (cs > kMaxCluster) cs = kMaxCluster;
  if (cs < 1) cs = 1;
  return cs;
}

template <typename T, int DPH>
static int launch_repair_t(RepairArgs a, cudaStream_t stream) {
  constexpr int NST = 1;
  a.stage_pred = 0;
  const size_t smem = repair_layout<DPH, NST, T>(a, nullptr, nullptr);
  if (smem > 220 * 1024) return -2;
  auto kern = a.L.b % 32 == 0 ? repair_kernel<T, DPH, NST, true> : repair_kernel<T, DPH, NST, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  const int cs = repair_cluster_size(a);
  a.cluster = cs;
  if (a.chain)
    return launch_pdl(kern, dim3(static_cast<unsigned>(a.rows) * cs), dim3(kNW * 32), smem, stream, cs, a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.rows) * cs, 1, 1);
  cfg.blockDim = dim3(kNW * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, a));
}

template <typename T>
static int launch_repair_dt(const RepairArgs& a, cudaStream_t stream) {
  const uintptr_t pk = reinterpret_cast<uintptr_t>(a.L.k) | reinterpret_cast<uintptr_t>(a.L.v);
  const bool aligned = (pk & 15) == 0 && (a.d * static_cast<int>(sizeof(T))) % 16 == 0 &&
                       (a.L.page_table == nullptr || a.L.b % a.L.page_size == 0) && a.L.kv_request_stride % 8 == 0;
  const size_t fast_stage = static_cast<size_t>(kNW) * 2 * 32 * a.d * sizeof(T);
  if (aligned && fast_stage <= 128 * 1024) {
    if (a.d == 64) return launch_repair_t<T, 4>(a, stream);
    if (a.d == 128) return launch_repair_t<T, 8>(a, stream);
  }
  if (a.d > 1024) return -3;
  return launch_repair_t<T, 0>(a, stream);
}

int launch_repair(const RepairArgs& a, int kv_dtype, cudaStream_t stream) {
  if (a.rows == 0) return 0;
  const int rc = launch_attend(a, kv_dtype, stream);
  if (rc != 1) return rc;
  switch (kv_dtype) {
    case kF32: return launch_repair_dt<float>(a, stream);
    case kF16: return launch_repair_dt<__half>(a, stream);
    default: return launch_repair_dt<__nv_bfloat16>(a, stream);
  }
}

int set_wait_limit_repair(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
