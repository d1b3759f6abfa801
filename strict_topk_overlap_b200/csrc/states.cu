// K2: per-block softmax states over lists of KV blocks, plus the per-row
// grouping / merge epilogues of speculation.
//
// Replaces kernels.py:42-71 (_partial), :74-91 (_merge), :94-117 (_group),
// :263-278 (_mass_only), :281-309 (_compact_group), :312-356 (_compact_values),
// :384-407 (_wrong_aggregate); gqa.py:29-59 (_partial incl. REPAIR slot
// search); gqa_hierarchical.py:22-52 (_packed_partials, per-block states).
//
// Design: persistent CTAs whose warps each stream one (row, block) job at a
// time through a private shared-memory stage (bulk copies on an mbarrier,
// L2 prefetch ahead) and reduce it with half-warp 128-bit tiles (see
// block_state.cuh); misaligned or odd shapes take a plain-load generic kernel
// with the same math.

#include <algorithm>

#include "block_state.cuh"

namespace stk {



struct JobInfo {
  int row, slot;
  long long bid;
  bool active;
};

// Whole-warp job resolution (uniform result in every lane).
__device__ __forceinline__ JobInfo resolve_job(const JobArgs& a, long long job, int lane) {
  JobInfo j;
  j.row = static_cast<int>(job / a.s);
  j.slot = static_cast<int>(job - static_cast<long long>(j.row) * a.s);
  j.bid = load_id(a.ids, a.ids64, job);
  bool act = true;
  if (a.active_mode == 1) act = a.active[j.row] != 0;
  else if (a.active_mode == 2) act = a.active[job] != 0;
  if (a.active_invert) act = !act;
  if (j.bid < 0) act = false;
  if (a.pred != nullptr) {
    int found = -1;
    for (int p = lane; p < a.sp; p += 32) {
      if (load_id(a.pred, a.pred64, static_cast<long long>(j.row) * a.sp + p) == j.bid) found = max(found, p);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(kFull, found, o));
    if (a.slot_out && lane == 0) a.slot_out[job] = found;
    if (found >= 0) act = false;
  }
  if (act) {
    const int r = j.row / a.hq;
    const int nb = request_blocks(a.L, r);
    if (j.bid >= nb) {
      if (lane == 0) report(a.status, kStatusBadBlockId);
      act = false;
    }
  }
  j.active = act;
  return j;
}

// Outputs of a job that reads no KV: the reference writes (-inf, 0, 0).
__device__ __forceinline__ void write_inactive(const JobArgs& a, long long job, int lane) {
  if (a.pred != nullptr) return;  // repair scratch: hits keep no state
  if (a.mode != kModeFixed) {
    if (lane == 0) {
      a.m[job] = neg_inf();
      a.l[job] = 0.f;
    }
    if (a.mode == kModeFull)
      for (int dd = lane; dd < a.d; dd += 32) a.u[job * a.d + dd] = 0.f;
  } else {
    if (lane == 0 && a.l) a.l[job] = 0.f;
    for (int dd = lane; dd < a.d; dd += 32) {
      a.u[job * a.d + dd] = 0.f;
      if (a.uabs) a.uabs[job * a.d + dd] = 0.f;
    }
  }
}

// ------------------------------------------------------------------ fast path
// Persistent CTAs, one per SM. CTA c owns the contiguous job range
// [njobs*c/C, njobs*(c+1)/C), so consecutive jobs mostly share a row (and q).
// Warp w of the CTA serves jobs j0 + w, j0 + w + nw, ... by itself:
//   * 32 of its jobs at a time are resolved lane-parallel (one lane per job:
//     row, block id, activity), so metadata costs one load round trip per 32
//     jobs;
//   * the warp owns NS stages (a ring): the K/V blocks of its first NS jobs
//     are copied at once (lane 0, bulk copies, one per page segment, on the
//     stage's mbarrier), and the copy of job k + NS is issued into job k's
//     stage as soon as job k has been reduced, so with NS = 2 the next block
//     is landing while the current one is reduced; jobs further ahead are
//     prefetched into L2 (cp.async.bulk.prefetch.L2) kWarpPrefetch deep;
//   * the warp reduces each block with half-warp 128-bit tiles
//     (warp_block_state).

constexpr int kFastMaxWarps = 16;
constexpr int kWarpPrefetch = 3;
constexpr int kQRowsStaged = 4;  // q rows of a CTA's range staged in shared memory up front
// Dynamic shared memory the stages may use: 144 KB (9 warps of 16 KiB stages
// at C1), so that the CTAs of a selector that runs beside this kernel still
// fit on the same SM; measured on cold inputs, more stage memory per CTA
// (192 or 224 KB) was not faster.
constexpr size_t kFastStageBudget = 144 * 1024;

#ifdef STK_TRACE
// [cta][warp][8] timeline of the block-state kernel (profiling builds only).
static __device__ unsigned long long g_jobs_trace[148 * kFastMaxWarps * 8];
extern "C" __attribute__((visibility("default"))) void* stk_trace_jobs() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_jobs_trace);
  return p;
}
#define JT(ev) do { if (blockIdx.x < 148 && lane == 0) STK_TRACE_AT(g_jobs_trace, (blockIdx.x * kFastMaxWarps + warp) * 8 + (ev)); } while (0)
#else
#define JT(ev) ((void)0)
#endif

template <typename T, int DPH, int MODE, bool FULL32, int NS>
__global__ void __launch_bounds__(kFastMaxWarps * 32, 1) jobs_fast_kernel(JobArgs a) {
  constexpr int D = 16 * DPH;
  constexpr bool kWantV = MODE != kModeMass;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ uint64_t bar[kFastMaxWarps * NS];
  __shared__ __align__(16) float sq[kQRowsStaged * D];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int B = a.L.b;
  const size_t stage_elems = static_cast<size_t>(B) * D * (kWantV ? 2 : 1);
  T* stages = reinterpret_cast<T*>(smem_raw) + static_cast<size_t>(warp) * NS * stage_elems;
  uint64_t* mb = &bar[warp * NS];
  const unsigned bytes = static_cast<unsigned>(B) * D * sizeof(T) * (kWantV ? 2u : 1u);

  const int njobs = a.rows * a.s;
  const int j0 = static_cast<int>(static_cast<long long>(njobs) * blockIdx.x / gridDim.x);
  const int j1 = static_cast<int>(static_cast<long long>(njobs) * (blockIdx.x + 1) / gridDim.x);
  const int mine = j1 - j0 > warp ? (j1 - j0 - warp + nw - 1) / nw : 0;  // jobs of this warp
  JT(0);
  if (a.chain) pdl_release();
  if (lane < NS) {
    mbar_init(&mb[lane], 1);
    fence_barrier_init();
  }
  // The q rows of this range are loaded before any KV traffic is queued
  // (a load issued behind the range's bulk traffic waits for all of it).
  const int row_first = j1 > j0 ? j0 / a.s : 0;
  const int nq = j1 > j0 ? min(kQRowsStaged, (j1 - 1) / a.s - row_first + 1) : 0;
  for (int i = threadIdx.x; i < nq * D; i += blockDim.x)
    sq[i] = load_any(a.q, a.q_dtype, static_cast<long long>(row_first) * D + i);

  // Lane-parallel resolution of this warp's jobs [base, base + 32).
  long long lb = -1;  // lane's block id, -1 when inactive
  int lrow = 0;
  auto resolve = [&](int base) {
    const int k = base + lane;
    lb = -1;
    lrow = 0;
    if (k < mine) {
      const int job = j0 + warp + k * nw;
      const int row = job / a.s;
      lrow = row;
      long long bid = load_id(a.ids, a.ids64, job);
      bool act = bid >= 0;
      if (a.active_mode == 1) act = act && ((a.active[row] != 0) != (a.active_invert != 0));
      else if (a.active_mode == 2) act = act && ((a.active[job] != 0) != (a.active_invert != 0));
      else if (a.active_mode == 3) act = act && reinterpret_cast<const int*>(a.active)[job] < 0;
      else if (a.active_invert) act = false;
      if (act && bid >= request_blocks(a.L, row / a.hq)) {
        report(a.status, kStatusBadBlockId);
        act = false;
      }
      lb = act ? bid : -1;
    }
  };
  auto issue = [&](int slot, long long bid, int row) {
    const int r = row / a.hq;
    mbar_arrive_expect_tx(&mb[slot], bytes);
    issue_block_copy<T>(a.L, r, (row - r * a.hq) / a.g, bid, stages + slot * stage_elems, kWantV, &mb[slot]);
  };
  auto prefetch_lane = [&]() {
    if (lb >= 0) {
      const int r = lrow / a.hq;
      prefetch_block<T>(a.L, r, (lrow - r * a.hq) / a.g, lb, kWantV);
    }
  };

  int base = 0;
  resolve(0);
  __syncthreads();  // q rows staged, barriers initialised
  // Ring of the next NS jobs (k .. k + NS - 1): block id (-1 inactive) and row.
  long long fb[NS];
  int fr[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    fb[i] = __shfl_sync(kFull, lb, i);
    fr[i] = __shfl_sync(kFull, lrow, i);
    if (i >= mine) fb[i] = -1;
    if (fb[i] >= 0 && lane == 0) issue(i, fb[i], fr[i]);
  }
  // L2 window: jobs NS .. NS + win - 1 now, then one per job (job k + NS
  // is asked for at the start of job k either way).
  const int win = a.l2_lean ? 0 : kWarpPrefetch - 1;
  if (lane >= NS && lane < NS + win) prefetch_lane();
  JT(1);

  unsigned phase = 0;  // bit s: parity of stage s's next completion
  float qf[DPH];
  int q_row = -1;
  int it = 0;
#pragma unroll 1
  for (int k = 0; k < mine; ++k) {
    const int job = j0 + warp + k * nw;
    const int slot = k % NS;
    const long long cb = fb[0];
    const int crow = fr[0];
    // The job that will reuse this stage: k + NS.
    const int kk = k + NS;
    long long nb = -1;
    int nrow = 0;
    if (kk < mine) {
      if (kk - base == 32) {
        base += 32;
        resolve(base);
      }
      nb = __shfl_sync(kFull, lb, kk - base);
      nrow = __shfl_sync(kFull, lrow, kk - base);
    }
    {
      const int pf = k + NS + win - base;
      if (k + NS + win < mine && pf >= 0 && pf < 32 && lane == pf) prefetch_lane();
    }
    if (cb < 0) {
      // Inactive slot: (-inf, 0, 0) as the reference writes; repair scratch keeps no state.
      if (a.pred == nullptr) {
        if (MODE != kModeFixed) {
          if (lane == 0) { a.m[job] = neg_inf(); a.l[job] = 0.f; }
          if (MODE == kModeFull && lane < 16) {
            float z[DPH];
#pragma unroll
            for (int j = 0; j < DPH; ++j) z[j] = 0.f;
            store_vec<DPH>(a.u + static_cast<long long>(job) * D + lane * DPH, z);
          }
        } else {
          if (lane == 0 && a.l) a.l[job] = 0.f;
          if (lane < 16) {
            float z[DPH];
#pragma unroll
            for (int j = 0; j < DPH; ++j) z[j] = 0.f;
            store_vec<DPH>(a.u + static_cast<long long>(job) * D + lane * DPH, z);
            if (a.uabs) store_vec<DPH>(a.uabs + static_cast<long long>(job) * D + lane * DPH, z);
          }
        }
      }
      // The stage is idle: start job k + NS's copy.
      if (nb >= 0 && lane == 0) issue(slot, nb, nrow);
    } else {
      if (crow != q_row) {
        q_row = crow;
        if (crow - row_first < nq) {
#pragma unroll
          for (int j = 0; j < DPH; ++j) qf[j] = sq[(crow - row_first) * D + (lane & 15) * DPH + j];
        } else {
          load_q<DPH>(a.q, a.q_dtype, static_cast<long long>(crow) * D + (lane & 15) * DPH, qf);
        }
      }
      const float frame = MODE == kModeFixed ? a.frame[crow] : 0.f;
      if (it < 1) JT(2);
      const bool ok = mbar_wait(&mb[slot], (phase >> slot) & 1u, a.status);
      phase ^= 1u << slot;
      if (it < 2) JT(3 + 3 * it);
      if (!ok) {
        // The ring's later jobs may have copies in flight too: wait for them
        // (bounded) before this warp stops using its stages.
#pragma unroll
        for (int i = 1; i < NS; ++i) {
          const int st2 = (k + i) % NS;
          if (fb[i] >= 0) mbar_wait_for(&mb[st2], (phase >> st2) & 1u, c_wait_ns);
        }
        if (a.chain) pdl_wait();
        return;
      }
      const T* stage = stages + slot * stage_elems;
      float m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
      for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
      warp_block_state<T, DPH, MODE, FULL32>(stage, stage + static_cast<size_t>(B) * D, B, qf, a.scale, frame, m, l,
                                             u, ua, lane);
      __syncwarp();
      if (it == 0) JT(5);
      // The stage is free: start job k + NS's copy before writing results.
      if (nb >= 0 && lane == 0) issue(slot, nb, nrow);
      if (MODE != kModeFixed) {
        if (lane == 0) { a.m[job] = m; a.l[job] = l; }
      } else if (lane == 0 && a.l) {
        a.l[job] = l;
      }
      if (kWantV && lane < 16) {
        store_vec<DPH>(a.u + static_cast<long long>(job) * D + lane * DPH, u);
        if (MODE == kModeFixed && a.uabs) store_vec<DPH>(a.uabs + static_cast<long long>(job) * D + lane * DPH, ua);
      }
      if (it < 2) JT(4 + 3 * it);
      ++it;
    }
    // Advance the ring.
#pragma unroll
    for (int i = 0; i + 1 < NS; ++i) {
      fb[i] = fb[i + 1];
      fr[i] = fr[i + 1];
    }
    fb[NS - 1] = nb;
    fr[NS - 1] = nrow;
  }
  if (a.chain) pdl_wait();  // this grid completes only after its predecessor
}

// ------------------------------------------------------------------ tiny blocks, wide groups
// Per-block states for blocks of NB <= 8 tokens when several query heads
// share a KV head (12 heads per KV head, 4-token blocks,
// one list per group). One warp takes one (request, KV head, slot): it reads
// the block of the group's first head once and computes the state of every
// head of the group whose ID at that slot is the same; a head with another
// ID then reads its own block (asked into L2 at the start of the slot). Lane
// l owns dims [DPL l, DPL l + DPL) of every token, so a token row is one
// coalesced warp load, and the group's q rows are staged per warp with
// cp.async while the IDs and the block load. The per-(row, block) jobs
// above would read each 2 KiB block once per query head and spend a 32-token
// chunk on 4 tokens. States as everywhere: s = (k . q) * scale, m = max s,
// l = sum exp(s - m), u = sum exp(s - m) v; (-inf, 0, 0) for a negative or
// out-of-range ID (the latter also reported in the status word).
constexpr int kGroupJobWarps = 8;
constexpr int kGroupJobMaxG = 16;

template <int BYTES>
__device__ __forceinline__ void cp_async_ca(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(smem_u32(smem)), "l"(gmem), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Transposed butterfly over NB values: on exit every lane of the group of
// 32 / NB lanes holding token t = lane / (32 / NB) has the warp's sum of v[t].
template <int NB>
__device__ __forceinline__ float transpose_sum(float (&v)[NB], int lane) {
#pragma unroll
  for (int cnt = NB, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
    const int half = cnt >> 1;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? v[i] : v[i + half];
      const float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, off);
    }
  }
  float x = v[0];
#pragma unroll
  for (int off = 16 / NB; off > 0; off >>= 1) x += __shfl_xor_sync(kFull, x, off);
  return x;
}

template <typename T, int DPL, int NB>
__device__ __forceinline__ void load_tiny_block(const T* base, int lane, float (&x)[NB][DPL]) {
  constexpr int D = 32 * DPL;
#pragma unroll
  for (int t = 0; t < NB; ++t) load_vec<T, DPL>(base + static_cast<size_t>(t) * D + lane * DPL, x[t]);
}

template <int DPL, int NB>
__device__ __forceinline__ void tiny_block_state(const float (&qf)[DPL], const float (&kf)[NB][DPL],
                                                 const float (&vf)[NB][DPL], float scale, int lane, float& m,
                                                 float& l, float (&u)[DPL]) {
  constexpr int kLanesPerTok = 32 / NB;
  float p[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc = fmaf(kf[t][j], qf[j], acc);
    p[t] = acc;
  }
  const float s = transpose_sum<NB>(p, lane) * scale;  // logit of token lane / kLanesPerTok
  float mx = s;
#pragma unroll
  for (int off = 16; off >= kLanesPerTok; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
  const float e = expf(s - mx);
  float sum = e;
#pragma unroll
  for (int off = 16; off >= kLanesPerTok; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
  m = mx;
  l = sum;
#pragma unroll
  for (int j = 0; j < DPL; ++j) u[j] = 0.f;
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    const float w = __shfl_sync(kFull, e, t * kLanesPerTok);
#pragma unroll
    for (int j = 0; j < DPL; ++j) u[j] = fmaf(w, vf[t][j], u[j]);
  }
}

// CTAs per SM the register budget is set for (no spills at 4 x 4 and 8 x 4 values per lane).
template <int DPL, int NB>
constexpr int group_ctas_per_sm() { return NB * DPL > 16 ? 2 : (NB * DPL == 16 ? 3 : 4); }

template <typename T, int DPL, int NB>
__global__ void __launch_bounds__(kGroupJobWarps * 32, group_ctas_per_sm<DPL, NB>()) jobs_group_kernel(JobArgs a) {
  constexpr int D = 32 * DPL;
  extern __shared__ __align__(16) unsigned char gq_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T* wq = reinterpret_cast<T*>(gq_raw) + static_cast<size_t>(warp) * kGroupJobMaxG * D + lane * DPL;
  const T* Q = static_cast<const T*>(a.q);
  const T* K = static_cast<const T*>(a.L.k);
  const T* V = static_cast<const T*>(a.L.v);
  const int hkv = a.hq / a.g;
  const long long tasks = static_cast<long long>(a.rows / a.hq) * hkv * a.s;
  const long long stride = static_cast<long long>(gridDim.x) * kGroupJobWarps;
  constexpr unsigned kBlockBytes = static_cast<unsigned>(NB * D * sizeof(T));
#pragma unroll 1
  for (long long t = static_cast<long long>(blockIdx.x) * kGroupJobWarps + warp; t < tasks; t += stride) {
    const int j = static_cast<int>(t % a.s);
    const long long rk = t / a.s;
    const int kv = static_cast<int>(rk % hkv);
    const int r = static_cast<int>(rk / hkv);
    const int row0 = r * a.hq + kv * a.g;
    const int nblk = request_blocks(a.L, r);
    // The group's q rows (each lane copies, and later reads, its own dims).
    for (int h = 0; h < a.g; ++h)
      cp_async_ca<DPL * sizeof(T)>(wq + h * D, Q + static_cast<long long>(row0 + h) * D + lane * DPL);
    cp_async_commit();
    // Lane h < g: head h's ID at this slot.
    long long my = -1;
    if (lane < a.g) my = load_id(a.ids, a.ids64, static_cast<long long>(row0 + lane) * a.s + j);
    const long long lead = __shfl_sync(kFull, my, 0);
    const bool valid = my >= 0 && my < nblk;
    if (lane < a.g && my >= nblk) report(a.status, kStatusBadBlockId);
    if (lane < a.g && valid && my != lead) {
      const long long off = block_seg(a.L, r, kv, my, 0).elem_off;
      bulk_prefetch_l2(K + off, kBlockBytes);
      bulk_prefetch_l2(V + off, kBlockBytes);
    }
    const unsigned shared_heads = __ballot_sync(kFull, lane < a.g && valid && my == lead);
    const unsigned own_heads = __ballot_sync(kFull, lane < a.g && valid && my != lead);
    const unsigned void_heads = __ballot_sync(kFull, lane < a.g && !valid);
    float kf[NB][DPL], vf[NB][DPL];
    if (shared_heads) {
      const long long off = block_seg(a.L, r, kv, lead, 0).elem_off;
      load_tiny_block<T, DPL, NB>(K + off, lane, kf);
      load_tiny_block<T, DPL, NB>(V + off, lane, vf);
    }
    cp_async_wait_all();
    auto finish = [&](int h, float m, float l, const float (&u)[DPL]) {
      const long long job = static_cast<long long>(row0 + h) * a.s + j;
      if (lane == 0) {
        a.m[job] = m;
        a.l[job] = l;
      }
      store_vec<DPL>(a.u + job * D + lane * DPL, u);
    };
    auto one_head = [&](int h) {
      float qf[DPL], u[DPL], m, l;
      load_vec<T, DPL>(wq + h * D, qf);
      tiny_block_state<DPL, NB>(qf, kf, vf, a.scale, lane, m, l, u);
      finish(h, m, l, u);
    };
#pragma unroll 1
    for (unsigned w = shared_heads; w; w &= w - 1) one_head(__ffs(w) - 1);
    // Heads whose ID differs from the first head's: each reads its own block.
#pragma unroll 1
    for (unsigned w = own_heads; w; w &= w - 1) {
      const int h = __ffs(w) - 1;
      const long long off = block_seg(a.L, r, kv, __shfl_sync(kFull, my, h), 0).elem_off;
      load_tiny_block<T, DPL, NB>(K + off, lane, kf);
      load_tiny_block<T, DPL, NB>(V + off, lane, vf);
      one_head(h);
    }
#pragma unroll 1
    for (unsigned w = void_heads; w; w &= w - 1) {
      float z[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) z[i] = 0.f;
      finish(__ffs(w) - 1, neg_inf(), 0.f, z);
    }
  }
}

// Dense K/V, full states, no masks or slot search, whole requests, tiny
// blocks, 2..16 query heads per KV head, q in the K/V dtype.
static bool group_eligible(const JobArgs& a, int elem, int dtype) {
  if (a.mode != kModeFull || a.pred != nullptr || a.active_mode != 0 || a.active_invert || a.chain) return false;
  if (a.L.page_table != nullptr || a.q_dtype != dtype) return false;
  if (a.g < 2 || a.g > kGroupJobMaxG || a.hq % a.g || a.rows % a.hq) return false;
  if (a.d != 64 && a.d != 128) return false;
  if (a.L.b != 2 && a.L.b != 4 && a.L.b != 8) return false;
  if ((a.L.b * a.d * elem) % 16) return false;  // L2 prefetch granularity
  const uintptr_t pk = reinterpret_cast<uintptr_t>(a.L.k), pv = reinterpret_cast<uintptr_t>(a.L.v);
  const uintptr_t pq = reinterpret_cast<uintptr_t>(a.q);
  if ((pk | pv | pq) & 15) return false;
  if (a.L.kv_request_stride % 8) return false;
  return true;
}

template <typename T, int DPL, int NB>
static int launch_group_nb(const JobArgs& a, int num_sms, cudaStream_t stream) {
  const long long tasks = static_cast<long long>(a.rows / a.hq) * (a.hq / a.g) * a.s;
  constexpr int kPerSm = group_ctas_per_sm<DPL, NB>();
  long long ctas = (tasks + kGroupJobWarps - 1) / kGroupJobWarps;
  const long long cap = static_cast<long long>(num_sms) * kPerSm;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  const size_t smem = static_cast<size_t>(kGroupJobWarps) * kGroupJobMaxG * 32 * DPL * sizeof(T);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(jobs_group_kernel<T, DPL, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  jobs_group_kernel<T, DPL, NB><<<static_cast<unsigned>(ctas), kGroupJobWarps * 32, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

template <typename T, int DPL>
static int launch_group_d(const JobArgs& a, int num_sms, cudaStream_t stream) {
  switch (a.L.b) {
    case 2: return launch_group_nb<T, DPL, 2>(a, num_sms, stream);
    case 4: return launch_group_nb<T, DPL, 4>(a, num_sms, stream);
    default: return launch_group_nb<T, DPL, 8>(a, num_sms, stream);
  }
}

template <typename T>
static int launch_group(const JobArgs& a, int num_sms, cudaStream_t stream) {
  return a.d == 64 ? launch_group_d<T, 2>(a, num_sms, stream) : launch_group_d<T, 4>(a, num_sms, stream);
}

// ------------------------------------------------------------------ generic path
// Any D <= 1024, any B, any alignment. Lane = token for QK, lane = dim for PV.
template <typename T>
__global__ void __launch_bounds__(128) jobs_generic_kernel(JobArgs a) {
  extern __shared__ float gsm[];  // per warp: q[d], u[d], ua[d]
  __shared__ float ws[4][32];
  __shared__ long long offs[4][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  const int D = a.d;
  float* qs = gsm + static_cast<size_t>(warp) * 3 * D;
  float* us = qs + D;
  float* uas = us + D;
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  const long long W = static_cast<long long>(gridDim.x) * wpc;
  const T* K = static_cast<const T*>(a.L.k);
  const T* V = static_cast<const T*>(a.L.v);
  const bool want_v = a.mode != kModeMass;
  if (a.chain) pdl_release();

  for (long long job = static_cast<long long>(blockIdx.x) * wpc + warp; job < njobs; job += W) {
    const JobInfo ji = resolve_job(a, job, lane);
    if (!ji.active) {
      write_inactive(a, job, lane);
      continue;
    }
    const int r = ji.row / a.hq;
    const int kv = (ji.row - r * a.hq) / a.g;
    __syncwarp();
    for (int dd = lane; dd < D; dd += 32) {
      qs[dd] = load_any(a.q, a.q_dtype, static_cast<long long>(ji.row) * D + dd);
      us[dd] = 0.f;
      uas[dd] = 0.f;
    }
    __syncwarp();
    const float frame = a.mode == kModeFixed ? a.frame[ji.row] : 0.f;
    float m = neg_inf(), l = 0.f;
    for (int t0 = 0; t0 < a.L.b; t0 += 32) {
      const int t = t0 + lane;
      const int ntok = min(32, a.L.b - t0);
      long long toff = 0;
      float s = neg_inf();
      if (t < a.L.b) {
        int seg = 0, within = t;
        if (a.L.page_table != nullptr) { seg = t / a.L.page_size; within = t - seg * a.L.page_size; }
        const BlockSeg sg = block_seg(a.L, r, kv, ji.bid, seg);
        toff = sg.elem_off + static_cast<long long>(within) * D;
        float acc = 0.f;
        for (int dd = 0; dd < D; ++dd) acc = fmaf(to_f32(K[toff + dd]), qs[dd], acc);
        s = acc * a.scale;
      }
      float w, alpha = 1.f;
      if (a.mode == kModeFixed) {
        w = t < a.L.b ? expf(s - frame) : 0.f;
        l += warp_sum(w);
      } else {
        const float mn = fmaxf(m, warp_max(s));
        alpha = expf(m - mn);
        w = t < a.L.b ? expf(s - mn) : 0.f;
        l = l * alpha + warp_sum(w);
        m = mn;
      }
      if (want_v) {
        ws[warp][lane] = w;
        offs[warp][lane] = toff;
        __syncwarp();
        for (int dd = lane; dd < D; dd += 32) {
          float acc = us[dd] * alpha, aacc = uas[dd];
          for (int tt = 0; tt < ntok; ++tt) {
            const float prod = ws[warp][tt] * to_f32(V[offs[warp][tt] + dd]);
            acc += prod;
            aacc += fabsf(prod);
          }
          us[dd] = acc;
          uas[dd] = aacc;
        }
        __syncwarp();
      }
    }
    __syncwarp();
    if (a.mode != kModeFixed) {
      if (lane == 0) { a.m[job] = m; a.l[job] = l; }
    } else if (lane == 0 && a.l) {
      a.l[job] = l;
    }
    if (want_v) {
      for (int dd = lane; dd < D; dd += 32) {
        a.u[job * D + dd] = us[dd];
        if (a.mode == kModeFixed && a.uabs) a.uabs[job * D + dd] = uas[dd];
      }
    }
  }
  if (a.chain) pdl_wait();  // this grid completes only after its predecessor
}

// ------------------------------------------------------------------ epilogues

// merge_partials (kernels.py:74-91): one CTA of 16 warps per row. Every
// thread takes a stripe of slots for M (max included m, or 0 if none) and
// the weights exp(m - M); warp k then folds slots k, k + 16, ... with 4
// consecutive dims per lane and eight slots' loads in flight, and the warps'
// parts add in warp order (the result does not depend on timing).
__global__ void __launch_bounds__(512) merge_kernel(const float* m, const float* l, const float* u,
                                                   const unsigned char* include, int s, int d, float* out) {
  extern __shared__ __align__(16) float msm[];  // w[s], then part[16][d]
  __shared__ float red[16];
  constexpr int kWarps = 16;
  constexpr int kBatch = 8;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* w = msm;
  float* part = msm + ((s + 3) & ~3);
  const long long base = static_cast<long long>(row) * s;
  float mx = neg_inf();
  for (int i = tid; i < s; i += blockDim.x)
    if (include == nullptr || include[base + i]) mx = fmaxf(mx, m[base + i]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = neg_inf();
#pragma unroll
  for (int k = 0; k < kWarps; ++k) M = fmaxf(M, red[k]);
  if (M == neg_inf()) M = 0.f;
  __syncthreads();
  float z = 0.f;
  for (int i = tid; i < s; i += blockDim.x) {
    const bool inc = include == nullptr || include[base + i];
    const float wi = inc ? expf(m[base + i] - M) : 0.f;
    w[i] = wi;
    if (inc) z += wi * l[base + i];
  }
  z = warp_sum(z);
  if (lane == 0) red[warp] = z;
  __syncthreads();
  float Z = 0.f;
#pragma unroll
  for (int k = 0; k < kWarps; ++k) Z += red[k];
  Z = fmaxf(Z, 1e-30f);
  for (int d0 = 0; d0 < d; d0 += 128) {
    const int dd = d0 + 4 * lane;
    const bool live = dd < d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = warp; i0 < s; i0 += kBatch * kWarps) {
      float4 x[kBatch];
      float wi[kBatch];
#pragma unroll
      for (int c = 0; c < kBatch; ++c) {
        const int i = i0 + c * kWarps;
        wi[c] = i < s ? w[i] : 0.f;
        x[c] = (wi[c] != 0.f && live) ? *reinterpret_cast<const float4*>(u + (base + i) * d + dd)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int c = 0; c < kBatch; ++c) {
        acc.x = fmaf(wi[c], x[c].x, acc.x);
        acc.y = fmaf(wi[c], x[c].y, acc.y);
        acc.z = fmaf(wi[c], x[c].z, acc.z);
        acc.w = fmaf(wi[c], x[c].w, acc.w);
      }
    }
    if (live) *reinterpret_cast<float4*>(part + warp * d + dd) = acc;
  }
  __syncthreads();
  for (int dd = tid; dd < d; dd += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) acc += part[k * d + dd];
    out[static_cast<long long>(row) * d + dd] = acc / Z;
  }
}

// merge_partials (kernels.py:74-91) for head dims that are not a multiple
// of 4: one CTA per row. Warp 0 forms the weights exp(m - M) (M = max
// included m, or 0 if none); threads then reduce the numerators over slots
// with coalesced loads, eight slots in flight.
__global__ void __launch_bounds__(256) merge_scalar_kernel(const float* m, const float* l, const float* u,
                                                   const unsigned char* include, int s, int d, float* out) {
  extern __shared__ __align__(16) float msm[];  // w[s]
  __shared__ float sZ;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  float* w = msm;
  const long long base = static_cast<long long>(row) * s;
  if (tid < 32) {
    float M = neg_inf();
    for (int i = lane; i < s; i += 32) {
      const bool inc = include == nullptr || include[base + i];
      if (inc) M = fmaxf(M, m[base + i]);
    }
    M = warp_max(M);
    if (M == neg_inf()) M = 0.f;
    float z = 0.f;
    for (int i = lane; i < s; i += 32) {
      const bool inc = include == nullptr || include[base + i];
      const float wi = inc ? expf(m[base + i] - M) : 0.f;
      w[i] = wi;
      if (inc) z += wi * l[base + i];
    }
    z = warp_sum(z);
    if (lane == 0) sZ = fmaxf(z, 1e-30f);
  }
  __syncthreads();
  const float z = sZ;
  for (int dd = tid; dd < d; dd += blockDim.x) {
    const float* ur = u + base * d + dd;
    float acc = 0.f;
    int i = 0;
    for (; i + 8 <= s; i += 8) {
      float x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = ur[static_cast<long long>(i + j) * d];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(w[i + j], x[j], acc);
    }
    for (; i < s; ++i) acc = fmaf(w[i], ur[static_cast<long long>(i) * d], acc);
    out[static_cast<long long>(row) * d + dd] = acc / z;
  }
}

// LSE reduction that keeps the state unnormalised: per row, M = max over
// included slots of m (-inf when none), Z = sum exp(m - M) l, U = sum exp(m - M) u.
// The context-parallel path reduces each shard's per-block states to one
// state per row this way before the shards' states are exchanged.
__global__ void __launch_bounds__(512) reduce_states_kernel(const float* m, const float* l, const float* u,
                                                            const unsigned char* include, int s, int d, float* m_out,
                                                            float* l_out, float* u_out) {
  // rsm: w[s] (slot weights), then part[16][d] (each warp's numerators).
  extern __shared__ __align__(16) float rsm[];
  __shared__ float red[16];
  constexpr int kWarps = 16;
  constexpr int kBatch = 8;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* w = rsm;
  float* part = rsm + ((s + 3) & ~3);
  const long long base = static_cast<long long>(row) * s;
  auto included = [&](int i) { return (include == nullptr || include[base + i]) && m[base + i] != neg_inf(); };
  // M and Z over every thread's stripe of slots, then the warps in order.
  float mx = neg_inf();
  for (int i = tid; i < s; i += blockDim.x)
    if (included(i)) mx = fmaxf(mx, m[base + i]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = neg_inf();
#pragma unroll
  for (int k = 0; k < kWarps; ++k) M = fmaxf(M, red[k]);
  __syncthreads();
  float z = 0.f;
  for (int i = tid; i < s; i += blockDim.x) {
    const bool inc = included(i);
    const float wi = inc ? expf(m[base + i] - M) : 0.f;
    w[i] = wi;
    z += inc ? wi * l[base + i] : 0.f;
  }
  z = warp_sum(z);
  if (lane == 0) red[warp] = z;
  __syncthreads();
  if (tid == 0) {
    float Z = 0.f;
    for (int k = 0; k < kWarps; ++k) Z += red[k];
    m_out[row] = M;
    l_out[row] = Z;
  }
  // Warp k folds slots k, k + 16, ... (lane: 4 consecutive dims per 128),
  // eight slots' loads in flight at a time; the warps' parts are then added
  // in warp order, so the result does not depend on timing.
  for (int d0 = 0; d0 < d; d0 += 128) {
    const int dd = d0 + 4 * lane;
    const bool live = dd < d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = warp; i0 < s; i0 += kBatch * kWarps) {
      float4 x[kBatch];
      float wi[kBatch];
#pragma unroll
      for (int c = 0; c < kBatch; ++c) {
        const int i = i0 + c * kWarps;
        wi[c] = i < s ? w[i] : 0.f;
        x[c] = (wi[c] != 0.f && live) ? *reinterpret_cast<const float4*>(u + (base + i) * d + dd)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int c = 0; c < kBatch; ++c) {
        acc.x = fmaf(wi[c], x[c].x, acc.x);
        acc.y = fmaf(wi[c], x[c].y, acc.y);
        acc.z = fmaf(wi[c], x[c].z, acc.z);
        acc.w = fmaf(wi[c], x[c].w, acc.w);
      }
    }
    if (live) *reinterpret_cast<float4*>(part + warp * d + dd) = acc;
  }
  __syncthreads();
  for (int dd = tid; dd < d; dd += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) acc += part[k * d + dd];
    u_out[static_cast<long long>(row) * d + dd] = acc;
  }
}

int launch_reduce_states(const float* m, const float* l, const float* u, const unsigned char* include, int rows,
                         int s, int d, float* m_out, float* l_out, float* u_out, cudaStream_t stream) {
  if (d % 4) return -1;  // 16-byte numerator rows
  const size_t smem = (static_cast<size_t>((s + 3) & ~3) + 16 * static_cast<size_t>(d)) * 4;
  if (smem > 200 * 1024) return -1;
  cudaFuncSetAttribute(reduce_states_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  reduce_states_kernel<<<rows, 512, smem, stream>>>(m, l, u, include, s, d, m_out, l_out, u_out);
  return static_cast<int>(cudaGetLastError());
}

// Slots whose per-dimension loads the grouping kernels issue together.
constexpr int kSlotBatch = 32;

// Hybrid grouping (kernels.py:94-117): high = mass >= tau * total mass,
// low aggregate at low_m = max low m, absolute numerator envelope. The
// row's (m, l) are staged in shared memory in one pass; warp 0 takes the
// slots 32 at a time (warp max / sum reductions); then every thread folds
// dims.
__global__ void hybrid_group_kernel(const float* m, const float* l, const float* u, int s, int d, float tau,
                                    unsigned char* high, float* low_m, float* low_l, float* low_u, float* low_abs) {
  extern __shared__ float hs[];  // alpha[s], then the row's m[s] and l[s]
  float* ms = hs + s;
  float* ls = ms + s;
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const long long base = static_cast<long long>(row) * s;
  // Launched as a programmatic dependent (chained step): the states come
  // from the preceding kernel. Both calls are no-ops in a plain launch.
  pdl_release();
  pdl_wait();
  // The row's (m, l) are read from global memory once, by every thread.
  for (int i = threadIdx.x; i < s; i += blockDim.x) {
    ms[i] = m[base + i];
    ls[i] = l[base + i];
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float gm = neg_inf();
    for (int i = lane; i < s; i += 32) gm = fmaxf(gm, ms[i]);
    gm = warp_max(gm);
    float total = 0.f;
    for (int i = lane; i < s; i += 32) total += expf(ms[i] - gm) * ls[i];
    total = warp_sum(total);
    float lm = neg_inf();
    for (int i = lane; i < s; i += 32) {
      const float mass = expf(ms[i] - gm) * ls[i];
      const bool hi = mass >= tau * total;
      high[base + i] = hi;
      hs[i] = hi ? 0.f : 1.f;
      if (!hi) lm = fmaxf(lm, ms[i]);
    }
    lm = warp_max(lm);
    if (lm == neg_inf()) lm = 0.f;
    float zz = 0.f;
    for (int i = lane; i < s; i += 32) {
      const float al = hs[i] != 0.f ? expf(ms[i] - lm) : 0.f;
      hs[i] = al;
      zz += al * ls[i];
    }
    zz = warp_sum(zz);
    if (lane == 0) {
      low_m[row] = lm;
      low_l[row] = zz;
    }
  }
  __syncthreads();
  // Slot order is kept (the sums are sequential in i); the loads are issued
  // kSlotBatch at a time, so a row costs s / kSlotBatch round trips to the
  // just-written states, not s.
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float uv = 0.f, ua = 0.f;
    int i = 0;
    for (; i + kSlotBatch <= s; i += kSlotBatch) {
      float x[kSlotBatch];
#pragma unroll
      for (int j = 0; j < kSlotBatch; ++j) x[j] = u[(base + i + j) * d + dd];
#pragma unroll
      for (int j = 0; j < kSlotBatch; ++j) {
        const float al = hs[i + j];
        uv += al * x[j];
        ua += al * fabsf(x[j]);
      }
    }
    for (; i < s; ++i) {
      const float al = hs[i];
      const float x = u[(base + i) * d + dd];
      uv += al * x;
      ua += al * fabsf(x);
    }
    low_u[static_cast<long long>(row) * d + dd] = uv;
    low_abs[static_cast<long long>(row) * d + dd] = ua;
  }
}

// Compact grouping (kernels.py:281-309): capacity-C packing of high blocks in
// predicted order with overflow spilled to the low group. One warp per row,
// slots 32 at a time; the high blocks' ranks in predicted order come from a
// ballot prefix count carried across the chunks.
__global__ void compact_group_kernel(const float* pm, const float* pl, const void* pred, int pred64, int s, int c,
                                     float tau, unsigned char* high, void* rids, float* low_m, float* low_l,
                                     unsigned char* overflow) {
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  const long long base = static_cast<long long>(row) * s;
  float gm = neg_inf();
  for (int i = lane; i < s; i += 32) gm = fmaxf(gm, pm[base + i]);
  gm = warp_max(gm);
  float total = 0.f;
  for (int i = lane; i < s; i += 32) total += expf(pm[base + i] - gm) * pl[base + i];
  total = warp_sum(total);
  for (int cc = lane; cc < c; cc += 32) store_id(rids, pred64, static_cast<long long>(row) * c + cc, -1);
  __syncwarp();
  int rank = 0;  // high blocks before this chunk
  float lm = neg_inf();
  for (int i0 = 0; i0 < s; i0 += 32) {
    const int i = i0 + lane;
    bool hi = false;
    if (i < s) hi = (expf(pm[base + i] - gm) * pl[base + i]) >= tau * total;
    const unsigned bal = __ballot_sync(kFull, hi);
    const int my = rank + __popc(bal & ((1u << lane) - 1)) + 1;  // 1-based rank among high blocks
    if (hi) {
      if (my <= c) store_id(rids, pred64, static_cast<long long>(row) * c + my - 1, load_id(pred, pred64, base + i));
      else hi = false;
    }
    if (i < s) {
      high[base + i] = hi;
      if (!hi) lm = fmaxf(lm, pm[base + i]);
    }
    rank += __popc(bal);
  }
  if (lane == 0) overflow[row] = rank > c;
  lm = warp_max(lm);
  if (lm == neg_inf()) lm = 0.f;
  float ll = 0.f;
  for (int i = lane; i < s; i += 32)
    if (!high[base + i]) ll += expf(pm[base + i] - lm) * pl[base + i];
  ll = warp_sum(ll);
  if (lane == 0) {
    low_m[row] = lm;
    low_l[row] = ll;
  }
}

// Sum per-slot vectors in slot order: out[row, :] = sum_i x[row, i, :].
__global__ void slot_sum_kernel(const float* x, const float* y, int s, int d, float* out_x, float* out_y) {
  const int row = blockIdx.x;
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float ax = 0.f, ay = 0.f;
    int i = 0;
    for (; i + kSlotBatch <= s; i += kSlotBatch) {  // batched loads, sums in slot order
      float bx[kSlotBatch], by[kSlotBatch];
#pragma unroll
      for (int t = 0; t < kSlotBatch; ++t) {
        const long long j = (static_cast<long long>(row) * s + i + t) * d + dd;
        bx[t] = x[j];
        by[t] = y ? y[j] : 0.f;
      }
#pragma unroll
      for (int t = 0; t < kSlotBatch; ++t) {
        ax += bx[t];
        if (y) ay += by[t];
      }
    }
    for (; i < s; ++i) {
      const long long j = (static_cast<long long>(row) * s + i) * d + dd;
      ax += x[j];
      if (y) ay += y[j];
    }
    out_x[static_cast<long long>(row) * d + dd] = ax;
    if (y) out_y[static_cast<long long>(row) * d + dd] = ay;
  }
}

// ------------------------------------------------------------------ host side

static size_t ws_stage_bytes(const JobArgs& a, int elem) {
  return static_cast<size_t>(a.L.b) * a.d * elem * (a.mode == kModeMass ? 1 : 2);
}

static bool fast_eligible(const JobArgs& a, int elem) {
  if (a.d != 64 && a.d != 128 && a.d != 256) return false;
  if (a.pred != nullptr) return false;  // slot search: generic kernel
  if (static_cast<long long>(a.rows) * a.s > 0x7fffffffll) return false;
  // At least four whole-block stages must fit the shared-memory plan.
  if (4 * ws_stage_bytes(a, elem) > 200 * 1024) return false;
  const uintptr_t pk = reinterpret_cast<uintptr_t>(a.L.k), pv = reinterpret_cast<uintptr_t>(a.L.v);
  if ((pk | pv) & 15) return false;
  if ((a.d * elem) % 16) return false;
  if (a.L.page_table != nullptr && (a.L.b % a.L.page_size)) return false;
  if (a.L.kv_request_stride % 8) return false;
  return true;
}


template <typename T, int DPH, int MODE, int NS>
static int launch_fast_ns(const JobArgs& a, int num_sms, cudaStream_t stream) {
  const size_t stage = ws_stage_bytes(a, sizeof(T)) * NS;
  size_t nw = kFastStageBudget / stage;
  if (nw > kFastMaxWarps) nw = kFastMaxWarps;
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  long long ctas = num_sms;
  if (a.chain && a.sm_skip > 0 && a.sm_skip <= num_sms / 2) ctas = num_sms - a.sm_skip;
  // Small problems: fewer CTAs so that no warp is left without a job.
  if (njobs < ctas * static_cast<long long>(nw)) ctas = (njobs + nw - 1) / nw;
  if (ctas < 1) ctas = 1;
  const size_t smem = stage * nw;
  auto kern = a.L.b % 32 == 0 ? jobs_fast_kernel<T, DPH, MODE, true, NS> : jobs_fast_kernel<T, DPH, MODE, false, NS>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  if (a.chain) return launch_pdl(kern, dim3(static_cast<unsigned>(ctas)), dim3(static_cast<unsigned>(nw * 32)), smem,
                                 stream, 0, a);
  kern<<<static_cast<unsigned>(ctas), static_cast<unsigned>(nw * 32), smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

// One stage per warp. Measured on cold inputs (C1), two stages per warp with
// half the warps were slower (11.3 µs against 10.9 µs per launch); with the
// L2 window already pulling later jobs, more warps beat deeper rings. For
// 4-token blocks an eight-stage ring was slower still
// (114 µs against 73 µs per launch).
template <typename T, int DPH, int MODE>
static int launch_fast_t(const JobArgs& a, int num_sms, cudaStream_t stream) {
  return launch_fast_ns<T, DPH, MODE, 1>(a, num_sms, stream);
}

template <typename T, int MODE>
static int launch_fast_d(const JobArgs& a, int num_sms, cudaStream_t stream) {
  switch (a.d) {
    case 64: return launch_fast_t<T, 4, MODE>(a, num_sms, stream);
    case 128: return launch_fast_t<T, 8, MODE>(a, num_sms, stream);
    default: return launch_fast_t<T, 16, MODE>(a, num_sms, stream);
  }
}

// The predicted-slot search of a job list whose hits are skipped (the
// context-parallel shard states): slot_out[job] = the highest pred slot of
// the row holding the job's block, -1 when none (one warp per job).
__global__ void __launch_bounds__(256) slot_search_kernel(JobArgs a) {
  const int lane = threadIdx.x & 31;
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  const long long nw = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long job = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; job < njobs;
       job += nw) {
    const int row = static_cast<int>(job / a.s);
    const long long bid = load_id(a.ids, a.ids64, job);
    int found = -1;
    if (bid >= 0)
      for (int p = lane; p < a.sp; p += 32)
        if (load_id(a.pred, a.pred64, static_cast<long long>(row) * a.sp + p) == bid) found = max(found, p);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(kFull, found, o));
    if (lane == 0) a.slot_out[job] = found;
  }
}

template <typename T>
static int launch_jobs_t(const JobArgs& a, int num_sms, cudaStream_t stream) {
  if (a.pred != nullptr && a.slot_out != nullptr && !a.chain && a.active_mode == 0 && !a.active_invert) {
    // Hits skipped: the slot search first, then the fast kernel over the
    // misses (active iff slot_out < 0; hits keep no state, as a.pred is set).
    JobArgs b = a;
    b.pred = nullptr;
    if (fast_eligible(b, sizeof(T))) {
      const long long njobs = static_cast<long long>(a.rows) * a.s;
      const long long ctas = std::min<long long>((njobs + 7) / 8, static_cast<long long>(num_sms) * 8);
      slot_search_kernel<<<static_cast<unsigned>(ctas), 256, 0, stream>>>(a);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return static_cast<int>(e);
      b.pred = a.pred;
      b.active = reinterpret_cast<const unsigned char*>(a.slot_out);
      b.active_mode = 3;
      switch (b.mode) {
        case kModeFull: return launch_fast_d<T, kModeFull>(b, num_sms, stream);
        case kModeMass: return launch_fast_d<T, kModeMass>(b, num_sms, stream);
        default: return launch_fast_d<T, kModeFixed>(b, num_sms, stream);
      }
    }
  }
  constexpr int kCode = sizeof(T) == 4 ? kF32 : (std::is_same<T, __half>::value ? kF16 : kBF16);
  if (group_eligible(a, sizeof(T), kCode)) return launch_group<T>(a, num_sms, stream);
  if (fast_eligible(a, sizeof(T))) {
    switch (a.mode) {
      case kModeFull: return launch_fast_d<T, kModeFull>(a, num_sms, stream);
      case kModeMass: return launch_fast_d<T, kModeMass>(a, num_sms, stream);
      default: return launch_fast_d<T, kModeFixed>(a, num_sms, stream);
    }
  }
  const size_t smem = static_cast<size_t>(4) * 3 * a.d * sizeof(float);
  cudaFuncSetAttribute(jobs_generic_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  long long ctas = (njobs + 3) / 4;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  if (a.chain) return launch_pdl(jobs_generic_kernel<T>, dim3(static_cast<unsigned>(ctas)), dim3(128), smem, stream, 0, a);
  jobs_generic_kernel<T><<<static_cast<unsigned>(ctas), 128, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int launch_jobs(const JobArgs& a, int kv_dtype, int num_sms, cudaStream_t stream) {
  if (static_cast<long long>(a.rows) * a.s == 0) return 0;
  switch (kv_dtype) {
    case kF32: return launch_jobs_t<float>(a, num_sms, stream);
    case kF16: return launch_jobs_t<__half>(a, num_sms, stream);
    default: return launch_jobs_t<__nv_bfloat16>(a, num_sms, stream);
  }
}

int launch_merge(const float* m, const float* l, const float* u, const unsigned char* include, int rows, int s, int d,
                 float* out, cudaStream_t stream) {
  const size_t wide_smem = (static_cast<size_t>((s + 3) & ~3) + 16 * static_cast<size_t>(d)) * 4;
  if (d % 4 == 0 && wide_smem <= 200 * 1024) {
    const size_t smem = wide_smem;
    cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    merge_kernel<<<rows, 512, smem, stream>>>(m, l, u, include, s, d, out);
    return static_cast<int>(cudaGetLastError());
  }
  const size_t smem = static_cast<size_t>(s) * 4;
  if (smem > 200 * 1024) return -1;
  cudaFuncSetAttribute(merge_scalar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  merge_scalar_kernel<<<rows, 256, smem, stream>>>(m, l, u, include, s, d, out);
  return static_cast<int>(cudaGetLastError());
}

int launch_hybrid_group(const float* m, const float* l, const float* u, int rows, int s, int d, float tau,
                        unsigned char* high, float* low_m, float* low_l, float* low_u, float* low_abs,
                        cudaStream_t stream, bool chain) {
  const size_t smem = static_cast<size_t>(s) * 3 * sizeof(float);
  if (smem > 48 * 1024) cudaFuncSetAttribute(hybrid_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
  if (chain)
    return launch_pdl(hybrid_group_kernel, dim3(rows), dim3(128), smem, stream, 0, m, l, u, s, d, tau, high, low_m,
                      low_l, low_u, low_abs);
  hybrid_group_kernel<<<rows, 128, smem, stream>>>(m, l, u, s, d, tau, high, low_m, low_l, low_u, low_abs);
  return static_cast<int>(cudaGetLastError());
}

int launch_compact_group(const float* pm, const float* pl, const void* pred, int pred64, int rows, int s, int c,
                         float tau, unsigned char* high, void* rids, float* low_m, float* low_l,
                         unsigned char* overflow, cudaStream_t stream) {
  compact_group_kernel<<<rows, 32, 0, stream>>>(pm, pl, pred, pred64, s, c, tau, high, rids, low_m, low_l, overflow);
  return static_cast<int>(cudaGetLastError());
}

int launch_slot_sum(const float* x, const float* y, int rows, int s, int d, float* out_x, float* out_y,
                    cudaStream_t stream) {
  slot_sum_kernel<<<rows, 128, 0, stream>>>(x, y, s, d, out_x, out_y);
  return static_cast<int>(cudaGetLastError());
}

// touch_kv (kernels.py:250-260): per (row, slot, 1024-element tile) checksum
// of K + V over the block's elements, read in token-major order.
template <typename T>
__global__ void touch_kernel(KVLayout L, int hq, int g, const void* ids, int ids64, int s, float* out) {
  const int row = blockIdx.x, slot = blockIdx.y, tile = blockIdx.z;
  const int ntiles = gridDim.z;
  const int r = row / hq, kv = (row - r * hq) / g;
  const long long bid = load_id(ids, ids64, static_cast<long long>(row) * s + slot);
  __shared__ float red[32];
  float acc = 0.f;
  if (bid >= 0 && bid < request_blocks(L, r)) {
    const T* K = static_cast<const T*>(L.k);
    const T* V = static_cast<const T*>(L.v);
    const int total = L.b * L.d;
    for (int x = tile * 1024 + threadIdx.x; x < min(total, (tile + 1) * 1024); x += blockDim.x) {
      const int t = x / L.d, dd = x - t * L.d;
      int seg = 0, within = t;
      if (L.page_table != nullptr) { seg = t / L.page_size; within = t - seg * L.page_size; }
      const long long o = block_seg(L, r, kv, bid, seg).elem_off + static_cast<long long>(within) * L.d + dd;
      acc += to_f32(K[o]) + to_f32(V[o]);
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
    out[(static_cast<long long>(row) * s + slot) * ntiles + tile] = t;
  }
}

int launch_touch(const KVLayout& L, int rows, int hq, int g, const void* ids, int ids64, int s, float* out,
                 int kv_dtype, cudaStream_t stream) {
  const int ntiles = (L.b * L.d + 1023) / 1024;
  dim3 grid(rows, s, ntiles);
  switch (kv_dtype) {
    case kF32: touch_kernel<float><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
    case kF16: touch_kernel<__half><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
    default: touch_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
  }
  return static_cast<int>(cudaGetLastError());
}

int set_wait_limit_states(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
