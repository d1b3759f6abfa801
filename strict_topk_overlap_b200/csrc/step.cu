// The whole decode step in one persistent, cooperative launch.
//
// Replaces, for one dense request (D = 128, 32-token blocks, 16-bit K/V):
//   * the speculative saved step of the reference harness
//     (benchmarks/run_benchmark.py:99-118): selection (selector.py:8-43,
//     gqa.py:15-26,145-161) || predicted-block states (kernels.py:42-71,
//     gqa.py:29-59,128-137), then the saved repair (gqa.py:62-104,186-188);
//   * the serial step (critical_path.py:110, run_benchmark.py:139):
//     selection, then exact attention over the selected blocks
//     (kernels.py:445-447, gqa.py:140-142).
//
// Why one launch: at decode sizes every stage is latency-bound. Launched
// separately, each kernel pays a launch, a cold instruction cache and a grid
// drain before its successor's wait returns; the predicted-block stream can
// only overlap the Top-K kernel's latency. Here the metadata stream, the
// predicted-block stream and the per-row selections run concurrently on all
// SMs, and each row's repair starts as soon as its own inputs are ready.
//
// Grid: one CTA per SM, launched cooperatively so that every CTA is resident
// and a CTA may wait for another's progress (each such wait is bounded by
// the library's wait limit and reports STK_STATUS_WAIT_TIMEOUT when it runs
// out). Every CTA scores its share of the metadata. The last hq CTAs are
// row CTAs: CTA grid - hq + r then selects row r's strict Top-K (the second
// stage of the two-stage selection, topk.cuh) and finishes row r. The other
// (work) CTAs then compute per-block states: of the predicted blocks
// (speculative step, right behind their metadata), or of the selected blocks
// as each row's selection is published (serial step).
//
// Inside a CTA, warp 11 issues 1-D bulk copies into a ring of 11 stages of
// 16 KiB (each on a "full" mbarrier with the copy's byte count) in item
// order: first the CTA's metadata items (16 blocks of one KV head: their lo
// rows, then their hi rows), then its block items (one block's K then V).
// Item it goes to stage it % 11 and is reduced by warp it % 11, which then
// releases the stage on its "empty" mbarrier: each stage has one consumer
// warp, which therefore waits on the stage's phases one after the other (a
// parity wait cannot tell a phase from the one two phases later, so two
// warps must never take turns on one stage). Warps 12..15 join for the
// selection and the row's repair. The small loads (q, predicted IDs) are
// issued before any bulk copy: a load queued behind the bulk stream waits
// for all of it.
//
// Cross-CTA progress goes through counters in the workspace's control
// block, which must be zero before the first call on a workspace; the last
// CTA to finish a call zeroes it again:
//   ctrl[mh]                metadata items done for KV head mh,
//   ctrl[hkv + r]           block states done for row r,
//   ctrl[hkv + hq + r]      row r's selection published (serial step),
//   ctrl[hkv + 2 hq]        CTAs finished.
// A writer publishes after its global writes with a fence and an atomic add;
// a reader waits with acquire loads and reads the data through L2.

#include "block_state.cuh"
#include "common.cuh"

#ifdef STK_TRACE
namespace stk {
// [cta][32] timeline of the fused step (profiling builds only).
static __device__ unsigned long long g_step_trace[256 * 32];
static __device__ long long g_step_clk[256 * 8];
}  // namespace stk
// Phases of the selection inside the fused step: events 16 + ev, thread 0
// (global timer), and the SM cycle counter beside it.
#define STK_TOPK_PROBE(ev) do { if (threadIdx.x == 0 && blockIdx.x < 256) { STK_TRACE_AT(stk::g_step_trace, blockIdx.x * 32 + 16 + (ev)); stk::g_step_clk[blockIdx.x * 8 + (ev)] = clock64(); } } while (0)
#endif
#include "topk.cuh"

namespace stk {

constexpr int kStepThreads = 512;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepStages = 11;               // ring stages = consumer warps 0..10
constexpr int kStepProducer = kStepStages;     // warp 11 issues the bulk copies
constexpr int kStepD = 128;
constexpr int kStepB = 32;
constexpr int kStepDPH = kStepD / 16;
constexpr int kStageBytes = 2 * kStepB * kStepD * 2;            // one 16-bit K+V block: 16 KiB
constexpr int kMetaItemBlocks = kStageBytes / (2 * kStepD * 4);  // 16 blocks of FP32 lo + hi
constexpr int kStepMaxList = 256;                                // topk and predicted-list limit
constexpr int kStepMaxBlocks = 4096;                             // blocks per request limit

#ifdef STK_TRACE
extern "C" __attribute__((visibility("default"))) int stk_trace_step_clk(void* host) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_step_clk, sizeof(g_step_clk)));
}
extern "C" __attribute__((visibility("default"))) int stk_trace_step_read(void* host, size_t bytes, int clear) {
  int rc = static_cast<int>(cudaMemcpyFromSymbol(host, g_step_trace, bytes));
  if (!rc && clear) {
    static unsigned long long zeros[256 * 32];
    rc = static_cast<int>(cudaMemcpyToSymbol(g_step_trace, zeros, sizeof(zeros)));
  }
  return rc;
}
#define SPT(ev) do { if (blockIdx.x < 256) STK_TRACE_AT(g_step_trace, blockIdx.x * 32 + (ev)); } while (0)
#else
#define SPT(ev) ((void)0)
#endif


__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: wait until *p >= target, bounded by the library's wait limit.
__device__ bool wait_count(const unsigned* p, unsigned target) {
  if (ld_acquire_gpu(p) >= target) return true;
  const unsigned long long t0 = global_ns(), limit = c_wait_ns;
  while (ld_acquire_gpu(p) < target) {
    __nanosleep(64);
    if (global_ns() - t0 > limit) return false;
  }
  return true;
}

// One thread, after the writes it publishes are ordered before it (warp or
// CTA barrier): make them visible GPU-wide, then count.
__device__ __forceinline__ void publish(unsigned* p) {
  __threadfence();
  atomicAdd(p, 1u);
}

// Fold a block state (m, l, u) into a running LSE state (wm, wl, wu).
__device__ __forceinline__ void fold_state(float& wm, float& wl, float (&wu)[kStepDPH], float m, float l,
                                           const float (&u)[kStepDPH]) {
  if (!(m > neg_inf())) return;
  const float M = fmaxf(wm, m);
  const float a = expf(wm - M);
  const float b = expf(m - M);
  wl = wl * a + l * b;
#pragma unroll
  for (int j = 0; j < kStepDPH; ++j) wu[j] = wu[j] * a + u[j] * b;
  wm = M;
}

// Score intervals of one metadata item: up to 16 blocks of KV head mh for
// its G query heads, staged as lo rows [16][D] then hi rows [16][D]. Lane =
// block-in-half * 4 + quarter of D, and every lane takes one block of each
// half (bA and bA + 8), so the query chunks it loads serve two blocks and it
// keeps 2 G independent sums. Per block and head the sum, its radius and the
// rounding are those of bound_interval_kernel (select.cu): each lane sums its
// D / 4 dims in order with FP32 FMA, two shuffle levels finish the sum, and
// the interval is widened by 2 (D/4 + 2) u ||q||_1 max|lo, hi| + 2^-118 and
// rounded outward.
template <int GM>
__device__ __forceinline__ void score_item(const StepArgs& a, const float* slo, const float* shi, const float* qs,
                                           const float* qn1, int mh, int b0, int nb, int G, int lane) {
  constexpr int D = kStepD;
  constexpr float kErrFactor = 2.f * (D / 4 + 2) * 0x1p-24f;
  const int p = lane & 3;
  const int bA = lane >> 2, bB = bA + 8;
  const bool liveA = bA < nb, liveB = bB < nb;
  const float4* LA = reinterpret_cast<const float4*>(slo + (liveA ? bA : 0) * D);
  const float4* HA = reinterpret_cast<const float4*>(shi + (liveA ? bA : 0) * D);
  const float4* LB = reinterpret_cast<const float4*>(slo + (liveB ? bB : 0) * D);
  const float4* HB = reinterpret_cast<const float4*>(shi + (liveB ? bB : 0) * D);
  const float* qrow = qs + mh * G * D;
  float sA[GM], sB[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) { sA[g] = 0.f; sB[g] = 0.f; }
  float mA = 0.f, mB = 0.f;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < D / 16; ++i) {
    const int c = p + 4 * i;
    const float4 la = liveA ? LA[c] : z, ha = liveA ? HA[c] : z;
    const float4 lb = liveB ? LB[c] : z, hb = liveB ? HB[c] : z;
    mA = fmaxf(mA, fmaxf(fmaxf(fabsf(la.x), fabsf(ha.x)), fmaxf(fabsf(la.y), fabsf(ha.y))));
    mA = fmaxf(mA, fmaxf(fmaxf(fabsf(la.z), fabsf(ha.z)), fmaxf(fabsf(la.w), fabsf(ha.w))));
    mB = fmaxf(mB, fmaxf(fmaxf(fabsf(lb.x), fabsf(hb.x)), fmaxf(fabsf(lb.y), fabsf(hb.y))));
    mB = fmaxf(mB, fmaxf(fmaxf(fabsf(lb.z), fabsf(hb.z)), fmaxf(fabsf(lb.w), fabsf(hb.w))));
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float4 qq = *reinterpret_cast<const float4*>(qrow + g * D + 4 * c);
        sA[g] = fmaf(qq.x, qq.x >= 0.f ? ha.x : la.x, sA[g]);
        sB[g] = fmaf(qq.x, qq.x >= 0.f ? hb.x : lb.x, sB[g]);
        sA[g] = fmaf(qq.y, qq.y >= 0.f ? ha.y : la.y, sA[g]);
        sB[g] = fmaf(qq.y, qq.y >= 0.f ? hb.y : lb.y, sB[g]);
        sA[g] = fmaf(qq.z, qq.z >= 0.f ? ha.z : la.z, sA[g]);
        sB[g] = fmaf(qq.z, qq.z >= 0.f ? hb.z : lb.z, sB[g]);
        sA[g] = fmaf(qq.w, qq.w >= 0.f ? ha.w : la.w, sA[g]);
        sB[g] = fmaf(qq.w, qq.w >= 0.f ? hb.w : lb.w, sB[g]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    sA[g] += __shfl_xor_sync(kFull, sA[g], 1);
    sB[g] += __shfl_xor_sync(kFull, sB[g], 1);
    sA[g] += __shfl_xor_sync(kFull, sA[g], 2);
    sB[g] += __shfl_xor_sync(kFull, sB[g], 2);
  }
  mA = fmaxf(mA, __shfl_xor_sync(kFull, mA, 1));
  mB = fmaxf(mB, __shfl_xor_sync(kFull, mB, 1));
  mA = fmaxf(mA, __shfl_xor_sync(kFull, mA, 2));
  mB = fmaxf(mB, __shfl_xor_sync(kFull, mB, 2));
  const float inf = __int_as_float(0x7f800000);
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G && (g & 3) == p) {
      const float qn = qn1[mh * G + g];
      float2* out = a.bounds + static_cast<long long>(mh * G + g) * a.n + b0;
      if (liveA) {
        const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn, mA), kErrFactor), 0x1p-118f);
        float2 iv = make_float2(__fsub_rd(sA[g], e), __fadd_ru(sA[g], e));
        if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
        out[bA] = iv;
      }
      if (liveB) {
        const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn, mB), kErrFactor), 0x1p-118f);
        float2 iv = make_float2(__fsub_rd(sB[g], e), __fadd_ru(sB[g], e));
        if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
        out[bB] = iv;
      }
    }
  }
}

template <typename T, int E, int GM>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(StepArgs a) {
  constexpr int D = kStepD;
  constexpr int DPH = kStepDPH;
  constexpr int NS = kStepStages;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full_bar[NS], empty_bar[NS];
  __shared__ int item_ok[NS];
  __shared__ volatile int s_abort;
  __shared__ int s_sel[kStepMaxList], s_pid[kStepMaxList], s_miss[kStepMaxList], s_hit[kStepMaxList];
  __shared__ int s_nmiss, s_nhit;
  __shared__ unsigned s_pmask[kStepMaxBlocks / 32], s_amask[kStepMaxBlocks / 32];
  __shared__ float s_wm[kStepWarps], s_wl[kStepWarps];
  __shared__ __align__(16) float s_wu[kStepWarps][D];
  __shared__ uint64_t fold_bar;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hq = a.hq, hkv = a.hkv, n = a.n, K = a.topk;
  const int G = hq / hkv;
  const int grid = gridDim.x;
  const int W = grid - hq;  // work CTAs; CTA W + r is row r's CTA
  const bool row_cta = static_cast<int>(blockIdx.x) >= W;
  const int row = row_cta ? static_cast<int>(blockIdx.x) - W : -1;
  const bool serial = a.sp == 0;
  const int S = serial ? K : a.sp;
  const int ipH = (n + kMetaItemBlocks - 1) / kMetaItemBlocks;  // metadata items per KV head
  const int n_meta = hkv * ipH;
  // Every CTA c scores metadata items c, c + grid, ...; work CTA c then takes
  // jobs [j0, j1) of the hq * S (row, slot) block states.
  const int my_meta = static_cast<int>(blockIdx.x) < n_meta ? (n_meta - 1 - static_cast<int>(blockIdx.x)) / grid + 1 : 0;
  const long long J = static_cast<long long>(hq) * S;
  const int j0 = row_cta ? 0 : static_cast<int>(J * blockIdx.x / W);
  const int j1 = row_cta ? 0 : static_cast<int>(J * (blockIdx.x + 1) / W);
  const int my_jobs = j1 - j0;
  const int n_items = my_meta + my_jobs;
  unsigned* head_done = a.ctrl;
  unsigned* row_states = a.ctrl + hkv;
  unsigned* row_ready = a.ctrl + hkv + hq;
  unsigned* ctas_done = a.ctrl + hkv + 2 * hq;

  float* qs = reinterpret_cast<float*>(smem);  // [hq][D] FP32
  float* qn1 = qs + hq * D;                     // [hq] ||q||_1, rounded up
  unsigned char* pool = smem + ((static_cast<size_t>(hq) * D + hq) * 4 + 127) / 128 * 128;
  const T* Kp = static_cast<const T*>(a.k);
  const T* Vp = static_cast<const T*>(a.v);
  constexpr unsigned kBlockBytes = kStepB * D * sizeof(T);

  // ---------------------------------------------------------------- set-up
  if (tid == 0) SPT(0);
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(&fold_bar, 1);
    fence_barrier_init();
    s_abort = 0;
  }
  __syncthreads();

  // Issues item `it` into stage it % NS once the consumer of item it - NS has
  // released it. An item it cannot fill (a bad ID, or after an abort) is
  // completed without a copy and flagged, so that its consumer skips it.
  auto produce = [&](int it, int kind, int mh, long long first, long long id) {
    const int st = it % NS;
    if (it >= NS && !mbar_wait(&empty_bar[st], ((it / NS) - 1) & 1u, a.status)) s_abort = 1;
    unsigned char* stage = pool + static_cast<size_t>(st) * kStageBytes;
    if (kind == 0) {  // metadata: rows [first, first + nb) of KV head mh
      const int nb = min(kMetaItemBlocks, n - static_cast<int>(first));
      const unsigned bytes = static_cast<unsigned>(nb) * D * 4;
      const long long off = (static_cast<long long>(mh) * n + first) * D;
      item_ok[st] = 1;
      mbar_arrive_expect_tx(&full_bar[st], 2 * bytes);
      bulk_g2s(stage, a.lo + off, bytes, &full_bar[st]);
      bulk_g2s(stage + kStageBytes / 2, a.hi + off, bytes, &full_bar[st]);
    } else if (id >= 0 && id < n && !s_abort) {  // one block of KV head mh
      const long long off = (static_cast<long long>(mh) * n + id) * kStepB * D;
      item_ok[st] = 1;
      mbar_arrive_expect_tx(&full_bar[st], 2 * kBlockBytes);
      bulk_g2s(stage, Kp + off, kBlockBytes, &full_bar[st]);
      bulk_g2s(stage + kBlockBytes, Vp + off, kBlockBytes, &full_bar[st]);
    } else {
      if (id >= n) report(a.status, kStatusBadBlockId);
      item_ok[st] = 0;
      mbar_arrive(&full_bar[st]);
    }
  };
  auto meta_item = [&](int it, int& mh, int& b0) {
    const int m = static_cast<int>(blockIdx.x) + it * grid;
    mh = m / ipH;
    b0 = (m % ipH) * kMetaItemBlocks;
  };

  // The small loads are issued first and consumed after the bulk copies are
  // queued: q (16 bytes per thread), the predicted IDs of this CTA's first
  // jobs (producer lanes) or of its row (row CTA).
  const int qvals = hq * D;
  const int qper = a.q_dtype == kF32 ? 4 : 8;  // values per 16-byte load
  float qv[2][8];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int i = (c * kStepThreads + tid) * qper;
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[c][e] = 0.f;
    if (i < qvals) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.q) +
                                                           static_cast<long long>(i) * (a.q_dtype == kF32 ? 4 : 2)));
      if (a.q_dtype == kF32) {
        qv[c][0] = __uint_as_float(x.x); qv[c][1] = __uint_as_float(x.y);
        qv[c][2] = __uint_as_float(x.z); qv[c][3] = __uint_as_float(x.w);
      } else {
        const unsigned w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (a.q_dtype == kBF16) {
            qv[c][2 * e] = __uint_as_float(w4[e] << 16);
            qv[c][2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
            qv[c][2 * e] = f.x;
            qv[c][2 * e + 1] = f.y;
          }
        }
      }
    }
  }
  long long lid = -1;  // producer lane: predicted ID of job j0 + jb + lane
  int jb = 0;
  if (warp == kStepProducer && !serial && lane < my_jobs) lid = load_id(a.pred, a.pred64, j0 + lane);
  if (row_cta && !serial)
    for (int i = tid; i < a.sp; i += kStepThreads)
      s_pid[i] = static_cast<int>(load_id(a.pred, a.pred64, static_cast<long long>(row) * a.sp + i));
  // Metadata items into the free stages at once, one producer lane each.
  const int n_first = min(my_meta, NS);
  if (warp == kStepProducer && lane < n_first) {
    int mh, b0;
    meta_item(lane, mh, b0);
    produce(lane, 0, mh, b0, 0);
  }
  if (tid == 0) SPT(2);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int i = (c * kStepThreads + tid) * qper;
    if (i < qvals)
      for (int e = 0; e < qper; ++e) qs[i + e] = qv[c][e];
  }
  __syncthreads();
  for (int t = warp; t < hq; t += kStepWarps) {
    float sum = 0.f;
    for (int dd = lane; dd < D; dd += 32) sum = __fadd_ru(sum, fabsf(qs[t * D + dd]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_ru(sum, __shfl_xor_sync(kFull, sum, o));
    if (lane == 0) qn1[t] = sum;
  }
  __syncthreads();
  if (tid == 0) SPT(1);

  // ---------------------------------------------------------------- ring: metadata, then block states
  if (warp == kStepProducer) {
    int ready_row = -1;  // serial: rows whose selection this warp has seen published
    long long sid = -1;  // serial: selected ID of job sb + lane
    int sb = -1;
    for (int it = n_first; it < n_items; ++it) {
      if (it < my_meta) {
        if (lane == 0) {
          int mh, b0;
          meta_item(it, mh, b0);
          produce(it, 0, mh, b0, 0);
        }
      } else {
        const int jl = it - my_meta;  // this CTA's job index
        const int job = j0 + jl;
        const int r = job / S;
        long long id = -1;
        if (!serial) {
          if (jl - jb == 32) {
            jb += 32;
            lid = jb + lane < my_jobs ? load_id(a.pred, a.pred64, j0 + jb + lane) : -1;
          }
          id = __shfl_sync(kFull, lid, jl - jb);
        } else {
          if (r > ready_row) {
            if (lane == 0 && !s_abort && !wait_count(&row_ready[r], 1)) {
              report(a.status, kStatusWaitTimeout);
              s_abort = 1;
            }
            __syncwarp();
            ready_row = r;
            sb = -1;
          }
          if (sb < 0 || job - sb >= 32) {
            // The selected IDs of the next 32 jobs of row r (job = r * K + slot).
            sb = job;
            const int jj = job + lane;
            sid = (!s_abort && jj < j1 && jj / S == r) ? __ldcg(a.selected + jj) : -1;
          }
          id = __shfl_sync(kFull, sid, job - sb);
        }
        if (lane == 0) produce(it, 1, r / G, 0, id);
      }
      if (lane == 0 && it == my_meta) SPT(3);
      if (lane == 0 && it == NS) SPT(30);
      if (lane == 0 && it == 2 * NS) SPT(31);
      __syncwarp();
    }
    if (lane == 0) SPT(4);
  } else if (warp < NS) {
    // Consumers: item it belongs to warp it % NS (one consumer per stage).
    // Block-state completions are published per row in batches (one fence
    // per row change and one at the end), metadata items one by one: the
    // selections wait on them.
    int pend_row = -1, pend = 0;
    if (lane == 0 && warp == 0) SPT(12);
    for (int it = warp; it < n_items; it += NS) {
      const int st = it % NS;
      const bool landed = mbar_wait(&full_bar[st], (it / NS) & 1u, a.status);
      if (lane == 0 && it == 0) SPT(13);
      if (lane == 0 && warp == 0 && it / NS < 3) SPT(24 + it / NS);
      if (!landed) s_abort = 1;
      const bool ok = landed && item_ok[st] != 0;
      const unsigned char* stage = pool + static_cast<size_t>(st) * kStageBytes;
      if (it < my_meta) {
        int mh, b0;
        meta_item(it, mh, b0);
        if (ok)
          score_item<GM>(a, reinterpret_cast<const float*>(stage),
                         reinterpret_cast<const float*>(stage + kStageBytes / 2), qs, qn1, mh, b0,
                         min(kMetaItemBlocks, n - b0), G, lane);
        __syncwarp();
        if (lane == 0 && warp == 0 && it == 0) SPT(22);
        if (lane == 0) {
          mbar_arrive(&empty_bar[st]);
          publish(&head_done[mh]);
        }
      } else {
        // One block's softmax state for (row r, slot).
        const int job = j0 + (it - my_meta);
        const int r = job / S, slot = job - r * S;
        float m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
        for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
        if (ok) {
          float qf[DPH];
#pragma unroll
          for (int j = 0; j < DPH; ++j) qf[j] = qs[r * D + (lane & 15) * DPH + j];
          const T* ks = reinterpret_cast<const T*>(stage);
          warp_block_state<T, DPH, kModeFull, true>(ks, ks + kStepB * D, kStepB, qf, a.scale, 0.f, m, l, u, ua,
                                                    lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);
        const long long o = static_cast<long long>(r) * S + slot;
        if (lane == 0) {
          a.sm[o] = m;
          a.sl[o] = l;
        }
        if (lane < 16) store_vec<DPH>(a.su + o * D + lane * DPH, u);
        __syncwarp();
        if (lane == 0 && warp == 0 && it == NS) SPT(23);
        if (lane == 0) {
          if (r != pend_row && pend > 0) {
            __threadfence();
            atomicAdd(&row_states[pend_row], static_cast<unsigned>(pend));
            pend = 0;
          }
          pend_row = r;
          ++pend;
        }
      }
      if (lane == 0 && warp == 0 && it / NS < 3) SPT(27 + it / NS);
    }
    if (lane == 0 && pend > 0) {
      __threadfence();
      atomicAdd(&row_states[pend_row], static_cast<unsigned>(pend));
    }
    if (lane == 0 && warp == 0) SPT(14);
  }

  // ---------------------------------------------------------------- row CTAs
  __syncthreads();
  if (row_cta) {
    const float* qrow = qs + row * D;
    const int mh = row / G;
    if (tid == 0) SPT(5);
    if (tid == 0 && !s_abort && !wait_count(&head_done[mh], static_cast<unsigned>(ipH))) {
      report(a.status, kStatusWaitTimeout);
      s_abort = 1;
    }
    __syncthreads();
    if (tid == 0) SPT(6);
    if (!s_abort) {
      SelectArgs sa{};
      sa.R = 1; sa.hsel = hq; sa.topk = K; sa.n = n; sa.block_offsets = nullptr; sa.total_blocks = n;
      sa.id_base = 0; sa.ids_out = a.selected; sa.keys_out = nullptr; sa.status = a.status;
      sa.bounds = a.bounds; sa.q = a.q; sa.q_dtype = a.q_dtype; sa.lo = a.lo; sa.hi = a.hi;
      sa.hq = hq; sa.hmeta = hkv; sa.d = D; sa.group_select = 0;
      bounded_select_core<E, kStepThreads>(sa, row, qrow, true);
#ifdef STK_TOPK_TWICE
      __syncthreads();
      if (tid == 0) SPT(21);
      bounded_select_core<E, kStepThreads>(sa, row, qrow, true);
#endif
    }
    __syncthreads();
    if (tid == 0) SPT(7);
    for (int i = tid; i < K; i += kStepThreads) s_sel[i] = a.selected[static_cast<long long>(row) * K + i];
    if (serial && tid == 0 && !s_abort) publish(&row_ready[row]);
    __syncthreads();

    float wm = neg_inf(), wl = 0.f, wu[DPH];
#pragma unroll
    for (int j = 0; j < DPH; ++j) wu[j] = 0.f;
    int n_fold = K;  // retained states to fold
    const int* fold_slot = nullptr;
    if (!serial) {
      // Saved repair: misses (A not in P) computed here, hits (P slots in A)
      // taken from the block states the work CTAs wrote.
      for (int i = tid; i < (n + 31) / 32; i += kStepThreads) { s_pmask[i] = 0u; s_amask[i] = 0u; }
      __syncthreads();
      for (int i = tid; i < a.sp; i += kStepThreads) {
        const int id = s_pid[i];
        if (id >= 0 && id < n) atomicOr(&s_pmask[id >> 5], 1u << (id & 31));
      }
      for (int i = tid; i < K; i += kStepThreads) {
        const int id = s_sel[i];
        if (id >= 0 && id < n) atomicOr(&s_amask[id >> 5], 1u << (id & 31));
      }
      __syncthreads();
      if (warp == 0) {
        int nm = 0;
        for (int b = 0; b < K; b += 32) {
          const int id = b + lane < K ? s_sel[b + lane] : -1;
          const bool miss = id >= 0 && !((s_pmask[id >> 5] >> (id & 31)) & 1u);
          const unsigned bal = __ballot_sync(kFull, miss);
          if (miss) s_miss[nm + __popc(bal & ((1u << lane) - 1u))] = id;
          nm += __popc(bal);
        }
        int nh = 0;
        for (int b = 0; b < a.sp; b += 32) {
          const int id = b + lane < a.sp ? s_pid[b + lane] : -1;
          const bool hit = id >= 0 && id < n && ((s_amask[id >> 5] >> (id & 31)) & 1u);
          const unsigned bal = __ballot_sync(kFull, hit);
          if (hit) s_hit[nh + __popc(bal & ((1u << lane) - 1u))] = b + lane;
          nh += __popc(bal);
        }
        if (lane == 0) { s_nmiss = nm; s_nhit = nh; }
      }
      __syncthreads();
      const int nmiss = s_abort ? 0 : s_nmiss;
      // Misses through the ring, continuing after this CTA's metadata items.
      if (warp == kStepProducer) {
        for (int i = 0; i < nmiss; ++i) {
          if (lane == 0) produce(n_items + i, 1, mh, 0, s_miss[i]);
          __syncwarp();
        }
      } else if (warp < NS) {
        // Item n_items + i belongs to warp (n_items + i) % NS, like every item of the ring.
        for (int i = (warp - n_items % NS + NS) % NS; i < nmiss; i += NS) {
          const int it = n_items + i;
          const int st = it % NS;
          const bool landed = mbar_wait(&full_bar[st], (it / NS) & 1u, a.status);
          if (lane == 0 && i < NS) SPT(15);
          if (!landed) s_abort = 1;
          if (landed && item_ok[st]) {
            float qf[DPH], m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
            for (int j = 0; j < DPH; ++j) { qf[j] = qrow[(lane & 15) * DPH + j]; u[j] = 0.f; ua[j] = 0.f; }
            const T* ks = reinterpret_cast<const T*>(pool + static_cast<size_t>(st) * kStageBytes);
            warp_block_state<T, DPH, kModeFull, true>(ks, ks + kStepB * D, kStepB, qf, a.scale, 0.f, m, l, u, ua,
                                                      lane);
            fold_state(wm, wl, wu, m, l, u);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_bar[st]);
        }
      }
      n_fold = s_nhit;
      fold_slot = s_hit;
    }
    if (tid == 0) SPT(8);
    // The row's S block states are complete: bring their numerators into
    // shared memory with one bulk copy (S x D FP32, once the ring's stages
    // are drained), and their (m, l) with plain loads through L2.
    __syncthreads();
    float* st_u = reinterpret_cast<float*>(pool);
    float* st_m = reinterpret_cast<float*>(pool + static_cast<size_t>(S) * D * 4);
    float* st_l = st_m + S;
    if (tid == 0) {
      if (!s_abort && !wait_count(&row_states[row], static_cast<unsigned>(S))) {
        report(a.status, kStatusWaitTimeout);
        s_abort = 1;
      }
      SPT(9);
      if (!s_abort) {
        // The numerators were written by other CTAs (generic proxy) and are
        // read here by the bulk-copy (async) proxy.
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const unsigned bytes = static_cast<unsigned>(S) * D * 4;
        mbar_arrive_expect_tx(&fold_bar, bytes);
        bulk_g2s(st_u, a.su + static_cast<long long>(row) * S * D, bytes, &fold_bar);
      }
    }
    __syncthreads();
    if (!s_abort) {
      for (int i = tid; i < S; i += kStepThreads) {
        st_m[i] = __ldcg(a.sm + static_cast<long long>(row) * S + i);
        st_l[i] = __ldcg(a.sl + static_cast<long long>(row) * S + i);
      }
    }
    const bool have_u = !s_abort && mbar_wait(&fold_bar, 0, a.status);
    if (!have_u) s_abort = 1;
    __syncthreads();
    if (!s_abort) {
      for (int i = warp; i < n_fold; i += kStepWarps) {
        const int slot = fold_slot ? fold_slot[i] : i;
        float u[DPH];
#pragma unroll
        for (int j = 0; j < DPH; ++j) u[j] = st_u[slot * D + (lane & 15) * DPH + j];
        fold_state(wm, wl, wu, st_m[slot], st_l[slot], u);
      }
    }
    if (lane == 0) { s_wm[warp] = wm; s_wl[warp] = wl; }
    if (lane < 16) store_vec<DPH>(&s_wu[warp][lane * DPH], wu);
    __syncthreads();
    if (tid < D && !s_abort) {
      float M = neg_inf();
      for (int w = 0; w < kStepWarps; ++w) M = fmaxf(M, s_wm[w]);
      float Z = 0.f, U = 0.f;
      for (int w = 0; w < kStepWarps; ++w) {
        if (s_wm[w] > neg_inf()) {
          const float x = expf(s_wm[w] - M);
          Z += x * s_wl[w];
          U += x * s_wu[w][tid];
        }
      }
      a.out[static_cast<long long>(row) * D + tid] = U / fmaxf(Z, 1e-30f);
    }
    if (tid == 0) SPT(10);
  }

  // ---------------------------------------------------------------- exit
  // Every wait of this CTA is over; the last CTA to get here zeroes the
  // control block for the next call.
  __syncthreads();
  if (tid == 0) SPT(11);
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(ctas_done, 1u) == static_cast<unsigned>(grid) - 1) {
      for (int i = 0; i < hkv + 2 * hq; ++i) atomicExch(a.ctrl + i, 0u);
      atomicExch(ctas_done, 0u);
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ host side

size_t decode_step_smem(int hq) {
  return ((static_cast<size_t>(hq) * kStepD + hq) * 4 + 127) / 128 * 128 +
         static_cast<size_t>(kStepStages) * kStageBytes;
}

const char* decode_step_unsupported(int hq, int hkv, int n, int b, int d, int kv_dtype, int topk, int sp,
                                    int num_sms) {
  if (d != kStepD || b != kStepB) return "the fused step takes head dim 128 and 32-token blocks";
  if (kv_dtype != kBF16 && kv_dtype != kF16) return "the fused step takes 16-bit K/V";
  if (hq % hkv != 0 || hq / hkv > 16) return "the fused step takes at most 16 query heads per KV head";
  if (static_cast<size_t>(hq) * kStepD > 4096) return "the fused step stages at most 4096 query values";
  if (n > kStepMaxBlocks || n < topk) return "the fused step takes topk <= blocks <= 4096";
  if (topk > kStepMaxList || sp > kStepMaxList) return "the fused step takes lists of at most 256 blocks";
  const int slots = sp > 0 ? sp : topk;
  if (static_cast<size_t>(slots) * (kStepD + 2) * 4 > static_cast<size_t>(kStepStages) * kStageBytes)
    return "the fused step folds at most 336 block states per row";
  if (2 * hq >= num_sms) return "the fused step needs more than two SMs per query head";
  return nullptr;
}

template <typename T, int E, int GM>
static int launch_step_t(const StepArgs& a, int num_sms, cudaStream_t stream) {
  auto kern = decode_step_kernel<T, E, GM>;
  const size_t smem = decode_step_smem(a.hq);
  cudaFuncAttributes fa;
  int dev = 0, optin = 0;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e == cudaSuccess) e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (fa.sharedSizeBytes + smem > static_cast<size_t>(optin)) return -1;  // outside the plan on this device
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  prefer_shared(kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, a));
}

template <typename T>
static int launch_step_d(const StepArgs& a, int num_sms, cudaStream_t stream) {
  const int G = a.hq / a.hkv;
  if (a.n <= 2048) return G <= 4 ? launch_step_t<T, 4, 4>(a, num_sms, stream) : launch_step_t<T, 4, 16>(a, num_sms, stream);
  return G <= 4 ? launch_step_t<T, 8, 4>(a, num_sms, stream) : launch_step_t<T, 8, 16>(a, num_sms, stream);
}

int launch_decode_step(const StepArgs& a, int kv_dtype, int num_sms, cudaStream_t stream) {
  return kv_dtype == kBF16 ? launch_step_d<__nv_bfloat16>(a, num_sms, stream)
                           : launch_step_d<__half>(a, num_sms, stream);
}

int set_wait_limit_step(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
