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
// A row CTA's phase: it polls the row's score slots (coalesced, exchanged
// through the ring's first stages) and selects; in the speculative step
// the misses then go to stages 0..7, the row's predicted states arrive in
// stages 8..10 with bulk copies once every work CTA has written them, and
// the helpers with consumers 8..10 fold the hits from there while
// consumers 0..7 reduce the misses; the warps' states merge in warp order.
//
// Cross-CTA progress goes through counters in the workspace's control
// block, which must be zero before the first call on a workspace; the last
// CTA to finish a call zeroes it again:
//   ctrl[mh]                metadata items done for KV head mh (counted; the
//                           row CTAs poll their score slots instead of
//                           waiting for it),
//   ctrl[hkv + r]           block states done for row r,
//   ctrl[hkv + hq + r]      row r's selection published (serial step),
//   ctrl[hkv + 2 hq]        CTAs finished.
// A writer publishes after its global writes with a fence and an atomic add;
// a reader waits with acquire loads and reads the data through L2.

#include <type_traits>

#include "block_state.cuh"
#include "common.cuh"

#ifdef STK_TRACE
namespace stk {
// Timeline of the fused step (profiling builds only): [cta][128] global
// timer stamps. Probes record into shared memory (a global store could wait
// behind this SM's bulk copies and delay the release that follows it); each
// CTA copies its record out at exit.
static __device__ unsigned long long g_step_trace[256 * 128];
static __shared__ unsigned long long s_trc[128];
static __shared__ unsigned s_trc_meta;  // scored metadata items of this CTA
// [launch % 64][first CTA start, last CTA exit] over consecutive launches.
static __device__ unsigned long long g_step_span[2 * 64];
static __device__ unsigned g_step_launch;
}  // namespace stk
// Phases of the selection inside the fused step: events 16 + ev.
#define STK_TOPK_PROBE(ev) do { if (threadIdx.x == 0) stk::s_trc[16 + (ev)] = stk::global_ns(); } while (0)
#endif
#include "topk.cuh"

namespace stk {

constexpr int kStepThreads = 512;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepStages = 11;               // ring stages = consumer warps 0..10
constexpr int kStepProducer = kStepStages;     // warp 11 issues the bulk copies
constexpr int kStepHelper0 = kStepProducer + 1;  // warps 12..15 (selection, repair folds)
constexpr int kStepD = 128;
constexpr int kStepB = 32;
constexpr int kStepDPH = kStepD / 16;
constexpr int kStageBytes = 2 * kStepB * kStepD * 2;            // one 16-bit K+V block: 16 KiB
constexpr int kMetaItemBlocks = kStageBytes / (2 * kStepD * 4);  // 16 blocks of FP32 lo + hi
constexpr int kStepMaxList = 256;                                // topk and predicted-list limit
constexpr int kStepMaxBlocks = 4096;                             // blocks per request limit
constexpr int kItemEnd = -1;                                     // stage descriptor: no more items
constexpr int kItemLocal = 1 << 30;                              // descriptor of row-local block i: kItemLocal + i
// Serial step: the share of each row's selected blocks that its own row CTA
// reduces (times 4 / (hq * topk / grid)); the rest go to the work CTAs.
#ifndef STK_STEP_LOCAL_SHARE4
#define STK_STEP_LOCAL_SHARE4 5
#endif

#ifdef STK_TRACE
extern "C" __attribute__((visibility("default"))) int stk_trace_step_read(void* host, size_t bytes, int clear) {
  int rc = static_cast<int>(cudaMemcpyFromSymbol(host, g_step_trace, bytes));
  if (!rc && clear) {
    static unsigned long long zeros[256 * 128];
    rc = static_cast<int>(cudaMemcpyToSymbol(g_step_trace, zeros, sizeof(zeros)));
  }
  return rc;
}
extern "C" __attribute__((visibility("default"))) int stk_trace_step_spans(void* host, int reset) {
  int rc = static_cast<int>(cudaMemcpyFromSymbol(host, g_step_span, sizeof(g_step_span)));
  if (!rc && reset) {
    static unsigned long long init[2 * 64];
    for (int i = 0; i < 2 * 64; ++i) init[i] = (i & 1) ? 0ull : ~0ull;
    unsigned zero = 0;
    rc = static_cast<int>(cudaMemcpyToSymbol(g_step_span, init, sizeof(init)));
    if (!rc) rc = static_cast<int>(cudaMemcpyToSymbol(g_step_launch, &zero, sizeof(zero)));
  }
  return rc;
}
#define SPT(ev) (s_trc[(ev)] = global_ns())
#define SPT_RAW(slot, val) (s_trc[(slot)] = (val))
#define SPAN_START() do { if (threadIdx.x == 0) atomicMin(&g_step_span[2 * (g_step_launch & 63)], global_ns()); } while (0)
#define SPAN_END() do { g_step_span[2 * (g_step_launch & 63) + 1] = global_ns(); ++g_step_launch; } while (0)
#else
#define SPT(ev) ((void)0)
#define SPT_RAW(slot, val) ((void)0)
#define SPAN_START() ((void)0)
#define SPAN_END() ((void)0)
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
__device__ __forceinline__ void publish(unsigned* p, unsigned count = 1u) {
  __threadfence();
  atomicAdd(p, count);
}

// Non-blocking probe of an mbarrier phase (acquire, CTA scope).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Named barrier over the warps other than the producer (480 threads).
// Warps 0..11 (consumers and producer): the miss list of the speculative
// row phase is published to them alone, so that the helper warps can start
// folding the buffered hits as soon as the selection ends.
__device__ __forceinline__ void sync_list_warps() {
  asm volatile("bar.sync 3, %0;" ::"n"((kStepStages + 1) * 32) : "memory");
}
__device__ __forceinline__ void sync_non_producer() {
  asm volatile("bar.sync 1, %0;" ::"n"(kStepThreads - 32) : "memory");
}
// Barrier 2: the producer arrives once its barriers are initialised, the
// other warps wait there before their first barrier access.
__device__ __forceinline__ void barriers_ready_arrive() {
  asm volatile("bar.arrive 2, %0;" ::"n"(kStepThreads) : "memory");
}
__device__ __forceinline__ void barriers_ready_wait() {
  asm volatile("bar.sync 2, %0;" ::"n"(kStepThreads) : "memory");
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
// its G query heads, staged as lo rows [16][D] then hi rows [16][D].
//
// Lane l owns dims [4l, 4l + 4): every warp-wide 128-bit load reads one whole
// 512-byte row (conflict-free), and q of four heads stays in registers split
// by sign, q+ = max(q, 0) and q- = min(q, 0), so that the sign-selected bound
// term q (q >= 0 ? hi : lo) is q+ hi + q- lo: two FMAs, one of them adding an
// exact zero. Per group of 4 blocks and 4 heads each lane forms 16 partial
// sums (its 4 dims in order); a transposed butterfly (xor 8, 4, 2, 1) and one
// xor-16 add leave the total of (block j, head g) in lanes 4 j + g and
// 16 + 4 j + g. Every nonzero term passes through at most 4 + 5 roundings,
// fewer than the D / 4 + 2 that the interval radius
// 2 (D/4 + 2) u ||q||_1 max|lo, hi| + 2^-118 of bound_interval_kernel
// (select.cu) covers, so the interval, rounded outward, contains the block's
// FP64 score (an infinite bound makes a NaN sum, and the interval then spans
// everything). The interval is written as one 8-byte store into a slot that
// reads zero until then.
template <int GM>
__device__ __forceinline__ void score_item(const StepArgs& a, const float* slo, const float* shi, const float* qs,
                                           const float* qn1, int mh, int b0, int nb, int G, int lane) {
  constexpr int D = kStepD;
  constexpr float kErrFactor = 2.f * (D / 4 + 2) * 0x1p-24f;
  const float inf = __int_as_float(0x7f800000);
#pragma unroll 1
  for (int g0 = 0; g0 < G; g0 += 4) {
    float4 qp[4], qn[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float4 q = (g0 + g < G) ? *reinterpret_cast<const float4*>(qs + (mh * G + g0 + g) * D + 4 * lane)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      qp[g] = make_float4(q.x >= 0.f ? q.x : 0.f, q.y >= 0.f ? q.y : 0.f, q.z >= 0.f ? q.z : 0.f,
                          q.w >= 0.f ? q.w : 0.f);
      qn[g] = make_float4(q.x >= 0.f ? 0.f : q.x, q.y >= 0.f ? 0.f : q.y, q.z >= 0.f ? 0.f : q.z,
                          q.w >= 0.f ? 0.f : q.w);
    }
#pragma unroll 1
    for (int bq = 0; bq < kMetaItemBlocks && bq < nb; bq += 4) {
      float part[16];
      float mx[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int b = bq + j;
        float4 l4 = make_float4(0.f, 0.f, 0.f, 0.f), h4 = l4;
        if (b < nb) {
          l4 = *reinterpret_cast<const float4*>(slo + b * D + 4 * lane);
          h4 = *reinterpret_cast<const float4*>(shi + b * D + 4 * lane);
        }
        mx[j] = fmaxf(fmaxf(fmaxf(fabsf(l4.x), fabsf(h4.x)), fmaxf(fabsf(l4.y), fabsf(h4.y))),
                      fmaxf(fmaxf(fabsf(l4.z), fabsf(h4.z)), fmaxf(fabsf(l4.w), fabsf(h4.w))));
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float acc = qp[g].x * h4.x;
          acc = fmaf(qn[g].x, l4.x, acc);
          acc = fmaf(qp[g].y, h4.y, acc);
          acc = fmaf(qn[g].y, l4.y, acc);
          acc = fmaf(qp[g].z, h4.z, acc);
          acc = fmaf(qn[g].z, l4.z, acc);
          acc = fmaf(qp[g].w, h4.w, acc);
          acc = fmaf(qn[g].w, l4.w, acc);
          part[4 * j + g] = acc;
        }
      }
      // Sums: transposed over lane bits 3..0, then the two lane halves.
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
          const float send = upper ? part[i] : part[i + off];
          const float keep = upper ? part[i + off] : part[i];
          part[i] = keep + __shfl_xor_sync(kFull, send, off);
        }
      }
      const float sum = part[0] + __shfl_xor_sync(kFull, part[0], 16);
      // Block maxima: transposed over lane bits 3, 2, then the rest.
#pragma unroll
      for (int off = 8, cnt = 2; off >= 4; off >>= 1, cnt >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < cnt; ++i) {
          const float send = upper ? mx[i] : mx[i + cnt];
          const float keep = upper ? mx[i + cnt] : mx[i];
          mx[i] = fmaxf(keep, __shfl_xor_sync(kFull, send, off));
        }
      }
      float bm = mx[0];
      bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
      bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 2));
      bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 1));
      const int j = (lane >> 2) & 3, g = lane & 3, b = bq + j, head = g0 + g;
      if (lane < 16 && b < nb && head < G) {
        const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn1[mh * G + head], bm), kErrFactor), 0x1p-118f);
        float lo = __fsub_rd(sum, e), up = __fadd_ru(sum, e);
        if (!(lo <= up)) { lo = -inf; up = inf; }
        *reinterpret_cast<unsigned long long*>(a.bounds + static_cast<long long>(mh * G + head) * a.n + b0 + b) =
            static_cast<unsigned long long>(__float_as_uint(lo)) |
            (static_cast<unsigned long long>(__float_as_uint(up)) << 32);
      }
    }
  }
}

// Relaxed GPU-scope add (no ordering: readers of what it counts check the
// data itself).
__device__ __forceinline__ void red_relaxed_gpu(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Shared-memory counter add with release semantics at CTA scope: the warp's
// global writes before it (ordered by __syncwarp) are visible to a thread of
// the CTA that reads the counter with ld_acquire_cta.
__device__ __forceinline__ void red_release_cta(unsigned* p, unsigned v) {
  asm volatile("red.release.cta.shared::cta.add.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

constexpr int kStepPublisher = kStepHelper0;  // warp 12 forwards the CTA's completions GPU-wide
constexpr int kStepMaxHeads = 32;             // hq (and so hkv) limit: hq * D <= 4096

template <typename T, int E, int GM>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(StepArgs a) {
  constexpr int D = kStepD;
  constexpr int DPH = kStepDPH;
  constexpr int NS = kStepStages;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full_bar[NS], empty_bar[NS], q_bar, hit_bar;
  __shared__ int s_desc[NS], item_ok[NS];
  __shared__ volatile int s_abort;
  __shared__ bool s_last;
  __shared__ int s_sel[kStepMaxList], s_pid[kStepMaxList], s_loc[kStepMaxList], s_glb[kStepMaxList];
  __shared__ int s_nloc, s_nglb;
  __shared__ unsigned s_pmask[kStepMaxBlocks / 32], s_amask[kStepMaxBlocks / 32];
  __shared__ unsigned s_row_cnt[kStepMaxHeads];
  __shared__ float s_wm[kStepWarps], s_wl[kStepWarps];
  __shared__ __align__(16) float s_wu[kStepWarps][D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hq = a.hq, hkv = a.hkv, n = a.n, K = a.topk;
  const int G = hq / hkv;
  const int grid = gridDim.x;
  const int W = grid - hq;  // work CTAs; CTA W + r is row r's CTA
  const bool row_cta = static_cast<int>(blockIdx.x) >= W;
  const int row = row_cta ? static_cast<int>(blockIdx.x) - W : -1;
  const bool serial = a.sp == 0;
  const int S = serial ? K : a.sp;
  // Serial step: row r's CTA reduces the first xl of its selected blocks
  // itself; the other K - xl go to the work CTAs through the states buffer.
  const int xl = serial ? min(K, (hq * K * STK_STEP_LOCAL_SHARE4 + 4 * grid - 1) / (4 * grid)) : 0;
  const int SJ = S - xl;  // per-row block states computed by work CTAs
  const int ipH = (n + kMetaItemBlocks - 1) / kMetaItemBlocks;  // metadata items per KV head
  const int n_meta = hkv * ipH;
  // Every CTA c scores metadata items c, c + grid, ...; work CTA c then takes
  // jobs [j0, j1) of the hq * SJ (row, slot) block states.
  const int my_meta = static_cast<int>(blockIdx.x) < n_meta ? (n_meta - 1 - static_cast<int>(blockIdx.x)) / grid + 1 : 0;
  const long long J = static_cast<long long>(hq) * SJ;
  const int j0 = row_cta ? 0 : static_cast<int>(J * blockIdx.x / W);
  const int j1 = row_cta ? 0 : static_cast<int>(J * (blockIdx.x + 1) / W);
  const int my_jobs = j1 - j0;
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

  auto meta_item = [&](int it, int& mh, int& b0) {
    const int m = static_cast<int>(blockIdx.x) + it * grid;
    mh = m / ipH;
    b0 = (m % ipH) * kMetaItemBlocks;
  };
  // Block ID of this CTA's job jl (slot xl + ... of its row): the predicted
  // list (speculative step) or the published selection (serial step).
  auto job_id = [&](int jl) -> long long {
    if (jl < 0 || jl >= my_jobs) return -1;
    const int jj = j0 + jl, r = jj / SJ;
    const long long o = static_cast<long long>(r) * (serial ? K : S) + xl + (jj - r * SJ);
    if (!serial) return load_id(a.pred, a.pred64, o);
    // Serial step: the row CTA publishes ID + 1 into the zeroed tags.
    int t = ld_relaxed_gpu_s32(a.sel_tag + o);
    if (t == 0) {
      const unsigned long long t0 = global_ns();
      while ((t = ld_relaxed_gpu_s32(a.sel_tag + o)) == 0) {
        __nanosleep(100);
        if (global_ns() - t0 > c_wait_ns) {
          report(a.status, kStatusWaitTimeout);
          s_abort = 1;
          return -1;
        }
      }
    }
    return static_cast<long long>(t) - 1;
  };

  // ---------------------------------------------------------------- producer (warp 11)
  // Lane c < NS of the producer warp serves stage c. Each pass, every lane
  // whose stage has been released takes the next unissued item, so one pass
  // issues into all free stages at once and a slow item holds only its own
  // stage. An item that cannot be filled (bad ID, abort) is completed
  // without a copy and flagged, so that its consumer skips it.
  unsigned my_uses = 0;  // producer lane c < NS: items issued into stage c
  int npass = 0;         // profiling builds: passes that issued
  auto lane_free = [&]() {
    return lane < NS && (my_uses == 0 || mbar_test_wait(&empty_bar[lane], (my_uses - 1u) & 1u));
  };
  // kind 0 = metadata rows [first, first + 16) of KV head mh, 1 = K and V of
  // block id of KV head mh, 2 = end (no copy).
  auto fill_lane = [&](int code, int kind, int mh, long long first, long long id) {
    const int st = lane;
    unsigned char* stage = pool + static_cast<size_t>(st) * kStageBytes;
    s_desc[st] = code;
    if (kind == 0) {
      const int nb = min(kMetaItemBlocks, n - static_cast<int>(first));
      const unsigned bytes = static_cast<unsigned>(nb) * D * 4;
      const long long off = (static_cast<long long>(mh) * n + first) * D;
      item_ok[st] = 1;
      mbar_arrive_expect_tx(&full_bar[st], 2 * bytes);
      bulk_g2s(stage, a.lo + off, bytes, &full_bar[st]);
      bulk_g2s(stage + kStageBytes / 2, a.hi + off, bytes, &full_bar[st]);
    } else if (kind == 1 && id >= 0 && id < n && !s_abort) {
      const long long off = (static_cast<long long>(mh) * n + id) * kStepB * D;
      item_ok[st] = 1;
      mbar_arrive_expect_tx(&full_bar[st], 2 * kBlockBytes);
      bulk_g2s(stage, Kp + off, kBlockBytes, &full_bar[st]);
      bulk_g2s(stage + kBlockBytes, Vp + off, kBlockBytes, &full_bar[st]);
    } else {
      if (kind == 1 && id >= n) report(a.status, kStatusBadBlockId);
      item_ok[st] = 0;
      mbar_arrive(&full_bar[st]);
    }
    ++my_uses;
  };
  // Issue items [0, count): prepare(next) runs on every lane before a pass;
  // item_of(i, ...) runs on every lane (i < 0: none) and describes item i.
  auto produce = [&](int count, auto&& prepare, auto&& item_of) {
    int next = 0;
    unsigned long long t0 = 0;
    bool waiting = false;
    while (next < count && !s_abort) {
      const bool fr = lane_free();
      const unsigned fm = __ballot_sync(kFull, fr);
      if (fm == 0) {
        if (!waiting) {
          t0 = global_ns();
          waiting = true;
        } else if (global_ns() - t0 > c_wait_ns) {
          if (lane == 0) report(a.status, kStatusWaitTimeout);
          s_abort = 1;
        }
        continue;
      }
      waiting = false;
      prepare(next);
      const int rank = __popc(fm & ((1u << lane) - 1u));
      const int take = min(__popc(fm), count - next);
      const bool mine = fr && rank < take;
      int code = kItemEnd, kind = 2, mh = 0;
      long long first = 0, id = -1;
      item_of(mine ? next + rank : -1, code, kind, mh, first, id);
      if (mine) fill_lane(code, kind, mh, first, id);
      if (lane == 0 && npass < 32) {
        SPT_RAW(64 + npass, global_ns());
        SPT_RAW(96 + npass, static_cast<unsigned long long>(take) | (static_cast<unsigned long long>(next) << 16));
      }
      ++npass;
      next += take;
      __syncwarp();
    }
  };
  auto produce_ends = [&](int nstages) {
    bool ended = lane >= nstages;
    unsigned long long t0 = global_ns();
    while (!__all_sync(kFull, ended) && !s_abort) {
      if (!ended && lane_free()) {
        fill_lane(kItemEnd, 2, 0, 0, 0);
        ended = true;
      }
      if (global_ns() - t0 > c_wait_ns) {
        if (lane == 0) report(a.status, kStatusWaitTimeout);
        s_abort = 1;
      }
    }
  };

  // ---------------------------------------------------------------- set-up
#ifdef STK_TRACE
  const unsigned long long t_start = global_ns();
  if (warp == kStepProducer) {
    for (int i = lane; i < 128; i += 32) s_trc[i] = 0ull;
    s_trc_meta = 0u;
  }
#endif
  SPAN_START();
  const int n_first = min(my_meta, NS);
  // q arrives by one bulk copy queued ahead of the metadata (a load queued
  // behind this SM's bulk copies would wait for all of them): FP32 q straight
  // into qs, 16-bit q into s_wu (free until the row's final merge) and then
  // widened.
  const int qbytes = hq * D * (a.q_dtype == kF32 ? 4 : 2);
  void* q_dst = a.q_dtype == kF32 ? static_cast<void*>(qs) : static_cast<void*>(&s_wu[0][0]);
  long long lid_a = -1, lid_b = -1;  // producer lane: IDs of jobs jb + lane and jb + 32 + lane
  int jb = 0;
  if (warp == kStepProducer) {
    // Barriers and counters, q, then the first metadata items at once (one
    // lane each), before anything else of the CTA.
    if (lane == 0) {
      for (int i = 0; i < NS; ++i) {
        mbar_init(&full_bar[i], 1);
        mbar_init(&empty_bar[i], 1);
      }
      mbar_init(&q_bar, 1);
      mbar_init(&hit_bar, 1);
      fence_barrier_init();
      s_abort = 0;
      mbar_arrive_expect_tx(&q_bar, static_cast<unsigned>(qbytes));
      bulk_g2s(q_dst, a.q, static_cast<unsigned>(qbytes), &q_bar);
    }
    s_row_cnt[lane] = 0u;
    __syncwarp();
    barriers_ready_arrive();
    if (lane < n_first) {
      int mh, b0;
      meta_item(lane, mh, b0);
      fill_lane(lane, 0, mh, b0, 0);
    }
    __syncwarp();
    if (lane == 0) SPT(2);
    if (!serial) {
      lid_a = job_id(lane);
      lid_b = job_id(32 + lane);
    }
  } else {
    // q as FP32 in shared memory and its per-head ||q||_1 rounded up; the
    // producer does not take part.
    const int t = tid < kStepProducer * 32 ? tid : tid - 32;
    if (row_cta && !serial)
      for (int i = t; i < a.sp; i += kStepThreads - 32)
        s_pid[i] = static_cast<int>(load_id(a.pred, a.pred64, static_cast<long long>(row) * a.sp + i));
    barriers_ready_wait();
#ifdef STK_TRACE
    if (tid == 0) s_trc[0] = t_start;
#endif
    if (!mbar_wait(&q_bar, 0, a.status)) s_abort = 1;
    if (a.q_dtype != kF32) {
      const unsigned* raw = reinterpret_cast<const unsigned*>(&s_wu[0][0]);
      sync_non_producer();
      for (int i = t; i < hq * D / 2; i += kStepThreads - 32) {
        const unsigned w = raw[i];
        float lo, hi;
        if (a.q_dtype == kBF16) {
          lo = __uint_as_float(w << 16);
          hi = __uint_as_float(w & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
          lo = f.x;
          hi = f.y;
        }
        qs[2 * i] = lo;
        qs[2 * i + 1] = hi;
      }
    }
    sync_non_producer();
    const int wv = warp < kStepProducer ? warp : warp - 1;
    for (int h = wv; h < hq; h += kStepWarps - 1) {
      float sum = 0.f;
      for (int dd = lane; dd < D; dd += 32) sum = __fadd_ru(sum, fabsf(qs[h * D + dd]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum = __fadd_ru(sum, __shfl_xor_sync(kFull, sum, o));
      if (lane == 0) qn1[h] = sum;
    }
    sync_non_producer();
    if (tid == 0) SPT(1);
  }

  // ---------------------------------------------------------------- the ring
  // Consumer warp c (c < NS) owns stage c: it takes the stage's items one
  // phase after another until an end descriptor. A scored metadata item
  // counts for its KV head, a job's block state (written to the states
  // buffer) for its row, in shared-memory counters that the publisher warp
  // forwards to the control block; row-local blocks (misses, or the serial
  // row's own share) fold into the warp's running state (wm, wl, wu).
  unsigned kph = 0;  // phases this consumer has taken from its stage
  auto consume = [&](auto local_tag, const float* qrow_local, float& wm, float& wl, float (&wu)[DPH]) {
    constexpr bool kLocal = decltype(local_tag)::value;
    const int st = warp;
    const unsigned char* stage = pool + static_cast<size_t>(st) * kStageBytes;
    while (true) {
      const bool landed = mbar_wait(&full_bar[st], kph & 1u, a.status);
      if (!landed) {
        s_abort = 1;
        break;
      }
      if (lane == 0 && warp == 0 && kph < 16) SPT(32 + 2 * kph);
      ++kph;
      const int code = s_desc[st];
      const bool ok = item_ok[st] != 0;
      if (code == kItemEnd) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);
        break;
      }
      if (code < my_meta) {
        int mh, b0;
        meta_item(code, mh, b0);
#ifdef STK_SCORE_TWICE
        if (ok && warp == 0 && kph == 1) {
          if (lane == 0) SPT(25);
          score_item<GM>(a, reinterpret_cast<const float*>(stage),
                         reinterpret_cast<const float*>(stage + kStageBytes / 2), qs, qn1, mh, b0,
                         min(kMetaItemBlocks, n - b0), G, lane);
          __syncwarp();
          if (lane == 0) SPT(26);
        }
#endif
        if (ok)
          score_item<GM>(a, reinterpret_cast<const float*>(stage),
                         reinterpret_cast<const float*>(stage + kStageBytes / 2), qs, qn1, mh, b0,
                         min(kMetaItemBlocks, n - b0), G, lane);
        __syncwarp();
#ifdef STK_SCORE_TWICE
        if (warp == 0 && kph == 1 && lane == 0) SPT(27);
#endif
        if (lane == 0) {
          mbar_arrive(&empty_bar[st]);
          red_relaxed_gpu(&head_done[mh], 1u);
#ifdef STK_TRACE
          if (atomicAdd(&s_trc_meta, 1u) == static_cast<unsigned>(my_meta) - 1u) SPT(21);
#endif
        }
      } else if (code < kItemLocal) {
        const int job = j0 + (code - my_meta);
        const int r = job / SJ, slot = xl + (job - r * SJ);
        float m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
        for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
        if (ok) {
          float qf[DPH];
#pragma unroll
          for (int j = 0; j < DPH; ++j) qf[j] = qs[r * D + (lane & 15) * DPH + j];
          const T* ks = reinterpret_cast<const T*>(stage);
#ifdef STK_SCORE_TWICE
          if (warp == 0 && (code - my_meta) < 64 && s_trc[28] == 0) {
            if (lane == 0) SPT(28);
            float m2 = neg_inf(), l2 = 0.f, u2[DPH], ua2[DPH];
#pragma unroll
            for (int j = 0; j < DPH; ++j) { u2[j] = 0.f; ua2[j] = 0.f; }
            warp_block_state<T, DPH, kModeFull, true>(ks, ks + kStepB * D, kStepB, qf, a.scale, 0.f, m2, l2, u2, ua2,
                                                      lane);
            __syncwarp();
            if (lane == 0) SPT(29);
            warp_block_state<T, DPH, kModeFull, true>(ks, ks + kStepB * D, kStepB, qf, a.scale, 0.f, m, l, u, ua,
                                                      lane);
            __syncwarp();
            if (lane == 0) SPT(30);
          } else
#endif
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
        if (lane == 0) red_release_cta(&s_row_cnt[r], 1u);
      } else if constexpr (kLocal) {
        if (ok) {
          float qf[DPH], m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
          for (int j = 0; j < DPH; ++j) { qf[j] = qrow_local[(lane & 15) * DPH + j]; u[j] = 0.f; ua[j] = 0.f; }
          const T* ks = reinterpret_cast<const T*>(stage);
          warp_block_state<T, DPH, kModeFull, true>(ks, ks + kStepB * D, kStepB, qf, a.scale, 0.f, m, l, u, ua,
                                                    lane);
          fold_state(wm, wl, wu, m, l, u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);
        if (lane == 0 && warp == 0) SPT(15);
      }
      if (lane == 0 && warp == 0 && kph <= 16) SPT(33 + 2 * (kph - 1));
    }
  };

  if (warp == kStepProducer) {
    // First phase: the remaining metadata items, the CTA's jobs, then one
    // end descriptor per stage.
    produce(my_meta - n_first, [&](int) {},
            [&](int i, int& code, int& kind, int& mh, long long& first, long long&) {
              if (i < 0) return;
              int b0;
              code = n_first + i;
              kind = 0;
              meta_item(code, mh, b0);
              first = b0;
            });
    if (my_jobs > 0) {
      if (serial) {
        // The rows of [j0, j1) publish their selections as tags; their
        // row_ready counts tell when to start reading them.
        if (lane == 0)
          for (int r = j0 / SJ; r <= (j1 - 1) / SJ && !s_abort; ++r)
            if (!wait_count(&row_ready[r], 1)) {
              report(a.status, kStatusWaitTimeout);
              s_abort = 1;
            }
        __syncwarp();
        if (!s_abort) lid_a = job_id(lane);
        if (!s_abort) lid_b = job_id(32 + lane);
      }
      if (lane == 0) SPT(3);
      produce(my_jobs,
              [&](int next) {
                if (next >= jb + 32) {  // slide the ID window
                  jb += 32;
                  lid_a = lid_b;
                  lid_b = job_id(jb + 32 + lane);
                }
              },
              [&](int i, int& code, int& kind, int& mh, long long&, long long& id) {
                const int off = i < 0 ? 0 : i - jb;
                const long long va = __shfl_sync(kFull, lid_a, off & 31);
                long long vb = -1;  // read only when needed: it may still be loading
                if (__any_sync(kFull, off >= 32)) vb = __shfl_sync(kFull, lid_b, off & 31);
                if (i < 0) return;
                code = my_meta + i;
                kind = 1;
                mh = ((j0 + i) / SJ) / G;
                id = off < 32 ? va : vb;
              });
    }
    produce_ends(NS);
    if (lane == 0) SPT(4);
  } else if (warp < NS) {
    if (lane == 0 && warp == 0) SPT(12);
    float dm = 0.f, dl = 0.f, du[DPH];
    consume(std::false_type{}, nullptr, dm, dl, du);
    if (lane == 0 && warp == 0) SPT(14);
  } else if (warp == kStepPublisher) {
    // Forward the CTA's block-state completions GPU-wide: one fence per
    // batch (a GPU-scope fence waits behind this SM's bulk copies, so it is
    // kept off the consumers). Lane r < hq: row r's block states.
    unsigned pub_r = 0;
    const unsigned want = static_cast<unsigned>(my_jobs);
    unsigned long long t0 = global_ns();
    while (want > 0) {
      const unsigned cr = lane < hq ? ld_acquire_cta(&s_row_cnt[lane]) : 0u;
      const bool fresh = cr != pub_r;
      if (__any_sync(kFull, fresh)) {
        if (fresh) {
          __threadfence();
          atomicAdd(&row_states[lane], cr - pub_r);
        }
        pub_r = cr;
        t0 = global_ns();
      }
      if (static_cast<unsigned>(warp_sum_int(static_cast<int>(pub_r))) >= want || s_abort) break;
      if (global_ns() - t0 > c_wait_ns) {
        if (lane == 0) report(a.status, kStatusWaitTimeout);
        s_abort = 1;
        break;
      }
      __nanosleep(64);
    }
    if (lane == 0) SPT(13);
  }

  // ---------------------------------------------------------------- row CTAs
  __syncthreads();
  if (row_cta) {
    const float* qrow = qs + row * D;
    const int mh = row / G;
    if (tid == 0) SPT(5);
    // Membership of the predicted list (speculative step), the selection's
    // mask and the row-local list start empty; the predicted IDs arrived at
    // kernel start.
    for (int i = tid; i < (n + 31) / 32; i += kStepThreads) { s_pmask[i] = 0u; s_amask[i] = 0u; }
    __syncthreads();
    if (!serial)
      for (int i = tid; i < a.sp; i += kStepThreads) {
        const int id = s_pid[i];
        if (id >= 0 && id < n) atomicOr(&s_pmask[id >> 5], 1u << (id & 31));
      }
    // No wait for the head's metadata count: the selection polls the row's
    // score slots (each fills with one 8-byte store) and starts as soon as
    // the last one lands, with a bounded wait of its own.
    __syncthreads();
    if (tid == 0) SPT(6);
    // Row-local blocks: the misses (A not in P) of the saved repair, or the
    // serial row's first xl selected blocks. While the selection runs, the
    // blocks its intervals already classify as selected and that P lacks are
    // asked into L2 (their copies, issued once the list is final, then hit
    // L2); each selected block sets its bit in the selection's mask and
    // flags its output position when it is a miss.
    struct RowHook {
      const StepArgs* a;
      int* s_mflag;
      unsigned* s_pmask;
      unsigned* s_amask;
      int mh, n;
      bool serial;
      __device__ void sure_in(int id) const {
        if (serial || ((s_pmask[id >> 5] >> (id & 31)) & 1u)) return;
        const long long off = (static_cast<long long>(mh) * n + id) * kStepB * kStepD;
        constexpr unsigned kBytes = kStepB * kStepD * sizeof(T);
        bulk_prefetch_l2(static_cast<const T*>(a->k) + off, kBytes);
        bulk_prefetch_l2(static_cast<const T*>(a->v) + off, kBytes);
      }
      __device__ void selected(int pos, int id, bool) const {
        atomicOr(&s_amask[id >> 5], 1u << (id & 31));
        s_mflag[pos] = serial ? 0 : !((s_pmask[id >> 5] >> (id & 31)) & 1u);
      }
    };
    const RowHook hook{&a, s_loc, s_pmask, s_amask, mh, n, serial};
    if (!s_abort) {
      SelectArgs sa{};
      sa.R = 1; sa.hsel = hq; sa.topk = K; sa.n = n; sa.block_offsets = nullptr; sa.total_blocks = n;
      sa.id_base = 0; sa.ids_out = a.selected; sa.keys_out = nullptr; sa.status = a.status;
      sa.bounds = a.bounds; sa.q = a.q; sa.q_dtype = a.q_dtype; sa.lo = a.lo; sa.hi = a.hi;
      sa.hq = hq; sa.hmeta = hkv; sa.d = D; sa.group_select = 0;
      // The ring's first three stages hold no copy from the end of the scoring
      // phase until the first miss is issued: they stage the row's intervals.
      static_assert(3 * kStageBytes >= (kStepMaxBlocks + kStepMaxBlocks / 16) * 8 && kStepStages >= 3, "interval stage");
      bounded_select_core<E, kStepThreads, true, RowHook>(sa, row, qrow, true, s_sel, hook,
                                                          reinterpret_cast<float2*>(pool));
    }
    __syncthreads();
    if (tid == 0) SPT(7);
    // The ascending list of row-local blocks (warp 0; s_loc held the miss
    // flags of the output positions).
    if (warp == 0) {
      int nm = 0;
      for (int b = 0; b < K; b += 32) {
        const int pos = b + lane;
        const bool take = pos < K && (serial ? pos < xl : s_loc[pos] != 0);
        const int id = pos < K ? s_sel[pos] : -1;
        const unsigned bal = __ballot_sync(kFull, take);
        __syncwarp();
        if (take) s_glb[nm + __popc(bal & ((1u << lane) - 1u))] = id;
        nm += __popc(bal);
      }
      __syncwarp();
      for (int i = lane; i < nm; i += 32) s_loc[i] = s_glb[i];
      if (lane == 0) s_nloc = nm;
    }
    if (serial) {
      for (int i = xl + tid; i < K; i += kStepThreads) a.sel_tag[static_cast<long long>(row) * K + i] = s_sel[i] + 1;
      __syncthreads();
    } else if (warp < kStepHelper0) {
      sync_list_warps();  // the helpers need only the selection's mask, complete above
    }
    if (serial && tid == 0 && !s_abort) red_relaxed_gpu(&row_ready[row], 1u);
    const int nloc = (s_abort || (!serial && warp >= kStepHelper0)) ? 0 : s_nloc;
    // Block states to fold from the buffer: the hits (P slots whose block is
    // in A), or the serial row's slots xl .. K - 1.
    const int nglb = s_abort ? 0 : (serial ? K - xl : a.sp);
    float wm = neg_inf(), wl = 0.f, wu[DPH];
#pragma unroll
    for (int j = 0; j < DPH; ++j) wu[j] = 0.f;
    // Without the shared-memory hits below (serial step, or a predicted list
    // too large for three stages), the buffered states are folded from L2 by
    // the helper warps 12..15, eight per memory round trip, in a fixed slot
    // order, while the consumers take the row-local blocks.
    constexpr int nfw = kStepWarps - kStepHelper0;
    const int fw = warp - kStepHelper0;
    const long long rb = static_cast<long long>(row) * S;
    // Speculative step with a predicted list whose states fit three stages:
    // the misses use stages 0 .. NS - 4 only, the row's predicted states
    // (u, then m, then l) arrive in the last three stages with bulk copies
    // as soon as every work CTA has written them, and seven warps (the
    // helpers and the three consumers without a stage) fold the hits from
    // shared memory.
    constexpr int kHitStages = 3;
    const bool smem_hits = !serial && a.sp % 4 == 0 && a.sp * (D + 2) * 4 <= kHitStages * kStageBytes;
    const int NR = smem_hits ? NS - kHitStages : NS;  // stages of the row-local blocks
    constexpr int nhw = kHitStages + nfw;              // hit-folding warps in that case
    const int hw = warp >= kStepHelper0 ? kHitStages + (warp - kStepHelper0) : warp - (NS - kHitStages);
    float* hit_u = reinterpret_cast<float*>(pool + static_cast<size_t>(NS - kHitStages) * kStageBytes);
    float* hit_m = hit_u + a.sp * D;
    float* hit_l = hit_m + a.sp;
    // Buffer slot of fold i (serial: xl + i; speculative: P slot i when its
    // block is in A), or -1.
    auto fold_slot = [&](int i) {
      if (i >= nglb) return -1;
      if (serial) return xl + i;
      const int id = s_pid[i];
      return (id >= 0 && id < n && ((s_amask[id >> 5] >> (id & 31)) & 1u)) ? i : -1;
    };
    auto fold_buffered = [&]() {
      if (lane == 0 && nglb > 0 && !s_abort && !wait_count(&row_states[row], static_cast<unsigned>(SJ))) {
        report(a.status, kStatusWaitTimeout);
        s_abort = 1;
      }
      __syncwarp();
      if (fw == 0 && lane == 0) SPT(110);
      if (s_abort) return;
      constexpr int kBatch = 8;
      for (int i0 = fw; i0 < nglb; i0 += kBatch * nfw) {
        float mm[kBatch], ll[kBatch], uu[kBatch][DPH];
#pragma unroll
        for (int c = 0; c < kBatch; ++c) {
          const int slot = fold_slot(i0 + c * nfw);
          mm[c] = neg_inf();
          ll[c] = 0.f;
          if (slot >= 0) {
            const long long o = rb + slot;
            mm[c] = __ldcg(a.sm + o);
            ll[c] = __ldcg(a.sl + o);
            const float4* up = reinterpret_cast<const float4*>(a.su + o * D + (lane & 15) * DPH);
            const float4 x0 = __ldcg(up), x1 = __ldcg(up + 1);
            uu[c][0] = x0.x; uu[c][1] = x0.y; uu[c][2] = x0.z; uu[c][3] = x0.w;
            uu[c][4] = x1.x; uu[c][5] = x1.y; uu[c][6] = x1.z; uu[c][7] = x1.w;
          } else {
#pragma unroll
            for (int j = 0; j < DPH; ++j) uu[c][j] = 0.f;
          }
        }
        if (fw == 0 && lane == 0 && i0 == fw) SPT(111);
#pragma unroll
        for (int c = 0; c < kBatch; ++c) fold_state(wm, wl, wu, mm[c], ll[c], uu[c]);
      }
    };
    // Shared-memory hits: the first helper lane waits for the row's states
    // and issues their copy; every hit-folding warp then folds P slots
    // hw, hw + nhw, ... in order.
    auto fold_smem = [&]() {
      if (warp == kStepHelper0 && lane == 0) {
        bool ok = !s_abort && wait_count(&row_states[row], static_cast<unsigned>(SJ));
        if (ok) {
          // The states were written by other CTAs through the generic proxy
          // and acquired above; the bulk copy reads them through the async
          // proxy.
          asm volatile("fence.proxy.async.global;" ::: "memory");
          const unsigned ub = static_cast<unsigned>(a.sp) * D * 4, mb = static_cast<unsigned>(a.sp) * 4;
          mbar_arrive_expect_tx(&hit_bar, ub + 2 * mb);
          bulk_g2s(hit_u, a.su + rb * D, ub, &hit_bar);
          bulk_g2s(hit_m, a.sm + rb, mb, &hit_bar);
          bulk_g2s(hit_l, a.sl + rb, mb, &hit_bar);
        } else {
          report(a.status, kStatusWaitTimeout);
          s_abort = 1;
          mbar_arrive(&hit_bar);  // complete the phase without data
        }
      }
      if (!mbar_wait(&hit_bar, 0u, a.status)) s_abort = 1;
      __syncwarp();
      if (warp == kStepHelper0 && lane == 0) SPT(110);
      if (s_abort) return;
      for (int i = hw; i < a.sp; i += nhw) {
        if (fold_slot(i) < 0) continue;
        float uu[DPH];
        const float4* up = reinterpret_cast<const float4*>(hit_u + static_cast<size_t>(i) * D + (lane & 15) * DPH);
        const float4 x0 = up[0], x1 = up[1];
        uu[0] = x0.x; uu[1] = x0.y; uu[2] = x0.z; uu[3] = x0.w;
        uu[4] = x1.x; uu[5] = x1.y; uu[6] = x1.z; uu[7] = x1.w;
        fold_state(wm, wl, wu, hit_m[i], hit_l[i], uu);
      }
    };
    if (warp == kStepProducer) {
      if (lane == 0) SPT(123);
      // Row-local block i goes to stage i % NR, so that each consumer folds
      // a fixed subsequence of the list in order: the result does not depend
      // on timing.
      for (int base = 0; base < nloc && !s_abort; base += NR) {
        bool done = lane >= NR || base + lane >= nloc;
        const unsigned long long t0 = global_ns();
        while (!__all_sync(kFull, done) && !s_abort) {
          if (!done && lane_free()) {
            fill_lane(kItemLocal + base + lane, 1, mh, 0, s_loc[base + lane]);
            done = true;
          }
          if (global_ns() - t0 > c_wait_ns) {
            if (lane == 0) report(a.status, kStatusWaitTimeout);
            s_abort = 1;
          }
        }
      }
      if (lane == 0) SPT(8);
      produce_ends(NR);
      if (lane == 0) SPT(23);
    } else if (warp < NR) {
      consume(std::true_type{}, qrow, wm, wl, wu);
      if (lane == 0 && warp == 0) SPT(24);
    } else if (warp < NS) {
      fold_smem();  // smem_hits: the consumers of the hit stages
    } else {
      if (smem_hits) fold_smem(); else fold_buffered();
      if (warp == kStepHelper0 && lane == 0) SPT(9);
      // The row's score slots go back to zero for the next call.
      unsigned long long* slots = reinterpret_cast<unsigned long long*>(a.bounds + static_cast<long long>(row) * n);
      for (int i = tid - kStepHelper0 * 32; i < n; i += nfw * 32) slots[i] = 0ull;
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
#ifdef STK_TRACE
  __syncthreads();
  if (blockIdx.x < 256)
    for (int i = tid; i < 128; i += kStepThreads) g_step_trace[blockIdx.x * 128 + i] = s_trc[i];
#endif
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(ctas_done, 1u) == static_cast<unsigned>(grid) - 1;
  }
  __syncthreads();
  if (s_last) {
    // Every other CTA is done: zero the serial tags and the control block.
    if (serial)
      for (int i = tid; i < hq * K; i += kStepThreads) a.sel_tag[i] = 0;
    if (tid == 0) {
      for (int i = 0; i < hkv + 2 * hq; ++i) atomicExch(a.ctrl + i, 0u);
      atomicExch(ctas_done, 0u);
      SPAN_END();
    }
    __threadfence();
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
