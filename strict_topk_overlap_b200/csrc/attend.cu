// Exact / saved / union attention over a row's selected blocks, one launch.
//
// Replaces, for the plain-LSE-merge repairs (no guards):
//   kernels.py:437-447       exact_attention / merge_partials(block_partials)
//   gqa.py:29-104,140-142    gqa.exact, REPAIR _partial + _merge_repair
//                            (repair_saved, repair_union)
//   gqa_light.py:10-60       _repair_light (saved semantics)
//   gqa_hierarchical.py:99-144 exact / repair_saved / repair_saved_shared
//
// One thread-block cluster of CS CTAs (kAW warps each) serves one
// (request, query head) row:
//   1. every CTA loads the row's selected IDs A (and predicted IDs P), marks
//      P in a shared-memory bitmap and lists the blocks to compute in A
//      order — all of A (exact) or A minus P (saved, union);
//   2. CTA c takes list entries c, c + CS, ...: it asks L2 for all of their
//      blocks (cp.async.bulk.prefetch.L2), then each warp streams its entries
//      through a private stage with bulk copies and folds each block's state
//      into a per-warp LSE state; the CTA also folds retained prediction
//      slots c, c + CS, ... (saved: P slots whose ID is in A; union: all);
//   3. each CTA pushes its partial (M, Z, U[D]) into rank 0's shared memory
//      with distributed-shared-memory stores (after a split cluster barrier,
//      armed at kernel start, confirms every CTA of the cluster has started);
//      after one more cluster barrier rank 0 merges the CS partials in rank
//      order and writes the row's output.
// Waits on bulk copies are bounded; a warp whose wait ran out records the
// status and stops, and its CTA still reaches the cluster barrier.
#include <cooperative_groups.h>

#include "block_state.cuh"

namespace cg = cooperative_groups;

namespace stk {

constexpr int kAW = 4;           // warps per CTA
constexpr int kAttendCluster = 8;

#ifdef STK_TRACE
// [cta][8] timeline of the attend kernel (profiling builds only).
static __device__ unsigned long long g_attend_trace[4096 * 8];
extern "C" __attribute__((visibility("default"))) void* stk_trace_attend() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_attend_trace);
  return p;
}
#define AT(ev) do { if (blockIdx.x < 4096 && threadIdx.x == 0) STK_TRACE_AT(g_attend_trace, blockIdx.x * 8 + (ev)); } while (0)
#else
#define AT(ev) ((void)0)
#endif

struct AttendSmem {
  long long* a_ids;  // [sa]
  long long* p_ids;  // [sp]
  unsigned* bitA;    // [nwords]
  unsigned* bitP;    // [nwords]
  int* list;         // [sa] entries (indices into A) to compute
  float* qv;         // [d]
  float* wU;         // [kAW][d] per-warp numerators
  float* pushU;      // [CS][d] partial numerators pushed by each CTA (rank 0's copy is read)
  float* pushS;      // [CS][2] partial (M, Z)
  float* rm;         // [ns] retained-slot maxima of this CTA's slots rank, rank + CS, ...
  float* rl;         // [ns] retained-slot normalisers
  float* ru;         // [ns][d] retained-slot numerators
};

template <int DPH, typename T>
__host__ __device__ inline size_t attend_layout(const RepairArgs& a, int cs, AttendSmem* S, unsigned char* base) {
  const int D = a.d;
  size_t off = 0;
  auto take = [&](size_t bytes, size_t align) {
    off = (off + align - 1) & ~(align - 1);
    const size_t at = off;
    off += bytes;
    return at;
  };
  const size_t st = take(static_cast<size_t>(kAW) * 2 * 32 * D * sizeof(T), 128);
  (void)st;
  const int nwords = (a.max_n + 31) / 32;
  const size_t ai = take(static_cast<size_t>(a.sa) * 8, 16), pi = take(static_cast<size_t>(a.sp) * 8, 16);
  const size_t ba = take(static_cast<size_t>(nwords) * 4, 16), bp = take(static_cast<size_t>(nwords) * 4, 16);
  const size_t li = take(static_cast<size_t>(a.sa) * 4, 16);
  const size_t qv = take(static_cast<size_t>(D) * 4, 16);
  const size_t wu = take(static_cast<size_t>(kAW) * D * 4, 16);
  const size_t pu = take(static_cast<size_t>(cs) * D * 4, 16);
  const size_t ps = take(static_cast<size_t>(cs) * 8, 16);
  const int ns = a.pmode == kPredNone ? 0 : (a.sp + cs - 1) / cs;
  const size_t rm = take(static_cast<size_t>(ns) * 4, 16), rl = take(static_cast<size_t>(ns) * 4, 16);
  const size_t ru = take(static_cast<size_t>(ns) * D * 4, 16);
  if (S != nullptr) {
    S->a_ids = reinterpret_cast<long long*>(base + ai);
    S->p_ids = reinterpret_cast<long long*>(base + pi);
    S->bitA = reinterpret_cast<unsigned*>(base + ba);
    S->bitP = reinterpret_cast<unsigned*>(base + bp);
    S->list = reinterpret_cast<int*>(base + li);
    S->qv = reinterpret_cast<float*>(base + qv);
    S->wU = reinterpret_cast<float*>(base + wu);
    S->pushU = reinterpret_cast<float*>(base + pu);
    S->pushS = reinterpret_cast<float*>(base + ps);
    S->rm = reinterpret_cast<float*>(base + rm);
    S->rl = reinterpret_cast<float*>(base + rl);
    S->ru = reinterpret_cast<float*>(base + ru);
  }
  return off;
}

// One warp folds a block state (m, l, u in half-warp layout) into its
// running LSE state (wm, wl in registers; numerators in smem row U).
template <int DPH>
__device__ __forceinline__ void fold_state(float& wm, float& wl, float* U, float m, float l, const float (&u)[DPH],
                                           int lane) {
  if (m == neg_inf()) return;
  const float mn = fmaxf(wm, m);
  const float a1 = wm == neg_inf() ? 0.f : expf(wm - mn), a2 = expf(m - mn);
  if (lane < 16) {
#pragma unroll
    for (int j = 0; j < DPH; ++j) {
      float* p = U + lane * DPH + j;
      *p = *p * a1 + u[j] * a2;
    }
  }
  wl = wl * a1 + l * a2;
  wm = mn;
}

template <typename T, int DPH, bool FULL32>
__global__ void __launch_bounds__(kAW * 32) attend_kernel(RepairArgs a) {
  constexpr int D = 16 * DPH;
  constexpr int kChunk = 32 * D;  // elements of one 32-token chunk of K (or V)
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar[kAW];
  __shared__ int sh_cnt[kAW + 1];
  __shared__ float sh_w[kAW][2];
  __shared__ float sh_keep[2];

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  // A launch whose cluster shape differs from the host's plan (rows x CS
  // CTAs in clusters of CS) would map CTAs to the wrong rows: refuse it.
  if (CS != a.cluster || gridDim.x != static_cast<unsigned>(a.rows) * a.cluster) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x / CS;
  const int r = row / a.hq;
  const int kv = (row - r * a.hq) / a.g;
  const int nblocks = request_blocks(a.L, r);
  const bool has_pred = a.pmode != kPredNone;

  AttendSmem S;
  attend_layout<DPH, T>(a, CS, &S, smem);
  T* stage = reinterpret_cast<T*>(smem) + static_cast<size_t>(warp) * 2 * kChunk;
  uint64_t* mb = &bar[warp];
  const int nwords = (a.max_n + 31) / 32;

  // Announce this CTA to the cluster (its shared memory is live); the
  // matching wait comes before the first remote store into rank 0.
  AT(0);
  pdl_release();
  cluster_arrive_relaxed();

  // ---- 1. IDs, q, bitmaps, the list of blocks to compute.
  // Everything except the selected IDs A is ready when this kernel starts
  // (q and P come from the host or from kernels this launch fully depends
  // on); it is loaded before waiting for the preceding kernel, which may be
  // the one writing A. These small loads also go out before any of this
  // kernel's bulk traffic (a load issued behind it waits for all of it).
  if (lane == 0) {
    mbar_init(mb, 1);
    fence_barrier_init();
  }
  for (int i = tid; i < nwords; i += blockDim.x) { S.bitA[i] = 0u; S.bitP[i] = 0u; }
  for (int i = tid; i < kAW * D; i += blockDim.x) S.wU[i] = 0.f;
  if (has_pred)
    for (int i = tid; i < a.sp; i += blockDim.x)
      S.p_ids[i] = load_id(a.pred, a.pred64, static_cast<long long>(row) * a.sp + i);
  for (int dd = tid; dd < D; dd += blockDim.x) S.qv[dd] = load_any(a.q, a.q_dtype, static_cast<long long>(row) * D + dd);
  // This CTA's prediction slots rank, rank + CS, ...
  const int ns = has_pred ? (a.sp - rank + CS - 1) / CS : 0;
  auto load_states = [&]() {
    const long long sr = static_cast<long long>(row) * a.sc;
    for (int i = tid; i < ns; i += blockDim.x) {
      S.rm[i] = a.pm[sr + rank + i * CS];
      S.rl[i] = a.pl[sr + rank + i * CS];
    }
    for (int i = tid; i < ns * D; i += blockDim.x) {
      const int si = i / D, dd = i - si * D;
      S.ru[i] = a.pu[(sr + rank + si * CS) * D + dd];
    }
  };
  if (has_pred && !a.chain) load_states();
  __syncthreads();
  if (has_pred)
    for (int i = tid; i < a.sp; i += blockDim.x) {
      const long long id = S.p_ids[i];
      if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); S.p_ids[i] = -1; continue; }
      atomicOr(&S.bitP[id >> 5], 1u << (id & 31));
    }
  pdl_wait();  // A (and, chained, the prediction states) may come from the preceding kernel
  for (int i = tid; i < a.sa; i += blockDim.x) S.a_ids[i] = load_id(a.sel, a.sel64, static_cast<long long>(row) * a.sa + i);
  if (has_pred && a.chain) load_states();
  __syncthreads();
  AT(1);
  for (int i = tid; i < a.sa; i += blockDim.x) {
    const long long id = S.a_ids[i];
    if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); S.a_ids[i] = -1; continue; }
    atomicOr(&S.bitA[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  // List = A entries to compute, in A order (block-wide ballot prefix).
  int total = 0;
  for (int base = 0; base < a.sa; base += blockDim.x) {
    const int i = base + tid;
    bool need = false;
    if (i < a.sa) {
      const long long id = S.a_ids[i];
      need = id >= 0 && !(has_pred && ((S.bitP[id >> 5] >> (id & 31)) & 1u));
    }
    const unsigned bal = __ballot_sync(kFull, need);
    if (lane == 0) sh_cnt[warp] = __popc(bal);
    __syncthreads();
    int before = total;
    for (int w = 0; w < warp; ++w) before += sh_cnt[w];
    if (need) S.list[before + __popc(bal & ((1u << lane) - 1))] = i;
    for (int w = 0; w < kAW; ++w) total += sh_cnt[w];
    __syncthreads();
  }
  const int count = total;
  AT(2);

  // ---- 2. this CTA's share: L2 prefetch, first copies, retained slots, blocks.
  for (int k = rank + CS * tid; k < count; k += CS * blockDim.x)
    prefetch_block<T>(a.L, r, kv, S.a_ids[S.list[k]], true);
  const int nchunks = (a.L.b + 31) / 32;
  const int kfirst = rank + CS * warp, kstep = CS * kAW;
  const unsigned chunk_bytes_full = 32u * D * sizeof(T);
  auto issue = [&](int k, int c) {
    const long long bid = S.a_ids[S.list[k]];
    const int t0 = c * 32, ntok = FULL32 ? 32 : min(32, a.L.b - t0);
    T* ks = stage;
    T* vs = stage + kChunk;
    const unsigned bytes = FULL32 ? chunk_bytes_full : static_cast<unsigned>(ntok * D * sizeof(T));
    mbar_arrive_expect_tx(mb, 2 * bytes);
    const T* K = static_cast<const T*>(a.L.k);
    const T* V = static_cast<const T*>(a.L.v);
    if (a.L.page_table == nullptr) {
      const long long o = block_seg(a.L, r, kv, bid, 0).elem_off + static_cast<long long>(t0) * D;
      bulk_g2s(ks, K + o, bytes, mb);
      bulk_g2s(vs, V + o, bytes, mb);
    } else {
      for (int t = t0; t < t0 + ntok;) {
        const int pg = t / a.L.page_size, po = t - pg * a.L.page_size;
        const int cnt = min(a.L.page_size - po, t0 + ntok - t);
        const long long o = block_seg(a.L, r, kv, bid, pg).elem_off + static_cast<long long>(po) * D;
        const unsigned sb = static_cast<unsigned>(cnt * D * sizeof(T));
        bulk_g2s(ks + (t - t0) * D, K + o, sb, mb);
        bulk_g2s(vs + (t - t0) * D, V + o, sb, mb);
        t += cnt;
      }
    }
  };
  if (kfirst < count && lane == 0) issue(kfirst, 0);
  AT(3);

  // Retained prediction slots of this CTA (saved: hits; union: every slot),
  // weights relative to the CTA's own maximum.
  if (has_pred) {
    if (warp == 0) {
      // keep flags into rm: -inf marks a slot that is not retained.
      float M = neg_inf();
      for (int i = lane; i < ns; i += 32) {
        const long long id = S.p_ids[rank + i * CS];
        const bool keep = id >= 0 && (a.variant == kVarUnion || ((S.bitA[id >> 5] >> (id & 31)) & 1u));
        if (!keep) S.rm[i] = neg_inf();
        M = fmaxf(M, S.rm[i]);
      }
      M = warp_max(M);
      float Z = 0.f;
      for (int i = lane; i < ns; i += 32)
        if (S.rm[i] != neg_inf()) Z += expf(S.rm[i] - M) * S.rl[i];
      Z = warp_sum(Z);
      if (lane == 0) { sh_keep[0] = M; sh_keep[1] = Z; }
    }
    __syncthreads();
  } else if (tid == 0) {
    sh_keep[0] = neg_inf();
    sh_keep[1] = 0.f;
  }

  float qf[DPH];
#pragma unroll
  for (int j = 0; j < DPH; ++j) qf[j] = S.qv[(lane & 15) * DPH + j];
  float wm = neg_inf(), wl = 0.f;
  float* myU = S.wU + warp * D;
  unsigned phase = 0;
  bool ok = true;
#pragma unroll 1
  for (int k = kfirst; k < count && ok; k += kstep) {
    float m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
    for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      ok = mbar_wait(mb, phase, a.status);
      phase ^= 1u;
      if (!ok) break;
      const int ntok = FULL32 ? 32 : min(32, a.L.b - c * 32);
      warp_block_state<T, DPH, kModeFull, FULL32>(stage, stage + kChunk, ntok, qf, a.scale, 0.f, m, l, u, ua, lane);
      __syncwarp();
      // Stage free: the next chunk of this block, or this warp's next block.
      if (lane == 0) {
        if (c + 1 < nchunks) issue(k, c + 1);
        else if (k + kstep < count) issue(k + kstep, 0);
      }
    }
    if (ok) fold_state<DPH>(wm, wl, myU, m, l, u, lane);
  }
  if (lane == 0) { sh_w[warp][0] = wm; sh_w[warp][1] = wl; }
  AT(4);
  __syncthreads();
  AT(5);

  // ---- 3. CTA partial -> rank 0 (distributed shared memory), merge there.
  float M = sh_keep[0];
  for (int w = 0; w < kAW; ++w) M = fmaxf(M, sh_w[w][0]);
  cluster_wait();  // every CTA of the cluster has started
  float* dstU = cluster.map_shared_rank(S.pushU, 0) + rank * D;
  for (int dd = tid; dd < D; dd += blockDim.x) {
    float U = 0.f;
    for (int w = 0; w < kAW; ++w)
      if (sh_w[w][0] != neg_inf()) U += expf(sh_w[w][0] - M) * S.wU[w * D + dd];
    if (has_pred && sh_keep[0] != neg_inf()) {
      // Retained numerators of this CTA's slots, weighted at M.
      float R = 0.f;
      for (int i = 0; i < ns; ++i)
        if (S.rm[i] != neg_inf()) R = fmaf(expf(S.rm[i] - M), S.ru[i * D + dd], R);
      U += R;
    }
    dstU[dd] = U;
  }
  if (tid == 0) {
    float Z = sh_keep[0] != neg_inf() ? expf(sh_keep[0] - M) * sh_keep[1] : 0.f;
    for (int w = 0; w < kAW; ++w)
      if (sh_w[w][0] != neg_inf()) Z += expf(sh_w[w][0] - M) * sh_w[w][1];
    float* dstS = cluster.map_shared_rank(S.pushS, 0) + rank * 2;
    dstS[0] = M;
    dstS[1] = Z;
  }
  AT(6);
  cluster.sync();
  AT(7);
  if (rank != 0) return;
  float GM = neg_inf();
  for (int c = 0; c < CS; ++c) GM = fmaxf(GM, S.pushS[c * 2]);
  float GZ = 0.f;
  for (int c = 0; c < CS; ++c)
    if (S.pushS[c * 2] != neg_inf()) GZ += expf(S.pushS[c * 2] - GM) * S.pushS[c * 2 + 1];
  for (int dd = tid; dd < D; dd += blockDim.x) {
    float U = 0.f;
    for (int c = 0; c < CS; ++c)
      if (S.pushS[c * 2] != neg_inf()) U += expf(S.pushS[c * 2] - GM) * S.pushU[c * D + dd];
    a.out[static_cast<long long>(row) * D + dd] = U / fmaxf(GZ, 1e-30f);
  }
  if (tid == 0) {
    if (a.fallback) a.fallback[row] = 0;
    if (a.remaining) a.remaining[row] = 1.f;
    if (a.approx) a.approx[row] = 0;
    if (a.extra) a.extra[row] = 0.f;
    if (a.pos_out) a.pos_out[row] = count;
    if (a.total_out) a.total_out[row] = count;
  }
}

// ------------------------------------------------------------------ saved repair, one CTA per row
// The low-latency form of the saved / union repair (reference gqa_light.py:
// one program per query head): one CTA of kLW warps per row, no cluster.
// Predicted IDs and q are loaded before waiting for the preceding kernel
// (the one writing A), and so are the prediction states' m and l unless
// that kernel also wrote them (a.chain). After the wait A's misses are
// listed and each warp starts streaming its first miss through a private
// stage; while those copies land, every warp folds its share of the
// retained slots' numerators (saved: P slots whose ID is in A; union: all)
// straight from global memory, then reduces its misses; one merge in warp
// order writes the row's output.
constexpr int kLW = 8;

template <typename T, int DPH, bool FULL32, int LW>
__global__ void __launch_bounds__(LW * 32) light_kernel(RepairArgs a) {
  constexpr int D = 16 * DPH;
  constexpr int kChunk = 32 * D;
  constexpr int kDL = D / 32;  // dims per lane in the retained fold
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar[LW];
  __shared__ float sh_w[LW + 1][2];
  __shared__ int sh_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int r = row / a.hq;
  const int kv = (row - r * a.hq) / a.g;
  const int nblocks = request_blocks(a.L, r);
  const int nwords = (a.max_n + 31) / 32;
  AT(0);
  pdl_release();

  // Shared memory: stages [LW][2][32][D] T, then the row's bookkeeping.
  T* stage = reinterpret_cast<T*>(smem) + static_cast<size_t>(warp) * 2 * kChunk;
  size_t off = static_cast<size_t>(LW) * 2 * kChunk * sizeof(T);
  auto carve = [&](size_t bytes) {
    off = (off + 15) & ~size_t(15);
    unsigned char* p = smem + off;
    off += bytes;
    return p;
  };
  float* pm_s = reinterpret_cast<float*>(carve(static_cast<size_t>(a.sp) * 4));
  float* pl_s = reinterpret_cast<float*>(carve(static_cast<size_t>(a.sp) * 4));
  long long* p_ids = reinterpret_cast<long long*>(carve(static_cast<size_t>(a.sp) * 8));
  long long* a_ids = reinterpret_cast<long long*>(carve(static_cast<size_t>(a.sa) * 8));
  unsigned* bitA = reinterpret_cast<unsigned*>(carve(static_cast<size_t>(nwords) * 4));
  unsigned* bitP = reinterpret_cast<unsigned*>(carve(static_cast<size_t>(nwords) * 4));
  int* list = reinterpret_cast<int*>(carve(static_cast<size_t>(a.sa) * 4));
  float* qv = reinterpret_cast<float*>(carve(static_cast<size_t>(D) * 4));
  float* wU = reinterpret_cast<float*>(carve(static_cast<size_t>(LW) * D * 4));  // miss numerators per warp
  float* wR = reinterpret_cast<float*>(carve(static_cast<size_t>(LW) * D * 4));  // retained numerators per warp

  if (lane == 0) {
    mbar_init(&bar[warp], 1);
    fence_barrier_init();
  }
  // ---- before the wait: everything the preceding kernel does not write.
  const long long sr = static_cast<long long>(row) * a.sp;
  auto load_ml = [&]() {
    for (int i = tid; i < a.sp; i += blockDim.x) {
      pm_s[i] = a.pm[sr + i];
      pl_s[i] = a.pl[sr + i];
    }
  };
  for (int i = tid; i < nwords; i += blockDim.x) { bitA[i] = 0u; bitP[i] = 0u; }
  for (int i = tid; i < a.sp; i += blockDim.x) p_ids[i] = load_id(a.pred, a.pred64, sr + i);
  for (int dd = tid; dd < D; dd += blockDim.x) qv[dd] = load_any(a.q, a.q_dtype, static_cast<long long>(row) * D + dd);
  if (!a.chain) load_ml();
  __syncthreads();
  for (int i = tid; i < a.sp; i += blockDim.x) {
    const long long id = p_ids[i];
    if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); p_ids[i] = -1; continue; }
    atomicOr(&bitP[id >> 5], 1u << (id & 31));
  }
  pdl_wait();  // A (and, chained, the prediction states) come from the preceding kernel
  AT(1);
  if (a.chain) load_ml();
  for (int i = tid; i < a.sa; i += blockDim.x) {
    long long id = load_id(a.sel, a.sel64, static_cast<long long>(row) * a.sa + i);
    if (id < 0 || id >= nblocks) { report(a.status, kStatusBadBlockId); id = -1; }
    a_ids[i] = id;
    if (id >= 0) atomicOr(&bitA[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  // Misses (A entries not in P), in A order.
  if (warp == 0) {
    int n = 0;
    for (int base = 0; base < a.sa; base += 32) {
      const int i = base + lane;
      bool miss = false;
      if (i < a.sa) {
        const long long id = a_ids[i];
        miss = id >= 0 && !((bitP[id >> 5] >> (id & 31)) & 1u);
      }
      const unsigned bal = __ballot_sync(kFull, miss);
      if (miss) list[n + __popc(bal & ((1u << lane) - 1))] = i;
      n += __popc(bal);
    }
    if (lane == 0) sh_total = n;
  }
  __syncthreads();
  const int count = sh_total;
  AT(2);

  // Blocks shorter than a 32-token chunk (e.g. 4-token blocks) are gathered
  // mp = 32 / B misses to a stage: the misses are folded into one state
  // anyway, so one reduction covers them all.
  const int mp = (!FULL32 && a.L.b < 32 && 32 % a.L.b == 0) ? 32 / a.L.b : 1;
  const int ngroups = (count + mp - 1) / mp;
  const int nchunks = mp > 1 ? 1 : (a.L.b + 31) / 32;
  auto issue = [&](int kg, int c) {
    const T* K = static_cast<const T*>(a.L.k);
    const T* V = static_cast<const T*>(a.L.v);
    if (mp > 1) {
      const int k0 = kg * mp, nk = min(mp, count - k0);
      mbar_arrive_expect_tx(&bar[warp], static_cast<unsigned>(2 * nk * a.L.b * D * sizeof(T)));
      const int nseg = block_nseg(a.L);
      for (int j = 0; j < nk; ++j) {
        const long long bid = a_ids[list[k0 + j]];
        for (int sg = 0; sg < nseg; ++sg) {
          const BlockSeg seg = block_seg(a.L, r, kv, bid, sg);
          const unsigned sb = static_cast<unsigned>(seg.tokens * D * sizeof(T));
          const size_t dst = static_cast<size_t>(j * a.L.b + sg * seg.tokens) * D;
          bulk_g2s(stage + dst, K + seg.elem_off, sb, &bar[warp]);
          bulk_g2s(stage + kChunk + dst, V + seg.elem_off, sb, &bar[warp]);
        }
      }
      return;
    }
    const long long bid = a_ids[list[kg]];
    const int t0 = c * 32, ntok = FULL32 ? 32 : min(32, a.L.b - t0);
    const unsigned bytes = static_cast<unsigned>(ntok * D * sizeof(T));
    mbar_arrive_expect_tx(&bar[warp], 2 * bytes);
    if (a.L.page_table == nullptr) {
      const long long o = block_seg(a.L, r, kv, bid, 0).elem_off + static_cast<long long>(t0) * D;
      bulk_g2s(stage, K + o, bytes, &bar[warp]);
      bulk_g2s(stage + kChunk, V + o, bytes, &bar[warp]);
    } else {
      for (int t = t0; t < t0 + ntok;) {
        const int pg = t / a.L.page_size, po = t - pg * a.L.page_size;
        const int cnt = min(a.L.page_size - po, t0 + ntok - t);
        const long long o = block_seg(a.L, r, kv, bid, pg).elem_off + static_cast<long long>(po) * D;
        const unsigned sb = static_cast<unsigned>(cnt * D * sizeof(T));
        bulk_g2s(stage + (t - t0) * D, K + o, sb, &bar[warp]);
        bulk_g2s(stage + kChunk + (t - t0) * D, V + o, sb, &bar[warp]);
        t += cnt;
      }
    }
  };
  if (warp < ngroups && lane == 0) issue(warp, 0);
  AT(3);
  // Later misses (beyond one stage per warp) are prefetched into L2 now.
  for (int k = LW * mp + tid; k < count; k += blockDim.x) prefetch_block<T>(a.L, r, kv, a_ids[list[k]], true);

  // Retained slots while the copies land: every warp finds their max Mr;
  // warp w folds slots w, w + LW, ... with weights exp(m - Mr); the last
  // warp also records (Mr, Zr).
  float Mr = neg_inf();
  auto kept = [&](int c) {
    const long long id = p_ids[c];
    return id >= 0 && (a.variant == kVarUnion || ((bitA[id >> 5] >> (id & 31)) & 1u));
  };
  for (int c = lane; c < a.sp; c += 32)
    if (kept(c)) Mr = fmaxf(Mr, pm_s[c]);
  Mr = warp_max(Mr);
  if (warp == LW - 1) {
    float Zr = 0.f;
    for (int c = lane; c < a.sp; c += 32)
      if (kept(c) && pm_s[c] != neg_inf()) Zr += expf(pm_s[c] - Mr) * pl_s[c];
    Zr = warp_sum(Zr);
    if (lane == 0) { sh_w[LW][0] = Mr; sh_w[LW][1] = Zr; }
  }
  {
    // Eight slots' numerators are loaded before any is used (one memory
    // round trip per eight slots, not one per slot).
    constexpr int kBatch = 8;
    float R[kDL];
#pragma unroll
    for (int j = 0; j < kDL; ++j) R[j] = 0.f;
    for (int c0 = warp; c0 < a.sp; c0 += LW * kBatch) {
      float v[kBatch][kDL], w[kBatch];
#pragma unroll
      for (int t = 0; t < kBatch; ++t) {
        const int c = c0 + t * LW;
        w[t] = 0.f;
        if (c < a.sp) {
          const float* pu = a.pu + (sr + c) * D;
#pragma unroll
          for (int j = 0; j < kDL; ++j) v[t][j] = pu[j * 32 + lane];
          if (kept(c) && pm_s[c] != neg_inf()) w[t] = expf(pm_s[c] - Mr);
        } else {
#pragma unroll
          for (int j = 0; j < kDL; ++j) v[t][j] = 0.f;
        }
      }
#pragma unroll
      for (int t = 0; t < kBatch; ++t)
#pragma unroll
        for (int j = 0; j < kDL; ++j) R[j] = fmaf(w[t], v[t][j], R[j]);
    }
#pragma unroll
    for (int j = 0; j < kDL; ++j) wR[warp * D + j * 32 + lane] = R[j];
  }

  float qf[DPH];
#pragma unroll
  for (int j = 0; j < DPH; ++j) qf[j] = qv[(lane & 15) * DPH + j];
  float wm = neg_inf(), wl = 0.f;
  float* myU = wU + warp * D;
  for (int dd = lane; dd < D; dd += 32) myU[dd] = 0.f;
  __syncwarp();
  unsigned phase = 0;
  bool ok = true;
#pragma unroll 1
  for (int k = warp; k < ngroups && ok; k += LW) {
    float m = neg_inf(), l = 0.f, u[DPH], ua[DPH];
#pragma unroll
    for (int j = 0; j < DPH; ++j) { u[j] = 0.f; ua[j] = 0.f; }
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      ok = mbar_wait(&bar[warp], phase, a.status);
      phase ^= 1u;
      if (!ok) break;
      const int ntok = mp > 1 ? a.L.b * min(mp, count - k * mp) : (FULL32 ? 32 : min(32, a.L.b - c * 32));
      warp_block_state<T, DPH, kModeFull, FULL32>(stage, stage + kChunk, ntok, qf, a.scale, 0.f, m, l, u, ua, lane);
      __syncwarp();
      if (lane == 0) {
        if (c + 1 < nchunks) issue(k, c + 1);
        else if (k + LW < ngroups) issue(k + LW, 0);
      }
    }
    if (ok) fold_state<DPH>(wm, wl, myU, m, l, u, lane);
  }
  if (lane == 0) { sh_w[warp][0] = wm; sh_w[warp][1] = wl; }
  __syncthreads();
  AT(4);
  // Final merge: warps in order, then the retained slots.
  float M = sh_w[LW][0];
  for (int w = 0; w < LW; ++w) M = fmaxf(M, sh_w[w][0]);
  float Z = sh_w[LW][0] != neg_inf() ? expf(sh_w[LW][0] - M) * sh_w[LW][1] : 0.f;
  for (int w = 0; w < LW; ++w)
    if (sh_w[w][0] != neg_inf()) Z += expf(sh_w[w][0] - M) * sh_w[w][1];
  const float kscale = sh_w[LW][0] != neg_inf() ? expf(sh_w[LW][0] - M) : 0.f;
  for (int dd = tid; dd < D; dd += blockDim.x) {
    float U = 0.f;
    for (int w = 0; w < LW; ++w)
      if (sh_w[w][0] != neg_inf()) U += expf(sh_w[w][0] - M) * wU[w * D + dd];
    if (kscale != 0.f) {
      float R = 0.f;
      for (int w = 0; w < LW; ++w) R += wR[w * D + dd];
      U += kscale * R;
    }
    a.out[static_cast<long long>(row) * D + dd] = U / fmaxf(Z, 1e-30f);
  }
  if (tid == 0) {
    if (a.fallback) a.fallback[row] = 0;
    if (a.remaining) a.remaining[row] = 1.f;
    if (a.approx) a.approx[row] = 0;
    if (a.extra) a.extra[row] = 0.f;
    if (a.pos_out) a.pos_out[row] = count;
    if (a.total_out) a.total_out[row] = count;
  }
  AT(7);
}

template <typename T, int DPH, int LW>
static int launch_light_lw(const RepairArgs& a, cudaStream_t stream) {
  const int nwords = (a.max_n + 31) / 32;
  const int D = a.d;
  size_t smem = static_cast<size_t>(LW) * 2 * 32 * D * sizeof(T);
  auto add = [&](size_t b) { smem = ((smem + 15) & ~size_t(15)) + b; };
  add(static_cast<size_t>(a.sp) * 4); add(static_cast<size_t>(a.sp) * 4);
  add(static_cast<size_t>(a.sp) * 8); add(static_cast<size_t>(a.sa) * 8); add(static_cast<size_t>(nwords) * 4);
  add(static_cast<size_t>(nwords) * 4); add(static_cast<size_t>(a.sa) * 4); add(static_cast<size_t>(D) * 4);
  add(static_cast<size_t>(LW) * D * 4); add(static_cast<size_t>(LW) * D * 4);
  if (smem > 225 * 1024) return 1;
  auto kern = a.L.b % 32 == 0 ? light_kernel<T, DPH, true, LW> : light_kernel<T, DPH, false, LW>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  return launch_pdl(kern, dim3(static_cast<unsigned>(a.rows)), dim3(LW * 32), smem, stream, 0, a);
}

// A row's CTA takes kLW warps and kLW stages; a batch of rows at least
// twice the SM count (batched requests) takes half as many per row, so that
// three rows' CTAs share an SM and their latencies overlap.
static int current_sm_count() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    v = 0;
  return v > 0 ? v : 148;
}

template <typename T, int DPH>
static int launch_light_t(const RepairArgs& a, cudaStream_t stream) {
  if (a.rows >= 2 * current_sm_count()) return launch_light_lw<T, DPH, kLW / 2>(a, stream);
  return launch_light_lw<T, DPH, kLW>(a, stream);
}

// ------------------------------------------------------------------ host side

template <typename T, int DPH>
static int launch_attend_t(RepairArgs a, cudaStream_t stream) {
  const int jobs = a.sa;
  int cs = (jobs + kAW - 1) / kAW;
  if (cs > kAttendCluster) cs = kAttendCluster;
  if (cs < 1) cs = 1;
  a.cluster = cs;
  const size_t smem = attend_layout<DPH, T>(a, cs, nullptr, nullptr);
  if (smem > 220 * 1024) return -2;
  auto kern = a.L.b % 32 == 0 ? attend_kernel<T, DPH, true> : attend_kernel<T, DPH, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  return launch_pdl(kern, dim3(static_cast<unsigned>(a.rows) * cs), dim3(kAW * 32), smem, stream, cs, a);
}

// Returns 1 when the fast attend kernel does not apply (the caller then uses
// the general repair kernel), else the launch status.
int launch_attend(const RepairArgs& a, int kv_dtype, cudaStream_t stream) {
  const bool plain = a.pmode == kPredNone || (a.pmode == kPredSaved && (a.variant == kVarSaved || a.variant == kVarUnion));
  if (!plain || a.rows == 0) return 1;
  if (a.pmode == kPredSaved && a.sc != a.sp) return 1;
  const int esz = kv_dtype == kF32 ? 4 : 2;
  const uintptr_t pk = reinterpret_cast<uintptr_t>(a.L.k) | reinterpret_cast<uintptr_t>(a.L.v);
  const bool aligned = (pk & 15) == 0 && (a.d * esz) % 16 == 0 &&
                       (a.L.page_table == nullptr || a.L.b % a.L.page_size == 0) && a.L.kv_request_stride % 8 == 0;
  if (!aligned || (a.d != 64 && a.d != 128)) return 1;
  // Saved / union with a prediction: the one-CTA-per-row form when its stages
  // and the row's staged prediction states fit in shared memory.
  if (a.pmode == kPredSaved && kv_dtype != kF32 && (reinterpret_cast<uintptr_t>(a.pu) & 15) == 0) {
    const int rc = kv_dtype == kF16 ? (a.d == 64 ? launch_light_t<__half, 4>(a, stream) : launch_light_t<__half, 8>(a, stream))
                                    : (a.d == 64 ? launch_light_t<__nv_bfloat16, 4>(a, stream)
                                                 : launch_light_t<__nv_bfloat16, 8>(a, stream));
    if (rc != 1) return rc;
  }
  switch (kv_dtype) {
    case kF32: return a.d == 64 ? launch_attend_t<float, 4>(a, stream) : launch_attend_t<float, 8>(a, stream);
    case kF16: return a.d == 64 ? launch_attend_t<__half, 4>(a, stream) : launch_attend_t<__half, 8>(a, stream);
    default: return a.d == 64 ? launch_attend_t<__nv_bfloat16, 4>(a, stream) : launch_attend_t<__nv_bfloat16, 8>(a, stream);
  }
}

int set_wait_limit_attend(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
