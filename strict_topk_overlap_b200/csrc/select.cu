// K1: min/max query-sign-bound block scoring and strict Top-K selection.
//
// Replaces selector.py:8-20 (_score), gqa.py:15-26 (_bound_score) and the
// torch.topk call of selector.py:43 / gqa.py:161.
//
// Score definition (fixed, documented order so that IDs are bit-exact with
// the CPU oracle): for query row h and block n with metadata row b = (lo|hi)
// chosen per dimension by the sign of q (q >= 0 -> hi),
//     lane l (0..31) owns dims [l*c, min((l+1)*c, D)), c = ceil(D / 32);
//     part_l = (((0 + q_d0*b_d0) + q_d1*b_d1) + ...) over its dims, in FP64;
//     score  = xor-butterfly sum of part_l over lanes with offsets 16,8,4,2,1.
// Every product of an f32/f16/bf16 q with an f32 bound is exact in FP64, so
// the only roundings are the additions above, in that order.
//
// Group ("shared") selection scores a KV head by the FP64 sum, in ascending
// query-head order, of its query heads' scores.
//
// Scoring is HBM-bound on the metadata stream: each CTA pulls one tile of
// lo/hi rows (one meta head, tn consecutive blocks) into shared memory with
// two 1-D bulk copies, so every CTA's whole tile is in flight at once, then
// reduces from shared memory.
//
// Top-K: per selection row, the K largest scores, ties to the lower block
// index, written in ascending block-ID order. Radix select over 64-bit
// order-preserving keys held in registers (8-bit digits, leading common bits
// skipped, two barriers per digit), then one packed block scan that places
// every selected ID at its ascending-order position.

#ifdef STK_TRACE
// [cta][8] timeline of the Top-K kernels (profiling builds only): 0 start,
// 1..5 the bounded core's phase probes, 6 after the dependency wait, 7 end.
namespace stk {
static __device__ unsigned long long g_topk_trace[4096 * 8];
}
#define STK_TOPK_PROBE(ev) \
  do { if (blockIdx.x < 4096 && threadIdx.x == 0) stk::g_topk_trace[blockIdx.x * 8 + 1 + (ev)] = stk::global_ns(); } while (0)
#endif
#include "topk.cuh"

namespace stk {

#ifdef STK_TRACE
extern "C" __attribute__((visibility("default"))) void* stk_trace_topk() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_topk_trace);
  return p;
}
#define KT(ev) do { if (blockIdx.x < 4096 && threadIdx.x == 0) STK_TRACE_AT(g_topk_trace, blockIdx.x * 8 + (ev)); } while (0)
static __device__ unsigned long long g_score_trace[4096 * 4];
extern "C" __attribute__((visibility("default"))) void* stk_trace_score() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, g_score_trace);
  return p;
}
#define ST(ev) do { unsigned _b = blockIdx.y * gridDim.x + blockIdx.x; if (_b < 4096 && threadIdx.x == 0) STK_TRACE_AT(g_score_trace, _b * 4 + (ev)); } while (0)
#else
#define KT(ev) ((void)0)
#define ST(ev) ((void)0)
#endif

__device__ __forceinline__ int find_request(const int* offs, int R, int gb) {
  if (offs == nullptr) return 0;
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (offs[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  return lo;
}

constexpr int kScoreThreads = 128;
constexpr int kQReq = 2;  // requests whose q rows are staged per tile

struct ScoreTile {
  int tn;        // rows per tile
  int bulk;      // lo/hi rows are 16-byte multiples and aligned
};

template <int C>
__global__ void __launch_bounds__(kScoreThreads) score_generic_kernel(ScoreArgs a, ScoreTile t) {
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ uint64_t bar;
  __shared__ int req0;
  const int G = a.hq / a.hmeta;
  const int D = a.d;
  const int tn = t.tn;
  const int mh = blockIdx.y;
  const int row0 = blockIdx.x * tn;
  const int nrows = min(tn, a.total_blocks - row0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  float* slo = reinterpret_cast<float*>(sm);
  float* shi = slo + static_cast<size_t>(tn) * D;
  double* sq = reinterpret_cast<double*>(shi + static_cast<size_t>(tn) * D);  // [kQReq][G][D]
  double* s64 = sq + static_cast<size_t>(kQReq) * G * D;                        // [tn * G]
  int* srr = reinterpret_cast<int*>(s64 + static_cast<size_t>(tn) * G);          // [tn]
  const long long moff = (static_cast<long long>(mh) * a.total_blocks + row0) * D;

  if (tid == 0) {
    req0 = find_request(a.block_offsets, a.R, row0);
    if (t.bulk) {
      mbar_init(&bar, 1);
      fence_barrier_init();
      const unsigned bytes = static_cast<unsigned>(nrows) * D * 4;
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_g2s(slo, a.lo + moff, bytes, &bar);
      bulk_g2s(shi, a.hi + moff, bytes, &bar);
    }
  }
  __syncthreads();
  if (!t.bulk) {
    for (int i = tid; i < nrows * D; i += blockDim.x) {
      slo[i] = a.lo[moff + i];
      shi[i] = a.hi[moff + i];
    }
  }
  const int r0 = req0;
  for (int i = tid; i < kQReq * G * D; i += blockDim.x) {
    const int rr = i / (G * D), rem = i - rr * G * D;
    const int g = rem / D, dd = rem - g * D;
    const int r = r0 + rr;
    sq[i] = r < a.R ? static_cast<double>(load_any(a.q, a.q_dtype, (static_cast<long long>(r) * a.hq + mh * G + g) * D + dd))
                    : 0.0;
  }
  if (t.bulk && !mbar_wait(&bar, 0, a.status)) return;
  __syncthreads();

  // Per-row request index relative to r0 (tiles rarely span requests).
  for (int rl = tid; rl < nrows; rl += blockDim.x) srr[rl] = find_request(a.block_offsets, a.R, row0 + rl) - r0;
  __syncthreads();

  // Each warp takes a contiguous run of (row, head) pairs; lanes own dims.
  // Lane partial: FP64 FMA chain over its dims (each product is exact, so
  // fma(q, b, acc) rounds exactly like acc + q*b); then the xor butterfly.
  const int pairs = nrows * G;
  const int c = (D + 31) / 32;
  const int per_warp = (pairs + nwarps - 1) / nwarps;
  const int p_beg = warp * per_warp, p_end = min(pairs, p_beg + per_warp);
  int rloc = p_beg / G, g = p_beg - rloc * G;
#pragma unroll 4
  for (int pair = p_beg; pair < p_end; ++pair) {
    const float* lr = slo + rloc * D;
    const float* hr = shi + rloc * D;
    const int rr = srr[rloc];
    double acc = 0.0;
    if (rr < kQReq) {
      const double* qr = sq + (rr * G + g) * D;
      if constexpr (C == 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(lr + lane * 4);
        const float4 h4 = *reinterpret_cast<const float4*>(hr + lane * 4);
        const double2 q01 = *reinterpret_cast<const double2*>(qr + lane * 4);
        const double2 q23 = *reinterpret_cast<const double2*>(qr + lane * 4 + 2);
        acc = __fma_rn(q01.x, static_cast<double>(q01.x >= 0.0 ? h4.x : l4.x), acc);
        acc = __fma_rn(q01.y, static_cast<double>(q01.y >= 0.0 ? h4.y : l4.y), acc);
        acc = __fma_rn(q23.x, static_cast<double>(q23.x >= 0.0 ? h4.z : l4.z), acc);
        acc = __fma_rn(q23.y, static_cast<double>(q23.y >= 0.0 ? h4.w : l4.w), acc);
      } else {
        for (int dd = lane * c; dd < min((lane + 1) * c, D); ++dd) {
          const double qv = qr[dd];
          acc = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? hr[dd] : lr[dd]), acc);
        }
      }
    } else {
      // Tile spans more requests than are staged: read q from global memory.
      const long long qoff = (static_cast<long long>(r0 + rr) * a.hq + mh * G + g) * D;
      for (int dd = lane * c; dd < min((lane + 1) * c, D); ++dd) {
        const double qv = static_cast<double>(load_any(a.q, a.q_dtype, qoff + dd));
        acc = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? hr[dd] : lr[dd]), acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
    if (lane == 0) s64[pair] = acc;
    if (++g == G) { g = 0; ++rloc; }
  }
  __syncthreads();

  for (int pair = tid; pair < pairs; pair += blockDim.x) {
    const int rl = pair / G, g = pair - rl * G;
    const int gb = row0 + rl;
    const int h = mh * G + g;
    const double s = s64[pair];
    if (a.scores_f32) a.scores_f32[static_cast<long long>(h) * a.total_blocks + gb] = __double2float_rn(s);
    if (a.scores_f64 && !a.group_select) a.scores_f64[static_cast<long long>(h) * a.total_blocks + gb] = s;
  }
  if (a.scores_f64 && a.group_select) {
    for (int rl = tid; rl < nrows; rl += blockDim.x) {
      double acc = 0.0;
      for (int g = 0; g < G; ++g) acc = __dadd_rn(acc, s64[rl * G + g]);
      a.scores_f64[static_cast<long long>(mh) * a.total_blocks + row0 + rl] = acc;
    }
  }
}


// ------------------------------------------------------------------ tiled scorer
// The fast scorer for D = 32 * C (C = 2, 4, 8). One CTA scores kTileBlocks
// consecutive blocks of one meta head for all G query heads of that head.
// Each warp owns 8 blocks; lane = part * 8 + b (part 0..3, b = block in warp).
//
// Bit-exact restatement of the fixed order above: write p[c] for the lane-c
// partial of the reference order (dims [cC, cC+C), sequential FP64 FMA). The
// xor butterfly over offsets 16, 8, 4, 2, 1 is, from any lane's point of
// view, the balanced binary tree over the leaves L_k = p[bitrev5(k)] taken in
// order k = 0..31 (the pair at offset 16 is (L_2i, L_2i+1), at offset 8 the
// pairs of those, ...); FP64 addition is commutative, so every lane ends with
// the same value and so does this tree. Part j here reduces the subtree of
// leaves k in [8j, 8j+8) with a 3-level stack, and two shuffle levels (xor 8:
// parts 0+1, 2+3; xor 16: the halves) finish it.
//
// lo/hi rows are staged with one 1-D bulk copy per row into rows padded to
// D + 4 floats, so the 8 lanes of a shared-memory phase (same part, 8
// blocks) hit 8 different bank quads; q rows are FP64 in shared memory and
// read as broadcasts.

constexpr int kTileWarps = 4;
constexpr int kTileBlocks = 8 * kTileWarps;
constexpr int kTileRowGroup = 4;  // query heads reduced together per lo/hi chunk load

__device__ __forceinline__ int bitrev5(int k) { return static_cast<int>(__brev(static_cast<unsigned>(k)) >> 27); }

// Leaf value for a row whose request's q is not staged (tiles that span more
// than kQReq requests, i.e. requests shorter than a tile): q from global
// memory. Kept out of line so that the hot loop stays small.
template <int C>
__device__ __noinline__ double leaf_global_q(const ScoreArgs& a, long long qoff, const float* lo_c, const float* hi_c) {
  double v = 0.0;
  for (int e = 0; e < C; ++e) {
    const double qv = static_cast<double>(load_any(a.q, a.q_dtype, qoff + e));
    v = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? hi_c[e] : lo_c[e]), v);
  }
  return v;
}

template <int C, bool G4>
__global__ void __launch_bounds__(kTileWarps * 32) score_tiled_kernel(ScoreArgs a, int bulk) {
  constexpr int D = 32 * C;
  constexpr int RS = D + 4;  // padded row stride (floats)
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ uint64_t bar;
  __shared__ int req0;
  const int G = a.hq / a.hmeta;
  const int mh = blockIdx.y;
  const int row0 = blockIdx.x * kTileBlocks;
  const int nrows = min(kTileBlocks, a.total_blocks - row0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* slo = reinterpret_cast<float*>(sm);
  float* shi = slo + kTileBlocks * RS;
  // q split by sign: qp = q where q >= 0 (else +0), qn = q where q < 0 (else +0),
  // as FP64 rows [kQReq][G][D] each.
  double* qp = reinterpret_cast<double*>(shi + kTileBlocks * RS);
  double* qn = qp + static_cast<size_t>(kQReq) * G * D;
  const long long moff = (static_cast<long long>(mh) * a.total_blocks + row0) * D;
  ST(0);
  pdl_release();  // the Top-K kernel may launch now; it waits for this grid to finish

  // q first: a load issued behind the tile's bulk copies would wait for them.
  const int r0 = find_request(a.block_offsets, a.R, row0);
  constexpr int kQPer = 8;  // q elements per thread per pass
  for (int i0 = 0; i0 < kQReq * G * D; i0 += kQPer * static_cast<int>(blockDim.x)) {
    float qv[kQPer];
#pragma unroll
    for (int e = 0; e < kQPer; ++e) {
      const int i = i0 + e * blockDim.x + tid;
      qv[e] = 0.f;
      if (i < kQReq * G * D) {
        const int rr = i / (G * D), rem = i - rr * G * D;
        if (r0 + rr < a.R) qv[e] = load_any(a.q, a.q_dtype, (static_cast<long long>(r0 + rr) * a.hq + mh * G) * D + rem);
      }
    }
    if (i0 == 0 && tid == 0) {
      req0 = r0;
      if (bulk) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, static_cast<unsigned>(2 * nrows * D * 4));
      }
    }
    if (i0 == 0) __syncthreads();
    if (i0 == 0 && bulk && warp == 0) {
      for (int rr = lane; rr < nrows; rr += 32) {
        bulk_g2s(slo + rr * RS, a.lo + moff + static_cast<long long>(rr) * D, D * 4, &bar);
        bulk_g2s(shi + rr * RS, a.hi + moff + static_cast<long long>(rr) * D, D * 4, &bar);
      }
    }
#pragma unroll
    for (int e = 0; e < kQPer; ++e) {
      const int i = i0 + e * blockDim.x + tid;
      if (i < kQReq * G * D) {
        // q >= 0 picks hi: -0.0 goes with the non-negative side, as in the reference.
        const bool pos = qv[e] >= 0.f;
        qp[i] = pos ? static_cast<double>(qv[e]) : 0.0;
        qn[i] = pos ? 0.0 : static_cast<double>(qv[e]);
      }
    }
  }
  if (!bulk) {
    for (int i = tid; i < nrows * D; i += blockDim.x) {
      const int rr = i / D, dd = i - rr * D;
      slo[rr * RS + dd] = a.lo[moff + i];
      shi[rr * RS + dd] = a.hi[moff + i];
    }
  }
  ST(1);
  if (bulk && !mbar_wait(&bar, 0, a.status)) return;
  __syncthreads();
  ST(2);

  const int part = lane >> 3, b = lane & 7;
  const int rl = warp * 8 + b;  // tile row of this lane
  const bool live = rl < nrows;
  const int gb = row0 + rl;
  const int rr = live ? find_request(a.block_offsets, a.R, gb) - req0 : 0;
  const float* lr = slo + rl * RS;
  const float* hr = shi + rl * RS;
  double grp = 0.0;

  // Per element: fma(qn, lo, fma(qp, hi, v)). One of qp / qn is zero, and
  // fma(0, x, t) == t for finite x, so this rounds exactly like
  // fma(q, q >= 0 ? hi : lo, v) without a select.
#pragma unroll 1
  for (int g0 = 0; g0 < G; g0 += kTileRowGroup) {
    const int ng = G4 ? kTileRowGroup : min(kTileRowGroup, G - g0);
    double st[kTileRowGroup][3];
    double leaf_done[kTileRowGroup];
#pragma unroll
    for (int kl = 0; kl < 8; ++kl) {
      const int c = bitrev5(part * 8 + kl);
      double lo_c[C], hi_c[C];
#pragma unroll
      for (int e = 0; e < C; e += (C >= 4 ? 4 : 2)) {
        if constexpr (C >= 4) {
          const float4 x = *reinterpret_cast<const float4*>(lr + c * C + e);
          const float4 y = *reinterpret_cast<const float4*>(hr + c * C + e);
          lo_c[e] = x.x; lo_c[e + 1] = x.y; lo_c[e + 2] = x.z; lo_c[e + 3] = x.w;
          hi_c[e] = y.x; hi_c[e + 1] = y.y; hi_c[e + 2] = y.z; hi_c[e + 3] = y.w;
        } else {
          const float2 x = *reinterpret_cast<const float2*>(lr + c * C + e);
          const float2 y = *reinterpret_cast<const float2*>(hr + c * C + e);
          lo_c[e] = x.x; lo_c[e + 1] = x.y;
          hi_c[e] = y.x; hi_c[e + 1] = y.y;
        }
      }
#pragma unroll
      for (int gi = 0; gi < kTileRowGroup; ++gi) {
        if (G4 || gi < ng) {
          double v = 0.0;
          if (rr < kQReq) {
            const int qo = (rr * G + g0 + gi) * D + c * C;
#pragma unroll
            for (int e = 0; e < C; ++e) v = __fma_rn(qn[qo + e], lo_c[e], __fma_rn(qp[qo + e], hi_c[e], v));
          } else {
            float lf[C], hf[C];
#pragma unroll
            for (int e = 0; e < C; ++e) { lf[e] = static_cast<float>(lo_c[e]); hf[e] = static_cast<float>(hi_c[e]); }
            v = leaf_global_q<C>(a, (static_cast<long long>(req0 + rr) * a.hq + mh * G + g0 + gi) * D + c * C, lf,
                                 hf);
          }
          // Balanced-tree push of leaf kl (levels resolved at compile time).
          if ((kl & 1) == 0) {
            st[gi][0] = v;
          } else {
            v = __dadd_rn(st[gi][0], v);
            if ((kl & 2) == 0) {
              st[gi][1] = v;
            } else {
              v = __dadd_rn(st[gi][1], v);
              if ((kl & 4) == 0) st[gi][2] = v;
              else leaf_done[gi] = __dadd_rn(st[gi][2], v);
            }
          }
        }
      }
    }
#pragma unroll
    for (int gi = 0; gi < kTileRowGroup; ++gi) {
      double v = (G4 || gi < ng) ? leaf_done[gi] : 0.0;
      v = __dadd_rn(v, __shfl_xor_sync(kFull, v, 8));
      v = __dadd_rn(v, __shfl_xor_sync(kFull, v, 16));
      if ((G4 || gi < ng) && part == 0 && live) {
        const int h = mh * G + g0 + gi;
        if (a.scores_f32) a.scores_f32[static_cast<long long>(h) * a.total_blocks + gb] = __double2float_rn(v);
        if (a.scores_f64 && !a.group_select) a.scores_f64[static_cast<long long>(h) * a.total_blocks + gb] = v;
        grp = __dadd_rn(grp, v);
      }
    }
  }
  if (a.scores_f64 && a.group_select && part == 0 && live)
    a.scores_f64[static_cast<long long>(mh) * a.total_blocks + gb] = grp;
  ST(3);
}


template <int E>
__global__ void __launch_bounds__(512) select_topk_kernel(SelectArgs a) {
  KT(0);
  pdl_release();
  pdl_wait();  // scores come from the preceding scoring kernel
  const int row = blockIdx.x;
  const int r = row / a.hsel, hs = row - r * a.hsel;
  const int off = a.block_offsets ? a.block_offsets[r] : 0;
  const int n = a.block_offsets ? a.block_offsets[r + 1] - off : a.n;
  if (n < a.topk || n > static_cast<int>(blockDim.x) * E) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  const double* src = a.scores + static_cast<long long>(hs) * a.total_blocks + off;
  unsigned long long key[E];
  const int beg = threadIdx.x * E;
#pragma unroll
  for (int j = 0; j < E; ++j) key[j] = beg + j < n ? order_key(src[beg + j]) : 0ull;
  KT(1);
  const int base = a.id_base;
  select_registers<E>(key, n, a.topk, [base](int i) { return base + i; },
                      a.ids_out + static_cast<long long>(row) * a.topk,
                      a.keys_out ? a.keys_out + static_cast<long long>(row) * a.topk : nullptr);
  KT(2);
}

// Candidate merge (context-parallel and segmented selection): each row has
// `ncand` (key, id) candidates gathered from several shards in ascending-ID
// order (each shard's list is ascending and shards own increasing ID
// ranges), so position order equals ID order and the same selection resolves
// ties toward the lower ID.
template <int E>
__global__ void __launch_bounds__(512) merge_candidates_kernel(MergeArgs a) {
  const int row = blockIdx.x;
  const int n = a.ncand;
  if (n < a.topk || n > static_cast<int>(blockDim.x) * E) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  const unsigned long long* ksrc = a.keys + static_cast<long long>(row) * n;
  const int* isrc = a.ids + static_cast<long long>(row) * n;
  unsigned long long key[E];
  const int beg = threadIdx.x * E;
#pragma unroll
  for (int j = 0; j < E; ++j) key[j] = beg + j < n ? ksrc[beg + j] : 0ull;
  select_registers<E>(key, n, a.topk, [isrc](int i) { return isrc[i]; },
                      a.ids_out + static_cast<long long>(row) * a.topk, nullptr);
}

// ------------------------------------------------------------------ two-stage selection
// Stage 1, the interval scorer: the FP32 score s of every (row, block) with
// the same q-sign bound, and a rigorous radius e, written as the interval
// [s - e, s + e] rounded outward. The exact FP64 fixed-order score lies in
// it. Each lane sums D/4 dims with FP32 FMA (exact products, one rounding per
// step) and two shuffle levels finish the sum, so every term passes through
// at most D/4 + 2 roundings and |s - S| <= gamma_{D/4+2} * sum_d |q_d b_d|
// (recursive-summation bound, Higham, "Accuracy and Stability of Numerical
// Algorithms", 2nd ed., eq. 4.4; gamma_k = k u / (1 - k u), u = 2^-24), and
// sum_d |q_d b_d| <= ||q||_1 * max_d max(|lo_d|, |hi_d|), with ||q||_1 summed
// under upward rounding. The radius takes 2 (D/4 + 2) u, which also covers
// the FP64 score's own roundings (relative 2^-53 each) and, for group
// selection, the FP64 sum over the group; an absolute 2^-118 covers
// underflow. Non-finite inputs give the interval (-inf, +inf). A CTA's
// metadata (32 consecutive rows of one head: two contiguous ranges of lo and
// hi) lands in shared memory through two bulk copies on one mbarrier, so the
// whole tile is one DRAM request per array instead of 16 register loads per
// lane.
//
// Stage 2, per selection row: with T the K-th largest lower end and U the
// (K+1)-th largest upper end, a block whose upper end is below T is beaten
// by K blocks (out); a block whose lower end is above U can be beaten, or
// tied from a lower index, only by blocks whose upper end exceeds U — at most
// K of them, itself included — so it is in. Only the remaining blocks, whose
// intervals straddle the boundary (typically none to a few per row), get
// their exact FP64 score, recomputed in the fixed order above from q and
// lo/hi, and the best K - #in of them by (score, lower index) complete the
// selection: the result is the strict Top-K of the FP64 scores. T and U are
// located in 2048-bin histograms of a monotone map of the interval ends over
// the row's range; comparing bins instead of values keeps both tests
// conservative, so no radix passes over 64-bit keys are needed.

constexpr int kBWarps = 4;
constexpr int kBTile = kBWarps * 8;  // blocks per CTA: 8 per warp, 4 lanes per block

// Per-lane FP32 sum of query head mh * G + g (and the lane's largest
// metadata magnitude) for lanes whose request's q is not staged (tiles that
// span more than kQReq requests): q and metadata from global memory.
template <int C>
__device__ __forceinline__ float2 bound_lane_global(const ScoreArgs& a, int r, int mh, int G, int g, long long gb,
                                                 int p) {
  constexpr int D = 32 * C;
  const float* lr = a.lo + (static_cast<long long>(mh) * a.total_blocks + gb) * D;
  const float* hr = a.hi + (static_cast<long long>(mh) * a.total_blocks + gb) * D;
  const long long qoff = (static_cast<long long>(r) * a.hq + mh * G + g) * D;
  float m = 0.f, s = 0.f;
  for (int i = 0; i < D / 16; ++i) {
    for (int e = 0; e < 4; ++e) {
      const int dd = 4 * (p + 4 * i) + e;
      const float l = lr[dd], h = hr[dd];
      m = fmaxf(m, fmaxf(fabsf(l), fabsf(h)));
      const float qv = load_any(a.q, a.q_dtype, qoff + dd);
      s = fmaf(qv, qv >= 0.f ? h : l, s);
    }
  }
  return make_float2(s, m);
}

template <int C, int GM>
__global__ void __launch_bounds__(kBWarps * 32) bound_interval_kernel(ScoreArgs a, float2* __restrict__ out) {
  constexpr int D = 32 * C;
  constexpr int NI = D / 16;           // 16-byte chunks per lane per metadata row
  constexpr int NBAT = NI < 8 ? NI : 8;  // chunks in flight per batch
  constexpr float kErrFactor = 2.f * (D / 4 + 2) * 0x1p-24f;
  extern __shared__ __align__(16) float qs[];  // [kQReq][G][D] q as float, then [kQReq][G] ||q||_1
  const int G = a.hq / a.hmeta;
  const int mh = blockIdx.y;
  const int row0 = blockIdx.x * kBTile;
  const int nrows = min(kBTile, a.total_blocks - row0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = kQReq * G * D;
  float* qn1 = qs + nq;
  // Group selection: per staged request the group's Q+ and Q- rows
  // ([kQReq][2][D]) and its ||q||_1 (4 floats reserved).
  float* qsum = qs + ((nq + kQReq * G + 3) & ~3);
  float* qng = qsum + kQReq * 2 * D;
  // The tile's metadata rows, [kBTile][D] lo then hi: two contiguous ranges
  // of the metadata, each brought in by one bulk copy.
  float* slo = qng + 4;
  float* shi = slo + kBTile * D;
  __shared__ uint64_t meta_bar;
  ST(0);
  pdl_release();  // the Top-K kernel may launch now; it waits for this grid to finish
  if (threadIdx.x == 0) {
    mbar_init(&meta_bar, 1);
    fence_barrier_init();
    const unsigned bytes = static_cast<unsigned>(nrows * D * sizeof(float));
    const long long moff = (static_cast<long long>(mh) * a.total_blocks + row0) * D;
    mbar_arrive_expect_tx(&meta_bar, 2 * bytes);
    bulk_g2s(slo, a.lo + moff, bytes, &meta_bar);
    bulk_g2s(shi, a.hi + moff, bytes, &meta_bar);
  }

  // q first: loads issued behind the metadata stream would wait for it. The
  // staged requests' rows of this meta head are G * D consecutive elements
  // each; they are read in 8-element chunks (16-byte loads for 16-bit q),
  // two chunks in flight per thread, and rows of absent requests are zero.
  const int r0 = find_request(a.block_offsets, a.R, row0);
  {
    const int nreq = max(0, min(kQReq, a.R - r0));
    const int chunks = G * D / 8;
    const bool vec = (reinterpret_cast<uintptr_t>(a.q) & 15) == 0;
    for (int i = nreq * G * D + tid; i < nq; i += blockDim.x) qs[i] = 0.f;
    for (int c0 = 0; c0 < nreq * chunks; c0 += 2 * blockDim.x) {
      float x[2][8];
      int dst[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = c0 + u * blockDim.x + tid;
        dst[u] = -1;
        if (c < nreq * chunks) {
          const int rr = c / chunks, cc = c - rr * chunks;
          const long long src = (static_cast<long long>(r0 + rr) * a.hq + mh * G) * D + cc * 8;
          dst[u] = rr * G * D + cc * 8;
          if (vec && a.q_dtype == kF32) {
            load_vec<float, 8>(static_cast<const float*>(a.q) + src, x[u]);
          } else if (vec && a.q_dtype == kBF16) {
            load_vec<__nv_bfloat16, 8>(static_cast<const __nv_bfloat16*>(a.q) + src, x[u]);
          } else if (vec && a.q_dtype == kF16) {
            load_vec<__half, 8>(static_cast<const __half*>(a.q) + src, x[u]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[u][e] = load_any(a.q, a.q_dtype, src + e);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (dst[u] >= 0) {
          float4* d4 = reinterpret_cast<float4*>(qs + dst[u]);
          d4[0] = make_float4(x[u][0], x[u][1], x[u][2], x[u][3]);
          d4[1] = make_float4(x[u][4], x[u][5], x[u][6], x[u][7]);
        }
      }
    }
  }
#ifdef STK_QFIRST
  __syncthreads();  // every warp's q loads are issued before any metadata load
#endif
  // This lane's block (b) and quarter (p): chunks p, p + 4, p + 8, ... of the row.
  const int b = lane >> 2, p = lane & 3;
  const int rl = warp * 8 + b;
  const bool live = rl < nrows;
  const long long gb = row0 + (live ? rl : 0);
  const float4* L4 = reinterpret_cast<const float4*>(slo + (live ? rl : 0) * D);
  const float4* H4 = reinterpret_cast<const float4*>(shi + (live ? rl : 0) * D);
  float4 lv[NBAT], hv[NBAT];
  __syncthreads();
  // ||q||_1 per staged row, rounded up at every step.
  for (int t = warp; t < kQReq * G; t += kBWarps) {
    float sum = 0.f;
    for (int dd = lane; dd < D; dd += 32) sum = __fadd_ru(sum, fabsf(qs[t * D + dd]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_ru(sum, __shfl_xor_sync(kFull, sum, o));
    if (lane == 0) qn1[t] = sum;
  }
  __syncthreads();
  if (C == 4 && a.group_select) {
    // q . (q >= 0 ? hi : lo) = max(q, 0) hi + min(q, 0) lo, so the group's
    // score is one dot product of the metadata row with Q+ = sum_g max(q_g, 0)
    // and Q- = sum_g min(q_g, 0) (heads ascending, FP32). Its interval
    // radius is the per-head radii's sum: kErrFactor * sum_g ||q_g||_1 *
    // max|lo, hi|. Same-sign sums give |Q^ - Q| <= gamma_11 |Q| (G <= 12;
    // gamma_15 for G = 16), and each term of the dot passes 8 + 5 roundings,
    // so the FP32 score is within (gamma_13 (1 + gamma_15) + gamma_15) of
    // that bound's base: 28 u against the 2 (D/4 + 2) u = 68 u it takes.
    for (int i = tid; i < kQReq * D; i += blockDim.x) {
      const int rq = i / D, dd = i - rq * D;
      float qp = 0.f, qm = 0.f;
      for (int g = 0; g < G; ++g) {
        const float x = qs[(rq * G + g) * D + dd];
        qp += x > 0.f ? x : 0.f;
        qm += x < 0.f ? x : (x == x ? 0.f : x);  // a NaN q stays visible
      }
      qsum[(rq * 2) * D + dd] = qp;
      qsum[(rq * 2 + 1) * D + dd] = qm;
    }
    if (tid < kQReq) {
      float nsum = 0.f;
      for (int g = 0; g < G; ++g) nsum = __fadd_ru(nsum, qn1[tid * G + g]);
      qng[tid] = nsum;
    }
    __syncthreads();
  }
  ST(1);
  if (!mbar_wait(&meta_bar, 0, a.status)) return;  // bounded; the status records a wait that gave up

  const int rr = (live && a.block_offsets) ? find_request(a.block_offsets, a.R, static_cast<int>(gb)) - r0 : 0;
  if constexpr (C == 4) {
    // D = 128: lane l owns dims [4l, 4l + 4), so every warp-wide 128-bit
    // load reads one whole 512-byte metadata (or q) row, conflict-free. Per
    // group of 4 blocks and 4 heads each lane forms 16 partial sums (its 4
    // dims in order, FP32 FMA on the sign-selected bound); a transposed
    // butterfly (xor 8, 4, 2, 1) and one xor-16 add leave the total of
    // (block j, head g) in lanes 4 j + g and 16 + 4 j + g. Every term passes
    // through at most 4 + 5 roundings, within the D/4 + 2 the radius covers.
    // Lane b * 4 + p of the lane layout below held block b of the warp; its
    // request index rr is read from lane 4 b.
    if (__all_sync(kFull, !live || rr < kQReq)) {
      const float4* slo4 = reinterpret_cast<const float4*>(slo);
      const float4* shi4 = reinterpret_cast<const float4*>(shi);
      const float4* qs4 = reinterpret_cast<const float4*>(qs);
      const float inf = __int_as_float(0x7f800000);
      if (a.group_select) {
        // The warp's 8 blocks at once: 8 partial dots per lane, a transposed
        // butterfly (xor 16, 8, 4) and xor 2, 1 leave block j's score in
        // lanes 4 j .. 4 j + 3; the largest |lo|, |hi| likewise.
        const float4* qs4g = reinterpret_cast<const float4*>(qsum);
        float part[8], mx[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int rl2 = warp * 8 + j;
          const bool lj = rl2 < nrows;
          const int rrj = __shfl_sync(kFull, rr, 4 * j);
          const float4 l4 = lj ? slo4[rl2 * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 h4 = lj ? shi4[rl2 * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 qp = qs4g[(rrj * 2) * 32 + lane];
          const float4 qm = qs4g[(rrj * 2 + 1) * 32 + lane];
          float acc = qp.x * h4.x;
          acc = fmaf(qp.y, h4.y, acc);
          acc = fmaf(qp.z, h4.z, acc);
          acc = fmaf(qp.w, h4.w, acc);
          acc = fmaf(qm.x, l4.x, acc);
          acc = fmaf(qm.y, l4.y, acc);
          acc = fmaf(qm.z, l4.z, acc);
          acc = fmaf(qm.w, l4.w, acc);
          part[j] = acc;
          mx[j] = fmaxf(fmaxf(fmaxf(fabsf(l4.x), fabsf(h4.x)), fmaxf(fabsf(l4.y), fabsf(h4.y))),
                        fmaxf(fmaxf(fabsf(l4.z), fabsf(h4.z)), fmaxf(fabsf(l4.w), fabsf(h4.w))));
        }
#pragma unroll
        for (int off = 16, cnt = 4; off >= 4; off >>= 1, cnt >>= 1) {
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int i = 0; i < cnt; ++i) {
            const float send = upper ? part[i] : part[i + cnt];
            const float keep = upper ? part[i + cnt] : part[i];
            part[i] = keep + __shfl_xor_sync(kFull, send, off);
            const float msend = upper ? mx[i] : mx[i + cnt];
            const float mkeep = upper ? mx[i + cnt] : mx[i];
            mx[i] = fmaxf(mkeep, __shfl_xor_sync(kFull, msend, off));
          }
        }
        float sum = part[0], bm = mx[0];
        sum += __shfl_xor_sync(kFull, sum, 2);
        sum += __shfl_xor_sync(kFull, sum, 1);
        bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 2));
        bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 1));
        const int j = lane >> 2;
        const int rl2 = warp * 8 + j;
        const int rrj = __shfl_sync(kFull, rr, 4 * j);
        if ((lane & 3) == 0 && rl2 < nrows) {
          const float e = __fadd_ru(__fmul_ru(__fmul_ru(qng[rrj], bm), kErrFactor), 0x1p-118f);
          float2 iv = make_float2(__fsub_rd(sum, e), __fadd_ru(sum, e));
          if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
          out[static_cast<long long>(mh) * a.total_blocks + row0 + rl2] = iv;
        }
        ST(3);
        return;
      }
#pragma unroll 1
      for (int grp = 0; grp < 2; ++grp) {
        const int bb = warp * 8 + grp * 4;  // tile-local first block of the group
        float gl = 0.f, gu = 0.f;           // group selection: lanes 4 j accumulate block j
#pragma unroll 1
        for (int g0 = 0; g0 < G; g0 += 4) {
          float part[16];
          float mx[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int rl2 = bb + j;
            const bool lj = rl2 < nrows;
            const int rrj = __shfl_sync(kFull, rr, 4 * (grp * 4 + j));
            const float4 l4 = lj ? slo4[rl2 * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 h4 = lj ? shi4[rl2 * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
            mx[j] = fmaxf(fmaxf(fmaxf(fabsf(l4.x), fabsf(h4.x)), fmaxf(fabsf(l4.y), fabsf(h4.y))),
                          fmaxf(fmaxf(fabsf(l4.z), fabsf(h4.z)), fmaxf(fabsf(l4.w), fabsf(h4.w))));
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const float4 q = (lj && g0 + g < G) ? qs4[(rrj * G + g0 + g) * 32 + lane]
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
              float acc = q.x * (q.x >= 0.f ? h4.x : l4.x);
              acc = fmaf(q.y, q.y >= 0.f ? h4.y : l4.y, acc);
              acc = fmaf(q.z, q.z >= 0.f ? h4.z : l4.z, acc);
              acc = fmaf(q.w, q.w >= 0.f ? h4.w : l4.w, acc);
              part[4 * j + g] = acc;
            }
          }
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
          const int j = (lane >> 2) & 3, g = lane & 3, head = g0 + g;
          const int rl2 = bb + j;
          const bool lj = rl2 < nrows && head < G;
          const int rrj = __shfl_sync(kFull, rr, 4 * (grp * 4 + j));
          float lo = 0.f, up = 0.f;
          if (lj) {
            const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn1[rrj * G + head], bm), kErrFactor), 0x1p-118f);
            lo = __fsub_rd(sum, e);
            up = __fadd_ru(sum, e);
            if (!(lo <= up)) { lo = -inf; up = inf; }
          }
          if (!a.group_select) {
            if (lane < 16 && lj)
              out[static_cast<long long>(mh * G + head) * a.total_blocks + row0 + rl2] = make_float2(lo, up);
          } else {
            // The group's sum: heads of the chunk (lanes 4 j .. 4 j + 3), then
            // chunk after chunk, rounded outward at every step.
            lo = __fadd_rd(lo, __shfl_xor_sync(kFull, lo, 1));
            up = __fadd_ru(up, __shfl_xor_sync(kFull, up, 1));
            lo = __fadd_rd(lo, __shfl_xor_sync(kFull, lo, 2));
            up = __fadd_ru(up, __shfl_xor_sync(kFull, up, 2));
            gl = __fadd_rd(gl, lo);
            gu = __fadd_ru(gu, up);
          }
        }
        if (a.group_select && lane < 16 && (lane & 3) == 0 && bb + (lane >> 2) < nrows) {
          float2 iv = make_float2(gl, gu);
          if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
          out[static_cast<long long>(mh) * a.total_blocks + row0 + bb + (lane >> 2)] = iv;
        }
      }
      ST(3);
      return;
    }
  }
  float s[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) s[g] = 0.f;
  float mabs = 0.f;
  const bool staged = rr < kQReq;
  if (__all_sync(kFull, staged)) {
    const float* qrow = qs + rr * G * D;
#pragma unroll
    for (int bat = 0; bat < NI / NBAT; ++bat) {
#pragma unroll
      for (int i = 0; i < NBAT; ++i) {
        lv[i] = live ? L4[p + 4 * (bat * NBAT + i)] : make_float4(0.f, 0.f, 0.f, 0.f);
        hv[i] = live ? H4[p + 4 * (bat * NBAT + i)] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < NBAT; ++i) {
        const float4 l = lv[i], h = hv[i];
        mabs = fmaxf(mabs, fmaxf(fmaxf(fabsf(l.x), fabsf(h.x)), fmaxf(fabsf(l.y), fabsf(h.y))));
        mabs = fmaxf(mabs, fmaxf(fmaxf(fabsf(l.z), fabsf(h.z)), fmaxf(fabsf(l.w), fabsf(h.w))));
        const int off = 4 * (p + 4 * (bat * NBAT + i));
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g < G) {
            const float4 qq = *reinterpret_cast<const float4*>(qrow + g * D + off);
            s[g] = fmaf(qq.x, qq.x >= 0.f ? h.x : l.x, s[g]);
            s[g] = fmaf(qq.y, qq.y >= 0.f ? h.y : l.y, s[g]);
            s[g] = fmaf(qq.z, qq.z >= 0.f ? h.z : l.z, s[g]);
            s[g] = fmaf(qq.w, qq.w >= 0.f ? h.w : l.w, s[g]);
          }
        }
      }
    }
  } else if (live) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float2 sm = bound_lane_global<C>(a, r0 + rr, mh, G, g, gb, p);
        s[g] = sm.x;
        mabs = sm.y;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    s[g] += __shfl_xor_sync(kFull, s[g], 1);
    s[g] += __shfl_xor_sync(kFull, s[g], 2);
  }
  mabs = fmaxf(mabs, __shfl_xor_sync(kFull, mabs, 1));
  mabs = fmaxf(mabs, __shfl_xor_sync(kFull, mabs, 2));
  ST(2);
  if (!live) return;
  const float inf = __int_as_float(0x7f800000);
  if (!a.group_select) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G && (g & 3) == p) {
        const float qn = staged ? qn1[rr * G + g] : inf;
        const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn, mabs), kErrFactor), 0x1p-118f);
        float2 iv = make_float2(__fsub_rd(s[g], e), __fadd_ru(s[g], e));
        if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
        out[static_cast<long long>(mh * G + g) * a.total_blocks + gb] = iv;
      }
    }
  } else if (p == 0) {
    float gl = 0.f, gu = 0.f;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float qn = staged ? qn1[rr * G + g] : inf;
        const float e = __fadd_ru(__fmul_ru(__fmul_ru(qn, mabs), kErrFactor), 0x1p-118f);
        gl = __fadd_rd(gl, __fsub_rd(s[g], e));
        gu = __fadd_ru(gu, __fadd_ru(s[g], e));
      }
    }
    float2 iv = make_float2(gl, gu);
    if (!(iv.x <= iv.y)) iv = make_float2(-inf, inf);
    out[static_cast<long long>(mh) * a.total_blocks + gb] = iv;
  }
  ST(3);
}

template <int E, int NT>
__global__ void __launch_bounds__(NT, 1) select_bounded_kernel(SelectArgs a) {
  __shared__ __align__(16) float qsm[kQStage];  // the row's query heads, FP32, for exact rescoring
  extern __shared__ float2 sel_stage[];          // the row's intervals (n + n / 16 slots)
  KT(0);
  pdl_release();
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int r = row / a.hsel, hs = row - r * a.hsel;
  const int off = a.block_offsets ? a.block_offsets[r] : 0;
  const int n = a.block_offsets ? a.block_offsets[r + 1] - off : a.n;
  if (n < a.topk || n > NT * E) {
    pdl_wait();
    if (tid == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  const int G = a.hq / a.hmeta;
  const int q_heads = a.group_select ? G : 1;
  const bool q_staged = q_heads * a.d <= kQStage;
  if (q_staged) {
    // q is an input, not the scorer's output: staged before the wait.
    const long long q0 = (static_cast<long long>(r) * a.hq + (a.group_select ? hs * G : hs)) * a.d;
    for (int i = tid; i < q_heads * a.d; i += NT) qsm[i] = load_any(a.q, a.q_dtype, q0 + i);
  }
  pdl_wait();  // bounds come from the preceding interval scorer
  KT(6);
  bounded_select_core<E, NT>(a, row, qsm, q_staged, nullptr, NoSelectHook(), sel_stage);
  KT(7);
}

// ------------------------------------------------------------------ host side

int launch_score(const ScoreArgs& a, cudaStream_t stream) {
  const int G = a.hq / a.hmeta;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.lo) | reinterpret_cast<uintptr_t>(a.hi)) & 15) == 0;
  if (a.d == 64 || a.d == 128 || a.d == 256) {
    const int rs = a.d + 4;
    const size_t smem = static_cast<size_t>(2) * kTileBlocks * rs * 4 + static_cast<size_t>(2) * kQReq * G * a.d * 8;
    if (smem <= 200 * 1024) {
      const int tiles = (a.total_blocks + kTileBlocks - 1) / kTileBlocks;
      dim3 grid(tiles, a.hmeta);
      const int bulk = aligned ? 1 : 0;
      const bool g4 = G % kTileRowGroup == 0;
      auto kern = a.d == 64 ? (g4 ? score_tiled_kernel<2, true> : score_tiled_kernel<2, false>)
                            : (a.d == 128 ? (g4 ? score_tiled_kernel<4, true> : score_tiled_kernel<4, false>)
                                          : (g4 ? score_tiled_kernel<8, true> : score_tiled_kernel<8, false>));
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      prefer_shared(kern);
      kern<<<grid, kTileWarps * 32, smem, stream>>>(a, bulk);
      return static_cast<int>(cudaGetLastError());
    }
  }
  ScoreTile t;
  t.tn = max(4, min(64, (128 + G - 1) / G));
  t.bulk = aligned && (a.d % 4 == 0);
  const int tiles = (a.total_blocks + t.tn - 1) / t.tn;
  dim3 grid(tiles, a.hmeta);
  const size_t smem = static_cast<size_t>(t.tn) * a.d * 4 * 2 + static_cast<size_t>(kQReq) * G * a.d * 8 +
                      static_cast<size_t>(t.tn) * G * 8 + static_cast<size_t>(t.tn) * 4 + 16;
  if (smem > 200 * 1024) return -1;
  cudaFuncSetAttribute(score_generic_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  score_generic_kernel<0><<<grid, kScoreThreads, smem, stream>>>(a, t);
  return static_cast<int>(cudaGetLastError());
}

template <int E>
static int launch_topk_e(const SelectArgs& a, int threads, cudaStream_t stream) {
  prefer_shared(select_topk_kernel<E>);
  return launch_pdl(select_topk_kernel<E>, dim3(a.R * a.hsel), dim3(threads), 0, stream, 0, a);
}

int launch_select(const SelectArgs& a, int max_n, cudaStream_t stream) {
  if (max_n <= 1024) return launch_topk_e<4>(a, 256, stream);
  if (max_n <= 2048) return launch_topk_e<4>(a, 512, stream);
  if (max_n <= 4096) return launch_topk_e<8>(a, 512, stream);
  if (max_n <= 8192) return launch_topk_e<16>(a, 512, stream);
  if (max_n <= 16384) return launch_topk_e<32>(a, 512, stream);
  return -1;
}

int launch_bounds(const ScoreArgs& a, float2* bounds, cudaStream_t stream) {
  const int G = a.hq / a.hmeta;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.lo) | reinterpret_cast<uintptr_t>(a.hi)) & 15) == 0;
  if (!aligned || G > 16 || (a.d != 64 && a.d != 128 && a.d != 256)) return 1;
  // q rows and their norms (rounded up to 16 bytes), then the tile's lo and hi rows.
  const size_t smem = (((static_cast<size_t>(kQReq) * G * a.d + kQReq * G) + 3) & ~static_cast<size_t>(3)) * 4 +
                      (static_cast<size_t>(kQReq) * 2 * a.d + 4) * 4 + static_cast<size_t>(2) * kBTile * a.d * 4;
  const dim3 grid((a.total_blocks + kBTile - 1) / kBTile, a.hmeta);
  void (*kern)(ScoreArgs, float2*);
  if (a.d == 64) kern = G <= 4 ? bound_interval_kernel<2, 4> : bound_interval_kernel<2, 16>;
  else if (a.d == 128) kern = G <= 4 ? bound_interval_kernel<4, 4> : bound_interval_kernel<4, 16>;
  else kern = G <= 4 ? bound_interval_kernel<8, 4> : bound_interval_kernel<8, 16>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  kern<<<grid, kBWarps * 32, smem, stream>>>(a, bounds);
  return static_cast<int>(cudaGetLastError());
}

template <int E, int NT>
static int launch_bounded_e(const SelectArgs& a, cudaStream_t stream) {
  constexpr size_t smem = static_cast<size_t>(E * NT + (E * NT) / 16) * sizeof(float2);
  cudaFuncSetAttribute(select_bounded_kernel<E, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  prefer_shared(select_bounded_kernel<E, NT>);
  return launch_pdl(select_bounded_kernel<E, NT>, dim3(a.R * a.hsel), dim3(NT), smem, stream, 0, a);
}

int launch_select_bounded(const SelectArgs& a, int max_n, cudaStream_t stream) {
  if (max_n <= 1024) return launch_bounded_e<4, 256>(a, stream);
  if (max_n <= 2048) return launch_bounded_e<4, 512>(a, stream);
  if (max_n <= 4096) return launch_bounded_e<8, 512>(a, stream);
  if (max_n <= 8192) return launch_bounded_e<16, 512>(a, stream);
  if (max_n <= 16384) return launch_bounded_e<32, 512>(a, stream);
  return -1;
}

int launch_merge_candidates(const MergeArgs& a, cudaStream_t stream) {
  if (a.ncand <= 1024) {
    merge_candidates_kernel<8><<<a.rows, 128, 0, stream>>>(a);
  } else if (a.ncand <= 4096) {
    merge_candidates_kernel<16><<<a.rows, 256, 0, stream>>>(a);
  } else if (a.ncand <= 16384) {
    merge_candidates_kernel<32><<<a.rows, 512, 0, stream>>>(a);
  } else {
    return -1;
  }
  return static_cast<int>(cudaGetLastError());
}

int set_wait_limit_select(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
