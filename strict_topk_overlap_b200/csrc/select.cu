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

#include "internal.cuh"

namespace stk {

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
__global__ void __launch_bounds__(kScoreThreads) score_kernel(ScoreArgs a, ScoreTile t) {
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

// ------------------------------------------------------------------ Top-K

__device__ __forceinline__ unsigned long long order_key(double x) {
  unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(x + 0.0));
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

__device__ __forceinline__ unsigned long long warp_or64(unsigned long long x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x |= __shfl_xor_sync(kFull, x, o);
  return x;
}

// Radix select over E register-resident keys per thread; thread t owns
// positions [t*E, t*E+E). Writes the chosen positions' IDs (id_of) in
// ascending position order.
template <int E, typename IdOf>
__device__ void select_registers(const unsigned long long (&key)[E], int n, int topk, IdOf id_of, int* out,
                                 unsigned long long* keys_out) {
  __shared__ unsigned hist[2][256];
  __shared__ unsigned long long sh_or, sh_k0;
  __shared__ int sh_bin, sh_above, sh_cnt;
  __shared__ unsigned warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = blockDim.x >> 5;
  const int beg = tid * E;

  if (tid == 0) { sh_or = 0; sh_k0 = key[0]; }
  for (int i = tid; i < 512; i += blockDim.x) (&hist[0][0])[i] = 0;
  __syncthreads();
  const unsigned long long k0 = sh_k0;
  unsigned long long diff = 0;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if (beg + j < n) diff |= key[j] ^ k0;
  diff = warp_or64(diff);
  if (lane == 0 && diff) atomicOr(&sh_or, diff);
  __syncthreads();
  diff = sh_or;

  unsigned long long prefix, mask;
  int kk = topk;
  bool take_all = false;
  if (diff == 0) {
    mask = ~0ull;
    prefix = k0;
  } else {
    const int hb = 63 - __clzll(diff);
    mask = (hb == 63) ? 0ull : ~((2ull << hb) - 1ull);
    prefix = k0 & mask;
    int buf = 0;
    for (int shift = (hb / 8) * 8; shift >= 0; shift -= 8) {
#pragma unroll
      for (int j = 0; j < E; ++j) {
        // Lanes holding the same digit add once (warp-aggregated atomics).
        const bool cand = beg + j < n && (key[j] & mask) == prefix;
        const unsigned digit = cand ? static_cast<unsigned>((key[j] >> shift) & 0xFF) : 0xFFFFFFFFu;
        const unsigned grp = __match_any_sync(kFull, digit);
        if (cand && lane == __ffs(grp) - 1) atomicAdd(&hist[buf][digit], static_cast<unsigned>(__popc(grp)));
      }
      __syncthreads();
      if (warp == 0) {
        unsigned local[8];
        unsigned sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { local[j] = hist[buf][255 - (lane * 8 + j)]; sum += local[j]; }
        unsigned inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(kFull, inc, o);
          if (lane >= o) inc += y;
        }
        const unsigned excl = inc - sum;
        const bool crosses = excl < static_cast<unsigned>(kk) && inc >= static_cast<unsigned>(kk);
        const unsigned who = __ballot_sync(kFull, crosses);
        if (lane == __ffs(who) - 1) {
          unsigned run = excl;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (run + local[j] >= static_cast<unsigned>(kk)) {
              sh_bin = 255 - (lane * 8 + j);
              sh_above = static_cast<int>(run);
              sh_cnt = static_cast<int>(local[j]);
              break;
            }
            run += local[j];
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) hist[buf ^ 1][lane * 8 + j] = 0;
      }
      __syncthreads();
      prefix |= static_cast<unsigned long long>(sh_bin) << shift;
      mask |= 0xFFull << shift;
      kk -= sh_above;
      const int cnt = sh_cnt;
      buf ^= 1;
      if (cnt == kk) { take_all = true; break; }
    }
  }
  if (take_all) kk = n;

  // Packed scan: (#above, #in-region) before this thread's first position.
  unsigned n_gt = 0, n_eq = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    if (beg + j < n) {
      const unsigned long long km = key[j] & mask;
      n_gt += km > prefix;
      n_eq += km == prefix;
    }
  }
  const unsigned packed = (n_gt << 16) | n_eq;
  unsigned inc = packed;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const unsigned t = lane < nw ? warp_tot[lane] : 0u;
    unsigned ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(kFull, ti, o);
      if (lane >= o) ti += y;
    }
    if (lane < nw) warp_tot[lane] = ti - t;
  }
  __syncthreads();
  const unsigned excl = inc - packed + warp_tot[warp];
  unsigned gt_before = excl >> 16, eq_before = excl & 0xFFFFu;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    if (beg + j < n) {
      const unsigned long long km = key[j] & mask;
      bool s = km > prefix;
      if (km == prefix) s = static_cast<int>(eq_before) < kk;
      if (s) {
        const int pos = static_cast<int>(gt_before) + min(static_cast<int>(eq_before), kk);
        if (pos < topk) {
          out[pos] = id_of(beg + j);
          if (keys_out) keys_out[pos] = key[j];
        }
      }
      gt_before += km > prefix;
      eq_before += km == prefix;
    }
  }
}

template <int E>
__global__ void __launch_bounds__(512) select_topk_kernel(SelectArgs a) {
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
  const int base = a.id_base;
  select_registers<E>(key, n, a.topk, [base](int i) { return base + i; },
                      a.ids_out + static_cast<long long>(row) * a.topk,
                      a.keys_out ? a.keys_out + static_cast<long long>(row) * a.topk : nullptr);
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

// ------------------------------------------------------------------ host side

int launch_score(const ScoreArgs& a, cudaStream_t stream) {
  const int G = a.hq / a.hmeta;
  ScoreTile t;
  t.tn = max(4, min(64, (128 + G - 1) / G));
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.lo) | reinterpret_cast<uintptr_t>(a.hi)) & 15) == 0;
  t.bulk = aligned && (a.d % 4 == 0);
  const int tiles = (a.total_blocks + t.tn - 1) / t.tn;
  dim3 grid(tiles, a.hmeta);
  const size_t smem = static_cast<size_t>(t.tn) * a.d * 4 * 2 + static_cast<size_t>(kQReq) * G * a.d * 8 +
                      static_cast<size_t>(t.tn) * G * 8 + static_cast<size_t>(t.tn) * 4 + 16;
  if (smem > 200 * 1024) return -1;
  if (a.d == 128) {
    cudaFuncSetAttribute(score_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    score_kernel<4><<<grid, kScoreThreads, smem, stream>>>(a, t);
  } else {
    cudaFuncSetAttribute(score_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    score_kernel<0><<<grid, kScoreThreads, smem, stream>>>(a, t);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_select(const SelectArgs& a, int max_n, cudaStream_t stream) {
  const int rows = a.R * a.hsel;
  if (max_n <= 1024) {
    select_topk_kernel<8><<<rows, 128, 0, stream>>>(a);
  } else if (max_n <= 4096) {
    select_topk_kernel<16><<<rows, 256, 0, stream>>>(a);
  } else if (max_n <= 16384) {
    select_topk_kernel<32><<<rows, 512, 0, stream>>>(a);
  } else {
    return -1;
  }
  return static_cast<int>(cudaGetLastError());
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

}  // namespace stk
