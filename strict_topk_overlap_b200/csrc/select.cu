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
// Top-K: per selection row, the K largest scores, ties to the lower block
// index, written in ascending block-ID order. Radix select over 64-bit
// order-preserving keys in shared memory (8-bit digits, leading common bits
// skipped), followed by an index-ordered block scan that resolves ties.

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

// One CTA: one meta head, TN consecutive global blocks, all G query heads of
// that meta head. Pairs (row, g) are processed 32 at a time per warp.
template <int C>
__global__ void __launch_bounds__(256) score_kernel(ScoreArgs a, int tn) {
  extern __shared__ double s64[];  // [tn * G]
  const int G = a.hq / a.hmeta;
  const int mh = blockIdx.y;
  const int row0 = blockIdx.x * tn;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int pairs = tn * G;
  const int c = (a.d + 31) / 32;

  for (int base = warp * 32; base < pairs; base += nwarps * 32) {
    double part[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) part[i] = 0.0;
    int last_row = -1;
    float lo_v[C > 0 ? C : 1], hi_v[C > 0 ? C : 1];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int pair = base + i;
      const int rloc = pair / G;
      const int g = pair - rloc * G;
      const int gb = row0 + rloc;
      if (pair < pairs && gb < a.total_blocks) {
        if (rloc != last_row) {
          last_row = rloc;
          const long long moff = (static_cast<long long>(mh) * a.total_blocks + gb) * a.d;
          if constexpr (C == 4) {
            float4 x = *reinterpret_cast<const float4*>(a.lo + moff + lane * 4);
            float4 y = *reinterpret_cast<const float4*>(a.hi + moff + lane * 4);
            lo_v[0] = x.x; lo_v[1] = x.y; lo_v[2] = x.z; lo_v[3] = x.w;
            hi_v[0] = y.x; hi_v[1] = y.y; hi_v[2] = y.z; hi_v[3] = y.w;
          } else if constexpr (C > 0) {
#pragma unroll
            for (int j = 0; j < C; ++j) {
              const int dd = lane * C + j;
              lo_v[j] = dd < a.d ? a.lo[moff + dd] : 0.f;
              hi_v[j] = dd < a.d ? a.hi[moff + dd] : 0.f;
            }
          }
        }
        const int r = find_request(a.block_offsets, a.R, gb);
        const long long qoff = (static_cast<long long>(r) * a.hq + mh * G + g) * a.d;
        double acc = 0.0;
        if constexpr (C > 0) {
#pragma unroll
          for (int j = 0; j < C; ++j) {
            const int dd = lane * C + j;
            if (dd < a.d) {
              const float qv = load_any(a.q, a.q_dtype, qoff + dd);
              const float bv = qv >= 0.f ? hi_v[j] : lo_v[j];
              acc = __dadd_rn(acc, __dmul_rn(static_cast<double>(qv), static_cast<double>(bv)));
            }
          }
        } else {
          const long long moff = (static_cast<long long>(mh) * a.total_blocks + gb) * a.d;
          for (int dd = lane * c; dd < min((lane + 1) * c, a.d); ++dd) {
            const float qv = load_any(a.q, a.q_dtype, qoff + dd);
            const float bv = qv >= 0.f ? a.hi[moff + dd] : a.lo[moff + dd];
            acc = __dadd_rn(acc, __dmul_rn(static_cast<double>(qv), static_cast<double>(bv)));
          }
        }
        part[i] = acc;
      }
    }
    transpose_reduce32(part, lane);
    const int pair = base + lane;
    if (pair < pairs) s64[pair] = part[0];
  }
  __syncthreads();

  // Outputs.
  for (int pair = threadIdx.x; pair < pairs; pair += blockDim.x) {
    const int rloc = pair / G;
    const int g = pair - rloc * G;
    const int gb = row0 + rloc;
    if (gb >= a.total_blocks) continue;
    const int h = mh * G + g;
    const double s = s64[pair];
    if (a.scores_f32) a.scores_f32[static_cast<long long>(h) * a.total_blocks + gb] = __double2float_rn(s);
    if (a.scores_f64 && !a.group_select) a.scores_f64[static_cast<long long>(h) * a.total_blocks + gb] = s;
  }
  if (a.scores_f64 && a.group_select) {
    for (int rloc = threadIdx.x; rloc < tn; rloc += blockDim.x) {
      const int gb = row0 + rloc;
      if (gb >= a.total_blocks) continue;
      double acc = 0.0;
      for (int g = 0; g < G; ++g) acc = __dadd_rn(acc, s64[rloc * G + g]);
      a.scores_f64[static_cast<long long>(mh) * a.total_blocks + gb] = acc;
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

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int x, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nw ? warp_tot[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(kFull, ti, o);
      if (lane >= o) ti += y;
    }
    if (lane < nw) warp_tot[lane] = ti - t;
    if (lane == 31) *total = ti;
  }
  __syncthreads();
  const int res = inc - x + warp_tot[warp];
  __syncthreads();
  return res;
}

// Selection core shared by the plain and the candidate-merge kernels:
// `keys` holds n ordered keys in shared memory, `idx_of(i)` maps a position to
// the ID written out. Positions are ordered by (key desc, id asc) when the
// caller lays out positions in ascending-ID order.
template <typename IdOf>
__device__ void select_core(const unsigned long long* keys, int n, int topk, IdOf idx_of, int* ids_out,
                            unsigned long long* keys_out) {
  __shared__ unsigned hist[256];
  __shared__ int sh_bin, sh_above, sh_count;
  __shared__ unsigned long long sh_or;
  __shared__ int warp_tot[32];
  __shared__ int sh_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = blockDim.x;

  // Common leading bits.
  const unsigned long long k0 = keys[0];
  unsigned long long diff = 0;
  for (int i = tid; i < n; i += T) diff |= keys[i] ^ k0;
  diff = warp_or64(diff);
  if (tid == 0) sh_or = 0;
  __syncthreads();
  if (lane == 0) atomicOr(&sh_or, diff);
  __syncthreads();
  diff = sh_or;

  unsigned long long prefix = 0, mask = 0;
  int kk = topk;
  bool take_all_eq = false;
  if (diff == 0) {
    mask = ~0ull;
    prefix = k0;
    take_all_eq = (kk == n);
  } else {
    const int hb = 63 - __clzll(diff);
    mask = (hb == 63) ? 0ull : ~((2ull << hb) - 1ull);
    prefix = k0 & mask;
    for (int shift = (hb / 8) * 8; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += T) hist[i] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += T) {
        const unsigned long long k = keys[i];
        if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        // Suffix scan from the top bin downwards: lane l owns bins [255-8l-7, 255-8l].
        int local[8];
        int sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { local[j] = hist[255 - (lane * 8 + j)]; sum += local[j]; }
        int inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int y = __shfl_up_sync(kFull, inc, o);
          if (lane >= o) inc += y;
        }
        const int excl = inc - sum;
        const bool crosses = (excl < kk) && (inc >= kk);
        const unsigned who = __ballot_sync(kFull, crosses);
        if (lane == __ffs(who) - 1) {
          int run = excl;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (run + local[j] >= kk) {
              sh_bin = 255 - (lane * 8 + j);
              sh_above = run;
              sh_count = local[j];
              break;
            }
            run += local[j];
          }
        }
      }
      __syncthreads();
      const int bin = sh_bin, above = sh_above, cnt = sh_count;
      __syncthreads();
      prefix |= static_cast<unsigned long long>(bin) << shift;
      mask |= 0xFFull << shift;
      kk -= above;
      if (cnt == kk) { take_all_eq = true; break; }
    }
  }

  // Resolve: key above the region -> selected; in region -> selected if
  // take_all_eq, else the kk lowest positions.
  const int E = (n + T - 1) / T;
  const int beg = min(tid * E, n), end = min(beg + E, n);
  int n_eq = 0;
  for (int i = beg; i < end; ++i) n_eq += ((keys[i] & mask) == prefix);
  int eq_rank = block_exclusive_scan(n_eq, warp_tot, &sh_total);
  int n_sel = 0;
  {
    int er = eq_rank;
    for (int i = beg; i < end; ++i) {
      const unsigned long long km = keys[i] & mask;
      bool s = km > prefix;
      if (km == prefix) { s = take_all_eq || er < kk; ++er; }
      n_sel += s;
    }
  }
  int pos = block_exclusive_scan(n_sel, warp_tot, &sh_total);
  {
    int er = eq_rank;
    for (int i = beg; i < end; ++i) {
      const unsigned long long km = keys[i] & mask;
      bool s = km > prefix;
      if (km == prefix) { s = take_all_eq || er < kk; ++er; }
      if (s && pos < topk) {
        ids_out[pos] = idx_of(i);
        if (keys_out) keys_out[pos] = keys[i];
        ++pos;
      }
    }
  }
}

__global__ void __launch_bounds__(512) select_topk_kernel(SelectArgs a) {
  extern __shared__ unsigned long long skeys[];
  const int row = blockIdx.x;
  const int r = row / a.hsel, hs = row - r * a.hsel;
  const int off = a.block_offsets ? a.block_offsets[r] : 0;
  const int n = a.block_offsets ? a.block_offsets[r + 1] - off : a.n;
  const double* src = a.scores + static_cast<long long>(hs) * a.total_blocks + off;
  for (int i = threadIdx.x; i < n; i += blockDim.x) skeys[i] = order_key(src[i]);
  __syncthreads();
  if (n < a.topk) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  const int base = a.id_base;
  select_core(skeys, n, a.topk, [base](int i) { return base + i; },
              a.ids_out + static_cast<long long>(row) * a.topk,
              a.keys_out ? a.keys_out + static_cast<long long>(row) * a.topk : nullptr);
}

// Candidate merge (context-parallel and segmented selection): each row has
// `ncand` (key, id) candidates gathered from several shards, laid out in
// ascending-ID order (each shard's list is ascending and shards own
// increasing ID ranges), so position order equals ID order and the same
// selection core resolves ties toward the lower ID.

__global__ void __launch_bounds__(512) merge_candidates_kernel(MergeArgs a) {
  extern __shared__ unsigned long long smem[];
  unsigned long long* skeys = smem;                    // ncand
  int* sids = reinterpret_cast<int*>(smem + a.ncand);  // ncand
  const int row = blockIdx.x;
  const unsigned long long* ksrc = a.keys + static_cast<long long>(row) * a.ncand;
  const int* isrc = a.ids + static_cast<long long>(row) * a.ncand;
  for (int i = threadIdx.x; i < a.ncand; i += blockDim.x) {
    skeys[i] = ksrc[i];
    sids[i] = isrc[i];
  }
  __syncthreads();
  if (a.ncand < a.topk) {
    if (threadIdx.x == 0) report(a.status, kStatusShapeOverflow);
    return;
  }
  select_core(skeys, a.ncand, a.topk, [sids](int i) { return sids[i]; },
              a.ids_out + static_cast<long long>(row) * a.topk, nullptr);
}

// ------------------------------------------------------------------ host side

int launch_score(const ScoreArgs& a, cudaStream_t stream) {
  const int G = a.hq / a.hmeta;
  const int tn = max(1, 512 / G);
  const int tiles = (a.total_blocks + tn - 1) / tn;
  dim3 grid(tiles, a.hmeta);
  const size_t smem = static_cast<size_t>(tn) * G * sizeof(double);
  const int c = (a.d + 31) / 32;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.lo) | reinterpret_cast<uintptr_t>(a.hi)) & 15) == 0;
  const bool vec4 = (c == 4) && (a.d == 128) && aligned;
  if (vec4) {
    score_kernel<4><<<grid, 256, smem, stream>>>(a, tn);
  } else if (c <= 8 && a.d == c * 32) {
    switch (c) {
      case 1: score_kernel<1><<<grid, 256, smem, stream>>>(a, tn); break;
      case 2: score_kernel<2><<<grid, 256, smem, stream>>>(a, tn); break;
      case 8: score_kernel<8><<<grid, 256, smem, stream>>>(a, tn); break;
      default: score_kernel<0><<<grid, 256, smem, stream>>>(a, tn); break;
    }
  } else {
    score_kernel<0><<<grid, 256, smem, stream>>>(a, tn);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_select(const SelectArgs& a, int max_n, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(max_n) * sizeof(unsigned long long);
  if (smem > 200 * 1024) return -1;
  cudaFuncSetAttribute(select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  const int threads = max_n >= 4096 ? 512 : (max_n >= 1024 ? 256 : 128);
  select_topk_kernel<<<a.R * a.hsel, threads, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int launch_merge_candidates(const MergeArgs& a, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(a.ncand) * (sizeof(unsigned long long) + sizeof(int));
  if (smem > 200 * 1024) return -1;
  cudaFuncSetAttribute(merge_candidates_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  merge_candidates_kernel<<<a.rows, 256, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace stk
