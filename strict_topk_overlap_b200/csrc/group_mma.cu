// Tensor-core attention for wide GQA groups with a shared block list
// (12 query heads per KV head, 4-token blocks, one Top-K
// list per KV group). All G <= 16 query heads of a KV head form one 16-row
// MMA tile, so each selected K/V block is read once per group instead of
// once per query head, and QK^T and PV run on the tensor cores
// (mma.sync m16n8k16, bf16 or f16 inputs, FP32 accumulation).
//
// Replaces, for shared lists, the per-head attention of
// gqa_hierarchical.py:55-112 (_packed_partials + _reduce) and gqa.py:140-142.
//
// Grid: (splits, hkv). A CTA of four warps takes kTokensPerCta consecutive
// tokens of its KV head's list (whole blocks, gathered into shared memory
// with one bulk copy per block, issued by the lanes of warp 0), each warp 16
// of them (64 per CTA: config 2's 2,048 tokens per group give 256 CTAs):
//   S = Q K^T (2 n-tiles of 8 tokens x 8 k-steps of 16 dims), scaled by
//   D^-1/2 in FP32; a row-wise softmax over the warp's 16 tokens; O = P V
//   with P split into a bf16 (or f16) high part and the residual's low part,
//   two MMAs per tile, so the weights keep ~16 bits instead of 8.
// The four warps' (m, l, O) merge in shared memory; the CTA writes one
// unnormalised state per (query head, split), and merge_kernel finishes the
// rows. MMA fragment layouts follow the PTX ISA's m16n8k16 description
// (A row-major 16x16, B column-major 16x8, C 16x8 FP32).

#include <type_traits>

#include "internal.cuh"

namespace stk {

constexpr int kGroupWarps = 4;
constexpr int kTokensPerWarp = 16;
constexpr int kSTiles = kTokensPerWarp / 8;   // QK n-tiles of 8 tokens
constexpr int kPSteps = kTokensPerWarp / 16;  // PV k-steps of 16 tokens
constexpr int kTokensPerCta = kGroupWarps * kTokensPerWarp;

struct GroupArgs {
  KVLayout L;        // dense [hkv, n, b, d]
  const void* q;     // [hkv * G, d], same dtype as K/V
  int G;             // query heads per KV head (<= 16)
  const int* ids;    // [hkv, sa] shared block list per KV head
  int sa;
  const int* counts; // optional [hkv]: list length per KV head (the rest of its row is unused)
  float scale;
  int splits;
  float* m;          // [hkv * G, splits]
  float* l;
  float* u;          // [hkv * G, splits, d]
  int* status;
};

template <typename T>
__device__ __forceinline__ unsigned pack2(float lo, float hi);
template <>
__device__ __forceinline__ unsigned pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const unsigned*>(&v);
}
template <>
__device__ __forceinline__ unsigned pack2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const unsigned*>(&v);
}
template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float round_to<__half>(float x) { return __half2float(__float2half_rn(x)); }

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kGroupWarps * 32) group_mma_kernel(GroupArgs a) {
  constexpr int NT = D / 8;   // PV n-tiles (8 dims each)
  constexpr int KS = D / 16;  // QK k-steps (16 dims each)
  extern __shared__ __align__(128) unsigned char gsm[];
  T* Qs = reinterpret_cast<T*>(gsm);                 // [16][D]
  T* Ks = Qs + 16 * D;                               // [kTokensPerCta][D]
  T* Vs = Ks + kTokensPerCta * D;                    // [kTokensPerCta][D]
  float* wO = reinterpret_cast<float*>(Vs + kTokensPerCta * D);  // [warps][16][D]
  float* wM = wO + kGroupWarps * 16 * D;             // [warps][16]
  float* wL = wM + kGroupWarps * 16;                 // [warps][16]
  __shared__ uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, h = blockIdx.y;
  const int B = a.L.b;
  const int bpc = kTokensPerCta / B;                 // blocks per CTA
  const int j0 = split * bpc;
  const int len = a.counts ? min(a.sa, a.counts[h]) : a.sa;
  const int nb = max(0, min(bpc, len - j0));         // blocks of this CTA
  const int ntok = nb * B;
  const T* K = static_cast<const T*>(a.L.k);
  const T* V = static_cast<const T*>(a.L.v);
  const unsigned blk_bytes = static_cast<unsigned>(B * D * sizeof(T));

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0 && nb > 0) {
    if (lane == 0) mbar_arrive_expect_tx(&bar, 2u * blk_bytes * static_cast<unsigned>(nb));
    __syncwarp();
    for (int j = lane; j < nb; j += 32) {
      int bid = a.ids[static_cast<long long>(h) * a.sa + j0 + j];
      if (bid < 0 || bid >= a.L.n) {
        report(a.status, kStatusBadBlockId);
        bid = 0;  // keeps the expected byte count; the row is flagged
      }
      const long long off = (static_cast<long long>(h) * a.L.n + bid) * B * D;
      bulk_g2s(Ks + j * B * D, K + off, blk_bytes, &bar);
      bulk_g2s(Vs + j * B * D, V + off, blk_bytes, &bar);
    }
  }
  // Tokens past the list's end (last split) are zero, so that their zero
  // weights multiply finite values.
  for (int i = ntok * D + tid; i < kTokensPerCta * D; i += blockDim.x) {
    Ks[i] = T(0.f);
    Vs[i] = T(0.f);
  }
  // Q tile: rows >= G are zero.
  const T* Q = static_cast<const T*>(a.q) + static_cast<long long>(h) * a.G * D;
  for (int i = tid; i < 16 * D; i += blockDim.x) {
    const int r = i / D;
    Qs[i] = r < a.G ? Q[static_cast<long long>(r) * D + (i - r * D)] : T(0.f);
  }
  __syncthreads();
  const bool ok = nb == 0 || mbar_wait(&bar, 0, a.status);

  const int g = lane >> 2, t4 = lane & 3;
  const int tw0 = warp * kTokensPerWarp;  // this warp's first token
  float mrow[2] = {neg_inf(), neg_inf()}, lrow[2] = {0.f, 0.f};
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  if (ok && tw0 < ntok) {
    // ---- S = Q K^T over the warp's tokens.
    float s[kSTiles][4];
#pragma unroll
    for (int n = 0; n < kSTiles; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      unsigned af[4];
      const int c = ks * 16 + t4 * 2;
      af[0] = *reinterpret_cast<const unsigned*>(Qs + g * D + c);
      af[1] = *reinterpret_cast<const unsigned*>(Qs + (g + 8) * D + c);
      af[2] = *reinterpret_cast<const unsigned*>(Qs + g * D + c + 8);
      af[3] = *reinterpret_cast<const unsigned*>(Qs + (g + 8) * D + c + 8);
#pragma unroll
      for (int n = 0; n < kSTiles; ++n) {
        const T* kr = Ks + (tw0 + n * 8 + g) * D + c;  // token n*8+g, dims c, c+1 (and +8)
        const unsigned b0 = *reinterpret_cast<const unsigned*>(kr);
        const unsigned b1 = *reinterpret_cast<const unsigned*>(kr + 8);
        mma16816<T>(s[n], af, b0, b1);
      }
    }
    // ---- row-wise softmax over the warp's tokens (rows g and g + 8).
#pragma unroll
    for (int n = 0; n < kSTiles; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tw0 + n * 8 + t4 * 2 + (e & 1);
        s[n][e] = tok < ntok ? s[n][e] * a.scale : neg_inf();
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = neg_inf();
#pragma unroll
      for (int n = 0; n < kSTiles; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
      mrow[hr] = mx;
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < kSTiles; ++n) {
#pragma unroll
        for (int e = 2 * hr; e < 2 * hr + 2; ++e) {
          const float p = s[n][e] == neg_inf() ? 0.f : expf(s[n][e] - mx);
          s[n][e] = p;
          sum += p;
        }
      }
      sum += __shfl_xor_sync(kFull, sum, 1);
      sum += __shfl_xor_sync(kFull, sum, 2);
      lrow[hr] = sum;
    }
    // ---- O = P V: P as A fragments (hi and lo halves), V as column-major B.
#pragma unroll
    for (int kt = 0; kt < kPSteps; ++kt) {  // 16-token k-steps
      unsigned ph[4], pl[4];
      const float* s0 = s[2 * kt];
      const float* s1 = s[2 * kt + 1];
      const float v8[8] = {s0[0], s0[1], s0[2], s0[3], s1[0], s1[1], s1[2], s1[3]};
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        hi[e] = round_to<T>(v8[e]);
        lo[e] = v8[e] - hi[e];
      }
      ph[0] = pack2<T>(hi[0], hi[1]); ph[1] = pack2<T>(hi[2], hi[3]);
      ph[2] = pack2<T>(hi[4], hi[5]); ph[3] = pack2<T>(hi[6], hi[7]);
      pl[0] = pack2<T>(lo[0], lo[1]); pl[1] = pack2<T>(lo[2], lo[3]);
      pl[2] = pack2<T>(lo[4], lo[5]); pl[3] = pack2<T>(lo[6], lo[7]);
      const int tk = tw0 + kt * 16 + t4 * 2;  // tokens tk, tk+1 (b0) and tk+8, tk+9 (b1)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int col = n * 8 + g;
        const T* v0 = Vs + tk * D + col;
        T x0 = v0[0], x1 = v0[D], x2 = v0[8 * D], x3 = v0[9 * D];
        const unsigned b0 = (static_cast<unsigned>(*reinterpret_cast<const unsigned short*>(&x1)) << 16) |
                            *reinterpret_cast<const unsigned short*>(&x0);
        const unsigned b1 = (static_cast<unsigned>(*reinterpret_cast<const unsigned short*>(&x3)) << 16) |
                            *reinterpret_cast<const unsigned short*>(&x2);
        mma16816<T>(o[n], ph, b0, b1);
        mma16816<T>(o[n], pl, b0, b1);
      }
    }
  }
  // ---- merge the four warps: each warp parks (m, l, O) in shared memory.
  float* myO = wO + warp * 16 * D;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int col = n * 8 + t4 * 2;
    myO[g * D + col] = o[n][0];
    myO[g * D + col + 1] = o[n][1];
    myO[(g + 8) * D + col] = o[n][2];
    myO[(g + 8) * D + col + 1] = o[n][3];
  }
  if (t4 == 0) {
    wM[warp * 16 + g] = mrow[0];
    wM[warp * 16 + g + 8] = mrow[1];
    wL[warp * 16 + g] = lrow[0];
    wL[warp * 16 + g + 8] = lrow[1];
  }
  __syncthreads();
  for (int i = tid; i < a.G * D; i += blockDim.x) {
    const int r = i / D, dd = i - r * D;
    float M = neg_inf();
#pragma unroll
    for (int w = 0; w < kGroupWarps; ++w) M = fmaxf(M, wM[w * 16 + r]);
    float Z = 0.f, U = 0.f;
    if (M != neg_inf()) {
#pragma unroll
      for (int w = 0; w < kGroupWarps; ++w) {
        const float mw = wM[w * 16 + r];
        if (mw == neg_inf()) continue;
        const float c = expf(mw - M);
        Z += c * wL[w * 16 + r];
        U += c * wO[(w * 16 + r) * D + dd];
      }
    }
    const long long row = static_cast<long long>(h) * a.G + r;
    if (dd == 0) {
      a.m[row * a.splits + split] = M;
      a.l[row * a.splits + split] = Z;
    }
    a.u[(row * a.splits + split) * D + dd] = U;
  }
}

size_t group_mma_smem(int d, int esize) {
  return static_cast<size_t>(16 + 2 * kTokensPerCta) * d * esize + static_cast<size_t>(kGroupWarps) * 16 * d * 4 +
         static_cast<size_t>(kGroupWarps) * 16 * 4 * 2;
}

int group_mma_splits(int sa, int b) { return (sa * b + kTokensPerCta - 1) / kTokensPerCta; }

int launch_group_mma(const KVLayout& L, int kv_dtype, const void* q, int G, const int* ids, int sa, float scale,
                     float* m, float* l, float* u, int* status, cudaStream_t stream) {
  GroupArgs a{};
  a.L = L; a.q = q; a.G = G; a.ids = ids; a.sa = sa; a.scale = scale;
  a.splits = group_mma_splits(sa, L.b);
  a.m = m; a.l = l; a.u = u; a.status = status;
  const size_t smem = group_mma_smem(L.d, 2);
  const dim3 grid(static_cast<unsigned>(a.splits), static_cast<unsigned>(L.hkv));
  void (*kern)(GroupArgs);
  if (kv_dtype == kBF16) kern = L.d == 64 ? group_mma_kernel<__nv_bfloat16, 64> : group_mma_kernel<__nv_bfloat16, 128>;
  else kern = L.d == 64 ? group_mma_kernel<__half, 64> : group_mma_kernel<__half, 128>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  kern<<<grid, kGroupWarps * 32, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ shared saved repair
// gqa_hierarchical.repair_saved_shared (gqa_hierarchical.py:137-144) for
// groups whose query heads share one selected list A and one predicted
// list P: the misses (A not in P) are then the same for every head of a
// group, so they run on the tensor-core group tile above (each missed block
// read once per group), and each head folds its own saved states of the hits
// (P slots whose block is in A). Membership comes from the group's first row.

// Per KV head h (one CTA): the misses of row h * G in A order, their count,
// and the hit flag of every P slot.
__global__ void __launch_bounds__(256) group_miss_kernel(const int* sel, int sa, const int* pred, int sp, int G, int n,
                                                         int* miss, int* count, unsigned char* hit, int* status) {
  extern __shared__ unsigned gmask[];  // P bits [nw], then A bits [nw]
  __shared__ int wtot[8];
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = (n + 31) / 32;
  unsigned* pb = gmask;
  unsigned* ab = gmask + nw;
  const int* arow = sel + static_cast<long long>(h) * G * sa;
  const int* prow = pred + static_cast<long long>(h) * G * sp;
  for (int i = tid; i < 2 * nw; i += blockDim.x) gmask[i] = 0u;
  __syncthreads();
  for (int i = tid; i < sp; i += blockDim.x) {
    const int id = prow[i];
    if (id >= 0 && id < n) atomicOr(&pb[id >> 5], 1u << (id & 31));
  }
  for (int i = tid; i < sa; i += blockDim.x) {
    const int id = arow[i];
    if (id >= 0 && id < n) atomicOr(&ab[id >> 5], 1u << (id & 31));
    else report(status, kStatusBadBlockId);
  }
  __syncthreads();
  for (int i = tid; i < sp; i += blockDim.x) {
    const int id = prow[i];
    hit[static_cast<long long>(h) * sp + i] = (id >= 0 && id < n && ((ab[id >> 5] >> (id & 31)) & 1u)) ? 1 : 0;
  }
  // Misses in A order: chunks of 256 entries, one ballot per warp.
  int base = 0;
  for (int c0 = 0; c0 < sa; c0 += blockDim.x) {
    const int i = c0 + tid;
    const int id = i < sa ? arow[i] : -1;
    const bool m = id >= 0 && id < n && !((pb[id >> 5] >> (id & 31)) & 1u);
    const unsigned bal = __ballot_sync(kFull, m);
    if (lane == 0) wtot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) {
      before += w < warp ? wtot[w] : 0;
      total += wtot[w];
    }
    if (m) miss[static_cast<long long>(h) * sa + base + before + __popc(bal & ((1u << lane) - 1u))] = id;
    base += total;
    __syncthreads();
  }
  if (tid == 0) count[h] = base;
}

// Per row r (query head; one CTA of 16 warps): M over the row's hits and
// the group tile's split states, then every source's weight; warp k folds
// sources k, k + 16, ... (hits in P-slot order, then splits) with 4
// consecutive dims per lane, eight sources' loads in flight; the warps'
// parts add in warp order, so the result does not depend on timing.
__global__ void __launch_bounds__(512) group_repair_merge_kernel(const float* pm, const float* pl, const float* pu,
                                                                 const unsigned char* hit, int sp, const float* sm,
                                                                 const float* sl, const float* su, int splits, int G,
                                                                 int d, float* out) {
  extern __shared__ __align__(16) float gms[];  // w[sp + splits], part[16][d]
  __shared__ float red[16];
  constexpr int kWarps = 16;
  constexpr int kBatch = 8;
  const int r = blockIdx.x, h = r / G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ns = sp + splits;
  float* w = gms;
  float* part = gms + ((ns + 3) & ~3);
  const unsigned char* hr = hit + static_cast<long long>(h) * sp;
  const long long pr = static_cast<long long>(r) * sp, srow = static_cast<long long>(r) * splits;
  auto src_m = [&](int i) { return i < sp ? (hr[i] ? pm[pr + i] : neg_inf()) : sm[srow + i - sp]; };
  float mx = neg_inf();
  for (int i = tid; i < ns; i += blockDim.x) mx = fmaxf(mx, src_m(i));
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = neg_inf();
#pragma unroll
  for (int k = 0; k < kWarps; ++k) M = fmaxf(M, red[k]);
  __syncthreads();
  float z = 0.f;
  for (int i = tid; i < ns; i += blockDim.x) {
    const float mi = src_m(i);
    const float wi = (M != neg_inf() && mi != neg_inf()) ? expf(mi - M) : 0.f;
    w[i] = wi;
    z += wi * (i < sp ? pl[pr + i] : sl[srow + i - sp]);
  }
  z = warp_sum(z);
  if (lane == 0) red[warp] = z;
  __syncthreads();
  float Z = 0.f;
#pragma unroll
  for (int k = 0; k < kWarps; ++k) Z += red[k];
  for (int d0 = 0; d0 < d; d0 += 128) {
    const int dd = d0 + 4 * lane;
    const bool live = dd < d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = warp; i0 < ns; i0 += kBatch * kWarps) {
      float4 x[kBatch];
      float wi[kBatch];
#pragma unroll
      for (int c = 0; c < kBatch; ++c) {
        const int i = i0 + c * kWarps;
        wi[c] = i < ns ? w[i] : 0.f;
        const float* src = i < sp ? pu + (pr + i) * d : su + (srow + i - sp) * d;
        x[c] = (wi[c] != 0.f && live) ? *reinterpret_cast<const float4*>(src + dd) : make_float4(0.f, 0.f, 0.f, 0.f);
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
    float U = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) U += part[k * d + dd];
    out[static_cast<long long>(r) * d + dd] = U / fmaxf(Z, 1e-30f);
  }
}

int launch_group_repair(const KVLayout& L, int kv_dtype, const void* q, int G, float scale, const int* sel, int sa,
                        const int* pred, int sp, const float* pm, const float* pl, const float* pu, int* miss, int* count,
                        unsigned char* hit, float* sm, float* sl, float* su, float* out, int* status,
                        cudaStream_t stream) {
  const int hkv = L.hkv;
  const size_t msmem = static_cast<size_t>(2 * ((L.n + 31) / 32)) * 4;
  if (msmem > 48 * 1024)
    cudaFuncSetAttribute(group_miss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(msmem));
  group_miss_kernel<<<hkv, 256, msmem, stream>>>(sel, sa, pred, sp, G, L.n, miss, count, hit, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  GroupArgs a{};
  a.L = L; a.q = q; a.G = G; a.ids = miss; a.sa = sa; a.counts = count; a.scale = scale;
  a.splits = group_mma_splits(sa, L.b);
  a.m = sm; a.l = sl; a.u = su; a.status = status;
  const size_t smem = group_mma_smem(L.d, 2);
  const dim3 grid(static_cast<unsigned>(a.splits), static_cast<unsigned>(hkv));
  void (*kern)(GroupArgs);
  if (kv_dtype == kBF16) kern = L.d == 64 ? group_mma_kernel<__nv_bfloat16, 64> : group_mma_kernel<__nv_bfloat16, 128>;
  else kern = L.d == 64 ? group_mma_kernel<__half, 64> : group_mma_kernel<__half, 128>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  prefer_shared(kern);
  kern<<<grid, kGroupWarps * 32, smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  const size_t gsm = (static_cast<size_t>((sp + a.splits + 3) & ~3) + 16 * static_cast<size_t>(L.d)) * 4;
  if (gsm > 48 * 1024)
    cudaFuncSetAttribute(group_repair_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(gsm));
  group_repair_merge_kernel<<<hkv * G, 512, gsm, stream>>>(pm, pl, pu, hit, sp, sm, sl, su, a.splits, G, L.d, out);
  return static_cast<int>(cudaGetLastError());
}

int set_wait_limit_group_mma(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace stk
