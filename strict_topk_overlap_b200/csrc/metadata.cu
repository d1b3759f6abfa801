// Block metadata (per-block, per-dimension min / max of K over the block's
// tokens) and the decode-loop token append that keeps it current.
//
// Replaces the prefill-time `lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()`
// of benchmarks/run_benchmark.py:42-43 and experiments/trace_replay.py:68
// (the reference builds it outside its timed region) and adds what a real
// decode loop needs on top: writing one new token per request into the
// cache and folding it into its block's bounds, so the metadata is never
// rebuilt. Min / max propagate NaN like torch.amin / amax.
//
// HBM-bound: build reads B·D·esize bytes of K and writes 2·D·4 bytes per
// (block, KV head); append moves D elements of K and of V plus 2·D·4 bytes of
// metadata per (request, KV head).

#include "internal.cuh"

namespace stk {

__device__ __forceinline__ float nan_min(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b);
}
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

// Request of global metadata row gb (binary search over block_offsets).
__device__ __forceinline__ int request_of_block(const KVLayout& L, int R, int gb) {
  if (L.block_offsets == nullptr) return 0;
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (L.block_offsets[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One CTA per (metadata row, KV head); threads over dims, tokens in order.
template <typename T>
__global__ void __launch_bounds__(128) build_metadata_kernel(KVLayout L, int R, int total, float* lo, float* hi) {
  const int gb = blockIdx.x, kv = blockIdx.y;
  const int r = request_of_block(L, R, gb);
  const long long bid = gb - (L.block_offsets ? L.block_offsets[r] : 0);
  const T* K = static_cast<const T*>(L.k);
  const int nseg = block_nseg(L);
  const float inf = __int_as_float(0x7f800000);
  for (int dd = threadIdx.x; dd < L.d; dd += blockDim.x) {
    float mn = inf, mx = -inf;
    for (int s = 0; s < nseg; ++s) {
      const BlockSeg seg = block_seg(L, r, kv, bid, s);
      for (int t = 0; t < seg.tokens; ++t) {
        const float x = to_f32(K[seg.elem_off + static_cast<long long>(t) * L.d + dd]);
        mn = nan_min(mn, x);
        mx = nan_max(mx, x);
      }
    }
    const long long o = (static_cast<long long>(kv) * total + gb) * L.d + dd;
    lo[o] = mn;
    hi[o] = mx;
  }
}

// Token `pos[r]` of request r (block pos / B, slot pos % B) for every KV
// head: write k_new / v_new [R, hkv, D] into the cache and fold the key into
// the block's bounds (the first token of a block resets them).
template <typename T>
__global__ void __launch_bounds__(128) append_token_kernel(KVLayout L, int R, int total, const T* k_new, const T* v_new,
                                                           const int* pos, float* lo, float* hi, int* status) {
  const int r = blockIdx.x, kv = blockIdx.y;
  const int p = pos[r];
  const int j = p / L.b, t = p - j * L.b;
  if (p < 0 || j >= request_blocks(L, r)) {
    if (threadIdx.x == 0) report(status, kStatusBadBlockId);
    return;
  }
  const int s = t / L.page_size, ts = t - s * L.page_size;
  const BlockSeg seg = block_seg(L, r, kv, j, s);
  T* K = static_cast<T*>(const_cast<void*>(L.k));
  T* V = static_cast<T*>(const_cast<void*>(L.v));
  const long long dst = seg.elem_off + static_cast<long long>(ts) * L.d;
  const long long src = (static_cast<long long>(r) * L.hkv + kv) * L.d;
  const long long gb = (L.block_offsets ? L.block_offsets[r] : 0) + j;
  for (int dd = threadIdx.x; dd < L.d; dd += blockDim.x) {
    const T kx = k_new[src + dd];
    K[dst + dd] = kx;
    V[dst + dd] = v_new[src + dd];
    const float x = to_f32(kx);
    const long long o = (static_cast<long long>(kv) * total + gb) * L.d + dd;
    if (t == 0) {
      lo[o] = x;
      hi[o] = x;
    } else {
      lo[o] = nan_min(lo[o], x);
      hi[o] = nan_max(hi[o], x);
    }
  }
}

int launch_build_metadata(const KVLayout& L, int R, int total, int kv_dtype, float* lo, float* hi, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(total), static_cast<unsigned>(L.hkv));
  switch (kv_dtype) {
    case kF32: build_metadata_kernel<float><<<grid, 128, 0, stream>>>(L, R, total, lo, hi); break;
    case kF16: build_metadata_kernel<__half><<<grid, 128, 0, stream>>>(L, R, total, lo, hi); break;
    default: build_metadata_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(L, R, total, lo, hi); break;
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_append_token(const KVLayout& L, int R, int total, int kv_dtype, const void* k_new, const void* v_new,
                        const int* pos, float* lo, float* hi, int* status, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(R), static_cast<unsigned>(L.hkv));
  switch (kv_dtype) {
    case kF32:
      append_token_kernel<float><<<grid, 128, 0, stream>>>(L, R, total, static_cast<const float*>(k_new),
                                                           static_cast<const float*>(v_new), pos, lo, hi, status);
      break;
    case kF16:
      append_token_kernel<__half><<<grid, 128, 0, stream>>>(L, R, total, static_cast<const __half*>(k_new),
                                                            static_cast<const __half*>(v_new), pos, lo, hi, status);
      break;
    default:
      append_token_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(L, R, total,
                                                                   static_cast<const __nv_bfloat16*>(k_new),
                                                                   static_cast<const __nv_bfloat16*>(v_new), pos, lo,
                                                                   hi, status);
      break;
  }
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ predictor
// Next step's predicted block list from earlier selections (the policies of
// experiments/hisparse_cache_trace.py:40-57 `predict` and
// experiments/predictor_rank_trace.py:37-48 `interleave`):
//   previous_step   the first `budget` IDs of the previous step's ranking;
//   previous_layer  the first `budget` IDs of the previous layer's ranking;
//   rank_interleave slots alternate between the two rankings (the step's
//                   first), each slot taking its source's next ID not yet
//                   taken.
// A ranking is a selection row ordered by score, best first, ties to the
// lower block ID: by the rows' 64-bit order keys (descending, then position)
// when they are given, else the rows' own order. One CTA per row; the
// ranking is a counting rank; the interleave walks the slots in one thread
// with a bitmap of taken IDs. A source that runs out (the reference raises
// there) hands its slots to the other one; slots neither can fill get -1.

constexpr int kPredictThreads = 128;

__global__ void __launch_bounds__(kPredictThreads) predict_kernel(int policy, const int* step_ids,
                                                                  const unsigned long long* step_keys, int ks,
                                                                  const int* layer_ids,
                                                                  const unsigned long long* layer_keys, int kl,
                                                                  int n_blocks, int budget, int* out, int* status) {
  extern __shared__ int psm[];
  int* rs = psm;        // [ks] ranked step list
  int* rl = rs + ks;    // [kl] ranked layer list
  unsigned* seen = reinterpret_cast<unsigned*>(rl + kl);  // [(n_blocks + 31) / 32]
  const int row = blockIdx.x;
  const int nwords = (n_blocks + 31) / 32;
  auto rank_into = [&](const int* ids, const unsigned long long* keys, int k, int* dst) {
    if (ids == nullptr) return;
    const int* src = ids + static_cast<long long>(row) * k;
    const unsigned long long* ksrc = keys ? keys + static_cast<long long>(row) * k : nullptr;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      int rank = i;
      if (ksrc) {
        const unsigned long long ki = ksrc[i];
        rank = 0;
        for (int j = 0; j < k; ++j) {
          const unsigned long long kj = ksrc[j];
          rank += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
        }
      }
      dst[rank] = src[i];
    }
  };
  rank_into(step_ids, step_keys, ks, rs);
  rank_into(layer_ids, layer_keys, kl, rl);
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) seen[i] = 0u;
  __syncthreads();
  int* o = out + static_cast<long long>(row) * budget;
  if (policy != kPredictRankInterleave) {
    const int* src = policy == kPredictPreviousStep ? rs : rl;
    const int k = policy == kPredictPreviousStep ? ks : kl;
    for (int i = threadIdx.x; i < budget; i += blockDim.x) o[i] = i < k ? src[i] : -1;
    return;
  }
  if (threadIdx.x != 0) return;
  int ps = 0, pl = 0;
  auto take = [&](const int* src, int k, int& p) -> int {
    while (p < k) {
      const int b = src[p++];
      if (b < 0 || b >= n_blocks) {
        report(status, kStatusBadBlockId);
        continue;
      }
      if (!((seen[b >> 5] >> (b & 31)) & 1u)) {
        seen[b >> 5] |= 1u << (b & 31);
        return b;
      }
    }
    return -1;
  };
  for (int slot = 0; slot < budget; ++slot) {
    int b = (slot & 1) == 0 ? take(rs, ks, ps) : take(rl, kl, pl);
    if (b < 0) b = (slot & 1) == 0 ? take(rl, kl, pl) : take(rs, ks, ps);
    o[slot] = b;
  }
}

int launch_predict(int policy, const int* step_ids, const unsigned long long* step_keys, int ks, const int* layer_ids,
                   const unsigned long long* layer_keys, int kl, int rows, int n_blocks, int budget, int* out,
                   int* status, cudaStream_t stream) {
  const size_t smem = (static_cast<size_t>(ks) + kl) * 4 + static_cast<size_t>((n_blocks + 31) / 32) * 4;
  if (smem > 200 * 1024) return -1;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(predict_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  predict_kernel<<<rows, kPredictThreads, smem, stream>>>(policy, step_ids, step_keys, ks, layer_ids, layer_keys, kl,
                                                          n_blocks, budget, out, status);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace stk
