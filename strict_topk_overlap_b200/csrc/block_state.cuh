// Warp-level reduction of one shared-memory-staged KV block into an FP32
// softmax state. Shared by the block-state (speculation) and repair kernels.
//
// Layout ("half-warp tiles"): the block's K and V are [B, D] token-major in
// shared memory. Lane l belongs to half h = l / 16 and owns the DPH = D / 16
// dims [i*DPH, (i+1)*DPH) of q, K and V, i = l % 16. Half h takes the tokens
// 2s + h of every 32-token chunk, so each warp-wide 128-bit load covers two
// whole K (or V) rows.
//   QK: every lane forms 16 partial dot products (its dims, its half's
//       tokens); a transposed butterfly inside each half (xor 8, 4, 2, 1)
//       leaves the logit of token 2i + h in lane 16h + i.
//   PV: every lane accumulates its dims over its half's tokens, the weight of
//       token t broadcast from lane 16 (t % 2) + t / 2; one xor-16 exchange
//       adds the halves, so both halves end with the full numerator.
#pragma once
#include <type_traits>

#include "internal.cuh"

namespace stk {

// Widen N (a multiple of 8 for 16-bit, 4 for 32-bit types) consecutive
// elements at a 16-byte aligned shared-memory address to FP32.
template <typename T, int N>
__device__ __forceinline__ void load_row_slice(const T* p, float (&out)[N]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 x = *reinterpret_cast<const float4*>(p + i);
      out[i] = x.x; out[i + 1] = x.y; out[i + 2] = x.z; out[i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      const uint4 x = *reinterpret_cast<const uint4*>(p + i);
      const unsigned w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          out[i + 2 * j] = __uint_as_float(w[j] << 16);
          out[i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        } else {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
          const float2 f = __half22float2(h);
          out[i + 2 * j] = f.x;
          out[i + 2 * j + 1] = f.y;
        }
      }
    }
  }
}

// Transposed butterfly over the 16 lanes of each half-warp: on entry each
// lane holds 16 values v[0..15]; on exit lane 16h + i holds in v[0] the sum
// over its half's lanes of v[i].
__device__ __forceinline__ void transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, off);
    }
  }
}

// Reduces tokens [0, B) of the staged block. On entry (m, l, u, ua) hold the
// running state (m = -inf, l = 0, u = ua = 0 for a fresh block).
//   kModeFull : online softmax, m = max logit, l = sum exp(s - m), u = sum exp(s - m) v.
//   kModeMass : (m, l) only; V is not read.
//   kModeFixed: l = sum exp(s - frame), u = sum exp(s - frame) v, ua = sum |exp(s - frame) v|.
// Logits are s = (k . q) * scale in FP32; q holds this lane's DPH dims.
// On exit every lane holds u / ua for its dims (both halves agree).
// FULL32: B is a multiple of 32, so every 32-token chunk is full and the
// token loops carry no per-token predicates (which otherwise keep the
// compiler from hoisting the shared-memory loads; about 3x slower).
template <typename T, int DPH, int MODE, bool FULL32>
__device__ __forceinline__ void warp_block_state(const T* kst, const T* vst, int B, const float (&qf)[DPH],
                                                 float scale, float frame, float& m, float& l, float (&u)[DPH],
                                                 float (&ua)[DPH], int lane) {
  constexpr int D = 16 * DPH;
  constexpr bool kWantV = MODE != kModeMass;
  const int half = lane >> 4, li = lane & 15;
  // Half 0 carries the incoming numerators (rescaled with the running max),
  // half 1 starts from zero; the halves are added at the end.
  float pu[DPH], pa[DPH];
#pragma unroll
  for (int j = 0; j < DPH; ++j) {
    pu[j] = half ? 0.f : u[j];
    pa[j] = half ? 0.f : ua[j];
  }
#pragma unroll 1
  for (int t0 = 0; t0 < B; t0 += 32) {
    const int ntok = FULL32 ? 32 : min(32, B - t0);
    const T* ks = kst + static_cast<size_t>(t0 + half) * D + li * DPH;
    const T* vs = vst + static_cast<size_t>(t0 + half) * D + li * DPH;
    float p[16];
#pragma unroll
    for (int s2 = 0; s2 < 16; ++s2) {
      p[s2] = 0.f;
      if (FULL32 || 2 * s2 + half < ntok) {
        float kk[DPH];
        load_row_slice<T, DPH>(ks + static_cast<size_t>(2 * s2) * D, kk);
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < DPH; ++j) acc = fmaf(kk[j], qf[j], acc);
        p[s2] = acc;
      }
    }
    transpose_reduce16(p, lane);
    const int tok = 2 * li + half;  // token whose logit this lane holds
    const bool live = FULL32 || tok < ntok;
    const float s = live ? p[0] * scale : neg_inf();
    float w;
    if (MODE == kModeFixed) {
      w = live ? expf(s - frame) : 0.f;
      l += warp_sum(w);
    } else {
      const float mn = fmaxf(m, warp_max(s));
      const float alpha = expf(m - mn);
      w = live ? expf(s - mn) : 0.f;
      l = l * alpha + warp_sum(w);
      m = mn;
      if (kWantV) {
#pragma unroll
        for (int j = 0; j < DPH; ++j) pu[j] *= alpha;
      }
    }
    if (kWantV) {
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        const float wt = __shfl_sync(kFull, w, (lane & 16) + s2);
        if (FULL32 || 2 * s2 + half < ntok) {
          float vv[DPH];
          load_row_slice<T, DPH>(vs + static_cast<size_t>(2 * s2) * D, vv);
#pragma unroll
          for (int j = 0; j < DPH; ++j) {
            pu[j] = fmaf(wt, vv[j], pu[j]);
            if (MODE == kModeFixed) pa[j] += fabsf(wt * vv[j]);
          }
        }
      }
    }
  }
  if (kWantV) {
    // Add the two halves' numerators (both halves then hold the sum).
#pragma unroll
    for (int j = 0; j < DPH; ++j) {
      u[j] = pu[j] + __shfl_xor_sync(kFull, pu[j], 16);
      if (MODE == kModeFixed) ua[j] = pa[j] + __shfl_xor_sync(kFull, pa[j], 16);
    }
  }
}

// L2 prefetch of one block's K (and V). Called by one lane. A segment whose
// address or size is not a multiple of 16 bytes (odd head dims) is skipped:
// the bulk prefetch requires both, and it is only a hint.
template <typename T>
__device__ __forceinline__ void prefetch_block(const KVLayout& L, int r, int kv, long long bid, bool want_v) {
  const T* K = static_cast<const T*>(L.k);
  const T* V = static_cast<const T*>(L.v);
  const int nseg = block_nseg(L);
  for (int sg = 0; sg < nseg; ++sg) {
    const BlockSeg seg = block_seg(L, r, kv, bid, sg);
    const unsigned sb = static_cast<unsigned>(seg.tokens) * L.d * sizeof(T);
    const T* kp = K + seg.elem_off;
    const T* vp = V + seg.elem_off;
    if ((sb & 15u) != 0 || ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) & 15u) != 0) continue;
    bulk_prefetch_l2(kp, sb);
    if (want_v) bulk_prefetch_l2(vp, sb);
  }
}

// Issue the bulk copies of one (request, kv head, block) into a stage laid
// out as K [B, D] then V [B, D] (V skipped when want_v is false). Called by
// one lane; the caller arms `bar` with expect_tx for the block's bytes.
template <typename T>
__device__ __forceinline__ void issue_block_copy(const KVLayout& L, int r, int kv, long long bid, T* stage, bool want_v,
                                                 uint64_t* bar) {
  const T* K = static_cast<const T*>(L.k);
  const T* V = static_cast<const T*>(L.v);
  T* vs = stage + static_cast<size_t>(L.b) * L.d;
  const int nseg = block_nseg(L);
  for (int sg = 0; sg < nseg; ++sg) {
    const BlockSeg seg = block_seg(L, r, kv, bid, sg);
    const unsigned sb = static_cast<unsigned>(seg.tokens) * L.d * sizeof(T);
    const size_t dst = static_cast<size_t>(sg) * seg.tokens * L.d;
    bulk_g2s(stage + dst, K + seg.elem_off, sb, bar);
    if (want_v) bulk_g2s(vs + dst, V + seg.elem_off, sb, bar);
  }
}

}  // namespace stk
