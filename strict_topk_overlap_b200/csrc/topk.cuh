// Strict Top-K building blocks shared by the selection kernels (select.cu)
// and the fused decode-step kernel (step.cu): order keys, the register radix
// select, the exact FP64 rescoring of a block in the library's fixed order,
// and the second stage of the two-stage (interval) selection.
//
// Replaces the torch.topk call of selector.py:43 / gqa.py:161 (and the
// scoring half it consumes, selector.py:8-20, gqa.py:15-26). The score order
// and the interval argument are described in select.cu.
#pragma once

#include "internal.cuh"

// Phase probes of bounded_select_core (profiling builds of a caller define it).
#ifndef STK_TOPK_PROBE
#define STK_TOPK_PROBE(ev) ((void)0)
#endif

namespace stk {

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const void* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
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
// ascending position order; ties (equal keys) go to the lower position.
//
// MSB-first 4-bit digits over the bits in which the keys differ (the common
// prefix is skipped). One pass = one block barrier: every thread counts its
// candidate keys per digit in 8-bit fields, repacks them as eight 32-bit
// words of 16-bit fields summed over the warp by redux.sync, lane 0 stores
// the warp's counts (double-buffered by pass parity), and after the barrier
// every warp adds the warps' counts itself and finds the bin holding the
// K-th key, so no second barrier is needed. Once the boundary bin holds at
// most one key per thread, its keys are compacted into shared memory and the
// remaining passes run over that short list. The loop ends as soon as the
// boundary bin's keys are all selected. A final block scan places every
// selected ID at its ascending output position.
constexpr int kSelMaxWarps = 16;

// Given this thread's per-digit counts (8-bit fields, bins 0..7 in lo8,
// 8..15 in hi8), sum them over the block and return (bin, keys above it,
// keys in it) for the K-th largest; `buf` is this pass's count buffer.
__device__ __forceinline__ void radix_boundary(unsigned long long lo8, unsigned long long hi8, unsigned (*buf)[8],
                                               int kk, int& bin, int& above, int& cnt) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  unsigned w[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const unsigned xl = static_cast<unsigned>(lo8 >> (16 * i)), xh = static_cast<unsigned>(hi8 >> (16 * i));
    w[i] = (xl & 0xffu) | ((xl & 0xff00u) << 8);
    w[4 + i] = (xh & 0xffu) | ((xh & 0xff00u) << 8);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = __reduce_add_sync(kFull, w[i]);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) buf[warp][i] = w[i];
  }
  __syncthreads();
  // Lane i (< 16) takes bin 15 - i: an inclusive lane scan counts keys in
  // bins >= 15 - i. Every warp does this (same result), no second barrier.
  unsigned c = 0;
  if (lane < 16) {
    const int b = 15 - lane;
    for (int ww = 0; ww < nw; ++ww) c += (buf[ww][b >> 1] >> ((b & 1) * 16)) & 0xffffu;
  }
  unsigned inc = c;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) {
    const unsigned y = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += y;
  }
  const unsigned excl = inc - c;
  const unsigned hit = __ballot_sync(kFull, lane < 16 && excl < static_cast<unsigned>(kk) && inc >= static_cast<unsigned>(kk));
  const int src = hit ? __ffs(hit) - 1 : 0;  // exactly one lane crosses when kk <= candidates
  bin = 15 - src;
  above = static_cast<int>(__shfl_sync(kFull, excl, src));
  cnt = static_cast<int>(__shfl_sync(kFull, c, src));
}

template <int E, typename IdOf>
__device__ void select_registers(const unsigned long long (&key)[E], int n, int topk, IdOf id_of, int* out,
                                 unsigned long long* keys_out) {
  static_assert(E <= 255, "per-thread digit counts use 8-bit fields");
  __shared__ unsigned wc[2][kSelMaxWarps][8];
  __shared__ unsigned long long sh_or, sh_k0;
  __shared__ unsigned long long clist[512];  // compacted boundary-bin keys (<= one per thread)
  __shared__ unsigned warp_tot[kSelMaxWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = blockDim.x >> 5;
  const int beg = tid * E;

  if (tid == 0) { sh_or = 0; sh_k0 = key[0]; }
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
    int shift = (hb / 4) * 4;
    int parity = 0;
    bool compacted = false;
    int nlist = 0;
#pragma unroll 1
    for (; shift >= 0; shift -= 4, parity ^= 1) {
      unsigned long long lo8 = 0, hi8 = 0;
      if (!compacted) {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if (beg + j < n && (key[j] & mask) == prefix) {
            const unsigned d = static_cast<unsigned>(key[j] >> shift) & 15u;
            const unsigned long long inc = 1ull << ((d & 7u) * 8u);
            if (d < 8) lo8 += inc; else hi8 += inc;
          }
        }
      } else if (tid < nlist) {
        const unsigned long long kt = clist[tid];
        if ((kt & mask) == prefix) {
          const unsigned d = static_cast<unsigned>(kt >> shift) & 15u;
          const unsigned long long inc = 1ull << ((d & 7u) * 8u);
          if (d < 8) lo8 += inc; else hi8 += inc;
        }
      }
      int bin, above, cnt;
      radix_boundary(lo8, hi8, wc[parity], kk, bin, above, cnt);
      prefix |= static_cast<unsigned long long>(bin) << shift;
      mask |= 0xFull << shift;
      kk -= above;
      if (cnt == kk) { take_all = true; break; }
      if (!compacted && cnt <= static_cast<int>(blockDim.x) && cnt <= 512 && shift >= 4) {
        // Compact the boundary bin's keys (prefix now includes this digit).
        unsigned mine = 0;
#pragma unroll
        for (int j = 0; j < E; ++j) mine += (beg + j < n && (key[j] & mask) == prefix) ? 1u : 0u;
        unsigned inc = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(kFull, inc, o);
          if (lane >= o) inc += y;
        }
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        unsigned pos = inc - mine;
        for (int w2 = 0; w2 < warp; ++w2) pos += warp_tot[w2];
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (beg + j < n && (key[j] & mask) == prefix) clist[pos++] = key[j];
        nlist = cnt;
        compacted = true;
        __syncthreads();
      }
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
  __syncthreads();
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  unsigned excl = inc - packed;
  for (int w = 0; w < warp; ++w) excl += warp_tot[w];
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

// Exact FP64 score of (request r, query head h, metadata row gb) in the
// fixed order of the file header: lane l sums dims [l*c, (l+1)*c) with FP64
// FMA from zero, then the xor butterfly 16, 8, 4, 2, 1. Warp-collective.
__device__ __forceinline__ double exact_head_score(const SelectArgs& a, int r, int h, long long gb, int lane) {
  const int D = a.d, c = (D + 31) / 32;
  const int G = a.hq / a.hmeta;
  const long long qoff = (static_cast<long long>(r) * a.hq + h) * D;
  const long long moff = (static_cast<long long>(h / G) * a.total_blocks + gb) * D;
  double acc = 0.0;
  const int d1 = min((lane + 1) * c, D);
  for (int dd = lane * c; dd < d1; ++dd) {
    const double qv = static_cast<double>(load_any(a.q, a.q_dtype, qoff + dd));
    acc = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? a.hi[moff + dd] : a.lo[moff + dd]), acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
  return acc;
}

// Exact order key of selection row hs (a query head, or a KV head summing
// its query heads' scores in ascending order) at metadata row gb.
__device__ __forceinline__ unsigned long long exact_row_key(const SelectArgs& a, int r, int hs, long long gb,
                                                            int lane) {
  if (!a.group_select) return order_key(exact_head_score(a, r, hs, gb, lane));
  const int G = a.hq / a.hmeta;
  double grp = 0.0;
  for (int g = 0; g < G; ++g) grp = __dadd_rn(grp, exact_head_score(a, r, hs * G + g, gb, lane));
  return order_key(grp);
}

// The same exact key with the row's query heads staged in shared memory as
// FP32 (qsm [heads][D], heads = G for group rows, else 1) and the block's
// metadata loaded once for all heads: one memory round trip per block. For
// the interval path only (D <= 256, so each lane owns at most 8 dims).
__device__ __forceinline__ unsigned long long exact_row_key_staged(const SelectArgs& a, int hs, long long gb, int lane,
                                                                   const float* qsm) {
  const int D = a.d, c = (D + 31) / 32;
  const int G = a.hq / a.hmeta;
  const int heads = a.group_select ? G : 1;
  const int mh = a.group_select ? hs : hs / G;
  const long long moff = (static_cast<long long>(mh) * a.total_blocks + gb) * D;
  float lo_r[8], hi_r[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int dd = lane * c + e;
    lo_r[e] = (e < c && dd < D) ? a.lo[moff + dd] : 0.f;
    hi_r[e] = (e < c && dd < D) ? a.hi[moff + dd] : 0.f;
  }
  double grp = 0.0;
  for (int g = 0; g < heads; ++g) {
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int dd = lane * c + e;
      if (e < c && dd < D) {
        const double qv = static_cast<double>(qsm[g * D + dd]);
        acc = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? hi_r[e] : lo_r[e]), acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
    if (!a.group_select) return order_key(acc);
    grp = __dadd_rn(grp, acc);
  }
  return order_key(grp);
}

// Exact order keys of NK metadata rows gb[] (live[] false: skipped, key 0)
// with the rows' metadata loads all in flight before any arithmetic; each
// key is exact_row_key_staged's, computed in the same order.
template <int NK>
__device__ __forceinline__ void exact_row_keys_staged(const SelectArgs& a, int hs, const long long (&gb)[NK],
                                                      const bool (&live)[NK], int lane, const float* qsm,
                                                      unsigned long long (&key)[NK]) {
  const int D = a.d, c = (D + 31) / 32;
  const int G = a.hq / a.hmeta;
  const int heads = a.group_select ? G : 1;
  const int mh = a.group_select ? hs : hs / G;
  float lo_r[NK][8], hi_r[NK][8];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const long long moff = (static_cast<long long>(mh) * a.total_blocks + gb[k]) * D;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int dd = lane * c + e;
      const bool ok = live[k] && e < c && dd < D;
      lo_r[k][e] = ok ? a.lo[moff + dd] : 0.f;
      hi_r[k][e] = ok ? a.hi[moff + dd] : 0.f;
    }
  }
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    double grp = 0.0, one = 0.0;
    for (int g = 0; g < heads; ++g) {
      double acc = 0.0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int dd = lane * c + e;
        if (e < c && dd < D) {
          const double qv = static_cast<double>(qsm[g * D + dd]);
          acc = __fma_rn(qv, static_cast<double>(qv >= 0.0 ? hi_r[k][e] : lo_r[k][e]), acc);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
      if (!a.group_select) { one = acc; break; }
      grp = __dadd_rn(grp, acc);
    }
    key[k] = live[k] ? order_key(a.group_select ? grp : one) : 0ull;
  }
}

constexpr int kHistBins = 2048;
constexpr int kUncMax = 256;  // straddling blocks resolved by ranking; more take the radix path
constexpr int kQStage = 2048;  // staged query floats per Top-K CTA (heads x D)
constexpr unsigned char kClsOut = 0, kClsIn = 1, kClsUnc = 2;

__device__ __forceinline__ int hist_bin(float x, float mn, float scale) {
  const int b = __float2int_rd((x - mn) * scale);  // monotone in x; NaN (0 * inf) maps to 0
  return min(kHistBins - 1, max(0, b));
}

// Block-wide exclusive scan of one unsigned per thread over NT (<= 1024)
// threads; returns the exclusive prefix and writes the block total to
// *total. One barrier: each warp scans the per-warp totals itself with
// shuffles.
template <int NT>
__device__ __forceinline__ unsigned block_exclusive_scan(unsigned v, unsigned* wsum, unsigned* total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  const unsigned x = lane < NW ? wsum[lane] : 0u;
  unsigned sc = x;
#pragma unroll
  for (int o = 1; o < NW; o <<= 1) {
    const unsigned y = __shfl_up_sync(kFull, sc, o);
    if (lane >= o) sc += y;
  }
  *total = __shfl_sync(kFull, sc, NW - 1);
  return __shfl_sync(kFull, sc - x, warp) + inc - v;
}

// The second stage of the two-stage selection, for selection row `row` of
// `a`, run by every thread of the calling CTA (NT threads, NT <= 512 and
// E * NT >= the row's blocks, checked by the caller). `qsm` holds
// the row's query heads as FP32 ([G][D] for a group row, [D] otherwise) when
// `q_staged`; otherwise exact rescoring reads q from global memory. The
// interval bounds are read through L2 (ld.global.cg), so they may come from
// other CTAs of the calling kernel. Writes the row's IDs ascending (and,
// with a.keys_out, their exact order keys).
// With kPoll, the row's intervals are still being written by other CTAs of
// the calling kernel, each as one 8-byte store into a slot that was zero:
// a slot reads zero until its interval lands (no valid interval is all-zero
// bits: its lower end, rounded down, is never +0), so each thread re-reads
// its zero slots until they fill (bounded by the wait limit).
// ids_smem (optional): the IDs are also written there, in output order.
// hook (optional): hook.sure_in(id) runs once per block known to be selected
// as soon as the intervals classify it (before any exact rescoring), and
// hook.selected(pos, id, was_sure_in) once per selected block as its output
// position is written; both on the thread that owns the block.
// stage (optional): shared memory for n + n / 16 intervals. The row's
// intervals are then read (or, with kPoll, polled) with coalesced loads
// (thread t takes t, t + NT, ...) into it, one 8-byte slot of padding after
// every 16, so that each thread's E contiguous intervals read back without
// bank conflicts; read directly, each warp load of them spans E * 32 slots.
struct NoSelectHook {
  __device__ void sure_in(int) const {}
  __device__ void selected(int, int, bool) const {}
};
template <int E, int NT, bool kPoll = false, typename Hook = NoSelectHook>
__device__ void bounded_select_core(const SelectArgs& a, int row, const float* qsm, bool q_staged,
                                    int* ids_smem = nullptr, const Hook& hook = Hook(), float2* stage = nullptr) {
  static_assert(NT % 32 == 0 && NT <= 512 && kHistBins % NT == 0, "selection block shape");
  constexpr int NW = NT / 32;
  __shared__ unsigned hist[kHistBins];  // low 16 bits: lower ends; high 16 bits: upper ends
  __shared__ unsigned wsum[2][kSelMaxWarps];
  __shared__ float wmn[kSelMaxWarps], wmx[kSelMaxWarps];
  __shared__ int s_bt, s_bu;
  __shared__ int unc_pos[kUncMax];
  __shared__ unsigned long long unc_key[kUncMax];
  __shared__ unsigned char unc_sel[kUncMax];
  __shared__ unsigned char cls_s[512 * E];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nw = NW;
  const int r = row / a.hsel, hs = row - r * a.hsel;
  const int off = a.block_offsets ? a.block_offsets[r] : 0;
  const int n = a.block_offsets ? a.block_offsets[r + 1] - off : a.n;
  const int K = a.topk;
  int* out = a.ids_out + static_cast<long long>(row) * K;
  float2* src = a.bounds + static_cast<long long>(hs) * a.total_blocks + off;
  const int beg = tid * E;
  const float inf = __int_as_float(0x7f800000);
  auto row_key = [&](long long gb) {
    return q_staged ? exact_row_key_staged(a, hs, gb, lane, qsm) : exact_row_key(a, r, hs, gb, lane);
  };

  {
#pragma unroll
    for (int i = tid; i < kHistBins; i += NT) hist[i] = 0u;
    if (tid == 0) { s_bt = 0; s_bu = 0; }
    float lo_[E], up_[E];
    float mn = inf, mx = -inf;
    if constexpr (kPoll) {
      // With a stage, thread t polls slots t, t + NT, ... (coalesced) and the
      // slots are then exchanged through shared memory as in the plain path.
      const int pb = stage != nullptr ? tid : beg;
      const int ps = stage != nullptr ? NT : 1;
      unsigned long long raw[E];
#pragma unroll
      for (int j = 0; j < E; ++j) raw[j] = pb + j * ps < n ? ld_relaxed_gpu_u64(src + pb + j * ps) : 1ull;
      bool missing = false;
#pragma unroll
      for (int j = 0; j < E; ++j) missing |= raw[j] == 0ull;
      if (missing) {
        const unsigned long long t0 = global_ns();
        while (missing) {
          __nanosleep(100);
          missing = false;
#pragma unroll
          for (int j = 0; j < E; ++j) {
            if (raw[j] == 0ull) raw[j] = ld_relaxed_gpu_u64(src + pb + j * ps);
            missing |= raw[j] == 0ull;
          }
          if (missing && global_ns() - t0 > c_wait_ns) {
            report(a.status, kStatusWaitTimeout);
            break;
          }
        }
      }
      if (stage != nullptr) {
        unsigned long long* st64 = reinterpret_cast<unsigned long long*>(stage);
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const int i = tid + j * NT;
          if (i < n) st64[i + (i >> 4)] = raw[j];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const int i = beg + j;
          raw[j] = i < n ? st64[i + (i >> 4)] : 1ull;
        }
      }
#pragma unroll
      for (int j = 0; j < E; ++j) {
        lo_[j] = inf;
        up_[j] = -inf;
        if (beg + j < n) {
          lo_[j] = __uint_as_float(static_cast<unsigned>(raw[j]));
          up_[j] = __uint_as_float(static_cast<unsigned>(raw[j] >> 32));
          if (raw[j] == 0ull) { lo_[j] = -inf; up_[j] = inf; }
          if (lo_[j] > -inf) mn = fminf(mn, lo_[j]);
          if (up_[j] < inf) mx = fmaxf(mx, up_[j]);
        }
      }
    } else {
      if (stage != nullptr) {
        float2 t[E];
#pragma unroll
        for (int k = 0; k < E; ++k) {
          const int i = k * NT + tid;
          if (i < n) t[k] = __ldcg(src + i);
        }
#pragma unroll
        for (int k = 0; k < E; ++k) {
          const int i = k * NT + tid;
          if (i < n) stage[i + (i >> 4)] = t[k];
        }
        __syncthreads();
      }
#pragma unroll
      for (int j = 0; j < E; ++j) {
        lo_[j] = inf;
        up_[j] = -inf;
        if (beg + j < n) {
          const int i = beg + j;
          const float2 v = stage != nullptr ? stage[i + (i >> 4)] : __ldcg(src + i);
          lo_[j] = v.x;
          up_[j] = v.y;
          if (v.x > -inf) mn = fminf(mn, v.x);
          if (v.y < inf) mx = fmaxf(mx, v.y);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(kFull, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    }
    if (lane == 0) { wmn[warp] = mn; wmx[warp] = mx; }
    __syncthreads();
    STK_TOPK_PROBE(0);
    mn = lane < NW ? wmn[lane] : inf;
    mx = lane < NW ? wmx[lane] : -inf;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // every lane ends with the block's extremes
      mn = fminf(mn, __shfl_xor_sync(kFull, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    }
    float scale = 0.f;
    if (mx > mn) scale = fminf(static_cast<float>(kHistBins) / (mx - mn), 0x1p100f);
    if (!(mn < inf)) mn = 0.f;

    if (n == K) {
      // Everything is selected.
      for (int i = tid; i < n; i += NT) {
        out[i] = a.id_base + i;
        if (ids_smem) ids_smem[i] = a.id_base + i;
        hook.selected(i, a.id_base + i, false);
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) {
        if (beg + j < n) {
          atomicAdd(&hist[hist_bin(lo_[j], mn, scale)], 1u);
          atomicAdd(&hist[hist_bin(up_[j], mn, scale)], 1u << 16);
        }
      }
      __syncthreads();
      STK_TOPK_PROBE(1);
      // Suffix counts: thread t owns bins [kHistBins - (t+1)*per, kHistBins - t*per), scanned downward.
      constexpr int per = kHistBins / NT;
      const int top = kHistBins - 1 - tid * per;
      unsigned hv[per], loc = 0;
#pragma unroll
      for (int i = 0; i < per; ++i) {
        hv[i] = hist[top - i];
        loc += hv[i];
      }
      unsigned tot;
      unsigned c = block_exclusive_scan<NT>(loc, wsum[0], &tot);
#pragma unroll
      for (int i = 0; i < per; ++i) {
        const unsigned h = hv[i];
        const unsigned lo_before = c & 0xffffu, up_before = c >> 16;
        c += h;
        if (lo_before < static_cast<unsigned>(K) && (c & 0xffffu) >= static_cast<unsigned>(K)) s_bt = top - i;
        if (up_before < static_cast<unsigned>(K + 1) && (c >> 16) >= static_cast<unsigned>(K + 1)) s_bu = top - i;
      }
      __syncthreads();
      STK_TOPK_PROBE(2);
      const int bt = s_bt, bu = s_bu;
      // Classify: in (lower-end bin above U's bin), out (upper-end bin below T's bin), straddling.
      unsigned char cls[E];
      unsigned n_in = 0, n_unc = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        cls[j] = kClsOut;
        if (beg + j < n) {
          if (hist_bin(lo_[j], mn, scale) > bu) cls[j] = kClsIn;
          else if (hist_bin(up_[j], mn, scale) >= bt) cls[j] = kClsUnc;
          n_in += cls[j] == kClsIn;
          n_unc += cls[j] == kClsUnc;
        }
      }
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (cls[j] == kClsIn) hook.sure_in(a.id_base + beg + j);
      const unsigned packed = (n_in << 16) | n_unc;
      const unsigned ex = block_exclusive_scan<NT>(packed, wsum[1], &tot);
      const int total_in = static_cast<int>(tot >> 16), total_unc = static_cast<int>(tot & 0xffffu);
      STK_TOPK_PROBE(3);
      int need = K - total_in;
      if (need < 0 || need > total_unc) {  // cannot happen for valid intervals
        if (tid == 0) report(a.status, kStatusShapeOverflow);
        need = max(0, min(need, total_unc));
      }
      if (need < total_unc && total_unc > kUncMax) {
        // Many straddling blocks (ties, flat metadata): exact keys for all of
        // them, written over the row's bounds slots (every thread has read its
        // own), then the radix select over keys in = max, out = 0, straddling
        // = exact (sure-in blocks are at most K, so all of them are taken).
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (beg + j < n) cls_s[beg + j] = cls[j];
        __syncthreads();
        unsigned long long* scratch = reinterpret_cast<unsigned long long*>(src);
        for (int pos = warp; pos < n; pos += nw) {
          if (cls_s[pos] != kClsUnc) continue;
          const unsigned long long k = row_key(static_cast<long long>(off) + pos);
          if (lane == 0) scratch[pos] = k;
        }
        __syncthreads();
        unsigned long long key[E];
#pragma unroll
        for (int j = 0; j < E; ++j)
          key[j] = cls[j] == kClsIn ? ~0ull : (cls[j] == kClsUnc ? __ldcg(scratch + beg + j) : 0ull);
        const int base = a.id_base;
        select_registers<E>(key, n, K, [base](int i) { return base + i; }, out, nullptr);
        __syncthreads();  // this CTA's ID writes are visible to the whole CTA
        for (int i = tid; i < K; i += NT) {
          if (ids_smem) ids_smem[i] = out[i];
          hook.selected(i, out[i], cls_s[out[i] - a.id_base] == kClsIn);
        }
      } else {
        unsigned idx = ex & 0xffffu;
        if (need < total_unc) {
#pragma unroll
          for (int j = 0; j < E; ++j) {
            if (cls[j] == kClsUnc) unc_pos[idx++] = beg + j;
          }
          __syncthreads();
          for (int t = warp; t < total_unc; t += nw) {
            const unsigned long long k = row_key(static_cast<long long>(off) + unc_pos[t]);
            if (lane == 0) unc_key[t] = k;
          }
          __syncthreads();
          for (int t = tid; t < total_unc; t += NT) {
            const unsigned long long kt = unc_key[t];
            int rank = 0;
            for (int j = 0; j < total_unc; ++j) {
              const unsigned long long kj = unc_key[j];
              rank += (kj > kt || (kj == kt && j < t)) ? 1 : 0;
            }
            unc_sel[t] = rank < need ? 1 : 0;
          }
          __syncthreads();
        }
        STK_TOPK_PROBE(4);
        // Final flags and ascending output positions.
        idx = ex & 0xffffu;
        unsigned mine = 0;
        bool sel[E];
#pragma unroll
        for (int j = 0; j < E; ++j) {
          sel[j] = cls[j] == kClsIn;
          if (cls[j] == kClsUnc) {
            sel[j] = need == total_unc ? true : unc_sel[idx] != 0;
            ++idx;
          }
          mine += sel[j] ? 1u : 0u;
        }
        unsigned all;
        unsigned pos = block_exclusive_scan<NT>(mine, wsum[0], &all);
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if (sel[j]) {
            if (ids_smem) ids_smem[pos] = a.id_base + beg + j;
            hook.selected(static_cast<int>(pos), a.id_base + beg + j, cls[j] == kClsIn);
            out[pos++] = a.id_base + beg + j;
          }
        }
      }
    }
  }
  if (a.keys_out) {
    __syncthreads();  // this CTA's ID writes are visible to the whole CTA
    if (q_staged) {
      // Four keys per warp at a time: their metadata loads overlap.
      constexpr int NK = 4;
      for (int t0 = warp; t0 < K; t0 += NK * nw) {
        long long gbk[NK];
        bool lk[NK];
        unsigned long long kk[NK];
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int t = t0 + k * nw;
          lk[k] = t < K;
          gbk[k] = lk[k] ? static_cast<long long>(off) + (out[t] - a.id_base) : 0;
        }
        exact_row_keys_staged<NK>(a, hs, gbk, lk, lane, qsm, kk);
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < NK; ++k)
            if (lk[k]) a.keys_out[static_cast<long long>(row) * K + t0 + k * nw] = kk[k];
        }
      }
    } else {
      for (int t = warp; t < K; t += nw) {
        const int pos = out[t] - a.id_base;
        const unsigned long long k = row_key(static_cast<long long>(off) + pos);
        if (lane == 0) a.keys_out[static_cast<long long>(row) * K + t] = k;
      }
    }
  }
}

}  // namespace stk
