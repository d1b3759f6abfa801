// Shared device helpers for the sm_100a strict-Top-K speculative decode kernels.
//
// Conventions used by every kernel in this library:
//  * Q is [rows, D] in f32/f16/bf16 (runtime dtype), read and widened to FP32.
//  * K/V are either dense [Hkv, N, B, D] or paged [pages, Hkv, page, D] with a
//    per-request block->page table; the element type is a template parameter.
//  * A "row" is one (request, query head) pair: row = r * Hq + h, kv = h / G.
//  * All softmax states are FP32 (m, l, u) with m the block max logit,
//    l = sum exp(s - m), u = sum exp(s - m) * v, and s = (k . q) * D^-0.5.
//  * Waits on asynchronous copies are bounded; a wait that runs out records
//    an error code in the optional status word and the kernel returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace stk {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Error codes written to the optional device status word (first writer wins).
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,    // a bounded mbarrier wait ran out
  kStatusBadBlockId = 2,     // a block id outside [0, N) was met
  kStatusShapeOverflow = 3,  // a per-row size exceeded the kernel's static bound
};

constexpr unsigned kFull = 0xffffffffu;
__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

__device__ __forceinline__ void report(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

__device__ __forceinline__ float load_any(const void* p, int dtype, long long i) {
  if (dtype == kF32) return static_cast<const float*>(p)[i];
  if (dtype == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ long long load_id(const void* p, int is64, long long i) {
  return is64 ? static_cast<const long long*>(p)[i] : static_cast<long long>(static_cast<const int*>(p)[i]);
}

__device__ __forceinline__ void store_id(void* p, int is64, long long i, long long v) {
  if (is64) static_cast<long long*>(p)[i] = v; else static_cast<int*>(p)[i] = static_cast<int>(v);
}

// Load N consecutive elements of T (N * sizeof(T) bytes, naturally aligned to
// the vector width) and widen them to FP32.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[N]) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  if constexpr (sizeof(T) == 4) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        float4 x = *reinterpret_cast<const float4*>(p + i);
        out[i] = x.x; out[i + 1] = x.y; out[i + 2] = x.z; out[i + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = to_f32(p[i]);
    }
  } else {
    static_assert(sizeof(T) == 2, "16-bit element expected");
    if constexpr (kBytes % 16 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 8) {
        uint4 x = *reinterpret_cast<const uint4*>(p + i);
        const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
        for (int j = 0; j < 8; ++j) out[i + j] = to_f32(e[j]);
      }
    } else if constexpr (kBytes % 8 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        uint2 x = *reinterpret_cast<const uint2*>(p + i);
        const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
        for (int j = 0; j < 4; ++j) out[i + j] = to_f32(e[j]);
      }
    } else if constexpr (kBytes % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        uint32_t x = *reinterpret_cast<const uint32_t*>(p + i);
        const T* e = reinterpret_cast<const T*>(&x);
        out[i] = to_f32(e[0]); out[i + 1] = to_f32(e[1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = to_f32(p[i]);
    }
  }
}

// q row slice [off, off + N) of a runtime-dtype tensor, widened to FP32.
template <int N>
__device__ __forceinline__ void load_q(const void* q, int dtype, long long off, float (&out)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) out[j] = load_any(q, dtype, off + j);
}

// Store N consecutive floats (16-byte aligned when N % 4 == 0).
template <int N>
__device__ __forceinline__ void store_vec(float* p, const float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = v[i];
  }
}

// ---------------------------------------------------------------- warp math
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}
__device__ __forceinline__ int warp_sum_int(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

// Transposed butterfly: on entry each lane holds 32 partial values v[0..31];
// on exit lane t holds in v[0] the sum over lanes of v[t]. The pairing order
// (xor 16, 8, 4, 2, 1) is the same tree as a per-value xor butterfly, so the
// result for every t is bit-identical to reducing v[t] alone that way.
template <typename F>
__device__ __forceinline__ void transpose_reduce32(F (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      F send = upper ? v[i] : v[i + off];
      F keep = upper ? v[i + off] : v[i];
      F recv = __shfl_xor_sync(kFull, send, off);
      v[i] = keep + recv;
    }
  }
}

// ---------------------------------------------------------------- async copies
// 1-D bulk copies (cp.async.bulk) global -> shared, completed on an mbarrier.
// Addresses and sizes must be 16-byte multiples; callers check on the host.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make initialised barriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Ask L2 to fetch `bytes` (16-byte aligned, multiple of 16) starting at
// `src`; no completion is tracked. Later bulk copies of the same bytes then
// hit L2 instead of waiting a full DRAM round trip.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Timeline probes: compiled in only with -DSTK_TRACE (a profiling build of
// the library); otherwise they vanish. STK_TRACE_AT(buf, i) stores the
// global nanosecond timer at buf[i].
#ifdef STK_TRACE
#define STK_TRACE_AT(buf, i) ((buf)[(i)] = global_ns())
#else
#define STK_TRACE_AT(buf, i) ((void)0)
#endif

// Bounded wait: try_wait (which itself blocks for a short, system-defined
// time) until the phase completes, giving up once c_wait_ns of wall time
// have passed (default 2 s, far above any legal copy time); a wait that gives
// up records kStatusWaitTimeout, then waits once more, with the same limit,
// for the copies still in flight on that barrier (so that its caller does not
// leave shared memory that a late copy could still write), and returns false.
//
// The limit is a runtime value: one copy per translation unit (internal
// linkage), all of them written by stk_set_wait_limit_ns for the current
// device through set_wait_limit_this_unit().
static __constant__ unsigned long long c_wait_ns = 2000000000ull;

static inline int set_wait_limit_this_unit(unsigned long long ns) {
  return static_cast<int>(cudaMemcpyToSymbol(c_wait_ns, &ns, sizeof(ns)));
}

__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, unsigned parity, unsigned long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
#ifdef STK_WAIT_BACKOFF
    __nanosleep(STK_WAIT_BACKOFF);
#endif
    if (global_ns() - t0 > limit) return false;
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int* status) {
  const unsigned long long limit = c_wait_ns;
  if (mbar_wait_for(bar, parity, limit)) return true;
  report(status, kStatusWaitTimeout);
  mbar_wait_for(bar, parity, limit);  // drain: bounded as well
  return false;
}

// ---------------------------------------------------------------- clusters
// Split cluster barrier. The CTAs of a cluster are co-scheduled but need not
// have started when a sibling runs, so a CTA arrives here first thing and
// waits before its first distributed-shared-memory access; the next
// cluster-wide barrier then starts a new phase. Every thread of every CTA
// must execute each arrive and wait once (warp-converged).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// its predecessor on the stream is still running; pdl_wait() blocks until
// that predecessor has completed and its writes are visible (a no-op for an
// ordinary launch). pdl_release() lets this kernel's own dependents launch
// early. Code before pdl_wait() must not read the predecessor's outputs.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- KV layout
// Addressing for one (request, kv head, block). A block is `nseg` segments of
// `seg_tokens` contiguous tokens; dense layouts have one segment per block,
// paged layouts one segment per page.
struct KVLayout {
  const void* k;
  const void* v;
  int hkv, n, b, d;            // n = blocks per request (dense), b = tokens per block
  const int* page_table;       // paged: [total_blocks * pages_per_block] page ids; null = dense
  const int* block_offsets;    // [R + 1] global block offsets per request (paged / batched); may be null
  int page_size;               // paged: tokens per page (divides b)
  long long kv_request_stride; // dense, batched: elements between requests' KV (0 for a single request)
};

struct BlockSeg {
  long long elem_off;  // element offset of the segment start within K (same for V)
  int tokens;
};

__device__ __forceinline__ int request_blocks(const KVLayout& L, int r) {
  return L.block_offsets ? (L.block_offsets[r + 1] - L.block_offsets[r]) : L.n;
}

// Segment `s` of block `bid` of request `r`, kv head `kv`.
__device__ __forceinline__ BlockSeg block_seg(const KVLayout& L, int r, int kv, long long bid, int s) {
  BlockSeg out;
  if (L.page_table == nullptr) {
    out.elem_off = r * L.kv_request_stride + ((static_cast<long long>(kv) * L.n + bid) * L.b) * L.d;
    out.tokens = L.b;
  } else {
    const int ppb = L.b / L.page_size;
    const long long gb = static_cast<long long>(L.block_offsets ? L.block_offsets[r] : 0) + bid;
    const long long page = L.page_table[gb * ppb + s];
    out.elem_off = ((page * L.hkv + kv) * L.page_size) * L.d;
    out.tokens = L.page_size;
  }
  return out;
}

__device__ __forceinline__ int block_nseg(const KVLayout& L) {
  return L.page_table == nullptr ? 1 : L.b / L.page_size;
}

}  // namespace stk
