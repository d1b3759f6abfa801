// K2: per-block softmax states over lists of KV blocks, plus the per-row
// grouping / merge epilogues of speculation.
//
// Replaces kernels.py:42-71 (_partial), :74-91 (_merge), :94-117 (_group),
// :263-278 (_mass_only), :281-309 (_compact_group), :312-356 (_compact_values),
// :384-407 (_wrong_aggregate); gqa.py:29-59 (_partial incl. REPAIR slot
// search); gqa_hierarchical.py:22-52 (_packed_partials, per-block states).
//
// Design: one warp owns one (row, block) job at a time. Each warp keeps a
// private ring of NST shared-memory stages; lane 0 streams 32-token K/V
// chunks into them with 1-D bulk copies (cp.async.bulk) completed on a
// per-stage mbarrier, while the whole warp reduces the previous chunk:
//   QK : lane l owns dims [l*DPL, (l+1)*DPL); 32 token partials are reduced
//        with one transposed butterfly, leaving token t's logit in lane t;
//   PV : lane l accumulates its DPL output dims over the chunk's tokens.
// Misaligned or odd shapes take a plain-load generic kernel with the same math.

#include "internal.cuh"

namespace stk {



struct JobInfo {
  int row, slot;
  long long bid;
  bool active;
};

// Whole-warp job resolution (uniform result in every lane).
__device__ __forceinline__ JobInfo resolve_job(const JobArgs& a, long long job, int lane) {
  JobInfo j;
  j.row = static_cast<int>(job / a.s);
  j.slot = static_cast<int>(job - static_cast<long long>(j.row) * a.s);
  j.bid = load_id(a.ids, a.ids64, job);
  bool act = true;
  if (a.active_mode == 1) act = a.active[j.row] != 0;
  else if (a.active_mode == 2) act = a.active[job] != 0;
  if (a.active_invert) act = !act;
  if (j.bid < 0) act = false;
  if (a.pred != nullptr) {
    int found = -1;
    for (int p = lane; p < a.sp; p += 32) {
      if (load_id(a.pred, a.pred64, static_cast<long long>(j.row) * a.sp + p) == j.bid) found = max(found, p);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(kFull, found, o));
    if (a.slot_out && lane == 0) a.slot_out[job] = found;
    if (found >= 0) act = false;
  }
  if (act) {
    const int r = j.row / a.hq;
    const int nb = request_blocks(a.L, r);
    if (j.bid >= nb) {
      if (lane == 0) report(a.status, kStatusBadBlockId);
      act = false;
    }
  }
  j.active = act;
  return j;
}

// Outputs of a job that reads no KV: the reference writes (-inf, 0, 0).
__device__ __forceinline__ void write_inactive(const JobArgs& a, long long job, int lane) {
  if (a.pred != nullptr) return;  // repair scratch: hits keep no state
  if (a.mode != kModeFixed) {
    if (lane == 0) {
      a.m[job] = neg_inf();
      a.l[job] = 0.f;
    }
    if (a.mode == kModeFull)
      for (int dd = lane; dd < a.d; dd += 32) a.u[job * a.d + dd] = 0.f;
  } else {
    if (lane == 0 && a.l) a.l[job] = 0.f;
    for (int dd = lane; dd < a.d; dd += 32) {
      a.u[job * a.d + dd] = 0.f;
      if (a.uabs) a.uabs[job * a.d + dd] = 0.f;
    }
  }
}

// ------------------------------------------------------------------ fast path

template <typename T, int DPL, int MODE, int NST>
__global__ void __launch_bounds__(128) jobs_fast_kernel(JobArgs a) {
  constexpr int D = 32 * DPL;
  constexpr int kChunkElems = 32 * D;
  constexpr bool kWantV = MODE != kModeMass;
  constexpr int kStageElems = kChunkElems * (kWantV ? 2 : 1);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ uint64_t bars[4 * NST];
  __shared__ int info_row[4 * NST], info_slot[4 * NST], info_chunk[4 * NST];
  __shared__ long long info_bid[4 * NST];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  T* stages = reinterpret_cast<T*>(smem_raw) + static_cast<size_t>(warp) * NST * kStageElems;
  uint64_t* bar = bars + warp * NST;
  int* irow = info_row + warp * NST;
  int* islot = info_slot + warp * NST;
  int* ichunk = info_chunk + warp * NST;
  long long* ibid = info_bid + warp * NST;

  if (lane == 0) {
    for (int st = 0; st < NST; ++st) mbar_init(&bar[st], 1);
    fence_barrier_init();
  }
  __syncwarp();

  const long long njobs = static_cast<long long>(a.rows) * a.s;
  const long long W = static_cast<long long>(gridDim.x) * wpc;
  const int nchunks = (a.L.b + 31) / 32;
  const int nseg_page = (a.L.page_table != nullptr) ? a.L.page_size : 0;

  // Issue cursor (uniform across the warp).
  long long ijob = static_cast<long long>(blockIdx.x) * wpc + warp;
  int ichunk_cur = 0;
  JobInfo iinfo;
  auto advance_to_active = [&](bool first) {
    if (!first) {
      if (++ichunk_cur < nchunks) return;
      ichunk_cur = 0;
      ijob += W;
    }
    while (ijob < njobs) {
      iinfo = resolve_job(a, ijob, lane);
      if (iinfo.active) return;
      write_inactive(a, ijob, lane);
      ijob += W;
    }
  };
  auto issue = [&](int st) {
    if (ijob >= njobs) {
      if (lane == 0) irow[st] = -1;
      return;
    }
    if (lane == 0) {
      const int r = iinfo.row / a.hq;
      const int kv = (iinfo.row - r * a.hq) / a.g;
      const int t0 = ichunk_cur * 32;
      const int ntok = min(32, a.L.b - t0);
      irow[st] = iinfo.row;
      islot[st] = iinfo.slot;
      ichunk[st] = ichunk_cur;
      ibid[st] = iinfo.bid;
      T* ks = stages + static_cast<size_t>(st) * kStageElems;
      T* vs = ks + kChunkElems;
      const unsigned bytes = static_cast<unsigned>(ntok * D * sizeof(T));
      mbar_arrive_expect_tx(&bar[st], kWantV ? 2 * bytes : bytes);
      const T* K = static_cast<const T*>(a.L.k);
      const T* V = static_cast<const T*>(a.L.v);
      if (nseg_page == 0) {
        const BlockSeg sg = block_seg(a.L, r, kv, iinfo.bid, 0);
        const long long off = sg.elem_off + static_cast<long long>(t0) * D;
        bulk_g2s(ks, K + off, bytes, &bar[st]);
        if (kWantV) bulk_g2s(vs, V + off, bytes, &bar[st]);
      } else {
        for (int t = t0; t < t0 + ntok;) {
          const int pg = t / nseg_page, o = t - pg * nseg_page;
          const int cnt = min(nseg_page - o, t0 + ntok - t);
          const BlockSeg sg = block_seg(a.L, r, kv, iinfo.bid, pg);
          const long long off = sg.elem_off + static_cast<long long>(o) * D;
          const unsigned sb = static_cast<unsigned>(cnt * D * sizeof(T));
          bulk_g2s(ks + (t - t0) * D, K + off, sb, &bar[st]);
          if (kWantV) bulk_g2s(vs + (t - t0) * D, V + off, sb, &bar[st]);
          t += cnt;
        }
      }
    }
    advance_to_active(false);
  };

  advance_to_active(true);
#pragma unroll 1
  for (int st = 0; st < NST; ++st) issue(st);
  __syncwarp();

  unsigned phase = 0;  // bit st = parity of stage st
  float qf[DPL];
  int q_row = -1;
  float m = neg_inf(), l = 0.f;
  float u[DPL], ua[DPL];
  float frame = 0.f;

#pragma unroll 1
  for (long long item = 0;; ++item) {
    const int st = static_cast<int>(item % NST);
    __syncwarp();
    const int row = irow[st];
    if (row < 0) break;
    const int slot = islot[st], chunk = ichunk[st];
    if (!mbar_wait(&bar[st], (phase >> st) & 1u, a.status)) return;
    phase ^= 1u << st;
    const int t0 = chunk * 32;
    const int ntok = min(32, a.L.b - t0);
    if (chunk == 0) {
      if (row != q_row) {
        q_row = row;
#pragma unroll
        for (int j = 0; j < DPL; ++j) qf[j] = load_any(a.q, a.q_dtype, static_cast<long long>(row) * D + lane * DPL + j);
      }
      m = neg_inf();
      l = 0.f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) { u[j] = 0.f; ua[j] = 0.f; }
      if (MODE == kModeFixed) frame = a.frame[row];
    }
    const T* ks = stages + static_cast<size_t>(st) * kStageElems;
    const T* vs = ks + kChunkElems;

    float p[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      p[t] = 0.f;
      if (t < ntok) {
        float kv[DPL];
        load_vec<T, DPL>(ks + t * D + lane * DPL, kv);
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc = fmaf(kv[j], qf[j], acc);
        p[t] = acc;
      }
    }
    transpose_reduce32(p, lane);
    const float s = lane < ntok ? p[0] * a.scale : neg_inf();

    float w;
    if (MODE == kModeFixed) {
      w = lane < ntok ? expf(s - frame) : 0.f;
      l += warp_sum(w);
    } else {
      const float mc = warp_max(s);
      const float mn = fmaxf(m, mc);
      const float alpha = expf(m - mn);
      w = lane < ntok ? expf(s - mn) : 0.f;
      l = l * alpha + warp_sum(w);
      m = mn;
      if (kWantV) {
#pragma unroll
        for (int j = 0; j < DPL; ++j) u[j] *= alpha;
      }
    }
    if (kWantV) {
#pragma unroll 4
      for (int t = 0; t < ntok; ++t) {
        const float wt = __shfl_sync(kFull, w, t);
        float vv[DPL];
        load_vec<T, DPL>(vs + t * D + lane * DPL, vv);
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          const float prod = wt * vv[j];
          u[j] += prod;
          if (MODE == kModeFixed) ua[j] += fabsf(prod);
        }
      }
    }
    __syncwarp();
    // Stage consumed: refill it before writing results.
    issue(st);

    if (chunk == (a.L.b + 31) / 32 - 1) {
      const long long job = static_cast<long long>(row) * a.s + slot;
      if (MODE != kModeFixed) {
        if (lane == 0) { a.m[job] = m; a.l[job] = l; }
      } else if (lane == 0 && a.l) {
        a.l[job] = l;
      }
      if (kWantV) {
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          a.u[job * D + lane * DPL + j] = u[j];
          if (MODE == kModeFixed && a.uabs) a.uabs[job * D + lane * DPL + j] = ua[j];
        }
      }
    }
  }
}

// ------------------------------------------------------------------ generic path
// Any D <= 1024, any B, any alignment. Lane = token for QK, lane = dim for PV.
template <typename T>
__global__ void __launch_bounds__(128) jobs_generic_kernel(JobArgs a) {
  extern __shared__ float gsm[];  // per warp: q[d], u[d], ua[d]
  __shared__ float ws[4][32];
  __shared__ long long offs[4][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  const int D = a.d;
  float* qs = gsm + static_cast<size_t>(warp) * 3 * D;
  float* us = qs + D;
  float* uas = us + D;
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  const long long W = static_cast<long long>(gridDim.x) * wpc;
  const T* K = static_cast<const T*>(a.L.k);
  const T* V = static_cast<const T*>(a.L.v);
  const bool want_v = a.mode != kModeMass;

  for (long long job = static_cast<long long>(blockIdx.x) * wpc + warp; job < njobs; job += W) {
    const JobInfo ji = resolve_job(a, job, lane);
    if (!ji.active) {
      write_inactive(a, job, lane);
      continue;
    }
    const int r = ji.row / a.hq;
    const int kv = (ji.row - r * a.hq) / a.g;
    __syncwarp();
    for (int dd = lane; dd < D; dd += 32) {
      qs[dd] = load_any(a.q, a.q_dtype, static_cast<long long>(ji.row) * D + dd);
      us[dd] = 0.f;
      uas[dd] = 0.f;
    }
    __syncwarp();
    const float frame = a.mode == kModeFixed ? a.frame[ji.row] : 0.f;
    float m = neg_inf(), l = 0.f;
    for (int t0 = 0; t0 < a.L.b; t0 += 32) {
      const int t = t0 + lane;
      const int ntok = min(32, a.L.b - t0);
      long long toff = 0;
      float s = neg_inf();
      if (t < a.L.b) {
        int seg = 0, within = t;
        if (a.L.page_table != nullptr) { seg = t / a.L.page_size; within = t - seg * a.L.page_size; }
        const BlockSeg sg = block_seg(a.L, r, kv, ji.bid, seg);
        toff = sg.elem_off + static_cast<long long>(within) * D;
        float acc = 0.f;
        for (int dd = 0; dd < D; ++dd) acc = fmaf(to_f32(K[toff + dd]), qs[dd], acc);
        s = acc * a.scale;
      }
      float w, alpha = 1.f;
      if (a.mode == kModeFixed) {
        w = t < a.L.b ? expf(s - frame) : 0.f;
        l += warp_sum(w);
      } else {
        const float mn = fmaxf(m, warp_max(s));
        alpha = expf(m - mn);
        w = t < a.L.b ? expf(s - mn) : 0.f;
        l = l * alpha + warp_sum(w);
        m = mn;
      }
      if (want_v) {
        ws[warp][lane] = w;
        offs[warp][lane] = toff;
        __syncwarp();
        for (int dd = lane; dd < D; dd += 32) {
          float acc = us[dd] * alpha, aacc = uas[dd];
          for (int tt = 0; tt < ntok; ++tt) {
            const float prod = ws[warp][tt] * to_f32(V[offs[warp][tt] + dd]);
            acc += prod;
            aacc += fabsf(prod);
          }
          us[dd] = acc;
          uas[dd] = aacc;
        }
        __syncwarp();
      }
    }
    __syncwarp();
    if (a.mode != kModeFixed) {
      if (lane == 0) { a.m[job] = m; a.l[job] = l; }
    } else if (lane == 0 && a.l) {
      a.l[job] = l;
    }
    if (want_v) {
      for (int dd = lane; dd < D; dd += 32) {
        a.u[job * D + dd] = us[dd];
        if (a.mode == kModeFixed && a.uabs) a.uabs[job * D + dd] = uas[dd];
      }
    }
  }
}

// ------------------------------------------------------------------ epilogues

// merge_partials (kernels.py:74-91): one CTA per row, threads over dims.
__global__ void merge_kernel(const float* m, const float* l, const float* u, const unsigned char* include, int s,
                             int d, float* out) {
  const int row = blockIdx.x;
  __shared__ float sM;
  __shared__ float sZ;
  if (threadIdx.x == 0) {
    float M = neg_inf();
    for (int i = 0; i < s; ++i) {
      const bool inc = include == nullptr || include[static_cast<long long>(row) * s + i];
      if (inc) M = fmaxf(M, m[static_cast<long long>(row) * s + i]);
    }
    if (M == neg_inf()) M = 0.f;
    float z = 0.f;
    for (int i = 0; i < s; ++i) {
      const bool inc = include == nullptr || include[static_cast<long long>(row) * s + i];
      if (inc) z += expf(m[static_cast<long long>(row) * s + i] - M) * l[static_cast<long long>(row) * s + i];
    }
    sM = M;
    sZ = fmaxf(z, 1e-30f);
  }
  __syncthreads();
  const float M = sM, z = sZ;
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < s; ++i) {
      const long long j = static_cast<long long>(row) * s + i;
      const bool inc = include == nullptr || include[j];
      if (inc) acc += expf(m[j] - M) * u[j * d + dd];
    }
    out[static_cast<long long>(row) * d + dd] = acc / z;
  }
}

// Hybrid grouping (kernels.py:94-117): high = mass >= tau * total mass,
// low aggregate at low_m = max low m, absolute numerator envelope.
__global__ void hybrid_group_kernel(const float* m, const float* l, const float* u, int s, int d, float tau,
                                    unsigned char* high, float* low_m, float* low_l, float* low_u, float* low_abs) {
  extern __shared__ float hs[];  // alpha[s]
  const int row = blockIdx.x;
  const long long base = static_cast<long long>(row) * s;
  if (threadIdx.x == 0) {
    float gm = neg_inf();
    for (int i = 0; i < s; ++i) gm = fmaxf(gm, m[base + i]);
    float total = 0.f;
    for (int i = 0; i < s; ++i) total += expf(m[base + i] - gm) * l[base + i];
    float lm = neg_inf();
    for (int i = 0; i < s; ++i) {
      const float mass = expf(m[base + i] - gm) * l[base + i];
      const bool hi = mass >= tau * total;
      high[base + i] = hi;
      hs[i] = hi ? 0.f : 1.f;
      if (!hi) lm = fmaxf(lm, m[base + i]);
    }
    if (lm == neg_inf()) lm = 0.f;
    float zz = 0.f;
    for (int i = 0; i < s; ++i) {
      const float al = hs[i] != 0.f ? expf(m[base + i] - lm) : 0.f;
      hs[i] = al;
      zz += al * l[base + i];
    }
    low_m[row] = lm;
    low_l[row] = zz;
  }
  __syncthreads();
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float uv = 0.f, ua = 0.f;
    for (int i = 0; i < s; ++i) {
      const float al = hs[i];
      const float x = u[(base + i) * d + dd];
      uv += al * x;
      ua += al * fabsf(x);
    }
    low_u[static_cast<long long>(row) * d + dd] = uv;
    low_abs[static_cast<long long>(row) * d + dd] = ua;
  }
}

// Compact grouping (kernels.py:281-309): capacity-C packing of high blocks in
// predicted order with overflow spilled to the low group.
__global__ void compact_group_kernel(const float* pm, const float* pl, const void* pred, int pred64, int s, int c,
                                     float tau, unsigned char* high, void* rids, float* low_m, float* low_l,
                                     unsigned char* overflow) {
  const int row = blockIdx.x;
  if (threadIdx.x != 0) return;
  const long long base = static_cast<long long>(row) * s;
  float gm = neg_inf();
  for (int i = 0; i < s; ++i) gm = fmaxf(gm, pm[base + i]);
  float total = 0.f;
  for (int i = 0; i < s; ++i) total += expf(pm[base + i] - gm) * pl[base + i];
  int count = 0;
  for (int i = 0; i < s; ++i) count += (expf(pm[base + i] - gm) * pl[base + i]) >= tau * total;
  overflow[row] = count > c;
  int rank = 0;
  for (int cc = 0; cc < c; ++cc) store_id(rids, pred64, static_cast<long long>(row) * c + cc, -1);
  float lm = neg_inf();
  for (int i = 0; i < s; ++i) {
    bool hi = (expf(pm[base + i] - gm) * pl[base + i]) >= tau * total;
    if (hi) {
      ++rank;
      if (rank <= c) store_id(rids, pred64, static_cast<long long>(row) * c + rank - 1, load_id(pred, pred64, base + i));
      else hi = false;
    }
    high[base + i] = hi;
    if (!hi) lm = fmaxf(lm, pm[base + i]);
  }
  if (lm == neg_inf()) lm = 0.f;
  float ll = 0.f;
  for (int i = 0; i < s; ++i)
    if (!high[base + i]) ll += expf(pm[base + i] - lm) * pl[base + i];
  low_m[row] = lm;
  low_l[row] = ll;
}

// Sum per-slot vectors in slot order: out[row, :] = sum_i x[row, i, :].
__global__ void slot_sum_kernel(const float* x, const float* y, int s, int d, float* out_x, float* out_y) {
  const int row = blockIdx.x;
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float ax = 0.f, ay = 0.f;
    for (int i = 0; i < s; ++i) {
      const long long j = (static_cast<long long>(row) * s + i) * d + dd;
      ax += x[j];
      if (y) ay += y[j];
    }
    out_x[static_cast<long long>(row) * d + dd] = ax;
    if (y) out_y[static_cast<long long>(row) * d + dd] = ay;
  }
}

// ------------------------------------------------------------------ host side

static bool fast_eligible(const JobArgs& a, int elem) {
  if (a.d != 64 && a.d != 128 && a.d != 256) return false;
  // Four warps with at least one stage each must fit the shared-memory plan.
  const size_t stage = static_cast<size_t>(32) * a.d * elem * (a.mode == kModeMass ? 1 : 2);
  if (4 * stage > 200 * 1024) return false;
  const uintptr_t pk = reinterpret_cast<uintptr_t>(a.L.k), pv = reinterpret_cast<uintptr_t>(a.L.v);
  if ((pk | pv) & 15) return false;
  if ((a.d * elem) % 16) return false;
  if (a.L.page_table != nullptr && (a.L.b % a.L.page_size)) return false;
  if (a.L.kv_request_stride % 8) return false;
  return true;
}

template <typename T, int DPL, int MODE>
constexpr size_t fast_stage_bytes() {
  return static_cast<size_t>(32) * 32 * DPL * sizeof(T) * (MODE == kModeMass ? 1 : 2);
}

template <typename T, int DPL, int MODE>
static int launch_fast_t(const JobArgs& a, int num_sms, cudaStream_t stream) {
  constexpr size_t kStage = fast_stage_bytes<T, DPL, MODE>();
  constexpr int NST = (4 * 3 * kStage <= 200 * 1024) ? 3 : ((4 * 2 * kStage <= 200 * 1024) ? 2 : 1);
  const size_t stage = kStage;
  const size_t smem = stage * NST * 4;
  auto kern = jobs_fast_kernel<T, DPL, MODE, NST>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  long long ctas = (njobs + 3) / 4;
  const long long cap = static_cast<long long>(num_sms) * (smem <= 110 * 1024 ? 2 : 1);
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  kern<<<static_cast<unsigned>(ctas), 128, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

template <typename T, int MODE>
static int launch_fast_d(const JobArgs& a, int num_sms, cudaStream_t stream) {
  switch (a.d) {
    case 64: return launch_fast_t<T, 2, MODE>(a, num_sms, stream);
    case 128: return launch_fast_t<T, 4, MODE>(a, num_sms, stream);
    default: return launch_fast_t<T, 8, MODE>(a, num_sms, stream);
  }
}

template <typename T>
static int launch_jobs_t(const JobArgs& a, int num_sms, cudaStream_t stream) {
  if (fast_eligible(a, sizeof(T))) {
    switch (a.mode) {
      case kModeFull: return launch_fast_d<T, kModeFull>(a, num_sms, stream);
      case kModeMass: return launch_fast_d<T, kModeMass>(a, num_sms, stream);
      default: return launch_fast_d<T, kModeFixed>(a, num_sms, stream);
    }
  }
  const size_t smem = static_cast<size_t>(4) * 3 * a.d * sizeof(float);
  cudaFuncSetAttribute(jobs_generic_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  const long long njobs = static_cast<long long>(a.rows) * a.s;
  long long ctas = (njobs + 3) / 4;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  jobs_generic_kernel<T><<<static_cast<unsigned>(ctas), 128, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int launch_jobs(const JobArgs& a, int kv_dtype, int num_sms, cudaStream_t stream) {
  if (static_cast<long long>(a.rows) * a.s == 0) return 0;
  switch (kv_dtype) {
    case kF32: return launch_jobs_t<float>(a, num_sms, stream);
    case kF16: return launch_jobs_t<__half>(a, num_sms, stream);
    default: return launch_jobs_t<__nv_bfloat16>(a, num_sms, stream);
  }
}

int launch_merge(const float* m, const float* l, const float* u, const unsigned char* include, int rows, int s, int d,
                 float* out, cudaStream_t stream) {
  merge_kernel<<<rows, 128, 0, stream>>>(m, l, u, include, s, d, out);
  return static_cast<int>(cudaGetLastError());
}

int launch_hybrid_group(const float* m, const float* l, const float* u, int rows, int s, int d, float tau,
                        unsigned char* high, float* low_m, float* low_l, float* low_u, float* low_abs,
                        cudaStream_t stream) {
  hybrid_group_kernel<<<rows, 128, s * sizeof(float), stream>>>(m, l, u, s, d, tau, high, low_m, low_l, low_u,
                                                                  low_abs);
  return static_cast<int>(cudaGetLastError());
}

int launch_compact_group(const float* pm, const float* pl, const void* pred, int pred64, int rows, int s, int c,
                         float tau, unsigned char* high, void* rids, float* low_m, float* low_l,
                         unsigned char* overflow, cudaStream_t stream) {
  compact_group_kernel<<<rows, 32, 0, stream>>>(pm, pl, pred, pred64, s, c, tau, high, rids, low_m, low_l, overflow);
  return static_cast<int>(cudaGetLastError());
}

int launch_slot_sum(const float* x, const float* y, int rows, int s, int d, float* out_x, float* out_y,
                    cudaStream_t stream) {
  slot_sum_kernel<<<rows, 128, 0, stream>>>(x, y, s, d, out_x, out_y);
  return static_cast<int>(cudaGetLastError());
}

// touch_kv (kernels.py:250-260): per (row, slot, 1024-element tile) checksum
// of K + V over the block's elements, read in token-major order.
template <typename T>
__global__ void touch_kernel(KVLayout L, int hq, int g, const void* ids, int ids64, int s, float* out) {
  const int row = blockIdx.x, slot = blockIdx.y, tile = blockIdx.z;
  const int ntiles = gridDim.z;
  const int r = row / hq, kv = (row - r * hq) / g;
  const long long bid = load_id(ids, ids64, static_cast<long long>(row) * s + slot);
  __shared__ float red[32];
  float acc = 0.f;
  if (bid >= 0 && bid < request_blocks(L, r)) {
    const T* K = static_cast<const T*>(L.k);
    const T* V = static_cast<const T*>(L.v);
    const int total = L.b * L.d;
    for (int x = tile * 1024 + threadIdx.x; x < min(total, (tile + 1) * 1024); x += blockDim.x) {
      const int t = x / L.d, dd = x - t * L.d;
      int seg = 0, within = t;
      if (L.page_table != nullptr) { seg = t / L.page_size; within = t - seg * L.page_size; }
      const long long o = block_seg(L, r, kv, bid, seg).elem_off + static_cast<long long>(within) * L.d + dd;
      acc += to_f32(K[o]) + to_f32(V[o]);
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
    out[(static_cast<long long>(row) * s + slot) * ntiles + tile] = t;
  }
}

int launch_touch(const KVLayout& L, int rows, int hq, int g, const void* ids, int ids64, int s, float* out,
                 int kv_dtype, cudaStream_t stream) {
  const int ntiles = (L.b * L.d + 1023) / 1024;
  dim3 grid(rows, s, ntiles);
  switch (kv_dtype) {
    case kF32: touch_kernel<float><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
    case kF16: touch_kernel<__half><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
    default: touch_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(L, hq, g, ids, ids64, s, out); break;
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace stk
