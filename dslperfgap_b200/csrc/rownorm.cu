// rownorm.cu — row-normalising kernels: layer_norm, rms_norm, softmax,
// log_softmax (sm_100a).
//
// All four read a row, reduce it to one or two statistics, and write a row of
// the same length. Three kernel shapes cover every input:
//
//  * resident_kernel: the row is split over a group of `tpr` threads (a warp
//    for short rows, up to a 1024-thread CTA for 128 KiB rows), each holding
//    VPT 16-byte vectors in registers. HBM is read once and written once; the
//    statistics are warp-shuffle + shared-memory reductions. Used whenever the
//    row is 16-byte vectorisable and fits (<= 8192 vectors).
//  * stream_kernel: one CTA per row, two passes. Pass 1 streams the row into
//    per-thread online statistics (Welford / running max+sum); pass 2 re-reads
//    the row (an L2 hit: a CTA's row is at most a few hundred KiB) and writes
//    the output. Used for rows too long for registers and for unaligned or
//    odd-length rows (scalar variant).
//  * strided_log_softmax_kernel: log_softmax over a non-last dim of an
//    [M, N, K] tensor; each thread owns one (m, k) column, reads are coalesced
//    across k.
//
// Numerics: fp32 accumulation, one rounding at the store, NaN-propagating max
// (torch semantics: a NaN anywhere in a softmax row poisons the row).
#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"
#include "pipe.cuh"

namespace dslpg {

enum RowOp : int { kLayerNorm = 0, kRmsNorm = 1, kSoftmax = 2, kLogSoftmax = 3 };

struct RowArgs {
  const void* x;
  void* y;
  const void* w;  // layer_norm / rms_norm weight [N] (dtype wdt)
  const void* b;  // layer_norm bias [N] (dtype wdt) or nullptr
  int64_t M;
  int N;
  int nvec;   // N / elements-per-vector (vector paths)
  int tpr;    // threads per row
  int rpc;    // rows per CTA (resident kernel)
  float eps;
  float inv_n;  // 1 / N
  int wdt;    // weight dtype code
  int wvec;   // 1: weight/bias have x's dtype and are 16-byte aligned
};

// log_softmax(x, dtype=Tout) first converts x to Tout (a no-op when Tout is fp32).
template <typename Tin, typename Tout>
constexpr bool kRoundIn = !std::is_same<Tin, Tout>::value && !std::is_same<Tout, float>::value;

template <typename Tin, typename Tout>
DSLPG_DEV float in_value(float v) {
  if constexpr (kRoundIn<Tin, Tout>) return round_to<Tout>(v);
  return v;
}

// Weight (and bias) elements [j*E, j*E+E) as fp32. The resident kernel is only
// used when weight and bias have x's dtype and are 16-byte aligned.
template <typename Tin, int E>
DSLPG_DEV void load_weight(const void* p, int j, float* out) {
  if (p == nullptr) {
#pragma unroll
    for (int i = 0; i < E; ++i) out[i] = 0.f;
    return;
  }
  unpack<Tin>(ld_keep(static_cast<const Tin*>(p) + static_cast<int64_t>(j) * E), out);
}

// ============================================================================
// Per-row math shared by the resident and TMA kernels
// ============================================================================
// Weight (or bias) vector j of a row as raw 16-byte data (zeros if p is null).
// Read through L1: every row of a CTA reads the same vectors.
template <typename Tin>
DSLPG_DEV Vec16 weight_vec(const void* p, int j) {
  if (p == nullptr) return Vec16{{0u, 0u, 0u, 0u}};
  return ld_keep(static_cast<const Tin*>(p) + static_cast<int64_t>(j) * Elt<Tin>::kPerVec);
}

// Normalise one row whose VPT 16-byte vectors (elements [j*E, j*E+E) with
// j = t + k*tpr) this thread holds in v; masked vectors (ok[k] false, always
// the trailing ones) hold zeros. Stores the thread's part of the output row
// yr. Every thread of the row group calls it. Element arithmetic runs on fp32
// pairs, two lanes per fma/add/mul.f32x2 instruction.
template <int OP, typename Tin, typename Tout, int VPT, int CACHE_LIMIT, class Red>
DSLPG_DEV void normalize_row(const RowArgs& a, const Vec16 (&v)[VPT], const bool (&ok)[VPT], int t,
                             Tout* yr, Red& rd) {
  constexpr int E = Elt<Tin>::kPerVec;
  constexpr int P = E / 2;
  // Up to CACHE_LIMIT fp32 values per thread are kept unpacked (softmax keeps
  // the exp values there, so each element costs one ex2); longer slices stay
  // packed and are unpacked again in each phase.
  constexpr bool kCache = VPT * E <= CACHE_LIMIT;

  auto load_pair = [&](int k, int p) -> f32x2 {
    f32x2 x = unpack_pair<Tin>(v[k], p);
    if constexpr (kRoundIn<Tin, Tout>) {
      float x0, x1;
      upk2(x, x0, x1);
      x = pk2(round_to<Tout>(x0), round_to<Tout>(x1));
    }
    return x;
  };
  f32x2 fr[kCache ? VPT : 1][P];
  if constexpr (kCache) {
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int p = 0; p < P; ++p) fr[k][p] = load_pair(k, p);
  }
  auto pair = [&](int k, int p) -> f32x2 {
    if constexpr (kCache) return fr[k][p];
    else return load_pair(k, p);
  };
  auto store = [&](int k, const f32x2 (&y)[P]) {
    StorePairs<Tout, P>::run(yr + static_cast<int64_t>(t + k * a.tpr) * E, y);
  };

  if constexpr (OP == kRmsNorm) {
    f32x2 ss2 = pk2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const f32x2 x = pair(k, p);
        ss2 = fma2(x, x, ss2);
      }
    const float ss = rd.template reduce<SumOp>(hsum2(ss2));
    const float inv = rsqrtf(ss * a.inv_n + a.eps);
    const f32x2 inv2 = pk2(inv, inv);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (!ok[k]) continue;
      const Vec16 wk = weight_vec<Tin>(a.w, t + k * a.tpr);
      f32x2 y[P];
#pragma unroll
      for (int p = 0; p < P; ++p) y[p] = mul2(mul2(pair(k, p), inv2), unpack_pair<Tin>(wk, p));
      store(k, y);
    }
  } else if constexpr (OP == kLayerNorm) {
    // The sum and the sum of squares in one exchange; var = E[x^2] - mean^2
    // is kept only where that difference cannot cancel badly (mean^2 <= 16 var:
    // relative error below 1e-6). Other rows (a large offset against a small
    // spread, or inf/NaN) take the exact second pass over (x - mean)^2. The
    // test is on values every thread of the row holds, so the branch is uniform.
    f32x2 s2 = pk2(0.f, 0.f), q2 = pk2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const f32x2 x = pair(k, p);  // masked vectors hold zeros
        s2 = add2(s2, x);
        q2 = fma2(x, x, q2);
      }
    float sum = hsum2(s2), sq = hsum2(q2);
    rd.sum_pair(sum, sq);
    const float mean = sum * a.inv_n;
    const f32x2 nmean2 = pk2(-mean, -mean);
    float var = fmaf(sq, a.inv_n, -mean * mean);
    if (!(mean * mean <= 16.f * var)) {
      q2 = pk2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!ok[k]) continue;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const f32x2 d = add2(pair(k, p), nmean2);
          q2 = fma2(d, d, q2);
        }
      }
      var = rd.template reduce_own<SumOp>(hsum2(q2)) * a.inv_n;  // only this row's group is here
    }
    const float rstd = rsqrtf(var + a.eps);
    const f32x2 rstd2 = pk2(rstd, rstd);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (!ok[k]) continue;
      const int j = t + k * a.tpr;
      const Vec16 wk = weight_vec<Tin>(a.w, j), bk = weight_vec<Tin>(a.b, j);
      f32x2 y[P];
#pragma unroll
      for (int p = 0; p < P; ++p)
        y[p] = fma2(mul2(add2(pair(k, p), nmean2), rstd2), unpack_pair<Tin>(wk, p), unpack_pair<Tin>(bk, p));
      store(k, y);
    }
  } else {  // kSoftmax / kLogSoftmax
    float m;
    if constexpr (!kRoundIn<Tin, Tout>) {
      // max on the stored values; masked vectors count as -inf
      if (ok[VPT - 1]) {
        m = RawExtreme<Tin, VPT, false>::run(v);
      } else {
        constexpr uint32_t ni = NegInfWord<Tin>::v;
        Vec16 vm[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) vm[k] = ok[k] ? v[k] : Vec16{{ni, ni, ni, ni}};
        m = RawExtreme<Tin, VPT, false>::run(vm);
      }
    } else {
      m = kNegInf;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!ok[k]) continue;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          float x0, x1;
          upk2(pair(k, p), x0, x1);
          m = max_nan(m, max_nan(x0, x1));
        }
      }
    }
    m = rd.template reduce<MaxOp>(m);
    const f32x2 nm2 = pk2(-m, -m), l2e2 = pk2(kLog2e, kLog2e);
    f32x2 s2 = pk2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (!ok[k]) continue;
#pragma unroll
      for (int p = 0; p < P; ++p) {
        float t0, t1;
        upk2(mul2(add2(pair(k, p), nm2), l2e2), t0, t1);
        const f32x2 e = pk2(ex2(t0), ex2(t1));
        if constexpr (kCache && OP == kSoftmax) fr[k][p] = e;
        s2 = add2(s2, e);
      }
    }
    const float s = rd.template reduce<SumOp>(hsum2(s2));
    if constexpr (OP == kSoftmax) {
      const float inv = 1.0f / s;
      const f32x2 inv2 = pk2(inv, inv);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!ok[k]) continue;
        f32x2 y[P];
#pragma unroll
        for (int p = 0; p < P; ++p) {
          if constexpr (kCache) {
            y[p] = mul2(fr[k][p], inv2);
          } else {
            float t0, t1;
            upk2(mul2(add2(pair(k, p), nm2), l2e2), t0, t1);
            y[p] = mul2(pk2(ex2(t0), ex2(t1)), inv2);
          }
        }
        store(k, y);
      }
    } else {
      const float ls = logf(s);
      const f32x2 nls2 = pk2(-ls, -ls);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!ok[k]) continue;
        f32x2 y[P];
#pragma unroll
        for (int p = 0; p < P; ++p) y[p] = add2(add2(pair(k, p), nm2), nls2);
        store(k, y);
      }
    }
  }
}

// ============================================================================
// Resident kernel: rows read straight into registers
// ============================================================================
// PD = rows loaded ahead of the one being reduced (0, 1 or 2), so that every
// thread keeps PD rows of loads in flight while it reduces.
template <int OP, typename Tin, typename Tout, int VPT, int PD>
__global__ void __launch_bounds__(1024) resident_kernel(const RowArgs a) {
  constexpr int E = Elt<Tin>::kPerVec;
  __shared__ float red[2][32];
  __shared__ float red2[OP == kLayerNorm ? 2 : 1][64];

  const int g = threadIdx.x / a.tpr;
  const int t = threadIdx.x - g * a.tpr;
  GroupReducer rd{red, a.tpr >> 5, g * (a.tpr >> 5), 0, red2, 0};

  auto load_row = [&](Vec16* dst, int64_t row) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int j = t + k * a.tpr;
      dst[k] = Vec16{{0u, 0u, 0u, 0u}};
      if (row < a.M && j < a.nvec)
        dst[k] = ld_stream(static_cast<const Tin*>(a.x) + row * a.N + static_cast<int64_t>(j) * E);
    }
  };

  const int64_t step = static_cast<int64_t>(gridDim.x) * a.rpc;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * a.rpc + g;
  Vec16 q0[PD >= 1 ? VPT : 1], q1[PD >= 2 ? VPT : 1];
  if constexpr (PD >= 1) load_row(q0, first);
  if constexpr (PD >= 2) load_row(q1, first + step);

  for (int64_t base = static_cast<int64_t>(blockIdx.x) * a.rpc; base < a.M; base += step) {
    const int64_t row = base + g;
    Vec16 v[VPT];
    if constexpr (PD == 0) {
      load_row(v, row);
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) v[k] = q0[k];
      if constexpr (PD == 2) {
#pragma unroll
        for (int k = 0; k < VPT; ++k) q0[k] = q1[k];
        load_row(q1, row + 2 * step);
      } else {
        load_row(q0, row + step);
      }
    }
    bool ok[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) ok[k] = row < a.M && (t + k * a.tpr) < a.nvec;
    // 16 cached values: the prefetch buffers need the other registers.
    // log_softmax re-reads x in its output phase: recomputing the unpack there
    // is cheaper than the registers a cached copy costs in occupancy.
    normalize_row<OP, Tin, Tout, VPT, (OP == kLogSoftmax ? 0 : 16)>(a, v, ok, t,
                                                                    static_cast<Tout*>(a.y) + row * a.N, rd);
  }
}

// ============================================================================
// TMA kernel: rows streamed into a shared-memory ring by bulk copies
// ============================================================================
// Counts waits that ran out of time in this file's kernels (read and reset
// by dslpg_take_wait_timeouts).
static __device__ unsigned int g_wait_timeouts;

// Warp 0 lane 0 is the producer: it copies each of the CTA's rows (rows
// blockIdx.x, blockIdx.x + gridDim.x, ...) into the next ring slot. Warps 1..
// are the a.tpr consumers: each waits for the row, copies its VPT vectors to
// registers, releases the slot, and normalises the row with stores straight
// from registers. A wait that runs out of time sets `abort`: every thread then
// still runs the same loop (so the consumers' named barriers stay matched) but
// skips the remaining waits; the producer stops issuing and drains.
template <int OP, typename Tin, typename Tout, int VPT>
__global__ void __launch_bounds__(1024) tma_norm_kernel(const RowArgs a, int stages,
                                                        unsigned long long limit_ns) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int E = Elt<Tin>::kPerVec;
  __shared__ volatile int abort_flag;
  const int ncw = (blockDim.x >> 5) - 1;
  const uint32_t row_bytes = static_cast<uint32_t>(a.N) * sizeof(Tin);
  if (threadIdx.x == 0) abort_flag = 0;
  float* red;
  const Ring ring = ring_setup(smem, row_bytes, stages, ncw, &red);  // includes __syncthreads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t u = 0;
      for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x, ++u) {
        if (abort_flag) break;
        if (u >= static_cast<uint32_t>(stages) && !mbar_wait(ring.empty_bar(u), ring.parity(u) ^ 1u, limit_ns)) {
          atomicAdd(&g_wait_timeouts, 1u);
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(ring.full_bar(u), row_bytes);
        bulk_load(ring.slot(u), static_cast<const Tin*>(a.x) + row * a.N, row_bytes, ring.full_bar(u), pol);
      }
      if (!ring_drain(ring, u)) atomicAdd(&g_wait_timeouts, 1u);
    }
    return;
  }

  const int t = threadIdx.x - 32;
  ConsumerReducer rd{red, ncw, 0};
  uint32_t u = 0;
  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x, ++u) {
    if (!abort_flag && !mbar_wait(ring.full_bar(u), ring.parity(u), limit_ns)) {
      atomicAdd(&g_wait_timeouts, 1u);
      abort_flag = 1;
    }
    Vec16 v[VPT];
    bool ok[VPT];
    const uint32_t slot = ring.slot(u);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int j = t + k * a.tpr;
      ok[k] = j < a.nvec;
      v[k] = Vec16{{0u, 0u, 0u, 0u}};
      if (ok[k]) v[k] = lds16(slot + 16u * j);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(ring.empty_bar(u));
    if (abort_flag) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) ok[k] = false;  // no stores after a timeout
    }
    normalize_row<OP, Tin, Tout, VPT, 32>(a, v, ok, t, static_cast<Tout*>(a.y) + row * a.N, rd);
  }
}

// ============================================================================
// Stream kernel (two passes; any length and alignment)
// ============================================================================
// Running statistics of one thread.
struct Welford {
  float n, mean, m2;
};

DSLPG_DEV Welford welford_merge(Welford a, Welford b) {
  const float n = a.n + b.n;
  if (n == 0.f) return a;
  const float d = b.mean - a.mean;
  const float fb = b.n / n;
  Welford r;
  r.n = n;
  r.mean = a.mean + d * fb;
  r.m2 = a.m2 + b.m2 + d * d * a.n * fb;
  return r;
}

// Online max / sum-of-exp update with a chunk of values (invalid ones are -inf).
DSLPG_DEV void online_update(float& m, float& s, const float* f, int n) {
  float cm = kNegInf;
  for (int i = 0; i < n; ++i) cm = max_nan(cm, f[i]);
  const float nm = max_nan(m, cm);
  if (nm == kNegInf) return;  // every value so far is -inf: nothing to add
  s = (m == nm) ? s : s * exp_shifted(m - nm);
  for (int i = 0; i < n; ++i) s += exp_shifted(f[i] - nm);
  m = nm;
}

// Combine (max, sum) pairs of one row spread over the CTA; returns the row's.
DSLPG_DEV void block_merge_ms(float& m, float& s, float* red0, float* red1) {
  const int nw = blockDim.x >> 5;
  const float gm = group_reduce<MaxOp>(m, red0, nw, 0);
  const float sc = (m == gm) ? s : s * exp_shifted(m - gm);
  s = group_reduce<SumOp>(sc, red1, nw, 0);
  m = gm;
}

DSLPG_DEV Welford warp_merge_welford(Welford w) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Welford other;
    other.n = __shfl_down_sync(0xffffffffu, w.n, o);
    other.mean = __shfl_down_sync(0xffffffffu, w.mean, o);
    other.m2 = __shfl_down_sync(0xffffffffu, w.m2, o);
    w = welford_merge(w, other);
  }
  // lane 0 holds the warp's statistics; broadcast them.
  w.n = __shfl_sync(0xffffffffu, w.n, 0);
  w.mean = __shfl_sync(0xffffffffu, w.mean, 0);
  w.m2 = __shfl_sync(0xffffffffu, w.m2, 0);
  return w;
}

DSLPG_DEV Welford block_merge_welford(Welford w, float* sh /* [3][32] */) {
  w = warp_merge_welford(w);
  const int nw = blockDim.x >> 5;
  if (nw == 1) return w;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sh[wid] = w.n;
    sh[32 + wid] = w.mean;
    sh[64 + wid] = w.m2;
  }
  __syncthreads();
  Welford r{0.f, 0.f, 0.f};
  if (lane < nw) r = Welford{sh[lane], sh[32 + lane], sh[64 + lane]};
  r = warp_merge_welford(r);
  __syncthreads();  // sh may be reused by the caller's next row
  return r;
}

template <typename Tin, int V>
DSLPG_DEV void load_unit(const Tin* xr, int j, bool ok, float* f) {
  if constexpr (V == 1) {
    f[0] = ok ? to_f(xr[j]) : 0.f;
  } else {
    Vec16 v{{0u, 0u, 0u, 0u}};
    if (ok) v = ld_stream(xr + static_cast<int64_t>(j) * V);
    unpack<Tin>(v, f);
  }
}

template <typename Tin, int V>
DSLPG_DEV void load_weight_unit(const RowArgs& a, const void* p, int j, float* w) {
  if (p == nullptr) {
#pragma unroll
    for (int i = 0; i < V; ++i) w[i] = 0.f;
  } else if (V > 1 && a.wvec) {
    load_weight<Tin, V>(p, j, w);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) w[i] = load_any(p, static_cast<int64_t>(j) * V + i, a.wdt);
  }
}

template <typename Tout, int V>
DSLPG_DEV void store_unit(Tout* yr, int j, const float* f) {
  if constexpr (V == 1) {
    yr[j] = from_f<Tout>(f[0]);
  } else {
    StoreOut<Tout, V>::run(yr + static_cast<int64_t>(j) * V, f);
  }
}

template <int OP, typename Tin, typename Tout, int V>
__global__ void __launch_bounds__(1024) stream_kernel(const RowArgs a) {
  constexpr int U = 4;  // units in flight per thread per iteration
  __shared__ float sh[3][32];
  __shared__ float sh_w[96];
  const int t = threadIdx.x;
  const int tpr = blockDim.x;
  const int units = (V == 1) ? a.N : a.nvec;
  const float n_f = static_cast<float>(a.N);

  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    const Tin* xr = static_cast<const Tin*>(a.x) + row * a.N;
    Tout* yr = static_cast<Tout*>(a.y) + row * a.N;

    // ---- pass 1: statistics
    float ss = 0.f;                 // rms_norm
    Welford wf{0.f, 0.f, 0.f};      // layer_norm
    float m = kNegInf, s = 0.f;     // softmax family
    for (int j0 = t; j0 < units; j0 += U * tpr) {
      float f[U][V];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        ok[u] = j < units;
        load_unit<Tin, V>(xr, j, ok[u], f[u]);
#pragma unroll
        for (int i = 0; i < V; ++i) f[u][i] = in_value<Tin, Tout>(f[u][i]);
      }
      if constexpr (OP == kRmsNorm) {
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int i = 0; i < V; ++i) ss = fmaf(f[u][i], f[u][i], ss);
      } else if constexpr (OP == kLayerNorm) {
        float c = 0.f, cs = 0.f;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!ok[u]) continue;
          c += V;
#pragma unroll
          for (int i = 0; i < V; ++i) cs += f[u][i];
        }
        if (c > 0.f) {
          const float cmean = cs / c;
          float cm2 = 0.f;
#pragma unroll
          for (int u = 0; u < U; ++u) {
            if (!ok[u]) continue;
#pragma unroll
            for (int i = 0; i < V; ++i) {
              const float d = f[u][i] - cmean;
              cm2 = fmaf(d, d, cm2);
            }
          }
          wf = welford_merge(wf, Welford{c, cmean, cm2});
        }
      } else {
        float flat[U * V];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int i = 0; i < V; ++i) flat[u * V + i] = ok[u] ? f[u][i] : kNegInf;
        online_update(m, s, flat, U * V);
      }
    }

    // ---- combine across the CTA
    float p0 = 0.f, p1 = 0.f;  // per-op parameters of pass 2
    if constexpr (OP == kRmsNorm) {
      ss = group_reduce<SumOp>(ss, sh[0], tpr >> 5, 0);
      p0 = 1.0f / sqrtf(ss / n_f + a.eps);
    } else if constexpr (OP == kLayerNorm) {
      wf = block_merge_welford(wf, sh_w);
      p0 = wf.mean;
      p1 = 1.0f / sqrtf(wf.m2 / n_f + a.eps);
    } else {
      block_merge_ms(m, s, sh[0], sh[1]);
      if (!(fabsf(m) < kPosInf)) s = __int_as_float(0x7fc00000);  // non-finite max: NaN row
      p0 = m;
      p1 = (OP == kSoftmax) ? 1.0f / s : logf(s);
    }

    // ---- pass 2: output (re-read; the row is L2-resident)
    for (int j0 = t; j0 < units; j0 += U * tpr) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        if (j >= units) continue;
        float f[V];
        load_unit<Tin, V>(xr, j, true, f);
#pragma unroll
        for (int i = 0; i < V; ++i) f[i] = in_value<Tin, Tout>(f[i]);
        if constexpr (OP == kRmsNorm) {
          float w[V];
          load_weight_unit<Tin, V>(a, a.w, j, w);
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] = (f[i] * p0) * w[i];
        } else if constexpr (OP == kLayerNorm) {
          float w[V], bb[V];
          load_weight_unit<Tin, V>(a, a.w, j, w);
          load_weight_unit<Tin, V>(a, a.b, j, bb);
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] = fmaf((f[i] - p0) * p1, w[i], bb[i]);
        } else if constexpr (OP == kSoftmax) {
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] = exp_shifted(f[i] - p0) * p1;
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] = (f[i] - p0) - p1;
        }
        store_unit<Tout, V>(yr, j, f);
      }
    }
    __syncthreads();  // shared buffers are reused by the next row
  }
}

// ============================================================================
// Cluster kernel: a long row split over the CTAs of a thread-block cluster
// ============================================================================
// Each row is split into C contiguous slices of slice_vecs 16-byte vectors,
// one per CTA of a cluster of C (up to 8 portable CTAs of 1024 threads). A CTA
// holds its slice in registers, VPT vectors per thread, prefetching the next
// row's slice while it reduces this one, exactly as the resident kernel does
// within one CTA; the row statistics come from ClusterReducer. HBM is read
// once and written once. Clusters loop over rows.
template <int OP, typename Tin, typename Tout, int VPT>
__global__ void __launch_bounds__(1024) cluster_norm_kernel(const RowArgs a, int slice_vecs) {
  __shared__ float red[2][32];
  __shared__ float slots[2];
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr int E = Elt<Tin>::kPerVec;
  const int C = static_cast<int>(cl.num_blocks());
  const int rank = static_cast<int>(cl.block_rank());
  const int64_t nclusters = gridDim.x / C;
  const int64_t cid = blockIdx.x / C;
  const int t = threadIdx.x;
  const int v0 = rank * slice_vecs;
  const int nv = max(0, min(a.nvec, v0 + slice_vecs) - v0);

  // The slice seen as a row of its own (statistics still use 1/N of the row).
  RowArgs s = a;
  s.tpr = blockDim.x;
  s.nvec = nv;
  if (a.w) s.w = static_cast<const Tin*>(a.w) + static_cast<int64_t>(v0) * E;
  if (a.b) s.b = static_cast<const Tin*>(a.b) + static_cast<int64_t>(v0) * E;
  ClusterReducer rd{slots, red, 0, C};

  auto load_row = [&](Vec16* dst, int64_t row) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int j = t + k * s.tpr;
      dst[k] = Vec16{{0u, 0u, 0u, 0u}};
      if (row < a.M && j < nv)
        dst[k] = ld_stream(static_cast<const Tin*>(a.x) + row * a.N + static_cast<int64_t>(v0 + j) * E);
    }
  };
  Vec16 nxt[VPT];
  load_row(nxt, cid);
  for (int64_t row = cid; row < a.M; row += nclusters) {
    Vec16 v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) v[k] = nxt[k];
    load_row(nxt, row + nclusters);
    bool ok[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) ok[k] = (t + k * s.tpr) < nv;
    normalize_row<OP, Tin, Tout, VPT, (OP == kLogSoftmax ? 0 : 16)>(
        s, v, ok, t, static_cast<Tout*>(a.y) + row * a.N + static_cast<int64_t>(v0) * E, rd);
  }
  cl.sync();  // no CTA leaves while another may still read its exchange slots
}

// ============================================================================
// log_softmax over the middle axis of [M, N, K]
// ============================================================================
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) strided_log_softmax_kernel(const Tin* __restrict__ x,
                                                                  Tout* __restrict__ y, int64_t M,
                                                                  int64_t N, int64_t K) {
  const int64_t cols = M * K;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t mi = c / K;
    const int64_t k = c - mi * K;
    const Tin* xc = x + mi * N * K + k;
    Tout* yc = y + mi * N * K + k;
    float m = kNegInf, s = 0.f;
    for (int64_t n = 0; n < N; ++n) {
      float f = in_value<Tin, Tout>(to_f(xc[n * K]));
      online_update(m, s, &f, 1);
    }
    if (!(fabsf(m) < kPosInf)) s = __int_as_float(0x7fc00000);
    const float ls = logf(s);
    for (int64_t n = 0; n < N; ++n) {
      const float f = in_value<Tin, Tout>(to_f(xc[n * K]));
      yc[n * K] = from_f<Tout>((f - m) - ls);
    }
  }
}

// ============================================================================
// Host dispatch
// ============================================================================
namespace {

inline int round_up32(int v) { return (v + 31) & ~31; }

template <int OP, typename Tin, typename Tout, int VPT, int PD = (VPT <= 4 ? 1 : 0)>
cudaError_t launch_resident(RowArgs a, cudaStream_t st) {
  a.tpr = round_up32((a.nvec + VPT - 1) / VPT);
  a.rpc = a.tpr >= 256 ? 1 : 256 / a.tpr;
  const int block = a.tpr * a.rpc;
  const void* fn = reinterpret_cast<const void*>(&resident_kernel<OP, Tin, Tout, VPT, PD>);
  const int grid = persistent_grid(fn, block, 0, (a.M + a.rpc - 1) / a.rpc);
  resident_kernel<OP, Tin, Tout, VPT, PD><<<grid, block, 0, st>>>(a);
  return cudaGetLastError();
}

template <int OP, typename Tin, typename Tout, int V>
cudaError_t launch_stream(RowArgs a, cudaStream_t st) {
  const int units = V == 1 ? a.N : a.nvec;
  int block = round_up32((units + 3) / 4);
  block = block < 32 ? 32 : (block > 1024 ? 1024 : block);
  a.tpr = block;
  a.rpc = 1;
  const void* fn = reinterpret_cast<const void*>(&stream_kernel<OP, Tin, Tout, V>);
  const int grid = persistent_grid(fn, block, 0, a.M);
  stream_kernel<OP, Tin, Tout, V><<<grid, block, 0, st>>>(a);
  return cudaGetLastError();
}

// Largest row (in 16-byte vectors) kept in registers: 128 KiB of fp32 (8 vectors
// per thread over 1024 threads) or 64 KiB of 16-bit data (4 vectors per thread;
// 8 packed 16-bit vectors per thread do not fit the 64-register budget).

// Shared memory given to a TMA CTA's ring (a few CTAs fit on one SM).
constexpr uint32_t kTmaRingBytes = 64u * 1024u;
// Longest row (bytes) the TMA kernel takes.
constexpr uint32_t kTmaMaxRow = 32768u;

template <int OP, typename Tin, typename Tout, int VPT>
cudaError_t launch_tma(RowArgs a, cudaStream_t st) {
  a.tpr = round_up32((a.nvec + VPT - 1) / VPT);
  a.rpc = 1;
  const int block = a.tpr + 32;
  const uint32_t row_bytes = static_cast<uint32_t>(a.N) * sizeof(Tin);
  uint32_t stages = kTmaRingBytes / row_bytes;
  stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
  const size_t smem = RingLayout::total_bytes(row_bytes, static_cast<int>(stages));
  const void* fn = reinterpret_cast<const void*>(&tma_norm_kernel<OP, Tin, Tout, VPT>);
  if (cudaError_t e = allow_dynamic_smem(fn, smem)) return e;
  const int grid = persistent_grid(fn, block, smem, a.M);
  tma_norm_kernel<OP, Tin, Tout, VPT><<<grid, block, smem, st>>>(a, static_cast<int>(stages), kWaitLimitNs);
  return cudaGetLastError();
}

// Cluster split: 1024-thread CTAs holding VPT vectors per thread, clusters of
// 2-8 CTAs (portable sizes): rows up to 8 * 1024 * 4 vectors (512 KiB of
// 16-bit data, 1 MiB of fp32 with 8 vectors per thread).
template <int OP, typename Tin, typename Tout, int VPT>
cudaError_t launch_cluster_v(RowArgs a, int C, cudaStream_t st) {
  const int slice_vecs = (a.nvec + C - 1) / C;
  const int block = 1024;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(C * sm_count());
  const int max_clusters = max_active_clusters(
      reinterpret_cast<const void*>(&cluster_norm_kernel<OP, Tin, Tout, VPT>), cfg, C, sm_count() / C);
  const int64_t nclusters = a.M < max_clusters ? a.M : max_clusters;
  cfg.gridDim = dim3(static_cast<unsigned>(nclusters * C));
  return cudaLaunchKernelEx(&cfg, cluster_norm_kernel<OP, Tin, Tout, VPT>, a, slice_vecs);
}

// Launch the cluster kernel; returns cudaErrorNotSupported when the row does
// not fit (the caller then streams it).
template <int OP, typename Tin, typename Tout>
cudaError_t launch_cluster(RowArgs a, cudaStream_t st) {
  constexpr int E = Elt<Tin>::kPerVec;
  constexpr int kVpt = (E == 4) ? 4 : 2;  // 16 elements per thread, as the resident kernel
  int C = (a.nvec + 1024 * kVpt - 1) / (1024 * kVpt);
  if (C < 2) C = 2;
  if (C <= 8) return launch_cluster_v<OP, Tin, Tout, kVpt>(a, C, st);
  // twice the vectors per thread
  C = (a.nvec + 1024 * 2 * kVpt - 1) / (1024 * 2 * kVpt);
  if (C <= 8) return launch_cluster_v<OP, Tin, Tout, 2 * kVpt>(a, C, st);
  return cudaErrorNotSupported;
}

template <int OP, typename Tin, typename Tout>
cudaError_t dispatch_rows(RowArgs a, cudaStream_t st) {
  constexpr int E = Elt<Tin>::kPerVec;
  const int path = kernel_path();
  const bool vec = (a.N % E == 0) && aligned(a.x, 16) &&
                   aligned(a.y, E * static_cast<int>(sizeof(Tout)));
  const bool weights_ok = (OP != kLayerNorm && OP != kRmsNorm) || a.wvec;
  if (vec && weights_ok && path != DSLPG_PATH_STREAM) {
    a.nvec = a.N / E;
    const uint32_t row_bytes = static_cast<uint32_t>(a.N) * sizeof(Tin);
    // The TMA pipeline is measured slower than register-resident rows on B200
    // for every benchmark shape, so it runs only when selected explicitly.
    if (path == DSLPG_PATH_TMA && row_bytes <= kTmaMaxRow) {
      // 32 elements per thread; fewer when the row is short.
      constexpr int kV = 32 / E;
      if (a.nvec >= 32 * kV) return launch_tma<OP, Tin, Tout, kV>(a, st);
      if (a.nvec > 32) return launch_tma<OP, Tin, Tout, 2>(a, st);
      return launch_tma<OP, Tin, Tout, 1>(a, st);
    }
    // Largest row (in 16-byte vectors) kept in registers: 128 KiB of fp32 (8
    // vectors per thread over 1024 threads) or 64 KiB of 16-bit data (4 vectors
    // per thread; 8 packed 16-bit vectors per thread do not fit the
    // 64-register budget).
    const int max_resident = (E == 4) ? 8192 : 4096;
    if (path == DSLPG_PATH_CLUSTER) {
      const cudaError_t e = launch_cluster<OP, Tin, Tout>(a, st);
      if (e != cudaErrorNotSupported) return e;
      cudaGetLastError();
    }
    if (a.nvec <= max_resident && path != DSLPG_PATH_TMA && path != DSLPG_PATH_CLUSTER) {
      // About 16 elements per thread (4 fp32 or 2 16-bit vectors), more only
      // when the row would need more than 1024 threads, fewer for short rows.
      constexpr int kBase = (E == 4) ? 4 : 2;
      // log_softmax: 32 elements per thread measured faster (fewer threads
      // per row to reduce over; its element work is the lightest).
      if constexpr (OP == kLogSoftmax && E == 8) {
        if (a.nvec >= 128 && a.nvec <= 4 * 1024) return launch_resident<OP, Tin, Tout, 4>(a, st);
      }
      if constexpr (E == 4) {
        if (a.nvec > 4 * 1024) return launch_resident<OP, Tin, Tout, 8>(a, st);
      }
      if (a.nvec > kBase * 1024) return launch_resident<OP, Tin, Tout, 4>(a, st);
      if (a.nvec >= 32 * kBase) {
        // softmax: two rows of loads in flight (free in registers at its occupancy)
        if constexpr (OP == kSoftmax && kBase == 2) return launch_resident<OP, Tin, Tout, 2, 2>(a, st);
        return launch_resident<OP, Tin, Tout, kBase>(a, st);
      }
      if (a.nvec > 32) return launch_resident<OP, Tin, Tout, 2>(a, st);
      return launch_resident<OP, Tin, Tout, 1>(a, st);
    }
    // Longer rows. Measured on B200: with at least as many rows as SMs the
    // two-pass stream kernel is faster (one cluster barrier per reduction
    // serialises a row across its CTAs); with fewer rows the cluster split
    // brings more SMs to each row (8 rows of 64K bf16: 10 us against 16 us).
    if (path != DSLPG_PATH_TMA && a.M < sm_count()) {
      const cudaError_t e = launch_cluster<OP, Tin, Tout>(a, st);
      if (e != cudaErrorNotSupported) return e;
      cudaGetLastError();  // clear a not-supported status
    }
    if (vec) return launch_stream<OP, Tin, Tout, E>(a, st);
  }
  if (vec) {
    a.nvec = a.N / E;
    return launch_stream<OP, Tin, Tout, E>(a, st);
  }
  a.nvec = 0;
  return launch_stream<OP, Tin, Tout, 1>(a, st);
}

template <int OP, typename Tin>
cudaError_t dispatch_out(RowArgs a, int out_dt, cudaStream_t st) {
  switch (out_dt) {
    case DSLPG_F32: return dispatch_rows<OP, Tin, float>(a, st);
    case DSLPG_F16: return dispatch_rows<OP, Tin, __half>(a, st);
    default: return dispatch_rows<OP, Tin, __nv_bfloat16>(a, st);
  }
}

template <int OP>
cudaError_t dispatch_in(RowArgs a, int in_dt, int out_dt, cudaStream_t st) {
  switch (in_dt) {
    case DSLPG_F32: return dispatch_out<OP, float>(a, out_dt, st);
    case DSLPG_F16: return dispatch_out<OP, __half>(a, out_dt, st);
    default: return dispatch_out<OP, __nv_bfloat16>(a, out_dt, st);
  }
}

// Same-dtype ops only instantiate the diagonal.
template <int OP>
cudaError_t dispatch_same(RowArgs a, int dt, cudaStream_t st) {
  switch (dt) {
    case DSLPG_F32: return dispatch_rows<OP, float, float>(a, st);
    case DSLPG_F16: return dispatch_rows<OP, __half, __half>(a, st);
    default: return dispatch_rows<OP, __nv_bfloat16, __nv_bfloat16>(a, st);
  }
}

int check_rows(const void* x, const void* y, int64_t M, int64_t N) {
  if (x == nullptr || y == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0 || N > 0x7fffffff) return DSLPG_ERR_BAD_SHAPE;
  return DSLPG_OK;
}

RowArgs make_args(const void* x, void* y, const void* w, const void* b, int64_t M, int64_t N,
                  int x_dt, int w_dt, float eps) {
  RowArgs a{};
  a.x = x;
  a.y = y;
  a.w = w;
  a.b = b;
  a.M = M;
  a.N = static_cast<int>(N);
  a.eps = eps;
  a.inv_n = 1.0f / static_cast<float>(N);
  a.wdt = w_dt;
  a.wvec = (w != nullptr && w_dt == x_dt && aligned(w, 16) && (b == nullptr || aligned(b, 16)))
               ? 1
               : 0;
  return a;
}

}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_layer_norm_fwd(const void* x, const void* weight, const void* bias, void* y,
                                    int64_t M, int64_t N, int x_dtype, int w_dtype, float eps,
                                    cudaStream_t stream) {
  if (int rc = check_rows(x, y, M, N)) return rc;
  if (weight == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (!(eps >= 0.f) || !(eps < kPosInf)) return DSLPG_ERR_BAD_EPS;
  if (M == 0 || N == 0) return DSLPG_OK;
  RowArgs a = make_args(x, y, weight, bias, M, N, x_dtype, w_dtype, eps);
  return static_cast<int>(dispatch_same<kLayerNorm>(a, x_dtype, stream));
}

extern "C" int dslpg_rms_norm_fwd(const void* x, const void* weight, void* y, int64_t M, int64_t N,
                                  int x_dtype, int w_dtype, float eps, cudaStream_t stream) {
  if (int rc = check_rows(x, y, M, N)) return rc;
  if (weight == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (!(eps >= 0.f) || !(eps < kPosInf)) return DSLPG_ERR_BAD_EPS;
  if (M == 0 || N == 0) return DSLPG_OK;
  RowArgs a = make_args(x, y, weight, nullptr, M, N, x_dtype, w_dtype, eps);
  return static_cast<int>(dispatch_same<kRmsNorm>(a, x_dtype, stream));
}

extern "C" int dslpg_softmax_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                                 cudaStream_t stream) {
  if (int rc = check_rows(x, y, M, N)) return rc;
  if (!is_float_dtype(dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (M == 0 || N == 0) return DSLPG_OK;
  RowArgs a = make_args(x, y, nullptr, nullptr, M, N, dtype, dtype, 0.f);
  return static_cast<int>(dispatch_same<kSoftmax>(a, dtype, stream));
}

namespace {
template <typename Tin, typename Tout>
cudaError_t launch_strided(const void* x, void* y, int64_t M, int64_t N, int64_t K,
                           cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&strided_log_softmax_kernel<Tin, Tout>);
  const int64_t cols = M * K;
  const int grid = persistent_grid(fn, 256, 0, (cols + 255) / 256);
  strided_log_softmax_kernel<Tin, Tout><<<grid, 256, 0, st>>>(static_cast<const Tin*>(x),
                                                              static_cast<Tout*>(y), M, N, K);
  return cudaGetLastError();
}
template <typename Tin>
cudaError_t strided_out(const void* x, void* y, int64_t M, int64_t N, int64_t K, int out_dt,
                        cudaStream_t st) {
  switch (out_dt) {
    case DSLPG_F32: return launch_strided<Tin, float>(x, y, M, N, K, st);
    case DSLPG_F16: return launch_strided<Tin, __half>(x, y, M, N, K, st);
    default: return launch_strided<Tin, __nv_bfloat16>(x, y, M, N, K, st);
  }
}
}  // namespace

extern "C" int dslpg_log_softmax_fwd(const void* x, void* y, int64_t M, int64_t N, int64_t K,
                                     int in_dtype, int out_dtype, cudaStream_t stream) {
  if (int rc = check_rows(x, y, M, N)) return rc;
  if (K < 1) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(in_dtype) || !is_float_dtype(out_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (M == 0 || N == 0) return DSLPG_OK;
  if (K == 1) {
    RowArgs a = make_args(x, y, nullptr, nullptr, M, N, in_dtype, in_dtype, 0.f);
    return static_cast<int>(dispatch_in<kLogSoftmax>(a, in_dtype, out_dtype, stream));
  }
  cudaError_t e;
  switch (in_dtype) {
    case DSLPG_F32: e = strided_out<float>(x, y, M, N, K, out_dtype, stream); break;
    case DSLPG_F16: e = strided_out<__half>(x, y, M, N, K, out_dtype, stream); break;
    default: e = strided_out<__nv_bfloat16>(x, y, M, N, K, out_dtype, stream); break;
  }
  return static_cast<int>(e);
}

namespace dslpg {
unsigned int take_wait_timeouts_rownorm() {
  unsigned int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero));
  return v;
}
}  // namespace dslpg
