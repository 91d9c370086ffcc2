// rowstat.cu — reductions of a row (or row segment) to a few scalars:
// logsumexp and the blockwise cross-entropy forward (sm_100a).
//
// One kernel, rowstat_kernel, streams each work item (a row for logsumexp, a
// (row, column block) pair for cross-entropy) exactly once from HBM with
// 16-byte loads, U vectors in flight per thread, and keeps an online
// (max, sum of exp) pair per thread in the log2 domain:
//     t = x * scale * log2(e);  m = max t;  s = sum 2^(t - m)
// so each element costs one multiply, one max, one subtract, one SFU ex2 and
// one add. Per-thread pairs are merged with warp shuffles and a shared-memory
// step, and lse = (m + log2 s) * ln 2.
//
// Work item i maps to row r = i / nseg, block cb = i % nseg, so consecutive
// work items touch consecutive memory. Cross-entropy outputs land at flat
// index cb * n_rows + r, the layout of
// ViperBench/cross_entropy/triton_impl.py:46,75-76.
#include "common.cuh"
#include "pipe.cuh"
#include "xent_grad.cuh"

namespace dslpg {

enum StatKind : int { kLse = 0, kXent = 1 };

struct StatArgs {
  const void* x;
  int64_t M;      // rows
  int64_t N;      // columns
  int64_t ld;     // row stride in elements
  int64_t seg;    // segment (column block) length
  int64_t nseg;   // segments per row
  int tpr;        // threads per work item
  int rpc;        // work items per CTA
  float c;        // scale * log2(e)
  void* out;      // logsumexp: [M] of x's dtype
  // cross-entropy
  const void* labels;
  int label64;
  float* loss;
  float* lse;
  float* zloss;
  float smoothing, scale, lse_sq, total_classes;
  int64_t ignored, class_start;
  int split;
};

constexpr float kNaN = __builtin_nanf("");

// Fold a chunk of n log2-domain values into the running (m, s).
template <int n>
DSLPG_DEV void fold_chunk(float& m, float& s, const float* t) {
  float cm = t[0];
#pragma unroll
  for (int i = 1; i < n; ++i) cm = max_nan(cm, t[i]);
  const float nm = max_nan(m, cm);
  if (nm == kNegInf) return;  // nothing but -inf so far
  float acc = (m == nm) ? s : s * ex2(m - nm);
#pragma unroll
  for (int i = 0; i < n; ++i) acc += ex2(t[i] - nm);
  s = acc;
  m = nm;
}

// Fold NV full 16-byte vectors of T (every element valid) into the running
// (m, s) of t = x * c in the log2 domain; with SMOOTH also add the plain sum of
// x to `sum`. The chunk's extreme is found on the stored values (two 16-bit
// values per instruction); each element then costs half an fma.f32x2, one
// ex2 and half an add.f32x2. x * c - m is formed with a single rounding (fma),
// so the largest element contributes 2^r with |r| at most half an ulp of m.
template <typename T, int NV, bool SMOOTH, int POLY = 0>
DSLPG_DEV void fold_vecs(float& m, float& s, float& sum, const Vec16 (&v)[NV], float c) {
  constexpr int P = Elt<T>::kPerVec / 2;
  if constexpr (SMOOTH) {
    f32x2 s2 = pk2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int p = 0; p < P; ++p) s2 = add2(s2, unpack_pair<T>(v[k], p));
    sum += hsum2(s2);
  }
  // max(x * c) is c * max(x) for c >= 0 and c * min(x) for c < 0 (rounding
  // is monotonic); c == 0 gives 0 (NaN for non-finite x), as x * 0 does.
  const float ext = (c >= 0.f) ? RawExtreme<T, NV, false>::run(v) : RawExtreme<T, NV, true>::run(v);
  const float nm = max_nan(m, ext * c);
  if (nm == kNegInf) return;  // nothing but -inf so far
  const f32x2 c2 = pk2(c, c), nnm2 = pk2(-nm, -nm);
  f32x2 acc0 = pk2(0.f, 0.f), acc1 = pk2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const f32x2 d = fma2(unpack_pair<T>(v[k], p), c2, nnm2);
      f32x2 e;
      if (POLY > 0 && (k * P + p) % POLY == POLY - 1) {
        e = exp2_poly2(d);  // every POLY-th pair on the FMA pipe
      } else {
        float d0, d1;
        upk2(d, d0, d1);
        e = pk2(ex2(d0), ex2(d1));
      }
      if ((k * P + p) & 1) acc1 = add2(acc1, e);
      else acc0 = add2(acc0, e);
    }
  s = ((m == nm) ? s : s * ex2(m - nm)) + hsum2(add2(acc0, acc1));
  m = nm;
}

// fold_vecs for a partial chunk: vectors with ok[k] false are left out.
template <typename T, int NV, bool SMOOTH>
DSLPG_DEV void fold_vecs_masked(float& m, float& s, float& sum, const Vec16 (&v)[NV], const bool (&ok)[NV],
                                float c) {
  constexpr int E = Elt<T>::kPerVec;
  float tv[NV * E];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float f[E];
    unpack<T>(v[k], f);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      tv[k * E + i] = ok[k] ? f[i] * c : kNegInf;
      if constexpr (SMOOTH) sum += ok[k] ? f[i] : 0.f;
    }
  }
  fold_chunk<NV * E>(m, s, tv);
}

// The label of row r and, when it falls in the block [col0, hi), its scaled
// logit: loaded when the item starts, so the two dependent loads overlap the
// item's stream instead of following it.
struct LabelPick {
  int64_t label;
  float xl;      // logit[label] * scale (0 when the label is not in the block)
  bool in_block;
};

template <typename T>
DSLPG_DEV LabelPick pick_label(const StatArgs& a, int64_t r, int64_t cb, int64_t col0) {
  LabelPick p;
  p.label = a.label64 ? static_cast<const int64_t*>(a.labels)[r]
                      : static_cast<int64_t>(static_cast<const int32_t*>(a.labels)[r]);
  const int64_t adj = p.label - a.class_start;
  const int64_t hi = (cb + 1) * a.seg < a.N ? (cb + 1) * a.seg : a.N;
  p.in_block = p.label != a.ignored && adj >= col0 && adj < hi;
  p.xl = p.in_block ? to_f(static_cast<const T*>(a.x)[r * a.ld + adj]) * a.scale : 0.f;
  return p;
}

// Write the results of work item (row r, block cb) from the merged online
// statistics: gm = max of t, gs = sum of 2^(t - gm), gsum = sum of x (SMOOTH),
// and (cross-entropy) the item's label pick.
template <int KIND, typename T, bool SMOOTH>
DSLPG_DEV void finish_item(const StatArgs& a, int64_t r, int64_t cb, float gm, float gs, float gsum,
                           const LabelPick& lp) {
  const float lse_fin = (gm + log2f(gs)) * kLn2;
  if constexpr (KIND == kLse) {
    // torch.logsumexp shifts by the max only when it is finite.
    float v = lse_fin;
    if (gm == kPosInf) v = kPosInf;
    else if (gm == kNegInf) v = kNegInf;
    static_cast<T*>(a.out)[r] = from_f<T>(v);
  } else {
    const float lse = (fabsf(gm) < kPosInf) ? lse_fin : kNaN;
    const int64_t oi = cb * a.M + r;
    a.lse[oi] = lse;
    float loss = 0.f, z = 0.f;
    if (lp.label != a.ignored) {
      const float lse_term = a.split ? 0.f : lse;
      const float sum_logits = gsum * a.scale;
      if (lp.in_block) {
        if constexpr (SMOOTH)
          loss = lse_term - a.smoothing * sum_logits / a.total_classes - (1.f - a.smoothing) * lp.xl;
        else
          loss = lse_term - lp.xl;
      } else if constexpr (SMOOTH) {
        loss = a.smoothing * (lse_term - sum_logits / a.total_classes);
      }
      if (!a.split) {
        z = a.lse_sq * lse * lse;
        loss += z;
      }
    }
    a.loss[oi] = loss;
    a.zloss[oi] = z;
  }
}

// finish_item with the label loaded at the end (kernels that do not prefetch it).
template <int KIND, typename T, bool SMOOTH>
DSLPG_DEV void finish_item(const StatArgs& a, int64_t r, int64_t cb, int64_t col0, float gm, float gs,
                           float gsum) {
  LabelPick lp{0, 0.f, false};
  if constexpr (KIND == kXent) lp = pick_label<T>(a, r, cb, col0);
  finish_item<KIND, T, SMOOTH>(a, r, cb, gm, gs, gsum, lp);
}

template <int KIND, typename T, int V, bool SMOOTH, int POLY, bool PF = false, int UV = 4, int MINB = 1>
__global__ void __launch_bounds__(256, MINB) rowstat_kernel(const StatArgs a) {
  constexpr int U = (V == 1) ? 8 : UV;  // loads in flight per thread per iteration
  __shared__ float red[2][32];
  const int g = threadIdx.x / a.tpr;
  const int t = threadIdx.x - g * a.tpr;
  const int nw = a.tpr >> 5;
  const int first_warp = g * nw;
  int buf = 0;
  const int64_t items = a.M * a.nseg;
  const int64_t step = static_cast<int64_t>(gridDim.x) * a.rpc;

  for (int64_t base = static_cast<int64_t>(blockIdx.x) * a.rpc; base < items; base += step) {
    const int64_t item = base + g;
    const bool iv = item < items;
    const int64_t r = iv ? item / a.nseg : 0;
    const int64_t cb = iv ? item - r * a.nseg : 0;
    const int64_t col0 = cb * a.seg;
    const int64_t len = iv ? ((a.N - col0) < a.seg ? (a.N - col0) : a.seg) : 0;
    const T* xs = static_cast<const T*>(a.x) + r * a.ld + col0;

    LabelPick lp{0, 0.f, false};
    if constexpr (KIND == kXent)
      if (t == 0 && iv) lp = pick_label<T>(a, r, cb, col0);
    // logsumexp: the same kind of row-start scalar read (the item's first
    // element), consumed at the finish. Measured on B200, logsumexp bf16
    // [8192,128256]: 0.903 -> 0.947 of the measured copy bandwidth, repeatable,
    // at unchanged occupancy; why it helps (the compiled schedule differs) is
    // not established.
    if constexpr (KIND == kLse)
      if (t == 0 && iv) lp.xl = to_f(static_cast<const T*>(a.x)[r * a.ld + col0]);
    float m = kNegInf, s = 0.f, sum = 0.f;
    int64_t done = 0;
    if constexpr (V > 1) {
      const int64_t nv = len / V;
      const int64_t stride = static_cast<int64_t>(U) * a.tpr;
      auto load = [&](Vec16 (&dst)[U], int64_t j0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
          dst[u] = Vec16{{0u, 0u, 0u, 0u}};
          if (j < nv) dst[u] = ld_stream(xs + j * V);
        }
      };
      Vec16 nx[PF ? U : 1];
      if constexpr (PF) load(nx, t);
      for (int64_t j0 = t; j0 < nv; j0 += stride) {
        Vec16 v[U];
        if constexpr (PF) {
#pragma unroll
          for (int u = 0; u < U; ++u) v[u] = nx[u];
          if (j0 + stride < nv) load(nx, j0 + stride);
        } else {
          load(v, j0);
        }
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) ok[u] = j0 + static_cast<int64_t>(u) * a.tpr < nv;
        if (ok[U - 1]) fold_vecs<T, U, SMOOTH, POLY>(m, s, sum, v, a.c);
        else fold_vecs_masked<T, U, SMOOTH>(m, s, sum, v, ok, a.c);
      }
      done = nv * V;
    }
    // Scalar remainder (the whole item on the scalar path).
    for (int64_t j0 = done + t; j0 < len; j0 += static_cast<int64_t>(U) * a.tpr) {
      float tv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
        float f = 0.f;
        if (j < len) f = to_f(xs[j]);
        if constexpr (SMOOTH) sum += f;
        tv[u] = (j < len) ? f * a.c : kNegInf;
      }
      fold_chunk<U>(m, s, tv);
    }

    // Merge the group's (m, s) pairs.
    const float gm = group_reduce<MaxOp>(m, red[buf], nw, first_warp);
    buf ^= 1;
    const float sc = (m == gm) ? s : s * ex2(m - gm);
    const float gs = group_reduce<SumOp>(sc, red[buf], nw, first_warp);
    buf ^= 1;
    float gsum = 0.f;
    if constexpr (SMOOTH) {
      gsum = group_reduce<SumOp>(sum, red[buf], nw, first_warp);
      buf ^= 1;
    }

    if constexpr (KIND == kLse) asm volatile("" ::"f"(lp.xl));  // keeps the row-start read
    if (t == 0 && iv) finish_item<KIND, T, SMOOTH>(a, r, cb, gm, gs, gsum, lp);
  }
}

// Cross-entropy forward and backward in one kernel, for a row that is one
// column block (BLOCK_SIZE >= n_cols) and a dloss known before the forward
// (a mean or sum of the losses). One CTA of fused_threads() per row, one CTA per
// SM: pass 1 streams the row from HBM into the online statistics (as
// rowstat_kernel) and writes loss / lse / z_loss; pass 2 reads the row again,
// now from L2 (the rows in flight take about 250 KiB each, 148 of them well
// inside the 126 MB L2), and writes dlogits with the backward's arithmetic.
// HBM traffic: the logits once and dlogits once, against the logits twice for
// a forward followed by a backward. Pass 1 reads with an L2 evict-last policy.
DSLPG_DEV Vec16 ld_policy(const void* p, uint64_t pol) {
  Vec16 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
      : "l"(p), "l"(pol));
  return v;
}

struct FusedArgs {
  StatArgs s;
  const void* dloss;
  int dloss_dt;
  int64_t dloss_stride;
  void* dx;
  int64_t ldo;
  int nvec;  // N / V on the vector path
};

// Threads per row: 1024; 512 with smoothing, whose extra sum of the logits
// does not fit the 64 registers a thread has at 1024 threads.
#ifndef DSLPG_FUSED_CTAS
#define DSLPG_FUSED_CTAS 1  // CTAs per SM
#endif
template <bool SMOOTH>
constexpr int fused_threads() {
  return (SMOOTH ? 512 : 1024) / DSLPG_FUSED_CTAS;
}

// 16-byte loads in flight per thread in pass 2 (with the next chunk prefetched)
#ifndef DSLPG_FUSED_PASS2_U
#define DSLPG_FUSED_PASS2_U 2
#endif

template <typename T, int V, bool SMOOTH>
__global__ void __launch_bounds__(fused_threads<SMOOTH>(), DSLPG_FUSED_CTAS) xent_fused_kernel(const FusedArgs f) {
  constexpr int U = 4;
  constexpr int kFusedThreads = fused_threads<SMOOTH>();
  const StatArgs& a = f.s;
  __shared__ float red[2][32];
  const int t = threadIdx.x, nw = kFusedThreads / 32;
  int buf = 0;
  for (int64_t r = blockIdx.x; r < a.M; r += gridDim.x) {
    const T* xr = static_cast<const T*>(a.x) + r * a.ld;
    // every thread needs the label and dloss (pass 2); loaded now, their latency hides behind pass 1
    const LabelPick lp = pick_label<T>(a, r, 0, 0);
    const float dl_row = load_any(f.dloss, r * f.dloss_stride, f.dloss_dt);
    float m = kNegInf, s = 0.f, sum = 0.f;
    // pass 1 marks the row's lines evict-last so that pass 2 finds them in L2
    // (without the hint it read about 1.8x the logits from DRAM)
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    if constexpr (V > 1) {
      const int64_t nv = f.nvec, stride = static_cast<int64_t>(U) * kFusedThreads;
      auto load = [&](Vec16 (&dst)[U], int64_t j0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * kFusedThreads;
          dst[u] = Vec16{{0u, 0u, 0u, 0u}};
          if (j < nv) dst[u] = ld_policy(xr + j * V, pol);
        }
      };
      Vec16 nx[U];
      load(nx, t);
      for (int64_t j0 = t; j0 < nv; j0 += stride) {
        Vec16 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = nx[u];
        if (j0 + stride < nv) load(nx, j0 + stride);
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) ok[u] = j0 + static_cast<int64_t>(u) * kFusedThreads < nv;
        if (ok[U - 1]) fold_vecs<T, U, SMOOTH, 4>(m, s, sum, v, a.c);
        else fold_vecs_masked<T, U, SMOOTH>(m, s, sum, v, ok, a.c);
      }
    } else {
      for (int64_t j0 = t; j0 < a.N; j0 += static_cast<int64_t>(U) * kFusedThreads) {
        float tv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * kFusedThreads;
          float x = 0.f;
          if (j < a.N) x = to_f(xr[j]);
          if constexpr (SMOOTH) sum += x;
          tv[u] = (j < a.N) ? x * a.c : kNegInf;
        }
        fold_chunk<U>(m, s, tv);
      }
    }
    const float gm = group_reduce<MaxOp>(m, red[buf], nw, 0);
    buf ^= 1;
    const float gs = group_reduce<SumOp>((m == gm) ? s : s * ex2(m - gm), red[buf], nw, 0);
    buf ^= 1;
    float gsum = 0.f;
    if constexpr (SMOOTH) {
      gsum = group_reduce<SumOp>(sum, red[buf], nw, 0);
      buf ^= 1;
    }
    if (t == 0) finish_item<kXent, T, SMOOTH>(a, r, 0, gm, gs, gsum, lp);
    // the lse finish_item stored, formed the same way by every thread
    const float lse = (fabsf(gm) < kPosInf) ? (gm + log2f(gs)) * kLn2 : kNaN;
    const float dl = (lp.label != a.ignored) ? dl_row : 0.f;
    const GradRow b =
        grad_row_consts(dl, a.scale, lse, a.lse_sq, SMOOTH, a.smoothing, a.total_classes, lp.label, a.class_start);
    grad_row<T, V, DSLPG_FUSED_PASS2_U>(xr, static_cast<T*>(f.dx) + r * f.ldo, f.nvec, a.N, b, a.scale, SMOOTH, t,
                                        kFusedThreads);
  }
}

// Counts waits that ran out of time in this file's kernels.
static __device__ unsigned int g_wait_timeouts;

// TMA-pipelined variant for long work items (vocab-sized rows): warp 0 lane 0
// streams each item of the CTA (items blockIdx.x, blockIdx.x + gridDim.x, ...)
// in chunks of up to chunk_bytes into the shared-memory ring; the consumer
// warps fold every chunk into per-thread online statistics (VPC vectors per
// thread per chunk), release the slot, and merge per item. Timeouts are
// handled as in the normalising TMA kernel: the loop shape never changes, so
// the consumers' named barriers stay matched.
template <int KIND, typename T, bool SMOOTH, int VPC>
__global__ void __launch_bounds__(544) tma_stat_kernel(const StatArgs a, int stages, uint32_t chunk_bytes,
                                                        unsigned long long limit_ns) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int E = Elt<T>::kPerVec;
  __shared__ volatile int abort_flag;
  const int ncw = (blockDim.x >> 5) - 1;
  const int C = ncw * 32;
  if (threadIdx.x == 0) abort_flag = 0;
  float* red;
  const Ring ring = ring_setup(smem, chunk_bytes, stages, ncw, &red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t items = a.M * a.nseg;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t u = 0;
      bool stop = false;
      for (int64_t item = blockIdx.x; item < items && !stop; item += gridDim.x) {
        const int64_t r = item / a.nseg, cb = item - r * a.nseg;
        const int64_t col0 = cb * a.seg;
        const int64_t len = (a.N - col0) < a.seg ? (a.N - col0) : a.seg;
        const char* src = reinterpret_cast<const char*>(static_cast<const T*>(a.x) + r * a.ld + col0);
        const uint32_t bytes = static_cast<uint32_t>(len * sizeof(T));
        for (uint32_t off = 0; off < bytes; off += chunk_bytes, ++u) {
          if (abort_flag) { stop = true; break; }
          if (u >= static_cast<uint32_t>(stages) && !mbar_wait(ring.empty_bar(u), ring.parity(u) ^ 1u, limit_ns)) {
            atomicAdd(&g_wait_timeouts, 1u);
            abort_flag = 1;
            stop = true;
            break;
          }
          const uint32_t n = (bytes - off) < chunk_bytes ? (bytes - off) : chunk_bytes;
          mbar_arrive_expect_tx(ring.full_bar(u), n);
          bulk_load(ring.slot(u), src + off, n, ring.full_bar(u), pol);
        }
      }
      if (!ring_drain(ring, u)) atomicAdd(&g_wait_timeouts, 1u);
    }
    return;
  }

  const int t = threadIdx.x - 32;
  ConsumerReducer rd{red, ncw, 0};
  uint32_t u = 0;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int64_t r = item / a.nseg, cb = item - r * a.nseg;
    const int64_t col0 = cb * a.seg;
    const int64_t len = (a.N - col0) < a.seg ? (a.N - col0) : a.seg;
    const uint32_t bytes = static_cast<uint32_t>(len * sizeof(T));
    float m = kNegInf, s = 0.f, sum = 0.f;
    for (uint32_t off = 0; off < bytes; off += chunk_bytes, ++u) {
      if (!abort_flag && !mbar_wait(ring.full_bar(u), ring.parity(u), limit_ns)) {
        atomicAdd(&g_wait_timeouts, 1u);
        abort_flag = 1;
      }
      const uint32_t nv = ((bytes - off) < chunk_bytes ? (bytes - off) : chunk_bytes) / 16u;
      const uint32_t slot = ring.slot(u);
      Vec16 v[VPC];
#pragma unroll
      for (int k = 0; k < VPC; ++k) {
        const uint32_t j = t + k * C;
        v[k] = Vec16{{0u, 0u, 0u, 0u}};
        if (j < nv) v[k] = lds16(slot + 16u * j);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(ring.empty_bar(u));
      bool ok[VPC];
#pragma unroll
      for (int k = 0; k < VPC; ++k) ok[k] = static_cast<uint32_t>(t + k * C) < nv;
      if (ok[VPC - 1]) fold_vecs<T, VPC, SMOOTH>(m, s, sum, v, a.c);
      else fold_vecs_masked<T, VPC, SMOOTH>(m, s, sum, v, ok, a.c);
    }
    const float gm = rd.template reduce<MaxOp>(m);
    const float sc = (m == gm) ? s : s * ex2(m - gm);
    const float gs = rd.template reduce<SumOp>(sc);
    float gsum = 0.f;
    if constexpr (SMOOTH) gsum = rd.template reduce<SumOp>(sum);
    if (t == 0 && !abort_flag) finish_item<KIND, T, SMOOTH>(a, r, cb, col0, gm, gs, gsum);
  }
}

// Few long work items: each item split over the CTAs of a thread-block
// cluster. Every CTA folds its contiguous slice of the item (the same online
// fold as rowstat_kernel, next loads prefetched), the per-CTA (max, sum[, x
// sum]) are merged through distributed shared memory (ClusterReducer), and
// rank 0 writes the item's results. Clusters loop over items.
template <int KIND, typename T, bool SMOOTH>
__global__ void __launch_bounds__(512) cluster_stat_kernel(const StatArgs a, int64_t slice_vecs) {
  constexpr int V = Elt<T>::kPerVec;
  constexpr int U = 4;
  __shared__ float red[2][32];
  __shared__ float slots[2];
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int C = static_cast<int>(cl.num_blocks());
  const int rank = static_cast<int>(cl.block_rank());
  const int64_t nclusters = gridDim.x / C;
  const int64_t cid = blockIdx.x / C;
  const int t = threadIdx.x, nt = blockDim.x;
  const int64_t items = a.M * a.nseg;
  ClusterReducer rd{slots, red, 0, C};

  for (int64_t item = cid; item < items; item += nclusters) {
    const int64_t r = item / a.nseg, cb = item - r * a.nseg;
    const int64_t col0 = cb * a.seg;
    const int64_t len = (a.N - col0) < a.seg ? (a.N - col0) : a.seg;
    const int64_t nvi = len / V;
    const int64_t j_lo = rank * slice_vecs;
    const int64_t j_hi = (j_lo + slice_vecs) < nvi ? (j_lo + slice_vecs) : nvi;
    const T* xs = static_cast<const T*>(a.x) + r * a.ld + col0;
    float m = kNegInf, s = 0.f, sum = 0.f;
    auto load = [&](Vec16 (&dst)[U], int64_t j0) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + static_cast<int64_t>(u) * nt;
        dst[u] = Vec16{{0u, 0u, 0u, 0u}};
        if (j < j_hi) dst[u] = ld_stream(xs + j * V);
      }
    };
    Vec16 nx[U];
    load(nx, j_lo + t);
    for (int64_t j0 = j_lo + t; j0 < j_hi; j0 += static_cast<int64_t>(U) * nt) {
      Vec16 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = nx[u];
      load(nx, j0 + static_cast<int64_t>(U) * nt);
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) ok[u] = j0 + static_cast<int64_t>(u) * nt < j_hi;
      if (ok[U - 1]) fold_vecs<T, U, SMOOTH, 4>(m, s, sum, v, a.c);
      else fold_vecs_masked<T, U, SMOOTH>(m, s, sum, v, ok, a.c);
    }
    const float gm = rd.template reduce<MaxOp>(m);
    const float sc = (m == gm) ? s : s * ex2(m - gm);
    const float gs = rd.template reduce<SumOp>(sc);
    float gsum = 0.f;
    if constexpr (SMOOTH) gsum = rd.template reduce<SumOp>(sum);
    if (rank == 0 && t == 0) finish_item<KIND, T, SMOOTH>(a, r, cb, col0, gm, gs, gsum);
  }
  cl.sync();  // no CTA leaves while another may still read its exchange slots
}

namespace {

inline int round_up32(int v) { return (v + 31) & ~31; }

template <int KIND, typename T, int V, bool SMOOTH, int POLY = 0, bool PF = false, int UV = 4, int MINB = 1>
cudaError_t launch_stat(StatArgs a, cudaStream_t st) {
  // Threads per work item: about 16 vectors (or 64 scalars) per thread per item.
  const int64_t units = (V > 1) ? a.seg / V : a.seg;
  const int64_t per_thread = (V > 1) ? 16 : 64;
  int64_t want = (units + per_thread - 1) / per_thread;
  int tpr = static_cast<int>(want > 256 ? 256 : want);
  tpr = round_up32(tpr < 32 ? 32 : tpr);
  a.tpr = tpr;
  a.rpc = tpr >= 256 ? 1 : 256 / tpr;
  const int block = a.tpr * a.rpc;
  const void* fn = reinterpret_cast<const void*>(&rowstat_kernel<KIND, T, V, SMOOTH, POLY, PF, UV, MINB>);
  const int64_t items = a.M * a.nseg;
  const int grid = persistent_grid(fn, block, 0, (items + a.rpc - 1) / a.rpc);
  rowstat_kernel<KIND, T, V, SMOOTH, POLY, PF, UV, MINB><<<grid, block, 0, st>>>(a);
  return cudaGetLastError();
}

// TMA path (selected explicitly): work items streamed in chunks of
// kTmaChunk bytes through a ring of kTmaStages slots (two CTAs per SM).
constexpr uint32_t kTmaChunk = 16u * 1024u;
constexpr int kTmaStages = 6;
constexpr int kTmaConsumers = 256;

template <int KIND, typename T, bool SMOOTH, int VPC>
cudaError_t launch_tma_stat_v(StatArgs a, cudaStream_t st, int consumers, int stages) {
  a.tpr = consumers;
  a.rpc = 1;
  const int block = consumers + 32;
  const size_t smem = RingLayout::total_bytes(kTmaChunk, stages);
  const void* fn = reinterpret_cast<const void*>(&tma_stat_kernel<KIND, T, SMOOTH, VPC>);
  if (cudaError_t e = allow_dynamic_smem(fn, smem)) return e;
  const int grid = persistent_grid(fn, block, smem, a.M * a.nseg);
  tma_stat_kernel<KIND, T, SMOOTH, VPC><<<grid, block, smem, st>>>(a, stages, kTmaChunk, kWaitLimitNs);
  return cudaGetLastError();
}

template <int KIND, typename T, bool SMOOTH>
cudaError_t launch_tma_stat(StatArgs a, cudaStream_t st) {
  return launch_tma_stat_v<KIND, T, SMOOTH, 4>(a, st, kTmaConsumers, kTmaStages);
}

// Cluster split for few long items: returns cudaErrorNotSupported when it
// does not apply.
template <int KIND, typename T, bool SMOOTH>
cudaError_t launch_cluster_stat(StatArgs a, cudaStream_t st) {
  constexpr int V = Elt<T>::kPerVec;
  const int64_t items = a.M * a.nseg;
  const int64_t nv = a.seg / V;  // vectors of a full item
  // about 32 vectors per thread of a 512-thread CTA per slice
  int64_t C = (nv + 32 * 512 - 1) / (32 * 512);
  if (C < 2) C = 2;
  if (C > 8) C = 8;
  const int64_t slice_vecs = (nv + C - 1) / C;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(512);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(C * sm_count()));
  const int max_clusters = max_active_clusters(reinterpret_cast<const void*>(&cluster_stat_kernel<KIND, T, SMOOTH>),
                                               cfg, static_cast<int>(C), static_cast<int>(sm_count() / C));
  const int64_t nclusters = items < max_clusters ? items : max_clusters;
  cfg.gridDim = dim3(static_cast<unsigned>(nclusters * C));
  return cudaLaunchKernelEx(&cfg, cluster_stat_kernel<KIND, T, SMOOTH>, a, slice_vecs);
}

template <int KIND, typename T, bool SMOOTH>
cudaError_t dispatch_vec(StatArgs a, cudaStream_t st) {
  constexpr int E = Elt<T>::kPerVec;
  const int path = kernel_path();
  const bool vec = aligned(a.x, 16) && (a.ld % E == 0) && (a.seg % E == 0);
  // every item's byte count must be a multiple of 16 for the bulk copies
  const bool tma_ok = vec && (a.N % E == 0);
  const int64_t item_bytes = a.seg * static_cast<int64_t>(sizeof(T));
  // Explicit selection only: the register kernel is measured faster on B200.
  if (tma_ok && path == DSLPG_PATH_TMA && item_bytes > 0)
    return launch_tma_stat<KIND, T, SMOOTH>(a, st);
  // Measured best on B200 for vocab-sized rows: next loads prefetched, one
  // exponential pair in four on the FMA pipe, registers bounded to three
  // CTAs per SM.
  // Few long items (fewer than SMs, at least 128 KiB each): one cluster of
  // CTAs per item instead of one CTA group. Measured on B200: 4 rows of 1M
  // bf16 16 us against 94 us; 64 rows of 128256 bf16 14 us against 19 us.
  const bool few_long = a.M * a.nseg < sm_count() && item_bytes >= 128 * 1024;
  if (tma_ok && (path == DSLPG_PATH_CLUSTER || (path == DSLPG_PATH_AUTO && few_long)))
    return launch_cluster_stat<KIND, T, SMOOTH>(a, st);
  // With smoothing (the extra sum of the logits) the register bound of three
  // CTAs spilled; two CTAs hold it in registers (vocab rows: 4982 against
  // 4933 GB/s).
  if (vec && path != DSLPG_PATH_STREAM)
    return launch_stat<KIND, T, E, SMOOTH, 4, true, 4, (SMOOTH ? 2 : 3)>(a, st);
  return launch_stat<KIND, T, 1, SMOOTH>(a, st);
}

template <int KIND, bool SMOOTH>
cudaError_t dispatch_dtype(StatArgs a, int dt, cudaStream_t st) {
  switch (dt) {
    case DSLPG_F32: return dispatch_vec<KIND, float, SMOOTH>(a, st);
    case DSLPG_F16: return dispatch_vec<KIND, __half, SMOOTH>(a, st);
    default: return dispatch_vec<KIND, __nv_bfloat16, SMOOTH>(a, st);
  }
}

template <typename T, bool SMOOTH>
cudaError_t launch_fused_t(FusedArgs f, cudaStream_t st) {
  constexpr int E = Elt<T>::kPerVec;
  const bool vec = aligned(f.s.x, 16) && aligned(f.dx, 16) && f.s.N % E == 0 && f.s.ld % E == 0 && f.ldo % E == 0 &&
                   f.s.N / E <= 0x7fffffff;
  const int64_t cap = static_cast<int64_t>(sm_count()) * DSLPG_FUSED_CTAS;  // rows in flight stay in L2
  const int64_t rows = f.s.M < cap ? f.s.M : cap;
  if (vec) {
    f.nvec = static_cast<int>(f.s.N / E);
    xent_fused_kernel<T, E, SMOOTH><<<static_cast<int>(rows), fused_threads<SMOOTH>(), 0, st>>>(f);
  } else {
    f.nvec = 0;
    xent_fused_kernel<T, 1, SMOOTH><<<static_cast<int>(rows), fused_threads<SMOOTH>(), 0, st>>>(f);
  }
  return cudaGetLastError();
}

template <bool SMOOTH>
cudaError_t launch_fused(FusedArgs f, int dt, cudaStream_t st) {
  switch (dt) {
    case DSLPG_F32: return launch_fused_t<float, SMOOTH>(f, st);
    case DSLPG_F16: return launch_fused_t<__half, SMOOTH>(f, st);
    default: return launch_fused_t<__nv_bfloat16, SMOOTH>(f, st);
  }
}

}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_logsumexp_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                                   cudaStream_t stream) {
  if (x == nullptr || y == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (M == 0) return DSLPG_OK;
  if (N == 0) return DSLPG_ERR_BAD_SHAPE;  // torch.logsumexp of an empty row is -inf; callers handle it
  StatArgs a{};
  a.x = x;
  a.M = M;
  a.N = N;
  a.ld = N;
  a.seg = N;
  a.nseg = 1;
  a.c = kLog2e;
  a.out = y;
  return static_cast<int>(dispatch_dtype<kLse, false>(a, dtype, stream));
}

extern "C" int dslpg_cross_entropy_fwd(const void* logits, const void* labels, float* loss,
                                       float* lse, float* z_loss, int64_t n_rows, int64_t n_cols,
                                       int64_t logits_row_stride, int logits_dtype,
                                       int labels_dtype, float smoothing, float logit_scale,
                                       float lse_square_scale, int64_t ignored_index,
                                       float total_classes, int64_t class_start_idx,
                                       int64_t block_size, int has_smoothing, int split,
                                       cudaStream_t stream) {
  if (!logits || !labels || !loss || !lse || !z_loss) return DSLPG_ERR_NULL_POINTER;
  if (n_rows < 0 || n_cols < 0 || block_size <= 0 || logits_row_stride < n_cols)
    return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(logits_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (labels_dtype != DSLPG_I32 && labels_dtype != DSLPG_I64) return DSLPG_ERR_BAD_DTYPE;
  if (n_rows == 0 || n_cols == 0) return DSLPG_OK;
  StatArgs a{};
  a.x = logits;
  a.M = n_rows;
  a.N = n_cols;
  a.ld = logits_row_stride;
  // One segment per column block; a block wider than the row is the whole row.
  a.seg = block_size < n_cols ? block_size : n_cols;
  a.nseg = (n_cols + block_size - 1) / block_size;
  a.c = logit_scale * kLog2e;
  a.labels = labels;
  a.label64 = labels_dtype == DSLPG_I64 ? 1 : 0;
  a.loss = loss;
  a.lse = lse;
  a.zloss = z_loss;
  a.smoothing = smoothing;
  a.scale = logit_scale;
  a.lse_sq = lse_square_scale;
  a.total_classes = total_classes;
  a.ignored = ignored_index;
  a.class_start = class_start_idx;
  a.split = split ? 1 : 0;
  cudaError_t e = has_smoothing ? dispatch_dtype<kXent, true>(a, logits_dtype, stream)
                                : dispatch_dtype<kXent, false>(a, logits_dtype, stream);
  return static_cast<int>(e);
}

namespace dslpg {
unsigned int take_wait_timeouts_rowstat() {
  unsigned int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero));
  return v;
}
}  // namespace dslpg

extern "C" int dslpg_cross_entropy_fwd_bwd(const void* logits, const void* labels, const void* dloss, int dloss_dtype,
                                           int64_t dloss_stride, float* loss, float* lse, float* z_loss,
                                           void* dlogits, int64_t n_rows, int64_t n_cols, int64_t logits_row_stride,
                                           int64_t dlogits_row_stride, int logits_dtype, int labels_dtype,
                                           float smoothing, float logit_scale, float lse_square_scale,
                                           int64_t ignored_index, float total_classes, int64_t class_start_idx,
                                           int has_smoothing, cudaStream_t stream) {
  if (!logits || !labels || !dloss || !loss || !lse || !z_loss || !dlogits) return DSLPG_ERR_NULL_POINTER;
  if (n_rows < 0 || n_cols < 0 || logits_row_stride < n_cols || dlogits_row_stride < n_cols || dloss_stride < 0)
    return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(logits_dtype) || !is_float_dtype(dloss_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (labels_dtype != DSLPG_I32 && labels_dtype != DSLPG_I64) return DSLPG_ERR_BAD_DTYPE;
  if (n_rows == 0 || n_cols == 0) return DSLPG_OK;
  FusedArgs f{};
  StatArgs& a = f.s;
  a.x = logits;
  a.M = n_rows;
  a.N = n_cols;
  a.ld = logits_row_stride;
  a.seg = n_cols;
  a.nseg = 1;
  a.c = logit_scale * kLog2e;
  a.labels = labels;
  a.label64 = labels_dtype == DSLPG_I64 ? 1 : 0;
  a.loss = loss;
  a.lse = lse;
  a.zloss = z_loss;
  a.smoothing = smoothing;
  a.scale = logit_scale;
  a.lse_sq = lse_square_scale;
  a.total_classes = total_classes;
  a.ignored = ignored_index;
  a.class_start = class_start_idx;
  a.split = 0;
  f.dloss = dloss;
  f.dloss_dt = dloss_dtype;
  f.dloss_stride = dloss_stride;
  f.dx = dlogits;
  f.ldo = dlogits_row_stride;
  cudaError_t e = has_smoothing ? launch_fused<true>(f, logits_dtype, stream) : launch_fused<false>(f, logits_dtype, stream);
  return static_cast<int>(e);
}
