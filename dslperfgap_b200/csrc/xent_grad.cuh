// xent_grad.cuh — the cross-entropy gradient of one row, shared by the
// backward kernel (xent_bwd.cu) and the fused forward + backward kernel
// (rowstat.cu).
//
// dlogits[c] = (dloss * scale) * p, where
//   p = exp(logits[c] * scale - lse);  p += 2 * lse_sq * lse * p;
//   p -= (1 - smoothing) (or 1 without smoothing) at the label's column;
//   p -= smoothing / total_classes (with smoothing);
// and rows whose label is ignored_index have dloss = 0. This is the
// arithmetic of ViperBench/cross_entropy/triton_impl.py:79-120 and
// pytorch_impl.py:93-141.
#pragma once

#include "common.cuh"

namespace dslpg {

// Per-row constants of the gradient.
struct GradRow {
  float k1;      // dloss * scale
  float lse;
  float fac;     // 2 * lse_sq * lse
  float sn;      // smoothing / total_classes (0 without smoothing)
  float lab;     // subtracted at the label column
  int64_t adj;   // label column (label - class_start)
};

DSLPG_DEV GradRow grad_row_consts(float dl, float scale, float lse, float lse_sq, bool smooth, float smoothing,
                                  float total_classes, int64_t label, int64_t class_start) {
  GradRow b;
  b.k1 = dl * scale;
  b.lse = lse;
  b.fac = 2.0f * lse_sq * lse;
  b.sn = smooth ? smoothing / total_classes : 0.f;
  b.lab = smooth ? (1.0f - smoothing) : 1.0f;
  b.adj = label - class_start;
  return b;
}

// The gradient of one element, exactly in the reference's order of operations.
DSLPG_DEV float grad_elem(const GradRow& b, float x, float scale, bool is_label, bool smooth) {
  float p = exp_shifted(x * scale - b.lse);
  p = p + b.fac * p;
  if (is_label) p = p - b.lab;
  if (smooth) p = p - b.sn;
  return b.k1 * p;
}

// Write the N gradients of one row (xr -> yr) with the tpr threads t of a
// group: 16-byte vectors (V > 1, nvec = N / V) or scalars (V == 1). The label
// column is rewritten afterwards by the thread that wrote its vector, so it is
// ordered after that thread's own vector store.
// LAST_USE: the row's loads carry an L2 evict-first policy (its last read).
// U: 16-byte loads in flight per thread.
template <typename T, int V, bool LAST_USE = false, int U = 4>
DSLPG_DEV void grad_row(const T* xr, T* yr, int nvec, int64_t N, const GradRow& b, float scale, bool smooth, int t,
                        int tpr) {
  if constexpr (V > 1) {
    constexpr int P = V / 2;
    const f32x2 nl2 = pk2(-b.lse * kLog2e, -b.lse * kLog2e);
    const f32x2 l2e2 = pk2(kLog2e * scale, kLog2e * scale);
    const f32x2 fac2 = pk2(b.fac, b.fac), nsn2 = pk2(-b.sn, -b.sn), k12 = pk2(b.k1, b.k1);
    uint64_t pol = 0;
    if constexpr (LAST_USE) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    for (int j0 = t; j0 < nvec; j0 += U * tpr) {
      Vec16 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        v[u] = Vec16{{0u, 0u, 0u, 0u}};
        if (j < nvec) {
          if constexpr (LAST_USE) {
            asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                : "=r"(v[u].w[0]), "=r"(v[u].w[1]), "=r"(v[u].w[2]), "=r"(v[u].w[3])
                : "l"(xr + static_cast<int64_t>(j) * V), "l"(pol));
          } else {
            v[u] = ld_stream(xr + static_cast<int64_t>(j) * V);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        if (j >= nvec) continue;
        f32x2 y[P];
#pragma unroll
        for (int p = 0; p < P; ++p) {
          // exp(x * scale - lse) = 2^(x * scale * log2e - lse * log2e)
          float d0, d1;
          upk2(fma2(unpack_pair<T>(v[u], p), l2e2, nl2), d0, d1);
          f32x2 e = pk2(ex2(d0), ex2(d1));
          e = fma2(fac2, e, e);
          if (smooth) e = add2(e, nsn2);
          y[p] = mul2(k12, e);
        }
        StorePairs<T, P>::run(yr + static_cast<int64_t>(j) * V, y);
      }
    }
  } else {
    for (int64_t c = t; c < N; c += tpr) yr[c] = from_f<T>(grad_elem(b, to_f(xr[c]), scale, false, smooth));
  }
  if (b.adj >= 0 && b.adj < N) {
    const int64_t unit = (V > 1) ? b.adj / V : b.adj;
    if (static_cast<int>(unit % tpr) == t) yr[b.adj] = from_f<T>(grad_elem(b, to_f(xr[b.adj]), scale, true, smooth));
  }
}

}  // namespace dslpg
