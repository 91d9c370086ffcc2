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

// The per-row constants of the vector path, packed in f32x2 pairs.
struct GradPairs {
  f32x2 nl2, l2e2, fac2, nsn2, k12;
};

DSLPG_DEV GradPairs grad_pairs(const GradRow& b, float scale) {
  GradPairs c;
  c.nl2 = pk2(-b.lse * kLog2e, -b.lse * kLog2e);
  c.l2e2 = pk2(kLog2e * scale, kLog2e * scale);
  c.fac2 = pk2(b.fac, b.fac);
  c.nsn2 = pk2(-b.sn, -b.sn);
  c.k12 = pk2(b.k1, b.k1);
  return c;
}

// The gradients of one 16-byte vector of logits, stored at dst.
template <typename T>
DSLPG_DEV void grad_vec(const Vec16& v, const GradPairs& c, bool smooth, T* dst) {
  constexpr int P = Elt<T>::kPerVec / 2;
  f32x2 y[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    // exp(x * scale - lse) = 2^(x * scale * log2e - lse * log2e)
    float d0, d1;
    upk2(fma2(unpack_pair<T>(v, p), c.l2e2, c.nl2), d0, d1);
    f32x2 e = pk2(ex2(d0), ex2(d1));
    e = fma2(c.fac2, e, e);
    if (smooth) e = add2(e, c.nsn2);
    y[p] = mul2(c.k12, e);
  }
  StorePairs<T, P>::run(dst, y);
}

// The label column of a row, rewritten by the thread that wrote its vector
// (V > 1) or element (V == 1), after that thread's own store.
template <typename T, int V>
DSLPG_DEV void grad_label_fix(const T* xr, T* yr, int64_t N, const GradRow& b, float scale, bool smooth, int t,
                              int tpr) {
  if (b.adj >= 0 && b.adj < N) {
    const int64_t unit = (V > 1) ? b.adj / V : b.adj;
    if (static_cast<int>(unit % tpr) == t) yr[b.adj] = from_f<T>(grad_elem(b, to_f(xr[b.adj]), scale, true, smooth));
  }
}

// Write the N gradients of one row (xr -> yr) with the tpr threads t of a
// group: 16-byte vectors (V > 1, nvec = N / V) or scalars (V == 1), then the
// label column. U: 16-byte loads in flight per thread.
template <typename T, int V, int U = 4>
DSLPG_DEV void grad_row(const T* xr, T* yr, int nvec, int64_t N, const GradRow& b, float scale, bool smooth, int t,
                        int tpr) {
  if constexpr (V > 1) {
    const GradPairs c = grad_pairs(b, scale);
    // the next chunk's loads are issued before this chunk's math and stores
    auto load = [&](Vec16 (&dst)[U], int j0) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        dst[u] = Vec16{{0u, 0u, 0u, 0u}};
        if (j < nvec) dst[u] = ld_stream(xr + static_cast<int64_t>(j) * V);
      }
    };
    Vec16 nx[U];
    load(nx, t);
    for (int j0 = t; j0 < nvec; j0 += U * tpr) {
      Vec16 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = nx[u];
      if (j0 + U * tpr < nvec) load(nx, j0 + U * tpr);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * tpr;
        if (j < nvec) grad_vec<T>(v[u], c, smooth, yr + static_cast<int64_t>(j) * V);
      }
    }
  } else {
    for (int64_t c = t; c < N; c += tpr) yr[c] = from_f<T>(grad_elem(b, to_f(xr[c]), scale, false, smooth));
  }
  grad_label_fix<T, V>(xr, yr, N, b, scale, smooth, t, tpr);
}

}  // namespace dslpg
