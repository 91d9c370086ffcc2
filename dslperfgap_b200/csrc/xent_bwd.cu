// xent_bwd.cu — blockwise cross-entropy backward (sm_100a).
//
// dlogits[r, c] = (dloss[r] * scale) * p, where
//   p = exp(logits[r, c] * scale - lse[r]);  p += 2 * lse_sq * lse[r] * p;
//   p -= (1 - smoothing) (or 1 without smoothing) at the label's column;
//   p -= smoothing / total_classes (with smoothing);
// and rows whose label is ignored_index have dloss = 0. This is the
// arithmetic of ViperBench/cross_entropy/triton_impl.py:79-120 and
// pytorch_impl.py:93-141. Column blocks only tile the computation there, so
// the result does not depend on BLOCK_SIZE.
//
// There is no reduction: each row is streamed once (read logits, write
// dlogits) by one CTA with 16-byte vectors; the label column is rewritten
// after the row by the thread that owns its vector, in program order after
// its own vector store.
#include "common.cuh"

namespace dslpg {

struct BwdArgs {
  const void* dloss;
  int dloss_dt;
  int64_t dloss_stride;
  const void* x;
  const float* lse;
  const void* labels;
  int label64;
  void* dx;
  int64_t M, N, ld, ldo;
  int nvec;
  float smoothing, scale, lse_sq, total_classes;
  int64_t ignored, class_start;
  int has_smoothing;
};

// Per-row constants.
struct BwdRow {
  float k1;      // dloss * scale
  float lse;
  float fac;     // 2 * lse_sq * lse
  float sn;      // smoothing / total_classes (0 without smoothing)
  float lab;     // subtracted at the label column
  int64_t adj;   // label column (label - class_start)
};

DSLPG_DEV BwdRow bwd_row(const BwdArgs& a, int64_t r) {
  BwdRow b;
  const int64_t label = a.label64 ? static_cast<const int64_t*>(a.labels)[r]
                                  : static_cast<int64_t>(static_cast<const int32_t*>(a.labels)[r]);
  const float dl = (label != a.ignored) ? load_any(a.dloss, r * a.dloss_stride, a.dloss_dt) : 0.f;
  b.k1 = dl * a.scale;
  b.lse = a.lse[r];
  b.fac = 2.0f * a.lse_sq * b.lse;
  b.sn = a.has_smoothing ? a.smoothing / a.total_classes : 0.f;
  b.lab = a.has_smoothing ? (1.0f - a.smoothing) : 1.0f;
  b.adj = label - a.class_start;
  return b;
}

// The gradient of one element, exactly in the reference's order of operations.
DSLPG_DEV float bwd_elem(const BwdRow& b, float x, float scale, bool is_label, bool smooth) {
  float p = exp_shifted(x * scale - b.lse);
  p = p + b.fac * p;
  if (is_label) p = p - b.lab;
  if (smooth) p = p - b.sn;
  return b.k1 * p;
}

template <typename T, int V>
__global__ void __launch_bounds__(256) xent_bwd_kernel(const BwdArgs a) {
  constexpr int U = 4;
  const int t = threadIdx.x, tpr = blockDim.x;
  const bool smooth = a.has_smoothing != 0;
  for (int64_t r = blockIdx.x; r < a.M; r += gridDim.x) {
    const BwdRow b = bwd_row(a, r);
    const T* xr = static_cast<const T*>(a.x) + r * a.ld;
    T* yr = static_cast<T*>(a.dx) + r * a.ldo;
    if constexpr (V > 1) {
      constexpr int P = V / 2;
      const f32x2 sc2 = pk2(a.scale, a.scale), nl2 = pk2(-b.lse * kLog2e, -b.lse * kLog2e);
      const f32x2 l2e2 = pk2(kLog2e * a.scale, kLog2e * a.scale);
      const f32x2 fac2 = pk2(b.fac, b.fac), nsn2 = pk2(-b.sn, -b.sn), k12 = pk2(b.k1, b.k1);
      (void)sc2;
      for (int j0 = t; j0 < a.nvec; j0 += U * tpr) {
        Vec16 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int j = j0 + u * tpr;
          v[u] = Vec16{{0u, 0u, 0u, 0u}};
          if (j < a.nvec) v[u] = ld_stream(xr + static_cast<int64_t>(j) * V);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int j = j0 + u * tpr;
          if (j >= a.nvec) continue;
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
      for (int64_t c = t; c < a.N; c += tpr) {
        yr[c] = from_f<T>(bwd_elem(b, to_f(xr[c]), a.scale, false, smooth));
      }
    }
    // The label column: rewritten by the thread that wrote its vector.
    if (b.adj >= 0 && b.adj < a.N) {
      const int64_t unit = (V > 1) ? b.adj / V : b.adj;
      if (static_cast<int>(unit % tpr) == t) {
        yr[b.adj] = from_f<T>(bwd_elem(b, to_f(xr[b.adj]), a.scale, true, smooth));
      }
    }
  }
}

namespace {
template <typename T>
cudaError_t launch_bwd(BwdArgs a, cudaStream_t st) {
  constexpr int E = Elt<T>::kPerVec;
  const bool vec = aligned(a.x, 16) && aligned(a.dx, 16) && (a.N % E == 0) && (a.ld % E == 0) &&
                   (a.ldo % E == 0) && a.N / E <= 0x7fffffff;
  const int block = 256;
  if (vec) {
    a.nvec = static_cast<int>(a.N / E);
    const void* fn = reinterpret_cast<const void*>(&xent_bwd_kernel<T, E>);
    const int grid = persistent_grid(fn, block, 0, a.M);
    xent_bwd_kernel<T, E><<<grid, block, 0, st>>>(a);
  } else {
    a.nvec = 0;
    const void* fn = reinterpret_cast<const void*>(&xent_bwd_kernel<T, 1>);
    const int grid = persistent_grid(fn, block, 0, a.M);
    xent_bwd_kernel<T, 1><<<grid, block, 0, st>>>(a);
  }
  return cudaGetLastError();
}
}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_cross_entropy_bwd(const void* dloss, int dloss_dtype, int64_t dloss_stride,
                                       const void* logits, const float* lse, const void* labels,
                                       void* dlogits, int64_t n_rows, int64_t n_cols,
                                       int64_t logits_row_stride, int64_t dlogits_row_stride,
                                       int logits_dtype, int labels_dtype, float smoothing,
                                       float logit_scale, float lse_square_scale,
                                       int64_t ignored_index, float total_classes,
                                       int64_t class_start_idx, int has_smoothing,
                                       cudaStream_t stream) {
  if (!dloss || !logits || !lse || !labels || !dlogits) return DSLPG_ERR_NULL_POINTER;
  if (n_rows < 0 || n_cols < 0 || logits_row_stride < n_cols || dlogits_row_stride < n_cols ||
      dloss_stride < 0)
    return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(logits_dtype) || !is_float_dtype(dloss_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (labels_dtype != DSLPG_I32 && labels_dtype != DSLPG_I64) return DSLPG_ERR_BAD_DTYPE;
  if (n_rows == 0 || n_cols == 0) return DSLPG_OK;
  BwdArgs a{};
  a.dloss = dloss;
  a.dloss_dt = dloss_dtype;
  a.dloss_stride = dloss_stride;
  a.x = logits;
  a.lse = lse;
  a.labels = labels;
  a.label64 = labels_dtype == DSLPG_I64 ? 1 : 0;
  a.dx = dlogits;
  a.M = n_rows;
  a.N = n_cols;
  a.ld = logits_row_stride;
  a.ldo = dlogits_row_stride;
  a.smoothing = smoothing;
  a.scale = logit_scale;
  a.lse_sq = lse_square_scale;
  a.total_classes = total_classes;
  a.ignored = ignored_index;
  a.class_start = class_start_idx;
  a.has_smoothing = has_smoothing ? 1 : 0;
  cudaError_t e;
  switch (logits_dtype) {
    case DSLPG_F32: e = launch_bwd<float>(a, stream); break;
    case DSLPG_F16: e = launch_bwd<__half>(a, stream); break;
    default: e = launch_bwd<__nv_bfloat16>(a, stream); break;
  }
  return static_cast<int>(e);
}
