// reduce.cu — the sibling row reductions: mean, max with index, argmax
// (sm_100a).
//
// A tensor reduced over one axis (or a run of adjacent axes) is viewed as
// [M, N, K] with N the reduced extent:
//  * reduce_rows_kernel (K == 1): a group of threads per row streams it with
//    16-byte loads, U vectors in flight per thread. mean accumulates fp32
//    pairs; max / argmax take each vector's maximum on the stored values (two
//    16-bit values per instruction), keep the first vector that raises the
//    running maximum in registers, and locate the element once per row.
//  * reduce_cols_kernel (K > 1): one thread per (m, k), reads coalesced across k.
// Index semantics are torch's: the first NaN wins (a NaN is the maximum), and
// among equal maxima the smallest index wins.
#include <type_traits>

#include "common.cuh"

namespace dslpg {

enum RedOp : int { kMean = 0, kMax = 1, kArgmax = 2 };

struct RedArgs {
  const void* x;
  void* val;        // mean / max values (may be null for argmax)
  int64_t* idx;     // max / argmax indices
  int64_t M, N, K;
  int nvec;         // N / elements per vector (row kernel, vector path)
  int tpr, rpc;
  float inv_n;
};

// mean(x, dtype=Tout) converts x to Tout first (a no-op when Tout is fp32).
template <typename Tin, typename Tout>
constexpr bool kRedRound = !std::is_same<Tin, Tout>::value && !std::is_same<Tout, float>::value;

// (value, index) with torch's max order: NaN above everything, ties to the
// smaller index.
struct ArgBest {
  float v;
  int64_t i;
};
DSLPG_DEV bool arg_better(float bv, int64_t bi, float av, int64_t ai) {
  const bool bn = bv != bv, an = av != av;
  if (bn || an) return bn && (!an || bi < ai);
  return bv > av || (bv == av && bi < ai);
}

DSLPG_DEV ArgBest warp_arg_reduce(ArgBest a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, a.v, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, a.i, o);
    if (arg_better(ov, oi, a.v, a.i)) a = ArgBest{ov, oi};
  }
  return a;
}

template <int OP, typename Tin, typename Tout, int V, int MINB = 1>
__global__ void __launch_bounds__(256, MINB) reduce_rows_kernel(const RedArgs a) {
  constexpr int U = (V == 1) ? 8 : 4;
  __shared__ float red_v[32];
  __shared__ int64_t red_i[32];
  const int g = threadIdx.x / a.tpr;
  const int t = threadIdx.x - g * a.tpr;
  const int nw = a.tpr >> 5, first_warp = g * nw, lane = threadIdx.x & 31;
  const int64_t step = static_cast<int64_t>(gridDim.x) * a.rpc;

  // the first chunk of a row's loads (U vectors per thread)
  Vec16 nx[V > 1 ? U : 1];
  auto first_chunk = [&](int64_t row) {
    if constexpr (V > 1) {
      const Tin* xr = static_cast<const Tin*>(a.x) + row * a.N;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = t + static_cast<int64_t>(u) * a.tpr;
        nx[u] = Vec16{{0u, 0u, 0u, 0u}};
        if (row < a.M && j < a.nvec) nx[u] = ld_stream(xr + j * V);
      }
    }
  };
  first_chunk(static_cast<int64_t>(blockIdx.x) * a.rpc + g);
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * a.rpc; base < a.M; base += step) {
    const int64_t row = base + g;
    const bool rv = row < a.M;
    const Tin* xr = static_cast<const Tin*>(a.x) + (rv ? row : 0) * a.N;
    f32x2 sum2 = pk2(0.f, 0.f);
    ArgBest best{kNegInf, INT64_MAX};
    int64_t best_j = -1;  // vector path: the vector holding best.v, and its data
    Vec16 best_vec{{0u, 0u, 0u, 0u}};
    const int64_t units = rv ? ((V > 1) ? a.nvec : a.N) : 0;

    for (int64_t j0 = t; j0 < units; j0 += static_cast<int64_t>(U) * a.tpr) {
      if constexpr (V > 1) {
        constexpr int P = V / 2;
        Vec16 v[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          ok[u] = j0 + static_cast<int64_t>(u) * a.tpr < units;
          v[u] = nx[u];
        }
        // prefetch the next chunk before working on this one
        const int64_t jn = j0 + static_cast<int64_t>(U) * a.tpr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = jn + static_cast<int64_t>(u) * a.tpr;
          nx[u] = Vec16{{0u, 0u, 0u, 0u}};
          if (j < units) nx[u] = ld_stream(xr + j * V);
        }
        if constexpr (OP == kMean) {
#pragma unroll
          for (int u = 0; u < U; ++u)
#pragma unroll
            for (int p = 0; p < P; ++p) {
              f32x2 x = unpack_pair<Tin>(v[u], p);
              if constexpr (kRedRound<Tin, Tout>) {
                float x0, x1;
                upk2(x, x0, x1);
                x = pk2(round_to<Tout>(x0), round_to<Tout>(x1));
              }
              sum2 = add2(sum2, x);  // masked vectors are zeros
            }
        } else {
          // per vector: its maximum on the stored values; keep the first
          // vector holding a new running maximum (and its raw data)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            if (!ok[u]) continue;
            const Vec16 one[1] = {v[u]};
            const float m = RawExtreme<Tin, 1, false>::run(one);
            const bool mn = m != m, bn = best.v != best.v;
            if (mn ? !bn : (!bn && m > best.v)) {
              best.v = m;
              best_j = j0 + static_cast<int64_t>(u) * a.tpr;
              best_vec = v[u];
            }
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
          if (j >= units) continue;
          float f = to_f(xr[j]);
          if constexpr (kRedRound<Tin, Tout>) f = round_to<Tout>(f);
          if constexpr (OP == kMean) {
            sum2 = add2(sum2, pk2(f, 0.f));
          } else {
            if (arg_better(f, j, best.v, best.i)) best = ArgBest{f, j};
          }
        }
      }
    }

    // The next row's first loads fly during this row's merge (max / argmax:
    // 0.830 -> 0.845 of measured HBM; it costs max / argmax a 4-byte spill).
    first_chunk(row + step);
    if constexpr (OP != kMean && V > 1) {
      if (best_j >= 0) {  // first position of the maximum (or first NaN) in its vector
        float f[V];
        unpack<Tin>(best_vec, f);
        bool found = false;
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const bool hit = (best.v != best.v) ? (f[i] != f[i]) : (f[i] == best.v);
          if (!found && hit) {
            found = true;
            best.i = best_j * V + i;
          }
        }
      }
    }

    // merge over the row group
    if constexpr (OP == kMean) {
      float s = group_reduce<SumOp>(hsum2(sum2), red_v, nw, first_warp);
      if (t == 0 && rv) static_cast<Tout*>(a.val)[row] = from_f<Tout>(s * a.inv_n);
      __syncthreads();
    } else {
      best = warp_arg_reduce(best);
      if (nw > 1) {
        if (lane == 0) {
          red_v[threadIdx.x >> 5] = best.v;
          red_i[threadIdx.x >> 5] = best.i;
        }
        __syncthreads();
        ArgBest b{kNegInf, INT64_MAX};
        if (lane < nw) b = ArgBest{red_v[first_warp + lane], red_i[first_warp + lane]};
        best = warp_arg_reduce(b);
      }
      if (t == 0 && rv) {
        if constexpr (OP == kMax) static_cast<Tin*>(a.val)[row] = from_f<Tin>(best.v);
        a.idx[row] = best.i == INT64_MAX ? 0 : best.i;
      }
      __syncthreads();
    }
  }
}

template <int OP, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) reduce_cols_kernel(const RedArgs a) {
  const int64_t cols = a.M * a.K;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t mi = c / a.K, k = c - mi * a.K;
    const Tin* xc = static_cast<const Tin*>(a.x) + mi * a.N * a.K + k;
    if constexpr (OP == kMean) {
      float s = 0.f;
      for (int64_t n = 0; n < a.N; ++n) {
        float f = to_f(xc[n * a.K]);
        if constexpr (kRedRound<Tin, Tout>) f = round_to<Tout>(f);
        s += f;
      }
      static_cast<Tout*>(a.val)[c] = from_f<Tout>(s * a.inv_n);
    } else {
      ArgBest best{kNegInf, INT64_MAX};
      for (int64_t n = 0; n < a.N; ++n) {
        const float f = to_f(xc[n * a.K]);
        if (arg_better(f, n, best.v, best.i)) best = ArgBest{f, n};
      }
      if constexpr (OP == kMax) static_cast<Tin*>(a.val)[c] = from_f<Tin>(best.v);
      a.idx[c] = best.i == INT64_MAX ? 0 : best.i;
    }
  }
}

namespace {

inline int round_up32(int v) { return (v + 31) & ~31; }

template <int OP, typename Tin, typename Tout, int V, int MINB = 1>
cudaError_t launch_rows(RedArgs a, cudaStream_t st) {
  const int64_t units = (V > 1) ? a.nvec : a.N;
  // Vectors per thread per row: max / argmax pay a fixed per-row cost (the
  // 64-bit index merge and the re-read of the winning chunk), so they take
  // longer slices.
#ifndef DSLPG_RED_PER_THREAD_MAX
#define DSLPG_RED_PER_THREAD_MAX 64
#endif
  const int64_t per_thread = (V > 1) ? (OP == kMean ? 16 : DSLPG_RED_PER_THREAD_MAX) : 64;
  int64_t want = (units + per_thread - 1) / per_thread;
  int tpr = static_cast<int>(want > 256 ? 256 : want);
  tpr = round_up32(tpr < 32 ? 32 : tpr);
  a.tpr = tpr;
  a.rpc = tpr >= 256 ? 1 : 256 / tpr;
  const int block = a.tpr * a.rpc;
  const void* fn = reinterpret_cast<const void*>(&reduce_rows_kernel<OP, Tin, Tout, V, MINB>);
#ifdef DSLPG_RED_NONPERSISTENT
  const int grid = static_cast<int>((a.M + a.rpc - 1) / a.rpc);
#else
  const int grid = persistent_grid(fn, block, 0, (a.M + a.rpc - 1) / a.rpc);
#endif
  reduce_rows_kernel<OP, Tin, Tout, V, MINB><<<grid, block, 0, st>>>(a);
  return cudaGetLastError();
}

template <int OP, typename Tin, typename Tout>
cudaError_t launch_red(RedArgs a, cudaStream_t st) {
  constexpr int E = Elt<Tin>::kPerVec;
  if (a.K > 1) {
    const void* fn = reinterpret_cast<const void*>(&reduce_cols_kernel<OP, Tin, Tout>);
    const int grid = persistent_grid(fn, 256, 0, (a.M * a.K + 255) / 256);
    reduce_cols_kernel<OP, Tin, Tout><<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
  }
  if (aligned(a.x, 16) && a.N % E == 0 && a.N / E <= 0x7fffffff) {
    a.nvec = static_cast<int>(a.N / E);
    // max / argmax: registers bounded to four CTAs per SM (measured faster)
#ifndef DSLPG_RED_MINB_MAX
#define DSLPG_RED_MINB_MAX 4
#endif
    if constexpr (OP != kMean) return launch_rows<OP, Tin, Tout, E, DSLPG_RED_MINB_MAX>(a, st);
    return launch_rows<OP, Tin, Tout, E>(a, st);
  }
  return launch_rows<OP, Tin, Tout, 1>(a, st);
}

template <int OP, typename Tin>
cudaError_t red_out(RedArgs a, int out_dt, cudaStream_t st) {
  if constexpr (OP != kMean) {
    return launch_red<OP, Tin, Tin>(a, st);
  } else {
    switch (out_dt) {
      case DSLPG_F32: return launch_red<OP, Tin, float>(a, st);
      case DSLPG_F16: return launch_red<OP, Tin, __half>(a, st);
      default: return launch_red<OP, Tin, __nv_bfloat16>(a, st);
    }
  }
}

template <int OP>
cudaError_t red_in(RedArgs a, int in_dt, int out_dt, cudaStream_t st) {
  switch (in_dt) {
    case DSLPG_F32: return red_out<OP, float>(a, out_dt, st);
    case DSLPG_F16: return red_out<OP, __half>(a, out_dt, st);
    default: return red_out<OP, __nv_bfloat16>(a, out_dt, st);
  }
}

int check_red(const void* x, int64_t M, int64_t N, int64_t K, int in_dt) {
  if (x == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0 || K < 1) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(in_dt)) return DSLPG_ERR_BAD_DTYPE;
  return DSLPG_OK;
}

RedArgs make_red(const void* x, void* val, int64_t* idx, int64_t M, int64_t N, int64_t K) {
  RedArgs a{};
  a.x = x;
  a.val = val;
  a.idx = idx;
  a.M = M;
  a.N = N;
  a.K = K;
  a.inv_n = N > 0 ? 1.0f / static_cast<float>(N) : 0.f;
  return a;
}

}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_mean_reduction(const void* x, void* y, int64_t M, int64_t N, int64_t K, int in_dtype,
                                    int out_dtype, cudaStream_t stream) {
  if (int rc = check_red(x, M, N, K, in_dtype)) return rc;
  if (y == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (!is_float_dtype(out_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (M == 0) return DSLPG_OK;
  if (N == 0) return DSLPG_ERR_BAD_SHAPE;  // the mean of nothing is NaN; callers handle it
  return static_cast<int>(red_in<kMean>(make_red(x, y, nullptr, M, N, K), in_dtype, out_dtype, stream));
}

extern "C" int dslpg_max_reduction(const void* x, void* values, int64_t* indices, int64_t M, int64_t N,
                                   int64_t K, int dtype, cudaStream_t stream) {
  if (int rc = check_red(x, M, N, K, dtype)) return rc;
  if (values == nullptr || indices == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M == 0) return DSLPG_OK;
  if (N == 0) return DSLPG_ERR_BAD_SHAPE;  // torch raises for an empty reduced dim
  return static_cast<int>(red_in<kMax>(make_red(x, values, indices, M, N, K), dtype, dtype, stream));
}

extern "C" int dslpg_argmax(const void* x, int64_t* indices, int64_t M, int64_t N, int64_t K, int dtype,
                            cudaStream_t stream) {
  if (int rc = check_red(x, M, N, K, dtype)) return rc;
  if (indices == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M == 0) return DSLPG_OK;
  if (N == 0) return DSLPG_ERR_BAD_SHAPE;
  return static_cast<int>(red_in<kArgmax>(make_red(x, nullptr, indices, M, N, K), dtype, dtype, stream));
}
