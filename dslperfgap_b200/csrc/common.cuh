// common.cuh — shared device helpers for the row-reduction kernels (sm_100a).
//
// Everything here is memory-movement and reduction plumbing: 16-byte vector
// loads and stores with cache hints, fp16/bf16 <-> fp32 unpacking, NaN-
// propagating max, warp and row-group reductions, and the host-side launch
// helpers (SM count, occupancy-sized persistent grids).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/dslpg_b200.h"

#define DSLPG_DEV __device__ __forceinline__

namespace dslpg {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.69314718055994531f;
constexpr float kNegInf = -__builtin_huge_valf();
constexpr float kPosInf = __builtin_huge_valf();

// ----------------------------------------------------------------------------
// Storage types
// ----------------------------------------------------------------------------
struct alignas(16) Vec16 {
  uint32_t w[4];
};

template <typename T> struct Elt;
template <> struct Elt<float> { static constexpr int kPerVec = 4; };
template <> struct Elt<__half> { static constexpr int kPerVec = 8; };
template <> struct Elt<__nv_bfloat16> { static constexpr int kPerVec = 8; };

DSLPG_DEV float to_f(float v) { return v; }
DSLPG_DEV float to_f(__half v) { return __half2float(v); }
DSLPG_DEV float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> DSLPG_DEV T from_f(float v);
template <> DSLPG_DEV float from_f<float>(float v) { return v; }
template <> DSLPG_DEV __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> DSLPG_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round v to T's precision and back (exact when T is fp32).
template <typename T> DSLPG_DEV float round_to(float v) { return to_f(from_f<T>(v)); }

// Scalar load of element i of an array whose dtype is only known at run time.
DSLPG_DEV float load_any(const void* p, int64_t i, int dt) {
  if (dt == DSLPG_F32) return __ldg(static_cast<const float*>(p) + i);
  if (dt == DSLPG_F16) return __half2float(__ldg(static_cast<const __half*>(p) + i));
  return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p) + i));
}

// ----------------------------------------------------------------------------
// Vector memory ops
// ----------------------------------------------------------------------------
// Cache hints of the streaming loads and stores. Measured on B200 (same box,
// interleaved runs): plain stores beat st.global.cs by 2-3 points of HBM
// bandwidth on every read+write kernel; an .L2::256B load prefetch hint
// changed nothing. Both stay selectable at build time for re-measurement.
#ifndef DSLPG_LD_L2_256B
#define DSLPG_LD_L2_256B 0
#endif
#ifndef DSLPG_ST_CS
#define DSLPG_ST_CS 0
#endif
#if DSLPG_LD_L2_256B
#define DSLPG_LD_HINT ".L1::no_allocate.L2::256B"
#else
#define DSLPG_LD_HINT ".L1::no_allocate"
#endif
#if DSLPG_ST_CS
#define DSLPG_ST_HINT ".cs"
#else
#define DSLPG_ST_HINT ""
#endif

// Read-once activations: do not allocate in L1 (the row is read once from HBM).
DSLPG_DEV Vec16 ld_stream(const void* p) {
  Vec16 v;
  asm volatile("ld.global.nc" DSLPG_LD_HINT ".v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
      : "l"(p));
  return v;
}

// Data re-read by many rows (weight / bias vectors): keep in L1.
DSLPG_DEV Vec16 ld_keep(const void* p) {
  Vec16 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
      : "l"(p));
  return v;
}

DSLPG_DEV void st_stream(void* p, const Vec16& v) {
  asm volatile("st.global" DSLPG_ST_HINT ".v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
               "r"(v.w[2]), "r"(v.w[3])
               : "memory");
}

DSLPG_DEV void st_stream8(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global" DSLPG_ST_HINT ".v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

// Unpack one 16-byte vector of T into fp32 (Elt<T>::kPerVec values).
template <typename T> DSLPG_DEV void unpack(const Vec16& v, float* f);
template <> DSLPG_DEV void unpack<float>(const Vec16& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(v.w[i]);
}
template <> DSLPG_DEV void unpack<__nv_bfloat16>(const Vec16& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(v.w[i] << 16);
    f[2 * i + 1] = __uint_as_float(v.w[i] & 0xffff0000u);
  }
}
template <> DSLPG_DEV void unpack<__half>(const Vec16& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&v.w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Pack two fp32 values into one 32-bit word of T (T 16-bit), round to nearest even.
template <typename T> DSLPG_DEV uint32_t pack2(float a, float b);
template <> DSLPG_DEV uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> DSLPG_DEV uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Store E fp32 values as E elements of T at p (p aligned to E * sizeof(T)).
// E is 4 or 8; the store is 8, 16 or 32 bytes.
template <typename T, int E> struct StoreOut;
template <int E> struct StoreOut<float, E> {
  static DSLPG_DEV void run(void* p, const float* f) {
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      Vec16 v;
#pragma unroll
      for (int i = 0; i < 4; ++i) v.w[i] = __float_as_uint(f[4 * q + i]);
      st_stream(static_cast<char*>(p) + 16 * q, v);
    }
  }
};
template <typename T16> struct Store16Bit {
  template <int E> static DSLPG_DEV void run(void* p, const float* f) {
    if constexpr (E == 4) {
      st_stream8(p, pack2<T16>(f[0], f[1]), pack2<T16>(f[2], f[3]));
    } else {
      Vec16 v;
#pragma unroll
      for (int i = 0; i < 4; ++i) v.w[i] = pack2<T16>(f[2 * i], f[2 * i + 1]);
      st_stream(p, v);
    }
  }
};
template <int E> struct StoreOut<__half, E> {
  static DSLPG_DEV void run(void* p, const float* f) { Store16Bit<__half>::run<E>(p, f); }
};
template <int E> struct StoreOut<__nv_bfloat16, E> {
  static DSLPG_DEV void run(void* p, const float* f) { Store16Bit<__nv_bfloat16>::run<E>(p, f); }
};

// ----------------------------------------------------------------------------
// Arithmetic
// ----------------------------------------------------------------------------
// 2^x on the SFU; x = -inf gives 0, NaN stays NaN. Results below 2^-126 flush
// to zero, which only drops terms < 1e-38 relative to the largest one.
DSLPG_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(d) for d = x - max (d <= 0 in normal use).
DSLPG_DEV float exp_shifted(float d) { return ex2(d * kLog2e); }

// max that returns NaN when either operand is NaN (torch's amax semantics).
DSLPG_DEV float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Raw bit pattern of two -inf values of T in one 32-bit word (one for fp32).
template <typename T> struct NegInfWord;
template <> struct NegInfWord<float> { static constexpr uint32_t v = 0xff800000u; };
template <> struct NegInfWord<__half> { static constexpr uint32_t v = 0xfc00fc00u; };
template <> struct NegInfWord<__nv_bfloat16> { static constexpr uint32_t v = 0xff80ff80u; };

// ----------------------------------------------------------------------------
// Packed fp32 pairs (sm_100a fma/add/mul .f32x2: two lanes per instruction)
// ----------------------------------------------------------------------------
typedef unsigned long long f32x2;

DSLPG_DEV f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
DSLPG_DEV void upk2(f32x2 v, float& a, float& b) { asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
DSLPG_DEV f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
DSLPG_DEV f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
DSLPG_DEV f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
DSLPG_DEV float hsum2(f32x2 v) {
  float a, b;
  upk2(v, a, b);
  return a + b;
}

// Elements (2p, 2p+1) of a 16-byte vector of T as an fp32 pair,
// p in [0, Elt<T>::kPerVec / 2).
template <typename T> DSLPG_DEV f32x2 unpack_pair(const Vec16& v, int p);
template <> DSLPG_DEV f32x2 unpack_pair<float>(const Vec16& v, int p) {
  return pk2(__uint_as_float(v.w[2 * p]), __uint_as_float(v.w[2 * p + 1]));
}
template <> DSLPG_DEV f32x2 unpack_pair<__nv_bfloat16>(const Vec16& v, int p) {
  return pk2(__uint_as_float(v.w[p] << 16), __uint_as_float(v.w[p] & 0xffff0000u));
}
template <> DSLPG_DEV f32x2 unpack_pair<__half>(const Vec16& v, int p) {
  float2 t = __half22float2(*reinterpret_cast<const __half2*>(&v.w[p]));
  return pk2(t.x, t.y);
}

// Store the 2P values of P fp32 pairs as 2P elements of T at p (aligned to
// 2P * sizeof(T)), rounding to nearest even.
template <typename T, int P> struct StorePairs;
template <int P> struct StorePairs<float, P> {
  static DSLPG_DEV void run(void* p, const f32x2* y) {
#pragma unroll
    for (int q = 0; q < P / 2; ++q) {
      float a, b, c, d;
      upk2(y[2 * q], a, b);
      upk2(y[2 * q + 1], c, d);
      st_stream(static_cast<char*>(p) + 16 * q,
                Vec16{{__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d)}});
    }
  }
};
template <typename T16, int P> struct StorePairs16 {
  static DSLPG_DEV void run(void* p, const f32x2* y) {
    uint32_t w[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float a, b;
      upk2(y[i], a, b);
      w[i] = pack2<T16>(a, b);
    }
    if constexpr (P == 2) st_stream8(p, w[0], w[1]);
    else st_stream(p, Vec16{{w[0], w[1], w[2], w[3]}});
  }
};
template <int P> struct StorePairs<__half, P> : StorePairs16<__half, P> {};
template <int P> struct StorePairs<__nv_bfloat16, P> : StorePairs16<__nv_bfloat16, P> {};

// Largest (MIN: smallest) element of NV vectors of T, compared on the stored
// values (16-bit values two per instruction, fp32 three-input), as fp32;
// NaN-propagating.
template <typename T, int NV, bool MIN> struct RawExtreme;
template <int NV, bool MIN> struct RawExtreme<float, NV, MIN> {
  static DSLPG_DEV float op3(float a, float b, float c) {
    float r;
    if constexpr (MIN) asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    else asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
  }
  static DSLPG_DEV float run(const Vec16 (&v)[NV]) {
    float f[4 * NV];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) f[4 * k + i] = __uint_as_float(v[k].w[i]);
    // a tree of three-input steps
#pragma unroll
    for (int n = 4 * NV; n > 1; n = (n + 2) / 3) {
#pragma unroll
      for (int i = 0; i < (n + 2) / 3; ++i) {
        const float a = f[3 * i];
        const float b = (3 * i + 1 < n) ? f[3 * i + 1] : a;
        const float c = (3 * i + 2 < n) ? f[3 * i + 2] : a;
        f[i] = op3(a, b, c);
      }
    }
    return f[0];
  }
};
template <typename T16, int NV, bool MIN> struct RawExtreme16 {
  static DSLPG_DEV uint32_t op(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (std::is_same<T16, __nv_bfloat16>::value) {
      if constexpr (MIN) asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
      else asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    } else {
      if constexpr (MIN) asm("min.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
      else asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    }
    return r;
  }
  static DSLPG_DEV float run(const Vec16 (&v)[NV]) {
    uint32_t w[4 * NV];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) w[4 * k + i] = v[k].w[i];
#pragma unroll
    for (int n = 4 * NV; n > 1; n = (n + 1) / 2) {
#pragma unroll
      for (int i = 0; i < n / 2; ++i) w[i] = op(w[2 * i], w[2 * i + 1]);
      if (n & 1) w[n / 2] = w[n - 1];
    }
    const f32x2 pr = unpack_pair<T16>(Vec16{{w[0], 0u, 0u, 0u}}, 0);
    float a, b, r;
    upk2(pr, a, b);
    if constexpr (MIN) asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    else asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
  }
};
template <int NV, bool MIN> struct RawExtreme<__nv_bfloat16, NV, MIN> : RawExtreme16<__nv_bfloat16, NV, MIN> {};
template <int NV, bool MIN> struct RawExtreme<__half, NV, MIN> : RawExtreme16<__half, NV, MIN> {};

// 2^d for both lanes of a pair on the FMA and integer pipes, leaving the SFU
// free (used for a share of the exponentials of the long-row reductions, whose
// throughput is otherwise bounded by the SFU). Method: d = n + f with
// n = round(d) (added to 1.5 * 2^23, whose low mantissa bits then hold n) and
// |f| <= 1/2; 2^f from a degree-4 polynomial whose coefficients were fitted
// for this library by iteratively reweighted least squares on Chebyshev nodes
// (max relative error 2.7e-6 in fp32 over [-1/2, 1/2]); n is added to the
// exponent field. Lanes below -126 are clamped there: their 2^d < 1.2e-38 is
// negligible next to the 1 of the largest term; a NaN lane becomes a finite
// value, which callers tolerate because a NaN already poisons the running
// maximum (see fold_vecs).
DSLPG_DEV f32x2 exp2_poly2(f32x2 d) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  float d0, d1;
  upk2(d, d0, d1);
  const f32x2 dc = pk2(fmaxf(d0, -126.0f), fmaxf(d1, -126.0f));
  const f32x2 t = add2(dc, pk2(kRound, kRound));
  const f32x2 n = add2(t, pk2(-kRound, -kRound));
  const f32x2 f = fma2(n, pk2(-1.0f, -1.0f), dc);
  f32x2 p = fma2(pk2(0.009570095f, 0.009570095f), f, pk2(0.05591786f, 0.05591786f));
  p = fma2(p, f, pk2(0.24024744f, 0.24024744f));
  p = fma2(p, f, pk2(0.69312179f, 0.69312179f));
  p = fma2(p, f, pk2(0.99999928f, 0.99999928f));
  float t0, t1, p0, p1;
  upk2(t, t0, t1);
  upk2(p, p0, p1);
  return pk2(__int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23)),
             __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23)));
}

struct SumOp {
  static DSLPG_DEV float identity() { return 0.f; }
  static DSLPG_DEV float apply(float a, float b) { return a + b; }
};
struct MaxOp {
  static DSLPG_DEV float identity() { return kNegInf; }
  static DSLPG_DEV float apply(float a, float b) { return max_nan(a, b); }
};

// Butterfly reduction: every lane ends with the same bits.
template <class Op> DSLPG_DEV float warp_reduce(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = Op::apply(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Reduction over a row group of `nw` consecutive warps (group g of the CTA).
// `red` is a 32-float shared buffer indexed by the CTA's warp number. All
// threads of the CTA must call this (it contains a __syncthreads when nw > 1).
// Alternate between two buffers for back-to-back reductions: a buffer may be
// rewritten only after the next barrier.
template <class Op>
DSLPG_DEV float group_reduce(float v, float* red, int nw, int first_warp) {
  v = warp_reduce<Op>(v);
  if (nw == 1) return v;
  const int lane = threadIdx.x & 31;
  if (lane == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = lane < nw ? red[first_warp + lane] : Op::identity();
  return warp_reduce<Op>(r);
}

// ----------------------------------------------------------------------------
// Host helpers
// ----------------------------------------------------------------------------
// SM count of the current device (cached per device).
int sm_count();

// Persistent grid: enough CTAs to fill every SM at full occupancy, but no more
// than there is work for. `kernel` is the kernel's host stub.
int persistent_grid(const void* kernel, int block, size_t smem, int64_t work_ctas);

// Allow `kernel` to use `bytes` of dynamic shared memory (cached per device).
cudaError_t allow_dynamic_smem(const void* kernel, size_t bytes);
// Co-resident clusters of `cluster_size` CTAs for launch configuration `cfg`
// (cudaOccupancyMaxActiveClusters), cached per device, kernel, block and shared
// memory under the occupancy cache's lock; `fallback` when the query fails.
int max_active_clusters(const void* kernel, const cudaLaunchConfig_t& cfg, int cluster_size, int fallback);

// Kernel-shape override (DSLPG_PATH_*), set by dslpg_set_kernel_path.
int kernel_path();

// Per-file counters of bounded waits that ran out of time (read and reset).
unsigned int take_wait_timeouts_rownorm();
unsigned int take_wait_timeouts_rowstat();
unsigned int take_wait_timeouts_ff();

inline int dtype_size(int dt) { return dt == DSLPG_F32 ? 4 : 2; }
inline bool is_float_dtype(int dt) { return dt == DSLPG_F32 || dt == DSLPG_F16 || dt == DSLPG_BF16; }
inline bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

}  // namespace dslpg
