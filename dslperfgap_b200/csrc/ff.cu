// ff.cu — Llama feed-forward with the RMSNorm fused around a tcgen05 dual
// GEMM (sm_100a): ViperBench linear_activation.kernel_ff.
//
//   a_norm[m] = rsqrt(sum_k x[m,k]^2 / K + 1e-6)             (fp32)
//   xs[m,k]   = x[m,k] * rms_w[k]                              (rounded to fp16)
//   acc1 = xs @ w1^T, acc3 = xs @ w3^T                         (fp16 in, fp32 acc)
//   out  = silu(a_norm * acc1) * (a_norm * acc3)               (stored as fp16)
// (ViperBench/linear_activation/pytorch_impl.py:5-54.)
//
// Two kernels:
//  * ff_prologue_kernel: one pass over x per row (a warp per row): a_norm and xs.
//  * ff_gemm2_kernel (M > 128): CTA pairs on 256x128 tiles with
//    tcgen05.mma.cta_group::2 — described where it is defined;
//  * ff_gemv_kernel (M <= 3 by default): one warp per output column streaming
//    the weight rows, for decode-like shapes — described where it is defined;
//  * ff_gemm_kernel (M <= 128): persistent, one CTA per SM walking 128x128 output tiles,
//    warp-specialised:
//      warp 0 (one lane)  TMA tensor loads of xs / w1 / w3 tiles (BK = 64,
//                         128-byte swizzle) into a 4-stage shared-memory ring;
//      warp 1             allocates all 512 TMEM columns: two buffers of
//                         (acc1 | acc3); one lane issues tcgen05.mma (M=128,
//                         N=128, K=16, fp16 -> fp32), tcgen05.commit releases
//                         each stage and hands a finished buffer to the epilogue;
//      warps 2-5          the epilogue: tcgen05.ld of both accumulators, the
//                         a_norm scale, the SiLU gate, fp16 stores — while the
//                         MMAs of the next tile run into the other buffer.
// No TMA multicast; no peer memory. Every mbarrier wait is bounded (1 s of
// %globaltimer); a wait that runs out records a device counter, the kernel
// finishes its control flow without further waits or stores, the producer
// drains its copies and the TMEM columns are freed before the CTA exits.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "pipe.cuh"

namespace dslpg {

static __device__ unsigned int g_ff_timeouts;

constexpr int kBM = 128, kBN = 128, kBK = 64, kStages = 4;
constexpr uint32_t kTileA = kBM * kBK * 2;  // 16 KiB
constexpr uint32_t kTileB = kBN * kBK * 2;  // 16 KiB
constexpr uint32_t kStageBytes = kTileA + 2 * kTileB;
constexpr uint32_t kTmemCols = 512;  // two buffers of (acc1 | acc3), 128 columns each
constexpr uint32_t kFfThreads = 192;
constexpr size_t kFfSmem = 1024 + kStages * kStageBytes + 1024;  // alignment + ring + barriers

// ---------------------------------------------------------------- prologue
// One warp per row (8 rows per CTA of 256 threads, rows strided over a
// persistent grid), 16-byte vectors with 4 in flight per lane; K % 8 == 0.
__global__ void __launch_bounds__(256) ff_prologue_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                          __half* __restrict__ xs, float* __restrict__ a_norm,
                                                          int64_t M, int K) {
  constexpr int U = 4;
  const int nvec = K / 8, lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t m = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); m < M; m += warps) {
    const __half* xr = x + m * K;
    __half* yr = xs + m * K;
    float ss = 0.f;
    for (int j0 = lane; j0 < nvec; j0 += 32 * U) {
      Vec16 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (j0 + 32 * u < nvec) v[u] = ld_stream(xr + static_cast<int64_t>(j0 + 32 * u) * 8);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + 32 * u;
        if (j >= nvec) break;
        const Vec16 wv = ld_keep(w + static_cast<int64_t>(j) * 8);
        Vec16 o;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 a = *reinterpret_cast<const __half2*>(&v[u].w[i]);
          const __half2 b = *reinterpret_cast<const __half2*>(&wv.w[i]);
          const float2 af = __half22float2(a);
          ss = fmaf(af.x, af.x, ss);
          ss = fmaf(af.y, af.y, ss);
          const __half2 p = __hmul2(a, b);  // x * rms_w in fp16, as the reference
          o.w[i] = *reinterpret_cast<const uint32_t*>(&p);
        }
        st_stream(yr + static_cast<int64_t>(j) * 8, o);
      }
    }
    ss = warp_reduce<SumOp>(ss);
    if (lane == 0) a_norm[m] = rsqrtf(ss / static_cast<float>(K) + 1e-6f);
  }
}

// ------------------------------------------------------------------ tcgen05
// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle
// (rows of 64 fp16 = 128 bytes; 8-row atoms 1024 bytes apart): start address,
// stride byte offset 1024, descriptor version 1, layout SWIZZLE_128B.
DSLPG_DEV uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;            // version
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, M = 128, N = 128 (one of w1 / w3) or 256 (w1 and w3 stacked).
template <int N>
constexpr uint32_t idesc_m128() {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}

template <int N>
DSLPG_DEV void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc_m128<N>()), "r"(accumulate));
}

DSLPG_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

DSLPG_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

#define DSLPG_R32(r) \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
  "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),        \
  "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),       \
  "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one row per lane).
DSLPG_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%"
      "20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : DSLPG_R32(r)
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

DSLPG_DEV float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// out = silu(a_norm * acc1) * (a_norm * acc3) for 32 columns of one row, in
// f32x2 pairs: sigmoid(g) = 1 / (1 + 2^(-g log2 e)) with the SFU's ex2 and
// reciprocal (a few fp32 ulps, far below the fp16 output's rounding), then
// rounded to fp16 pairs.
DSLPG_DEV void gate_pack(const uint32_t (&r1)[32], const uint32_t (&r3)[32], float an, uint32_t (&packed)[16]) {
  const f32x2 an2 = pk2(an, an), nl2 = pk2(-kLog2e, -kLog2e), one2 = pk2(1.0f, 1.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const f32x2 g = mul2(pk2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1])), an2);
    const f32x2 u = mul2(pk2(__uint_as_float(r3[2 * i]), __uint_as_float(r3[2 * i + 1])), an2);
    float t0, t1;
    upk2(mul2(g, nl2), t0, t1);
    float d0, d1;
    upk2(add2(pk2(ex2(t0), ex2(t1)), one2), d0, d1);
    float v0, v1;
    upk2(mul2(mul2(g, pk2(rcp_approx(d0), rcp_approx(d1))), u), v0, v1);
    packed[i] = pack2<__half>(v0, v1);
  }
}

struct FfArgs {
  const float* a_norm;
  __half* out;
  int64_t M, N;
  int K;
};

// Tile order of the persistent grid: groups of up to kGroupM row tiles; inside
// a group the row tile varies fastest, so the CTAs running at one time share a
// few weight tiles (read from DRAM once) and the group's xs rows stay in L2.
#ifndef DSLPG_FF_GROUP_M
#define DSLPG_FF_GROUP_M 16
#endif
constexpr int kGroupM = DSLPG_FF_GROUP_M;

DSLPG_DEV void tile_coords(int t, int mt, int nt, int& tm, int& tn) {
  const int per_group = kGroupM * nt;
  const int g = t / per_group, r = t - g * per_group;
  const int gm = min(kGroupM, mt - g * kGroupM);
  tm = g * kGroupM + r % gm;
  tn = r / gm;
}

__global__ void __launch_bounds__(kFfThreads, 1)
    ff_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b1,
                   const __grid_constant__ CUtensorMap map_b3, const FfArgs a) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t ring = (raw + 1023u) & ~1023u;  // 1024-aligned for the 128-byte swizzle atoms
  const uint32_t bars = ring + kStages * kStageBytes;
  // full[s], empty[s]: the stage ring; tfull[b], tempty[b]: the two TMEM
  // accumulator buffers; done: every MMA issued has completed.
  const uint32_t full0 = bars, empty0 = bars + 8u * kStages;
  const uint32_t tfull0 = bars + 16u * kStages, tempty0 = tfull0 + 16u, done_bar = tfull0 + 32u;
  const int mt = static_cast<int>((a.M + kBM - 1) / kBM), nt = static_cast<int>((a.N + kBN - 1) / kBN);
  const int tiles = mt * nt;
  const int kblocks = (a.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 4);  // one arrival per epilogue warp
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {  // TMEM: two buffers of (acc1 | acc3)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t it = 0;  // stage uses issued so far
      for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, mt, nt, tm, tn);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (abort_flag) break;
          if (it >= kStages && !mbar_wait(empty0 + 8u * s, ph ^ 1u, kWaitLimitNs)) {
            atomicAdd(&g_ff_timeouts, 1u);
            abort_flag = 1;
            break;
          }
          const uint32_t st = ring + s * kStageBytes;
          mbar_arrive_expect_tx(full0 + 8u * s, kStageBytes);
          tma_load_2d(st, &map_a, kb * kBK, tm * kBM, full0 + 8u * s);
          tma_load_2d(st + kTileA, &map_b1, kb * kBK, tn * kBN, full0 + 8u * s);
          tma_load_2d(st + kTileA + kTileB, &map_b3, kb * kBK, tn * kBN, full0 + 8u * s);
        }
      }
      // drain: no copy may still be landing when the CTA exits
      for (uint32_t u = (it > kStages ? it - kStages : 0); u < it; ++u)
        if (!mbar_wait(full0 + 8u * (u % kStages), (u / kStages) & 1u, kWaitLimitNs)) atomicAdd(&g_ff_timeouts, 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      uint32_t it = 0, j = 0;
      for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x, ++j) {
        const uint32_t b = j & 1u;
        if (j >= 2 && !mbar_wait(tempty0 + 8u * b, ((j >> 1) & 1u) ^ 1u, kWaitLimitNs)) {
          atomicAdd(&g_ff_timeouts, 1u);
          abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_base = tmem + b * 2u * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (abort_flag) break;
          if (!mbar_wait(full0 + 8u * s, (it / kStages) & 1u, kWaitLimitNs)) {
            atomicAdd(&g_ff_timeouts, 1u);
            abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = ring + s * kStageBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {  // K = 16 per MMA: 32 bytes into the swizzled rows
            const uint64_t ad = smem_desc_sw128(st + 32u * k);
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#ifdef DSLPG_FF1_TWO_MMAS
            const uint64_t b1 = smem_desc_sw128(st + kTileA + 32u * k);
            const uint64_t b3 = smem_desc_sw128(st + kTileA + kTileB + 32u * k);
            umma_f16<kBN>(acc_base, ad, b1, acc);
            umma_f16<kBN>(acc_base + kBN, ad, b3, acc);
#else
            // the w1 tile and the w3 tile lie back to back (128 rows each, 1024-byte
            // row groups), one 256-row operand: TMEM columns 0-127 get acc1, 128-255 acc3
            umma_f16<2 * kBN>(acc_base, ad, smem_desc_sw128(st + kTileA + 32u * k), acc);
#endif
          }
          umma_commit(empty0 + 8u * s);  // the stage is free once these MMAs have read it
        }
        umma_commit(tfull0 + 8u * b);  // the tile's accumulators are complete
      }
      umma_commit(done_bar);  // every MMA issued so far has completed
      if (!mbar_wait(done_bar, 0u, kWaitLimitNs)) atomicAdd(&g_ff_timeouts, 1u);
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
    uint32_t j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      if (abort_flag) break;
      const uint32_t b = j & 1u;
      if (!mbar_wait(tfull0 + 8u * b, (j >> 1) & 1u, kWaitLimitNs)) {
        atomicAdd(&g_ff_timeouts, 1u);
        abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int tm, tn;
      tile_coords(t, mt, nt, tm, tn);
      const int64_t m = static_cast<int64_t>(tm) * kBM + 32 * q + lane;
      const int64_t n0 = static_cast<int64_t>(tn) * kBN;
      const bool row_ok = m < a.M;
      const float an = row_ok ? a.a_norm[m] : 0.f;
      const uint32_t lane_addr = tmem + b * 2u * kBN + (static_cast<uint32_t>(32 * q) << 16);
      __half* orow = a.out + m * a.N;
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r1[32], r3[32];
        tmem_ld32(lane_addr + 32u * c, r1);
        tmem_ld32(lane_addr + kBN + 32u * c, r3);
        if (c == kBN / 32 - 1) {  // both accumulators read: hand the buffer back to the MMA warp
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty0 + 8u * b);
        }
        if (!row_ok) continue;
        const int64_t nb = n0 + 32 * c;
        uint32_t packed[16];
        gate_pack(r1, r3, an, packed);
        if (nb + 32 <= a.N && (a.N % 8) == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            st_stream(orow + nb + 8 * i, Vec16{{packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]}});
        } else {
          for (int i = 0; i < 32; ++i) {
            if (nb + i >= a.N) break;
            const uint32_t w = packed[i >> 1];
            orow[nb + i] = __ushort_as_half(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xffffu)));
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------- two-SM (CTA pair)
// ff_gemm2_kernel: the same computation with 256x128 output tiles per CTA pair
// (a cluster of 2 on neighbouring SMs) and ONE tcgen05.mma.cta_group::2 of
// M = 256, N = 256 per K step, whose B operand is the w1 tile (128 rows, from
// CTA 0's shared memory) stacked on the w3 tile (128 rows, from CTA 1's): the
// accumulator's columns 0-127 are acc1 and 128-255 acc3. CTA r loads rows
// [128r, 128r+128) of the xs tile and the w1 (r = 0) or w3 (r = 1) tile, so
// each SM brings in 32 KiB per K-block of 64 (48 KiB with one CTA per tile)
// and reads 64 bytes of operands per tensor cycle (A no longer read twice);
// 6 stages fit in shared memory. Each CTA's TMEM holds its 128 rows of
// acc1 | acc3 (two buffers, 512 columns).
// Barriers: CTA 0's full[s] counts both CTAs' bytes (CTA 1's copies signal
// it); empty[s] and tfull[b] are signalled in both CTAs by a multicast
// tcgen05.commit; CTA 0's tempty[b] takes one arrival per epilogue warp of
// both CTAs. TMA loads have no multicast.
#ifndef DSLPG_FF_STAGES
#define DSLPG_FF_STAGES 6
#endif
constexpr int kStages2 = DSLPG_FF_STAGES;
constexpr uint32_t kStage2Bytes = kTileA + kTileB;  // xs half-tile + this CTA's w1 or w3 tile
constexpr size_t kFfSmem2 = 1024 + kStages2 * kStage2Bytes + 1024;
// M = 256 (across the pair), N = 256 (w1 | w3), fp16 inputs, fp32 accumulator, K-major A and B.
constexpr uint32_t kIdesc2 =
    (1u << 4) | (static_cast<uint32_t>((2 * kBN) >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);

DSLPG_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

DSLPG_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of the same variable in CTA `rank` of the cluster.
DSLPG_DEV uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

DSLPG_DEV void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// mbar_wait with cluster-scope acquire, for barriers the peer CTA signals.
DSLPG_DEV bool mbar_wait_cl(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
  for (int n = 0;; ++n) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((n & 63) == 63 && global_ns() - t0 > limit_ns) return false;
  }
}

DSLPG_DEV void umma2_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc2), "r"(accumulate));
}

// Arrive on barrier `bar` (same offset) in both CTAs of the pair once every
// MMA issued so far by this thread has completed.
DSLPG_DEV void umma2_commit_both(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// Tensor load into this CTA's shared memory that signals `cluster_bar`, which
// may be in either CTA of the pair.
DSLPG_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kFfThreads, 1)
    ff_gemm2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b1,
                    const __grid_constant__ CUtensorMap map_b3, const FfArgs a) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t ring = (raw + 1023u) & ~1023u;  // same offset in both CTAs: the MMA reads both at it
  const uint32_t bars = ring + kStages2 * kStage2Bytes;
  const uint32_t full0 = bars, empty0 = bars + 8u * kStages2;
  const uint32_t tfull0 = bars + 16u * kStages2, tempty0 = tfull0 + 16u, done_bar = tfull0 + 32u;
  const int mt = static_cast<int>((a.M + 2 * kBM - 1) / (2 * kBM)), nt = static_cast<int>((a.N + kBN - 1) / kBN);
  const int tiles = mt * nt;
  const int kblocks = (a.K + kBK - 1) / kBK;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {  // one warp of each CTA allocates for the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ---------------------------------------------------------- producers
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = pair; t < tiles && !abort_flag; t += pairs) {
        int tm, tn;
        tile_coords(t, mt, nt, tm, tn);
        const int arow = tm * 2 * kBM + static_cast<int>(rank) * kBM;
        const CUtensorMap* map_b = rank == 0 ? &map_b1 : &map_b3;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kStages2, ph = (it / kStages2) & 1u;
          if (abort_flag) break;
          if (it >= kStages2 && !mbar_wait_cl(empty0 + 8u * s, ph ^ 1u, kWaitLimitNs)) {
            atomicAdd(&g_ff_timeouts, 1u);
            abort_flag = 1;
            break;
          }
          const uint32_t st = ring + s * kStage2Bytes;
          const uint32_t fb = map_to_rank(full0 + 8u * s, 0);
#ifdef DSLPG_FF_DIAG_NO_LOAD  // diagnostic builds only: after the first fill, MMAs re-read stale tiles
          if (it >= kStages2) {
            if (rank == 0) mbar_arrive(full0 + 8u * s);
            continue;
          }
#endif
          if (rank == 0) mbar_arrive_expect_tx(full0 + 8u * s, 2 * kStage2Bytes);
          tma_load_2d_pair(st, &map_a, kb * kBK, arow, fb);
          tma_load_2d_pair(st + kTileA, map_b, kb * kBK, tn * kBN, fb);
        }
      }
      // CTA 0's full barriers count the copies of both CTAs: it drains them
      if (rank == 0)
        for (uint32_t u = (it > kStages2 ? it - kStages2 : 0); u < it; ++u)
          if (!mbar_wait_cl(full0 + 8u * (u % kStages2), (u / kStages2) & 1u, kWaitLimitNs))
            atomicAdd(&g_ff_timeouts, 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA (CTA 0)
    if (lane == 0 && rank == 0) {
      uint32_t it = 0, j = 0;
      for (int t = pair; t < tiles && !abort_flag; t += pairs, ++j) {
        const uint32_t b = j & 1u;
        if (j >= 2 && !mbar_wait_cl(tempty0 + 8u * b, ((j >> 1) & 1u) ^ 1u, kWaitLimitNs)) {
          atomicAdd(&g_ff_timeouts, 1u);
          abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_base = tmem + b * 2u * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kStages2;
          if (abort_flag) break;
          if (!mbar_wait_cl(full0 + 8u * s, (it / kStages2) & 1u, kWaitLimitNs)) {
            atomicAdd(&g_ff_timeouts, 1u);
            abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = ring + s * kStage2Bytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(st + 32u * k);
            const uint64_t bd = smem_desc_sw128(st + kTileA + 32u * k);
            umma2_f16(acc_base, ad, bd, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma2_commit_both(empty0 + 8u * s);
        }
        umma2_commit_both(tfull0 + 8u * b);
      }
      umma2_commit_both(done_bar);
      if (!mbar_wait_cl(done_bar, 0u, kWaitLimitNs)) atomicAdd(&g_ff_timeouts, 1u);
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t tempty_leader = map_to_rank(tempty0, 0);
    uint32_t j = 0;
    for (int t = pair; t < tiles; t += pairs, ++j) {
      if (abort_flag) break;
      const uint32_t b = j & 1u;
      if (!mbar_wait_cl(tfull0 + 8u * b, (j >> 1) & 1u, kWaitLimitNs)) {
        atomicAdd(&g_ff_timeouts, 1u);
        abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int tm, tn;
      tile_coords(t, mt, nt, tm, tn);
      const int64_t m = static_cast<int64_t>(tm) * 2 * kBM + static_cast<int64_t>(rank) * kBM + 32 * q + lane;
      const int64_t n0 = static_cast<int64_t>(tn) * kBN;
      const bool row_ok = m < a.M;
      const float an = row_ok ? a.a_norm[m] : 0.f;
      const uint32_t lane_addr = tmem + b * 2u * kBN + (static_cast<uint32_t>(32 * q) << 16);
      __half* orow = a.out + m * a.N;
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r1[32], r3[32];
        tmem_ld32(lane_addr + 32u * c, r1);
        tmem_ld32(lane_addr + kBN + 32u * c, r3);
        if (c == kBN / 32 - 1) {  // both accumulators read: hand the buffer back to CTA 0's MMA thread
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(tempty_leader + 8u * b);
        }
        #ifdef DSLPG_FF_DIAG_NO_EPILOGUE  // diagnostic builds only: time the main loop without the epilogue's math and stores
        continue;
#endif
        if (!row_ok) continue;
        const int64_t nb = n0 + 32 * c;
        uint32_t packed[16];
        gate_pack(r1, r3, an, packed);
        if (nb + 32 <= a.N && (a.N % 8) == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            st_stream(orow + nb + 8 * i, Vec16{{packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]}});
        } else {
          for (int i = 0; i < 32; ++i) {
            if (nb + i >= a.N) break;
            const uint32_t w = packed[i >> 1];
            orow[nb + i] = __ushort_as_half(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xffffu)));
          }
        }
      }
    }
  }

  // Neither CTA leaves (nor frees TMEM) while the pair's MMAs, copies or
  // remote arrivals may still touch its memory.
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------- few rows (GEMV)
// ff_gemv_kernel: M <= 3 by default (decode-like). Reading the weights is the
// whole cost, and the tensor-core kernels read each weight row in 128-byte
// pieces, 256 rows at a time. Here one warp takes one output column n at a
// time and streams the weight rows w1[n] and w3[n] contiguously (512 bytes per
// warp load, U loads of each in flight), against the M rows of xs staged in
// shared memory; fp32 accumulation on f32x2 pairs, a warp butterfly, and lane
// m applies the a_norm scale and the SiLU gate of row m.
constexpr int kGemvMaxRows = 8;   // the kernel's limit (DSLPG_PATH_STREAM forces it up to here)
constexpr int kGemvAutoRows = 3;  // chosen by default up to here. Measured per call (K = 4096,
                                  // N = 16384) against the tensor-core kernel: 50.7 / 68.0 us at M = 1,
                                  // 52.9 / 68.7 at M = 2, 65.8 / 68.4 at M = 3, even at M = 4, 117 / 72
                                  // at M = 8 (its CUDA-core FMAs grow with M)
constexpr int kGemvThreads = 256;
constexpr int kGemvMaxSmem = 96 * 1024;  // xs staged per CTA: M * K * 2 bytes at most

template <int MB>
__global__ void __launch_bounds__(kGemvThreads) ff_gemv_kernel(const __half* __restrict__ xs,
                                                               const __half* __restrict__ w1,
                                                               const __half* __restrict__ w3, const FfArgs a) {
  constexpr int U = 4;
  extern __shared__ __align__(16) unsigned char smem_g[];
  const int K = a.K, M = static_cast<int>(a.M), kv = K / 8;
  Vec16* sx = reinterpret_cast<Vec16*>(smem_g);  // [M][kv]
  for (int i = threadIdx.x; i < M * kv; i += kGemvThreads) sx[i] = ld_keep(xs + static_cast<int64_t>(i) * 8);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kGemvThreads / 32);
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * (kGemvThreads / 32) + (threadIdx.x >> 5); n < a.N;
       n += nwarps) {
    const __half* r1 = w1 + n * K;
    const __half* r3 = w3 + n * K;
    f32x2 acc1[MB], acc3[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) acc1[m] = acc3[m] = pk2(0.f, 0.f);
    for (int j0 = lane; j0 < kv; j0 += 32 * U) {
      Vec16 v1[U], v3[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + 32 * u;
        if (j < kv) {
          v1[u] = ld_stream(r1 + static_cast<int64_t>(j) * 8);
          v3[u] = ld_stream(r3 + static_cast<int64_t>(j) * 8);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + 32 * u;
        if (j >= kv) continue;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m >= M) break;
          const Vec16 xv = sx[m * kv + j];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const f32x2 xp = unpack_pair<__half>(xv, p);
            acc1[m] = fma2(unpack_pair<__half>(v1[u], p), xp, acc1[m]);
            acc3[m] = fma2(unpack_pair<__half>(v3[u], p), xp, acc3[m]);
          }
        }
      }
    }
    float mine1 = 0.f, mine3 = 0.f;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      if (m >= M) break;
      const float s1 = warp_reduce<SumOp>(hsum2(acc1[m]));
      const float s3 = warp_reduce<SumOp>(hsum2(acc3[m]));
      if (lane == m) {
        mine1 = s1;
        mine3 = s3;
      }
    }
    if (lane < M) {
      const float an = a.a_norm[lane];
      const float g = mine1 * an, u = mine3 * an;
      const float sig = rcp_approx(1.0f + ex2(-g * kLog2e));
      a.out[static_cast<int64_t>(lane) * a.N + n] = __float2half_rn((g * sig) * u);
    }
  }
}

namespace {
template <int MB>
cudaError_t launch_gemv(const __half* xs, const __half* w1, const __half* w3, const FfArgs& args, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&ff_gemv_kernel<MB>);
  const size_t smem = static_cast<size_t>(args.M) * args.K * 2;
  if (cudaError_t e = allow_dynamic_smem(fn, smem)) return e;
  const int grid = persistent_grid(fn, kGemvThreads, smem, (args.N + 7) / 8);
  ff_gemv_kernel<MB><<<grid, kGemvThreads, smem, st>>>(xs, w1, w3, args);
  return cudaGetLastError();
}
}  // namespace

// ------------------------------------------------------------------- host
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [rows, K] fp16 row-major, boxes of box_rows rows x 64 columns, 128-byte swizzle,
// zero fill out of bounds.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int K, uint32_t box_rows = 128) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {kBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

unsigned int take_wait_timeouts_ff() {
  unsigned int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_ff_timeouts, sizeof(v));
  cudaMemcpyToSymbol(g_ff_timeouts, &zero, sizeof(zero));
  return v;
}

}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_kernel_ff_workspace_bytes(int64_t M, int64_t K, int64_t* bytes) {
  if (bytes == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || K < 0) return DSLPG_ERR_BAD_SHAPE;
  // xs [M, K] fp16 (256-byte aligned), then a_norm [M] fp32
  *bytes = ((M * K * 2 + 255) / 256) * 256 + M * 4;
  return DSLPG_OK;
}

extern "C" int dslpg_kernel_ff(const void* x, const void* w1, const void* w3, const void* rms_w, void* out,
                               int64_t M, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                               cudaStream_t stream) {
  if (!x || !w1 || !w3 || !rms_w || !out || !workspace) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0 || K <= 0 || K % 8 != 0 || K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff)
    return DSLPG_ERR_BAD_SHAPE;
  int64_t need = 0;
  dslpg_kernel_ff_workspace_bytes(M, K, &need);
  if (workspace_bytes < need) return DSLPG_ERR_BAD_ARGUMENT;
  if (!aligned(x, 16) || !aligned(w1, 16) || !aligned(w3, 16) || !aligned(rms_w, 16) || !aligned(out, 16) ||
      !aligned(workspace, 256))
    return DSLPG_ERR_BAD_ARGUMENT;
  if (M == 0 || N == 0) return DSLPG_OK;
  __half* xs = static_cast<__half*>(workspace);
  float* a_norm = reinterpret_cast<float*>(static_cast<char*>(workspace) + ((M * K * 2 + 255) / 256) * 256);

  const int pgrid = persistent_grid(reinterpret_cast<const void*>(&ff_prologue_kernel), 256, 0, (M + 7) / 8);
  ff_prologue_kernel<<<pgrid, 256, 0, stream>>>(static_cast<const __half*>(x), static_cast<const __half*>(rms_w), xs,
                                                a_norm, M, static_cast<int>(K));
  if (cudaError_t e = cudaGetLastError()) return static_cast<int>(e);

  FfArgs args{a_norm, static_cast<__half*>(out), M, N, static_cast<int>(K)};
  const int path = kernel_path();
  // Few rows: the weight-streaming kernel (DSLPG_PATH_STREAM forces it where it applies).
  const bool gemv_fits = M <= kGemvMaxRows && M * K * 2 <= kGemvMaxSmem;
  if (gemv_fits && ((path == DSLPG_PATH_AUTO && M <= kGemvAutoRows) || path == DSLPG_PATH_STREAM)) {
    const __half* w1h = static_cast<const __half*>(w1);
    const __half* w3h = static_cast<const __half*>(w3);
    cudaError_t e;
    if (M == 1) e = launch_gemv<1>(xs, w1h, w3h, args, stream);
    else if (M == 2) e = launch_gemv<2>(xs, w1h, w3h, args, stream);
    else if (M <= 4) e = launch_gemv<4>(xs, w1h, w3h, args, stream);
    else e = launch_gemv<8>(xs, w1h, w3h, args, stream);
    return static_cast<int>(e);
  }
  const bool use_pair = path == DSLPG_PATH_CLUSTER || (path != DSLPG_PATH_RESIDENT && M > kBM);
  CUtensorMap ma, mb1, mb3;
  if (!make_map(&ma, xs, M, static_cast<int>(K)) || !make_map(&mb1, w1, N, static_cast<int>(K)) ||
      !make_map(&mb3, w3, N, static_cast<int>(K)))
    return static_cast<int>(cudaErrorInvalidValue);
  if (use_pair) {
    const int64_t tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
    if (tiles > 0x3fffffff) return DSLPG_ERR_BAD_SHAPE;
    const void* fn = reinterpret_cast<const void*>(&ff_gemm2_kernel);
    if (cudaError_t e = allow_dynamic_smem(fn, kFfSmem2)) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kFfThreads);
    cfg.dynamicSmemBytes = kFfSmem2;
    cfg.stream = stream;
    cfg.gridDim = dim3(2);
    // co-resident CTA pairs on this device (cached per device with the occupancy figures)
    const int max_pairs = max_active_clusters(fn, cfg, 2, sm_count() / 2);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * std::min<int64_t>(tiles, max_pairs)));
    return static_cast<int>(cudaLaunchKernelEx(&cfg, ff_gemm2_kernel, ma, mb1, mb3, args));
  }
  const void* fn = reinterpret_cast<const void*>(&ff_gemm_kernel);
  if (cudaError_t e = allow_dynamic_smem(fn, kFfSmem)) return static_cast<int>(e);
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  if (tiles > 0x7fffffff) return DSLPG_ERR_BAD_SHAPE;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));  // one CTA per SM (TMEM: all 512 columns)
  ff_gemm_kernel<<<grid, kFfThreads, kFfSmem, stream>>>(ma, mb1, mb3, args);
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------ static-scratch entry
// dslpg_kernel_ff for callers that cannot allocate device memory per call (a
// C / FFI host with no device allocator of its own, or a loop that must not
// pay cudaMalloc / cudaFree's device-wide synchronisation). xs and a_norm go to
// this file-scope scratch instead of a caller workspace; nothing in it must
// start at zero, since the prologue writes every byte the GEMM reads. One
// scratch per device: overlapping calls on a device race on it.
namespace dslpg {
namespace {
constexpr int64_t kStaticScratchBytes = DSLPG_KERNEL_FF_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_ff_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchAddr {
  unsigned long long ctx_id = 0;  // the CUDA context the address belongs to (0: none yet)
  void* addr = nullptr;
};
ScratchAddr g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// The unique id of the calling thread's current CUDA context (0 when it cannot
// be read). A device reset or a new primary context gets a new id, which is
// what makes a cached scratch address stale.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetCurrentFn>(p) : nullptr;
  }();
  static CtxGetIdFn get_id = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetIdFn>(p) : nullptr;
  }();
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// The scratch's device address in the current device's current context. The
// lookup (cudaGetSymbolAddress, with that device current) is the set-up step:
// it runs on the first call on each device, and again only after the device's
// context has been replaced (for example after cudaDeviceReset), since the
// module's addresses belong to the context that loaded it.
cudaError_t static_scratch(void** out) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& slot = g_scratch_addr[dev];
  unsigned long long id = current_context_id();
  if (slot.addr == nullptr || id == 0 || slot.ctx_id != id) {
    void* p = nullptr;
    if (cudaError_t e = cudaGetSymbolAddress(&p, g_ff_scratch)) return e;
    if (id == 0) id = current_context_id();  // the lookup made the context current
    slot.addr = p;
    slot.ctx_id = id;
  }
  *out = slot.addr;
  return cudaSuccess;
}
}  // namespace
}  // namespace dslpg

extern "C" int dslpg_kernel_ff_static(const void* x, const void* w1, const void* w3, const void* rms_w, void* out,
                                      int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (!x || !w1 || !w3 || !rms_w || !out) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0 || K <= 0 || K % 8 != 0 || K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff)
    return DSLPG_ERR_BAD_SHAPE;
  if (M > 0 && K > kStaticScratchBytes / (2 * M)) return DSLPG_ERR_TOO_LARGE;  // before M * K can overflow
  int64_t need = 0;
  dslpg_kernel_ff_workspace_bytes(M, K, &need);
  if (need > kStaticScratchBytes) return DSLPG_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return DSLPG_OK;
  void* scratch = nullptr;
  if (cudaError_t e = static_scratch(&scratch)) return static_cast<int>(e);
  return dslpg_kernel_ff(x, w1, w3, rms_w, out, M, N, K, scratch, kStaticScratchBytes, stream);
}
