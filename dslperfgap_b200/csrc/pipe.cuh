// pipe.cuh — TMA bulk-copy pipeline plumbing for sm_100a.
//
// A CTA is one producer warp plus C consumer threads. The producer's lane 0
// streams fixed-size stages (a row, or a chunk of a long row) from global
// memory into a ring of S shared-memory slots with `cp.async.bulk` (plain
// bulk copies into the CTA's own shared memory, never multicast); each slot
// has a "full" mbarrier (transaction-counted) and an "empty" mbarrier (one
// arrival per consumer warp). Consumers wait on full[s], read their slice,
// and release the slot; so the memory system always has up to S stages per
// CTA in flight regardless of how many registers the consumers use.
//
// Every wait is bounded in wall-clock time (%globaltimer). A wait that runs
// out records the event in a per-translation-unit device counter, which the
// host reads back with dslpg_take_wait_timeouts(), and the waiting thread
// abandons the kernel; the producer always waits (again bounded) for the
// copies it issued before the CTA exits, so no copy is left in flight.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace dslpg {

// Wall-clock limit of any single wait: far above any legitimate wait.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s

DSLPG_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DSLPG_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

DSLPG_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
DSLPG_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

DSLPG_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

DSLPG_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

DSLPG_DEV bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity of barrier `bar` has completed.
// Returns false if `limit_ns` of wall-clock time passed first.
DSLPG_DEV bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_test(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

// Policy for read-once data: evict first from L2.
DSLPG_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Bulk copy `bytes` (multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on mbarrier `bar`.
DSLPG_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

DSLPG_DEV Vec16 lds16(uint32_t addr) {
  Vec16 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "r"(addr));
  return v;
}

// Barrier among the consumer threads only (named barrier 1).
DSLPG_DEV void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Reduction over all consumer threads (warps 1.. of the CTA). `red` holds 32
// floats; alternate two buffers between back-to-back reductions.
template <class Op>
DSLPG_DEV float consumer_reduce(float v, float* red, int ncw) {
  v = warp_reduce<Op>(v);
  if (ncw == 1) return v;
  const int lane = threadIdx.x & 31;
  if (lane == 0) red[(threadIdx.x >> 5) - 1] = v;
  consumer_sync(ncw * 32);
  float r = lane < ncw ? red[lane] : Op::identity();
  return warp_reduce<Op>(r);
}

// Reductions over the threads of a row group of the register-resident kernel.
struct GroupReducer {
  float (*red)[32];
  int nw, first_warp, buf;
  float (*red2)[64];  // pair sums (LayerNorm), double-buffered with their own toggle
  int buf2;
  template <class Op> DSLPG_DEV float reduce(float v) {
    v = group_reduce<Op>(v, red[buf], nw, first_warp);
    buf ^= 1;
    return v;
  }
  // A reduction that only this row group's threads take part in (a branch
  // that other groups of the CTA may skip): its barrier is the group's own
  // named barrier (1 + group index; at most 8 groups of one warp each, which
  // need no barrier, or 4 groups of two warps and more).
  template <class Op> DSLPG_DEV float reduce_own(float v) {
    v = warp_reduce<Op>(v);
    if (nw == 1) return v;
    float* r = red[buf];
    buf ^= 1;
    const int lane = threadIdx.x & 31;
    if (lane == 0) r[threadIdx.x >> 5] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + first_warp / nw), "r"(nw * 32) : "memory");
    float q = lane < nw ? r[first_warp + lane] : Op::identity();
    return warp_reduce<Op>(q);
  }
  // Two sums in one exchange: both values ride the same shuffles and barrier.
  DSLPG_DEV void sum_pair(float& a, float& b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (nw == 1) return;
    float* r = red2[buf2];
    buf2 ^= 1;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) {
      r[2 * w] = a;
      r[2 * w + 1] = b;
    }
    __syncthreads();
    a = lane < nw ? r[2 * (first_warp + lane)] : 0.f;
    b = lane < nw ? r[2 * (first_warp + lane) + 1] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
  }
};

// Reductions over the consumer threads of a TMA-pipelined CTA.
struct ConsumerReducer {
  float* red;  // [2][32]
  int ncw, buf;
  template <class Op> DSLPG_DEV float reduce(float v) {
    v = consumer_reduce<Op>(v, red + 32 * buf, ncw);
    buf ^= 1;
    return v;
  }
  DSLPG_DEV void sum_pair(float& a, float& b) {
    a = reduce<SumOp>(a);
    b = reduce<SumOp>(b);
  }
  // one row per CTA or cluster: every thread takes the same branches
  template <class Op> DSLPG_DEV float reduce_own(float v) { return reduce<Op>(v); }
};

// Reductions over a whole cluster: a CTA-wide reduction, the C per-CTA values
// exchanged through distributed shared memory after one cluster barrier, and
// combined in rank order by every thread (so all CTAs agree bit for bit). The
// exchange slots are double-buffered: a slot is rewritten two reductions
// later, after a cluster barrier that follows every read of it.
struct ClusterReducer {
  float* slots;  // [2] in this CTA's shared memory
  float (*red)[32];
  int buf, C;
  template <class Op> DSLPG_DEV float reduce(float v) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    v = group_reduce<Op>(v, red[buf], blockDim.x >> 5, 0);
    if (threadIdx.x == 0) slots[buf] = v;
    cl.sync();
    float r = *cl.map_shared_rank(&slots[buf], 0);
    for (int q = 1; q < C; ++q) r = Op::apply(r, *cl.map_shared_rank(&slots[buf], q));
    buf ^= 1;
    return r;
  }
  DSLPG_DEV void sum_pair(float& a, float& b) {
    a = reduce<SumOp>(a);
    b = reduce<SumOp>(b);
  }
  // one row per CTA or cluster: every thread takes the same branches
  template <class Op> DSLPG_DEV float reduce_own(float v) { return reduce<Op>(v); }
};

// Ring bookkeeping: use number u of the ring (0, 1, 2, ...) maps to slot
// u % S and phase u / S.
struct Ring {
  uint32_t base;   // shared address of slot 0
  uint32_t full;   // shared address of full[0] (8 bytes per barrier)
  uint32_t empty;  // shared address of empty[0]
  uint32_t slot_bytes;
  int stages;
  DSLPG_DEV uint32_t slot(uint32_t u) const { return base + (u % stages) * slot_bytes; }
  DSLPG_DEV uint32_t full_bar(uint32_t u) const { return full + 8u * (u % stages); }
  DSLPG_DEV uint32_t empty_bar(uint32_t u) const { return empty + 8u * (u % stages); }
  DSLPG_DEV uint32_t parity(uint32_t u) const { return (u / stages) & 1u; }
};

// Layout of the dynamic shared memory: S slots, then 2*S barriers, then
// scratch for reductions.
struct RingLayout {
  static constexpr uint32_t kAlign = 128;
  static __host__ __device__ uint32_t barriers_offset(uint32_t slot_bytes, int stages) {
    return (slot_bytes * stages + 15u) & ~15u;
  }
  static __host__ __device__ uint32_t total_bytes(uint32_t slot_bytes, int stages) {
    return barriers_offset(slot_bytes, stages) + 16u * stages + 2u * 32u * 4u;
  }
};

// Set up the ring in dynamic shared memory (called by every thread).
DSLPG_DEV Ring ring_setup(unsigned char* smem, uint32_t slot_bytes, int stages, int consumer_warps,
                          float** red_out) {
  Ring r;
  r.base = smem_u32(smem);
  const uint32_t boff = RingLayout::barriers_offset(slot_bytes, stages);
  r.full = r.base + boff;
  r.empty = r.full + 8u * stages;
  r.slot_bytes = slot_bytes;
  r.stages = stages;
  *red_out = reinterpret_cast<float*>(smem + boff + 16u * stages);
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(r.full + 8u * s, 1);
      mbar_init(r.empty + 8u * s, consumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  return r;
}

// Producer-side drain: wait (bounded) for the last copy issued into every
// slot, so that no bulk copy into this CTA's shared memory is still in flight
// when the CTA exits. `issued` is the number of ring uses the producer made.
DSLPG_DEV bool ring_drain(const Ring& r, uint32_t issued) {
  bool ok = true;
  const uint32_t first = issued > static_cast<uint32_t>(r.stages) ? issued - r.stages : 0;
  for (uint32_t u = first; u < issued; ++u) ok = mbar_wait(r.full_bar(u), r.parity(u), kWaitLimitNs) && ok;
  return ok;
}

}  // namespace dslpg
