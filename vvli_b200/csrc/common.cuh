// common.cuh - device helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define VVLI_DEV __device__ __forceinline__

namespace vvli {

constexpr int kWarp = 32;

// ---------------------------------------------------------------- bf16
// bf16ToF32 (src/llm.zig:791-793): the 16 bits become the high half of an f32.
VVLI_DEV float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
VVLI_DEV float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }
VVLI_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// f32ToBf16 (src/llm.zig:799-803): round to nearest even on the bit pattern.
VVLI_DEV uint16_t f32_to_bf16(float v) {
  uint32_t bits = __float_as_uint(v);
  return static_cast<uint16_t>((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

// ---------------------------------------------------------------- memory
// Streaming 128-bit load of read-only weights: non-coherent path, no L1 allocation.
VVLI_DEV uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Fire-and-forget bulk prefetch of [p, p+bytes) into L2 (bytes multiple of 16).
VVLI_DEV void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// griddepcontrol.wait blocks until every prerequisite grid has completed and
// its memory is visible; a no-op when the launch had no programmatic edge.
VVLI_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream start launching its CTAs now.
VVLI_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- reductions
VVLI_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

VVLI_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Argmax candidate order of llm.argmax (src/llm.zig:778-789): the larger
// value wins; equal values keep the lower index (first index wins ties).
VVLI_DEV bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

VVLI_DEV void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

// ---------------------------------------------------------------- synthetic weights
// Counter-based generator, bit-identical to oracle/vvli_ref_cpu.cpp:
// SplitMix64 outputs -> twelve 16-bit uniforms -> Irwin-Hall sum (exact in
// fp32) -> * std in fp32 -> f32ToBf16.
VVLI_DEV uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// ---------------------------------------------------------------- mbarrier + bulk copy (TMA, no multicast)
VVLI_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

VVLI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the async (bulk-copy) proxy.
VVLI_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

VVLI_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
VVLI_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
VVLI_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
VVLI_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait
constexpr int kErrTimeout = 22;                    // VVLI_ERR_TIMEOUT

// Bounded wait for the completion of phase `parity` of an mbarrier.  On
// timeout it records VVLI_ERR_TIMEOUT in *err and returns false.
VVLI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, kErrTimeout);
      return false;
    }
  }
}

// Bulk copy global -> shared (the CTA's own shared memory), completing
// `bytes` of transaction count on `bar`.  16-byte aligned, bytes % 16 == 0.
VVLI_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Barrier among the first `count` threads (named barrier `id`, 1..15).
VVLI_DEV void named_barrier(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

}  // namespace vvli
