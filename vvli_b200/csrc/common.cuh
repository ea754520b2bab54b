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

}  // namespace vvli
