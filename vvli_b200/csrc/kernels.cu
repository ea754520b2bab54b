#include <cuda_fp16.h>
// kernels.cu - decode-step kernels for sm_100a.
//
// One decode token per layer runs five kernels, chained with programmatic
// dependent launch (PDL) inside one CUDA graph:
//   gemv<PLAIN>    rmsnorm(x) prologue, fused q|k|v rows, + bias      (src/llm.zig:736-740)
//   attention      RoPE on q and k, KV write, flash-decode, combine   (src/llm.zig:742-755)
//   gemv<PLAIN>    o_proj + residual add                               (src/llm.zig:756-757)
//   gemv<SILU_MUL> rmsnorm prologue, gate|up rows, silu(g)*u          (src/llm.zig:759-763)
//   gemv<PLAIN>    down_proj + residual add                            (src/llm.zig:764-765)
// and the LM head is gemv<ARGMAX> with the final-norm prologue
// (src/llm.zig:727-728) and llm.argmax fused (src/llm.zig:778-789).
#include "common.cuh"
#include "device_fns.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>

namespace vvli {

// Row epilogue shared by both GEMV kernels: sums a row's k-split partials in
// a fixed order, then applies bias / residual (linearRange + addInto,
// src/llm.zig:1271-1275, 1389-1396) or silu(g)*u (siluMulInto,
// src/llm.zig:1382-1387); tracks the argmax for the LM head.
template <int EPI>
__device__ void gemv_epilogue(const GemvParams& p, const float* part, int S, int r0, int nrows, int tid,
                              int nthreads, int lane, int warp, float* wv, int* wi, int* last_flag,
                              bool use_named_barrier) {
  constexpr int NPHYS = (EPI == EPI_SILU_MUL) ? 2 : 1;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (int rl = tid; rl < nrows; rl += nthreads) {
    const int r = r0 + rl;
    float a = 0.f;
    if (EPI == EPI_SILU_MUL) {
      float g = 0.f, u = 0.f;
      for (int s = 0; s < S; ++s) {
        g += part[(NPHYS * rl) * S + s];
        u += part[(NPHYS * rl + 1) * S + s];
      }
      a = (g / (1.0f + expf(-g))) * u;
    } else {
      for (int s = 0; s < S; ++s) a += part[rl * S + s];
      if (p.bias) a = a + bf16_to_f32(p.bias[r]);
      if (p.residual) a = p.residual[r] + a;
    }
    p.y[r] = a;
    if (EPI == EPI_ARGMAX && better(a, r + p.row_base, best_v, best_i)) {
      best_v = a;
      best_i = r + p.row_base;
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
    // CTA argmax, then the last CTA to finish reduces the per-CTA results.
    const int nwarps = nthreads / kWarp;
    warp_argmax(best_v, best_i);
    if (lane == 0) {
      wv[warp] = best_v;
      wi[warp] = best_i;
    }
    if (use_named_barrier) named_barrier(1, nthreads); else __syncthreads();
    if (tid == 0) {
      float bv = wv[0];
      int bi = wi[0];
      for (int i = 1; i < nwarps; ++i)
        if (better(wv[i], wi[i], bv, bi)) {
          bv = wv[i];
          bi = wi[i];
        }
      p.part_val[blockIdx.x] = bv;
      p.part_idx[blockIdx.x] = bi;
      __threadfence();
      *last_flag = atomicAdd(p.counter, 1u) == gridDim.x - 1;
      if (*last_flag) {
        __threadfence();
        float bv2 = __ldcg(p.part_val);
        int bi2 = __ldcg(p.part_idx);
        for (unsigned b = 1; b < gridDim.x; ++b) {
          const float v = __ldcg(p.part_val + b);
          const int i = __ldcg(p.part_idx + b);
          if (better(v, i, bv2, bi2)) {
            bv2 = v;
            bi2 = i;
          }
        }
        *p.counter = 0;
        if (p.finalize) {
          publish_argmax(p.st, p.seq_tokens, bi2);
        } else {
          p.local_best[0] = bv2;
          p.local_best[1] = __int_as_float(bi2);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- GEMV: bulk-copy pipeline
// y = W . x for bf16 W [N, K] and fp32 x with fp32 accumulation (linearInto,
// src/llm.zig:1228-1275).  HBM-bound: each weight byte is read once.
//
// CTA b owns the contiguous rows [b*N/G, (b+1)*N/G), one CTA per SM.  Warp 8
// is the producer: one lane streams the CTA's rows through a ring of
// `nst` shared-memory stages with cp.async.bulk (R whole rows per stage,
// completion counted on a full-barrier), starting before the PDL wait, so
// the weights of this kernel are in flight while the previous kernel
// finishes.  Warps 0-7 consume: warp w always owns k-split w % S of a row,
// so the matching slice of x (after the fused RMSNorm) lives in registers
// for the whole kernel, and every 16-byte weight chunk is read once from
// shared memory.  Row partials meet in shared memory and are summed in a
// fixed order (deterministic).  Every mbarrier wait is bounded (2 s) and
// reports VVLI_ERR_TIMEOUT through StepState.err.
constexpr int kTmaMaxConsumerWarps = 16;

template <int EPI, int MAXC, bool ILP2>
__global__ void __launch_bounds__((kTmaMaxConsumerWarps + 1) * kWarp, 1) gemv_tma_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kTmaMaxConsumerWarps];
  __shared__ float wv[kTmaMaxConsumerWarps];
  __shared__ int wi[kTmaMaxConsumerWarps];
  __shared__ int last_flag;
  constexpr int NPHYS = (EPI == EPI_SILU_MUL) ? 2 : 1;
  const int CW = static_cast<int>(blockDim.x / kWarp) - 1;  // consumer warps; the last warp produces
  const int NC = CW * kWarp;
  const int K = p.K, N = p.N, S = p.S, R = p.R, nst = p.nst;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = static_cast<int>((static_cast<long long>(blockIdx.x) * N) / gridDim.x);
  const int r1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * N) / gridDim.x);
  const int nrows = r1 - r0;
  const int nstages = (nrows + R - 1) / R;
  const size_t row_bytes = static_cast<size_t>(K) * 2;
  uint8_t* ring = smem;
  float* part = reinterpret_cast<float*>(smem + static_cast<size_t>(nst) * p.stage_bytes);
  const size_t part_floats = static_cast<size_t>(p.part_rows) * NPHYS * S;
  uint64_t* full = reinterpret_cast<uint64_t*>(part + ((part_floats + 1) & ~static_cast<size_t>(1)));
  uint64_t* empty = full + nst;
  int* err = p.st ? &p.st->err : nullptr;

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CW) {  // producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nstages; ++i) {
        const int slot = i % nst;
        if (i >= nst && !mbar_wait(&empty[slot], ((i / nst) - 1) & 1, err)) break;
        const int rows_here = min(R, nrows - i * R);
        const uint32_t bytes = static_cast<uint32_t>(rows_here * row_bytes);
        mbar_arrive_expect_tx(&full[slot], bytes * NPHYS);
#pragma unroll
        for (int ph = 0; ph < NPHYS; ++ph)
          bulk_g2s(ring + static_cast<size_t>(slot) * p.stage_bytes + ph * R * row_bytes,
                   p.W + static_cast<size_t>(r0 + i * R + ph * p.pair_offset) * K, bytes, &full[slot]);
        issued = i + 1;
        if (i + 1 == min(nst, nstages) && p.next_W) {
          // Warm L2 with the head of this CTA's rows in the next GEMV (one
          // stage-sized window per matrix), so its first stages skip DRAM latency.
          const int n0 = static_cast<int>((static_cast<long long>(blockIdx.x) * p.next_N) / gridDim.x);
          const int n1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * p.next_N) / gridDim.x);
          const size_t nb = static_cast<size_t>(n1 - n0) * p.next_K * 2;
          const uint32_t pre = static_cast<uint32_t>(nb < static_cast<size_t>(p.stage_bytes) ? nb : p.stage_bytes);
          if (pre >= 16) {
            prefetch_l2_bulk(p.next_W + static_cast<size_t>(n0) * p.next_K, pre & ~15u);
            if (p.next_pair_offset)
              prefetch_l2_bulk(p.next_W + static_cast<size_t>(n0 + p.next_pair_offset) * p.next_K, pre & ~15u);
          }
        }
      }
      // Every copy this thread issued has landed before the CTA may exit.
      for (int i = max(0, issued - nst); i < issued; ++i) mbar_wait(&full[i % nst], (i / nst) & 1, err);
    }
    return;
  }

  // ---- consumers
  grid_dependency_wait();
  grid_launch_dependents();
  float scale = 1.f;
  if (p.norm_w) {  // rmsNormInto (src/llm.zig:1287-1300), fused
    float ss = 0.f;
    for (int i = tid; i < K; i += NC) ss = fmaf(p.x[i], p.x[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_barrier(1, NC);
    float t = 0.f;
    for (int i = 0; i < CW; ++i) t += red[i];
    scale = 1.0f / sqrtf(t / static_cast<float>(K) + p.eps);
  }
  const int cpr = K >> 3;
  const int split = warp % S;
  const int cbeg = split * p.SZ;
  const int cend = min(cpr, cbeg + p.SZ);
  float xr[MAXC][8];
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int c = cbeg + lane + kWarp * j;
    if (j < p.cpl && c < cend) {
      const float4 a = *reinterpret_cast<const float4*>(p.x + c * 8);
      const float4 b = *reinterpret_cast<const float4*>(p.x + c * 8 + 4);
      xr[j][0] = a.x, xr[j][1] = a.y, xr[j][2] = a.z, xr[j][3] = a.w;
      xr[j][4] = b.x, xr[j][5] = b.y, xr[j][6] = b.z, xr[j][7] = b.w;
      if (p.norm_w) {
        const uint4 wn = *reinterpret_cast<const uint4*>(p.norm_w + c * 8);
        const float nw[8] = {bf16_lo(wn.x), bf16_hi(wn.x), bf16_lo(wn.y), bf16_hi(wn.y),
                             bf16_lo(wn.z), bf16_hi(wn.z), bf16_lo(wn.w), bf16_hi(wn.w)};
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[j][e] = xr[j][e] * nw[e] * scale;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xr[j][e] = 0.f;
    }
  }

  // Dot product of this warp's x slice with one row split held in the stage.
  auto row_dot = [&](const uint8_t* rp) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      const int c = cbeg + lane + kWarp * j;
      if (j < p.cpl && c < cend) acc += dot8(*reinterpret_cast<const uint4*>(rp + c * 16), xr[j]);
    }
    return acc;
  };
  auto pair_row = [&](int pi, int& ph, int& row) {
    const int t = pi / S;
    ph = (NPHYS == 2) ? (t & 1) : 0;
    row = (NPHYS == 2) ? (t >> 1) : t;
  };

  const int pairs = R * NPHYS * S;
  for (int i = 0; i < nstages; ++i) {
    const int slot = i % nst;
    if (!mbar_wait(&full[slot], (i / nst) & 1, err)) break;
    const int rows_here = min(R, nrows - i * R);
    const uint8_t* stg = ring + static_cast<size_t>(slot) * p.stage_bytes;
    if constexpr (ILP2) {
      // Two rows per iteration (pairs pi and pi + CW share this warp's split).
      for (int pi = warp; pi < pairs; pi += 2 * CW) {
        int pha, rowa, phb, rowb;
        pair_row(pi, pha, rowa);
        pair_row(pi + CW, phb, rowb);
        const bool va = rowa < rows_here;
        const bool vb = pi + CW < pairs && rowb < rows_here;
        const float a = va ? row_dot(stg + pha * R * row_bytes + rowa * row_bytes) : 0.f;
        const float b = vb ? row_dot(stg + phb * R * row_bytes + rowb * row_bytes) : 0.f;
        const float v = warp_sum2(a, b, lane);
        if (lane == 0 && va) part[((i * R + rowa) * NPHYS + pha) * S + split] = v;
        if (lane == 16 && vb) part[((i * R + rowb) * NPHYS + phb) * S + split] = v;
      }
    } else {
      for (int pi = warp; pi < pairs; pi += CW) {
        int ph, row;
        pair_row(pi, ph, row);
        if (row < rows_here) {
          const float acc = warp_sum(row_dot(stg + ph * R * row_bytes + row * row_bytes));
          if (lane == 0) part[((i * R + row) * NPHYS + ph) * S + split] = acc;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  named_barrier(1, NC);
  gemv_epilogue<EPI>(p, part, S, r0, nrows, tid, NC, lane, warp, wv, wi, &last_flag, true);
}

// ---------------------------------------------------------------- GEMV: register streaming (long rows)
// Fallback for K > 16384: 128-bit non-coherent loads straight into registers,
// 4 work items (row x 128 chunks) in flight per warp, x from shared memory.
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / kWarp;
constexpr int kItemChunks = 128;
constexpr int kItemsInFlight = 4;

template <int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_stream_kernel(const GemvParams p) {
  extern __shared__ __align__(16) float smem_f[];
  __shared__ float red[32];
  __shared__ float wv[kGemvWarps];
  __shared__ int wi[kGemvWarps];
  __shared__ int last_flag;
  constexpr int NPHYS = (EPI == EPI_SILU_MUL) ? 2 : 1;
  const int K = p.K, N = p.N;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = static_cast<int>((static_cast<long long>(blockIdx.x) * N) / gridDim.x);
  const int r1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * N) / gridDim.x);
  const int nrows = r1 - r0;
  const int cpr = K >> 3;
  const int S = (cpr + kItemChunks - 1) / kItemChunks;
  float* xs = smem_f;
  float* part = smem_f + K;
  grid_dependency_wait();
  grid_launch_dependents();
  if (p.norm_w) {
    float ss = 0.f;
    for (int i = tid; i < K; i += kGemvThreads) ss = fmaf(p.x[i], p.x[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < kGemvWarps; ++i) t += red[i];
    const float scale = 1.0f / sqrtf(t / static_cast<float>(K) + p.eps);
    for (int i = tid; i < K; i += kGemvThreads) xs[i] = p.x[i] * bf16_to_f32(p.norm_w[i]) * scale;
  } else {
    for (int i = tid * 4; i < K; i += kGemvThreads * 4)
      *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(p.x + i);
  }
  __syncthreads();
  const int items = nrows * NPHYS * S;
  for (int base = warp; base < items; base += kGemvWarps * kItemsInFlight) {
    uint4 w[kItemsInFlight][4];
    int cb[kItemsInFlight];
#pragma unroll
    for (int u = 0; u < kItemsInFlight; ++u) {
      const int item = base + kGemvWarps * u;
      const bool ok = item < items;
      int sp = 0, ph = 0, rl = 0;
      if (ok) {
        sp = item % S;
        const int t = item / S;
        ph = (NPHYS == 2) ? (t & 1) : 0;
        rl = (NPHYS == 2) ? (t >> 1) : t;
      }
      const uint16_t* row = p.W + static_cast<size_t>(r0 + rl + ph * p.pair_offset) * K;
      cb[u] = sp * kItemChunks;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cb[u] + lane + kWarp * j;
        w[u][j] = (ok && c < cpr) ? ld_stream(row + static_cast<size_t>(c) * 8) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kItemsInFlight; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cb[u] + lane + kWarp * j;
        if (c < cpr) acc += dot8(w[u][j], xs + c * 8);
      }
      acc = warp_sum(acc);
      const int item = base + kGemvWarps * u;
      if (lane == 0 && item < items) part[item] = acc;
    }
  }
  __syncthreads();
  gemv_epilogue<EPI>(p, part, S, r0, nrows, tid, kGemvThreads, lane, warp, wv, wi, &last_flag, false);
}

// ---------------------------------------------------------------- GEMV launch
template <typename Kern, typename... Args>
static cudaError_t launch_ex(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// Pipeline shape of the bulk-copy GEMV: consumer warps per CTA, stage and
// ring bytes.  Defaults are set by configure_kernels (env overrides
// VVLI_GEMV_CONSUMER_WARPS, VVLI_GEMV_STAGE_BYTES, VVLI_GEMV_RING_BYTES).
static int g_consumer_warps = 16;
static int g_stage_target = 65536;
static int g_ring_budget = 196608;

template <int EPI, int MAXC, bool ILP2>
static cudaError_t launch_tma(const GemvParams& p, int grid, size_t smem, cudaStream_t s, bool pdl) {
  return launch_ex(gemv_tma_kernel<EPI, MAXC, ILP2>, dim3(grid), dim3((g_consumer_warps + 1) * kWarp), smem, s, pdl,
                   p);
}

template <int EPI>
static cudaError_t launch_tma_variant(const GemvParams& p, int grid, size_t smem, cudaStream_t s, bool pdl) {
  if (p.cpl <= 4) return launch_tma<EPI, 4, true>(p, grid, smem, s, pdl);
  return launch_tma<EPI, 8, false>(p, grid, smem, s, pdl);
}

cudaError_t launch_gemv(int epi, GemvParams p, int sm_count, cudaStream_t s, bool pdl) {
  const int nphys = epi == EPI_SILU_MUL ? 2 : 1;
  const int cpr = p.K / 8;
  const size_t row_bytes = static_cast<size_t>(p.K) * 2;
  int S = 1;
  while (S < g_consumer_warps && S * 128 < cpr) S *= 2;  // S divides the consumer warp count
  const int SZ = (cpr + S - 1) / S;
  const int cpl = (SZ + kWarp - 1) / kWarp;
  if (cpl <= 8 && row_bytes * nphys <= 65536) {
    const int grid = p.N < sm_count ? p.N : sm_count;
    // Rows per stage: enough (row, split) pairs for every consumer warp (two
    // each when it interleaves two rows), within the stage budget.
    const int want_pairs = g_consumer_warps * (cpl <= 4 ? 2 : 1);
    int R = (want_pairs + S * nphys - 1) / (S * nphys);
    while (R > 1 && R * row_bytes * nphys > static_cast<size_t>(g_stage_target)) R /= 2;
    R = R < 1 ? 1 : R;
    p.S = S;
    p.SZ = SZ;
    p.cpl = cpl;
    p.R = R;
    p.stage_bytes = static_cast<int>(R * row_bytes * nphys);
    int nst = g_ring_budget / p.stage_bytes;
    p.nst = nst < 2 ? 2 : (nst > 8 ? 8 : nst);
    p.part_rows = (p.N + grid - 1) / grid + 1;
    const size_t part_floats = static_cast<size_t>(p.part_rows) * nphys * S;
    const size_t smem = static_cast<size_t>(p.nst) * p.stage_bytes + ((part_floats + 1) & ~size_t(1)) * 4 +
                        2 * p.nst * sizeof(uint64_t);
    switch (epi) {
      case EPI_PLAIN: return launch_tma_variant<EPI_PLAIN>(p, grid, smem, s, pdl);
      case EPI_SILU_MUL: return launch_tma_variant<EPI_SILU_MUL>(p, grid, smem, s, pdl);
      default: return launch_tma_variant<EPI_ARGMAX>(p, grid, smem, s, pdl);
    }
  }
  const int grid = p.N < 2 * sm_count ? p.N : 2 * sm_count;
  const int Sst = (cpr + kItemChunks - 1) / kItemChunks;
  const size_t rows = (static_cast<size_t>(p.N) + grid - 1) / grid + 1;
  const size_t smem = static_cast<size_t>(p.K) * 4 + rows * nphys * Sst * 4;
  switch (epi) {
    case EPI_PLAIN: return launch_ex(gemv_stream_kernel<EPI_PLAIN>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
    case EPI_SILU_MUL:
      return launch_ex(gemv_stream_kernel<EPI_SILU_MUL>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
    default: return launch_ex(gemv_stream_kernel<EPI_ARGMAX>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
  }
}

// ---------------------------------------------------------------- attention (decode)
// computeAttentionInto (src/llm.zig:1302-1335) for one token over the paged
// fp32 KV cache.  CTA (g, s) serves kv head g and the pages s, s + A,
// s + 2A, ... of positions 0..pos, where A = min(gridDim.y, pages) CTAs are
// active.  It rotates its group's q heads; the CTA holding the last page
// rotates the new k and writes k and v at `pos`.  Per page: q.k/sqrt(d)
// scores in shared memory (LP lanes per position, 128-bit loads), an online
// softmax (running max and sum per head), and P.V with one (head, dim) pair
// per thread.  The last CTA of a kv head merges the A partial (o, max, sum)
// triples with weights exp(m_s - M).
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / kWarp;
constexpr int kMaxAcc = 16;  // (group * head_dim) / 128 <= 16

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int last_flag;
  const int G = p.group, d = p.d;
  float* qs = sm;                  // [G][d]
  float* sc = qs + G * d;          // [G][kPage]
  float* mrun = sc + G * kPage;    // [G]
  float* lrun = mrun + G;          // [G]
  float* alpha = lrun + G;         // [G]
  float* wsplit = alpha + G;       // [G][splits] (combine)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = blockIdx.x, s = blockIdx.y;

  grid_dependency_wait();
  grid_launch_dependents();
  const int pos = p.st->pos;
  if (pos < 0 || pos >= p.st->max_seq) {
    if (g == 0 && s == 0 && tid == 0) p.st->err = 1;  // VVLI_ERR_CONTEXT_FULL
    return;
  }
  const int n_ctx = pos + 1;
  const int pages = (n_ctx + kPage - 1) / kPage;
  const int active = min(static_cast<int>(gridDim.y), pages);
  if (s >= active) return;
  const int half = d / 2;

  const float* qg = p.qkv + static_cast<size_t>(g) * G * d;
  for (int idx = tid; idx < G * half; idx += kAttnThreads) {
    const int hh = idx / half;
    rope_rotate(p.rope, pos, idx % half, d, qg + hh * d, qs + hh * d);
  }
  if ((pages - 1) % active == s) {
    const float* kn = p.qkv + static_cast<size_t>(p.nq) * d + static_cast<size_t>(g) * d;
    const float* vn = kn + static_cast<size_t>(p.nkv) * d;
    const size_t off = kv_off(p.page_table, pos, g, p.nkv, d);
    for (int i = tid; i < half; i += kAttnThreads) rope_rotate(p.rope, pos, i, d, kn, p.k_cache + off);
    for (int i = tid; i < d; i += kAttnThreads) p.v_cache[off + i] = vn[i];
  }
  for (int hh = tid; hh < G; hh += kAttnThreads) {
    mrun[hh] = -INFINITY;
    lrun[hh] = 0.f;
  }
  __syncthreads();

  // Score layout: EPL elements per lane (<= 32, multiple of 4), LP lanes per position.
  const int EPL = d < 32 ? d : 32;
  const int LP = d / EPL;
  const int PPW = kWarp / LP;                 // positions per warp per pass
  const int pp = lane / LP, qq = lane % LP;
  const int nacc = (G * d + kAttnThreads - 1) / kAttnThreads;
  float acc[kMaxAcc];
#pragma unroll
  for (int k = 0; k < kMaxAcc; ++k) acc[k] = 0.f;

  for (int page = s; page < pages; page += active) {
    const int t0 = page * kPage;
    const int n = min(kPage, n_ctx - t0);
    for (int base = warp * PPW; base < n; base += kAttnWarps * PPW) {
      const int i = base + pp;
      float kv[32];
      const bool ok = i < n && lane < PPW * LP;
      if (ok) {
        const float* kr = p.k_cache + kv_off(p.page_table, t0 + i, g, p.nkv, d) + qq * EPL;
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          if (e < EPL) *reinterpret_cast<float4*>(kv + e) = *reinterpret_cast<const float4*>(kr + e);
      }
      for (int hh = 0; hh < G; ++hh) {
        float dot = 0.f;
        if (ok) {
          const float* qh = qs + hh * d + qq * EPL;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < EPL) dot = fmaf(qh[e], kv[e], dot);
        }
        for (int o = 1; o < LP; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (ok && qq == 0) sc[hh * kPage + i] = dot * p.inv_sqrt_d;
      }
    }
    __syncthreads();
    for (int hh = warp; hh < G; hh += kAttnWarps) {  // online softmax (softmaxInPlace, src/llm.zig:1408-1419)
      float m = -INFINITY;
      for (int i = lane; i < n; i += kWarp) m = fmaxf(m, sc[hh * kPage + i]);
      m = warp_max(m);
      const float mnew = fmaxf(mrun[hh], m);
      float l = 0.f;
      for (int i = lane; i < n; i += kWarp) {
        const float e = expf(sc[hh * kPage + i] - mnew);
        sc[hh * kPage + i] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float a = expf(mrun[hh] - mnew);  // 0 on the first page (mrun = -inf)
        alpha[hh] = a;
        lrun[hh] = lrun[hh] * a + l;
        mrun[hh] = mnew;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMaxAcc; ++k) {
      const int idx = tid + k * kAttnThreads;
      if (k < nacc && idx < G * d) {
        const int hh = idx / d, e = idx % d;
        float a = acc[k] * alpha[hh];
        const float* vb = p.v_cache + e;
#pragma unroll 8
        for (int i = 0; i < n; ++i) a = fmaf(sc[hh * kPage + i], vb[kv_off(p.page_table, t0 + i, g, p.nkv, d)], a);
        acc[k] = a;
      }
    }
    __syncthreads();
  }

  // Partial (o, m, l) of this split.
#pragma unroll
  for (int k = 0; k < kMaxAcc; ++k) {
    const int idx = tid + k * kAttnThreads;
    if (k < nacc && idx < G * d) {
      const int hh = idx / d, e = idx % d;
      p.part[(static_cast<size_t>(g * G + hh) * p.splits + s) * (d + 2) + e] = acc[k];
    }
  }
  for (int hh = tid; hh < G; hh += kAttnThreads) {
    float* pp2 = p.part + (static_cast<size_t>(g * G + hh) * p.splits + s) * (d + 2);
    pp2[d] = mrun[hh];
    pp2[d + 1] = lrun[hh];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = atomicAdd(&p.counters[g], 1u) == static_cast<unsigned>(active) - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // Merge the active splits: weights exp(m_s - M) per head and split.
  for (int hh = warp; hh < G; hh += kAttnWarps) {
    const float* base = p.part + static_cast<size_t>(g * G + hh) * p.splits * (d + 2);
    float M = -INFINITY;
    for (int sp = lane; sp < active; sp += kWarp) M = fmaxf(M, __ldcg(base + sp * (d + 2) + d));
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < active; sp += kWarp) {
      const float w = expf(__ldcg(base + sp * (d + 2) + d) - M);
      wsplit[hh * p.splits + sp] = w;
      L = fmaf(__ldcg(base + sp * (d + 2) + d + 1), w, L);
    }
    L = warp_sum(L);
    if (lane == 0) alpha[hh] = 1.0f / L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * d; idx += kAttnThreads) {
    const int hh = idx / d, e = idx % d;
    const float* base = p.part + static_cast<size_t>(g * G + hh) * p.splits * (d + 2) + e;
    float o = 0.f;
    for (int sp = 0; sp < active; ++sp) o = fmaf(__ldcg(base + sp * (d + 2)), wsplit[hh * p.splits + sp], o);
    p.out[static_cast<size_t>(g * G + hh) * d + e] = o * alpha[hh];
  }
  if (tid == 0) p.counters[g] = 0;
}

size_t attention_smem_bytes(int group, int d, int splits) {
  return (static_cast<size_t>(group) * d + static_cast<size_t>(group) * kPage + 3 * group +
          static_cast<size_t>(group) * splits) * 4;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  return launch_ex(attention_decode_kernel, dim3(p.nkv, p.splits), dim3(kAttnThreads),
                   attention_smem_bytes(p.group, p.d, p.splits), s, pdl, p);
}

// ---------------------------------------------------------------- embedding
// copyEmbeddingToken (src/llm.zig:1373-1380) or forwardEmbedding's memcpy
// (src/llm.zig:716): x = table[seq_tokens[pos]] as fp32, or the caller's row.
__global__ void embed_kernel(const EmbedParams p) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int pos = p.st->pos;
  if (p.st->use_embedding) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.h; i += gridDim.x * blockDim.x) p.x[i] = p.emb_in[i];
    return;
  }
  int tok = (pos >= 0 && pos < p.st->max_seq) ? p.seq_tokens[pos] : 0;
  if (tok < 0 || tok >= p.vocab) {
    if (blockIdx.x == 0 && threadIdx.x == 0) p.st->err = 3;  // VVLI_ERR_INVALID_TOKEN
    tok = 0;
  }
  const uint16_t* row = p.table + static_cast<size_t>(tok) * p.h;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.h; i += gridDim.x * blockDim.x)
    p.x[i] = bf16_to_f32(row[i]);
}

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl) {
  const int blocks = (p.h + 255) / 256;
  return launch_ex(embed_kernel, dim3(blocks < 32 ? blocks : 32), dim3(256), 0, s, pdl, p);
}

// ---------------------------------------------------------------- tensor-parallel argmax
// Ranks hold increasing vocab shards; their (value, index) pairs are scanned
// in rank order with the llm.argmax rule.
__global__ void tp_argmax_finalize_kernel(const float* all_best, int ranks, StepState* st, int* seq_tokens) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float bv = all_best[0];
  int bi = __float_as_int(all_best[1]);
  for (int r = 1; r < ranks; ++r) {
    const float v = all_best[2 * r];
    const int i = __float_as_int(all_best[2 * r + 1]);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  publish_argmax(st, seq_tokens, bi);
}

cudaError_t launch_tp_argmax_finalize(const float* all_best, int ranks, StepState* st, int* seq_tokens,
                                      cudaStream_t s) {
  tp_argmax_finalize_kernel<<<1, 32, 0, s>>>(all_best, ranks, st, seq_tokens);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- transpose
__global__ void transpose_bf16_kernel(const uint16_t* src, uint16_t* dst, int rows, int cols) {
  __shared__ uint16_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[static_cast<size_t>(r) * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[static_cast<size_t>(c) * rows + r] = tile[threadIdx.x][i];
  }
}

cudaError_t launch_transpose_bf16(const uint16_t* src, uint16_t* dst, int rows, int cols, cudaStream_t s) {
  const dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose_bf16_kernel<<<grid, dim3(32, 8), 0, s>>>(src, dst, rows, cols);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- synthetic weights
__device__ uint16_t synth_value(uint64_t key, uint64_t idx) {
  constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
  uint32_t s = 0;
#pragma unroll
  for (uint64_t j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + (3 * idx + j + 1) * kGolden);
    s += static_cast<uint32_t>(h & 0xffff) + static_cast<uint32_t>((h >> 16) & 0xffff) +
         static_cast<uint32_t>((h >> 32) & 0xffff) + static_cast<uint32_t>(h >> 48);
  }
  const float z = __fmul_rn(__int2float_rn(static_cast<int>(s) - 393210), 1.0f / 65536.0f);
  return f32_to_bf16(__fmul_rn(z, 0.02f));
}

// Fills a rows x cols piece of a tensor whose full row length is src_ld,
// starting at (row0, col0) of the tensor.  kind 1 = norm weights (1.0).
__global__ void synth_fill_kernel(uint16_t* dst, uint64_t key, uint64_t rows, uint64_t cols, uint64_t src_ld,
                                  uint64_t row0, uint64_t col0, int kind) {
  const uint64_t total = rows * cols;
  for (uint64_t e = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = e / cols, c = e % cols;
    dst[e] = kind == 1 ? static_cast<uint16_t>(0x3F80) : synth_value(key, (row0 + r) * src_ld + col0 + c);
  }
}

cudaError_t launch_synth_fill(uint16_t* dst, uint64_t key, uint64_t rows, uint64_t cols, uint64_t src_ld,
                              uint64_t row0, uint64_t col0, int kind, cudaStream_t s) {
  const uint64_t total = rows * cols;
  uint64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks == 0) return cudaSuccess;
  synth_fill_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(dst, key, rows, cols, src_ld, row0, col0, kind);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- rotary pair rows
// dst row (head*d + 2j) <- src row (head*d + j); dst row (head*d + 2j + 1) <- src row (head*d + j + d/2).
__global__ void pair_rows_kernel(uint16_t* dst, const uint16_t* src, int rows, int K, int d) {
  const size_t total = static_cast<size_t>(rows) * K;
  for (size_t e = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(e / K), c = static_cast<int>(e % K);
    const int head = r / d, i = r % d;
    const int src_row = head * d + ((i & 1) ? i / 2 + d / 2 : i / 2);
    dst[e] = src[static_cast<size_t>(src_row) * K + c];
  }
}

// GGML block quantisation of bf16 rows, one thread per 32-weight block, with
// the published rules in plain fp32 steps (no contraction), so a host
// restatement with the same steps gives the same blocks:
//   Q8_0: d = amax / 127, q = roundf(x * (1 / d)) (halves away from zero);
//   Q4_0: d = m / -8 (m: the first weight of largest magnitude),
//         n = min(15, trunc(x * (1 / d) + 8.5)).
// Output rows use the device layout of kernels.h (quants, then fp16 scales).
__global__ void quantize_rows_kernel(const uint16_t* __restrict__ src, uint64_t rows, int K, int fmt,
                                     uint8_t* __restrict__ dst, int row_bytes) {
  const int nb = K / 32;
  const uint64_t total = rows * static_cast<uint64_t>(nb);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / nb;
    const int b = static_cast<int>(i % nb);
    const uint16_t* x = src + r * K + b * 32;
    uint8_t* row = dst + r * row_bytes;
    float v[32];
    float amax = 0.f, m = 0.f;
    for (int j = 0; j < 32; ++j) {
      v[j] = bf16_to_f32(x[j]);
      if (fabsf(v[j]) > amax) {
        amax = fabsf(v[j]);
        m = v[j];
      }
    }
    if (fmt == kFmtQ8) {
      const float d = __fdiv_rn(amax, 127.0f);
      const float inv = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      for (int j = 0; j < 32; ++j) {
        const float q = fminf(127.f, fmaxf(-127.f, roundf(__fmul_rn(v[j], inv))));
        row[b * 32 + j] = static_cast<uint8_t>(static_cast<int8_t>(q));
      }
      *reinterpret_cast<__half*>(row + K + 2 * b) = __float2half_rn(d);
    } else {
      const float d = __fdiv_rn(m, -8.0f);
      const float inv = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      uint8_t n[32];
      for (int j = 0; j < 32; ++j) {
        const float t = truncf(__fadd_rn(__fmul_rn(v[j], inv), 8.5f));
        n[j] = static_cast<uint8_t>(fminf(15.f, fmaxf(0.f, t)));
      }
      for (int j = 0; j < 16; ++j) row[b * 16 + j] = static_cast<uint8_t>(n[j] | (n[j + 16] << 4));
      *reinterpret_cast<__half*>(row + K / 2 + 2 * b) = __float2half_rn(d);
    }
  }
}

cudaError_t launch_quantize_rows(const uint16_t* src, uint64_t rows, int K, int fmt, uint8_t* dst, cudaStream_t s) {
  if (fmt != kFmtQ8 && fmt != kFmtQ4) return cudaErrorInvalidValue;
  const uint64_t blocks = rows * (K / 32);
  const unsigned grid = static_cast<unsigned>(std::min<uint64_t>((blocks + 255) / 256, 8192));
  quantize_rows_kernel<<<grid, 256, 0, s>>>(src, rows, K, fmt, dst, row_bytes_of(fmt, K));
  return cudaGetLastError();
}

cudaError_t launch_pair_rows(uint16_t* w, uint16_t* bias, uint16_t* tmp, int rows, int K, int d, cudaStream_t s) {
  cudaError_t e = cudaMemcpyAsync(tmp, w, static_cast<size_t>(rows) * K * 2, cudaMemcpyDeviceToDevice, s);
  if (e) return e;
  pair_rows_kernel<<<148 * 8, 256, 0, s>>>(w, tmp, rows, K, d);
  if ((e = cudaGetLastError())) return e;
  if (bias) {
    if ((e = cudaMemcpyAsync(tmp, bias, static_cast<size_t>(rows) * 2, cudaMemcpyDeviceToDevice, s))) return e;
    pair_rows_kernel<<<8, 256, 0, s>>>(bias, tmp, rows, 1, d);
    if ((e = cudaGetLastError())) return e;
  }
  return cudaSuccess;
}

template <typename Kern>
static cudaError_t allow_dynamic_smem(Kern k, int max_smem_optin) {
  // The opt-in limit covers static plus dynamic shared memory.
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k);
  if (e) return e;
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              max_smem_optin - static_cast<int>(fa.sharedSizeBytes));
}

static int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : fallback;
}

cudaError_t configure_kernels(int max_smem_optin) {
  // Clamped to what the kernel's thread bound and shared memory allow.
  // 8 or 16: every k-split count (1, 2, 4, 8) must divide the consumer warps.
  g_consumer_warps = env_int("VVLI_GEMV_CONSUMER_WARPS", 16) <= 8 ? 8 : kTmaMaxConsumerWarps;
  g_stage_target = std::min(65536, std::max(4096, env_int("VVLI_GEMV_STAGE_BYTES", 65536)));
  g_ring_budget = std::min(200 * 1024, std::max(2 * g_stage_target, env_int("VVLI_GEMV_RING_BYTES", 196608)));
  cudaError_t e;
#define VVLI_ALLOW(k) \
  if ((e = allow_dynamic_smem(k, max_smem_optin))) return e;
  VVLI_ALLOW((gemv_tma_kernel<EPI_PLAIN, 4, true>));
  VVLI_ALLOW((gemv_tma_kernel<EPI_PLAIN, 8, false>));
  VVLI_ALLOW((gemv_tma_kernel<EPI_SILU_MUL, 4, true>));
  VVLI_ALLOW((gemv_tma_kernel<EPI_SILU_MUL, 8, false>));
  VVLI_ALLOW((gemv_tma_kernel<EPI_ARGMAX, 4, true>));
  VVLI_ALLOW((gemv_tma_kernel<EPI_ARGMAX, 8, false>));
  VVLI_ALLOW(gemv_stream_kernel<EPI_PLAIN>);
  VVLI_ALLOW(gemv_stream_kernel<EPI_SILU_MUL>);
  VVLI_ALLOW(gemv_stream_kernel<EPI_ARGMAX>);
  VVLI_ALLOW(attention_decode_kernel);
#undef VVLI_ALLOW
  return cudaSuccess;
}

}  // namespace vvli
