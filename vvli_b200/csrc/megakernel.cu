// megakernel.cu - one persistent, cooperative kernel per decode step.
//
// The step of Runner.forwardCurrentEmbedding (src/llm.zig:720-766) is a list
// of phases: embed, then per layer q|k|v GEMV, attention, o_proj (+residual),
// gate|up (silu*mul), down_proj (+residual), and the LM head with argmax.
// One CTA per SM runs them all:
//   * warp 16 is the producer.  It walks every GEMV phase of the step in
//     order and streams this CTA's rows of each weight matrix through a ring
//     of shared-memory stages with cp.async.bulk.  Weights do not depend on
//     activations, so it never waits for a phase boundary: while the
//     consumers run attention or wait at a grid barrier, the next matrix is
//     already arriving.  HBM stays busy across the whole step.
//   * warps 0-15 consume: they wait at a grid barrier for the phase input,
//     run the phase (GEMV rows from the ring, or attention items), write
//     their outputs and meet at the next grid barrier.
// All cross-CTA data is read through L2 (ld.global.cg).  Every wait (ring
// stages, grid barrier, tensor-parallel flags) is bounded and reports
// VVLI_ERR_TIMEOUT in StepState.err.  Under tensor parallelism the
// all-reduce after o_proj and down_proj is fused into their epilogues: each
// CTA stores its partial rows into every peer's receive buffer over NVLink,
// raises a flag on each peer, waits for the peers' flags for its rows and
// adds the partials in rank order.
#include <cuda_fp16.h>

#include <algorithm>

#include "device_fns.cuh"
#include "kernels.h"

namespace vvli {

constexpr int kCW = kMegaConsumerWarps;
constexpr int kNC = kCW * kWarp;


// ---------------------------------------------------------------- sync helpers
VVLI_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
VVLI_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
VVLI_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier of the consumer threads of every CTA (the producers never
// join).  A 64-bit counter only grows: every CTA adds one per barrier with a
// fire-and-forget release reduction, and barrier k of step `epoch` is passed
// once the counter reaches (epoch * barriers_per_step + k + 1) * CTAs.  No
// CTA waits for its own atomic to return and nothing is reset, so a barrier
// costs about one memory round trip.  Split in two so a CTA can issue work
// for its next phase between arriving and waiting.  The wait is bounded.
VVLI_DEV uint64_t ld_acquire_gpu_u64(const unsigned long long* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ void grid_arrive(unsigned long long* bar) {
  named_barrier(1, kNC);
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ bool grid_wait(const unsigned long long* bar, uint64_t target, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (ld_acquire_gpu_u64(bar) < target) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 0; ld_acquire_gpu_u64(bar) < target; ++it) {
        if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
          atomicExch(err, kErrTimeout);
          ok = 0;
          break;
        }
      }
    }
  }
  named_barrier(1, kNC);
  return ok != 0;
}

VVLI_DEV void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// The fp32 half of *w once its high half is `epoch` (a peer's 8-byte store
// over NVLink); bounded: on timeout VVLI_ERR_TIMEOUT and 0.
VVLI_DEV float word_of_epoch(const unsigned long long* w, unsigned epoch, int* err) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
    if (static_cast<unsigned>(v >> 32) == epoch) return __uint_as_float(static_cast<unsigned>(v));
    if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
      atomicExch(err, kErrTimeout);
      return 0.f;
    }
  }
}

// Bounded wait until *flag == value (a peer's release store over NVLink).
VVLI_DEV bool wait_flag_sys(const unsigned* flag, unsigned value, int* err) {
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_sys(flag) != value) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicExch(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// First row of CTA b's range of N rows; ranges start at multiples of `align`.
VVLI_DEV int cta_row(int N, int b, int align) {
  if (b >= static_cast<int>(gridDim.x)) return N;
  const int r = static_cast<int>((static_cast<long long>(b) * N) / gridDim.x);
  return r - r % align;
}
VVLI_DEV int cta_row0(int N) { return cta_row(N, blockIdx.x, 1); }
VVLI_DEV int cta_row1(int N) { return cta_row(N, blockIdx.x + 1, 1); }

// Block-wide sum over the consumer threads, result on thread 0.
__device__ float consumer_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  named_barrier(1, kNC);
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kCW; ++i) t += red[i];
  named_barrier(1, kNC);
  return t;
}

// Optional timeline: per phase and CTA, [0] consumers start, [1] inputs
// loaded, [2] rows consumed, [3] outputs written, [4] grid barrier passed,
// [5] producer issued the phase's first stage.
VVLI_DEV void trace_mark(const MegaParams& P, int f, int k) {
  if (P.trace) P.trace[(static_cast<size_t>(f) * gridDim.x + blockIdx.x) * 6 + k] = global_timer_ns();
}

// Fixed-point accumulators of the fused down_proj (see MegaPhase::acc_out):
// v -> round(v * 2^32) as a 64-bit integer; integer sums do not depend on
// the order of the adds, so the result is the same on every run.
VVLI_DEV long long to_fixed(float v) {
  const double t = static_cast<double>(v) * kAccScale;
  return __double2ll_rn(fmin(fmax(t, -9.0e18), 9.0e18));
}
VVLI_DEV float from_fixed(long long v) { return static_cast<float>(static_cast<double>(v) * (1.0 / kAccScale)); }

// ---------------------------------------------------------------- producer
// Cursor over this CTA's stages of every GEMV phase of the step, in order.
struct StageCursor {
  int f = -1, i = 0, nstages = 0, r0 = 0, nrows = 0;
  __device__ bool next(const MegaParams& P) {  // moves to the next stage; false at the end
    ++i;
    while (i >= nstages) {
      if (++f >= P.nphases) return false;
      const MegaPhase& ph = P.phases[f];
      if (ph.kind != MK_GEMV) continue;
      r0 = cta_row(ph.N, blockIdx.x, ph.row_align);
      nrows = cta_row(ph.N, blockIdx.x + 1, ph.row_align) - r0;
      nstages = (nrows + ph.R - 1) / ph.R;
      i = 0;
    }
    return true;
  }
};

__device__ void mega_producer(const MegaParams& P, uint8_t* ring, uint64_t* full, uint64_t* empty, int* err) {
  StageCursor cur;  // i = 0 >= nstages = 0: the first next() loads the first GEMV phase
  uint32_t gi = 0;
  int last_f = -1;
  while (cur.next(P)) {
    const MegaPhase& ph = P.phases[cur.f];
    if (cur.f != last_f) {
      trace_mark(P, cur.f, 5);
      last_f = cur.f;
    }
    const uint32_t slot = gi % P.nst;
    if (gi >= static_cast<uint32_t>(P.nst) && !mbar_wait(&empty[slot], ((gi / P.nst) - 1) & 1, err)) break;
    const size_t row_bytes = static_cast<size_t>(ph.row_bytes);
    const int rows_here = min(ph.R, cur.nrows - cur.i * ph.R);
    const uint32_t bytes = static_cast<uint32_t>(rows_here * row_bytes);
    mbar_arrive_expect_tx(&full[slot], bytes * ph.nphys);
    for (int q = 0; q < ph.nphys; ++q)
      bulk_g2s(ring + static_cast<size_t>(slot) * P.slot_bytes + q * ph.R * row_bytes,
               reinterpret_cast<const uint8_t*>(ph.W) +
                   static_cast<size_t>(cur.r0 + cur.i * ph.R + q * ph.pair_offset) * row_bytes,
               bytes, &full[slot]);
    ++gi;
  }
  // Every issued copy lands before the CTA exits.
  const uint32_t first = gi > static_cast<uint32_t>(P.nst) ? gi - P.nst : 0;
  for (uint32_t i = first; i < gi; ++i) mbar_wait(&full[i % P.nst], (i / P.nst) & 1, err);
}

// ---------------------------------------------------------------- weight formats
// A consumer lane reads 16-byte chunks of a row: 8 bf16 weights, 16 Q8_0
// quants (half a block) or 32 Q4_0 nibbles (a whole block), and holds the
// matching input elements in registers (32 floats in every format).
template <int FMT>
struct WFmt {
  static constexpr int EPC = FMT == kFmtBF16 ? 8 : FMT == kFmtQ8 ? 16 : 32;  // weights per chunk
  static constexpr int MAXC = 32 / EPC;                                      // chunks per lane
};

// Byte k of `t` as a float: the byte becomes the mantissa of 2^23 + byte, and
// the bias is subtracted exactly (one permute and one add per weight, on the
// fp32 pipe).
VVLI_DEV float byte_as_float(uint32_t t, int k, float bias) {
  return __int_as_float(__byte_perm(t, 0x4B000000u, 0x7540u + k)) - bias;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue, two lanes of
// fp32 arithmetic, each rounded like the scalar instruction).
typedef unsigned long long f32x2;
VVLI_DEV f32x2 pack_f2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
VVLI_DEV f32x2 pack_u2(uint32_t a, uint32_t b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
VVLI_DEV f32x2 fma_f2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
VVLI_DEV f32x2 add_f2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
VVLI_DEV float sum_f2(f32x2 a) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a));
  return lo + hi;
}

// Bytes k and k + 1 of `t` as the pair (2^23 + byte) - bias, exactly.
VVLI_DEV f32x2 bytes_as_f2(uint32_t t, int k, f32x2 neg_bias) {
  return add_f2(pack_u2(__byte_perm(t, 0x4B000000u, 0x7540u + k), __byte_perm(t, 0x4B000000u, 0x7540u + k + 1)),
                neg_bias);
}

// sum_i q_i * x_i over the 16 int8 quants of a chunk (x ^ 0x80 maps q to
// q + 128); x2 holds the 16 inputs as 8 pairs.
VVLI_DEV float dot16_q8(uint4 w, const f32x2* x2) {
  const uint32_t wd[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
  const f32x2 nb = pack_f2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  f32x2 acc[2] = {0ull, 0ull};  // two independent chains
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    acc[0] = fma_f2(bytes_as_f2(wd[m], 0, nb), x2[2 * m], acc[0]);
    acc[1] = fma_f2(bytes_as_f2(wd[m], 2, nb), x2[2 * m + 1], acc[1]);
  }
  return sum_f2(add_f2(acc[0], acc[1]));
}

// sum_i (n_i - 8) * x_i over the 32 nibbles of a Q4_0 block: byte j holds
// weight j (low nibble) and weight j + 16 (high nibble); x2 holds 16 pairs.
VVLI_DEV float dot32_q4(uint4 w, const f32x2* x2) {
  const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
  const f32x2 nb = pack_f2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
  f32x2 acc[4] = {0ull, 0ull, 0ull, 0ull};  // four independent chains
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t lo = wd[m] & 0x0F0F0F0Fu, hi = (wd[m] >> 4) & 0x0F0F0F0Fu;
    acc[0] = fma_f2(bytes_as_f2(lo, 0, nb), x2[2 * m], acc[0]);
    acc[1] = fma_f2(bytes_as_f2(lo, 2, nb), x2[2 * m + 1], acc[1]);
    acc[2] = fma_f2(bytes_as_f2(hi, 0, nb), x2[8 + 2 * m], acc[2]);
    acc[3] = fma_f2(bytes_as_f2(hi, 2, nb), x2[8 + 2 * m + 1], acc[3]);
  }
  return sum_f2(add_f2(add_f2(acc[0], acc[1]), add_f2(acc[2], acc[3])));
}

VVLI_DEV float half_at(const uint8_t* p) { return __half2float(*reinterpret_cast<const __half*>(p)); }

// ---------------------------------------------------------------- GEMV phase (consumers)
template <int MAXC, int FMT>
__device__ void mega_gemv(const MegaParams& P, const MegaPhase& ph, uint8_t* ring, float* part, uint64_t* full,
                          uint64_t* empty, uint32_t& gi, float* red, float* wv, int* wi, int* err, unsigned epoch0,
                          int f, float* ffs, float* xres, float4* xs) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int EPC = WFmt<FMT>::EPC;
  const int K = ph.K, S = ph.S, R = ph.R, nphys = ph.nphys;
  const int r0 = cta_row(ph.N, blockIdx.x, ph.row_align);
  const int nrows = cta_row(ph.N, blockIdx.x + 1, ph.row_align) - r0;
  const int nstages = (nrows + R - 1) / R;
  const size_t row_bytes = static_cast<size_t>(ph.row_bytes);
  const int qbytes = quant_bytes(FMT, K);  // Q formats: the scales follow the quants
  // Inputs: this warp's slice of x times the norm weights.  RMSNorm's scale
  // is one scalar, so it multiplies the finished dot products in the
  // epilogue: W.(x*w*s) = s * W.(x*w).  Warp 0 sums the per-CTA squares
  // meanwhile; nothing waits for it before the rows are consumed.
  const int cpr = K / EPC;
  const int split = warp % S;
  const int cbeg = split * ph.SZ;
  const int cend = min(cpr, cbeg + ph.SZ);
  float ssq_lane = 0.f;
  if (ph.norm_w && warp == 0 && !ph.acc_in) {
    float v[8];  // up to 256 CTAs, all loads in flight together
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int b = lane + k * kWarp;
      v[k] = b < static_cast<int>(gridDim.x) ? __ldcg(P.ssq + b) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) ssq_lane += v[k];
  }
  // With S <= 2 splits, eight or more warps hold each slice of x: the CTA
  // then reads x from L2 once into shared memory and the warps take their
  // slices there (measured: Qwen2.5-0.5B's prologue 6.2 -> 3.8 us; with S = 4
  // the Llama-3-8B step was slower).
  // Block-quantised phases stage x too: a lane's 16 or 32 inputs lie 64 or
  // 128 bytes apart from its neighbours', a pattern that serves L2 poorly.
  // Shared memory holds chunk c's float4 q at c * P4 + (q ^ sw(c)), so the 8
  // lanes of one 128-bit access hit different banks.
  constexpr int P4 = EPC / 4;  // float4s per chunk
  const bool staged = (S <= 2 || FMT != kFmtBF16) && !ph.acc_in && K <= P.xstage_floats;
  auto sw = [](int c) { return P4 == 8 ? (c & 7) : P4 == 4 ? ((c >> 1) & 3) : ((c >> 2) & 1); };
  if (staged) {
    const float4* x4 = reinterpret_cast<const float4*>(ph.x);
    for (int i = tid; i < K / 4; i += kNC) {
      const int c = i / P4, q = i % P4;
      xs[c * P4 + (q ^ sw(c))] = __ldcg(x4 + i);
    }
    named_barrier(1, kNC);
  }
  // bf16: the inputs as floats; Q formats: as fp32 pairs for the f32x2 dots.
  constexpr bool kBf = FMT == kFmtBF16;
  float xr[kBf ? MAXC : 1][kBf ? EPC : 1];
  f32x2 x2[kBf ? 1 : MAXC][kBf ? 1 : EPC / 2];
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int c = cbeg + lane + kWarp * j;
    const bool live = j < ph.cpl && c < cend;
    if constexpr (kBf) {
      if (live) {
#pragma unroll
        for (int q = 0; q < EPC / 4; ++q) {
          const float4 a = staged ? xs[c * P4 + (q ^ sw(c))] : __ldcg(reinterpret_cast<const float4*>(ph.x + c * EPC + 4 * q));
          xr[j][4 * q] = a.x, xr[j][4 * q + 1] = a.y, xr[j][4 * q + 2] = a.z, xr[j][4 * q + 3] = a.w;
        }
        if (ph.acc_in) {  // the previous layer's down_proj, still in its fixed-point accumulator
          const longlong2* ap = reinterpret_cast<const longlong2*>(ph.acc_in + c * 8);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const longlong2 t = __ldcg(ap + q);
            xr[j][2 * q] = xr[j][2 * q] + from_fixed(t.x);
            xr[j][2 * q + 1] = xr[j][2 * q + 1] + from_fixed(t.y);
          }
          if (warp < S) {  // warps 0..S-1 hold each slice of x once: the sum of squares here
#pragma unroll
            for (int e = 0; e < 8; ++e) ssq_lane = fmaf(xr[j][e], xr[j][e], ssq_lane);
          }
        }
        if (ph.norm_w) {
          const uint4 wn = *reinterpret_cast<const uint4*>(ph.norm_w + c * EPC);
          const float nw[8] = {bf16_lo(wn.x), bf16_hi(wn.x), bf16_lo(wn.y), bf16_hi(wn.y),
                               bf16_lo(wn.z), bf16_hi(wn.z), bf16_lo(wn.w), bf16_hi(wn.w)};
#pragma unroll
          for (int e = 0; e < 8; ++e) xr[j][e] = xr[j][e] * nw[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPC; ++e) xr[j][e] = 0.f;
      }
    } else {
      if (live) {
#pragma unroll
        for (int q = 0; q < EPC / 4; ++q) {
          const float4 a = staged ? xs[c * P4 + (q ^ sw(c))] : __ldcg(reinterpret_cast<const float4*>(ph.x + c * EPC + 4 * q));
          x2[j][2 * q] = pack_f2(a.x, a.y);
          x2[j][2 * q + 1] = pack_f2(a.z, a.w);
        }
        if (ph.norm_w) {  // x * w, rounded once per element like the scalar product
#pragma unroll
          for (int q = 0; q < EPC / 8; ++q) {
            const uint4 wn = *reinterpret_cast<const uint4*>(ph.norm_w + c * EPC + 8 * q);
            const uint32_t ww[4] = {wn.x, wn.y, wn.z, wn.w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
              x2[j][4 * q + t] = fma_f2(x2[j][4 * q + t], pack_f2(bf16_lo(ww[t]), bf16_hi(ww[t])), 0ull);
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPC / 2; ++e) x2[j][e] = 0ull;
      }
    }
  }
  auto row_dot = [&](const uint8_t* rp) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      const int c = cbeg + lane + kWarp * j;
      if (j < ph.cpl && c < cend) {
        const uint4 w = *reinterpret_cast<const uint4*>(rp + c * 16);
        if constexpr (FMT == kFmtBF16) {
          acc += dot8(w, xr[j]);
        } else if constexpr (FMT == kFmtQ8) {  // weight = d * q, d shared by the two chunks of a block
          acc = fmaf(dot16_q8(w, x2[j]), half_at(rp + qbytes + (c >> 1) * 2), acc);
        } else {  // weight = d * (n - 8)
          acc = fmaf(dot32_q4(w, x2[j]), half_at(rp + qbytes + c * 2), acc);
        }
      }
    }
    return acc;
  };
  if (P.hidden && ph.acc_in && ph.hidden_layer >= 0) {  // debugging: the finished layer's output
    for (int r = cta_row0(K) + tid; r < cta_row1(K); r += kNC)
      P.hidden[static_cast<size_t>(ph.hidden_layer) * K + r] = __ldcg(ph.x + r) + from_fixed(__ldcg(ph.acc_in + r));
  }
  if (tid == 0) trace_mark(P, f, 1);
  if (ph.epi == ME_QKV && P.phases[f + 1].kind == MK_ATTN && tid < 4) {
    // This CTA's attention item of the next phase: warm L2 with its K and V
    // pages of positions before `pos` (its own token is written later).
    const MegaPhase& at = P.phases[f + 1];
    const int pos = P.st->pos;
    const int pages = (pos + 1 + kPage - 1) / kPage;
    const int A = min(P.splits, pages);
    if (static_cast<int>(blockIdx.x) < P.nkv * A) {
      const int g = blockIdx.x / A, s0 = blockIdx.x % A;
      int k = 0;
      for (int page = s0; page < pages; page += A, ++k) {
        if ((k & 3) != tid) continue;
        const size_t off = kv_off(P.page_table, page * kPage, g, P.nkv, P.d);
        const uint32_t bytes = static_cast<uint32_t>(kPage * P.d * 4);
        prefetch_l2_bulk(at.k_cache + off, bytes);
        prefetch_l2_bulk(at.v_cache + off, bytes);
      }
    }
  }
  const int pairs = R * nphys * S;
  for (int i = 0; i < nstages; ++i, ++gi) {
    const uint32_t slot = gi % P.nst;
    if (!mbar_wait(&full[slot], (gi / P.nst) & 1, err)) break;
    const int rows_here = min(R, nrows - i * R);
    const uint8_t* stg = ring + static_cast<size_t>(slot) * P.slot_bytes;
    for (int pi = warp; pi < pairs; pi += 2 * kCW) {
      const int pb = pi + kCW;
      const int ta = pi / S, tb = pb / S;
      const int pha = nphys == 2 ? (ta & 1) : 0, rowa = nphys == 2 ? (ta >> 1) : ta;
      const int phb = nphys == 2 ? (tb & 1) : 0, rowb = nphys == 2 ? (tb >> 1) : tb;
      const bool va = rowa < rows_here;
      const bool vb = pb < pairs && rowb < rows_here;
      const float a = va ? row_dot(stg + pha * R * row_bytes + rowa * row_bytes) : 0.f;
      const float b = vb ? row_dot(stg + phb * R * row_bytes + rowb * row_bytes) : 0.f;
      const float v = warp_sum2(a, b, lane);
      if (lane == 0 && va) part[((i * R + rowa) * nphys + pha) * S + split] = v;
      if (lane == 16 && vb) part[((i * R + rowb) * nphys + phb) * S + split] = v;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  __shared__ float scale_sh;
  if (ph.acc_in && ph.norm_w) {
    const float t = warp_sum(ssq_lane);
    if (lane == 0 && warp < S) red[warp] = t;
    named_barrier(1, kNC);
    if (tid == 0) {
      float tt = 0.f;
      for (int w = 0; w < S; ++w) tt += red[w];
      scale_sh = 1.0f / sqrtf(tt / static_cast<float>(K) + P.eps);
    }
  } else if (warp == 0) {
    const float t = warp_sum(ssq_lane);
    if (lane == 0) scale_sh = ph.norm_w ? 1.0f / sqrtf(t / static_cast<float>(K) + P.eps) : 1.0f;
  }
  named_barrier(1, kNC);
  if (tid == 0) trace_mark(P, f, 2);
  const float scale = scale_sh;

  // ---- epilogue
  if (ph.epi == ME_QKV) {
    // q|k|v rows with the bias (src/llm.zig:738-740); q and k rotated
    // (applyRoPE, src/llm.zig:742-743; rows hold rotary pairs side by side);
    // k and v go straight into the KV cache at `pos` (src/llm.zig:744-745).
    const int pos = P.st->pos;
    const bool pos_ok = pos >= 0 && pos < P.st->max_seq;
    const int d = P.d, qr = P.nq * d, kr = P.nkv * d;
    for (int pr = tid; pr < nrows / 2; pr += kNC) {
      const int ra = r0 + 2 * pr;
      float a = 0.f, b = 0.f;
      for (int s = 0; s < S; ++s) {
        a += part[(2 * pr) * S + s];
        b += part[(2 * pr + 1) * S + s];
      }
      a *= scale;
      b *= scale;
      if (ph.bias) {
        a = a + bf16_to_f32(ph.bias[ra]);
        b = b + bf16_to_f32(ph.bias[ra + 1]);
      }
      if (ra < qr + kr) {
        const int di = ra % d;  // pair j = di / 2 of the head, frequency index 2j
        const float ang = static_cast<float>(pos) * rope_inv_freq(P.rope, di, d);
        float sn, cs;
        sincosf(ang, &sn, &cs);
        const float x0 = a, x1 = b;
        a = x0 * cs - x1 * sn;
        b = x0 * sn + x1 * cs;
      }
      if (ra < qr) {
        ph.y[ra] = a;
        ph.y[ra + 1] = b;
      } else if (pos_ok) {
        const bool is_k = ra < qr + kr;
        const int rel = is_k ? ra - qr : ra - qr - kr;
        const size_t off = kv_off(P.page_table, pos, rel / d, P.nkv, d) + rel % d;
        float* cache = is_k ? ph.k_cache : ph.v_cache;
        cache[off] = a;
        cache[off + 1] = b;
      }
    }
    return;
  }
  if (ph.epi == ME_STORE || ph.epi == ME_SILU) {
    for (int rl = tid; rl < nrows; rl += kNC) {
      const int r = r0 + rl;
      float a;
      if (ph.epi == ME_SILU) {
        float g = 0.f, u = 0.f;
        for (int s = 0; s < S; ++s) {
          g += part[(2 * rl) * S + s];
          u += part[(2 * rl + 1) * S + s];
        }
        g *= scale;
        u *= scale;
        a = (g / (1.0f + expf(-g))) * u;  // siluMulInto, src/llm.zig:1382-1387
      } else {
        a = 0.f;
        for (int s = 0; s < S; ++s) a += part[rl * S + s];
        a *= scale;
        if (ph.bias) a = a + bf16_to_f32(ph.bias[r]);
      }
      if (ph.ff_smem) {
        ffs[rl] = a;  // read by the ME_AXPY phase that follows in this CTA
      } else {
        ph.y[r] = a;
      }
    }
    return;
  }
  if (ph.epi == ME_RESIDUAL) {
    // x[r] = x[r] + W.x (addInto, src/llm.zig:757, 765); under tensor
    // parallelism the partials of all ranks are exchanged first.
    float ss = 0.f;
    if (P.tp > 1) {
      // Flag values grow by one per residual phase: (step * 2L + index + 1).
      const unsigned epoch = epoch0 * static_cast<unsigned>(P.n_ar) + static_cast<unsigned>(ph.ar_index) + 1u;
      const int par = ph.ar_index & 1;
      const size_t slot_off = static_cast<size_t>(par) * P.tp * P.h;
      // Each partial row travels as one 8-byte word (epoch, fp32 bits) to
      // every rank; a word is stored and loaded whole, so the receiver
      // polls the data itself: no fence and no separate flag.  The thread
      // that sends row rl is the one that sums it, and the same rows on
      // every rank belong to the same CTA index.
      for (int rl = tid; rl < nrows; rl += kNC) {
        float a = 0.f;
        for (int s = 0; s < S; ++s) a += part[rl * S + s];
        const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(a);
        for (int q = 0; q < P.tp; ++q) st_relaxed_sys_u64(P.peer_recv[q] + slot_off + static_cast<size_t>(P.rank) * P.h + r0 + rl, w);
      }
      const unsigned long long* recv = P.peer_recv[P.rank] + slot_off;
      for (int rl = tid; rl < nrows; rl += kNC) {
        const int r = r0 + rl;
        float a = 0.f;
        for (int q = 0; q < P.tp; ++q) a += word_of_epoch(recv + static_cast<size_t>(q) * P.h + r, epoch, err);
        const float xn = __ldcg(P.x + r) + a;
        P.x[r] = xn;
        ss = fmaf(xn, xn, ss);
        if (P.hidden && (ph.ar_index & 1)) P.hidden[static_cast<size_t>(ph.layer) * P.h + r] = xn;
      }
    } else {
      for (int rl = tid; rl < nrows; rl += kNC) {
        const int r = r0 + rl;
        float a = 0.f;
        for (int s = 0; s < S; ++s) a += part[rl * S + s];
        float xo = P.xres ? xres[rl] : __ldcg(P.x + r);  // this CTA's own rows of x
        if (ph.acc_fold) {  // the previous layer's down_proj joins the residual stream here
          xo = xo + from_fixed(__ldcg(ph.acc_fold + r));
          ph.acc_fold[r] = 0;
        }
        const float xn = xo + a;
        P.x[r] = xn;
        if (P.xres) xres[rl] = xn;
        ss = fmaf(xn, xn, ss);
        if (P.hidden && (ph.ar_index & 1)) P.hidden[static_cast<size_t>(ph.layer) * P.h + r] = xn;
      }
    }
    ss = consumer_sum(ss, red);
    if (tid == 0) P.ssq[blockIdx.x] = ss;
    return;
  }
  // ME_ARGMAX: logits and llm.argmax (src/llm.zig:778-789).
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (int rl = tid; rl < nrows; rl += kNC) {
    const int r = r0 + rl;
    float a = 0.f;
    for (int s = 0; s < S; ++s) a += part[rl * S + s];
    a *= scale;
    ph.y[r] = a;
    if (better(a, r + P.row_base, best_v, best_i)) {
      best_v = a;
      best_i = r + P.row_base;
    }
  }
  warp_argmax(best_v, best_i);
  if (lane == 0) {
    wv[warp] = best_v;
    wi[warp] = best_i;
  }
  named_barrier(1, kNC);
  if (tid == 0) {
    float bv = wv[0];
    int bi = wi[0];
    for (int i = 1; i < kCW; ++i)
      if (better(wv[i], wi[i], bv, bi)) {
        bv = wv[i];
        bi = wi[i];
      }
    P.amax_val[blockIdx.x] = bv;
    P.amax_idx[blockIdx.x] = bi;
    __threadfence();
    if (atomicAdd(P.amax_counter, 1u) == gridDim.x - 1) {
      __threadfence();
      float gv = __ldcg(P.amax_val);
      int gidx = __ldcg(P.amax_idx);
      for (unsigned b = 1; b < gridDim.x; ++b) {
        const float v = __ldcg(P.amax_val + b);
        const int i = __ldcg(P.amax_idx + b);
        if (better(v, i, gv, gidx)) {
          gv = v;
          gidx = i;
        }
      }
      *P.amax_counter = 0;
      if (P.tp > 1) {
        // Exchange (value, index) with every rank; ranks hold increasing vocab shards.
        const unsigned epoch = epoch0 + 1u;
        for (int q = 0; q < P.tp; ++q) {
          P.peer_best[q][2 * P.rank] = gv;
          P.peer_best[q][2 * P.rank + 1] = __int_as_float(gidx);
        }
        __threadfence_system();
        for (int q = 0; q < P.tp; ++q) st_release_sys(P.peer_best_flag[q] + P.rank, epoch);
        float bv2 = 0.f;
        int bi2 = 0;
        for (int q = 0; q < P.tp; ++q) {
          wait_flag_sys(P.peer_best_flag[P.rank] + q, epoch, err);
          const float v = __ldcg(P.peer_best[P.rank] + 2 * q);
          const int i = __float_as_int(__ldcg(P.peer_best[P.rank] + 2 * q + 1));
          if (q == 0 || better(v, i, bv2, bi2)) {
            bv2 = v;
            bi2 = i;
          }
        }
        gidx = bi2;
      }
      publish_argmax(P.st, P.seq_tokens, gidx);
      *P.epoch = epoch0 + 1u;
    }
  }
}

// ---------------------------------------------------------------- fused down_proj (consumers)
// down_proj = W_down . ff computed as a sum of rows of W_down^T scaled by this
// CTA's own ff values (the gate|up rows it just produced, kept in shared
// memory): thread t owns output elements [8t, 8t + 8) (and +4096 when h >
// 4096), every 16-byte weight chunk is read once, and the CTA's h-wide
// partial goes to the fixed-point accumulator with 64-bit integer atomics.
// No grid barrier separates it from gate|up, so the weight ring keeps
// streaming from one matrix into the next.
__device__ void mega_axpy(const MegaParams& P, const MegaPhase& ph, uint8_t* ring, uint64_t* full, uint64_t* empty,
                          uint32_t& gi, const float* ffs, int* err, int f) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int K = ph.K, R = ph.R;
  const int r0 = cta_row(ph.N, blockIdx.x, ph.row_align);
  const int nrows = cta_row(ph.N, blockIdx.x + 1, ph.row_align) - r0;
  const int nstages = (nrows + R - 1) / R;
  const size_t row_bytes = static_cast<size_t>(K) * 2;
  const int chunks = K >> 3;
  float acc[2][8];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[q][e] = 0.f;
  if (tid == 0) trace_mark(P, f, 1);
  for (int i = 0; i < nstages; ++i, ++gi) {
    const uint32_t slot = gi % P.nst;
    if (!mbar_wait(&full[slot], (gi / P.nst) & 1, err)) break;
    const int rows_here = min(R, nrows - i * R);
    const uint8_t* stg = ring + static_cast<size_t>(slot) * P.slot_bytes;
    for (int j = 0; j < rows_here; ++j) {
      const float w = ffs[i * R + j];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int c = tid + q * kNC;
        if (c < chunks) {
          const uint4 v = *reinterpret_cast<const uint4*>(stg + j * row_bytes + c * 16);
          acc[q][0] = fmaf(w, bf16_lo(v.x), acc[q][0]);
          acc[q][1] = fmaf(w, bf16_hi(v.x), acc[q][1]);
          acc[q][2] = fmaf(w, bf16_lo(v.y), acc[q][2]);
          acc[q][3] = fmaf(w, bf16_hi(v.y), acc[q][3]);
          acc[q][4] = fmaf(w, bf16_lo(v.z), acc[q][4]);
          acc[q][5] = fmaf(w, bf16_hi(v.z), acc[q][5]);
          acc[q][6] = fmaf(w, bf16_lo(v.w), acc[q][6]);
          acc[q][7] = fmaf(w, bf16_hi(v.w), acc[q][7]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (tid == 0) trace_mark(P, f, 2);
  unsigned long long* out = reinterpret_cast<unsigned long long*>(ph.acc_out);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int c = tid + q * kNC;
    if (c < chunks) {
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(out + c * 8 + e, static_cast<unsigned long long>(to_fixed(acc[q][e])));
    }
  }
}

// ---------------------------------------------------------------- attention phase (consumers)
// computeAttentionInto (src/llm.zig:1302-1335): work item (kv head g, page
// group s) of A = min(splits, pages) groups.  Loads are batched so the item
// costs few dependent memory round trips under full weight streaming: q,
// the new k and v, and the first page's K rows are fetched together; the
// new position's k and v come from shared memory, not from the cache that
// this CTA has just written.  The last CTA of a kv head merges the A
// partial (o, max, sum) triples, loading them all at once.
constexpr int kMaxSplitsMerged = 16;

__device__ void mega_attention(const MegaParams& P, const MegaPhase& ph, float* sm, int* err, int f) {
  __shared__ int last_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.group, d = P.d;
  const int pos = P.st->pos;
  if (pos < 0 || pos >= P.st->max_seq) {
    if (blockIdx.x == 0 && tid == 0) atomicExch(err, 1);  // VVLI_ERR_CONTEXT_FULL
    return;
  }
  const int n_ctx = pos + 1;
  const int pages = (n_ctx + kPage - 1) / kPage;
  const int A = min(P.splits, pages);
  const int items = P.nkv * A;
  float* qs = sm;               // [G][d] rotated q
  float* sc = qs + G * d;       // [G][kPage], then the P.V reduction [kNC/d][G][d]
  float* mrun = sc + G * kPage + (kNC / d) * G * d;
  float* lrun = mrun + G;
  float* alpha = lrun + G;
  float* wsplit = alpha + G;    // [G][splits]
  int* pt_sh = reinterpret_cast<int*>(wsplit + G * P.splits);  // page numbers of this item
  const int EPL = d < 32 ? d : 32;
  const int LP = d / EPL;
  const int PPW = kWarp / LP;
  const int pp = lane / LP, qq = lane % LP;
  const int nacc = (G * d + kNC - 1) / kNC;  // <= 4

  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int g = item / A, s = item % A;
    // One round trip: the group's rotated q (written by the q|k|v epilogue)
    // and the page numbers of this item's pages.
    const float* qg = P.qkv + static_cast<size_t>(g) * G * d;
    for (int idx = tid; idx < G * d; idx += kNC) qs[idx] = __ldcg(qg + idx);
    for (int k = tid, page = s + tid * A; page < pages; k += kNC, page += kNC * A) pt_sh[k] = __ldcg(P.page_table + page);
    for (int hh = tid; hh < G; hh += kNC) {
      mrun[hh] = -INFINITY;
      lrun[hh] = 0.f;
    }
    named_barrier(1, kNC);
    if (tid == 0) trace_mark(P, f, 1);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int NPG = kNC / d;
    for (int page = s, pk = 0; page < pages; page += A, ++pk) {
      const int t0 = page * kPage;
      const int n = min(kPage, n_ctx - t0);
      const size_t page_base = (static_cast<size_t>(pt_sh[pk] * P.nkv + g) * kPage) * d;  // [page][kv head][kPage][d]
      // K rows for the scores and V rows for P.V are loaded together.
      // Lane qq of a position holds float4 number j * LP + qq of the key, so
      // the LP lanes of a position read LP * 16 contiguous bytes per load.
      const int nf4 = EPL / 4;
      const int i = warp * PPW + pp;  // score position of this lane (first pass)
      float4 kv[8];
      {
        const bool ok = i < n;
        const float4* kr = reinterpret_cast<const float4*>(ph.k_cache + page_base + static_cast<size_t>(ok ? i : 0) * d);
#pragma unroll
        for (int j = 0; j < 8; ++j) kv[j] = (ok && j < nf4) ? __ldcg(kr + j * LP + qq) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float v[16];
      const int ve = tid % d, vpg = tid / d;
      const float* vb = ph.v_cache + page_base + ve;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int iv = vpg + u * NPG;
        v[u] = (tid < NPG * d && iv < n) ? __ldcg(vb + static_cast<size_t>(iv) * d) : 0.f;
      }
      for (int pass = 0, base = warp * PPW; base < n; ++pass, base += kCW * PPW) {
        const int ip = base + pp;
        const bool ok = ip < n;
        if (pass > 0) {  // positions beyond the first pass
          const float4* kr = reinterpret_cast<const float4*>(ph.k_cache + page_base + static_cast<size_t>(ok ? ip : 0) * d);
#pragma unroll
          for (int j = 0; j < 8; ++j) kv[j] = (ok && j < nf4) ? __ldcg(kr + j * LP + qq) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int hh = 0; hh < G; ++hh) {
          const float4* qh = reinterpret_cast<const float4*>(qs + hh * d);
          float dot = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j < nf4) {
              const float4 q4 = qh[j * LP + qq];
              dot = fmaf(q4.x, kv[j].x, fmaf(q4.y, kv[j].y, fmaf(q4.z, kv[j].z, fmaf(q4.w, kv[j].w, dot))));
            }
          }
          for (int o = 1; o < LP; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (ok && qq == 0) sc[hh * kPage + ip] = dot * P.inv_sqrt_d;
        }
      }
      named_barrier(1, kNC);
      if (tid == 0 && pk == 0) trace_mark(P, f, 5);
      for (int hh = warp; hh < G; hh += kCW) {  // online softmax (softmaxInPlace, src/llm.zig:1408-1419)
        float m = -INFINITY;
        for (int ii = lane; ii < n; ii += kWarp) m = fmaxf(m, sc[hh * kPage + ii]);
        m = warp_max(m);
        const float mnew = fmaxf(mrun[hh], m);
        float l = 0.f;
        for (int ii = lane; ii < n; ii += kWarp) {
          const float e = expf(sc[hh * kPage + ii] - mnew);
          sc[hh * kPage + ii] = e;
          l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
          const float a = expf(mrun[hh] - mnew);
          alpha[hh] = a;
          lrun[hh] = lrun[hh] * a + l;
          mrun[hh] = mnew;
        }
      }
      named_barrier(1, kNC);
      // P.V: thread (position group vpg, dim ve) uses each V element for all
      // q heads of the group; groups meet in shared memory.
      float* red = sc + G * kPage;  // [NPG][G][d]
      if (tid < NPG * d) {
        float ah[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int iv = vpg + u * NPG;
          if (iv < n) {
#pragma unroll
            for (int hh = 0; hh < 8; ++hh)
              if (hh < G) ah[hh] = fmaf(sc[hh * kPage + iv], v[u], ah[hh]);
          }
        }
#pragma unroll
        for (int hh = 0; hh < 8; ++hh)
          if (hh < G) red[(vpg * G + hh) * d + ve] = ah[hh];
      }
      named_barrier(1, kNC);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = tid + k * kNC;
        if (k < nacc && idx < G * d) {
          const int hh = idx / d, e = idx % d;
          float a = 0.f;
          for (int pg = 0; pg < NPG; ++pg) a += red[(pg * G + hh) * d + e];
          acc[k] = acc[k] * alpha[hh] + a;
        }
      }
      named_barrier(1, kNC);
    }
    if (tid == 0) trace_mark(P, f, 2);
    if (A == 1) {  // one split: normalise directly
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = tid + k * kNC;
        if (k < nacc && idx < G * d) P.attn[static_cast<size_t>(g * G) * d + idx] = acc[k] / lrun[idx / d];
      }
      named_barrier(1, kNC);
      continue;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = tid + k * kNC;
      if (k < nacc && idx < G * d) {
        const int hh = idx / d, e = idx % d;
        P.attn_part[(static_cast<size_t>(g * G + hh) * P.splits + s) * (d + 2) + e] = acc[k];
      }
    }
    for (int hh = tid; hh < G; hh += kNC) {
      float* pp2 = P.attn_part + (static_cast<size_t>(g * G + hh) * P.splits + s) * (d + 2);
      pp2[d] = mrun[hh];
      pp2[d + 1] = lrun[hh];
    }
    __threadfence();
    named_barrier(1, kNC);
    if (tid == 0) last_flag = atomicAdd(&P.attn_counters[g], 1u) == static_cast<unsigned>(A) - 1;
    named_barrier(1, kNC);
    if (last_flag) {
      __threadfence();
      // Weights exp(m_s - M) / L per head and split.  The o partials of the
      // first element a thread merges are loaded before the weights are
      // computed, so the merge costs one round trip for G * d <= 512.
      float ov[kMaxSplitsMerged];
      auto load_ov = [&](int idx) {
        const float* base = P.attn_part + static_cast<size_t>(g * G + idx / d) * P.splits * (d + 2) + idx % d;
#pragma unroll
        for (int sp = 0; sp < kMaxSplitsMerged; ++sp)
          if (sp < A) ov[sp] = __ldcg(base + sp * (d + 2));
      };
      if (tid < G * d) load_ov(tid);
      for (int hh = warp; hh < G; hh += kCW) {
        const float* base = P.attn_part + static_cast<size_t>(g * G + hh) * P.splits * (d + 2);
        const float m = lane < A ? __ldcg(base + lane * (d + 2) + d) : -INFINITY;
        const float l = lane < A ? __ldcg(base + lane * (d + 2) + d + 1) : 0.f;
        const float M = warp_max(m);
        const float w = lane < A ? expf(m - M) : 0.f;
        const float L = warp_sum(l * w);
        if (lane < A) wsplit[hh * P.splits + lane] = w / L;
      }
      named_barrier(1, kNC);
      for (int idx = tid; idx < G * d; idx += kNC) {
        if (idx != tid) load_ov(idx);
        const int hh = idx / d;
        float o = 0.f;
#pragma unroll
        for (int sp = 0; sp < kMaxSplitsMerged; ++sp)
          if (sp < A) o = fmaf(ov[sp], wsplit[hh * P.splits + sp], o);
        P.attn[static_cast<size_t>(g * G) * d + idx] = o;
      }
      if (tid == 0) P.attn_counters[g] = 0;
    }
    named_barrier(1, kNC);
  }
}

// ---------------------------------------------------------------- embed phase
// copyEmbeddingToken (src/llm.zig:1373-1380) / forwardEmbedding's copy.
__device__ void mega_embed(const MegaParams& P, float* red, int* err, float* xres) {
  const int tid = threadIdx.x;
  const int r0 = cta_row0(P.h), r1 = cta_row1(P.h);
  const int pos = P.st->pos;
  int tok = (pos >= 0 && pos < P.st->max_seq) ? P.seq_tokens[pos] : 0;
  if (!P.st->use_embedding && (tok < 0 || tok >= P.vocab)) {
    if (blockIdx.x == 0 && tid == 0) atomicExch(err, 3);  // VVLI_ERR_INVALID_TOKEN
    tok = 0;
  }
  float ss = 0.f;
  const uint8_t* erow = reinterpret_cast<const uint8_t*>(P.emb) + static_cast<size_t>(tok) * P.emb_row_bytes;
  for (int r = r0 + tid; r < r1; r += kNC) {
    float v;
    if (P.st->use_embedding) {
      v = P.emb_in[r];
    } else if (P.emb_fmt == kFmtQ8) {  // d * q
      v = half_at(erow + P.h + (r >> 5) * 2) * static_cast<float>(static_cast<int8_t>(erow[r]));
    } else if (P.emb_fmt == kFmtQ4) {  // d * (n - 8), GGML nibble order
      const int b = r >> 5, e = r & 31;
      const uint8_t byte = erow[b * 16 + (e & 15)];
      const int nib = e < 16 ? (byte & 15) : (byte >> 4);
      v = half_at(erow + P.h / 2 + b * 2) * static_cast<float>(nib - 8);
    } else {
      v = bf16_to_f32(reinterpret_cast<const uint16_t*>(erow)[r]);
    }
    P.x[r] = v;
    if (P.xres) xres[r - r0] = v;
    ss = fmaf(v, v, ss);
  }
  ss = consumer_sum(ss, red);
  if (tid == 0) P.ssq[blockIdx.x] = ss;
  if (P.acc_zero)  // the last step's final down_proj accumulator, read by its LM head
    for (int r = r0 + tid; r < r1; r += kNC) P.acc_zero[r] = 0;
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(kMegaThreads, 1) decode_megakernel(const MegaParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kCW];
  __shared__ float wv[kCW];
  __shared__ int wi[kCW];
  __shared__ float ffs[kMaxFfRows];  // gate|up outputs of this CTA for the fused down_proj
  __shared__ float xres[kMaxResRows];  // this CTA's rows of x (MegaParams::xres)
  const int tid = threadIdx.x, warp = tid >> 5;
  uint8_t* ring = smem;
  float* part = reinterpret_cast<float*>(smem + static_cast<size_t>(P.nst) * P.slot_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(part + ((P.part_floats + 1) & ~1));
  uint64_t* empty = full + P.nst;
  // a GEMV phase's input vector (P.xstage_floats; see mega_gemv), 16-byte aligned
  float4* xstage = reinterpret_cast<float4*>((reinterpret_cast<uintptr_t>(empty + P.nst) + 15) & ~uintptr_t(15));
  int* err = &P.st->err;

  if (tid == 0) {
    for (int i = 0; i < P.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCW);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == kCW) {
    if ((tid & 31) == 0) mega_producer(P, ring, full, empty, err);
    return;
  }
  uint32_t gi = 0;
  uint32_t nbar = 0;  // barriers passed in this step
  const unsigned epoch0 = __ldcg(P.epoch);
  for (int f = 0; f < P.nphases; ++f) {
    const MegaPhase& ph = P.phases[f];
    if (tid == 0) trace_mark(P, f, 0);
    if (ph.kind == MK_EMBED) {
      mega_embed(P, red, err, xres);
    } else if (ph.kind == MK_ATTN) {
      mega_attention(P, ph, part, err, f);
    } else if (ph.epi == ME_AXPY) {
      mega_axpy(P, ph, ring, full, empty, gi, ffs, err, f);
    } else {
      if (ph.fmt == kFmtQ8)
        mega_gemv<2, kFmtQ8>(P, ph, ring, part, full, empty, gi, red, wv, wi, err, epoch0, f, ffs, xres, xstage);
      else if (ph.fmt == kFmtQ4)
        mega_gemv<1, kFmtQ4>(P, ph, ring, part, full, empty, gi, red, wv, wi, err, epoch0, f, ffs, xres, xstage);
      else
        mega_gemv<4, kFmtBF16>(P, ph, ring, part, full, empty, gi, red, wv, wi, err, epoch0, f, ffs, xres, xstage);
    }
    if (tid == 0) trace_mark(P, f, 3);
    if (f + 1 < P.nphases && P.phases[f + 1].no_barrier) {
      named_barrier(1, kNC);  // the next phase reads only what this CTA wrote
    } else if (f + 1 < P.nphases) {
      grid_arrive(P.bar);
      // While the other CTAs arrive: warm L1/L2 with the next phase's
      // constant vectors (norm weights, biases) of this CTA.
      const MegaPhase& nx = P.phases[f + 1];
      if (nx.kind == MK_GEMV) {
        if (nx.norm_w && (tid + 1) * 64 <= nx.K * 2) prefetch_l2_bulk(nx.norm_w + tid * 32, 64);
      }
      // A barrier that gave up ends this CTA; the producer's own bounded
      // waits then end it too.
      const uint64_t target = (static_cast<uint64_t>(epoch0) * P.bars_per_step + nbar + 1) * gridDim.x;
      ++nbar;
      if (!grid_wait(P.bar, target, err)) break;
    }
    if (tid == 0) trace_mark(P, f, 4);
  }
}

cudaError_t launch_megakernel(const MegaParams& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMegaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_megakernel, p);
}

bool plan_mega_gemv(MegaPhase& ph, int stage_cap) {
  const int epc = ph.fmt == kFmtBF16 ? WFmt<kFmtBF16>::EPC : ph.fmt == kFmtQ8 ? WFmt<kFmtQ8>::EPC : WFmt<kFmtQ4>::EPC;
  const int maxc = 32 / epc;
  if (ph.K % (ph.fmt == kFmtBF16 ? 8 : 32)) return false;
  const int cpr = ph.K / epc;
  const size_t row_bytes = static_cast<size_t>(ph.row_bytes);
  int S = 1;
  while (S < kCW && S * kWarp * maxc < cpr) S *= 2;
  ph.S = S;
  ph.SZ = (cpr + S - 1) / S;
  ph.cpl = (ph.SZ + kWarp - 1) / kWarp;
  if (ph.cpl > maxc) return false;
  const int want_pairs = 2 * kCW;
  int R = (want_pairs + S * ph.nphys - 1) / (S * ph.nphys);
  while (R > 1 && R * row_bytes * ph.nphys > static_cast<size_t>(stage_cap)) R /= 2;
  // Shorter rows (block-quantised ones) take more rows per stage, so the ring
  // keeps as many bytes in flight as with bf16 rows.
  R = std::max(R, static_cast<int>(static_cast<size_t>(stage_cap) / (row_bytes * ph.nphys)));
  ph.R = R < 1 ? 1 : R;
  ph.stage_bytes = static_cast<int>(ph.R * row_bytes * ph.nphys);
  return true;
}

size_t mega_attention_floats(int group, int d, int splits, int max_pages) {
  // q, scores, P.V reduction [threads/d][group][d], running max/sum/alpha, merge weights, page numbers
  return static_cast<size_t>(group) * d + static_cast<size_t>(group) * kPage +
         static_cast<size_t>(kNC / d) * group * d + 3 * group + static_cast<size_t>(group) * splits +
         static_cast<size_t>((max_pages + splits - 1) / splits);
}

cudaError_t configure_megakernel(int max_smem_optin) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, decode_megakernel);
  if (e) return e;
  return cudaFuncSetAttribute(decode_megakernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              max_smem_optin - static_cast<int>(fa.sharedSizeBytes));
}

}  // namespace vvli
