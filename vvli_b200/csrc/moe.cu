// moe.cu - mixture-of-experts feed-forward block (OLMoE) for decode batches.
//
// x += MoE(rmsnorm(x) * norm_w) for T token rows, as the OLMoE decoder layer
// applies its sparse block after attention.  The reference parses OLMoE
// configs (src/llm.zig:45-48, 111-133, 210-214) and counts their parameters
// (src/llm.zig:261-264) but stops before any arithmetic (src/main.zig:
// 590-611); the arithmetic follows the published OLMoE block (transformers
// 5.5.0, models/olmoe/modeling_olmoe.py: OlmoeTopKRouter, OlmoeExperts),
// restated in oracle/moe_ref.py.
//
// Five launches on the caller's stream, HBM-bound on the expert weights; the
// last four are programmatic dependents of the one before (each starts
// while its predecessor runs and waits for it before reading its output):
//   1. moe_logits_kernel, CTA = (8 experts, token): RMSNorm of the row in
//      shared memory (written to the workspace once), a warp per router
//      logit.
//   2. moe_group_kernel, one CTA: softmax and top-k of every token (a warp
//      per token; larger probability first, lower index on ties; weights
//      renormalised when norm_topk_prob), then the (token, slot) pairs
//      grouped by expert in token order (warp ballots), the experts'
//      counts and offsets, the list of the routed experts in ascending
//      order, and each token's pairs sorted by expert index.
//   3. moe_expert_kernel<true>: gate|up rows of every routed expert times its
//      tokens' normed rows, silu(gate) * up per pair; then
//      4. moe_expert_kernel<false>: the down rows times those.  Persistent
//      grids (the CTAs resident at once) walk the (routed expert, row tile)
//      items, so only the routed experts' weights are read and no CTA is
//      spent on an expert without tokens.  A warp streams 8 weight rows
//      with 16-byte loads, two steps in flight, and multiplies them with up
//      to 3 tokens staged in shared memory (the token count of a pass is a
//      template parameter; each weight is unpacked once per step); an
//      expert with more tokens is taken 3 at a time (its tile comes back
//      from L2).
//   5. moe_combine_kernel, one CTA per token: x += sum of w_e * down_e(...)
//      over the token's experts in ascending expert index (the order of the
//      OLMoE experts loop), so the result does not depend on timing.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <mutex>
#include <string>

#include "../../include/vvli_cuda.h"
#include "common.cuh"

namespace vvli {
void set_last_error(const std::string& what);  // runtime.cu
}

using namespace vvli;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTokens = 4096;
constexpr int kMaxDim = 8192;
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;
constexpr int kTG = 3;           // tokens multiplied per pass over a weight tile
constexpr int kKC = 2048;        // activation elements staged per chunk
constexpr int kRowsPerWarp = 8;  // weight rows a warp streams together

struct MoeDev {
  int T, h, I, E, k, norm_topk;
  float eps;
  float* x;
  const uint16_t* norm_w;
  const uint16_t* router;
  const uint16_t* gate_up;
  const uint16_t* down;
  // workspace
  float* xn;        // [T][h]
  float* logits;    // [T][E] router logits (then the group kernel's scratch)
  int* topk_idx;    // [T][k]
  float* topk_w;    // [T][k]
  int* cnt;         // [E]
  int* off;         // [E]
  int* act;         // [E] routed experts, ascending
  int* n_act;       // [1]
  int* pair_tok;    // [T*k] token of pair q (pairs grouped by expert)
  int* tok_rank;    // [T*k] rank of (token, slot) among the token's experts by index
  int* tok_q;       // [T][k] the token's pairs, ascending expert index
  float* tok_w;     // [T][k] their weights
  float* f;         // [T*k][I] silu(gate) * up
  float* yd;        // [T*k][h] down rows . f
  // optional outputs
  int32_t* out_idx;
  float* out_w;
};

struct WsLayout {
  size_t xn, logits, idx, w, cnt, off, act, nact, pair_tok, tok_rank, tok_q, tok_w, f, yd, total;
};

size_t up256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

WsLayout ws_layout(uint64_t T, uint64_t h, uint64_t I, uint64_t E, uint64_t k) {
  WsLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = up256(o + bytes);
    return at;
  };
  L.xn = take(T * h * 4);
  L.logits = take(T * E * 4);
  L.idx = take(T * k * 4);
  L.w = take(T * k * 4);
  L.cnt = take(E * 4);
  L.off = take(E * 4);
  L.act = take(E * 4);
  L.nact = take(4);
  L.pair_tok = take(T * k * 4);
  L.tok_rank = take(T * k * 4);
  L.tok_q = take(T * k * 4);
  L.tok_w = take(T * k * 4);
  L.f = take(T * k * I * 4);
  L.yd = take(T * k * h * 4);
  L.total = o;
  return L;
}

// Eight bf16 weights (one 16-byte load) times eight activations.
VVLI_DEV float dot8(const uint4& w, const float4& a, const float4& b, float acc) {
  acc = fmaf(bf16_lo(w.x), a.x, acc);
  acc = fmaf(bf16_hi(w.x), a.y, acc);
  acc = fmaf(bf16_lo(w.y), a.z, acc);
  acc = fmaf(bf16_hi(w.y), a.w, acc);
  acc = fmaf(bf16_lo(w.z), b.x, acc);
  acc = fmaf(bf16_hi(w.z), b.y, acc);
  acc = fmaf(bf16_lo(w.w), b.z, acc);
  acc = fmaf(bf16_hi(w.w), b.w, acc);
  return acc;
}

// Streaming 16-byte load of read-only weights that the compiler may schedule
// freely (no volatile): the loads of one chunk go out together.
VVLI_DEV uint4 ld_weights(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// 1. RMSNorm and the router logits (OlmoeTopKRouter.forward, first half).
//    CTA = (8 experts, token): the row is normalised in shared memory (the
//    CTA of experts 0-7 also writes it to xn), then a warp per expert.
__global__ void __launch_bounds__(kThreads) moe_logits_kernel(const MoeDev p) {
  extern __shared__ float xs[];  // xn [h]
  __shared__ float red[kWarps];
  const int t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  grid_launch_dependents();  // the next kernel waits for this one's completion before reading
  const float* xr = p.x + static_cast<size_t>(t) * p.h;
  float ss = 0.f;
  for (int i = tid; i < p.h; i += kThreads) {
    const float v = xr[i];
    xs[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += red[w];
  // rmsNormInto (src/llm.zig:1287-1300)
  const float scale = 1.0f / sqrtf(tot / static_cast<float>(p.h) + p.eps);
  float* xo = p.xn + static_cast<size_t>(t) * p.h;
  for (int i = tid; i < p.h; i += kThreads) {
    const float v = xs[i] * scale * bf16_to_f32(p.norm_w[i]);
    xs[i] = v;
    if (blockIdx.x == 0) xo[i] = v;
  }
  __syncthreads();
  const int e = blockIdx.x * kWarps + warp;
  if (e >= p.E) return;
  const uint16_t* wr = p.router + static_cast<size_t>(e) * p.h;  // h % 8 == 0: 16-byte rows
  float a = 0.f;
#pragma unroll 8
  for (int k0 = lane * 8; k0 < p.h; k0 += 256)
    a = dot8(ld_weights(wr + k0), *reinterpret_cast<const float4*>(xs + k0),
             *reinterpret_cast<const float4*>(xs + k0 + 4), a);
  a = warp_sum(a);
  if (lane == 0) p.logits[static_cast<size_t>(t) * p.E + e] = a;
}

// 2. Softmax and top-k of every token (OlmoeTopKRouter.forward, second
//    half; a warp per token, its router row in registers), then the pairs
//    grouped by expert in token order (warp ballots), the experts' counts
//    and offsets, the list of the routed experts in ascending order, and per
//    token its pairs sorted by expert index for the combine.  One CTA.
__global__ void __launch_bounds__(1024) moe_group_kernel(const MoeDev p) {
  constexpr int kPerLane = kMaxExperts / 32;
  __shared__ int cnt_s[kMaxExperts], off_s[kMaxExperts], act_s[kMaxExperts];
  __shared__ int wsum[32], wact[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  grid_launch_dependents();
  grid_dependency_wait();  // the router logits come from the previous kernel
  for (int t = warp; t < p.T; t += nw) {
    const float* lg = p.logits + static_cast<size_t>(t) * p.E;
    float v[kPerLane];  // expert lane + 32 c
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < kPerLane; ++c) {
      const int e = lane + 32 * c;
      v[c] = e < p.E ? lg[e] : -INFINITY;
      m = fmaxf(m, v[c]);
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kPerLane; ++c) {
      const int e = lane + 32 * c;
      v[c] = e < p.E ? expf(v[c] - m) : -2.f;  // -2: never a candidate
      if (e < p.E) s += v[c];
    }
    s = warp_sum(s);
    float sel_v = 0.f, sum = 0.f;  // lane j keeps slot j
    int sel_i = INT_MAX;
    for (int j = 0; j < p.k; ++j) {
      float bv = -1.f;
      int bi = INT_MAX;
#pragma unroll
      for (int c = 0; c < kPerLane; ++c)
        if (better(v[c], lane + 32 * c, bv, bi)) bv = v[c], bi = lane + 32 * c;
      warp_argmax(bv, bi);
      if (bi >= p.E) bi = 0, bv = 0.f;  // NaN logits leave no candidate: keep the index in range
      const float pv = bv / s;
      if (lane == j) sel_v = pv, sel_i = bi;
      sum += pv;  // slot order, larger first
#pragma unroll
      for (int c = 0; c < kPerLane; ++c)
        if (lane + 32 * c == bi) v[c] = -2.f;  // not chosen again
    }
    // rank of slot `lane` among the token's experts by index (ties: slot order)
    int rank = 0;
    for (int l = 0; l < p.k; ++l) {
      const int other = __shfl_sync(0xffffffffu, sel_i, l);
      rank += (other < sel_i) || (other == sel_i && l < lane);
    }
    if (lane < p.k) {
      const float w = p.norm_topk ? sel_v / sum : sel_v;
      const size_t at = static_cast<size_t>(t) * p.k + lane;
      p.topk_idx[at] = sel_i;
      p.topk_w[at] = w;
      p.tok_rank[at] = rank;
      if (p.out_idx) p.out_idx[at] = sel_i;
      if (p.out_w) p.out_w[at] = w;
    }
  }
  __syncthreads();
  // counts: a warp per expert, 32 pairs per ballot
  const int n = p.T * p.k;
  for (int e = warp; e < p.E; e += nw) {
    int c = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      c += __popc(__ballot_sync(0xffffffffu, i < n && p.topk_idx[i] == e));
    }
    if (lane == 0) cnt_s[e] = c;
  }
  __syncthreads();
  // exclusive scans of the counts and of the routed flags (E <= 1024 = blockDim)
  {
    const int c = tid < p.E ? cnt_s[tid] : 0;
    const int f = c > 0;
    int sc = c, sf = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, sc, o), b = __shfl_up_sync(0xffffffffu, sf, o);
      if (lane >= o) sc += a, sf += b;
    }
    if (lane == 31) wsum[warp] = sc, wact[warp] = sf;
    __syncthreads();
    if (warp == 0) {
      int a = wsum[lane], b = wact[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
        if (lane >= o) a += x, b += y;
      }
      wsum[lane] = a, wact[lane] = b;  // inclusive over warps
    }
    __syncthreads();
    const int base_c = warp ? wsum[warp - 1] : 0, base_f = warp ? wact[warp - 1] : 0;
    if (tid < p.E) {
      off_s[tid] = base_c + sc - c;
      p.cnt[tid] = c;
      p.off[tid] = base_c + sc - c;
      if (f) act_s[base_f + sf - 1] = tid;
    }
    if (tid == 0) *p.n_act = wact[31];
  }
  __syncthreads();
  for (int a = tid; a < wact[31]; a += blockDim.x) p.act[a] = act_s[a];
  // placement: pair i of expert e goes to off[e] + (pairs of e before i)
  for (int e = warp; e < p.E; e += nw) {
    int q = off_s[e];
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      const bool mine = i < n && p.topk_idx[i] == e;
      const unsigned mask = __ballot_sync(0xffffffffu, mine);
      if (mine) {
        const int qi = q + __popc(mask & lt);
        const int t = i / p.k;
        p.pair_tok[qi] = t;
        const size_t at = static_cast<size_t>(t) * p.k + p.tok_rank[i];
        p.tok_q[at] = qi;
        p.tok_w[at] = p.topk_w[i];
      }
      q += __popc(mask);
    }
  }
}

// 3. Weight tiles of the routed experts times their tokens (OlmoeExperts.forward).
//    GATEUP: rows r of gate and up (4 output rows per warp: 8 weight rows),
//            f[q][r] = silu(gate_r . xn) * (up_r . xn);
//    else:   rows r of down (8 per warp), yd[q][r] = down_r . f[q].
//    Persistent: CTA b takes items b, b + grid, ... of the list (routed
//    expert slot, row tile), slot-major, until the slot passes n_act.
// One pass of a warp's 8 weight rows over K with NG tokens (pairs q .. q+NG-1),
// then its outputs.  Weight row i: (i < 4 ? b0 : b1) + (i % 4) * K, live when
// i % 4 < (i < 4 ? n0 : n1).  The tokens' activations are staged in shared
// memory chunk by chunk; each weight is unpacked once per step and used for
// all NG tokens; two steps of weights are in flight.  Sums in element order.
template <bool GATEUP, int NG>
__device__ __forceinline__ void expert_pass(const MoeDev& p, const uint16_t* b0, const uint16_t* b1, int n0, int n1,
                                            int K, int R, int r_base, int q, float* xs) {
  constexpr int kOut = GATEUP ? kRowsPerWarp / 2 : kRowsPerWarp;
  const int tid = threadIdx.x, lane = tid & 31;
  auto row = [&](int i) { return (i < 4 ? b0 : b1) + static_cast<size_t>(i & 3) * K; };
  auto live = [&](int i) { return (i & 3) < (i < 4 ? n0 : n1); };
  float acc[kRowsPerWarp][NG];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int u = 0; u < NG; ++u) acc[i][u] = 0.f;
  for (int c0 = 0; c0 < K; c0 += kKC) {
    const int kc = min(kKC, K - c0);
    // the chunk's first weights go out before the activations are staged
    uint4 cur[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
      cur[i] = (live(i) && lane * 8 < kc) ? ld_weights(row(i) + c0 + lane * 8) : make_uint4(0, 0, 0, 0);
    __syncthreads();  // the previous chunk's readers are done
    const int kc4 = kc >> 2;  // K % 8 == 0: rows and chunks start on 16-byte boundaries
    for (int idx = tid; idx < NG * kc4; idx += kThreads) {
      const int u = idx / kc4, kk = (idx - u * kc4) * 4;
      const float* src = GATEUP ? p.xn + static_cast<size_t>(p.pair_tok[q + u]) * K : p.f + static_cast<size_t>(q + u) * K;
      *reinterpret_cast<float4*>(xs + u * kKC + kk) = *reinterpret_cast<const float4*>(src + c0 + kk);
    }
    __syncthreads();
    for (int k0 = lane * 8; k0 < kc; k0 += 256) {
      uint4 nxt[kRowsPerWarp];
      const bool more = k0 + 256 < kc;
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i)
        nxt[i] = (live(i) && more) ? ld_weights(row(i) + c0 + k0 + 256) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float4 xv[NG];
#pragma unroll
        for (int u = 0; u < NG; ++u) xv[u] = *reinterpret_cast<const float4*>(xs + u * kKC + k0 + 4 * half);
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
          const uint32_t w0 = half ? cur[i].z : cur[i].x, w1 = half ? cur[i].w : cur[i].y;
          const float a0 = bf16_lo(w0), a1 = bf16_hi(w0), a2 = bf16_lo(w1), a3 = bf16_hi(w1);
#pragma unroll
          for (int u = 0; u < NG; ++u) {
            float t = acc[i][u];
            t = fmaf(a0, xv[u].x, t);
            t = fmaf(a1, xv[u].y, t);
            t = fmaf(a2, xv[u].z, t);
            t = fmaf(a3, xv[u].w, t);
            acc[i][u] = t;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i) cur[i] = nxt[i];
    }
  }
  // every lane gets the sums; lane (i, u) stores one of them
#pragma unroll
  for (int i = 0; i < kOut; ++i) {
#pragma unroll
    for (int u = 0; u < NG; ++u) {
      const float s0 = warp_sum(acc[i][u]);
      float val = s0;
      if constexpr (GATEUP) {
        const float up = warp_sum(acc[kOut + i][u]);
        val = (s0 / (1.0f + expf(-s0))) * up;  // silu(gate) * up
      }
      const int out = r_base + i;
      if (lane == i * NG + u && out < R) {
        const size_t qq = static_cast<size_t>(q + u);
        if constexpr (GATEUP)
          p.f[qq * p.I + out] = val;
        else
          p.yd[qq * p.h + out] = val;
      }
    }
  }
}

template <bool GATEUP>
__global__ void __launch_bounds__(kThreads, 2) moe_expert_kernel(const MoeDev p) {
  extern __shared__ float xs[];  // [kTG][kKC]
  const int K = GATEUP ? p.h : p.I;
  const int R = GATEUP ? p.I : p.h;  // output rows of an expert
  constexpr int kOut = GATEUP ? kRowsPerWarp / 2 : kRowsPerWarp;
  constexpr int kTileRows = kWarps * kOut;
  const int tiles = (R + kTileRows - 1) / kTileRows;
  grid_launch_dependents();
  grid_dependency_wait();  // the routing (and for down, f) comes from the previous kernels
  const int n_act = *p.n_act;
  const int warp = threadIdx.x >> 5;
  for (int item = blockIdx.x;; item += gridDim.x) {
    const int slot = item / tiles;
    if (slot >= n_act) break;  // uniform over the CTA
    const int e = p.act[slot];
    const int cnt = p.cnt[e], q0 = p.off[e];
    const int r_base = ((item - slot * tiles) * kWarps + warp) * kOut;
    const uint16_t* W = GATEUP ? p.gate_up + static_cast<size_t>(e) * 2 * p.I * p.h
                               : p.down + static_cast<size_t>(e) * p.h * p.I;
    // GATEUP: gate rows r_base .. +3, then the matching up rows I + r_base .. +3; else rows r_base .. +7
    const int left = max(0, R - r_base);
    const int n0 = min(4, left), n1 = GATEUP ? n0 : max(0, min(4, left - 4));
    const uint16_t* b0 = W + static_cast<size_t>(left ? r_base : 0) * K;
    const uint16_t* b1 = GATEUP ? W + static_cast<size_t>(left ? p.I + r_base : 0) * K : b0 + 4 * static_cast<size_t>(K);
    for (int g0 = 0; g0 < cnt; g0 += kTG) {
      switch (min(kTG, cnt - g0)) {  // the pass's token count as a compile-time constant
        case 1: expert_pass<GATEUP, 1>(p, b0, b1, n0, n1, K, R, r_base, q0 + g0, xs); break;
        case 2: expert_pass<GATEUP, 2>(p, b0, b1, n0, n1, K, R, r_base, q0 + g0, xs); break;
        default: expert_pass<GATEUP, 3>(p, b0, b1, n0, n1, K, R, r_base, q0 + g0, xs); break;
      }
    }
  }
}

// 5. x += sum over the token's experts, ascending expert index, of w * yd.
//    The token's pair list goes to shared memory first; the experts' rows
//    are loaded eight at a time and added in order.
__global__ void __launch_bounds__(kThreads) moe_combine_kernel(const MoeDev p) {
  __shared__ int sq[kMaxTopK];
  __shared__ float sw[kMaxTopK];
  const int t = blockIdx.x, tid = threadIdx.x;
  grid_dependency_wait();  // the pairs and yd come from the previous kernels
  if (tid < p.k) {
    sq[tid] = p.tok_q[static_cast<size_t>(t) * p.k + tid];
    sw[tid] = p.tok_w[static_cast<size_t>(t) * p.k + tid];
  }
  __syncthreads();
  float* xr = p.x + static_cast<size_t>(t) * p.h;
  for (int c = tid; c < p.h; c += kThreads) {
    float y = 0.f;
    int j = 0;
    for (; j + 8 <= p.k; j += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = p.yd[static_cast<size_t>(sq[j + u]) * p.h + c];
#pragma unroll
      for (int u = 0; u < 8; ++u) y += sw[j + u] * v[u];
    }
    for (; j < p.k; ++j) y += sw[j] * p.yd[static_cast<size_t>(sq[j]) * p.h + c];
    xr[c] = xr[c] + y;
  }
}

int fail(int code, const std::string& why) {
  set_last_error("moe_ffn: " + why);
  return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Sizes the kernels take; "" when they do, else the reason.
std::string check_sizes(uint64_t T, uint64_t h, uint64_t I, uint64_t E, uint64_t k) {
  if (T < 1 || T > kMaxTokens) return "tokens must be in [1, " + std::to_string(kMaxTokens) + "]";
  if (h < 8 || h > kMaxDim || h % 8) return "hidden must be a multiple of 8 in [8, " + std::to_string(kMaxDim) + "]";
  if (I < 8 || I > kMaxDim || I % 8) return "inter must be a multiple of 8 in [8, " + std::to_string(kMaxDim) + "]";
  if (E < 1 || E > kMaxExperts) return "experts must be in [1, " + std::to_string(kMaxExperts) + "]";
  if (k < 1 || k > E || k > kMaxTopK) return "top_k must be in [1, min(experts, " + std::to_string(kMaxTopK) + ")]";
  return "";
}

// CTAs of each expert kernel resident at once on `device` (SMs x blocks per
// SM), looked up once per device.
cudaError_t expert_residency(int device, int* out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int cached[kMaxDevices][2] = {};
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[device][0]) {
    int sms = 0, b0 = 0, b1 = 0;
    const size_t smem = static_cast<size_t>(kTG) * kKC * sizeof(float);
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b0, moe_expert_kernel<true>, kThreads, smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b1, moe_expert_kernel<false>, kThreads, smem);
    if (e != cudaSuccess) return e;
    cached[device][0] = std::max(1, sms * b0);
    cached[device][1] = std::max(1, sms * b1);
  }
  out[0] = cached[device][0];
  out[1] = cached[device][1];
  return cudaSuccess;
}

struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" uint64_t vvli_cuda_moe_workspace_bytes(uint64_t tokens, uint64_t hidden, uint64_t inter, uint64_t experts,
                                                  uint64_t top_k) {
  if (!check_sizes(tokens, hidden, inter, experts, top_k).empty()) return 0;
  return ws_layout(tokens, hidden, inter, experts, top_k).total;
}

extern "C" int vvli_cuda_moe_ffn(int device, const vvli_moe_args* a, void* stream) {
  if (!a) return fail(VVLI_ERR_INVALID_ARGUMENT, "null arguments");
  const std::string bad = check_sizes(a->tokens, a->hidden, a->inter, a->experts, a->top_k);
  if (!bad.empty()) return fail(VVLI_ERR_INVALID_ARGUMENT, bad);
  if (!a->x || !a->norm_w || !a->router || !a->gate_up || !a->down || !a->workspace)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(a->router) || !aligned16(a->gate_up) || !aligned16(a->down) || !aligned16(a->x))
    return fail(VVLI_ERR_INVALID_ARGUMENT, "x, router, gate_up and down must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(a->workspace) & 255u)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  if (!(a->rms_eps >= 0.f)) return fail(VVLI_ERR_INVALID_ARGUMENT, "rms_eps must be >= 0");
  const WsLayout L = ws_layout(a->tokens, a->hidden, a->inter, a->experts, a->top_k);
  if (a->workspace_bytes < L.total)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "workspace_bytes " + std::to_string(a->workspace_bytes) + " < " +
                                               std::to_string(L.total) + " (vvli_cuda_moe_workspace_bytes)");
  DeviceGuard guard;
  cudaError_t e = cudaGetDevice(&guard.prev);
  if (e == cudaSuccess) e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(VVLI_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));

  MoeDev p{};
  p.T = static_cast<int>(a->tokens), p.h = static_cast<int>(a->hidden), p.I = static_cast<int>(a->inter);
  p.E = static_cast<int>(a->experts), p.k = static_cast<int>(a->top_k), p.norm_topk = a->norm_topk_prob != 0;
  p.eps = a->rms_eps;
  p.x = a->x, p.norm_w = a->norm_w, p.router = a->router, p.gate_up = a->gate_up, p.down = a->down;
  char* ws = static_cast<char*>(a->workspace);
  p.xn = reinterpret_cast<float*>(ws + L.xn);
  p.logits = reinterpret_cast<float*>(ws + L.logits);
  p.topk_idx = reinterpret_cast<int*>(ws + L.idx);
  p.topk_w = reinterpret_cast<float*>(ws + L.w);
  p.cnt = reinterpret_cast<int*>(ws + L.cnt);
  p.off = reinterpret_cast<int*>(ws + L.off);
  p.act = reinterpret_cast<int*>(ws + L.act);
  p.n_act = reinterpret_cast<int*>(ws + L.nact);
  p.pair_tok = reinterpret_cast<int*>(ws + L.pair_tok);
  p.tok_rank = reinterpret_cast<int*>(ws + L.tok_rank);
  p.tok_q = reinterpret_cast<int*>(ws + L.tok_q);
  p.tok_w = reinterpret_cast<float*>(ws + L.tok_w);
  p.f = reinterpret_cast<float*>(ws + L.f);
  p.yd = reinterpret_cast<float*>(ws + L.yd);
  p.out_idx = a->topk_index, p.out_w = a->topk_weight;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int resident[2];
  if ((e = expert_residency(device, resident)) != cudaSuccess)
    return fail(VVLI_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(e));
  const size_t logits_smem = static_cast<size_t>(p.h) * sizeof(float);       // <= 32 KB
  const size_t expert_smem = static_cast<size_t>(kTG) * kKC * sizeof(float);  // 24 KB
  moe_logits_kernel<<<dim3((p.E + kWarps - 1) / kWarps, p.T), kThreads, logits_smem, s>>>(p);
  // the later kernels are programmatic dependents: they launch while the
  // previous one runs and wait (griddepcontrol.wait) before reading its output
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  auto launch = [&](auto kernel, dim3 grid, int threads, size_t smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
  };
  // persistent grids: no more CTAs than are resident at once, nor than (expert, tile) items
  const long gu_items = static_cast<long>(p.E) * ((p.I + kWarps * kRowsPerWarp / 2 - 1) / (kWarps * kRowsPerWarp / 2));
  const long dn_items = static_cast<long>(p.E) * ((p.h + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp));
  if ((e = launch(moe_group_kernel, dim3(1), 1024, 0)) == cudaSuccess &&
      (e = launch(moe_expert_kernel<true>, dim3(static_cast<unsigned>(std::min<long>(gu_items, resident[0]))), kThreads,
                  expert_smem)) == cudaSuccess &&
      (e = launch(moe_expert_kernel<false>, dim3(static_cast<unsigned>(std::min<long>(dn_items, resident[1]))), kThreads,
                  expert_smem)) == cudaSuccess)
    e = launch(moe_combine_kernel, dim3(p.T), kThreads, 0);
  if (e != cudaSuccess) return fail(VVLI_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VVLI_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return VVLI_OK;
}
