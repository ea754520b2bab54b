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
// Five launches on the caller's stream, HBM-bound on the expert weights:
//   1. moe_logits_kernel, CTA = (8 experts, token): RMSNorm of the row in
//      shared memory (written to the workspace once), a warp per router
//      logit.
//   2. moe_group_kernel, one CTA: softmax and top-k of every token (a warp
//      per token; larger probability first, lower index on ties; weights
//      renormalised when norm_topk_prob), then the (token, slot) pairs
//      grouped by expert in token order, the experts' counts and offsets,
//      and the list of the routed experts in ascending order.
//   3. moe_expert_kernel<true>: gate|up rows of every routed expert times its
//      tokens' normed rows, silu(gate) * up per pair; then
//      4. moe_expert_kernel<false>: the down rows times those.  Persistent
//      grids (the CTAs resident at once) walk the (routed expert, row tile)
//      items, so only the routed experts' weights are read and no CTA is
//      spent on an expert without tokens.  A warp streams 8 weight rows
//      with 16-byte loads, two steps in flight, and multiplies them with up
//      to 4 tokens staged in shared memory; an expert with more tokens is
//      taken 4 at a time (its tile comes back from L2).
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
constexpr int kTG = 4;           // tokens multiplied per pass over a weight tile
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
  int* slot_q;      // [T*k] pair of (token, slot)
  float* f;         // [T*k][I] silu(gate) * up
  float* yd;        // [T*k][h] down rows . f
  // optional outputs
  int32_t* out_idx;
  float* out_w;
};

struct WsLayout {
  size_t xn, logits, idx, w, cnt, off, act, nact, pair_tok, slot_q, f, yd, total;
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
  L.slot_q = take(T * k * 4);
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
//    half; a warp per token), then the pairs grouped by expert (token order
//    inside an expert), the experts' counts and offsets and the list of the
//    routed experts in ascending order.  One CTA.
__global__ void __launch_bounds__(1024) moe_group_kernel(const MoeDev p) {
  __shared__ int cnt_s[kMaxExperts], off_s[kMaxExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  for (int t = warp; t < p.T; t += nw) {
    float* lg = p.logits + static_cast<size_t>(t) * p.E;  // this warp's row, reused as scratch
    float m = -INFINITY;
    for (int e = lane; e < p.E; e += 32) m = fmaxf(m, lg[e]);
    m = warp_max(m);
    float s = 0.f;
    for (int e = lane; e < p.E; e += 32) {
      const float v = expf(lg[e] - m);
      lg[e] = v;
      s += v;
    }
    s = warp_sum(s);
    __syncwarp();
    float sel_v = 0.f, sum = 0.f;  // lane j keeps slot j
    int sel_i = 0;
    for (int j = 0; j < p.k; ++j) {
      float bv = -1.f;
      int bi = INT_MAX;
      for (int e = lane; e < p.E; e += 32)
        if (better(lg[e], e, bv, bi)) bv = lg[e], bi = e;
      warp_argmax(bv, bi);
      if (bi >= p.E) bi = 0, bv = 0.f;  // NaN logits leave no candidate: keep the index in range
      const float pv = bv / s;
      if (lane == j) sel_v = pv, sel_i = bi;
      sum += pv;  // slot order, larger first
      __syncwarp();
      if (lane == 0) lg[bi] = -2.f;  // below every probability: not chosen again
      __syncwarp();
    }
    if (lane < p.k) {
      const float w = p.norm_topk ? sel_v / sum : sel_v;
      const size_t at = static_cast<size_t>(t) * p.k + lane;
      p.topk_idx[at] = sel_i;
      p.topk_w[at] = w;
      if (p.out_idx) p.out_idx[at] = sel_i;
      if (p.out_w) p.out_w[at] = w;
    }
  }
  __syncthreads();
  const int n = p.T * p.k;
  for (int e = tid; e < p.E; e += blockDim.x) {
    int c = 0;
    for (int i = 0; i < n; ++i) c += p.topk_idx[i] == e;
    cnt_s[e] = c;
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0, a = 0;
    for (int e = 0; e < p.E; ++e) {
      off_s[e] = o;
      o += cnt_s[e];
      if (cnt_s[e]) p.act[a++] = e;
    }
    *p.n_act = a;
  }
  __syncthreads();
  for (int e = tid; e < p.E; e += blockDim.x) {
    p.cnt[e] = cnt_s[e];
    p.off[e] = off_s[e];
    int q = off_s[e];
    for (int i = 0; i < n; ++i)
      if (p.topk_idx[i] == e) {
        p.pair_tok[q] = i / p.k;
        p.slot_q[i] = q;
        ++q;
      }
  }
}

// 3. Weight tiles of the routed experts times their tokens (OlmoeExperts.forward).
//    GATEUP: rows r of gate and up (4 output rows per warp: 8 weight rows),
//            f[q][r] = silu(gate_r . xn) * (up_r . xn);
//    else:   rows r of down (8 per warp), yd[q][r] = down_r . f[q].
//    Persistent: CTA b takes items b, b + grid, ... of the list (routed
//    expert slot, row tile), slot-major, until the slot passes n_act.
template <bool GATEUP>
__global__ void __launch_bounds__(kThreads) moe_expert_kernel(const MoeDev p) {
  extern __shared__ float xs[];  // [kTG][kKC]
  const int K = GATEUP ? p.h : p.I;
  const int R = GATEUP ? p.I : p.h;  // output rows of an expert
  constexpr int kOut = GATEUP ? kRowsPerWarp / 2 : kRowsPerWarp;
  constexpr int kTileRows = kWarps * kOut;
  const int tiles = (R + kTileRows - 1) / kTileRows;
  const int n_act = *p.n_act;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int item = blockIdx.x;; item += gridDim.x) {
    const int slot = item / tiles;
    if (slot >= n_act) break;  // uniform over the CTA
    const int e = p.act[slot];
    const int cnt = p.cnt[e], q0 = p.off[e];
    const int r_base = ((item - slot * tiles) * kWarps + warp) * kOut;
    const uint16_t* W = GATEUP ? p.gate_up + static_cast<size_t>(e) * 2 * p.I * p.h
                               : p.down + static_cast<size_t>(e) * p.h * p.I;
    const uint16_t* rows[kRowsPerWarp];
    bool live[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int out = r_base + (GATEUP ? (i % kOut) : i);
      live[i] = out < R;
      const int wrow = GATEUP ? (i < kOut ? out : p.I + out) : out;  // gate rows, then the matching up rows
      rows[i] = W + static_cast<size_t>(live[i] ? wrow : 0) * K;
    }
    for (int g0 = 0; g0 < cnt; g0 += kTG) {
      const int ng = min(kTG, cnt - g0);
      float acc[kRowsPerWarp][kTG];
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
        for (int u = 0; u < kTG; ++u) acc[i][u] = 0.f;
      for (int c0 = 0; c0 < K; c0 += kKC) {
        const int kc = min(kKC, K - c0);
        // the chunk's first weights go out before the activations are staged
        uint4 cur[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i)
          cur[i] = (live[i] && lane * 8 < kc) ? ld_weights(rows[i] + c0 + lane * 8) : make_uint4(0, 0, 0, 0);
        __syncthreads();  // the previous chunk's readers are done
        for (int idx = tid; idx < ng * kc; idx += kThreads) {
          const int u = idx / kc, kk = idx - u * kc;
          const int q = q0 + g0 + u;
          const float* src = GATEUP ? p.xn + static_cast<size_t>(p.pair_tok[q]) * K : p.f + static_cast<size_t>(q) * K;
          xs[u * kKC + kk] = src[c0 + kk];
        }
        __syncthreads();
        for (int k0 = lane * 8; k0 < kc; k0 += 256) {
          // two steps of weights in flight: the next step's loads before this step's math
          uint4 nxt[kRowsPerWarp];
          const bool more = k0 + 256 < kc;
#pragma unroll
          for (int i = 0; i < kRowsPerWarp; ++i)
            nxt[i] = (live[i] && more) ? ld_weights(rows[i] + c0 + k0 + 256) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int u = 0; u < kTG; ++u) {
            if (u < ng) {
              const float4 a = *reinterpret_cast<const float4*>(xs + u * kKC + k0);
              const float4 b = *reinterpret_cast<const float4*>(xs + u * kKC + k0 + 4);
#pragma unroll
              for (int i = 0; i < kRowsPerWarp; ++i) acc[i][u] = dot8(cur[i], a, b, acc[i][u]);
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
        for (int u = 0; u < kTG; ++u) {
          const float s0 = warp_sum(acc[i][u]);
          float val = s0;
          if constexpr (GATEUP) {
            const float up = warp_sum(acc[kOut + i][u]);
            val = (s0 / (1.0f + expf(-s0))) * up;  // silu(gate) * up
          }
          const int out = r_base + i;
          if (lane == i * kTG + u && u < ng && out < R) {
            const size_t q = static_cast<size_t>(q0 + g0 + u);
            if constexpr (GATEUP)
              p.f[q * p.I + out] = val;
            else
              p.yd[q * p.h + out] = val;
          }
        }
      }
    }
  }
}

// 4. x += sum over the token's experts, ascending expert index, of w * yd.
__global__ void __launch_bounds__(kThreads) moe_combine_kernel(const MoeDev p) {
  __shared__ int sq[kMaxTopK];
  __shared__ float sw[kMaxTopK];
  const int t = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    int es[kMaxTopK];
    for (int j = 0; j < p.k; ++j) {
      const size_t at = static_cast<size_t>(t) * p.k + j;
      int e = p.topk_idx[at], q = p.slot_q[at];
      float w = p.topk_w[at];
      int pos = j;
      while (pos > 0 && es[pos - 1] > e) {  // insertion sort by expert index
        es[pos] = es[pos - 1];
        sq[pos] = sq[pos - 1];
        sw[pos] = sw[pos - 1];
        --pos;
      }
      es[pos] = e, sq[pos] = q, sw[pos] = w;
    }
  }
  __syncthreads();
  float* xr = p.x + static_cast<size_t>(t) * p.h;
  for (int c = tid; c < p.h; c += kThreads) {
    float y = 0.f;
    for (int j = 0; j < p.k; ++j) y += sw[j] * p.yd[static_cast<size_t>(sq[j]) * p.h + c];
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
  p.slot_q = reinterpret_cast<int*>(ws + L.slot_q);
  p.f = reinterpret_cast<float*>(ws + L.f);
  p.yd = reinterpret_cast<float*>(ws + L.yd);
  p.out_idx = a->topk_index, p.out_w = a->topk_weight;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int resident[2];
  if ((e = expert_residency(device, resident)) != cudaSuccess)
    return fail(VVLI_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(e));
  const size_t logits_smem = static_cast<size_t>(p.h) * sizeof(float);       // <= 32 KB
  const size_t expert_smem = static_cast<size_t>(kTG) * kKC * sizeof(float);  // 32 KB
  moe_logits_kernel<<<dim3((p.E + kWarps - 1) / kWarps, p.T), kThreads, logits_smem, s>>>(p);
  moe_group_kernel<<<1, 1024, 0, s>>>(p);
  // persistent grids: no more CTAs than are resident at once, nor than (expert, tile) items
  const long gu_items = static_cast<long>(p.E) * ((p.I + kWarps * kRowsPerWarp / 2 - 1) / (kWarps * kRowsPerWarp / 2));
  const long dn_items = static_cast<long>(p.E) * ((p.h + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp));
  moe_expert_kernel<true><<<static_cast<unsigned>(std::min<long>(gu_items, resident[0])), kThreads, expert_smem, s>>>(p);
  moe_expert_kernel<false><<<static_cast<unsigned>(std::min<long>(dn_items, resident[1])), kThreads, expert_smem, s>>>(p);
  moe_combine_kernel<<<p.T, kThreads, 0, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VVLI_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return VVLI_OK;
}
