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
// Four launches on the caller's stream, all HBM-bound on the expert weights:
//   1. moe_route_kernel, one CTA per token: RMSNorm into the workspace, the
//      router's E dot products (a warp per expert), softmax and the top-k
//      experts (larger probability first, lower index on ties), their
//      weights (renormalised when norm_topk_prob).
//   2. moe_group_kernel, one CTA: the (token, slot) pairs grouped by expert
//      in token order, the experts' counts and offsets, and the list of the
//      experts that got a token, in ascending order.
//   3. moe_expert_kernel<true>: gate|up rows of every routed expert times its
//      tokens' normed rows, silu(gate) * up per pair; then
//      moe_expert_kernel<false>: the down rows times those.  CTA = (row
//      tile, slot in the routed-expert list): CTAs past the list's length
//      return at once, so only the routed experts' weights are read.  A
//      warp streams 8 weight rows with 16-byte loads and multiplies them
//      with up to 4 tokens staged in shared memory; an expert with more
//      tokens is taken 4 at a time (its tile comes back from L2).
//   4. moe_combine_kernel, one CTA per token: x += sum of w_e * down_e(...)
//      over the token's experts in ascending expert index (the order of the
//      OLMoE experts loop), so the result does not depend on timing.
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <cmath>
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
  size_t xn, idx, w, cnt, off, act, nact, pair_tok, slot_q, f, yd, total;
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

// 1. RMSNorm, router, softmax, top-k (OlmoeTopKRouter.forward).
__global__ void __launch_bounds__(kThreads) moe_route_kernel(const MoeDev p) {
  extern __shared__ float sh[];  // xn [h], router logits / exponentials [E]
  float* xs = sh;
  float* lg = sh + p.h;
  __shared__ float red[kWarps];
  __shared__ int sel_i[kMaxTopK];
  __shared__ float sel_v[kMaxTopK];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    xo[i] = v;
  }
  __syncthreads();
  // router logits, a warp per expert (h % 8 == 0: 16-byte rows)
  for (int e = warp; e < p.E; e += kWarps) {
    const uint16_t* wr = p.router + static_cast<size_t>(e) * p.h;
    float a = 0.f;
    for (int k0 = lane * 8; k0 < p.h; k0 += 256) {
      const uint4 u = ld_stream(wr + k0);
      a = dot8(u, *reinterpret_cast<const float4*>(xs + k0), *reinterpret_cast<const float4*>(xs + k0 + 4), a);
    }
    a = warp_sum(a);
    if (lane == 0) lg[e] = a;
  }
  __syncthreads();
  if (warp != 0) return;
  // softmax over all experts, then k rounds of a warp argmax
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
  for (int j = 0; j < p.k; ++j) {
    float bv = -1.f;
    int bi = INT_MAX;
    for (int e = lane; e < p.E; e += 32)
      if (better(lg[e], e, bv, bi)) bv = lg[e], bi = e;
    warp_argmax(bv, bi);
    if (lane == 0) {
      if (bi >= p.E) bi = 0, bv = 0.f;  // NaN logits leave no candidate: keep the index in range
      sel_i[j] = bi;
      sel_v[j] = bv / s;
      lg[bi] = -2.f;  // below every probability: not chosen again
    }
    __syncwarp();
  }
  if (lane == 0) {
    float norm = 1.f;
    if (p.norm_topk) {
      float sum = 0.f;
      for (int j = 0; j < p.k; ++j) sum += sel_v[j];
      norm = sum;
    }
    for (int j = 0; j < p.k; ++j) {
      const float w = p.norm_topk ? sel_v[j] / norm : sel_v[j];
      const size_t at = static_cast<size_t>(t) * p.k + j;
      p.topk_idx[at] = sel_i[j];
      p.topk_w[at] = w;
      if (p.out_idx) p.out_idx[at] = sel_i[j];
      if (p.out_w) p.out_w[at] = w;
    }
  }
}

// 2. Pairs grouped by expert (token order inside an expert), one CTA.
__global__ void __launch_bounds__(1024) moe_group_kernel(const MoeDev p) {
  __shared__ int cnt_s[kMaxExperts], off_s[kMaxExperts];
  const int n = p.T * p.k, tid = threadIdx.x;
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

// 3. One weight tile of one routed expert times its tokens (OlmoeExperts.forward).
//    GATEUP: rows r of gate and up (4 output rows per warp: 8 weight rows),
//            f[q][r] = silu(gate_r . xn) * (up_r . xn);
//    else:   rows r of down (8 per warp), yd[q][r] = down_r . f[q].
template <bool GATEUP>
__global__ void __launch_bounds__(kThreads) moe_expert_kernel(const MoeDev p) {
  extern __shared__ float xs[];  // [kTG][kKC]
  const int slot = blockIdx.y;
  if (slot >= *p.n_act) return;  // uniform over the CTA
  const int e = p.act[slot];
  const int cnt = p.cnt[e], q0 = p.off[e];
  const int K = GATEUP ? p.h : p.I;
  const int R = GATEUP ? p.I : p.h;  // output rows of the expert
  constexpr int kOut = GATEUP ? kRowsPerWarp / 2 : kRowsPerWarp;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r_base = (blockIdx.x * kWarps + warp) * kOut;
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
      __syncthreads();  // the previous chunk's readers are done
      for (int idx = tid; idx < kTG * kc; idx += kThreads) {
        const int u = idx / kc, kk = idx - u * kc;
        float v = 0.f;
        if (u < ng) {
          const int q = q0 + g0 + u;
          const float* src = GATEUP ? p.xn + static_cast<size_t>(p.pair_tok[q]) * K : p.f + static_cast<size_t>(q) * K;
          v = src[c0 + kk];
        }
        xs[u * kKC + kk] = v;
      }
      __syncthreads();
#pragma unroll 2
      for (int k0 = lane * 8; k0 < kc; k0 += 256) {
        uint4 wv[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) wv[i] = live[i] ? ld_stream(rows[i] + c0 + k0) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < kTG; ++u) {
          if (u < ng) {
            const float4 a = *reinterpret_cast<const float4*>(xs + u * kKC + k0);
            const float4 b = *reinterpret_cast<const float4*>(xs + u * kKC + k0 + 4);
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) acc[i][u] = dot8(wv[i], a, b, acc[i][u]);
          }
        }
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
  const size_t route_smem = static_cast<size_t>(p.h + p.E) * sizeof(float);  // <= 36 KB
  const size_t expert_smem = static_cast<size_t>(kTG) * kKC * sizeof(float);  // 32 KB
  moe_route_kernel<<<p.T, kThreads, route_smem, s>>>(p);
  moe_group_kernel<<<1, 1024, 0, s>>>(p);
  const unsigned gu_tiles = static_cast<unsigned>((p.I + kWarps * kRowsPerWarp / 2 - 1) / (kWarps * kRowsPerWarp / 2));
  const unsigned dn_tiles = static_cast<unsigned>((p.h + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp));
  moe_expert_kernel<true><<<dim3(gu_tiles, p.E), kThreads, expert_smem, s>>>(p);
  moe_expert_kernel<false><<<dim3(dn_tiles, p.E), kThreads, expert_smem, s>>>(p);
  moe_combine_kernel<<<p.T, kThreads, 0, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VVLI_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return VVLI_OK;
}
