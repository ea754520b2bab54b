// kernels.cu - decode-step kernels for sm_100a.
//
// One decode token per layer runs five kernels, chained with programmatic
// dependent launch (PDL) inside one CUDA graph:
//   gemv<PLAIN>   rmsnorm(x) prologue, fused q|k|v rows, + bias      (src/llm.zig:736-740)
//   attention     RoPE on q and k, KV write, flash-decode, combine   (src/llm.zig:742-755)
//   gemv<PLAIN>   o_proj + residual add                               (src/llm.zig:756-757)
//   gemv<SILU_MUL> rmsnorm prologue, gate|up rows, silu(g)*u          (src/llm.zig:759-763)
//   gemv<PLAIN>   down_proj + residual add                            (src/llm.zig:764-765)
// and the LM head is gemv<ARGMAX> with the final-norm prologue
// (src/llm.zig:727-728) and llm.argmax fused (src/llm.zig:778-789).
#include "common.cuh"
#include "kernels.h"

namespace vvli {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / kWarp;
constexpr int kItemChunks = 128;       // 16-byte chunks per work item (4 per lane)
constexpr int kItemsInFlight = 4;      // items per warp per iteration
constexpr uint32_t kPrefetchBytes = 32768;

// ---------------------------------------------------------------- block helpers
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];  // fixed order: deterministic
  return t;
}

// Fused RMSNorm prologue (rmsNormInto, src/llm.zig:1287-1300) or plain copy
// of the input vector into shared memory.
__device__ void load_input(float* xs, const float* x, const uint16_t* norm_w, float eps, int K, float* red) {
  const int tid = threadIdx.x;
  if (norm_w) {
    float ss = 0.f;
    for (int i = tid; i < K; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
    for (int i = tid; i < K; i += blockDim.x) xs[i] = x[i] * bf16_to_f32(norm_w[i]) * scale;
  } else {
    for (int i = tid * 4; i < K; i += blockDim.x * 4)
      *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
  }
}

VVLI_DEV float dot8(uint4 w, const float* xs) {
  const float4 a = *reinterpret_cast<const float4*>(xs);
  const float4 b = *reinterpret_cast<const float4*>(xs + 4);
  float acc = bf16_lo(w.x) * a.x;
  acc = fmaf(bf16_hi(w.x), a.y, acc);
  acc = fmaf(bf16_lo(w.y), a.z, acc);
  acc = fmaf(bf16_hi(w.y), a.w, acc);
  acc = fmaf(bf16_lo(w.z), b.x, acc);
  acc = fmaf(bf16_hi(w.z), b.y, acc);
  acc = fmaf(bf16_lo(w.w), b.z, acc);
  acc = fmaf(bf16_hi(w.w), b.w, acc);
  return acc;
}

// Publishes the step's argmax and advances the device step state: the token
// following position `pos` is the argmax unless it is a prompt token.
__device__ void publish_argmax(StepState* st, int* seq_tokens, int best) {
  st->argmax = best;
  const int np = st->pos + 1;
  if (np <= st->max_seq && np >= st->prompt_len) seq_tokens[np] = best;  // seq_tokens has max_seq + 1 slots
  st->pos = np;
}

// ---------------------------------------------------------------- GEMV
// y = W . x for bf16 W [N, K] and fp32 x, fp32 accumulation (linearInto,
// src/llm.zig:1228-1275).  HBM-bound: every weight byte is read once with
// 128-bit non-coherent loads.  CTA b owns the contiguous rows
// [b*N/G, (b+1)*N/G); its work is split into items of one row x up to 128
// 16-byte chunks, and every warp keeps 4 items (16 loads per lane) in flight.
// Item partial sums meet in shared memory and are added in a fixed order,
// so results are deterministic.  Before waiting on the previous kernel the
// CTA asks L2 to prefetch the head of its rows, which overlaps the launch
// gap and the previous kernel's tail.
template <int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float red[32];
  __shared__ int last_flag;
  constexpr int NPHYS = (EPI == EPI_SILU_MUL) ? 2 : 1;
  const int K = p.K, N = p.N;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = static_cast<int>((static_cast<long long>(blockIdx.x) * N) / gridDim.x);
  const int r1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * N) / gridDim.x);
  const int nrows = r1 - r0;
  const int cpr = K >> 3;
  const int S = (cpr + kItemChunks - 1) / kItemChunks;
  float* xs = smem;
  float* part = smem + K;

  if (tid == 0 && nrows > 0) {
    const size_t bytes = static_cast<size_t>(nrows) * K * 2;
    const uint32_t pre = static_cast<uint32_t>(bytes < kPrefetchBytes ? bytes : kPrefetchBytes);
#pragma unroll
    for (int ph = 0; ph < NPHYS; ++ph)
      prefetch_l2_bulk(p.W + static_cast<size_t>(r0 + ph * p.pair_offset) * K, pre);
  }
  grid_dependency_wait();
  grid_launch_dependents();

  load_input(xs, p.x, p.norm_w, p.eps, K, red);
  __syncthreads();

  const int items = nrows * NPHYS * S;
  for (int base = warp; base < items; base += kGemvWarps * kItemsInFlight) {
    uint4 w[kItemsInFlight][4];
    int cbase[kItemsInFlight];
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
      cbase[u] = sp * kItemChunks;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cbase[u] + lane + kWarp * j;
        w[u][j] = (ok && c < cpr) ? ld_stream(row + static_cast<size_t>(c) * 8) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kItemsInFlight; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cbase[u] + lane + kWarp * j;
        if (c < cpr) acc += dot8(w[u][j], xs + c * 8);
      }
      acc = warp_sum(acc);
      const int item = base + kGemvWarps * u;
      if (lane == 0 && item < items) part[item] = acc;
    }
  }
  __syncthreads();

  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (int rl = tid; rl < nrows; rl += kGemvThreads) {
    const int r = r0 + rl;
    float a = 0.f;
    if (EPI == EPI_SILU_MUL) {
      float g = 0.f, u = 0.f;
      for (int s = 0; s < S; ++s) {
        g += part[(2 * rl) * S + s];
        u += part[(2 * rl + 1) * S + s];
      }
      a = (g / (1.0f + expf(-g))) * u;  // siluMulInto, src/llm.zig:1382-1387
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
    warp_argmax(best_v, best_i);
    __shared__ float wv[kGemvWarps];
    __shared__ int wi[kGemvWarps];
    if (lane == 0) {
      wv[warp] = best_v;
      wi[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
      float bv = wv[0];
      int bi = wi[0];
      for (int i = 1; i < kGemvWarps; ++i)
        if (better(wv[i], wi[i], bv, bi)) {
          bv = wv[i];
          bi = wi[i];
        }
      p.part_val[blockIdx.x] = bv;
      p.part_idx[blockIdx.x] = bi;
      __threadfence();
      last_flag = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last_flag && tid == 0) {
      __threadfence();
      const volatile float* pv = p.part_val;
      const volatile int* pi = p.part_idx;
      float bv = pv[0];
      int bi = pi[0];
      for (unsigned b = 1; b < gridDim.x; ++b)
        if (better(pv[b], pi[b], bv, bi)) {
          bv = pv[b];
          bi = pi[b];
        }
      *p.counter = 0;
      if (p.finalize) {
        publish_argmax(p.st, p.seq_tokens, bi);
      } else {
        p.local_best[0] = bv;
        p.local_best[1] = __int_as_float(bi);
      }
    }
  }
}

size_t gemv_smem_bytes(int epi, int N, int K, int grid) {
  const int nphys = epi == EPI_SILU_MUL ? 2 : 1;
  const int S = (K / 8 + kItemChunks - 1) / kItemChunks;
  const size_t rows = (static_cast<size_t>(N) + grid - 1) / grid + 1;
  return static_cast<size_t>(K) * 4 + rows * nphys * S * 4;
}

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

cudaError_t launch_gemv(int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
  const size_t smem = gemv_smem_bytes(epi, p.N, p.K, grid);
  switch (epi) {
    case EPI_PLAIN: return launch_ex(gemv_kernel<EPI_PLAIN>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
    case EPI_SILU_MUL: return launch_ex(gemv_kernel<EPI_SILU_MUL>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
    default: return launch_ex(gemv_kernel<EPI_ARGMAX>, dim3(grid), dim3(kGemvThreads), smem, s, pdl, p);
  }
}

// ---------------------------------------------------------------- RoPE
// Inverse frequency of rotary pair `dim_index` (rotatePair, src/llm.zig:1361-1364)
// with the optional llama3 rope_scaling rule.
__device__ float rope_inv_freq(const RopeParams& r, int dim_index, int d) {
  const float exponent = static_cast<float>(dim_index) / static_cast<float>(d);
  float inv_freq = 1.0f / powf(r.theta, exponent);
  if (r.scaling == 1) {
    const float two_pi = 6.283185307179586f;
    const float low_wavelen = r.orig / r.low;
    const float high_wavelen = r.orig / r.high;
    const float wavelen = two_pi / inv_freq;
    if (wavelen > low_wavelen) {
      inv_freq = inv_freq / r.factor;
    } else if (!(wavelen < high_wavelen)) {
      const float smooth = (r.orig / wavelen - r.low) / (r.high - r.low);
      inv_freq = (1.0f - smooth) * inv_freq / r.factor + smooth * inv_freq;
    }
  }
  return inv_freq;
}

// Pair i of a head (0 <= i < d/2): element indices and the frequency index
// (applyRoPE, src/llm.zig:1337-1359).
VVLI_DEV void rope_pair(int layout, int i, int d, int& first, int& second, int& dim_index) {
  if (layout == 0) {
    first = 2 * i;
    second = 2 * i + 1;
    dim_index = 2 * i;
  } else {
    first = i;
    second = i + d / 2;
    dim_index = 2 * i;
  }
}

// ---------------------------------------------------------------- attention (decode)
// One CTA per (kv head, split of positions 0..pos).  It rotates the q heads
// of its group, and the split holding `pos` rotates the new k and writes k
// and v into the paged KV cache.  Scores (q.k/sqrt(d)) and an unnormalised
// softmax stay in shared memory; P.V is accumulated per warp.  The last CTA
// of a kv head combines the splits' (o, max, sum) into the output
// (computeAttentionInto, src/llm.zig:1302-1335).
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / kWarp;
constexpr int kMaxEpl = 8;     // head_dim <= 256
constexpr int kHeadBatch = 8;  // q heads accumulated together

VVLI_DEV const float* kv_row(const float* cache, const int* pt, int t, int g, int nkv, int d) {
  const int page = pt[t / kPage];
  return cache + (static_cast<size_t>(page * nkv + g) * kPage + (t % kPage)) * d;
}

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int last_flag;
  const int G = p.group, d = p.d;
  float* qs = sm;                      // [G][d]
  float* sc = qs + G * d;              // [G][chunk_cap]
  float* wred = sc + G * p.chunk_cap;  // [warps][kHeadBatch][d]
  float* stat = wred + kAttnWarps * kHeadBatch * d;  // [G][2]  (max, sum)
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
  const int chunk = (n_ctx + p.splits - 1) / p.splits;
  const int t0 = s * chunk;
  const int t1 = min(n_ctx, t0 + chunk);
  const int half = d / 2;

  // RoPE of this group's q heads into shared memory.
  const float* qg = p.qkv + static_cast<size_t>(g) * G * d;
  for (int idx = tid; idx < G * half; idx += kAttnThreads) {
    const int hh = idx / half, i = idx % half;
    int a, b, di;
    rope_pair(p.rope.layout, i, d, a, b, di);
    const float ang = static_cast<float>(pos) * rope_inv_freq(p.rope, di, d);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float x0 = qg[hh * d + a], x1 = qg[hh * d + b];
    qs[hh * d + a] = x0 * cs - x1 * sn;
    qs[hh * d + b] = x0 * sn + x1 * cs;
  }
  // The split that holds `pos` writes the rotated k and the v of this token.
  if (t0 < t1 && t1 == n_ctx) {
    const float* kn = p.qkv + static_cast<size_t>(p.nq) * d + static_cast<size_t>(g) * d;
    const float* vn = kn + static_cast<size_t>(p.nkv) * d;
    float* kr = const_cast<float*>(kv_row(p.k_cache, p.page_table, pos, g, p.nkv, d));
    float* vr = const_cast<float*>(kv_row(p.v_cache, p.page_table, pos, g, p.nkv, d));
    for (int i = tid; i < half; i += kAttnThreads) {
      int a, b, di;
      rope_pair(p.rope.layout, i, d, a, b, di);
      const float ang = static_cast<float>(pos) * rope_inv_freq(p.rope, di, d);
      float sn, cs;
      sincosf(ang, &sn, &cs);
      const float x0 = kn[a], x1 = kn[b];
      kr[a] = x0 * cs - x1 * sn;
      kr[b] = x0 * sn + x1 * cs;
    }
    for (int i = tid; i < d; i += kAttnThreads) vr[i] = vn[i];
  }
  __syncthreads();

  const int n = t1 > t0 ? t1 - t0 : 0;
  // Scores.
  for (int t = t0 + warp; t < t1; t += kAttnWarps) {
    const float* kr = kv_row(p.k_cache, p.page_table, t, g, p.nkv, d);
    float kv[kMaxEpl];
#pragma unroll
    for (int j = 0; j < kMaxEpl; ++j) kv[j] = (lane + kWarp * j < d) ? kr[lane + kWarp * j] : 0.f;
    for (int hh = 0; hh < G; ++hh) {
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxEpl; ++j)
        if (lane + kWarp * j < d) dot = fmaf(qs[hh * d + lane + kWarp * j], kv[j], dot);
      dot = warp_sum(dot);
      if (lane == 0) sc[hh * p.chunk_cap + (t - t0)] = dot * p.inv_sqrt_d;
    }
  }
  __syncthreads();
  // Per-head max and unnormalised exp (softmaxInPlace, src/llm.zig:1408-1419).
  for (int hh = warp; hh < G; hh += kAttnWarps) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += kWarp) m = fmaxf(m, sc[hh * p.chunk_cap + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < n; i += kWarp) {
      const float e = expf(sc[hh * p.chunk_cap + i] - m);
      sc[hh * p.chunk_cap + i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * hh] = m;
      stat[2 * hh + 1] = l;
    }
  }
  __syncthreads();
  // P.V in batches of q heads; each warp owns a stride of positions.
  for (int hb = 0; hb < G; hb += kHeadBatch) {
    const int nb = min(kHeadBatch, G - hb);
    float acc[kHeadBatch][kMaxEpl];
#pragma unroll
    for (int a = 0; a < kHeadBatch; ++a)
#pragma unroll
      for (int j = 0; j < kMaxEpl; ++j) acc[a][j] = 0.f;
    for (int t = t0 + warp; t < t1; t += kAttnWarps) {
      const float* vr = kv_row(p.v_cache, p.page_table, t, g, p.nkv, d);
      float vv[kMaxEpl];
#pragma unroll
      for (int j = 0; j < kMaxEpl; ++j) vv[j] = (lane + kWarp * j < d) ? vr[lane + kWarp * j] : 0.f;
#pragma unroll
      for (int a = 0; a < kHeadBatch; ++a) {
        if (a < nb) {
          const float pr = sc[(hb + a) * p.chunk_cap + (t - t0)];
#pragma unroll
          for (int j = 0; j < kMaxEpl; ++j) acc[a][j] = fmaf(pr, vv[j], acc[a][j]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < kHeadBatch; ++a)
#pragma unroll
      for (int j = 0; j < kMaxEpl; ++j)
        if (a < nb && lane + kWarp * j < d) wred[(warp * kHeadBatch + a) * d + lane + kWarp * j] = acc[a][j];
    __syncthreads();
    for (int idx = tid; idx < nb * d; idx += kAttnThreads) {
      const int a = idx / d, e = idx % d;
      float o = 0.f;
      for (int w = 0; w < kAttnWarps; ++w) o += wred[(w * kHeadBatch + a) * d + e];
      const int qh = g * G + hb + a;
      p.part[(static_cast<size_t>(qh) * p.splits + s) * (d + 2) + e] = o;
    }
    __syncthreads();
  }
  for (int hh = tid; hh < G; hh += kAttnThreads) {
    const int qh = g * G + hh;
    float* pp = p.part + (static_cast<size_t>(qh) * p.splits + s) * (d + 2);
    pp[d] = n > 0 ? stat[2 * hh] : -INFINITY;
    pp[d + 1] = n > 0 ? stat[2 * hh + 1] : 0.f;
  }

  // The last split of this kv head combines all splits.
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = atomicAdd(&p.counters[g], 1u) == static_cast<unsigned>(p.splits) - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  for (int idx = tid; idx < G * d; idx += kAttnThreads) {
    const int hh = idx / d, e = idx % d;
    const int qh = g * G + hh;
    const volatile float* base = p.part + static_cast<size_t>(qh) * p.splits * (d + 2);
    float M = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, base[sp * (d + 2) + d]);
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < p.splits; ++sp) {
      const float m = base[sp * (d + 2) + d];
      if (m == -INFINITY) continue;
      const float sc2 = expf(m - M);
      L = fmaf(base[sp * (d + 2) + d + 1], sc2, L);
      O = fmaf(base[sp * (d + 2) + e], sc2, O);
    }
    p.out[static_cast<size_t>(qh) * d + e] = O / L;
  }
  if (tid == 0) p.counters[g] = 0;
}

size_t attention_smem_bytes(int group, int d, int chunk_cap) {
  return (static_cast<size_t>(group) * d + static_cast<size_t>(group) * chunk_cap +
          static_cast<size_t>(kAttnWarps) * kHeadBatch * d + 2 * group) * 4;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  return launch_ex(attention_decode_kernel, dim3(p.nkv, p.splits), dim3(kAttnThreads),
                   attention_smem_bytes(p.group, p.d, p.chunk_cap), s, pdl, p);
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

template <typename Kern>
static cudaError_t allow_dynamic_smem(Kern k, int max_smem_optin) {
  // The opt-in limit covers static plus dynamic shared memory.
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k);
  if (e) return e;
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              max_smem_optin - static_cast<int>(fa.sharedSizeBytes));
}

cudaError_t configure_kernels(int max_smem_optin) {
  cudaError_t e;
  if ((e = allow_dynamic_smem(gemv_kernel<EPI_PLAIN>, max_smem_optin))) return e;
  if ((e = allow_dynamic_smem(gemv_kernel<EPI_SILU_MUL>, max_smem_optin))) return e;
  if ((e = allow_dynamic_smem(gemv_kernel<EPI_ARGMAX>, max_smem_optin))) return e;
  return allow_dynamic_smem(attention_decode_kernel, max_smem_optin);
}

}  // namespace vvli
