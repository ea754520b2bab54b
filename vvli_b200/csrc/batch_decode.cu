// batch_decode.cu - SIMT parts of a decode batch: attention of every row over
// its own sequence's paged KV cache, and the argmax of every logits row.
//
// Row b of a batch is sequence slot b: its KV pages are
// page_table[b * seq_pages ..] and its token sits at row_pos[b].  The
// attention is computeAttentionInto (src/llm.zig:1302-1335) per q head with
// an online softmax over tiles of 64 positions; long contexts split the
// positions over `splits` CTAs per (row, kv head), and the last CTA to finish
// merges the partial (o, max, sum) triples.  The output is written as the
// bf16 hi / lo pair the o_proj GEMM reads.
#include "batch.cuh"
#include "device_fns.cuh"

namespace vvli {

namespace {

constexpr int kBaThreads = 256;
constexpr int kBaTile = 64;

VVLI_DEV void split_pair(float v, uint16_t* hi, uint16_t* lo) {
  const uint16_t h = f32_to_bf16(v);
  *hi = h;
  *lo = f32_to_bf16(v - bf16_to_f32(h));
}

__global__ void __launch_bounds__(kBaThreads) batch_attention_kernel(const BatchAttnParams p) {
  extern __shared__ float sm[];
  const int G = p.group, d = p.d;
  float* qs = sm;                // [G][d]
  float* sc = qs + G * d;        // [G][kBaTile]
  float* mrun = sc + G * kBaTile;
  float* lrun = mrun + G;
  float* alpha = lrun + G;
  __shared__ int last_flag;
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = p.row_pos[b];
  const int n_ctx = pos + 1;
  const int chunk = (n_ctx + p.splits - 1) / p.splits;
  const int t_begin = s * chunk, t_end = min(n_ctx, t_begin + chunk);
  const int* pt = p.page_table + static_cast<size_t>(b) * p.seq_pages;
  const int qd = p.nq * d;
  for (int i = tid; i < G * d; i += kBaThreads) qs[i] = p.q[static_cast<size_t>(b) * qd + static_cast<size_t>(g * G) * d + i];
  for (int i = tid; i < G; i += kBaThreads) {
    mrun[i] = -INFINITY;
    lrun[i] = 0.f;
  }
  __syncthreads();
  const int nacc = (G * d + kBaThreads - 1) / kBaThreads;  // <= 4 (G <= 8, d <= 128)
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t0 = t_begin; t0 < t_end; t0 += kBaTile) {
    const int n = min(kBaTile, t_end - t0);
    // scores: one (head, position) per thread
    for (int i = tid; i < G * kBaTile; i += kBaThreads) {
      const int hh = i / kBaTile, j = i % kBaTile;
      float v = -INFINITY;
      if (j < n) {
        const float4* kr = reinterpret_cast<const float4*>(p.k_cache + kv_off(pt, t0 + j, g, p.nkv, d));
        const float4* qh = reinterpret_cast<const float4*>(qs + hh * d);
        float dot = 0.f;
        for (int e = 0; e < d / 4; ++e) {
          const float4 kk = kr[e], qq = qh[e];
          dot = fmaf(qq.x, kk.x, dot);
          dot = fmaf(qq.y, kk.y, dot);
          dot = fmaf(qq.z, kk.z, dot);
          dot = fmaf(qq.w, kk.w, dot);
        }
        v = dot * p.inv_sqrt_d;
      }
      sc[hh * kBaTile + j] = v;
    }
    __syncthreads();
    // online softmax, one warp per head (softmaxInPlace, src/llm.zig:1408-1419)
    for (int hh = warp; hh < G; hh += kBaThreads / 32) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[hh * kBaTile + j]);
      m = warp_max(m);
      const float mnew = fmaxf(mrun[hh], m);
      float l = 0.f;
      for (int j = lane; j < kBaTile; j += 32) {
        const float e = j < n ? expf(sc[hh * kBaTile + j] - mnew) : 0.f;
        sc[hh * kBaTile + j] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float a = mrun[hh] == -INFINITY ? 0.f : expf(mrun[hh] - mnew);
        alpha[hh] = a;
        lrun[hh] = lrun[hh] * a + l;
        mrun[hh] = mnew;
      }
    }
    __syncthreads();
    // P.V (addScaled, src/llm.zig:1398-1406): output element (head, dim) per thread
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = tid + k * kBaThreads;
      if (k < nacc && idx < G * d) {
        const int hh = idx / d, e = idx % d;
        float a = 0.f;
        for (int j = 0; j < n; ++j) a = fmaf(sc[hh * kBaTile + j], p.v_cache[kv_off(pt, t0 + j, g, p.nkv, d) + e], a);
        acc[k] = acc[k] * alpha[hh] + a;
      }
    }
    __syncthreads();
  }
  const size_t out_row = static_cast<size_t>(b) * qd + static_cast<size_t>(g * G) * d;
  if (p.splits == 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = tid + k * kBaThreads;
      if (k < nacc && idx < G * d) split_pair(acc[k] / lrun[idx / d], p.out_hi + out_row + idx, p.out_lo + out_row + idx);
    }
    return;
  }
  // partial (o, m, l) of this split: part[b][head][split][d + 2]
  float* part_b = p.part + static_cast<size_t>(b) * p.nq * p.splits * (d + 2);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int idx = tid + k * kBaThreads;
    if (k < nacc && idx < G * d) {
      const int hh = idx / d, e = idx % d;
      part_b[(static_cast<size_t>(g * G + hh) * p.splits + s) * (d + 2) + e] = acc[k];
    }
  }
  for (int hh = tid; hh < G; hh += kBaThreads) {
    float* q2 = part_b + (static_cast<size_t>(g * G + hh) * p.splits + s) * (d + 2);
    q2[d] = mrun[hh];
    q2[d + 1] = lrun[hh];
  }
  __threadfence();
  __syncthreads();
  unsigned* counter = p.counters + static_cast<size_t>(b) * p.nkv + g;
  if (tid == 0) last_flag = atomicAdd(counter, 1u) == static_cast<unsigned>(p.splits) - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  for (int idx = tid; idx < G * d; idx += kBaThreads) {
    const int hh = idx / d, e = idx % d;
    const float* base = part_b + static_cast<size_t>(g * G + hh) * p.splits * (d + 2);
    float M = -INFINITY;
    for (int q = 0; q < p.splits; ++q) M = fmaxf(M, __ldcg(base + q * (d + 2) + d));
    float L = 0.f, o = 0.f;
    for (int q = 0; q < p.splits; ++q) {
      const float m = __ldcg(base + q * (d + 2) + d);
      const float w = m == -INFINITY ? 0.f : expf(m - M);
      L = fmaf(__ldcg(base + q * (d + 2) + d + 1), w, L);
      o = fmaf(__ldcg(base + q * (d + 2) + e), w, o);
    }
    split_pair(o / L, p.out_hi + out_row + idx, p.out_lo + out_row + idx);
  }
  if (tid == 0) *counter = 0;
}

// llm.argmax (src/llm.zig:778-789) of every row; out[2 * b] = value, out[2 * b + 1] = index + row_base.
__global__ void __launch_bounds__(1024) rows_argmax_kernel(const float* logits, int n, int ld, int row_base, float* out) {
  __shared__ float wv[32];
  __shared__ int wi[32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* v = logits + static_cast<size_t>(b) * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < n; i += 1024)
    if (better(v[i], i, bv, bi)) {
      bv = v[i];
      bi = i;
    }
  warp_argmax(bv, bi);
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = wv[lane];
    bi = wi[lane];
    warp_argmax(bv, bi);
    if (lane == 0) {
      if (row_base == 0 && isnan(v[0])) {  // llm.argmax never replaces a NaN in element 0
        bv = v[0];
        bi = 0;
      } else if (bi == 0x7fffffff) {  // all NaN in this vocabulary shard: never the winner
        bv = __int_as_float(0x7fc00000);
      } else {
        bi += row_base;
      }
      out[2 * b] = bv;
      out[2 * b + 1] = __int_as_float(bi);
    }
  }
}

// Under tensor parallelism: the winner over the ranks' (value, index) pairs of every row.
__global__ void rows_argmax_merge_kernel(const float* all, int ranks, int B, int* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = all[2 * b];
  int bi = __float_as_int(all[2 * b + 1]);
  for (int r = 1; r < ranks; ++r) {
    const float v = all[static_cast<size_t>(r) * 2 * B + 2 * b];
    const int i = __float_as_int(all[static_cast<size_t>(r) * 2 * B + 2 * b + 1]);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  out[b] = bi;
}

__global__ void rows_argmax_index_kernel(const float* best, int B, int* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) out[b] = __float_as_int(best[2 * b + 1]);
}

}  // namespace

size_t batch_attention_smem(int group, int d) {
  return (static_cast<size_t>(group) * d + static_cast<size_t>(group) * kBaTile + 3 * group) * 4;
}

cudaError_t launch_batch_attention(const BatchAttnParams& p, int B, cudaStream_t s) {
  const dim3 grid(p.splits, p.nkv, B);
  batch_attention_kernel<<<grid, kBaThreads, batch_attention_smem(p.group, p.d), s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_rows_argmax(const float* logits, int B, int n, int ld, int row_base, float* best, cudaStream_t s) {
  rows_argmax_kernel<<<B, 1024, 0, s>>>(logits, n, ld, row_base, best);
  return cudaGetLastError();
}

cudaError_t launch_rows_argmax_merge(const float* all, int ranks, int B, int* out, cudaStream_t s) {
  rows_argmax_merge_kernel<<<(B + 127) / 128, 128, 0, s>>>(all, ranks, B, out);
  return cudaGetLastError();
}

cudaError_t launch_rows_argmax_index(const float* best, int B, int* out, cudaStream_t s) {
  rows_argmax_index_kernel<<<(B + 127) / 128, 128, 0, s>>>(best, B, out);
  return cudaGetLastError();
}

}  // namespace vvli
