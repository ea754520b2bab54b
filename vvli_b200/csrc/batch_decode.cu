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
#include <algorithm>
#include <cstdlib>

#include "batch.cuh"
#include "device_fns.cuh"

namespace vvli {

namespace {

constexpr int kBaThreads = 512;
constexpr int kBaTile = kPage;  // positions per tile: one KV page
constexpr int kBaMaxSlots = 8;

VVLI_DEV void split_pair(float v, uint16_t* hi, uint16_t* lo) {
  const uint16_t h = f32_to_bf16(v);
  *hi = h;
  *lo = f32_to_bf16(v - bf16_to_f32(h));
}

// CTA = (split s, kv head g, row b).  Split s owns a contiguous range of the
// row's 64-position pages; each page's K and V rows ([kPage][d] fp32, one
// contiguous block per kv head) arrive with two cp.async.bulk copies into a
// ring of `nslots` shared-memory slots.  Every warp runs its own online
// softmax over 4 positions of each page (positions 4w .. 4w + 3): lane l holds
// dims [l*DPL, (l+1)*DPL) of the key, of every q head (q in registers) and of
// the warp's output accumulators; the heads' dot products meet in a shuffle
// reduce-scatter, the 5 GH exponentials of a page are computed once each,
// spread over the lanes.  No block-wide barrier per page: a warp releases a
// slot on its `empty` barrier and thread 0 refills it once all warps have.
// At the end the 16 warps' (max, sum, o) triples merge in shared memory.
template <int GH>
VVLI_DEV int head_lane(int h) {  // a lane holding head h's sum after reduce_heads4 / reduce_heads8
  return GH == 4 ? (h >> 1) * 16 + (h & 1) * 8 : (h >> 2) * 16 + ((h >> 1) & 1) * 8 + (h & 1) * 4;
}

template <int DPL, int GH>
__global__ void __launch_bounds__(kBaThreads) batch_attention_kernel(const BatchAttnParams p) {
  constexpr int kWarps = kBaThreads / 32;
  constexpr int kPosPerWarp = kBaTile / kWarps;  // 4
  extern __shared__ __align__(128) float sm[];
  const int G = p.group, d = p.d, nslot = p.nslots;
  const int page_floats = kPage * d;
  float* kv = sm;                              // [nslot][K | V][kPage][d]
  float* qs = kv + nslot * 2 * page_floats;    // [G][d]
  float* wacc = qs + G * d;                    // [warps][G][d] the warps' output accumulators
  float* wml = wacc + kWarps * G * d;          // [warps][G][2] their (max, sum)
  float* mrun = wml + kWarps * G * 2;          // [G] merged max
  float* lrun = mrun + G;                      // [G] merged sum
  __shared__ __align__(8) uint64_t full[kBaMaxSlots];
  __shared__ __align__(8) uint64_t empty[kBaMaxSlots];
  __shared__ int last_flag;
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = p.row_pos[b];
  const int n_ctx = pos + 1;
  const int np = (n_ctx + kPage - 1) / kPage;
  const int per = (np + p.splits - 1) / p.splits;
  const int p_begin = min(np, s * per), p_end = min(np, p_begin + per);
  const int* pt = p.page_table + static_cast<size_t>(b) * p.seq_pages;
  const int qd = p.nq * d;
  grid_launch_dependents();
  if (tid == 0) {
    for (int i = 0; i < nslot; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int page, int slot) {  // thread 0
    const int rows = min(kPage, n_ctx - page * kPage);
    const uint32_t bytes = static_cast<uint32_t>(rows * d * 4);
    const size_t off = kv_off(pt, page * kPage, g, p.nkv, d);
    float* kb = kv + static_cast<size_t>(slot) * 2 * page_floats;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the slot come first
    mbar_arrive_expect_tx(&full[slot], 2 * bytes);
    bulk_g2s(kb, p.k_cache + off, bytes, &full[slot]);
    bulk_g2s(kb + page_floats, p.v_cache + off, bytes, &full[slot]);
  };
  int issued = 0;
  // Pages before the row's last one hold earlier positions only, which the
  // previous kernel (the q|k|v GEMM writing position `pos`) does not touch:
  // they are fetched before the dependency wait.
  if (tid == 0)
    for (; issued < nslot && p_begin + issued < min(p_end, np - 1); ++issued) issue(p_begin + issued, issued);
  grid_dependency_wait();
  for (int i = tid; i < G * d; i += kBaThreads) qs[i] = p.q[static_cast<size_t>(b) * qd + static_cast<size_t>(g * G) * d + i];
  __syncthreads();
  if (tid == 0)
    for (; issued < nslot && p_begin + issued < p_end; ++issued) issue(p_begin + issued, issued);
  // this lane's slice of every q head of the group, and of the warp's outputs
  const bool lane_on = lane * DPL < d;
  float qr[GH][DPL], acc[GH][DPL], m[GH], l[GH];
#pragma unroll
  for (int hh = 0; hh < GH; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      qr[hh][k] = (hh < G && lane_on) ? qs[hh * d + lane * DPL + k] : 0.f;
      acc[hh][k] = 0.f;
    }
  }
  bool ok = true;
  for (int page = p_begin, it = 0; page < p_end; ++page, ++it) {
    const int slot = it % nslot;
    if (!(ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], (it / nslot) & 1, p.err)))) break;
    const int n = min(kPage, n_ctx - page * kPage);
    const float* ks = kv + static_cast<size_t>(slot) * 2 * page_floats;
    const float* vs = ks + page_floats;
    // scores of this warp's positions for every head (all lanes)
    float sc[kPosPerWarp][GH];
#pragma unroll
    for (int jj = 0; jj < kPosPerWarp; ++jj) {
      const int j = warp * kPosPerWarp + jj;
      const bool valid = j < n;
      float kx[DPL];
      if constexpr (DPL == 4) {
        const float4 t = (valid && lane_on) ? *reinterpret_cast<const float4*>(ks + j * d + lane * 4)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        kx[0] = t.x, kx[1] = t.y, kx[2] = t.z, kx[3] = t.w;
      } else if constexpr (DPL == 2) {
        const float2 t = (valid && lane_on) ? *reinterpret_cast<const float2*>(ks + j * d + lane * 2) : make_float2(0.f, 0.f);
        kx[0] = t.x, kx[1] = t.y;
      } else {
        kx[0] = (valid && lane_on) ? ks[j * d + lane] : 0.f;
      }
      float part[GH];
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < DPL; ++k) a = fmaf(qr[hh][k], kx[k], a);
        part[hh] = a;
      }
      const float dot = GH == 4 ? reduce_heads4(part, lane) : reduce_heads8(part, lane);
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        const float v = __shfl_sync(0xffffffffu, dot, head_lane<GH>(hh));
        sc[jj][hh] = valid ? v * p.inv_sqrt_d : -INFINITY;
      }
    }
    // online softmax (softmaxInPlace, src/llm.zig:1408-1419) over the warp's
    // positions: the page's new maxima, then its 5 GH exponentials, one per
    // lane (two rounds for GH = 8), shared by shuffles
    float mnew[GH];
#pragma unroll
    for (int hh = 0; hh < GH; ++hh) {
      float bm = sc[0][hh];
#pragma unroll
      for (int jj = 1; jj < kPosPerWarp; ++jj) bm = fmaxf(bm, sc[jj][hh]);
      mnew[hh] = fmaxf(m[hh], bm);
    }
    constexpr int kNexp = (kPosPerWarp + 1) * GH;
    float e[(kNexp + 31) / 32];
#pragma unroll
    for (int r = 0; r < (kNexp + 31) / 32; ++r) {
      const int vidx = lane + 32 * r;
      float x = -INFINITY, mm = -INFINITY;
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
#pragma unroll
        for (int jj = 0; jj < kPosPerWarp; ++jj)
          if (vidx == jj * GH + hh) x = sc[jj][hh], mm = mnew[hh];
        if (vidx == kPosPerWarp * GH + hh) x = m[hh], mm = mnew[hh];
      }
      e[r] = (x == -INFINITY || mm == -INFINITY) ? 0.f : expf(x - mm);
    }
    float pr[kPosPerWarp][GH], alpha[GH];
#pragma unroll
    for (int hh = 0; hh < GH; ++hh) {
#pragma unroll
      for (int jj = 0; jj < kPosPerWarp; ++jj) {
        const int vidx = jj * GH + hh;
        pr[jj][hh] = __shfl_sync(0xffffffffu, e[vidx / 32], vidx % 32);
      }
      const int vidx = kPosPerWarp * GH + hh;
      alpha[hh] = __shfl_sync(0xffffffffu, e[vidx / 32], vidx % 32);
      float ls = 0.f;
#pragma unroll
      for (int jj = 0; jj < kPosPerWarp; ++jj) ls += pr[jj][hh];
      l[hh] = l[hh] * alpha[hh] + ls;
      m[hh] = mnew[hh];
#pragma unroll
      for (int k = 0; k < DPL; ++k) acc[hh][k] *= alpha[hh];
    }
    // P.V (addScaled, src/llm.zig:1398-1406)
#pragma unroll
    for (int jj = 0; jj < kPosPerWarp; ++jj) {
      const int j = warp * kPosPerWarp + jj;
      if (j >= n || !lane_on) continue;  // rows past n were never copied
      float vx[DPL];
      if constexpr (DPL == 4) {
        const float4 t = *reinterpret_cast<const float4*>(vs + j * d + lane * 4);
        vx[0] = t.x, vx[1] = t.y, vx[2] = t.z, vx[3] = t.w;
      } else if constexpr (DPL == 2) {
        const float2 t = *reinterpret_cast<const float2*>(vs + j * d + lane * 2);
        vx[0] = t.x, vx[1] = t.y;
      } else {
        vx[0] = vs[j * d + lane];
      }
#pragma unroll
      for (int hh = 0; hh < GH; ++hh)
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[hh][k] = fmaf(pr[jj][hh], vx[k], acc[hh][k]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done with the slot
    if (tid == 0 && p_begin + issued < p_end) {  // all warps done with it: the next page goes in
      if (!mbar_wait(&empty[slot], (it / nslot) & 1, p.err)) {
        ok = false;
      } else {
        issue(p_begin + issued, slot);
        ++issued;
      }
    }
    if (!__all_sync(0xffffffffu, ok)) break;
  }
  // a copy that never landed or a slot never released: let the copies in
  // flight finish before the CTA exits
  if (__syncthreads_or(ok ? 0 : 1)) {
    if (tid == 0)
      for (int i = max(0, issued - nslot); i < issued; ++i) mbar_wait(&full[i % nslot], (i / nslot) & 1, p.err);
    __syncthreads();
    return;
  }
  // the warps' (max, sum, o) into shared memory, merged per (head, dim)
#pragma unroll
  for (int hh = 0; hh < GH; ++hh) {
    if (hh >= G) break;
    if (lane_on)
#pragma unroll
      for (int k = 0; k < DPL; ++k) wacc[(warp * G + hh) * d + lane * DPL + k] = acc[hh][k];
    if (lane == 0) {
      wml[(warp * G + hh) * 2] = m[hh];
      wml[(warp * G + hh) * 2 + 1] = l[hh];
    }
  }
  __syncthreads();
  const int nacc = (G * d + kBaThreads - 1) / kBaThreads;  // <= 2 (G * d <= 1024)
  float o_acc[2] = {0.f, 0.f};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = tid + k * kBaThreads;
    if (k < nacc && idx < G * d) {
      const int hh = idx / d, e2 = idx % d;
      float M = -INFINITY;
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wml[(w * G + hh) * 2]);
      float L = 0.f, o = 0.f;
      for (int w = 0; w < kWarps; ++w) {
        const float mw = wml[(w * G + hh) * 2];
        const float wt = mw == -INFINITY ? 0.f : expf(mw - M);
        L = fmaf(wml[(w * G + hh) * 2 + 1], wt, L);
        o = fmaf(wacc[(w * G + hh) * d + e2], wt, o);
      }
      o_acc[k] = o;
      if (e2 == 0) {
        mrun[hh] = M;
        lrun[hh] = L;
      }
    }
  }
  __syncthreads();
  const size_t out_row = static_cast<size_t>(b) * qd + static_cast<size_t>(g * G) * d;
  if (p.splits == 1) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = tid + k * kBaThreads;
      if (k < nacc && idx < G * d) split_pair(o_acc[k] / lrun[idx / d], p.out_hi + out_row + idx, p.out_lo + out_row + idx);
    }
    return;
  }
  // partial (o, m, l) of this split: part[b][head][split][d + 2]
  float* part_b = p.part + static_cast<size_t>(b) * p.nq * p.splits * (d + 2);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int idx = tid + k * kBaThreads;
    if (k < nacc && idx < G * d) {
      const int hh = idx / d, e = idx % d;
      part_b[(static_cast<size_t>(g * G + hh) * p.splits + s) * (d + 2) + e] = o_acc[k];
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
  grid_launch_dependents();
  grid_dependency_wait();
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
  grid_dependency_wait();
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
  grid_dependency_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) out[b] = __float_as_int(best[2 * b + 1]);
}

}  // namespace

int batch_attention_slots(int d) {
  (void)d;
  const char* env = getenv("VVLI_BATCH_ATTN_SLOTS");
  if (env && atoi(env) >= 1) return std::min(kBaMaxSlots, atoi(env));
  // Two pages in flight per CTA (one CTA per SM at 512 threads): 4.87 ms per
  // 8B step at batch 16, context 512, against 5.19 with one and 4.88 with three.
  return 2;
}

int batch_attention_ctas_per_sm(int group, int d, int slots) {
  const size_t smem = batch_attention_smem(group, d, slots);
  int n = 0;
  auto occ = [&](auto kern) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kBaThreads, smem))
      n = 1;
  };
  if (group <= 4)
    d > 64 ? occ(batch_attention_kernel<4, 4>) : d > 32 ? occ(batch_attention_kernel<2, 4>) : occ(batch_attention_kernel<1, 4>);
  else
    d > 64 ? occ(batch_attention_kernel<4, 8>) : d > 32 ? occ(batch_attention_kernel<2, 8>) : occ(batch_attention_kernel<1, 8>);
  return std::max(1, n);
}

size_t batch_attention_smem(int group, int d, int slots) {
  constexpr int kWarps = kBaThreads / 32;
  return (2 * static_cast<size_t>(slots) * kPage * d + static_cast<size_t>(group) * d +
          static_cast<size_t>(kWarps) * group * d + static_cast<size_t>(kWarps) * group * 2 + 2 * group) * 4;
}

template <typename Kern, typename... Args>
static cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
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

cudaError_t launch_batch_attention(const BatchAttnParams& p, int B, cudaStream_t s, bool pdl) {
  const size_t smem = batch_attention_smem(p.group, p.d, p.nslots);
  const dim3 grid(p.splits, p.nkv, B);
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    return e ? e : launch_pdl(kern, grid, dim3(kBaThreads), smem, s, pdl, p);
  };
  if (p.group <= 4) {
    if (p.d > 64) return go(batch_attention_kernel<4, 4>);
    if (p.d > 32) return go(batch_attention_kernel<2, 4>);
    return go(batch_attention_kernel<1, 4>);
  }
  if (p.d > 64) return go(batch_attention_kernel<4, 8>);
  if (p.d > 32) return go(batch_attention_kernel<2, 8>);
  return go(batch_attention_kernel<1, 8>);
}

cudaError_t launch_rows_argmax(const float* logits, int B, int n, int ld, int row_base, float* best, cudaStream_t s,
                               bool pdl) {
  return launch_pdl(rows_argmax_kernel, dim3(B), dim3(1024), 0, s, pdl, logits, n, ld, row_base, best);
}

cudaError_t launch_rows_argmax_merge(const float* all, int ranks, int B, int* out, cudaStream_t s) {
  rows_argmax_merge_kernel<<<(B + 127) / 128, 128, 0, s>>>(all, ranks, B, out);
  return cudaGetLastError();
}

// Each thread first stores its elements to every rank as one 8-byte word
// (epoch, value) — stored and loaded whole, so no fence or flag is needed —
// then polls its own block until every rank's word for those elements has
// the epoch.  All CTAs are resident (grid <= 2 per SM), so a rank never waits
// for a peer CTA that has not started.
__global__ void __launch_bounds__(256) tp_exchange_kernel(const float* src, int n, float* dst, int gather,
                                                          const TpExchange x) {
  const int stride = gridDim.x * blockDim.x;
  const size_t par = static_cast<size_t>(x.epoch & 1) * x.tp * x.cap;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const unsigned long long w = (static_cast<unsigned long long>(x.epoch) << 32) | __float_as_uint(src[i]);
    for (int q = 0; q < x.tp; ++q)
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(x.block[q] + par + static_cast<size_t>(x.rank) * x.cap + i),
                   "l"(w)
                   : "memory");
  }
  const unsigned long long* own = x.block[x.rank] + par;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float sum = 0.f;
    for (int q = 0; q < x.tp; ++q) {
      const unsigned long long* wp = own + static_cast<size_t>(q) * x.cap + i;
      unsigned long long v;
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 0;; ++it) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(wp) : "memory");
        if (static_cast<unsigned>(v >> 32) == x.epoch) break;
        if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
          atomicExch(x.err, kErrTimeout);
          v = 0;
          break;
        }
      }
      const float f = __uint_as_float(static_cast<unsigned>(v));
      if (gather)
        dst[static_cast<size_t>(q) * n + i] = f;
      else
        sum += f;
    }
    if (!gather) dst[i] = sum;
  }
}

cudaError_t launch_tp_exchange(const float* src, int n, float* dst, int gather, const TpExchange& x, int sm_count,
                               cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (n > x.cap || x.tp > kTpxMax || x.epoch == 0) return cudaErrorInvalidValue;
  const int grid = std::max(1, std::min((n + 255) / 256, 2 * sm_count));
  tp_exchange_kernel<<<grid, 256, 0, s>>>(src, n, dst, gather, x);
  return cudaGetLastError();
}

cudaError_t launch_rows_argmax_index(const float* best, int B, int* out, cudaStream_t s, bool pdl) {
  return launch_pdl(rows_argmax_index_kernel, dim3((B + 127) / 128), dim3(128), 0, s, pdl, best, B, out);
}

}  // namespace vvli
