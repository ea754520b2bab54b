// attn_tc.cu - causal prompt attention on the tensor cores (tcgen05, TMEM).
//
// computeAttentionInto (src/llm.zig:1302-1335) for every token of a prompt
// chunk, all q heads of one kv head per CTA, in flash form:
//   * CTA = (kv head g, block of 128 / G tokens): its 128 query rows are the
//     group's q heads x tokens (row r = token r / G, head r % G), the M of
//     every MMA.  Keys come in tiles of 64 positions, one KV page.
//   * The reference works in fp32; q, k, v, and the probabilities enter the
//     tensor cores as bf16 hi + lo pairs (v = hi + lo to about 16 bits), and
//     each product is hi.hi + hi.lo + lo.hi: three kind::f16 MMAs into one
//     fp32 accumulator in TMEM (the dropped lo.lo term is below fp32
//     rounding of the sum).
//   * S = Q K^T (128 x 64) lands in TMEM; each of the 128 worker threads owns
//     one query row (one TMEM lane), so the online softmax (scale, causal
//     mask, running max and sum) needs no shuffles.  P (hi / lo) goes to
//     shared memory as the A operand of P V; P V (128 x d) lands in TMEM and
//     is added to the row's output kept in registers, O = O * alpha + P V.
//   * Operands are written to shared memory by the worker threads in the
//     layout a 128-byte-swizzled TMA load would produce (rows of 128 bytes,
//     the 16-byte chunk c of row r stored at chunk c ^ (r % 8), 8-row groups
//     of 1024 bytes), K-major: Q and K by rows, V transposed (d rows of 64
//     keys) so it is the K-major B operand of P V.
//   * Warp 0 allocates TMEM and one of its threads issues the MMAs; warps
//     1-4 (TMEM lanes 32 (w % 4) ..) convert operands, run the softmax and
//     keep the output.  Every wait is bounded.
#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "device_fns.cuh"
#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace vvli {

namespace {

constexpr int kAtRows = 128;   // query rows per CTA: M of every MMA, TMEM lanes
constexpr int kAtKeys = 64;    // keys per tile: one KV page
constexpr int kAtWorkers = 128;
constexpr int kAtThreads = 32 + kAtWorkers;

template <int D>
struct AtLayout {
  static constexpr uint32_t q_tile = kAtRows * D * 2;         // bytes of Q hi (or lo): D / 64 atoms of 128 rows
  static constexpr uint32_t k_tile = kAtKeys * D * 2;         // D / 64 atoms of 64 rows
  static constexpr uint32_t v_tile = D * kAtKeys * 2;         // one atom of D rows (64 keys)
  static constexpr uint32_t p_tile = kAtRows * kAtKeys * 2;   // one atom of 128 rows
  static constexpr uint32_t q_hi = 0, q_lo = q_hi + q_tile;
  static constexpr uint32_t k_hi = q_lo + q_tile, k_lo = k_hi + k_tile;
  static constexpr uint32_t v_hi = k_lo + k_tile, v_lo = v_hi + v_tile;
  static constexpr uint32_t p_hi = v_lo + v_tile, p_lo = p_hi + p_tile;
  static constexpr uint32_t bars = p_lo + p_tile;             // 4 mbarriers + TMEM address
  static constexpr uint32_t smem = bars + 64 + 1024;          // + alignment slack
  static constexpr uint32_t tmem_cols = 64 + D <= 128 ? 128 : 256;  // S at column 0, P V at column 64
  static constexpr uint32_t s_idesc = umma_idesc(kAtRows, kAtKeys);
  static constexpr uint32_t pv_idesc = umma_idesc(kAtRows, D);
};

// Byte offset of the 16-byte chunk holding elements [8c, 8c + 8) of row r in
// a K-major, 128-byte-swizzled tile of `rows` rows (K split in 64-element atoms).
VVLI_DEV uint32_t sw_chunk(int rows, int r, int c) {
  return static_cast<uint32_t>((c >> 3) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// hi / lo bf16 pairs of 8 floats, packed as two 16-byte chunks.
VVLI_DEV void split8(const float* v, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint16_t h0, l0, h1, l1;
    split_bf16(v[2 * i], h0, l0);
    split_bf16(v[2 * i + 1], h1, l1);
    h[i] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
    l[i] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

VVLI_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(kAtThreads, 1) prefill_attn_tc_kernel(const PrefillAttnParams p) {
  using L = AtLayout<D>;
  extern __shared__ uint8_t at_raw[];
  const uint32_t raw = smem_u32(at_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  uint8_t* sm = at_raw + (base - raw);
  uint64_t* kv_ready = reinterpret_cast<uint64_t*>(sm + L::bars);  // workers wrote Q (first tile), K, V
  uint64_t* s_full = kv_ready + 1;                                  // S = Q K^T is in TMEM
  uint64_t* p_ready = kv_ready + 2;                                 // workers wrote P
  uint64_t* pv_full = kv_ready + 3;                                 // P V is in TMEM
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(kv_ready + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group, g = blockIdx.x;
  const int BQ = kAtRows / G;
  const int t0 = blockIdx.y * BQ;
  const int nt = min(BQ, p.M - t0);
  const int rows = G * nt;
  const int last_pos = p.pos0 + t0 + nt - 1;
  const int ntiles = (last_pos + kAtKeys) / kAtKeys;
  const int qd = p.nq * D;

  if (threadIdx.x == 0) {
    mbar_init(kv_ready, kAtWorkers);
    mbar_init(s_full, 1);
    mbar_init(p_ready, kAtWorkers);
    mbar_init(pv_full, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(L::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // ---- MMA issuer
      int ns = 0, npv = 0;  // commits issued
      for (int j = 0; j < ntiles; ++j) {
        if (!mbar_wait(kv_ready, j & 1, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {  // S = Q K^T over d, 16 per MMA
          const uint32_t ka = (ks >> 2) * (kAtRows * 128) + (ks & 3) * 32;
          const uint32_t kb = (ks >> 2) * (kAtKeys * 128) + (ks & 3) * 32;
          const uint64_t qh = umma_desc(base + L::q_hi + ka), ql = umma_desc(base + L::q_lo + ka);
          const uint64_t kh = umma_desc(base + L::k_hi + kb), kl = umma_desc(base + L::k_lo + kb);
          umma_bf16(tmem, qh, kh, L::s_idesc, ks != 0);
          umma_bf16(tmem, qh, kl, L::s_idesc, 1u);
          umma_bf16(tmem, ql, kh, L::s_idesc, 1u);
        }
        umma_commit(s_full);
        ++ns;
        if (!mbar_wait(p_ready, j & 1, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kAtKeys / 16; ++ks) {  // P V over the tile's keys
          const uint64_t ph = umma_desc(base + L::p_hi + ks * 32), pl = umma_desc(base + L::p_lo + ks * 32);
          const uint64_t vh = umma_desc(base + L::v_hi + ks * 32), vl = umma_desc(base + L::v_lo + ks * 32);
          umma_bf16(tmem + 64, ph, vh, L::pv_idesc, ks != 0);
          umma_bf16(tmem + 64, ph, vl, L::pv_idesc, 1u);
          umma_bf16(tmem + 64, pl, vh, L::pv_idesc, 1u);
        }
        umma_commit(pv_full);
        ++npv;
      }
      // Every MMA has finished before TMEM is released (already so unless a wait gave up).
      if (ns > 0) mbar_wait(s_full, (ns - 1) & 1, p.err);
      if (npv > 0) mbar_wait(pv_full, (npv - 1) & 1, p.err);
    }
  } else {  // ---- workers: row R = TMEM lane
    const int wt = threadIdx.x - 32;  // 0 .. 127
    const int R = 32 * (warp & 3) + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    const int qpos = R < rows ? p.pos0 + t0 + R / G : -1;
    // Q (hi / lo), zero rows past `rows`
    for (int it = wt; it < kAtRows * (D / 8); it += kAtWorkers) {
      const int r = it / (D / 8), c = it % (D / 8);
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (r < rows) {
        const float4* src = reinterpret_cast<const float4*>(
            p.q + static_cast<size_t>(t0 + r / G) * qd + static_cast<size_t>(g * G + r % G) * D + c * 8);
        const float4 a = src[0], b = src[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
      }
      uint4 hi, lo;
      split8(v, hi, lo);
      const uint32_t off = sw_chunk(kAtRows, r, c);
      *reinterpret_cast<uint4*>(sm + L::q_hi + off) = hi;
      *reinterpret_cast<uint4*>(sm + L::q_lo + off) = lo;
    }
    float o[D];
#pragma unroll
    for (int e = 0; e < D; ++e) o[e] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int j0 = j * kAtKeys;
      const int nkeys = min(kAtKeys, last_pos + 1 - j0);
      const size_t kvb = kv_off(p.page_table, j0, g, p.nkv, D);  // the tile's rows are contiguous
      // K by rows (zero past nkeys)
      for (int it = wt; it < kAtKeys * (D / 8); it += kAtWorkers) {
        const int r = it / (D / 8), c = it % (D / 8);
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (r < nkeys) {
          const float4* src = reinterpret_cast<const float4*>(p.k_cache + kvb + static_cast<size_t>(r) * D + c * 8);
          const float4 a = __ldcg(src), b = __ldcg(src + 1);
          v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        }
        uint4 hi, lo;
        split8(v, hi, lo);
        const uint32_t off = sw_chunk(kAtKeys, r, c);
        *reinterpret_cast<uint4*>(sm + L::k_hi + off) = hi;
        *reinterpret_cast<uint4*>(sm + L::k_lo + off) = lo;
      }
      // V transposed: item (dims 8eb.., keys 8jc..) -> 8 chunks, one per dim (zero past nkeys)
      for (int it = wt; it < (D / 8) * (kAtKeys / 8); it += kAtWorkers) {
        const int eb = it % (D / 8), jc = it / (D / 8);
        float t[8][8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int key = 8 * jc + jj;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
          if (key < nkeys) {
            const float4* src =
                reinterpret_cast<const float4*>(p.v_cache + kvb + static_cast<size_t>(key) * D + eb * 8);
            a = __ldcg(src), b = __ldcg(src + 1);
          }
          t[0][jj] = a.x, t[1][jj] = a.y, t[2][jj] = a.z, t[3][jj] = a.w;
          t[4][jj] = b.x, t[5][jj] = b.y, t[6][jj] = b.z, t[7][jj] = b.w;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          uint4 hi, lo;
          split8(t[e], hi, lo);
          const uint32_t off = sw_chunk(D, 8 * eb + e, jc);
          *reinterpret_cast<uint4*>(sm + L::v_hi + off) = hi;
          *reinterpret_cast<uint4*>(sm + L::v_lo + off) = lo;
        }
      }
      fence_async_smem();  // generic-proxy writes, read by the tensor cores
      tc_fence_before();   // this thread's TMEM loads of the last tile come first
      mbar_arrive(kv_ready);
      // ---- softmax of S (softmaxInPlace, src/llm.zig:1408-1419, online form)
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      float s[kAtKeys];
      tmem_ld32(trow, s);
      tmem_ld32(trow + 32, s + 32);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAtKeys; ++c) {
        s[c] = (c < nkeys && j0 + c <= qpos) ? s[c] * p.inv_sqrt_d : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const float mnew = fmaxf(m, mt);
      const float alpha = m == -INFINITY ? 0.f : expf(m - mnew);
      float sum = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < kAtKeys / 8; ++c8) {
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pv[i] = mnew == -INFINITY ? 0.f : expf(s[8 * c8 + i] - mnew);
          sum += pv[i];
        }
        uint4 hi, lo;
        split8(pv, hi, lo);
        const uint32_t off = sw_chunk(kAtRows, R, c8);
        *reinterpret_cast<uint4*>(sm + L::p_hi + off) = hi;
        *reinterpret_cast<uint4*>(sm + L::p_lo + off) = lo;
      }
      l = l * alpha + sum;
      m = mnew;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
      // ---- O = O * alpha + P V (addScaled, src/llm.zig:1398-1406)
      ok = __all_sync(0xffffffffu, mbar_wait(pv_full, j & 1, p.err));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float v[32];
        tmem_ld32(trow + 64 + cc * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[cc * 32 + i] = fmaf(o[cc * 32 + i], alpha, v[i]);
      }
    }
    if (ok && R < rows) {
      const size_t orow = static_cast<size_t>(t0 + R / G) * qd + static_cast<size_t>(g * G + R % G) * D;
      const float inv = 1.0f / l;
#pragma unroll
      for (int e = 0; e < D; ++e) split_bf16(o[e] * inv, p.out_hi[orow + e], p.out_lo[orow + e]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols) : "memory");
  }
}

template <int D>
cudaError_t launch_at(const PrefillAttnParams& p, cudaStream_t s) {
  const int BQ = kAtRows / p.group;
  const dim3 grid(p.nkv, (p.M + BQ - 1) / BQ);
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(AtLayout<D>::smem));
  if (e) return e;
  prefill_attn_tc_kernel<D><<<grid, kAtThreads, AtLayout<D>::smem, s>>>(p);
  return cudaGetLastError();
}

__global__ void fill_f32_kernel(float* p, size_t n, uint64_t key, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
    p[i] = scale * (static_cast<float>(h >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f);
  }
}

// max |a - b| over the hi + lo outputs of two kernels, and max |b|.
__global__ void compare_pairs_kernel(const uint16_t* ah, const uint16_t* al, const uint16_t* bh, const uint16_t* bl,
                                     size_t n, float* out) {
  float d = 0.f, mx = 0.f;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float a = bf16_to_f32(ah[i]) + bf16_to_f32(al[i]);
    const float b = bf16_to_f32(bh[i]) + bf16_to_f32(bl[i]);
    d = fmaxf(d, fabsf(a - b));
    mx = fmaxf(mx, fabsf(b));
    if (a != a) d = INFINITY;  // NaN
  }
  atomicMax(reinterpret_cast<int*>(out), __float_as_int(d));
  atomicMax(reinterpret_cast<int*>(out) + 1, __float_as_int(mx));
}

}  // namespace

cudaError_t attention_tc_selftest(int d, int group, int M, int pos0, uint64_t seed, float* max_rel_err) {
  const int nkv = 2, nq = nkv * group, total = pos0 + M, pages = (total + kPage - 1) / kPage;
  const size_t qn = static_cast<size_t>(M) * nq * d, kvn = static_cast<size_t>(pages) * nkv * kPage * d;
  float *q = nullptr, *kc = nullptr, *vc = nullptr, *res = nullptr;
  uint16_t* outs = nullptr;
  int *pt = nullptr, *err = nullptr;
  cudaError_t e;
  auto cleanup = [&]() { cudaFree(q), cudaFree(kc), cudaFree(vc), cudaFree(res), cudaFree(outs), cudaFree(pt), cudaFree(err); };
  if ((e = cudaMalloc(&q, qn * 4)) || (e = cudaMalloc(&kc, kvn * 4)) || (e = cudaMalloc(&vc, kvn * 4)) ||
      (e = cudaMalloc(&res, 8)) || (e = cudaMalloc(&outs, 4 * qn * 2)) || (e = cudaMalloc(&pt, pages * 4)) ||
      (e = cudaMalloc(&err, 4))) {
    cleanup();
    return e;
  }
  std::vector<int> hpt(pages);
  for (int i = 0; i < pages; ++i) hpt[i] = (i * 7 + 3) % pages;  // a scrambled page table
  cudaMemcpy(pt, hpt.data(), pages * 4, cudaMemcpyHostToDevice);
  cudaMemset(res, 0, 8);
  cudaMemset(err, 0, 4);
  fill_f32_kernel<<<256, 256>>>(q, qn, seed * 5 + 1, 2.0f);
  fill_f32_kernel<<<256, 256>>>(kc, kvn, seed * 5 + 2, 2.0f);
  fill_f32_kernel<<<256, 256>>>(vc, kvn, seed * 5 + 3, 1.0f);
  PrefillAttnParams a{q, kc, vc, pt, outs, outs + qn, M, nq, nkv, d, group, pos0, 1.0f / sqrtf(static_cast<float>(d)), err};
  PrefillAttnParams b = a;
  b.out_hi = outs + 2 * qn, b.out_lo = outs + 3 * qn;
  if ((e = launch_prefill_attention_simt(a, 0)) || (e = launch_prefill_attention_tc(b, 0))) {
    cleanup();
    return e;
  }
  compare_pairs_kernel<<<256, 256>>>(b.out_hi, b.out_lo, a.out_hi, a.out_lo, qn, res);
  float h[2] = {0.f, 0.f};
  int herr = 0;
  e = cudaMemcpy(h, res, 8, cudaMemcpyDeviceToHost);
  if (!e) e = cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
  cleanup();
  if (e) return e;
  *max_rel_err = herr ? INFINITY : h[0] / fmaxf(h[1], 1e-30f);
  return cudaSuccess;
}

bool prefill_attention_tc_supported(int d, int group) { return (d == 64 || d == 128) && group >= 1 && group <= 8; }

cudaError_t launch_prefill_attention_tc(const PrefillAttnParams& p, cudaStream_t s) {
  if (!prefill_attention_tc_supported(p.d, p.group)) return cudaErrorInvalidValue;
  return p.d == 128 ? launch_at<128>(p, s) : launch_at<64>(p, s);
}

}  // namespace vvli
