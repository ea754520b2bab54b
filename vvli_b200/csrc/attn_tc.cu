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
//   * S = Q K^T (128 x 64) lands in TMEM (two buffers: S of tile j + 2 is
//     computed while the softmax works on tile j + 1); two softmax threads
//     own one query row (one TMEM lane), 32 key columns each, so the online
//     softmax (scale, causal mask, running max and sum) needs no shuffles.  P (hi / lo) goes to
//     shared memory as the A operand of P V, which accumulates O (128 x d) in
//     TMEM; when a row's max moves, its O is rescaled in TMEM first.
//   * Operands are written to shared memory by the worker threads in the
//     layout a 128-byte-swizzled TMA load would produce (rows of 128 bytes,
//     the 16-byte chunk c of row r stored at chunk c ^ (r % 8), 8-row groups
//     of 1024 bytes), K-major: Q and K by rows, V transposed (d rows of 64
//     keys) so it is the K-major B operand of P V.
//   * A pre-pass (kv_tiles_kernel) writes every 64-position tile of the
//     layer's K and V, once, as the hi / lo image of a shared-memory K / V
//     buffer; an attention CTA fetches each tile with one bulk copy into a
//     double buffer, so the many query blocks that read a tile do not
//     convert it again.
//   * Warps 0-7 convert Q, then run the softmax and write the output: warp w
//     takes TMEM lanes 32 (w % 4) .. and key columns 32 (w / 4) .., the two
//     halves of a row meeting once per tile for the row max; warp 8
//     allocates TMEM and one of its threads issues the K / V copies and the
//     MMAs, whichever is ready first.  Every wait is bounded.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "device_fns.cuh"
#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace vvli {

namespace {

constexpr int kAtRows = 128;        // query rows per CTA: M of every MMA, TMEM lanes
constexpr int kAtKeys = 64;         // keys per tile: one KV page
constexpr int kAtSoftmax = 256;     // warps 0-7: row 32 (w % 4) + lane, key columns 32 (w / 4) ..
constexpr int kAtConv = 128;        // threads of the K / V pre-pass
constexpr int kAtThreads = kAtSoftmax + 32;  // warp 8: TMEM, the K / V copies and the MMAs
// A row's reference max moves only when a score exceeds it by more than
// this (natural log): exp(s - m) then stays below e^8, so the output in TMEM
// is rescaled rarely; the result is the same up to fp32 rounding.
constexpr float kAtRescale = 8.0f;

template <int D>
struct AtLayout {
  static constexpr uint32_t q_tile = kAtRows * D * 2;         // bytes of Q hi (or lo): D / 64 atoms of 128 rows
  static constexpr uint32_t k_tile = kAtKeys * D * 2;         // D / 64 atoms of 64 rows
  static constexpr uint32_t v_tile = D * kAtKeys * 2;         // one atom of D rows (64 keys)
  static constexpr uint32_t p_tile = kAtRows * kAtKeys * 2;   // one atom of 128 rows
  static constexpr uint32_t kv_buf = 2 * k_tile + 2 * v_tile;  // K hi, K lo, V^T hi, V^T lo
  static constexpr uint32_t k_hi = 0, k_lo = k_tile, v_hi = 2 * k_tile, v_lo = 2 * k_tile + v_tile;  // in a buffer
  static constexpr uint32_t q_hi = 0, q_lo = q_tile;
  static constexpr uint32_t kv0 = 2 * q_tile;                 // two K / V buffers (tile j uses j % 2)
  static constexpr uint32_t p_hi = kv0 + 2 * kv_buf, p_lo = p_hi + p_tile;
  static constexpr uint32_t bars = p_lo + p_tile;             // 9 mbarriers + TMEM address
  static constexpr uint32_t smem = bars + 128 + 1024;         // + alignment slack
  static constexpr uint32_t o_col = 128;                      // S of even / odd tiles at columns 0 / 64, O at 128
  static constexpr uint32_t tmem_cols = 256;
  static constexpr uint32_t s_idesc = umma_idesc(kAtRows, kAtKeys);
  static constexpr uint32_t pv_idesc = umma_idesc(kAtRows, D);
};

// Byte offset of the 16-byte chunk holding elements [8c, 8c + 8) of row r in
// a K-major, 128-byte-swizzled tile of `rows` rows (K split in 64-element atoms).
VVLI_DEV uint32_t sw_chunk(int rows, int r, int c) {
  return static_cast<uint32_t>((c >> 3) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// hi / lo bf16 pairs (round to nearest even) of 8 floats, packed as two 16-byte chunks.
VVLI_DEV void split8(const float* v, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 hb = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    const float2 hf = __bfloat1622float2(hb);
    const __nv_bfloat162 lb = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&hb);
    l[i] = *reinterpret_cast<const uint32_t*>(&lb);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

VVLI_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

VVLI_DEV void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Rows [r0, r0 + n * 128 / (D / 8)) of a row-major fp32 source -> hi / lo
// chunks of a swizzled tile: N items per converter thread, item i = (row,
// chunk) of index ct + i * 128; all loads are issued before the first store.
template <int D, int N, typename Src>
VVLI_DEV void convert_rows(Src src, int nrows_valid, int tile_rows, uint8_t* hi, uint8_t* lo, int ct) {
  float4 a[N][2];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int it = ct + i * kAtConv, r = it / (D / 8), c = it % (D / 8);
    if (r < nrows_valid) {
      const float4* p = src(r, c);
      a[i][0] = __ldcg(p), a[i][1] = __ldcg(p + 1);
    } else {
      a[i][0] = a[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int it = ct + i * kAtConv, r = it / (D / 8), c = it % (D / 8);
    const float v[8] = {a[i][0].x, a[i][0].y, a[i][0].z, a[i][0].w, a[i][1].x, a[i][1].y, a[i][1].z, a[i][1].w};
    uint4 h, l;
    split8(v, h, l);
    const uint32_t off = sw_chunk(tile_rows, r, c);
    *reinterpret_cast<uint4*>(hi + off) = h;
    *reinterpret_cast<uint4*>(lo + off) = l;
  }
}

// One tile (64 positions) of kv head g of a layer's K and V into the image of
// a shared-memory K / V buffer (K hi, K lo by rows; V^T hi, V^T lo), rows past
// nkeys zero.  128 threads.
template <int D>
VVLI_DEV void convert_kv_tile(const float* k_tile, const float* v_tile, int nkeys, uint8_t* kvb, int ct) {
  using L = AtLayout<D>;
  // K by rows
  convert_rows<D, D / 16>(
      [&](int r, int c) { return reinterpret_cast<const float4*>(k_tile + static_cast<size_t>(r) * D + c * 8); },
      nkeys, kAtKeys, kvb + L::k_hi, kvb + L::k_lo, ct);
  // V transposed: item (dims 8eb.., keys 8jc..) -> 8 chunks, one per dim
  if (ct < D) {
    // the 8 threads of a key chunk group write one row's 8 chunks (no bank conflicts in shared memory)
    const int jc = ct % 8, eb = ct / 8;
    float t[8][8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int key = 8 * jc + jj;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (key < nkeys) {
        const float4* src = reinterpret_cast<const float4*>(v_tile + static_cast<size_t>(key) * D + eb * 8);
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
      *reinterpret_cast<uint4*>(kvb + L::v_hi + off) = hi;
      *reinterpret_cast<uint4*>(kvb + L::v_lo + off) = lo;
    }
  }
}

// Pre-pass: every tile (64 positions) of positions [0, npos) of every kv head
// as the hi / lo image of a K / V buffer, tiles[(tile * nkv + g)], so the
// attention CTAs (many per tile) copy them instead of converting them again.
template <int D>
__global__ void __launch_bounds__(kAtConv) kv_tiles_kernel(const float* k_cache, const float* v_cache,
                                                           const int* page_table, int npos, int nkv, uint8_t* tiles) {
  using L = AtLayout<D>;
  const int j = blockIdx.x, g = blockIdx.y;
  const int nkeys = min(kAtKeys, npos - j * kAtKeys);
  const size_t tb = kv_off(page_table, j * kAtKeys, g, nkv, D);  // the tile's rows are contiguous
  convert_kv_tile<D>(k_cache + tb, v_cache + tb, nkeys, tiles + (static_cast<size_t>(j) * nkv + g) * L::kv_buf,
                     threadIdx.x);
}

template <int D>
__global__ void __launch_bounds__(kAtThreads, 1) prefill_attn_tc_kernel(const PrefillAttnParams p) {
  using L = AtLayout<D>;
  extern __shared__ uint8_t at_raw[];
  const uint32_t raw = smem_u32(at_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  uint8_t* sm = at_raw + (base - raw);
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(sm + L::bars);  // [2] converters wrote K / V (and Q)
  uint64_t* kv_empty = kv_full + 2;                                 // [2] the MMAs that read a buffer are done
  uint64_t* s_full = kv_full + 4;                                   // [2] S = Q K^T of an even / odd tile is in TMEM
  uint64_t* p_ready = kv_full + 6;                                  // softmax wrote P (and rescaled O)
  uint64_t* pv_full = kv_full + 7;                                  // O += P V is done
  uint64_t* q_ready = kv_full + 8;                                  // converters wrote Q
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(kv_full + 9);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group, g = blockIdx.x;
  const int BQ = kAtRows / G;
  // Token blocks in reverse: the later blocks see more keys (causal), so the
  // longest CTAs start in the first wave and the short ones fill the tail.
  const int t0 = (gridDim.y - 1 - blockIdx.y) * BQ;
  const int nt = min(BQ, p.M - t0);
  const int rows = G * nt;
  const int last_pos = p.pos0 + t0 + nt - 1;
  const int ntiles = (last_pos + kAtKeys) / kAtKeys;
  const int qd = p.nq * D;

  if (threadIdx.x == 0) {
    mbar_init(&kv_full[0], 1);  // the K / V copy: one arrival with its byte count
    mbar_init(&kv_full[1], 1);
    mbar_init(q_ready, kAtSoftmax);
    mbar_init(&kv_empty[0], 1);
    mbar_init(&kv_empty[1], 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_ready, kAtSoftmax);
    mbar_init(pv_full, 1);
    fence_barrier_init();
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(L::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 8) {
    if (lane == 0) {  // ---- MMA issuer
      // The start address is the descriptor's low field (address >> 4, smem < 256 KB):
      // an operand at base + off has descriptor desc(base) + (off >> 4).
      const uint64_t dq_hi = umma_desc(base + L::q_hi), dq_lo = umma_desc(base + L::q_lo);
      const uint64_t dp_hi = umma_desc(base + L::p_hi), dp_lo = umma_desc(base + L::p_lo);
      const uint64_t dkv0 = umma_desc(base + L::kv0);
      // S of tile j into columns 64 (j % 2).  The thread issues whichever is
      // ready first: P V of the next tile once its P is written, or S of a
      // later tile once its K / V are in and its S buffer has been read (the
      // P V of the tile two before was issued), so neither waits on the other.
      auto issue_s = [&](int j) {
        tc_fence_after();
        const uint32_t kvo = (j & 1) * L::kv_buf;  // this tile's K / V buffer, from kv0
        const uint32_t sacc = tmem + static_cast<uint32_t>((j & 1) * 64);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {  // S = Q K^T over d, 16 per MMA
          const uint32_t ka = (ks >> 2) * (kAtRows * 128) + (ks & 3) * 32;
          const uint32_t kb = (ks >> 2) * (kAtKeys * 128) + (ks & 3) * 32;
          const uint64_t qh = dq_hi + (ka >> 4), ql = dq_lo + (ka >> 4);
          const uint64_t kh = dkv0 + ((kvo + L::k_hi + kb) >> 4), kl = dkv0 + ((kvo + L::k_lo + kb) >> 4);
          umma_bf16(sacc, qh, kh, L::s_idesc, ks != 0);
          umma_bf16(sacc, qh, kl, L::s_idesc, 1u);
          umma_bf16(sacc, ql, kh, L::s_idesc, 1u);
        }
        umma_commit(&s_full[j & 1]);
      };
      auto issue_pv = [&](int j) {
        tc_fence_after();
        const uint32_t kvo = (j & 1) * L::kv_buf;
#pragma unroll
        for (int ks = 0; ks < kAtKeys / 16; ++ks) {  // O += P V over the tile's keys
          const uint64_t ph = dp_hi + (ks * 32 >> 4), pl = dp_lo + (ks * 32 >> 4);
          const uint64_t vh = dkv0 + ((kvo + L::v_hi + ks * 32) >> 4), vl = dkv0 + ((kvo + L::v_lo + ks * 32) >> 4);
          umma_bf16(tmem + L::o_col, ph, vh, L::pv_idesc, (j | ks) != 0);
          umma_bf16(tmem + L::o_col, ph, vl, L::pv_idesc, 1u);
          umma_bf16(tmem + L::o_col, pl, vh, L::pv_idesc, 1u);
        }
        umma_commit(pv_full);
        umma_commit(&kv_empty[j & 1]);
      };
      // The K / V tile images of the pre-pass, one bulk copy per tile into the
      // double buffer, as soon as the P V of the tile two before has read it.
      auto issue_copy = [&](int j) {
        mbar_arrive_expect_tx(&kv_full[j & 1], L::kv_buf);
        bulk_g2s(sm + L::kv0 + (j & 1) * L::kv_buf, p.kv_tiles + (static_cast<size_t>(j) * p.nkv + g) * L::kv_buf,
                 L::kv_buf, &kv_full[j & 1]);
      };
      int nc = 0, ns = 0, npv = 0;  // tiles copied / whose S / P V MMAs were issued
      bool qok = false;
      uint64_t t0 = 0;
      while (npv < ntiles) {
        bool moved = false;
        if (nc < ntiles && (nc < 2 || mbar_try_wait(&kv_empty[nc & 1], ((nc >> 1) - 1) & 1))) {
          issue_copy(nc++);
          moved = true;
        }
        if (!qok) qok = mbar_try_wait(q_ready, 0);
        if (qok && ns < nc && ns <= npv + 1 && mbar_try_wait(&kv_full[ns & 1], (ns >> 1) & 1)) {
          issue_s(ns++);
          moved = true;
        } else if (npv < ns && mbar_try_wait(p_ready, npv & 1)) {
          issue_pv(npv++);
          moved = true;
        }
        if (moved) {
          t0 = 0;
        } else {
          const uint64_t now = global_timer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            if (p.err) atomicExch(p.err, kErrTimeout);
            break;
          }
        }
      }
      const int done = npv;
      // Every MMA has finished before TMEM is released (already so unless a wait gave up).
      if (done > 0) mbar_wait(&kv_empty[(done - 1) & 1], ((done - 1) >> 1) & 1, p.err);
    }
  } else {  // ---- softmax: row R = TMEM lane, key columns 32 h .. (softmaxInPlace, src/llm.zig:1408-1419, online form)
    __shared__ float xrow[2][kAtRows];  // the two halves' row max, then their row sums
    const int st = threadIdx.x;         // 0 .. 255
    const int h = warp >> 2;            // half of the key columns (and of the output dims)
    const int R = 32 * (warp & 3) + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    const int qpos = R < rows ? p.pos0 + t0 + R / G : -1;
    // Q (hi / lo) by all softmax threads, zero rows past `rows`
    for (int it0 = 0; it0 < kAtRows * (D / 8); it0 += 8 * kAtSoftmax) {
      float4 a[8][2];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int it = it0 + st + i * kAtSoftmax, r = it / (D / 8), c = it % (D / 8);
        a[i][0] = a[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (it < kAtRows * (D / 8) && r < rows) {
          const float4* src = reinterpret_cast<const float4*>(p.q + static_cast<size_t>(t0 + r / G) * qd +
                                                              static_cast<size_t>(g * G + r % G) * D + c * 8);
          a[i][0] = __ldcg(src), a[i][1] = __ldcg(src + 1);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int it = it0 + st + i * kAtSoftmax, r = it / (D / 8), c = it % (D / 8);
        if (it >= kAtRows * (D / 8)) continue;
        const float v[8] = {a[i][0].x, a[i][0].y, a[i][0].z, a[i][0].w, a[i][1].x, a[i][1].y, a[i][1].z, a[i][1].w};
        uint4 hi, lo;
        split8(v, hi, lo);
        const uint32_t off = sw_chunk(kAtRows, r, c);
        *reinterpret_cast<uint4*>(sm + L::q_hi + off) = hi;
        *reinterpret_cast<uint4*>(sm + L::q_lo + off) = lo;
      }
    }
    fence_async_smem();  // generic-proxy writes, read by the tensor cores
    mbar_arrive(q_ready);
    float m = -INFINITY, l = 0.f;  // l: this half's share of the row sum
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int j0 = j * kAtKeys + 32 * h;  // position of this thread's first key column
      const int nkeys = min(kAtKeys, last_pos + 1 - j * kAtKeys) - 32 * h;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err)))) break;
      tc_fence_after();
      float s[32];
      tmem_ld32(trow + (j & 1) * 64 + 32 * h, s);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        s[c] = (c < nkeys && j0 + c <= qpos) ? s[c] * p.inv_sqrt_d : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      xrow[h][R] = mt;
      named_barrier(1, kAtSoftmax);
      mt = fmaxf(xrow[0][R], xrow[1][R]);
      const bool move = mt > m + kAtRescale;  // false while the row has no key yet (mt = -inf)
      const float mnew = move ? mt : m;
      const float alpha = move ? (m == -INFINITY ? 0.f : __expf(m - mnew)) : 1.f;
      // P is free and O complete once the last tile's P V is done
      if (j > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(pv_full, (j - 1) & 1, p.err)))) break;
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {  // this half of O = O * alpha (warp-collective)
#pragma unroll 1
        for (int cc = 0; cc < D / 64; ++cc) {
          float v[32];
          const uint32_t col = L::o_col + h * (D / 2) + cc * 32;
          tmem_ld32(trow + col, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(trow + col, v);
        }
      }
      float sum = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pv[i] = mnew == -INFINITY ? 0.f : __expf(s[8 * c8 + i] - mnew);
          sum += pv[i];
        }
        uint4 hi, lo;
        split8(pv, hi, lo);
        const uint32_t off = sw_chunk(kAtRows, R, 4 * h + c8);
        *reinterpret_cast<uint4*>(sm + L::p_hi + off) = hi;
        *reinterpret_cast<uint4*>(sm + L::p_lo + off) = lo;
      }
      l = l * alpha + sum;
      m = mnew;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
    }
    ok = ok && __all_sync(0xffffffffu, mbar_wait(pv_full, (ntiles - 1) & 1, p.err));
    named_barrier(1, kAtSoftmax);  // both halves are past their last read of xrow
    xrow[h][R] = l;
    named_barrier(1, kAtSoftmax);
    if (ok) {
      tc_fence_after();
      const size_t orow = static_cast<size_t>(t0 + R / G) * qd + static_cast<size_t>(g * G + R % G) * D;
      const float inv = 1.0f / (xrow[0][R] + xrow[1][R]);
#pragma unroll 1
      for (int cc = 0; cc < D / 64; ++cc) {
        float v[32];
        const int e0 = h * (D / 2) + cc * 32;
        tmem_ld32(trow + L::o_col + e0, v);
        if (R < rows) {
#pragma unroll
          for (int i = 0; i < 32; ++i) split_bf16(v[i] * inv, p.out_hi[orow + e0 + i], p.out_lo[orow + e0 + i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols) : "memory");
  }
}

template <int D>
cudaError_t launch_at(const PrefillAttnParams& p, cudaStream_t s) {
  const int npos = p.pos0 + p.M;
  const dim3 tgrid((npos + kAtKeys - 1) / kAtKeys, p.nkv);
  kv_tiles_kernel<D><<<tgrid, kAtConv, 0, s>>>(p.k_cache, p.v_cache, p.page_table, npos, p.nkv, p.kv_tiles);
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
  uint8_t* ws = nullptr;
  if ((e = cudaMalloc(&ws, prefill_attention_tc_workspace(d, nkv, total)))) {
    cleanup();
    return e;
  }
  PrefillAttnParams a{q, kc, vc, pt, outs, outs + qn, M, nq, nkv, d, group, pos0, 1.0f / sqrtf(static_cast<float>(d)), err,
                      ws};
  PrefillAttnParams b = a;
  b.out_hi = outs + 2 * qn, b.out_lo = outs + 3 * qn;
  if ((e = launch_prefill_attention_simt(a, 0)) || (e = launch_prefill_attention_tc(b, 0))) {
    cleanup();
    return e;
  }
  compare_pairs_kernel<<<256, 256>>>(b.out_hi, b.out_lo, a.out_hi, a.out_lo, qn, res);
  cudaFree(ws);
  float h[2] = {0.f, 0.f};
  int herr = 0;
  e = cudaMemcpy(h, res, 8, cudaMemcpyDeviceToHost);
  if (!e) e = cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
  cleanup();
  if (e) return e;
  *max_rel_err = herr ? INFINITY : h[0] / fmaxf(h[1], 1e-30f);
  return cudaSuccess;
}

size_t prefill_attention_tc_workspace(int d, int nkv, int max_pos) {
  const size_t tiles = (static_cast<size_t>(max_pos) + kAtKeys - 1) / kAtKeys;
  return tiles * nkv * (d == 128 ? AtLayout<128>::kv_buf : AtLayout<64>::kv_buf);
}

bool prefill_attention_tc_supported(int d, int group) { return (d == 64 || d == 128) && group >= 1 && group <= 8; }

cudaError_t launch_prefill_attention_tc(const PrefillAttnParams& p, cudaStream_t s) {
  if (!prefill_attention_tc_supported(p.d, p.group) || !p.kv_tiles) return cudaErrorInvalidValue;
  return p.d == 128 ? launch_at<128>(p, s) : launch_at<64>(p, s);
}

}  // namespace vvli
