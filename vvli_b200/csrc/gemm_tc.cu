// gemm_tc.cu - prefill on the tensor cores (tcgen05 + TMEM + TMA) and its SIMT helpers.
//
// The reference prefills one token at a time (src/generator.zig:243-251), so
// every weight matrix is read once per prompt token.  Here a prompt chunk of
// M tokens runs each linear layer as one GEMM C[M, N] = A[M, K] . W[N, K]^T:
//   * 128 x 256 output tile per CTA, 64-element k-blocks (128-byte rows,
//     128-byte swizzle), 3-stage ring of shared-memory stages;
//   * warp 0: TMA producer (cp.async.bulk.tensor 2-D, no multicast);
//     warp 1: allocates 2 x 256 TMEM columns (two accumulators), one thread
//     issues tcgen05.mma.cta_group::1.kind::f16 (bf16 x bf16 -> fp32 in
//     TMEM) and frees stages with tcgen05.commit; warps 2-9: epilogue,
//     tcgen05.ld of the accumulator (TMEM lane = token row);
//   * persistent CTAs (one per SM at most); stream-K shares of the last
//     waves' k-blocks when whole tiles would leave SMs idle (launch_gemm_tc);
//     a CTA-pair variant (tcgen05.mma.cta_group::2, 256-row tiles) is opt-in;
//   * activations are fp32 in the reference.  They enter the tensor cores as
//     two bf16 operands, hi = bf16(a) and lo = bf16(a - hi), and both MMAs
//     accumulate into the same TMEM tile, so A is represented to about 16
//     mantissa bits while W (bf16 already) is exact;
//   * epilogues: q|k|v (+bias, RoPE on q and k, k and v into the paged KV
//     cache), residual add into the fp32 hidden rows, and silu(g)*u written
//     as the next GEMM's hi/lo operand.
// All mbarrier waits are bounded and report VVLI_ERR_TIMEOUT through p.err.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <vector>
#include <climits>
#include <cstdlib>

#include "device_fns.cuh"
#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace vvli {

constexpr uint32_t kTileA = kGemmBM * kGemmBK * 2;   // 16 KB
constexpr int kGemmThreads = 320;      // single-CTA kernel: producer, MMA, 8 epilogue warps
constexpr int kPairThreads = 192;      // CTA-pair kernel: producer, MMA, 4 epilogue warps
constexpr int kEpiTileFloats = 32 * 32;  // an epilogue warp's transpose tile (XOR-swizzled)

// Tile shape per output width BN (256, or 128 for matrices with few column
// tiles, so the grid still covers the SMs): stages fill ~192 KB.
template <int BN>
struct TcLayout {
  static constexpr uint32_t tile_b = BN * kGemmBK * 2;
  static constexpr uint32_t stage = 2 * kTileA + tile_b;  // A_hi | A_lo | B
  static constexpr int stages = (192 * 1024) / stage;
  static constexpr uint32_t tmem_cols = 2 * BN;  // two accumulators: tile i + 1's MMAs run during tile i's epilogue
  static constexpr uint32_t idesc = umma_idesc(kGemmBM, BN);
  static constexpr size_t smem =
      static_cast<size_t>(stages) * stage + 1024 /*align*/ + 256 /*barriers*/ + 8 * kEpiTileFloats * 4 /*epilogue tiles*/;
};

// Stream-K hand-off: a writer publishes its part with a release store of the
// launch's epoch; the finisher's bounded acquire spin reports
// VVLI_ERR_TIMEOUT through *err when a flag never arrives.
VVLI_DEV void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
VVLI_DEV bool wait_flag_gpu(const unsigned* p, unsigned v, int* err) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    unsigned x;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(x) : "l"(p) : "memory");
    if (x == v) return true;
    if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, kErrTimeout);
      return false;
    }
    __nanosleep(64);
  }
}

size_t gemm_tc_streamk_ws_floats(int sm_count) { return static_cast<size_t>(sm_count) * 256 * kGemmBM; }

// Epilogue of one accumulator tile: warp wq of each set of four owns TMEM
// lanes (rows) m0 + 32 wq .. and takes the 32-column chunks half, half +
// halves, ...; n0 is the tile's first output column.
// The later parts of a split tile, in k order, are in the sk_ws slots of
// CTAs j * sk_mt + sk_mem for j in [sk_w0, sk_w1) (none when equal).
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, uint32_t trow, int m0, int n0, int wq, int lane,
                                              float* epi_t, int half, int halves, int sk_w0 = 0, int sk_w1 = 0,
                                              int sk_mt = 1, int sk_mem = 0) {
  const int lrow = wq * 32 + lane;
  auto add_parts = [&](float* v, int col0) {
    for (int j = sk_w0; j < sk_w1; ++j) {
      const int c = j * sk_mt + sk_mem;  // the writer's CTA
      const float* ws = p.sk_ws + static_cast<size_t>(c) * BN * kGemmBM + static_cast<size_t>(col0) * kGemmBM + lrow;
      float w[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = __ldcg(ws + j * kGemmBM);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w[j];
    }
  };
  {
    // The accumulator arrives one row per lane (TMEM lane = row); each
    // 32 x 32 chunk is turned around in this warp's shared tile so that the
    // lanes then walk a row's 32 consecutive columns: every global load
    // and store of the epilogue is a coalesced row segment.
    tc_fence_after();
    float v[32];
    const int wrow0 = m0 + wq * 32;  // first row of this warp's 32
    auto transpose_in = [&](const float* src) {
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) epi_t[lane * 32 + (j ^ lane)] = src[j];
      __syncwarp();
    };
    if constexpr (EPI == GE_SILU) {
      float u[32];
      for (int c = half; c < 4; c += halves) {
        tmem_ld32(trow + c * 32, v);        // gate columns
        tmem_ld32(trow + 128 + c * 32, u);  // up columns
        add_parts(v, c * 32);
        add_parts(u, 128 + c * 32);
        float g[32];
        transpose_in(v);
#pragma unroll
        for (int r = 0; r < 32; ++r) g[r] = epi_t[r * 32 + (lane ^ r)];
        transpose_in(u);
        const int n = n0 + c * 32 + lane;
        if (n < p.N) {
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int row_r = wrow0 + r;
            if (row_r >= p.M) break;
            const float f = (g[r] / (1.0f + expf(-g[r]))) * epi_t[r * 32 + (lane ^ r)];  // siluMulInto, src/llm.zig:1382-1387
            const size_t o = static_cast<size_t>(row_r) * p.ld_out + n;
            split_bf16(f, p.out_hi[o], p.out_lo[o]);
          }
        }
      }
    } else {
      // q|k|v: lane r holds the KV page of row wrow0 + r, looked up once per tile
      int my_page = 0;
      if constexpr (EPI == GE_QKV) {
        if (lane < p.M - wrow0 && p.page_table) my_page = p.page_table[(p.pos0 + wrow0 + lane) / kPage];
      }
      for (int c = half; c < BN / 32; c += halves) {
        tmem_ld32(trow + c * 32, v);
        add_parts(v, c * 32);
        transpose_in(v);
        const int n = n0 + c * 32 + lane;
        // The rows' steps are independent: fully unrolled, so that each
        // warp (one per sub-partition) keeps its loads and math in flight
        // together rather than one row's latency at a time.
        const int rows = min(32, p.M - wrow0);
        if constexpr (EPI == GE_RESID) {
          if (n < p.N) {
            float* y = p.y + static_cast<size_t>(wrow0) * p.ldy + n;
            float old[32];
#pragma unroll
            for (int r = 0; r < 32; ++r) old[r] = (p.add_residual && r < rows) ? y[static_cast<size_t>(r) * p.ldy] : 0.f;
#pragma unroll
            for (int r = 0; r < 32; ++r)
              if (r < rows) y[static_cast<size_t>(r) * p.ldy] = old[r] + epi_t[r * 32 + (lane ^ r)];  // addInto
          }
        } else {  // GE_QKV: column n of rows wrow0 ..; rotary pairs (n, n ^ 1) sit in neighbouring lanes
          const bool live = n < p.N;
          const bool rot = n < p.q_rows + p.kv_rows;  // q and k rows hold rotary pairs side by side
          const bool odd = n & 1;
          const float bias = live && p.bias ? bf16_to_f32(p.bias[n]) : 0.f;
          const float inv_freq = rot ? rope_inv_freq(p.rope, (n & ~1) % p.d, p.d) : 0.f;
          const bool is_q = n < p.q_rows;
          const bool is_k = !is_q && rot;
          const int rel = is_q ? 0 : (is_k ? n - p.q_rows : n - p.q_rows - p.kv_rows);
          float* cache = is_k ? p.k_cache : p.v_cache;
          const size_t head_off = static_cast<size_t>(rel / p.d) * kPage * p.d + rel % p.d;
          // Rows r and r + 1 together: the pair's even lane takes the angle
          // of row r, the odd lane that of row r + 1, and they swap
          // (one sincosf per lane per two rows).
#pragma unroll 4
          for (int r = 0; r < 32; r += 2) {
            float sn = 0.f, cs = 1.f;
            if (rot) sincosf(static_cast<float>(p.pos0 + wrow0 + r + (odd ? 1 : 0)) * inv_freq, &sn, &cs);
            const float osn = __shfl_xor_sync(0xffffffffu, sn, 1), ocs = __shfl_xor_sync(0xffffffffu, cs, 1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = r + h;
              float x = epi_t[rr * 32 + (lane ^ rr)];
              if (p.bias) x = x + bias;
              const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
              const int page = __shfl_sync(0xffffffffu, my_page, rr);
              const int pos = p.pos0 + wrow0 + rr;
              if (rot) {
                const bool own = (h == 1) == odd;  // this lane computed row rr's angle
                const float s1 = own ? sn : osn, c1 = own ? cs : ocs;
                const float x0 = odd ? partner : x, x1 = odd ? x : partner;
                x = odd ? x0 * s1 + x1 * c1 : x0 * c1 - x1 * s1;
              }
              if (live && rr < rows) {
                if (is_q)
                  p.y[static_cast<size_t>(wrow0 + rr) * p.ldy + n] = x;
                else  // kv_off: [page][kv head][position in page][d]
                  cache[static_cast<size_t>(page) * p.nkv * kPage * p.d + static_cast<size_t>(pos % kPage) * p.d +
                        head_off] = x;
              }
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- GEMM kernel
template <int EPI, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                   const __grid_constant__ CUtensorMap tm_w, const GemmParams p) {
  using L = TcLayout<BN>;
  constexpr int kGemmStages = L::stages;
  constexpr uint32_t kStageBytes = L::stage;
  constexpr uint32_t kTileB = L::tile_b;
  constexpr uint32_t kTmemCols = L::tmem_cols;
  constexpr uint32_t kIdesc = L::idesc;
  static_assert(EPI != GE_SILU || BN == 256, "gate|up tiles hold 128 gate and 128 up columns");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  uint8_t* sm = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kGemmStages * kStageBytes);
  uint64_t* empty = full + kGemmStages;
  uint64_t* tmem_full = empty + kGemmStages;  // [2] an accumulator holds a finished tile
  uint64_t* tmem_empty = tmem_full + 2;       // [2] the epilogue has read it
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  // epilogue warps' 32 x 33 transpose tiles, after the 256 bytes of barriers
  // epilogue warps' transpose tiles, after the 256 bytes of barriers
  float* epi_t = reinterpret_cast<float*>(sm + kGemmStages * kStageBytes + 256) +
                 ((threadIdx.x >> 5) >= 2 ? (threadIdx.x >> 5) - 2 : 0) * kEpiTileFloats;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr bool kPair = EPI == GE_SILU;
  // Persistent: CTA b takes tiles b, b + grid, ...  Row tiles vary fastest,
  // so the CTAs reading one weight tile run together and share its L2 lines
  // (each weight tile comes from HBM about once).
  const int mt = (p.M + kGemmBM - 1) / kGemmBM;
  const int ntiles = mt * p.n_tiles;
  auto tile_m0 = [&](int t) { return (t % mt) * kGemmBM; };
  auto tile_n0 = [&](int t) { return (t / mt) * (kPair ? BN / 2 : BN); };  // first output column
  // Work segments (tile, k-blocks [kb0, kb1)) of this CTA, in order: whole
  // tiles b, b + G, ... (G = grid); with stream-K, whole tiles for the first
  // sk_dp_waves waves, then a share of the rest, so that no partial last
  // wave of whole tiles leaves SMs idle.  The CTAs go in groups of mt (G is a
  // multiple of mt): group j takes the equal share [j U / NG, (j + 1) U / NG)
  // of the U = (remaining column tiles) x k-blocks units, and its member m
  // does row tile m of each, so the mt CTAs reading one weight tile still
  // read the same k-blocks together (L2 reuse).  A member's share starts
  // inside a tile only with its first stream-K segment (a writer) and ends
  // inside one only with its last (the finisher of that tile), so finishers
  // wait only on writers' first segments: no cycle.
  const bool sk = p.sk_ws != nullptr;
  const int dp_waves = sk ? p.sk_dp_waves : INT_MAX;
  const int t_sk = sk ? dp_waves * static_cast<int>(gridDim.x) : ntiles;  // first stream-K tile (a multiple of mt)
  const int ng = static_cast<int>(gridDim.x) / mt, grp = blockIdx.x / mt, mem = blockIdx.x % mt;
  const long long U = static_cast<long long>(ntiles - t_sk) / mt * p.nk;
  auto share = [&](int j) { return static_cast<long long>(j) * U / ng; };
  struct Cursor {
    long long u, uend;
    int iter;
  };
  auto seg_start = [&]() { return Cursor{sk ? share(grp) : 0, sk ? share(grp + 1) : 0, 0}; };
  auto next_seg = [&](Cursor& cu, int& t, int& kb0, int& kb1) -> bool {
    if (cu.iter < dp_waves) {
      t = static_cast<int>(blockIdx.x) + cu.iter++ * static_cast<int>(gridDim.x);
      kb0 = 0, kb1 = p.nk;
      if (t < t_sk) return true;
      cu.iter = dp_waves;  // whole tiles done (without stream-K: all of them)
    }
    if (cu.u >= cu.uend) return false;
    t = t_sk + static_cast<int>(cu.u / p.nk) * mt + mem;
    kb0 = static_cast<int>(cu.u % p.nk);
    kb1 = static_cast<int>(min(static_cast<long long>(p.nk), kb0 + (cu.uend - cu.u)));
    cu.u += kb1 - kb0;
    return true;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&tmem_full[0], 1);
    mbar_init(&tmem_full[1], 1);
    mbar_init(&tmem_empty[0], 256);  // every epilogue thread
    mbar_init(&tmem_empty[1], 256);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer: every k-block of every tile of this CTA, one ring
      const uint32_t bytes = (p.two_a ? 2 * kTileA : kTileA) + kTileB;
      int issued = 0;  // k-blocks issued over all segments
      bool ok = true;
      Cursor cu = seg_start();
      int t, kb0, kb1;
      while (ok && next_seg(cu, t, kb0, kb1)) {
        const int m0 = tile_m0(t), n0 = tile_n0(t);
        const int rb0 = n0;
        const int rb1 = kPair ? p.pair_offset + n0 : n0 + BN / 2;
        for (int kb = kb0; kb < kb1; ++kb, ++issued) {
          const int s = issued % kGemmStages;
          if (issued >= kGemmStages && !(ok = mbar_wait(&empty[s], ((issued / kGemmStages) - 1) & 1, p.err))) break;
          mbar_arrive_expect_tx(&full[s], bytes);
          const uint32_t st = base + s * kStageBytes;
          const int x = kb * kGemmBK;
          tma_load_2d(st, &tm_a_hi, x, m0, &full[s]);
          if (p.two_a) tma_load_2d(st + kTileA, &tm_a_lo, x, m0, &full[s]);
          tma_load_2d(st + 2 * kTileA, &tm_w, x, rb0, &full[s]);
          if (BN == 256) tma_load_2d(st + 2 * kTileA + kTileB / 2, &tm_w, x, rb1, &full[s]);
        }
      }
      for (int i = issued > kGemmStages ? issued - kGemmStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kGemmStages], (i / kGemmStages) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer: tile i into accumulator i % 2
      bool ok = true;
      int used = 0;  // k-blocks consumed over all segments
      int i = 0;     // segments of this CTA
      Cursor cu = seg_start();
      int t, kb0, kb1;
      for (; ok && next_seg(cu, t, kb0, kb1); ++i) {
        const int buf = i & 1;
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * BN);
        if (i >= 2 && !(ok = mbar_wait(&tmem_empty[buf], ((i >> 1) - 1) & 1, p.err))) break;
        tc_fence_after();
        for (int kb = kb0; kb < kb1; ++kb, ++used) {
          const int s = used % kGemmStages;
          if (!(ok = mbar_wait(&full[s], (used / kGemmStages) & 1, p.err))) break;
          tc_fence_after();
          const uint32_t st = base + s * kStageBytes;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {  // UMMA_K = 16 bf16 = 32 bytes
            const uint64_t bdesc = umma_desc(st + 2 * kTileA + k * 32);
            umma_bf16(acc, umma_desc(st + k * 32), bdesc, kIdesc, (kb != kb0 || k != 0) ? 1u : 0u);
            if (p.two_a) umma_bf16(acc, umma_desc(st + kTileA + k * 32), bdesc, kIdesc, 1u);
          }
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) umma_commit(&tmem_full[buf]);
      }
    }
  } else {  // ---- epilogue: warps 2-9, TMEM lanes 32 * (warp % 4) ..
    // Two warps per TMEM lane quarter (a warp may read only lanes
    // 32 (warp % 4) ..), each taking every other 32-column chunk.
    const int wq = warp & 3, half = (warp - 2) >> 2;
    const int lrow = wq * 32 + lane;
    __shared__ int sk_ok;
    int i = 0;
    Cursor cu = seg_start();
    int t, kb0, kb1;
    for (; next_seg(cu, t, kb0, kb1); ++i) {
    const int buf = i & 1;
    const int m0 = tile_m0(t), n0 = tile_n0(t);
    const uint32_t trow = tmem + (static_cast<uint32_t>(wq * 32) << 16) + static_cast<uint32_t>(buf * BN);
    // tcgen05.ld is warp-collective: the warp goes on only if every lane saw the accumulator.
    if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[buf], (i >> 1) & 1, p.err))) break;
    if (kb0 > 0) {
      // A later part of a split tile: the raw accumulator goes to this CTA's
      // workspace slot, column-major so that the lanes' stores coalesce.
      tc_fence_after();
      float v[32];
      float* ws = p.sk_ws + static_cast<size_t>(blockIdx.x) * BN * kGemmBM + lrow;
      for (int c = half; c < BN / 32; c += 2) {
        tmem_ld32(trow + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) ws[static_cast<size_t>(c * 32 + j) * kGemmBM] = v[j];
      }
      __threadfence();
      named_barrier(1, 256);
      if (threadIdx.x == 64) st_release_gpu(p.sk_flags + blockIdx.x, p.sk_epoch);
      tc_fence_before();
      mbar_arrive(&tmem_empty[buf]);
      continue;
    }
    // The first part of a split tile finishes it: the same member of groups
    // grp + 1 .. g_end - 1 holds the rest of its k-blocks, each as its first
    // segment (CTA j * mt + mem of group j).
    int g_end = grp + 1;
    if (sk && t >= t_sk && kb1 < p.nk) {
      const long long tend = static_cast<long long>((t - t_sk) / mt + 1) * p.nk;
      while (g_end < ng && share(g_end) < tend) ++g_end;
      if (threadIdx.x == 64) {
        sk_ok = 1;
        for (int j = grp + 1; j < g_end && sk_ok; ++j)
          if (!wait_flag_gpu(p.sk_flags + j * mt + mem, p.sk_epoch, p.err)) sk_ok = 0;
      }
      named_barrier(1, 256);
      if (!sk_ok) break;
    }
    epilogue_tile<EPI, BN>(p, trow, m0, n0, wq, lane, epi_t, half, 2, grp + 1, g_end, mt, mem);
    tc_fence_before();  // this warp's TMEM loads of the tile come before the MMAs that reuse it
    mbar_arrive(&tmem_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------- CTA-pair GEMM (cta_group::2)
// Tiles of 256 rows x 256 columns per CTA pair (a 2-CTA cluster): CTA r loads
// rows m0 + 128 r .. of A (hi and lo) and its half of the tile's weight rows
// (rank 0 the first 128 columns, rank 1 the second; for gate|up, 128 gate and
// 128 up rows), and one 256 x 256 x 16 MMA of the leader (rank 0) reads A
// from both CTAs and B from both halves.  Each CTA's TMEM holds its 128 rows
// x 256 columns, so each SM loads 48 KB per k-block for the work that costs a
// 128 x 256 tile 64 KB: a quarter less L2-to-SM traffic.  Measured, it is no
// faster than the single-CTA kernel (which already issues at the measured
// tensor peak inside a wave), so prefill uses it only when VVLI_GEMM_PAIR=1.
// Both CTAs' loads complete on the leader's `full` barriers; the
// leader's commits free both CTAs' stages and announce both accumulators;
// both CTAs' epilogue warps release an accumulator on the leader's barrier.
// No load is multicast.  Every wait is bounded (VVLI_ERR_TIMEOUT in p.err).
struct TcPairLayout {
  static constexpr uint32_t tile_b = 128 * kGemmBK * 2;        // this CTA's half of B: 16 KB
  static constexpr uint32_t stage = 2 * kTileA + tile_b;      // A_hi | A_lo | B half: 48 KB
  static constexpr int stages = 4;
  static constexpr uint32_t tmem_cols = 512;                  // two 256-column accumulators
  static constexpr uint32_t idesc = umma_idesc(256, 256);
  static constexpr size_t smem = static_cast<size_t>(stages) * stage + 1024 + 256 + 4 * kEpiTileFloats * 4;
};

template <int EPI>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                        const __grid_constant__ CUtensorMap tm_w, const GemmParams p) {
  using L = TcPairLayout;
  constexpr int kStages = L::stages;
  constexpr bool kPair = EPI == GE_SILU;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * L::stage);
  uint64_t* empty = full + kStages;
  uint64_t* tmem_full = empty + kStages;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;   // [2], the leader's counts both CTAs' epilogue warps
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  float* epi_t = reinterpret_cast<float*>(sm + kStages * L::stage + 256) + ((threadIdx.x >> 5) & 3) * kEpiTileFloats;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cr = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int mt = (p.M + 255) / 256;
  const int ntiles = mt * p.n_tiles;
  auto tile_m0 = [&](int t) { return (t % mt) * 256; };
  auto tile_n0 = [&](int t) { return (t / mt) * (kPair ? 128 : 256); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&tmem_full[0], 1);
    mbar_init(&tmem_full[1], 1);
    mbar_init(&tmem_empty[0], 8);  // 4 epilogue warps x 2 CTAs
    mbar_init(&tmem_empty[1], 8);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(L::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncwarp();        // the cluster barrier is warp-aligned
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs): this CTA's A rows and B half
      const uint32_t bytes = (p.two_a ? 2 * kTileA : kTileA) + L::tile_b;
      int issued = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs) {
        const int m0 = tile_m0(t) + 128 * static_cast<int>(cr), n0 = tile_n0(t);
        const int rb = cr == 0 ? n0 : (kPair ? p.pair_offset + n0 : n0 + 128);
        for (int kb = 0; kb < p.nk; ++kb, ++issued) {
          const int s = issued % kStages;
          if (issued >= kStages && !(ok = mbar_wait(&empty[s], ((issued / kStages) - 1) & 1, p.err))) break;
          if (cr == 0) mbar_arrive_expect_tx(&full[s], 2 * bytes);
          const uint32_t bar = cluster_addr(smem_u32(&full[s]), 0);
          const uint32_t st = base + s * L::stage;
          const int x = kb * kGemmBK;
          tma_load_2d_pair(st, &tm_a_hi, x, m0, bar);
          if (p.two_a) tma_load_2d_pair(st + kTileA, &tm_a_lo, x, m0, bar);
          tma_load_2d_pair(st + 2 * kTileA, &tm_w, x, rb, bar);
        }
      }
      // Before this CTA may exit, its last copies must have landed: the
      // leader sees them on `full`, the peer through the MMAs' release of its stages.
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
        if (cr == 0)
          mbar_wait(&full[i % kStages], (i / kStages) & 1, p.err);
        else
          mbar_wait(&empty[i % kStages], (i / kStages) & 1, p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && cr == 0) {  // ---- MMA issuer (leader only): tile i into accumulator i % 2 of both CTAs
      bool ok = true;
      int used = 0, i = 0;
      const uint32_t peer_empty0 = cluster_addr(smem_u32(&empty[0]), 1);
      const uint32_t peer_tfull0 = cluster_addr(smem_u32(&tmem_full[0]), 1);
      for (int t = pair; t < ntiles && ok; t += npairs, ++i) {
        const int buf = i & 1;
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * 256);
        if (i >= 2 && !(ok = mbar_wait(&tmem_empty[buf], ((i >> 1) - 1) & 1, p.err))) break;
        tc_fence_after();
        for (int kb = 0; kb < p.nk; ++kb, ++used) {
          const int s = used % kStages;
          if (!(ok = mbar_wait(&full[s], (used / kStages) & 1, p.err))) break;
          tc_fence_after();
          const uint32_t st = base + s * L::stage;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t bdesc = umma_desc(st + 2 * kTileA + k * 32);
            umma_bf16_pair(acc, umma_desc(st + k * 32), bdesc, L::idesc, (kb | k) != 0);
            if (p.two_a) umma_bf16_pair(acc, umma_desc(st + kTileA + k * 32), bdesc, L::idesc, 1u);
          }
          umma_commit_pair(cluster_addr(smem_u32(&empty[s]), 0));  // both CTAs' stage s is free
          umma_commit_pair(peer_empty0 + s * 8);
        }
        if (ok) {
          umma_commit_pair(cluster_addr(smem_u32(&tmem_full[buf]), 0));
          umma_commit_pair(peer_tfull0 + buf * 8);
        }
      }
    }
  } else {  // ---- epilogue warps 2-5 (both CTAs): this CTA's 128 rows of the tile
    const int wq = warp & 3;
    const uint32_t leader_te0 = cluster_addr(smem_u32(&tmem_empty[0]), 0);
    int i = 0;
    for (int t = pair; t < ntiles; t += npairs, ++i) {
      const int buf = i & 1;
      const int m0 = tile_m0(t) + 128 * static_cast<int>(cr), n0 = tile_n0(t);
      const uint32_t trow = tmem + (static_cast<uint32_t>(wq * 32) << 16) + static_cast<uint32_t>(buf * 256);
      if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[buf], (i >> 1) & 1, p.err))) break;
      epilogue_tile<EPI, 256>(p, trow, m0, n0, wq, lane, epi_t, 0, 1);
      tc_fence_before();  // this warp's TMEM loads come before the MMAs that reuse the accumulator
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_te0 + buf * 8);
    }
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // neither CTA leaves while the other may still signal it or use its TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols) : "memory");
  }
}

cudaError_t launch_gemm_tc(const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& w,
                           const GemmParams& p, cudaStream_t s) {
  const int mt = (p.M + kGemmBM - 1) / kGemmBM;
  // Residual GEMMs (o_proj, down_proj: few output columns) take 128-wide tiles
  // when 256-wide ones would leave most SMs idle, unless the k-blocks are
  // many (>= 128) and stream-K can spread the 256-wide tiles' k-blocks over
  // the SMs instead: half the B traffic per MMA of 128-wide tiles (8B
  // down_proj on 512 tokens 131.7 -> 109.5 us; o_proj, 64 k-blocks, 45.1 ->
  // 47.5 us, so it keeps the narrow tiles).
  static const bool sk_off = getenv("VVLI_STREAMK") && getenv("VVLI_STREAMK")[0] == '0';
  const bool narrow = p.epi == GE_RESID && ((p.N + 255) / 256) * mt < 96 && (!p.sk_ws || sk_off || p.nk < 128);
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  GemmParams q = p;
  // Persistent: one CTA per SM at most.  Stream-K spreads the k-blocks of the
  // last one to two waves' tiles evenly over all SMs when whole tiles would
  // leave more than a fifth of the waves' slots idle (measured: 8B gate|up on
  // 512 tokens, 448 tiles = 3.03 waves, 195 -> 177 us; fuller waves lose a
  // little to the split parts); at least 4 k-blocks of a tile per CTA keeps
  // the parts few.
  if (sk_off) q.sk_ws = nullptr;
  // The grid is a multiple of the row tiles mt (groups of CTAs sharing a weight tile).
  auto grid_of = [&](int tiles) {
    const int G = std::max(1, sms / mt) * mt;
    if (!q.sk_ws || mt > sms) {
      q.sk_ws = nullptr;
      return std::min(tiles, sms);
    }
    const int waves = (tiles + G - 1) / G;
    if (!(tiles < 0.8 * waves * G)) {
      q.sk_ws = nullptr;  // whole-tile waves at least 80% full: splitting costs more than it balances
      return std::min(tiles, sms);
    }
    q.sk_dp_waves = tiles > G ? tiles / G - 1 : 0;
    if (q.sk_dp_waves) return G;
    const long long units = static_cast<long long>(tiles / mt) * p.nk;  // per group member
    const long long groups = std::max(1LL, std::min<long long>(G / mt, units / std::min(p.nk, 4)));
    return static_cast<int>(groups) * mt;
  };
  if (narrow) {
    q.n_tiles = (p.N + 127) / 128;
    const int grid = grid_of(mt * q.n_tiles);
    gemm_tc_kernel<GE_RESID, 128><<<grid, kGemmThreads, TcLayout<128>::smem, s>>>(a_hi, a_lo, w, q);
    return cudaGetLastError();
  }
  const int cols = p.epi == GE_SILU ? 128 : 256;
  q.n_tiles = (p.N + cols - 1) / cols;
  // CTA pairs (256-row tiles, VVLI_GEMM_PAIR=1 above 128 rows): a quarter
  // less L2 traffic for the same waves, measured no faster (the single-CTA
  // kernel already issues at the measured tensor peak inside a wave), so off.
  static const bool pair_on = getenv("VVLI_GEMM_PAIR") && getenv("VVLI_GEMM_PAIR")[0] == '1';
  if ((p.M > kGemmBM && pair_on && !p.force_single) || p.force_pair) {
    static int max_pairs = 0;
    if (!max_pairs) {
      cudaLaunchConfig_t oc = {};
      oc.gridDim = dim3(2 * sms);
      oc.blockDim = dim3(kPairThreads);
      oc.dynamicSmemBytes = TcPairLayout::smem;
      cudaLaunchAttribute ca[1];
      ca[0].id = cudaLaunchAttributeClusterDimension;
      ca[0].val.clusterDim.x = 2, ca[0].val.clusterDim.y = 1, ca[0].val.clusterDim.z = 1;
      oc.attrs = ca;
      oc.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&max_pairs, gemm_tc_pair_kernel<GE_RESID>, &oc) != cudaSuccess || max_pairs < 1)
        max_pairs = sms / 2;
    }
    const int pairs = std::min((p.M + 255) / 256 * q.n_tiles, max_pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kPairThreads);
    cfg.dynamicSmemBytes = TcPairLayout::smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (p.epi) {
      case GE_QKV: return cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel<GE_QKV>, a_hi, a_lo, w, q);
      case GE_RESID: return cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel<GE_RESID>, a_hi, a_lo, w, q);
      default: return cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel<GE_SILU>, a_hi, a_lo, w, q);
    }
  }
  const int grid = grid_of(mt * q.n_tiles);
  constexpr size_t smem = TcLayout<256>::smem;
  switch (p.epi) {
    case GE_QKV: gemm_tc_kernel<GE_QKV, 256><<<grid, kGemmThreads, smem, s>>>(a_hi, a_lo, w, q); break;
    case GE_RESID: gemm_tc_kernel<GE_RESID, 256><<<grid, kGemmThreads, smem, s>>>(a_hi, a_lo, w, q); break;
    default: gemm_tc_kernel<GE_SILU, 256><<<grid, kGemmThreads, smem, s>>>(a_hi, a_lo, w, q); break;
  }
  return cudaGetLastError();
}

cudaError_t configure_gemm_tc(int max_smem_optin) {
  if (static_cast<int>(TcLayout<256>::smem) > max_smem_optin || static_cast<int>(TcLayout<128>::smem) > max_smem_optin)
    return cudaErrorInvalidValue;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(gemm_tc_kernel<GE_QKV, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcLayout<256>::smem)) ||
      (e = cudaFuncSetAttribute(gemm_tc_kernel<GE_RESID, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcLayout<256>::smem)) ||
      (e = cudaFuncSetAttribute(gemm_tc_kernel<GE_SILU, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcLayout<256>::smem)) ||
      (e = cudaFuncSetAttribute(gemm_tc_kernel<GE_RESID, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcLayout<128>::smem)))
    return e;
  if (static_cast<int>(TcPairLayout::smem) > max_smem_optin) return cudaErrorInvalidValue;
  if ((e = cudaFuncSetAttribute(gemm_tc_pair_kernel<GE_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcPairLayout::smem)) ||
      (e = cudaFuncSetAttribute(gemm_tc_pair_kernel<GE_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcPairLayout::smem)) ||
      (e = cudaFuncSetAttribute(gemm_tc_pair_kernel<GE_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TcPairLayout::smem)))
    return e;
  return cudaSuccess;
}

// ---------------------------------------------------------------- tensor maps
cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode),
                                            cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !encode) return cudaErrorNotSupported;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- SIMT helpers
__global__ void prefill_embed_kernel(const uint16_t* table, const int* tokens, int M, int h, float* x) {
  const size_t total = static_cast<size_t>(M) * h;
  for (size_t e = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(e / h), i = static_cast<int>(e % h);
    x[e] = bf16_to_f32(table[static_cast<size_t>(tokens[m]) * h + i]);
  }
}

cudaError_t launch_prefill_embed(const uint16_t* table, const int* tokens, int M, int h, float* x, cudaStream_t s) {
  const size_t total = static_cast<size_t>(M) * h;
  const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 148 * 16));
  prefill_embed_kernel<<<blocks, 256, 0, s>>>(table, tokens, M, h, x);
  return cudaGetLastError();
}

// rmsNormInto (src/llm.zig:1287-1300) of every row, written as bf16 hi + lo.
// One CTA per row; each thread loads its PER elements at once (a row costs
// one memory round trip, which matters for the few rows of a decode batch).
template <int PER>
__global__ void __launch_bounds__(512) norm_split_kernel(const float* x, const uint16_t* w, float eps, int h,
                                                          uint16_t* hi, uint16_t* lo) {
  __shared__ float red[16];
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  grid_launch_dependents();
  grid_dependency_wait();  // no-op without a programmatic edge
  const float* xr = x + static_cast<size_t>(m) * h;
  float v[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = tid + k * 512;
    v[k] = i < h ? xr[i] : 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) ss = fmaf(v[k], v[k], ss);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) t += red[i];
  const float scale = 1.0f / sqrtf(t / static_cast<float>(h) + eps);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = tid + k * 512;
    if (i < h) split_bf16(v[k] * bf16_to_f32(w[i]) * scale, hi[static_cast<size_t>(m) * h + i], lo[static_cast<size_t>(m) * h + i]);
  }
}

cudaError_t launch_norm_split(const float* x, const uint16_t* w, float eps, int M, int h, uint16_t* hi, uint16_t* lo,
                              cudaStream_t s, bool pdl) {
  const int per = (h + 511) / 512;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(512);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (per <= 2) return cudaLaunchKernelEx(&cfg, norm_split_kernel<2>, x, w, eps, h, hi, lo);
  if (per <= 4) return cudaLaunchKernelEx(&cfg, norm_split_kernel<4>, x, w, eps, h, hi, lo);
  if (per <= 8) return cudaLaunchKernelEx(&cfg, norm_split_kernel<8>, x, w, eps, h, hi, lo);
  if (per <= 16) return cudaLaunchKernelEx(&cfg, norm_split_kernel<16>, x, w, eps, h, hi, lo);
  if (per <= 32) return cudaLaunchKernelEx(&cfg, norm_split_kernel<32>, x, w, eps, h, hi, lo);
  return cudaErrorInvalidValue;  // hidden sizes above 16384
}

// Causal attention of a prompt chunk (computeAttentionInto per token,
// src/llm.zig:1302-1335): CTA = (kv head g, block of QB tokens), rows = the
// group's q heads x tokens; 32-position K/V tiles staged in shared memory
// (K rows padded by one float against bank conflicts); one warp per row at a
// time with an online softmax; output as bf16 hi/lo for the o_proj GEMM.
constexpr int kPaTile = 32;
constexpr int kPaThreads = 256;
constexpr int kPaAcc = 32;  // fp32 accumulators per lane: rows_per_warp * dims_per_lane

template <int DPL>  // dims per lane = ceil(head_dim / 32)
__global__ void __launch_bounds__(kPaThreads) prefill_attention_kernel(const PrefillAttnParams p) {
  extern __shared__ float pa[];
  const int d = p.d, G = p.group, g = blockIdx.x;
  constexpr int dpl = DPL;
  constexpr int rpw = kPaAcc / DPL;  // rows per warp
  const int QB = max(1, (rpw * (kPaThreads / 32)) / G);  // tokens per CTA
  const int t0 = blockIdx.y * QB;
  const int nt = min(QB, p.M - t0);
  const int rows = G * nt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qs = pa;                                  // [rows][d]
  float* ks = qs + static_cast<size_t>(G) * QB * d;  // [kPaTile][d + 1]
  float* vs = ks + kPaTile * (d + 1);              // [kPaTile][d]
  for (int idx = threadIdx.x; idx < rows * d; idx += kPaThreads) {
    const int r = idx / d, e = idx % d;
    const int hh = r % G, t = r / G;
    qs[idx] = p.q[static_cast<size_t>(t0 + t) * p.nq * d + static_cast<size_t>(g * G + hh) * d + e];
  }
  float acc[kPaAcc], mrun[rpw], lrun[rpw];
#pragma unroll
  for (int i = 0; i < kPaAcc; ++i) acc[i] = 0.f;
#pragma unroll
  for (int i = 0; i < rpw; ++i) {
    mrun[i] = -INFINITY;
    lrun[i] = 0.f;
  }
  const int last_pos = p.pos0 + t0 + nt - 1;
  for (int base = 0; base <= last_pos; base += kPaTile) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kPaTile * d; idx += kPaThreads) {
      const int i = idx / d, e = idx % d;
      const int pos = base + i;
      float kv = 0.f, vv = 0.f;
      if (pos <= last_pos) {
        const size_t off = kv_off(p.page_table, pos, g, p.nkv, d) + e;
        kv = p.k_cache[off];
        vv = p.v_cache[off];
      }
      ks[i * (d + 1) + e] = kv;
      vs[i * d + e] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < rpw; ++rr) {
      const int r = warp * rpw + rr;
      if (r >= rows) continue;
      const int pos_r = p.pos0 + t0 + r / G;  // this row's token position (causal limit)
      const float* qr = qs + static_cast<size_t>(r) * d;
      float sc = -INFINITY;
      if (base + lane <= pos_r) {
        float dot = 0.f;
        for (int e = 0; e < d; ++e) dot = fmaf(qr[e], ks[lane * (d + 1) + e], dot);
        sc = dot * p.inv_sqrt_d;
      }
      const float mt = warp_max(sc);
      const float mnew = fmaxf(mrun[rr], mt);
      const float pr = sc == -INFINITY ? 0.f : expf(sc - mnew);
      const float alpha = mrun[rr] == -INFINITY ? 0.f : expf(mrun[rr] - mnew);
      lrun[rr] = lrun[rr] * alpha + warp_sum(pr);
      mrun[rr] = mnew;
#pragma unroll
      for (int j = 0; j < dpl; ++j) {
        const int e = lane + 32 * j;
        float a = acc[rr * dpl + j] * alpha;
        for (int i = 0; i < kPaTile; ++i) {
          const float pi = __shfl_sync(0xffffffffu, pr, i);
          if (e < d) a = fmaf(pi, vs[i * d + e], a);
        }
        acc[rr * dpl + j] = a;
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < rpw; ++rr) {
    const int r = warp * rpw + rr;
    if (r >= rows) continue;
    const int hh = r % G, t = r / G;
    const size_t orow = static_cast<size_t>(t0 + t) * p.nq * d + static_cast<size_t>(g * G + hh) * d;
#pragma unroll
    for (int j = 0; j < dpl; ++j) {
      const int e = lane + 32 * j;
      if (e < d) split_bf16(acc[rr * dpl + j] / lrun[rr], p.out_hi[orow + e], p.out_lo[orow + e]);
    }
  }
}

// Register-blocked causal attention for head_dim 64 / 128 (flash form).
// CTA = (kv head g, block of BQ = 128 / G tokens): its 128 query rows are the
// group's q heads x tokens (row r = token r / G, head r % G).  Key tiles of 64
// positions (one KV page) are staged transposed (K) and as-is (V) in shared
// memory; thread t owns query rows 4 (t / 8) .. + 3, and score columns
// 8 (t % 8) .. + 7 of a tile (32 scores from 3 shared loads per k), then
// output dims (t % 8) D / 8 .. of its 4 rows for P.V.  Online softmax per row
// across the row's 8 lanes; causal mask by position.  Output as bf16 hi / lo
// for the o_proj GEMM.
constexpr int kFaThreads = 256;
constexpr int kFaRows = 128;
constexpr int kFaKeys = 64;
constexpr int kFaPs = kFaKeys + 1;  // P row stride (bank spread)

template <int D>
size_t flash_smem_floats() {
  return static_cast<size_t>(D) * kFaRows + static_cast<size_t>(D) * kFaKeys + static_cast<size_t>(kFaKeys) * D +
         static_cast<size_t>(kFaRows) * kFaPs;
}

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1) prefill_flash_kernel(const PrefillAttnParams p) {
  extern __shared__ __align__(16) float fa[];
  constexpr int DD = D / 8;  // output dims per thread
  float* qt = fa;                           // [D][128]   Q^T
  float* kt = qt + D * kFaRows;             // [D][64]    K^T
  float* vs = kt + D * kFaKeys;             // [64][D]
  float* ps = vs + kFaKeys * D;             // [128][65]  probabilities
  const int G = p.group, g = blockIdx.x;
  const int BQ = kFaRows / G;
  const int t0 = blockIdx.y * BQ;
  const int nt = min(BQ, p.M - t0);
  const int rows = G * nt;
  const int tid = threadIdx.x, rg = tid >> 3, cg = tid & 7;
  const int qd = p.nq * D;
  // Q^T: thread reads 4 consecutive dims of a row, writes 4 rows of qt
  for (int idx = tid; idx < kFaRows * (D / 4); idx += kFaThreads) {
    const int r = idx % kFaRows, k4 = idx / kFaRows;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) {
      const int t = r / G, hh = r % G;
      v = *reinterpret_cast<const float4*>(p.q + static_cast<size_t>(t0 + t) * qd + static_cast<size_t>(g * G + hh) * D + 4 * k4);
    }
    qt[(4 * k4 + 0) * kFaRows + r] = v.x;
    qt[(4 * k4 + 1) * kFaRows + r] = v.y;
    qt[(4 * k4 + 2) * kFaRows + r] = v.z;
    qt[(4 * k4 + 3) * kFaRows + r] = v.w;
  }
  // this thread's rows: query positions (rows past `rows` are padding)
  int qpos[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rg + i;
    qpos[i] = r < rows ? p.pos0 + t0 + r / G : -1;
  }
  float o[4][DD];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DD; ++e) o[i][e] = 0.f;
  }
  const int last_pos = p.pos0 + t0 + nt - 1;
  for (int j0 = 0; j0 <= last_pos; j0 += kFaKeys) {
    __syncthreads();  // previous tile's K, V and P are no longer read
    const int nkeys = min(kFaKeys, last_pos + 1 - j0);
    const size_t base = kv_off(p.page_table, j0, g, p.nkv, D);  // a tile is one page: rows contiguous
    for (int idx = tid; idx < kFaKeys * (D / 4); idx += kFaThreads) {
      const int j = idx % kFaKeys, k4 = idx / kFaKeys;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (j < nkeys) {
        kv = *reinterpret_cast<const float4*>(p.k_cache + base + static_cast<size_t>(j) * D + 4 * k4);
        vv = *reinterpret_cast<const float4*>(p.v_cache + base + static_cast<size_t>(j) * D + 4 * k4);
      }
      kt[(4 * k4 + 0) * kFaKeys + j] = kv.x;
      kt[(4 * k4 + 1) * kFaKeys + j] = kv.y;
      kt[(4 * k4 + 2) * kFaKeys + j] = kv.z;
      kt[(4 * k4 + 3) * kFaKeys + j] = kv.w;
      *reinterpret_cast<float4*>(vs + j * D + 4 * k4) = vv;
    }
    __syncthreads();
    // S = Q K^T for rows 4rg.., keys 8cg..
    float sc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) sc[i][c] = 0.f;
#pragma unroll 4
    for (int k = 0; k < D; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(qt + k * kFaRows + 4 * rg);
      const float4 b0 = *reinterpret_cast<const float4*>(kt + k * kFaKeys + 8 * cg);
      const float4 b1 = *reinterpret_cast<const float4*>(kt + k * kFaKeys + 8 * cg + 4);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) sc[i][c] = fmaf(av[i], bv[c], sc[i][c]);
    }
    // online softmax over the row's 8 lanes (softmaxInPlace, src/llm.zig:1408-1419)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int kp = j0 + 8 * cg + c;
        sc[i][c] = (kp <= qpos[i] && 8 * cg + c < nkeys) ? sc[i][c] * p.inv_sqrt_d : -INFINITY;
        mt = fmaxf(mt, sc[i][c]);
      }
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      const float mnew = fmaxf(m[i], mt);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float e = mnew == -INFINITY ? 0.f : expf(sc[i][c] - mnew);
        ps[(4 * rg + i) * kFaPs + 8 * cg + c] = e;
        sum += e;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      const float alpha = m[i] == -INFINITY ? 0.f : expf(m[i] - mnew);
      l[i] = l[i] * alpha + sum;
      m[i] = mnew;
#pragma unroll
      for (int e = 0; e < DD; ++e) o[i][e] *= alpha;
    }
    __syncthreads();
    // O += P V (addScaled, src/llm.zig:1398-1406) for rows 4rg.., dims cg*DD..
#pragma unroll 2
    for (int j = 0; j < nkeys; ++j) {
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = ps[(4 * rg + i) * kFaPs + j];
      const float4* vr = reinterpret_cast<const float4*>(vs + j * D + cg * DD);
#pragma unroll
      for (int e4 = 0; e4 < DD / 4; ++e4) {
        const float4 v = vr[e4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[i][4 * e4 + 0] = fmaf(pr[i], v.x, o[i][4 * e4 + 0]);
          o[i][4 * e4 + 1] = fmaf(pr[i], v.y, o[i][4 * e4 + 1]);
          o[i][4 * e4 + 2] = fmaf(pr[i], v.z, o[i][4 * e4 + 2]);
          o[i][4 * e4 + 3] = fmaf(pr[i], v.w, o[i][4 * e4 + 3]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rg + i;
    if (r >= rows) continue;
    const int t = r / G, hh = r % G;
    const size_t orow = static_cast<size_t>(t0 + t) * qd + static_cast<size_t>(g * G + hh) * D + cg * DD;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int e = 0; e < DD; ++e) split_bf16(o[i][e] * inv, p.out_hi[orow + e], p.out_lo[orow + e]);
  }
}

template <int D>
static cudaError_t launch_flash(const PrefillAttnParams& p, cudaStream_t s) {
  const int BQ = kFaRows / p.group;
  const dim3 grid(p.nkv, (p.M + BQ - 1) / BQ);
  const size_t smem = flash_smem_floats<D>() * 4;
  cudaError_t e = cudaFuncSetAttribute(prefill_flash_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e) return e;
  prefill_flash_kernel<D><<<grid, kFaThreads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int DPL>
static cudaError_t launch_pa(const PrefillAttnParams& p, cudaStream_t s) {
  constexpr int rpw = kPaAcc / DPL;
  const int QB = std::max(1, (rpw * (kPaThreads / 32)) / p.group);
  const dim3 grid(p.nkv, (p.M + QB - 1) / QB);
  const size_t smem = (static_cast<size_t>(p.group) * QB * p.d + kPaTile * (p.d + 1) + kPaTile * p.d) * 4;
  cudaError_t e = cudaFuncSetAttribute(prefill_attention_kernel<DPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e) return e;
  prefill_attention_kernel<DPL><<<grid, kPaThreads, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill_attention(const PrefillAttnParams& p, cudaStream_t s) {
  static const bool tc = !(getenv("VVLI_ATTN_TC") && getenv("VVLI_ATTN_TC")[0] == '0');
  if (tc && p.kv_tiles && prefill_attention_tc_supported(p.d, p.group)) return launch_prefill_attention_tc(p, s);
  return launch_prefill_attention_simt(p, s);
}

cudaError_t launch_prefill_attention_simt(const PrefillAttnParams& p, cudaStream_t s) {
  if (p.group <= 8 && kFaRows / p.group >= 1) {
    if (p.d == 128) return launch_flash<128>(p, s);
    if (p.d == 64) return launch_flash<64>(p, s);
  }
  const int dpl = (p.d + 31) / 32;
  if (dpl <= 1) return launch_pa<1>(p, s);
  if (dpl <= 2) return launch_pa<2>(p, s);
  if (dpl <= 4) return launch_pa<4>(p, s);
  return launch_pa<8>(p, s);
}

// ---------------------------------------------------------------- self-test
__global__ void fill_bf16_kernel(uint16_t* p, size_t n, uint64_t key, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
    const float u = static_cast<float>(static_cast<int>(h & 0xffff) - 32768) * (1.0f / 32768.0f);
    p[i] = f32_to_bf16(u * scale);
  }
}

__global__ void gemm_ref_kernel(const uint16_t* ahi, const uint16_t* alo, const uint16_t* w, int M, int N, int K,
                                int two_a, float* c) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  if (n >= N) return;
  double acc = 0.0;
  for (int k = 0; k < K; ++k) {
    double a = bf16_to_f32(ahi[static_cast<size_t>(m) * K + k]);
    if (two_a) a += bf16_to_f32(alo[static_cast<size_t>(m) * K + k]);
    acc += a * bf16_to_f32(w[static_cast<size_t>(n) * K + k]);
  }
  c[static_cast<size_t>(m) * N + n] = static_cast<float>(acc);
}

__global__ void max_rel_err_kernel(const float* a, const float* b, size_t n, float* out) {
  float worst = 0.f, scale = 0.f;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    worst = fmaxf(worst, fabsf(a[i] - b[i]));
    scale = fmaxf(scale, fabsf(b[i]));
  }
  worst = warp_max(worst);
  scale = warp_max(scale);
  __shared__ float w_sh[32], s_sh[32];
  if ((threadIdx.x & 31) == 0) {
    w_sh[threadIdx.x >> 5] = worst;
    s_sh[threadIdx.x >> 5] = scale;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (unsigned i = 1; i < blockDim.x / 32; ++i) {
      worst = fmaxf(worst, w_sh[i]);
      scale = fmaxf(scale, s_sh[i]);
    }
    *out = worst / fmaxf(scale, 1e-30f);
  }
}

// Runs C = A . W^T through the tensor-core GEMM and a SIMT fp64-accumulating
// reference on random data; *max_rel_err = max |C - ref| / max |ref|.
cudaError_t gemm_tc_selftest(int M, int N, int K, int two_a, int kernel, uint64_t seed, float* max_rel_err) {
  const bool skinny = kernel == 1;
  cudaError_t e;
  int dev = 0, optin = 0;
  if ((e = cudaGetDevice(&dev))) return e;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if ((e = configure_gemm_tc(optin))) return e;
  if (skinny && (M > kSkinnyMaxRows || (e = configure_gemm_skinny(optin)))) return e ? e : cudaErrorInvalidValue;
  uint16_t *ahi = nullptr, *alo = nullptr, *w = nullptr;
  float *c = nullptr, *ref = nullptr, *err_out = nullptr, *sk_ws = nullptr, *c2 = nullptr;
  int* err = nullptr;
  unsigned* sk_flags = nullptr;
  const bool streamk = kernel == 3;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto cleanup = [&]() {
    cudaFree(ahi), cudaFree(alo), cudaFree(w), cudaFree(c), cudaFree(ref), cudaFree(err_out), cudaFree(err);
    cudaFree(sk_ws), cudaFree(sk_flags), cudaFree(c2);
  };
  if (streamk && ((e = cudaMalloc(&sk_ws, gemm_tc_streamk_ws_floats(sms) * 4)) ||
                  (e = cudaMalloc(&sk_flags, static_cast<size_t>(sms) * 4)) ||
                  (e = cudaMemset(sk_flags, 0, static_cast<size_t>(sms) * 4)) ||
                  (e = cudaMalloc(&c2, static_cast<size_t>(M) * N * 4)))) {
    cleanup();
    return e;
  }
  if ((e = cudaMalloc(&ahi, static_cast<size_t>(M) * K * 2)) || (e = cudaMalloc(&alo, static_cast<size_t>(M) * K * 2)) ||
      (e = cudaMalloc(&w, static_cast<size_t>(N) * K * 2)) || (e = cudaMalloc(&c, static_cast<size_t>(M) * N * 4)) ||
      (e = cudaMalloc(&ref, static_cast<size_t>(M) * N * 4)) || (e = cudaMalloc(&err_out, 4)) ||
      (e = cudaMalloc(&err, 4))) {
    cleanup();
    return e;
  }
  cudaMemset(err, 0, 4);
  fill_bf16_kernel<<<256, 256>>>(ahi, static_cast<size_t>(M) * K, seed * 3 + 1, 1.0f);
  fill_bf16_kernel<<<256, 256>>>(alo, static_cast<size_t>(M) * K, seed * 3 + 2, 1.0f / 256);
  fill_bf16_kernel<<<256, 256>>>(w, static_cast<size_t>(N) * K, seed * 3 + 3, 0.05f);
  CUtensorMap mhi, mlo, mw;
  const uint32_t box_a = skinny ? static_cast<uint32_t>(skinny_nb(M)) : static_cast<uint32_t>(kGemmBM);
  if ((e = make_tmap_bf16(&mhi, ahi, M, K, box_a)) || (e = make_tmap_bf16(&mlo, alo, M, K, box_a)) ||
      (e = make_tmap_bf16(&mw, w, N, K, kGemmBN / 2))) {
    cleanup();
    return e;
  }
  GemmParams p{};
  p.M = M, p.N = N, p.K = K, p.nk = (K + kGemmBK - 1) / kGemmBK, p.two_a = two_a, p.epi = GE_RESID;
  p.y = c, p.ldy = N, p.add_residual = 0, p.err = err;
  p.force_pair = kernel == 2 ? 1 : 0;
  if ((kernel == 0 || streamk) && M > kGemmBM) p.force_single = 1;
  p.sk_ws = sk_ws, p.sk_flags = sk_flags, p.sk_epoch = 1;
  if ((e = skinny ? launch_gemm_skinny(mhi, mlo, mw, p, skinny_split(p.epi, M, N, p.nk, sms), 0) : launch_gemm_tc(mhi, mlo, mw, p, 0))) {
    cleanup();
    return e;
  }
  if (streamk) {  // the next launch reuses the flags at the next epoch: the same C, bit for bit
    p.y = c2, p.sk_epoch = 2;
    int same = 0;
    if (!(e = launch_gemm_tc(mhi, mlo, mw, p, 0)) && !(e = cudaDeviceSynchronize())) {
      std::vector<float> h0(static_cast<size_t>(M) * N), h1(h0.size());
      if (!(e = cudaMemcpy(h0.data(), c, h0.size() * 4, cudaMemcpyDeviceToHost)) &&
          !(e = cudaMemcpy(h1.data(), c2, h1.size() * 4, cudaMemcpyDeviceToHost)))
        same = std::memcmp(h0.data(), h1.data(), h0.size() * 4) == 0;
    }
    if (!e && !same) e = cudaErrorUnknown;
    if (e) {
      cleanup();
      return e;
    }
  }
  gemm_ref_kernel<<<dim3((N + 127) / 128, M), 128>>>(ahi, alo, w, M, N, K, two_a, ref);
  max_rel_err_kernel<<<1, 1024>>>(c, ref, static_cast<size_t>(M) * N, err_out);
  int herr = 0;
  if ((e = cudaMemcpy(max_rel_err, err_out, 4, cudaMemcpyDeviceToHost)) ||
      (e = cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost))) {
    cleanup();
    return e;
  }
  cleanup();
  return herr ? cudaErrorTimeout : cudaSuccess;
}

}  // namespace vvli
