// gemm_skinny.cu - linear layers of a decode batch (B <= 32 rows) on the tensor cores.
//
// With few activation rows the weight matrix is the big operand, so the
// roles are swapped: each CTA owns 128 weight rows (the MMA's M = 128, the
// TMEM lanes) and multiplies them with all B activation rows (N = 16 or 32),
// D^T[128, NB] = W[128, K] . X[NB, K]^T, so no tensor work is spent on
// padding rows and every weight byte is read once per batch.
//   * warp 0: TMA producer (W tile 128 x 64 and the X hi / lo tiles NB x 64
//     per k-block, 128-byte swizzle, no multicast), a ring of stages filling
//     about 200 KB of shared memory;
//   * warp 1: TMEM allocation and the MMA issuer
//     (tcgen05.mma.cta_group::1.kind::f16, two MMAs per k-step for the hi and
//     lo halves of the fp32 activations, a second accumulator for the up rows
//     of gate|up);
//   * warps 2-5: epilogue, one weight row per thread, its NB batch values
//     read with tcgen05.ld.
// Matrices with few 128-row tiles split K over a thread-block cluster of S
// CTAs (S <= 8); the partial accumulators meet in the leader's registers
// through distributed shared memory, added in cluster-rank order, so the
// result does not depend on timing.  Every mbarrier wait is bounded and
// reports VVLI_ERR_TIMEOUT through p.err; every thread reaches both cluster
// barriers whatever happened before.
#include <cooperative_groups.h>

#include <algorithm>

#include "device_fns.cuh"
#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace vvli {

namespace {

constexpr int kSkBM = 128;
constexpr int kSkThreads = 192;
constexpr uint32_t kSkTileW = kSkBM * kGemmBK * 2;  // 16 KB
constexpr int kSkMaxSplit = 8;

template <int NB, bool PAIR>
struct SkLayout {
  static constexpr uint32_t tile_x = NB * kGemmBK * 2;  // NB rows of 128 bytes
  static constexpr uint32_t w_bytes = (PAIR ? 2 : 1) * kSkTileW;
  static constexpr uint32_t stage = w_bytes + 2 * tile_x;
  static constexpr int stages = (200 * 1024) / stage < 12 ? (200 * 1024) / stage : 12;
  static constexpr int acc_cols = PAIR ? 2 * NB : NB;
  static constexpr uint32_t tmem_cols = acc_cols < 32 ? 32 : acc_cols;
  static constexpr size_t smem = static_cast<size_t>(stages) * stage + 1024 + 256;
  static_assert(tile_x % 1024 == 0, "X tiles stay 1024-byte aligned");
  static_assert(static_cast<size_t>(acc_cols) * kSkBM * 4 <= static_cast<size_t>(stages) * stage,
                "the cluster reduction reuses the stage memory");
};

VVLI_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <int NB>
VVLI_DEV void tmem_ld_nb(uint32_t taddr, float* v) {
  if constexpr (NB == 16) {
    tmem_ld16(taddr, v);
  } else {
    tmem_ld32(taddr, v);
  }
}

template <int EPI, int NB>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_x_hi, const __grid_constant__ CUtensorMap tm_x_lo,
                       const __grid_constant__ CUtensorMap tm_w, const GemmParams p) {
  constexpr bool kPair = EPI == GE_SILU;
  using L = SkLayout<NB, kPair>;
  constexpr uint32_t kIdescSk = umma_idesc(kSkBM, NB);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::stages * L::stage);
  uint64_t* empty = full + L::stages;
  uint64_t* tmem_full = empty + L::stages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_full + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kSkBM;
  const int S = gridDim.y;
  const int split = blockIdx.y;
  const int kb0 = split * p.nk / S, kb1 = (split + 1) * p.nk / S;
  const uint32_t crank = S > 1 ? cluster_ctarank() : 0u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(L::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  float acc[NB];
  float accu[kPair ? NB : 1];
  bool have = false;
  grid_launch_dependents();  // the next kernel may start its own weight stream on free SMs
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      const uint32_t bytes = L::w_bytes + (p.two_a ? 2 : 1) * L::tile_x;
      // The weights do not depend on the previous kernel: the first ring's
      // worth goes out before the dependency wait, the activations after it.
      const int pre = min(L::stages, kb1 - kb0);
      for (int i = 0; i < pre; ++i) {
        const uint32_t st = base + i * L::stage;
        const int x = (kb0 + i) * kGemmBK;
        mbar_arrive_expect_tx(&full[i], bytes);
        tma_load_2d(st, &tm_w, x, r0, &full[i]);
        if (kPair) tma_load_2d(st + kSkTileW, &tm_w, x, p.pair_offset + r0, &full[i]);
      }
      grid_dependency_wait();
      for (int i = 0; i < pre; ++i) {
        const uint32_t st = base + i * L::stage;
        const int x = (kb0 + i) * kGemmBK;
        tma_load_2d(st + L::w_bytes, &tm_x_hi, x, 0, &full[i]);
        if (p.two_a) tma_load_2d(st + L::w_bytes + L::tile_x, &tm_x_lo, x, 0, &full[i]);
      }
      int issued = pre;
      for (int kb = kb0 + pre; kb < kb1; ++kb) {
        const int i = kb - kb0, s = i % L::stages;
        if (i >= L::stages && !mbar_wait(&empty[s], ((i / L::stages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], bytes);
        const uint32_t st = base + s * L::stage;
        const int x = kb * kGemmBK;
        tma_load_2d(st, &tm_w, x, r0, &full[s]);
        if (kPair) tma_load_2d(st + kSkTileW, &tm_w, x, p.pair_offset + r0, &full[s]);
        tma_load_2d(st + L::w_bytes, &tm_x_hi, x, 0, &full[s]);
        if (p.two_a) tma_load_2d(st + L::w_bytes + L::tile_x, &tm_x_lo, x, 0, &full[s]);
        issued = i + 1;
      }
      for (int i = issued > L::stages ? issued - L::stages : 0; i < issued; ++i)
        mbar_wait(&full[i % L::stages], (i / L::stages) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      bool ok = true;
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        const int i = kb - kb0, s = i % L::stages;
        if (!(ok = mbar_wait(&full[s], (i / L::stages) & 1, p.err))) break;
        tc_fence_after();
        const uint32_t st = base + s * L::stage;
#pragma unroll
        for (int k = 0; k < kGemmBK / 16; ++k) {
          const uint64_t xh = umma_desc(st + L::w_bytes + k * 32);
          const uint64_t xl = umma_desc(st + L::w_bytes + L::tile_x + k * 32);
          const uint64_t wa = umma_desc(st + k * 32);
          umma_bf16(tmem, wa, xh, kIdescSk, (i | k) != 0);
          if (p.two_a) umma_bf16(tmem, wa, xl, kIdescSk, 1u);
          if (kPair) {
            const uint64_t wb = umma_desc(st + kSkTileW + k * 32);
            umma_bf16(tmem + NB, wb, xh, kIdescSk, (i | k) != 0);
            if (p.two_a) umma_bf16(tmem + NB, wb, xl, kIdescSk, 1u);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(tmem_full);
    }
  } else {  // ---- epilogue warps: read this thread's weight row
    grid_dependency_wait();  // the epilogue reads and writes the previous kernel's outputs
    const int wq = warp & 3;
    const uint32_t trow = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    // tcgen05.ld is warp-collective: the warp goes on only if every lane saw the accumulator.
    const bool ok = __all_sync(0xffffffffu, mbar_wait(tmem_full, 0, p.err));
    if (ok) {
      tc_fence_after();
      tmem_ld_nb<NB>(trow, acc);
      if constexpr (kPair) tmem_ld_nb<NB>(trow + NB, accu);
      have = true;
    }
  }

  // ---- split-K: partial accumulators meet in the leader (cluster rank 0).
  __syncwarp();  // the cluster barriers below are warp-aligned
  if (S > 1) {
    float* red = reinterpret_cast<float*>(sm);  // [acc_cols][128], the stages are idle now
    const int row_local = (warp & 3) * 32 + lane;
    if (warp >= 2 && crank != 0) {
#pragma unroll
      for (int c = 0; c < NB; ++c) {
        red[c * kSkBM + row_local] = have ? acc[c] : 0.f;
        if constexpr (kPair) red[(NB + c) * kSkBM + row_local] = have ? accu[c] : 0.f;
      }
    }
    cluster_sync_all();
    if (warp >= 2 && crank == 0) {
      // Plain loads through the peers' generic shared-memory addresses: all of
      // a peer's values are in flight together; peers are added in rank order.
      cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
      for (int q = 1; q < S; ++q) {
        const float* peer = cluster.map_shared_rank(red, static_cast<unsigned>(q));
        float pv[NB], pu[kPair ? NB : 1];
#pragma unroll
        for (int c = 0; c < NB; ++c) {
          pv[c] = peer[c * kSkBM + row_local];
          if constexpr (kPair) pu[c] = peer[(NB + c) * kSkBM + row_local];
        }
#pragma unroll
        for (int c = 0; c < NB; ++c) {
          acc[c] += pv[c];
          if constexpr (kPair) accu[c] += pu[c];
        }
      }
    }
    cluster_sync_all();
  }

  // ---- epilogue (the leader of a split, or the only CTA)
  if (warp >= 2 && have && crank == 0) {
    const int r = r0 + (warp & 3) * 32 + lane;
    const int M = p.M;
    // The batch rows' steps are independent: predicated rather than cut
    // short, so the unrolled loads and math of all rows are in flight together.
    if constexpr (EPI == GE_SILU) {
      if (r < p.N) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < M) {
            const float g = acc[b];
            const float f = (g / (1.0f + expf(-g))) * accu[b];  // siluMulInto, src/llm.zig:1382-1387
            split_bf16(f, p.out_hi[static_cast<size_t>(b) * p.ld_out + r], p.out_lo[static_cast<size_t>(b) * p.ld_out + r]);
          }
        }
      }
    } else if constexpr (EPI == GE_RESID) {
      if (r < p.N) {
        float old[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) old[b] = (p.add_residual && b < M) ? p.y[static_cast<size_t>(b) * p.ldy + r] : 0.f;
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b < M) p.y[static_cast<size_t>(b) * p.ldy + r] = old[b] + acc[b];  // addInto, src/llm.zig:1389-1396
      }
    } else {  // GE_QKV: batch row b is sequence slot b at position row_pos[b]
      const bool rot = r < p.q_rows + p.kv_rows;  // uniform over the warp (regions are whole heads)
      const bool odd = r & 1;
      const float inv_freq = rot ? rope_inv_freq(p.rope, (r & ~1) % p.d, p.d) : 0.f;
      const float bias = (p.bias && r < p.N) ? bf16_to_f32(p.bias[r]) : 0.f;
      const bool is_q = r < p.q_rows;
      const bool is_k = !is_q && rot;
      const int rel = is_q ? 0 : (is_k ? r - p.q_rows : r - p.q_rows - p.kv_rows);
      float* cache = is_k ? p.k_cache : p.v_cache;
      const size_t head_off = static_cast<size_t>(rel / p.d) * kPage * p.d + rel % p.d;
      // lane b holds batch row b's position and the KV page it falls in
      const int my_pos = lane < M ? p.row_pos[lane] : 0;
      const int my_page = lane < M ? p.page_table[static_cast<size_t>(lane) * p.seq_pages + my_pos / kPage] : 0;
#pragma unroll
      for (int b = 0; b < NB; b += 2) {
        // the rotary pair's even lane takes row b's angle, the odd lane row b + 1's
        float sn = 0.f, cs = 1.f;
        const int pos_mine = __shfl_sync(0xffffffffu, my_pos, b + (odd ? 1 : 0));
        if (rot) sincosf(static_cast<float>(pos_mine) * inv_freq, &sn, &cs);
        const float osn = __shfl_xor_sync(0xffffffffu, sn, 1), ocs = __shfl_xor_sync(0xffffffffu, cs, 1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int bb = b + h;
          float a = acc[bb];
          if (p.bias) a = a + bias;
          const float other = __shfl_xor_sync(0xffffffffu, a, 1);  // the rotary partner row
          const int pos = __shfl_sync(0xffffffffu, my_pos, bb);
          const int page = __shfl_sync(0xffffffffu, my_page, bb);
          if (rot) {
            const bool own = (h == 1) == odd;
            const float s1 = own ? sn : osn, c1 = own ? cs : ocs;
            a = odd ? other * s1 + a * c1 : a * c1 - other * s1;
          }
          if (r < p.N && bb < M) {
            if (is_q)
              p.y[static_cast<size_t>(bb) * p.ldy + r] = a;
            else  // kv_off: [page][kv head][position in page][d]
              cache[static_cast<size_t>(page) * p.nkv * kPage * p.d + static_cast<size_t>(pos % kPage) * p.d + head_off] = a;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols) : "memory");
  }
}

template <int EPI, int NB>
cudaError_t launch_sk(const CUtensorMap& xh, const CUtensorMap& xl, const CUtensorMap& w, const GemmParams& p, int S,
                      bool pdl, cudaStream_t s) {
  using L = SkLayout<NB, EPI == GE_SILU>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + kSkBM - 1) / kSkBM, S);
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = L::smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gemm_skinny_kernel<EPI, NB>, xh, xl, w, p);
}

// Clusters of each size that fit on the device at once (cudaOccupancyMaxActiveClusters),
// per [epilogue][NB 16 / 32][cluster size].
int g_max_clusters[3][2][kSkMaxSplit + 1] = {};

template <int EPI, int NB>
cudaError_t configure_sk() {
  using L = SkLayout<NB, EPI == GE_SILU>;
  cudaError_t e = cudaFuncSetAttribute(gemm_skinny_kernel<EPI, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L::smem));
  if (e) return e;
  for (int S = 1; S <= kSkMaxSplit; ++S) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, S);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = L::smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_skinny_kernel<EPI, NB>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    g_max_clusters[EPI][NB == 16 ? 0 : 1][S] = n;
  }
  return cudaSuccess;
}

}  // namespace

int skinny_nb(int M) { return M <= 16 ? 16 : 32; }

// K split: the most CTAs per weight tile such that every cluster of the launch
// is resident at once (one wave) and no CTA gets an empty K range.
int skinny_split(int epi, int M, int N, int nk, int sm_count) {
  const int tiles = (N + kSkBM - 1) / kSkBM;
  const int* maxc = g_max_clusters[epi < 0 || epi > 2 ? 1 : epi][skinny_nb(M) == 16 ? 0 : 1];
  int best = 1;
  for (int S = 2; S <= std::min(kSkMaxSplit, nk); ++S)
    if (tiles * S <= sm_count && tiles <= maxc[S]) best = S;
  return best;
}

cudaError_t launch_gemm_skinny(const CUtensorMap& x_hi, const CUtensorMap& x_lo, const CUtensorMap& w,
                               const GemmParams& p, int split, cudaStream_t s, bool pdl) {
  if (p.M < 1 || p.M > kSkinnyMaxRows || split < 1 || split > kSkMaxSplit) return cudaErrorInvalidValue;
  const bool nb16 = skinny_nb(p.M) == 16;
  switch (p.epi) {
    case GE_QKV:
      return nb16 ? launch_sk<GE_QKV, 16>(x_hi, x_lo, w, p, split, pdl, s) : launch_sk<GE_QKV, 32>(x_hi, x_lo, w, p, split, pdl, s);
    case GE_RESID:
      return nb16 ? launch_sk<GE_RESID, 16>(x_hi, x_lo, w, p, split, pdl, s)
                  : launch_sk<GE_RESID, 32>(x_hi, x_lo, w, p, split, pdl, s);
    default:
      return nb16 ? launch_sk<GE_SILU, 16>(x_hi, x_lo, w, p, split, pdl, s) : launch_sk<GE_SILU, 32>(x_hi, x_lo, w, p, split, pdl, s);
  }
}

cudaError_t configure_gemm_skinny(int max_smem_optin) {
  if (static_cast<int>(SkLayout<32, true>::smem) > max_smem_optin) return cudaErrorInvalidValue;
  cudaError_t e;
  if ((e = configure_sk<GE_QKV, 16>()) || (e = configure_sk<GE_QKV, 32>()) || (e = configure_sk<GE_RESID, 16>()) ||
      (e = configure_sk<GE_RESID, 32>()) || (e = configure_sk<GE_SILU, 16>()) || (e = configure_sk<GE_SILU, 32>()))
    return e;
  return cudaSuccess;
}

}  // namespace vvli
