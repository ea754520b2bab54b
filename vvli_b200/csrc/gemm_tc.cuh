// gemm_tc.cuh - tcgen05 (5th-generation tensor core) GEMM for prefill.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace vvli {

enum GemmEpi { GE_QKV = 0, GE_RESID = 1, GE_SILU = 2 };

constexpr int kGemmBM = 128;  // tokens per tile (TMEM lanes)
constexpr int kGemmBN = 256;  // output columns per tile (TMEM columns)
constexpr int kGemmBK = 64;   // bf16 elements per k-block (one 128-byte swizzled row)

struct GemmParams {
  int M, N, K;           // C[M, N] = A[M, K] . W[N, K]^T; N = columns produced (pair: per matrix)
  int n_tiles;           // column tiles (set by launch_gemm_tc)
  int pair_offset;       // GE_SILU: row offset of the `up` rows in W (gate rows first)
  int nk;                // k-blocks = ceil(K / 64)
  int two_a;             // 1: A = A_hi + A_lo (two MMAs per k-step, near-fp32 activations)
  int epi;               // GemmEpi
  // GE_QKV: q -> y [M, q_rows] fp32 (rotated); k, v -> KV cache at positions pos0 + m
  float* y;
  int ldy;
  const uint16_t* bias;
  int q_rows, kv_rows, d, nkv, pos0;
  RopeParams rope;
  float* k_cache;
  float* v_cache;
  const int* page_table;
  // GE_RESID: x[m, n] = (add_residual ? x[m, n] : 0) + acc (x = y, ld = ldy)
  int add_residual;
  // GE_SILU: ff = silu(g) * u written as bf16 hi / lo [M, ld_out]
  uint16_t* out_hi;
  uint16_t* out_lo;
  int ld_out;
  int* err;              // VVLI_ERR_TIMEOUT on a bounded wait giving up
  // decode batches (gemm_skinny, GE_QKV): row b is sequence slot b at position row_pos[b];
  // its pages are page_table[b * seq_pages ..]
  const int* row_pos;
  int seq_pages;
  // gemm_tc self-test: force the CTA-pair kernel (256-row tiles) or the single-CTA one
  int force_pair, force_single;
  // Stream-K (gemm_tc single-CTA kernel, optional): after sk_dp_waves waves of
  // whole tiles, every CTA takes an equal share of the remaining (tile,
  // k-block) units; a tile split across CTAs is finished by the CTA holding
  // its first k-blocks, which adds the later parts' accumulators (workspace
  // slot = the writer's CTA index, [BN][128] floats) in k order.
  float* sk_ws;          // null: whole tiles only
  unsigned* sk_flags;    // [grid]: slot b holds this launch's part when sk_flags[b] == sk_epoch
  unsigned sk_epoch;     // > 0, a new value per launch
  int sk_dp_waves;       // set by launch_gemm_tc
};
// Stream-K workspace floats for launch_gemm_tc on `sm_count` SMs (flags: sm_count).
size_t gemm_tc_streamk_ws_floats(int sm_count);

// Encodes a 2-D bf16 tensor map [rows, cols] (cols contiguous) with a
// {64, box_rows} box and 128-byte swizzle, the layout the UMMA descriptors use.
cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

cudaError_t launch_gemm_tc(const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& w,
                           const GemmParams& p, cudaStream_t s);
cudaError_t configure_gemm_tc(int max_smem_optin);
cudaError_t gemm_tc_selftest(int M, int N, int K, int two_a, int skinny, uint64_t seed, float* max_rel_err);

// Decode-batch GEMM (B <= kSkinnyMaxRows activation rows): C[B, N] = X[B, K] . W[N, K]^T with the
// weight rows as the MMA's M operand.  X maps: box {64, skinny_nb(B)} rows; W map: box {64, 128}.
// `split` CTAs of a cluster share K (skinny_split picks it).
constexpr int kSkinnyMaxRows = 32;
int skinny_nb(int M);
int skinny_split(int epi, int M, int N, int nk, int sm_count);
// pdl: programmatic edge to the previous kernel (weights stream before the dependency wait).
cudaError_t launch_gemm_skinny(const CUtensorMap& x_hi, const CUtensorMap& x_lo, const CUtensorMap& w,
                               const GemmParams& p, int split, cudaStream_t s, bool pdl = false);
cudaError_t configure_gemm_skinny(int max_smem_optin);

// Prefill helpers (SIMT): embedding gather, RMSNorm into bf16 hi/lo, causal attention.
cudaError_t launch_prefill_embed(const uint16_t* table, const int* tokens, int M, int h, float* x, cudaStream_t s);
cudaError_t launch_norm_split(const float* x, const uint16_t* w, float eps, int M, int h, uint16_t* hi, uint16_t* lo,
                              cudaStream_t s, bool pdl = false);
struct PrefillAttnParams {
  const float* q;        // [M, nq*d] rotated
  const float* k_cache;  // this layer
  const float* v_cache;
  const int* page_table;
  uint16_t* out_hi;      // [M, nq*d] bf16 hi / lo
  uint16_t* out_lo;
  int M, nq, nkv, d, group, pos0;
  float inv_sqrt_d;
  int* err;              // VVLI_ERR_TIMEOUT when a bounded wait gives up (may be null)
  uint8_t* kv_tiles;     // tensor-core kernel's workspace: prefill_attention_tc_workspace bytes
};
size_t prefill_attention_tc_workspace(int d, int nkv, int max_pos);
// Tensor-core kernel when it takes the shape (and VVLI_ATTN_TC is not 0), else the SIMT kernels.
cudaError_t launch_prefill_attention(const PrefillAttnParams& p, cudaStream_t s);
cudaError_t launch_prefill_attention_simt(const PrefillAttnParams& p, cudaStream_t s);
bool prefill_attention_tc_supported(int d, int group);
cudaError_t launch_prefill_attention_tc(const PrefillAttnParams& p, cudaStream_t s);
// Random q, K, V (d, group, M tokens after pos0 positions, scrambled page table): the
// tensor-core kernel against the SIMT flash kernel; *max_rel_err = max |diff| / max |out|.
cudaError_t attention_tc_selftest(int d, int group, int M, int pos0, uint64_t seed, float* max_rel_err);

}  // namespace vvli
