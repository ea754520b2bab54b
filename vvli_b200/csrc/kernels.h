// kernels.h - parameter blocks and launchers of the decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vvli {

// Device-resident scalars of the current step.  The captured step graph
// reads them, so one graph serves every position and token.
struct StepState {
  int pos;            // position of the token being processed
  int prompt_len;     // seq_tokens[0, prompt_len) are fixed prompt tokens
  int max_seq;        // KV capacity in positions
  int use_embedding;  // 1: x comes from emb_in instead of the embedding table
  int argmax;         // argmax of the last logits
  int err;            // non-zero: a kernel found an invalid state (VVLI_ERR_* code)
  int batch;          // rows of the batched step
  int pad;
};

struct RopeParams {
  float theta;
  int layout;   // 0 interleaved, 1 split-half
  int scaling;  // 0 none, 1 llama3
  float factor, low, high, orig;
};

enum GemvEpilogue { EPI_PLAIN = 0, EPI_SILU_MUL = 1, EPI_ARGMAX = 2 };

struct GemvParams {
  const uint16_t* W;       // [rows, K] bf16 row-major; rows of a pair start at W + pair_offset*K
  int N;                   // output rows
  int K;                   // input length, multiple of 8
  int pair_offset;         // EPI_SILU_MUL: row offset of the `up` matrix
  const float* x;          // input vector [K]
  const uint16_t* norm_w;  // non-null: x := rmsnorm(x) * norm_w (fused prologue)
  float eps;
  const uint16_t* bias;    // [N] or null
  const float* residual;   // [N] or null: y = residual + W.x
  float* y;                // [N]
  // EPI_ARGMAX
  float* part_val;         // [gridDim.x]
  int* part_idx;           // [gridDim.x]
  unsigned* counter;       // last-CTA ticket, reset by the last CTA
  int row_base;            // global index of row 0 (vocab shard offset)
  int finalize;            // 1: last CTA publishes argmax and advances StepState
  float* local_best;       // finalize == 0: {value, index-as-float-bits} for the TP gather
  StepState* st;
  int* seq_tokens;
  // bulk-copy pipeline plan (filled by launch_gemv)
  int S;            // k-splits per row (1, 2, 4, 8 or 16); warp w owns split w % S
  int SZ;           // 16-byte chunks per split
  int cpl;          // chunks per lane per split
  int R;            // rows per stage (per matrix of a pair)
  int nst;          // stages in the ring
  int stage_bytes;  // bytes per stage
  int part_rows;    // rows reserved per CTA in the partial-sum area
  // The GEMV that follows in the step: its head is prefetched into L2.
  const uint16_t* next_W;
  int next_N, next_K, next_pair_offset;
};

struct AttnParams {
  const float* qkv;        // [nq*d | nkv*d | nkv*d] of this token (rank-local heads)
  float* k_cache;          // this layer: [pages][nkv][kPage][d]
  float* v_cache;
  const int* page_table;   // [max_pages]
  float* out;              // [nq*d]
  float* part;             // [nq][splits][d+2] partial (o, m, l)
  unsigned* counters;      // [nkv]
  StepState* st;
  int nq, nkv, d, group, splits;
  float inv_sqrt_d;
  RopeParams rope;
};

constexpr int kPage = 64;  // KV positions per page

struct EmbedParams {
  const uint16_t* table;  // [V, h]
  const float* emb_in;    // [h] caller embedding
  const int* seq_tokens;
  StepState* st;
  float* x;
  int h;
  int vocab;
};

// ---------------------------------------------------------------- decode megakernel
// One cooperative launch runs a whole decode step as a list of phases.
enum MegaKind { MK_EMBED = 0, MK_GEMV = 1, MK_ATTN = 2 };
enum MegaEpi { ME_STORE = 0, ME_RESIDUAL = 1, ME_SILU = 2, ME_ARGMAX = 3, ME_QKV = 4, ME_AXPY = 5 };

// Fixed-point scale of the down_proj accumulators (x contributions are added as
// round(v * 2^32) in 64-bit integers, so their sum does not depend on the order).
constexpr double kAccScale = 4294967296.0;
constexpr int kMaxFfRows = 256;  // gate|up rows per CTA kept in shared memory for ME_AXPY
constexpr int kMaxTp = 8;
constexpr int kMaxResRows = 64;  // rows of x a CTA can keep in shared memory (MegaParams::xres)
// Weight storage of a matrix.  bf16: rows of K bf16.  Q8_0 / Q4_0 (GGML
// blocks of 32 weights along a row, an fp16 scale each): a row holds its K
// int8 quants (Q8_0) or K/2 nibble bytes (Q4_0, GGML's order: byte j of a
// block carries weight j in the low nibble and weight j + 16 in the high
// one), then the K/32 fp16 scales, padded to a 16-byte multiple.
enum WeightFormat { kFmtBF16 = 0, kFmtQ8 = 1, kFmtQ4 = 2 };
inline __host__ __device__ int quant_bytes(int fmt, int K) { return fmt == kFmtQ8 ? K : K / 2; }
inline __host__ __device__ int row_bytes_of(int fmt, int K) {
  return fmt == kFmtBF16 ? 2 * K : (quant_bytes(fmt, K) + K / 16 + 15) / 16 * 16;
}

constexpr int kMegaConsumerWarps = 16;
constexpr int kMegaXStageMax = 4096;  // longest GEMV input staged in shared memory
constexpr int kMegaThreads = (kMegaConsumerWarps + 1) * 32;

struct MegaPhase {
  int kind;                // MegaKind
  int epi;                 // MegaEpi (GEMV phases)
  int layer;
  int nphys;               // 2: gate|up pair
  const uint16_t* W;       // [N (x nphys), K] rows in format `fmt`, row_bytes apart
  int N, K, pair_offset;
  int fmt, row_bytes;      // WeightFormat, bytes per row
  int S, SZ, cpl, R, stage_bytes;  // streaming plan (see launch_gemv)
  const uint16_t* norm_w;  // non-null: input = rmsnorm(x) * norm_w, x = the residual stream
  const float* x;          // input vector
  float* y;                // output vector
  const uint16_t* bias;
  float* k_cache;          // MK_ATTN and ME_QKV: this layer's K and V pages
  float* v_cache;
  int ar_index;            // ME_RESIDUAL: 2*layer (o_proj) or 2*layer+1 (down_proj)
  int row_align;           // CTA row ranges start at multiples of this (2 for ME_QKV: rotary pairs)
  // down_proj fused into gate|up (tp = 1): the CTA's silu(g)*u rows stay in shared
  // memory (ff_smem) and the next phase (ME_AXPY, no grid barrier before it) streams
  // the matching rows of down_proj^T, adding its h-wide partial into acc_out.
  int ff_smem;             // ME_SILU: outputs to shared memory instead of y
  int no_barrier;          // entered straight from the previous phase
  long long* acc_out;      // ME_AXPY: fixed-point accumulator [h]
  long long* acc_in;       // prologue: x := x + acc_in * 2^-32, sum of squares computed locally
  long long* acc_fold;     // ME_RESIDUAL: residual x[r] + acc_fold[r] * 2^-32, then acc_fold[r] = 0
  int hidden_layer;        // prologue with acc_in and debugging: layer whose output is written to hidden
};

struct MegaParams {
  const MegaPhase* phases;
  int nphases;
  int nst, slot_bytes, part_floats;  // shared-memory ring and partial-sum area
  int xstage_floats;       // shared-memory staging of GEMV inputs (phases with S <= 2), 0: none
  StepState* st;
  int* seq_tokens;
  const uint16_t* emb;
  int emb_fmt, emb_row_bytes;  // the embedding's WeightFormat and bytes per row
  const float* emb_in;
  int h, vocab;
  float* x;                // residual stream [h]
  float* ssq;              // [gridDim.x] per-CTA sums of squares of x
  int xres;                // 1: each CTA keeps its rows of x in shared memory across the step
  float eps;
  unsigned long long* bar; // grid barrier arrivals (grows forever; see megakernel.cu)
  unsigned* epoch;         // increases by one per step (tensor-parallel flag values)
  int n_ar;                // residual phases per step (2 * layers)
  int bars_per_step;       // grid barriers per step (phases entered without one are not counted)
  long long* acc_zero;     // [h] accumulator the embed phase clears (the last layer's)
  // attention
  const float* qkv;
  float* attn;
  float* attn_part;
  unsigned* attn_counters;
  const int* page_table;
  int nq, nkv, d, group, splits;
  float inv_sqrt_d;
  RopeParams rope;
  // LM head argmax
  float* amax_val;
  int* amax_idx;
  unsigned* amax_counter;
  int row_base;
  float* hidden;           // non-null: x after each layer, [layers][h]
  uint64_t* trace;         // non-null: %globaltimer per [phase][cta][6] (see megakernel.cu)
  // tensor parallelism: every peer's receive rows [2][tp][h], flags [2][tp][grid],
  // argmax slots [tp][2] and their flags [tp]
  int tp, rank;
  unsigned long long* peer_recv[kMaxTp];  // [2][tp][h] words: epoch << 32 | fp32 bits of a partial row
  unsigned* peer_flags[kMaxTp];
  float* peer_best[kMaxTp];
  unsigned* peer_best_flag[kMaxTp];
};

cudaError_t launch_megakernel(const MegaParams& p, int grid, size_t smem, cudaStream_t s);
cudaError_t configure_megakernel(int max_smem_optin);
// Streaming plan of one GEMV for the megakernel (16 consumer warps, stages <= stage_cap bytes).
// ph.fmt, ph.K, ph.nphys and ph.row_bytes must be set; false when a row is too long for the plan.
bool plan_mega_gemv(MegaPhase& ph, int stage_cap);
size_t mega_attention_floats(int group, int d, int splits, int max_pages);

// Launchers (pdl: launch with a programmatic edge to the previous kernel).
cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl);
// Launches the GEMV on `sm_count` SMs: the bulk-copy pipeline kernel when a
// row fits a stage (K <= 16384), else the register-streaming kernel.
cudaError_t launch_gemv(int epi, GemvParams p, int sm_count, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl);
size_t attention_smem_bytes(int group, int d, int splits);
cudaError_t launch_tp_argmax_finalize(const float* all_best, int ranks, StepState* st, int* seq_tokens,
                                      cudaStream_t s);
cudaError_t launch_synth_fill(uint16_t* dst, uint64_t key, uint64_t rows, uint64_t cols, uint64_t src_ld,
                              uint64_t row0, uint64_t col0, int kind, cudaStream_t s);
cudaError_t configure_kernels(int max_smem_optin);
// Reorders the q and k rows (and biases) of a fused q|k|v matrix so that the
// two elements of every split-half rotary pair (i, i + d/2) sit on adjacent
// rows (2i, 2i + 1): on the device, split-half RoPE becomes the interleaved
// rule.  `rows` = q rows + k rows (whole heads of d rows), `tmp` holds rows x K.
// bf16 rows [rows, K] -> GGML Q8_0 / Q4_0 blocks in the device row layout (K % 32 == 0).
cudaError_t launch_quantize_rows(const uint16_t* src, uint64_t rows, int K, int fmt, uint8_t* dst, cudaStream_t s);
cudaError_t launch_pair_rows(uint16_t* w, uint16_t* bias, uint16_t* tmp, int rows, int K, int d, cudaStream_t s);
// dst[cols][rows] = src[rows][cols]^T (bf16).
cudaError_t launch_transpose_bf16(const uint16_t* src, uint16_t* dst, int rows, int cols, cudaStream_t s);

}  // namespace vvli
