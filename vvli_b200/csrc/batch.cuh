// batch.cuh - SIMT kernels of a decode batch (see batch_decode.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vvli {

struct BatchAttnParams {
  const float* q;          // [B][nq * d] rotated q of every row
  const float* k_cache;    // this layer: [pages][nkv][kPage][d]
  const float* v_cache;
  const int* page_table;   // row b uses page_table[b * seq_pages ..]
  int seq_pages;
  const int* row_pos;      // [B] position of each row's token
  float* part;             // [B][nq][splits][d + 2] partial (o, max, sum)
  unsigned* counters;      // [B][nkv], zero between launches
  uint16_t* out_hi;        // [B][nq * d] bf16 hi / lo of the attention output
  uint16_t* out_lo;
  int nq, nkv, d, group, splits;
  int nslots;              // pages in flight per CTA (batch_attention_slots)
  float inv_sqrt_d;
  int* err;                // VVLI_ERR_TIMEOUT when a page copy never lands
};

int batch_attention_slots(int d);
// Resident CTAs per SM of the attention kernel with `slots` pages in flight.
int batch_attention_ctas_per_sm(int group, int d, int slots);
size_t batch_attention_smem(int group, int d, int slots);
// pdl: programmatic edge to the previous kernel (earlier pages are fetched before the wait).
cudaError_t launch_batch_attention(const BatchAttnParams& p, int B, cudaStream_t s, bool pdl = false);
// Per-row llm.argmax of B rows of n logits (row stride ld, indices offset by row_base):
// best[2b] = value, best[2b+1] = index bits.
cudaError_t launch_rows_argmax(const float* logits, int B, int n, int ld, int row_base, float* best, cudaStream_t s,
                               bool pdl = false);
// Winner per row over `ranks` gathered best arrays ([ranks][B][2]).
cudaError_t launch_rows_argmax_merge(const float* all, int ranks, int B, int* out, cudaStream_t s);
cudaError_t launch_rows_argmax_index(const float* best, int B, int* out, cudaStream_t s, bool pdl = false);

// Tensor-parallel exchange over peer memory (every rank's block mapped in
// every process): block q holds [2 parities][tp][cap] words, each the
// exchange's epoch in the high half and an fp32 value in the low half.
constexpr int kTpxMax = 8;
struct TpExchange {
  unsigned long long* block[kTpxMax];
  int tp, rank, cap;
  unsigned epoch;  // > 0, a new value per exchange, the same on every rank
  int* err;        // VVLI_ERR_TIMEOUT when a peer's word never arrives
};
// gather = 0: dst[i] = sum over ranks (in rank order) of src[i], i < n;
// gather = 1: dst[q * n + i] = rank q's src[i].  n <= cap.
cudaError_t launch_tp_exchange(const float* src, int n, float* dst, int gather, const TpExchange& x, int sm_count,
                               cudaStream_t s);

}  // namespace vvli
