// sampler.cuh - Sampler.next (src/generator.zig:97-126, 338-463) on the device.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vvli {

// Candidate lists up to this length are selected and sorted inside one CTA;
// longer ones (top_k = 0 or large) take the sorted-vocabulary path.
constexpr int kSampleSmallK = 4096;
// top_k <= kSampleFastK (the reference's default is 40) takes a two-pass path:
// per-1024-id CTAs keep their best k (warp sorting networks and a merge tree),
// one CTA merges those lists (at most kSampleFastMaxCand / 64 of them: a
// vocabulary of up to 262,144 tokens).
constexpr int kSampleFastK = 64;
constexpr int kSampleFastMaxCand = 16384;

struct SampleState {
  unsigned long long rng[4];  // xoshiro256++ state, advanced when a draw happens
  int token;                  // result
  int path;                   // 0: token is final; 1: the long-candidate path must run
  int k;                      // candidates of the long path's scan
  int n_sort;                 // keys the long path sorts (those its scan can reach)
};

struct SampleParams {
  const float* logits;
  int V;
  const unsigned* stamp;      // stamp[i] == call: token i is among the last repeat_last_n
  unsigned call;
  // top-k path: when stamp is null, the last repeat_last_n tokens themselves
  const uint32_t* recent;
  int n_recent;
  float temperature, top_p, repeat_penalty;
  unsigned long long top_k;
  unsigned* key32;            // [V] scratch: order-preserving keys of the finite adjusted logits, 0 = none
  unsigned long long* key64;  // [V] scratch: (key32 << 32) | ~id of the long path's candidates, unsorted
  unsigned long long* key64_sorted;  // [V] scratch: the same keys, descending
  float* probs;               // [V] scratch of the long path
  SampleState* st;
};

// Recent tokens that travel inside the fused top-k kernel's parameters.
constexpr int kSampleArgRecent = 256;

// The fused top-k step: everything it reads from the host is in here.
struct FastSampleArgs {
  SampleParams p;                // p.st unused; p.recent used when n_recent > kSampleArgRecent
  unsigned long long rng[4];     // xoshiro256++ state before the step
  int k, nlists;                 // top_k, lists merged by the last CTA (a power of two >= CTAs)
  unsigned long long* cand;      // [CTAs * k] scratch
  unsigned* nfin;                // [CTAs] scratch
  unsigned* done;                // CTA counter, 0 between calls
  SampleState* out;              // token and the state after the step (page-locked host memory, mapped)
  int recent_in_args;            // 1: the recent tokens are recent[0, p.n_recent)
  uint32_t recent[kSampleArgRecent];
};

// Marks recent[0, n) (tokens >= V skipped) with `call` (buildRepeatCounts
// only decides whether a token's count is non-zero).
cudaError_t launch_sample_mark(const uint32_t* recent, int n, unsigned* stamp, unsigned call, int V, cudaStream_t s);
// Greedy-with-penalties or the whole short-candidate sampling path; sets
// st->path = 1 when the candidate list is longer than kSampleSmallK.
cudaError_t launch_sample(const SampleParams& p, cudaStream_t s);
// The long-candidate path: sort the st->n_sort keys that launch_sample left
// in key64 (n_sort, read back by the host), then probabilities, top-p and
// the draw over the first st->k.
cudaError_t launch_sample_long(const SampleParams& p, int n_sort, cudaStream_t s);
// top_k in [1, kSampleFastK] with temperature > 0, one launch: CTA b keeps the
// best k of ids [1024 b, 1024 b + 1024), the last CTA to finish merges the
// lists and draws.  cand holds ceil(V / 1024) * k keys, nfin ceil(V / 1024) counts.
cudaError_t launch_sample_fast(const FastSampleArgs& a, cudaStream_t s);
cudaError_t configure_sampler();

}  // namespace vvli
