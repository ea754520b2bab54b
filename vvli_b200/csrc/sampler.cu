// sampler.cu - Sampler.next (src/generator.zig:97-126, 338-463) on the device.
//
// One CTA of 1024 threads does the whole step for candidate lists of up to
// kSampleSmallK entries (the reference's default top_k is 40):
//   1. adjusted logits (adjustedLogit, :399-402) from the logits and a
//      per-token stamp of the last repeat_last_n tokens (only "count != 0"
//      matters to the reference);
//   2. temperature <= 0: the penalised argmax (greedyWithPenalties, :362-374);
//   3. else the top-k candidates by (adjusted logit desc, id asc) - the order
//      insertTopCandidate/bubbleCandidateUp leave them in (:404-422) - found
//      by a three-level radix select over order-preserving 32-bit keys, with
//      ties at the threshold taken in id order, then a bitonic sort in
//      shared memory;
//   4. exp((l - max) / T), the sequential fp32 sums, the top-p cut and the
//      cumulative draw (prepareProbabilities/sampleCandidate, :428-463) on one
//      thread, in the reference's order, so the sums round the same way.
// Longer candidate lists (top_k = 0 or > kSampleSmallK) run step 4 over the
// sorted list, where the scan stops at the first probability below half an
// ulp of its running sum (every later one is smaller: the sum can no longer
// change).  The running sum is >= 1 from the first candidate on (the maximum,
// exp(0)), so a candidate with (l - max) / T < -17.5 (probability below
// 2.6e-8 < 2^-24) is never reached: only the keys above that cut are sorted,
// in 8,192-key chunks in shared memory, each key then placed by its rank
// among the other chunks (binary searches).
//
// The uniform draw is random.float(f32) of Zig's DefaultPrng: xoshiro256++
// (the published generator) with the float built from 23 mantissa bits and a
// leading-zero count for the exponent.  It is drawn only when the reference
// draws it: temperature > 0 and at least one finite candidate.
#include <algorithm>

#include "common.cuh"
#include "sampler.cuh"

namespace vvli {
namespace {

constexpr int kST = 1024;   // threads of the sampling CTA
constexpr int kBins = 4096;  // radix-select histogram (12 bits)
constexpr size_t kSampleSmem = static_cast<size_t>(kSampleSmallK) * (8 + 4);
constexpr int kSortChunk = 8192;       // keys sorted per CTA on the long path
constexpr float kLongCut = -17.5f;     // (l - max) / T below this: never reached by the long path's scan

// Finite floats -> unsigned keys in the same order (never 0; +0 and -0 equal).
VVLI_DEV unsigned order_key(float s) {
  const unsigned u = __float_as_uint(s == 0.0f ? 0.0f : s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
VVLI_DEV float key_value(unsigned k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }
VVLI_DEV unsigned long long make_key64(unsigned k, int id) {
  return (static_cast<unsigned long long>(k) << 32) | (0xffffffffu - static_cast<unsigned>(id));
}
VVLI_DEV unsigned key64_id(unsigned long long k) { return 0xffffffffu - static_cast<unsigned>(k & 0xffffffffull); }

VVLI_DEV float adjusted_logit(float l, bool recent, float rp) {  // :399-402
  if (!recent || rp <= 1.0f) return l;
  return l < 0.0f ? l * rp : l / rp;
}

VVLI_DEV unsigned long long rotl64(unsigned long long x, int k) { return (x << k) | (x >> (64 - k)); }
VVLI_DEV unsigned long long xoshiro_next(unsigned long long* s) {
  const unsigned long long r = rotl64(s[0] + s[3], 23) + s[0];
  const unsigned long long t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return r;
}
// random.float(f32): uniform in [0, 1) with the exponent from leading zeros.
VVLI_DEV float xoshiro_float(unsigned long long* s) {
  const unsigned long long rand = xoshiro_next(s);
  int lz = __clzll(static_cast<long long>(rand));
  if (lz >= 41) {
    lz = 41 + __clzll(static_cast<long long>(xoshiro_next(s)));
    if (lz == 41 + 64) lz += __clz(static_cast<int>(static_cast<unsigned>(xoshiro_next(s)) | 0x7ffu));
  }
  return __uint_as_float((static_cast<unsigned>(126 - lz) << 23) | static_cast<unsigned>(rand & 0x7fffffull));
}

// exp of an fp32 argument, rounded once to fp32 from a double-precision exp.
VVLI_DEV float prob_of(float logit, float max_logit, float t) {
  const float pr = static_cast<float>(exp(static_cast<double>((logit - max_logit) / t)));
  return isfinite(pr) ? pr : 0.0f;
}

// Adding p (or anything smaller) to `sum` leaves it unchanged.
VVLI_DEV bool negligible(float p, float sum) { return p < 0.5f * (nextafterf(sum, INFINITY) - sum); }

// Exclusive prefix sum over the CTA's threads in index order; *total = sum.
__device__ unsigned block_excl_scan(unsigned v, unsigned* wsum, unsigned* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    unsigned w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  const unsigned excl = x - v + (warp > 0 ? wsum[warp - 1] : 0u);
  *total = wsum[31];
  __syncthreads();
  return excl;
}

// Argmax over the CTA (first index of the maximum, NaN never chosen); result on all threads.
__device__ int block_argmax(float v, int i, float* wv, int* wi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  warp_argmax(v, i);
  if (lane == 0) {
    wv[warp] = v;
    wi[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    v = wv[lane];
    i = wi[lane];
    warp_argmax(v, i);
    if (lane == 0) wi[0] = i;
  }
  __syncthreads();
  const int r = wi[0];
  __syncthreads();
  return r;
}

// prepareProbabilities (:428-449) and sampleCandidate (:451-463) over the k
// keys cand[0, k), sorted descending, in shared memory; every thread calls it.
__device__ void finish_sorted(const SampleParams& p, const unsigned long long* rng_in, SampleState* st,
                              const unsigned long long* cand, float* probs, unsigned k) {
  const int tid = threadIdx.x;
  const float t = fmaxf(p.temperature, 1e-6f);
  const float mx = key_value(static_cast<unsigned>(cand[0] >> 32));
  for (int j = tid; j < static_cast<int>(k); j += blockDim.x) probs[j] = prob_of(key_value(static_cast<unsigned>(cand[j] >> 32)), mx, t);
  __syncthreads();
  if (tid == 0) {
    float total = 0.0f;
    for (unsigned j = 0; j < k; ++j) total += probs[j];
    unsigned count = k;
    if (!(total > 0.0f) || !isfinite(total)) {
      count = 1;
    } else if (p.top_p < 1.0f) {
      float cum = 0.0f;
      for (unsigned j = 0; j < k; ++j) {
        cum += probs[j];
        if (cum / total >= p.top_p) {
          count = j + 1;
          break;
        }
      }
    }
    unsigned long long s[4] = {rng_in[0], rng_in[1], rng_in[2], rng_in[3]};
    const float u = xoshiro_float(s);
    float total2 = 0.0f;
    for (unsigned j = 0; j < count; ++j) total2 += probs[j];
    unsigned tok = key64_id(cand[0]);
    if (total2 > 0.0f && isfinite(total2)) {
      const float target = fminf(u, 0.99999994f) * total2;
      float cum = 0.0f;
      tok = key64_id(cand[count - 1]);
      for (unsigned j = 0; j < count; ++j) {
        cum += probs[j];
        if (target <= cum) {
          tok = key64_id(cand[j]);
          break;
        }
      }
    }
    for (int q = 0; q < 4; ++q) st->rng[q] = s[q];
    st->token = static_cast<int>(tok);
    st->path = 0;
  }
}

// ---------------------------------------------------------------- small top-k (k <= kSampleFastK)
// Sorting networks on 64-key lists held two keys per lane (index lane and
// lane + 32), descending.  Keys are unique (the id is in the low bits) except
// the zeros of padding and non-finite logits, which sort last.
VVLI_DEV unsigned long long kmax(unsigned long long a, unsigned long long b) { return a > b ? a : b; }
VVLI_DEV unsigned long long kmin(unsigned long long a, unsigned long long b) { return a < b ? a : b; }

// One compare-exchange at `stride` (< 32) for the element of index `idx`:
// the lower index of a pair keeps the larger key when `desc`.
VVLI_DEV unsigned long long cx_step(unsigned long long v, int idx, int stride, bool desc) {
  const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, stride);
  return ((idx & stride) == 0) == desc ? kmax(v, o) : kmin(v, o);
}

// Bitonic sort of 64 keys, descending.
VVLI_DEV void warp_sort64(unsigned long long& r0, unsigned long long& r1, int lane) {
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride == 32) {
        const unsigned long long hi = kmax(r0, r1), lo = kmin(r0, r1);
        r0 = hi, r1 = lo;
      } else {
        r0 = cx_step(r0, lane, stride, size == 64 || (lane & size) == 0);
        r1 = cx_step(r1, lane + 32, stride, size == 64 || ((lane + 32) & size) == 0);
      }
    }
  }
}

// Top 64 of two descending 64-lists a and b (shared memory), descending, into
// out (which may be a): max(a[i], b[63 - i]) is a bitonic sequence holding the
// 64 largest keys, then a bitonic merge sorts it.
VVLI_DEV void warp_merge64(const unsigned long long* a, const unsigned long long* b, unsigned long long* out,
                           int lane) {
  unsigned long long r0 = kmax(a[lane], b[63 - lane]);
  unsigned long long r1 = kmax(a[lane + 32], b[31 - lane]);
  __syncwarp();
  {
    const unsigned long long hi = kmax(r0, r1), lo = kmin(r0, r1);
    r0 = hi, r1 = lo;
  }
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
    r0 = cx_step(r0, lane, stride, true);
    r1 = cx_step(r1, lane + 32, stride, true);
  }
  out[lane] = r0;
  out[lane + 32] = r1;
}

// Merges n (a power of two) 64-lists lists[i * 64] in place, pairwise by
// levels, into lists[0]; every thread of the CTA calls it.
__device__ void merge_lists(unsigned long long* lists, int n) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  for (int step = 1; step < n; step <<= 1) {
    for (int m = warp; m < n / (2 * step); m += warps) {
      unsigned long long* a = lists + static_cast<size_t>(2 * step * m) * 64;
      warp_merge64(a, a + static_cast<size_t>(step) * 64, a, lane);
    }
    __syncthreads();
  }
}

// CTA b takes ids [1024 b, 1024 b + 1024): each warp sorts 64 of them, the
// CTA merges its 16 lists and writes its best k to cand[b * k ..] and its
// count of finite adjusted logits to nfin[b].  The last CTA to finish (a
// counter) merges every CTA's list in CTA order, so the result does not
// depend on which CTA that is, and runs the probabilities, top-p and draw.
__global__ void __launch_bounds__(512) topk_sample_kernel(const __grid_constant__ FastSampleArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* lists = reinterpret_cast<unsigned long long*>(smem);  // [max(16, nlists)][64]
  float* probs = reinterpret_cast<float*>(lists + static_cast<size_t>(max(16, a.nlists)) * 64);  // [kSampleFastK]
  __shared__ unsigned wcount[16];
  __shared__ unsigned recent_bits[32];  // ids [1024 b, 1024 b + 1024) among the recent tokens
  __shared__ unsigned last;
  const SampleParams& p = a.p;
  const int k = a.k;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = blockIdx.x * 1024;
  if (!p.stamp) {
    const uint32_t* rec = a.recent_in_args ? a.recent : p.recent;
    if (threadIdx.x < 32) recent_bits[threadIdx.x] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < p.n_recent; i += blockDim.x) {
      const int t = static_cast<int>(rec[i]) - base;
      if (t >= 0 && t < 1024) atomicOr(&recent_bits[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
  }
  unsigned long long r[2];
  unsigned mine = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int id = base + warp * 64 + lane + 32 * h;
    r[h] = 0ull;
    if (id < p.V) {
      const int t = id - base;
      const bool rec = p.stamp ? p.stamp[id] == p.call : ((recent_bits[t >> 5] >> (t & 31)) & 1u) != 0;
      const float s = adjusted_logit(p.logits[id], rec, p.repeat_penalty);
      if (isfinite(s)) {
        r[h] = make_key64(order_key(s), id);
        ++mine;
      }
    }
  }
  mine = __reduce_add_sync(0xffffffffu, mine);
  if (lane == 0) wcount[warp] = mine;
  warp_sort64(r[0], r[1], lane);
  lists[warp * 64 + lane] = r[0];
  lists[warp * 64 + lane + 32] = r[1];
  __syncthreads();
  merge_lists(lists, 16);
  for (int i = threadIdx.x; i < k; i += blockDim.x) a.cand[static_cast<size_t>(blockIdx.x) * k + i] = lists[i];
  if (threadIdx.x == 0) {
    unsigned t = 0;
    for (int w = 0; w < 16; ++w) t += wcount[w];
    a.nfin[blockIdx.x] = t;
  }
  // publish this CTA's list, then count it in
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(a.done, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int nblk = gridDim.x;
  unsigned c = 0;
  for (int b = threadIdx.x; b < nblk; b += blockDim.x) c += __ldcg(a.nfin + b);
  c = __reduce_add_sync(0xffffffffu, c);
  if (lane == 0) wcount[warp] = c;
  __syncthreads();
  unsigned n_finite = 0;
  for (int w = 0; w < 16; ++w) n_finite += wcount[w];
  if (threadIdx.x == 0) *a.done = 0;  // ready for the next call (stream order)
  SampleState* st = a.out;
  if (n_finite == 0) {  // no candidate: llm.argmax of the raw logits (:115), rare
    if (threadIdx.x == 0) {
      float bv = p.logits[0];
      int bi = 0;
      for (int i = 1; i < p.V; ++i)
        if (p.logits[i] > bv) {
          bv = p.logits[i];
          bi = i;
        }
      for (int q = 0; q < 4; ++q) st->rng[q] = a.rng[q];
      st->token = bi;
      st->path = 0;
    }
    return;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.nlists * 64; i += blockDim.x) {
    const int b = i >> 6, j = i & 63;
    lists[i] = (b < nblk && j < k) ? __ldcg(a.cand + static_cast<size_t>(b) * k + j) : 0ull;
  }
  __syncthreads();
  merge_lists(lists, a.nlists);
  finish_sorted(p, a.rng, st, lists, probs, min(static_cast<unsigned>(k), n_finite));
}

__global__ void sample_mark_kernel(const uint32_t* recent, int n, unsigned* stamp, unsigned call, int V) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const uint32_t t = recent[i];
    if (t < static_cast<uint32_t>(V)) stamp[t] = call;
  }
}

__global__ void __launch_bounds__(kST, 1) sample_kernel(const SampleParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);  // [kSampleSmallK]
  float* probs = reinterpret_cast<float*>(cand + kSampleSmallK);            // [kSampleSmallK]
  __shared__ unsigned hist[kBins];
  __shared__ unsigned wsum[32];
  __shared__ float wv[32];
  __shared__ int wi[32];
  __shared__ unsigned found[2];
  const int tid = threadIdx.x;
  const int V = p.V;
  const float rp = p.repeat_penalty;
  SampleState* st = p.st;

  if (p.temperature <= 0.0f) {
    // greedyWithPenalties (:362-374): strict '>' from element 0, so a NaN
    // there is never replaced and NaNs elsewhere never win.
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += kST) {
      const float s = adjusted_logit(p.logits[i], p.stamp[i] == p.call, rp);
      if (better(s, i, bv, bi)) {
        bv = s;
        bi = i;
      }
    }
    const int best = block_argmax(bv, bi, wv, wi);
    if (tid == 0) {
      const float s0 = adjusted_logit(p.logits[0], p.stamp[0] == p.call, rp);
      st->token = isnan(s0) || best == 0x7fffffff ? 0 : best;
      st->path = 0;
    }
    return;
  }

  // Keys of the finite adjusted logits (buildCandidates skips the others, :384, :392).
  unsigned nfin = 0;
  for (int i = tid; i < V; i += kST) {
    const float s = adjusted_logit(p.logits[i], p.stamp[i] == p.call, rp);
    const bool fin = isfinite(s);
    p.key32[i] = fin ? order_key(s) : 0u;
    nfin += fin ? 1u : 0u;
  }
  unsigned n_finite;
  block_excl_scan(nfin, wsum, &n_finite);  // its barriers also publish key32 to the CTA
  if (n_finite == 0) {
    // No candidate: llm.argmax of the raw logits (:115).
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += kST) {
      const float l = p.logits[i];
      if (better(l, i, bv, bi)) {
        bv = l;
        bi = i;
      }
    }
    const int best = block_argmax(bv, bi, wv, wi);
    if (tid == 0) {
      st->token = isnan(p.logits[0]) || best == 0x7fffffff ? 0 : best;
      st->path = 0;
    }
    return;
  }
  const unsigned long long limit = p.top_k == 0 ? static_cast<unsigned long long>(V)
                                                : (p.top_k < static_cast<unsigned long long>(V) ? p.top_k : V);
  const unsigned k = static_cast<unsigned>(limit < n_finite ? limit : n_finite);
  if (k > static_cast<unsigned>(kSampleSmallK)) {
    // The keys that the long path's scan can reach, compacted in id order.
    unsigned km = 0;
    for (int i = tid; i < V; i += kST) km = max(km, p.key32[i]);
    km = __reduce_max_sync(0xffffffffu, km);
    if ((tid & 31) == 0) wsum[tid >> 5] = km;
    __syncthreads();
    km = 0;
    for (int w = 0; w < kST / 32; ++w) km = max(km, wsum[w]);
    __syncthreads();
    const float mx = key_value(km);
    const float t = fmaxf(p.temperature, 1e-6f);
    auto keep = [&](unsigned kk) { return kk != 0 && (key_value(kk) - mx) / t >= kLongCut; };
    const int C = (V + kST - 1) / kST;
    const int i0 = min(V, tid * C), i1 = min(V, i0 + C);
    unsigned nk = 0;
    for (int i = i0; i < i1; ++i) nk += keep(p.key32[i]) ? 1u : 0u;
    unsigned n_keep;
    unsigned o = block_excl_scan(nk, wsum, &n_keep);
    for (int i = i0; i < i1; ++i)
      if (keep(p.key32[i])) p.key64[o++] = make_key64(p.key32[i], i);
    if (tid == 0) {
      st->path = 1;
      st->k = static_cast<int>(min(k, n_keep));
      st->n_sort = static_cast<int>(n_keep);
    }
    return;
  }

  // Radix select: the k-th largest key (threshold tau) in three levels.
  unsigned prefix = 0, mask = 0, need = k;
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
  for (int lv = 0; lv < 3; ++lv) {
    const int nb = 1 << widths[lv], sh = shifts[lv];
    for (int b = tid; b < nb; b += kST) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kST) {
      const unsigned kk = p.key32[i];
      if (kk != 0 && (kk & mask) == prefix) atomicAdd(&hist[(kk >> sh) & (nb - 1)], 1u);
    }
    __syncthreads();
    const int bpt = nb >= kST ? nb / kST : 1;
    const int b0 = tid * bpt;
    unsigned local = 0;
    for (int j = 0; j < bpt; ++j)
      if (b0 + j < nb) local += hist[b0 + j];
    unsigned total;
    const unsigned excl = block_excl_scan(local, wsum, &total);
    unsigned run = total - excl - local;  // keys in the bins of higher-numbered threads
    for (int j = bpt - 1; j >= 0; --j) {
      const int b = b0 + j;
      if (b >= nb) continue;
      const unsigned h = hist[b];
      if (run < need && run + h >= need) {
        found[0] = static_cast<unsigned>(b);
        found[1] = run;
      }
      run += h;
    }
    __syncthreads();
    need -= found[1];
    prefix |= found[0] << sh;
    mask |= static_cast<unsigned>(nb - 1) << sh;
    __syncthreads();
  }
  const unsigned tau = prefix;
  const unsigned c_gt = k - need;  // keys above tau; `need` keys equal to tau are taken, lowest ids first

  // Compaction in id order: thread t scans ids [t*C, (t+1)*C).
  const int C = (V + kST - 1) / kST;
  const int i0 = min(V, tid * C), i1 = min(V, i0 + C);
  unsigned ngt = 0, neq = 0;
  for (int i = i0; i < i1; ++i) {
    const unsigned kk = p.key32[i];
    ngt += kk > tau ? 1u : 0u;
    neq += kk == tau ? 1u : 0u;
  }
  unsigned tot_gt, tot_eq;
  unsigned og = block_excl_scan(ngt, wsum, &tot_gt);
  unsigned oe = block_excl_scan(neq, wsum, &tot_eq);
  for (int i = i0; i < i1; ++i) {
    const unsigned kk = p.key32[i];
    if (kk > tau) {
      cand[og++] = make_key64(kk, i);
    } else if (kk == tau) {
      if (oe < need) cand[c_gt + oe] = make_key64(kk, i);
      ++oe;
    }
  }
  int N = 1;
  while (N < static_cast<int>(k)) N <<= 1;
  for (int j = static_cast<int>(k) + tid; j < N; j += kST) cand[j] = 0ull;
  __syncthreads();
  // Bitonic sort, descending.
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < N / 2; i += kST) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = cand[lo], b = cand[hi];
        if ((a < b) == desc) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  finish_sorted(p, p.st->rng, p.st, cand, probs, k);
}

// Sorts keys[c * kSortChunk ..] (n keys in all) descending, chunk c per CTA,
// into out (which may be keys).
__global__ void __launch_bounds__(1024) sort_chunk_kernel(const unsigned long long* keys, int n,
                                                          unsigned long long* out) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* a = reinterpret_cast<unsigned long long*>(smem);  // [kSortChunk]
  const int base = blockIdx.x * kSortChunk;
  const int len = min(kSortChunk, n - base);
  int N = 64;
  while (N < len) N <<= 1;
  for (int i = threadIdx.x; i < N; i += blockDim.x) a[i] = i < len ? keys[base + i] : 0ull;
  __syncthreads();
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < N / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < len; i += blockDim.x) out[base + i] = a[i];
}

// Key g of the sorted chunks goes to its place in the whole list: its index
// in its chunk plus, for every other chunk, the number of keys there above it
// (keys are distinct: the id is part of the key).
__global__ void rank_place_kernel(const unsigned long long* chunks, int n, unsigned long long* out) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const unsigned long long x = chunks[g];
  const int mine = g / kSortChunk;
  int pos = g - mine * kSortChunk;
  for (int c = 0; c * kSortChunk < n; ++c) {
    if (c == mine) continue;
    const unsigned long long* a = chunks + static_cast<size_t>(c) * kSortChunk;
    int lo = 0, hi = min(kSortChunk, n - c * kSortChunk);  // first index with a[idx] < x
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (a[mid] > x)
        lo = mid + 1;
      else
        hi = mid;
    }
    pos += lo;
  }
  out[pos] = x;
}

// Step 4 over the first st->k keys of the sorted candidates.
__global__ void __launch_bounds__(kST, 1) sample_long_kernel(const SampleParams p) {
  SampleState* st = p.st;
  const int k = st->k;
  const unsigned long long* keys = p.key64_sorted;
  const float t = fmaxf(p.temperature, 1e-6f);
  const float mx = key_value(static_cast<unsigned>(keys[0] >> 32));
  for (int j = threadIdx.x; j < k; j += kST) p.probs[j] = prob_of(key_value(static_cast<unsigned>(keys[j] >> 32)), mx, t);
  __syncthreads();
  if (threadIdx.x != 0) return;
  const float* pr = p.probs;
  float total = 0.0f;
  for (int j = 0; j < k; ++j) {
    if (negligible(pr[j], total)) break;
    total += pr[j];
  }
  int count = k;
  float total2 = total;
  if (!(total > 0.0f) || !isfinite(total)) {
    count = 1;
    total2 = pr[0];
  } else if (p.top_p < 1.0f) {
    float cum = 0.0f;
    for (int j = 0; j < k; ++j) {
      if (negligible(pr[j], cum)) break;
      cum += pr[j];
      if (cum / total >= p.top_p) {
        count = j + 1;
        break;
      }
    }
    total2 = cum;  // the sum of the first `count` probabilities, added in the same order
  }
  unsigned long long s[4] = {st->rng[0], st->rng[1], st->rng[2], st->rng[3]};
  const float u = xoshiro_float(s);
  unsigned tok = key64_id(keys[0]);
  if (total2 > 0.0f && isfinite(total2)) {
    const float target = fminf(u, 0.99999994f) * total2;
    float cum = 0.0f;
    tok = key64_id(keys[min(count, k) - 1]);
    for (int j = 0; j < count; ++j) {
      if (negligible(pr[j], cum)) break;
      cum += pr[j];
      if (target <= cum) {
        tok = key64_id(keys[j]);
        break;
      }
    }
  }
  for (int q = 0; q < 4; ++q) st->rng[q] = s[q];
  st->token = static_cast<int>(tok);
  st->path = 0;
}

}  // namespace

cudaError_t launch_sample_mark(const uint32_t* recent, int n, unsigned* stamp, unsigned call, int V, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  sample_mark_kernel<<<(n + 255) / 256, 256, 0, s>>>(recent, n, stamp, call, V);
  return cudaGetLastError();
}

cudaError_t launch_sample(const SampleParams& p, cudaStream_t s) {
  sample_kernel<<<1, kST, kSampleSmem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sample_long(const SampleParams& p, int n_sort, cudaStream_t s) {
  if (n_sort < 1 || n_sort > p.V) return cudaErrorInvalidValue;
  const int chunks = (n_sort + kSortChunk - 1) / kSortChunk;
  const size_t smem = static_cast<size_t>(kSortChunk) * 8;
  if (chunks == 1) {
    sort_chunk_kernel<<<1, 1024, smem, s>>>(p.key64, n_sort, p.key64_sorted);
  } else {
    sort_chunk_kernel<<<chunks, 1024, smem, s>>>(p.key64, n_sort, p.key64);
    rank_place_kernel<<<(n_sort + 255) / 256, 256, 0, s>>>(p.key64, n_sort, p.key64_sorted);
  }
  sample_long_kernel<<<1, kST, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sample_fast(const FastSampleArgs& a, cudaStream_t s) {
  const int nblk = (a.p.V + 1023) / 1024;
  if (a.k < 1 || a.k > kSampleFastK || a.nlists < nblk || a.nlists * 64 > kSampleFastMaxCand ||
      (a.recent_in_args && a.p.n_recent > kSampleArgRecent))
    return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(std::max(16, a.nlists)) * 64 * 8 + kSampleFastK * 4;
  topk_sample_kernel<<<nblk, 512, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t configure_sampler() {
  cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSampleSmem));
  if (e) return e;
  e = cudaFuncSetAttribute(sort_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSortChunk * 8);
  if (e) return e;
  return cudaFuncSetAttribute(topk_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(static_cast<size_t>(kSampleFastMaxCand) * 8 + kSampleFastK * 4));
}

}  // namespace vvli
