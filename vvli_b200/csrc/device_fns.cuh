// device_fns.cuh - device functions shared by the decode kernels and the megakernel.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace vvli {

// ---------------------------------------------------------------- shared helpers
VVLI_DEV float dot8(uint4 w, const float* x) {
  float acc = bf16_lo(w.x) * x[0];
  acc = fmaf(bf16_hi(w.x), x[1], acc);
  acc = fmaf(bf16_lo(w.y), x[2], acc);
  acc = fmaf(bf16_hi(w.y), x[3], acc);
  acc = fmaf(bf16_lo(w.z), x[4], acc);
  acc = fmaf(bf16_hi(w.z), x[5], acc);
  acc = fmaf(bf16_lo(w.w), x[6], acc);
  acc = fmaf(bf16_hi(w.w), x[7], acc);
  return acc;
}

// Publishes the step's argmax and advances the device step state: the token
// following position `pos` is the argmax unless it is a prompt token.
VVLI_DEV void publish_argmax(StepState* st, int* seq_tokens, int best) {
  st->argmax = best;
  const int np = st->pos + 1;
  if (np <= st->max_seq && np >= st->prompt_len) seq_tokens[np] = best;  // seq_tokens has max_seq + 1 slots
  st->pos = np;
}

// Sums a (lanes 0-15 get it) and b (lanes 16-31 get it) over the warp with
// one butterfly: the first exchange swaps halves, so two reductions cost
// five shuffles.
VVLI_DEV float warp_sum2(float a, float b, int lane) {
  const bool hi = lane & 16;
  float v = hi ? b : a;
  v += __shfl_xor_sync(0xffffffffu, hi ? a : b, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- RoPE
// Inverse frequency of rotary pair `dim_index` (rotatePair, src/llm.zig:1361-1364)
// with the optional llama3 rope_scaling rule.
VVLI_DEV float rope_inv_freq(const RopeParams& r, int dim_index, int d) {
  const float exponent = static_cast<float>(dim_index) / static_cast<float>(d);
  float inv_freq = 1.0f / powf(r.theta, exponent);
  if (r.scaling == 1) {
    const float two_pi = 6.283185307179586f;
    const float low_wavelen = r.orig / r.low;
    const float high_wavelen = r.orig / r.high;
    const float wavelen = two_pi / inv_freq;
    if (wavelen > low_wavelen) {
      inv_freq = inv_freq / r.factor;
    } else if (!(wavelen < high_wavelen)) {
      const float smooth = (r.orig / wavelen - r.low) / (r.high - r.low);
      inv_freq = (1.0f - smooth) * inv_freq / r.factor + smooth * inv_freq;
    }
  }
  return inv_freq;
}

// Pair i of a head (0 <= i < d/2): element indices and the frequency index
// (applyRoPE, src/llm.zig:1337-1359).
VVLI_DEV void rope_pair(int layout, int i, int d, int& first, int& second, int& dim_index) {
  if (layout == 0) {
    first = 2 * i;
    second = 2 * i + 1;
  } else {
    first = i;
    second = i + d / 2;
  }
  dim_index = 2 * i;
}

VVLI_DEV void rope_rotate(const RopeParams& rp, int pos, int i, int d, const float* src, float* dst) {
  int a, b, di;
  rope_pair(rp.layout, i, d, a, b, di);
  const float ang = static_cast<float>(pos) * rope_inv_freq(rp, di, d);
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const float x0 = src[a], x1 = src[b];
  dst[a] = x0 * cs - x1 * sn;
  dst[b] = x0 * sn + x1 * cs;
}

VVLI_DEV size_t kv_off(const int* pt, int t, int g, int nkv, int d) {
  const int page = pt[t / kPage];
  return (static_cast<size_t>(page * nkv + g) * kPage + (t % kPage)) * d;
}

// Sum over the warp of p[0..7] (one partial dot product per q head of the
// group): three exchange-halving steps leave head (bit2 + 2 bit3 + 4 bit4) of
// the lane index in each lane, two more finish the sum (9 shuffles in all).
VVLI_DEV float reduce_heads8(const float* p, int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float q[4], r[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = b4 ? p[i + 4] : p[i], send = b4 ? p[i] : p[i + 4];
    q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b3 ? q[i + 2] : q[i], send = b3 ? q[i] : q[i + 2];
    r[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float t = (b2 ? r[1] : r[0]) + __shfl_xor_sync(0xffffffffu, b2 ? r[0] : r[1], 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return t;
}

// The same for four heads p[0..3]: two exchange-halving steps leave head
// (bit3 + 2 bit4) of the lane index in each lane, three more finish the sum.
VVLI_DEV float reduce_heads4(const float* p, int lane) {
  const bool b4 = lane & 16, b3 = lane & 8;
  float q[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b4 ? p[i + 2] : p[i], send = b4 ? p[i] : p[i + 2];
    q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float t = (b3 ? q[1] : q[0]) + __shfl_xor_sync(0xffffffffu, b3 ? q[0] : q[1], 8);
  t += __shfl_xor_sync(0xffffffffu, t, 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return t;
}

}  // namespace vvli
