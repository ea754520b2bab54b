// vvli_ref_cpu.cpp - TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of VVLI's dense decoder path, used as the parity oracle and
// as the timed CPU baseline.  Only tests/, __graft_entry__.smoke() and the
// cpu-baseline / reference arms of bench.py load it; the product library
// (vvli_b200/libvvli_cuda.so) never links or calls it.
//
// The reference is Zig 0.16 (no Zig toolchain exists on this machine), so
// this file follows its source line by line:
//   src/llm.zig:720-766     forward op order (forwardCurrentEmbedding / forwardLayer)
//   src/llm.zig:1228-1285   linearInto / linearRange / resolveWorkerCount (threads per call)
//   src/llm.zig:1445-1466   dotBf16: simd_lanes partial sums, ordered reduce, FMA tail
//   src/llm.zig:1287-1300   rmsNormInto (+ sumSquares :1421-1431)
//   src/llm.zig:1302-1335   computeAttentionInto (+ softmaxInPlace :1408-1419, addScaled :1398-1406)
//   src/llm.zig:1337-1371   applyRoPE / rotatePair
//   src/llm.zig:1382-1396   siluMulInto / addInto
//   src/llm.zig:778-803     argmax, bf16ToF32, f32ToBf16
//   src/llm.zig:488-537, 814-837  weight blob layout (assignSlices / storageElementCount)
//   src/generator.zig:142-175, 338-463  greedy loop and Sampler helpers
// Zig's default float mode is strict: a*b+c is two roundings unless written
// @mulAdd.  This file is compiled with -ffp-contract=off and uses std::fma
// exactly where the reference writes @mulAdd.
//
// Parity pins: the reference's known-answer tests (src/llm.zig:1690-1782,
// src/tensor.zig:848-878, src/generator.zig:491-512) and fp32 `transformers`
// forwards of the same weights (tests/golden/).  Transcendentals use libm's
// expf/powf/sinf/cosf where Zig uses its own std.math; they agree to ulps.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <thread>
#include <vector>

#include "../include/vvli_cuda.h"

namespace {

constexpr size_t kMaxWorkerThreads = 64;      // src/llm.zig:11
constexpr size_t kElemsPerCacheLine = 32;     // 64-byte alignment of bf16 tensors, src/llm.zig:1499-1504

// ---------------------------------------------------------------- bf16 (src/llm.zig:791-803)
inline float bf16_to_f32(uint16_t bits) {
  uint32_t u = static_cast<uint32_t>(bits) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t f32_to_bf16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  uint32_t rounded = bits + 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<uint16_t>(rounded >> 16);
}

// ---------------------------------------------------------------- config helpers (src/llm.zig:195-276)
inline uint64_t head_dim(const vvli_model_config& c) { return c.hidden_size / c.num_attention_heads; }
inline uint64_t kv_dim(const vvli_model_config& c) { return c.num_key_value_heads * head_dim(c); }
inline uint64_t kv_group(const vvli_model_config& c) { return c.num_attention_heads / c.num_key_value_heads; }

int validate(const vvli_model_config& c) {
  if (c.vocab_size == 0 || c.hidden_size == 0 || c.intermediate_size == 0 || c.num_hidden_layers == 0 ||
      c.num_attention_heads == 0 || c.num_key_value_heads == 0 || c.max_position_embeddings == 0)
    return VVLI_ERR_INVALID_CONFIG;
  if (c.hidden_size % c.num_attention_heads != 0) return VVLI_ERR_INVALID_CONFIG;
  if (c.num_attention_heads % c.num_key_value_heads != 0) return VVLI_ERR_INVALID_CONFIG;
  if (head_dim(c) % 2 != 0) return VVLI_ERR_INVALID_CONFIG;
  if (c.num_experts == 0) {
    if (c.num_experts_per_token != 0) return VVLI_ERR_INVALID_CONFIG;
  } else {
    if (c.num_experts_per_token == 0 || c.num_experts_per_token > c.num_experts) return VVLI_ERR_INVALID_CONFIG;
    return VVLI_ERR_UNSUPPORTED_ARCH;  // supportsDenseRunner() is false for MoE
  }
  if (c.architecture == VVLI_ARCH_OLMOE) return VVLI_ERR_UNSUPPORTED_ARCH;
  return VVLI_OK;
}

inline uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Offsets of one layer's tensors inside the blob (assignSlices, src/llm.zig:488-522).
struct LayerOffsets {
  uint64_t input_norm, q, q_bias, k, k_bias, v, v_bias, o, post_norm, gate, up, down;
};

struct BlobLayout {
  uint64_t embedding = 0;
  std::vector<LayerOffsets> layers;
  uint64_t final_norm = 0;
  uint64_t lm_head = UINT64_MAX;
  uint64_t total = 0;
};

BlobLayout blob_layout(const vvli_model_config& c) {
  BlobLayout b;
  uint64_t cur = 0;
  auto take = [&](uint64_t len) {
    cur = align_up(cur, kElemsPerCacheLine);
    uint64_t start = cur;
    cur += len;
    return start;
  };
  const uint64_t h = c.hidden_size, kv = kv_dim(c), inter = c.intermediate_size;
  b.embedding = take(c.vocab_size * h);
  b.layers.resize(c.num_hidden_layers);
  for (auto& L : b.layers) {
    L.input_norm = take(h);
    L.q = take(h * h);
    L.q_bias = c.qkv_bias ? take(h) : UINT64_MAX;
    L.k = take(kv * h);
    L.k_bias = c.qkv_bias ? take(kv) : UINT64_MAX;
    L.v = take(kv * h);
    L.v_bias = c.qkv_bias ? take(kv) : UINT64_MAX;
    L.o = take(h * h);
    L.post_norm = take(h);
    L.gate = take(inter * h);
    L.up = take(inter * h);
    L.down = take(h * inter);
  }
  b.final_norm = take(h);
  if (!c.tie_word_embeddings) b.lm_head = take(c.vocab_size * h);
  // storageElementCount aligns each addition's start but not the end (src/llm.zig:1490-1493).
  b.total = cur;
  return b;
}

// ---------------------------------------------------------------- synthetic weights
// Counter-based generator shared bit-for-bit with the device generator in
// vvli_b200/csrc/weights.cu: SplitMix64 outputs -> twelve 16-bit uniforms ->
// Irwin-Hall sum (exact in fp32) -> * std in fp32 -> reference f32ToBf16.
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

inline uint64_t tensor_key(uint64_t seed, uint64_t tensor_id) {
  return mix64(seed ^ mix64(tensor_id + 0x632BE59BD9B4E019ull));
}

inline uint16_t synth_value(uint64_t key, uint64_t idx, float stddev) {
  uint32_t s = 0;
  for (uint64_t j = 0; j < 3; ++j) {
    uint64_t hsh = mix64(key + (3 * idx + j + 1) * kGolden);
    s += static_cast<uint32_t>(hsh & 0xffff) + static_cast<uint32_t>((hsh >> 16) & 0xffff) +
         static_cast<uint32_t>((hsh >> 32) & 0xffff) + static_cast<uint32_t>(hsh >> 48);
  }
  float z = static_cast<float>(static_cast<int32_t>(s) - 393210) * (1.0f / 65536.0f);
  return f32_to_bf16(z * stddev);
}

struct TensorSpec {
  uint64_t offset, len, tensor_id;
  int kind;  // 0 = normal(std), 1 = ones
};

std::vector<TensorSpec> tensor_specs(const vvli_model_config& c, const BlobLayout& b) {
  const uint64_t h = c.hidden_size, kv = kv_dim(c), inter = c.intermediate_size;
  std::vector<TensorSpec> s;
  s.push_back({b.embedding, c.vocab_size * h, 0, 0});
  for (uint64_t l = 0; l < c.num_hidden_layers; ++l) {
    const auto& L = b.layers[l];
    const uint64_t base = 1 + 12 * l;
    s.push_back({L.input_norm, h, base + 0, 1});
    s.push_back({L.q, h * h, base + 1, 0});
    if (c.qkv_bias) s.push_back({L.q_bias, h, base + 2, 0});
    s.push_back({L.k, kv * h, base + 3, 0});
    if (c.qkv_bias) s.push_back({L.k_bias, kv, base + 4, 0});
    s.push_back({L.v, kv * h, base + 5, 0});
    if (c.qkv_bias) s.push_back({L.v_bias, kv, base + 6, 0});
    s.push_back({L.o, h * h, base + 7, 0});
    s.push_back({L.post_norm, h, base + 8, 1});
    s.push_back({L.gate, inter * h, base + 9, 0});
    s.push_back({L.up, inter * h, base + 10, 0});
    s.push_back({L.down, h * inter, base + 11, 0});
  }
  s.push_back({b.final_norm, h, 1 + 12 * c.num_hidden_layers, 1});
  if (!c.tie_word_embeddings) s.push_back({b.lm_head, c.vocab_size * h, 2 + 12 * c.num_hidden_layers, 0});
  return s;
}

// ---------------------------------------------------------------- kernels
// dotBf16 / dotF32 (src/llm.zig:1433-1455): L strided partial sums (mul then
// add, two roundings), ordered horizontal reduce, FMA tail.
template <int L>
__attribute__((target_clones("avx512f", "avx2", "default")))
float dot_bf16(const uint16_t* a, const float* b, size_t n) {
  float acc[L];
  for (int l = 0; l < L; ++l) acc[l] = 0.0f;
  size_t i = 0;
  for (; i + L <= n; i += L) {
    for (int l = 0; l < L; ++l) {
      float p = bf16_to_f32(a[i + l]) * b[i + l];
      acc[l] = acc[l] + p;
    }
  }
  float sum = 0.0f;
  for (int l = 0; l < L; ++l) sum = sum + acc[l];
  for (; i < n; ++i) sum = std::fma(bf16_to_f32(a[i]), b[i], sum);
  return sum;
}

template <int L>
float dot_f32(const float* a, const float* b, size_t n) {
  float acc[L];
  for (int l = 0; l < L; ++l) acc[l] = 0.0f;
  size_t i = 0;
  for (; i + L <= n; i += L)
    for (int l = 0; l < L; ++l) acc[l] = acc[l] + a[i + l] * b[i + l];
  float sum = 0.0f;
  for (int l = 0; l < L; ++l) sum = sum + acc[l];
  for (; i < n; ++i) sum = std::fma(a[i], b[i], sum);
  return sum;
}

// One weight element as f32: bf16 bits widened, or an f32 weight as is
// (Matrix storage .bf16 / .f32 of the reference).
inline float wval(uint16_t v) { return bf16_to_f32(v); }
inline float wval(float v) { return v; }
template <int L>
float dot_w(const uint16_t* a, const float* b, size_t n) { return dot_bf16<L>(a, b, n); }
template <int L>
float dot_w(const float* a, const float* b, size_t n) { return dot_f32<L>(a, b, n); }

template <int L>
float sum_squares(const float* v, size_t n) {  // src/llm.zig:1421-1431
  float acc[L];
  for (int l = 0; l < L; ++l) acc[l] = 0.0f;
  size_t i = 0;
  for (; i + L <= n; i += L)
    for (int l = 0; l < L; ++l) acc[l] = acc[l] + v[i + l] * v[i + l];
  float sum = 0.0f;
  for (int l = 0; l < L; ++l) sum = sum + acc[l];
  for (; i < n; ++i) sum = std::fma(v[i], v[i], sum);
  return sum;
}

// rmsNormInto (src/llm.zig:1287-1300); weight is bf16 (or f32 when w_f32).
template <int L>
void rms_norm(float* out, const float* in, const uint16_t* w_bf16, const float* w_f32, size_t n, float eps) {
  const float mean_square = sum_squares<L>(in, n) / static_cast<float>(n);
  const float scale = 1.0f / std::sqrt(mean_square + eps);
  for (size_t i = 0; i < n; ++i) {
    const float w = w_f32 ? w_f32[i] : bf16_to_f32(w_bf16[i]);
    out[i] = in[i] * w * scale;
  }
}

// softmaxInPlace (src/llm.zig:1408-1419).
void softmax_in_place(float* v, size_t n) {
  float mx = v[0];
  for (size_t i = 1; i < n; ++i) mx = std::max(mx, v[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    v[i] = std::exp(v[i] - mx);
    sum += v[i];
  }
  const float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) v[i] *= inv;
}

// addScaled (src/llm.zig:1398-1406): vector body mul-then-add, FMA tail.
template <int L>
void add_scaled(float* out, const float* values, float scale, size_t n) {
  size_t i = 0;
  for (; i + L <= n; i += L)
    for (int l = 0; l < L; ++l) out[i + l] = out[i + l] + values[i + l] * scale;
  for (; i < n; ++i) out[i] = std::fma(values[i], scale, out[i]);
}

// Inverse frequency of rotary pair `dim_index` (src/llm.zig:1361-1364), with
// the optional llama3 rope_scaling extension (not in the reference, which
// ignores rope_scaling): the published Llama 3.1 frequency rule, wavelength
// bands [orig/high, orig/low] interpolated between inv_freq and inv_freq/factor.
float rope_inv_freq(const vvli_model_config& c, size_t dim_index, float dim_f) {
  const float exponent = static_cast<float>(dim_index) / dim_f;
  float inv_freq = 1.0f / std::pow(c.rope_theta, exponent);
  if (c.rope_scaling_type == VVLI_ROPE_SCALING_LLAMA3) {
    const float two_pi = 6.283185307179586f;
    const float orig = static_cast<float>(c.rope_original_max_position);
    const float low_wavelen = orig / c.rope_low_freq_factor;
    const float high_wavelen = orig / c.rope_high_freq_factor;
    const float wavelen = two_pi / inv_freq;
    if (wavelen > low_wavelen) {
      inv_freq = inv_freq / c.rope_scaling_factor;
    } else if (!(wavelen < high_wavelen)) {
      const float smooth = (orig / wavelen - c.rope_low_freq_factor) /
                           (c.rope_high_freq_factor - c.rope_low_freq_factor);
      inv_freq = (1.0f - smooth) * inv_freq / c.rope_scaling_factor + smooth * inv_freq;
    }
  }
  return inv_freq;
}

// applyRoPE / rotatePair (src/llm.zig:1337-1371).
void apply_rope(float* values, size_t heads, size_t hd, size_t position, const vvli_model_config& c) {
  const float pos_f = static_cast<float>(position);
  const float dim_f = static_cast<float>(hd);
  auto rotate = [&](float* v, size_t first, size_t second, size_t dim_index) {
    const float inv_freq = rope_inv_freq(c, dim_index, dim_f);
    const float angle = pos_f * inv_freq;
    const float cs = std::cos(angle), sn = std::sin(angle);
    const float x0 = v[first], x1 = v[second];
    v[first] = x0 * cs - x1 * sn;
    v[second] = x0 * sn + x1 * cs;
  };
  for (size_t head = 0; head < heads; ++head) {
    float* hs = values + head * hd;
    if (c.rope_layout == VVLI_ROPE_INTERLEAVED) {
      for (size_t i = 0; i < hd; i += 2) rotate(hs, i, i + 1, i);
    } else {
      const size_t half = hd / 2;
      for (size_t i = 0; i < half; ++i) rotate(hs, i, i + half, i * 2);
    }
  }
}

// argmax (src/llm.zig:778-789): strict >, first index wins ties.
size_t argmax(const float* v, size_t n) {
  size_t best = 0;
  float bv = v[0];
  for (size_t i = 1; i < n; ++i)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return best;
}

// ---------------------------------------------------------------- linearInto (src/llm.zig:1228-1285)
struct RuntimeOptions {
  size_t thread_count = 0;          // 0 = host CPU count
  size_t min_rows_per_thread = 64;
};

size_t resolve_worker_count(size_t rows, const RuntimeOptions& o) {
  if (rows == 0) return 1;
  size_t requested = o.thread_count == 0 ? std::max<size_t>(1, std::thread::hardware_concurrency()) : o.thread_count;
  if (requested <= 1) return 1;
  const size_t min_rows = std::max<size_t>(o.min_rows_per_thread, 1);
  const size_t useful = std::max<size_t>(1, rows / min_rows);
  return std::max<size_t>(1, std::min(std::min(requested, useful), kMaxWorkerThreads));
}

template <int L, typename T>
void linear_range(float* out, const T* W, size_t K, const float* x, const T* bias, size_t start, size_t end) {
  for (size_t row = start; row < end; ++row)
    out[row] = dot_w<L>(W + row * K, x, K) + (bias ? wval(bias[row]) : 0.0f);
}

// A fresh set of OS threads per call, as the reference spawns and joins
// std.Thread workers inside every linearInto.
template <int L, typename T>
void linear_into(float* out, const T* W, size_t N, size_t K, const float* x, const T* bias,
                 const RuntimeOptions& o) {
  const size_t workers = resolve_worker_count(N, o);
  if (workers == 1) {
    linear_range<L, T>(out, W, K, x, bias, 0, N);
    return;
  }
  const size_t per = (N + workers - 1) / workers;
  std::vector<std::thread> threads;
  threads.reserve(workers);
  size_t spawned = 0;
  for (; spawned + 1 < workers; ++spawned) {
    const size_t start = std::min(spawned * per, N);
    const size_t end = std::min(start + per, N);
    threads.emplace_back([=] { linear_range<L, T>(out, W, K, x, bias, start, end); });
  }
  linear_range<L, T>(out, W, K, x, bias, std::min(spawned * per, N), N);
  for (auto& t : threads) t.join();
}

// ---------------------------------------------------------------- Runner (src/llm.zig:688-776)
struct Runner {
  vvli_model_config cfg{};
  BlobLayout layout;
  std::vector<uint16_t> owned;  // set when the runner generated its own weights
  const uint16_t* blob = nullptr;
  // f32 weights in the same layout (element offsets of the bf16 blob), used
  // instead of `blob` when set: the reference's .f32 Matrix storage, which
  // dequantised GGUF tensors (Q8_0, Q4_0) need.
  const float* blob_f32 = nullptr;
  size_t max_seq = 0;
  RuntimeOptions opts;
  int lanes = 16;
  std::vector<float> keys, values;
  std::vector<float> x, residual, norm, q, k, v, attention, projected, gate, up, ff, scores, logits;
  std::vector<float> hidden;  // x after every layer, [layers][hidden]
  // Checker conveniences (never set by the timed CPU baseline): attention
  // over q heads on several threads, and a forward that stops before the LM
  // head.  Neither changes the arithmetic of any value that is produced.
  size_t attention_threads = 1;
  bool skip_lm_head = false;
  std::vector<float> head_scores;  // [attention_threads][max_seq]
};

// One q head of computeAttentionInto; `used` is that head's score scratch.
template <int L>
void attention_head(Runner& r, size_t layer, size_t position, size_t qh, float* used) {
  const auto& c = r.cfg;
  const size_t hd = head_dim(c), group = kv_group(c), kvd = kv_dim(c);
  const float inv_sqrt_head = 1.0f / std::sqrt(static_cast<float>(hd));
  {
    const size_t kvh = qh / group;
    const float* qs = r.q.data() + qh * hd;
    for (size_t t = 0; t <= position; ++t) {
      const float* key = r.keys.data() + (layer * r.max_seq + t) * kvd + kvh * hd;
      used[t] = dot_f32<L>(qs, key, hd) * inv_sqrt_head;
    }
    softmax_in_place(used, position + 1);
    float* oh = r.attention.data() + qh * hd;
    std::fill(oh, oh + hd, 0.0f);
    for (size_t t = 0; t <= position; ++t) {
      const float* val = r.values.data() + (layer * r.max_seq + t) * kvd + kvh * hd;
      add_scaled<L>(oh, val, used[t], hd);
    }
  }
}

template <int L>
void attention_into(Runner& r, size_t layer, size_t position) {  // src/llm.zig:1302-1335
  const size_t heads = r.cfg.num_attention_heads;
  std::fill(r.attention.begin(), r.attention.end(), 0.0f);
  const size_t T = std::min(r.attention_threads, heads);
  if (T <= 1) {  // the reference: one thread, heads in order
    for (size_t qh = 0; qh < heads; ++qh) attention_head<L>(r, layer, position, qh, r.scores.data());
    return;
  }
  // Checker only: heads are independent, so splitting them over threads
  // gives every output the same arithmetic as the sequential loop.
  std::vector<std::thread> ts;
  for (size_t t = 0; t < T; ++t)
    ts.emplace_back([&, t] {
      for (size_t qh = t; qh < heads; qh += T) attention_head<L>(r, layer, position, qh, r.head_scores.data() + t * r.max_seq);
    });
  for (auto& th : ts) th.join();
}

// rmsNormInto with a weight of either storage.
template <int L>
void rms_norm_w(float* out, const float* in, const uint16_t* w, size_t n, float eps) {
  rms_norm<L>(out, in, w, nullptr, n, eps);
}
template <int L>
void rms_norm_w(float* out, const float* in, const float* w, size_t n, float eps) {
  rms_norm<L>(out, in, nullptr, w, n, eps);
}

template <int L, typename T>
void forward_current(Runner& r, size_t position, const T* B) {  // src/llm.zig:720-766
  const auto& c = r.cfg;
  const size_t h = c.hidden_size, kvd = kv_dim(c), inter = c.intermediate_size, hd = head_dim(c);
  for (size_t l = 0; l < c.num_hidden_layers; ++l) {
    const auto& Lo = r.layout.layers[l];
    auto bias = [&](uint64_t off) -> const T* { return off == UINT64_MAX ? nullptr : B + off; };
    std::copy(r.x.begin(), r.x.end(), r.residual.begin());
    rms_norm_w<L>(r.norm.data(), r.x.data(), B + Lo.input_norm, h, c.rms_norm_eps);
    linear_into<L, T>(r.q.data(), B + Lo.q, h, h, r.norm.data(), bias(Lo.q_bias), r.opts);
    linear_into<L, T>(r.k.data(), B + Lo.k, kvd, h, r.norm.data(), bias(Lo.k_bias), r.opts);
    linear_into<L, T>(r.v.data(), B + Lo.v, kvd, h, r.norm.data(), bias(Lo.v_bias), r.opts);
    apply_rope(r.q.data(), c.num_attention_heads, hd, position, c);
    apply_rope(r.k.data(), c.num_key_value_heads, hd, position, c);
    std::copy(r.k.begin(), r.k.end(), r.keys.begin() + (l * r.max_seq + position) * kvd);
    std::copy(r.v.begin(), r.v.end(), r.values.begin() + (l * r.max_seq + position) * kvd);
    attention_into<L>(r, l, position);
    linear_into<L, T>(r.projected.data(), B + Lo.o, h, h, r.attention.data(), nullptr, r.opts);
    for (size_t i = 0; i < h; ++i) r.x[i] = r.residual[i] + r.projected[i];
    std::copy(r.x.begin(), r.x.end(), r.residual.begin());
    rms_norm_w<L>(r.norm.data(), r.x.data(), B + Lo.post_norm, h, c.rms_norm_eps);
    linear_into<L, T>(r.gate.data(), B + Lo.gate, inter, h, r.norm.data(), nullptr, r.opts);
    linear_into<L, T>(r.up.data(), B + Lo.up, inter, h, r.norm.data(), nullptr, r.opts);
    for (size_t i = 0; i < inter; ++i) {
      const float g = r.gate[i];
      r.ff[i] = (g / (1.0f + std::exp(-g))) * r.up[i];
    }
    linear_into<L, T>(r.projected.data(), B + Lo.down, h, inter, r.ff.data(), nullptr, r.opts);
    for (size_t i = 0; i < h; ++i) r.x[i] = r.residual[i] + r.projected[i];
    std::copy(r.x.begin(), r.x.end(), r.hidden.begin() + l * h);
  }
  if (r.skip_lm_head) return;
  rms_norm_w<L>(r.norm.data(), r.x.data(), B + r.layout.final_norm, h, c.rms_norm_eps);
  const uint64_t head = r.layout.lm_head == UINT64_MAX ? r.layout.embedding : r.layout.lm_head;
  linear_into<L, T>(r.logits.data(), B + head, c.vocab_size, h, r.norm.data(), nullptr, r.opts);
}

void forward_dispatch(Runner& r, size_t position) {
  switch (r.lanes) {
    case 4: r.blob_f32 ? forward_current<4>(r, position, r.blob_f32) : forward_current<4>(r, position, r.blob); break;
    case 8: r.blob_f32 ? forward_current<8>(r, position, r.blob_f32) : forward_current<8>(r, position, r.blob); break;
    default:
      r.blob_f32 ? forward_current<16>(r, position, r.blob_f32) : forward_current<16>(r, position, r.blob);
      break;
  }
}

int host_simd_lanes() {
  // std.simd.suggestVectorLength(f32) on the build CPU: 512-bit -> 16, 256-bit -> 8, else 4.
  if (__builtin_cpu_supports("avx512f")) return 16;
  if (__builtin_cpu_supports("avx2")) return 8;
  return 4;
}

void parallel_for(size_t n, size_t threads, const auto& fn) {
  if (threads <= 1 || n < 1024) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> ts;
  const size_t per = (n + threads - 1) / threads;
  for (size_t t = 0; t < threads; ++t) {
    const size_t s = std::min(n, t * per), e = std::min(n, s + per);
    if (s < e) ts.emplace_back([&, s, e] { fn(s, e); });
  }
  for (auto& t : ts) t.join();
}

void fill_synthetic(const vvli_model_config& c, uint64_t seed, uint16_t* blob, uint64_t n, size_t threads) {
  const BlobLayout b = blob_layout(c);
  std::memset(blob, 0, n * sizeof(uint16_t));
  for (const auto& t : tensor_specs(c, b)) {
    uint16_t* dst = blob + t.offset;
    if (t.kind == 1) {
      std::fill(dst, dst + t.len, static_cast<uint16_t>(0x3F80));
      continue;
    }
    const uint64_t key = tensor_key(seed, t.tensor_id);
    parallel_for(t.len, threads, [&](size_t s, size_t e) {
      for (size_t i = s; i < e; ++i) dst[i] = synth_value(key, i, 0.02f);
    });
  }
}

}  // namespace

// ================================================================ C ABI (ctypes)
extern "C" {

uint16_t ref_f32_to_bf16(float v) { return f32_to_bf16(v); }
float ref_bf16_to_f32(uint16_t b) { return bf16_to_f32(b); }
int ref_host_simd_lanes() { return host_simd_lanes(); }
int ref_validate(const vvli_model_config* c) { return validate(*c); }

uint64_t ref_storage_elements(const vvli_model_config* c) { return blob_layout(*c).total; }

// Offsets of every tensor, in blob order, as (offset, len, tensor_id) triples.
uint64_t ref_tensor_table(const vvli_model_config* c, uint64_t* out, uint64_t cap) {
  const auto specs = tensor_specs(*c, blob_layout(*c));
  for (size_t i = 0; i < specs.size() && i < cap; ++i) {
    out[3 * i] = specs[i].offset;
    out[3 * i + 1] = specs[i].len;
    out[3 * i + 2] = specs[i].tensor_id;
  }
  return specs.size();
}

void ref_fill_synthetic(const vvli_model_config* c, uint64_t seed, uint16_t* blob, uint64_t n, uint64_t threads) {
  fill_synthetic(*c, seed, blob, n, threads ? threads : std::max(1u, std::thread::hardware_concurrency()));
}

// OwnedModel.fillDeterministicForTesting, bf16 kind (src/llm.zig:466-477).
void ref_fill_deterministic(uint16_t* blob, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) {
    const int32_t centered = static_cast<int32_t>(i % 251) - 125;
    blob[i] = f32_to_bf16(static_cast<float>(centered) * 0.001f);
  }
}

void ref_rms_norm(float* out, const float* in, const float* w, uint64_t n, float eps, int lanes) {
  if (lanes == 4) rms_norm<4>(out, in, nullptr, w, n, eps);
  else if (lanes == 8) rms_norm<8>(out, in, nullptr, w, n, eps);
  else rms_norm<16>(out, in, nullptr, w, n, eps);
}

void ref_softmax(float* v, uint64_t n) { softmax_in_place(v, n); }
uint64_t ref_argmax(const float* v, uint64_t n) { return argmax(v, n); }

void ref_apply_rope(float* values, uint64_t heads, uint64_t hd, uint64_t position, const vvli_model_config* c) {
  apply_rope(values, heads, hd, position, *c);
}

void ref_linear(float* out, const uint16_t* W, uint64_t N, uint64_t K, const float* x, const uint16_t* bias,
                uint64_t threads, int lanes) {
  RuntimeOptions o;
  o.thread_count = threads;
  if (lanes == 4) linear_into<4>(out, W, N, K, x, bias, o);
  else if (lanes == 8) linear_into<8>(out, W, N, K, x, bias, o);
  else linear_into<16>(out, W, N, K, x, bias, o);
}

// Runner lifecycle.  `blob` must outlive the runner unless `synthetic_seed`
// >= 0, in which case the runner generates and owns its weights.
void* ref_runner_create(const vvli_model_config* c, const uint16_t* blob, uint64_t n_elements, int64_t synthetic_seed,
                        uint64_t max_seq, uint64_t threads, uint64_t min_rows_per_thread, int lanes, int* status) {
  *status = validate(*c);
  if (*status != VVLI_OK) return nullptr;
  if (max_seq == 0 || max_seq > c->max_position_embeddings) {
    *status = VVLI_ERR_INVALID_CONFIG;
    return nullptr;
  }
  auto r = std::make_unique<Runner>();
  r->cfg = *c;
  r->layout = blob_layout(*c);
  if (synthetic_seed >= 0) {
    r->owned.resize(r->layout.total);
    fill_synthetic(*c, static_cast<uint64_t>(synthetic_seed), r->owned.data(), r->layout.total,
                   threads ? threads : std::max(1u, std::thread::hardware_concurrency()));
    r->blob = r->owned.data();
  } else {
    if (blob == nullptr || n_elements < r->layout.total) {
      *status = VVLI_ERR_INVALID_WEIGHT;
      return nullptr;
    }
    r->blob = blob;
  }
  r->max_seq = max_seq;
  r->opts.thread_count = threads;
  r->opts.min_rows_per_thread = min_rows_per_thread ? min_rows_per_thread : 64;
  r->lanes = lanes > 0 ? lanes : host_simd_lanes();
  const size_t h = c->hidden_size, kvd = kv_dim(*c), inter = c->intermediate_size;
  r->keys.assign(c->num_hidden_layers * max_seq * kvd, 0.0f);
  r->values.assign(c->num_hidden_layers * max_seq * kvd, 0.0f);
  r->x.resize(h);
  r->residual.resize(h);
  r->norm.resize(h);
  r->q.resize(h);
  r->k.resize(kvd);
  r->v.resize(kvd);
  r->attention.resize(h);
  r->projected.resize(std::max(h, inter));
  r->gate.resize(inter);
  r->up.resize(inter);
  r->ff.resize(inter);
  r->scores.resize(max_seq);
  r->logits.resize(c->vocab_size);
  r->hidden.assign(c->num_hidden_layers * h, 0.0f);
  *status = VVLI_OK;
  return r.release();
}

// A runner over f32 weights in the bf16 blob's layout (n_elements f32
// values, kept by the caller for the runner's life): the reference's .f32
// Matrix storage, for models whose tensors are dequantised GGUF blocks.
void* ref_runner_create_f32(const vvli_model_config* c, const float* blob, uint64_t n_elements, uint64_t max_seq,
                            uint64_t threads, uint64_t min_rows_per_thread, int lanes, int* status) {
  if (!blob || n_elements < blob_layout(*c).total) {
    *status = VVLI_ERR_INVALID_WEIGHT;
    return nullptr;
  }
  // The bf16 blob pointer is never read when blob_f32 is set; a dummy keeps
  // the bf16 creation path's checks.
  static const uint16_t dummy = 0;
  auto* r = static_cast<Runner*>(ref_runner_create(c, &dummy, UINT64_MAX, -1, max_seq, threads,
                                                   min_rows_per_thread, lanes, status));
  if (!r) return nullptr;
  r->blob = nullptr;
  r->blob_f32 = blob;
  return r;
}

void ref_runner_destroy(void* p) { delete static_cast<Runner*>(p); }

const uint16_t* ref_runner_blob(void* p) { return static_cast<Runner*>(p)->blob; }

void ref_runner_reset(void* p) {  // KVCache.clear (src/llm.zig:576-579)
  auto* r = static_cast<Runner*>(p);
  std::fill(r->keys.begin(), r->keys.end(), 0.0f);
  std::fill(r->values.begin(), r->values.end(), 0.0f);
}

// Runner.forwardToken (src/llm.zig:702-709) + copyEmbeddingToken (:1373-1380).
int ref_runner_forward_token(void* p, uint32_t token, uint64_t position, float* logits_out) {
  auto* r = static_cast<Runner*>(p);
  if (token >= r->cfg.vocab_size) return VVLI_ERR_INVALID_TOKEN;
  if (position >= r->max_seq) return VVLI_ERR_CONTEXT_FULL;
  const uint64_t row = r->layout.embedding + static_cast<uint64_t>(token) * r->cfg.hidden_size;
  for (size_t i = 0; i < r->cfg.hidden_size; ++i)
    r->x[i] = r->blob_f32 ? r->blob_f32[row + i] : bf16_to_f32(r->blob[row + i]);
  forward_dispatch(*r, position);
  if (logits_out) std::copy(r->logits.begin(), r->logits.end(), logits_out);
  return VVLI_OK;
}

// Runner.forwardEmbedding (src/llm.zig:711-718).
int ref_runner_forward_embedding(void* p, const float* embedding, uint64_t position, float* logits_out) {
  auto* r = static_cast<Runner*>(p);
  if (position >= r->max_seq) return VVLI_ERR_CONTEXT_FULL;
  std::copy(embedding, embedding + r->cfg.hidden_size, r->x.begin());
  forward_dispatch(*r, position);
  if (logits_out) std::copy(r->logits.begin(), r->logits.end(), logits_out);
  return VVLI_OK;
}

// Checker only: runs heads of computeAttentionInto on `threads` threads
// (1 = the reference's sequential loop).  Results are bit-identical.
void ref_runner_set_attention_threads(void* p, uint64_t threads) {
  auto* r = static_cast<Runner*>(p);
  r->attention_threads = std::max<uint64_t>(1, threads);
  r->head_scores.assign(r->attention_threads * r->max_seq, 0.0f);
}

// Checker only: forwardToken over tokens[0, n) at positions start.., with the
// final norm and LM head run for the last token alone (earlier positions'
// logits are never read by a prompt loop).  Every hidden state and the last
// logits are what n forwardToken calls give.
int ref_runner_prefill(void* p, const uint32_t* tokens, uint64_t n, uint64_t start, float* logits_out) {
  auto* r = static_cast<Runner*>(p);
  for (uint64_t i = 0; i < n; ++i) {
    r->skip_lm_head = i + 1 < n;
    const int st = ref_runner_forward_token(p, tokens[i], start + i, i + 1 < n ? nullptr : logits_out);
    r->skip_lm_head = false;
    if (st) return st;
  }
  return VVLI_OK;
}

void ref_runner_hidden(void* p, uint64_t layer, float* out) {
  auto* r = static_cast<Runner*>(p);
  const size_t h = r->cfg.hidden_size;
  std::copy(r->hidden.begin() + layer * h, r->hidden.begin() + (layer + 1) * h, out);
}

void ref_runner_logits(void* p, float* out) {
  auto* r = static_cast<Runner*>(p);
  std::copy(r->logits.begin(), r->logits.end(), out);
}

// generateGreedy (src/generator.zig:142-175).  eos < 0 means no eos.
int ref_generate_greedy(void* p, const uint32_t* prompt, uint64_t n_prompt, uint64_t max_new, int64_t eos,
                        uint32_t* out, uint64_t* produced_out) {
  auto* r = static_cast<Runner*>(p);
  if (n_prompt == 0) return VVLI_ERR_EMPTY_PROMPT;
  uint64_t position = 0;
  for (uint64_t i = 0; i < n_prompt; ++i) {
    int st = ref_runner_forward_token(p, prompt[i], position, nullptr);
    if (st) return st;
    ++position;
  }
  uint64_t produced = 0;
  while (produced < max_new) {
    const uint32_t next = static_cast<uint32_t>(argmax(r->logits.data(), r->cfg.vocab_size));
    out[produced] = next;
    if (eos >= 0 && next == static_cast<uint32_t>(eos)) {
      ++produced;
      break;
    }
    int st = ref_runner_forward_token(p, next, position, nullptr);
    if (st) return st;
    ++position;
    ++produced;
  }
  *produced_out = produced;
  return VVLI_OK;
}

// ---------------------------------------------------------------- Sampler helpers (src/generator.zig:338-463)
int ref_validate_sampling(float temperature, float top_p, float repeat_penalty) {
  if (temperature < 0.0f || std::isnan(temperature)) return VVLI_ERR_INVALID_SAMPLING;
  if (top_p <= 0.0f || top_p > 1.0f || std::isnan(top_p)) return VVLI_ERR_INVALID_SAMPLING;
  if (repeat_penalty < 1.0f || std::isnan(repeat_penalty)) return VVLI_ERR_INVALID_SAMPLING;
  return VVLI_OK;
}

void ref_build_repeat_counts(uint16_t* counts, uint64_t n, const uint32_t* prompt, uint64_t n_prompt,
                             const uint32_t* generated, uint64_t n_generated, float repeat_penalty,
                             uint64_t repeat_last_n) {
  std::fill(counts, counts + n, 0);
  if (repeat_penalty <= 1.0f || repeat_last_n == 0) return;
  const uint64_t total = n_prompt + n_generated;
  const uint64_t start = total > repeat_last_n ? total - repeat_last_n : 0;
  for (uint64_t i = start; i < total; ++i) {
    const uint32_t tok = i < n_prompt ? prompt[i] : generated[i - n_prompt];
    if (tok >= n) continue;
    if (counts[tok] != 0xffff) ++counts[tok];
  }
}

static inline float adjusted_logit(float logit, uint16_t count, float rp) {  // :399-402
  if (count == 0 || rp <= 1.0f) return logit;
  return logit < 0.0f ? logit * rp : logit / rp;
}

uint32_t ref_greedy_with_penalties(const float* logits, const uint16_t* counts, uint64_t n, float rp) {  // :362-374
  uint32_t best = 0;
  float bl = adjusted_logit(logits[0], counts[0], rp);
  for (uint64_t i = 1; i < n; ++i) {
    const float s = adjusted_logit(logits[i], counts[i], rp);
    if (s > bl) {
      bl = s;
      best = static_cast<uint32_t>(i);
    }
  }
  return best;
}

struct Candidate {
  uint32_t id;
  float logit;
  float probability;
};

// buildCandidates (:376-397) with insertTopCandidate/bubbleCandidateUp (:404-422).
uint64_t ref_build_candidates(Candidate* cands, const float* logits, const uint16_t* counts, uint64_t n,
                              uint64_t top_k, float rp) {
  const uint64_t limit = top_k == 0 ? n : std::min<uint64_t>(top_k, n);
  uint64_t count = 0;
  if (limit == n) {
    for (uint64_t i = 0; i < n; ++i) {
      const float s = adjusted_logit(logits[i], counts[i], rp);
      if (!std::isfinite(s)) continue;
      cands[count++] = {static_cast<uint32_t>(i), s, 0.0f};
    }
    // std.sort.pdq is not stable; candidates with equal logits may come out
    // in either order there.  A stable sort is one valid outcome.
    std::stable_sort(cands, cands + count, [](const Candidate& a, const Candidate& b) { return a.logit > b.logit; });
    return count;
  }
  for (uint64_t i = 0; i < n; ++i) {
    const float s = adjusted_logit(logits[i], counts[i], rp);
    if (!std::isfinite(s)) continue;
    Candidate c{static_cast<uint32_t>(i), s, 0.0f};
    if (limit == 0) continue;
    uint64_t at;
    if (count < limit) {
      cands[count] = c;
      at = count++;
    } else {
      if (c.logit <= cands[count - 1].logit) continue;
      cands[count - 1] = c;
      at = count - 1;
    }
    while (at > 0 && cands[at].logit > cands[at - 1].logit) {
      std::swap(cands[at], cands[at - 1]);
      --at;
    }
  }
  return count;
}

// prepareProbabilities (:428-449).
uint64_t ref_prepare_probabilities(Candidate* cands, uint64_t n, float temperature, float top_p) {
  if (n == 0) return 0;
  const float t = std::max(temperature, 1e-6f);
  const float mx = cands[0].logit;
  float total = 0.0f;
  for (uint64_t i = 0; i < n; ++i) {
    const float pr = std::exp((cands[i].logit - mx) / t);
    cands[i].probability = std::isfinite(pr) ? pr : 0.0f;
    total += cands[i].probability;
  }
  if (total <= 0.0f || !std::isfinite(total)) return 1;
  if (top_p >= 1.0f) return n;
  float cum = 0.0f;
  for (uint64_t i = 0; i < n; ++i) {
    cum += cands[i].probability;
    if (cum / total >= top_p) return i + 1;
  }
  return n;
}

// sampleCandidate (:451-463).
uint32_t ref_sample_candidate(const Candidate* cands, uint64_t n, float random_unit) {
  float total = 0.0f;
  for (uint64_t i = 0; i < n; ++i) total += cands[i].probability;
  if (total <= 0.0f || !std::isfinite(total)) return cands[0].id;
  const float target = std::min(random_unit, 0.99999994f) * total;
  float cum = 0.0f;
  for (uint64_t i = 0; i < n; ++i) {
    cum += cands[i].probability;
    if (target <= cum) return cands[i].id;
  }
  return cands[n - 1].id;
}

uint64_t ref_candidate_size() { return sizeof(Candidate); }

// Sampler.next (:97-126) given the uniform draw the PRNG would produce.
int ref_sampler_next(const float* logits, uint64_t n, const uint32_t* prompt, uint64_t n_prompt,
                     const uint32_t* generated, uint64_t n_generated, const vvli_sample_options* o, float random_unit,
                     uint32_t* out) {
  int st = ref_validate_sampling(o->temperature, o->top_p, o->repeat_penalty);
  if (st) return st;
  std::vector<uint16_t> counts(n);
  ref_build_repeat_counts(counts.data(), n, prompt, n_prompt, generated, n_generated, o->repeat_penalty,
                          o->repeat_last_n);
  if (o->temperature <= 0.0f) {
    *out = ref_greedy_with_penalties(logits, counts.data(), n, o->repeat_penalty);
    return VVLI_OK;
  }
  std::vector<Candidate> cands(n);
  const uint64_t cc = ref_build_candidates(cands.data(), logits, counts.data(), n, o->top_k, o->repeat_penalty);
  if (cc == 0) {
    *out = static_cast<uint32_t>(argmax(logits, n));
    return VVLI_OK;
  }
  const uint64_t sc = ref_prepare_probabilities(cands.data(), cc, o->temperature, o->top_p);
  if (sc == 0) {
    *out = cands[0].id;
    return VVLI_OK;
  }
  *out = ref_sample_candidate(cands.data(), sc, random_unit);
  return VVLI_OK;
}

}  // extern "C"
