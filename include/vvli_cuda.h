/*
 * vvli_cuda.h - C ABI of the B200 (sm_100a) decoder runtime.
 *
 * This is the drop-in boundary for VVLI's dense decoder hot path.  The Zig host
 * (src/main.zig, src/generator.zig) binds these functions with @cImport and
 * links libvvli_cuda.so from build.zig; every entry point uses plain pointers,
 * sizes and the plain-C structs below (no C++ or torch types).  Each function
 * names the reference interface it replaces as path:line inside VVLI.
 *
 * Conventions (the reference's own FFI convention, src/gpu/metal_smoke.zig:5-11:
 * an extern struct for results and an int return code):
 *   - every function returns int: VVLI_OK (0) on success, a VVLI_ERR_* code
 *     otherwise; vvli_cuda_strerror() maps codes to text;
 *   - a context is single-caller (like llm.Runner, src/llm.zig:688-700) and
 *     every call is synchronous on return;
 *   - host buffers passed in are only read during the call; output buffers are
 *     host memory written before the call returns.
 */
#ifndef VVLI_CUDA_H
#define VVLI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes.  1..10 map 1:1 onto llm.Error (src/llm.zig:17-27) and
 * generator.Error (src/generator.zig:8-12), 11..13 onto gguf.Error
 * (src/gguf.zig:7-12); 20.. are added by this runtime. */
enum vvli_status {
  VVLI_OK = 0,
  VVLI_ERR_CONTEXT_FULL = 1,          /* llm.Error.ContextFull */
  VVLI_ERR_INVALID_CONFIG = 2,        /* llm.Error.InvalidConfig */
  VVLI_ERR_INVALID_TOKEN = 3,         /* llm.Error.InvalidToken */
  VVLI_ERR_INVALID_WEIGHT = 4,        /* llm.Error.InvalidWeight */
  VVLI_ERR_UNSUPPORTED_DTYPE = 5,     /* llm.Error.UnsupportedDType */
  VVLI_ERR_UNSUPPORTED_ARCH = 6,      /* llm.Error.UnsupportedModelArchitecture */
  VVLI_ERR_EMPTY_PROMPT = 7,          /* generator.Error.EmptyPrompt */
  VVLI_ERR_OUTPUT_TOO_SMALL = 8,      /* generator.Error.OutputTooSmall */
  VVLI_ERR_INVALID_SAMPLING = 9,      /* generator.Error.InvalidSamplingOptions */
  VVLI_ERR_MISSING_TENSOR = 10,       /* llm.Error.MissingSafetensorsTensor */
  VVLI_ERR_INVALID_GGUF = 11,         /* gguf.Error.InvalidGguf */
  VVLI_ERR_UNSUPPORTED_GGUF_VERSION = 12, /* gguf.Error.UnsupportedGgufVersion */
  VVLI_ERR_UNSUPPORTED_METADATA_TYPE = 13, /* gguf.Error.UnsupportedMetadataType */
  VVLI_ERR_CUDA = 20,                 /* a CUDA runtime call failed */
  VVLI_ERR_NCCL = 21,                 /* an NCCL call failed or NCCL is missing */
  VVLI_ERR_TIMEOUT = 22,              /* a bounded device-side wait gave up */
  VVLI_ERR_OOM = 23,                  /* device allocation failed */
  VVLI_ERR_NOT_LOADED = 24,           /* forward called before weights were loaded */
  VVLI_ERR_INVALID_ARGUMENT = 25,     /* null pointer, bad size or bad rank */
  VVLI_ERR_UNIMPLEMENTED = 26
};

/* llm.Architecture (src/llm.zig:29-43). */
enum vvli_architecture {
  VVLI_ARCH_LLAMA = 0,
  VVLI_ARCH_MISTRAL = 1,
  VVLI_ARCH_OLMOE = 2,
  VVLI_ARCH_QWEN2 = 3
};

/* llm.RopeLayout (src/llm.zig:50-53). */
enum vvli_rope_layout {
  VVLI_ROPE_INTERLEAVED = 0,
  VVLI_ROPE_SPLIT_HALF = 1
};

/* Extension: rope_scaling from config.json.  The reference ignores it
 * (src/llm.zig:98-145 never reads it); VVLI_ROPE_SCALING_NONE reproduces the
 * reference exactly. */
enum vvli_rope_scaling {
  VVLI_ROPE_SCALING_NONE = 0,
  VVLI_ROPE_SCALING_LLAMA3 = 1
};

/* Mirror of llm.Config (src/llm.zig:77-96) plus the rope_scaling extension. */
typedef struct vvli_model_config {
  uint64_t vocab_size;
  uint64_t hidden_size;
  uint64_t intermediate_size;
  uint64_t num_hidden_layers;
  uint64_t num_attention_heads;
  uint64_t num_key_value_heads;
  uint64_t max_position_embeddings;
  uint64_t num_experts;            /* 0 = dense (FeedForwardKind.dense) */
  uint64_t num_experts_per_token;
  uint32_t architecture;           /* enum vvli_architecture */
  uint32_t rope_layout;            /* enum vvli_rope_layout */
  float rope_theta;
  float rms_norm_eps;
  uint32_t tie_word_embeddings;    /* bool */
  uint32_t qkv_bias;               /* bool */
  uint32_t qk_norm;                /* bool; only OLMoE sets it, which is rejected */
  uint32_t eos_token_id;
  uint32_t pad_token_id;
  uint32_t rope_scaling_type;      /* enum vvli_rope_scaling */
  float rope_scaling_factor;
  float rope_low_freq_factor;
  float rope_high_freq_factor;
  uint32_t _pad0;
  uint64_t rope_original_max_position;
} vvli_model_config;

/* Per-call options of the decode path. */
typedef struct vvli_generate_stats {
  uint64_t prompt_tokens;
  uint64_t generated_tokens;
  int64_t prefill_nanoseconds;     /* generator.Stats (src/generator.zig:25-43) */
  int64_t decode_nanoseconds;
  int64_t total_nanoseconds;
} vvli_generate_stats;

/* generator.Options sampling fields (src/generator.zig:14-23).  eos < 0 means
 * "no eos" (eos_token_id = null). */
typedef struct vvli_sample_options {
  float temperature;
  float top_p;
  uint64_t top_k;
  float repeat_penalty;
  uint32_t _pad0;
  uint64_t repeat_last_n;
} vvli_sample_options;

typedef struct vvli_ctx vvli_ctx;

/* Size of the opaque NCCL unique id blob (ncclUniqueId is 128 bytes). */
#define VVLI_NCCL_ID_BYTES 128

/* Text for a status code.  Replaces writeAppError's error names
 * (src/main.zig:438-467).  Never returns NULL. */
const char* vvli_cuda_strerror(int status);

/* Text of the last failure on the calling thread (the failing call and the
 * CUDA/NCCL message), or "" if none.  Valid until the next call. */
const char* vvli_cuda_last_error(void);

/* Number of bf16 elements of the host weight blob for `cfg`, with every tensor
 * at a 64-byte aligned offset.  Replaces llm.storageElementCount
 * (src/llm.zig:814-837) for kind = .bf16. */
int vvli_cuda_storage_elements(const vvli_model_config* cfg, uint64_t* out_elements);

/* Fills `id` (VVLI_NCCL_ID_BYTES bytes) with a fresh NCCL unique id, to be
 * shared by the caller with every tensor-parallel rank before
 * vvli_cuda_create.  No counterpart in the reference (it has no
 * collectives); needed for the tensor-parallel split of src/llm.zig:732-766. */
int vvli_cuda_nccl_unique_id(void* id);

/* The tensor-parallel weight plan of rank `tp_rank` of `tp_size`, without a
 * GPU: one row of 9 uint64 per copied piece {device element offset, tensor id
 * in blob order, blob element offset of the tensor, rows, cols, source row
 * length, first source row, first source column, kind (0 matrix/bias, 1 norm)}.
 * q/k/v and gate/up are split by heads / rows, o_proj and down_proj by
 * columns, the LM head by vocabulary rows.  Writes at most `cap` rows to `out`
 * (may be NULL) and the total to `count`.  No counterpart in the reference,
 * which has no sharding; it describes how this runtime slices the
 * llm.OwnedModel blob (src/llm.zig:488-537). */
int vvli_cuda_tp_plan(const vvli_model_config* cfg, int tp_rank, int tp_size, uint64_t* out, uint64_t cap,
                      uint64_t* count);

/* Creates a context on `device` for rank `tp_rank` of `tp_size` ranks.
 * Replaces KVCache.init + Scratch.init + Runner.init
 * (src/llm.zig:546-562, 626-668, 694-700; called from src/main.zig:161-171).
 * `max_seq` mirrors KVCache.init's max_seq_len (0 < max_seq <=
 * max_position_embeddings, else VVLI_ERR_INVALID_CONFIG).  `max_batch` bounds
 * vvli_cuda_forward_batch and vvli_cuda_prefill chunk sizes.  For tp_size > 1,
 * `nccl_unique_id` must be the same blob on all ranks. */
int vvli_cuda_create(const vvli_model_config* cfg, int device, int tp_rank, int tp_size,
                     const void* nccl_unique_id, uint64_t max_seq, uint64_t max_batch,
                     vvli_ctx** out_ctx);

/* Uploads the bf16 weight blob laid out exactly as llm.OwnedModel.storage_bf16
 * (src/llm.zig:415-537: embedding; per layer [input_norm, q, q_bias?, k,
 * k_bias?, v, v_bias?, o, post_norm, gate, up, down]; final_norm; lm_head?).
 * Each rank copies only its own tensor-parallel shard.  Replaces the
 * safetensors/GGUF loaders' final copy into OwnedModel (src/llm.zig:923-1006);
 * the caller keeps ownership of `blob`. */
int vvli_cuda_load_weights(vvli_ctx* ctx, const uint16_t* blob, uint64_t n_elements);

/* Loads this rank's weights straight from a safetensors file
 * (loadOwnedFromSafetensorsFile + loadSafetensorsIntoOwnedModel,
 * src/llm.zig:859-883, 923-1006): the file is memory-mapped and only the
 * pieces of this rank's shard are copied to the device; F32 tensors are
 * rounded to bf16 with the reference's f32ToBf16 on the device.  Errors as
 * copyTensorIntoWeight: VVLI_ERR_MISSING_TENSOR, VVLI_ERR_UNSUPPORTED_DTYPE
 * (not BF16 / F32), VVLI_ERR_INVALID_WEIGHT (shape or byte range); a file
 * that cannot be opened gives VVLI_ERR_INVALID_ARGUMENT.  Same effect as
 * vvli_cuda_load_weights on the blob the reference would build. */
int vvli_cuda_load_safetensors(vvli_ctx* ctx, const char* path);

/* Loads this rank's weights straight from a GGUF file (loadOwnedFromGgufFile
 * + loadGgufIntoOwnedModel + copyGgufTensorIntoWeight, src/llm.zig:885-921,
 * 1008-1138; gguf.parse, src/gguf.zig:234-287).  The context's config must be
 * the one Config.fromGguf builds from the same file (src/llm.zig:153-193):
 * rope_layout INTERLEAVED (else VVLI_ERR_INVALID_CONFIG) and no q/k/v biases
 * (else VVLI_ERR_UNSUPPORTED_ARCH, as the reference).  Tensors may be F32,
 * F16 or BF16; F32 and F16 are rounded with f32ToBf16 on the device.  Errors:
 * VVLI_ERR_INVALID_GGUF, VVLI_ERR_UNSUPPORTED_GGUF_VERSION,
 * VVLI_ERR_UNSUPPORTED_METADATA_TYPE (as gguf.parse), then as
 * copyGgufTensorIntoWeight: VVLI_ERR_MISSING_TENSOR,
 * VVLI_ERR_UNSUPPORTED_DTYPE (a quantised type), VVLI_ERR_INVALID_WEIGHT
 * (element count or byte range); a file that cannot be opened gives
 * VVLI_ERR_INVALID_ARGUMENT. */
int vvli_cuda_load_gguf(vvli_ctx* ctx, const char* path);

/* Benchmark helper with no counterpart in the reference: fills the device
 * weights with the seeded synthetic model (every matrix and bias
 * ~N(0, 0.02) by a 12-term Irwin-Hall sum, norms 1.0), bit-identical to the
 * host generator that the CPU baseline uses, without a host blob. */
int vvli_cuda_fill_synthetic(vvli_ctx* ctx, uint64_t seed);

/* The same synthetic model with every matrix (embedding, q/k/v, o,
 * gate/up, down, LM head) block-quantised on the device: format 1 = GGML
 * Q8_0, 2 = GGML Q4_0 (32 weights and an fp16 scale per block; norms and
 * biases stay bf16).  The blocks are those a GGUF file of these weights
 * quantised with the published rules holds, so the model equals a
 * vvli_cuda_load_gguf of such a file.  No counterpart in the reference (it
 * rejects quantised tensors, src/llm.zig:1083); tp_size 1 only. */
int vvli_cuda_fill_synthetic_quantized(vvli_ctx* ctx, uint64_t seed, int format);

/* Zeroes the KV cache.  Replaces KVCache.clear (src/llm.zig:576-579). */
int vvli_cuda_reset(vvli_ctx* ctx);

/* One token through all layers at `position`.  Replaces Runner.forwardToken
 * (src/llm.zig:702-709).  Errors: VVLI_ERR_INVALID_TOKEN when token >= vocab,
 * VVLI_ERR_CONTEXT_FULL when position >= max_seq.  `logits_out` (vocab floats,
 * may be NULL) receives the logits the reference returns as a borrowed slice;
 * `argmax_out` (may be NULL) receives llm.argmax of them (src/llm.zig:778-789,
 * first index wins ties). */
int vvli_cuda_forward_token(vvli_ctx* ctx, uint32_t token, uint64_t position,
                            float* logits_out, uint32_t* argmax_out);

/* Like vvli_cuda_forward_token with a caller-supplied fp32 embedding of
 * hidden_size floats.  Replaces Runner.forwardEmbedding (src/llm.zig:711-718). */
int vvli_cuda_forward_embedding(vvli_ctx* ctx, const float* embedding, uint64_t position,
                                float* logits_out, uint32_t* argmax_out);

/* Runs `n` prompt tokens at positions start_position.. in one batched pass
 * (tensor-core GEMMs and causal attention).  Equal, within tolerance, to n
 * sequential vvli_cuda_forward_token calls; only the last token's logits are
 * returned.  Replaces the per-token prefill loop of
 * generateGreedyMeasuredInternal (src/generator.zig:243-251). */
int vvli_cuda_prefill(vvli_ctx* ctx, const uint32_t* tokens, uint64_t n, uint64_t start_position,
                      float* last_logits_out, uint32_t* argmax_out);

/* Greedy generation entirely on the device: prefill `prompt`, then emit up to
 * max_new_tokens argmax tokens, each fed back without a host round trip.
 * Stops after emitting eos when eos_token_id >= 0.  Replaces generateGreedy /
 * generateGreedyInto / generateGreedyMeasured with --greedy
 * (src/generator.zig:142-175, 221-325).  `out` holds max_new_tokens entries;
 * `out_count` receives the number produced; `stats` (may be NULL) receives
 * the generator.Stats timings measured with the same boundaries. */
int vvli_cuda_generate_greedy(vvli_ctx* ctx, const uint32_t* prompt, uint64_t n_prompt,
                              uint64_t max_new_tokens, int64_t eos_token_id, uint32_t* out,
                              uint64_t* out_count, vvli_generate_stats* stats);

/* Continues greedy decoding on the device from the state the last forward
 * left: runs n_steps forwards, each fed the argmax of the one before (the
 * decode loop of generateGreedyInto, src/generator.zig:311-323, with the
 * argmax taken on the device).  `out_tokens` (n_steps entries, may be NULL)
 * receives the argmax of each forward; `device_ms` (may be NULL) the
 * CUDA-event time of the n_steps forwards.  VVLI_ERR_CONTEXT_FULL when the
 * last forward would pass max_seq. */
int vvli_cuda_decode(vvli_ctx* ctx, uint64_t n_steps, uint32_t* out_tokens, float* device_ms);

/* Sampler.next (src/generator.zig:97-126, 338-463) on the device, over
 * `logits_or_null` (vocab_size host floats, uploaded) or, when it is NULL,
 * the logits of the last forward call (forward_token / forward_embedding /
 * prefill / decode), which stay on the device.  `recent` holds the prompt tokens followed by the
 * generated ones (or at least their last repeat_last_n); repeat penalties
 * apply to the last repeat_last_n of them.  temperature <= 0: penalised
 * argmax.  Otherwise top-k by (adjusted logit desc, id asc), exp((l - max)/T),
 * the top-p cut and the cumulative draw, with the sums in the reference's
 * order.  `rng_state` is the xoshiro256++ state of std.Random.DefaultPrng; it
 * is advanced by random.float(f32) exactly when the reference draws (T > 0
 * and a finite candidate exists).  Invalid options: VVLI_ERR_INVALID_SAMPLING
 * (validateSamplingOptions, :338-342).  Under tensor parallelism every rank
 * makes the call with the same state and gets the same token. */
int vvli_cuda_sample(vvli_ctx* ctx, const vvli_sample_options* options, const float* logits_or_null,
                     const uint32_t* recent, uint64_t n_recent, uint64_t rng_state[4], uint32_t* out_token);

/* Measurement helper with no counterpart in the reference: times one decode
 * kernel alone with CUDA events on the context's stream, cycling over every
 * layer's weights so that no launch finds its weights in L2.  kernel: 0 q|k|v
 * GEMV, 1 o_proj GEMV, 2 gate|up GEMV, 3 down GEMV, 4 LM-head GEMV.
 * `avg_ms` receives the mean launch duration, `bytes` the algorithmic HBM
 * bytes of one launch (weights, norm/bias vectors, input and output). */
int vvli_cuda_time_kernel(vvli_ctx* ctx, int kernel, int reps, float* avg_ms, double* bytes);

/* Copies the residual stream x after layer `layer` of the last forward call
 * (hidden_size floats); after vvli_cuda_prefill, that of the prompt's last
 * token.  Debug entry point for per-layer parity; the reference keeps it in
 * Scratch.x (src/llm.zig:612, 757, 765).  Requires debug capture to be on
 * (vvli_cuda_set_debug) during that call. */
int vvli_cuda_set_debug(vvli_ctx* ctx, int enabled);
int vvli_cuda_debug_hidden(vvli_ctx* ctx, int layer, float* out);

/* Reads a numeric property of the context: "megakernel" (1 when the step
 * runs as one persistent kernel), "sm_count", "graph", "mega_ring_bytes",
 * "mega_phases", "kernels_per_step", "weight_bytes", "tc_prefill" (1 when
 * prefill runs on the tensor cores).  No counterpart in the
 * reference; for benchmarks and tests. */
int vvli_cuda_query(vvli_ctx* ctx, const char* key, double* out);

/* Megakernel timeline of the last step when the context was created with
 * VVLI_TRACE=1 in the environment: %globaltimer ns per [phase][CTA][6] =
 * consumers start, inputs loaded, rows consumed, outputs written, grid
 * barrier passed, producer's first stage of the phase.  `count` receives the
 * number of values (0 without tracing); `out` is filled when cap >= count. */
int vvli_cuda_trace(vvli_ctx* ctx, uint64_t* out, uint64_t cap, uint64_t* count);

/* Self-test of the tensor-core (tcgen05) GEMMs, with no counterpart in the
 * reference: C[M,N] = (A_hi + A_lo)[M,K] . W[N,K]^T on random bf16 data
 * (two_a = 0: A_hi only) against a SIMT fp64-accumulating reference on
 * `device`; `max_rel_err` = max |C - ref| / max |ref|.  kernel 0: the prefill
 * GEMM on single CTAs (128 x 256 tiles); kernel 1: the decode-batch GEMM
 * (M <= 32 rows, weight rows as the MMA's M operand, split-K over a
 * cluster); kernel 2: the prefill GEMM on CTA pairs (256 x 256 tiles,
 * cta_group::2, opt-in with VVLI_GEMM_PAIR=1); kernel 3: the prefill GEMM
 * with the stream-K schedule prefill runs (the last waves' k-blocks shared
 * evenly by all SMs, split tiles summed in k order), run twice to check that
 * the result repeats bit for bit. */
int vvli_cuda_gemm_selftest(int device, int kernel, int M, int N, int K, int two_a, uint64_t seed,
                            float* max_rel_err);

/* Times the isolated linear op y[M,N] = x[M,K] . W[N,K]^T (W bf16, x and y
 * fp32; linearInto, src/llm.zig:1228-1285, over M independent rows) on
 * `device`, through the kernel the decoder uses for M rows: the bulk-copy
 * GEMV (M = 1, kernel_used 0), the decode-batch tensor-core GEMM (M <= 32,
 * 1; M <= 64 as two 32-row launches, 2) or the prefill tensor-core GEMM
 * (M > 64, 3).  Weight copies are rotated so that together they exceed twice
 * the L2 size.  `avg_ms` = mean time per op over `reps` (CUDA events; the
 * fp32 -> bf16 hi/lo split of x is included), `bytes` = 2NK + 4MK + 4MN,
 * `flops` = 2MNK.  Measurement hook (BASELINE op sweep); no counterpart in
 * the reference.  Needs N even and K a multiple of 8. */
int vvli_cuda_op_bench(int device, int M, int N, int K, int reps, float* avg_ms, double* bytes, double* flops,
                       int* kernel_used);

/* Self-test of the tensor-core prompt attention, with no counterpart in the
 * reference: random q, K and V (head_dim d of 64 or 128, `group` q heads per
 * kv head, 2 kv heads, `tokens` query tokens at positions pos0 .., a
 * scrambled page table) through the tcgen05 kernel and the SIMT flash kernel
 * on `device`; `max_rel_err` = max |difference| / max |SIMT output|. */
int vvli_cuda_attention_selftest(int device, int d, int group, int tokens, int pos0, uint64_t seed,
                                 float* max_rel_err);

/* Prompt prefill of B independent sequences, with no counterpart in the
 * reference (which prefills one token at a time, src/generator.zig:243-251):
 * sequence b is tokens[sum(lengths[0..b)), + lengths[b]) at positions
 * 0..lengths[b]-1 of sequence slot b (the KV pages vvli_cuda_forward_batch
 * row b uses), each through the tensor-core prefill.  last_logits (may be
 * NULL) receives B x vocab_size floats, the logits of each sequence's last
 * token; argmax_out (may be NULL) B greedy tokens.  B <= max_batch; every
 * length in 1..max_seq.  Decoding continues with vvli_cuda_forward_batch;
 * slot 0 is also left ready for vvli_cuda_forward_token at position
 * lengths[0].  VVLI_ERR_UNIMPLEMENTED when the context has no tensor-core
 * prefill. */
int vvli_cuda_prefill_batch(vvli_ctx* ctx, const uint32_t* tokens, const uint64_t* lengths, uint64_t B,
                            float* last_logits, uint32_t* argmax_out);

/* One decode step of `batch` independent sequences, with no counterpart in
 * the reference (which decodes one sequence): row b is sequence slot b, with
 * its own KV cache (slot 0 is the cache forward_token uses), and computes what
 * Runner.forwardToken (src/llm.zig:702-709) computes for tokens[b] at
 * positions[b] on that sequence.  The linear layers run as tensor-core GEMMs
 * that read every weight once per 32 rows (bf16 hi + lo activations, fp32
 * accumulation), so rows agree with forward_token to about 1e-3 of the
 * logits' scale.  `logits_out` [batch][vocab_size] and `argmax_out` [batch]
 * may be NULL.  batch <= max_batch of vvli_cuda_create; a token >= vocab_size
 * gives VVLI_ERR_INVALID_TOKEN, a position >= max_seq VVLI_ERR_CONTEXT_FULL.
 * The single-sequence state (next position, logits used by
 * vvli_cuda_sample) is not changed. */
int vvli_cuda_forward_batch(vvli_ctx* ctx, const uint32_t* tokens, const uint64_t* positions, uint64_t batch,
                            float* logits_out, uint32_t* argmax_out);

/* Greedy token choice over `rows` rows of `n` fp32 logits that are already in
 * device memory (row r at logits + r * n), writing the index of each row's
 * maximum to tokens[r] (device memory).  It has no counterpart in the
 * reference; it returns what llm.argmax (src/llm.zig:778-789) returns for each
 * row: the first maximal index, NaNs never chosen except that a NaN in
 * element 0 gives 0.
 *
 * The library allocates nothing for this call and needs no context: it is for
 * callers that own the whole device's memory (a serving engine whose pool has
 * already claimed HBM for its KV cache, where a library cudaMalloc would fail
 * or eat into the pool) or that cannot afford cudaFree's device-wide
 * synchronisation.  Its scratch is one static device array of 33,024 bytes
 * per device, so the limits are rows <= 64 and rows * ceil(n / 4096) <= 4096
 * (n <= 16,777,216 for one row); larger requests, null or misaligned pointers,
 * and ranges whose first or last byte is not device memory of `device` (or
 * managed memory) return VVLI_ERR_INVALID_ARGUMENT with the reason in
 * vvli_cuda_last_error().  Only the two ends are checked, so a buffer that a
 * virtual-memory pool (cuMemCreate + cuMemMap) maps as several chunks is
 * accepted.
 *
 * The work is queued on `stream` (a cudaStream_t; NULL = the legacy default
 * stream) and tokens[] is valid once that stream has been synchronised.  The
 * caller's current device is restored before returning.
 *
 * The first call on each device does one-time setup (the scratch address is
 * looked up, which may load this library's device code); make that first
 * call before any stream capture begins.  The address is kept for the life of
 * the process, so resetting a device (cudaDeviceReset) after its first call
 * is not supported.  The scratch's per-row arrival
 * counters must be zero when a call starts: they are zero when the device
 * code loads and every completed call leaves them zero.  Calls that overlap
 * on one device (two streams, or two host threads, without ordering between
 * them) share the scratch and race: results are then wrong and the counters
 * may stay non-zero for later calls.  Order calls on one device, e.g. issue
 * them all on one stream. */
int vvli_cuda_argmax_rows_static(int device, const float* logits, uint64_t rows, uint64_t n, int32_t* tokens,
                                 void* stream);

/* ---------------------------------------------------------------- mixture of experts
 * The sparse feed-forward block of OLMoE, which the reference detects and
 * rejects (src/llm.zig:45-48, 210-214, 261-264; src/main.zig:590-611):
 *   x[t] += sum over the top_k experts e of softmax(router . xn)[e] *
 *           down_e . (silu(gate_e . xn) * (up_e . xn)),  xn = rmsnorm(x[t]) * norm_w
 * for every token row t, with the experts chosen by router probability
 * (larger first, lower index on ties) and their weights divided by their
 * sum when norm_topk_prob is set (the OLMoE block of transformers 5.5.0).
 * The experts' contributions are added in ascending expert index, so the
 * result does not depend on timing.  Only the routed experts' weights are
 * read.  All pointers are device memory of `device`; weights are bf16.
 * Needs no context; allocates nothing: the caller passes a workspace of
 * vvli_cuda_moe_workspace_bytes(...) bytes.  Limits: tokens <= 4096,
 * hidden and inter multiples of 8 up to 8192, experts <= 1024,
 * top_k <= min(experts, 32); x, router, gate_up and down 16-byte aligned,
 * the workspace 256-byte aligned.  Other sizes or pointers return
 * VVLI_ERR_INVALID_ARGUMENT with the reason in vvli_cuda_last_error().
 * The work is queued on `stream` (a cudaStream_t; NULL = the legacy default
 * stream); the caller's current device is restored before returning. */
typedef struct vvli_moe_args {
  uint64_t tokens;          /* rows of x */
  uint64_t hidden;          /* h */
  uint64_t inter;           /* I, one expert's intermediate size */
  uint64_t experts;         /* E */
  uint64_t top_k;           /* experts per token */
  int32_t norm_topk_prob;   /* 1: the chosen weights are divided by their sum (OLMoE: 0) */
  float rms_eps;
  float* x;                 /* [tokens][h] f32 residual rows, updated in place */
  const uint16_t* norm_w;   /* [h] the post-attention RMSNorm weight */
  const uint16_t* router;   /* [E][h] */
  const uint16_t* gate_up;  /* [E][2 I][h]: the I gate rows, then the I up rows */
  const uint16_t* down;     /* [E][h][I] */
  void* workspace;
  uint64_t workspace_bytes;
  int32_t* topk_index;      /* optional [tokens][top_k] out: chosen experts, larger weight first */
  float* topk_weight;       /* optional [tokens][top_k] out: their weights */
} vvli_moe_args;

/* Workspace bytes vvli_cuda_moe_ffn needs for these sizes; 0 if it does not take them. */
uint64_t vvli_cuda_moe_workspace_bytes(uint64_t tokens, uint64_t hidden, uint64_t inter, uint64_t experts,
                                       uint64_t top_k);
int vvli_cuda_moe_ffn(int device, const vvli_moe_args* args, void* stream);

/* Device-side timing of the last forward in milliseconds (CUDA events). */
int vvli_cuda_last_forward_ms(vvli_ctx* ctx, float* out_ms);

/* Destroys the context and frees all device memory. */
int vvli_cuda_destroy(vvli_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* VVLI_CUDA_H */
