// runtime.cu - the C ABI of include/vvli_cuda.h.
//
// A context owns one GPU's share of the model: its tensor-parallel weight
// shard in one device allocation, a paged fp32 KV cache, the activation
// buffers of one decode step, and a CUDA graph of that step.  The graph
// reads the token and position from device memory (StepState), so one
// capture serves every call; generation and prefill replay it back to back
// without host round trips.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/vvli_cuda.h"
#include "gemm_tc.cuh"
#include "batch.cuh"
#include "kernels.h"
#include "loader.h"
#include "sampler.cuh"

using namespace vvli;

static_assert(sizeof(vvli_model_config) == 136, "vvli_model_config layout is part of the ABI");

namespace {

thread_local std::string g_last_error;

}  // namespace

namespace vvli {
// Lets other translation units of the library report through vvli_cuda_last_error.
void set_last_error(const std::string& what) { g_last_error = what; }
}  // namespace vvli

namespace {

// ---------------------------------------------------------------- NCCL (loaded at run time)
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = "libnccl.so.2 not found";
      return a;
    }
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    a.ok = sym(a.GetUniqueId, "ncclGetUniqueId") && sym(a.CommInitRankConfig, "ncclCommInitRankConfig") &&
           sym(a.CommGetAsyncError, "ncclCommGetAsyncError") && sym(a.AllReduce, "ncclAllReduce") &&
           sym(a.AllGather, "ncclAllGather") && sym(a.CommDestroy, "ncclCommDestroy") &&
           sym(a.CommAbort, "ncclCommAbort") && sym(a.GetErrorString, "ncclGetErrorString");
    if (!a.ok) a.why = "libnccl is missing a required symbol";
    return a;
  }();
  return api;
}

// ---------------------------------------------------------------- reference blob layout
// assignSlices / storageElementCount (src/llm.zig:488-537, 814-837).
struct LayerOff {
  uint64_t in_norm, q, qb, k, kb, v, vb, o, post, gate, up, down;
};
struct BlobLayout {
  uint64_t emb = 0, final_norm = 0, lm_head = UINT64_MAX, total = 0;
  std::vector<LayerOff> layers;
};

BlobLayout blob_layout(const vvli_model_config& c) {
  BlobLayout b;
  uint64_t cur = 0;
  auto take = [&](uint64_t n) {
    cur = (cur + 31) / 32 * 32;
    const uint64_t s = cur;
    cur += n;
    return s;
  };
  const uint64_t h = c.hidden_size, kv = c.num_key_value_heads * (c.hidden_size / c.num_attention_heads),
                 I = c.intermediate_size;
  b.emb = take(c.vocab_size * h);
  b.layers.resize(c.num_hidden_layers);
  for (auto& L : b.layers) {
    L.in_norm = take(h);
    L.q = take(h * h);
    L.qb = c.qkv_bias ? take(h) : UINT64_MAX;
    L.k = take(kv * h);
    L.kb = c.qkv_bias ? take(kv) : UINT64_MAX;
    L.v = take(kv * h);
    L.vb = c.qkv_bias ? take(kv) : UINT64_MAX;
    L.o = take(h * h);
    L.post = take(h);
    L.gate = take(I * h);
    L.up = take(I * h);
    L.down = take(h * I);
  }
  b.final_norm = take(h);
  if (!c.tie_word_embeddings) b.lm_head = take(c.vocab_size * h);
  b.total = cur;
  return b;
}

uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
uint64_t tensor_key(uint64_t seed, uint64_t tid) { return mix64(seed ^ mix64(tid + 0x632BE59BD9B4E019ull)); }

// One rectangular piece of a reference tensor copied into the device layout.
struct Piece {
  uint64_t dst;        // element offset in the device allocation
  uint64_t tensor_id;  // blob order id (synthetic generator key)
  uint64_t src;        // element offset of the tensor in the host blob
  uint64_t rows, cols, src_ld, row0, col0;
  int kind;            // 0 matrix/bias, 1 norm weights
  // The fused matrix this piece belongs to (q|k|v, gate|up, or the matrix
  // itself): its element offset and this piece's first row in it.  A
  // quantised matrix is stored from the group's offset with its own row size.
  uint64_t group_base, group_row;
};

struct DevLayer {
  uint64_t in_norm, w_qkv, b_qkv, w_o, post, w_gu, w_down;
  int f_qkv = kFmtBF16, f_o = kFmtBF16, f_gu = kFmtBF16, f_down = kFmtBF16;  // WeightFormat of each matrix
};

}  // namespace

struct vvli_ctx {
  vvli_model_config cfg{};
  int device = 0, tp_rank = 0, tp_size = 1;
  int sm_count = 148;
  uint64_t max_seq = 0, max_batch = 1;
  // dimensions
  int h = 0, L = 0, nq = 0, nkv = 0, d = 0, group = 0, I = 0, V = 0;
  int nq_l = 0, nkv_l = 0, q_rows = 0, kv_rows = 0, I_l = 0, V_l = 0, V_lr = 0, v0 = 0;
  // weights
  std::vector<Piece> pieces;
  std::vector<DevLayer> lay;
  uint64_t off_emb = 0, off_final = 0, off_lm = 0, weight_elems = 0;
  bool lm_aliases_emb = false;
  uint16_t* w = nullptr;
  bool loaded = false;
  // Matrix formats (WeightFormat): bf16 unless a GGUF file held Q8_0 / Q4_0
  // blocks; `quant` when any matrix is block-quantised.
  int f_emb = kFmtBF16, f_lm = kFmtBF16;
  bool quant = false;
  int smem_optin = 0;
  int plan_sig = 0;              // formats the megakernel plan was made for (0: all bf16)
  bool want_mega = false;        // megakernel wanted (VVLI_MEGAKERNEL not 0)
  bool tc_prefill_planned = false;
  bool rows_paired = false;      // q/k rows already in rotary-pair order (quantised synthetic fill)
  // KV cache and step buffers
  float* kv = nullptr;
  size_t kv_layer_floats = 0;  // K (or V) floats per layer
  int max_pages = 0;
  int* page_table = nullptr;
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *ff = nullptr, *logits = nullptr, *logits_full = nullptr,
        *emb_in = nullptr, *hidden = nullptr, *attn_part = nullptr, *amax_val = nullptr, *best = nullptr,
        *all_best = nullptr;
  int* amax_idx = nullptr;
  unsigned* counters = nullptr;  // [nkv_l] attention + [1] argmax
  int* seq_tokens = nullptr;
  StepState* st = nullptr;
  // launch shapes
  int attn_splits = 1;
  // host staging (pinned)
  StepState* h_st = nullptr;
  int* h_tok = nullptr;
  // execution
  cudaStream_t stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  bool debug = false;
  bool use_pdl = true;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  ncclComm_t comm = nullptr;
  // decode megakernel (one cooperative launch per step)
  bool use_mega = false;
  std::vector<MegaPhase> h_phases;
  MegaPhase* d_phases = nullptr;
  MegaParams mp{};
  size_t mega_smem = 0;
  float* ssq = nullptr;
  unsigned long long* bar = nullptr;  // megakernel barrier arrivals
  unsigned* epoch = nullptr;
  int mega_splits = 1;
  uint64_t* trace = nullptr;  // VVLI_TRACE=1: megakernel timeline
  // tensor-parallel megakernel: this rank's exchange block (receive rows, flags,
  // argmax slots) and every rank's block mapped into this process (CUDA IPC)
  uint8_t* peer_block = nullptr;
  TpExchange xch{};  // decode batches' all-reduces and logits gathers over the peer blocks (when mapped)
  void* peer_base[kMaxTp] = {};
  uint16_t* w_downT = nullptr;  // fused down_proj: W_down^T per layer [I_l][h]
  long long* acc = nullptr;     // fused down_proj: fixed-point accumulators [2][h]
  // tensor-core prefill
  bool tc_prefill = false;
  int pf_cap = 0;
  float *pf_x = nullptr, *pf_q = nullptr;
  uint16_t *pf_ahi = nullptr, *pf_alo = nullptr, *pf_fhi = nullptr, *pf_flo = nullptr;
  int* pf_tokens = nullptr;
  uint8_t* pf_kvt = nullptr;  // tensor-core attention: hi / lo images of the layer's K / V tiles
  float* pf_skws = nullptr;     // stream-K parts of the GEMMs, one slot per SM
  unsigned* pf_skflags = nullptr;
  unsigned pf_sk_epoch = 0;     // a new value per GEMM launch
  CUtensorMap tm_ah_hi{}, tm_ah_lo{}, tm_aq_hi{}, tm_aq_lo{}, tm_f_hi{}, tm_f_lo{};
  std::vector<CUtensorMap> tm_w;  // per layer: q|k|v, o, gate|up, down
  // decode batches (allocated on first use): chunks of up to kSkinnyMaxRows rows
  bool bt_ready = false;
  int bt_splits_max = 0;
  int bt_attn_per_sm = 0;  // resident attention CTAs per SM
  float *bt_x = nullptr, *bt_q = nullptr, *bt_logits = nullptr, *bt_best = nullptr, *bt_all_best = nullptr,
        *bt_part = nullptr, *bt_logits_all = nullptr;
  uint16_t *bt_ahi = nullptr, *bt_alo = nullptr, *bt_fhi = nullptr, *bt_flo = nullptr;
  int *bt_tokens = nullptr, *bt_pos = nullptr, *bt_idx = nullptr;
  unsigned* bt_counters = nullptr;
  CUtensorMap tmb_h[2][2]{}, tmb_q[2][2]{}, tmb_f[2][2]{};  // [nb 16 / 32][hi / lo]
  CUtensorMap tm_lm{};
  // device sampler (allocated on first use)
  unsigned* smp_stamp = nullptr;
  unsigned* smp_key32 = nullptr;
  unsigned long long *smp_key64 = nullptr, *smp_key64_sorted = nullptr;
  float* smp_probs = nullptr;
  float* smp_logits = nullptr;
  uint32_t* smp_recent = nullptr;
  SampleState* smp_state = nullptr;
  SampleState* h_smp_state = nullptr;
  uint32_t* h_smp_recent = nullptr;  // page-locked staging of the recent tokens
  SampleState* h_smp_out = nullptr;  // fused top-k step's result: page-locked host memory the kernel writes
  SampleState* d_smp_out = nullptr;  // its device address
  unsigned* smp_done = nullptr;      // fused top-k step's CTA counter
  unsigned smp_call = 0;
};

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) return VVLI_ERR_OOM;
  return VVLI_ERR_CUDA;
}

#define CK(call)                                                    \
  do {                                                              \
    cudaError_t e_ = (call);                                        \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);             \
  } while (0)

int nccl_wait(vvli_ctx* c, ncclResult_t r, const char* what) {
  auto& n = nccl();
  const double limit_s = getenv("VVLI_NCCL_TIMEOUT_S") ? atof(getenv("VVLI_NCCL_TIMEOUT_S")) : 120.0;
  const auto t0 = std::chrono::steady_clock::now();
  // A non-blocking communicator finishes enqueueing within microseconds:
  // poll without sleeping at first (a 50 us sleep per collective made a
  // decode batch, two all-reduces per layer, host-bound), then back off.
  for (uint32_t it = 0; r == ncclInProgress; ++it) {
    if (it < 256)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(it < 4096 ? 2 : 50));
    if (n.CommGetAsyncError(c->comm, &r) != ncclSuccess) break;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit_s) {
      g_last_error = std::string(what) + ": timed out";
      n.CommAbort(c->comm);
      c->comm = nullptr;
      return VVLI_ERR_TIMEOUT;
    }
  }
  if (r != ncclSuccess) {
    g_last_error = std::string(what) + ": " + n.GetErrorString(r);
    return VVLI_ERR_NCCL;
  }
  return VVLI_OK;
}

int tp_collective(vvli_ctx* c, const float* src, float* dst, size_t n, bool gather, cudaStream_t s, const char* what);

int validate_config(const vvli_model_config& c) {  // Config.validate (src/llm.zig:195-216)
  if (c.vocab_size == 0 || c.hidden_size == 0 || c.intermediate_size == 0 || c.num_hidden_layers == 0 ||
      c.num_attention_heads == 0 || c.num_key_value_heads == 0 || c.max_position_embeddings == 0)
    return VVLI_ERR_INVALID_CONFIG;
  if (c.hidden_size % c.num_attention_heads) return VVLI_ERR_INVALID_CONFIG;
  if (c.num_attention_heads % c.num_key_value_heads) return VVLI_ERR_INVALID_CONFIG;
  if ((c.hidden_size / c.num_attention_heads) % 2) return VVLI_ERR_INVALID_CONFIG;
  if (c.num_experts != 0) {
    if (c.num_experts_per_token == 0 || c.num_experts_per_token > c.num_experts) return VVLI_ERR_INVALID_CONFIG;
    return VVLI_ERR_UNSUPPORTED_ARCH;
  }
  if (c.num_experts_per_token != 0) return VVLI_ERR_INVALID_CONFIG;
  if (c.architecture == VVLI_ARCH_OLMOE || c.architecture > VVLI_ARCH_QWEN2) return VVLI_ERR_UNSUPPORTED_ARCH;
  return VVLI_OK;
}

uint64_t align128(uint64_t v) { return (v + 127) / 128 * 128; }

// Device layout of this rank's shard and the pieces that fill it.
void plan_weights(vvli_ctx* c) {
  const auto& cfg = c->cfg;
  const BlobLayout b = blob_layout(cfg);
  const uint64_t h = c->h, r = c->tp_rank;
  uint64_t cur = 0;
  auto alloc = [&](uint64_t n) {
    const uint64_t s = cur;
    cur = align128(cur + n);
    return s;
  };
  auto mat = [&](uint64_t dst, uint64_t tid, uint64_t src, uint64_t rows, uint64_t cols, uint64_t ld, uint64_t row0,
                 uint64_t col0, int kind, uint64_t group_base = UINT64_MAX, uint64_t group_row = 0) {
    c->pieces.push_back({dst, tid, src, rows, cols, ld, row0, col0, kind, group_base == UINT64_MAX ? dst : group_base,
                         group_row});
  };
  c->off_emb = alloc(static_cast<uint64_t>(c->V) * h);
  mat(c->off_emb, 0, b.emb, c->V, h, h, 0, 0, 0);
  c->lay.resize(c->L);
  const uint64_t qr = c->q_rows, kr = c->kv_rows, Il = c->I_l;
  for (int l = 0; l < c->L; ++l) {
    const auto& B = b.layers[l];
    auto& D = c->lay[l];
    const uint64_t base = 1 + 12ull * l;
    D.in_norm = alloc(h);
    mat(D.in_norm, base + 0, B.in_norm, 1, h, h, 0, 0, 1);
    D.w_qkv = alloc((qr + 2 * kr) * h);
    mat(D.w_qkv, base + 1, B.q, qr, h, h, r * qr, 0, 0, D.w_qkv, 0);
    mat(D.w_qkv + qr * h, base + 3, B.k, kr, h, h, r * kr, 0, 0, D.w_qkv, qr);
    mat(D.w_qkv + (qr + kr) * h, base + 5, B.v, kr, h, h, r * kr, 0, 0, D.w_qkv, qr + kr);
    D.b_qkv = UINT64_MAX;
    if (cfg.qkv_bias) {
      D.b_qkv = alloc(qr + 2 * kr);
      mat(D.b_qkv, base + 2, B.qb, 1, qr, h, 0, r * qr, 0);
      mat(D.b_qkv + qr, base + 4, B.kb, 1, kr, c->nkv * c->d, 0, r * kr, 0);
      mat(D.b_qkv + qr + kr, base + 6, B.vb, 1, kr, c->nkv * c->d, 0, r * kr, 0);
    }
    D.w_o = alloc(h * qr);
    mat(D.w_o, base + 7, B.o, h, qr, h, 0, r * qr, 0);
    D.post = alloc(h);
    mat(D.post, base + 8, B.post, 1, h, h, 0, 0, 1);
    D.w_gu = alloc(2 * Il * h);
    mat(D.w_gu, base + 9, B.gate, Il, h, h, r * Il, 0, 0, D.w_gu, 0);
    mat(D.w_gu + Il * h, base + 10, B.up, Il, h, h, r * Il, 0, 0, D.w_gu, Il);
    D.w_down = alloc(h * Il);
    mat(D.w_down, base + 11, B.down, h, Il, c->I, 0, r * Il, 0);
  }
  c->off_final = alloc(h);
  mat(c->off_final, 1 + 12ull * c->L, b.final_norm, 1, h, h, 0, 0, 1);
  if (cfg.tie_word_embeddings && c->tp_size == 1) {
    c->lm_aliases_emb = true;
    c->off_lm = c->off_emb;
  } else {
    c->off_lm = alloc(static_cast<uint64_t>(c->V_lr) * h);
    if (cfg.tie_word_embeddings)
      mat(c->off_lm, 0, b.emb, c->V_lr, h, h, c->v0, 0, 0);
    else
      mat(c->off_lm, 2 + 12ull * c->L, b.lm_head, c->V_lr, h, h, c->v0, 0, 0);
  }
  c->weight_elems = cur;
}

// Model and shard dimensions of rank `tp_rank` of `tp_size` (no CUDA calls).
int fill_dims(vvli_ctx* c, const vvli_model_config& cfg, int tp_rank, int tp_size) {
  const uint64_t d = cfg.hidden_size / cfg.num_attention_heads;
  c->cfg = cfg;
  c->tp_rank = tp_rank;
  c->tp_size = tp_size;
  c->h = static_cast<int>(cfg.hidden_size);
  c->L = static_cast<int>(cfg.num_hidden_layers);
  c->nq = static_cast<int>(cfg.num_attention_heads);
  c->nkv = static_cast<int>(cfg.num_key_value_heads);
  c->d = static_cast<int>(d);
  c->group = c->nq / c->nkv;
  c->I = static_cast<int>(cfg.intermediate_size);
  c->V = static_cast<int>(cfg.vocab_size);
  c->nq_l = c->nq / tp_size;
  c->nkv_l = c->nkv / tp_size;
  c->q_rows = c->nq_l * c->d;
  c->kv_rows = c->nkv_l * c->d;
  c->I_l = c->I / tp_size;
  c->V_l = (c->V + tp_size - 1) / tp_size;
  c->v0 = tp_rank * c->V_l;
  c->V_lr = std::max(0, std::min(c->V, c->v0 + c->V_l) - c->v0);
  return c->V_lr > 0 ? VVLI_OK : VVLI_ERR_INVALID_CONFIG;
}

// Phase table and launch parameters of the decode megakernel.  Returns
// false when a shape is outside what the megakernel takes (the per-kernel
// path then runs the step).
template <typename T>
int dalloc(T** p, size_t count);

bool plan_megakernel(vvli_ctx* c, int smem_optin) {
  const uint16_t* W = c->w;
  // Ring shape: two 64 KB stages.  Shared memory taken from the L1 carve-out
  // slows the latency-bound phase changes more than a deeper ring speeds the
  // weight stream (measured on Llama-3-8B).
  const int stage_cap = getenv("VVLI_MEGA_STAGE_CAP") ? std::max(4096, atoi(getenv("VVLI_MEGA_STAGE_CAP"))) : 65536;
  std::vector<MegaPhase> ph;
  bool plan_ok = true;
  auto gemv = [&](int epi, int layer, const uint16_t* w, int N, int K, int nphys, const uint16_t* norm,
                  const float* x, float* y, const uint16_t* bias, int ar_index, int fmt = kFmtBF16) {
    MegaPhase m{};
    m.kind = MK_GEMV, m.epi = epi, m.layer = layer, m.nphys = nphys, m.W = w, m.N = N, m.K = K;
    m.fmt = fmt, m.row_bytes = row_bytes_of(fmt, K);
    m.pair_offset = nphys == 2 ? N : 0;
    m.norm_w = norm, m.x = x, m.y = y, m.bias = bias, m.ar_index = ar_index, m.row_align = 1;
    plan_ok = plan_mega_gemv(m, stage_cap) && plan_ok;
    ph.push_back(m);
  };
  MegaPhase e{};
  e.kind = MK_EMBED;
  ph.push_back(e);
  // down_proj fused into gate|up (see MegaPhase::acc_out), opt-in with
  // VVLI_MEGA_FUSED_DOWN=1: it removes a grid barrier per layer, but the 64-bit
  // integer atomics of the fixed-point reduction (h per CTA) and the wider
  // accumulator reads cost more than the barrier saves (Llama-3-8B: 4.09 vs
  // 3.74 ms per token).  Each CTA's gate|up rows must fit the shared-memory ff
  // buffer and a thread owns at most 16 outputs.
  const char* fd = getenv("VVLI_MEGA_FUSED_DOWN");
  const bool fused = fd && fd[0] == '1' && c->tp_size == 1 && !c->quant && c->h % 8 == 0 &&
                     c->h <= 2 * 8 * kMegaConsumerWarps * 32 &&
                     (c->I_l + c->sm_count - 1) / c->sm_count + 1 <= kMaxFfRows;
  long long* acc[2] = {nullptr, nullptr};
  if (fused && !c->w_downT) {
    if (dalloc(&c->w_downT, static_cast<size_t>(c->L) * c->I_l * c->h) || dalloc(&c->acc, 2 * static_cast<size_t>(c->h)))
      return false;
  }
  if (fused) {
    acc[0] = c->acc;
    acc[1] = c->acc + c->h;
  }
  for (int l = 0; l < c->L; ++l) {
    const DevLayer& D = c->lay[l];
    gemv(ME_QKV, l, W + D.w_qkv, c->q_rows + 2 * c->kv_rows, c->h, 1, W + D.in_norm, c->x, c->qkv,
         D.b_qkv == UINT64_MAX ? nullptr : W + D.b_qkv, 0, D.f_qkv);
    ph.back().k_cache = c->kv + static_cast<size_t>(2 * l) * c->kv_layer_floats;
    ph.back().v_cache = ph.back().k_cache + c->kv_layer_floats;
    ph.back().row_align = 2;
    if (fused && l > 0) ph.back().acc_in = acc[(l - 1) & 1], ph.back().hidden_layer = l - 1;
    MegaPhase a{};
    a.kind = MK_ATTN, a.layer = l;
    a.k_cache = c->kv + static_cast<size_t>(2 * l) * c->kv_layer_floats;
    a.v_cache = a.k_cache + c->kv_layer_floats;
    ph.push_back(a);
    gemv(ME_RESIDUAL, l, W + D.w_o, c->h, c->q_rows, 1, nullptr, c->attn, c->x, nullptr, 2 * l, D.f_o);
    if (fused && l > 0) ph.back().acc_fold = acc[(l - 1) & 1];
    if (fused) {
      gemv(ME_SILU, l, W + D.w_gu, c->I_l, c->h, 2, W + D.post, c->x, nullptr, nullptr, 0);
      ph.back().ff_smem = 1;
      MegaPhase dn{};
      dn.kind = MK_GEMV, dn.epi = ME_AXPY, dn.layer = l, dn.nphys = 1, dn.no_barrier = 1, dn.row_align = 1;
      dn.W = c->w_downT + static_cast<size_t>(l) * c->I_l * c->h, dn.N = c->I_l, dn.K = c->h;
      dn.S = 1, dn.SZ = 0, dn.cpl = 0, dn.fmt = kFmtBF16, dn.row_bytes = 2 * c->h;
      dn.R = std::max(1, 65536 / (2 * c->h));
      dn.stage_bytes = dn.R * 2 * c->h;
      dn.acc_out = acc[l & 1];
      ph.push_back(dn);
    } else {
      gemv(ME_SILU, l, W + D.w_gu, c->I_l, c->h, 2, W + D.post, c->x, c->ff, nullptr, 0, D.f_gu);
      gemv(ME_RESIDUAL, l, W + D.w_down, c->h, c->I_l, 1, nullptr, c->ff, c->x, nullptr, 2 * l + 1, D.f_down);
    }
  }
  gemv(ME_ARGMAX, -1, W + c->off_lm, c->V_lr, c->h, 1, W + c->off_final, c->x, c->logits, nullptr, 0, c->f_lm);
  if (!plan_ok) return false;
  if (fused) ph.back().acc_in = acc[(c->L - 1) & 1], ph.back().hidden_layer = c->L - 1;
  for (MegaPhase& m : ph)
    if (!m.acc_in) m.hidden_layer = -1;

  const int grid = c->sm_count;
  int slot = 0;
  size_t part = mega_attention_floats(c->group, c->d, c->mega_splits, c->max_pages);
  for (const MegaPhase& m : ph) {
    if (m.kind != MK_GEMV) continue;
    if (c->group > 8 || (kMegaThreads - 32) % c->d || (kMegaThreads - 32) / c->d * 16 < kPage) return false;
    slot = std::max(slot, m.stage_bytes);
    part = std::max(part, static_cast<size_t>((m.N + grid - 1) / grid + 2) * m.nphys * m.S);
  }
  const size_t fixed = ((part + 1) & ~size_t(1)) * 4 + 2 * 8 * sizeof(uint64_t) + 1024;
  int nst = static_cast<int>(std::min<size_t>(8, (static_cast<size_t>(smem_optin) - fixed) / slot));
  // Two stages measured best: a deeper ring keeps more weight copies in
  // flight, which lengthens every latency-bound access of the phase changes.
  nst = std::min(nst, getenv("VVLI_MEGA_STAGES") ? std::max(2, atoi(getenv("VVLI_MEGA_STAGES"))) : 2);
  if (nst < 2) return false;
  // GEMV inputs that eight or more warps share (S <= 2), and those of
  // block-quantised phases, are staged in shared memory.
  int xstage = 0;
  for (const MegaPhase& m : ph)
    if (m.kind == MK_GEMV && (m.S <= 2 || m.fmt != kFmtBF16) && !m.acc_in && m.epi != ME_AXPY &&
        m.K <= kMegaXStageMax)
      xstage = std::max(xstage, m.K);
  c->mega_smem = static_cast<size_t>(nst) * slot + ((part + 1) & ~size_t(1)) * 4 + 2 * nst * sizeof(uint64_t) +
                 (xstage ? 16 + static_cast<size_t>(xstage) * 4 : 0);
  if (c->d_phases) cudaFree(c->d_phases);  // a re-plan after a load that changed the weight formats
  c->d_phases = nullptr;
  if (cudaMalloc(&c->d_phases, ph.size() * sizeof(MegaPhase)) != cudaSuccess) return false;
  if (cudaMemcpy(c->d_phases, ph.data(), ph.size() * sizeof(MegaPhase), cudaMemcpyHostToDevice) != cudaSuccess)
    return false;
  c->h_phases = ph;
  MegaParams& P = c->mp;
  P = MegaParams{};
  P.phases = c->d_phases;
  P.nphases = static_cast<int>(ph.size());
  P.nst = nst;
  P.slot_bytes = slot;
  P.part_floats = static_cast<int>(part);
  P.xstage_floats = xstage;
  P.st = c->st;
  P.seq_tokens = c->seq_tokens;
  P.emb = W + c->off_emb;
  P.emb_fmt = c->f_emb;
  P.emb_row_bytes = row_bytes_of(c->f_emb, c->h);
  P.emb_in = c->emb_in;
  P.h = c->h;
  P.vocab = c->V;
  P.x = c->x;
  P.ssq = c->ssq;
  P.eps = c->cfg.rms_norm_eps;
  P.bar = c->bar;
  P.epoch = c->epoch;
  P.n_ar = 2 * c->L;
  // Each CTA owns the same rows of x in the embed, o_proj and down_proj
  // phases, so it can keep them in shared memory instead of reading them back.
  P.xres = (c->tp_size == 1 && !fused && (c->h + grid - 1) / grid <= kMaxResRows) ? 1 : 0;
  P.bars_per_step = static_cast<int>(ph.size()) - 1;
  for (const MegaPhase& m : ph) P.bars_per_step -= m.no_barrier ? 1 : 0;
  P.acc_zero = fused ? acc[(c->L - 1) & 1] : nullptr;
  P.qkv = c->qkv;
  P.attn = c->attn;
  P.attn_part = c->attn_part;
  P.attn_counters = c->counters;
  P.page_table = c->page_table;
  P.nq = c->nq_l;
  P.nkv = c->nkv_l;
  P.d = c->d;
  P.group = c->group;
  P.splits = c->mega_splits;
  P.inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(c->d));
  P.rope = RopeParams{c->cfg.rope_theta, VVLI_ROPE_INTERLEAVED, static_cast<int>(c->cfg.rope_scaling_type),
                      c->cfg.rope_scaling_factor, c->cfg.rope_low_freq_factor, c->cfg.rope_high_freq_factor,
                      static_cast<float>(c->cfg.rope_original_max_position)};
  P.amax_val = c->amax_val;
  P.amax_idx = c->amax_idx;
  P.amax_counter = c->counters + c->nkv_l;
  P.row_base = c->v0;
  P.tp = c->tp_size;
  P.rank = c->tp_rank;
  const char* tr = getenv("VVLI_TRACE");
  if (c->trace) cudaFree(c->trace);
  c->trace = nullptr;
  if (tr && tr[0] == '1' &&
      cudaMalloc(&c->trace, ph.size() * grid * 6 * sizeof(uint64_t)) == cudaSuccess) {
    cudaMemset(c->trace, 0, ph.size() * grid * 6 * sizeof(uint64_t));
    P.trace = c->trace;
  }
  return true;
}

int enqueue_mega(vvli_ctx* c, cudaStream_t s, bool debug) {
  MegaParams P = c->mp;
  P.hidden = debug ? c->hidden : nullptr;
  CK(launch_megakernel(P, c->sm_count, c->mega_smem, s));
  return VVLI_OK;
}

// Final RMSNorm + LM head + argmax of c->x (src/llm.zig:727-728, 778-789);
// under tensor parallelism the vocab shards' winners are gathered.
int enqueue_lm_head(vvli_ctx* c, cudaStream_t s, bool pdl) {
  const bool tp = c->tp_size > 1;
  const uint16_t* W = c->w;
  GemvParams lm{};
  lm.W = W + c->off_lm;
  lm.N = c->V_lr;
  lm.K = c->h;
  lm.x = c->x;
  lm.norm_w = W + c->off_final;
  lm.eps = c->cfg.rms_norm_eps;
  lm.y = c->logits;
  lm.part_val = c->amax_val;
  lm.part_idx = c->amax_idx;
  lm.counter = c->counters + c->nkv_l;
  lm.row_base = c->v0;
  lm.finalize = tp ? 0 : 1;
  lm.local_best = c->best;
  lm.st = c->st;
  lm.seq_tokens = c->seq_tokens;
  CK(launch_gemv(EPI_ARGMAX, lm, c->sm_count, s, pdl && !tp));
  if (tp) {
    int st = nccl_wait(c, nccl().AllGather(c->best, c->all_best, 2, ncclFloat32, c->comm, s), "allgather");
    if (st) return st;
    CK(launch_tp_argmax_finalize(c->all_best, c->tp_size, c->st, c->seq_tokens, s));
  }
  return VVLI_OK;
}

int enqueue_step(vvli_ctx* c, cudaStream_t s, bool debug) {
  if (c->use_mega) return enqueue_mega(c, s, debug);
  const bool pdl = c->use_pdl && !debug;
  const bool tp = c->tp_size > 1;
  const uint16_t* W = c->w;
  EmbedParams ep{W + c->off_emb, c->emb_in, c->seq_tokens, c->st, c->x, c->h, c->V};
  CK(launch_embed(ep, s, false));
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(c->d));
  // q and k rows are stored in rotary-pair order (see after_load): the device
  // applies the interleaved rule for both layouts.
  RopeParams rope{c->cfg.rope_theta, VVLI_ROPE_INTERLEAVED, static_cast<int>(c->cfg.rope_scaling_type),
                  c->cfg.rope_scaling_factor, c->cfg.rope_low_freq_factor, c->cfg.rope_high_freq_factor,
                  static_cast<float>(c->cfg.rope_original_max_position)};
  auto next_qkv = [&](GemvParams& g, int l) {  // l = next layer, or L for the LM head
    if (l < c->L) {
      g.next_W = W + c->lay[l].w_qkv, g.next_N = c->q_rows + 2 * c->kv_rows, g.next_K = c->h;
    } else {
      g.next_W = W + c->off_lm, g.next_N = c->V_lr, g.next_K = c->h;
    }
  };
  for (int l = 0; l < c->L; ++l) {
    const DevLayer& D = c->lay[l];
    GemvParams q{};
    q.next_W = W + D.w_o, q.next_N = c->h, q.next_K = c->q_rows;
    q.W = W + D.w_qkv;
    q.N = c->q_rows + 2 * c->kv_rows;
    q.K = c->h;
    q.x = c->x;
    q.norm_w = W + D.in_norm;
    q.eps = c->cfg.rms_norm_eps;
    q.bias = D.b_qkv == UINT64_MAX ? nullptr : W + D.b_qkv;
    q.st = c->st;
    q.y = c->qkv;
    CK(launch_gemv(EPI_PLAIN, q, c->sm_count, s, pdl && !(tp && l > 0)));  // no PDL edge after a collective

    AttnParams a{};
    a.qkv = c->qkv;
    a.k_cache = c->kv + static_cast<size_t>(2 * l) * c->kv_layer_floats;
    a.v_cache = a.k_cache + c->kv_layer_floats;
    a.page_table = c->page_table;
    a.out = c->attn;
    a.part = c->attn_part;
    a.counters = c->counters;
    a.st = c->st;
    a.nq = c->nq_l;
    a.nkv = c->nkv_l;
    a.d = c->d;
    a.group = c->group;
    a.splits = c->attn_splits;
    a.inv_sqrt_d = inv_sqrt_d;
    a.rope = rope;
    CK(launch_attention(a, s, pdl));

    GemvParams o{};
    o.next_W = W + D.w_gu, o.next_N = c->I_l, o.next_K = c->h, o.next_pair_offset = c->I_l;
    o.W = W + D.w_o;
    o.N = c->h;
    o.K = c->q_rows;
    o.x = c->attn;
    o.residual = c->tp_rank == 0 ? c->x : nullptr;
    o.st = c->st;
    o.y = c->x;
    CK(launch_gemv(EPI_PLAIN, o, c->sm_count, s, pdl));
    if (tp) {
      int st = nccl_wait(c, nccl().AllReduce(c->x, c->x, c->h, ncclFloat32, ncclSum, c->comm, s), "allreduce");
      if (st) return st;
    }

    GemvParams gu{};
    gu.next_W = W + D.w_down, gu.next_N = c->h, gu.next_K = c->I_l;
    gu.W = W + D.w_gu;
    gu.N = c->I_l;
    gu.K = c->h;
    gu.pair_offset = c->I_l;
    gu.x = c->x;
    gu.norm_w = W + D.post;
    gu.eps = c->cfg.rms_norm_eps;
    gu.st = c->st;
    gu.y = c->ff;
    CK(launch_gemv(EPI_SILU_MUL, gu, c->sm_count, s, pdl && !tp));

    GemvParams dn{};
    next_qkv(dn, l + 1);
    dn.W = W + D.w_down;
    dn.N = c->h;
    dn.K = c->I_l;
    dn.x = c->ff;
    dn.residual = c->tp_rank == 0 ? c->x : nullptr;
    dn.st = c->st;
    dn.y = c->x;
    CK(launch_gemv(EPI_PLAIN, dn, c->sm_count, s, pdl));
    if (tp) {
      int st = nccl_wait(c, nccl().AllReduce(c->x, c->x, c->h, ncclFloat32, ncclSum, c->comm, s), "allreduce");
      if (st) return st;
    }
    if (debug) CK(cudaMemcpyAsync(c->hidden + static_cast<size_t>(l) * c->h, c->x, c->h * 4, cudaMemcpyDeviceToDevice, s));
  }
  return enqueue_lm_head(c, s, pdl);
}

template <typename T>
int dalloc(T** p, size_t count) {
  CK(cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T)));
  CK(cudaMemset(*p, 0, std::max<size_t>(count, 1) * sizeof(T)));
  return VVLI_OK;
}

// ---------------------------------------------------------------- tensor-core prefill
// Tensor maps of every weight matrix for the tcgen05 GEMM (K-major rows,
// 64 x 128 boxes, 128-byte swizzle).
int plan_tc_prefill(vvli_ctx* c) {
  c->tm_w.resize(4 * c->L);
  for (int l = 0; l < c->L; ++l) {
    const DevLayer& D = c->lay[l];
    cudaError_t e;
    if ((e = make_tmap_bf16(&c->tm_w[4 * l + 0], c->w + D.w_qkv, c->q_rows + 2 * c->kv_rows, c->h, 128)) ||
        (e = make_tmap_bf16(&c->tm_w[4 * l + 1], c->w + D.w_o, c->h, c->q_rows, 128)) ||
        (e = make_tmap_bf16(&c->tm_w[4 * l + 2], c->w + D.w_gu, 2 * c->I_l, c->h, 128)) ||
        (e = make_tmap_bf16(&c->tm_w[4 * l + 3], c->w + D.w_down, c->h, c->I_l, 128)))
      return cuda_fail(e, "make_tmap_bf16 (weights)");
  }
  return VVLI_OK;
}

// Activation buffers of a prompt chunk of up to pf_cap tokens (allocated on
// the first tensor-core prefill).
int ensure_prefill_buffers(vvli_ctx* c) {
  if (c->pf_cap) return VVLI_OK;
  const int cap = static_cast<int>(std::min<uint64_t>(c->max_seq, 2048));
  const size_t ka = std::max(c->h, c->q_rows);
  int st;
  if ((st = dalloc(&c->pf_x, static_cast<size_t>(cap) * c->h)) || (st = dalloc(&c->pf_q, static_cast<size_t>(cap) * c->q_rows)) ||
      (st = dalloc(&c->pf_ahi, cap * ka)) || (st = dalloc(&c->pf_alo, cap * ka)) ||
      (st = dalloc(&c->pf_fhi, static_cast<size_t>(cap) * c->I_l)) ||
      (st = dalloc(&c->pf_flo, static_cast<size_t>(cap) * c->I_l)) || (st = dalloc(&c->pf_tokens, cap)) ||
      (st = dalloc(&c->pf_skws, gemm_tc_streamk_ws_floats(c->sm_count))) ||
      (st = dalloc(&c->pf_skflags, static_cast<size_t>(c->sm_count))) ||
      (prefill_attention_tc_supported(c->d, c->group) &&
       (st = dalloc(&c->pf_kvt, prefill_attention_tc_workspace(c->d, c->nkv_l, static_cast<int>(c->max_seq))))))
    return st;
  cudaError_t e;
  if ((e = make_tmap_bf16(&c->tm_ah_hi, c->pf_ahi, cap, c->h, 128)) ||
      (e = make_tmap_bf16(&c->tm_ah_lo, c->pf_alo, cap, c->h, 128)) ||
      (e = make_tmap_bf16(&c->tm_aq_hi, c->pf_ahi, cap, c->q_rows, 128)) ||
      (e = make_tmap_bf16(&c->tm_aq_lo, c->pf_alo, cap, c->q_rows, 128)) ||
      (e = make_tmap_bf16(&c->tm_f_hi, c->pf_fhi, cap, c->I_l, 128)) ||
      (e = make_tmap_bf16(&c->tm_f_lo, c->pf_flo, cap, c->I_l, 128)))
    return cuda_fail(e, "make_tmap_bf16 (activations)");
  c->pf_cap = cap;
  return VVLI_OK;
}

// Runs tokens[0, n) at positions start.. with one tensor-core GEMM per linear
// layer and chunk (prefill of the reference's per-token loop,
// src/generator.zig:243-251), then the LM head of the last token.
int prefill_tc(vvli_ctx* c, const uint32_t* tokens, uint64_t n, uint64_t start, int slot = 0) {
  int st;
  if ((st = ensure_prefill_buffers(c))) return st;
  cudaStream_t s = c->stream;
  // Sequence slot `slot` owns pages [slot * pps, (slot + 1) * pps) of the page table.
  const int* page_table = c->page_table + static_cast<size_t>(slot) * ((c->max_seq + kPage - 1) / kPage);
  const uint16_t* W = c->w;
  const bool tp = c->tp_size > 1;
  RopeParams rope{c->cfg.rope_theta, VVLI_ROPE_INTERLEAVED, static_cast<int>(c->cfg.rope_scaling_type),
                  c->cfg.rope_scaling_factor, c->cfg.rope_low_freq_factor, c->cfg.rope_high_freq_factor,
                  static_cast<float>(c->cfg.rope_original_max_position)};
  int* err = &c->st->err;
  // Every GEMM balances its last waves' k-blocks over the SMs (stream-K).
  auto streamk = [&](GemmParams& g) {
    g.sk_ws = c->pf_skws, g.sk_flags = c->pf_skflags;
    if (++c->pf_sk_epoch == 0) ++c->pf_sk_epoch;
    g.sk_epoch = c->pf_sk_epoch;
  };
  int M = 0;
  for (uint64_t c0 = 0; c0 < n; c0 += c->pf_cap) {
    M = static_cast<int>(std::min<uint64_t>(c->pf_cap, n - c0));
    const int pos0 = static_cast<int>(start + c0);
    CK(cudaMemcpyAsync(c->pf_tokens, tokens + c0, M * sizeof(int), cudaMemcpyHostToDevice, s));
    CK(launch_prefill_embed(W + c->off_emb, c->pf_tokens, M, c->h, c->pf_x, s));
    for (int l = 0; l < c->L; ++l) {
      const DevLayer& D = c->lay[l];
      float* kc = c->kv + static_cast<size_t>(2 * l) * c->kv_layer_floats;
      float* vc = kc + c->kv_layer_floats;
      CK(launch_norm_split(c->pf_x, W + D.in_norm, c->cfg.rms_norm_eps, M, c->h, c->pf_ahi, c->pf_alo, s));
      GemmParams g{};
      g.M = M, g.two_a = 1, g.err = err;
      g.N = c->q_rows + 2 * c->kv_rows, g.K = c->h, g.epi = GE_QKV, g.y = c->pf_q, g.ldy = c->q_rows;
      g.bias = D.b_qkv == UINT64_MAX ? nullptr : W + D.b_qkv;
      g.q_rows = c->q_rows, g.kv_rows = c->kv_rows, g.d = c->d, g.nkv = c->nkv_l, g.pos0 = pos0, g.rope = rope;
      g.k_cache = kc, g.v_cache = vc, g.page_table = page_table;
      g.nk = (g.K + kGemmBK - 1) / kGemmBK;
      streamk(g);
      CK(launch_gemm_tc(c->tm_ah_hi, c->tm_ah_lo, c->tm_w[4 * l + 0], g, s));
      PrefillAttnParams a{c->pf_q, kc, vc, page_table, c->pf_ahi, c->pf_alo, M, c->nq_l, c->nkv_l, c->d,
                          c->group, pos0, 1.0f / sqrtf(static_cast<float>(c->d)), err, c->pf_kvt};
      CK(launch_prefill_attention(a, s));
      GemmParams o{};
      o.M = M, o.two_a = 1, o.err = err, o.N = c->h, o.K = c->q_rows, o.epi = GE_RESID, o.y = c->pf_x, o.ldy = c->h;
      o.add_residual = c->tp_rank == 0 ? 1 : 0, o.nk = (o.K + kGemmBK - 1) / kGemmBK;
      streamk(o);
      CK(launch_gemm_tc(c->tm_aq_hi, c->tm_aq_lo, c->tm_w[4 * l + 1], o, s));
      if (tp && (st = nccl_wait(c, nccl().AllReduce(c->pf_x, c->pf_x, static_cast<size_t>(M) * c->h, ncclFloat32,
                                                     ncclSum, c->comm, s), "allreduce")))
        return st;
      CK(launch_norm_split(c->pf_x, W + D.post, c->cfg.rms_norm_eps, M, c->h, c->pf_ahi, c->pf_alo, s));
      GemmParams gu{};
      gu.M = M, gu.two_a = 1, gu.err = err, gu.N = c->I_l, gu.K = c->h, gu.epi = GE_SILU, gu.pair_offset = c->I_l;
      gu.out_hi = c->pf_fhi, gu.out_lo = c->pf_flo, gu.ld_out = c->I_l, gu.nk = (gu.K + kGemmBK - 1) / kGemmBK;
      streamk(gu);
      CK(launch_gemm_tc(c->tm_ah_hi, c->tm_ah_lo, c->tm_w[4 * l + 2], gu, s));
      GemmParams dn{};
      dn.M = M, dn.two_a = 1, dn.err = err, dn.N = c->h, dn.K = c->I_l, dn.epi = GE_RESID, dn.y = c->pf_x;
      dn.ldy = c->h, dn.add_residual = c->tp_rank == 0 ? 1 : 0, dn.nk = (dn.K + kGemmBK - 1) / kGemmBK;
      streamk(dn);
      CK(launch_gemm_tc(c->tm_f_hi, c->tm_f_lo, c->tm_w[4 * l + 3], dn, s));
      if (tp && (st = nccl_wait(c, nccl().AllReduce(c->pf_x, c->pf_x, static_cast<size_t>(M) * c->h, ncclFloat32,
                                                     ncclSum, c->comm, s), "allreduce")))
        return st;
      // Debug mode: the residual stream of the chunk's last token after each
      // layer (vvli_cuda_debug_hidden reads the prompt's last token).
      if (c->debug)
        CK(cudaMemcpyAsync(c->hidden + static_cast<size_t>(l) * c->h, c->pf_x + static_cast<size_t>(M - 1) * c->h,
                           c->h * sizeof(float), cudaMemcpyDeviceToDevice, s));
    }
  }
  // The last token's hidden state goes through the final norm and LM head.
  CK(cudaMemcpyAsync(c->x, c->pf_x + static_cast<size_t>(M - 1) * c->h, c->h * sizeof(float),
                     cudaMemcpyDeviceToDevice, s));
  return enqueue_lm_head(c, s, false);
}

// ---------------------------------------------------------------- decode batches
// Buffers and tensor maps of a batch chunk (kSkinnyMaxRows rows), allocated on first use.
int ensure_batch_buffers(vvli_ctx* c) {
  if (c->bt_ready) return VVLI_OK;
  constexpr int R = kSkinnyMaxRows;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device);
  CK(configure_gemm_skinny(optin));
  if (c->tm_w.empty()) {
    const int st0 = plan_tc_prefill(c);
    if (st0) return st0;
  }
  const size_t ka = std::max(c->h, c->q_rows);
  c->bt_splits_max = 16;
  int st;
  if ((st = dalloc(&c->bt_x, static_cast<size_t>(R) * c->h)) || (st = dalloc(&c->bt_q, static_cast<size_t>(R) * c->q_rows)) ||
      (st = dalloc(&c->bt_ahi, R * ka)) || (st = dalloc(&c->bt_alo, R * ka)) ||
      (st = dalloc(&c->bt_fhi, static_cast<size_t>(R) * c->I_l)) || (st = dalloc(&c->bt_flo, static_cast<size_t>(R) * c->I_l)) ||
      (st = dalloc(&c->bt_logits, static_cast<size_t>(R) * c->V_l)) ||
      (st = dalloc(&c->bt_logits_all, c->tp_size > 1 ? static_cast<size_t>(R) * c->V_l * c->tp_size : 1)) ||
      (st = dalloc(&c->bt_best, 2 * R)) || (st = dalloc(&c->bt_all_best, 2 * R * c->tp_size)) ||
      (st = dalloc(&c->bt_part, static_cast<size_t>(R) * c->nq_l * c->bt_splits_max * (c->d + 2))) ||
      (st = dalloc(&c->bt_tokens, R)) || (st = dalloc(&c->bt_pos, R)) || (st = dalloc(&c->bt_idx, R)) ||
      (st = dalloc(&c->bt_counters, static_cast<size_t>(R) * c->nkv_l)))
    return st;
  cudaError_t e;
  for (int v = 0; v < 2; ++v) {
    const uint32_t nb = v == 0 ? 16 : 32;
    if ((e = make_tmap_bf16(&c->tmb_h[v][0], c->bt_ahi, R, c->h, nb)) ||
        (e = make_tmap_bf16(&c->tmb_h[v][1], c->bt_alo, R, c->h, nb)) ||
        (e = make_tmap_bf16(&c->tmb_q[v][0], c->bt_ahi, R, c->q_rows, nb)) ||
        (e = make_tmap_bf16(&c->tmb_q[v][1], c->bt_alo, R, c->q_rows, nb)) ||
        (e = make_tmap_bf16(&c->tmb_f[v][0], c->bt_fhi, R, c->I_l, nb)) ||
        (e = make_tmap_bf16(&c->tmb_f[v][1], c->bt_flo, R, c->I_l, nb)))
      return cuda_fail(e, "make_tmap_bf16 (batch activations)");
  }
  if ((e = make_tmap_bf16(&c->tm_lm, c->w + c->off_lm, c->V_lr, c->h, 128)))
    return cuda_fail(e, "make_tmap_bf16 (lm head)");
  c->bt_ready = true;
  return VVLI_OK;
}

// One chunk of B <= kSkinnyMaxRows rows (row b = sequence slot `slot0 + b`):
// every linear layer is one skinny tensor-core GEMM that reads its weights
// once for the whole chunk.  Leaves logits in bt_logits [B][V_l] and the
// per-row argmax in bt_idx.
int forward_batch_chunk(vvli_ctx* c, const uint32_t* tokens, const uint64_t* positions, int B, int slot0) {
  cudaStream_t s = c->stream;
  const uint16_t* W = c->w;
  const bool tp = c->tp_size > 1;
  int* err = &c->st->err;
  const int pps = static_cast<int>((c->max_seq + kPage - 1) / kPage);  // pages per sequence slot
  std::vector<int> hbuf(2 * B);
  int max_pos = 0;
  for (int b = 0; b < B; ++b) {
    hbuf[b] = static_cast<int>(tokens[b]);
    hbuf[B + b] = static_cast<int>(positions[b]);
    max_pos = std::max(max_pos, hbuf[B + b]);
  }
  CK(cudaMemcpyAsync(c->bt_tokens, hbuf.data(), B * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(c->bt_pos, hbuf.data() + B, B * sizeof(int), cudaMemcpyHostToDevice, s));
  const int v = skinny_nb(B) == 16 ? 0 : 1;
  RopeParams rope{c->cfg.rope_theta, VVLI_ROPE_INTERLEAVED, static_cast<int>(c->cfg.rope_scaling_type),
                  c->cfg.rope_scaling_factor, c->cfg.rope_low_freq_factor, c->cfg.rope_high_freq_factor,
                  static_cast<float>(c->cfg.rope_original_max_position)};
  // Attention splits: (row, kv head, split) CTAs filling the resident slots once, at least a page each.
  const int slots = batch_attention_slots(c->d);
  if (!c->bt_attn_per_sm) c->bt_attn_per_sm = batch_attention_ctas_per_sm(c->group, c->d, slots);
  const int resident = c->sm_count * c->bt_attn_per_sm;
  const int want = std::max(1, (resident + B * c->nkv_l / 2) / std::max(1, B * c->nkv_l));
  const int splits = std::max(1, std::min({c->bt_splits_max, want, (max_pos + kPage) / kPage}));
  // Programmatic edges between consecutive kernels (weights stream before the
  // dependency wait); none next to NCCL collectives.
  const bool pdl = !tp;
  auto gemm = [&](const CUtensorMap* x, const CUtensorMap& w, GemmParams g, bool edge) -> int {
    g.M = B, g.two_a = 1, g.err = err, g.nk = (g.K + kGemmBK - 1) / kGemmBK;
    const int n_rows = g.N;
    CK(launch_gemm_skinny(x[0], x[1], w, g, skinny_split(g.epi, B, n_rows, g.nk, c->sm_count), s, edge));
    return VVLI_OK;
  };
  int st;
  CK(launch_prefill_embed(W + c->off_emb, c->bt_tokens, B, c->h, c->bt_x, s));
  for (int l = 0; l < c->L; ++l) {
    const DevLayer& D = c->lay[l];
    float* kc = c->kv + static_cast<size_t>(2 * l) * c->kv_layer_floats;
    float* vc = kc + c->kv_layer_floats;
    CK(launch_norm_split(c->bt_x, W + D.in_norm, c->cfg.rms_norm_eps, B, c->h, c->bt_ahi, c->bt_alo, s, pdl));
    GemmParams q{};
    q.N = c->q_rows + 2 * c->kv_rows, q.K = c->h, q.epi = GE_QKV, q.y = c->bt_q, q.ldy = c->q_rows;
    q.bias = D.b_qkv == UINT64_MAX ? nullptr : W + D.b_qkv;
    q.q_rows = c->q_rows, q.kv_rows = c->kv_rows, q.d = c->d, q.nkv = c->nkv_l, q.rope = rope;
    q.k_cache = kc, q.v_cache = vc, q.page_table = c->page_table + static_cast<size_t>(slot0) * pps;
    q.row_pos = c->bt_pos, q.seq_pages = pps;
    if ((st = gemm(c->tmb_h[v], c->tm_w[4 * l + 0], q, pdl))) return st;
    BatchAttnParams a{};
    a.q = c->bt_q, a.k_cache = kc, a.v_cache = vc, a.page_table = c->page_table + static_cast<size_t>(slot0) * pps;
    a.seq_pages = pps, a.row_pos = c->bt_pos, a.part = c->bt_part, a.counters = c->bt_counters;
    a.out_hi = c->bt_ahi, a.out_lo = c->bt_alo, a.nq = c->nq_l, a.nkv = c->nkv_l, a.d = c->d, a.group = c->group;
    a.splits = splits, a.nslots = slots, a.inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(c->d));
    a.err = err;
    CK(launch_batch_attention(a, B, s, pdl));
    GemmParams o{};
    o.N = c->h, o.K = c->q_rows, o.epi = GE_RESID, o.y = c->bt_x, o.ldy = c->h, o.add_residual = c->tp_rank == 0;
    if ((st = gemm(c->tmb_q[v], c->tm_w[4 * l + 1], o, pdl))) return st;
    if (tp && (st = tp_collective(c, c->bt_x, c->bt_x, static_cast<size_t>(B) * c->h, false, s, "allreduce"))) return st;
    CK(launch_norm_split(c->bt_x, W + D.post, c->cfg.rms_norm_eps, B, c->h, c->bt_ahi, c->bt_alo, s, pdl));
    GemmParams gu{};
    gu.N = c->I_l, gu.K = c->h, gu.epi = GE_SILU, gu.pair_offset = c->I_l;
    gu.out_hi = c->bt_fhi, gu.out_lo = c->bt_flo, gu.ld_out = c->I_l;
    if ((st = gemm(c->tmb_h[v], c->tm_w[4 * l + 2], gu, pdl))) return st;
    GemmParams dn{};
    dn.N = c->h, dn.K = c->I_l, dn.epi = GE_RESID, dn.y = c->bt_x, dn.ldy = c->h, dn.add_residual = c->tp_rank == 0;
    if ((st = gemm(c->tmb_f[v], c->tm_w[4 * l + 3], dn, pdl))) return st;
    if (tp && (st = tp_collective(c, c->bt_x, c->bt_x, static_cast<size_t>(B) * c->h, false, s, "allreduce"))) return st;
  }
  // final norm + LM head of every row (src/llm.zig:727-728), then llm.argmax per row
  CK(launch_norm_split(c->bt_x, W + c->off_final, c->cfg.rms_norm_eps, B, c->h, c->bt_ahi, c->bt_alo, s, pdl));
  GemmParams lm{};
  lm.N = c->V_lr, lm.K = c->h, lm.epi = GE_RESID, lm.y = c->bt_logits, lm.ldy = c->V_l, lm.add_residual = 0;
  if ((st = gemm(c->tmb_h[v], c->tm_lm, lm, pdl))) return st;
  CK(launch_rows_argmax(c->bt_logits, B, c->V_lr, c->V_l, c->v0, c->bt_best, s, pdl));  // this rank's real rows only
  if (tp) {
    if ((st = tp_collective(c, c->bt_best, c->bt_all_best, 2 * static_cast<size_t>(B), true, s, "allgather"))) return st;
    CK(launch_rows_argmax_merge(c->bt_all_best, c->tp_size, B, c->bt_idx, s));
  } else {
    CK(launch_rows_argmax_index(c->bt_best, B, c->bt_idx, s, pdl));
  }
  return VVLI_OK;
}

int build_graph(vvli_ctx* c) {
  if (c->graph) {
    cudaGraphExecDestroy(c->graph);
    c->graph = nullptr;
  }
  if (getenv("VVLI_NO_GRAPH")) return VVLI_OK;
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int st = enqueue_step(c, c->stream, false);
  cudaError_t e = cudaStreamEndCapture(c->stream, &g);
  if (st != VVLI_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  // A step that cannot be captured still runs, launched directly.
  if (e != cudaSuccess) {
    cudaGetLastError();
    return VVLI_OK;
  }
  e = cudaGraphInstantiate(&c->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    c->graph = nullptr;
  }
  return VVLI_OK;
}

// Launches `steps` decode steps (graph replays, or eager steps in debug mode).
int run_steps(vvli_ctx* c, int steps) {
  for (int i = 0; i < steps; ++i) {
    if (c->debug || !c->graph) {
      int st = enqueue_step(c, c->stream, c->debug);
      if (st) return st;
    } else {
      CK(cudaGraphLaunch(c->graph, c->stream));
    }
  }
  return VVLI_OK;
}

int stage_state(vvli_ctx* c, int pos, int prompt_len, int use_emb) {
  StepState* h = c->h_st;
  h->pos = pos;
  h->prompt_len = prompt_len;
  h->max_seq = static_cast<int>(c->max_seq);
  h->use_embedding = use_emb;
  h->argmax = -1;
  h->err = 0;
  h->batch = 1;
  CK(cudaMemcpyAsync(c->st, h, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
  return VVLI_OK;
}

int finish_state(vvli_ctx* c) {
  CK(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  if (c->h_st->err) {
    g_last_error = "device step reported an error";
    // An aborted megakernel step leaves its barrier count and epoch out of
    // step with each other: start both over.
    if (c->use_mega) {
      cudaMemsetAsync(c->bar, 0, sizeof(unsigned long long), c->stream);
      cudaMemsetAsync(c->epoch, 0, sizeof(unsigned), c->stream);
      if (c->acc) cudaMemsetAsync(c->acc, 0, 2 * static_cast<size_t>(c->h) * sizeof(long long), c->stream);
      cudaStreamSynchronize(c->stream);
    }
    return c->h_st->err;
  }
  return VVLI_OK;
}

// Sum (gather = false) or gather (true) of n floats per rank: through the
// mapped peer blocks when there are any (one kernel, tagged words, sums in
// rank order), else NCCL.  Every rank makes the same calls in the same order.
int tp_collective(vvli_ctx* c, const float* src, float* dst, size_t n, bool gather, cudaStream_t s, const char* what) {
  if (c->xch.block[0] && n <= static_cast<size_t>(c->xch.cap)) {
    if (++c->xch.epoch == 0) ++c->xch.epoch;
    CK(launch_tp_exchange(src, static_cast<int>(n), dst, gather ? 1 : 0, c->xch, c->sm_count, s));
    return VVLI_OK;
  }
  return nccl_wait(c,
                   gather ? nccl().AllGather(src, dst, n, ncclFloat32, c->comm, s)
                          : nccl().AllReduce(src, dst, n, ncclFloat32, ncclSum, c->comm, s),
                   what);
}

int copy_logits(vvli_ctx* c, float* out) {
  if (!out) return VVLI_OK;
  if (c->tp_size > 1) {
    int st = tp_collective(c, c->logits, c->logits_full, c->V_l, true, c->stream, "allgather logits");
    if (st) return st;
    CK(cudaMemcpyAsync(out, c->logits_full, static_cast<size_t>(c->V) * 4, cudaMemcpyDeviceToHost, c->stream));
  } else {
    CK(cudaMemcpyAsync(out, c->logits, static_cast<size_t>(c->V) * 4, cudaMemcpyDeviceToHost, c->stream));
  }
  return VVLI_OK;
}

void free_ctx(vvli_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->graph) cudaGraphExecDestroy(c->graph);
  for (int q = 0; q < kMaxTp; ++q)
    if (c->peer_base[q] && c->peer_base[q] != c->peer_block) cudaIpcCloseMemHandle(c->peer_base[q]);
  if (c->peer_block) cudaFree(c->peer_block);
  if (c->comm) nccl().CommDestroy(c->comm);
  void* dev[] = {c->w, c->kv, c->page_table, c->x, c->qkv, c->attn, c->ff, c->logits, c->logits_full, c->emb_in,
                 c->hidden, c->attn_part, c->amax_val, c->amax_idx, c->best, c->all_best, c->counters,
                 c->seq_tokens, c->st, c->ssq, c->bar, c->epoch, c->d_phases, c->trace, c->w_downT, c->acc, c->pf_x, c->pf_q,
                 c->pf_ahi, c->pf_alo, c->pf_fhi, c->pf_flo, c->pf_tokens, c->pf_kvt, c->pf_skws, c->pf_skflags, c->smp_stamp, c->smp_key32,
                 c->smp_key64, c->smp_key64_sorted, c->smp_probs, c->smp_logits, c->smp_state, c->smp_done,
                 c->bt_x, c->bt_q, c->bt_logits, c->bt_best, c->bt_all_best, c->bt_part, c->bt_logits_all, c->bt_ahi,
                 c->bt_alo, c->bt_fhi, c->bt_flo, c->bt_tokens, c->bt_pos, c->bt_idx, c->bt_counters};
  for (void* p : dev)
    if (p) cudaFree(p);
  if (c->h_st) cudaFreeHost(c->h_st);
  if (c->h_tok) cudaFreeHost(c->h_tok);
  if (c->h_smp_state) cudaFreeHost(c->h_smp_state);  // the recent-token staging lives in the same block
  if (c->h_smp_out) cudaFreeHost(c->h_smp_out);
  if (c->ev0) cudaEventDestroy(c->ev0);
  if (c->ev1) cudaEventDestroy(c->ev1);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}


}  // namespace

// ================================================================ C ABI
extern "C" {

const char* vvli_cuda_strerror(int status) {
  switch (status) {
    case VVLI_OK: return "ok";
    case VVLI_ERR_CONTEXT_FULL: return "ContextFull";
    case VVLI_ERR_INVALID_CONFIG: return "InvalidConfig";
    case VVLI_ERR_INVALID_TOKEN: return "InvalidToken";
    case VVLI_ERR_INVALID_WEIGHT: return "InvalidWeight";
    case VVLI_ERR_UNSUPPORTED_DTYPE: return "UnsupportedDType";
    case VVLI_ERR_UNSUPPORTED_ARCH: return "UnsupportedModelArchitecture";
    case VVLI_ERR_EMPTY_PROMPT: return "EmptyPrompt";
    case VVLI_ERR_OUTPUT_TOO_SMALL: return "OutputTooSmall";
    case VVLI_ERR_INVALID_SAMPLING: return "InvalidSamplingOptions";
    case VVLI_ERR_MISSING_TENSOR: return "MissingSafetensorsTensor";
    case VVLI_ERR_INVALID_GGUF: return "InvalidGguf";
    case VVLI_ERR_UNSUPPORTED_GGUF_VERSION: return "UnsupportedGgufVersion";
    case VVLI_ERR_UNSUPPORTED_METADATA_TYPE: return "UnsupportedMetadataType";
    case VVLI_ERR_CUDA: return "CudaError";
    case VVLI_ERR_NCCL: return "NcclError";
    case VVLI_ERR_TIMEOUT: return "Timeout";
    case VVLI_ERR_OOM: return "OutOfMemory";
    case VVLI_ERR_NOT_LOADED: return "WeightsNotLoaded";
    case VVLI_ERR_INVALID_ARGUMENT: return "InvalidArgument";
    case VVLI_ERR_UNIMPLEMENTED: return "Unimplemented";
    default: return "UnknownError";
  }
}

const char* vvli_cuda_last_error(void) { return g_last_error.c_str(); }

int vvli_cuda_storage_elements(const vvli_model_config* cfg, uint64_t* out) {
  if (!cfg || !out) return VVLI_ERR_INVALID_ARGUMENT;
  int st = validate_config(*cfg);
  if (st == VVLI_ERR_INVALID_CONFIG) return st;
  *out = blob_layout(*cfg).total;
  return VVLI_OK;
}

int vvli_cuda_tp_plan(const vvli_model_config* cfg, int tp_rank, int tp_size, uint64_t* out, uint64_t cap,
                      uint64_t* count) {
  if (!cfg || !count || tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return VVLI_ERR_INVALID_ARGUMENT;
  int st = validate_config(*cfg);
  if (st) return st;
  if (cfg->num_key_value_heads % tp_size || cfg->intermediate_size % (8ull * tp_size)) return VVLI_ERR_INVALID_CONFIG;
  vvli_ctx tmp;
  if ((st = fill_dims(&tmp, *cfg, tp_rank, tp_size))) return st;
  plan_weights(&tmp);
  *count = tmp.pieces.size();
  for (size_t i = 0; i < tmp.pieces.size() && out && i < cap; ++i) {
    const Piece& p = tmp.pieces[i];
    const uint64_t row[9] = {p.dst, p.tensor_id, p.src, p.rows, p.cols, p.src_ld, p.row0, p.col0,
                             static_cast<uint64_t>(p.kind)};
    std::memcpy(out + 9 * i, row, sizeof(row));
  }
  return VVLI_OK;
}

int vvli_cuda_nccl_unique_id(void* id) {
  if (!id) return VVLI_ERR_INVALID_ARGUMENT;
  auto& n = nccl();
  if (!n.ok) {
    g_last_error = n.why;
    return VVLI_ERR_NCCL;
  }
  ncclUniqueId uid;
  ncclResult_t r = n.GetUniqueId(&uid);
  if (r != ncclSuccess) return VVLI_ERR_NCCL;
  static_assert(sizeof(ncclUniqueId) == VVLI_NCCL_ID_BYTES, "ncclUniqueId size");
  std::memcpy(id, &uid, sizeof(uid));
  return VVLI_OK;
}

static int setup_tp_peers(vvli_ctx* c);

int vvli_cuda_create(const vvli_model_config* cfg, int device, int tp_rank, int tp_size, const void* nccl_unique_id,
                     uint64_t max_seq, uint64_t max_batch, vvli_ctx** out_ctx) {
  if (!cfg || !out_ctx) return VVLI_ERR_INVALID_ARGUMENT;
  *out_ctx = nullptr;
  int st = validate_config(*cfg);
  if (st) return st;
  if (max_seq == 0 || max_seq > cfg->max_position_embeddings || max_seq > (1u << 30)) return VVLI_ERR_INVALID_CONFIG;
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return VVLI_ERR_INVALID_ARGUMENT;
  if (tp_size > 1 && !nccl_unique_id) return VVLI_ERR_INVALID_ARGUMENT;
  const uint64_t d = cfg->hidden_size / cfg->num_attention_heads;
  // Shapes the kernels take: 16-byte weight rows; head_dim a multiple of 4 up to 32, or 64, 128, 256; q heads per kv head x head_dim <= 2048.
  const bool d_ok = (d <= 32 && d % 4 == 0) || d == 64 || d == 128 || d == 256;
  if (cfg->hidden_size % 8 || cfg->intermediate_size % 8 || !d_ok ||
      (cfg->num_attention_heads / cfg->num_key_value_heads) * d > 2048)
    return VVLI_ERR_UNSUPPORTED_ARCH;
  if (cfg->num_key_value_heads % tp_size || cfg->intermediate_size % (8ull * tp_size)) return VVLI_ERR_INVALID_CONFIG;
  if (((cfg->num_attention_heads / tp_size) * d) % 8) return VVLI_ERR_INVALID_CONFIG;

  auto* c = new vvli_ctx();
  if (fill_dims(c, *cfg, tp_rank, tp_size) != VVLI_OK) {
    delete c;
    return VVLI_ERR_INVALID_CONFIG;
  }
  c->device = device;
  c->max_seq = max_seq;
  c->max_batch = std::max<uint64_t>(1, max_batch);

  auto fail = [&](int code) {
    free_ctx(c);
    return code;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e) return fail(cuda_fail(e, "cudaSetDevice"));
  int smem_optin = 0;
  cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if ((e = configure_kernels(smem_optin))) return fail(cuda_fail(e, "configure_kernels"));
  if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking))) return fail(cuda_fail(e, "stream"));
  cudaEventCreate(&c->ev0);
  cudaEventCreate(&c->ev1);

  plan_weights(c);
  if ((st = dalloc(&c->w, c->weight_elems))) return fail(st);

  // Paged KV cache: [layer][K|V][page][kv_head][kPage][d] fp32.
  c->max_pages = static_cast<int>((max_seq + kPage - 1) / kPage) * static_cast<int>(c->max_batch);
  c->kv_layer_floats = static_cast<size_t>(c->max_pages) * c->nkv_l * kPage * c->d;
  if ((st = dalloc(&c->kv, 2 * c->kv_layer_floats * c->L))) return fail(st);
  if ((st = dalloc(&c->page_table, c->max_pages))) return fail(st);
  std::vector<int> pt(c->max_pages);
  for (int i = 0; i < c->max_pages; ++i) pt[i] = i;
  if ((e = cudaMemcpy(c->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice))) return fail(cuda_fail(e, "pt"));

  // Attention: one CTA per (kv head, group of 64-position pages); about two
  // CTAs per SM over the kv heads once the context is long enough.
  {
    const int pages = static_cast<int>((max_seq + kPage - 1) / kPage);
    c->attn_splits = std::max(1, std::min(pages, (2 * c->sm_count + c->nkv_l - 1) / c->nkv_l));
    c->mega_splits = std::max(1, std::min({pages, c->sm_count / c->nkv_l, 16}));  // the merge stages <= 16 splits
    if (attention_smem_bytes(c->group, c->d, c->attn_splits) > static_cast<size_t>(smem_optin)) {
      delete c;
      return VVLI_ERR_UNSUPPORTED_ARCH;
    }
  }
  const size_t B = c->max_batch;
  if ((st = dalloc(&c->x, B * c->h)) || (st = dalloc(&c->qkv, B * (c->q_rows + 2 * c->kv_rows))) ||
      (st = dalloc(&c->attn, B * c->q_rows)) || (st = dalloc(&c->ff, B * c->I_l)) ||
      (st = dalloc(&c->logits, B * static_cast<size_t>(c->V_l))) ||
      (st = dalloc(&c->logits_full, static_cast<size_t>(c->V_l) * tp_size)) || (st = dalloc(&c->emb_in, c->h)) ||
      (st = dalloc(&c->hidden, static_cast<size_t>(c->L) * c->h)) ||
      (st = dalloc(&c->attn_part, static_cast<size_t>(c->nq_l) * std::max(c->attn_splits, c->mega_splits) * (c->d + 2))) ||
      (st = dalloc(&c->ssq, c->sm_count)) || (st = dalloc(&c->bar, 1)) || (st = dalloc(&c->epoch, 1)) ||
      (st = dalloc(&c->amax_val, 2 * c->sm_count)) || (st = dalloc(&c->amax_idx, 2 * c->sm_count)) ||
      (st = dalloc(&c->best, 2)) || (st = dalloc(&c->all_best, 2 * tp_size)) ||
      (st = dalloc(&c->counters, c->nkv_l + 1)) || (st = dalloc(&c->seq_tokens, max_seq + 1)) ||
      (st = dalloc(&c->st, 1)))
    return fail(st);
  if ((e = cudaMallocHost(&c->h_st, sizeof(StepState))) || (e = cudaMallocHost(&c->h_tok, 64 * sizeof(int))))
    return fail(cuda_fail(e, "cudaMallocHost"));

  if (tp_size > 1) {
    auto& n = nccl();
    if (!n.ok) {
      g_last_error = n.why;
      return fail(VVLI_ERR_NCCL);
    }
    ncclUniqueId uid;
    std::memcpy(&uid, nccl_unique_id, sizeof(uid));
    ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
    ncfg.blocking = 0;
    ncclResult_t r = n.CommInitRankConfig(&c->comm, tp_size, uid, tp_rank, &ncfg);
    if ((st = nccl_wait(c, r, "ncclCommInitRankConfig"))) return fail(st);
  }
  {
    const char* tc_env = getenv("VVLI_TC_PREFILL");
    if (!(tc_env && tc_env[0] == '0') && configure_gemm_tc(smem_optin) == cudaSuccess && plan_tc_prefill(c) == VVLI_OK)
      c->tc_prefill = c->tc_prefill_planned = true;
    cudaGetLastError();
  }
  c->smem_optin = smem_optin;
  const char* mega_env = getenv("VVLI_MEGAKERNEL");
  const bool want_mega = !(mega_env && mega_env[0] == '0') && tp_size <= kMaxTp;
  c->want_mega = want_mega;
  if (want_mega) {
    if ((e = configure_megakernel(smem_optin))) return fail(cuda_fail(e, "configure_megakernel"));
    c->use_mega = plan_megakernel(c, smem_optin);
    // Under tensor parallelism the megakernel needs every peer's exchange block;
    // without it (no peer access) the per-kernel step with NCCL runs instead.
    if (!c->use_mega) g_last_error = "megakernel: no plan fits this model";
    if (c->use_mega && tp_size > 1 && setup_tp_peers(c) != VVLI_OK) {
      c->use_mega = false;  // g_last_error says why
      cudaGetLastError();
    }
  }
  if (tp_size > 1) {
    // Every rank must take the same path (a megakernel rank waits for peers'
    // flags, a per-kernel rank for NCCL): the megakernel runs only if all
    // ranks could set it up.
    int* flag = nullptr;
    int mine = c->use_mega ? 1 : 0, all = 0;
    if ((e = cudaMalloc(&flag, sizeof(int)))) return fail(cuda_fail(e, "cudaMalloc"));
    cudaMemcpy(flag, &mine, sizeof(int), cudaMemcpyHostToDevice);
    st = nccl_wait(c, nccl().AllReduce(flag, flag, 1, ncclInt32, ncclMin, c->comm, c->stream), "allreduce (path)");
    if (st == VVLI_OK) e = cudaStreamSynchronize(c->stream);
    if (st == VVLI_OK && e == cudaSuccess) e = cudaMemcpy(&all, flag, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(flag);
    if (st) return fail(st);
    c->use_mega = all == 1;
  }
  *out_ctx = c;
  return VVLI_OK;
}

// Tensor-parallel megakernel: each rank allocates one exchange block — the
// receive words of the o_proj / down_proj partial sums [2 parities][tp][h]
// (each an 8-byte word: the exchange's epoch and the row's fp32 bits), flags
// [2][tp][CTAs], and the LM-head argmax slots [tp][2] with flags [tp] —
// exports it as a CUDA IPC handle, gathers every rank's handle over NCCL and
// maps the peers' blocks.  The megakernel then stores its partials straight
// into every peer's block over NVLink (plain stores, no multicast) and polls,
// bounded, its own block until every word carries the exchange's epoch.
static int setup_tp_peers(vvli_ctx* c) {
  const int tp = c->tp_size, grid = c->sm_count;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t recv_off = 0, recv_bytes = 2ull * tp * c->h * 8;
  const size_t flag_off = up(recv_off + recv_bytes), flag_bytes = 2ull * tp * grid * 4;
  const size_t best_off = up(flag_off + flag_bytes), best_bytes = 2ull * tp * 4;
  const size_t bflag_off = up(best_off + best_bytes), bflag_bytes = static_cast<size_t>(tp) * 4;
  const int xcap = std::max(c->V_l, kSkinnyMaxRows * c->h);
  const size_t xch_off = up(bflag_off + bflag_bytes), xch_bytes = 2ull * tp * xcap * 8;
  const size_t total = up(xch_off + xch_bytes);
  CK(cudaMalloc(&c->peer_block, total));
  CK(cudaMemset(c->peer_block, 0, total));
  cudaIpcMemHandle_t mine;
  CK(cudaIpcGetMemHandle(&mine, c->peer_block));
  uint8_t* ids = nullptr;
  CK(cudaMalloc(&ids, sizeof(cudaIpcMemHandle_t) * tp));
  std::vector<cudaIpcMemHandle_t> all(tp);
  int st = VVLI_OK;
  cudaError_t e = cudaMemcpy(ids + sizeof(mine) * c->tp_rank, &mine, sizeof(mine), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    st = nccl_wait(c, nccl().AllGather(ids + sizeof(mine) * c->tp_rank, ids, sizeof(mine), ncclChar, c->comm, c->stream),
                   "allgather ipc handles");
  // the gather runs on c->stream (non-blocking): wait for it before reading
  if (e == cudaSuccess && st == VVLI_OK) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess && st == VVLI_OK) e = cudaMemcpy(all.data(), ids, sizeof(mine) * tp, cudaMemcpyDeviceToHost);
  cudaFree(ids);
  if (st) return st;
  if (e) return cuda_fail(e, "ipc handle exchange");
  MegaParams& P = c->mp;
  for (int q = 0; q < tp; ++q) {
    void* base = c->peer_block;
    if (q != c->tp_rank) {
      e = cudaIpcOpenMemHandle(&base, all[q], cudaIpcMemLazyEnablePeerAccess);
      if (e) return cuda_fail(e, "cudaIpcOpenMemHandle (peer exchange block)");
    }
    c->peer_base[q] = base;
    uint8_t* b = static_cast<uint8_t*>(base);
    P.peer_recv[q] = reinterpret_cast<unsigned long long*>(b + recv_off);
    P.peer_flags[q] = reinterpret_cast<unsigned*>(b + flag_off);
    P.peer_best[q] = reinterpret_cast<float*>(b + best_off);
    P.peer_best_flag[q] = reinterpret_cast<unsigned*>(b + bflag_off);
    c->xch.block[q] = reinterpret_cast<unsigned long long*>(b + xch_off);
  }
  c->xch.tp = tp, c->xch.rank = c->tp_rank, c->xch.cap = xcap, c->xch.epoch = 0, c->xch.err = &c->st->err;
  return VVLI_OK;
}

// Bytes of every weight matrix of this rank as stored (bf16 rows or quantised
// rows with their scales): what one decode step streams besides norms and KV.
static uint64_t weight_stream_bytes(const vvli_ctx* c) {
  uint64_t b = 0;
  for (const DevLayer& D : c->lay) {
    b += static_cast<uint64_t>(c->q_rows + 2 * c->kv_rows) * row_bytes_of(D.f_qkv, c->h);
    b += static_cast<uint64_t>(c->h) * row_bytes_of(D.f_o, c->q_rows);
    b += 2ull * c->I_l * row_bytes_of(D.f_gu, c->h);
    b += static_cast<uint64_t>(c->h) * row_bytes_of(D.f_down, c->I_l);
  }
  return b + static_cast<uint64_t>(c->V_lr) * row_bytes_of(c->f_lm, c->h);
}

// Every matrix back to bf16 (the blob, safetensors and synthetic loads).
static void set_bf16_formats(vvli_ctx* c) {
  for (DevLayer& D : c->lay) D.f_qkv = D.f_o = D.f_gu = D.f_down = kFmtBF16;
  c->f_emb = c->f_lm = kFmtBF16;
  c->quant = false;
}

// Formats of a GGUF load from the format each piece was stored in: the pieces
// of a fused matrix (q|k|v, gate|up) must agree.  Block-quantised matrices
// run only in the single-GPU decode megakernel.
static int set_loaded_formats(vvli_ctx* c, const std::vector<int>& piece_fmt) {
  std::map<uint64_t, int> fmt;  // tensor id -> format
  for (size_t i = 0; i < c->pieces.size(); ++i) fmt[c->pieces[i].tensor_id] = piece_fmt[i];
  auto f = [&](uint64_t id) { auto it = fmt.find(id); return it == fmt.end() ? static_cast<int>(kFmtBF16) : it->second; };
  bool ok = true;
  c->quant = false;
  for (int l = 0; l < c->L; ++l) {
    DevLayer& D = c->lay[l];
    const uint64_t base = 1 + 12ull * l;
    D.f_qkv = f(base + 1);
    ok = ok && f(base + 3) == D.f_qkv && f(base + 5) == D.f_qkv;
    D.f_o = f(base + 7);
    D.f_gu = f(base + 9);
    ok = ok && f(base + 10) == D.f_gu;
    D.f_down = f(base + 11);
    c->quant = c->quant || D.f_qkv || D.f_o || D.f_gu || D.f_down;
  }
  c->f_emb = f(0);
  c->f_lm = c->lm_aliases_emb ? c->f_emb : f(2 + 12ull * c->L);
  c->quant = c->quant || c->f_emb || c->f_lm;
  if (!ok) {
    g_last_error = "q, k and v (and gate and up) of a layer must share one tensor type";
    set_bf16_formats(c);
    return VVLI_ERR_UNSUPPORTED_DTYPE;
  }
  if (c->quant && c->tp_size > 1) {
    g_last_error = "block-quantised (Q8_0 / Q4_0) GGUF tensors run on one GPU (tp_size 1)";
    set_bf16_formats(c);
    return VVLI_ERR_UNSUPPORTED_DTYPE;
  }
  return VVLI_OK;
}

static int after_load(vvli_ctx* c) {
  // The megakernel plan follows the matrix formats: plan again when a load
  // changed them (tp = 1 only; quantised loads require it).
  int sig = c->f_emb * 3 + c->f_lm;
  for (const DevLayer& D : c->lay) sig = sig * 7 + D.f_qkv * 27 + D.f_o * 9 + D.f_gu * 3 + D.f_down;
  if (sig != c->plan_sig && c->tp_size == 1 && c->smem_optin) {
    c->use_mega = c->want_mega && plan_megakernel(c, c->smem_optin);
    c->plan_sig = sig;
    // the new plan starts its barrier count and step epoch from zero
    CK(cudaMemsetAsync(c->bar, 0, sizeof(unsigned long long), c->stream));
    CK(cudaMemsetAsync(c->epoch, 0, sizeof(unsigned), c->stream));
  }
  c->tc_prefill = c->tc_prefill_planned && !c->quant;
  if (c->quant && !c->use_mega) {
    g_last_error = "block-quantised weights need the decode megakernel (VVLI_MEGAKERNEL unset and a plan that fits)";
    set_bf16_formats(c);
    c->loaded = false;
    return VVLI_ERR_UNSUPPORTED_DTYPE;
  }
  // Split-half RoPE: put rotary pairs on adjacent q/k rows (device layout).
  if (c->cfg.rope_layout == VVLI_ROPE_SPLIT_HALF && !c->rows_paired) {
    const int rows = c->q_rows + c->kv_rows;
    uint16_t* tmp = nullptr;
    CK(cudaMalloc(&tmp, static_cast<size_t>(rows) * c->h * 2));
    for (int l = 0; l < c->L; ++l) {
      const DevLayer& D = c->lay[l];
      cudaError_t e = launch_pair_rows(c->w + D.w_qkv, D.b_qkv == UINT64_MAX ? nullptr : c->w + D.b_qkv, tmp, rows,
                                       c->h, c->d, c->stream);
      if (e) {
        cudaFree(tmp);
        return cuda_fail(e, "launch_pair_rows");
      }
    }
    CK(cudaStreamSynchronize(c->stream));
    cudaFree(tmp);
  }
  if (c->w_downT) {  // fused down_proj streams W_down^T rows
    for (int l = 0; l < c->L; ++l)
      CK(launch_transpose_bf16(c->w + c->lay[l].w_down, c->w_downT + static_cast<size_t>(l) * c->I_l * c->h, c->h,
                               c->I_l, c->stream));
  }
  CK(cudaStreamSynchronize(c->stream));
  c->rows_paired = false;
  c->loaded = true;
  return build_graph(c);
}

int vvli_cuda_load_weights(vvli_ctx* c, const uint16_t* blob, uint64_t n) {
  if (!c || !blob) return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(c->device));
  if (n < blob_layout(c->cfg).total) return VVLI_ERR_INVALID_WEIGHT;
  set_bf16_formats(c);
  for (const Piece& p : c->pieces) {
    const uint16_t* src = blob + p.src + p.row0 * p.src_ld + p.col0;
    if (p.rows == 1) {
      CK(cudaMemcpyAsync(c->w + p.dst, src, p.cols * 2, cudaMemcpyHostToDevice, c->stream));
    } else {
      CK(cudaMemcpy2DAsync(c->w + p.dst, p.cols * 2, src, p.src_ld * 2, p.cols * 2, p.rows, cudaMemcpyHostToDevice,
                           c->stream));
    }
  }
  return after_load(c);
}

// Element count of the reference tensor with blob order id `id`.
static uint64_t tensor_elems(const vvli_model_config& cfg, uint64_t id) {
  const uint64_t h = cfg.hidden_size, kv = cfg.num_key_value_heads * (cfg.hidden_size / cfg.num_attention_heads),
                 I = cfg.intermediate_size, V = cfg.vocab_size, L = cfg.num_hidden_layers;
  if (id == 0 || id == 2 + 12 * L) return V * h;
  if (id == 1 + 12 * L) return h;
  switch ((id - 1) % 12) {
    case 0: case 2: case 8: return h;           // norms, q bias
    case 1: case 7: return h * h;               // q, o
    case 3: case 5: return kv * h;              // k, v
    case 4: case 6: return kv;                  // k, v bias
    default: return I * h;                      // gate, up, down
  }
}

// This rank's shard plan as file pieces (the loaders read nothing else).
static std::vector<LoadPiece> load_pieces(const vvli_ctx* c) {
  std::vector<LoadPiece> lp;
  lp.reserve(c->pieces.size());
  for (const Piece& p : c->pieces)
    lp.push_back(LoadPiece{p.tensor_id, tensor_elems(c->cfg, p.tensor_id), p.dst, p.rows, p.cols, p.src_ld, p.row0,
                           p.col0, p.group_base, p.group_row});
  return lp;
}

int vvli_cuda_load_safetensors(vvli_ctx* c, const char* path) {
  if (!c || !path) return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(c->device));
  std::string why;
  set_bf16_formats(c);
  const int st = upload_safetensors(path, load_pieces(c), c->L, c->w, c->stream, &why);
  if (st != VVLI_OK) {
    g_last_error = why;
    return st;
  }
  return after_load(c);
}

int vvli_cuda_load_gguf(vvli_ctx* c, const char* path) {
  if (!c || !path) return VVLI_ERR_INVALID_ARGUMENT;
  if (c->cfg.qkv_bias) return VVLI_ERR_UNSUPPORTED_ARCH;  // loadGgufIntoOwnedModel (src/llm.zig:1011)
  if (c->cfg.rope_layout != VVLI_ROPE_INTERLEAVED) {
    g_last_error = "a GGUF model needs rope_layout INTERLEAVED (Config.fromGguf)";
    return VVLI_ERR_INVALID_CONFIG;
  }
  CK(cudaSetDevice(c->device));
  std::string why;
  std::vector<int> piece_fmt;
  int st = upload_gguf(path, load_pieces(c), c->L, c->w, c->stream, &why, &piece_fmt);
  if (st != VVLI_OK) {
    g_last_error = why;
    set_bf16_formats(c);
    return st;
  }
  if ((st = set_loaded_formats(c, piece_fmt))) return st;
  return after_load(c);
}

int vvli_cuda_fill_synthetic(vvli_ctx* c, uint64_t seed) {
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(c->device));
  set_bf16_formats(c);
  for (const Piece& p : c->pieces)
    CK(launch_synth_fill(c->w + p.dst, tensor_key(seed, p.tensor_id), p.rows, p.cols, p.src_ld, p.row0, p.col0,
                         p.kind, c->stream));
  return after_load(c);
}

int vvli_cuda_fill_synthetic_quantized(vvli_ctx* c, uint64_t seed, int format) {
  if (!c || (format != kFmtQ8 && format != kFmtQ4)) return VVLI_ERR_INVALID_ARGUMENT;
  if (c->tp_size > 1) {
    g_last_error = "block-quantised weights run on one GPU (tp_size 1)";
    return VVLI_ERR_UNSUPPORTED_DTYPE;
  }
  if (c->h % 32 || c->I_l % 32 || c->q_rows % 32) {
    g_last_error = "block quantisation needs hidden, intermediate and q widths that are multiples of 32";
    return VVLI_ERR_UNSUPPORTED_DTYPE;
  }
  CK(cudaSetDevice(c->device));
  set_bf16_formats(c);
  c->loaded = false;
  for (const Piece& p : c->pieces)
    CK(launch_synth_fill(c->w + p.dst, tensor_key(seed, p.tensor_id), p.rows, p.cols, p.src_ld, p.row0, p.col0,
                         p.kind, c->stream));
  // Rotary-pair row order first (it moves whole bf16 rows; blocks lie along rows).
  if (c->cfg.rope_layout == VVLI_ROPE_SPLIT_HALF) {
    const int rows = c->q_rows + c->kv_rows;
    uint16_t* tmp = nullptr;
    CK(cudaMalloc(&tmp, static_cast<size_t>(rows) * c->h * 2));
    for (int l = 0; l < c->L; ++l) {
      const DevLayer& D = c->lay[l];
      cudaError_t e = launch_pair_rows(c->w + D.w_qkv, D.b_qkv == UINT64_MAX ? nullptr : c->w + D.b_qkv, tmp, rows,
                                       c->h, c->d, c->stream);
      if (e) {
        cudaFree(tmp);
        return cuda_fail(e, "launch_pair_rows");
      }
    }
    CK(cudaStreamSynchronize(c->stream));
    cudaFree(tmp);
  }
  // Every matrix (embedding, q|k|v, o, gate|up, down, LM head) quantised in
  // place from a bf16 copy.
  struct Mat { uint64_t off, rows; int K; };
  std::vector<Mat> mats;
  mats.push_back({c->off_emb, static_cast<uint64_t>(c->V), c->h});
  for (const DevLayer& D : c->lay) {
    mats.push_back({D.w_qkv, static_cast<uint64_t>(c->q_rows + 2 * c->kv_rows), c->h});
    mats.push_back({D.w_o, static_cast<uint64_t>(c->h), c->q_rows});
    mats.push_back({D.w_gu, 2ull * c->I_l, c->h});
    mats.push_back({D.w_down, static_cast<uint64_t>(c->h), c->I_l});
  }
  if (!c->lm_aliases_emb) mats.push_back({c->off_lm, static_cast<uint64_t>(c->V_lr), c->h});
  size_t big = 0;
  for (const Mat& m : mats) big = std::max<size_t>(big, m.rows * m.K);
  uint16_t* stage = nullptr;
  CK(cudaMalloc(&stage, big * 2));
  cudaError_t e = cudaSuccess;
  for (const Mat& m : mats) {
    if ((e = cudaMemcpyAsync(stage, c->w + m.off, m.rows * m.K * 2, cudaMemcpyDeviceToDevice, c->stream))) break;
    if ((e = launch_quantize_rows(stage, m.rows, m.K, format, reinterpret_cast<uint8_t*>(c->w + m.off), c->stream)))
      break;
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  cudaFree(stage);
  if (e) return cuda_fail(e, "quantise weights");
  for (DevLayer& D : c->lay) D.f_qkv = D.f_o = D.f_gu = D.f_down = format;
  c->f_emb = c->f_lm = format;
  c->quant = true;
  c->rows_paired = true;
  return after_load(c);
}

int vvli_cuda_reset(vvli_ctx* c) {  // KVCache.clear (src/llm.zig:576-579)
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(c->device));
  CK(cudaMemsetAsync(c->kv, 0, 2 * c->kv_layer_floats * c->L * sizeof(float), c->stream));
  CK(cudaStreamSynchronize(c->stream));
  return VVLI_OK;
}

static int forward_common(vvli_ctx* c, uint64_t position, float* logits_out, uint32_t* argmax_out, int use_emb) {
  int st;
  if ((st = stage_state(c, static_cast<int>(position), 0, use_emb))) return st;
  CK(cudaEventRecord(c->ev0, c->stream));
  if ((st = run_steps(c, 1))) return st;
  CK(cudaEventRecord(c->ev1, c->stream));
  if ((st = copy_logits(c, logits_out))) return st;
  if ((st = finish_state(c))) return st;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  if (argmax_out) *argmax_out = static_cast<uint32_t>(c->h_st->argmax);
  return VVLI_OK;
}

int vvli_cuda_forward_token(vvli_ctx* c, uint32_t token, uint64_t position, float* logits_out, uint32_t* argmax_out) {
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (token >= c->cfg.vocab_size) return VVLI_ERR_INVALID_TOKEN;
  if (position >= c->max_seq) return VVLI_ERR_CONTEXT_FULL;
  CK(cudaSetDevice(c->device));
  c->h_tok[0] = static_cast<int>(token);
  CK(cudaMemcpyAsync(c->seq_tokens + position, c->h_tok, sizeof(int), cudaMemcpyHostToDevice, c->stream));
  return forward_common(c, position, logits_out, argmax_out, 0);
}

int vvli_cuda_forward_embedding(vvli_ctx* c, const float* emb, uint64_t position, float* logits_out,
                                uint32_t* argmax_out) {
  if (!c || !emb) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (position >= c->max_seq) return VVLI_ERR_CONTEXT_FULL;
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpyAsync(c->emb_in, emb, static_cast<size_t>(c->h) * 4, cudaMemcpyHostToDevice, c->stream));
  return forward_common(c, position, logits_out, argmax_out, 1);
}

int vvli_cuda_prefill(vvli_ctx* c, const uint32_t* tokens, uint64_t n, uint64_t start, float* last_logits,
                      uint32_t* argmax_out) {
  if (!c || (!tokens && n)) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (n == 0) return VVLI_ERR_EMPTY_PROMPT;
  for (uint64_t i = 0; i < n; ++i)
    if (tokens[i] >= c->cfg.vocab_size) return VVLI_ERR_INVALID_TOKEN;
  if (start + n > c->max_seq) return VVLI_ERR_CONTEXT_FULL;
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpyAsync(c->seq_tokens + start, tokens, n * sizeof(int), cudaMemcpyHostToDevice, c->stream));
  int st;
  const bool tc = c->tc_prefill && n >= 2;
  // The tensor-core path ends in the LM head of the last token, which
  // publishes its argmax and advances the state from position start + n - 1.
  if ((st = stage_state(c, static_cast<int>(tc ? start + n - 1 : start), static_cast<int>(start + n), 0))) return st;
  CK(cudaEventRecord(c->ev0, c->stream));
  if (tc) {
    if ((st = prefill_tc(c, tokens, n, start))) return st;
  } else if ((st = run_steps(c, static_cast<int>(n)))) {
    return st;
  }
  CK(cudaEventRecord(c->ev1, c->stream));
  if ((st = copy_logits(c, last_logits))) return st;
  if ((st = finish_state(c))) return st;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  if (argmax_out) *argmax_out = static_cast<uint32_t>(c->h_st->argmax);
  return VVLI_OK;
}

int vvli_cuda_prefill_batch(vvli_ctx* c, const uint32_t* tokens, const uint64_t* lengths, uint64_t B,
                            float* last_logits, uint32_t* argmax_out) {
  if (!c || (B && (!tokens || !lengths))) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (c->quant) {
    g_last_error = "prefill of several sequences runs on bf16 weights only (this model is block-quantised)";
    return VVLI_ERR_UNIMPLEMENTED;
  }
  if (B == 0) return VVLI_OK;
  if (B > c->max_batch) {
    g_last_error = "prefill of " + std::to_string(B) + " sequences exceeds the context's max_batch " +
                   std::to_string(c->max_batch);
    return VVLI_ERR_INVALID_ARGUMENT;
  }
  uint64_t total = 0;
  for (uint64_t b = 0; b < B; ++b) {
    if (lengths[b] == 0) return VVLI_ERR_EMPTY_PROMPT;
    if (lengths[b] > c->max_seq) return VVLI_ERR_CONTEXT_FULL;
    total += lengths[b];
  }
  for (uint64_t i = 0; i < total; ++i)
    if (tokens[i] >= c->cfg.vocab_size) return VVLI_ERR_INVALID_TOKEN;
  if (!c->tc_prefill) {
    g_last_error = "prefill of several sequences needs the tensor-core prefill path";
    return VVLI_ERR_UNIMPLEMENTED;
  }
  CK(cudaSetDevice(c->device));
  int st;
  float ms_total = 0.f;
  uint64_t off = 0;
  for (uint64_t b = 0; b < B; ++b) {
    const uint64_t n = lengths[b];
    // The LM head of the sequence's last token publishes its argmax through the
    // step state; only sequence 0 (slot 0, the single-sequence slot) also
    // records it as its next token.
    if ((st = stage_state(c, static_cast<int>(n - 1), static_cast<int>(b == 0 ? n : n + 1), 0))) return st;
    CK(cudaEventRecord(c->ev0, c->stream));
    if ((st = prefill_tc(c, tokens + off, n, 0, static_cast<int>(b)))) return st;
    CK(cudaEventRecord(c->ev1, c->stream));
    if ((st = copy_logits(c, last_logits ? last_logits + b * static_cast<size_t>(c->cfg.vocab_size) : nullptr)))
      return st;
    if ((st = finish_state(c))) return st;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    ms_total += ms;
    if (argmax_out) argmax_out[b] = static_cast<uint32_t>(c->h_st->argmax);
    off += n;
  }
  c->last_ms = ms_total;
  return VVLI_OK;
}

int vvli_cuda_forward_batch(vvli_ctx* c, const uint32_t* tokens, const uint64_t* positions, uint64_t B,
                            float* logits_out, uint32_t* argmax_out) {
  if (!c || (B && (!tokens || !positions))) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (c->quant) {
    g_last_error = "decode batches run on bf16 weights only (this model is block-quantised)";
    return VVLI_ERR_UNIMPLEMENTED;
  }
  if (B == 0) return VVLI_OK;
  if (B > c->max_batch) {
    g_last_error = "batch of " + std::to_string(B) + " rows exceeds the context's max_batch " + std::to_string(c->max_batch);
    return VVLI_ERR_INVALID_ARGUMENT;
  }
  for (uint64_t b = 0; b < B; ++b) {
    if (tokens[b] >= c->cfg.vocab_size) return VVLI_ERR_INVALID_TOKEN;  // src/llm.zig:704
    if (positions[b] >= c->max_seq) return VVLI_ERR_CONTEXT_FULL;     // src/llm.zig:705
  }
  if (c->group * c->d > 1024 || c->group > 8 || c->d > 128 || c->d % 4) {
    g_last_error = "decode batch: needs head_dim <= 128 (a multiple of 4) and at most 8 q heads per kv head";
    return VVLI_ERR_UNIMPLEMENTED;
  }
  CK(cudaSetDevice(c->device));
  int st;
  if ((st = ensure_batch_buffers(c))) return st;
  cudaStream_t s = c->stream;
  CK(cudaMemsetAsync(&c->st->err, 0, sizeof(int), s));
  CK(cudaEventRecord(c->ev0, s));
  const size_t V = c->V;
  for (uint64_t b0 = 0; b0 < B; b0 += kSkinnyMaxRows) {
    const int n = static_cast<int>(std::min<uint64_t>(kSkinnyMaxRows, B - b0));
    if ((st = forward_batch_chunk(c, tokens + b0, positions + b0, n, static_cast<int>(b0)))) return st;
    if (logits_out) {
      float* dst = logits_out + b0 * V;
      if (c->tp_size > 1) {
        if ((st = nccl_wait(c, nccl().AllGather(c->bt_logits, c->bt_logits_all, static_cast<size_t>(n) * c->V_l,
                                                ncclFloat32, c->comm, s), "allgather logits")))
          return st;
        for (int r = 0; r < c->tp_size; ++r) {
          const int vr = std::max(0, std::min(c->V, (r + 1) * c->V_l) - r * c->V_l);
          if (vr == 0) continue;
          CK(cudaMemcpy2DAsync(dst + static_cast<size_t>(r) * c->V_l, V * 4,
                               c->bt_logits_all + static_cast<size_t>(r) * n * c->V_l, static_cast<size_t>(c->V_l) * 4,
                               static_cast<size_t>(vr) * 4, n, cudaMemcpyDeviceToHost, s));
        }
      } else {
        CK(cudaMemcpy2DAsync(dst, V * 4, c->bt_logits, static_cast<size_t>(c->V_l) * 4, V * 4, n, cudaMemcpyDeviceToHost, s));
      }
    }
    CK(cudaMemcpyAsync(c->h_tok, c->bt_idx, n * sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (argmax_out)
      for (int b = 0; b < n; ++b) argmax_out[b0 + b] = static_cast<uint32_t>(c->h_tok[b]);
  }
  CK(cudaEventRecord(c->ev1, s));
  int err = 0;
  CK(cudaMemcpyAsync(&c->h_st->err, &c->st->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  err = c->h_st->err;
  if (err) {
    c->h_st->err = 0;
    CK(cudaMemsetAsync(&c->st->err, 0, sizeof(int), s));
    CK(cudaMemsetAsync(c->bt_counters, 0, static_cast<size_t>(kSkinnyMaxRows) * c->nkv_l * sizeof(unsigned), s));
    CK(cudaStreamSynchronize(s));
    g_last_error = "decode batch: a bounded wait gave up";
    return err;
  }
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  return VVLI_OK;
}

int vvli_cuda_generate_greedy(vvli_ctx* c, const uint32_t* prompt, uint64_t n_prompt, uint64_t max_new, int64_t eos,
                              uint32_t* out, uint64_t* out_count, vvli_generate_stats* stats) {
  if (!c || !out_count || (!out && max_new) || (!prompt && n_prompt)) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (n_prompt == 0) return VVLI_ERR_EMPTY_PROMPT;  // generateGreedy, src/generator.zig:148
  *out_count = 0;
  using clk = std::chrono::steady_clock;
  const auto t_start = clk::now();
  uint32_t first = 0;
  int st = vvli_cuda_prefill(c, prompt, n_prompt, 0, nullptr, &first);
  if (st) return st;
  const auto t_prefill = clk::now();
  // Decode (src/generator.zig:160-172): emit token k; stop after eos; else
  // forward token k at position n_prompt + k, whose argmax is token k + 1.
  // Forward k stores token k + 1 in seq_tokens[n_prompt + k + 1] on the
  // device, so steps run in chunks and the host only reads tokens back once
  // per chunk to look for eos.  Forwards past an eos are speculative: their
  // tokens are dropped.  As in the reference, the last emitted token is
  // forwarded too.
  uint64_t known = 0, scanned = 0, forwards = 0, result = 0;
  if (max_new) {
    out[0] = first;
    known = 1;
  }
  std::vector<int> buf;
  for (;;) {
    bool stop = false;
    for (; scanned < known; ++scanned)
      if (eos >= 0 && out[scanned] == static_cast<uint32_t>(eos)) {
        result = scanned + 1;
        stop = true;
        break;
      }
    if (stop) break;
    if (forwards >= max_new) {
      result = max_new;
      break;
    }
    const uint64_t pos = n_prompt + forwards;
    if (pos >= c->max_seq) return VVLI_ERR_CONTEXT_FULL;
    const uint64_t chunk = std::min<uint64_t>({max_new - forwards, c->max_seq - pos, forwards < 8 ? uint64_t{8} : uint64_t{64}});
    if ((st = run_steps(c, static_cast<int>(chunk)))) return st;
    buf.resize(chunk);
    CK(cudaMemcpyAsync(buf.data(), c->seq_tokens + pos + 1, chunk * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    if ((st = finish_state(c))) return st;
    for (uint64_t i = 0; i < chunk && forwards + 1 + i < max_new; ++i)
      out[forwards + 1 + i] = static_cast<uint32_t>(buf[i]);
    forwards += chunk;
    known = std::min<uint64_t>(max_new, forwards + 1);
  }
  *out_count = result;
  const auto t_end = clk::now();
  if (stats) {
    stats->prompt_tokens = n_prompt;
    stats->generated_tokens = result;
    stats->prefill_nanoseconds = std::chrono::duration_cast<std::chrono::nanoseconds>(t_prefill - t_start).count();
    stats->decode_nanoseconds = std::chrono::duration_cast<std::chrono::nanoseconds>(t_end - t_prefill).count();
    stats->total_nanoseconds = std::chrono::duration_cast<std::chrono::nanoseconds>(t_end - t_start).count();
  }
  return VVLI_OK;
}

int vvli_cuda_decode(vvli_ctx* c, uint64_t n_steps, uint32_t* out_tokens, float* device_ms) {
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (n_steps == 0) return VVLI_OK;
  CK(cudaSetDevice(c->device));
  const uint64_t pos0 = static_cast<uint64_t>(c->h_st->pos);  // next position, left by the last forward
  if (pos0 + n_steps > c->max_seq) return VVLI_ERR_CONTEXT_FULL;
  int st;
  CK(cudaEventRecord(c->ev0, c->stream));
  if ((st = run_steps(c, static_cast<int>(n_steps)))) return st;
  CK(cudaEventRecord(c->ev1, c->stream));
  if (out_tokens)
    CK(cudaMemcpyAsync(out_tokens, c->seq_tokens + pos0 + 1, n_steps * sizeof(int), cudaMemcpyDeviceToHost,
                       c->stream));
  if ((st = finish_state(c))) return st;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  if (device_ms) *device_ms = c->last_ms;
  return VVLI_OK;
}

// ---------------------------------------------------------------- sampling
namespace {
constexpr int kSampleRecentCap = 4096;  // recent tokens marked per copy
constexpr size_t kSampleStateBytes = 64;  // SampleState, padded; the recent tokens follow it
static_assert(sizeof(SampleState) <= kSampleStateBytes, "the recent tokens follow the step state");

int ensure_sampler(vvli_ctx* c) {
  if (c->smp_state) return VVLI_OK;
  const size_t V = static_cast<size_t>(c->V);
  int st;
  auto alloc = [&](void** p, size_t bytes) -> int {
    const cudaError_t e = cudaMalloc(p, bytes);
    return e == cudaSuccess ? VVLI_OK : cuda_fail(e, "sampler buffers");
  };
  if ((st = alloc(reinterpret_cast<void**>(&c->smp_stamp), V * 4)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_key32), V * 4)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_key64), V * 8)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_key64_sorted), V * 8)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_probs), V * 4)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_logits), V * 4)) ||
      (st = alloc(reinterpret_cast<void**>(&c->smp_state), kSampleStateBytes + kSampleRecentCap * 4)))
    return st;
  // The step state and the recent tokens sit in one block (device and
  // page-locked host), so one copy sends both.
  c->smp_recent = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(c->smp_state) + kSampleStateBytes);
  CK(cudaMallocHost(&c->h_smp_state, kSampleStateBytes + kSampleRecentCap * 4));
  if ((st = alloc(reinterpret_cast<void**>(&c->smp_done), 4))) return st;
  CK(cudaMemset(c->smp_done, 0, 4));
  CK(cudaHostAlloc(&c->h_smp_out, kSampleStateBytes, cudaHostAllocMapped));
  CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->d_smp_out), c->h_smp_out, 0));
  c->h_smp_recent = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(c->h_smp_state) + kSampleStateBytes);
  CK(cudaMemset(c->smp_stamp, 0, V * 4));
  CK(configure_sampler());
  c->smp_call = 0;
  return VVLI_OK;
}
}  // namespace

int vvli_cuda_sample(vvli_ctx* c, const vvli_sample_options* o, const float* host_logits, const uint32_t* recent,
                     uint64_t n_recent, uint64_t* rng_state, uint32_t* out_token) {
  if (!c || !o || !rng_state || !out_token || (n_recent && !recent)) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  // validateSamplingOptions (src/generator.zig:338-342)
  if (o->temperature < 0.0f || std::isnan(o->temperature) || o->top_p <= 0.0f || o->top_p > 1.0f ||
      std::isnan(o->top_p) || o->repeat_penalty < 1.0f || std::isnan(o->repeat_penalty))
    return VVLI_ERR_INVALID_SAMPLING;
  CK(cudaSetDevice(c->device));
  int st;
  if ((st = ensure_sampler(c))) return st;
  const float* logits = c->logits;
  if (host_logits) {
    CK(cudaMemcpyAsync(c->smp_logits, host_logits, static_cast<size_t>(c->V) * 4, cudaMemcpyHostToDevice, c->stream));
    logits = c->smp_logits;
  } else if (c->tp_size > 1) {
    if ((st = tp_collective(c, c->logits, c->logits_full, c->V_l, true, c->stream, "allgather logits"))) return st;
    logits = c->logits_full;
  }
  const uint64_t limit = o->top_k == 0 ? c->V : std::min<uint64_t>(o->top_k, c->V);
  const int nblk = (c->V + 1023) / 1024;
  int nlists = 1;
  while (nlists < nblk) nlists <<= 1;
  const bool fast = o->temperature > 0.0f && limit <= static_cast<uint64_t>(kSampleFastK) &&
                    nlists * 64 <= kSampleFastMaxCand;
  // buildRepeatCounts (src/generator.zig:344-360): the last repeat_last_n tokens.
  const bool penalise = o->repeat_penalty > 1.0f && o->repeat_last_n > 0 && n_recent > 0;
  const uint64_t n_use = penalise ? std::min<uint64_t>(n_recent, o->repeat_last_n) : 0;
  const uint32_t* src = recent + (n_recent - n_use);
  // The top-k path reads the recent tokens itself (in its launch's parameters,
  // or one copy when there are many); the other paths read per-token stamps
  // marked here.
  const bool fold = fast && n_use <= static_cast<uint64_t>(kSampleRecentCap);
  if (!fold && ++c->smp_call == 0) {  // the stamps wrapped: start over
    CK(cudaMemsetAsync(c->smp_stamp, 0, static_cast<size_t>(c->V) * 4, c->stream));
    c->smp_call = 1;
  }
  if (!fold && n_use > 0) {
    for (uint64_t done = 0; done < n_use; done += kSampleRecentCap) {
      const int n = static_cast<int>(std::min<uint64_t>(kSampleRecentCap, n_use - done));
      std::memcpy(c->h_smp_recent, src + done, static_cast<size_t>(n) * 4);  // page-locked: an async copy
      CK(cudaMemcpyAsync(c->smp_recent, c->h_smp_recent, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice,
                         c->stream));
      CK(launch_sample_mark(c->smp_recent, n, c->smp_stamp, c->smp_call, c->V, c->stream));
      if (done + kSampleRecentCap < n_use) CK(cudaStreamSynchronize(c->stream));  // smp_recent is reused
    }
  }
  SampleParams p{};
  p.logits = logits;
  p.V = c->V;
  p.stamp = c->smp_stamp;
  p.call = c->smp_call;
  p.temperature = o->temperature;
  p.top_p = o->top_p;
  p.repeat_penalty = o->repeat_penalty;
  p.top_k = o->top_k;
  p.key32 = c->smp_key32;
  p.key64 = c->smp_key64;
  p.key64_sorted = c->smp_key64_sorted;
  p.probs = c->smp_probs;
  p.st = c->smp_state;
  if (fast) {
    // One launch: the state and up to kSampleArgRecent recent tokens travel in
    // its parameters, the result comes back through mapped host memory.
    FastSampleArgs a{};
    a.p = p;
    std::memcpy(a.rng, rng_state, sizeof(a.rng));
    a.k = static_cast<int>(limit);
    a.nlists = nlists;
    a.cand = c->smp_key64;  // V keys >= ceil(V / 1024) * 64
    a.nfin = c->smp_key32;
    a.done = c->smp_done;
    a.out = c->d_smp_out;
    if (fold) {
      a.p.stamp = nullptr;
      a.p.n_recent = static_cast<int>(n_use);
      if (n_use <= static_cast<uint64_t>(kSampleArgRecent)) {
        a.recent_in_args = 1;
        if (n_use) std::memcpy(a.recent, src, n_use * 4);
      } else {
        std::memcpy(c->h_smp_recent, src, n_use * 4);
        CK(cudaMemcpyAsync(c->smp_recent, c->h_smp_recent, n_use * 4, cudaMemcpyHostToDevice, c->stream));
        a.p.recent = c->smp_recent;
      }
    }
    SampleState* h = c->h_smp_out;
    h->token = -1;
    CK(launch_sample_fast(a, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    const int tok = reinterpret_cast<volatile SampleState*>(h)->token;
    if (tok < 0 || tok >= static_cast<int>(c->V)) {
      g_last_error = "sampler produced no token";
      return VVLI_ERR_CUDA;
    }
    std::memcpy(rng_state, h->rng, sizeof(h->rng));
    *out_token = static_cast<uint32_t>(tok);
    return VVLI_OK;
  }
  SampleState* h = c->h_smp_state;
  std::memcpy(h->rng, rng_state, sizeof(h->rng));
  h->token = -1;
  h->path = 0;
  h->k = 0;
  h->n_sort = 0;
  CK(cudaMemcpyAsync(c->smp_state, h, kSampleStateBytes, cudaMemcpyHostToDevice, c->stream));
  CK(launch_sample(p, c->stream));
  CK(cudaMemcpyAsync(h, c->smp_state, sizeof(SampleState), cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  if (h->path == 1) {
    CK(launch_sample_long(p, h->n_sort, c->stream));
    CK(cudaMemcpyAsync(h, c->smp_state, sizeof(SampleState), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
  }
  if (h->token < 0 || h->token >= static_cast<int>(c->V)) {
    g_last_error = "sampler produced no token";
    return VVLI_ERR_CUDA;
  }
  std::memcpy(rng_state, h->rng, sizeof(h->rng));
  *out_token = static_cast<uint32_t>(h->token);
  return VVLI_OK;
}

int vvli_cuda_time_kernel(vvli_ctx* c, int kernel, int reps, float* avg_ms, double* bytes) {
  if (!c || !avg_ms || !bytes || reps <= 0 || kernel < 0 || kernel > 4) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->loaded) return VVLI_ERR_NOT_LOADED;
  if (c->quant) {
    g_last_error = "the standalone decode kernels stream bf16 weights only (this model is block-quantised)";
    return VVLI_ERR_UNIMPLEMENTED;
  }
  CK(cudaSetDevice(c->device));
  const uint16_t* W = c->w;
  const double h = c->h;
  auto params = [&](int l, int& epi, double& b) {
    const DevLayer& D = c->lay[l % c->L];
    GemvParams p{};
    p.eps = c->cfg.rms_norm_eps;
    p.st = c->st;
    epi = EPI_PLAIN;
    switch (kernel) {
      case 0:
        p.W = W + D.w_qkv, p.N = c->q_rows + 2 * c->kv_rows, p.K = c->h, p.x = c->x, p.norm_w = W + D.in_norm;
        p.bias = D.b_qkv == UINT64_MAX ? nullptr : W + D.b_qkv, p.y = c->qkv;
        b = 2.0 * p.N * h + 4 * h + 2 * h + 4.0 * p.N + (p.bias ? 2.0 * p.N : 0);
        break;
      case 1:
        p.W = W + D.w_o, p.N = c->h, p.K = c->q_rows, p.x = c->attn, p.residual = c->x, p.y = c->x;
        b = 2.0 * p.N * p.K + 4.0 * p.K + 8.0 * p.N;
        break;
      case 2:
        p.W = W + D.w_gu, p.N = c->I_l, p.K = c->h, p.pair_offset = c->I_l, p.x = c->x, p.norm_w = W + D.post;
        p.y = c->ff, epi = EPI_SILU_MUL;
        b = 2.0 * 2 * p.N * h + 4 * h + 2 * h + 4.0 * p.N;
        break;
      case 3:
        p.W = W + D.w_down, p.N = c->h, p.K = c->I_l, p.x = c->ff, p.residual = c->x, p.y = c->x;
        b = 2.0 * p.N * p.K + 4.0 * p.K + 8.0 * p.N;
        break;
      default:
        p.W = W + c->off_lm, p.N = c->V_lr, p.K = c->h, p.x = c->x, p.norm_w = W + c->off_final, p.y = c->logits;
        p.part_val = c->amax_val, p.part_idx = c->amax_idx, p.counter = c->counters + c->nkv_l, p.row_base = c->v0;
        p.finalize = 0, p.local_best = c->best, p.st = c->st, p.seq_tokens = c->seq_tokens;
        epi = EPI_ARGMAX;
        b = 2.0 * p.N * h + 4 * h + 2 * h + 4.0 * p.N;
        break;
    }
    return p;
  };
  int epi = 0;
  double b = 0;
  for (int i = 0; i < 3; ++i) {  // warm-up
    GemvParams p = params(i, epi, b);
    CK(launch_gemv(epi, p, c->sm_count, c->stream, false));
  }
  CK(cudaEventRecord(c->ev0, c->stream));
  for (int i = 0; i < reps; ++i) {
    GemvParams p = params(i, epi, b);
    CK(launch_gemv(epi, p, c->sm_count, c->stream, false));
  }
  CK(cudaEventRecord(c->ev1, c->stream));
  CK(cudaEventSynchronize(c->ev1));
  float ms = 0;
  CK(cudaEventElapsedTime(&ms, c->ev0, c->ev1));
  *avg_ms = ms / reps;
  *bytes = b;
  return VVLI_OK;
}

int vvli_cuda_query(vvli_ctx* c, const char* key, double* out) {
  if (!c || !key || !out) return VVLI_ERR_INVALID_ARGUMENT;
  const std::string k(key);
  if (k == "megakernel") *out = c->use_mega ? 1 : 0;
  else if (k == "sm_count") *out = c->sm_count;
  else if (k == "graph") *out = c->graph ? 1 : 0;
  else if (k == "mega_ring_bytes") *out = c->use_mega ? static_cast<double>(c->mp.nst) * c->mp.slot_bytes : 0;
  else if (k == "mega_phases") *out = c->use_mega ? c->mp.nphases : 0;
  else if (k == "kernels_per_step")
    *out = c->use_mega ? 1 : 1 + 5.0 * c->L + 1 + (c->tp_size > 1 ? 1 : 0);
  else if (k == "weight_bytes") *out = static_cast<double>(c->weight_elems) * 2;
  else if (k == "tc_prefill") *out = c->tc_prefill ? 1 : 0;
  else if (k == "quantized") *out = c->quant ? 1 : 0;
  else if (k == "weight_stream_bytes") *out = static_cast<double>(weight_stream_bytes(c));
  else return VVLI_ERR_INVALID_ARGUMENT;
  return VVLI_OK;
}

int vvli_cuda_trace(vvli_ctx* c, uint64_t* out, uint64_t cap, uint64_t* count) {
  if (!c || !count) return VVLI_ERR_INVALID_ARGUMENT;
  *count = c->trace ? c->h_phases.size() * c->sm_count * 6 : 0;
  if (c->trace && out && cap >= *count) {
    CK(cudaSetDevice(c->device));
    CK(cudaMemcpy(out, c->trace, *count * sizeof(uint64_t), cudaMemcpyDeviceToHost));
  }
  return VVLI_OK;
}

int vvli_cuda_attention_selftest(int device, int d, int group, int tokens, int pos0, uint64_t seed,
                                 float* max_rel_err) {
  if (!max_rel_err || tokens <= 0 || pos0 < 0 || !prefill_attention_tc_supported(d, group))
    return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(device));
  CK(attention_tc_selftest(d, group, tokens, pos0, seed, max_rel_err));
  return VVLI_OK;
}

int vvli_cuda_gemm_selftest(int device, int kernel, int M, int N, int K, int two_a, uint64_t seed,
                            float* max_rel_err) {
  if (!max_rel_err || M <= 0 || N <= 0 || K <= 0 || K % 8 || N % 2 || kernel < 0 || kernel > 3 ||
      (kernel == 1 && M > kSkinnyMaxRows))
    return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(device));
  cudaError_t e = gemm_tc_selftest(M, N, K, two_a, kernel, seed, max_rel_err);
  if (e == cudaErrorTimeout) {
    g_last_error = "tensor-core GEMM: a bounded wait gave up";
    return VVLI_ERR_TIMEOUT;
  }
  CK(e);
  return VVLI_OK;
}

int vvli_cuda_set_debug(vvli_ctx* c, int enabled) {
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  c->debug = enabled != 0;
  return VVLI_OK;
}

int vvli_cuda_debug_hidden(vvli_ctx* c, int layer, float* out) {
  if (!c || !out || layer < 0 || layer >= c->L) return VVLI_ERR_INVALID_ARGUMENT;
  if (!c->debug) return VVLI_ERR_INVALID_ARGUMENT;
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpy(out, c->hidden + static_cast<size_t>(layer) * c->h, c->h * 4, cudaMemcpyDeviceToHost));
  return VVLI_OK;
}

int vvli_cuda_last_forward_ms(vvli_ctx* c, float* out_ms) {
  if (!c || !out_ms) return VVLI_ERR_INVALID_ARGUMENT;
  *out_ms = c->last_ms;
  return VVLI_OK;
}

int vvli_cuda_destroy(vvli_ctx* c) {
  if (!c) return VVLI_ERR_INVALID_ARGUMENT;
  free_ctx(c);
  return VVLI_OK;
}

}  // extern "C"
