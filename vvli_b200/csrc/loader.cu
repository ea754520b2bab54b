// loader.cu - weights straight from a safetensors or GGUF file into this rank's device layout.
//
// loadSafetensorsIntoOwnedModel (src/llm.zig:923-1006) copies every tensor of
// model.safetensors into one host blob; here each rank reads only the pieces
// its shard plan names, from the memory-mapped file to the device:
//   * the header is the JSON object at the start of the file (8-byte little
//     endian length, then {"name": {"dtype", "shape", "data_offsets"}});
//   * tensors are checked like copyTensorIntoWeight (:1149-1183): the name
//     must exist, dtype BF16 or F32, the shape's element count and the byte
//     range must match;
//   * BF16 rows are copied with one strided copy per piece; F32 rows are copied
//     to a device staging buffer and rounded with the reference's f32ToBf16
//     (round to nearest even, no NaN special case) by a kernel;
//   * the mapping is page-locked read-only (cudaHostRegister) when the system
//     allows it, so the copies are DMA from the page cache; otherwise they go
//     through the driver's pageable path.
//
// loadGgufIntoOwnedModel (src/llm.zig:1008-1065) does the same for a GGUF
// file (src/gguf.zig): the binary header and tensor table are parsed here,
// tensors are named token_embd / blk.N.* / output_norm / output, and may be
// F32, F16 or BF16 (copyGgufTensorIntoWeight, :1081-1138); F16 values are
// widened exactly and rounded with f32ToBf16 on the device.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_fp16.h>

#include <algorithm>
#include <functional>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/vvli_cuda.h"
#include "common.cuh"
#include "kernels.h"
#include "loader.h"

namespace vvli {

namespace {

// ---------------------------------------------------------------- JSON (the header's subset)
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(Json* out) {
    if (!value(out)) return false;
    ws();
    return p_ == end_;
  }

 private:
  const char* p_;
  const char* end_;
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if (static_cast<size_t>(end_ - p_) < n || memcmp(p_, s, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool string(std::string* out) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    out->clear();
    while (p_ < end_ && *p_ != '"') {
      char ch = *p_++;
      if (ch == '\\') {
        if (p_ >= end_) return false;
        const char e = *p_++;
        switch (e) {
          case '"': ch = '"'; break;
          case '\\': ch = '\\'; break;
          case '/': ch = '/'; break;
          case 'b': ch = '\b'; break;
          case 'f': ch = '\f'; break;
          case 'n': ch = '\n'; break;
          case 'r': ch = '\r'; break;
          case 't': ch = '\t'; break;
          case 'u': {  // tensor names are ASCII; other code points are kept as '?'
            if (end_ - p_ < 4) return false;
            p_ += 4;
            ch = '?';
            break;
          }
          default: return false;
        }
      }
      out->push_back(ch);
    }
    if (p_ >= end_) return false;
    ++p_;
    return true;
  }
  bool number(double* out) {
    const char* s = p_;
    while (p_ < end_ && (isdigit(static_cast<unsigned char>(*p_)) || *p_ == '-' || *p_ == '+' || *p_ == '.' ||
                         *p_ == 'e' || *p_ == 'E'))
      ++p_;
    if (p_ == s) return false;
    *out = strtod(std::string(s, p_).c_str(), nullptr);
    return true;
  }
  bool value(Json* v) {
    ws();
    if (p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->kind = Json::Obj;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        if (!value(&v->obj[key])) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      v->kind = Json::Arr;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        v->arr.emplace_back();
        if (!value(&v->arr.back())) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      v->kind = Json::Str;
      return string(&v->str);
    }
    if (lit("true")) {
      v->kind = Json::Bool, v->b = true;
      return true;
    }
    if (lit("false")) {
      v->kind = Json::Bool, v->b = false;
      return true;
    }
    if (lit("null")) {
      v->kind = Json::Null;
      return true;
    }
    v->kind = Json::Num;
    return number(&v->num);
  }
};

// The reference's tensor names (src/llm.zig:938-1005) by blob order id:
// 0 embedding, 1 + 12 l + {0 input norm, 1 q, 2 q bias, 3 k, 4 k bias, 5 v,
// 6 v bias, 7 o, 8 post norm, 9 gate, 10 up, 11 down}, then final norm, LM head.
std::string tensor_name(uint64_t id, int layers) {
  if (id == 0) return "model.embed_tokens.weight";
  if (id == 1 + 12ull * layers) return "model.norm.weight";
  if (id == 2 + 12ull * layers) return "lm_head.weight";
  const uint64_t l = (id - 1) / 12, k = (id - 1) % 12;
  static const char* kSuffix[12] = {"input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.q_proj.bias",
                                    "self_attn.k_proj.weight", "self_attn.k_proj.bias", "self_attn.v_proj.weight",
                                    "self_attn.v_proj.bias", "self_attn.o_proj.weight",
                                    "post_attention_layernorm.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                                    "mlp.down_proj.weight"};
  return "model.layers." + std::to_string(l) + "." + kSuffix[k];
}

// f32ToBf16 (src/llm.zig:795-803) of every element.
__global__ void f32_to_bf16_kernel(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = f32_to_bf16(src[i]);
}

// f32ToBf16(f16ToF32(bits)) of every element (src/llm.zig:795-803, 1119-1126):
// the half -> float widening is exact, the rounding is the reference's.
__global__ void f16_to_bf16_kernel(const uint16_t* src, uint16_t* dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = f32_to_bf16(__half2float(__ushort_as_half(src[i])));
}

struct Mapping {
  int fd = -1;
  void* base = MAP_FAILED;
  size_t size = 0;
  bool registered = false;
  ~Mapping() {
    if (registered) cudaHostUnregister(base);
    if (base != MAP_FAILED) munmap(base, size);
    if (fd >= 0) close(fd);
  }
  int open_file(const char* path, std::string* why) {
    fd = open(path, O_RDONLY);
    if (fd < 0) {
      *why = std::string("cannot open ") + path;
      return VVLI_ERR_INVALID_ARGUMENT;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
      *why = std::string("cannot stat ") + path;
      return VVLI_ERR_INVALID_ARGUMENT;
    }
    size = static_cast<size_t>(st.st_size);
    if (size == 0) return VVLI_OK;  // nothing to map; the format checks reject it
    base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (base == MAP_FAILED) {
      *why = std::string("cannot map ") + path;
      return VVLI_ERR_INVALID_ARGUMENT;
    }
    return VVLI_OK;
  }
  const uint8_t* bytes() const { return base == MAP_FAILED ? nullptr : static_cast<const uint8_t*>(base); }
  // DMA straight from the page cache when the mapping can be page-locked.
  void lock() {
    if (base == MAP_FAILED) return;
    registered = cudaHostRegister(base, size, cudaHostRegisterReadOnly) == cudaSuccess;
    if (!registered) cudaGetLastError();
  }
};

enum SrcType { kSrcBF16, kSrcF32, kSrcF16, kSrcQ8_0, kSrcQ4_0 };

// A checked source tensor: `count` elements of `type` at `data`.
struct SrcTensor {
  int type;
  uint64_t count;
  const uint8_t* data;
};

inline uint64_t src_elem_bytes(int type) { return type == kSrcF32 ? 4 : 2; }
// Bytes of a GGML block of 32 weights: an fp16 scale and 32 int8 (Q8_0) or 16
// bytes of nibbles (Q4_0).
inline uint64_t src_block_bytes(int type) { return type == kSrcQ8_0 ? 34 : 18; }
inline bool src_quantised(int type) { return type == kSrcQ8_0 || type == kSrcQ4_0; }

// GGML blocks of `rows` rows (nb blocks each, contiguous) -> the device row
// layout of kernels.h: the quants of every block of the row, then its scales.
__global__ void repack_blocks_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t rows,
                                     int nb, int q8, int row_bytes) {
  const int qb = q8 ? 32 : 16, bb = q8 ? 34 : 18;
  const uint64_t total = rows * static_cast<uint64_t>(nb);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / nb;
    const int b = static_cast<int>(i % nb);
    const uint8_t* blk = src + i * bb;
    uint8_t* row = dst + r * row_bytes;
    row[nb * qb + 2 * b] = blk[0];  // fp16 scale, little endian
    row[nb * qb + 2 * b + 1] = blk[1];
    for (int j = 0; j < qb; ++j) row[b * qb + j] = blk[2 + j];
  }
}

// Finds and checks the tensor of blob id `id`; returns a vvli_status.
using Lookup = std::function<int(uint64_t id, uint64_t expect_elems, SrcTensor*, std::string*)>;

// Copies every piece: BF16 rows with one strided copy, F32 / F16 rows through
// a device staging buffer and a rounding kernel.
int copy_pieces(const std::vector<LoadPiece>& pieces, const Lookup& lookup, uint16_t* w, cudaStream_t s,
                std::string* why, std::vector<int>* piece_fmt = nullptr) {
  void* stage = nullptr;
  constexpr size_t kStageBytes = 64ull << 20;
  int status = VVLI_OK;
  if (piece_fmt) piece_fmt->assign(pieces.size(), kFmtBF16);
  for (size_t pi = 0; pi < pieces.size(); ++pi) {
    const LoadPiece& p = pieces[pi];
    SrcTensor t{};
    if ((status = lookup(p.tensor_id, p.tensor_elems, &t, why)) != VVLI_OK) break;
    if (src_quantised(t.type)) {
      // Whole rows of blocks (the plan of a single rank): copy the blocks of
      // each staging chunk of rows, then repack them into the device rows.
      const int nb = static_cast<int>(p.cols / 32);
      const uint64_t row_src = static_cast<uint64_t>(nb) * src_block_bytes(t.type);
      const int fmt = t.type == kSrcQ8_0 ? kFmtQ8 : kFmtQ4;
      const int rb = row_bytes_of(fmt, static_cast<int>(p.cols));
      if (p.cols % 32 || p.col0 || p.src_ld != p.cols || p.rows == 1) {
        *why = "tensor " + std::to_string(p.tensor_id) + ": block-quantised tensors need whole rows of 32-weight "
               "blocks on one rank (a norm or bias must be F32, F16 or BF16)";
        status = VVLI_ERR_UNSUPPORTED_DTYPE;
        break;
      }
      if (!stage && cudaMalloc(&stage, kStageBytes) != cudaSuccess) {
        *why = "staging buffer for quantised tensors";
        status = VVLI_ERR_OOM;
        break;
      }
      uint8_t* dst = reinterpret_cast<uint8_t*>(w + p.group_base) + p.group_row * static_cast<uint64_t>(rb);
      const uint8_t* src = t.data + p.row0 * row_src;
      const uint64_t rows_per = std::max<uint64_t>(1, kStageBytes / row_src);
      cudaError_t e = cudaSuccess;
      for (uint64_t r = 0; r < p.rows && e == cudaSuccess; r += rows_per) {
        const uint64_t n = std::min(rows_per, p.rows - r);
        e = cudaMemcpyAsync(stage, src + r * row_src, n * row_src, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
          const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((n * nb + 255) / 256, 4096));
          repack_blocks_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(stage), dst + r * rb, n, nb,
                                                      fmt == kFmtQ8, rb);
          e = cudaGetLastError();
          if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the staging buffer is reused
        }
      }
      if (e != cudaSuccess) {
        *why = std::string("copying tensor ") + std::to_string(p.tensor_id) + ": " + cudaGetErrorString(e);
        status = e == cudaErrorMemoryAllocation ? VVLI_ERR_OOM : VVLI_ERR_CUDA;
        break;
      }
      if (piece_fmt) (*piece_fmt)[pi] = fmt;
      continue;
    }
    const uint64_t esz = src_elem_bytes(t.type);
    const uint8_t* src = t.data + (p.row0 * p.src_ld + p.col0) * esz;
    uint16_t* dst = w + p.dst;
    cudaError_t e;
    if (t.type == kSrcBF16) {
      e = cudaMemcpy2DAsync(dst, p.cols * 2, src, p.src_ld * 2, p.cols * 2, p.rows, cudaMemcpyHostToDevice, s);
    } else {
      if (!stage && (e = cudaMalloc(&stage, kStageBytes)) != cudaSuccess) {
        *why = "staging buffer for F32 / F16 tensors";
        status = VVLI_ERR_OOM;
        break;
      }
      const uint64_t rows_per = std::max<uint64_t>(1, kStageBytes / (p.cols * esz));
      e = cudaSuccess;
      for (uint64_t r = 0; r < p.rows && e == cudaSuccess; r += rows_per) {
        const uint64_t n = std::min(rows_per, p.rows - r);
        e = cudaMemcpy2DAsync(stage, p.cols * esz, src + r * p.src_ld * esz, p.src_ld * esz, p.cols * esz, n,
                              cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
          const size_t total = n * p.cols;
          const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 4096));
          if (t.type == kSrcF32)
            f32_to_bf16_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(stage), dst + r * p.cols, total);
          else
            f16_to_bf16_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint16_t*>(stage), dst + r * p.cols, total);
          e = cudaGetLastError();
          if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the staging buffer is reused
        }
      }
    }
    if (e != cudaSuccess) {
      *why = std::string("copying tensor ") + std::to_string(p.tensor_id) + ": " + cudaGetErrorString(e);
      status = VVLI_ERR_CUDA;
      break;
    }
  }
  const cudaError_t e = cudaStreamSynchronize(s);  // before the mapping goes away
  if (stage) cudaFree(stage);
  if (status == VVLI_OK && e != cudaSuccess) {
    *why = std::string("loading weights: ") + cudaGetErrorString(e);
    status = VVLI_ERR_CUDA;
  }
  return status;
}

// ---------------------------------------------------------------- GGUF (src/gguf.zig)
// The GGUF names of the reference's tensors (loadGgufIntoOwnedModel,
// src/llm.zig:1008-1065) by blob order id; GGUF models carry no q/k/v biases.
std::string gguf_tensor_name(uint64_t id, int layers) {
  if (id == 0) return "token_embd.weight";
  if (id == 1 + 12ull * layers) return "output_norm.weight";
  if (id == 2 + 12ull * layers) return "output.weight";
  const uint64_t l = (id - 1) / 12, k = (id - 1) % 12;
  static const char* kSuffix[12] = {"attn_norm.weight", "attn_q.weight", "attn_q.bias", "attn_k.weight",
                                    "attn_k.bias",      "attn_v.weight", "attn_v.bias", "attn_output.weight",
                                    "ffn_norm.weight",  "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
  return "blk." + std::to_string(l) + "." + kSuffix[k];
}

struct GgufTensor {
  uint32_t type;
  uint64_t count;   // 0 when the element count overflows
  uint64_t offset;  // from the start of the data section
};

// gguf.parse (src/gguf.zig:234-287): header, metadata (only general.alignment
// is kept), tensor table; little-endian reads bounded by the file size.
class GgufReader {
 public:
  GgufReader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  size_t index = 0;
  int status = VVLI_OK;

  bool bytes(size_t len, const uint8_t** out) {
    if (len > n_ - index) return fail(VVLI_ERR_INVALID_GGUF);
    *out = p_ + index;
    index += len;
    return true;
  }
  template <typename T>
  bool num(T* out) {
    const uint8_t* b;
    if (!bytes(sizeof(T), &b)) return false;
    memcpy(out, b, sizeof(T));  // little endian on every CUDA host
    return true;
  }
  bool str(std::string* out) {
    uint64_t len;
    const uint8_t* b;
    if (!num(&len) || !bytes(len, &b)) return false;
    out->assign(reinterpret_cast<const char*>(b), len);
    return true;
  }
  bool skip_str() {
    uint64_t len;
    const uint8_t* b;
    return num(&len) && bytes(len, &b);
  }
  // gguf.MetadataType (src/gguf.zig:16-30); other values are UnsupportedMetadataType.
  bool meta_type(uint32_t* t) {
    if (!num(t)) return false;
    if (*t > 12) return fail(VVLI_ERR_UNSUPPORTED_METADATA_TYPE);
    return true;
  }
  // Reader.skipMetadataValue (src/gguf.zig:340-355); arrays may nest.
  bool skip_value(uint32_t t, int depth = 0) {
    const uint8_t* b;
    switch (t) {
      case 0: case 1: case 7: return bytes(1, &b);
      case 2: case 3: return bytes(2, &b);
      case 4: case 5: case 6: return bytes(4, &b);
      case 10: case 11: case 12: return bytes(8, &b);
      case 8: return skip_str();
      default: {  // array
        uint32_t it;
        uint64_t len;
        if (depth > 64) return fail(VVLI_ERR_INVALID_GGUF);
        if (!meta_type(&it) || !num(&len)) return false;
        const size_t fixed = it == 8 || it == 9 ? 0 : (it <= 1 || it == 7 ? 1 : it <= 3 ? 2 : it <= 6 ? 4 : 8);
        if (fixed) {  // one bounds check for a whole array of numbers
          if (len > (n_ - index) / fixed) return fail(VVLI_ERR_INVALID_GGUF);
          index += len * fixed;
          return true;
        }
        for (uint64_t i = 0; i < len; ++i)
          if (!skip_value(it, depth + 1)) return false;
        return true;
      }
    }
  }
  // File.usizeValue (src/gguf.zig:149-162) of a value of type t; *ok = false
  // for a type it does not accept (or a negative integer).
  bool usize_value(uint32_t t, uint64_t* out, bool* ok) {
    *ok = true;
    switch (t) {
      case 0: { uint8_t v; if (!num(&v)) return false; *out = v; return true; }
      case 2: { uint16_t v; if (!num(&v)) return false; *out = v; return true; }
      case 4: { uint32_t v; if (!num(&v)) return false; *out = v; return true; }
      case 10: { uint64_t v; if (!num(&v)) return false; *out = v; return true; }
      case 1: { int8_t v; if (!num(&v)) return false; *ok = v >= 0; *out = static_cast<uint64_t>(v); return true; }
      case 3: { int16_t v; if (!num(&v)) return false; *ok = v >= 0; *out = static_cast<uint64_t>(v); return true; }
      case 5: { int32_t v; if (!num(&v)) return false; *ok = v >= 0; *out = static_cast<uint64_t>(v); return true; }
      case 11: { int64_t v; if (!num(&v)) return false; *ok = v >= 0; *out = static_cast<uint64_t>(v); return true; }
      default: *ok = false; return skip_value(t);
    }
  }

 private:
  const uint8_t* p_;
  size_t n_;
  bool fail(int st) {
    if (status == VVLI_OK) status = st;
    return false;
  }
};

// gguf.TensorType (src/gguf.zig:32-72): the values the reference accepts.
bool gguf_known_tensor_type(uint32_t t) {
  return t <= 3 || (t >= 6 && t <= 30) || t == 34 || t == 35 || t == 39;
}

int parse_gguf(const uint8_t* bytes, size_t n, std::map<std::string, GgufTensor>* tensors, uint64_t* data_start,
               std::string* why) {
  GgufReader r(bytes, n);
  const uint8_t* magic;
  uint32_t version;
  uint64_t tensor_count, metadata_count;
  auto bad = [&](const char* what) {
    *why = what;
    return r.status != VVLI_OK ? r.status : VVLI_ERR_INVALID_GGUF;
  };
  if (!r.bytes(4, &magic) || memcmp(magic, "GGUF", 4) != 0) return bad("not a GGUF file");
  if (!r.num(&version)) return bad("GGUF header is cut short");
  if (version < 2 || version > 3) {
    *why = "GGUF version " + std::to_string(version) + " (2 or 3 only)";
    return VVLI_ERR_UNSUPPORTED_GGUF_VERSION;
  }
  if (!r.num(&tensor_count) || !r.num(&metadata_count)) return bad("GGUF header is cut short");
  uint64_t alignment = 32;  // gguf.default_alignment
  bool have_alignment = false;
  for (uint64_t i = 0; i < metadata_count; ++i) {
    std::string key;
    uint32_t t;
    if (!r.str(&key) || !r.meta_type(&t)) return bad("malformed GGUF metadata");
    if (key == "general.alignment" && !have_alignment) {  // the first entry of a key wins
      have_alignment = true;
      uint64_t v;
      bool ok;
      if (!r.usize_value(t, &v, &ok)) return bad("malformed GGUF metadata");
      if (ok) alignment = v;
    } else if (!r.skip_value(t)) {
      return bad("malformed GGUF metadata");
    }
  }
  for (uint64_t i = 0; i < tensor_count; ++i) {
    std::string name;
    uint32_t dims;
    if (!r.str(&name) || !r.num(&dims)) return bad("malformed GGUF tensor table");
    if (dims == 0 || dims > 8) return bad("GGUF tensor with 0 or more than 8 dimensions");
    uint64_t count = 1;
    bool overflow = false;
    for (uint32_t d = 0; d < dims; ++d) {
      uint64_t v;
      if (!r.num(&v)) return bad("malformed GGUF tensor table");
      overflow |= __builtin_mul_overflow(count, v, &count);
    }
    GgufTensor t{};
    if (!r.num(&t.type)) return bad("malformed GGUF tensor table");
    if (!gguf_known_tensor_type(t.type)) {  // readEnum(TensorType) fails this way
      *why = name + " has an unknown GGUF tensor type " + std::to_string(t.type);
      return VVLI_ERR_UNSUPPORTED_METADATA_TYPE;
    }
    if (!r.num(&t.offset)) return bad("malformed GGUF tensor table");
    t.count = overflow ? 0 : count;
    tensors->emplace(name, t);  // File.tensor returns the first of a name
  }
  if (alignment == 0) return bad("general.alignment is 0");
  const uint64_t start = (r.index + alignment - 1) / alignment * alignment;
  if (start < r.index || start > n) return bad("GGUF data section starts past the end of the file");
  *data_start = start;
  return VVLI_OK;
}

}  // namespace

int upload_safetensors(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w,
                       cudaStream_t s, std::string* why) {
  Mapping m;
  int st = m.open_file(path, why);
  if (st != VVLI_OK) return st;
  if (m.size < 8) {
    *why = std::string("not a safetensors file: ") + path;
    return VVLI_ERR_INVALID_WEIGHT;
  }
  const uint8_t* bytes = m.bytes();
  uint64_t header_len = 0;
  memcpy(&header_len, bytes, 8);  // little endian on every CUDA host
  if (header_len > m.size - 8) {
    *why = "safetensors header runs past the end of the file";
    return VVLI_ERR_INVALID_WEIGHT;
  }
  Json header;
  if (!Parser(reinterpret_cast<const char*>(bytes + 8), header_len).parse(&header) || header.kind != Json::Obj) {
    *why = "safetensors header is not a JSON object";
    return VVLI_ERR_INVALID_WEIGHT;
  }
  const uint8_t* data = bytes + 8 + header_len;
  const size_t data_len = m.size - 8 - header_len;
  m.lock();
  // copyTensorIntoWeight (src/llm.zig:1149-1183): name, dtype BF16 or F32,
  // element count and byte range.
  auto lookup = [&](uint64_t id, uint64_t expect, SrcTensor* t, std::string* err) -> int {
    const std::string name = tensor_name(id, layers);
    auto it = header.obj.find(name);
    if (it == header.obj.end()) {
      *err = "missing tensor " + name;
      return VVLI_ERR_MISSING_TENSOR;
    }
    const Json& meta = it->second;
    auto dt = meta.obj.find("dtype");
    auto sh = meta.obj.find("shape");
    auto off = meta.obj.find("data_offsets");
    if (meta.kind != Json::Obj || dt == meta.obj.end() || sh == meta.obj.end() || off == meta.obj.end() ||
        sh->second.kind != Json::Arr || off->second.kind != Json::Arr || off->second.arr.size() != 2) {
      *err = "malformed entry for " + name;
      return VVLI_ERR_INVALID_WEIGHT;
    }
    const bool bf16 = dt->second.str == "BF16", f32 = dt->second.str == "F32";
    if (!bf16 && !f32) {
      *err = name + " has dtype " + dt->second.str + " (BF16 or F32 only)";
      return VVLI_ERR_UNSUPPORTED_DTYPE;
    }
    uint64_t count = 1;
    for (const Json& d : sh->second.arr) count *= static_cast<uint64_t>(d.num);
    const uint64_t start = static_cast<uint64_t>(off->second.arr[0].num);
    const uint64_t end = static_cast<uint64_t>(off->second.arr[1].num);
    const uint64_t esz = bf16 ? 2 : 4;
    if (count != expect || end < start || end > data_len || end - start != count * esz) {
      *err = "shape or byte range of " + name + " does not match the model config";
      return VVLI_ERR_INVALID_WEIGHT;
    }
    *t = SrcTensor{bf16 ? kSrcBF16 : kSrcF32, count, data + start};
    return VVLI_OK;
  };
  return copy_pieces(pieces, lookup, w, s, why);
}

int upload_gguf(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w, cudaStream_t s,
                std::string* why, std::vector<int>* piece_fmt) {
  Mapping m;
  int st = m.open_file(path, why);
  if (st != VVLI_OK) return st;
  std::map<std::string, GgufTensor> tensors;
  uint64_t data_start = 0;
  if ((st = parse_gguf(m.bytes(), m.size, &tensors, &data_start, why)) != VVLI_OK) return st;
  m.lock();
  // copyGgufTensorIntoWeight (src/llm.zig:1081-1138): name, native float
  // type (F32, F16, BF16), element count, byte range.
  auto lookup = [&](uint64_t id, uint64_t expect, SrcTensor* t, std::string* err) -> int {
    const std::string name = gguf_tensor_name(id, layers);
    auto it = tensors.find(name);
    if (it == tensors.end()) {
      *err = "missing tensor " + name;
      return VVLI_ERR_MISSING_TENSOR;
    }
    const GgufTensor& g = it->second;
    // F32, F16, BF16 as in the reference; Q8_0 (8) and Q4_0 (2), which the
    // reference rejects (src/llm.zig:1083), are kept as blocks for the
    // matrices (a norm or bias must stay a native float).
    const int type = g.type == 0 ? kSrcF32 : g.type == 1 ? kSrcF16 : g.type == 30 ? kSrcBF16
                   : g.type == 8 ? kSrcQ8_0 : g.type == 2 ? kSrcQ4_0 : -1;
    if (type < 0) {
      *err = name + " has GGUF tensor type " + std::to_string(g.type) + " (F32, F16, BF16, Q8_0 or Q4_0 only)";
      return VVLI_ERR_UNSUPPORTED_DTYPE;
    }
    if (g.count != expect) {
      *err = "element count of " + name + " does not match the model config";
      return VVLI_ERR_INVALID_WEIGHT;
    }
    if (src_quantised(type) && g.count % 32) {
      *err = name + ": a block-quantised tensor must hold whole 32-weight blocks";
      return VVLI_ERR_INVALID_WEIGHT;
    }
    const uint64_t len = src_quantised(type) ? g.count / 32 * src_block_bytes(type) : g.count * src_elem_bytes(type);
    uint64_t start, end;
    if (__builtin_add_overflow(data_start, g.offset, &start) || __builtin_add_overflow(start, len, &end) ||
        end > m.size) {
      *err = "byte range of " + name + " runs past the end of the file";
      return VVLI_ERR_INVALID_WEIGHT;
    }
    *t = SrcTensor{type, g.count, m.bytes() + start};
    return VVLI_OK;
  };
  return copy_pieces(pieces, lookup, w, s, why, piece_fmt);
}

}  // namespace vvli
