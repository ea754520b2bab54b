// loader.cu - weights straight from a safetensors file into this rank's device layout.
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
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/vvli_cuda.h"
#include "common.cuh"
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
};

}  // namespace

int upload_safetensors(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w,
                       cudaStream_t s, std::string* why) {
  Mapping m;
  m.fd = open(path, O_RDONLY);
  if (m.fd < 0) {
    *why = std::string("cannot open ") + path;
    return VVLI_ERR_INVALID_ARGUMENT;
  }
  struct stat st;
  if (fstat(m.fd, &st) != 0 || st.st_size < 8) {
    *why = std::string("not a safetensors file: ") + path;
    return VVLI_ERR_INVALID_WEIGHT;
  }
  m.size = static_cast<size_t>(st.st_size);
  m.base = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, m.fd, 0);
  if (m.base == MAP_FAILED) {
    *why = std::string("cannot map ") + path;
    return VVLI_ERR_INVALID_ARGUMENT;
  }
  const uint8_t* bytes = static_cast<const uint8_t*>(m.base);
  uint64_t header_len = 0;
  memcpy(&header_len, bytes, 8);  // little endian on every CUDA host
  if (8 + header_len > m.size) {
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
  // DMA straight from the page cache when the mapping can be page-locked.
  m.registered = cudaHostRegister(m.base, m.size, cudaHostRegisterReadOnly) == cudaSuccess;
  if (!m.registered) cudaGetLastError();

  float* stage = nullptr;
  constexpr size_t kStageBytes = 64ull << 20;
  int status = VVLI_OK;
  for (const LoadPiece& p : pieces) {
    const std::string name = tensor_name(p.tensor_id, layers);
    auto it = header.obj.find(name);
    if (it == header.obj.end()) {
      *why = "missing tensor " + name;
      status = VVLI_ERR_MISSING_TENSOR;
      break;
    }
    const Json& meta = it->second;
    auto dt = meta.obj.find("dtype");
    auto sh = meta.obj.find("shape");
    auto off = meta.obj.find("data_offsets");
    if (meta.kind != Json::Obj || dt == meta.obj.end() || sh == meta.obj.end() || off == meta.obj.end() ||
        sh->second.kind != Json::Arr || off->second.kind != Json::Arr || off->second.arr.size() != 2) {
      *why = "malformed entry for " + name;
      status = VVLI_ERR_INVALID_WEIGHT;
      break;
    }
    const bool bf16 = dt->second.str == "BF16", f32 = dt->second.str == "F32";
    if (!bf16 && !f32) {
      *why = name + " has dtype " + dt->second.str + " (BF16 or F32 only)";
      status = VVLI_ERR_UNSUPPORTED_DTYPE;
      break;
    }
    uint64_t count = 1;
    for (const Json& d : sh->second.arr) count *= static_cast<uint64_t>(d.num);
    const uint64_t start = static_cast<uint64_t>(off->second.arr[0].num), end = static_cast<uint64_t>(off->second.arr[1].num);
    const uint64_t esz = bf16 ? 2 : 4;
    if (count != p.tensor_elems || end < start || end > data_len || end - start != count * esz) {
      *why = "shape or byte range of " + name + " does not match the model config";
      status = VVLI_ERR_INVALID_WEIGHT;
      break;
    }
    const uint8_t* src = data + start + (p.row0 * p.src_ld + p.col0) * esz;
    uint16_t* dst = w + p.dst;
    cudaError_t e;
    if (bf16) {
      e = cudaMemcpy2DAsync(dst, p.cols * 2, src, p.src_ld * 2, p.cols * 2, p.rows, cudaMemcpyHostToDevice, s);
    } else {
      if (!stage && (e = cudaMalloc(&stage, kStageBytes)) != cudaSuccess) {
        *why = "staging buffer for F32 tensors";
        status = VVLI_ERR_OOM;
        break;
      }
      const uint64_t rows_per = std::max<uint64_t>(1, kStageBytes / (p.cols * 4));
      e = cudaSuccess;
      for (uint64_t r = 0; r < p.rows && e == cudaSuccess; r += rows_per) {
        const uint64_t n = std::min(rows_per, p.rows - r);
        e = cudaMemcpy2DAsync(stage, p.cols * 4, src + r * p.src_ld * 4, p.src_ld * 4, p.cols * 4, n,
                              cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
          const size_t total = n * p.cols;
          const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 4096));
          f32_to_bf16_kernel<<<blocks, 256, 0, s>>>(stage, dst + r * p.cols, total);
          e = cudaGetLastError();
          if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the staging buffer is reused
        }
      }
    }
    if (e != cudaSuccess) {
      *why = std::string("copying ") + name + ": " + cudaGetErrorString(e);
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

}  // namespace vvli
