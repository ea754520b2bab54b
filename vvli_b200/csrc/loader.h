// loader.h - safetensors / GGUF file -> device weight layout (see loader.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace vvli {

// One rectangular piece of a reference tensor (blob order id `tensor_id`,
// `tensor_elems` elements in all) copied to element offset `dst` of the
// device weights: rows x cols starting at (row0, col0), source row stride src_ld.
struct LoadPiece {
  uint64_t tensor_id, tensor_elems;
  uint64_t dst, rows, cols, src_ld, row0, col0;
};

// Returns a vvli_status; *why says what went wrong.
int upload_safetensors(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w,
                       cudaStream_t s, std::string* why);
int upload_gguf(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w, cudaStream_t s,
                std::string* why);

}  // namespace vvli
