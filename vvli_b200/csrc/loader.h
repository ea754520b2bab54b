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
  // The fused matrix the piece belongs to: element offset and this piece's
  // first row in it (where a block-quantised matrix stores its rows).
  uint64_t group_base, group_row;
};

// Returns a vvli_status; *why says what went wrong.
int upload_safetensors(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w,
                       cudaStream_t s, std::string* why);
// GGUF: F32 / F16 / BF16 tensors land as bf16; Q8_0 and Q4_0 matrices keep
// their blocks, repacked per row (kernels.h WeightFormat) from the group's
// offset.  piece_fmt[i] receives the WeightFormat piece i was stored in.
int upload_gguf(const char* path, const std::vector<LoadPiece>& pieces, int layers, uint16_t* w, cudaStream_t s,
                std::string* why, std::vector<int>* piece_fmt);

}  // namespace vvli
