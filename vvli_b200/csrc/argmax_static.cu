// argmax_static.cu - greedy token choice over rows of device logits, with no
// device allocation by the library.
//
// This is a standalone variant of the argmax reduction that ends the lm_head
// GEMV (EPI_ARGMAX in kernels.cu): every CTA reduces a slice of a row to one
// (value, index) partial, and the last CTA of the row to arrive reduces the
// partials.  The context-based path keeps those partials in buffers that
// vvli_cuda_create allocates; this variant keeps them in one file-scope
// static device array, so a call needs neither a context nor cudaMalloc.
//
// Which callers need it: a host that has already handed (nearly) all of the
// GPU's memory to its own pool - a serving engine that reserves HBM for its
// KV cache up front - cannot let a library call cudaMalloc, because the
// allocation fails or steals from the pool; and cudaFree synchronises the
// whole device, which a caller that keeps several streams busy cannot afford
// per token.  Such a caller produces logits with its own kernels and only
// wants the token ids written to memory it owns.
//
// Semantics follow llm.argmax (src/llm.zig:778-789): strict `>` in index
// order, so the first maximal index wins ties, a NaN never replaces the
// running best, and a NaN in element 0 makes the answer 0.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <mutex>
#include <string>

#include "../../include/vvli_cuda.h"
#include "common.cuh"

namespace vvli {
void set_last_error(const std::string& what);  // runtime.cu
}

using namespace vvli;

namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 16;
constexpr int kChunk = kThreads * kPerThread;   // logits one CTA reduces (4096)
constexpr int kMaxRows = 64;                    // rows per call
constexpr int kMaxPartials = 4096;              // CTAs per call over all rows
constexpr int kMaxDevices = 64;

// Scratch layout (bytes): [0, 256) per-row arrival counters (u32 x 64),
// [256, 16640) partial values (f32 x 4096), [16640, 33024) partial indices
// (i32 x 4096).  33,024 bytes per device in total.
constexpr size_t kCountersOff = 0;
constexpr size_t kValOff = kCountersOff + sizeof(unsigned int) * kMaxRows;
constexpr size_t kIdxOff = kValOff + sizeof(float) * kMaxPartials;
constexpr size_t kScratchBytes = kIdxOff + sizeof(int) * kMaxPartials;
static_assert(kValOff % 16 == 0 && kIdxOff % 16 == 0, "scratch sections stay 16-byte aligned");

// Static storage is zero when this library's device code is loaded.  The
// arrival counters MUST be zero when a call starts: the last CTA of each row
// writes its counter back to zero, so every completed call leaves them zero.
// The partials need no initial value (each is written before it is read).
static __device__ __align__(256) unsigned char g_argmax_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

__global__ void __launch_bounds__(kThreads) argmax_rows_static_kernel(const float* __restrict__ logits, int n,
                                                                      int ctas_per_row, int32_t* __restrict__ tokens,
                                                                      unsigned char* scratch) {
  unsigned int* arrivals = reinterpret_cast<unsigned int*>(scratch + kCountersOff);
  float* part_val = reinterpret_cast<float*>(scratch + kValOff);
  int* part_idx = reinterpret_cast<int*>(scratch + kIdxOff);
  __shared__ float wv[kThreads / kWarp];
  __shared__ int wi[kThreads / kWarp];
  __shared__ int last;

  const int row = blockIdx.y, cta = blockIdx.x, tid = threadIdx.x;
  const int warp = tid / kWarp, lane = tid % kWarp;
  const float* v = logits + static_cast<size_t>(row) * n;
  const int base = cta * kChunk + tid;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  float x[kPerThread];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int i = base + j * kThreads;
    x[j] = i < n ? __ldg(v + i) : -INFINITY;
  }
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int i = base + j * kThreads;
    if (i < n && better(x[j], i, bv, bi)) {
      bv = x[j];
      bi = i;
    }
  }
  warp_argmax(bv, bi);
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  const int slot = row * ctas_per_row + cta;
  if (tid == 0) {
    for (int w = 1; w < kThreads / kWarp; ++w)
      if (better(wv[w], wi[w], bv, bi)) {
        bv = wv[w];
        bi = wi[w];
      }
    part_val[slot] = bv;
    part_idx[slot] = bi;
    __threadfence();
    last = atomicAdd(arrivals + row, 1u) == static_cast<unsigned>(ctas_per_row) - 1;
  }
  __syncthreads();
  if (!last) return;

  // Last CTA of this row: reduce the row's partials (L2 reads, not L1).
  __threadfence();
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int c = tid; c < ctas_per_row; c += kThreads) {
    const float pv = __ldcg(part_val + row * ctas_per_row + c);
    const int pi = __ldcg(part_idx + row * ctas_per_row + c);
    if (better(pv, pi, bv, bi)) {
      bv = pv;
      bi = pi;
    }
  }
  warp_argmax(bv, bi);
  __syncthreads();  // every thread has read `last` and wv/wi before they are reused
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kThreads / kWarp; ++w)
      if (better(wv[w], wi[w], bv, bi)) {
        bv = wv[w];
        bi = wi[w];
      }
    // llm.argmax starts from element 0: a NaN there is never replaced.
    if (isnan(__ldg(v))) bi = 0;
    tokens[row] = bi;
    arrivals[row] = 0;  // the next call starts from zero
  }
}

int fail(int code, const std::string& why) {
  set_last_error(why);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  set_last_error(std::string("argmax (static scratch): ") + what + ": " + cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? VVLI_ERR_OOM : VVLI_ERR_CUDA;
}

// True when `p` is memory that `device` can read: device memory of `device`,
// or managed memory.
bool device_ptr_ok(const void* p, int device) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == device);
}

// True when the first and the last byte of [p, p + bytes) are memory that
// `device` can read.  Both ends are checked separately rather than asking for
// one allocation that covers the range: pools built on the virtual memory API
// (cuMemCreate + cuMemMap, e.g. torch's expandable segments) map a buffer as
// several physical chunks, and a buffer that spans two of them is valid.
bool device_range_ok(const void* p, size_t bytes, int device) {
  if (bytes == 0 || reinterpret_cast<uintptr_t>(p) > UINTPTR_MAX - (bytes - 1)) return false;
  return device_ptr_ok(p, device) && device_ptr_ok(static_cast<const char*>(p) + (bytes - 1), device);
}

// One-time setup per device (the device is current): look up the address of
// the static scratch.  This may load this library's device code.  The address
// is kept for the life of the process: a cudaDeviceReset after the first call
// unloads the device code, and the cached address is then stale, so a device
// reset is not supported once this entry point has run on that device.
int scratch_for(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    if (!p || reinterpret_cast<uintptr_t>(p) % 256 != 0)
      return fail(VVLI_ERR_CUDA, "argmax (static scratch): the scratch symbol has no usable device address");
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return VVLI_OK;
}

// Restores the caller's current device on every return path.
struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int vvli_cuda_argmax_rows_static(int device, const float* logits, uint64_t rows, uint64_t n,
                                            int32_t* tokens, void* stream) {
  if (!logits || !tokens) return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): null pointer");
  if (rows == 0 || n == 0) return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): empty logits");
  if (n > static_cast<uint64_t>(kMaxPartials) * kChunk)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): n = " + std::to_string(n) +
                                               " exceeds the limit of " +
                                               std::to_string(static_cast<uint64_t>(kMaxPartials) * kChunk) +
                                               " logits per row");
  if (rows > kMaxRows)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): " + std::to_string(rows) +
                                               " rows exceed the limit of " + std::to_string(kMaxRows) +
                                               " rows per call");
  const uint64_t ctas_per_row = (n + kChunk - 1) / kChunk;
  if (ctas_per_row * rows > static_cast<uint64_t>(kMaxPartials))
    return fail(VVLI_ERR_INVALID_ARGUMENT,
                "argmax (static scratch): rows * ceil(n / 4096) = " + std::to_string(ctas_per_row * rows) +
                    " exceeds the scratch limit of 4096 partials (rows " + std::to_string(rows) + ", n " +
                    std::to_string(n) + ")");
  if (reinterpret_cast<uintptr_t>(logits) % alignof(float) || reinterpret_cast<uintptr_t>(tokens) % alignof(int32_t))
    return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): misaligned pointer");
  if (device < 0 || device >= kMaxDevices)
    return fail(VVLI_ERR_INVALID_ARGUMENT, "argmax (static scratch): device ordinal out of range");

  DeviceGuard guard;
  cudaError_t e = cudaGetDevice(&guard.prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  if (!device_range_ok(logits, rows * n * sizeof(float), device))
    return fail(VVLI_ERR_INVALID_ARGUMENT,
                "argmax (static scratch): logits must be rows * n floats of device memory on device " +
                    std::to_string(device));
  if (!device_range_ok(tokens, rows * sizeof(int32_t), device))
    return fail(VVLI_ERR_INVALID_ARGUMENT,
                "argmax (static scratch): tokens must be rows int32 of device memory on device " +
                    std::to_string(device));

  void* scratch = nullptr;
  const int rc = scratch_for(device, &scratch);
  if (rc != VVLI_OK) return rc;
  const dim3 grid(static_cast<unsigned>(ctas_per_row), static_cast<unsigned>(rows));
  argmax_rows_static_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, static_cast<int>(n), static_cast<int>(ctas_per_row), tokens, static_cast<unsigned char*>(scratch));
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return VVLI_OK;
}
