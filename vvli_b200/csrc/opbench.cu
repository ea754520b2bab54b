// opbench.cu - the isolated linear-layer op of the decoder, timed alone.
//
// y[M, N] = x[M, K] . W[N, K]^T with W bf16 and x, y fp32 (linearInto,
// src/llm.zig:1228-1285, applied to M independent rows), through the kernel
// the decoder uses for that many rows:
//   M = 1        the bulk-copy GEMV (gemv_tma_kernel; fp32 x, fp32 sums);
//   M <= 32      the decode-batch tensor-core GEMM (gemm_skinny_kernel);
//   M <= 64      the same GEMM twice, 32 rows per launch (W read twice);
//   M > 64       the prefill tensor-core GEMM (gemm_tc_kernel).
// The tensor-core paths take x as bf16 hi + lo pairs; the split kernel that
// makes them from fp32 x is inside the timed region.  Weight copies are
// rotated so that the copies together exceed twice the L2 size and no launch
// finds its weights in L2.  Measurement hook only: nothing on the decode path
// calls it.
#include <algorithm>
#include <string>
#include <vector>

#include "../../include/vvli_cuda.h"
#include "gemm_tc.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace vvli {
void set_last_error(const std::string& what);  // runtime.cu
}

using namespace vvli;

namespace {

__global__ void opbench_fill_kernel(uint16_t* w, size_t n, uint64_t seed, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint64_t z = (i + 1) * 0x9E3779B97F4A7C15ull ^ seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float u = (static_cast<float>(z >> 40) * (1.0f / 16777216.0f)) - 0.5f;
    w[i] = f32_to_bf16(u * scale);
  }
}

__global__ void opbench_fill_f32_kernel(float* x, size_t n, uint64_t seed) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint64_t z = (i + 7) * 0xD6E8FEB86659FD93ull ^ seed;
    z = (z ^ (z >> 32)) * 0xD6E8FEB86659FD93ull;
    z ^= z >> 29;
    x[i] = static_cast<float>(z >> 40) * (2.0f / 16777216.0f) - 1.0f;
  }
}

// fp32 activations -> bf16 hi + lo operands of the tensor-core GEMMs.
__global__ void opbench_split_kernel(const float* __restrict__ x, size_t n, uint16_t* __restrict__ hi,
                                     uint16_t* __restrict__ lo) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    split_bf16(x[i], hi[i], lo[i]);
}

struct Buffers {
  std::vector<uint16_t*> w;
  float *x = nullptr, *y = nullptr;
  uint16_t *xhi = nullptr, *xlo = nullptr;
  int* err = nullptr;
  float* sk_ws = nullptr;  // stream-K parts of the prefill GEMM, as the decoder's prefill has them
  unsigned* sk_flags = nullptr;
  ~Buffers() {
    for (uint16_t* p : w) cudaFree(p);
    cudaFree(x), cudaFree(y), cudaFree(xhi), cudaFree(xlo), cudaFree(err), cudaFree(sk_ws), cudaFree(sk_flags);
  }
};

}  // namespace

extern "C" int vvli_cuda_op_bench(int device, int M, int N, int K, int reps, float* avg_ms, double* bytes,
                                  double* flops, int* kernel_used) {
  if (!avg_ms || !bytes || !flops || M < 1 || N < 2 || N % 2 || K < 8 || K % 8 || reps < 1) {
    set_last_error("op bench: needs M >= 1, even N >= 2, K a multiple of 8, reps >= 1");
    return VVLI_ERR_INVALID_ARGUMENT;
  }
  auto cuda_err = [](cudaError_t e, const char* what) {
    set_last_error(std::string("op bench: ") + what + ": " + cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? VVLI_ERR_OOM : VVLI_ERR_CUDA;
  };
  cudaError_t e;
  if ((e = cudaSetDevice(device))) return cuda_err(e, "cudaSetDevice");
  int optin = 0, l2 = 0, sms = 148;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if ((e = configure_kernels(optin)) || (e = configure_gemm_tc(optin)) || (e = configure_gemm_skinny(optin)))
    return cuda_err(e, "configure");
  const size_t wbytes = static_cast<size_t>(N) * K * 2;
  const size_t copies = std::max<size_t>(4, (2 * static_cast<size_t>(l2) + wbytes - 1) / wbytes + 1);
  const int kind = M == 1 ? 0 : M <= kSkinnyMaxRows ? 1 : M <= 2 * kSkinnyMaxRows ? 2 : 3;
  Buffers b;
  for (size_t i = 0; i < copies; ++i) {
    uint16_t* p = nullptr;
    if ((e = cudaMalloc(&p, wbytes))) return cuda_err(e, "weights");
    b.w.push_back(p);
    opbench_fill_kernel<<<1024, 256>>>(p, static_cast<size_t>(N) * K, 0x5EED0000ull + i, 0.08f);
  }
  const size_t xn = static_cast<size_t>(M) * K;
  // Activation rows allocated (zero beyond M) so that every TMA box lies inside its tensor.
  const int xrows = kind == 3 ? std::max(M, kGemmBM) : kind > 0 ? 2 * kSkinnyMaxRows : M;
  if ((e = cudaMalloc(&b.x, xn * 4)) || (e = cudaMalloc(&b.y, static_cast<size_t>(M) * N * 4)) ||
      (e = cudaMalloc(&b.xhi, static_cast<size_t>(xrows) * K * 2)) ||
      (e = cudaMalloc(&b.xlo, static_cast<size_t>(xrows) * K * 2)) || (e = cudaMalloc(&b.err, 4)))
    return cuda_err(e, "activations");
  if (kind == 3 && ((e = cudaMalloc(&b.sk_ws, gemm_tc_streamk_ws_floats(sms) * 4)) ||
                    (e = cudaMalloc(&b.sk_flags, static_cast<size_t>(sms) * 4)) ||
                    (e = cudaMemset(b.sk_flags, 0, static_cast<size_t>(sms) * 4))))
    return cuda_err(e, "stream-K workspace");
  unsigned sk_epoch = 0;
  cudaMemset(b.err, 0, 4);
  cudaMemset(b.xhi, 0, static_cast<size_t>(xrows) * K * 2);
  cudaMemset(b.xlo, 0, static_cast<size_t>(xrows) * K * 2);
  opbench_fill_f32_kernel<<<256, 256>>>(b.x, xn, 0xA11CEull);

  // Tensor maps: activations (one per 32-row half for kind 2) and every weight copy.
  std::vector<CUtensorMap> tw(copies);
  CUtensorMap th[2], tl[2];
  if (kind > 0) {
    const uint32_t box_x = kind == 3 ? static_cast<uint32_t>(kGemmBM) : static_cast<uint32_t>(skinny_nb(std::min(M, kSkinnyMaxRows)));
    const int halves = kind == 2 ? 2 : 1;
    for (int hf = 0; hf < halves; ++hf) {
      const int rows = kind == 3 ? xrows : kSkinnyMaxRows;
      const size_t off = static_cast<size_t>(hf) * kSkinnyMaxRows * K;
      if ((e = make_tmap_bf16(&th[hf], b.xhi + off, rows, K, box_x)) ||
          (e = make_tmap_bf16(&tl[hf], b.xlo + off, rows, K, box_x)))
        return cuda_err(e, "activation tensor maps");
    }
    for (size_t i = 0; i < copies; ++i)
      if ((e = make_tmap_bf16(&tw[i], b.w[i], N, K, kind == 3 ? kGemmBN / 2 : 128)))
        return cuda_err(e, "weight tensor maps");
  }
  cudaStream_t s = nullptr;
  if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking))) return cuda_err(e, "stream");
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  auto one = [&](size_t i) -> cudaError_t {
    if (kind == 0) {
      GemvParams p{};
      p.W = b.w[i], p.N = N, p.K = K, p.x = b.x, p.y = b.y;
      return launch_gemv(EPI_PLAIN, p, sms, s, false);
    }
    opbench_split_kernel<<<std::min<size_t>(1024, (xn + 255) / 256), 256, 0, s>>>(b.x, xn, b.xhi, b.xlo);
    GemmParams p{};
    p.N = N, p.K = K, p.nk = (K + kGemmBK - 1) / kGemmBK, p.two_a = 1, p.epi = GE_RESID, p.add_residual = 0;
    p.err = b.err, p.ldy = N;
    if (kind == 3) {
      p.M = M, p.y = b.y;
      p.sk_ws = b.sk_ws, p.sk_flags = b.sk_flags, p.sk_epoch = ++sk_epoch;
      return launch_gemm_tc(th[0], tl[0], tw[i], p, s);
    }
    for (int hf = 0; hf < (kind == 2 ? 2 : 1); ++hf) {
      p.M = kind == 2 ? std::min(kSkinnyMaxRows, M - hf * kSkinnyMaxRows) : M;
      p.y = b.y + static_cast<size_t>(hf) * kSkinnyMaxRows * N;
      cudaError_t le = launch_gemm_skinny(th[hf], tl[hf], tw[i], p, skinny_split(GE_RESID, p.M, N, p.nk, sms), s, false);
      if (le) return le;
    }
    return cudaSuccess;
  };
  int rc = VVLI_OK;
  for (size_t i = 0; i < std::min<size_t>(copies, 3) && rc == VVLI_OK; ++i)
    if ((e = one(i))) rc = cuda_err(e, "warm-up launch");
  if (rc == VVLI_OK && (e = cudaEventRecord(e0, s))) rc = cuda_err(e, "event");
  for (int r = 0; r < reps && rc == VVLI_OK; ++r)
    if ((e = one(static_cast<size_t>(r + 3) % copies))) rc = cuda_err(e, "launch");
  if (rc == VVLI_OK && ((e = cudaEventRecord(e1, s)) || (e = cudaEventSynchronize(e1)))) rc = cuda_err(e, "sync");
  float ms = 0.f;
  int herr = 0;
  if (rc == VVLI_OK) {
    cudaEventElapsedTime(&ms, e0, e1);
    cudaMemcpy(&herr, b.err, 4, cudaMemcpyDeviceToHost);
    if (herr) {
      set_last_error("op bench: a bounded wait of the GEMM gave up");
      rc = VVLI_ERR_TIMEOUT;
    }
  }
  cudaStreamSynchronize(s);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  if (rc != VVLI_OK) return rc;
  *avg_ms = ms / reps;
  *bytes = 2.0 * N * K + 4.0 * M * K + 4.0 * M * N;
  *flops = 2.0 * M * N * static_cast<double>(K);
  if (kernel_used) *kernel_used = kind;
  return VVLI_OK;
}
