// Shared device-side helpers for the executor's kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "common.h"

namespace mx {

#define MX_CUDA(call)                                                                                      \
  do {                                                                                                     \
    cudaError_t e_ = (call);                                                                               \
    if (e_ != cudaSuccess)                                                                                 \
      throw ::mx::Error(std::string(#call) + ": " + cudaGetErrorString(e_), MX_E_CUDA);                   \
  } while (0)

// A strided NHWC view of one plan buffer: pixel p, channel c lives at
// ptr[p * stride + c]. `stride` is the channel count of the buffer that owns
// the storage (a channel view of a wider buffer keeps its parent's stride).
struct View {
  float* ptr;
  int64_t stride;
  int64_t c;  // channels of this buffer
  int64_t npix;
};

inline unsigned blocks_for(int64_t n, int threads) { return unsigned((n + threads - 1) / threads); }

#ifdef __CUDACC__
// The activations, shared by the standalone elementwise kernels and the
// tensor-core epilogue so a fused step computes exactly what the separate
// op would (src/exec_cpu.rs: gelu with erf, the logistic sigmoid).
__device__ __forceinline__ float gelu_f(float a) { return 0.5f * a * (1.0f + erff(a * 0.70710677f)); }
__device__ __forceinline__ float sigmoid_f(float a) { return 1.0f / (1.0f + expf(-a)); }
#endif

}  // namespace mx
