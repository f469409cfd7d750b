// The channel mean (the CALayer squeeze, src/exec_gpu.rs:443-457) as a
// stand-alone entry point that allocates nothing.
//
// Who needs it: a caller that owns its device memory but may not allocate
// more of it - an engine that hands the GPU a fixed memory budget up front, a
// process running inside a CUDA stream capture (where cudaMalloc is not
// allowed), or an allocator-managed service that forbids stray allocations.
// The executor's own channel mean keeps its partial sums in a scratch buffer
// it allocates when the handle is created; this variant keeps them instead in
// one file-scope device array of fixed size that the library image carries,
// so a call does no cudaMalloc / cudaFree and calls no allocating routine.
//
// The array (kMaxScratch floats = 1 MiB) is held on every GPU that loads this
// library, until the process exits. It is shared by every call: each call
// writes every partial it later reads, so nothing has to start at zero, but
// two calls that overlap on the GPU (different streams, no ordering) race on
// it and give wrong results.
//
// The partition (one block per 512 pixels, at most 1024 blocks) and both
// kernels are the executor's own, so a call returns bit for bit what the
// executor's ChanMean step returns for the same tensor. The array holds that
// partition's 1024 partial rows for up to 256 channels, which is why the
// channel limit is 256 (the model's widest channel attention has 128).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "common.h"
#include "kernels_mem.cuh"
#include "maxim_b200.h"

namespace mx {
namespace {

constexpr int kMaxBlocks = 1024;                       // the executor's partition cap
constexpr int kMaxChannels = 256;
constexpr int kMaxScratch = kMaxBlocks * kMaxChannels;  // floats of partial sums (1 MiB)

__device__ __align__(256) float g_mean_scratch[kMaxScratch];

// Host code cannot use the array's name as a device address: in host code it
// names a host-side stand-in. The device address is looked up once per
// device, with that device current, and cached.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

float* scratch_on_current_device() {
  int dev = 0;
  MX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) throw Error(fmt("device %d is beyond the %d this entry point tracks", dev, kMaxDevices));
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mean_scratch);
    if (e != cudaSuccess || !p)
      throw Error(std::string("cudaGetSymbolAddress(channel-mean scratch): ") + cudaGetErrorString(e), MX_E_CUDA);
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace mx

using namespace mx;

extern "C" int mx_channel_mean_noalloc(const float* x, int64_t npix, int32_t c, int64_t pixel_stride, float* out,
                                       void* stream) {
  return guard([&] {
    if (!x || !out) throw Error("mx_channel_mean_noalloc: null pointer");
    if (npix <= 0 || npix >= (int64_t(1) << 31))
      throw Error(fmt("mx_channel_mean_noalloc: %lld pixels is outside 1 .. 2^31-1", (long long)npix));
    if (c <= 0 || c % 4 != 0 || c > kMaxChannels)
      throw Error(fmt("mx_channel_mean_noalloc: %d channels; this entry point takes a multiple of 4 up to %d (its "
                      "fixed scratch holds %d partial sums)",
                      c, kMaxChannels, kMaxScratch));
    if (pixel_stride < c || pixel_stride % 4 != 0 || pixel_stride >= (int64_t(1) << 31))
      throw Error(fmt("mx_channel_mean_noalloc: pixel stride %lld must be a multiple of 4 and at least c = %d",
                      (long long)pixel_stride, c));
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) throw Error("mx_channel_mean_noalloc: x must be 16-byte aligned");
    if (npix * pixel_stride >= (int64_t(1) << 31))
      throw Error("mx_channel_mean_noalloc: the input spans 2^31 or more floats");
    float* part = scratch_on_current_device();
    // The executor's partition: one block per 512 pixels, at most 1024
    // blocks; nb * c <= kMaxScratch by the channel limit above.
    const int nb = int(std::max<int64_t>(1, std::min<int64_t>((npix + 511) / 512, kMaxBlocks)));
    const int per = int((npix + nb - 1) / nb);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    chan_mean_partial_kernel<<<unsigned(nb), 256, 0, s>>>(int(npix), c / 4, per, x, int(pixel_stride), part);
    chan_mean_final_tree_kernel<<<unsigned(c), 256, 0, s>>>(nb, c, int(npix), part, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw Error(std::string("mx_channel_mean_noalloc: launch: ") + cudaGetErrorString(e), MX_E_CUDA);
  });
}
