// The reference pipeline's per-pixel image steps on the device, either side
// of the pass: 8-bit RGB samples to the plan's padded [3][H][W] input, and the
// padded prediction to the cropped 8-bit RGB the CLI writes
// (src/image.rs:40-104 for the 8-bit conversions, :116-141 and :171-207 for
// the reflections, :233-246 for the crop). Both are bit for bit the host
// pipeline's: the same divide by 255, the same reflections, and the same
// clamp, multiply, add and truncate, each rounded on its own.
#pragma once

#include <cstdint>

// torch's reflect (mirror about the edge without repeating it) for an index
// at most n - 1 outside [0, n).
__device__ __forceinline__ int reflect_px(int i, int n) { return i < 0 ? -i : (i >= n ? 2 * n - 2 - i : i); }

// One thread per padded pixel (grid-stride). The padded image is the even
// image reflected `top` rows / `left` columns out on each side, and the even
// image is the original reflected one row (column) out at the bottom (right)
// when its height (width) is odd; so padded (y, x) reads the original at the
// two reflections composed. The caller guarantees top < even_h,
// left < even_w, h >= 2 and w >= 2, which keeps every index in range.
// Reads are interleaved RGB bytes; each plane's writes are coalesced.
__global__ void __launch_bounds__(256) rgb8_to_padded_kernel(const uint8_t* __restrict__ src, int h, int w,
                                                             int even_h, int even_w, int top, int left, int H, int W,
                                                             float* __restrict__ dst) {
  const int64_t plane = int64_t(H) * W;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < plane; i += int64_t(gridDim.x) * blockDim.x) {
    const int y = int(i / W), x = int(i - int64_t(y) * W);
    const int sy = reflect_px(reflect_px(y - top, even_h), h);
    const int sx = reflect_px(reflect_px(x - left, even_w), w);
    const uint8_t* p = src + (int64_t(sy) * w + sx) * 3;
    // IEEE division (this build keeps -prec-div on), as the host's v / 255.0f.
    dst[i] = float(p[0]) / 255.0f;
    dst[plane + i] = float(p[1]) / 255.0f;
    dst[2 * plane + i] = float(p[2]) / 255.0f;
  }
}

// clamp(v, 0, 1) * 255 + 0.5, truncated: round half up to 8 bits, with the
// multiply and the add rounded separately as on the host. NaN gives 0 (what
// the reference's saturating `as u8` gives for a NaN).
__device__ __forceinline__ uint8_t quantize8(float v) {
  if (v != v) return 0;
  v = fminf(fmaxf(v, 0.0f), 1.0f);
  return uint8_t(__fadd_rn(__fmul_rn(v, 255.0f), 0.5f));
}

// One thread per output pixel (grid-stride): the prediction's [3][H][W]
// window at (hs, ws), oh x ow pixels, quantised and interleaved.
__global__ void __launch_bounds__(256) crop_to_rgb8_kernel(const float* __restrict__ pred, int H, int W, int hs,
                                                           int ws, int oh, int ow, uint8_t* __restrict__ dst) {
  const int64_t n = int64_t(oh) * ow, plane = int64_t(H) * W;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int y = int(i / ow), x = int(i - int64_t(y) * ow);
    const int64_t s = int64_t(hs + y) * W + (ws + x);
    uint8_t* d = dst + i * 3;
    d[0] = quantize8(pred[s]);
    d[1] = quantize8(pred[plane + s]);
    d[2] = quantize8(pred[2 * plane + s]);
  }
}
