// 3x3 pad-1 convolutions with three input or three output channels (the
// image-facing convs: the per-scale input convs 3 -> c and SAM Conv_2 3 -> c,
// the output convs and SAM Conv_1 c -> 3). Three channels cannot feed the
// tensor-core kernel (TMA rows must be 16-byte multiples and the MMA N is at
// least 16), and a general tiled SIMT GEMM wastes most of its tile on them, so
// each shape gets a direct kernel. Accumulation follows the reference's
// (ky, kx, ci) order from the bias (src/exec_cpu.rs:694-772), with FMA.
#pragma once

#include "gpu_common.cuh"

namespace mx {
namespace {

// c_in == 3: one thread per output pixel and per block of 32 output
// channels; the 27 weights of those channels sit in shared memory.
// W is [c_out][tap][3].
__global__ void __launch_bounds__(128) conv3x3_cin3_kernel(int h, int wd, int co, const float* __restrict__ x, int sx,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ bias, float* __restrict__ y,
                                                           int sy) {
  __shared__ float ws[32 * 27];
  __shared__ float bs[32];
  const int c0 = blockIdx.y * 32;
  for (int i = threadIdx.x; i < 32 * 27; i += blockDim.x) {
    int o = i / 27, k = i - o * 27;
    ws[i] = (c0 + o < co) ? w[size_t(c0 + o) * 27 + k] : 0.0f;
  }
  if (threadIdx.x < 32) bs[threadIdx.x] = (bias && c0 + threadIdx.x < co) ? bias[c0 + threadIdx.x] : 0.0f;
  __syncthreads();
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= h * wd) return;
  const int py = p / wd, px = p - py * wd;
  float in[27];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky)
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int iy = py + ky - 1, ix = px + kx - 1;
      const bool ok = iy >= 0 && iy < h && ix >= 0 && ix < wd;
      const float* s = x + size_t(iy * wd + ix) * sx;
#pragma unroll
      for (int c = 0; c < 3; ++c) in[(ky * 3 + kx) * 3 + c] = ok ? __ldg(s + c) : 0.0f;
    }
  float acc[32];
#pragma unroll
  for (int o = 0; o < 32; ++o) {
    float a = bs[o];
#pragma unroll
    for (int k = 0; k < 27; ++k) a = fmaf(in[k], ws[o * 27 + k], a);
    acc[o] = a;
  }
  float* d = y + size_t(p) * sy + c0;
  const int n = min(32, co - c0);
  if (n == 32 && (reinterpret_cast<uintptr_t>(d) % 16) == 0) {
#pragma unroll
    for (int o = 0; o < 32; o += 4) *reinterpret_cast<float4*>(d + o) = make_float4(acc[o], acc[o + 1], acc[o + 2], acc[o + 3]);
  } else {
#pragma unroll
    for (int o = 0; o < 32; ++o)
      if (o < n) d[o] = acc[o];
  }
}

// c_out == 3: a 16x16 block of output pixels per 256-thread block. Input
// channels go in chunks of 32 through a shared (18 x 18 pixel, 33-float
// padded) halo tile, so each input value is read from global once per block;
// each thread accumulates its pixel's 3 outputs. W is [3][tap][c_in].
__global__ void __launch_bounds__(256) conv3x3_cout3_kernel(int h, int wd, int ci, const float* __restrict__ x, int sx,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int sy) {
  constexpr int T = 16, HALO = T + 2, R = 33;
  __shared__ float tile[HALO * HALO * R];
  __shared__ float ws[3 * 9 * 32];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int x0 = blockIdx.x * T, y0 = blockIdx.y * T;
  float a0 = bias ? bias[0] : 0.0f, a1 = bias ? bias[1] : 0.0f, a2 = bias ? bias[2] : 0.0f;
  for (int cb = 0; cb < ci; cb += 32) {
    const int nc = min(32, ci - cb);
    __syncthreads();
    for (int i = threadIdx.x; i < HALO * HALO * 32; i += 256) {
      int pix = i >> 5, c = i & 31;
      int hy = pix / HALO, hx = pix - hy * HALO;
      int iy = y0 + hy - 1, ix = x0 + hx - 1;
      float v = 0.0f;
      if (c < nc && iy >= 0 && iy < h && ix >= 0 && ix < wd) v = __ldg(x + size_t(iy * wd + ix) * sx + cb + c);
      tile[pix * R + c] = v;
    }
    for (int i = threadIdx.x; i < 3 * 9 * 32; i += 256) {
      int o = i / (9 * 32), r = i - o * 9 * 32, t = r >> 5, c = r & 31;
      ws[i] = c < nc ? __ldg(w + (size_t(o) * 9 + t) * ci + cb + c) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const int ky = t / 3, kx = t - ky * 3;
      const float* s = tile + ((ty + ky) * HALO + tx + kx) * R;
      const float* w0 = ws + t * 32;
#pragma unroll 8
      for (int c = 0; c < 32; ++c) {
        const float v = s[c];
        a0 = fmaf(v, w0[c], a0);
        a1 = fmaf(v, w0[9 * 32 + c], a1);
        a2 = fmaf(v, w0[18 * 32 + c], a2);
      }
    }
  }
  const int py = y0 + ty, px = x0 + tx;
  if (py < h && px < wd) {
    float* d = y + size_t(py * wd + px) * sy;
    d[0] = a0;
    d[1] = a1;
    d[2] = a2;
  }
}

// The same two convs with their weights passed by value as a kernel
// parameter: the parameter space is a constant bank, so each multiply-add
// takes its weight as a constant operand and no instruction loads it. The
// loops over weights are fully unrolled (their indices are compile-time),
// and every output's sum runs in the same order as in the kernels above, so
// the results are theirs bit for bit.
//
// c_in == 3, one 32-output-channel chunk per launch: one output pixel per
// thread, all 32 outputs. The weights are [k = (ky, kx, c)][output], so the
// two weights of an output pair are one 8-byte constant: the multiply-adds
// run paired (f32x2), half the instructions and half the constant-bank
// reads (which set this kernel's pace when each multiply-add read its own).
struct alignas(16) Cin3Weights {
  float w[27 * 32];
  float b[32];
};
__global__ void __launch_bounds__(128) conv3x3_cin3c_kernel(int h, int wd, int n, const float* __restrict__ x, int sx,
                                                            float* __restrict__ y, int sy,
                                                            const __grid_constant__ Cin3Weights cw) {
  // A pixel past the end computes on zeros (its row of the staging buffer
  // is never stored) so that every thread reaches the barrier below.
  const int p = min(blockIdx.x * blockDim.x + threadIdx.x, h * wd - 1);
  const int py = p / wd, px = p - py * wd;
  float in[27];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky)
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int iy = py + ky - 1, ix = px + kx - 1;
      const bool ok = iy >= 0 && iy < h && ix >= 0 && ix < wd;
      const float* s = x + size_t(iy * wd + ix) * sx;
#pragma unroll
      for (int c = 0; c < 3; ++c) in[(ky * 3 + kx) * 3 + c] = ok ? __ldg(s + c) : 0.0f;
    }
  uint64_t acc2[16];
  const uint64_t* b2 = reinterpret_cast<const uint64_t*>(cw.b);
#pragma unroll
  for (int j = 0; j < 16; ++j) acc2[j] = b2[j];
#pragma unroll
  for (int k = 0; k < 27; ++k) {
    const uint64_t v = f2_pack(in[k], in[k]);
    const uint64_t* w2 = reinterpret_cast<const uint64_t*>(cw.w + k * 32);
#pragma unroll
    for (int j = 0; j < 16; ++j) acc2[j] = f2_fma(v, w2[j], acc2[j]);
  }
  float acc[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) f2_unpack(acc2[j], acc[2 * j], acc[2 * j + 1]);
  // The block's 128 x 32 outputs go through shared memory (rows padded to
  // 36 floats: conflict-free float4 access both ways), so each warp-wide
  // store writes four whole 128-byte pixel chunks instead of 32 scattered
  // 16-byte pieces.
  __shared__ float4 stage[128 * 9];
  const int t = threadIdx.x;
#pragma unroll
  for (int o = 0; o < 32; o += 4) stage[t * 9 + o / 4] = make_float4(acc[o], acc[o + 1], acc[o + 2], acc[o + 3]);
  __syncthreads();
  const int p0 = blockIdx.x * blockDim.x, npix = min(128, h * wd - p0);
  const bool vec = n == 32 && sy % 4 == 0 && (reinterpret_cast<uintptr_t>(y) % 16) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int f = t + 128 * i, pp = f >> 3, q = f & 7;
    if (pp >= npix) break;
    float* d = y + size_t(p0 + pp) * sy + 4 * q;
    const float4 v = stage[pp * 9 + q];
    if (vec) {
      *reinterpret_cast<float4*>(d) = v;
    } else {
      if (4 * q < n) d[0] = v.x;
      if (4 * q + 1 < n) d[1] = v.y;
      if (4 * q + 2 < n) d[2] = v.z;
      if (4 * q + 3 < n) d[3] = v.w;
    }
  }
}

// c_out == 3 with CI input channels (a multiple of 32; weights [o][tap][ci]):
// a 16x16 block of output pixels per 256-thread block, input channels in
// chunks of 32 through a shared halo tile read as float4s (rows padded to
// 36 floats: the eight float4 reads of a quarter-warp hit distinct banks).
template <int CI>
struct Cout3Weights {
  float w[3 * 9 * CI];
  float b[3];
};
template <int CI>
__global__ void __launch_bounds__(256) conv3x3_cout3c_kernel(int h, int wd, const float* __restrict__ x, int sx,
                                                             float* __restrict__ y, int sy,
                                                             const __grid_constant__ Cout3Weights<CI> cw) {
  constexpr int T = 16, HALO = T + 2, R = 36;
  __shared__ float4 tile[HALO * HALO * R / 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int x0 = blockIdx.x * T, y0 = blockIdx.y * T;
  float a0 = cw.b[0], a1 = cw.b[1], a2 = cw.b[2];
#pragma unroll
  for (int cb = 0; cb < CI; cb += 32) {
    if (cb) __syncthreads();
    for (int i = threadIdx.x; i < HALO * HALO * 8; i += 256) {
      const int pix = i >> 3, c4 = i & 7;
      const int hy = pix / HALO, hx = pix - hy * HALO;
      const int iy = y0 + hy - 1, ix = x0 + hx - 1;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (iy >= 0 && iy < h && ix >= 0 && ix < wd)
        v = __ldg(reinterpret_cast<const float4*>(x + size_t(iy * wd + ix) * sx + cb) + c4);
      tile[pix * (R / 4) + c4] = v;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const int ky = t / 3, kx = t - ky * 3;
      const float4* s = tile + ((ty + ky) * HALO + tx + kx) * (R / 4);
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) {
        const float4 v = s[c4];
        const int c = cb + 4 * c4;
        a0 = fmaf(v.x, cw.w[(0 * 9 + t) * CI + c], a0);
        a1 = fmaf(v.x, cw.w[(1 * 9 + t) * CI + c], a1);
        a2 = fmaf(v.x, cw.w[(2 * 9 + t) * CI + c], a2);
        a0 = fmaf(v.y, cw.w[(0 * 9 + t) * CI + c + 1], a0);
        a1 = fmaf(v.y, cw.w[(1 * 9 + t) * CI + c + 1], a1);
        a2 = fmaf(v.y, cw.w[(2 * 9 + t) * CI + c + 1], a2);
        a0 = fmaf(v.z, cw.w[(0 * 9 + t) * CI + c + 2], a0);
        a1 = fmaf(v.z, cw.w[(1 * 9 + t) * CI + c + 2], a1);
        a2 = fmaf(v.z, cw.w[(2 * 9 + t) * CI + c + 2], a2);
        a0 = fmaf(v.w, cw.w[(0 * 9 + t) * CI + c + 3], a0);
        a1 = fmaf(v.w, cw.w[(1 * 9 + t) * CI + c + 3], a1);
        a2 = fmaf(v.w, cw.w[(2 * 9 + t) * CI + c + 3], a2);
      }
    }
  }
  const int py = y0 + ty, px = x0 + tx;
  if (py < h && px < wd) {
    float* d = y + size_t(py * wd + px) * sy;
    d[0] = a0;
    d[1] = a1;
    d[2] = a2;
  }
}

}  // namespace
}  // namespace mx
