// The memory-bound op kernels and the SIMT contraction fallback of the
// executor, all over NHWC views (pixel-major, channels contiguous).
//
// Where the reference's CPU executor fixes an order of operations that decides
// the result - the LayerNorm statistics and the resize taps - these kernels use
// the non-contracting intrinsics (__fadd_rn / __fmul_rn / __fdiv_rn /
// __fsqrt_rn) in that same order, so they reproduce it bit for bit rather than
// letting the compiler fuse a multiply and an add into one rounding.
#pragma once

#include "gpu_common.cuh"

namespace mx {

enum EwKind { EW_COPY = 0, EW_ADD, EW_MUL, EW_GATE, EW_GELU, EW_LRELU, EW_SIGMOID };

template <int KIND>
__device__ __forceinline__ float ew_apply(float a, float b, float slope) {
  if constexpr (KIND == EW_COPY) return a;
  else if constexpr (KIND == EW_ADD) return a + b;
  else if constexpr (KIND == EW_MUL) return a * b;
  else if constexpr (KIND == EW_GATE) return a * (b + 1.0f);  // u * (v + 1)
  else if constexpr (KIND == EW_GELU) return gelu_f(a);
  else if constexpr (KIND == EW_LRELU) return a >= 0.0f ? a : slope * a;
  else return sigmoid_f(a);
}

// Elementwise over npix x c with strided operands, 4 channels per thread.
template <int KIND>
__global__ void ew_kernel4(int64_t npix, int c4, const float* __restrict__ a, int64_t sa, const float* __restrict__ b,
                           int64_t sb, float* __restrict__ d, int64_t sd, float slope) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= npix * c4) return;
  int64_t p = i / c4;
  int ch = int(i - p * c4) * 4;
  float4 x = *reinterpret_cast<const float4*>(a + p * sa + ch);
  float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
  if (KIND == EW_ADD || KIND == EW_MUL || KIND == EW_GATE) y = *reinterpret_cast<const float4*>(b + p * sb + ch);
  float4 r;
  r.x = ew_apply<KIND>(x.x, y.x, slope);
  r.y = ew_apply<KIND>(x.y, y.y, slope);
  r.z = ew_apply<KIND>(x.z, y.z, slope);
  r.w = ew_apply<KIND>(x.w, y.w, slope);
  *reinterpret_cast<float4*>(d + p * sd + ch) = r;
}

template <int KIND>
__global__ void ew_kernel1(int64_t npix, int c, const float* __restrict__ a, int64_t sa, const float* __restrict__ b,
                           int64_t sb, float* __restrict__ d, int64_t sd, float slope) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= npix * c) return;
  int64_t p = i / c;
  int ch = int(i - p * c);
  float y = 0.0f;
  if (KIND == EW_ADD || KIND == EW_MUL || KIND == EW_GATE) y = b[p * sb + ch];
  d[p * sd + ch] = ew_apply<KIND>(a[p * sa + ch], y, slope);
}

// Channel LayerNorm, one thread per pixel, in the reference's order: serial
// s1 = sum x and s2 = sum x*x over the pixel's channels, m = s1/c,
// var = s2/c - m*m, rstd = 1/sqrt(max(var,0) + eps), y = (x - m)*rstd*w + b
// (src/exec_cpu.rs:396-433).
__global__ void chan_ln_kernel1(int64_t npix, int c, const float* __restrict__ x, int64_t sx,
                                const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ y,
                                int64_t sy, float eps) {
  int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (p >= npix) return;
  const float* xp = x + p * sx;
  float s1 = 0.0f, s2 = 0.0f;
  for (int i = 0; i < c; ++i) {
    s1 = __fadd_rn(s1, xp[i]);
    s2 = __fadd_rn(s2, __fmul_rn(xp[i], xp[i]));
  }
  float nf = float(c);
  float m = __fdiv_rn(s1, nf);
  float var = __fsub_rn(__fdiv_rn(s2, nf), __fmul_rn(m, m));
  float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), eps)));
  float* yp = y + p * sy;
  for (int i = 0; i < c; ++i) yp[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xp[i], m), rstd), w[i]), bias[i]);
}

// The same with 16-byte accesses, for c % 4 == 0 and aligned operands.
__global__ void chan_ln_kernel4(int64_t npix, int c, const float* __restrict__ x, int64_t sx,
                                const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ y,
                                int64_t sy, float eps) {
  int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (p >= npix) return;
  const float* xp = x + p * sx;
  float s1 = 0.0f, s2 = 0.0f;
  for (int i = 0; i < c; i += 4) {
    float4 v = *reinterpret_cast<const float4*>(xp + i);
    s1 = __fadd_rn(s1, v.x);
    s2 = __fadd_rn(s2, __fmul_rn(v.x, v.x));
    s1 = __fadd_rn(s1, v.y);
    s2 = __fadd_rn(s2, __fmul_rn(v.y, v.y));
    s1 = __fadd_rn(s1, v.z);
    s2 = __fadd_rn(s2, __fmul_rn(v.z, v.z));
    s1 = __fadd_rn(s1, v.w);
    s2 = __fadd_rn(s2, __fmul_rn(v.w, v.w));
  }
  float nf = float(c);
  float m = __fdiv_rn(s1, nf);
  float var = __fsub_rn(__fdiv_rn(s2, nf), __fmul_rn(m, m));
  float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), eps)));
  float* yp = y + p * sy;
  for (int i = 0; i < c; i += 4) {
    float4 v = *reinterpret_cast<const float4*>(xp + i);
    float4 ww = *reinterpret_cast<const float4*>(w + i);
    float4 bb = *reinterpret_cast<const float4*>(bias + i);
    float4 r;
    r.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, m), rstd), ww.x), bb.x);
    r.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, m), rstd), ww.y), bb.y);
    r.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, m), rstd), ww.z), bb.z);
    r.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, m), rstd), ww.w), bb.w);
    *reinterpret_cast<float4*>(yp + i) = r;
  }
}

// Per-channel mean over the pixels (the CALayer squeeze): one block per channel.
__global__ void chan_mean_kernel(int64_t npix, const float* __restrict__ x, int64_t sx, float* __restrict__ d) {
  __shared__ float red[32];
  int ch = blockIdx.x;
  float s = 0.0f;
  for (int64_t p = threadIdx.x; p < npix; p += blockDim.x) s += x[p * sx + ch];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) d[ch] = s / float(npix);
  }
}

// out[p][c] = x[p][c] * s[c] (the CALayer excitation).
__global__ void chan_scale_kernel(int64_t npix, int c, const float* __restrict__ x, int64_t sx,
                                  const float* __restrict__ s, float* __restrict__ d, int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= npix * c) return;
  int64_t p = i / c;
  int ch = int(i - p * c);
  d[p * sd + ch] = x[p * sx + ch] * s[ch];
}

// Space <-> blocked permutation of whole pixels (src/exec_cpu.rs:1078-1103):
// blocked index e = g * psz + q, g = gy*gw + gx, q = fy*fw + fx.
__global__ void block_perm_kernel(int64_t total, int c, int wd, int gw, int fh, int fw, int gsz, int psz, int swap,
                                  int forward, const float* __restrict__ src, int64_t ss, float* __restrict__ dst,
                                  int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= total) return;
  int64_t e = i / c;
  int ch = int(i - e * c);
  int64_t g, q;
  if (swap) {
    q = e / gsz;
    g = e - q * gsz;
  } else {
    g = e / psz;
    q = e - g * psz;
  }
  int64_t gy = g / gw, gx = g - gy * gw, fy = q / fw, fx = q - fy * fw;
  int64_t pix = (gy * fh + fy) * wd + gx * fw + fx;
  if (forward) dst[e * sd + ch] = src[pix * ss + ch];
  else dst[pix * sd + ch] = src[e * ss + ch];
}

// jax nearest downsample: out[y][x] = in[y*s+off][x*s+off].
__global__ void down_s_kernel(int64_t total, int c, int wd, int ow, int stride, int off, const float* __restrict__ src,
                              int64_t ss, float* __restrict__ dst, int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= total) return;
  int64_t p = i / c;
  int ch = int(i - p * c);
  int64_t y = p / ow, x = p - y * ow;
  dst[p * sd + ch] = src[((y * stride + off) * wd + x * stride + off) * ss + ch];
}

// One axis of the jax bilinear resize from a host-built tap table: per output
// index o, taps j0[o] .. j0[o]+cnt[o]-1 with weights w[w0[o] ..], then
// acc / wsum[o] if wsum > 0 (src/exec_cpu.rs:1284-1322). Horizontal pass:
// rows of `rows` pixels, output column fastest.
struct TapTable {
  const int* j0;
  const int* w0;
  const int* cnt;
  const float* w;
  const float* wsum;
};

__global__ void resize_h_kernel(int64_t total, int c, int win, int wout, TapTable t, const float* __restrict__ src,
                                int64_t ss, float* __restrict__ dst, int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= total) return;  // total = rows * wout * c
  int64_t p = i / c;
  int ch = int(i - p * c);
  int64_t row = p / wout;
  int xo = int(p - row * wout);
  int j0 = t.j0[xo], w0 = t.w0[xo], n = t.cnt[xo];
  const float* s = src + (row * win + j0) * ss + ch;
  float acc = 0.0f;
  for (int k = 0; k < n; ++k) acc = __fadd_rn(acc, __fmul_rn(t.w[w0 + k], s[k * ss]));
  float sm = t.wsum[xo];
  dst[p * sd + ch] = sm > 0.0f ? __fdiv_rn(acc, sm) : acc;
}

__global__ void resize_v_kernel(int64_t total, int c, int hin, int hout, int wout, TapTable t,
                                const float* __restrict__ src, int64_t ss, float* __restrict__ dst, int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= total) return;  // total = hout * wout * c
  int64_t p = i / c;
  int ch = int(i - p * c);
  int yo = int(p / wout);
  int64_t x = p - int64_t(yo) * wout;
  int j0 = t.j0[yo], w0 = t.w0[yo], n = t.cnt[yo];
  const float* s = src + (int64_t(j0) * wout + x) * ss + ch;
  float acc = 0.0f;
  for (int k = 0; k < n; ++k) acc = __fadd_rn(acc, __fmul_rn(t.w[w0 + k], s[int64_t(k) * wout * ss]));
  float sm = t.wsum[yo];
  dst[p * sd + ch] = sm > 0.0f ? __fdiv_rn(acc, sm) : acc;
}

// [c][p] <-> [p][c] at the boundary (host images are NCHW).
__global__ void nchw_to_nhwc_kernel(int64_t npix, int c, const float* __restrict__ src, float* __restrict__ dst,
                                    int64_t sd) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= npix * c) return;
  int64_t ch = i / npix, p = i - ch * npix;
  dst[p * sd + ch] = src[i];
}

__global__ void nhwc_to_nchw_kernel(int64_t npix, int c, const float* __restrict__ src, int64_t ss,
                                    float* __restrict__ dst) {
  int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= npix * c) return;
  int64_t ch = i / npix, p = i - ch * npix;
  dst[i] = src[p * ss + ch];
}

// ---------------------------------------------------------------------------
// SIMT contraction: D[m][n] = init(m, n) + sum_k A(m, k) B(k, n) over a
// problem object that supplies the operand addressing (implicit GEMM). Used
// for the ops the tensor-core kernels do not take.
template <int BM, int BN, int TM, int TN, class Prob>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) simt_gemm_kernel(Prob pr) {
  constexpr int BK = 16, NT = (BM / TM) * (BN / TN);
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int z = blockIdx.z;
  const int64_t m0 = int64_t(blockIdx.x) * BM;
  const int n0 = blockIdx.y * BN;
  const int tid = threadIdx.x, tm = tid / (BN / TN), tn = tid % (BN / TN);
  const int64_t M = pr.M;
  const int N = pr.N, K = pr.K;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int64_t m = m0 + tm * TM + i;
      int n = n0 + tn * TN + j;
      acc[i][j] = (m < M && n < N) ? pr.init(z, m, n) : 0.0f;
    }
  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int e = tid; e < BM * BK; e += NT) {
      int kk = e % BK, mm = e / BK;
      int64_t m = m0 + mm;
      int k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? pr.a(z, m, k) : 0.0f;
    }
    for (int e = tid; e < BN * BK; e += NT) {
      int kk = e % BK, nn = e / BK;
      int n = n0 + nn, k = k0 + kk;
      Bs[kk][nn] = (n < N && k < K) ? pr.b(z, k, n) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][tm * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tn * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int64_t m = m0 + tm * TM + i;
      int n = n0 + tn * TN + j;
      if (m < M && n < N) pr.store(z, m, n, acc[i][j]);
    }
}

// 1x1 conv / Dense: y[m][n] = b[n] + sum_k x[m][k] W[n][k].
struct ProbConv1x1 {
  const float* x;
  int64_t sx;
  const float* w;  // [c_out][c_in]
  const float* bias;
  float* y;
  int64_t sy;
  int64_t M;
  int N, K;
  __device__ float a(int, int64_t m, int k) const { return x[m * sx + k]; }
  __device__ float b(int, int k, int n) const { return w[int64_t(n) * K + k]; }
  __device__ float init(int, int64_t, int n) const { return bias ? bias[n] : 0.0f; }
  __device__ void store(int, int64_t m, int n, float v) const { y[m * sy + n] = v; }
};

// A 1x1 conv over a handful of pixels (the channel-attention convs run on
// the 1x1 squeeze): one block per pixel and 128 outputs, the pixel's inputs
// staged in shared memory, each thread one output's sum - the bias, then
// c_in ascending (fused multiply-adds) - and the unary tail (EW_LRELU /
// EW_SIGMOID / EW_GELU, or none). W is [c_in][c_out], so a warp's weight
// reads are consecutive.
// With `stage_w`, the block first copies its [K][<=128] slice of W into
// shared memory in one coalesced sweep, so the sums wait on one round trip
// rather than one per k.
__global__ void __launch_bounds__(128) conv1x1_small_kernel(int K, int N, const float* __restrict__ x, int64_t sx,
                                                            const float* __restrict__ wt,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int64_t sy, int tail, float slope, int stage_w) {
  extern __shared__ float xs[];  // K inputs, then (stage_w) K x nb weights
  const int m = blockIdx.x, n0 = blockIdx.y * 128, n = n0 + threadIdx.x, nb = min(128, N - n0);
  float* ws = xs + K;
  for (int k = threadIdx.x; k < K; k += 128) xs[k] = x[int64_t(m) * sx + k];
  if (stage_w)
    for (int i = threadIdx.x; i < K * nb; i += 128) {
      const int k = i / nb, j = i - k * nb;
      ws[i] = wt[int64_t(k) * N + n0 + j];
    }
  __syncthreads();
  if (n >= N) return;
  float a = bias ? bias[n] : 0.0f;
  if (stage_w) {
    for (int k = 0; k < K; ++k) a = fmaf(xs[k], ws[k * nb + threadIdx.x], a);
  } else {
    for (int k = 0; k < K; ++k) a = fmaf(xs[k], wt[int64_t(k) * N + n], a);
  }
  if (tail == EW_LRELU) a = a >= 0.0f ? a : slope * a;
  else if (tail == EW_SIGMOID) a = sigmoid_f(a);
  else if (tail == EW_GELU) a = gelu_f(a);
  y[int64_t(m) * sy + n] = a;
}

// k x k conv, stride s, padding (pt, pl): k = tap * c_in + ci, tap = ky*ks + kx,
// the reference's (ky, kx, ic) order. W is [c_out][tap][c_in].
struct ProbConvKxK {
  const float* x;
  int64_t sx;
  const float* w;
  const float* bias;
  float* y;
  int64_t sy;
  int64_t M;
  int N, K;
  int ci, h, wd, oh, ow, ks, stride, pt, pl;
  __device__ float a(int, int64_t m, int k) const {
    int oy = int(m / ow), ox = int(m - int64_t(oy) * ow);
    int tap = k / ci, c = k - tap * ci;
    int ky = tap / ks, kx = tap - ky * ks;
    int iy = oy * stride + ky - pt, ix = ox * stride + kx - pl;
    if (iy < 0 || iy >= h || ix < 0 || ix >= wd) return 0.0f;
    return x[(int64_t(iy) * wd + ix) * sx + c];
  }
  __device__ float b(int, int k, int n) const { return w[int64_t(n) * K + k]; }
  __device__ float init(int, int64_t, int n) const { return bias ? bias[n] : 0.0f; }
  __device__ void store(int, int64_t m, int n, float v) const { y[m * sy + n] = v; }
};

// ConvTranspose 2x2 stride 2: n = tap * c_out + o, W is [tap*c_out + o][c_in];
// the bias is added last, as the reference does.
struct ProbConvT {
  const float* x;
  int64_t sx;
  const float* w;
  const float* bias;
  float* y;
  int64_t sy;
  int64_t M;
  int N, K;
  int co, wd;
  __device__ float a(int, int64_t m, int k) const { return x[m * sx + k]; }
  __device__ float b(int, int k, int n) const { return w[int64_t(n) * K + k]; }
  __device__ float init(int, int64_t, int) const { return 0.0f; }
  __device__ void store(int, int64_t m, int n, float v) const {
    int tap = n / co, o = n - tap * co;
    int ky = tap >> 1, kx = tap & 1;
    int64_t yy = m / wd, xx = m - yy * wd;
    float bv = bias ? bias[o] : 0.0f;
    y[((2 * yy + ky) * (2 * wd) + 2 * xx + kx) * sy + o] = bv + v;
  }
};

// Gating Dense over the grid axis (mode 0) of a blocked [gg][pp] pixel
// buffer: out[a][q][c] = bias[a] + sum_t W[a][t] x[t][q][c]; n = q * c + ch.
struct ProbGate0 {
  const float* x;
  int64_t sx;
  const float* w;  // [gg][gg], [out][in]
  const float* bias;
  float* y;
  int64_t sy;
  int64_t M;
  int N, K;
  int c, pp;
  __device__ float a(int, int64_t m, int k) const { return w[m * K + k]; }
  __device__ float b(int, int k, int n) const {
    int q = n / c, ch = n - q * c;
    return x[(int64_t(k) * pp + q) * sx + ch];
  }
  __device__ float init(int, int64_t m, int) const { return bias ? bias[m] : 0.0f; }
  __device__ void store(int, int64_t m, int n, float v) const {
    int q = n / c, ch = n - q * c;
    y[(m * pp + q) * sy + ch] = v;
  }
};

// Gating Dense over the within-block axis (mode 1), batched over the blocks:
// out[g][a][c] = bias[a] + sum_t W[a][t] x[g][t][c].
struct ProbGate1 {
  const float* x;
  int64_t sx;
  const float* w;  // [pp][pp]
  const float* bias;
  float* y;
  int64_t sy;
  int64_t M;
  int N, K;
  int pp;
  __device__ float a(int, int64_t m, int k) const { return w[m * K + k]; }
  __device__ float b(int g, int k, int n) const { return x[(int64_t(g) * pp + k) * sx + n]; }
  __device__ float init(int, int64_t m, int) const { return bias ? bias[m] : 0.0f; }
  __device__ void store(int g, int64_t m, int n, float v) const { y[(int64_t(g) * pp + m) * sy + n] = v; }
};

}  // namespace mx
