// Memory-bound op kernels, vectorised: every thread moves 16 bytes per access
// and consecutive threads touch consecutive addresses, with 32-bit index
// arithmetic (every tensor here has fewer than 2^31 elements; the host checks).
//
// These take the executor's NHWC views when channels come in multiples of 4
// and views are 16-byte aligned; the scalar kernels in kernels_simt.cuh cover
// everything else.
#pragma once

#include "gpu_common.cuh"

namespace mx {
// Internal linkage: more than one translation unit includes these kernels.
namespace {

// Space <-> blocked permutation of whole pixels, 4 channels per thread
// (src/exec_cpu.rs:1078-1103; blocked index e = g * psz + q).
__global__ void block_perm4_kernel(int total4, int c4, int wd, int gw, int fh, int fw, int gsz, int psz, int swap,
                                   int forward, const float* __restrict__ src, int ss, float* __restrict__ dst,
                                   int sd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total4) return;
  int e = i / c4;
  int ch = (i - e * c4) * 4;
  int g, q;
  if (swap) {
    q = e / gsz;
    g = e - q * gsz;
  } else {
    g = e / psz;
    q = e - g * psz;
  }
  int gy = g / gw, gx = g - gy * gw, fy = q / fw, fx = q - fy * fw;
  int pix = (gy * fh + fy) * wd + gx * fw + fx;
  if (forward)
    *reinterpret_cast<float4*>(dst + size_t(e) * sd + ch) =
        *reinterpret_cast<const float4*>(src + size_t(pix) * ss + ch);
  else
    *reinterpret_cast<float4*>(dst + size_t(pix) * sd + ch) =
        *reinterpret_cast<const float4*>(src + size_t(e) * ss + ch);
}

// Channel LayerNorm of P pixels per 128-thread block. The block's pixels are
// staged through shared memory (rows padded to C+1 floats so a thread walking
// its own row is conflict-free), then each pixel's statistics are taken
// serially in channel order - the reference's exact order (s1, s2 ascending,
// m = s1/c, var = s2/c - m*m, rstd = 1/sqrt(max(var,0)+eps),
// y = (x-m)*rstd*w + b; src/exec_cpu.rs:396-433) - with non-contracting
// intrinsics, so the result is bit-identical to the CPU path.
template <int C>
__global__ void __launch_bounds__(128) chan_ln_tile_kernel(int npix, const float* __restrict__ x, int sx,
                                                           const float* __restrict__ w, const float* __restrict__ b,
                                                           float* __restrict__ y, int sy, float eps) {
  constexpr int P = C <= 64 ? 128 : (C == 128 ? 64 : 32);
  constexpr int C4 = C / 4, R = C + 1;
  extern __shared__ float tile[];  // P * R, then P (mean, rstd) pairs
  float2* st = reinterpret_cast<float2*>(tile + ((P * R + 1) & ~1));
  const int p0 = blockIdx.x * P;
  const int np = min(P, npix - p0);
  for (int idx = threadIdx.x; idx < np * C4; idx += 128) {
    int r = idx / C4, c = (idx - r * C4) * 4;
    float4 v = *reinterpret_cast<const float4*>(x + size_t(p0 + r) * sx + c);
    float* t = tile + r * R + c;
    t[0] = v.x;
    t[1] = v.y;
    t[2] = v.z;
    t[3] = v.w;
  }
  __syncthreads();
  // The statistics, one pixel per thread, serially in channel order.
  if (threadIdx.x < np) {
    const float* t = tile + threadIdx.x * R;
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 8
    for (int i = 0; i < C; ++i) {
      float v = t[i];
      s1 = __fadd_rn(s1, v);
      s2 = __fadd_rn(s2, __fmul_rn(v, v));
    }
    const float nf = float(C);
    float m = __fdiv_rn(s1, nf);
    float var = __fsub_rn(__fdiv_rn(s2, nf), __fmul_rn(m, m));
    float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), eps)));
    st[threadIdx.x] = make_float2(m, rstd);
  }
  __syncthreads();
  // The normalisation, spread over all threads four channels at a time:
  // ((x - m) * rstd) * w + b, each operation rounded on its own (paired).
  for (int idx = threadIdx.x; idx < np * C4; idx += 128) {
    const int r = idx / C4, c = (idx - r * C4) * 4;
    const float* t = tile + r * R + c;
    const float2 ms = st[r];
    const float4 wv = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 bv = __ldg(reinterpret_cast<const float4*>(b + c));
    const uint64_t mm = f2_pack(ms.x, ms.x), rr = f2_pack(ms.y, ms.y);
    float4 o;
    f2_unpack(f2_add_after_mul(f2_mul(f2_mul(f2_sub(f2_pack(t[0], t[1]), mm), rr), f2_pack(wv.x, wv.y)),
                               f2_pack(bv.x, bv.y)),
              o.x, o.y);
    f2_unpack(f2_add_after_mul(f2_mul(f2_mul(f2_sub(f2_pack(t[2], t[3]), mm), rr), f2_pack(wv.z, wv.w)),
                               f2_pack(bv.z, bv.w)),
              o.z, o.w);
    *reinterpret_cast<float4*>(y + size_t(p0 + r) * sy + c) = o;
  }
}

// The statistics half of the same LayerNorm, for a consumer that normalises
// on load: per pixel (mean, 1 / sqrt(max(var, 0) + eps)) as two floats,
// computed exactly as chan_ln_tile_kernel computes them.
template <int C>
__global__ void __launch_bounds__(128) chan_stats_tile_kernel(int npix, const float* __restrict__ x, int sx,
                                                              float2* __restrict__ stats, float eps) {
  constexpr int P = C <= 64 ? 128 : (C == 128 ? 64 : 32);
  constexpr int C4 = C / 4, R = C + 1;
  extern __shared__ float tile[];  // P * R
  const int p0 = blockIdx.x * P;
  const int np = min(P, npix - p0);
  for (int idx = threadIdx.x; idx < np * C4; idx += 128) {
    int r = idx / C4, c = (idx - r * C4) * 4;
    float4 v = *reinterpret_cast<const float4*>(x + size_t(p0 + r) * sx + c);
    float* t = tile + r * R + c;
    t[0] = v.x;
    t[1] = v.y;
    t[2] = v.z;
    t[3] = v.w;
  }
  __syncthreads();
  if (threadIdx.x < np) {
    const float* t = tile + threadIdx.x * R;
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 8
    for (int i = 0; i < C; ++i) {
      float v = t[i];
      s1 = __fadd_rn(s1, v);
      s2 = __fadd_rn(s2, __fmul_rn(v, v));
    }
    const float nf = float(C);
    float m = __fdiv_rn(s1, nf);
    float var = __fsub_rn(__fdiv_rn(s2, nf), __fmul_rn(m, m));
    float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), eps)));
    stats[p0 + threadIdx.x] = make_float2(m, rstd);
  }
}

// Per-channel mean over the pixels (the CALayer squeeze) in two deterministic
// phases: block b sums its own pixel range per channel into part[b][c];
// then one thread per channel adds the blocks' partials in block order.
// 256 threads = R pixel rows x C4 channel quads.
__global__ void __launch_bounds__(256) chan_mean_partial_kernel(int npix, int c4, int per_block,
                                                                const float* __restrict__ x, int sx,
                                                                float* __restrict__ part) {
  __shared__ float4 red[256];
  const int rows = 256 / c4;
  const int r = threadIdx.x / c4, q = threadIdx.x - r * c4;
  const int p0 = blockIdx.x * per_block, p1 = min(npix, p0 + per_block);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r < rows)
    for (int p = p0 + r; p < p1; p += rows) {
      float4 v = *reinterpret_cast<const float4*>(x + size_t(p) * sx + q * 4);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  red[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x < c4) {
    float4 t = red[threadIdx.x];
    for (int k = 1; k < rows; ++k) {
      float4 u = red[k * c4 + threadIdx.x];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    *reinterpret_cast<float4*>(part + size_t(blockIdx.x) * c4 * 4 + threadIdx.x * 4) = t;
  }
}

__global__ void chan_mean_final_kernel(int nblocks, int c, int npix, const float* __restrict__ part,
                                       float* __restrict__ out) {
  int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= c) return;
  float s = 0.0f;
  for (int b = 0; b < nblocks; ++b) s += part[size_t(b) * c + ch];
  out[ch] = s / float(npix);
}

// The same second phase with one block per channel: each of 256 threads sums
// a fixed stride of the partials, then a fixed shared-memory tree adds the
// threads' sums, so the result is deterministic and the serial chain is
// nblocks / 256 adds instead of nblocks.
__global__ void __launch_bounds__(256) chan_mean_final_tree_kernel(int nblocks, int c, int npix,
                                                                   const float* __restrict__ part,
                                                                   float* __restrict__ out) {
  __shared__ float red[256];
  const int ch = blockIdx.x;
  float s = 0.0f;
  for (int b = threadIdx.x; b < nblocks; b += 256) s += part[size_t(b) * c + ch];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[ch] = red[0] / float(npix);
}

// out[p][c] = x[p][c] * s[c], 4 channels per thread.
__global__ void chan_scale4_kernel(int total4, int c4, const float* __restrict__ x, int sx,
                                   const float* __restrict__ s, float* __restrict__ d, int sd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total4) return;
  int p = i / c4, c = (i - p * c4) * 4;
  float4 v = *reinterpret_cast<const float4*>(x + size_t(p) * sx + c);
  float4 g = *reinterpret_cast<const float4*>(s + c);
  *reinterpret_cast<float4*>(d + size_t(p) * sd + c) = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
}

// x * s + r (channel scale, then the residual add) in one pass, with the two
// roundings of the separate ops: no fused multiply-add.
__global__ void chan_scale_add4_kernel(int total4, int c4, const float* __restrict__ x, int sx,
                                       const float* __restrict__ s, const float* __restrict__ r, int sr,
                                       float* __restrict__ d, int sd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total4) return;
  int p = i / c4, c = (i - p * c4) * 4;
  float4 v = *reinterpret_cast<const float4*>(x + size_t(p) * sx + c);
  float4 g = *reinterpret_cast<const float4*>(s + c);
  float4 e = *reinterpret_cast<const float4*>(r + size_t(p) * sr + c);
  *reinterpret_cast<float4*>(d + size_t(p) * sd + c) =
      make_float4(__fadd_rn(__fmul_rn(v.x, g.x), e.x), __fadd_rn(__fmul_rn(v.y, g.y), e.y),
                  __fadd_rn(__fmul_rn(v.z, g.z), e.z), __fadd_rn(__fmul_rn(v.w, g.w), e.w));
}

// ((x * s) + r) + r2: the channel scale and two residual adds in one pass,
// each operation rounded on its own as the three separate ops round it.
__global__ void chan_scale_add2_4_kernel(int total4, int c4, const float* __restrict__ x, int sx,
                                         const float* __restrict__ s, const float* __restrict__ r, int sr,
                                         const float* __restrict__ r2, int sr2, float* __restrict__ d, int sd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total4) return;
  int p = i / c4, c = (i - p * c4) * 4;
  float4 v = *reinterpret_cast<const float4*>(x + size_t(p) * sx + c);
  float4 g = *reinterpret_cast<const float4*>(s + c);
  float4 e = *reinterpret_cast<const float4*>(r + size_t(p) * sr + c);
  float4 f = *reinterpret_cast<const float4*>(r2 + size_t(p) * sr2 + c);
  *reinterpret_cast<float4*>(d + size_t(p) * sd + c) =
      make_float4(__fadd_rn(__fadd_rn(__fmul_rn(v.x, g.x), e.x), f.x),
                  __fadd_rn(__fadd_rn(__fmul_rn(v.y, g.y), e.y), f.y),
                  __fadd_rn(__fadd_rn(__fmul_rn(v.z, g.z), e.z), f.z),
                  __fadd_rn(__fadd_rn(__fmul_rn(v.w, g.w), e.w), f.w));
}

// Resize passes, 4 channels per thread, same tap tables and the same
// per-channel arithmetic as the scalar kernels (acc over taps ascending with
// non-contracting ops, then acc / wsum if wsum > 0). One block row of threads
// per output row (blockIdx.y), channels in groups of 4 along x; c4 (channels
// / 4) is a power of two, 1 << lg4.
struct TapTable4 {
  const int* j0;
  const int* w0;
  const int* cnt;
  const float* w;
  const float* wsum;
  // 1 / wsum where wsum is an exact power of two (then acc * wrcp is acc /
  // wsum bit for bit), else 0: the division is only paid where the taps were
  // clipped at the border.
  const float* wrcp;
};

// acc += w * v per channel, the product and the sum each rounded (no fused
// multiply-add).
__device__ __forceinline__ void tap_acc(float4& acc, float w, float4 v) {
  acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
  acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
  acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
  acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
}
// The same as paired f32x2 instructions (the same roundings, half the
// instructions), where the registers allow.
__device__ __forceinline__ void tap_acc_x2(float4& acc, float w, float4 v) {
  const uint64_t ww = f2_pack(w, w);
  f2_unpack(f2_add_after_mul(f2_mul(ww, f2_pack(v.x, v.y)), f2_pack(acc.x, acc.y)), acc.x, acc.y);
  f2_unpack(f2_add_after_mul(f2_mul(ww, f2_pack(v.z, v.w)), f2_pack(acc.z, acc.w)), acc.z, acc.w);
}
__device__ __forceinline__ float4 tap_norm(float4 acc, float sm, float rcp) {
  if (rcp != 0.0f)
    return make_float4(__fmul_rn(acc.x, rcp), __fmul_rn(acc.y, rcp), __fmul_rn(acc.z, rcp), __fmul_rn(acc.w, rcp));
  if (sm > 0.0f)
    return make_float4(__fdiv_rn(acc.x, sm), __fdiv_rn(acc.y, sm), __fdiv_rn(acc.z, sm), __fdiv_rn(acc.w, sm));
  return acc;
}

// Both passes are bound by load latency (each thread's taps wait in turn),
// so they are held to 32 registers for eight 256-thread blocks per SM.
// Horizontal pass: dst row r (of hin), column xo, from src row r.
__global__ void __launch_bounds__(256, 8) resize_h4_kernel(int lg4, int win, int wout, TapTable4 t, const float* __restrict__ src, int ss,
                                 float* __restrict__ dst, int sd) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (wout << lg4)) return;
  const int row = blockIdx.y, xo = i >> lg4, c = (i & ((1 << lg4) - 1)) * 4;
  const int j0 = __ldg(t.j0 + xo), w0 = __ldg(t.w0 + xo), n = __ldg(t.cnt + xo);
  const float* s = src + (size_t(row) * win + j0) * ss + c;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < n; ++k) tap_acc(acc, __ldg(t.w + w0 + k), *reinterpret_cast<const float4*>(s + size_t(k) * ss));
  *reinterpret_cast<float4*>(dst + (size_t(row) * wout + xo) * sd + c) =
      tap_norm(acc, __ldg(t.wsum + xo), __ldg(t.wrcp + xo));
}

// Vertical pass: dst row yo (of hout) from rows j0.. of the horizontal result.
__global__ void __launch_bounds__(256, 8) resize_v4_kernel(int lg4, int wout, TapTable4 t, const float* __restrict__ src, int ss,
                                 float* __restrict__ dst, int sd) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (wout << lg4)) return;
  const int yo = blockIdx.y, x = i >> lg4, c = (i & ((1 << lg4) - 1)) * 4;
  const int j0 = __ldg(t.j0 + yo), w0 = __ldg(t.w0 + yo), n = __ldg(t.cnt + yo);
  const float* s = src + (size_t(j0) * wout + x) * ss + c;
  const size_t step = size_t(wout) * ss;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < n; ++k) tap_acc(acc, __ldg(t.w + w0 + k), *reinterpret_cast<const float4*>(s + k * step));
  *reinterpret_cast<float4*>(dst + (size_t(yo) * wout + x) * sd + c) =
      tap_norm(acc, __ldg(t.wsum + yo), __ldg(t.wrcp + yo));
}

// Both passes in one launch, for upsampling (at most kRzTaps taps a side).
// A CTA makes output rows [y0, y0 + kRzTY) of a strip of output columns
// holding kRzTile floats a row (all channels). It first computes, into shared
// memory, the horizontal pass of every input row those output rows read
// (exactly what resize_h4_kernel writes to the intermediate), then the
// vertical pass from there. Values and summation order are those of the two
// kernels above, so the result is bit for bit theirs; the intermediate never
// goes through DRAM. The host uses it only where every tile needs at most
// kRzRows input rows; the kernel clamps to that bound all the same.
constexpr int kRzTY = 16, kRzRows = 11, kRzTile = 1024, kRzTaps = 3;
__global__ void __launch_bounds__(256) resize_hv4_kernel(int lg4, int win, int wout, int hout, TapTable4 tx,
                                                         TapTable4 ty, const float* __restrict__ src, int ss,
                                                         float* __restrict__ dst, int sd) {
  __shared__ float4 rows[kRzRows][kRzTile / 4];
  // The vertical taps of the CTA's output rows, read once by one warp:
  // first input row (relative to r_lo), tap count, weights, sum, reciprocal.
  __shared__ int s_j[kRzTY], s_n[kRzTY];
  __shared__ float s_w[kRzTY][kRzTaps], s_sum[kRzTY], s_rcp[kRzTY];
  __shared__ int s_rlo, s_nrows;
  const int f = threadIdx.x;  // float4 of a strip row: column f >> lg4, channels 4 (f & (c4 - 1))
  const int xo = blockIdx.x * ((kRzTile / 4) >> lg4) + (f >> lg4), c = (f & ((1 << lg4) - 1)) * 4;
  const bool xin = xo < wout;
  const int y0 = blockIdx.y * kRzTY, ny = min(kRzTY, hout - y0);
  if (f < 32) {
    int j = 1 << 30, hi = -1;
    if (f < ny) {
      const int yo = y0 + f;
      j = __ldg(ty.j0 + yo);
      const int n = __ldg(ty.cnt + yo), w0 = __ldg(ty.w0 + yo);
      hi = j + n - 1;
      s_n[f] = n;
#pragma unroll
      for (int k = 0; k < kRzTaps; ++k) s_w[f][k] = k < n ? __ldg(ty.w + w0 + k) : 0.0f;
      s_sum[f] = __ldg(ty.wsum + yo);
      s_rcp[f] = __ldg(ty.wrcp + yo);
    }
    int lo = j;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (f < ny) s_j[f] = j - lo;
    if (f == 0) s_rlo = lo, s_nrows = min(hi - lo + 1, kRzRows);
  }
  __syncthreads();
  const int r_lo = s_rlo, nrows = s_nrows;
  static_assert(kRzTaps == 3, "the vertical pass is written for three taps");
  if (xin) {
    // Four input rows at a time, all their taps' loads issued before any is
    // used (the loads, not the arithmetic, are what a thread waits on).
    const int j0 = __ldg(tx.j0 + xo), w0 = __ldg(tx.w0 + xo), n = min(__ldg(tx.cnt + xo), kRzTaps);
    const float sm = __ldg(tx.wsum + xo), rc = __ldg(tx.wrcp + xo);
    float w[kRzTaps];
#pragma unroll
    for (int k = 0; k < kRzTaps; ++k) w[k] = k < n ? __ldg(tx.w + w0 + k) : 0.0f;
    const float* base = src + (size_t(r_lo) * win + j0) * ss + c;
    const size_t rstep = size_t(win) * ss;
    for (int r0 = 0; r0 < nrows; r0 += 4) {
      float4 v[4][kRzTaps];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float* s = base + size_t(min(r0 + q, nrows - 1)) * rstep;
#pragma unroll
        for (int k = 0; k < kRzTaps; ++k)
          v[q][k] = k < n ? *reinterpret_cast<const float4*>(s + k * ss) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (r0 + q >= nrows) break;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kRzTaps; ++k)
          if (k < n) tap_acc_x2(acc, w[k], v[q][k]);
        rows[r0 + q][f] = tap_norm(acc, sm, rc);
      }
    }
  }
  __syncthreads();
  // Vertical pass, one output row per warp at a time: the row's taps are
  // read once into registers and serve all 256 float4s of the strip row
  // (eight per lane), and each warp-wide store covers consecutive floats.
  const int warp = f >> 5, lane = f & 31;
  const int xs = blockIdx.x * ((kRzTile / 4) >> lg4);  // the strip's first column
  const int cmask = (1 << lg4) - 1;
  for (int yy = warp; yy < ny; yy += 8) {
    const int j0 = s_j[yy], n = s_n[yy];
    const float w0 = s_w[yy][0], w1 = s_w[yy][1], w2 = s_w[yy][2], sm = s_sum[yy], rc = s_rcp[yy];
    const bool t0 = n > 0 && j0 < nrows, t1 = n > 1 && j0 + 1 < nrows, t2 = n > 2 && j0 + 2 < nrows;
    const float4* r0 = rows[min(j0, kRzRows - 1)];
    const float4* r1 = rows[min(j0 + 1, kRzRows - 1)];
    const float4* r2 = rows[min(j0 + 2, kRzRows - 1)];
    float* drow = dst + size_t(y0 + yy) * wout * sd;
#pragma unroll 4
    for (int g = lane; g < kRzTile / 4; g += 32) {
      const int x = xs + (g >> lg4);
      if (x >= wout) break;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t0) tap_acc_x2(acc, w0, r0[g]);
      if (t1) tap_acc_x2(acc, w1, r1[g]);
      if (t2) tap_acc_x2(acc, w2, r2[g]);
      *reinterpret_cast<float4*>(drow + size_t(x) * sd + (g & cmask) * 4) = tap_norm(acc, sm, rc);
    }
  }
}

}  // namespace
}  // namespace mx
