// Tensor-core implicit-GEMM convolution for sm_100a: tcgen05.mma kind::tf32
// with FP32 accumulators in TMEM, operands staged by TMA.
//
//   D[pixel][co] = bias[co] + sum_{tap, ci} X[pixel + off(tap)][ci] * W[co][tap][ci]
//
// covers the 1x1 convs / Dense channel mixing (TAPS = 1, pixels as a flat
// M axis) and the 3x3 pad-1 convs (TAPS = 9, 8x16-pixel tiles, each tap a
// shifted 3-D TMA box whose out-of-image part TMA fills with zeros - the
// padding costs nothing).
//
// Precision: each product is computed as a 3-pass TF32 split,
//   a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi,
// with a_hi exactly representable in TF32 (low 13 mantissa bits cleared) and
// a_lo = a - a_hi, so the sum carries ~21 significant bits per product and
// accumulates in FP32 - the fp32 accuracy class the parity bars need (plain
// TF32 measured 46-48 dB against the fp32 CPU path under the He-normal init,
// below the 50 dB bar). The weights' hi / lo pair is split on the host.
//
// Warp roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box (16 KB), B and B_lo blocks per k-block
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2-5   split: A -> (A_hi in place, A_lo beside it) per k-block
//   warps 6-9   epilogue: TMEM -> registers -> +bias -> swizzled smem -> TMA store
// Two TMEM accumulators let the epilogue of tile i overlap the MMAs of i+1.
#pragma once

#include <cuda.h>

#include "sm100.cuh"

namespace mx {

struct UmmaConvParams {
  int tiles;       // output tiles (128 pixels each)
  int tiles_x;     // TAPS == 9: tiles per image row (width / 16)
  int kb_per_tap;  // c_in / 32
  int c_in;
  const float* bias;  // [c_out] or null
  int* status;        // device status word (0 = ok)
};

template <int N>
struct UmmaCfg {
  static constexpr int STAGES = N <= 64 ? 4 : (N <= 128 ? 3 : 2);
  static constexpr int A_BYTES = 128 * 128;  // 128 rows x 32 fp32
  static constexpr int B_BYTES = N * 128;    // N rows x 32 fp32
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGING_BYTES = 2 * 128 * 128;
  static constexpr int TMEM_COLS = 2 * N;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + 8 * (3 * STAGES + 4) + 16;
};

enum : int {
  kErrProducer = 0x101,
  kErrSplit = 0x102,
  kErrMmaAcc = 0x103,
  kErrMmaLo = 0x104,
  kErrEpilogue = 0x105,
};

template <int N, int TAPS>
__global__ void __launch_bounds__(320, 1)
    umma_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmD,
                     UmmaConvParams p) {
  using C = UmmaCfg<N>;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = base + C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
  uint64_t* lo_ready = full + C::STAGES;
  uint64_t* empty = lo_ready + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int abort_flag;
  const volatile int* vabort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = TAPS * p.kb_per_tap;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&lo_ready[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    tma_prefetch(&tmBlo);
    tma_prefetch(&tmD);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&](int code) {
    atomicCAS(p.status, 0, code);
    abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x) {
        int m0 = 0, x0 = 0, y0 = 0;
        if (TAPS == 1) {
          m0 = t * 128;
        } else {
          y0 = (t / p.tiles_x) * 8;
          x0 = (t % p.tiles_x) * 16;
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, vabort)) {
            fail(kErrProducer);
            break;
          }
          uint8_t* st = base + s * C::STAGE_BYTES;
          const int tap = kb / p.kb_per_tap, cb = kb % p.kb_per_tap;
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + 2 * C::B_BYTES);
          if (TAPS == 1) {
            tma_load_2d(st, &tmA, &full[s], cb * 32, m0);
          } else {
            const int ky = tap / 3, kx = tap % 3;
            tma_load_3d(st, &tmA, &full[s], cb * 32, x0 + kx - 1, y0 + ky - 1);
          }
          const int kcol = tap * p.c_in + cb * 32;
          tma_load_2d(st + 2 * C::A_BYTES, &tmB, &full[s], kcol, 0);
          tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, &tmBlo, &full[s], kcol, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, N, 0, 0);
      uint32_t it = 0, tc = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
        const uint32_t acc = tc & 1, aph = (tc >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1, vabort)) {
          fail(kErrMmaAcc);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * N;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&lo_ready[s], ph, vabort)) {
            fail(kErrMmaLo);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(base + s * C::STAGE_BYTES);
          const uint32_t alo = a + C::A_BYTES, b = a + 2 * C::A_BYTES, blo = b + C::B_BYTES;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = desc_kmajor_sw128(a + 32 * k), dalo = desc_kmajor_sw128(alo + 32 * k);
            const uint64_t db = desc_kmajor_sw128(b + 32 * k), dblo = desc_kmajor_sw128(blo + 32 * k);
            mma_tf32(d, dalo, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            mma_tf32(d, da, dblo, idesc, 1u);
            mma_tf32(d, da, db, idesc, 1u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ split
    const int tid = threadIdx.x - 64;  // 0..127
    uint32_t it = 0;
    for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1;
        if (!mbar_wait(&full[s], ph, vabort)) {
          fail(kErrSplit);
          ok = false;
          break;
        }
        float4* a = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES) + tid * 8;
        float4* alo = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES + C::A_BYTES) + tid * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 v = a[i], h, l;
          h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
          h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
          h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
          h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
          l.x = v.x - h.x;
          l.y = v.y - h.y;
          l.z = v.z - h.z;
          l.w = v.w - h.w;
          a[i] = h;
          alo[i] = l;
        }
        fence_proxy_async_smem();
        mbar_arrive(&lo_ready[s]);
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 192;  // 0..127
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;     // tile row (pixel) this thread owns
    uint32_t tc = 0;
    int chunk = 0;
    for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
      const uint32_t acc = tc & 1, aph = (tc >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], aph, vabort)) {
        fail(kErrEpilogue);
        break;
      }
      tc_fence_after();
      int m0 = 0, x0 = 0, y0 = 0;
      if (TAPS == 1) {
        m0 = t * 128;
      } else {
        y0 = (t / p.tiles_x) * 8;
        x0 = (t % p.tiles_x) * 16;
      }
#pragma unroll 1
      for (int j = 0; j < N / 32; ++j, ++chunk) {
        float v[32];
        tmem_ld32(tmem + (uint32_t(q * 32) << 16) + acc * N + j * 32, v);
        if (p.bias) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + j * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float4 b = __ldg(b4 + i);
            v[4 * i] += b.x;
            v[4 * i + 1] += b.y;
            v[4 * i + 2] += b.z;
            v[4 * i + 3] += b.w;
          }
        }
        uint8_t* sb = staging + (chunk & 1) * (128 * 128);
        named_bar(1, 128);  // the buffer's previous store has been read (see below)
        float4* rowp = reinterpret_cast<float4*>(sb + row * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) rowp[i ^ (row & 7)] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        fence_proxy_async_smem();
        named_bar(1, 128);
        if (et == 0) {
          if (TAPS == 1) tma_store_2d(&tmD, sb, j * 32, m0);
          else tma_store_3d(&tmD, sb, j * 32, x0, y0);
          bulk_commit();
          bulk_wait_read<1>();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
    if (et == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace mx
