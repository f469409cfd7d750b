// Tensor-core contractions for sm_100a: tcgen05.mma kind::tf32 with FP32
// accumulators in TMEM, operands staged by TMA (no multicast).
//
// One persistent kernel, three problem shapes (MODE):
//   MODE_CONV1  1x1 conv / Dense:  D[pix][co] = b[co] + sum_ci X[pix][ci] W[co][ci]
//               M = 128 pixels of the flat pixel axis, K = c_in
//   MODE_CONV3  3x3 pad-1 conv:    K = (tap, ci); each tap's A block is a
//               shifted 3-D TMA box (8 rows x 16 columns x 32 channels) whose
//               out-of-image part TMA fills with zeros - the padding is free
//   MODE_GATE   gMLP gating Dense over a spatial axis of a blocked buffer:
//               D[(grp, c)][a] = b[a] + sum_t X[grp, t][c] W[a][t]
//               (MODE_GATE / MODE_GATE_GRID)
//               M = 4 groups x 32 channels, N = a, K = t. The activation is
//               the MN-major operand: for each t, 32 channels are contiguous
//               in NHWC, which is one 128-byte row of the canonical SW128
//               MN-major atom; the 3-D box (32 ch, 32 t, 4 groups) lands
//               exactly in that layout. Block gating (t = position inside a
//               block) and grid gating (t = the cell) differ only in the
//               tensor map's strides.
//
// Precision: every product is a 3-pass TF32 split,
//   a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi,
// with a_hi = a rounded to the nearest TF32 value and a_lo = a - a_hi rounded
// to TF32 again, so each product carries ~22 significant bits (plain TF32
// measured 46-48 dB against the fp32 CPU path under the He-normal init, below
// the 50 dB bar). Weights are split on the host, activations in the kernel.
// The hi*hi products and the two cross terms accumulate in separate TMEM
// regions, added in fp32 by the epilogue: the tensor core rounds its fp32
// accumulator at every MMA, and with one region the full-size running sum
// took three such roundings per k-step instead of one.
//
// Warp roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A block (16 KB), B and B_lo blocks per k-block
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2-5   split: A -> (A_hi in place, A_lo beside it) per k-block
//   warps 6-9   epilogue: TMEM -> registers -> +bias -> swizzled smem -> TMA store
// Two accumulator sets (N <= 128) let the epilogue of tile i overlap the MMAs
// of tile i+1; N = 256 has room for one set only.
// Every mbarrier wait is bounded in time; a wait that runs out records a code
// in the status word, the kernel unwinds and frees its TMEM.
#pragma once

#include <cuda.h>

#include "sm100.cuh"

namespace mx {

// MODE_GATE: block gating (t = position inside a block, groups = blocks);
// MODE_GATE_GRID: grid gating (t = the cell, groups = positions in a cell).
// The grid case loads and stores its 4 groups as 4 separate boxes so every
// tensor map keeps its strides in ascending order.
// MODE_CONV4: the 4x4 stride-2 SAME conv (Conv_down); its A box is read with
// a TMA traversal stride of 2 in both spatial dimensions.
enum : int { MODE_CONV1 = 0, MODE_CONV3 = 1, MODE_GATE = 2, MODE_GATE_GRID = 3, MODE_CONV4 = 4 };

struct UmmaConvParams {
  int tiles;       // output tiles
  int tiles_x;     // CONV3: tiles per image row (width / 16); GATE: group tiles (ceil(groups / 4))
  int kb_per_tap;  // k-blocks (of 32) per tap
  int c_in;        // K per tap (CONV) / K (GATE)
  int groups;      // GATE_GRID: positions per cell (boxes past it are skipped)
  int pad_t, pad_l;  // CONV4: SAME padding before the first row / column
  const float* bias;  // per output column, or null
  int* status;        // device status word (0 = ok)
};

template <int N>
struct UmmaCfg {
  static constexpr int STAGES = N <= 64 ? 4 : (N <= 128 ? 3 : 2);
  static constexpr int A_BYTES = 128 * 128;  // 128 rows x 32 fp32
  static constexpr int B_BYTES = N * 128;    // N rows x 32 fp32
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGING_BYTES = 2 * 128 * 128;
  // An accumulator set is two N-column fp32 regions: the hi*hi products and
  // the two cross terms, summed once in the epilogue. Sets are double
  // buffered (the epilogue drains one tile while the next accumulates) where
  // two fit in the 512 TMEM columns.
  static constexpr int ACC_SETS = 4 * N <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = ACC_SETS * 2 * N;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + 8 * (3 * STAGES + 4) + 16;
};

enum : int {
  kErrProducer = 0x101,
  kErrSplit = 0x102,
  kErrMmaAcc = 0x103,
  kErrMmaLo = 0x104,
  kErrEpilogue = 0x105,
};

// Round an fp32 value to the nearest TF32 value (ties to even), returned as
// fp32 with the low 13 mantissa bits clear, so the tensor core reads it
// exactly whatever it does with those bits. Finite inputs here are far below
// the overflow threshold, so the carry never reaches the exponent's top.
__device__ __forceinline__ float tf32_rne(float v) {
  uint32_t b = __float_as_uint(v);
  b = (b + 0xFFFu + ((b >> 13) & 1u)) & 0xFFFFE000u;
  return __uint_as_float(b);
}

template <int N, int MODE>
__global__ void __launch_bounds__(320, 1)
    umma_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmD,
                     UmmaConvParams p) {
  using C = UmmaCfg<N>;
  using namespace sm100;
  constexpr int TAPS = MODE == MODE_CONV3 ? 9 : (MODE == MODE_CONV4 ? 16 : 1);
  constexpr bool SPATIAL = MODE == MODE_CONV3 || MODE == MODE_CONV4;  // 8x16-pixel output tiles
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

  // Tile t -> its origin: CONV1 (m0), CONV3 (x0, y0), GATE (group g0, channel block cc).
  auto decode = [&](int t, int& a0, int& a1) {
    if (MODE == MODE_CONV1) {
      a0 = t * 128;
      a1 = 0;
    } else if (SPATIAL) {
      a0 = (t % p.tiles_x) * 16;
      a1 = (t / p.tiles_x) * 8;
    } else {
      a0 = (t % p.tiles_x) * 4;  // first group of the tile
      a1 = (t / p.tiles_x) * 32;  // first channel
    }
  };

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
        int a0, a1;
        decode(t, a0, a1);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, vabort)) {
            fail(kErrProducer);
            break;
          }
          uint8_t* st = base + s * C::STAGE_BYTES;
          const int tap = kb / p.kb_per_tap, cb = kb % p.kb_per_tap;
          int a_bytes = C::A_BYTES;
          if (MODE == MODE_GATE_GRID) a_bytes = 4096 * min(4, p.groups - a0);
          mbar_arrive_expect_tx(&full[s], a_bytes + 2 * C::B_BYTES);
          if (MODE == MODE_CONV1) {
            tma_load_2d(st, &tmA, &full[s], cb * 32, a0);
          } else if (MODE == MODE_CONV3) {
            const int ky = tap / 3, kx = tap % 3;
            tma_load_3d(st, &tmA, &full[s], cb * 32, a0 + kx - 1, a1 + ky - 1);
          } else if (MODE == MODE_CONV4) {
            // Output pixel (oy, ox) reads input (2oy + ky - pt, 2ox + kx - pl):
            // the tensor map steps 2 input pixels per box element.
            const int ky = tap >> 2, kx = tap & 3;
            tma_load_3d(st, &tmA, &full[s], cb * 32, 2 * a0 + kx - p.pad_l, 2 * a1 + ky - p.pad_t);
          } else if (MODE == MODE_GATE) {
            tma_load_3d(st, &tmA, &full[s], a1, kb * 32, a0);
          } else {
            // A box past the last position would read nothing; its rows
            // only feed accumulator rows that are never stored, so it is
            // skipped and the expected byte count below counts only real boxes.
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (a0 + g < p.groups) tma_load_3d(st + g * 4096, &tmA, &full[s], a1, a0 + g, kb * 32);
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
      constexpr bool GATE = MODE == MODE_GATE || MODE == MODE_GATE_GRID;
      constexpr uint32_t idesc = idesc_tf32(128, N, GATE ? 1 : 0, 0);
      uint32_t it = 0, tc = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
        const uint32_t acc = tc % C::ACC_SETS, aph = (tc / C::ACC_SETS) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1, vabort)) {
          fail(kErrMmaAcc);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * 2 * N, dx = d + N;
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
            uint64_t da, dalo;
            if (GATE) {
              // MN-major: k-step k covers K rows 8k..8k+7 of each 4 KB group block.
              da = desc_mnmajor_sw128_32b(a + 1024 * k, 4096);
              dalo = desc_mnmajor_sw128_32b(alo + 1024 * k, 4096);
            } else {
              da = desc_kmajor_sw128(a + 32 * k);
              dalo = desc_kmajor_sw128(alo + 32 * k);
            }
            const uint64_t db = desc_kmajor_sw128(b + 32 * k), dblo = desc_kmajor_sw128(blo + 32 * k);
            // The running sum of the hi*hi products takes one accumulator
            // update per k-step; the cross terms, about 2^-12 of its size,
            // go to their own region, so the accumulator's rounding at each
            // update is paid once per k-step at full magnitude, not three times.
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            mma_tf32(d, da, db, idesc, accum);
            mma_tf32(dx, dalo, db, idesc, accum);
            mma_tf32(dx, da, dblo, idesc, 1u);
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
        // Elementwise, so the layout does not matter; a warp touches 32
        // consecutive float4 (512 contiguous bytes) per access, which keeps
        // every shared-memory access free of bank conflicts.
        float4* a = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES) + tid;
        float4* alo = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES + C::A_BYTES) + tid;
#pragma unroll
        for (int i = 0; i < 8 * 128; i += 128) {
          float4 v = a[i], h, l;
          h.x = tf32_rne(v.x);
          h.y = tf32_rne(v.y);
          h.z = tf32_rne(v.z);
          h.w = tf32_rne(v.w);
          l.x = tf32_rne(v.x - h.x);
          l.y = tf32_rne(v.y - h.y);
          l.z = tf32_rne(v.z - h.z);
          l.w = tf32_rne(v.w - h.w);
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
    const int row = q * 32 + lane;     // accumulator row this thread owns
    uint32_t tc = 0;
    int chunk = 0;
    for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
      const uint32_t acc = tc % C::ACC_SETS, aph = (tc / C::ACC_SETS) & 1;
      if (!mbar_wait(&acc_full[acc], aph, vabort)) {
        fail(kErrEpilogue);
        break;
      }
      tc_fence_after();
      int a0, a1;
      decode(t, a0, a1);
#pragma unroll 1
      for (int j = 0; j < N / 32; ++j, ++chunk) {
        float v[32], x[32];
        const uint32_t col = tmem + (uint32_t(q * 32) << 16) + acc * 2 * N + j * 32;
        tmem_ld32(col, v);
        tmem_ld32(col + N, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += x[i];
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
        if (MODE == MODE_GATE || MODE == MODE_GATE_GRID) {
          // Staging is [group][a][channel]: this thread (group q, channel
          // lane) writes one float into each of its group's 32 rows.
          float* g = reinterpret_cast<float*>(sb + q * 4096);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int r = q * 32 + i;  // row within the 128-row staging tile
            g[i * 32 + (((lane >> 2) ^ (r & 7)) << 2) + (lane & 3)] = v[i];
          }
        } else {
          float4* rowp = reinterpret_cast<float4*>(sb + row * 128);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            rowp[i ^ (row & 7)] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
        fence_proxy_async_smem();
        named_bar(1, 128);
        if (et == 0) {
          if (MODE == MODE_CONV1) tma_store_2d(&tmD, sb, j * 32, a0);
          else if (SPATIAL) tma_store_3d(&tmD, sb, j * 32, a0, a1);
          else if (MODE == MODE_GATE) tma_store_3d(&tmD, sb, a1, j * 32, a0);
          else
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (a0 + g < p.groups) tma_store_3d(&tmD, sb + g * 4096, a1, a0 + g, j * 32);
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
