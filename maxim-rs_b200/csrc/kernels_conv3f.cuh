// The 3x3 pad-1 conv with 32 input and 32 output channels on the tensor
// cores, its three column taps side by side in N.
//
// The column-shift kernel (MODE_CONV3H) issues 72 MMAs per 128 output
// pixels at N = 64 and 32, and at that width an MMA costs the same ~25 ns
// whatever its N, so the MMA issue sets that kernel's pace. Here one
// instruction multiplies an A tile by the weights of all three column taps of
// a tap row, N = 3 x 32: D_kx[p] = sum over (ky, ci) of in(row(p) + ky - 1,
// col(p))[ci] W[ky][kx][ci][:], for every input column p of the tile. The
// output pixel at column o of the tile is then
//     D_0[o] + D_1[o + 1] + D_2[o + 2],
// the partial sums of the two neighbouring input columns, which the epilogue
// thread of column o takes from its neighbours' lanes by warp shuffle.
//
// Tile: 4 output rows x 30 output columns. The A box is the 32 input columns
// x 6 input rows around it (TMA zero-fills outside the image), 192 K-major
// rows of 32 channels; tap row ky reads its rows 32 ky .. 32 ky + 127, so
// TMEM lane 32 r + c holds input column c of output row r. A tile issues
// 3 tap rows x 4 k-steps x 2 MMAs: A_hi x [B_hi | B_lo] at N' = 192 and A_lo x
// B_hi at N = 96 (the 3xTF32 split of the other tensor-core convs: the hi*hi
// products in TMEM columns [0, 96), the cross terms in [96, 192)).
//
// The weights (3 tap rows x hi/lo x 3 column taps x 32 outputs x 32 inputs,
// 72 KB) stay in shared memory for the whole launch; two stages hold A and
// its TF32 residual A_lo.
//
// Warp roles as in umma_conv_kernel: 0 TMA producer, 1 MMA issuer, 2-9 the
// A_lo split, 10-17 the epilogue (two accumulator sets of four warps; warp q
// of a set drains output row q). Every wait is bounded.
#pragma once

#include "kernels_umma.cuh"

namespace mx {

struct Conv3fCfg {
  static constexpr int OUT_W = 30, OUT_H = 4;              // output pixels of a tile
  static constexpr int BOX_W = 32, BOX_H = 6;              // the input box around them
  static constexpr int A_BYTES = BOX_W * BOX_H * 128;      // 192 rows of 32 fp32
  static constexpr int NF = 96;                            // 3 column taps x 32 outputs
  static constexpr int W_KY_BYTES = 2 * NF * 128;          // one tap row's B: hi rows, then lo rows
  static constexpr int W_BYTES = 3 * W_KY_BYTES;
  static constexpr int STAGES = 2;
  static constexpr int STAGE_BYTES = 2 * A_BYTES;          // A, then A_lo
  static constexpr int SPLIT = 8;
  static constexpr int ACC_SETS = 2;
  static constexpr int ACC_COLS = 2 * NF;                  // hi*hi region, then the cross terms
  static constexpr int EPI_WARPS = 4 * ACC_SETS;
  static constexpr int EPI_WARP0 = 2 + SPLIT;
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
  static constexpr int STAGING_BYTES = EPI_WARPS * 4096;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES =
      1024 + W_BYTES + STAGES * STAGE_BYTES + STAGING_BYTES + 8 * (3 * STAGES + 2 * ACC_SETS + 1 + EPI_WARPS) + 16;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
  static_assert(ACC_SETS * ACC_COLS <= TMEM_COLS, "TMEM holds the accumulator sets");
};

// Six 32-lane x 8-column TMEM loads and one wait for all of them. The
// wait takes the destination registers as operands (in two statements of 24
// each, the second ordered after the first), so nothing reads them before the
// loads have landed.
__device__ __forceinline__ void tmem_ld8(uint32_t t, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(t)
               : "memory");
}
__device__ __forceinline__ void tmem_pass24(uint32_t (&a)[8], uint32_t (&b)[8], uint32_t (&c)[8], bool wait) {
  if (wait) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]), "+r"(c[4]), "+r"(c[5]), "+r"(c[6]), "+r"(c[7])
                 :
                 : "memory");
  } else {
    asm volatile("// tcgen05 load results"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]), "+r"(c[4]), "+r"(c[5]), "+r"(c[6]), "+r"(c[7])
                 :
                 : "memory");
  }
}
__device__ __forceinline__ void tmem_ld8x6(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3, uint32_t t4,
                                           uint32_t t5, float (&v)[6][8]) {
  uint32_t r0[8], r1[8], r2[8], r3[8], r4[8], r5[8];
  tmem_ld8(t0, r0);
  tmem_ld8(t1, r1);
  tmem_ld8(t2, r2);
  tmem_ld8(t3, r3);
  tmem_ld8(t4, r4);
  tmem_ld8(t5, r5);
  tmem_pass24(r0, r1, r2, true);
  tmem_pass24(r3, r4, r5, false);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[0][j] = __uint_as_float(r0[j]);
    v[1][j] = __uint_as_float(r1[j]);
    v[2][j] = __uint_as_float(r2[j]);
    v[3][j] = __uint_as_float(r3[j]);
    v[4][j] = __uint_as_float(r4[j]);
    v[5][j] = __uint_as_float(r5[j]);
  }
}

// p.tiles_x tiles across (ceil(width / 30)); p.e_w, p.e_h the image; p.epi
// the tail (UEPI_NONE / _GELU / _LRELU / _SIGMOID, or UEPI_ADD / _MUL with
// the second operand read through tmE, which has the output's geometry);
// p.bias 32 floats or null.
__global__ void __launch_bounds__(Conv3fCfg::THREADS, 1)
    umma_conv3f_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmE,
                       UmmaConvParams p) {
  using C = Conv3fCfg;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wsm = base;                                   // resident weights
  uint8_t* stg = base + C::W_BYTES;                      // stages: A, A_lo
  uint8_t* staging = stg + C::STAGES * C::STAGE_BYTES;   // one 4 KB buffer per epilogue warp
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
  uint64_t* lo_ready = full + C::STAGES;
  uint64_t* empty = lo_ready + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + C::ACC_SETS;
  uint64_t* wbar = acc_empty + C::ACC_SETS;
  uint64_t* ebar = wbar + 1;  // per epilogue warp: its operand row has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + C::EPI_WARPS);
  __shared__ int abort_flag;
  const volatile int* vabort = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&lo_ready[s], 32 * C::SPLIT);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < C::ACC_SETS; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(wbar, 1);
    for (int w = 0; w < C::EPI_WARPS; ++w) mbar_init(&ebar[w], 1);
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmW);
    tma_prefetch(&tmD);
    if (p.epi >= UEPI_ADD) tma_prefetch(&tmE);
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
  auto origin = [&](int t, int& x0, int& y0) {
    x0 = (t % p.tiles_x) * C::OUT_W;
    y0 = (t / p.tiles_x) * C::OUT_H;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(wbar, C::W_BYTES);
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) tma_load_2d(wsm + ky * C::W_KY_BYTES, &tmW, wbar, 0, ky * 2 * C::NF);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++it) {
        int x0, y0;
        origin(t, x0, y0);
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, vabort)) {
          fail(kErrProducer);
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::A_BYTES);
        tma_load_3d(stg + s * C::STAGE_BYTES, &tmA, &full[s], 0, x0 - 1, y0 - 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && mbar_wait(wbar, 0, vabort)) {
      tc_fence_after();
      constexpr uint32_t idesc2 = idesc_tf32(128, 2 * C::NF, 0, 0);  // A_hi x [B_hi | B_lo]
      constexpr uint32_t idesc = idesc_tf32(128, C::NF, 0, 0);       // A_lo x B_hi
      const uint64_t db0 = desc_kmajor_sw128(smem_u32(wsm));
      const uint32_t stg_u = smem_u32(stg);
      int s = 0;
      uint32_t ph = 0, tc = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
        const uint32_t acc = tc % C::ACC_SETS, aph = (tc / C::ACC_SETS) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1, vabort)) {
          fail(kErrMmaAcc);
          break;
        }
        tc_fence_after();
        if (!mbar_wait(&lo_ready[s], ph, vabort)) {
          fail(kErrMmaLo);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * C::ACC_COLS, dx = d + C::NF;
        const uint32_t a = stg_u + s * C::STAGE_BYTES;
        const uint64_t da0 = desc_kmajor_sw128(a), dl0 = desc_kmajor_sw128(a + C::A_BYTES);
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // Tap row ky: A rows from 32 ky (4 KB, 256 in the address field),
            // its B block 24 KB further per row; 32 bytes per K = 8 step.
            const uint64_t ra = 256u * ky + 2u * k, rb = uint64_t(C::W_KY_BYTES / 16) * ky + 2u * k;
            mma_tf32(d, da0 + ra, db0 + rb, idesc2, (ky > 0 || k > 0) ? 1u : 0u);
            mma_tf32(dx, dl0 + ra, db0 + rb, idesc, 1u);
          }
        mma_commit(&empty[s]);
        if (++s == C::STAGES) s = 0, ph ^= 1;
        mma_commit(&acc_full[acc]);
      }
    } else if (lane == 0 && !*vabort) {
      fail(kErrMmaLo);
    }
  } else if (warp < C::EPI_WARP0) {
    // ------------------------------------------------------------ split: A_lo
    const int tid = threadIdx.x - 64;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++it) {
      const int s = it % C::STAGES;
      const uint32_t ph = (it / C::STAGES) & 1;
      if (!mbar_wait(&full[s], ph, vabort)) {
        fail(kErrSplit);
        break;
      }
      const float4* a = reinterpret_cast<const float4*>(stg + s * C::STAGE_BYTES) + tid;
      float4* alo = reinterpret_cast<float4*>(stg + s * C::STAGE_BYTES + C::A_BYTES) + tid;
#pragma unroll
      for (int i = 0; i < C::A_BYTES / 16; i += 32 * C::SPLIT) {
        float4 l;
        tf32_residual4(a[i], &l.x);
        alo[i] = l;
      }
      fence_proxy_async_smem();
      mbar_arrive(&lo_ready[s]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - C::EPI_WARP0;
    const int set = ew >> 2;
    const int q = warp & 3;  // TMEM lane quarter = output row of the tile
    uint8_t* sb = staging + ew * 4096;
    float4* rowp = reinterpret_cast<float4*>(sb + lane * 128);
    const bool binary = p.epi >= UEPI_ADD;
    uint32_t use = 0, euse = 0;
    for (int t = blockIdx.x + set * gridDim.x; t < p.tiles; t += C::ACC_SETS * gridDim.x) {
      bool ok = mbar_wait(&acc_full[set], use & 1, vabort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) fail(kErrEpilogue);
        break;
      }
      tc_fence_after();
      int x0, y0;
      origin(t, x0, y0);
      // The previous store of this warp must have read the staging buffer.
      // A binary tail's operand row then comes by TMA into that buffer, in
      // the layout the results are staged in (a row past the image is
      // neither loaded nor stored).
      const bool row_in = y0 + q < p.e_h;
      if (lane == 0) {
        bulk_wait_read<0>();
        if (binary && row_in) {
          mbar_arrive_expect_tx(&ebar[ew], C::OUT_W * 128);
          tma_load_3d(sb, &tmE, &ebar[ew], 0, x0, y0 + q);
        }
      }
      __syncwarp();
      const uint32_t tb = tmem + (uint32_t(q * 32) << 16) + set * C::ACC_COLS;
      if (binary && row_in) {
        bool eok = mbar_wait(&ebar[ew], euse & 1, vabort);
        ++euse;
        eok = __all_sync(0xffffffffu, eok);
        if (!eok) {
          if (lane == 0) fail(kErrEpilogue);
          break;
        }
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        // Output channels 8g .. 8g + 7: the three column taps' partial sums,
        // hi*hi and cross regions each.
        float r[6][8];
        tmem_ld8x6(tb + 8 * g, tb + C::NF + 8 * g, tb + 32 + 8 * g, tb + C::NF + 32 + 8 * g, tb + 64 + 8 * g,
                   tb + C::NF + 64 + 8 * g, r);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          f2_add_to(r[0][i], r[0][i + 1], r[1][i], r[1][i + 1]);
          f2_add_to(r[2][i], r[2][i + 1], r[3][i], r[3][i + 1]);
          f2_add_to(r[4][i], r[4][i + 1], r[5][i], r[5][i + 1]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float s1 = __shfl_down_sync(0xffffffffu, r[2][i], 1);
          const float s2 = __shfl_down_sync(0xffffffffu, r[4][i], 2);
          v[i] = (r[0][i] + s1) + s2;
        }
        if (p.bias) {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias) + 2 * g);
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias) + 2 * g + 1);
          f2_add_to(v[0], v[1], b0.x, b0.y);
          f2_add_to(v[2], v[3], b0.z, b0.w);
          f2_add_to(v[4], v[5], b1.x, b1.y);
          f2_add_to(v[6], v[7], b1.z, b1.w);
        }
        if (binary) {
          // The operand's values where this thread stages its results (the
          // tensor-core kernel's order: the tail after the bias).
          const float4 e0 = rowp[(2 * g) ^ (lane & 7)], e1 = rowp[(2 * g + 1) ^ (lane & 7)];
          const float e[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
          if (p.epi == UEPI_ADD) {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] + e[i];
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = e[i] * v[i];
          }
        } else if (p.epi == UEPI_GELU) {
#pragma unroll
          for (int i = 0; i < 8; i += 2) gelu_f2(v[i], v[i + 1]);
        } else if (p.epi == UEPI_LRELU) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = v[i] >= 0.0f ? v[i] : p.slope * v[i];
        } else if (p.epi == UEPI_SIGMOID) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = sigmoid_f(v[i]);
        }
        rowp[(2 * g) ^ (lane & 7)] = make_float4(v[0], v[1], v[2], v[3]);
        rowp[(2 * g + 1) ^ (lane & 7)] = make_float4(v[4], v[5], v[6], v[7]);
      }
      // Everything this tile needs from TMEM has been read.
      tc_fence_before();
      mbar_arrive(&acc_empty[set]);
      ++use;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        // Staging rows 0..29 are output columns x0 .. x0 + 29 of row y0 + q;
        // TMA clips what lies outside the image.
        tma_store_3d(&tmD, sb, 0, x0, y0 + q);
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace mx
