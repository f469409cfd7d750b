// Tensor-core contractions for sm_100a: tcgen05.mma kind::tf32 with FP32
// accumulators in TMEM, operands staged by TMA (no multicast).
//
// One persistent kernel; the problem shapes (MODE):
//   MODE_CONV1  1x1 conv / Dense:  D[pix][co] = b[co] + sum_ci X[pix][ci] W[co][ci]
//               M = 128 pixels of the flat pixel axis, K = c_in
//   MODE_CONV3  3x3 pad-1 conv:    K = (tap, ci); each tap's A block is a
//               shifted 3-D TMA box (8 rows x 16 columns x 32 channels) whose
//               out-of-image part TMA fills with zeros - the padding is free
//   MODE_CONV4  4x4 stride-2 conv, the same with a stride-2 box
//   MODE_GATE   gMLP gating Dense over a spatial axis of a blocked buffer:
//               D[(grp, c)][a] = b[a] + sum_t X[grp, t][c] W[a][t]
//               (MODE_GATE / MODE_GATE_GRID / MODE_GATE_SP)
//               M = 4 groups x 32 channels, N = a, K = t. The activation is
//               the MN-major operand: for each t, 32 channels are contiguous
//               in NHWC, which is one 128-byte row of the canonical SW128
//               MN-major atom; the 3-D box (32 ch, 32 t, 4 groups) lands
//               exactly in that layout. Block gating (t = position inside a
//               block) and grid gating (t = the cell) differ only in the
//               tensor map's strides.
//   MODE_CONV3H the 3x3 conv for N <= 64 by column shift: a stage holds one
//               16 x 10 box (the tile's rows with their halo) for shift kx
//               and the weights of the three taps (ky, kx); tap ky reads the
//               box from row 16 ky. Each input pixel is split once per shift
//               rather than once per tap.
//   MODE_CONVT  2x2 stride-2 transposed conv: a 1x1 product with N = 4 co
//               whose four column groups are stored to the four output taps
//
// Precision: every product is a 3-pass TF32 split,
//   a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi,
// about 21 significant bits per product (plain TF32 measured 46-48 dB against
// the fp32 CPU path under the He-normal init, below the 50 dB bar). Weights
// are split on the host; for activations a_hi is the fp32 tile itself, which
// the tensor core reads truncated to TF32, and the split stage computes a_lo
// (tf32_residual). The hi*hi products and the cross terms accumulate in
// separate TMEM regions, added in fp32 by the epilogue: the tensor core
// rounds its fp32 accumulator at every MMA, and with one region the full-size
// running sum took more such roundings per k-step at full magnitude.
//
// Warp roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A block (16 KB), B and B_lo blocks per k-block
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2-5   split: A_lo per k-block (into TMEM for N <= 64 convolutions,
//   (or 2-9)    beside A in shared memory otherwise), LayerNorm on load
//   then        epilogue, four warps per accumulator set: TMEM -> registers
//               -> +bias -> [elementwise tail, second operand prefetched into
//               registers] -> swizzled smem -> TMA store
// Three accumulator sets (N <= 64) or two (N = 128) let the epilogue of
// earlier tiles overlap the MMAs of the next one.
// Every mbarrier wait is bounded in time; a wait that runs out records a code
// in the status word, the kernel unwinds and frees its TMEM.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "sm100.cuh"

namespace mx {

// MODE_GATE: block gating (t = position inside a block, groups = blocks);
// MODE_GATE_GRID: grid gating (t = the cell, groups = positions in a cell).
// The grid case loads and stores its 4 groups as 4 separate boxes so every
// tensor map keeps its strides in ascending order.
// MODE_CONV4: the 4x4 stride-2 SAME conv (Conv_down); its A box is read with
// a TMA traversal stride of 2 in both spatial dimensions.
// MODE_GATE_SP: either gating over a SPATIAL (plain NHWC) buffer, read and
// written through 5-D tensor maps over (channel, fx, gx, fy, gy), pixel
// (gy * fh + fy, gx * fw + fx), so no blocked copy of the activation exists.
// Like MODE_GATE_GRID it moves one (32 channel x 32 t) box per group, which
// lands as the same [group][t][channel] smem tile: grid gating (sp_mode 0,
// t = cell (gy, gx), group = (fy, fx)) takes 32 / gw rows of gw cells, block
// gating (sp_mode 1, t = (fy, fx), group = block (gy, gx)) 32 / fw rows of fw
// positions.
// MODE_CONVT: the 2x2 stride-2 transposed conv (Conv_up) as a 1x1 GEMM with
// N = 4 c_out columns (tap t = 2 dy + dx major, then output channel); each
// epilogue warp's 32 input pixels (one image-row segment) are stored to
// output pixels (2y + dy, 2x + dx) through a 5-D map over (c, dx, x, dy, y).
enum : int {
  MODE_CONV1 = 0,
  MODE_CONV3 = 1,
  MODE_GATE = 2,
  MODE_GATE_GRID = 3,
  MODE_CONV4 = 4,
  MODE_GATE_SP = 5,
  MODE_CONVT = 6,
  MODE_CONV3H = 7
};

// The elementwise tail applied to each output value v before the store, with
// e the same element of a second operand (same shape as the output), which
// the epilogue reads straight from global memory one chunk ahead of its use.
// Numbering matches the executor's.
enum : int { UEPI_NONE = 0, UEPI_GELU, UEPI_LRELU, UEPI_SIGMOID, UEPI_ADD, UEPI_MUL, UEPI_GATE };

struct UmmaConvParams {
  int tiles;       // output tiles (output blocks x n_slices)
  int n_slices;    // N-column slices per output block (the output has n_slices * N columns)
  int tiles_x;     // CONV3: tiles per image row (width / 16); GATE: group tiles (ceil(groups / 4))
  int kb_per_tap;  // k-blocks (of 32) per tap
  int c_in;        // K per tap (CONV) / K (GATE)
  int groups;      // GATE_GRID / GATE_SP: groups (boxes past the last are skipped)
  int pad_t, pad_l;  // CONV4: SAME padding before the first row / column
  int sp_mode;        // GATE_SP: 0 grid gating, 1 block gating
  int fw, gw, fh;     // GATE_SP: block width and height in pixels, blocks per row
  int sp_shift;       // GATE_SP: log2 of the contracted index's row length (gw or fw)
  int epi;            // UEPI_*
  float slope;        // UEPI_LRELU
  const float* eptr;  // the epilogue's second operand (NHWC view), or null
  int estride;        // its pixel stride in floats
  int e_npix;         // CONV1: output pixels
  int e_w, e_h;       // CONV3 / CONV4: output width, height; GATE_SP: image width
  int e_pp;           // GATE / GATE_GRID: pixels per block of the blocked buffer
  // LayerNorm on load (CONV1 / CONV3): A = LN(x) with per-input-pixel
  // (mean, rstd) and per-channel scale / bias; ln_stats null when off.
  const float2* ln_stats;
  const float* ln_scale;
  const float* ln_bias;
  int in_w, in_h;     // CONV1: input pixels in in_w; CONV3: input width, height
  int co;             // CONVT: output channels (columns per tap)
  // LayerNorm statistics written by the epilogue (row layouts): for group g,
  // output channels [st_c0[g], st_c0[g] + st_c) of every output pixel give
  // (mean, 1 / sqrt(max(var, 0) + st_eps)) at st_out[g][pixel]; null if off.
  float2* st_out[2];
  int st_c0[2];
  int st_c;
  float st_eps;
  // CONV1 LayerNorm of output columns [lo_col, lo_col + 32), written through
  // the fifth tensor map (tmL) beside the plain output; lo_scale null if off.
  int lo_col;
  int lo_only;  // the chunk itself has no reader: only its LayerNorm is stored
  // CONV1 with a binary tail: a second addend, v = (v + e) + e2, read through
  // tmL (then not a LayerNorm output) into the epilogue warp's staging buffer.
  int e2;
  const float* lo_scale;
  const float* lo_bias;
  const float* bias;  // per output column, or null
  int* status;        // device status word (0 = ok)
};

// GATE_SP: the 5-D coordinates (after the channel) of group G's box whose
// contracted (or produced) index starts at t0 (a multiple of 32; the index's
// row length is 1 << sp_shift). The group part (two divisions) is per tile;
// gate_sp_row gives the per-k-block part with a shift.
__device__ __forceinline__ void gate_sp_group(const UmmaConvParams& p, int G, int& fx, int& gx, int& fy, int& gy) {
  if (p.sp_mode == 0) {
    fx = G % p.fw, fy = G / p.fw, gx = 0, gy = 0;
  } else {
    gx = G % p.gw, gy = G / p.gw, fx = 0, fy = 0;
  }
}
__device__ __forceinline__ void gate_sp_coords(const UmmaConvParams& p, int G, int t0, int& fx, int& gx, int& fy,
                                               int& gy) {
  gate_sp_group(p, G, fx, gx, fy, gy);
  if (p.sp_mode == 0) gy = t0 >> p.sp_shift;
  else fy = t0 >> p.sp_shift;
}

// GELU runs on value pairs (f32x2): the same roundings as the scalar form
// (the elementwise kernels' gelu_f), half the instructions. The binary tails
// stay scalar: their operand registers leave the 96-register instances no
// room for pairing.
template <int KIND>
__device__ __forceinline__ void epi_chunk(float (&v)[16], const float (&e)[16], float slope) {
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    if (KIND == UEPI_GELU) {
      gelu_f2(v[i], v[i + 1]);
    } else if (KIND == UEPI_LRELU) {
      v[i] = v[i] >= 0.0f ? v[i] : slope * v[i];
      v[i + 1] = v[i + 1] >= 0.0f ? v[i + 1] : slope * v[i + 1];
    } else if (KIND == UEPI_SIGMOID) {
      v[i] = sigmoid_f(v[i]);
      v[i + 1] = sigmoid_f(v[i + 1]);
    } else if (KIND == UEPI_ADD) {
      v[i] = v[i] + e[i];
      v[i + 1] = v[i + 1] + e[i + 1];
    } else if (KIND == UEPI_MUL) {
      v[i] = e[i] * v[i];
      v[i + 1] = e[i + 1] * v[i + 1];
    } else if (KIND == UEPI_GATE) {
      v[i] = e[i] * (v[i] + 1.0f);
      v[i + 1] = e[i + 1] * (v[i + 1] + 1.0f);
    }
  }
}

// The tail over one chunk: one uniform branch on the kind, then 16
// independent straight-line evaluations.
__device__ __forceinline__ void epi_apply(int kind, float (&v)[16], const float (&e)[16], float slope) {
  switch (kind) {
    case UEPI_GELU: epi_chunk<UEPI_GELU>(v, e, slope); break;
    case UEPI_LRELU: epi_chunk<UEPI_LRELU>(v, e, slope); break;
    case UEPI_SIGMOID: epi_chunk<UEPI_SIGMOID>(v, e, slope); break;
    case UEPI_ADD: epi_chunk<UEPI_ADD>(v, e, slope); break;
    case UEPI_MUL: epi_chunk<UEPI_MUL>(v, e, slope); break;
    case UEPI_GATE: epi_chunk<UEPI_GATE>(v, e, slope); break;
    default: break;
  }
}

// Whether a kernel instance keeps A_lo (the residual half of the split A
// operand) in TMEM rather than shared memory: the convolutions with N <= 64.
// A_hi is always the fp32 tile in shared memory, which the tensor core reads
// as TF32 by dropping the 13 low mantissa bits. TMEM then holds the two
// accumulator sets (4N columns) and one 32-column A_lo slot per stage.
__host__ __device__ constexpr bool umma_tmem_a(int n, int mode) {
  return n <= 64 && (mode == MODE_CONV1 || mode == MODE_CONV3 || mode == MODE_CONV4);
}

template <int N, int MODE>
struct UmmaCfg {
  static constexpr bool TMEM_A = umma_tmem_a(N, MODE);
  static constexpr bool HALO = MODE == MODE_CONV3H;
  static constexpr int A_BYTES = (HALO ? 160 : 128) * 128;  // rows x 32 fp32
  static constexpr int B_BYTES = N * 128;                   // N rows x 32 fp32, per tap
  static constexpr int B_TAPS = HALO ? 3 : 1;               // taps per stage
  // A stage holds A (and A_lo unless it lives in TMEM), then B and B_lo of
  // each of its taps.
  static constexpr int STAGE_BYTES = (TMEM_A ? 1 : 2) * A_BYTES + 2 * B_TAPS * B_BYTES;
  static constexpr int STAGES =
      HALO ? (N <= 32 ? 3 : 2) : (TMEM_A ? (N <= 32 ? 6 : 4) : (N <= 64 ? 4 : 3));
  // The split stage: four warps for the 1x1 convs and the gating matmuls,
  // eight for the 3x3 and 4x4 convs. With A_lo in TMEM each warp writes its
  // TMEM lane quarter, and with eight, two per quarter take 16 of the
  // k-block's 32 columns each: the quarters whose warps share a
  // sub-partition with the producer or the MMA issuer set the pace unless
  // their work per warp is halved. With A_lo in shared memory (the halo box,
  // the 128-column 3x3) the eight warps share the tile's float4s.
  static constexpr int SPLIT = MODE == MODE_CONV3 || MODE == MODE_CONV4 || HALO ? 8 : 4;
  // An accumulator set is two N-column fp32 regions: the hi*hi products and
  // the two cross terms, summed once in the epilogue. Each set has its own
  // four epilogue warps, so while the next tile accumulates the epilogue
  // drains one tile (two sets) or two (three sets, for the 1x1 convs with
  // N <= 64, where TMEM has room for them beside the A_lo slots).
  static constexpr int ACC_SETS = TMEM_A && SPLIT == 4 ? 3 : 2;
  static constexpr int EPI_WARPS = 4 * ACC_SETS;
  // Warp 0 producer, warp 1 MMA issuer, SPLIT split warps, then the epilogue.
  static constexpr int EPI_WARP0 = 2 + SPLIT;
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
  static constexpr int STAGING_BYTES = EPI_WARPS * 4096;  // one 32-row x 32-column buffer per epilogue warp
  static constexpr int A_COL0 = ACC_SETS * 2 * N;  // first TMEM column of the A_lo slots
  static constexpr int TMEM_COLS = TMEM_A ? 512 : ACC_SETS * 2 * N;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES + STAGING_BYTES + 8 * (3 * STAGES + 2 * ACC_SETS + EPI_WARPS) + 16;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
  static_assert(!TMEM_A || A_COL0 + STAGES * 32 <= 512, "TMEM holds the accumulators and the A_lo slots");
  static_assert(2 * N <= 256, "one instruction covers B_hi and B_lo");
};

enum : int {
  kErrProducer = 0x101,
  kErrSplit = 0x102,
  kErrMmaAcc = 0x103,
  kErrMmaLo = 0x104,
  kErrEpilogue = 0x105,
};

// The A split. The tensor core reads an fp32 operand as TF32 by dropping
// its 13 low mantissa bits (checked on B200 with an exact 0/1 selector as B:
// every value, ties included, came back truncated), so the fp32 tile in
// shared memory is A_hi = trunc(v) as it stands and only the residual
// A_lo = v - trunc(v) is computed and stored. The subtraction is exact; the
// residual is then rounded to the nearest TF32 value, ties away from zero:
// adding half a TF32 ulp (bit 12) to the sign-magnitude bits does that,
// carrying into the exponent where it should, once the 13 low bits are
// cleared - and the tensor core clears them itself as it reads the operand,
// so the stored word keeps them (one instruction less per value). All on the
// integer and fp32 ALUs at the full issue rate (the TF32 conversion
// instruction runs on a slower pipe). A NaN residual would wrap to a zero
// TF32 value, but it only comes with a NaN or infinite A_hi, which the
// product carries.
__device__ __forceinline__ float tf32_residual(float v) {
  const float hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  const float r = __fsub_rn(v, hi);
  return __uint_as_float(__float_as_uint(r) + 0x1000u);
}
// The same for four values, the subtractions paired (f32x2).
__device__ __forceinline__ void tf32_residual4(const float4 v, float* o) {
  const float4 hi = make_float4(__uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                                __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                                __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                                __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
  float r0, r1, r2, r3;
  f2_unpack(f2_sub(f2_pack(v.x, v.y), f2_pack(hi.x, hi.y)), r0, r1);
  f2_unpack(f2_sub(f2_pack(v.z, v.w), f2_pack(hi.z, hi.w)), r2, r3);
  o[0] = __uint_as_float(__float_as_uint(r0) + 0x1000u);
  o[1] = __uint_as_float(__float_as_uint(r1) + 0x1000u);
  o[2] = __uint_as_float(__float_as_uint(r2) + 0x1000u);
  o[3] = __uint_as_float(__float_as_uint(r3) + 0x1000u);
}

// E: the epilogue's tail reads a second operand (UEPI_ADD / _MUL / _GATE).
// Instances without one keep no operand registers, which the 96-register
// 576-thread instances need for their paired GELU.
template <int N, int MODE, bool E>
__global__ void __launch_bounds__(UmmaCfg<N, MODE>::THREADS, 1)
    umma_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmD,
                     const __grid_constant__ CUtensorMap tmL, UmmaConvParams p) {
  using C = UmmaCfg<N, MODE>;
  constexpr bool TMEM_A = C::TMEM_A;
  using namespace sm100;
  constexpr bool HALO = C::HALO;
  // Stages per tile and channel block: taps, or column shifts (HALO).
  constexpr int TAPS = HALO ? 3 : (MODE == MODE_CONV3 ? 9 : (MODE == MODE_CONV4 ? 16 : 1));
  constexpr bool SPATIAL = MODE == MODE_CONV3 || MODE == MODE_CONV4 || HALO;  // 8x16-pixel output tiles
  constexpr bool GATE = MODE == MODE_GATE || MODE == MODE_GATE_GRID || MODE == MODE_GATE_SP;
  constexpr bool PER_GROUP = MODE == MODE_GATE_GRID || MODE == MODE_GATE_SP;  // one box per group
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = base + C::STAGES * C::STAGE_BYTES;  // 1024-byte aligned (stage sizes are multiples of 1 KB)
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
  uint64_t* lo_ready = full + C::STAGES;
  uint64_t* empty = lo_ready + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + C::ACC_SETS;
  uint64_t* ebar = acc_empty + C::ACC_SETS;  // per epilogue warp: its gate operand tile has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + C::EPI_WARPS);
  __shared__ int abort_flag;
  const volatile int* vabort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = TAPS * p.kb_per_tap;

  // Tile t -> its origin: CONV1 (first pixel a0), SPATIAL (x0, y0), GATE
  // (first group a0, first channel a1); n0 = the first output column (of
  // this N-column slice). The slices of one output block are consecutive
  // tiles, so the CTAs computing them read the same A tile at about the same
  // time and all but the first read it from L2.
  auto decode = [&](int t, int& a0, int& a1, int& n0) {
    n0 = (t % p.n_slices) * N;
    t /= p.n_slices;
    if (MODE == MODE_CONV1 || MODE == MODE_CONVT) {
      a0 = t * 128;
      a1 = 0;
    } else if (SPATIAL) {
      a0 = (t % p.tiles_x) * 16;
      a1 = (t / p.tiles_x) * 8;
    } else {
      a0 = (t % p.tiles_x) * 4;
      a1 = (t / p.tiles_x) * 32;
    }
  };

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
    for (int w = 0; w < C::EPI_WARPS; ++w) mbar_init(&ebar[w], 1);
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    tma_prefetch(&tmBlo);
    tma_prefetch(&tmD);
    if ((MODE == MODE_CONV1 && (p.lo_scale || p.e2)) || (GATE && E)) tma_prefetch(&tmL);
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
        int a0, a1, n0;
        decode(t, a0, a1, n0);
        // GATE_SP: each group's fixed coordinates, once per tile.
        int gfx[4] = {0, 0, 0, 0}, ggx[4] = {0, 0, 0, 0}, gfy[4] = {0, 0, 0, 0}, ggy[4] = {0, 0, 0, 0};
        if (MODE == MODE_GATE_SP) {
#pragma unroll
          for (int g = 0; g < 4; ++g) gate_sp_group(p, a0 + g, gfx[g], ggx[g], gfy[g], ggy[g]);
        }
        // (tap, channel block) of k-block kb, stepped without division.
        int tap = 0, cb = 0, ky = 0, kx = 0;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          if (kb > 0 && ++cb == p.kb_per_tap) {
            cb = 0;
            ++tap;
            if (++kx == (MODE == MODE_CONV4 ? 4 : 3)) kx = 0, ++ky;
          }
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, vabort)) {
            fail(kErrProducer);
            break;
          }
          uint8_t* st = base + s * C::STAGE_BYTES;
          int a_bytes = C::A_BYTES;
          if (PER_GROUP) a_bytes = 4096 * min(4, p.groups - a0);
          mbar_arrive_expect_tx(&full[s], a_bytes + 2 * C::B_TAPS * C::B_BYTES);
          if (MODE == MODE_CONV1 || MODE == MODE_CONVT) {
            tma_load_2d(st, &tmA, &full[s], cb * 32, a0);
          } else if (MODE == MODE_CONV3) {
            tma_load_3d(st, &tmA, &full[s], cb * 32, a0 + kx - 1, a1 + ky - 1);
          } else if (HALO) {
            // Column shift kx: the tile's 8 rows and the halo row on either
            // side, 16 x 10 pixels from (x0 + kx - 1, y0 - 1).
            tma_load_3d(st, &tmA, &full[s], cb * 32, a0 + kx - 1, a1 - 1);
          } else if (MODE == MODE_CONV4) {
            // Output pixel (oy, ox) reads input (2oy + ky - pt, 2ox + kx - pl):
            // the tensor map steps 2 input pixels per box element.
            tma_load_3d(st, &tmA, &full[s], cb * 32, 2 * a0 + kx - p.pad_l, 2 * a1 + ky - p.pad_t);
          } else if (MODE == MODE_GATE) {
            tma_load_3d(st, &tmA, &full[s], a1, kb * 32, a0);
          } else {
            // A box past the last group would read nothing; its rows only
            // feed accumulator rows that are never stored, so it is skipped
            // and the expected byte count above counts only real boxes.
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (a0 + g < p.groups) {
                if (MODE == MODE_GATE_GRID) {
                  tma_load_3d(st + g * 4096, &tmA, &full[s], a1, a0 + g, kb * 32);
                } else {
                  const int r = (kb * 32) >> p.sp_shift;
                  // (fx, gx, fy, gy): the contracted index runs along gy
                  // (grid gating) or fy (block gating).
                  tma_load_5d(st + g * 4096, &tmA, &full[s], a1, gfx[g], ggx[g], p.sp_mode == 0 ? gfy[g] : r,
                              p.sp_mode == 0 ? r : ggy[g]);
                }
              }
          }
          uint8_t* sbw = st + (TMEM_A ? 1 : 2) * C::A_BYTES;  // B follows A (and A_lo unless it lives in TMEM)
          if (HALO) {
            // The weights of taps (0, kx), (1, kx), (2, kx), hi then lo each.
#pragma unroll
            for (int r = 0; r < 3; ++r) {
              const int kcol = (r * 3 + kx) * p.c_in + cb * 32;
              tma_load_2d(sbw + r * 2 * C::B_BYTES, &tmB, &full[s], kcol, n0);
              tma_load_2d(sbw + r * 2 * C::B_BYTES + C::B_BYTES, &tmBlo, &full[s], kcol, n0);
            }
          } else {
            const int kcol = tap * p.c_in + cb * 32;
            tma_load_2d(sbw, &tmB, &full[s], kcol, n0);
            tma_load_2d(sbw + C::B_BYTES, &tmBlo, &full[s], kcol, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, N, GATE ? 1 : 0, 0);
      // B_lo sits right after B_hi in the stage (N rows each, whole 8-row
      // swizzle atoms), and the cross-term region right after the hi*hi one
      // in TMEM, so one N' = 2N instruction computes A_hi*B_hi and A_hi*B_lo
      // together. An MMA costs about the same below N = 128 whatever its
      // width, so the k-step takes two instructions instead of three.
      constexpr uint32_t idesc2 = idesc_tf32(128, 2 * N, GATE ? 1 : 0, 0);
      // The issuing thread shares its sub-partition with split and epilogue
      // warps, so its own instruction count per k-block sets part of the
      // pace: the stage and phase step without division, and each stage's
      // descriptors are built once per k-block and stepped by constants
      // (32 bytes along K = 2 in the address field; 1024 bytes = 64 for the
      // MN-major layout).
      const uint32_t base_u = smem_u32(base);
      constexpr uint32_t kStepK = GATE ? 64u : 2u;
      int s = 0;
      uint32_t ph = 0, tc = 0;
      for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x, ++tc) {
        const uint32_t acc = tc % C::ACC_SETS, aph = (tc / C::ACC_SETS) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1, vabort)) {
          fail(kErrMmaAcc);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * 2 * N, dx = d + N;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&lo_ready[s], ph, vabort)) {
            fail(kErrMmaLo);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = base_u + s * C::STAGE_BYTES;
          const uint32_t b = a + (TMEM_A ? 1 : 2) * C::A_BYTES, alo = a + C::A_BYTES;
          // TMEM_A: this stage's A_lo sits in TMEM columns [slot, slot + 32);
          // k-step k reads 8 of them.
          const uint32_t slot = tmem + C::A_COL0 + s * 32;
          const uint64_t da0 = GATE ? desc_mnmajor_sw128_32b(a, 4096) : desc_kmajor_sw128(a);
          const uint64_t dalo0 = GATE ? desc_mnmajor_sw128_32b(alo, 4096) : desc_kmajor_sw128(alo);
          const uint64_t db0 = desc_kmajor_sw128(b);
          // HALO: tap ky of the stage reads the box from row 16 ky (2 KB, 128
          // in the address field) and its weights from the ky-th B pair.
#pragma unroll
          for (int ky = 0; ky < C::B_TAPS; ++ky)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // GATE: MN-major, k-step k covers K rows 8k..8k+7 of each 4 KB
              // group block; otherwise K-major, 8 fp32 = 32 bytes per k-step.
              const uint32_t ra = 128u * ky, rb = uint32_t(2 * C::B_BYTES / 16) * ky;
              const uint64_t da = da0 + ra + kStepK * k, db = db0 + rb + 2u * k;
              // The running sum of the hi*hi products takes one accumulator
              // update per k-step; the cross terms, 2^-10 of its size or less,
              // go to their own region, so the accumulator's rounding at each
              // update is paid once per k-step at full magnitude.
              const uint32_t accum = (kb > 0 || ky > 0 || k > 0) ? 1u : 0u;
              mma_tf32(d, da, db, idesc2, accum);
              if (TMEM_A) {
                mma_tf32_ts(dx, slot + 8 * k, db, idesc, 1u);
              } else {
                mma_tf32(dx, dalo0 + ra + kStepK * k, db, idesc, 1u);
              }
            }
          mma_commit(&empty[s]);
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
      }
    }
  } else if (warp < C::EPI_WARP0) {
    // ------------------------------------------------------------ split
    const int tid = threadIdx.x - 64;  // 0 .. 32 * SPLIT - 1
    // TMEM_A with SPLIT = 8: warps 2-5 take columns 0-15 of each row, warps
    // 6-9 columns 16-31; otherwise one warp takes all 32.
    constexpr int NCH = 32 / 4 / (C::SPLIT / 4);  // float4 chunks of a row per thread
    const int half = (warp - 2) >> 2;
    uint32_t it = 0;
    // LayerNorm on load: the statistics of the input pixel behind A row r of
    // the current k-block, if that pixel is inside the image (rows outside
    // it are zero padding, which stays zero).
    int a0 = 0, a1 = 0, n0 = 0, cb = 0, ky = 0, kx = 0;
    auto ln_row = [&](int r, float& m, float& rs) -> bool {
      int pix = -1;
      if (MODE == MODE_CONV1) {
        if (a0 + r < p.in_w) pix = a0 + r;
      } else if (MODE == MODE_CONV3) {
        const int y = a1 + (r >> 4) + ky - 1, x = a0 + (r & 15) + kx - 1;
        if (y >= 0 && y < p.in_h && x >= 0 && x < p.in_w) pix = y * p.in_w + x;
      }
      if (pix < 0) return false;
      const float2 st = p.ln_stats[pix];
      m = st.x, rs = st.y;
      return true;
    };
    // (x - m) * rstd * scale + bias, in the LayerNorm kernel's exact order,
    // over 4 channels from ch (a multiple of 4; every thread reads the same
    // scale and bias, so the read-only cache serves them).
    // ((v - m) * rs) * w + b per channel, every operation rounded on its own
    // (the LayerNorm kernel's order), as paired f32x2 instructions.
    auto ln_apply4 = [&](float4 v, float m, float rs, int ch) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(p.ln_scale + ch));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p.ln_bias + ch));
      const uint64_t mm = f2_pack(m, m), rr = f2_pack(rs, rs);
      f2_unpack(f2_add_after_mul(f2_mul(f2_mul(f2_sub(f2_pack(v.x, v.y), mm), rr), f2_pack(w.x, w.y)),
                                 f2_pack(b.x, b.y)),
                v.x, v.y);
      f2_unpack(f2_add_after_mul(f2_mul(f2_mul(f2_sub(f2_pack(v.z, v.w), mm), rr), f2_pack(w.z, w.w)),
                                 f2_pack(b.z, b.w)),
                v.z, v.w);
      return v;
    };
    // In the 1x1 instances a thread's rows are the same for every k-block
    // of a tile (TMEM_A: row rq; otherwise rows tid / 8 + 16 j), so their
    // statistics are loaded once per tile, and a whole tile ahead: loaded
    // just before the A wait they would still be in flight when the tile
    // arrives (an L2 round trip, often to the far die, is longer than the
    // gap between two tiles). Bit j of ln_next: row j is inside the image.
    constexpr bool LN_AHEAD = MODE == MODE_CONV1;
    constexpr int LN_ROWS = TMEM_A ? 1 : 8;
    float2 st_next[LN_ROWS], st_cur[LN_ROWS];
#pragma unroll
    for (int j = 0; j < LN_ROWS; ++j) st_next[j] = st_cur[j] = make_float2(0.0f, 0.0f);
    uint32_t ln_next = 0, ln_cur = 0;
    auto fetch_stats = [&](int tn) {
      ln_next = 0;
      if (tn < p.tiles) {
        int b0, b1, m0;
        decode(tn, b0, b1, m0);
#pragma unroll
        for (int j = 0; j < LN_ROWS; ++j) {
          const int pix = b0 + (TMEM_A ? (warp & 3) * 32 + lane : (tid >> 3) + 16 * j);
          if (pix < p.in_w) {
            st_next[j] = p.ln_stats[pix];
            ln_next |= 1u << j;
          }
        }
      }
    };
    if (LN_AHEAD && p.ln_stats) fetch_stats(blockIdx.x);
    for (int t = blockIdx.x; t < p.tiles && !*vabort; t += gridDim.x) {
      bool ok = true;
      decode(t, a0, a1, n0);
      cb = 0, ky = 0, kx = 0;
      if (LN_AHEAD && p.ln_stats) {
#pragma unroll
        for (int j = 0; j < LN_ROWS; ++j) st_cur[j] = st_next[j];
        ln_cur = ln_next;
        fetch_stats(t + gridDim.x);
      }
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if (kb > 0 && ++cb == p.kb_per_tap) {
          cb = 0;
          if (++kx == 3) kx = 0, ++ky;
        }
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1;
        // LayerNorm on load: the statistics of this thread's rows (TMEM_A:
        // one row; otherwise the 8 rows tid / 8 + 16 i of its float4s). The
        // 1x1 instances have them from a tile ahead; elsewhere they depend on
        // the tap too and are loaded here, before the wait for the A tile.
        const int q = warp & 3, rq = q * 32 + lane;
        float lm = 0.0f, lr = 0.0f;
        bool ln = false;
        float lms[8], lrs[8];
        bool lns[8];
        if (p.ln_stats) {
          if (LN_AHEAD && TMEM_A) {
            ln = ln_cur & 1u, lm = st_cur[0].x, lr = st_cur[0].y;
          } else if (LN_AHEAD) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              lns[i] = (ln_cur >> i) & 1u, lms[i] = st_cur[i % LN_ROWS].x, lrs[i] = st_cur[i % LN_ROWS].y;
          } else if (TMEM_A) {
            ln = ln_row(rq, lm, lr);
          } else if (!GATE && !HALO) {
#pragma unroll
            for (int i = 0; i < 8; ++i) lns[i] = ln_row((tid >> 3) + 16 * i, lms[i], lrs[i]);
          }
        }
        if (!mbar_wait(&full[s], ph, vabort)) {
          fail(kErrSplit);
          ok = false;
          break;
        }
        if (TMEM_A) {
          // This warp's TMEM lane quarter: rows q*32 .. q*32+31 of A. Each
          // thread reads its row's columns (all 32 K values, or its half of
          // them; 128-byte swizzled) and writes their A_lo into the stage's
          // TMEM slot; with LayerNorm on load the normalised values also go
          // back into the tile (A_hi).
          const int r = rq;
          uint8_t* arow = base + s * C::STAGE_BYTES + r * 128;
          float lo[4 * NCH];
          if (p.ln_stats) {
            // Branch-free over the chunks (a row outside the image keeps its
            // zeros by selection), so the loads of all chunks and of the
            // scale and bias can be in flight together.
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
              const int cc = half * NCH + c;
              float4* p4 = reinterpret_cast<float4*>(arow + ((cc ^ (r & 7)) << 4));
              float4 v = *p4;
              const float4 u = ln_apply4(v, lm, lr, cb * 32 + 4 * cc);
              if (MODE == MODE_CONV1) {
                // A row past the last pixel only feeds an output row the
                // store clips, so it needs no selection (its statistics
                // are finite: zero, or an earlier row's).
                v = u;
              } else {
                v.x = ln ? u.x : v.x;
                v.y = ln ? u.y : v.y;
                v.z = ln ? u.z : v.z;
                v.w = ln ? u.w : v.w;
              }
              *p4 = v;
              tf32_residual4(v, lo + 4 * c);
            }
          } else {
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
              const int cc = half * NCH + c;  // float4 chunk of the row
              const float4 v = *reinterpret_cast<const float4*>(arow + ((cc ^ (r & 7)) << 4));
              tf32_residual4(v, lo + 4 * c);
            }
          }
          const uint32_t slot = tmem + (uint32_t(q * 32) << 16) + C::A_COL0 + s * 32;
          if (NCH == 8) {
            tmem_st32(slot, lo);
          } else {
            tmem_st16(slot + 16 * half, lo);
          }
          tmem_wait_st();
          if (p.ln_stats) fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(&lo_ready[s]);
          continue;
        }
        // Elementwise, so the layout does not matter; a warp touches 32
        // consecutive float4 (512 contiguous bytes) per access, which keeps
        // every shared-memory access free of bank conflicts.
        float4* a = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES) + tid;
        float4* alo = reinterpret_cast<float4*>(base + s * C::STAGE_BYTES + C::A_BYTES) + tid;
        // 32 * SPLIT split threads over the tile (HALO: the 160-row box).
        // Only the four-warp 1x1 instances normalise on load.
        // Branch-free over the float4s, as in the TMEM_A case.
        const bool norm = !GATE && !HALO && C::SPLIT == 4 && p.ln_stats;
#pragma unroll
        for (int i = 0; i < C::A_BYTES / 16; i += 32 * C::SPLIT) {
          float4 v = a[i], l;
          if (norm) {
            // float4 (tid + i) of the swizzled tile: row f / 8, chunk (f % 8) ^ (row % 8).
            const int f = tid + i, r = f >> 3, ch = cb * 32 + (((f & 7) ^ (r & 7)) << 2);
            const bool on = lns[i >> 7];
            const float4 u = ln_apply4(v, lms[i >> 7], lrs[i >> 7], ch);
            if (MODE == MODE_CONV1) {
              v = u;  // as above: rows past the last pixel feed clipped outputs
            } else {
              v.x = on ? u.x : v.x;
              v.y = on ? u.y : v.y;
              v.z = on ? u.z : v.z;
              v.w = on ? u.w : v.w;
            }
            a[i] = v;
          }
          tf32_residual4(v, &l.x);
          alo[i] = l;
        }
        fence_proxy_async_smem();
        mbar_arrive(&lo_ready[s]);
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // ACC_SETS sets of four warps; set `set` drains accumulator `set`, i.e.
    // every ACC_SETS-th tile, so that many tiles drain at once. A warp owns
    // the 32 accumulator rows of its TMEM lane quarter and stages and stores
    // them itself (one 4 KB staging buffer per warp), so no barrier joins the
    // epilogue warps.
    const int ew = warp - C::EPI_WARP0;  // 0 .. EPI_WARPS - 1
    const int set = ew >> 2;
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;  // accumulator row this thread owns
    // The gating instances take their second operand (the gate) by TMA into
    // the warp's staging buffer, in the layout the output is staged in, so
    // each thread reads its values where it then writes its results; the
    // others hold it in registers, loaded one chunk ahead.
    constexpr bool TMA_E = GATE && E;
    constexpr int NE = E && !GATE ? 32 : 1;  // operand values held per thread
    // A 1x1 conv's second addend comes the same way as the gate.
    const bool E2 = MODE == MODE_CONV1 && E && p.e2 != 0;
    uint8_t* sb = staging + ew * 4096;
    uint32_t euse = 0;  // operand tiles this warp has taken from ebar

    // The second operand's values for this thread in chunk j of tile t: its
    // output pixel's 32 channels.
    auto load_e = [&](int t, int j, float(&e)[NE]) {
      if constexpr (E && !GATE) {
        int a0, a1, n0;
        decode(t, a0, a1, n0);
        const int col = n0 + j * 32;
        int pix;
        bool ok;
        if (MODE == MODE_CONV1) {
          pix = a0 + row;
          ok = pix < p.e_npix;
        } else {
          const int y = a1 + (row >> 4), x = a0 + (row & 15);
          ok = y < p.e_h && x < p.e_w;
          pix = y * p.e_w + x;
        }
        const float4* src = reinterpret_cast<const float4*>(p.eptr + size_t(ok ? pix : 0) * p.estride + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = ok ? src[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          e[4 * i] = v.x, e[4 * i + 1] = v.y, e[4 * i + 2] = v.z, e[4 * i + 3] = v.w;
        }
      }
    };

    // The gate tile of chunk jj of tile tt: once the warp's previous store
    // has read the staging buffer, TMA loads the group's (32 channel x 32
    // position) box of the gate operand into it. It is issued as soon as the
    // previous chunk's store has gone out, so the load overlaps the wait for
    // the next accumulator and the TMEM loads (lane 0 only).
    auto gate_load = [&](int tt, int jj) {
      if (MODE == MODE_CONV1 && E2) {
        bulk_wait_read<0>();
        int b0, b1, m0;
        decode(tt, b0, b1, m0);
        mbar_arrive_expect_tx(&ebar[ew], 4096);
        tma_load_2d(sb, &tmL, &ebar[ew], m0 + jj * 32, b0 + 32 * q);
        return;
      }
      if constexpr (TMA_E) {
        bulk_wait_read<0>();
        int b0, b1, m0;
        decode(tt, b0, b1, m0);
        if (b0 + q >= p.groups) return;
        const int col = m0 + jj * 32;
        mbar_arrive_expect_tx(&ebar[ew], 4096);
        if (MODE == MODE_GATE) {
          tma_load_3d(sb, &tmL, &ebar[ew], b1, col, b0 + q);
        } else if (MODE == MODE_GATE_GRID) {
          tma_load_3d(sb, &tmL, &ebar[ew], b1, b0 + q, col);
        } else {
          int fx, gx, fy, gy;
          gate_sp_coords(p, b0 + q, col, fx, gx, fy, gy);
          tma_load_5d(sb, &tmL, &ebar[ew], b1, fx, gx, fy, gy);
        }
      }
    };
    const int tstep = C::ACC_SETS * gridDim.x;
    int t = blockIdx.x + set * gridDim.x, j = 0, a0 = 0, a1 = 0, n0 = 0;
    // LayerNorm statistics of this thread's output pixel, one serial pair of
    // sums per group, in channel order (the statistics kernel's order).
    float ss1[2] = {0.0f, 0.0f}, ss2[2] = {0.0f, 0.0f};
    uint32_t use = 0;  // how many tiles this set has taken from its accumulator
    // One chunk (32 columns), in two 16-column halves: drain from TMEM, add
    // the bias, apply the tail (operand values in `ecur`, loaded while the
    // previous chunk was finishing), stage and store, then start loading the
    // next chunk's operand values into `ecur`. Returns false when the
    // pipeline failed.
    auto step = [&](float(&ecur)[NE]) -> bool {
      if (j == 0) {
        bool ok = mbar_wait(&acc_full[set], use & 1, vabort);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0) fail(kErrEpilogue);
          return false;
        }
        tc_fence_after();
        decode(t, a0, a1, n0);
      }
      // A group past the last is neither loaded nor stored.
      const bool gvalid = GATE && a0 + q < p.groups;
      const uint32_t tcol = tmem + (uint32_t(q * 32) << 16) + set * 2 * N + j * 32;
      // The chunk whose LayerNorm this step also writes (below).
      const bool lnc = MODE == MODE_CONV1 && p.lo_scale != nullptr && n0 + j * 32 == p.lo_col;
#pragma unroll
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[16], x[16], e[16];
        tmem_ld16x2(tcol + h * 16, tcol + N + h * 16, v, x);
        // The two regions' sum and the bias: paired adds where the registers
        // allow (no second operand held), scalar adds otherwise; the same
        // roundings either way.
        if constexpr (E) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += x[i];
        } else {
#pragma unroll
          for (int i = 0; i < 16; i += 2) f2_add_to(v[i], v[i + 1], x[i], x[i + 1]);
        }
        if (p.bias) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0 + j * 32 + h * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 b = __ldg(b4 + i);
            if constexpr (E) {
              v[4 * i] += b.x;
              v[4 * i + 1] += b.y;
              v[4 * i + 2] += b.z;
              v[4 * i + 3] += b.w;
            } else {
              f2_add_to(v[4 * i], v[4 * i + 1], b.x, b.y);
              f2_add_to(v[4 * i + 2], v[4 * i + 3], b.z, b.w);
            }
          }
        }
        if constexpr (TMA_E) {
          if (h == 0 && gvalid) {
            bool ok = mbar_wait(&ebar[ew], euse & 1, vabort);
            ++euse;
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
              if (lane == 0) fail(kErrEpilogue);
              return false;
            }
          }
          // This thread's channel at positions h * 16 + i: where it stages
          // its results below.
          const float* g = reinterpret_cast<const float*>(sb);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int r = h * 16 + i;
            e[i] = gvalid ? g[r * 32 + (((lane >> 2) ^ (r & 7)) << 2) + (lane & 3)] : 0.0f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if constexpr (E) e[i] = ecur[h * 16 + i];
            else e[i] = 0.0f;
          }
        }
        epi_apply(p.epi, v, e, p.slope);
        if (E2) {
          // The second addend, where this thread stages its pixel's row.
          if (h == 0) {
            bool ok = mbar_wait(&ebar[ew], euse & 1, vabort);
            ++euse;
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
              if (lane == 0) fail(kErrEpilogue);
              return false;
            }
          }
          const float4* r4 = reinterpret_cast<const float4*>(sb + lane * 128);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 f = r4[(h * 4 + i) ^ (lane & 7)];
            v[4 * i] = v[4 * i] + f.x;
            v[4 * i + 1] = v[4 * i + 1] + f.y;
            v[4 * i + 2] = v[4 * i + 2] + f.z;
            v[4 * i + 3] = v[4 * i + 3] + f.w;
          }
        }
        if (!GATE && MODE != MODE_CONVT && p.st_out[0]) {
          const int colh = n0 + j * 32 + h * 16;
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            if (!p.st_out[g] || colh < p.st_c0[g] || colh >= p.st_c0[g] + p.st_c) continue;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              ss1[g] = __fadd_rn(ss1[g], v[i]);
              ss2[g] = __fadd_rn(ss2[g], __fmul_rn(v[i], v[i]));
            }
            if (colh + 16 == p.st_c0[g] + p.st_c) {
              int pix;
              bool in;
              if (MODE == MODE_CONV1) {
                pix = a0 + row;
                in = pix < p.e_npix;
              } else {
                const int y = a1 + (row >> 4), x = a0 + (row & 15);
                in = y < p.e_h && x < p.e_w;
                pix = y * p.e_w + x;
              }
              const float nf = float(p.st_c);
              const float m = __fdiv_rn(ss1[g], nf);
              const float var = __fsub_rn(__fdiv_rn(ss2[g], nf), __fmul_rn(m, m));
              const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), p.st_eps)));
              if (in) p.st_out[g][pix] = make_float2(m, rs);
              ss1[g] = 0.0f, ss2[g] = 0.0f;
            }
          }
        }
        if (!TMA_E && !E2 && h == 0) {
          // This warp's previous store must have read the staging buffer;
          // waiting only now lets that read overlap the TMEM loads and the
          // arithmetic above. (The gating instances waited before their
          // gate tile's load.)
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        if (GATE) {
          // Staging is [a][channel] for this warp's group: this thread
          // (channel lane) owns one float in each of the 32 rows.
          float* g = reinterpret_cast<float*>(sb);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int r = h * 16 + i;
            g[r * 32 + (((lane >> 2) ^ (r & 7)) << 2) + (lane & 3)] = v[i];
          }
        } else {
          float4* rowp = reinterpret_cast<float4*>(sb + lane * 128);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            rowp[(h * 4 + i) ^ (lane & 7)] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
      if (j == N / 32 - 1) {
        // Everything this tile needs from TMEM has been read.
        tc_fence_before();
        mbar_arrive(&acc_empty[set]);
        ++use;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int col = n0 + j * 32;
        if (MODE == MODE_CONV1) {
          if (!(lnc && p.lo_only)) tma_store_2d(&tmD, sb, col, a0 + 32 * q);
        } else if (MODE == MODE_CONVT) {
          // Rows a0 + 32q .. +31 are one row segment of the input image.
          const int pix = a0 + 32 * q;
          if (pix < p.e_npix) {
            const int tap = col / p.co, y = pix / p.e_w;
            tma_store_5d(&tmD, sb, col - tap * p.co, tap & 1, pix - y * p.e_w, tap >> 1, y);
          }
        } else if (SPATIAL) {
          tma_store_3d(&tmD, sb, col, a0, a1 + 2 * q);
        } else if (a0 + q < p.groups) {
          if (MODE == MODE_GATE) {
            tma_store_3d(&tmD, sb, a1, col, a0 + q);
          } else if (MODE == MODE_GATE_GRID) {
            tma_store_3d(&tmD, sb, a1, a0 + q, col);
          } else {
            int fx, gx, fy, gy;
            gate_sp_coords(p, a0 + q, col, fx, gx, fy, gy);
            tma_store_5d(&tmD, sb, a1, fx, gx, fy, gy);
          }
        }
        bulk_commit();
      }
      if (MODE == MODE_CONV1 && lnc) {
        // The LayerNorm of this pixel's 32 values, read back from the row
        // this thread just staged (the plain chunk's store only reads it), in
        // the LayerNorm kernel's order: serial sums over the channels, then
        // ((v - m) * rstd) * w + b, written over the row once that store has
        // read it.
        float4* rowp = reinterpret_cast<float4*>(sb + lane * 128);
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = rowp[i ^ (lane & 7)];
          s1 = __fadd_rn(s1, v.x), s2 = __fadd_rn(s2, __fmul_rn(v.x, v.x));
          s1 = __fadd_rn(s1, v.y), s2 = __fadd_rn(s2, __fmul_rn(v.y, v.y));
          s1 = __fadd_rn(s1, v.z), s2 = __fadd_rn(s2, __fmul_rn(v.z, v.z));
          s1 = __fadd_rn(s1, v.w), s2 = __fadd_rn(s2, __fmul_rn(v.w, v.w));
        }
        const float m = __fdiv_rn(s1, 32.0f);
        const float var = __fsub_rn(__fdiv_rn(s2, 32.0f), __fmul_rn(m, m));
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), p.st_eps)));
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 v = rowp[i ^ (lane & 7)];
          const float4 w = __ldg(reinterpret_cast<const float4*>(p.lo_scale) + i);
          const float4 b = __ldg(reinterpret_cast<const float4*>(p.lo_bias) + i);
          v.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, m), rs), w.x), b.x);
          v.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, m), rs), w.y), b.y);
          v.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, m), rs), w.z), b.z);
          v.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, m), rs), w.w), b.w);
          rowp[i ^ (lane & 7)] = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmL, sb, 0, a0 + 32 * q);
          bulk_commit();
        }
      }
      if (++j == N / 32) j = 0, t += tstep;
      if (E && !GATE && t < p.tiles) load_e(t, j, ecur);
      if ((TMA_E || E2) && lane == 0 && t < p.tiles) gate_load(t, j);
      return true;
    };

    float e[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) e[i] = 0.0f;
    if (E && !GATE && t < p.tiles) load_e(t, 0, e);
    if ((TMA_E || E2) && lane == 0 && t < p.tiles) gate_load(t, 0);
    while (t < p.tiles && step(e)) {
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
