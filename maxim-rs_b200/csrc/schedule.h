// The executor's own schedule of a plan: which ops run as one kernel, which
// disappear, and where every buffer lives in the arena.
//
// The plan (src/model.rs) is a list of single-purpose ops over one packed
// arena, laid out by the reference's live-range packer for that op list. On a
// B200 most of those ops are memory-bound passes over the whole activation,
// and many of them exist only to feed the next op. The schedule rewrites the
// op list into fewer, fatter steps and re-packs the arena for the new list:
//
//   * Epilogue fusion: the elementwise op that is the only reader of a
//     tensor-core GEMM's output (GELU, LeakyReLU, sigmoid, residual add,
//     multiply, the gMLP gate u * (v + 1)) is applied by the GEMM's epilogue,
//     which writes the elementwise op's destination directly.
//   * Copy forwarding: a Copy whose source has no other reader makes the
//     source's producer write the Copy's destination (a channel range of a
//     concatenation, usually) in place of the source.
//   * Block permutations: a forward space -> blocked permutation whose
//     blocked buffer only feeds per-pixel ops and gating matmuls is dropped;
//     those ops run on the spatial buffer unchanged (per-pixel ops do not care
//     about pixel order) and the gating matmul reads the blocks through a
//     5-D tensor map instead. The matching backward permutation becomes a
//     Copy, which copy forwarding then removes.
//   * LayerNorm on load: a channel LayerNorm whose only reader is a
//     tensor-core conv becomes a statistics step (per-pixel mean and
//     reciprocal standard deviation, in the reference's serial order) and
//     the conv normalises its A operand as it splits it, so the normalised
//     tensor is never written or read back.
//   * Packing: every buffer the rewritten list still touches gets an arena
//     range by first fit over the rewritten list's live ranges (largest
//     buffers first), 256-byte aligned.
//
// Each rewrite is taken only where data dependences allow it: the moved op's
// inputs are not written, and its destination is neither read nor written,
// between the producer and the op's original position. Values are computed
// by the same arithmetic in the same order as the unfused steps, so the
// fused pass is bit-identical to running the plan op by op.
#pragma once

#include <functional>
#include <vector>

#include "maxim_b200.h"

namespace mx {

// The elementwise tail of a fused step, applied to each value v of the
// primary op's output (e = the matching value of the step's second operand).
enum EpiKind : int {
  EPI_NONE = 0,
  EPI_GELU = 1,     // gelu(v)
  EPI_LRELU = 2,    // v >= 0 ? v : slope * v
  EPI_SIGMOID = 3,  // sigmoid(v)
  EPI_ADD = 4,      // v + e
  EPI_MUL = 5,      // e * v
  EPI_GATE = 6,     // e * (v + 1)   (gMLP gating: u * (gate + 1))
};

struct SchedStep {
  mx_op o{};                    // the primary op as executed (ids resolved, dst redirected, kind may become Copy)
  int32_t op = -1;              // the primary plan op
  std::vector<int32_t> covers;  // every plan op this step carries out, primary first
  int epi = EPI_NONE;
  int32_t epi_src = -1;         // the epilogue's second operand
  // A channel scale whose epilogue adds two residuals, ((x * s) + epi_src) +
  // epi_src2 (two consecutive residual adds); -1 otherwise.
  int32_t epi_src2 = -1;
  float epi_slope = 0.0f;
  // A gating matmul over spatial-order data: the plan op (a forward block
  // permutation, since dropped) whose blocking it reads through; -1 if it
  // reads a blocked buffer.
  int32_t gate_perm = -1;
  // A channel LayerNorm turned into its statistics: o.dst is the statistics
  // buffer (2 floats per pixel: mean, 1 / sqrt(var + eps)).
  bool stats_only = false;
  // A conv whose A operand is LayerNorm'd on load: the statistics buffer and
  // the LayerNorm's scale and bias weights (-1 when not).
  int32_t ln_stats = -1, ln_scale = -1, ln_bias = -1;
  // A tensor-core step whose epilogue also writes LayerNorm statistics of
  // (up to two) channel groups of its output: group g is output channels
  // [stats_c0[g], stats_c0[g] + stats_c), its statistics go to buffer
  // stats_out[g] (-1: unused).
  int32_t stats_out[2] = {-1, -1};
  int32_t stats_c0[2] = {0, 0};
  int32_t stats_c = 0;
  // A tensor-core 1x1 conv whose epilogue also writes the LayerNorm of the
  // 32 output channels [ln_out_c0, ln_out_c0 + 32) to buffer ln_out (-1: none),
  // with the LayerNorm's scale and bias weights: the LayerNorm op it covers.
  int32_t ln_out = -1, ln_out_c0 = 0, ln_out_scale = -1, ln_out_bias = -1, ln_out_op = -1;
  // ...and nothing else reads the chunk itself, so it is not stored.
  bool ln_out_only = false;
};

struct Schedule {
  std::vector<SchedStep> steps;
  std::vector<mx_buf> extra;  // buffers the schedule adds (ids n_bufs, n_bufs + 1, ...), each its own root
  std::vector<int64_t> offs;  // per buffer (plan's, then extra), in floats: the root's offset + the plan's view delta
  // Per plan buffer: for a root placed inside another root (3b, merged
  // placement), that root, whose pixel stride its views then have; -1 else.
  std::vector<int32_t> merged_into;
  int64_t arena_len = 0;      // floats
  int perms_dropped = 0;
  int ops_fused = 0;          // plan ops carried out inside another op's step
  int ln_on_load = 0;         // LayerNorms applied by their consumer
  int stats_in_epilogue = 0;  // of those, statistics written by the producer's epilogue
  int ln_in_epilogue = 0;     // LayerNorms written whole by their producer's epilogue
  int copies_elided = 0;      // Copies whose readers read the source instead
  int steps_moved = 0;        // producers run at their consumer's position to take it as an epilogue
  int copies_merged = 0;      // Copies of a whole root into a view of another, the two placed as one
};

struct ScheduleHooks {
  // Whether the op runs on the tensor-core kernel (whose epilogue takes EPI_*).
  std::function<bool(const mx_op&)> umma;
  // Whether a gating matmul can read spatial-order data blocked as `perm` describes.
  std::function<bool(const mx_op& gate, const mx_op& perm)> gate_spatial;
  // Whether buffer b can be a tensor-core operand or output of n channels.
  std::function<bool(int32_t b, int n)> tma_view;
  // Whether the op's kernel can LayerNorm its A operand on load.
  std::function<bool(const mx_op&)> ln_on_load;
  // Whether the op is a 1x1 conv over so few pixels that it runs on the
  // small-conv kernel, whose epilogue takes the unary tails (GELU / LeakyReLU
  // / sigmoid) but no second operand.
  std::function<bool(const mx_op&)> small_conv;
  // The output-column slice width of a tensor-core op whose epilogue can
  // write LayerNorm statistics (whole pixel rows per thread), 0 if it cannot.
  std::function<int(const mx_op&)> stats_slice;
};

// fuse = false gives the plan's op list unchanged (one step per op), packed
// afresh. Throws mx::Error on a plan whose views are not channel ranges.
Schedule build_schedule(const mx_plan& plan, const ScheduleHooks& hooks, bool fuse);

}  // namespace mx
