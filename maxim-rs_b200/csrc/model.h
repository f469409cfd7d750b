// The MAXIM graph as a flat op list over one activation arena (src/model.rs).
//
// The plan is built for ONE padded input shape. Ops name buffers by index; a
// buffer may be a VIEW (a channel range) of another buffer's storage, which is
// how the model's channel splits and concatenations cost nothing. `finish`
// packs every storage-owning buffer into one arena by live range, largest
// first (src/model.rs:1091-1234).
//
// The op record is the ABI's POD `mx_op`, so exporting the plan to the GPU
// executor or to the CPU oracle is a pointer hand-off.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "config.h"
#include "maxim_b200.h"

namespace mx {

class Weights;

// LayerNorm epsilon: flax's nn.LayerNorm default (src/model.rs:35).
constexpr float kEps = 1e-6f;

struct Plan {
  std::vector<mx_buf> bufs;
  std::vector<int64_t> offs;  // resolved element offsets
  std::vector<mx_op> ops;
  std::vector<std::vector<float>> weights;
  int64_t arena_len = 0;
  int32_t input = -1, output = -1;
  std::vector<std::pair<std::string, int32_t>> dumps;
  mx_buf shape{3, 0, 0};
  std::vector<std::string> labels;
  std::vector<int32_t> alias_parent;  // -1: owns its storage
  std::vector<int64_t> alias_delta;

  int64_t arena_bytes() const { return arena_len * 4; }
  int64_t weight_bytes() const;
  // The POD view of this plan, valid while the plan lives.
  mx_plan view() const;

 private:
  mutable std::vector<const float*> wptr_;
  mutable std::vector<int64_t> wlen_;
};

// `Builder::new(w, cfg)[.without_dumps()].build(h, wd)`.
std::unique_ptr<Plan> build_plan(const Weights& w, const Config& cfg, int64_t h, int64_t wd, bool dumps);

// The buffer operands of an op (`Op::operands`, src/model.rs:117-139): the
// list that drives liveness. dst first.
void op_operands(const mx_op& op, std::vector<int32_t>& out);
// A one-line description (`exec_cpu::describe`, src/exec_cpu.rs:1352-1376).
std::string describe(const mx_op& op);

}  // namespace mx
