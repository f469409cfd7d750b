// The six MAXIM variants and the task table (src/config.rs).
#pragma once

#include <string>

namespace mx {

class SafeTensors;

struct Config {
  std::string name;  // "S-1" .. "M-3"
  int features = 32;
  int depth = 3;
  int num_stages = 3;
  int num_groups = 2;
  int num_supervision_scales = 3;
  int num_outputs = 3;
  bool use_cross_gating = true;
  int high_res_stages = 2;
  int block_size_hr = 16;
  int block_size_lr = 8;
  // The grid size in CELLS per axis. The published code uses block_size_lr
  // for the low-res GRID size too, which is why this is 8 as well.
  int grid_size_hr = 16;
  int grid_size_lr = 8;
  int channels_reduction = 4;
  int num_bottleneck_blocks = 2;
  // "gMLP-<c>": not a model but ONE residual split-head multi-axis gMLP layer
  // (src/model.rs:576-603) over a c-channel input, block = grid = 16: the
  // isolated block op BASELINE's config 3 measures. `features` is c.
  bool block_only = false;

  // `Config::variant` (src/config.rs:34-62), plus "gMLP-<c>".
  static Config variant(const std::string& v);
  // `Config::of_checkpoint` (src/config.rs:71-100): the width is c_out of
  // `stage_0_encoder_block_0/Conv_0/kernel`, the stage count is the highest N
  // with a `stage_N_output_conv_1/kernel`.
  static Config of_checkpoint(const SafeTensors& f);
  // `Config::for_task` (src/config.rs:104-117).
  static Config for_task(const std::string& task);
};

}  // namespace mx
