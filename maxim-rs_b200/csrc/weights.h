// Parameter access and the layout conversions the executors read
// (src/weights.rs).
//
// Flax stores a conv kernel as [kh][kw][c_in][c_out] and a Dense as
// [c_in][c_out]. The plan keeps the reference's CPU layouts:
//   conv1x1 / Dense-as-1x1 -> [c_out][c_in]            (weights.rs:57-86)
//   k x k conv             -> [c_out][c_in][k][k]      (weights.rs:116-135)
//   ConvTranspose 2x2      -> [c_in][c_out][2][2], spatially FLIPPED
//                             (flax's ConvTranspose is the adjoint of its
//                             Conv; weights.rs:172-191)
//   gating Dense           -> [out][in]                (weights.rs:197-211)
// The GPU executor derives its own tensor-core layouts from these at upload.
//
// A Weights object can also run in SPEC mode: no file, every name "exists",
// and each request is recorded with the shape the builder expects. Running
// the builder against it yields the checkpoint's full parameter inventory,
// which is what a synthetic random-init checkpoint is generated from.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "config.h"

namespace mx {

class SafeTensors;

class Weights {
 public:
  static std::unique_ptr<Weights> open(const std::string& path);
  static std::unique_ptr<Weights> spec(const Config& cfg);
  ~Weights();

  Config config;

  bool has(const std::string& name) const;
  // A 1-D parameter of n values (LayerNorm scale/bias, conv bias).
  std::vector<float> vec(const std::string& name, int64_t n) const;
  // A 1x1 conv ([1,1,ci,co]) or Dense ([ci,co]) kernel as [co][ci]. `dense`
  // only tells SPEC mode which of the two shapes a checkpoint holds.
  std::vector<float> conv1x1(const std::string& name, int64_t ci, int64_t co, bool dense) const;
  // A k x k kernel as [co][ci][k][k].
  std::vector<float> convkxk(const std::string& name, int64_t k, int64_t ci, int64_t co) const;
  // A 2x2 transposed-conv kernel as [ci][co][2][2], spatially flipped.
  std::vector<float> convt2x2(const std::string& name, int64_t ci, int64_t co) const;
  // A square gating Dense (n x n) as [out][in].
  std::vector<float> dense(const std::string& name, int64_t n) const;

  bool spec_mode() const { return !file_; }
  // SPEC mode: every tensor the builder asked for, in request order.
  const std::vector<std::pair<std::string, std::vector<int64_t>>>& requested() const { return requested_; }

 private:
  Weights() = default;
  std::vector<int64_t> shape_of(const std::string& name) const;
  std::vector<float> raw(const std::string& name, const std::vector<int64_t>& expect) const;
  void record(const std::string& name, const std::vector<int64_t>& shape) const;

  std::unique_ptr<SafeTensors> file_;
  mutable std::vector<std::pair<std::string, std::vector<int64_t>>> requested_;
};

}  // namespace mx
