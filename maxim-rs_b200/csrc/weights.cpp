#include "weights.h"

#include "common.h"
#include "safetensors.h"

namespace mx {

namespace {
std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}
}  // namespace

std::unique_ptr<Weights> Weights::open(const std::string& path) {
  std::unique_ptr<Weights> w(new Weights());
  w->file_ = std::make_unique<SafeTensors>(path);
  w->config = Config::of_checkpoint(*w->file_);
  return w;
}

std::unique_ptr<Weights> Weights::spec(const Config& cfg) {
  std::unique_ptr<Weights> w(new Weights());
  w->config = cfg;
  return w;
}

Weights::~Weights() = default;

bool Weights::has(const std::string& name) const { return spec_mode() ? true : file_->contains(name); }

void Weights::record(const std::string& name, const std::vector<int64_t>& shape) const {
  requested_.emplace_back(name, shape);
}

std::vector<int64_t> Weights::shape_of(const std::string& name) const {
  if (!file_->contains(name)) throw Error(file_->path() + ": no tensor named " + name, MX_E_IO);
  return file_->info(name).shape;
}

std::vector<float> Weights::raw(const std::string& name, const std::vector<int64_t>& expect) const {
  auto s = shape_of(name);
  if (s != expect)
    throw Error(name + ": expected shape " + shape_str(expect) + ", the checkpoint has " + shape_str(s), MX_E_IO);
  return file_->f32(name);
}

std::vector<float> Weights::vec(const std::string& name, int64_t n) const {
  if (spec_mode()) {
    record(name, {n});
    return {};
  }
  return raw(name, {n});
}

std::vector<float> Weights::conv1x1(const std::string& name, int64_t ci, int64_t co, bool dense) const {
  if (spec_mode()) {
    record(name, dense ? std::vector<int64_t>{ci, co} : std::vector<int64_t>{1, 1, ci, co});
    return {};
  }
  // Either form is accepted whatever `dense` says, as weights.rs:57-86 does.
  auto s = shape_of(name);
  bool ok = (s.size() == 2 && s[0] == ci && s[1] == co) ||
            (s.size() == 4 && s[0] == 1 && s[1] == 1 && s[2] == ci && s[3] == co);
  if (!ok)
    throw Error(name + ": expected a 1x1 or Dense kernel for " + std::to_string(ci) + "->" + std::to_string(co) +
                    ", got " + shape_str(s),
                MX_E_IO);
  auto k = file_->f32(name);  // [ci][co]
  std::vector<float> out(size_t(ci * co));
  for (int64_t o = 0; o < co; ++o)
    for (int64_t i = 0; i < ci; ++i) out[o * ci + i] = k[i * co + o];
  return out;
}

std::vector<float> Weights::convkxk(const std::string& name, int64_t k, int64_t ci, int64_t co) const {
  if (spec_mode()) {
    record(name, {k, k, ci, co});
    return {};
  }
  auto src = raw(name, {k, k, ci, co});  // [ky][kx][ci][co]
  std::vector<float> out(src.size());
  for (int64_t oc = 0; oc < co; ++oc)
    for (int64_t ic = 0; ic < ci; ++ic)
      for (int64_t y = 0; y < k; ++y)
        for (int64_t x = 0; x < k; ++x) out[((oc * ci + ic) * k + y) * k + x] = src[((y * k + x) * ci + ic) * co + oc];
  return out;
}

std::vector<float> Weights::convt2x2(const std::string& name, int64_t ci, int64_t co) const {
  if (spec_mode()) {
    record(name, {2, 2, ci, co});
    return {};
  }
  auto src = raw(name, {2, 2, ci, co});
  std::vector<float> out(src.size());
  for (int64_t ic = 0; ic < ci; ++ic)
    for (int64_t oc = 0; oc < co; ++oc)
      for (int64_t y = 0; y < 2; ++y)
        for (int64_t x = 0; x < 2; ++x)
          out[((ic * co + oc) * 2 + y) * 2 + x] = src[((1 - y) * 2 + (1 - x)) * ci * co + ic * co + oc];
  return out;
}

std::vector<float> Weights::dense(const std::string& name, int64_t n) const {
  if (spec_mode()) {
    record(name, {n, n});
    return {};
  }
  auto src = raw(name, {n, n});  // [in][out]
  std::vector<float> out(src.size());
  for (int64_t o = 0; o < n; ++o)
    for (int64_t i = 0; i < n; ++i) out[o * n + i] = src[i * n + o];
  return out;
}

}  // namespace mx
