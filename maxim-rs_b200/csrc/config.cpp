#include "config.h"

#include <algorithm>
#include <cctype>

#include "common.h"
#include "safetensors.h"

namespace mx {

Config Config::variant(const std::string& v) {
  int features, stages;
  if (v == "S-1") features = 32, stages = 1;
  else if (v == "S-2") features = 32, stages = 2;
  else if (v == "S-3") features = 32, stages = 3;
  else if (v == "M-1") features = 64, stages = 1;
  else if (v == "M-2") features = 64, stages = 2;
  else if (v == "M-3") features = 64, stages = 3;
  else throw Error("unknown variant " + v + " (expected S-1..S-3, M-1..M-3)");
  Config c;
  c.name = v;
  c.features = features;
  c.num_stages = stages;
  return c;
}

Config Config::of_checkpoint(const SafeTensors& f) {
  const std::string name = "stage_0_encoder_block_0/Conv_0/kernel";
  if (!f.contains(name)) throw Error(name + " is missing (not a converted MAXIM checkpoint?)", MX_E_IO);
  const auto& s = f.info(name).shape;
  int64_t features = s.empty() ? 0 : s.back();
  int stages = 1;
  for (int n = 1; n < 3; ++n)
    if (f.contains("stage_" + std::to_string(n) + "_output_conv_1/kernel")) stages = n + 1;
  std::string v;
  if (features == 32) v = "S-" + std::to_string(stages);
  else if (features == 64) v = "M-" + std::to_string(stages);
  else
    throw Error(fmt("checkpoint has %lld features and %d stage(s), which is not one of the six published MAXIM "
                    "variants",
                    (long long)features, stages),
                MX_E_IO);
  return variant(v);
}

Config Config::for_task(const std::string& task) {
  std::string t = task;
  std::transform(t.begin(), t.end(), t.begin(), [](unsigned char ch) { return std::tolower(ch); });
  if (t == "denoising" || t == "deblurring") return variant("S-3");
  if (t == "deraining" || t == "dehazing" || t == "enhancement") return variant("S-2");
  throw Error("unknown task " + t + " (expected denoising, deblurring, deraining, dehazing, enhancement)");
}

}  // namespace mx
