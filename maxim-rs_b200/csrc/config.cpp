#include "config.h"

#include <algorithm>
#include <cctype>
#include <cstdlib>

#include "common.h"
#include "safetensors.h"

namespace mx {

// The tensor a checkpoint of the isolated gMLP layer is recognised by.
static const char* kBlockProbe = "SplitHeadMultiAxisGmlpLayer/in_project/kernel";

Config Config::variant(const std::string& v) {
  if (v.rfind("gMLP-", 0) == 0) {
    const int c = std::atoi(v.c_str() + 5);
    if (c <= 0 || c % 2 != 0 || v != "gMLP-" + std::to_string(c))
      throw Error("unknown variant " + v + " (gMLP-<c> takes an even channel count)");
    Config g;
    g.name = v;
    g.features = c;
    g.num_stages = 0;
    g.block_only = true;
    return g;
  }
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
  if (f.contains(kBlockProbe) && !f.contains("stage_0_encoder_block_0/Conv_0/kernel")) {
    const auto& s = f.info(kBlockProbe).shape;  // Dense [c][2c]
    if (s.size() != 2) throw Error(std::string(kBlockProbe) + " is not a Dense kernel", MX_E_IO);
    return variant("gMLP-" + std::to_string(s[0]));
  }
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
