// TEST INFRASTRUCTURE - the host side of the CPU baseline. Nothing in the
// product path links, loads or calls this file.
//
// The oracle library compiles the host contract's sources (safetensors
// reader, config, plan builder and packer, image pipeline: the C++
// restatement of src/weights.rs, src/config.rs, src/model.rs and
// src/image.rs) into itself with hidden visibility, and exports them here
// under `mxo_` names. A CPU-only timing of the reference's algorithm (the
// benchmark's reference arm) can then build its plan, read its checkpoint
// and pad its image without mapping the GPU product library at all.
#include "maxim_b200.h"

#define MXO_API extern "C" __attribute__((visibility("default")))

MXO_API size_t mxo_last_error(char* buf, size_t len) { return mx_last_error(buf, len); }

MXO_API int mxo_param_spec(const char* variant, char* buf, size_t len, size_t* needed) {
  return mx_param_spec(variant, buf, len, needed);
}

MXO_API int mxo_weights_open(const char* path, mx_weights** out) { return mx_weights_open(path, out); }
MXO_API void mxo_weights_free(mx_weights* w) { mx_weights_free(w); }

MXO_API int mxo_plan_build(const mx_weights* w, int32_t h, int32_t wd, int dumps, mx_plan_handle** out) {
  return mx_plan_build(w, h, wd, dumps, out);
}
MXO_API void mxo_plan_free(mx_plan_handle* p) { mx_plan_free(p); }
MXO_API const mx_plan* mxo_plan_view(const mx_plan_handle* p) { return mx_plan_view(p); }

MXO_API int mxo_preprocess(const mx_image* img, int32_t factor, mx_image* padded, int32_t* even_h, int32_t* even_w) {
  return mx_preprocess(img, factor, padded, even_h, even_w);
}
MXO_API void mxo_image_free(mx_image* img) { mx_image_free(img); }
