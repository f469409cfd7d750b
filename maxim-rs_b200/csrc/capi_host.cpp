// extern "C" entry points of the host contract (weights, plan, image).
#include <cerrno>
#include <climits>
#include <cstdarg>
#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "common.h"
#include "config.h"
#include "image.h"
#include "model.h"
#include "weights.h"

namespace mx {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

std::string fmt(const char* f, ...) {
  va_list ap;
  va_start(ap, f);
  va_list ap2;
  va_copy(ap2, ap);
  int n = vsnprintf(nullptr, 0, f, ap);
  va_end(ap);
  std::string s(size_t(n > 0 ? n : 0), '\0');
  if (n > 0) vsnprintf(&s[0], size_t(n) + 1, f, ap2);
  va_end(ap2);
  return s;
}

}  // namespace mx

struct mx_weights {
  std::unique_ptr<mx::Weights> w;
};

struct mx_plan_handle {
  std::unique_ptr<mx::Plan> plan;
  mx_plan view;
};

using namespace mx;

namespace {
void copy_str(const std::string& s, char* buf, size_t len) {
  if (!buf || len == 0) return;
  size_t n = std::min(s.size(), len - 1);
  memcpy(buf, s.data(), n);
  buf[n] = '\0';
}
mx_image to_c(Image&& img) {
  mx_image o{};
  o.c = int32_t(img.c), o.h = int32_t(img.h), o.w = int32_t(img.w);
  o.data = static_cast<float*>(malloc(img.data.size() * sizeof(float) + 1));
  if (!o.data) throw Error("host allocation failed", MX_E_OOM);
  memcpy(o.data, img.data.data(), img.data.size() * sizeof(float));
  return o;
}
Image from_c(const mx_image* m) {
  if (!m || !m->data || m->c <= 0 || m->h <= 0 || m->w <= 0) throw Error("invalid image");
  Image img(m->c, m->h, m->w);
  memcpy(img.data.data(), m->data, img.data.size() * sizeof(float));
  return img;
}
}  // namespace

extern "C" {

size_t mx_last_error(char* buf, size_t len) {
  copy_str(g_last_error, buf, len);
  return g_last_error.size();
}

int mx_weights_open(const char* path, mx_weights** out) {
  return guard([&] {
    if (!path || !out) throw Error("mx_weights_open: null argument");
    auto h = std::make_unique<mx_weights>();
    h->w = Weights::open(path);
    *out = h.release();
  });
}

void mx_weights_free(mx_weights* w) { delete w; }

int mx_weights_variant(const mx_weights* w, char* buf, size_t len) {
  return guard([&] {
    if (!w) throw Error("mx_weights_variant: null handle");
    copy_str(w->w->config.name, buf, len);
  });
}

int mx_param_spec(const char* variant, char* buf, size_t len, size_t* needed) {
  return guard([&] {
    if (!variant) throw Error("mx_param_spec: null variant");
    Config cfg = Config::variant(variant);
    auto w = Weights::spec(cfg);
    // The inventory does not depend on the image size; 64x64 is the smallest
    // plan every variant can build.
    build_plan(*w, cfg, 64, 64, false);
    std::string s;
    for (auto& kv : w->requested()) {
      s += kv.first + "\t";
      for (size_t i = 0; i < kv.second.size(); ++i) s += (i ? "," : "") + std::to_string(kv.second[i]);
      s += "\n";
    }
    if (needed) *needed = s.size() + 1;
    copy_str(s, buf, len);
  });
}

int mx_plan_build(const mx_weights* w, int32_t h, int32_t wd, int dumps, mx_plan_handle** out) {
  return guard([&] {
    if (!w || !out) throw Error("mx_plan_build: null argument");
    if (h <= 0 || wd <= 0) throw Error("mx_plan_build: the image shape must be positive");
    auto p = std::make_unique<mx_plan_handle>();
    p->plan = build_plan(*w->w, w->w->config, h, wd, dumps != 0);
    p->view = p->plan->view();
    *out = p.release();
  });
}

int mx_plan_build_variant(const char* variant, int32_t h, int32_t wd, int dumps, mx_plan_handle** out) {
  return guard([&] {
    if (!variant || !out) throw Error("mx_plan_build_variant: null argument");
    if (h <= 0 || wd <= 0) throw Error("mx_plan_build_variant: the image shape must be positive");
    Config cfg = Config::variant(variant);
    auto w = Weights::spec(cfg);
    auto p = std::make_unique<mx_plan_handle>();
    p->plan = build_plan(*w, cfg, h, wd, dumps != 0);
    p->view = p->plan->view();
    *out = p.release();
  });
}

void mx_plan_free(mx_plan_handle* p) { delete p; }

const mx_plan* mx_plan_view(const mx_plan_handle* p) { return p ? &p->view : nullptr; }

int32_t mx_plan_dump_count(const mx_plan_handle* p) { return p ? int32_t(p->plan->dumps.size()) : 0; }

int mx_plan_dump(const mx_plan_handle* p, int32_t i, char* name, size_t len, int32_t* id) {
  return guard([&] {
    if (!p || i < 0 || size_t(i) >= p->plan->dumps.size()) throw Error("mx_plan_dump: index out of range");
    copy_str(p->plan->dumps[size_t(i)].first, name, len);
    if (id) *id = p->plan->dumps[size_t(i)].second;
  });
}

int mx_plan_label(const mx_plan_handle* p, int32_t id, char* buf, size_t len) {
  return guard([&] {
    if (!p || id < 0 || size_t(id) >= p->plan->labels.size()) throw Error("mx_plan_label: id out of range");
    copy_str(p->plan->labels[size_t(id)], buf, len);
  });
}

void mx_image_free(mx_image* img) {
  if (img) {
    free(img->data);
    img->data = nullptr;
  }
}

int mx_png_read(const char* path, mx_image* out) {
  return guard([&] {
    if (!path || !out) throw Error("mx_png_read: null argument");
    *out = to_c(read_png(path));
  });
}

int mx_png_read_mem(const uint8_t* bytes, size_t n, mx_image* out) {
  return guard([&] {
    if (!bytes || !out) throw Error("mx_png_read_mem: null argument");
    *out = to_c(read_png_bytes(bytes, n, "<memory>"));
  });
}

int mx_png_write(const char* path, const mx_image* img) {
  return guard([&] {
    if (!path) throw Error("mx_png_write: null path");
    write_png(path, from_c(img));
  });
}

int mx_preprocess(const mx_image* img, int32_t factor, mx_image* padded, int32_t* even_h, int32_t* even_w) {
  return guard([&] {
    if (!padded || factor <= 0) throw Error("mx_preprocess: bad argument");
    Padded p = preprocess(from_c(img), factor);
    if (even_h) *even_h = int32_t(p.even_h);
    if (even_w) *even_w = int32_t(p.even_w);
    *padded = to_c(std::move(p.img));
  });
}

int mx_pad_geometry(int32_t h, int32_t w, int32_t factor, int32_t* padded_h, int32_t* padded_w, int32_t* even_h,
                    int32_t* even_w) {
  return guard([&] {
    if (h <= 0 || w <= 0 || factor <= 0) throw Error("mx_pad_geometry: bad argument");
    const PadGeometry g = pad_geometry(h, w, factor);
    if (padded_h) *padded_h = int32_t(g.h);
    if (padded_w) *padded_w = int32_t(g.w);
    if (even_h) *even_h = int32_t(g.even_h);
    if (even_w) *even_w = int32_t(g.even_w);
  });
}

void mx_image8_free(mx_image8* img) {
  if (img) {
    free(img->data);
    img->data = nullptr;
  }
}

int mx_png_size_mem(const uint8_t* bytes, size_t n, int32_t* h, int32_t* w) {
  return guard([&] {
    if (!bytes || !h || !w) throw Error("mx_png_size_mem: null argument");
    const auto hw = png_size(bytes, n, "<memory>");
    if (hw.first > INT32_MAX || hw.second > INT32_MAX) throw Error("PNG dimensions out of range", MX_E_IO);
    *h = int32_t(hw.first), *w = int32_t(hw.second);
  });
}

int mx_png_read_rgb8_mem(const uint8_t* bytes, size_t n, mx_image8* out) {
  return guard([&] {
    if (!bytes || !out) throw Error("mx_png_read_rgb8_mem: null argument");
    Rgb8 px = decode_png_rgb8(bytes, n, "<memory>");
    mx_image8 o{};
    o.c = 3, o.h = int32_t(px.h), o.w = int32_t(px.w);
    o.data = static_cast<uint8_t*>(malloc(px.data.size() + 1));
    if (!o.data) throw Error("host allocation failed", MX_E_OOM);
    memcpy(o.data, px.data.data(), px.data.size());
    *out = o;
  });
}

int mx_png_write_rgb8(const char* path, const mx_image8* img) {
  return guard([&] {
    if (!path || !img || !img->data || img->c != 3 || img->h <= 0 || img->w <= 0)
      throw Error("mx_png_write_rgb8: needs a 3-channel image and a path");
    const std::vector<uint8_t> bytes = encode_png_rgb8(img->data, img->h, img->w);
    FILE* f = fopen(path, "wb");
    if (!f) throw Error(std::string(path) + ": " + strerror(errno), MX_E_IO);
    size_t wr = fwrite(bytes.data(), 1, bytes.size(), f);
    int rc = fclose(f);
    if (wr != bytes.size() || rc != 0) throw Error(std::string(path) + ": write failed", MX_E_IO);
  });
}

int mx_crop_out(const mx_image* pred, int32_t orig_h, int32_t orig_w, int32_t even_h, int32_t even_w,
                mx_image* out) {
  return guard([&] {
    if (!out) throw Error("mx_crop_out: null output");
    *out = to_c(crop_out(from_c(pred), orig_h, orig_w, even_h, even_w));
  });
}

}  // extern "C"
