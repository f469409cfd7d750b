// The plan builder: one method per block of the reference model, with the
// same names and the same op and buffer order as src/model.rs:196-1076, so the
// op list, the buffer list and the packed arena come out identical (op and
// buffer counts and arena sizes are pinned by the tests against the figures
// the reference's own docs give).
#include "model.h"

#include <algorithm>
#include <cstdlib>
#include <limits>

#include "common.h"
#include "weights.h"

namespace mx {

namespace {

mx_op blank(int kind) {
  mx_op o{};
  o.kind = kind;
  o.dst = o.src = o.src2 = o.tmp = -1;
  o.w = o.wt = o.bias = o.scale = -1;
  return o;
}

// Flax's padding='SAME' for one axis (src/image.rs:108-112).
std::pair<int64_t, int64_t> same_pad(int64_t size, int64_t stride, int64_t k) {
  int64_t out = (size + stride - 1) / stride;
  int64_t total = std::max<int64_t>((out - 1) * stride + k - size, 0);
  return {total / 2, total - total / 2};
}

class Builder {
 public:
  Builder(const Weights& w, const Config& cfg, bool record) : w_(w), cfg_(cfg), record_(record) {
    deep_ = std::getenv("MAXIM_DEEP_DUMPS") != nullptr;
  }

  std::unique_ptr<Plan> build(int64_t h, int64_t wd);
  std::unique_ptr<Plan> build_block(int64_t h, int64_t wd);

 private:
  const Weights& w_;
  Config cfg_;
  std::vector<std::vector<float>> weights_;
  std::vector<mx_buf> bufs_;
  std::vector<std::string> labels_;
  std::vector<int32_t> alias_parent_;
  std::vector<int64_t> alias_delta_;
  std::vector<mx_op> ops_;
  std::vector<std::pair<std::string, int32_t>> named_;
  int up_index_ = 0;
  bool record_ = true;
  bool deep_ = false;

  int32_t buf(int64_t c, int64_t h, int64_t w, const char* label) {
    bufs_.push_back({c, h, w});
    labels_.emplace_back(label);
    alias_parent_.push_back(-1);
    alias_delta_.push_back(0);
    return int32_t(bufs_.size() - 1);
  }
  // A channel range of another buffer: no storage of its own.
  int32_t view(int32_t base, int64_t ch, int64_t c, const char* label) {
    mx_buf s = bufs_[base];
    bufs_.push_back({c, s.h, s.w});
    labels_.emplace_back(label);
    alias_parent_.push_back(base);
    alias_delta_.push_back(ch * s.h * s.w);
    return int32_t(bufs_.size() - 1);
  }
  void rec(const std::string& name, int32_t id) {
    if (record_) named_.emplace_back(name, id);
  }
  void deep_rec(const std::string& name, int32_t id) {
    if (deep_) rec(name, id);
  }
  int32_t weight(std::vector<float> v) {
    weights_.push_back(std::move(v));
    return int32_t(weights_.size() - 1);
  }
  int32_t own(const std::string& name, int64_t n) { return weight(w_.vec(name, n)); }
  // A bias that may be absent from the checkpoint: zeros stand in
  // (src/model.rs:274-283).
  int32_t own_or_zeros(const std::string& name, int64_t n) {
    if (w_.has(name)) return own(name, n);
    return weight(std::vector<float>(size_t(n), 0.0f));
  }
  int32_t opt_bias(const std::string& prefix, int64_t n) {
    std::string b = prefix + "/bias";
    return w_.has(b) ? own(b, n) : -1;
  }
  void push(const mx_op& o) { ops_.push_back(o); }
  int64_t len(int32_t id) const { return bufs_[id].c * bufs_[id].h * bufs_[id].w; }

  void chan_ln(int32_t dst, int32_t src, const std::string& prefix, int64_t c, int64_t hw) {
    int32_t s = own(prefix + "/scale", c);
    int32_t b = own_or_zeros(prefix + "/bias", c);
    mx_op o = blank(MX_OP_CHAN_LN);
    o.dst = dst, o.src = src, o.scale = s, o.bias = b, o.c = int32_t(c), o.hw = hw;
    push(o);
  }
  void conv1x1(int32_t dst, int32_t src, const std::string& prefix, int64_t ci, int64_t co, int64_t h, int64_t wd,
               bool dense) {
    int32_t w = weight(w_.conv1x1(prefix + "/kernel", ci, co, dense));
    int32_t bias = opt_bias(prefix, co);
    mx_op o = blank(MX_OP_CONV1X1);
    o.dst = dst, o.src = src, o.w = w, o.bias = bias;
    o.c_in = int32_t(ci), o.c_out = int32_t(co), o.h = int32_t(h), o.wd = int32_t(wd);
    push(o);
  }
  void conv3x3(int32_t dst, int32_t src, const std::string& prefix, int64_t ci, int64_t co, int64_t h, int64_t wd) {
    int32_t w = weight(w_.convkxk(prefix + "/kernel", 3, ci, co));
    int32_t bias = opt_bias(prefix, co);
    mx_op o = blank(MX_OP_CONV3X3);
    o.dst = dst, o.src = src, o.w = w, o.bias = bias;
    o.c_in = int32_t(ci), o.c_out = int32_t(co), o.h = int32_t(h), o.wd = int32_t(wd);
    push(o);
  }
  // Conv_down: 4x4 stride 2, SAME padding (src/model.rs:335-349).
  void conv_down(int32_t dst, int32_t src, const std::string& prefix, int64_t ci, int64_t co, int64_t h,
                 int64_t wd) {
    int32_t w = weight(w_.convkxk(prefix + "/kernel", 4, ci, co));
    int32_t bias = opt_bias(prefix, co);
    mx_op o = blank(MX_OP_CONV4X4S2);
    o.dst = dst, o.src = src, o.w = w, o.bias = bias;
    o.c_in = int32_t(ci), o.c_out = int32_t(co), o.h = int32_t(h), o.wd = int32_t(wd);
    o.oh = int32_t((h + 1) / 2), o.ow = int32_t((wd + 1) / 2);
    o.pad_top = int32_t(same_pad(h, 2, 4).first), o.pad_left = int32_t(same_pad(wd, 2, 4).first);
    push(o);
  }
  // ConvT_up: 2x2 stride 2 transposed; h/wd are the INPUT dims.
  void convt_up(int32_t dst, int32_t src, const std::string& prefix, int64_t ci, int64_t co, int64_t h,
                int64_t wd) {
    int32_t w = weight(w_.convt2x2(prefix + "/kernel", ci, co));
    int32_t bias = opt_bias(prefix, co);
    mx_op o = blank(MX_OP_CONVT2X2);
    o.dst = dst, o.src = src, o.w = w, o.bias = bias;
    o.c_in = int32_t(ci), o.c_out = int32_t(co), o.h = int32_t(h), o.wd = int32_t(wd);
    push(o);
  }
  void elem(int kind, int32_t dst, int32_t a, int32_t b, int64_t n, float slope = 0.0f) {
    mx_op o = blank(kind);
    o.dst = dst, o.src = a, o.src2 = b, o.n = n, o.slope = slope;
    push(o);
  }
  void gelu(int32_t dst, int32_t src, int64_t n) { elem(MX_OP_GELU, dst, src, -1, n); }
  void add(int32_t dst, int32_t a, int32_t b, int64_t n) { elem(MX_OP_ADD, dst, a, b, n); }
  void mul(int32_t dst, int32_t a, int32_t b, int64_t n) { elem(MX_OP_MUL, dst, a, b, n); }
  // jax `nearest` downsample: stride `factor`, offset factor/2 (src/model.rs:376-384).
  void nearest_down(int32_t dst, int32_t src, int64_t c, int64_t h, int64_t w, int64_t factor) {
    mx_op o = blank(MX_OP_DOWN_S);
    o.dst = dst, o.src = src, o.c = int32_t(c), o.h = int32_t(h), o.wd = int32_t(w);
    o.stride = int32_t(factor), o.off = int32_t(factor / 2);
    o.oh = int32_t(h / factor), o.ow = int32_t(w / factor);
    push(o);
  }
  // Bilinear resize (jax rule), a Copy when the shape does not change.
  void resize(int32_t dst, int32_t src, int64_t c, int64_t hin, int64_t win, int64_t hout, int64_t wout) {
    if (hin == hout && win == wout) {
      elem(MX_OP_COPY, dst, src, -1, c * hin * win);
      return;
    }
    int32_t tmp = buf(c, hin, wout, "resize_tmp");
    mx_op o = blank(MX_OP_RESIZE);
    o.dst = dst, o.src = src, o.tmp = tmp, o.c = int32_t(c);
    o.hin = int32_t(hin), o.win = int32_t(win), o.hout = int32_t(hout), o.wout = int32_t(wout);
    push(o);
  }
  void block_perm(int32_t dst, int32_t src, int64_t c, int64_t h, int64_t wd, int64_t gh, int64_t gw, int64_t fh,
                  int64_t fw, bool forward) {
    mx_op o = blank(MX_OP_BLOCK_PERM);
    o.dst = dst, o.src = src, o.c = int32_t(c), o.h = int32_t(h), o.wd = int32_t(wd);
    o.gh = int32_t(gh), o.gw = int32_t(gw), o.fh = int32_t(fh), o.fw = int32_t(fw);
    o.swap = 0, o.forward = forward ? 1 : 0;
    push(o);
  }
  void gate_mm(int32_t dst, int32_t src, int32_t w, int32_t bias, int64_t c, int64_t outer, int64_t inner, int mode) {
    mx_op o = blank(MX_OP_GATE_MM);
    o.dst = dst, o.src = src, o.w = w, o.bias = bias, o.c = int32_t(c);
    o.outer = int32_t(outer), o.inner = int32_t(inner), o.mode = mode;
    push(o);
  }

  // -- leaf blocks (src/model.rs:392-475) -----------------------------------
  int32_t calayer(const std::string& prefix, int32_t x, int64_t c, int64_t h, int64_t wd, int64_t red) {
    int64_t hw = h * wd;
    int32_t mean = buf(c, 1, 1, "ca_mean");
    {
      mx_op o = blank(MX_OP_CHAN_MEAN);
      o.dst = mean, o.src = x, o.c = int32_t(c), o.hw = hw;
      push(o);
    }
    deep_rec(prefix + "_mean", mean);
    int32_t sq = buf(c / red, 1, 1, "ca_squeeze");
    conv1x1(sq, mean, prefix + "/Conv_0", c, c / red, 1, 1, false);
    deep_rec(prefix + "_sq", sq);
    int32_t rl = buf(c / red, 1, 1, "ca_relu");
    elem(MX_OP_LRELU, rl, sq, -1, c / red, 0.0f);
    deep_rec(prefix + "_relu", rl);
    int32_t ex = buf(c, 1, 1, "ca_excite");
    conv1x1(ex, rl, prefix + "/Conv_1", c / red, c, 1, 1, false);
    deep_rec(prefix + "_excite", ex);
    int32_t sg = buf(c, 1, 1, "ca_sigmoid");
    elem(MX_OP_SIGMOID, sg, ex, -1, c);
    deep_rec(prefix + "_sigmoid", sg);
    int32_t out = buf(c, h, wd, "ca_out");
    {
      mx_op o = blank(MX_OP_CHAN_SCALE);
      o.dst = out, o.src = x, o.src2 = sg, o.c = int32_t(c), o.hw = hw;
      push(o);
    }
    return out;
  }

  int32_t rcab(const std::string& prefix, int32_t x, int64_t c, int64_t h, int64_t wd, int64_t red) {
    int64_t n = c * h * wd;
    int32_t y = buf(c, h, wd, "rcab_ln");
    chan_ln(y, x, prefix + "/LayerNorm", c, h * wd);
    deep_rec(prefix + "_ln", y);
    int32_t t = buf(c, h, wd, "rcab_conv1");
    conv3x3(t, y, prefix + "/conv1", c, c, h, wd);
    deep_rec(prefix + "_conv1", t);
    int32_t r = buf(c, h, wd, "rcab_lrelu");
    elem(MX_OP_LRELU, r, t, -1, n, 0.2f);
    deep_rec(prefix + "_lrelu", r);
    int32_t t2 = buf(c, h, wd, "rcab_conv2");
    conv3x3(t2, r, prefix + "/conv2", c, c, h, wd);
    deep_rec(prefix + "_conv2", t2);
    int32_t ca = calayer(prefix + "/channel_attention", t2, c, h, wd, red);
    deep_rec(prefix + "_ca", ca);
    int32_t out = buf(c, h, wd, "rcab_out");
    add(out, ca, x, n);
    return out;
  }

  int32_t rdcab(const std::string& prefix, int32_t x, int64_t c, int64_t h, int64_t wd, int64_t red) {
    int64_t n = c * h * wd;
    int32_t y = buf(c, h, wd, "rdcab_ln");
    chan_ln(y, x, prefix + "/LayerNorm", c, h * wd);
    int32_t c1 = buf(c, h, wd, "rdcab_dense0");
    conv1x1(c1, y, prefix + "/channel_mixing/Dense_0", c, c, h, wd, true);
    int32_t g = buf(c, h, wd, "rdcab_gelu");
    gelu(g, c1, n);
    int32_t c2 = buf(c, h, wd, "rdcab_dense1");
    conv1x1(c2, g, prefix + "/channel_mixing/Dense_1", c, c, h, wd, true);
    int32_t ca = calayer(prefix + "/channel_attention", c2, c, h, wd, red);
    int32_t out = buf(c, h, wd, "rdcab_out");
    add(out, ca, x, n);
    return out;
  }

  // Grid/Block gating unit: u * (Dense(layer_norm(v)) + 1) (src/model.rs:485-506).
  void gating(const std::string& prefix, int32_t u, int32_t v, int32_t dst, int64_t c, int64_t gg, int64_t pp,
              bool over_grid) {
    int64_t n = c * gg * pp;
    int32_t ln = buf(c, gg, pp, "gmlp_gate_ln");
    chan_ln(ln, v, prefix + "/intermediate_layernorm", c, gg * pp);
    int32_t g = buf(c, gg, pp, "gmlp_gate");
    int64_t nb = over_grid ? gg : pp;
    int32_t w = weight(w_.dense(prefix + "/Dense_0/kernel", nb));
    int32_t b = own_or_zeros(prefix + "/Dense_0/bias", nb);
    gate_mm(g, ln, w, b, c, gg, pp, over_grid ? 0 : 1);
    elem(MX_OP_GATE_APPLY, dst, u, g, n);
  }

  // One half of a multi-axis gMLP layer (src/model.rs:520-572).
  void gmlp_axis(const std::string& prefix, int32_t x, int32_t dst, int64_t c, int64_t h, int64_t wd, int64_t size,
                 bool over_grid) {
    int64_t gh, gw, fh, fw;
    if (over_grid) gh = size, gw = size, fh = h / size, fw = wd / size;
    else gh = h / size, gw = wd / size, fh = size, fw = size;
    if (gh == 0 || gw == 0 || fh == 0 || fw == 0)
      throw Error(fmt("%s: a %lld-%s does not fit a %lldx%lld feature map (cells %lldx%lld, %lldx%lld pixels) - the "
                      "input is too small for this model",
                      prefix.c_str(), (long long)size, over_grid ? "cell grid" : "pixel block", (long long)h,
                      (long long)wd, (long long)gh, (long long)gw, (long long)fh, (long long)fw));
    int64_t gg = gh * gw, pp = fh * fw;
    int32_t xb = buf(c, gg, pp, "gmlp_blocked");
    block_perm(xb, x, c, h, wd, gh, gw, fh, fw, true);
    deep_rec(prefix + "_blocked", xb);
    int32_t ln = buf(c, gg, pp, "gmlp_ln");
    chan_ln(ln, xb, prefix + "/LayerNorm", c, gg * pp);
    deep_rec(prefix + "_ln", ln);
    int32_t t = buf(2 * c, gg, pp, "gmlp_inproject");
    conv1x1(t, ln, prefix + "/in_project", c, 2 * c, gg, pp, true);
    deep_rec(prefix + "_inproject", t);
    int32_t tg = buf(2 * c, gg, pp, "gmlp_gelu");
    gelu(tg, t, 2 * c * gg * pp);
    deep_rec(prefix + "_gelu", tg);
    int32_t u = view(tg, 0, c, "gmlp_u");
    int32_t v = view(tg, c, c, "gmlp_v");
    int32_t gated = buf(c, gg, pp, "gmlp_gated");
    gating(prefix + (over_grid ? "/GridGatingUnit" : "/BlockGatingUnit"), u, v, gated, c, gg, pp, over_grid);
    deep_rec(prefix + "_gated", gated);
    int32_t proj = buf(c, gg, pp, "gmlp_outproject");
    conv1x1(proj, gated, prefix + "/out_project", c, c, gg, pp, true);
    deep_rec(prefix + "_proj", proj);
    int32_t mixed = buf(c, gg, pp, "gmlp_residual");
    add(mixed, proj, xb, c * gg * pp);
    block_perm(dst, mixed, c, h, wd, gh, gw, fh, fw, false);
  }

  // ResidualSplitHeadMultiAxisGmlpLayer (src/model.rs:576-603).
  int32_t split_head_gmlp(const std::string& prefix, int32_t x, int64_t c, int64_t h, int64_t wd, int64_t bs,
                          int64_t gs) {
    int32_t ln = buf(c, h, wd, "shg_ln");
    chan_ln(ln, x, prefix + "/LayerNorm_in", c, h * wd);
    int32_t t = buf(2 * c, h, wd, "shg_inproject");
    conv1x1(t, ln, prefix + "/in_project", c, 2 * c, h, wd, true);
    int32_t g = buf(2 * c, h, wd, "shg_gelu");
    gelu(g, t, 2 * c * h * wd);
    int32_t u = view(g, 0, c, "shg_u");
    int32_t v = view(g, c, c, "shg_v");
    gmlp_axis(prefix + "/GridGmlpLayer", u, u, c, h, wd, gs, true);
    gmlp_axis(prefix + "/BlockGmlpLayer", v, v, c, h, wd, bs, false);
    int32_t proj = buf(c, h, wd, "shg_outproject");
    conv1x1(proj, g, prefix + "/out_project", 2 * c, c, h, wd, true);
    int32_t out = buf(c, h, wd, "shg_out");
    add(out, proj, x, c * h * wd);
    return out;
  }

  // GetSpatialGatingWeights (src/model.rs:612-668).
  int32_t spatial_gating_weights(const std::string& prefix, int32_t x, int64_t c, int64_t h, int64_t wd, int64_t bs,
                                 int64_t gs) {
    int32_t ln = buf(c, h, wd, "sgw_ln");
    chan_ln(ln, x, prefix + "/LayerNorm_in", c, h * wd);
    int32_t t = buf(2 * c, h, wd, "sgw_inproject");
    conv1x1(t, ln, prefix + "/in_project", c, 2 * c, h, wd, true);
    int32_t g = buf(2 * c, h, wd, "sgw_gelu");
    gelu(g, t, 2 * c * h * wd);
    int32_t u = view(g, 0, c, "sgw_u");
    int32_t v = view(g, c, c, "sgw_v");

    int64_t gh = gs, gw = gs, fh = h / gh, fw = wd / gw, gg = gh * gw, pp = fh * fw;
    int32_t ub = buf(c, gg, pp, "sgw_u_blocked");
    block_perm(ub, u, c, h, wd, gh, gw, fh, fw, true);
    int32_t um = buf(c, gg, pp, "sgw_u_mixed");
    int32_t uw = weight(w_.dense(prefix + "/Dense_0/kernel", gg));
    int32_t ubias = own_or_zeros(prefix + "/Dense_0/bias", gg);
    gate_mm(um, ub, uw, ubias, c, gg, pp, 0);
    int32_t uu = buf(c, h, wd, "sgw_u_out");
    block_perm(uu, um, c, h, wd, gh, gw, fh, fw, false);

    int64_t fh2 = bs, fw2 = bs, gh2 = h / fh2, gw2 = wd / fw2, gg2 = gh2 * gw2, pp2 = fh2 * fw2;
    int32_t vb = buf(c, gg2, pp2, "sgw_v_blocked");
    block_perm(vb, v, c, h, wd, gh2, gw2, fh2, fw2, true);
    int32_t vm = buf(c, gg2, pp2, "sgw_v_mixed");
    int32_t vw = weight(w_.dense(prefix + "/Dense_1/kernel", pp2));
    int32_t vbias = own_or_zeros(prefix + "/Dense_1/bias", pp2);
    gate_mm(vm, vb, vw, vbias, c, gg2, pp2, 1);
    int32_t vv = buf(c, h, wd, "sgw_v_out");
    block_perm(vv, vm, c, h, wd, gh2, gw2, fh2, fw2, false);

    int32_t cat = buf(2 * c, h, wd, "sgw_cat");
    int32_t lo = view(cat, 0, c, "sgw_cat_lo");
    int32_t hi = view(cat, c, c, "sgw_cat_hi");
    elem(MX_OP_COPY, lo, uu, -1, c * h * wd);
    elem(MX_OP_COPY, hi, vv, -1, c * h * wd);
    int32_t out = buf(c, h, wd, "sgw_out");
    conv1x1(out, cat, prefix + "/out_project", 2 * c, c, h, wd, true);
    return out;
  }

  // CrossGatingBlock, returning (x, y) (src/model.rs:671-734).
  std::pair<int32_t, int32_t> cross_gating(const std::string& prefix, int32_t x, int64_t cx, int32_t y, int64_t cy,
                                           int64_t h, int64_t wd, int64_t f, int64_t bs, int64_t gs,
                                           bool upsample_y) {
    int64_t n = f * h * wd;
    int32_t y_up = y;
    if (upsample_y) {
      y_up = buf(f, h, wd, "cg_y_up");
      convt_up(y_up, y, prefix + "/ConvTranspose_0", cy, f, h / 2, wd / 2);
    }
    int32_t x0 = buf(f, h, wd, "cg_x0");
    conv1x1(x0, x, prefix + "/Conv_0", cx, f, h, wd, false);
    int32_t y0 = buf(f, h, wd, "cg_y0");
    conv1x1(y0, y_up, prefix + "/Conv_1", f, f, h, wd, false);

    int32_t xl = buf(f, h, wd, "cg_xln");
    chan_ln(xl, x0, prefix + "/LayerNorm_x", f, h * wd);
    int32_t xd = buf(f, h, wd, "cg_xdense");
    conv1x1(xd, xl, prefix + "/in_project_x", f, f, h, wd, true);
    int32_t xg = buf(f, h, wd, "cg_xgelu");
    gelu(xg, xd, n);
    int32_t gx = spatial_gating_weights(prefix + "/SplitHeadMultiAxisGating_x", xg, f, h, wd, bs, gs);

    int32_t yl = buf(f, h, wd, "cg_yln");
    chan_ln(yl, y0, prefix + "/LayerNorm_y", f, h * wd);
    int32_t yd = buf(f, h, wd, "cg_ydense");
    conv1x1(yd, yl, prefix + "/in_project_y", f, f, h, wd, true);
    int32_t yg = buf(f, h, wd, "cg_ygelu");
    gelu(yg, yd, n);
    int32_t gy = spatial_gating_weights(prefix + "/SplitHeadMultiAxisGating_y", yg, f, h, wd, bs, gs);

    int32_t ym = buf(f, h, wd, "cg_y_mul");
    mul(ym, yg, gx, n);
    int32_t yp = buf(f, h, wd, "cg_y_proj");
    conv1x1(yp, ym, prefix + "/out_project_y", f, f, h, wd, true);
    int32_t yo = buf(f, h, wd, "cg_y_out");
    add(yo, yp, y0, n);

    int32_t xm = buf(f, h, wd, "cg_x_mul");
    mul(xm, xg, gy, n);
    int32_t xp = buf(f, h, wd, "cg_x_proj");
    conv1x1(xp, xm, prefix + "/out_project_x", f, f, h, wd, true);
    int32_t xs = buf(f, h, wd, "cg_x_sum");
    add(xs, xp, yo, n);
    int32_t xo = buf(f, h, wd, "cg_x_out");
    add(xo, xs, x0, n);
    return {xo, yo};
  }

  std::pair<int64_t, int64_t> block_grid(int level) const {
    if (level < cfg_.high_res_stages) return {cfg_.block_size_hr, cfg_.grid_size_hr};
    return {cfg_.block_size_lr, cfg_.grid_size_lr};
  }

  // UpSampleRatio: resize to level `to`, then 1x1 to features_i
  // (src/model.rs:908-916; the name counter follows call order).
  int32_t upsampled(int32_t enc, int64_t c_in, int from, int to, int64_t h, int64_t wd, int64_t fi) {
    std::string name = "UpSampleRatio_" + std::to_string(up_index_++);
    int32_t r = buf(c_in, h >> to, wd >> to, "up_resize");
    resize(r, enc, c_in, h >> from, wd >> from, h >> to, wd >> to);
    int32_t o = buf(fi, h >> to, wd >> to, "up_conv");
    conv1x1(o, r, name + "/Conv_0", c_in, fi, h >> to, wd >> to, false);
    return o;
  }

  int32_t multiscale_signal(const std::vector<int32_t>& encs, int i, int64_t fi, int64_t h, int64_t wd) {
    int64_t ch = h >> i, cw = wd >> i;
    int32_t cat = buf(3 * fi, ch, cw, "cg_signal");
    for (size_t j = 0; j < encs.size(); ++j) {
      int32_t p = upsampled(encs[j], bufs_[encs[j]].c, int(j), i, h, wd, fi);
      int32_t dst = view(cat, int64_t(j) * fi, fi, "cg_signal_part");
      elem(MX_OP_COPY, dst, p, -1, fi * ch * cw);
    }
    return cat;
  }

  int32_t decoder_signal(const std::vector<int32_t>& skips, int i, int64_t fi, int64_t h, int64_t wd, int depth) {
    int64_t ch = h >> i, cw = wd >> i;
    int32_t cat = buf(3 * fi, ch, cw, "dec_signal");
    for (size_t j = 0; j < skips.size(); ++j) {
      int from = depth - 1 - int(j);
      int32_t p = upsampled(skips[j], bufs_[skips[j]].c, from, i, h, wd, fi);
      int32_t dst = view(cat, int64_t(j) * fi, fi, "dec_signal_part");
      elem(MX_OP_COPY, dst, p, -1, fi * ch * cw);
    }
    return cat;
  }

  // UNetEncoderBlock, returning (downsampled, bridge) (src/model.rs:954-1012).
  std::pair<int32_t, int32_t> unet_encoder_block(const std::string& prefix, int32_t x, int64_t f, int64_t bs,
                                                 int64_t gs, int ngroups, int64_t red, bool downsample, int32_t skip,
                                                 int32_t enc, int32_t dec, int64_t h, int64_t wd) {
    int64_t c_in = bufs_[x].c + (skip >= 0 ? bufs_[skip].c : 0);
    int32_t xin = x;
    if (skip >= 0) {
      // flax concatenates along the channel axis, in the order (x, skip).
      int32_t cat = buf(c_in, h, wd, "enc_skip_cat");
      int32_t a = view(cat, 0, bufs_[x].c, "enc_skip_x");
      int32_t b = view(cat, bufs_[x].c, bufs_[skip].c, "enc_skip_skip");
      elem(MX_OP_COPY, a, x, -1, len(x));
      elem(MX_OP_COPY, b, skip, -1, len(skip));
      xin = cat;
    }
    deep_rec(prefix + "_mid_cat", xin);
    int32_t t = buf(f, h, wd, "enc_conv");
    conv1x1(t, xin, prefix + "/Conv_0", c_in, f, h, wd, false);
    deep_rec(prefix + "_mid_conv", t);
    int32_t y = t;
    for (int g = 0; g < ngroups; ++g) {
      y = split_head_gmlp(prefix + "/SplitHeadMultiAxisGmlpLayer_" + std::to_string(g), y, f, h, wd, bs, gs);
      deep_rec(prefix + "_mid_g" + std::to_string(g) + "_gmlp", y);
      y = rcab(prefix + "/channel_attention_block_1" + std::to_string(g), y, f, h, wd, red);
      deep_rec(prefix + "_mid_g" + std::to_string(g) + "_rcab", y);
    }
    int32_t summed = buf(f, h, wd, "enc_residual");
    add(summed, y, t, f * h * wd);
    deep_rec(prefix + "_mid_sum", summed);
    int32_t out = summed;
    if (enc >= 0 && dec >= 0) {
      int32_t yd = buf(f, h, wd, "enc_encdec");
      add(yd, enc, dec, f * h * wd);
      out = cross_gating(prefix + "/cross_gating_block", summed, f, yd, f, h, wd, f, bs, gs, false).first;
    }
    if (downsample) {
      int32_t down = buf(f, (h + 1) / 2, (wd + 1) / 2, "enc_down");
      conv_down(down, out, prefix + "/Conv_1", f, f, h, wd);
      return {down, out};
    }
    return {out, out};
  }

  int32_t unet_decoder_block(const std::string& prefix, int32_t x, int32_t bridge, int64_t f, int64_t bs, int64_t gs,
                             int ngroups, int64_t red, int64_t h, int64_t wd) {
    int32_t up = buf(f, h, wd, "dec_up");
    convt_up(up, x, prefix + "/ConvTranspose_0", bufs_[x].c, f, h / 2, wd / 2);
    return unet_encoder_block(prefix + "/UNetEncoderBlock_0", up, f, bs, gs, ngroups, red, false, bridge, -1, -1, h,
                              wd)
        .first;
  }

  // The supervised attention module, returning (sam, image) (src/model.rs:1041-1061).
  std::pair<int32_t, int32_t> sam(const std::string& prefix, int32_t x, int32_t x_image, int64_t f, int64_t h,
                                  int64_t wd) {
    int64_t n = f * h * wd;
    int32_t x1 = buf(f, h, wd, "sam_x1");
    conv3x3(x1, x, prefix + "/Conv_0", f, f, h, wd);
    int32_t t = buf(3, h, wd, "sam_img_conv");
    conv3x3(t, x, prefix + "/Conv_1", f, 3, h, wd);
    int32_t image = buf(3, h, wd, "sam_image");
    add(image, t, x_image, 3 * h * wd);
    int32_t s = buf(f, h, wd, "sam_img_pre_sigmoid");
    conv3x3(s, image, prefix + "/Conv_2", 3, f, h, wd);
    int32_t gate = buf(f, h, wd, "sam_sigmoid");
    elem(MX_OP_SIGMOID, gate, s, -1, n);
    int32_t g = buf(f, h, wd, "sam_gated");
    mul(g, x1, gate, n);
    int32_t sm = buf(f, h, wd, "sam_out");
    add(sm, g, x, n);
    return {sm, image};
  }

  int32_t bottleneck(const std::string& prefix, int32_t x, int64_t f, int64_t h, int64_t wd, int64_t bs, int ngroups,
                     int64_t red) {
    int32_t t = buf(f, h, wd, "bn_inputproj");
    conv1x1(t, x, prefix + "/input_proj", bufs_[x].c, f, h, wd, false);
    int32_t y = t;
    for (int g = 0; g < ngroups; ++g) {
      y = split_head_gmlp(prefix + "/SplitHeadMultiAxisGmlpLayer_" + std::to_string(g), y, f, h, wd, bs, bs);
      y = rdcab(prefix + "/channel_attention_block_1_" + std::to_string(g), y, f, h, wd, red);
    }
    int32_t out = buf(f, h, wd, "bn_out");
    add(out, y, t, f * h * wd);
    return out;
  }

  std::unique_ptr<Plan> finish(int32_t input, int32_t output, mx_buf shape);
};

// One residual split-head multi-axis gMLP layer on its own (BASELINE's
// isolated block op): the same builder method the model calls
// (`split_head_gmlp`, src/model.rs:576-603), over a c-channel input.
std::unique_ptr<Plan> Builder::build_block(int64_t h, int64_t wd) {
  const int64_t c = cfg_.features;
  int32_t input = buf(c, h, wd, "input");
  rec("input", input);
  int32_t out = split_head_gmlp("SplitHeadMultiAxisGmlpLayer", input, c, h, wd, cfg_.block_size_hr,
                                cfg_.grid_size_hr);
  rec("final", out);
  return finish(input, out, mx_buf{c, h, wd});
}

std::unique_ptr<Plan> Builder::build(int64_t h, int64_t wd) {
  if (cfg_.block_only) return build_block(h, wd);
  const int depth = cfg_.depth, stages = cfg_.num_stages, nss = cfg_.num_supervision_scales;
  const int64_t features = cfg_.features;
  const int64_t red = cfg_.channels_reduction;
  const int ngroups = cfg_.num_groups;

  int32_t input = buf(3, h, wd, "input");
  rec("input", input);

  // The multi-scale input pyramid (jax nearest: shortcuts[i] is NOT
  // shortcuts[i-1] downsampled again).
  std::vector<int32_t> shortcuts{input};
  for (int i = 1; i < nss; ++i) {
    int64_t f = int64_t(1) << i;
    int32_t d = buf(3, h / f, wd / f, "shortcut");
    nearest_down(d, input, 3, h, wd, f);
    shortcuts.push_back(d);
  }

  std::vector<std::vector<int32_t>> outputs_all;
  std::vector<int32_t> sam_prev, encs_prev, decs_prev;
  auto pop = [](std::vector<int32_t>& v, const char* what) {
    if (v.empty()) throw Error(what);
    int32_t x = v.back();
    v.pop_back();
    return x;
  };

  for (int s = 0; s < stages; ++s) {
    std::string S = std::to_string(s);
    std::vector<int32_t> x_scales;
    for (int i = 0; i < nss; ++i) {
      int64_t c = (int64_t(1) << i) * features;
      int32_t xs = buf(c, h >> i, wd >> i, "input_conv");
      conv3x3(xs, shortcuts[i], "stage_" + S + "_input_conv_" + std::to_string(i), 3, c, h >> i, wd >> i);
      if (s > 0) {
        auto bg = block_grid(i);
        int32_t sm = pop(sam_prev, "stage input fuse: no SAM feature left");
        x_scales.push_back(cross_gating("stage_" + S + "_input_fuse_sam_" + std::to_string(i), xs, c, sm, c, h >> i,
                                        wd >> i, c, bg.first, bg.second, false)
                               .first);
      } else {
        x_scales.push_back(xs);
      }
      rec("stage" + S + "_input_conv" + std::to_string(i), x_scales.back());
    }

    // Encoder: every level downsamples, the last one included.
    std::vector<int32_t> encs;
    int32_t x = x_scales[0];
    for (int i = 0; i < depth; ++i) {
      auto bg = block_grid(i);
      int64_t fi = (int64_t(1) << i) * features;
      int64_t ch = h >> i, cw = wd >> i;
      int32_t skip = i < nss ? x_scales[i] : -1;
      int32_t enc_prev = s > 0 ? pop(encs_prev, "encoder: no enc feature left") : -1;
      int32_t dec_prev = s > 0 ? pop(decs_prev, "encoder: no dec feature left") : -1;
      auto r = unet_encoder_block("stage_" + S + "_encoder_block_" + std::to_string(i), x, fi, bg.first, bg.second,
                                  ngroups, red, true, skip, enc_prev, dec_prev, ch, cw);
      rec("stage" + S + "_enc" + std::to_string(i) + "_bridge", r.second);
      rec("stage" + S + "_enc" + std::to_string(i) + "_out", r.first);
      x = r.first;
      encs.push_back(r.second);
    }

    // The global bottleneck at h / 2^depth.
    int64_t global_c = (int64_t(1) << (depth - 1)) * features;
    int64_t bh = h >> depth, bw = wd >> depth;
    for (int i = 0; i < cfg_.num_bottleneck_blocks; ++i)
      x = bottleneck("stage_" + S + "_global_block_" + std::to_string(i), x, global_c, bh, bw, cfg_.block_size_lr,
                     ngroups, red);
    rec("stage" + S + "_global", x);
    int32_t global_feature = x;

    // Cross gating, coarse to fine.
    std::vector<int32_t> skip_features;
    for (int i = depth - 1; i >= 0; --i) {
      auto bg = block_grid(i);
      int64_t fi = (int64_t(1) << i) * features;
      int64_t ch = h >> i, cw = wd >> i;
      int32_t signal = multiscale_signal(encs, i, fi, h, wd);
      auto r = cross_gating("stage_" + S + "_cross_gating_block_" + std::to_string(i), signal, 3 * fi,
                            global_feature, global_c, ch, cw, fi, bg.first, bg.second, true);
      global_feature = r.second;
      global_c = fi;
      rec("stage" + S + "_skip" + std::to_string(i), r.first);
      skip_features.push_back(r.first);
    }

    // Decoder.
    std::vector<int32_t> outputs, decs, sam_new;
    for (int i = depth - 1; i >= 0; --i) {
      auto bg = block_grid(i);
      int64_t fi = (int64_t(1) << i) * features;
      int64_t ch = h >> i, cw = wd >> i;
      int32_t signal = decoder_signal(skip_features, i, fi, h, wd, depth);
      x = unet_decoder_block("stage_" + S + "_decoder_block_" + std::to_string(i), x, signal, fi, bg.first, bg.second,
                             ngroups, red, ch, cw);
      rec("stage" + S + "_dec" + std::to_string(i), x);
      decs.push_back(x);
      if (i < nss) {
        if (s + 1 < stages) {
          auto r = sam("stage_" + S + "_supervised_attention_module_" + std::to_string(i), x, shortcuts[i], fi, ch, cw);
          outputs.push_back(r.second);
          sam_new.push_back(r.first);
          rec("stage" + S + "_sam" + std::to_string(i), r.first);
        } else {
          int32_t o = buf(3, ch, cw, "output");
          conv3x3(o, x, "stage_" + S + "_output_conv_" + std::to_string(i), fi, 3, ch, cw);
          int32_t out = buf(3, ch, cw, "stage_out");
          add(out, o, shortcuts[i], 3 * ch * cw);
          outputs.push_back(out);
        }
        rec("stage" + S + "_out" + std::to_string(i), outputs.back());
      }
    }
    encs_prev.assign(encs.rbegin(), encs.rend());
    decs_prev = decs;
    sam_prev = sam_new;
    outputs_all.push_back(outputs);
  }
  if (outputs_all.empty() || outputs_all.back().empty()) throw Error("the model produced no output");
  int32_t output = outputs_all.back().back();
  rec("final", output);
  return finish(input, output, mx_buf{3, h, wd});
}

// Live-range packing, largest first (src/model.rs:1091-1234). The candidate
// offsets are the ends of every block already placed, ascending; the first one
// whose block overlaps no block live during [first, last] wins.
std::unique_ptr<Plan> Builder::finish(int32_t input, int32_t output, mx_buf shape) {
  const size_t n = bufs_.size();
  std::vector<size_t> base(n), delta(n);
  for (size_t i = 0; i < n; ++i) {
    if (alias_parent_[i] < 0) {
      base[i] = i;
      delta[i] = 0;
    } else {
      size_t p = size_t(alias_parent_[i]);
      base[i] = base[p];
      delta[i] = delta[p] + size_t(alias_delta_[i]);
    }
  }
  const size_t NONE = std::numeric_limits<size_t>::max();
  const size_t DEAD = NONE - 1;
  std::vector<size_t> first(n, NONE), last(n, 0);
  std::vector<int32_t> touch;
  std::vector<size_t> seen;
  for (size_t oi = 0; oi < ops_.size(); ++oi) {
    touch.clear();
    op_operands(ops_[oi], touch);
    seen.clear();
    for (int32_t t : touch) {
      size_t b = base[size_t(t)];
      if (std::find(seen.begin(), seen.end(), b) != seen.end()) continue;
      seen.push_back(b);
      if (first[b] == NONE) first[b] = oi;
      last[b] = oi;
    }
  }
  for (size_t i = 0; i < n; ++i)
    if (first[i] == NONE) first[i] = DEAD, last[i] = 0;
  // A named buffer survives to the end of the run (what --dump needs).
  for (auto& kv : named_) {
    size_t b = base[size_t(kv.second)];
    if (first[b] != DEAD) last[b] = ops_.empty() ? 0 : ops_.size() - 1;
  }
  auto blen = [&](size_t i) { return size_t(bufs_[i].c * bufs_[i].h * bufs_[i].w); };
  std::vector<size_t> order;
  for (size_t i = 0; i < n; ++i)
    if (base[i] == i && first[i] != DEAD) order.push_back(i);
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
    if (blen(a) != blen(b)) return blen(a) > blen(b);
    return first[a] < first[b];
  });
  struct Block {
    size_t start, end, off, size;
  };
  std::vector<Block> placed;
  placed.reserve(order.size());
  std::vector<size_t> off(n, 0);
  size_t arena_len = 0;
  std::vector<size_t> cands;
  std::vector<const Block*> live;
  for (size_t i : order) {
    size_t size = blen(i), start = first[i], end = last[i];
    cands.clear();
    cands.push_back(0);
    live.clear();
    for (const Block& b : placed) {
      cands.push_back(b.off + b.size);
      if (start <= b.end && b.start <= end) live.push_back(&b);
    }
    std::sort(cands.begin(), cands.end());
    cands.erase(std::unique(cands.begin(), cands.end()), cands.end());
    size_t chosen = NONE;
    for (size_t c : cands) {
      bool clash = false;
      for (const Block* b : live)
        if (c < b->off + b->size && b->off < c + size) {
          clash = true;
          break;
        }
      if (!clash) {
        chosen = c;
        break;
      }
    }
    size_t c = chosen == NONE ? arena_len : chosen;
    off[i] = c;
    arena_len = std::max(arena_len, c + size);
    placed.push_back({start, end, c, size});
  }

  auto plan = std::make_unique<Plan>();
  plan->offs.resize(n);
  for (size_t i = 0; i < n; ++i) plan->offs[i] = int64_t(off[base[i]] + delta[i]);
  plan->bufs = std::move(bufs_);
  plan->ops = std::move(ops_);
  plan->weights = std::move(weights_);
  plan->arena_len = int64_t(arena_len);
  plan->input = input;
  plan->output = output;
  plan->dumps = std::move(named_);
  plan->shape = shape;
  plan->labels = std::move(labels_);
  plan->alias_parent = std::move(alias_parent_);
  plan->alias_delta = std::move(alias_delta_);
  return plan;
}

}  // namespace

int64_t Plan::weight_bytes() const {
  int64_t b = 0;
  for (auto& w : weights) b += int64_t(w.size()) * 4;
  return b;
}

mx_plan Plan::view() const {
  wptr_.resize(weights.size());
  wlen_.resize(weights.size());
  for (size_t i = 0; i < weights.size(); ++i) {
    wptr_[i] = weights[i].data();
    wlen_[i] = int64_t(weights[i].size());
  }
  mx_plan v{};
  v.n_bufs = int32_t(bufs.size());
  v.bufs = bufs.data();
  v.offs = offs.data();
  v.alias_parent = alias_parent.data();
  v.alias_delta = alias_delta.data();
  v.n_ops = int32_t(ops.size());
  v.ops = ops.data();
  v.n_weights = int32_t(weights.size());
  v.weights = wptr_.data();
  v.weight_lens = wlen_.data();
  v.arena_len = arena_len;
  v.input = input;
  v.output = output;
  v.shape = shape;
  return v;
}

std::unique_ptr<Plan> build_plan(const Weights& w, const Config& cfg, int64_t h, int64_t wd, bool dumps) {
  Builder b(w, cfg, dumps);
  return b.build(h, wd);
}

void op_operands(const mx_op& op, std::vector<int32_t>& out) {
  switch (op.kind) {
    case MX_OP_ADD:
    case MX_OP_MUL:
    case MX_OP_GATE_APPLY:
    case MX_OP_CHAN_SCALE:
      out.insert(out.end(), {op.dst, op.src, op.src2});
      break;
    case MX_OP_RESIZE:
      out.insert(out.end(), {op.dst, op.src, op.tmp});
      break;
    default:
      out.insert(out.end(), {op.dst, op.src});
  }
}

std::string describe(const mx_op& o) {
  switch (o.kind) {
    case MX_OP_CONV1X1: return fmt("conv1x1 %d->%d @%dx%d", o.c_in, o.c_out, o.h, o.wd);
    case MX_OP_CONV3X3: return fmt("conv3x3 %d->%d @%dx%d", o.c_in, o.c_out, o.h, o.wd);
    case MX_OP_CONV4X4S2: return fmt("convdown %d->%d @%dx%d", o.c_in, o.c_out, o.h, o.wd);
    case MX_OP_CONVT2X2: return fmt("convt %d->%d @%dx%d", o.c_in, o.c_out, o.h, o.wd);
    case MX_OP_GATE_MM: return fmt("gatemm c=%d %dx%d mode%d", o.c, o.outer, o.inner, o.mode);
    case MX_OP_BLOCK_PERM: return fmt("blockperm %dx%d %dx%d %s", o.gh, o.gw, o.fh, o.fw, o.forward ? "in" : "out");
    case MX_OP_RESIZE: return fmt("resize %dx%d->%dx%d", o.hin, o.win, o.hout, o.wout);
    case MX_OP_CHAN_LN: return fmt("chanln %dx%lld", o.c, (long long)o.hw);
    case MX_OP_CHAN_SCALE: return fmt("chanscale %dx%lld", o.c, (long long)o.hw);
    case MX_OP_CHAN_MEAN: return fmt("chanmean %dx%lld", o.c, (long long)o.hw);
    case MX_OP_DOWN_S: return fmt("down stride%d off%d", o.stride, o.off);
    case MX_OP_COPY: return fmt("copy %lld", (long long)o.n);
    case MX_OP_ADD: return fmt("add %lld", (long long)o.n);
    case MX_OP_MUL: return fmt("mul %lld", (long long)o.n);
    case MX_OP_GATE_APPLY: return fmt("gate %lld", (long long)o.n);
    case MX_OP_GELU: return fmt("gelu %lld", (long long)o.n);
    case MX_OP_LRELU: return fmt("lrelu %lld", (long long)o.n);
    case MX_OP_SIGMOID: return fmt("sigmoid %lld", (long long)o.n);
  }
  return "?";
}

}  // namespace mx
