// TEST INFRASTRUCTURE - the parity oracle and the timed CPU baseline. Nothing
// in the product path links, loads or calls this file; only tests/, the smoke
// check and bench.py's CPU arms do, and only as the checker.
//
// A C++ restatement of the reference's CPU executor, src/exec_cpu.rs, which
// cannot be built here (no Rust toolchain; its `lightgpu`, `rayon` and `png`
// dependencies are not vendored). Every arm keeps the reference's order of
// operations term for term, so that its results match the Rust executor's:
//   Conv1x1   bias, then c_in ascending            (exec_cpu.rs:628-690)
//   Conv3x3   bias, then (ky, kx, ic) ascending    (exec_cpu.rs:694-772)
//   Conv4x4s2 bias, then (ky, kx, ic) ascending    (exec_cpu.rs:773-847)
//   ConvT2x2  taps from zero over ic, bias LAST    (exec_cpu.rs:848-914)
//   GateMm    bias, then t ascending, both modes   (exec_cpu.rs:915-1077)
//   ChanLn    serial s1, s2 over c; var = s2/n - m^2; rstd = 1/sqrt(max(var,0)+eps);
//             y = (x - m) * rstd * w + b           (exec_cpu.rs:359-455)
//   ChanMean  serial sum / hw                      (exec_cpu.rs:1118-1142)
//   Resize    tabulated jax taps, H then V pass, acc/wsum if wsum > 0
//                                                  (exec_cpu.rs:1143-1322)
//   BlockPerm / DownS / elementwise                (exec_cpu.rs:550-627, 1078-1117)
// GELU uses libm erff and sigmoid expf: the reference's `lightgpu::ops::cpu`
// twins live in an un-vendored git dependency with no pinned revision, so the
// last ulp of those two functions is not pinned (see the header of the test
// that compares this oracle with the reference's PyTorch transcription).
//
// Threads split the same axes the reference's rayon pool does (output
// channels, pixel blocks, rows); each output element's summation order is
// independent of the split, so the result does not depend on the thread count.
//
// Built with -ffp-contract=off: a fused multiply-add would change the rounding
// of every accumulation relative to the reference.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "maxim_b200.h"

namespace {

constexpr float kEps = 1e-6f;  // src/model.rs:35
constexpr int64_t PB = 256;    // pixels per conv1x1 task tile (exec_cpu.rs:37)

// A fixed pool of workers; run(n, f) calls f(0..n-1) across them and waits.
// Each run is its own Job with its own counters, so a worker still leaving
// the previous run can never claim (or count) a task of the next one.
class Pool {
 public:
  explicit Pool(int threads) : n_(std::max(1, threads)) {
    for (int i = 1; i < n_; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> l(m_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  void run(int64_t tasks, const std::function<void(int64_t)>& f) {
    if (tasks <= 0) return;
    if (n_ == 1 || tasks == 1) {
      for (int64_t i = 0; i < tasks; ++i) f(i);
      return;
    }
    auto job = std::make_shared<Job>();
    job->f = &f;
    job->total = tasks;
    {
      std::lock_guard<std::mutex> l(m_);
      job_ = job;
      ++gen_;
    }
    cv_.notify_all();
    work(*job);
    std::unique_lock<std::mutex> l(m_);
    done_cv_.wait(l, [&] { return job->done.load() == job->total; });
    job_.reset();
  }

 private:
  struct Job {
    const std::function<void(int64_t)>* f = nullptr;
    int64_t total = 0;
    std::atomic<int64_t> next{0}, done{0};
  };
  void work(Job& j) {
    for (;;) {
      int64_t i = j.next.fetch_add(1);
      if (i >= j.total) break;
      (*j.f)(i);
      if (j.done.fetch_add(1) + 1 == j.total) {
        std::lock_guard<std::mutex> l(m_);
        done_cv_.notify_all();
      }
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::shared_ptr<Job> j;
      {
        std::unique_lock<std::mutex> l(m_);
        cv_.wait(l, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
        j = job_;
      }
      if (j) work(*j);
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  std::shared_ptr<Job> job_;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

// The tabulated taps of one resize axis (`ResizeTaps`, exec_cpu.rs:1224-1282).
struct Taps {
  std::vector<int64_t> j0, w0;  // per output: first input index, first weight index
  std::vector<float> w, wsum;
  int64_t n_out;
  Taps(int64_t n_in, int64_t n_out_) : n_out(n_out_) {
    float inv = float(n_in) / float(n_out);
    float kscale = inv > 1.0f ? inv : 1.0f;
    for (int64_t o = 0; o < n_out; ++o) {
      float sample = (float(o) + 0.5f) * inv - 0.5f;
      int64_t a = int64_t(std::ceil(sample - kscale));
      int64_t b = int64_t(std::floor(sample + kscale));
      if (a < 0) a = 0;
      if (b > n_in - 1) b = n_in - 1;
      int64_t first = int64_t(w.size());
      float s = 0.0f;
      for (int64_t j = a; j <= b; ++j) {
        float d = std::fabs(sample - float(j)) / kscale;
        if (d < 1.0f) {
          float wv = 1.0f - d;
          w.push_back(wv);
          s += wv;
        }
      }
      j0.push_back(a);
      w0.push_back(first);
      wsum.push_back(s);
    }
  }
  int64_t count(int64_t o) const { return (o + 1 < n_out ? w0[o + 1] : int64_t(w.size())) - w0[o]; }
};

struct Ctx {
  const mx_plan& plan;
  float* arena;
  Pool& pool;

  float* p(int32_t id) const { return arena + plan.offs[id]; }
  const float* W(int32_t id) const { return plan.weights[id]; }
  int64_t blen(int32_t id) const { return plan.bufs[id].c * plan.bufs[id].h * plan.bufs[id].w; }

  // Flat elementwise split into tasks of at least 16384 elements
  // (PAR_MIN, exec_cpu.rs:106).
  template <class F>
  void flat(int64_t n, F f) {
    int64_t parts = std::max<int64_t>(1, std::min<int64_t>(n / 16384, pool.size() * 4));
    int64_t per = (n + parts - 1) / parts;
    pool.run(parts, [&](int64_t t) {
      int64_t a = t * per, b = std::min(n, a + per);
      for (int64_t i = a; i < b; ++i) f(i);
    });
  }

  void op(const mx_op& o);
};

void Ctx::op(const mx_op& o) {
  switch (o.kind) {
    case MX_OP_COPY: {
      float* d = p(o.dst);
      const float* s = p(o.src);
      flat(o.n, [&](int64_t i) { d[i] = s[i]; });
      break;
    }
    case MX_OP_ADD: {
      float* d = p(o.dst);
      const float *a = p(o.src), *b = p(o.src2);
      flat(o.n, [&](int64_t i) { d[i] = a[i] + b[i]; });
      break;
    }
    case MX_OP_MUL: {
      float* d = p(o.dst);
      const float *a = p(o.src), *b = p(o.src2);
      flat(o.n, [&](int64_t i) { d[i] = a[i] * b[i]; });
      break;
    }
    case MX_OP_GATE_APPLY: {  // u * (v + 1)
      float* d = p(o.dst);
      const float *u = p(o.src), *v = p(o.src2);
      flat(o.n, [&](int64_t i) { d[i] = u[i] * (v[i] + 1.0f); });
      break;
    }
    case MX_OP_GELU: {
      float* d = p(o.dst);
      const float* s = p(o.src);
      const float r2 = 0.70710677f;  // FRAC_1_SQRT_2 as f32
      flat(o.n, [&](int64_t i) {
        float x = s[i];
        d[i] = 0.5f * x * (1.0f + erff(x * r2));
      });
      break;
    }
    case MX_OP_LRELU: {
      float* d = p(o.dst);
      const float* s = p(o.src);
      float sl = o.slope;
      flat(o.n, [&](int64_t i) { d[i] = s[i] >= 0.0f ? s[i] : sl * s[i]; });
      break;
    }
    case MX_OP_SIGMOID: {
      float* d = p(o.dst);
      const float* s = p(o.src);
      flat(o.n, [&](int64_t i) { d[i] = 1.0f / (1.0f + expf(-s[i])); });
      break;
    }
    case MX_OP_CHAN_SCALE: {
      float* d = p(o.dst);
      const float *s = p(o.src), *sc = p(o.src2);
      int64_t hw = o.hw;
      pool.run(o.c, [&](int64_t ch) {
        for (int64_t i = 0; i < hw; ++i) d[ch * hw + i] = s[ch * hw + i] * sc[ch];
      });
      break;
    }
    case MX_OP_CHAN_MEAN: {
      float* d = p(o.dst);
      const float* s = p(o.src);
      for (int64_t ch = 0; ch < o.c; ++ch) {
        float acc = 0.0f;
        for (int64_t i = 0; i < o.hw; ++i) acc += s[ch * o.hw + i];
        d[ch] = acc / float(o.hw);
      }
      break;
    }
    case MX_OP_CHAN_LN: {
      const int64_t c = o.c, hw = o.hw;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float *sc = W(o.scale), *bi = W(o.bias);
      std::vector<float> table(static_cast<size_t>(2 * hw));
      const float nf = float(c);
      int64_t parts = std::max<int64_t>(1, std::min<int64_t>(hw / 4096, pool.size() * 4));
      int64_t per = (hw + parts - 1) / parts;
      pool.run(parts, [&](int64_t t) {
        for (int64_t px = t * per; px < std::min(hw, (t + 1) * per); ++px) {
          float s1 = 0.0f, s2 = 0.0f;
          for (int64_t ic = 0; ic < c; ++ic) {
            float v = s[ic * hw + px];
            s1 += v;
            s2 += v * v;
          }
          float m = s1 / nf;
          float var = s2 / nf - m * m;
          table[2 * px] = m;
          table[2 * px + 1] = 1.0f / std::sqrt(std::fmax(var, 0.0f) + kEps);
        }
      });
      pool.run(c, [&](int64_t ch) {
        float w = sc[ch], b = bi[ch];
        const float* sp = s + ch * hw;
        float* dp = d + ch * hw;
        for (int64_t px = 0; px < hw; ++px) dp[px] = (sp[px] - table[2 * px]) * table[2 * px + 1] * w + b;
      });
      break;
    }
    case MX_OP_CONV1X1: {
      const int64_t ci = o.c_in, co = o.c_out, plane = int64_t(o.h) * o.wd;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float* wt = W(o.w);
      const float* bs = o.bias >= 0 ? W(o.bias) : nullptr;
      int64_t blocks = (plane + PB - 1) / PB;
      pool.run(blocks, [&](int64_t k) {
        int64_t p0 = k * PB, np = std::min(PB, plane - p0);
        std::vector<float> tile(static_cast<size_t>(PB * ci)), acc(static_cast<size_t>(PB));
        for (int64_t ic = 0; ic < ci; ++ic) memcpy(&tile[size_t(ic * PB)], s + ic * plane + p0, size_t(np) * 4);
        for (int64_t oc = 0; oc < co; ++oc) {
          const float* wp = wt + oc * ci;
          float bv = bs ? bs[oc] : 0.0f;
          for (int64_t i = 0; i < np; ++i) acc[i] = bv;
          for (int64_t ic = 0; ic < ci; ++ic) {
            float wv = wp[ic];
            const float* ti = &tile[size_t(ic * PB)];
            for (int64_t i = 0; i < np; ++i) acc[i] += wv * ti[i];
          }
          memcpy(d + oc * plane + p0, acc.data(), size_t(np) * 4);
        }
      });
      break;
    }
    case MX_OP_CONV3X3: {
      const int64_t ci = o.c_in, co = o.c_out, h = o.h, wd = o.wd, plane = h * wd;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float* wt = W(o.w);
      const float* bs = o.bias >= 0 ? W(o.bias) : nullptr;
      // one task per (output channel, row block)
      int64_t rb = std::max<int64_t>(1, std::min<int64_t>(h, (pool.size() * 8 + co - 1) / co));
      int64_t rows = (h + rb - 1) / rb;
      pool.run(co * rb, [&](int64_t t) {
        int64_t oc = t / rb, y0 = (t % rb) * rows, y1 = std::min(h, y0 + rows);
        std::vector<float> row(static_cast<size_t>(wd + 2));
        float bv = bs ? bs[oc] : 0.0f;
        const float* wp = wt + oc * ci * 9;
        for (int64_t y = y0; y < y1; ++y) {
          std::fill(row.begin(), row.end(), bv);
          for (int64_t ky = 0; ky < 3; ++ky) {
            int64_t iy = y + ky - 1;
            if (iy < 0 || iy >= h) continue;
            for (int64_t kx = 0; kx < 3; ++kx) {
              int64_t shift = 2 - kx;
              for (int64_t ic = 0; ic < ci; ++ic) {
                float wv = wp[ic * 9 + ky * 3 + kx];
                const float* sr = s + ic * plane + iy * wd;
                float* r = row.data() + shift;
                for (int64_t i = 0; i < wd; ++i) r[i] += wv * sr[i];
              }
            }
          }
          memcpy(d + oc * plane + y * wd, row.data() + 1, size_t(wd) * 4);
        }
      });
      break;
    }
    case MX_OP_CONV4X4S2: {
      const int64_t ci = o.c_in, co = o.c_out, h = o.h, wd = o.wd, plane = h * wd;
      const int64_t oh = o.oh, ow = o.ow, pt = o.pad_top, pl = o.pad_left;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float* wt = W(o.w);
      const float* bs = o.bias >= 0 ? W(o.bias) : nullptr;
      pool.run(co, [&](int64_t oc) {
        float bv = bs ? bs[oc] : 0.0f;
        const float* wp = wt + oc * ci * 16;
        std::vector<float> acc(static_cast<size_t>(ow));
        for (int64_t oy = 0; oy < oh; ++oy) {
          std::fill(acc.begin(), acc.end(), bv);
          for (int64_t ky = 0; ky < 4; ++ky) {
            int64_t iy = oy * 2 + ky;
            if (iy < pt || iy - pt >= h) continue;
            iy -= pt;
            for (int64_t kx = 0; kx < 4; ++kx) {
              // floor((pl - kx + 1) / 2) clamped at 0; the upper bound keeps
              // the input column 2*ox + kx - pl at most wd - 1.
              int64_t num = pl - kx + 1;
              int64_t lo = std::max<int64_t>(0, num >= 0 ? num / 2 : -((-num + 1) / 2));
              int64_t hn = wd - 1 + pl - kx;
              int64_t hi = (hn >= 0 ? hn / 2 : -((-hn + 1) / 2)) + 1;
              hi = std::min<int64_t>(std::max<int64_t>(hi, 0), ow);
              for (int64_t ic = 0; ic < ci; ++ic) {
                float wv = wp[ic * 16 + ky * 4 + kx];
                const float* sr = s + ic * plane + iy * wd;
                for (int64_t ox = lo; ox < hi; ++ox) acc[ox] += wv * sr[ox * 2 + kx - pl];
              }
            }
          }
          memcpy(d + oc * oh * ow + oy * ow, acc.data(), size_t(ow) * 4);
        }
      });
      break;
    }
    case MX_OP_CONVT2X2: {
      const int64_t ci = o.c_in, co = o.c_out, h = o.h, wd = o.wd, plane = h * wd;
      const int64_t ow = wd * 2, oplane = h * 2 * ow;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float* wt = W(o.w);
      const float* bs = o.bias >= 0 ? W(o.bias) : nullptr;
      pool.run(co, [&](int64_t oc) {
        float bv = bs ? bs[oc] : 0.0f;
        std::vector<float> a0(static_cast<size_t>(wd)), a1(static_cast<size_t>(wd)), a2(static_cast<size_t>(wd)), a3(static_cast<size_t>(wd));
        for (int64_t y = 0; y < h; ++y) {
          std::fill(a0.begin(), a0.end(), 0.0f);
          std::fill(a1.begin(), a1.end(), 0.0f);
          std::fill(a2.begin(), a2.end(), 0.0f);
          std::fill(a3.begin(), a3.end(), 0.0f);
          for (int64_t ic = 0; ic < ci; ++ic) {
            const float* sr = s + ic * plane + y * wd;
            const float* wb = wt + (ic * co + oc) * 4;
            for (int64_t x = 0; x < wd; ++x) {
              float v = sr[x];
              a0[x] += wb[0] * v;
              a1[x] += wb[1] * v;
              a2[x] += wb[2] * v;
              a3[x] += wb[3] * v;
            }
          }
          float* r0 = d + oc * oplane + 2 * y * ow;
          float* r1 = r0 + ow;
          for (int64_t x = 0; x < wd; ++x) {
            r0[2 * x] = bv + a0[x];
            r0[2 * x + 1] = bv + a1[x];
            r1[2 * x] = bv + a2[x];
            r1[2 * x + 1] = bv + a3[x];
          }
        }
      });
      break;
    }
    case MX_OP_GATE_MM: {
      const int64_t c = o.c, outer = o.outer, inner = o.inner, pl = outer * inner;
      const float* s = p(o.src);
      float* d = p(o.dst);
      const float* wt = W(o.w);
      const float* bs = o.bias >= 0 ? W(o.bias) : nullptr;
      if (o.mode == 0) {
        // out[r][b] = bias[r] + sum_t w[r][t] x[t][b]; split by (gate, row block)
        int64_t rb = std::max<int64_t>(1, std::min<int64_t>(outer, (pool.size() * 8 + c - 1) / c));
        int64_t rows = (outer + rb - 1) / rb;
        pool.run(c * rb, [&](int64_t t) {
          int64_t ch = t / rb, r0 = (t % rb) * rows, r1 = std::min(outer, r0 + rows);
          const float* x = s + ch * pl;
          float* y = d + ch * pl;
          std::vector<float> row(static_cast<size_t>(inner));
          for (int64_t r = r0; r < r1; ++r) {
            const float* wa = wt + r * outer;
            float bv = bs ? bs[r] : 0.0f;
            std::fill(row.begin(), row.end(), bv);
            for (int64_t t_ = 0; t_ < outer; ++t_) {
              float wv = wa[t_];
              const float* xr = x + t_ * inner;
              for (int64_t b = 0; b < inner; ++b) row[b] += wv * xr[b];
            }
            memcpy(y + r * inner, row.data(), size_t(inner) * 4);
          }
        });
      } else {
        // out[i][a] = bias[a] + sum_t w[a][t] x[i][t]; split by (gate, row block)
        int64_t rb = std::max<int64_t>(1, std::min<int64_t>(outer, (pool.size() * 8 + c - 1) / c));
        int64_t rows = (outer + rb - 1) / rb;
        pool.run(c * rb, [&](int64_t t) {
          int64_t ch = t / rb, r0 = (t % rb) * rows, r1 = std::min(outer, r0 + rows);
          const float* x = s + ch * pl;
          float* y = d + ch * pl;
          for (int64_t i = r0; i < r1; ++i) {
            const float* xb = x + i * inner;
            for (int64_t a = 0; a < inner; ++a) {
              const float* wa = wt + a * inner;
              float acc = bs ? bs[a] : 0.0f;
              for (int64_t t_ = 0; t_ < inner; ++t_) acc += wa[t_] * xb[t_];
              y[i * inner + a] = acc;
            }
          }
        });
      }
      break;
    }
    case MX_OP_BLOCK_PERM: {
      const int64_t c = o.c, h = o.h, wd = o.wd, gh = o.gh, gw = o.gw, fh = o.fh, fw = o.fw;
      const int64_t gsz = gh * gw, psz = fh * fw, plane = h * wd;
      const float* s = p(o.src);
      float* d = p(o.dst);
      pool.run(c, [&](int64_t ch) {
        const float* pl = s + ch * plane;
        float* dl = d + ch * plane;
        for (int64_t gy = 0; gy < gh; ++gy)
          for (int64_t gx = 0; gx < gw; ++gx)
            for (int64_t fy = 0; fy < fh; ++fy)
              for (int64_t fx = 0; fx < fw; ++fx) {
                int64_t g = gy * gw + gx, q = fy * fw + fx;
                int64_t pix = (gy * fh + fy) * wd + gx * fw + fx;
                int64_t blk = o.swap ? q * gsz + g : g * psz + q;
                if (o.forward) dl[blk] = pl[pix];
                else dl[pix] = pl[blk];
              }
      });
      break;
    }
    case MX_OP_DOWN_S: {
      const int64_t ip = int64_t(o.h) * o.wd, op_ = int64_t(o.oh) * o.ow;
      const float* s = p(o.src);
      float* d = p(o.dst);
      pool.run(o.c, [&](int64_t ch) {
        for (int64_t y = 0; y < o.oh; ++y)
          for (int64_t x = 0; x < o.ow; ++x)
            d[ch * op_ + y * o.ow + x] = s[ch * ip + (y * o.stride + o.off) * o.wd + x * o.stride + o.off];
      });
      break;
    }
    case MX_OP_RESIZE: {
      const int64_t c = o.c, hin = o.hin, win = o.win, hout = o.hout, wout = o.wout;
      const float* s = p(o.src);
      float* t = p(o.tmp);
      float* d = p(o.dst);
      Taps tx(win, wout), ty(hin, hout);
      // horizontal pass: one row of tmp per (channel, input row)
      pool.run(c * hin, [&](int64_t r) {
        const float* sr = s + r * win;
        float* tr = t + r * wout;
        for (int64_t x = 0; x < wout; ++x) {
          int64_t j0 = tx.j0[x], w0 = tx.w0[x], n = tx.count(x);
          float acc = 0.0f;
          for (int64_t k = 0; k < n; ++k) acc += tx.w[w0 + k] * sr[j0 + k];
          float sm = tx.wsum[x];
          tr[x] = sm > 0.0f ? acc / sm : acc;
        }
      });
      // vertical pass: one output row per (channel, output row)
      pool.run(c * hout, [&](int64_t r) {
        int64_t ch = r / hout, oy = r % hout;
        const float* pl = t + ch * hin * wout;
        float* dr = d + r * wout;
        int64_t j0 = ty.j0[oy], w0 = ty.w0[oy], n = std::min<int64_t>(ty.count(oy), 64);
        float sm = ty.wsum[oy];
        for (int64_t x = 0; x < wout; ++x) {
          float acc = 0.0f;
          for (int64_t k = 0; k < n; ++k) acc += ty.w[w0 + k] * pl[(j0 + k) * wout + x];
          dr[x] = sm > 0.0f ? acc / sm : acc;
        }
      });
      break;
    }
    default:
      break;
  }
}

thread_local std::string g_err;

}  // namespace

extern "C" {

// Run the whole plan. `arena` holds plan->arena_len floats with the input
// image already at offs[input]. `threads` <= 0 means all hardware threads.
__attribute__((visibility("default"))) int mxo_run(const mx_plan* plan, float* arena, int threads) {
  if (!plan || !arena) return MX_E_INVALID;
  Pool pool(threads > 0 ? threads : int(std::thread::hardware_concurrency()));
  Ctx ctx{*plan, arena, pool};
  for (int32_t i = 0; i < plan->n_ops; ++i) ctx.op(plan->ops[i]);
  return MX_OK;
}

// Run ops [first, last) - the op-by-op walk `--verify-gpu` uses (`step`).
__attribute__((visibility("default"))) int mxo_run_range(const mx_plan* plan, float* arena, int32_t first,
                                                        int32_t last, int threads) {
  if (!plan || !arena || first < 0 || last > plan->n_ops || first > last) return MX_E_INVALID;
  Pool pool(threads > 0 ? threads : int(std::thread::hardware_concurrency()));
  Ctx ctx{*plan, arena, pool};
  for (int32_t i = first; i < last; ++i) ctx.op(plan->ops[i]);
  return MX_OK;
}

// The whole plan with every op's output rounded to bfloat16 (nearest, ties
// to even) as it is written: what storing activations in bf16 would do to
// the result, measured against mxo_run. Not the reference's arithmetic - a
// what-if for the storage precision of the activations.
__attribute__((visibility("default"))) int mxo_run_bf16_storage(const mx_plan* plan, float* arena, int threads) {
  if (!plan || !arena) return MX_E_INVALID;
  Pool pool(threads > 0 ? threads : int(std::thread::hardware_concurrency()));
  Ctx ctx{*plan, arena, pool};
  for (int32_t i = 0; i < plan->n_ops; ++i) {
    ctx.op(plan->ops[i]);
    float* d = ctx.p(plan->ops[i].dst);
    const int64_t n = ctx.blen(plan->ops[i].dst);  // a channel view is contiguous in [c][h][w]
    pool.run((n + 65535) / 65536, [&](int64_t t) {
      const int64_t e = std::min(n, (t + 1) * 65536);
      for (int64_t k = t * 65536; k < e; ++k) {
        uint32_t b;
        memcpy(&b, &d[k], 4);
        if ((b & 0x7f800000u) != 0x7f800000u) b = (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
        memcpy(&d[k], &b, 4);
      }
    });
  }
  return MX_OK;
}

}  // extern "C"
