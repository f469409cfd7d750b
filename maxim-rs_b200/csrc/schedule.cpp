// The executor's schedule: fusion, block-permutation removal and arena packing
// over a plan's op list. The plan's semantics are src/model.rs:66-112 (ops) and
// src/model.rs:1237-1272 (buffers, views, offsets); the reference packs the
// arena for its own op list (src/model.rs, Builder::finish), which is the
// layout the executor keeps for op-by-op stepping. This file packs afresh for
// the rewritten list with the same rule: first fit over live ranges.
#include "schedule.h"

#include <algorithm>
#include <climits>
#include <cstdint>

#include "common.h"

namespace mx {
namespace {

constexpr int32_t kNative = -1;  // data stored in the order the plan says

// Buffer geometry: every buffer is a channel range [lo, hi) of a root.
struct Geo {
  std::vector<int32_t> root;
  std::vector<int64_t> lo, hi;

  explicit Geo(const mx_plan& p) : root(size_t(p.n_bufs)), lo(size_t(p.n_bufs)), hi(size_t(p.n_bufs)) {
    for (int32_t b = 0; b < p.n_bufs; ++b) {
      int32_t r = b, guard_steps = 0;
      while (p.alias_parent[r] >= 0) {
        r = p.alias_parent[r];
        if (++guard_steps > p.n_bufs) throw Error("plan: the buffer views form a cycle");
      }
      root[size_t(b)] = r;
      const mx_buf& rb = p.bufs[r];
      const mx_buf& bb = p.bufs[b];
      const int64_t hw = rb.h * rb.w, delta = p.offs[b] - p.offs[r];
      if (bb.h * bb.w != hw || (hw > 0 && delta % hw != 0) || delta < 0)
        throw Error(fmt("plan: buffer %d is a view of %d that is not a channel range", b, r));
      lo[size_t(b)] = hw > 0 ? delta / hw : 0;
      hi[size_t(b)] = lo[size_t(b)] + bb.c;
      if (hi[size_t(b)] > rb.c) throw Error(fmt("plan: view %d runs past the channels of %d", b, r));
    }
  }
  bool overlap(int32_t a, int32_t b) const {
    if (a < 0 || b < 0) return false;
    return root[size_t(a)] == root[size_t(b)] && lo[size_t(a)] < hi[size_t(b)] && lo[size_t(b)] < hi[size_t(a)];
  }
  bool covers(int32_t a, int32_t t) const {
    return root[size_t(a)] == root[size_t(t)] && lo[size_t(a)] <= lo[size_t(t)] && hi[size_t(t)] <= hi[size_t(a)];
  }
  bool whole(int32_t a) const { return lo[size_t(a)] == 0 && hi[size_t(a)] == hi[size_t(root[size_t(a)])]; }
  // A buffer the schedule adds: a root of c channels. Returns its id.
  int32_t add(int64_t c) {
    const int32_t id = int32_t(root.size());
    root.push_back(id);
    lo.push_back(0);
    hi.push_back(c);
    return id;
  }
};

bool per_pixel_unary(int k) {
  return k == MX_OP_COPY || k == MX_OP_GELU || k == MX_OP_LRELU || k == MX_OP_SIGMOID || k == MX_OP_CHAN_LN ||
         k == MX_OP_CONV1X1;
}
bool per_pixel_binary(int k) { return k == MX_OP_ADD || k == MX_OP_MUL || k == MX_OP_GATE_APPLY; }
bool elementwise(int k) { return k <= MX_OP_SIGMOID; }

int writes_of(const mx_op& o, int32_t* w) {
  int n = 0;
  w[n++] = o.dst;
  if (o.kind == MX_OP_RESIZE && o.tmp >= 0) w[n++] = o.tmp;
  return n;
}
int reads_of(const mx_op& o, int32_t extra, int32_t* r) {
  int n = 0;
  if (o.src >= 0) r[n++] = o.src;
  if (o.src2 >= 0) r[n++] = o.src2;
  if (extra >= 0) r[n++] = extra;
  return n;
}
// Everything a scheduled step reads: its op's inputs, the epilogue
// operands and the LayerNorm statistics it normalises with. r holds 5.
int step_reads(const SchedStep& st, int32_t* r) {
  int n = reads_of(st.o, st.epi_src, r);
  if (st.epi_src2 >= 0) r[n++] = st.epi_src2;
  if (st.ln_stats >= 0) r[n++] = st.ln_stats;
  return n;
}
// Everything a scheduled step writes, the statistics and the LayerNorm of
// its epilogue included. w holds 5.
int step_writes(const SchedStep& st, int32_t* w) {
  int n = writes_of(st.o, w);
  for (int g = 0; g < 2; ++g)
    if (st.stats_out[g] >= 0) w[n++] = st.stats_out[g];
  if (st.ln_out >= 0) w[n++] = st.ln_out;
  return n;
}

// The outcome of dropping a set of forward block permutations.
struct PermSim {
  std::vector<int32_t> src, src2;  // per op: inputs with dropped permutations' outputs resolved
  std::vector<int32_t> gate_perm;  // per op
  std::vector<char> to_copy;       // per op: a backward permutation that became a Copy
};

// Walk the plan with the forward permutations in `drop` removed: the removed
// permutation's output is read from its (spatial) input instead, and every
// buffer carries the pixel order it is really stored in. Succeeds when every
// op sees inputs in an order it can handle: per-pixel ops any order (all
// inputs alike), gating matmuls a blocked order they can read through a
// tensor map, backward permutations the order they undo (they become
// Copies), everything else the plan's own order.
bool simulate(const mx_plan& p, const Geo& G, const ScheduleHooks& H, const std::vector<char>& drop, PermSim& out) {
  const int n = p.n_ops;
  std::vector<int32_t> subst(size_t(p.n_bufs), -1), sub_ord(size_t(p.n_bufs), kNative);
  std::vector<int32_t> rord(size_t(p.n_bufs), kNative);
  std::vector<char> written(size_t(p.n_bufs), 0);
  out.src.assign(size_t(n), -1);
  out.src2.assign(size_t(n), -1);
  out.gate_perm.assign(size_t(n), -1);
  out.to_copy.assign(size_t(n), 0);
  struct Active {
    int32_t y, x;
    int last;
  };
  std::vector<Active> active;
  for (int k = 0; k < n; ++k) {
    const mx_op& o = p.ops[k];
    for (size_t a = 0; a < active.size();) {
      if (active[a].last < k) {
        subst[size_t(active[a].y)] = -1;
        active.erase(active.begin() + long(a));
      } else {
        ++a;
      }
    }
    const int32_t in[2] = {o.src, o.src2};
    for (int32_t b : in)
      for (const Active& a : active)
        if (b >= 0 && G.overlap(b, a.y) && b != a.y) return false;  // a partial read of a dropped output
    auto ord = [&](int32_t b) { return subst[size_t(b)] >= 0 ? sub_ord[size_t(b)] : rord[size_t(G.root[size_t(b)])]; };
    auto res = [&](int32_t b) { return b >= 0 && subst[size_t(b)] >= 0 ? subst[size_t(b)] : b; };
    out.src[size_t(k)] = res(o.src);
    out.src2[size_t(k)] = res(o.src2);

    if (o.kind == MX_OP_BLOCK_PERM && o.forward && drop[size_t(k)]) {
      const int32_t x = o.src, y = o.dst;
      if (o.swap != 0 || subst[size_t(x)] >= 0 || ord(x) != kNative) return false;
      if (G.root[size_t(y)] != y || G.overlap(y, p.output) || G.overlap(y, p.input)) return false;
      int last = -1;
      for (int m = k + 1; m < n; ++m) {
        const mx_op& q = p.ops[m];
        int32_t r[3], w[2];
        const int nr = reads_of(q, -1, r), nw = writes_of(q, w);
        for (int i = 0; i < nr; ++i)
          if (G.overlap(r[i], y)) last = m;
        bool rewritten = false;
        for (int i = 0; i < nw; ++i) rewritten |= G.overlap(w[i], y);
        if (rewritten) break;
      }
      subst[size_t(y)] = x;
      sub_ord[size_t(y)] = k;
      active.push_back({y, x, last});
      continue;
    }

    int32_t out_ord = kNative;
    if (per_pixel_unary(o.kind)) {
      out_ord = ord(o.src);
    } else if (per_pixel_binary(o.kind)) {
      out_ord = ord(o.src);
      if (ord(o.src2) != out_ord) return false;
    } else if (o.kind == MX_OP_CHAN_SCALE) {
      out_ord = ord(o.src);
      if (ord(o.src2) != kNative) return false;  // the per-channel scale vector
    } else if (o.kind == MX_OP_GATE_MM) {
      out_ord = ord(o.src);
      if (out_ord != kNative) {
        const mx_op& P = p.ops[out_ord];
        if (o.c != P.c || int64_t(o.outer) != int64_t(P.gh) * P.gw || int64_t(o.inner) != int64_t(P.fh) * P.fw ||
            !H.gate_spatial(o, P))
          return false;
        out.gate_perm[size_t(k)] = out_ord;
      }
    } else if (o.kind == MX_OP_BLOCK_PERM && !o.forward) {
      const int32_t q = ord(o.src);
      if (q != kNative) {
        const mx_op& P = p.ops[q];
        if (P.gh != o.gh || P.gw != o.gw || P.fh != o.fh || P.fw != o.fw || P.swap != o.swap || P.h != o.h ||
            P.wd != o.wd || P.c != o.c)
          return false;
        out.to_copy[size_t(k)] = 1;
      }
    } else {
      for (int32_t b : in)
        if (b >= 0 && ord(b) != kNative) return false;
    }

    int32_t w[2];
    const int nw = writes_of(o, w);
    for (int i = 0; i < nw; ++i) {
      for (const Active& a : active)
        if (G.overlap(w[i], a.x) || G.overlap(w[i], a.y)) return false;
      const int32_t r = G.root[size_t(w[i])];
      const int32_t wo = i == 0 ? out_ord : kNative;
      if (G.whole(w[i]) || !written[size_t(r)]) rord[size_t(r)] = wo;
      else if (rord[size_t(r)] != wo) return false;
      written[size_t(r)] = 1;
    }
  }
  return rord[size_t(G.root[size_t(p.output)])] == kNative;
}

// The channel count of a tensor-core step's output tile rows.
int out_channels(const mx_op& o) { return o.kind == MX_OP_GATE_MM ? o.c : o.c_out; }

}  // namespace

Schedule build_schedule(const mx_plan& p, const ScheduleHooks& H, bool fuse) {
  Geo G(p);
  const int n = p.n_ops;
  Schedule S;

  // 1. Block permutations.
  std::vector<char> drop(size_t(n), 0);
  PermSim sim;
  if (fuse) {
    std::vector<int> cand;
    for (int k = 0; k < n; ++k)
      if (p.ops[k].kind == MX_OP_BLOCK_PERM && p.ops[k].forward && p.ops[k].swap == 0) cand.push_back(k);
    for (int k : cand) drop[size_t(k)] = 1;
    if (!simulate(p, G, H, drop, sim)) {
      for (int k : cand) drop[size_t(k)] = 0;
      for (int k : cand) {
        drop[size_t(k)] = 1;
        if (!simulate(p, G, H, drop, sim)) drop[size_t(k)] = 0;
      }
    }
  }
  if (!simulate(p, G, H, drop, sim)) throw Error("schedule: the plan's own op order failed the pixel-order check");

  std::vector<SchedStep> W;
  W.reserve(size_t(n));
  for (int k = 0; k < n; ++k) {
    if (drop[size_t(k)]) {
      ++S.perms_dropped;
      continue;
    }
    SchedStep s;
    s.o = p.ops[k];
    s.o.src = sim.src[size_t(k)];
    s.o.src2 = sim.src2[size_t(k)];
    if (sim.to_copy[size_t(k)]) {
      s.o.kind = MX_OP_COPY;
      s.o.n = int64_t(s.o.c) * s.o.h * s.o.wd;
    }
    s.op = k;
    s.covers.push_back(k);
    s.gate_perm = sim.gate_perm[size_t(k)];
    W.push_back(std::move(s));
  }

  // 2. Fold single consumers into their producers.
  std::vector<char> dead(W.size(), 0);
  for (size_t i = 0; fuse && i < W.size(); ++i) {
    if (dead[i]) continue;
    for (;;) {
      SchedStep& A = W[i];
      const int32_t T = A.o.dst;
      if (G.overlap(T, p.output) || A.o.kind == MX_OP_CHAN_MEAN) break;
      size_t j = SIZE_MAX;
      bool ok = true;
      for (size_t s = i + 1; s < W.size() && ok; ++s) {
        if (dead[s]) continue;
        int32_t r[5], w[2];
        const int nr = step_reads(W[s], r), nw = writes_of(W[s].o, w);
        for (int a = 0; a < nr; ++a)
          if (G.overlap(r[a], T)) {
            if (j != SIZE_MAX || r[a] != T) ok = false;
            else j = s;
          }
        bool gone = false;
        for (int a = 0; a < nw; ++a)
          if (G.overlap(w[a], T)) {
            if (G.covers(w[a], T)) gone = true;
            else ok = false;
          }
        if (gone) break;
      }
      if (!ok || j == SIZE_MAX) break;
      const SchedStep& B = W[j];
      int epi = -1;
      int32_t operand = -1;
      switch (B.o.kind) {
        case MX_OP_COPY:
          if (B.o.src == T) epi = EPI_NONE;
          break;
        case MX_OP_GELU:
          if (B.o.src == T && B.o.src2 < 0) epi = EPI_GELU;
          break;
        case MX_OP_LRELU:
          if (B.o.src == T && B.o.src2 < 0) epi = EPI_LRELU;
          break;
        case MX_OP_SIGMOID:
          if (B.o.src == T && B.o.src2 < 0) epi = EPI_SIGMOID;
          break;
        case MX_OP_ADD:
        case MX_OP_MUL:
          if ((B.o.src == T) != (B.o.src2 == T)) {
            epi = B.o.kind == MX_OP_ADD ? EPI_ADD : EPI_MUL;
            operand = B.o.src == T ? B.o.src2 : B.o.src;
          }
          break;
        case MX_OP_GATE_APPLY:  // dst = u * (v + 1) with src = u, src2 = v
          if (B.o.src2 == T && B.o.src != T) {
            epi = EPI_GATE;
            operand = B.o.src;
          }
          break;
        default:
          break;
      }
      if (epi < 0) break;
      const int32_t D = B.o.dst;
      const bool identity = epi == EPI_NONE;
      const bool umma = H.umma(A.o);
      if (identity) {
        if (umma && !H.tma_view(D, out_channels(A.o))) break;
      } else if (A.o.kind == MX_OP_CHAN_SCALE) {
        // The channel-attention tail x * s + residual: one pass over x and
        // the residual (all views 4-channel aligned for the vector kernel);
        // a second residual add that follows joins it too.
        if (epi != EPI_ADD || A.epi_src2 >= 0 || (A.epi != EPI_NONE && A.epi != EPI_ADD)) break;
        if (!H.tma_view(D, A.o.c) || !H.tma_view(operand, A.o.c) || !H.tma_view(A.o.src, A.o.c)) break;
      } else if (H.small_conv && H.small_conv(A.o)) {
        if (A.epi != EPI_NONE || operand >= 0 || (epi != EPI_GELU && epi != EPI_LRELU && epi != EPI_SIGMOID)) break;
      } else {
        // (A transposed conv's epilogue only forwards copies.) A 1x1 conv's
        // residual add takes a second add that follows it.
        const bool add2 = A.o.kind == MX_OP_CONV1X1 && A.epi == EPI_ADD && A.epi_src2 < 0 && epi == EPI_ADD;
        if (!umma || (A.epi != EPI_NONE && !add2) || A.o.kind == MX_OP_CONVT2X2) break;
        if (!H.tma_view(D, out_channels(A.o))) break;
        if (operand >= 0 && !H.tma_view(operand, out_channels(A.o))) break;
      }
      // Dependences between the producer and the consumer's own position.
      int32_t br[3];
      const int nbr = reads_of(B.o, -1, br);
      for (size_t s = i + 1; s < j && ok; ++s) {
        if (dead[s]) continue;
        int32_t r[5], w[2];
        const int nr = step_reads(W[s], r), nw = writes_of(W[s].o, w);
        for (int a = 0; a < nw; ++a) {
          for (int b = 0; b < nbr; ++b)
            if (br[b] != T && G.overlap(w[a], br[b])) ok = false;
          if (G.overlap(w[a], D)) ok = false;
        }
        for (int a = 0; a < nr; ++a)
          if (G.overlap(r[a], D)) ok = false;
      }
      // Where the consumer's position is what stands in the way (its other
      // operand is produced in between, most often), a tensor-core producer
      // with no epilogue yet can run there instead: nothing in between may
      // then write what it reads (its output has no other reader).
      bool sink = false;
      if (!ok && umma && A.epi == EPI_NONE && A.stats_out[0] < 0 && A.ln_out < 0 &&
          A.o.kind != MX_OP_CHAN_SCALE && !(H.small_conv && H.small_conv(A.o))) {
        int32_t ar2[5];
        const int na2 = step_reads(A, ar2);
        sink = true;
        for (size_t s = i + 1; s < j && sink; ++s) {
          if (dead[s]) continue;
          int32_t w[5];
          const int nw = step_writes(W[s], w);
          for (int a = 0; a < nw; ++a)
            for (int b = 0; b < na2; ++b)
              if (G.overlap(w[a], ar2[b])) sink = false;
        }
        ok = sink;
      }
      if (!ok) break;
      // The destination against what the producer itself reads: an exact
      // match is an in-place elementwise update (each value is read before
      // the same thread writes it), anything else is refused.
      int32_t ar[5];
      const int nar = step_reads(A, ar);
      for (int a = 0; a < nar; ++a)
        if (G.overlap(ar[a], D) &&
            !(ar[a] == D && (elementwise(A.o.kind) || ar[a] == A.epi_src || ar[a] == A.epi_src2)))
          ok = false;
      if (operand >= 0 && G.overlap(operand, D) && operand != D) ok = false;
      if (operand >= 0 && operand == D && !umma && A.o.kind != MX_OP_CHAN_SCALE) ok = false;
      if (G.overlap(D, T) && D != T) ok = false;
      if (!ok) break;
      if (sink) {
        // The fused step takes the consumer's place in the order.
        SchedStep moved = std::move(W[i]);
        const std::vector<int32_t> bc = W[j].covers;
        moved.o.dst = D;
        if (!identity) {
          moved.epi = epi;
          moved.epi_src = operand;
          moved.epi_slope = W[j].o.slope;
        }
        moved.covers.insert(moved.covers.end(), bc.begin(), bc.end());
        W[j] = std::move(moved);
        dead[i] = 1;
        S.ops_fused += int(bc.size());
        ++S.steps_moved;
        break;
      }
      A.o.dst = D;
      if (!identity && (A.o.kind == MX_OP_CHAN_SCALE || A.o.kind == MX_OP_CONV1X1) && A.epi == EPI_ADD) {
        A.epi_src2 = operand;
      } else if (!identity) {
        A.epi = epi;
        A.epi_src = operand;
        A.epi_slope = B.o.slope;
      }
      A.covers.insert(A.covers.end(), B.covers.begin(), B.covers.end());
      dead[j] = 1;
      S.ops_fused += int(B.covers.size());
    }
  }
  // 2b. Copy elision. A Copy left after folding has a source with other
  // readers (or no producer to fold into). Where its destination is a whole
  // buffer that later steps read only as a whole, and neither it nor the
  // source is written while it is still read, those readers read the source
  // instead and the Copy is removed (it moved the same values).
  for (size_t c = 0; fuse && c < W.size(); ++c) {
    if (dead[c] || W[c].o.kind != MX_OP_COPY || p.ops[W[c].op].kind != MX_OP_COPY || W[c].epi != EPI_NONE) continue;
    const int32_t D = W[c].o.dst, Sr = W[c].o.src;
    if (D < 0 || Sr < 0 || G.root[size_t(D)] != D || !G.whole(D) || G.overlap(D, p.output) || G.overlap(Sr, D))
      continue;
    const mx_buf& bd = p.bufs[D];
    const mx_buf& bs = p.bufs[Sr];
    if (bd.c != bs.c || bd.h != bs.h || bd.w != bs.w || W[c].o.n != bd.c * bd.h * bd.w) continue;
    if (!H.tma_view(Sr, int(bd.c)) && H.tma_view(D, int(bd.c))) continue;
    std::vector<size_t> rd;
    bool ok = true, src_written = false;
    for (size_t s = c + 1; s < W.size() && ok; ++s) {
      if (dead[s]) continue;
      int32_t r[5], w[5];
      const int nr = step_reads(W[s], r), nw = step_writes(W[s], w);
      bool reads_d = false;
      for (int a = 0; a < nr; ++a)
        if (G.overlap(r[a], D)) {
          if (r[a] != D) ok = false;
          reads_d = true;
        }
      if (reads_d) {
        if (src_written) ok = false;
        rd.push_back(s);
      }
      bool d_written = false;
      for (int a = 0; a < nw; ++a) {
        if (G.overlap(w[a], Sr)) src_written = true;
        if (G.overlap(w[a], D)) d_written = true;
      }
      if (d_written) break;
    }
    if (!ok || rd.empty()) continue;
    for (size_t s : rd) {
      SchedStep& R = W[s];
      if (R.o.src == D) R.o.src = Sr;
      if (R.o.src2 == D) R.o.src2 = Sr;
      if (R.epi_src == D) R.epi_src = Sr;
      if (R.epi_src2 == D) R.epi_src2 = Sr;
    }
    dead[c] = 1;
    ++S.copies_elided;
  }

  // 3. LayerNorm on load: a LayerNorm whose only reader is a conv that can
  // normalise its A operand becomes a statistics step, and the conv reads
  // the LayerNorm's input instead of its output.
  for (size_t j = 0; fuse && j < W.size(); ++j) {
    if (dead[j] || W[j].o.kind != MX_OP_CHAN_LN || W[j].stats_only) continue;
    const mx_op L = W[j].o;
    const int32_t x = L.src, y = L.dst;
    if (G.overlap(y, p.output) || G.overlap(x, y)) continue;
    size_t k = SIZE_MAX;
    bool ok = true;
    for (size_t s = j + 1; s < W.size() && ok; ++s) {
      if (dead[s]) continue;
      int32_t r[5], w[2];
      const int nr = step_reads(W[s], r), nw = writes_of(W[s].o, w);
      for (int a = 0; a < nr; ++a)
        if (G.overlap(r[a], y)) {
          if (k != SIZE_MAX || r[a] != y) ok = false;
          else k = s;
        }
      bool gone = false;
      for (int a = 0; a < nw; ++a)
        if (G.overlap(w[a], y)) {
          if (G.covers(w[a], y)) gone = true;
          else ok = false;
        }
      if (gone) break;
    }
    if (!ok || k == SIZE_MAX) continue;
    SchedStep& C = W[k];
    if (C.o.src != y || C.o.src2 == y || C.epi_src == y || C.epi_src2 == y || C.ln_stats >= 0) continue;
    mx_op as_read = C.o;
    as_read.src = x;
    if (!H.umma(as_read) || !H.ln_on_load(as_read)) continue;
    // x must still hold the LayerNorm's input when the conv runs, and the
    // conv must not write over it.
    for (size_t s = j + 1; s < k && ok; ++s) {
      if (dead[s]) continue;
      int32_t w[2];
      const int nw = writes_of(W[s].o, w);
      for (int a = 0; a < nw; ++a)
        if (G.overlap(w[a], x)) ok = false;
    }
    if (!ok || G.overlap(C.o.dst, x)) continue;
    const mx_buf& yb = p.bufs[y];
    const int32_t sb = G.add(2);
    S.extra.push_back(mx_buf{2, yb.h, yb.w});
    W[j].stats_only = true;
    W[j].o.dst = sb;
    C.o.src = x;
    C.ln_stats = sb;
    C.ln_scale = L.scale;
    C.ln_bias = L.bias;
    ++S.ln_on_load;
  }

  // 3b. Statistics from the producer: a statistics step whose input was
  // last written by a tensor-core conv's epilogue, as a 32-aligned channel
  // group inside one output slice of it, is computed by that epilogue (each
  // of its threads holds whole pixel rows, in channel order) and disappears.
  for (size_t j = 0; fuse && j < W.size(); ++j) {
    if (dead[j] || !W[j].stats_only) continue;
    const int32_t x = W[j].o.src, sb = W[j].o.dst;
    size_t i = SIZE_MAX;
    bool ok = true;
    for (size_t s = j; s-- > 0;) {
      if (dead[s]) continue;
      int32_t w[5];
      const int nw = step_writes(W[s], w);
      bool hit = false;
      for (int a = 0; a < nw; ++a) hit |= G.overlap(w[a], x);
      if (!hit) continue;
      if (G.covers(W[s].o.dst, x)) i = s;
      else ok = false;
      break;
    }
    if (!ok || i == SIZE_MAX) continue;
    SchedStep& P = W[i];
    const int slice = H.stats_slice(P.o);
    if (slice <= 0) continue;
    const int64_t c0 = G.lo[size_t(x)] - G.lo[size_t(P.o.dst)], c = G.hi[size_t(x)] - G.lo[size_t(x)];
    if (c0 % 32 != 0 || (c != 32 && c != 64 && c != 128) || c0 / slice != (c0 + c - 1) / slice) continue;
    if (P.stats_c != 0 && P.stats_c != c) continue;
    const int g = P.stats_out[0] < 0 ? 0 : (P.stats_out[1] < 0 ? 1 : -1);
    if (g < 0) continue;
    P.stats_out[g] = sb;
    P.stats_c0[g] = int32_t(c0);
    P.stats_c = int32_t(c);
    P.covers.insert(P.covers.end(), W[j].covers.begin(), W[j].covers.end());
    dead[j] = 1;
    ++S.stats_in_epilogue;
    ++S.ops_fused;
  }

  // 3c. LayerNorm from the producer: a LayerNorm over exactly one 32-column
  // chunk of a tensor-core 1x1 conv's output (whose epilogue threads hold
  // whole pixel rows) is computed by that epilogue, which writes the
  // normalised chunk to the LayerNorm's output as well as the chunk itself
  // to its own. The LayerNorm's output is then written at the conv's step,
  // so nothing between the two may touch it.
  for (size_t j = 0; fuse && j < W.size(); ++j) {
    if (dead[j] || W[j].o.kind != MX_OP_CHAN_LN || W[j].stats_only) continue;
    const mx_op L = W[j].o;
    const int32_t x = L.src, y = L.dst;
    size_t i = SIZE_MAX;
    bool ok = true;
    for (size_t s = j; s-- > 0;) {
      if (dead[s]) continue;
      int32_t w[5];
      const int nw = step_writes(W[s], w);
      bool hit = false;
      for (int a = 0; a < nw; ++a) hit |= G.overlap(w[a], x);
      if (!hit) continue;
      if (G.covers(W[s].o.dst, x)) i = s;
      else ok = false;
      break;
    }
    if (!ok || i == SIZE_MAX) continue;
    SchedStep& P = W[i];
    // (A step with a second addend reads it through the map a LayerNorm
    // output would use.)
    if (P.o.kind != MX_OP_CONV1X1 || P.ln_out >= 0 || P.epi_src2 >= 0 || H.stats_slice(P.o) <= 0 ||
        !H.tma_view(y, 32))
      continue;
    const int64_t c0 = G.lo[size_t(x)] - G.lo[size_t(P.o.dst)], c = G.hi[size_t(x)] - G.lo[size_t(x)];
    if (c != 32 || c0 % 32 != 0) continue;
    if (G.overlap(y, p.output) || G.overlap(y, P.o.dst)) continue;
    int32_t pr[5];
    const int npr = step_reads(P, pr);
    for (int a = 0; a < npr; ++a) ok = ok && !G.overlap(pr[a], y);
    for (size_t s = i + 1; s < j && ok; ++s) {
      if (dead[s]) continue;
      int32_t r[5], w[5];
      const int nr = step_reads(W[s], r), nw = step_writes(W[s], w);
      for (int a = 0; a < nr; ++a) ok = ok && !G.overlap(r[a], y);
      for (int a = 0; a < nw; ++a) ok = ok && !G.overlap(w[a], y);
    }
    if (!ok) continue;
    P.ln_out = y;
    P.ln_out_c0 = int32_t(c0);
    P.ln_out_scale = L.scale;
    P.ln_out_bias = L.bias;
    P.ln_out_op = W[j].op;
    // Whether any later step reads the chunk itself (before a step covers it
    // with new values): if none does, the epilogue stores only its LayerNorm.
    bool read = G.overlap(x, p.output);
    for (size_t s = i + 1; s < W.size() && !read; ++s) {
      if (dead[s] || s == j) continue;
      int32_t r[5], w[5];
      const int nr = step_reads(W[s], r), nw = step_writes(W[s], w);
      for (int a = 0; a < nr; ++a) read = read || G.overlap(r[a], x);
      bool gone = false;
      for (int a = 0; a < nw; ++a) gone = gone || G.covers(w[a], x);
      if (gone) break;
    }
    P.ln_out_only = !read;
    P.covers.insert(P.covers.end(), W[j].covers.begin(), W[j].covers.end());
    dead[j] = 1;
    ++S.ln_in_epilogue;
    ++S.ops_fused;
  }

  // 3b. Merged placement. A Copy of a whole root Sr into a view D of
  // another root (a concatenation copied into a wider one: the UpSampleRatio
  // inputs stacked ahead of their 1x1 conv) moves nothing if Sr is placed
  // where D is: the steps that write Sr's channel slices then write D's. That
  // takes: Sr read by the Copy alone, written only before it, and nothing
  // else touching D from Sr's first write to the Copy.
  std::vector<int32_t> merge_root(size_t(p.n_bufs), -1);
  std::vector<int64_t> merge_delta(size_t(p.n_bufs), 0);
  std::vector<char> merge_target(size_t(p.n_bufs), 0);
  for (size_t c = 0; fuse && c < W.size(); ++c) {
    if (dead[c] || W[c].o.kind != MX_OP_COPY || p.ops[W[c].op].kind != MX_OP_COPY || W[c].epi != EPI_NONE ||
        W[c].covers.size() != 1)
      continue;
    const int32_t Sr = W[c].o.src, D = W[c].o.dst;
    if (Sr < 0 || D < 0 || Sr >= p.n_bufs || D >= p.n_bufs || G.root[size_t(Sr)] != Sr) continue;
    const int32_t Dr = G.root[size_t(D)];
    if (Dr == Sr || merge_root[size_t(Sr)] >= 0 || merge_target[size_t(Sr)] || merge_root[size_t(Dr)] >= 0) continue;
    if (G.overlap(Sr, p.output) || G.overlap(Sr, p.input) || G.overlap(D, p.output) || G.overlap(D, p.input)) continue;
    const mx_buf& bs = p.bufs[Sr];
    const mx_buf& bd = p.bufs[D];
    if (bs.c != bd.c || bs.h != bd.h || bs.w != bd.w || W[c].o.n != bs.c * bs.h * bs.w) continue;
    bool ok = true;
    size_t first = SIZE_MAX;
    for (size_t s = 0; s < W.size() && ok; ++s) {
      if (dead[s] || s == c) continue;
      int32_t r[5], w[5];
      const int nr = step_reads(W[s], r), nw = step_writes(W[s], w);
      for (int a = 0; a < nr; ++a)
        if (r[a] >= 0 && G.root[size_t(r[a])] == Sr) ok = false;  // Sr has another reader
      for (int a = 0; a < nw; ++a)
        if (w[a] >= 0 && G.root[size_t(w[a])] == Sr) {
          if (s > c) ok = false;  // written after the Copy
          first = std::min(first, s);
        }
    }
    for (size_t s = first; ok && first != SIZE_MAX && s < c; ++s) {
      if (dead[s]) continue;
      int32_t r[5], w[5];
      const int nr = step_reads(W[s], r), nw = step_writes(W[s], w);
      for (int a = 0; a < nr; ++a) ok = ok && !G.overlap(r[a], D);
      for (int a = 0; a < nw; ++a) ok = ok && !G.overlap(w[a], D);
    }
    if (!ok) continue;
    merge_root[size_t(Sr)] = Dr;
    merge_delta[size_t(Sr)] = p.offs[D] - p.offs[Dr];
    merge_target[size_t(Dr)] = 1;
    dead[c] = 1;
    ++S.copies_merged;
  }

  for (size_t i = 0; i < W.size(); ++i)
    if (!dead[i]) S.steps.push_back(std::move(W[i]));

  // 4. Pack the roots the steps touch, by first fit over live ranges.
  const int m = int(S.steps.size());
  const int32_t nb = p.n_bufs + int32_t(S.extra.size());
  std::vector<int> first(size_t(nb), INT_MAX), last(size_t(nb), INT_MIN);
  // A merged root lives and is placed with the root it is merged into.
  auto placed = [&](int32_t r) { return r < p.n_bufs && merge_root[size_t(r)] >= 0 ? merge_root[size_t(r)] : r; };
  auto touch = [&](int32_t b, int t) {
    if (b < 0) return;
    const size_t r = size_t(placed(G.root[size_t(b)]));
    first[r] = std::min(first[r], t);
    last[r] = std::max(last[r], t);
  };
  touch(p.input, -1);
  touch(p.output, m);
  for (int t = 0; t < m; ++t) {
    int32_t r[5], w[5];
    const int nr = step_reads(S.steps[size_t(t)], r);
    const int nw = step_writes(S.steps[size_t(t)], w);
    for (int a = 0; a < nr; ++a) touch(r[a], t);
    for (int a = 0; a < nw; ++a) touch(w[a], t);
  }
  struct Slot {
    int32_t root;
    int64_t size, off;
  };
  std::vector<Slot> order;
  for (int32_t b = 0; b < nb; ++b)
    if (G.root[size_t(b)] == b && placed(b) == b && first[size_t(b)] <= last[size_t(b)]) {
      const mx_buf& bb = b < p.n_bufs ? p.bufs[b] : S.extra[size_t(b - p.n_bufs)];
      const int64_t len = bb.c * bb.h * bb.w;
      order.push_back({b, (len + 63) / 64 * 64, 0});
    }
  std::stable_sort(order.begin(), order.end(), [&](const Slot& a, const Slot& b) {
    if (a.size != b.size) return a.size > b.size;
    return first[size_t(a.root)] < first[size_t(b.root)];
  });
  std::vector<int64_t> root_off(size_t(nb), 0);
  std::vector<std::pair<int64_t, int64_t>> busy;
  for (size_t i = 0; i < order.size(); ++i) {
    Slot& s = order[i];
    busy.clear();
    for (size_t k = 0; k < i; ++k) {
      const Slot& q = order[k];
      if (first[size_t(q.root)] <= last[size_t(s.root)] && first[size_t(s.root)] <= last[size_t(q.root)])
        busy.push_back({q.off, q.off + q.size});
    }
    std::sort(busy.begin(), busy.end());
    int64_t off = 0;
    for (const auto& iv : busy) {
      if (off + s.size <= iv.first) break;
      off = std::max(off, iv.second);
    }
    s.off = off;
    root_off[size_t(s.root)] = off;
    S.arena_len = std::max(S.arena_len, off + s.size);
  }
  S.offs.resize(size_t(nb));
  for (int32_t b = 0; b < nb; ++b) {
    const int32_t r = G.root[size_t(b)];
    const int64_t at = placed(r) == r ? root_off[size_t(r)] : root_off[size_t(placed(r))] + merge_delta[size_t(r)];
    S.offs[size_t(b)] = at + (b < p.n_bufs ? p.offs[b] - p.offs[r] : 0);
  }
  S.arena_len = std::max<int64_t>(S.arena_len, 64);
  S.merged_into = std::move(merge_root);
  return S;
}

}  // namespace mx
