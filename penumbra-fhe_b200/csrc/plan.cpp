// plan.cpp -- graph -> batched ciphertext program (see plan.hpp for the construction).
#include "plan.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <functional>
#include <map>
#include <numeric>
#include <sstream>

namespace pnb {
namespace plan {

using ir::Error;
using ir::OpType;
typedef __int128 i128;

namespace {

[[noreturn]] void fail(const std::string& m) { throw Error(m); }

// smallest b >= 1 with -2^(b-1) <= lo and hi < 2^(b-1)
int bits_signed(int64_t lo, int64_t hi) {
  int b = 1;
  while (b < 64 && !((i128)lo >= -((i128)1 << (b - 1)) && (i128)hi < ((i128)1 << (b - 1)))) ++b;
  return b;
}

int64_t floor_shift(int64_t v, int s) { return s >= 63 ? (v < 0 ? -1 : 0) : (v >> s); }

i128 ceil_div(i128 a, i128 b) {  // b > 0
  i128 q = a / b;
  if ((a % b) != 0 && a > 0) ++q;
  return q;
}

uint64_t pow2(int e) { return e >= 64 ? 0 : (uint64_t)1 << e; }

struct Range {
  int64_t lo = 0, hi = 0;
};

int64_t to_i64(i128 v, const std::string& where) {
  if (v > (i128)INT64_MAX / 4 || v < (i128)INT64_MIN / 4)
    fail("value range of " + where + " exceeds what a 64-bit torus can hold exactly");
  return (int64_t)v;
}

// One element of a threshold node (Requant / Argmax): output = base + sum_j delta_j [y >= T_j].
struct Pair {
  int e;         // element
  int j;         // threshold index within the element (Requant: the clamp step j)
  int64_t T;     // y-space threshold
  int64_t delta;
};

}  // namespace

double ksms_log2_sigma(int n, int N, int k, int ks_base_log, int ks_level, double lwe_std) {
  const double kN = (double)k * N;
  const int kept = ks_base_log * ks_level;
  const double step = std::ldexp(1.0, 64 - kept);  // keyswitch rounds a_i to this step
  const double v_round = (kN / 2) * step * step / 12.0;
  const double half_b = std::ldexp(1.0, ks_base_log - 1);
  const double e_d2 = (4 * half_b * half_b + 2) / 12.0;  // balanced digit second moment
  const double s = lwe_std * std::ldexp(1.0, 64);
  const double v_key = kN * ks_level * e_d2 * s * s;
  const double ms_step = std::ldexp(1.0, 64 - (int)std::lround(std::log2(2.0 * N)));
  const double v_ms = (n / 2.0 + 1) * ms_step * ms_step / 12.0;
  return 0.5 * std::log2(v_round + v_key + v_ms);
}

std::vector<KeyLevel> default_levels(int n, int N, int k, double glwe_std) {
  // (base_log, level, measured output noise of the default set, relative cost)
  struct Row {
    int b, l;
    double sig, cost;
  };
  // noise measured on a B200 over 4096 bootstraps (rounded up); cost = measured time per
  // bootstrap relative to the single-level kernel (87.6k PBS/s against 44.6k, 29.4k, 23.7k,
  // 17.0k and 12.0k at batch 4096)
  static const Row rows[] = {{23, 1, 49.1, 1.0}, {15, 2, 42.0, 1.96}, {11, 3, 38.75, 2.98},
                             {10, 4, 36.6, 3.70}, {7, 6, 33.9, 5.15}, {5, 9, 32.3, 7.33}};
  const bool is_default = (n == 834 && N == 2048 && k == 1 &&
                           std::fabs(glwe_std - 2.845267479601915e-15) < 1e-20);
  std::vector<KeyLevel> out;
  if (N == 8192) {
    // the gadgets compiled for N = 8192; noise: key noise through the digits, gadget rounding
    // and the f64 product's error (relative 2^-51.1 of the product's spread, as measured at
    // N = 2048), the last two amplified by the secret key (1 + kN/2 terms)
    struct R8 {
      int b, l;
      double cost;
    };
    static const R8 r8[] = {{23, 1, 1.0}, {15, 2, 1.5}, {11, 4, 2.5}};
    const double s = glwe_std * std::ldexp(1.0, 64);
    for (const R8& r : r8) {
      const double B = std::ldexp(1.0, r.b);
      const double ed2 = B * B / 12.0;
      const double v1 = (double)n * (k + 1) * r.l * N * ed2 * s * s;
      const double eps = std::ldexp(1.0, 64 - r.b * r.l);
      const double v2 = (n / 2.0) * (1 + k * N / 2.0) * eps * eps / 12.0;
      const double sprod2 = std::exp2(-2 * 51.1) * N * ed2 * std::ldexp(1.0, 126) / 3.0;
      const double v3 = (double)n * (1 + k * N / 2.0) * (k + 1) * r.l * sprod2;
      KeyLevel L;
      L.base_log = r.b;
      L.level = r.l;
      L.cost = r.cost;
      L.log2_sigma = 0.5 * std::log2(v1 + v2 + v3);
      out.push_back(L);
    }
    return out;
  }
  for (const Row& r : rows) {
    KeyLevel L;
    L.base_log = r.b;
    L.level = r.l;
    L.cost = r.cost;
    if (is_default) {
      L.log2_sigma = r.sig;
    } else {
      // blind-rotation output: key noise through the gadget digits + gadget rounding,
      // plus 0.7 bit for the f64 transforms (what the measured set shows over this formula)
      const double B = std::ldexp(1.0, r.b), s = glwe_std * std::ldexp(1.0, 64);
      const double v1 = (double)n * (k + 1) * r.l * N * (B * B / 12.0) * s * s;
      const double eps = std::ldexp(1.0, 64 - r.b * r.l);
      const double v2 = (n / 2.0) * (1 + k * N / 2.0) * eps * eps / 12.0;
      L.log2_sigma = 0.5 * std::log2(v1 + v2) + 0.7;
    }
    out.push_back(L);
  }
  return out;
}

namespace {

struct Builder {
  const ir::Graph& g;
  Options o;
  Program P;
  double V_ksms;
  std::vector<int> lvl_order;  // levels sorted by cost

  // per IR tensor
  std::map<std::string, int> tid;
  std::vector<std::string> tname;
  std::vector<std::vector<Range>> range;
  std::vector<int> producer;  // node index or -1 (graph input)
  std::vector<int> cls;       // scale class (union-find)
  std::vector<int> scale;
  std::vector<double> vmax, var;
  std::vector<int> buf;
  std::vector<std::vector<int64_t>> k0s;  // per threshold node (see thresholds())
  // Share of a bootstrap read's noise budget granted to the value it reads (the rest is left to
  // the bootstrap outputs the chain adds before its next read).
  double vfrac = 0.5;

  Builder(const ir::Graph& gr, const Options& op) : g(gr), o(op) {}

  int find(int a) { return cls[a] == a ? a : cls[a] = find(cls[a]); }
  void unite(int a, int b) { cls[find(a)] = find(b); }

  int tensor(const std::string& n) {
    auto it = tid.find(n);
    if (it != tid.end()) return it->second;
    const int id = (int)tname.size();
    tid[n] = id;
    tname.push_back(n);
    range.emplace_back();
    producer.push_back(-1);
    cls.push_back(id);
    return id;
  }

  // ---- noise model -------------------------------------------------------------------
  // Largest variance of a ciphertext (at its own scale, LSB 2^E) that a bootstrap reading
  // cells of 2^cell_log2 may see while keeping z sigma below half a cell.
  double allowed(int cell_log2, int E) const {
    const double h = std::ldexp(1.0, cell_log2 - 1) / o.z;
    const double a = h * h - V_ksms;
    if (a <= 0) return -1;
    return a * std::ldexp(1.0, 2 * (E - cell_log2));
  }
  double lvar(int l) const {
    const double s = std::ldexp(1.0, 0) * std::exp2(o.levels[l].log2_sigma);
    return s * s;
  }
  // cheapest level whose output keeps v + V_l <= 0.9 * limit; -1 if none
  int pick(double v, double limit) const {
    for (int l : lvl_order)
      if (v + lvar(l) <= 0.9 * limit) return l;
    return -1;
  }

  // ---- program emission --------------------------------------------------------------
  int new_buf(int64_t elems, const std::string& name) {
    P.bufs.push_back({elems, name});
    return (int)P.bufs.size() - 1;
  }
  int tv(const TvSpec& s) {
    for (size_t i = 0; i < P.tvs.size(); ++i)
      if (P.tvs[i].lut_len == s.lut_len && P.tvs[i].val == s.val) return (int)i;
    P.tvs.push_back(s);
    return (int)P.tvs.size() - 1;
  }
  TvSpec const_tv(uint64_t c) {
    TvSpec s;
    s.lut_len = 0;  // 0 = constant over the whole half torus (no box centring)
    s.val = {c};
    return s;
  }
  void lin(int dst, std::vector<Term> terms, std::vector<uint64_t> cst, const std::string& w) {
    Instr I;
    I.kind = Kind::Lin;
    I.dst = dst;
    I.terms = std::move(terms);
    I.cst = std::move(cst);
    I.what = w;
    P.code.push_back(std::move(I));
  }
  void pbs(int dst, int src, int shift, uint64_t offset, int level, std::vector<int32_t> tvi,
           int64_t count, const std::string& w) {
    if (shift < 0 || shift > 63) fail("internal: bootstrap input shift out of range");
    Instr I;
    I.kind = Kind::Pbs;
    I.dst = dst;
    I.src = src;
    I.shift = shift;
    I.offset = offset;
    I.level = level;
    I.tv = std::move(tvi);
    I.what = w;
    P.code.push_back(std::move(I));
    P.pbs_per_sample += count;
    P.cost_per_sample += (double)count * o.levels[level].cost;
    if ((int)per_level.size() < (int)o.levels.size()) per_level.assign(o.levels.size(), 0);
    per_level[level] += count;
    P.pbs_per_level = per_level;
  }
  std::vector<int64_t> per_level;

  // A digit chain: the running value in buffer R (count elements per sample) at LSB scale
  // 2^E with noise variance V; X is the bootstrap output scratch (same element count).
  struct Chain {
    int R;
    int X;
    int64_t count;
    int E;
    double V;
  };

  // Key sets for a given window sequence (LSB first): each bootstrap takes the cheapest key
  // whose output keeps the next read within its budget.  False when some read is over budget.
  bool eval_windows(const Chain& c, const std::vector<int>& ws, int final_cell,
                    std::vector<int>* lv, double* Vend, double* cost) const {
    // read sequence: (cell, E) per read; pbs i adds noise before read i+1
    std::vector<std::pair<int, int>> reads;
    int E = c.E;
    for (int w : ws) {
      reads.push_back({64 - w, E});
      if (w >= 2) reads.push_back({64 - w, E});
      E += w;
    }
    reads.push_back({final_cell, E});
    double V = c.V;
    lv->clear();
    *cost = 0;
    for (size_t r = 0; r + 1 < reads.size(); ++r) {
      const double A = allowed(reads[r].first, reads[r].second);
      if (A < 0 || V > A) return false;
      const double An = allowed(reads[r + 1].first, reads[r + 1].second);
      const int l = pick(V, An);
      if (l < 0) return false;
      lv->push_back(l);
      V += lvar(l);
      *cost += o.levels[l].cost;
    }
    const double Af = allowed(reads.back().first, reads.back().second);
    if (Af < 0 || V > Af) return false;
    *Vend = V;
    return true;
  }

  // Remove the low k bits: the cheapest split into windows of 1..5 bits (every split for
  // k <= 17; for wider chains the first 12 bits are searched and the rest taken in fives).
  bool plan_windows(Chain c, int k, int final_cell, std::vector<int>* lv, double* Vend,
                    double* cost, std::vector<int>* ws_out = nullptr) {
    const int head = k <= 17 ? k : 12;
    std::vector<int> tail;
    for (int r = k - head; r > 0; r -= std::min(r, 5)) tail.push_back(std::min(r, 5));
    std::vector<int> cur, best_ws, best_lv, tmp_lv;
    double best = 1e300, best_V = 0;
    std::function<void(int)> rec = [&](int left) {
      if (left == 0) {
        std::vector<int> ws = cur;
        ws.insert(ws.end(), tail.begin(), tail.end());
        double V, cst;
        if (eval_windows(c, ws, final_cell, &tmp_lv, &V, &cst) && cst < best - 1e-9) {
          best = cst;
          best_ws = ws;
          best_lv = tmp_lv;
          best_V = V;
        }
        return;
      }
      for (int w = std::min(5, left); w >= 1; --w) {
        cur.push_back(w);
        rec(left - w);
        cur.pop_back();
      }
    };
    rec(head);
    if (best >= 1e300) return false;
    *lv = best_lv;
    *Vend = best_V;
    *cost = best;
    if (ws_out) *ws_out = best_ws;
    return true;
  }
  void emit_windows(Chain& c, const std::vector<int>& ws, const std::vector<int>& lv,
                    const std::string& what) {
    const int X = c.X;
    size_t li = 0;
    for (int w : ws) {
      const int shift = 64 - w - c.E;
      const uint64_t C = w >= 2 ? pow2(w - 2 + c.E) : pow2(c.E - 1);
      // top bit of the window through the negacyclic sign: out = +C (bit 0) or -C (bit 1)
      pbs(X, c.R, shift, pow2(63 - w), lv[li], {tv(const_tv(C))}, c.count,
          what + ": window sign at 2^" + std::to_string(c.E));
      c.V += lvar(lv[li++]);
      lin(c.R, {Term{c.R, {1}, {}}, Term{X, {1}, {}}}, {(uint64_t)0 - C}, what + ": clear bit");
      if (w >= 2) {
        TvSpec d;
        d.lut_len = 1 << (w - 1);
        for (int v = 0; v < d.lut_len; ++v) d.val.push_back((uint64_t)v << c.E);
        pbs(X, c.R, shift, 0, lv[li], {tv(d)}, c.count,
            what + ": window digits at 2^" + std::to_string(c.E));
        c.V += lvar(lv[li++]);
        lin(c.R, {Term{c.R, {1}, {}}, Term{X, {-1}, {}}}, {0}, what + ": clear digits");
      }
      c.E += w;
    }
  }

  // ---- graph analysis ----------------------------------------------------------------
  void ranges() {
    for (const auto& n : g.inputs) {
      const int t = tensor(n);
      (void)t;
    }
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& nd = g.nodes[ni];
      std::vector<int64_t> in_lens;
      for (const auto& i : nd.inputs) in_lens.push_back((int64_t)range[tensor(i)].size());
      const int64_t len = ir::output_length(nd.op, in_lens);
      const int t = tensor(nd.outputs[0]);
      producer[t] = (int)ni;
      const auto& X = range[tensor(nd.inputs[0])];
      std::vector<Range> R((size_t)len);
      const auto& op = nd.op;
      const std::string where = "node '" + nd.name + "'";
      switch (op.type) {
        case OpType::Linear:
          for (int64_t m = 0; m < len; ++m) {
            i128 lo = op.bias[m], hi = op.bias[m];
            for (size_t k = 0; k < X.size(); ++k) {
              const i128 w = op.weights[m][k];
              lo += w >= 0 ? w * X[k].lo : w * X[k].hi;
              hi += w >= 0 ? w * X[k].hi : w * X[k].lo;
            }
            R[m] = {to_i64(lo, where), to_i64(hi, where)};
          }
          break;
        case OpType::Conv2d: {
          const int oh = (op.in_h + 2 * op.padding - op.kernel_h) / op.stride + 1;
          const int ow = (op.in_w + 2 * op.padding - op.kernel_w) / op.stride + 1;
          for (size_t oc = 0; oc < op.weights.size(); ++oc)
            for (int oy = 0; oy < oh; ++oy)
              for (int ox = 0; ox < ow; ++ox) {
                i128 lo = op.bias[oc], hi = op.bias[oc];
                for (int ic = 0; ic < op.in_channels; ++ic)
                  for (int ky = 0; ky < op.kernel_h; ++ky)
                    for (int kx = 0; kx < op.kernel_w; ++kx) {
                      const int iy = oy * op.stride + ky - op.padding;
                      const int ix = ox * op.stride + kx - op.padding;
                      if (iy < 0 || ix < 0 || iy >= op.in_h || ix >= op.in_w) continue;
                      const i128 w = op.weights[oc][(ic * op.kernel_h + ky) * op.kernel_w + kx];
                      const Range& r = X[(size_t)ic * op.in_h * op.in_w + iy * op.in_w + ix];
                      lo += w >= 0 ? w * r.lo : w * r.hi;
                      hi += w >= 0 ? w * r.hi : w * r.lo;
                    }
                R[(oc * oh + oy) * ow + ox] = {to_i64(lo, where), to_i64(hi, where)};
              }
          break;
        }
        case OpType::Pool: {
          const int oh = (op.in_h - op.pool_h) / op.stride + 1;
          const int ow = (op.in_w - op.pool_w) / op.stride + 1;
          for (int c = 0; c < op.channels; ++c)
            for (int oy = 0; oy < oh; ++oy)
              for (int ox = 0; ox < ow; ++ox) {
                i128 lo = 0, hi = 0;
                bool first = true;
                for (int ky = 0; ky < op.pool_h; ++ky)
                  for (int kx = 0; kx < op.pool_w; ++kx) {
                    const Range& r = X[(size_t)c * op.in_h * op.in_w +
                                       (oy * op.stride + ky) * op.in_w + ox * op.stride + kx];
                    if (op.pool_avg) {
                      lo += r.lo;
                      hi += r.hi;
                    } else {
                      lo = first ? r.lo : std::max<i128>(lo, r.lo);
                      hi = first ? r.hi : std::max<i128>(hi, r.hi);
                    }
                    first = false;
                  }
                R[(c * oh + oy) * ow + ox] = {to_i64(lo, where), to_i64(hi, where)};
              }
          break;
        }
        case OpType::Requant: {
          const int64_t M = (1 << op.out_bits) - 1;
          int64_t lo = INT64_MAX, hi = INT64_MIN;
          for (int64_t c = 0; c <= M; ++c) {
            lo = std::min<int64_t>(lo, (int64_t)op.clamp_lut[c]);
            hi = std::max<int64_t>(hi, (int64_t)op.clamp_lut[c]);
          }
          for (auto& r : R) r = {lo, hi};
          break;
        }
        case OpType::Activation: {
          for (size_t e = 0; e < R.size(); ++e) {
            int64_t lo = INT64_MAX, hi = INT64_MIN;
            for (int64_t v = X[e].lo; v <= X[e].hi && v - X[e].lo < 64; ++v) {
              const int64_t y = (int64_t)op.lut[((v % 4) + 4) % 4];
              lo = std::min(lo, y);
              hi = std::max(hi, y);
            }
            R[e] = {lo, hi};
          }
          break;
        }
        case OpType::Argmax:
          R[0] = {0, 1};
          break;
        case OpType::Add: {
          const auto& Y = range[tensor(nd.inputs[1])];
          for (int64_t e = 0; e < len; ++e)
            R[e] = {to_i64((i128)X[e].lo + Y[e].lo, where), to_i64((i128)X[e].hi + Y[e].hi, where)};
          unite(tensor(nd.inputs[0]), tensor(nd.inputs[1]));
          break;
        }
      }
      if (op.type == OpType::Linear || op.type == OpType::Conv2d ||
          (op.type == OpType::Pool && (op.pool_avg || wide_max(X))) || op.type == OpType::Add)
        unite(t, tensor(nd.inputs[0]));
      range[t] = std::move(R);
      if (op.type == OpType::Linear || op.type == OpType::Conv2d) {
        for (const auto& row : op.weights)
          for (int64_t w : row)
            if (w < -128 || w > 127)
              fail("node '" + nd.name + "': weight " + std::to_string(w) +
                   " does not fit the int8 tensor-core contraction");
      }
    }
  }

  // Max pooling reads a tensor spanning at most four values with one pairwise lookup; wider
  // tensors go through the digits of each pairwise difference (emit_maxpool_wide).
  static bool wide_max(const std::vector<Range>& x) {
    int64_t lo = INT64_MAX, hi = INT64_MIN;
    for (const auto& r : x) {
      lo = std::min(lo, r.lo);
      hi = std::max(hi, r.hi);
    }
    return hi - lo > 3;
  }
  static void span_of(const std::vector<Range>& x, int64_t* lo, int64_t* hi) {
    *lo = INT64_MAX;
    *hi = INT64_MIN;
    for (const auto& r : x) {
      *lo = std::min(*lo, r.lo);
      *hi = std::max(*hi, r.hi);
    }
  }

  // thresholds of a Requant / Argmax node, per element
  // k0[e]: the clamp index every y of element e reaches (c0 plus the thresholds decided as
  // crossed); the output is clamp_lut[k0 + number of undecided thresholds crossed].
  void thresholds(const ir::Node& nd, const std::vector<Range>& y, std::vector<Pair>* pairs,
                  std::vector<int64_t>* base, std::vector<int64_t>* k0 = nullptr) {
    const auto& op = nd.op;
    base->assign(y.size(), 0);
    if (k0) k0->assign(y.size(), 0);
    pairs->clear();
    for (size_t e = 0; e < y.size(); ++e) {
      if (op.type == OpType::Argmax) {
        if (op.threshold <= y[e].lo) (*base)[e] = 1;
        else if (op.threshold <= y[e].hi) pairs->push_back({(int)e, 1, op.threshold, 1});
        continue;
      }
      uint64_t mult = op.mult, rb = op.round_bias;
      uint32_t s = op.shift;
      if (!op.mults.empty()) {
        const size_t ch = e / op.channel_size;
        mult = op.mults[ch];
        rb = op.round_biases[ch];
        s = op.shifts[ch];
      }
      const int64_t M = (1 << op.out_bits) - 1;
      const int64_t c0 = s >= 64 ? 0 : (int64_t)std::min<uint64_t>(rb >> s, (uint64_t)M);
      int64_t b = (int64_t)op.clamp_lut[c0];
      int64_t kk = c0;
      for (int64_t j = c0 + 1; j <= M; ++j) {
        const int64_t delta = (int64_t)op.clamp_lut[j] - (int64_t)op.clamp_lut[j - 1];
        // y >= T  <=>  mult*y + rb >= j*2^s  (for y >= 0; j*2^s > rb so T > 0)
        const i128 num = s >= 100 ? ((i128)1 << 100) : ((i128)j << s) - (i128)rb;
        const i128 T = ceil_div(num, (i128)mult);
        if (T <= y[e].lo) {
          b += delta;
          ++kk;
        } else if (T <= y[e].hi && delta != 0) {
          pairs->push_back({(int)e, (int)j, (int64_t)T, delta});
        }
      }
      (*base)[e] = b;
      if (k0) (*k0)[e] = kk;
    }
  }

  // bits the y-space chain must remove so that every (y - T) >> k fits 5 signed bits
  static void chain_bits(const std::vector<std::pair<int64_t, int64_t>>& v, int* k, int* bf) {
    for (int kk = 0; kk < 64; ++kk) {
      int b = 1;
      for (const auto& r : v) b = std::max(b, bits_signed(floor_shift(r.first, kk),
                                                          floor_shift(r.second, kk)));
      if (b <= 5) {
        *k = kk;
        *bf = b;
        return;
      }
    }
    *k = 63;
    *bf = 1;
  }

  // ---- top level ---------------------------------------------------------------------
  const InputSpec* spec_of(size_t gi) const {
    return gi < o.input_specs.size() ? &o.input_specs[gi] : nullptr;
  }

  void run() {
    if (o.check_budget) ir::check_graph_bit_width_budget(g);
    for (size_t i = 0; i < o.levels.size(); ++i) lvl_order.push_back((int)i);
    std::sort(lvl_order.begin(), lvl_order.end(),
              [&](int a, int b) { return o.levels[a].cost < o.levels[b].cost; });
    if (o.levels.empty()) fail("no bootstrap key sets given");
    V_ksms = std::exp2(2 * o.log2_ksms);
    if (o.input_lo > o.input_hi) fail("input range is empty");

    for (const auto& n : g.inputs) tensor(n);
    // graph inputs need a length: the first consumer's expectation
    for (const auto& n : g.inputs) {
      int64_t len = -1;
      for (const auto& nd : g.nodes)
        for (size_t q = 0; q < nd.inputs.size(); ++q)
          if (nd.inputs[q] == n && len < 0) {
            const auto& op = nd.op;
            switch (op.type) {
              case OpType::Linear: len = op.weights[0].size(); break;
              case OpType::Conv2d: len = (int64_t)op.in_channels * op.in_h * op.in_w; break;
              case OpType::Pool: len = (int64_t)op.channels * op.in_h * op.in_w; break;
              case OpType::Argmax: len = 1; break;
              default: break;
            }
          }
      const size_t gi = (size_t)(&n - &g.inputs[0]);
      const int64_t given = gi < o.input_lens.size() ? o.input_lens[gi] : 0;
      if (given > 0) {
        if (len >= 0 && len != given)
          fail("graph input '" + n + "' is given " + std::to_string(given) +
               " elements but its consumer expects " + std::to_string(len));
        len = given;
      }
      if (len < 0)
        fail("graph input '" + n + "' has no consumer that fixes its length (Linear, Conv2d, "
             "Pool or Argmax); pass its length explicitly");
      const InputSpec* sp = spec_of(gi);
      if (sp && sp->ranged && sp->lo > sp->hi) fail("graph input '" + n + "': empty value range");
      range[tensor(n)].assign((size_t)len, sp && sp->ranged ? Range{sp->lo, sp->hi}
                                                            : Range{o.input_lo, o.input_hi});
    }
    ranges();
    const int T = (int)tname.size();
    scale.assign(T, 63);
    vmax.assign(T, 1e300);
    var.assign(T, 0);
    buf.assign(T, -1);

    // per threshold node: pairs and base
    std::vector<std::vector<Pair>> pairs(g.nodes.size());
    std::vector<std::vector<int64_t>> bases(g.nodes.size());
    k0s.assign(g.nodes.size(), {});
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& nd = g.nodes[ni];
      if (nd.op.type == OpType::Requant || nd.op.type == OpType::Argmax)
        thresholds(nd, range[tensor(nd.inputs[0])], &pairs[ni], &bases[ni], &k0s[ni]);
    }

    // scale of each class: the widest signed range any member (or chain on it) must hold
    std::vector<int> cap(T, 62);
    auto tighten = [&](int t, int64_t lo, int64_t hi) {
      const int c = find(t);
      cap[c] = std::min(cap[c], 63 - bits_signed(lo, hi));
    };
    for (int t = 0; t < T; ++t)
      for (const auto& r : range[t]) tighten(t, r.lo, r.hi);
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& nd = g.nodes[ni];
      const int yt = tensor(nd.inputs[0]);
      for (const Pair& p : pairs[ni])
        tighten(yt, range[yt][p.e].lo - p.T, range[yt][p.e].hi - p.T);
      if (nd.op.type == OpType::Pool && !nd.op.pool_avg && wide_max(range[yt])) {
        // the pairwise differences a - b are split into digits at the input's scale
        int64_t lo, hi;
        span_of(range[yt], &lo, &hi);
        tighten(yt, lo - hi, hi - lo);
      } else if (nd.op.type == OpType::Activation ||
                 (nd.op.type == OpType::Pool && !nd.op.pool_avg)) {
        cap[find(yt)] = std::min(cap[find(yt)], 59);
      }
    }
    // A Requant reading a class rooted at a graph input sees fresh (tiny) noise, so the single
    // z = mult*y + rb chain is affordable there: leave room for z's wider range.
    std::vector<char> fresh(T, 0);
    for (int t = 0; t < T; ++t)
      if (producer[t] < 0) fresh[find(t)] = 1;
    for (size_t gi = 0; gi < g.inputs.size(); ++gi) {
      const InputSpec* sp = spec_of(gi);
      if (sp && (sp->scale > 0 || sp->log2_sigma > 0)) fresh[find(tensor(g.inputs[gi]))] = 0;
    }
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& op = g.nodes[ni].op;
      const int yt = tensor(g.nodes[ni].inputs[0]);
      if (op.type != OpType::Requant || pairs[ni].empty() || !fresh[find(yt)]) continue;
      bool uniform = true;
      for (uint32_t x : op.shifts) uniform = uniform && x == op.shifts[0];
      if (!uniform) continue;
      i128 zlo = 0, zhi = 0;
      bool first = true;
      for (const Pair& p : pairs[ni]) {
        const size_t ch = op.mults.empty() ? 0 : p.e / op.channel_size;
        const i128 m = op.mults.empty() ? op.mult : op.mults[ch];
        const i128 rb = op.mults.empty() ? op.round_bias : op.round_biases[ch];
        const i128 a = m * range[yt][p.e].lo + rb, b = m * range[yt][p.e].hi + rb;
        zlo = first ? a : std::min(zlo, a);
        zhi = first ? b : std::max(zhi, b);
        first = false;
      }
      if (zlo > -((i128)1 << 56) && zhi < ((i128)1 << 56)) tighten(yt, (int64_t)zlo, (int64_t)zhi);
    }
    // scales the caller pins: inputs arriving from earlier ops, outputs feeding later ones
    std::vector<int> forced(T, 0);
    auto force = [&](int t, int s, const std::string& what) {
      const int c = find(t);
      if (s > cap[c])
        fail(what + " at scale 2^" + std::to_string(s) + " leaves no room for the values it " +
             "must hold (at most 2^" + std::to_string(cap[c]) + ")");
      if (forced[c] && forced[c] != s)
        fail(what + ": scales 2^" + std::to_string(forced[c]) + " and 2^" + std::to_string(s) +
             " meet where one encoding is needed");
      forced[c] = s;
      cap[c] = s;
    };
    for (size_t gi = 0; gi < g.inputs.size(); ++gi) {
      const InputSpec* sp = spec_of(gi);
      if (sp && sp->scale > 0) force(tensor(g.inputs[gi]), sp->scale, "graph input '" + g.inputs[gi] + "'");
    }
    if (o.output_scale > 0)
      for (const auto& n : g.outputs) force(tensor(n), o.output_scale, "graph output '" + n + "'");
    for (int t = 0; t < T; ++t) {
      scale[t] = cap[find(t)];
      if (scale[t] < 8)
        fail("tensor '" + tname[t] + "' spans more than 55 bits; no exact encoding exists");
    }

    // backward pass: the largest noise each tensor may carry
    for (const auto& n : g.outputs) {
      const int t = tensor(n);
      const double h = std::ldexp(1.0, scale[t] - 1) / o.z;
      vmax[t] = std::min(vmax[t], h * h);
      if (o.output_log2_sigma > 0) vmax[t] = std::min(vmax[t], std::exp2(2 * o.output_log2_sigma));
    }
    for (int ni = (int)g.nodes.size() - 1; ni >= 0; --ni) {
      const auto& nd = g.nodes[ni];
      const int out = tensor(nd.outputs[0]);
      const int in = tensor(nd.inputs[0]);
      const auto& op = nd.op;
      switch (op.type) {
        case OpType::Linear:
        case OpType::Conv2d: {
          double w2 = 0;
          for (const auto& row : op.weights) {
            double s = 0;
            for (int64_t w : row) s += (double)w * w;
            w2 = std::max(w2, s);
          }
          vmax[in] = std::min(vmax[in], vmax[out] / std::max(w2, 1.0));
          break;
        }
        case OpType::Pool:
          if (op.pool_avg)
            vmax[in] = std::min(vmax[in], vmax[out] / (op.pool_h * op.pool_w));
          else if (wide_max(range[in]))  // a - b read in 2-bit windows (emit_maxpool_wide)
            vmax[in] = std::min(vmax[in], 0.25 * allowed(62, scale[in]));
          else  // read as 4a + b at cells of 2^59 (see emit_maxpool)
            vmax[in] = std::min(vmax[in], 0.9 * allowed(59, scale[in]) / 17.0);
          break;
        case OpType::Add:
          vmax[in] = std::min(vmax[in], vmax[out] / 2);
          vmax[tensor(nd.inputs[1])] = std::min(vmax[tensor(nd.inputs[1])], vmax[out] / 2);
          break;
        case OpType::Requant:
        case OpType::Argmax: {
          if (pairs[ni].empty()) break;
          std::vector<std::pair<int64_t, int64_t>> v;
          for (const Pair& p : pairs[ni])
            v.push_back({range[in][p.e].lo - p.T, range[in][p.e].hi - p.T});
          int k, bf;
          chain_bits(v, &k, &bf);
          const int cell = k > 0 ? 64 - std::min(k, 5) : 64 - bf;
          vmax[in] = std::min(vmax[in], vfrac * allowed(cell, scale[in]));
          break;
        }
        case OpType::Activation: {
          vmax[in] = std::min(vmax[in], vfrac * allowed(act_cell(range[in]), scale[in]));
          break;
        }
      }
    }

    // forward: buffers, variances and code
    P.opt = o;
    P.levels = o.levels;
    int64_t in_off = 0;
    for (size_t gi = 0; gi < g.inputs.size(); ++gi) {
      const std::string& n = g.inputs[gi];
      const int t = tensor(n);
      const InputSpec* sp = spec_of(gi);
      buf[t] = new_buf((int64_t)range[t].size(), n);
      const double ls = sp && sp->log2_sigma > 0 ? sp->log2_sigma : o.log2_fresh;
      const double s = std::exp2(ls);
      var[t] = s * s;
      TensorIO io;
      io.name = n;
      io.buf = buf[t];
      io.elems = (int64_t)range[t].size();
      io.scale = scale[t];
      io.log2_sigma = ls;
      io.lo = sp && sp->ranged ? sp->lo : o.input_lo;
      io.hi = sp && sp->ranged ? sp->hi : o.input_hi;
      P.inputs.push_back(io);
      in_off += io.elems;
      if (var[t] > vmax[t])
        fail("graph input '" + n + "': noise 2^" + std::to_string(ls) + " at scale 2^" +
             std::to_string(scale[t]) + " exceeds what its consumers tolerate (2^" +
             std::to_string(0.5 * std::log2(vmax[t])) + ")");
    }
    P.input_elems = in_off;
    std::ostringstream rep;
    for (size_t ni = 0; ni < g.nodes.size(); ++ni)
      emit_node((int)ni, pairs[ni], bases[ni], rep);
    int64_t out_off = 0;
    for (const auto& n : g.outputs) {
      const int t = tensor(n);
      if (buf[t] < 0) fail("graph output '" + n + "' is never produced");
      TensorIO io;
      io.name = n;
      io.buf = buf[t];
      io.elems = (int64_t)range[t].size();
      io.scale = scale[t];
      io.log2_sigma = 0.5 * std::log2(std::max(var[t], 1.0));
      io.lo = INT64_MAX;
      io.hi = INT64_MIN;
      for (const auto& r : range[t]) {
        io.lo = std::min(io.lo, r.lo);
        io.hi = std::max(io.hi, r.hi);
      }
      P.outputs.push_back(io);
      out_off += io.elems;
      if (var[t] > vmax[t] * 1.0000001)
        fail("output '" + n + "' noise (2^" + std::to_string(io.log2_sigma) +
             ") is too large to decode at scale 2^" + std::to_string(scale[t]));
    }
    P.output_elems = out_off;
    rep << "bootstraps per sample: " << P.pbs_per_sample << " (cost " << P.cost_per_sample
        << " single-level equivalents)";
    for (size_t l = 0; l < per_level.size(); ++l)
      if (per_level[l])
        rep << (l ? ", " : "; ") << "(2^" << o.levels[l].base_log << "," << o.levels[l].level
            << "): " << per_level[l];
    rep << "\n";
    P.report = rep.str();
  }

  static int act_cell(const std::vector<Range>& x) {
    int64_t lo = INT64_MAX, hi = INT64_MIN;
    for (const auto& r : x) {
      lo = std::min(lo, r.lo);
      hi = std::max(hi, r.hi);
    }
    const int64_t lo4 = lo >= 0 ? 0 : -((-lo + 3) / 4) * 4;
    const int64_t span = hi - lo4 + 1;
    int lb = 0;
    while ((1ll << lb) < span) ++lb;
    return 63 - lb;
  }

  // key level for the bootstrap that produces tensor t as a sum of `terms` outputs
  int out_level(int t, int terms, const std::string& who) {
    for (int l : lvl_order)
      if (terms * lvar(l) <= vmax[t]) return l;
    fail("node '" + who + "': no key set is precise enough for its consumers (need output "
         "noise below 2^" + std::to_string(0.5 * std::log2(vmax[t] / terms)) + ")");
  }

  void emit_node(int ni, const std::vector<Pair>& pairs, const std::vector<int64_t>& base,
                 std::ostringstream& rep) {
    const auto& nd = g.nodes[ni];
    const auto& op = nd.op;
    const int out = tensor(nd.outputs[0]);
    const int in = tensor(nd.inputs[0]);
    const int64_t E = (int64_t)range[out].size();
    buf[out] = new_buf(E, nd.outputs[0]);
    char line[512];
    switch (op.type) {
      case OpType::Linear:
      case OpType::Conv2d:
      case OpType::Pool: {
        if (op.type == OpType::Pool && !op.pool_avg) {
          if (wide_max(range[in])) emit_maxpool_wide(ni, rep);
          else emit_maxpool(ni, rep);
          return;
        }
        Instr I;
        I.kind = Kind::Contract;
        I.dst = buf[out];
        I.src = buf[in];
        I.bias_delta = pow2(scale[in]);
        double w2 = 0;
        if (op.type == OpType::Linear) {
          I.M = (int)op.weights.size();
          I.K = (int)op.weights[0].size();
          I.P = 1;
        } else if (op.type == OpType::Conv2d) {
          const int oh = (op.in_h + 2 * op.padding - op.kernel_h) / op.stride + 1;
          const int ow = (op.in_w + 2 * op.padding - op.kernel_w) / op.stride + 1;
          I.M = (int)op.weights.size();
          I.K = op.in_channels * op.kernel_h * op.kernel_w;
          I.P = oh * ow;
          I.gather.assign((size_t)I.P * I.K, -1);
          for (int oy = 0; oy < oh; ++oy)
            for (int ox = 0; ox < ow; ++ox)
              for (int ic = 0; ic < op.in_channels; ++ic)
                for (int ky = 0; ky < op.kernel_h; ++ky)
                  for (int kx = 0; kx < op.kernel_w; ++kx) {
                    const int iy = oy * op.stride + ky - op.padding;
                    const int ix = ox * op.stride + kx - op.padding;
                    if (iy < 0 || ix < 0 || iy >= op.in_h || ix >= op.in_w) continue;
                    I.gather[(size_t)(oy * ow + ox) * I.K + (ic * op.kernel_h + ky) * op.kernel_w +
                             kx] = ic * op.in_h * op.in_w + iy * op.in_w + ix;
                  }
        } else {
          const int oh = (op.in_h - op.pool_h) / op.stride + 1;
          const int ow = (op.in_w - op.pool_w) / op.stride + 1;
          I.M = 1;
          I.K = op.pool_h * op.pool_w;
          I.P = op.channels * oh * ow;
          I.gather.assign((size_t)I.P * I.K, -1);
          for (int c = 0; c < op.channels; ++c)
            for (int oy = 0; oy < oh; ++oy)
              for (int ox = 0; ox < ow; ++ox)
                for (int ky = 0; ky < op.pool_h; ++ky)
                  for (int kx = 0; kx < op.pool_w; ++kx)
                    I.gather[(size_t)((c * oh + oy) * ow + ox) * I.K + ky * op.pool_w + kx] =
                        c * op.in_h * op.in_w + (oy * op.stride + ky) * op.in_w + ox * op.stride +
                        kx;
          I.W.assign(I.K, 1);
          I.bias.assign(1, 0);
          w2 = I.K;
        }
        if (op.type != OpType::Pool) {
          I.W.resize((size_t)I.M * I.K);
          I.bias = op.bias;
          for (int m = 0; m < I.M; ++m) {
            double s = 0;
            for (int k = 0; k < I.K; ++k) {
              I.W[(size_t)m * I.K + k] = (int8_t)op.weights[m][k];
              s += (double)op.weights[m][k] * op.weights[m][k];
            }
            w2 = std::max(w2, s);
          }
        }
        I.what = nd.name;
        var[out] = var[in] * std::max(w2, 1.0);
        snprintf(line, sizeof line, "%-20s %-10s %d x %d (P=%d) at 2^%d, noise 2^%.1f\n",
                 nd.name.c_str(), op.name(), I.M, I.K, I.P, scale[in],
                 0.5 * std::log2(std::max(var[out], 1.0)));
        rep << line;
        P.code.push_back(std::move(I));
        return;
      }
      case OpType::Add: {
        const int in2 = tensor(nd.inputs[1]);
        if (scale[in] != scale[in2]) fail("internal: Add operands at different scales");
        lin(buf[out], {Term{buf[in], {1}, {}}, Term{buf[in2], {1}, {}}}, {0}, nd.name);
        var[out] = var[in] + var[in2];
        snprintf(line, sizeof line, "%-20s Add at 2^%d\n", nd.name.c_str(), scale[in]);
        rep << line;
        return;
      }
      case OpType::Activation: {
        const auto& X = range[in];
        int64_t lo = INT64_MAX, hi = INT64_MIN;
        for (const auto& r : X) {
          lo = std::min(lo, r.lo);
          hi = std::max(hi, r.hi);
        }
        const int64_t lo4 = lo >= 0 ? 0 : -((-lo + 3) / 4) * 4;
        const int cell = act_cell(X);
        TvSpec s;
        s.lut_len = 1 << (63 - cell);
        for (int c = 0; c < s.lut_len; ++c)
          s.val.push_back(op.lut[(((c + lo4) % 4) + 4) % 4] << scale[out]);
        const double A = allowed(cell, scale[in]);
        if (A < 0 || var[in] > A)
          fail("node '" + nd.name + "': Activation input too noisy for an exact lookup");
        const int lvl = out_level(out, 1, nd.name);
        pbs(buf[out], buf[in], cell - scale[in], (uint64_t)(-lo4) << cell, lvl, {tv(s)}, E,
            nd.name);
        var[out] = lvar(lvl);
        snprintf(line, sizeof line, "%-20s Activation  1 bootstrap/elem, key (%d,%d)\n",
                 nd.name.c_str(), o.levels[lvl].base_log, o.levels[lvl].level);
        rep << line;
        return;
      }
      case OpType::Requant:
      case OpType::Argmax:
        emit_threshold(ni, pairs, base, rep);
        return;
    }
  }

  // Max pooling of a tensor whose values span at most four integers [lo, lo+3] (a 2-bit
  // activation): a pairwise tree, max(a, b) = one 16-entry lookup bootstrap on
  // 4(a - lo) + (b - lo) read at cells of 2^59; inner results carry max - lo at scale 2^57.
  void emit_maxpool(int ni, std::ostringstream& rep) {
    const auto& nd = g.nodes[ni];
    const auto& op = nd.op;
    const int out = tensor(nd.outputs[0]);
    const int in = tensor(nd.inputs[0]);
    const int64_t E = (int64_t)range[out].size();
    const int ex = scale[in], eo = scale[out];
    int64_t lo = INT64_MAX;
    for (const auto& r : range[in]) lo = std::min(lo, r.lo);
    const int oh = (op.in_h - op.pool_h) / op.stride + 1;
    const int ow = (op.in_w - op.pool_w) / op.stride + 1;
    // operand t of output o: (buffer, element map, scale, offset removed?)
    struct Opd {
      int buf;
      std::vector<int32_t> map;  // per output element
      int scale;
      bool leaf;
    };
    std::vector<Opd> ops;
    for (int ky = 0; ky < op.pool_h; ++ky)
      for (int kx = 0; kx < op.pool_w; ++kx) {
        Opd d{buf[in], std::vector<int32_t>(E), ex, true};
        for (int c = 0; c < op.channels; ++c)
          for (int oy = 0; oy < oh; ++oy)
            for (int ox = 0; ox < ow; ++ox)
              d.map[(c * oh + oy) * ow + ox] = c * op.in_h * op.in_w +
                                               (oy * op.stride + ky) * op.in_w + ox * op.stride +
                                               kx;
        ops.push_back(std::move(d));
      }
    const double tmp_lim = 0.9 * allowed(59, 59) / 272.0;  // inner results read with 16 and 4
    int inner = -1;
    for (int l : lvl_order)
      if (lvar(l) <= tmp_lim) {
        inner = l;
        break;
      }
    if (inner < 0) fail("node '" + nd.name + "': no key set is precise enough for max pooling");
    const int fl = out_level(out, 1, nd.name);
    int level_no = 0;
    int64_t pbs_count = 0;
    if (ops.size() == 1) {
      // a 1x1 window: rescale through an identity lookup
      TvSpec sp;
      sp.lut_len = 4;
      for (int v = 0; v < 4; ++v) sp.val.push_back((uint64_t)(v + lo) << eo);
      const int X = new_buf(E, nd.name + ".in");
      lin(X, {Term{ops[0].buf, {(int64_t)pow2(61 - ex)}, ops[0].map}},
          {(uint64_t)0 - ((uint64_t)lo << 61)}, nd.name + ": stage");
      pbs(buf[out], X, 0, 0, fl, {tv(sp)}, E, nd.name + ": identity lookup");
      var[out] = lvar(fl);
      return;
    }
    while (ops.size() > 1) {
      const size_t np = ops.size() / 2;
      const bool last = ops.size() == 2;
      std::vector<Opd> next;
      for (size_t j = 0; j < np; ++j) {
        const Opd& a = ops[2 * j];
        const Opd& b = ops[2 * j + 1];
        const int D = new_buf(E, nd.name + ".pair");
        uint64_t c = 0;
        if (a.leaf) c -= (uint64_t)lo << 61;
        if (b.leaf) c -= (uint64_t)lo << 59;
        lin(D, {Term{a.buf, {(int64_t)pow2(61 - a.scale)}, a.map},
                Term{b.buf, {(int64_t)pow2(59 - b.scale)}, b.map}},
            {c}, nd.name + ": 4a + b");
        TvSpec sp;
        sp.lut_len = 16;
        for (int v = 0; v < 16; ++v) {
          const int m = std::max(v >> 2, v & 3);
          sp.val.push_back(last ? (uint64_t)(m + lo) << eo : (uint64_t)m << 57);
        }
        const int Y = last ? buf[out] : new_buf(E, nd.name + ".max");
        pbs(Y, D, 0, 0, last ? fl : inner, {tv(sp)}, E, nd.name + ": pairwise max");
        pbs_count += E;
        std::vector<int32_t> id(E);
        for (int64_t e = 0; e < E; ++e) id[e] = (int32_t)e;
        next.push_back(Opd{Y, id, 57, false});
      }
      if (ops.size() % 2) next.push_back(ops.back());
      ops = std::move(next);
      ++level_no;
    }
    var[out] = lvar(fl);
    char line[256];
    snprintf(line, sizeof line, "%-20s Pool(max)  %lld bootstraps/elem over %d tree levels, key %s\n",
             nd.name.c_str(), (long long)(pbs_count / std::max<int64_t>(E, 1)), level_no,
             key_name(fl).c_str());
    rep << line;
  }

  // Max pooling of wide values: a pairwise tree, max(a, b) = b + relu(a - b).  The difference d
  // is split LSB first into nd two's-complement digits of 2 bits (the radix split's peeling:
  // each window read through the negacyclic sign and a two-box lookup, once at the running
  // scale to clear the digit and once at 2^59 to form the digit g_i * 2^59); the top window's
  // sign read also emits s * 2^61, s = [d >= 0].  One lookup per digit on g_i 2^59 + s 2^61
  // (eight cells of 2^59) emits s g_i 4^i at the input's scale, and relu(d) is their sum (for
  // d >= 0 the top digit is 0 or 1; for d < 0 every term is 0).  Inner maxima stay at the
  // input's scale.
  void emit_maxpool_wide(int ni, std::ostringstream& rep) {
    const auto& nd = g.nodes[ni];
    const auto& op = nd.op;
    const int out = tensor(nd.outputs[0]);
    const int in = tensor(nd.inputs[0]);
    const int64_t E = (int64_t)range[out].size();
    const int ex = scale[in];
    if (scale[out] != ex) fail("internal: wide max pooling keeps the input's scale");
    int64_t lo, hi;
    span_of(range[in], &lo, &hi);
    const int ndg = (bits_signed(lo - hi, hi - lo) + 1) / 2;  // 2-bit digits of a - b
    if (ex + 2 * ndg > 64) fail("node '" + nd.name + "': no room for the differences' digits");
    const int oh = (op.in_h - op.pool_h) / op.stride + 1;
    const int ow = (op.in_w - op.pool_w) / op.stride + 1;
    struct Opd {
      int buf;
      std::vector<int32_t> map;  // per output element (empty: identity)
      double V;
    };
    std::vector<Opd> ops;
    for (int ky = 0; ky < op.pool_h; ++ky)
      for (int kx = 0; kx < op.pool_w; ++kx) {
        Opd d{buf[in], std::vector<int32_t>(E), var[in]};
        for (int c = 0; c < op.channels; ++c)
          for (int oy = 0; oy < oh; ++oy)
            for (int ox = 0; ox < ow; ++ox)
              d.map[(c * oh + oy) * ow + ox] = c * op.in_h * op.in_w +
                                               (oy * op.stride + ky) * op.in_w + ox * op.stride +
                                               kx;
        ops.push_back(std::move(d));
      }
    const int l0 = lvl_order[0];
    const double v_inner = 0.25 * allowed(62, ex);  // what an inner maximum may carry
    const int64_t pbs_before = P.pbs_per_sample;
    if (ops.size() == 1) {
      lin(buf[out], {Term{ops[0].buf, {1}, ops[0].map}}, {0}, nd.name + ": 1x1 window");
      var[out] = ops[0].V;
      return;
    }
    // scratch, shared by every pair
    const int R = new_buf(E, nd.name + ".d");
    const int Xc = new_buf(E, nd.name + ".clear");
    const int Xb = new_buf(E, nd.name + ".bit");
    const int Yb = new_buf(E, nd.name + ".low");
    const int S = new_buf(E, nd.name + ".sign");
    const int G = new_buf(E * ndg, nd.name + ".digits");
    const int W = new_buf(E * ndg, nd.name + ".terms");
    std::string keys;
    while (ops.size() > 1) {
      const bool last = ops.size() == 2;
      std::vector<Opd> next;
      for (size_t j = 0; j + 1 < ops.size(); j += 2) {
        const Opd& a = ops[j];
        const Opd& b = ops[j + 1];
        const double Vd = a.V + b.V;
        lin(R, {Term{a.buf, {1}, a.map}, Term{b.buf, {-1}, b.map}}, {0}, nd.name + ": a - b");
        Chain c{R, Xc, E, ex, Vd};
        std::vector<int> ws(ndg, 2), lv;
        double Vend = 0, cost = 0;
        if (!eval_windows(c, ws, 64, &lv, &Vend, &cost))
          fail("node '" + nd.name + "': max pooling input too noisy for exact differences");
        for (int i = 0; i < ndg; ++i) {
          const int Ei = ex + 2 * i;
          const int shift = 62 - Ei;
          const bool top = i == ndg - 1;
          std::vector<int32_t> gm(E * ndg, -1);
          for (int64_t e = 0; e < E; ++e) gm[e * ndg + i] = (int32_t)e;
          std::vector<uint64_t> gc(E * ndg, 0);
          for (int64_t e = 0; e < E; ++e) gc[e * ndg + i] = pow2(59);
          pbs(Xb, R, shift, pow2(61), l0, {tv(const_tv(pow2(59)))}, E, nd.name + ": digit sign");
          if (top)
            pbs(S, R, shift, pow2(61), l0, {tv(const_tv(pow2(60)))}, E, nd.name + ": sign of d");
          pbs(Xc, R, shift, pow2(61), lv[2 * i], {tv(const_tv(pow2(Ei)))}, E,
              nd.name + ": clear digit sign");
          lin(R, {Term{R, {1}, {}}, Term{Xc, {1}, {}}}, {(uint64_t)0 - pow2(Ei)},
              nd.name + ": clear top bit");
          TvSpec lb;
          lb.lut_len = 2;
          lb.val = {0, pow2(59)};
          pbs(Yb, R, shift, 0, l0, {tv(lb)}, E, nd.name + ": digit low bit");
          // G[e][i] = (2^59 - Xb) + Yb = g_i 2^59
          if (i == 0) {  // the first digit also clears the other digits' slots
            lin(G, {Term{Xb, {-1}, gm}, Term{Yb, {1}, gm}}, gc, nd.name + ": digit");
          } else {
            std::vector<int32_t> gid(E * ndg);
            for (int64_t q = 0; q < E * ndg; ++q) gid[q] = (int32_t)q;
            lin(G, {Term{G, {1}, gid}, Term{Xb, {-1}, gm}, Term{Yb, {1}, gm}}, gc,
                nd.name + ": digit");
          }
          if (!top) {
            TvSpec lc;
            lc.lut_len = 2;
            lc.val = {0, pow2(Ei)};
            pbs(Xc, R, shift, 0, lv[2 * i + 1], {tv(lc)}, E, nd.name + ": clear low bit");
            lin(R, {Term{R, {1}, {}}, Term{Xc, {-1}, {}}}, {0}, nd.name + ": clear low bit");
          }
        }
        // the terms s g_i 4^i at the input's scale: one lookup per digit on g_i 2^59 + s 2^61;
        // S = (sign read + 2^60) = s 2^61
        std::vector<int32_t> rep_s(E * ndg);
        for (int64_t q = 0; q < E * ndg; ++q) rep_s[q] = (int32_t)(q / ndg);
        lin(G, {Term{G, {1}, {}}, Term{S, {1}, rep_s}}, {pow2(60)}, nd.name + ": digit + sign");
        const double v_target = last ? vmax[out] : v_inner;
        int lt = -1;
        for (int l : lvl_order)
          if (b.V + ndg * lvar(l) <= 0.9 * v_target) {
            lt = l;
            break;
          }
        if (lt < 0) fail("node '" + nd.name + "': no key set is precise enough for max pooling");
        std::vector<int32_t> tvi(E * ndg);
        std::vector<int> tv_of(ndg);
        for (int i = 0; i < ndg; ++i) {
          TvSpec sp;
          sp.lut_len = 16;
          for (int v = 0; v < 16; ++v) {
            const int gdig = v & 3, sbit = (v >> 2) & 1;
            sp.val.push_back(v < 8 && sbit ? ((uint64_t)gdig << (2 * i)) << ex : 0);
          }
          tv_of[i] = tv(sp);
        }
        for (int64_t q = 0; q < E * ndg; ++q) tvi[q] = tv_of[q % ndg];
        pbs(W, G, 0, 0, lt, tvi, E * ndg, nd.name + ": s * digit");
        // max = b + sum of terms, into a fresh buffer (or the output)
        const int Y = last ? buf[out] : new_buf(E, nd.name + ".max");
        for (int i0 = 0; i0 < ndg; i0 += 2) {
          std::vector<Term> terms;
          terms.push_back(i0 == 0 ? Term{b.buf, {1}, b.map} : Term{Y, {1}, {}});
          for (int i = i0; i < std::min(ndg, i0 + 2); ++i) {
            std::vector<int32_t> m(E);
            for (int64_t e = 0; e < E; ++e) m[e] = (int32_t)(e * ndg + i);
            terms.push_back(Term{W, {1}, m});
          }
          lin(Y, terms, {0}, nd.name + ": b + relu(a - b)");
        }
        keys = key_name(lt);
        next.push_back(Opd{Y, {}, b.V + ndg * lvar(lt)});
      }
      if (ops.size() % 2) next.push_back(ops.back());
      ops = std::move(next);
    }
    var[out] = ops[0].V;
    char line[256];
    snprintf(line, sizeof line,
             "%-20s Pool(max)  %lld bootstraps/elem, differences in %d 2-bit digits, terms %s\n",
             nd.name.c_str(), (long long)((P.pbs_per_sample - pbs_before) / std::max<int64_t>(E, 1)),
             ndg, keys.c_str());
    rep << line;
  }

  void emit_threshold(int ni, const std::vector<Pair>& pairs, const std::vector<int64_t>& base,
                      std::ostringstream& rep) {
    const auto& nd = g.nodes[ni];
    const auto& op = nd.op;
    const int out = tensor(nd.outputs[0]);
    const int in = tensor(nd.inputs[0]);
    const int64_t E = (int64_t)range[out].size();
    const int ey = scale[in], ex = scale[out];
    const auto& Y = range[in];
    char line[512];
    std::vector<uint64_t> cst(E);
    for (int64_t e = 0; e < E; ++e) cst[e] = (uint64_t)base[e] << ex;
    if (pairs.empty()) {
      lin(buf[out], {}, cst, nd.name + ": constant");
      var[out] = 0;
      snprintf(line, sizeof line, "%-20s %-10s constant (every threshold decided by range)\n",
               nd.name.c_str(), op.name());
      rep << line;
      return;
    }
    int per_elem = 0;
    {
      std::vector<int> c(E, 0);
      for (const Pair& p : pairs) per_elem = std::max(per_elem, ++c[p.e]);
    }

    // ---- candidate 1: chains on v = y - T (y space) ----
    std::vector<std::pair<int64_t, int64_t>> vr;
    for (const Pair& p : pairs) vr.push_back({Y[p.e].lo - p.T, Y[p.e].hi - p.T});
    int ky, bfy;
    chain_bits(vr, &ky, &bfy);
    std::vector<int> lvy;
    double Vy_end = 0, costy = 0;
    std::vector<int> wsy, wsA, wsB;
    const bool y_ok =
        plan_windows(Chain{-1, -1, 0, ey, var[in]}, ky, 64 - bfy, &lvy, &Vy_end, &costy, &wsy);
    const int fl = out_level(out, per_elem, nd.name);
    costy = (costy + o.levels[fl].cost) * pairs.size();

    // ---- candidate 2: z = mult*y + rb with the low `shift` bits removed once ----
    bool z_ok = false;
    double costz = 1e300;
    std::vector<int> zel;  // elements with at least one undecided threshold
    std::vector<int> zidx(E, -1);
    std::vector<int> lvA, lvB;
    int s = 0, kB = 0, bfB = 1;
    bool z_lut = false;
    int64_t qmin = INT64_MAX, qmax = INT64_MIN;
    double VA_end = 0;
    if (op.type == OpType::Requant) {
      bool uniform = true;
      if (!op.shifts.empty())
        for (uint32_t x : op.shifts) uniform = uniform && x == op.shifts[0];
      s = op.shifts.empty() ? (int)op.shift : (int)op.shifts[0];
      for (const Pair& p : pairs)
        if (zidx[p.e] < 0) {
          zidx[p.e] = (int)zel.size();
          zel.push_back(p.e);
        }
      double m2 = 0;
      int64_t zlo = INT64_MAX, zhi = INT64_MIN;
      bool fits = uniform && s < 40;
      for (int e : zel) {
        const uint64_t mult = op.mults.empty() ? op.mult : op.mults[e / op.channel_size];
        const uint64_t rb = op.mults.empty() ? op.round_bias : op.round_biases[e / op.channel_size];
        m2 = std::max(m2, (double)mult * mult);
        const i128 a = (i128)mult * Y[e].lo + rb, b = (i128)mult * Y[e].hi + rb;
        if (a < -((i128)1 << 60) || b > ((i128)1 << 60)) {
          fits = false;
          break;
        }
        zlo = std::min<int64_t>(zlo, (int64_t)a);
        zhi = std::max<int64_t>(zhi, (int64_t)b);
        qmin = std::min(qmin, floor_shift((int64_t)a, s));
        qmax = std::max(qmax, floor_shift((int64_t)b, s));
      }
      if (fits && bits_signed(zlo, zhi) <= 63 - ey) {
        std::vector<std::pair<int64_t, int64_t>> qr;
        for (const Pair& p : pairs) {
          const uint64_t mult = op.mults.empty() ? op.mult : op.mults[p.e / op.channel_size];
          const uint64_t rb =
              op.mults.empty() ? op.round_bias : op.round_biases[p.e / op.channel_size];
          qr.push_back({floor_shift((int64_t)((i128)mult * Y[p.e].lo + rb), s) - p.j,
                        floor_shift((int64_t)((i128)mult * Y[p.e].hi + rb), s) - p.j});
        }
        int lut_cell = 59;
        if (qmax - qmin + 1 <= 16) {
          int lb = 0;
          while ((1ll << lb) < qmax - qmin + 1) ++lb;
          lut_cell = 63 - lb;
          z_lut = lut_cell >= ey + s;
        }
        if (!z_lut) {
          chain_bits(qr, &kB, &bfB);
        }
        const int cellA = z_lut ? lut_cell : (kB > 0 ? 64 - std::min(kB, 5) : 64 - bfB);
        double costA = 0;
        if (plan_windows(Chain{-1, -1, 0, ey, m2 * var[in]}, s, cellA, &lvA, &VA_end, &costA,
                         &wsA)) {
          if (z_lut) {
            const int lz = out_level(out, 1, nd.name);
            costz = (costA + o.levels[lz].cost) * zel.size();
            z_ok = true;
          } else {
            double VB_end = 0, costB = 0;
            if (plan_windows(Chain{-1, -1, 0, ey + s, VA_end}, kB, 64 - bfB, &lvB, &VB_end,
                             &costB, &wsB)) {
              costz = costA * zel.size() + (costB + o.levels[fl].cost) * pairs.size();
              z_ok = true;
            }
          }
        }
      }
    }
    if (!y_ok && !z_ok)
      fail("node '" + nd.name + "': no exact plan; the accumulator at scale 2^" +
           std::to_string(ey) + " carries noise 2^" +
           std::to_string(0.5 * std::log2(var[in])) + " against a range of " +
           std::to_string(ky + bfy) + " bits");

    const bool use_z = z_ok && (!y_ok || costz < costy);
    const int per_tv = -1;
    (void)per_tv;
    if (use_z) {
      const int64_t nz = (int64_t)zel.size();
      const int RA = new_buf(nz, nd.name + ".z");
      const int XA = new_buf(nz, nd.name + ".z.pbs");
      std::vector<int64_t> coef(nz);
      std::vector<int32_t> map(nz);
      std::vector<uint64_t> c(nz);
      double m2 = 0;
      for (int64_t i = 0; i < nz; ++i) {
        const int e = zel[i];
        const uint64_t mult = op.mults.empty() ? op.mult : op.mults[e / op.channel_size];
        const uint64_t rb = op.mults.empty() ? op.round_bias : op.round_biases[e / op.channel_size];
        coef[i] = (int64_t)mult;
        map[i] = e;
        c[i] = rb << ey;
        m2 = std::max(m2, (double)mult * mult);
      }
      lin(RA, {Term{buf[in], coef, map}}, c, nd.name + ": z = mult*y + rb");
      Chain ch{RA, XA, nz, ey, m2 * var[in]};
      emit_windows(ch, wsA, lvA, nd.name + " (z)");
      if (z_lut) {
        // q = z >> shift sits at scale 2^(ey+s): one lookup gives the whole output
        int lb = 0;
        while ((1ll << lb) < qmax - qmin + 1) ++lb;
        const int cell = 63 - lb;
        const int lz = out_level(out, 1, nd.name);
        std::map<int64_t, int> tv_of_c0;
        std::vector<int32_t> tvi(nz);
        const int64_t M = (1 << op.out_bits) - 1;
        for (int64_t i = 0; i < nz; ++i) {
          const int e = zel[i];
          const uint64_t rb = op.mults.empty() ? op.round_bias : op.round_biases[e / op.channel_size];
          const int64_t c0 = (int64_t)std::min<uint64_t>(rb >> s, (uint64_t)M);
          auto it = tv_of_c0.find(c0);
          if (it == tv_of_c0.end()) {
            TvSpec sp;
            sp.lut_len = 1 << lb;
            for (int q = 0; q < sp.lut_len; ++q) {
              const int64_t qq = std::min<int64_t>(std::max<int64_t>(q + qmin, c0), M);
              sp.val.push_back(op.clamp_lut[qq] << ex);
            }
            it = tv_of_c0.emplace(c0, tv(sp)).first;
          }
          tvi[i] = it->second;
        }
        const int X = XA;
        pbs(X, RA, cell - (ey + s), (uint64_t)(-qmin) << cell, lz, tvi, nz,
            nd.name + ": clamp lookup");
        std::vector<int32_t> omap(E, -1);
        for (int64_t i = 0; i < nz; ++i) {
          omap[zel[i]] = (int32_t)i;
          cst[zel[i]] = 0;
        }
        lin(buf[out], {Term{X, {1}, omap}}, cst, nd.name + ": assemble");
        var[out] = lvar(lz);
        snprintf(line, sizeof line,
                 "%-20s Requant    z-space: %zu elems remove %d bits (%zu bootstraps) + 1 lookup "
                 "key (%d,%d)\n",
                 nd.name.c_str(), zel.size(), s, lvA.size(), o.levels[lz].base_log,
                 o.levels[lz].level);
        rep << line;
        return;
      }
      // split into (threshold, element) pairs: v = q - j at scale 2^(ey+s)
      const int64_t np = (int64_t)pairs.size();
      const int RB = new_buf(np, nd.name + ".q");
      const int XB = new_buf(np, nd.name + ".q.pbs");
      std::vector<int32_t> pm(np);
      std::vector<uint64_t> pc(np);
      for (int64_t p = 0; p < np; ++p) {
        pm[p] = zidx[pairs[p].e];
        pc[p] = (uint64_t)0 - ((uint64_t)pairs[p].j << (ey + s));
      }
      lin(RB, {Term{RA, {1}, pm}}, pc, nd.name + ": per threshold");
      Chain cb{RB, XB, np, ey + s, ch.V};
      emit_windows(cb, wsB, lvB, nd.name + " (q)");
      const std::string fin = finish_pairs(cb, bfB, pairs, out, cst, fl, nd.name, ni);
      snprintf(line, sizeof line,
               "%-20s Requant    z-space: %zu elems remove %d bits, %zu pairs remove %d more "
               "(%zu+%zu bootstraps), %s\n",
               nd.name.c_str(), zel.size(), s, pairs.size(), kB, lvA.size(), lvB.size() + 1,
               fin.c_str());
      rep << line;
      return;
    }
    const int64_t np = (int64_t)pairs.size();
    const int R = new_buf(np, nd.name + ".v");
    const int Xv = new_buf(np, nd.name + ".v.pbs");
    std::vector<int32_t> pm(np);
    std::vector<uint64_t> pc(np);
    for (int64_t p = 0; p < np; ++p) {
      pm[p] = pairs[p].e;
      pc[p] = (uint64_t)0 - ((uint64_t)pairs[p].T << ey);
    }
    lin(R, {Term{buf[in], {1}, pm}}, pc, nd.name + ": v = y - T");
    Chain c{R, Xv, np, ey, var[in]};
    emit_windows(c, wsy, lvy, nd.name);
    const std::string fin = finish_pairs(c, bfy, pairs, out, cst, fl, nd.name, ni);
    std::string levels;
    for (int l : lvy) levels += key_name(l);
    snprintf(line, sizeof line, "%-20s %-10s y-space: %zu pairs remove %d bits [%s], %s\n",
             nd.name.c_str(), op.name(), pairs.size(), ky, levels.c_str(), fin.c_str());
    rep << line;
  }

  // ---- radix conversion ------------------------------------------------------------
  void setup_levels() {
    for (size_t i = 0; i < o.levels.size(); ++i) lvl_order.push_back((int)i);
    std::sort(lvl_order.begin(), lvl_order.end(),
              [&](int a, int b) { return o.levels[a].cost < o.levels[b].cost; });
    if (o.levels.empty()) fail("no bootstrap key sets given");
    V_ksms = std::exp2(2 * o.log2_ksms);
    P.opt = o;
    P.levels = o.levels;
  }

  TensorIO io_of(int b, const std::string& name, int64_t elems, int sc, double v, int64_t lo,
                 int64_t hi) {
    TensorIO io;
    io.name = name;
    io.buf = b;
    io.elems = elems;
    io.scale = sc;
    io.log2_sigma = 0.5 * std::log2(std::max(v, 1.0));
    io.lo = lo;
    io.hi = hi;
    return io;
  }

  // wide -> blocks: LSB-first, every digit's 2-bit window is read twice (its top bit through the
  // negacyclic sign, then the low bit by a two-box lookup); each read runs once at the wide
  // value's scale, whose outputs clear the digit from the running value, and once at the block
  // scale, whose outputs form the block.
  void run_split(const RadixSpec& r) {
    setup_levels();
    const int nb = r.num_blocks, mb = r.msg_bits;
    if (mb != 2) fail("radix split: blocks of " + std::to_string(mb) + " message bits are not "
                      "supported (the reference's blocks carry 2)");
    const int64_t E = r.elems;
    const int eb = 63 - r.msg_bits - r.carry_bits;  // block scale
    const InputSpec& w = r.wide;
    const int width = mb * nb;
    if (r.is_signed ? (w.lo < -((i128)1 << (width - 1)) || w.hi >= ((i128)1 << (width - 1)))
                    : (w.lo < 0 || w.hi >= ((i128)1 << width)))
      fail("radix split: values in [" + std::to_string(w.lo) + ", " + std::to_string(w.hi) +
           "] do not fit " + std::to_string(nb) + (r.is_signed ? " signed" : " unsigned") +
           " 2-bit blocks");
    const int s_in = w.scale;
    if (s_in < 1 || s_in + width > 64)
      fail("radix split: input scale 2^" + std::to_string(s_in) + " leaves no room for " +
           std::to_string(width) + " bits");
    const double v_in = std::exp2(2 * (w.log2_sigma > 0 ? w.log2_sigma : o.log2_fresh));
    // key sets of the clearing reads: every read of window i must see noise below its budget
    Chain c{-1, -1, E, s_in, v_in};
    std::vector<int> ws(nb, 2), lv;
    double Vend = 0, cost = 0;
    if (!eval_windows(c, ws, 64, &lv, &Vend, &cost))
      fail("radix split: the input's noise (2^" + std::to_string(0.5 * std::log2(v_in)) +
           ") at scale 2^" + std::to_string(s_in) + " is too large to read its digits exactly");
    const int l0 = lvl_order[0];
    // block outputs are read by the reference's own bootstraps: keep them well inside a cell
    const double blk_lim = std::pow(std::ldexp(1.0, eb - 1) / o.z, 2);
    if (2 * lvar(l0) > blk_lim) fail("radix split: the cheapest key set is too noisy for blocks");
    const int IN = new_buf(E, "wide");
    const int R = new_buf(E, "running");
    const int Xc = new_buf(E, "clear");
    const int Xb = new_buf(E, "block bit");
    const int Yb = new_buf(E, "block low bit");
    const int OUT = new_buf(E * nb, "blocks");
    P.inputs.push_back(io_of(IN, "wide", E, s_in, v_in, w.lo, w.hi));
    lin(R, {Term{IN, {1}, {}}}, {0}, "split: running value");
    double V = v_in;
    for (int i = 0; i < nb; ++i) {
      const int Ei = s_in + 2 * i;
      const int shift = 62 - Ei;
      const bool top = i == nb - 1;
      const std::string at = "digit " + std::to_string(i);
      // top bit of the window: +C (0) or -C (1) at the running scale and at the block scale
      pbs(Xc, R, shift, pow2(61), lv[2 * i], {tv(const_tv(pow2(Ei)))}, E, at + ": sign (clear)");
      pbs(Xb, R, shift, pow2(61), l0, {tv(const_tv(pow2(eb)))}, E, at + ": sign (block)");
      lin(R, {Term{R, {1}, {}}, Term{Xc, {1}, {}}}, {(uint64_t)0 - pow2(Ei)}, at + ": clear top");
      V += lvar(lv[2 * i]);
      // low bit of the window
      TvSpec lb;
      lb.lut_len = 2;
      lb.val = {0, pow2(eb)};
      pbs(Yb, R, shift, 0, l0, {tv(lb)}, E, at + ": low bit (block)");
      // block i = (2^eb - Xb) + Yb = (2 b1 + b0) 2^eb
      std::vector<int32_t> map(E * nb, -1);
      for (int64_t e = 0; e < E; ++e) map[e * nb + i] = (int32_t)e;
      std::vector<uint64_t> cst(E * nb, 0);
      for (int64_t e = 0; e < E; ++e) cst[e * nb + i] = pow2(eb);
      if (i == 0) {
        lin(OUT, {Term{Xb, {-1}, map}, Term{Yb, {1}, map}}, cst, at + ": block");
      } else {
        std::vector<int32_t> id(E * nb);
        for (int64_t q = 0; q < E * nb; ++q) id[q] = (int32_t)q;
        lin(OUT, {Term{OUT, {1}, id}, Term{Xb, {-1}, map}, Term{Yb, {1}, map}}, cst,
            at + ": block");
      }
      if (!top) {
        TvSpec lc;
        lc.lut_len = 2;
        lc.val = {0, pow2(Ei)};
        pbs(Xc, R, shift, 0, lv[2 * i + 1], {tv(lc)}, E, at + ": low bit (clear)");
        lin(R, {Term{R, {1}, {}}, Term{Xc, {-1}, {}}}, {0}, at + ": clear low");
        V += lvar(lv[2 * i + 1]);
      }
    }
    P.input_elems = E;
    P.outputs.push_back(io_of(OUT, "blocks", E * nb, eb, 2 * lvar(l0), 0, 3));
    P.output_elems = E * nb;
    std::ostringstream rep;
    rep << "radix split: " << E << " integers -> " << nb << " blocks each, "
        << P.pbs_per_sample / std::max<int64_t>(E, 1) << " bootstraps per integer\n";
    P.report = rep.str();
  }

  // blocks -> wide: one lookup per block, d -> its weighted digit at the output scale, summed.
  void run_merge(const RadixSpec& r) {
    setup_levels();
    const int nb = r.num_blocks, mb = r.msg_bits, space = 1 << (r.msg_bits + r.carry_bits);
    const int64_t E = r.elems;
    const int eb = 63 - r.msg_bits - r.carry_bits;
    const int dmax = r.block_max > 0 ? r.block_max : (1 << mb) - 1;
    if (dmax >= space) fail("radix merge: a block holds digits below " + std::to_string(space));
    if ((int64_t)nb * mb > 62) fail("radix merge: too many blocks for a 64-bit torus");
    // value range of the merged integer
    i128 lo = 0, hi = 0;
    for (int i = 0; i < nb; ++i) {
      const i128 wgt = (i128)1 << (mb * i);
      if (r.is_signed && i == nb - 1) {
        lo += -(i128)(1 << (mb - 1)) * wgt;
        hi += (i128)((1 << (mb - 1)) - 1) * wgt;
      } else {
        hi += (i128)dmax * wgt;
      }
    }
    const int cap = 63 - bits_signed(to_i64(lo, "radix merge"), to_i64(hi, "radix merge"));
    const int so = r.wide.scale > 0 ? r.wide.scale : cap;
    if (so > cap)
      fail("radix merge: output scale 2^" + std::to_string(so) + " leaves no room for " +
           std::to_string(nb * mb) + "-bit integers (at most 2^" + std::to_string(cap) + ")");
    double vmax_out = std::pow(std::ldexp(1.0, so - 1) / o.z, 2);
    if (r.wide.log2_sigma > 0) vmax_out = std::min(vmax_out, std::exp2(2 * r.wide.log2_sigma));
    int lvl = -1;
    for (int l : lvl_order)
      if (nb * lvar(l) <= vmax_out) {
        lvl = l;
        break;
      }
    if (lvl < 0)
      fail("radix merge: " + std::to_string(nb) + " blocks sum " + std::to_string(nb) +
           " bootstrap outputs, and no key set keeps that sum below 2^" +
           std::to_string(0.5 * std::log2(vmax_out)) + " (scale 2^" + std::to_string(so) + ")");
    const double v_blk = std::max(std::exp2(2 * o.log2_fresh), lvar(lvl_order[0]));
    if (v_blk > allowed(eb, eb)) fail("radix merge: block noise too large to read");
    const int IN = new_buf(E * nb, "blocks");
    const int X = new_buf(E * nb, "weighted");
    const int OUT = new_buf(E, "wide");
    P.inputs.push_back(io_of(IN, "blocks", E * nb, eb, v_blk, 0, dmax));
    std::vector<int32_t> tvi(E * nb);
    std::vector<int> tv_of(nb);
    for (int i = 0; i < nb; ++i) {
      TvSpec sp;
      sp.lut_len = space;
      const i128 wgt = (i128)1 << (mb * i);
      for (int d = 0; d < space; ++d) {
        i128 v = (i128)d * wgt;
        if (r.is_signed && i == nb - 1) {
          const int dm = d % (1 << mb);
          v = (i128)(dm >= (1 << (mb - 1)) ? dm - (1 << mb) : dm) * wgt;
        }
        sp.val.push_back((uint64_t)(int64_t)v << so);
      }
      tv_of[i] = tv(sp);
    }
    for (int64_t q = 0; q < E * nb; ++q) tvi[q] = tv_of[q % nb];
    pbs(X, IN, 0, 0, lvl, tvi, E * nb, "merge: weighted digits");
    for (int i0 = 0; i0 < nb; i0 += 3) {
      std::vector<Term> terms;
      if (i0 > 0) terms.push_back(Term{OUT, {1}, {}});
      for (int i = i0; i < std::min(nb, i0 + 3); ++i) {
        std::vector<int32_t> map(E);
        for (int64_t e = 0; e < E; ++e) map[e] = (int32_t)(e * nb + i);
        terms.push_back(Term{X, {1}, map});
      }
      lin(OUT, terms, {0}, "merge: sum of blocks");
    }
    P.input_elems = E * nb;
    P.outputs.push_back(io_of(OUT, "wide", E, so, nb * lvar(lvl), (int64_t)lo, (int64_t)hi));
    P.output_elems = E;
    std::ostringstream rep;
    rep << "radix merge: " << nb << " blocks -> 1 integer at 2^" << so << ", " << nb
        << " bootstraps with key " << key_name(lvl) << "\n";
    P.report = rep.str();
  }

  // Final sign read of every pair, then either
  //  (direct)   out = base + sum_j delta_j [v_j >= 0], each sign bootstrap emitting its term at
  //             the output scale with the key the output's consumers need, or
  //  (combined) each sign bootstrap emits a bit at 2^61 with the cheapest key, the bits of an
  //             element are summed into k (the undecided thresholds crossed), and one lookup
  //             bootstrap with the consumers' key emits clamp_lut[k0 + k] -- one precise
  //             bootstrap per element instead of one per threshold.
  std::string key_name(int l) const {
    return "(" + std::to_string(o.levels[l].base_log) + "," + std::to_string(o.levels[l].level) +
           ")";
  }
  // returns a description of the final stage for the plan report
  std::string finish_pairs(const Chain& c, int bf, const std::vector<Pair>& pairs, int out,
                           std::vector<uint64_t>& cst, int fl, const std::string& name, int ni) {
    const int64_t np = (int64_t)pairs.size();
    const int ex = scale[out];
    const int64_t E = (int64_t)cst.size();
    std::vector<std::vector<int32_t>> maps;
    std::vector<int> cnt(E, 0);
    for (int64_t p = 0; p < np; ++p) {
      const int e = pairs[p].e;
      const int t = cnt[e]++;
      if ((int)maps.size() <= t) maps.emplace_back(E, -1);
      maps[t][e] = (int32_t)p;
    }
    const int J = (int)maps.size();
    const auto& op = g.nodes[ni].op;
    // combined form: bits read back at cells of 2^61 (k <= 3 fits four cells)
    int lb = -1, ll = -1;
    int64_t ne = 0;
    for (int64_t e = 0; e < E; ++e) ne += cnt[e] > 0;
    if (op.type == OpType::Requant && J >= 2) {
      lb = pick(0, allowed(61, 61) / J);
      for (int l : lvl_order)
        if (lvar(l) <= vmax[out]) {
          ll = l;
          break;
        }
    }
    const double cost_direct = (double)np * o.levels[fl].cost;
    const double cost_comb = (lb < 0 || ll < 0) ? 1e300
                                                : (double)np * o.levels[lb].cost +
                                                      (double)ne * o.levels[ll].cost;
    const int X = c.X;
    if (cost_comb >= cost_direct) {
      std::vector<int32_t> tvi(np);
      std::map<int64_t, int> tv_of_delta;
      for (int64_t p = 0; p < np; ++p) {
        const int64_t d = pairs[p].delta;
        auto it = tv_of_delta.find(d);
        if (it == tv_of_delta.end())
          it = tv_of_delta.emplace(d, tv(const_tv((uint64_t)d << (ex - 1)))).first;
        tvi[p] = it->second;
        cst[pairs[p].e] += (uint64_t)d << (ex - 1);
      }
      pbs(X, c.R, 64 - bf - c.E, pow2(63 - bf), fl, tvi, np, name + ": final sign");
      std::vector<Term> terms;
      for (auto& m : maps) terms.push_back(Term{X, {1}, m});
      lin(buf[out], terms, cst, name + ": sum of thresholds");
      var[out] = (double)J * lvar(fl);
      return "final signs " + key_name(fl);
    }
    pbs(X, c.R, 64 - bf - c.E, pow2(63 - bf), lb, {tv(const_tv(pow2(60)))}, np,
        name + ": final sign (bit)");
    // S[i] = k_i * 2^61 over the elements with undecided thresholds
    std::vector<int32_t> elem_of(ne), idx_of(E, -1);
    {
      int64_t i = 0;
      for (int64_t e = 0; e < E; ++e)
        if (cnt[e] > 0) {
          idx_of[e] = (int32_t)i;
          elem_of[i++] = (int32_t)e;
        }
    }
    const int S = new_buf(ne, name + ".count");
    const int Y = new_buf(ne, name + ".lookup");
    std::vector<Term> terms;
    for (auto& m : maps) {
      std::vector<int32_t> mi(ne);
      for (int64_t i = 0; i < ne; ++i) mi[i] = m[elem_of[i]];
      terms.push_back(Term{X, {1}, mi});
    }
    std::vector<uint64_t> sc(ne);
    for (int64_t i = 0; i < ne; ++i) sc[i] = (uint64_t)cnt[elem_of[i]] << 60;
    lin(S, terms, sc, name + ": count of thresholds crossed");
    const int64_t M = (1 << op.out_bits) - 1;
    std::map<int64_t, int> tv_of_k0;
    std::vector<int32_t> tvi(ne);
    for (int64_t i = 0; i < ne; ++i) {
      const int64_t k0 = k0s[ni][elem_of[i]];
      auto it = tv_of_k0.find(k0);
      if (it == tv_of_k0.end()) {
        TvSpec sp;
        sp.lut_len = 4;
        for (int k = 0; k < 4; ++k) sp.val.push_back(op.clamp_lut[std::min<int64_t>(k0 + k, M)] << ex);
        it = tv_of_k0.emplace(k0, tv(sp)).first;
      }
      tvi[i] = it->second;
    }
    pbs(Y, S, 0, 0, ll, tvi, ne, name + ": clamp lookup of the count");
    std::vector<uint64_t> oc(E);
    for (int64_t e = 0; e < E; ++e) oc[e] = idx_of[e] >= 0 ? 0 : cst[e];
    lin(buf[out], {Term{Y, {1}, idx_of}}, oc, name + ": assemble");
    var[out] = lvar(ll);
    return "final sign bits " + key_name(lb) + " + one lookup " + key_name(ll);
  }
};

}  // namespace

Program build(const ir::Graph& g, const Options& o) {
  // How much of a chain's first read budget goes to its input (and so how precise the key sets
  // producing that input must be) trades cost between layers: try a few splits, keep the
  // cheapest program.
  Program best;
  bool have = false;
  std::string first_error;
  for (double f : {0.5, 0.6, 0.7, 0.8}) {
    try {
      Builder b(g, o);
      b.vfrac = f;
      b.run();
      if (!have || b.P.cost_per_sample < best.cost_per_sample) {
        best = std::move(b.P);
        have = true;
      }
    } catch (const Error& e) {
      if (first_error.empty()) first_error = e.what();
    }
  }
  if (!have) throw Error(first_error);
  return best;
}

Program build_radix(const RadixSpec& r, const Options& o) {
  static const ir::Graph empty;
  if (r.num_blocks < 1 || r.elems < 1) throw Error("radix program: need blocks and elements");
  Builder b(empty, o);
  if (r.to_blocks) b.run_split(r);
  else b.run_merge(r);
  return std::move(b.P);
}

// ---- noise-free execution ------------------------------------------------------------

static uint64_t tv_eval(const TvSpec& s, int N, int idx2n) {
  // coefficient 0 of X^(-idx) * tv, i.e. tv[idx] (idx < N) or -tv[idx - N]
  const bool neg = idx2n >= N;
  const int i = neg ? idx2n - N : idx2n;
  uint64_t v;
  if (s.lut_len == 0) {
    v = s.val[0];
  } else {
    const int box = N / s.lut_len, half = box / 2;
    const int m = (i + half) / box;
    v = m < s.lut_len ? s.val[m] : (uint64_t)0 - s.val[m - s.lut_len];
  }
  return neg ? (uint64_t)0 - v : v;
}

std::vector<uint64_t> materialize_tv(const TvSpec& s, int N) {
  std::vector<uint64_t> t(N);
  for (int i = 0; i < N; ++i) t[i] = tv_eval(s, N, i);
  return t;
}

void simulate(const Program& prog, const int64_t* inputs, int batch, int64_t* outputs,
              double* min_margin) {
  const int N = prog.opt.N;
  const int lg = (int)std::lround(std::log2(2.0 * N));
  std::vector<std::vector<uint64_t>> B(prog.bufs.size());
  for (size_t i = 0; i < prog.bufs.size(); ++i)
    B[i].assign((size_t)batch * prog.bufs[i].elems, 0);
  int64_t off = 0;
  for (const auto& io : prog.inputs) {
    for (int b = 0; b < batch; ++b)
      for (int64_t e = 0; e < io.elems; ++e)
        B[io.buf][(size_t)b * io.elems + e] =
            (uint64_t)inputs[(size_t)b * prog.input_elems + off + e] << io.scale;
    off += io.elems;
  }
  double margin = 1e300;
  for (const Instr& I : prog.code) {
    const int64_t E = prog.bufs[I.dst].elems;
    std::vector<uint64_t>& D = B[I.dst];
    if (I.kind == Kind::Contract) {
      const int64_t Es = prog.bufs[I.src].elems;
      const std::vector<uint64_t>& S = B[I.src];
      for (int b = 0; b < batch; ++b)
        for (int m = 0; m < I.M; ++m)
          for (int p = 0; p < I.P; ++p) {
            uint64_t acc = (uint64_t)I.bias[m] * I.bias_delta;
            for (int k = 0; k < I.K; ++k) {
              const int64_t src = I.gather.empty() ? k : I.gather[(size_t)p * I.K + k];
              if (src < 0) continue;
              acc += (uint64_t)(int64_t)I.W[(size_t)m * I.K + k] * S[(size_t)b * Es + src];
            }
            D[(size_t)b * E + (size_t)m * I.P + p] = acc;
          }
    } else if (I.kind == Kind::Lin) {
      std::vector<uint64_t> tmp((size_t)batch * E);
      for (int b = 0; b < batch; ++b)
        for (int64_t e = 0; e < E; ++e) {
          uint64_t acc = I.cst.size() == 1 ? I.cst[0] : I.cst[e];
          for (const Term& t : I.terms) {
            const int64_t src = t.map.empty() ? e : t.map[e];
            if (src < 0) continue;
            const int64_t c = t.coef.size() == 1 ? t.coef[0] : t.coef[e];
            acc += (uint64_t)c * B[t.src][(size_t)b * prog.bufs[t.src].elems + src];
          }
          tmp[(size_t)b * E + e] = acc;
        }
      D = std::move(tmp);
    } else {
      const std::vector<uint64_t>& S = B[I.src];
      std::vector<uint64_t> tmp((size_t)batch * E);
      for (int b = 0; b < batch; ++b)
        for (int64_t e = 0; e < E; ++e) {
          const uint64_t ph = (S[(size_t)b * E + e] << I.shift) + I.offset;
          const TvSpec& s = prog.tvs[I.tv.size() == 1 ? I.tv[0] : I.tv[e]];
          const int mod = 2 * N;
          // exact position in units of 2^(64-lg), rounded like the modulus switch
          const double u = std::ldexp((double)ph, -(64 - lg));
          const int idx = (int)(((ph >> (63 - lg)) + 1) >> 1) & (mod - 1);
          const uint64_t v = tv_eval(s, N, idx);
          tmp[(size_t)b * E + e] = v;
          // distance to the nearest index whose output differs
          for (int d = 1; d <= 256; ++d) {
            const int lo = (idx - d + mod) & (mod - 1), hi = (idx + d) & (mod - 1);
            const bool dl = tv_eval(s, N, lo) != v, dh = tv_eval(s, N, hi) != v;
            if (dl || dh) {
              // boundaries at idx -/+ (d - 0.5); measure from the unrounded position
              double frac = u - std::floor(u / mod) * mod - idx;
              if (frac > mod / 2) frac -= mod;
              if (frac < -mod / 2) frac += mod;
              double m = 1e300;
              if (dl) m = std::min(m, (d - 0.5) + frac);
              if (dh) m = std::min(m, (d - 0.5) - frac);
              margin = std::min(margin, m);
              break;
            }
          }
        }
      D = std::move(tmp);
    }
  }
  off = 0;
  for (const auto& io : prog.outputs) {
    for (int b = 0; b < batch; ++b)
      for (int64_t e = 0; e < io.elems; ++e) {
        const uint64_t ph = B[io.buf][(size_t)b * io.elems + e];
        // signed rounding decode at scale 2^scale
        const int64_t v = (int64_t)(ph + (io.scale > 0 ? ((uint64_t)1 << (io.scale - 1)) : 0)) >>
                          io.scale;
        outputs[(size_t)b * prog.output_elems + off + e] = v;
      }
    off += io.elems;
  }
  if (min_margin) *min_margin = margin;
}

}  // namespace plan
}  // namespace pnb
