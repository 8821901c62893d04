// Graph -> sm_100a kernels + host plan. See lower.hpp.
//
// What differs from the reference compiler, by design:
//  * Materialisation (lib/lower/fusion.ml:54-55 gives a buffer to every node
//    with fan-out >= 2). Here an element-wise node owns a buffer only when it
//    is an output; every other use recomputes it inline, and within one kernel
//    the fused expression DAG is hash-consed so a shared node is computed once
//    per element. A Philox normal feeding three consumers is generated once
//    in registers instead of round-tripping through HBM.
//  * Horizontal fusion. Kernel roots that range over the same index space and
//    do not depend on each other's results share one "map-reduce" launch: any
//    number of element-wise stores and flat reductions in one pass (saxpy's r
//    and sum r; the Greeks' four path sums; the cells of a skinny product).
//  * Invariant factoring. A flat add-reduction whose element is c * g(i), with
//    c loop-invariant but dependent on another reduction of the same pass, is
//    accumulated as sum g(i) and multiplied by c after the pass (sum is
//    linear). This is what lets a Grad-produced adjoint, whose seed is a
//    broadcast of the forward sum, join the forward sum's pass. Rounding
//    differs from the interpreter's sequential fold only within tolerance.
//  * Scalar tails. Outputs of one element that only need this pass's results
//    (price = mean * discount, the gradients) are evaluated by the last block
//    after the final fold, not by separate launches.
#include "lower.hpp"

#include <algorithm>
#include <cinttypes>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>
#include <unordered_map>
#include <cctype>
#include <cstdio>
#include <cstdlib>

#include "common.hpp"

namespace ccb {

int dt_size(Dt d) { return (d == DT_F32 || d == DT_I32) ? 4 : (d == DT_BOOL ? 1 : 8); }
const char* dt_name(Dt d) {
  static const char* n[] = {"f32", "f64", "i32", "i64", "bool"};
  return n[d];
}
const char* dt_ctype(Dt d) {
  static const char* n[] = {"float", "double", "int", "long long", "bool"};
  return n[d];
}
static bool is_float(Dt d) { return d == DT_F32 || d == DT_F64; }
static bool is_int(Dt d) { return d == DT_I32 || d == DT_I64; }

struct LowerError : std::runtime_error {
  int code;
  LowerError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
static void bad(const std::string& m) { throw LowerError(CCB_ERR_INVALID, m); }
static void unsupported(const std::string& m) { throw LowerError(CCB_ERR_UNSUPPORTED, m); }

// ===================================================================== parse
static Dt parse_dt(const std::string& s) {
  if (s == "f32") return DT_F32;
  if (s == "f64") return DT_F64;
  if (s == "i32") return DT_I32;
  if (s == "i64") return DT_I64;
  if (s == "bool") return DT_BOOL;
  bad("wire: unknown dtype " + s);
  return DT_F32;
}
static int lookup(const char* const* names, int n, const std::string& s, const char* what) {
  for (int k = 0; k < n; ++k)
    if (s == names[k]) return k;
  bad(std::string("wire: unknown ") + what + " " + s);
  return 0;
}
// Names are one token on the wire, '%', whitespace and control bytes written
// as %XX (two hex digits), the empty name as a lone '%'; decode them back to
// the caller's bytes.
static std::string wire_name(const std::string& s) {
  if (s == "%") return std::string();
  std::string out;
  out.reserve(s.size());
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i] != '%') {
      out += s[i];
      continue;
    }
    auto hex = [&](char c) -> int {
      if (c >= '0' && c <= '9') return c - '0';
      if (c >= 'a' && c <= 'f') return c - 'a' + 10;
      if (c >= 'A' && c <= 'F') return c - 'A' + 10;
      return -1;
    };
    int hi = i + 2 < s.size() ? hex(s[i + 1]) : -1, lo = i + 2 < s.size() ? hex(s[i + 2]) : -1;
    if (hi < 0 || lo < 0) bad("wire: bad %XX escape in name " + s);
    out += (char)(hi * 16 + lo);
    i += 2;
  }
  return out;
}
static const char* const kBin[] = {"add", "sub", "mul", "div", "min", "max", "bit_and", "bit_or", "bit_xor", "shl", "shr"};
static const char* const kUn[] = {"neg", "sqrt", "exp", "log", "abs", "sin", "cos", "erf", "erfinv"};
static const char* const kCmp[] = {"eq", "ne", "lt", "le", "gt", "ge"};
static const char* const kLogic[] = {"and", "or"};
static const char* const kTk[] = {"param", "iota", "map", "map2", "reduce", "scan", "gather", "scatter_add", "matmul", "reshape", "broadcast"};

int parse_graph(const char* text, GGraph& g) {
  try {
    std::istringstream in(text);
    std::string line;
    std::unordered_map<int64_t, int> eidx, tidx;
    bool header = false, ended = false;
    auto E = [&](int64_t id) {
      auto it = eidx.find(id);
      if (it == eidx.end()) bad("wire: unknown expression id " + std::to_string(id));
      return it->second;
    };
    auto T = [&](int64_t id) {
      auto it = tidx.find(id);
      if (it == tidx.end()) bad("wire: unknown tensor id " + std::to_string(id));
      return it->second;
    };
    while (std::getline(in, line)) {
      if (line.empty()) continue;
      std::istringstream ls(line);
      std::string tag;
      ls >> tag;
      if (tag == "ccbgraph") {
        int v = 0;
        ls >> v;
        if (v != 1) bad("wire: unsupported version");
        header = true;
      } else if (tag == "name") {
        ls >> g.name;
        g.name = wire_name(g.name);
      } else if (tag == "opt") {
        std::string key;
        ls >> key;
        if (key == "shard") {
          long long r = -1, w = 0;
          if (!(ls >> r >> w) || w < 1 || w > 32 || r < 0 || r >= w)
            bad("wire: opt shard <rank> <world> needs 0 <= rank < world <= 32");
          g.shard_rank = (int)r;
          g.shard_world = (int)w;
          continue;
        }
        std::string val;
        ls >> val;
        if (key != "matmul") bad("wire: unknown option " + key);
        if (val == "f32") g.matmul = MM_F32;
        else if (val == "tf32") g.matmul = MM_TF32;
        else bad("wire: matmul precision must be f32 or tf32, got " + val);
      } else if (tag == "e") {
        int64_t id;
        std::string dts, kind;
        ls >> id >> dts >> kind;
        GExpr e;
        e.dt = parse_dt(dts);
        if (kind == "const") {
          e.kind = E_CONST;
          std::string v;
          ls >> v;
          if (is_float(e.dt)) {
            uint64_t bits = std::stoull(v, nullptr, 16);
            std::memcpy(&e.f, &bits, 8);
          } else {
            e.i = std::stoll(v);
          }
        } else if (kind == "arg") {
          e.kind = E_ARG;
          ls >> e.i;
        } else if (kind == "index") {
          e.kind = E_INDEX;
        } else if (kind == "binop" || kind == "cmp" || kind == "logic") {
          std::string op;
          int64_t a, b;
          ls >> op >> a >> b;
          e.kind = kind == "binop" ? E_BINOP : (kind == "cmp" ? E_CMP : E_LOGIC);
          e.op = kind == "binop" ? lookup(kBin, 11, op, "binop") : (kind == "cmp" ? lookup(kCmp, 6, op, "cmp") : lookup(kLogic, 2, op, "logic"));
          e.a = E(a);
          e.b = E(b);
        } else if (kind == "unop") {
          std::string op;
          int64_t a;
          ls >> op >> a;
          e.kind = E_UNOP;
          e.op = lookup(kUn, 9, op, "unop");
          e.a = E(a);
        } else if (kind == "not" || kind == "cast") {
          int64_t a;
          ls >> a;
          e.kind = kind == "not" ? E_NOT : E_CAST;
          e.a = E(a);
        } else if (kind == "select") {
          int64_t c, a, b;
          ls >> c >> a >> b;
          e.kind = E_SELECT;
          e.a = E(c);
          e.b = E(a);
          e.c = E(b);
        } else {
          bad("wire: unknown expression kind " + kind);
        }
        if (ls.fail()) bad("wire: malformed line: " + line);
        eidx[id] = (int)g.ex.size();
        g.ex.push_back(e);
      } else if (tag == "t") {
        GTensor t;
        std::string dts, kind;
        int rank = 0;
        ls >> t.uid >> dts >> rank;
        t.dt = parse_dt(dts);
        t.shape.resize(rank);
        t.numel = 1;
        for (int k = 0; k < rank; ++k) {
          ls >> t.shape[k];
          t.numel *= t.shape[k];
        }
        ls >> kind;
        t.kind = lookup(kTk, 11, kind, "tensor kind");
        int64_t a, b, x, y, z, w;
        switch (t.kind) {
          case T_PARAM:
            ls >> t.name;
            t.name = wire_name(t.name);
            break;
          case T_IOTA: break;
          case T_MAP:
            ls >> a >> x >> z;
            t.dep0 = T(a);
            t.arg0 = E(x);
            t.body = E(z);
            break;
          case T_MAP2:
            ls >> a >> b >> x >> y >> z;
            t.dep0 = T(a);
            t.dep1 = T(b);
            t.arg0 = E(x);
            t.arg1 = E(y);
            t.body = E(z);
            break;
          case T_REDUCE:
          case T_SCAN:
            ls >> a >> x >> y >> z >> w;
            t.dep0 = T(a);
            t.arg0 = E(x);
            t.arg1 = E(y);
            t.body = E(z);
            t.init = E(w);
            break;
          case T_GATHER:
          case T_SCATTER:
          case T_MATMUL:
            ls >> a >> b;
            t.dep0 = T(a);
            t.dep1 = T(b);
            break;
          default:
            ls >> a;
            t.dep0 = T(a);
        }
        if (ls.fail()) bad("wire: malformed line: " + line);
        if (t.numel >= (int64_t(1) << 31)) unsupported("tensor of " + std::to_string(t.numel) + " elements: indices are int32");
        tidx[t.uid] = (int)g.ts.size();
        g.ts.push_back(t);
      } else if (tag == "o") {
        std::string nm;
        int64_t id;
        ls >> nm >> id;
        g.outputs.push_back({wire_name(nm), T(id)});
      } else if (tag == "end") {
        ended = true;
      } else {
        bad("wire: bad line: " + line);
      }
    }
    if (!header || !ended) bad("wire: truncated graph text");
  } catch (const LowerError& e) {
    return fail(e.code, e.what());
  } catch (const std::exception& e) {
    return fail(CCB_ERR_INVALID, std::string("wire: ") + e.what());
  }
  return CCB_OK;
}

// ===================================================================== kernel expression IR
// A hash-consed DAG of scalar operations over loads, the loop index and (in
// an epilogue) the final values of the pass's reductions.
// K_CAST with sub = 1: an I32 read as unsigned, to F64. K_FMA: a * b + c in
// one rounding; only made where the exact result is representable (the
// unsigned-word affine forms of fold()), so it equals the unfused chain.
enum KOp { K_CONST, K_INDEX, K_LOAD, K_BIN, K_UN, K_CMP, K_LOGIC, K_NOT, K_SELECT, K_CAST, K_REDVAL, K_CHECK, K_ARG, K_FMA };

struct KN {
  int op = K_CONST;
  Dt dt = DT_I32;
  int a = -1, b = -1, c = -1;
  int sub = 0;
  double f = 0;
  int64_t iv = 0;
  int buf = -1;
  // properties
  bool late = false;     // depends on a reduction of this pass (epilogue only)
  bool variant = false;  // depends on the loop index
  bool ranged = false;   // integer value range known
  int64_t lo = 0, hi = 0;
};

struct KCtx {
  std::vector<KN> n;
  std::unordered_map<std::string, int> hc;
  int64_t ilo = 0, ihi = 0;
  int index_node = -1;

  static std::string key(const KN& k) {
    char buf[200];
    uint64_t fb;
    std::memcpy(&fb, &k.f, 8);
    snprintf(buf, sizeof buf, "%d|%d|%d|%d|%d|%d|%" PRIx64 "|%" PRId64 "|%d", k.op, (int)k.dt, k.a, k.b, k.c, k.sub, fb, k.iv, k.buf);
    return buf;
  }

  int mk(KN k) {
    fold(k);
    if (k.op == K_CONST && is_int(k.dt)) {
      k.ranged = true;
      k.lo = k.hi = k.iv;
    }
    std::string ky = key(k);
    auto it = hc.find(ky);
    if (it != hc.end()) return it->second;
    props(k);
    if (k.ranged && k.lo == k.hi && k.dt == DT_I32 && k.op != K_CONST) {
      KN c;
      c.op = K_CONST;
      c.dt = DT_I32;
      c.iv = k.lo;
      return mk(c);
    }
    int id = (int)n.size();
    n.push_back(k);
    hc[ky] = id;
    return id;
  }

  int cint(Dt dt, int64_t v) {
    KN k;
    k.op = K_CONST;
    k.dt = dt;
    k.iv = v;
    return mk(k);
  }
  int cfloat(Dt dt, double v) {
    KN k;
    k.op = K_CONST;
    k.dt = dt;
    k.f = dt == DT_F32 ? (double)(float)v : v;
    return mk(k);
  }
  int one(Dt dt) { return is_float(dt) ? cfloat(dt, 1.0) : cint(dt, 1); }
  int index() {
    if (index_node < 0) {
      KN k;
      k.op = K_INDEX;
      k.dt = DT_I32;
      index_node = mk(k);
    }
    return index_node;
  }
  int bin(Dt dt, int op, int a, int b) {
    if (dt == DT_I32 && (op == B_ADD || op == B_SUB || op == B_MUL || op == B_DIV)) {
      const int r = affine_bin(op, a, b);
      if (r >= 0) return r;
    }
    return raw_bin(dt, op, a, b);
  }
  int raw_bin(Dt dt, int op, int a, int b) {
    KN k;
    k.op = K_BIN;
    k.dt = dt;
    k.sub = op;
    k.a = a;
    k.b = b;
    return mk(k);
  }

  // ---- exact affine forms of I32 values
  // An I32 value built from additions, subtractions and constant multiples
  // is kept as sum(c_j * atom_j) + k over "atoms" (nodes of any other kind),
  // in ascending atom order, so every spelling of the same index arithmetic
  // ((4i+1)/4, i + 2^22 - 2^22, ...) lands on one node. Coefficients wrap
  // modulo 2^32 exactly as the I32 arithmetic they replace. A division by a
  // positive constant is resolved only when value ranges prove it exact:
  // the numerator is non-negative (truncation = floor) and its part that is
  // not a multiple of the divisor stays inside [0, d).
  struct Aff {
    std::vector<std::pair<int, int64_t>> t;  // (atom node, coefficient)
    int64_t k = 0;
  };
  std::unordered_map<int, Aff> aff;  // sum nodes built by affine_build -> form

  static int64_t w32(int64_t v) { return (int64_t)(int32_t)(uint32_t)(uint64_t)v; }
  Aff aff_of(int id) const {
    Aff f;
    if (n[id].op == K_CONST) {
      f.k = n[id].iv;
      return f;
    }
    auto it = aff.find(id);
    if (it != aff.end()) return it->second;
    f.t.push_back({id, 1});
    return f;
  }
  static Aff aff_add(const Aff& a, const Aff& b, int64_t sb) {
    Aff r;
    size_t i = 0, j = 0;
    while (i < a.t.size() || j < b.t.size()) {
      int id;
      int64_t c;
      if (j >= b.t.size() || (i < a.t.size() && a.t[i].first < b.t[j].first)) {
        id = a.t[i].first, c = a.t[i].second, ++i;
      } else if (i >= a.t.size() || b.t[j].first < a.t[i].first) {
        id = b.t[j].first, c = w32(sb * b.t[j].second), ++j;
      } else {
        id = a.t[i].first, c = w32(a.t[i].second + sb * b.t[j].second), ++i, ++j;
      }
      if (c != 0) r.t.push_back({id, c});
    }
    r.k = w32(a.k + sb * b.k);
    return r;
  }
  static Aff aff_scale(const Aff& a, int64_t c) {
    Aff r;
    c = w32(c);
    if (c == 0) return r;
    for (auto& tm : a.t) {
      const int64_t v = w32(tm.second * c);
      if (v) r.t.push_back({tm.first, v});
    }
    r.k = w32(a.k * c);
    return r;
  }
  // The exact (unwrapped) range of the form's value, when every atom is ranged.
  bool aff_range(const Aff& f, int64_t& lo, int64_t& hi) const {
    lo = hi = f.k;
    for (auto& tm : f.t) {
      const KN& x = n[tm.first];
      if (!x.ranged) return false;
      const int64_t c = tm.second, e1 = c * x.lo, e2 = c * x.hi;
      lo += std::min(e1, e2);
      hi += std::max(e1, e2);
      if (lo < -(int64_t(1) << 40) || hi > (int64_t(1) << 40)) return false;
    }
    return true;
  }
  int affine_build(const Aff& f) {
    if (f.t.empty()) return cint(DT_I32, f.k);
    if (f.t.size() == 1 && f.t[0].second == 1 && f.k == 0) return f.t[0].first;
    int acc = -1;
    for (auto& tm : f.t) {
      const int64_t c = tm.second;
      if (c == -1 && acc >= 0) {
        acc = raw_bin(DT_I32, B_SUB, acc, tm.first);
        continue;
      }
      const int term = c == 1 ? tm.first : raw_bin(DT_I32, B_MUL, tm.first, cint(DT_I32, c));
      acc = acc < 0 ? term : raw_bin(DT_I32, B_ADD, acc, term);
    }
    if (f.k > 0 || f.k == INT32_MIN) acc = raw_bin(DT_I32, B_ADD, acc, cint(DT_I32, f.k));
    else if (f.k < 0) acc = raw_bin(DT_I32, B_SUB, acc, cint(DT_I32, -f.k));
    if (n[acc].op != K_CONST) aff[acc] = f;
    return acc;
  }
  int affine_bin(int op, int a, int b) {
    const Aff fa = aff_of(a), fb = aff_of(b);
    const bool ca = fa.t.empty(), cb = fb.t.empty();
    if (ca && cb) return -1;  // constant folding
    switch (op) {
      case B_ADD: return affine_build(aff_add(fa, fb, 1));
      case B_SUB: return affine_build(aff_add(fa, fb, -1));
      case B_MUL:
        if (ca) return affine_build(aff_scale(fb, fa.k));
        if (cb) return affine_build(aff_scale(fa, fb.k));
        return -1;
      case B_DIV: {
        if (!cb || fb.k <= 0) return -1;
        const int64_t d = fb.k;
        int64_t lo, hi;
        if (!aff_range(fa, lo, hi) || lo < 0 || hi > INT32_MAX) return -1;
        Aff y, rest;
        for (auto& tm : fa.t) {
          if (tm.second % d == 0) y.t.push_back({tm.first, tm.second / d});
          else rest.t.push_back(tm);
        }
        const int64_t q = fa.k >= 0 ? fa.k / d : -((-fa.k + d - 1) / d);
        rest.k = fa.k - q * d;  // in [0, d)
        int64_t rlo, rhi;
        if (!aff_range(rest, rlo, rhi) || rlo < 0 || rhi >= d) return -1;
        y.k = q;
        return affine_build(y);
      }
      default: return -1;
    }
  }
  int un(Dt dt, int op, int a) {
    KN k;
    k.op = K_UN;
    k.dt = dt;
    k.sub = op;
    k.a = a;
    return mk(k);
  }
  int load(Dt dt, int buf, int idx) {
    KN k;
    k.op = K_LOAD;
    k.dt = dt;
    k.buf = buf;
    k.a = idx;
    return mk(k);
  }

 private:
  static int64_t wrap(Dt dt, int64_t v) { return dt == DT_I32 ? (int64_t)(int32_t)(uint32_t)(uint64_t)v : v; }

  // Rng turns its I32 word into a float by reading it as unsigned through a
  // select on the sign (w < 0 ? double(w) + 2^32 : double(w)), then
  // (u + 0.5) * 2^-32, and Rng.normal takes 2u - 1 (rng.ml:61-74). Every value
  // of such a chain is U * s + t for the unsigned word U in [0, 2^32), a power
  // of two s and a constant t, and is exact in F64 while its significant bits
  // (from U * s's top bit down to the lowest bit of s and t) number at most
  // 53; each step of the chain then rounds nothing, so the whole chain equals
  // one unsigned conversion and one FMA of U, s and t, bit for bit. The
  // select becomes K_CAST sub 1; each affine step on it becomes K_FMA(U, s, t).
  bool unsigned_affine(int id, int& u, double& s, double& t) const {
    const KN& x = n[id];
    if (x.op == K_CAST && x.dt == DT_F64 && x.sub == 1) {
      u = id, s = 1.0, t = 0.0;
      return true;
    }
    if (x.op == K_CAST && x.dt == DT_F64 && n[x.a].dt == DT_F64) return unsigned_affine(x.a, u, s, t);
    if (x.op == K_FMA && x.dt == DT_F64) {
      u = x.a, s = n[x.b].f, t = n[x.c].f;
      return true;
    }
    return false;
  }
  static bool exact_affine(double s, double t) {
    int es = 0, et = 0;
    if (!(s > 0) || std::frexp(s, &es) != 0.5) return false;  // s a power of two: s = 2^(es - 1)
    const double top = 4294967296.0 * s + std::fabs(t);
    if (!(top < 1e300)) return false;
    int etop = 0;
    std::frexp(top, &etop);
    int low = es - 1;
    if (t != 0) {
      double m = std::frexp(t, &et);  // t = m * 2^et, 0.5 <= |m| < 1
      int lb = et - 53;               // the lowest set bit of t
      for (int i = 0; i < 53 && std::ldexp(m, 53 - i) == std::trunc(std::ldexp(m, 53 - i)); ++i) lb = et - 53 + i;
      low = std::min(low, lb);
    }
    return etop - low <= 53 && low > -1000;
  }
  bool fold_unsigned_word(KN& k) {
    auto cf = [&](int id, double& v) {
      if (id < 0 || n[id].op != K_CONST || n[id].dt != DT_F64) return false;
      v = n[id].f;
      return true;
    };
    if (k.op == K_SELECT) {
      const KN& c = n[k.a];
      if (!(c.op == K_CMP && c.sub == C_LT && n[c.a].dt == DT_I32 && n[c.b].op == K_CONST && n[c.b].iv == 0)) return false;
      const int w = c.a;
      const KN& f = n[k.c];
      if (!(f.op == K_CAST && f.sub == 0 && f.a == w)) return false;
      const KN& g = n[k.b];
      double big = 0;
      if (!(g.op == K_BIN && g.sub == B_ADD && ((g.a == k.c && cf(g.b, big)) || (g.b == k.c && cf(g.a, big))) &&
            big == 4294967296.0))
        return false;
      k = KN();
      k.op = K_CAST;
      k.dt = DT_F64;
      k.a = w;
      k.sub = 1;
      return true;
    }
    if (k.op != K_BIN || (k.sub != B_ADD && k.sub != B_SUB && k.sub != B_MUL)) return false;
    int u = -1;
    double s = 0, t = 0, c = 0;
    bool left = false;
    if (unsigned_affine(k.a, u, s, t) && cf(k.b, c)) left = true;
    else if (!(unsigned_affine(k.b, u, s, t) && cf(k.a, c))) return false;
    double s2 = s, t2 = t;
    if (k.sub == B_ADD) {
      t2 = t + c;
    } else if (k.sub == B_SUB) {
      if (!left) return false;  // c - (U s + t) is not of the form
      t2 = t - c;
    } else {
      int e = 0;
      if (!(c > 0) || std::frexp(c, &e) != 0.5) return false;  // scaling by a power of two only
      s2 = s * c;
      t2 = t * c;
    }
    // t +- c must be exact (the rounding error of the sum, by Knuth's
    // two-sum, is zero), and every value of both forms exact
    if (k.sub != B_MUL) {
      const double b = k.sub == B_ADD ? c : -c;
      const double bv = t2 - t, av = t2 - bv;
      if ((t - av) + (b - bv) != 0.0) return false;
    }
    if (!exact_affine(s2, t2) || !exact_affine(s, t)) return false;
    KN r;
    r.op = K_FMA;
    r.dt = DT_F64;
    r.a = u;
    r.b = cfloat(DT_F64, s2);
    r.c = cfloat(DT_F64, t2);
    k = r;
    return true;
  }

  // Exact integer simplification only (float folding is left to the device
  // compiler, which rounds exactly as the device does), and the exact
  // unsigned-word chains above.
  void fold(KN& k) {
    auto is_c = [&](int id, int64_t v) { return id >= 0 && n[id].op == K_CONST && is_int(n[id].dt) && n[id].iv == v; };
    if (k.op == K_CAST && n[k.a].op == K_CONST && is_int(k.dt) && is_int(n[k.a].dt)) {
      const Dt dt = k.dt;
      const int64_t v = n[k.a].iv;
      k = KN();
      k.op = K_CONST;
      k.dt = dt;
      k.iv = wrap(dt, v);
      return;
    }
    auto is_k = [&](int id) { return id >= 0 && n[id].op == K_CONST && !is_float(n[id].dt); };
    auto to_bool = [&](bool v) {
      k = KN();
      k.op = K_CONST;
      k.dt = DT_BOOL;
      k.iv = v ? 1 : 0;
    };
    if (k.op == K_CMP && is_k(k.a) && is_k(k.b)) {
      const int64_t x = n[k.a].iv, y = n[k.b].iv;
      const int c = k.sub;
      to_bool(c == C_EQ ? x == y : c == C_NE ? x != y : c == C_LT ? x < y : c == C_LE ? x <= y : c == C_GT ? x > y : x >= y);
      return;
    }
    if (k.op == K_NOT && is_k(k.a)) {
      to_bool(n[k.a].iv == 0);
      return;
    }
    if (k.op == K_LOGIC && is_k(k.a) && is_k(k.b)) {
      const bool x = n[k.a].iv != 0, y = n[k.b].iv != 0;
      to_bool(k.sub == 0 ? (x && y) : (x || y));
      return;
    }
    if (k.op == K_SELECT && (is_k(k.a) || k.b == k.c)) {
      const int pick = k.b == k.c ? k.b : (n[k.a].iv != 0 ? k.b : k.c);
      k = n[pick];
      return;
    }
    // one spelling for commuted operands: a+b = b+a and a*b = b*a exactly,
    // in IEEE arithmetic as in wrapping integers
    if (k.op == K_BIN && k.a > k.b &&
        (k.sub == B_ADD || k.sub == B_MUL || (is_int(k.dt) && (k.sub == B_AND || k.sub == B_OR || k.sub == B_XOR))))
      std::swap(k.a, k.b);
    if (k.dt == DT_F64 && fold_unsigned_word(k)) return;
    if (k.op == K_BIN && k.sub == B_MUL && is_float(k.dt)) {  // x * 1.0 == x exactly, NaN and -0 included
      auto one = [&](int id) { return n[id].op == K_CONST && n[id].f == 1.0; };
      if (one(k.a) || one(k.b)) {
        k = n[one(k.a) ? k.b : k.a];
        return;
      }
    }
    if (k.op != K_BIN || !is_int(k.dt)) return;
    if (n[k.a].op == K_CONST && n[k.b].op == K_CONST) {
      const int64_t x = n[k.a].iv, y = n[k.b].iv;
      const uint64_t ux = (uint64_t)x, uy = (uint64_t)y;
      const int bits = k.dt == DT_I32 ? 32 : 64;
      int64_t v;
      bool ok = true;
      switch (k.sub) {
        case B_ADD: v = (int64_t)(ux + uy); break;
        case B_SUB: v = (int64_t)(ux - uy); break;
        case B_MUL: v = (int64_t)(ux * uy); break;
        case B_DIV:
          ok = y != 0 && !(y == -1 && x == (k.dt == DT_I32 ? INT32_MIN : INT64_MIN));
          v = ok ? x / y : 0;
          break;
        case B_MIN: v = x < y ? x : y; break;
        case B_MAX: v = x > y ? x : y; break;
        case B_AND: v = x & y; break;
        case B_OR: v = x | y; break;
        case B_XOR: v = x ^ y; break;
        case B_SHL:
          v = bits == 32 ? (int64_t)(int32_t)((uint32_t)x << (y & 31)) : (int64_t)(ux << (y & 63));
          break;
        case B_SHR:
          v = bits == 32 ? (int64_t)(int32_t)((uint32_t)x >> (y & 31)) : (int64_t)(ux >> (y & 63));
          break;
        default: ok = false; v = 0;
      }
      if (ok) {
        const Dt dt = k.dt;
        k = KN();
        k.op = K_CONST;
        k.dt = dt;
        k.iv = wrap(dt, v);
      }
      return;
    }
    // identities: x+0, x-0, x*1, x^0, x|0, x<<0, x>>0 -> x; x*0, x&0 -> 0
    int keep = -1;
    switch (k.sub) {
      case B_ADD:
      case B_OR:
      case B_XOR:
        if (is_c(k.b, 0)) keep = k.a;
        else if (is_c(k.a, 0)) keep = k.b;
        break;
      case B_SUB:
      case B_SHL:
      case B_SHR:
        if (is_c(k.b, 0)) keep = k.a;
        break;
      case B_MUL:
        if (is_c(k.b, 1)) keep = k.a;
        else if (is_c(k.a, 1)) keep = k.b;
        else if (is_c(k.a, 0) || is_c(k.b, 0)) {
          const Dt dt = k.dt;
          k = KN();
          k.op = K_CONST;
          k.dt = dt;
          return;
        }
        break;
      case B_AND:
        if (is_c(k.a, 0) || is_c(k.b, 0)) {
          const Dt dt = k.dt;
          k = KN();
          k.op = K_CONST;
          k.dt = dt;
          return;
        }
        if (is_c(k.b, -1)) keep = k.a;
        else if (is_c(k.a, -1)) keep = k.b;
        break;
      default: break;
    }
    if (keep >= 0) k = n[keep];
  }

  void props(KN& k) {
    switch (k.op) {
      case K_CONST: break;
      case K_ARG: break;
      case K_INDEX:
        k.variant = true;
        k.ranged = true;
        k.lo = ilo;
        k.hi = ihi;
        break;
      case K_REDVAL: k.late = true; break;
      default: {
        for (int ch : {k.a, k.b, k.c})
          if (ch >= 0) {
            k.late = k.late || n[ch].late;
            k.variant = k.variant || n[ch].variant;
          }
      }
    }
    if (k.op == K_CHECK) {
      const KN& a = n[k.a];
      if (a.ranged && a.lo >= 0 && a.hi < k.iv) {
        k.ranged = true;
        k.lo = a.lo;
        k.hi = a.hi;
      }
    }
    if (k.op == K_BIN && k.dt == DT_I32) {
      const KN& a = n[k.a];
      const KN& b = n[k.b];
      if (a.ranged && b.ranged) {
        int64_t lo = 0, hi = 0;
        bool ok = true;
        switch (k.sub) {
          case B_ADD: lo = a.lo + b.lo; hi = a.hi + b.hi; break;
          case B_SUB: lo = a.lo - b.hi; hi = a.hi - b.lo; break;
          case B_MUL: {
            int64_t c[4] = {a.lo * b.lo, a.lo * b.hi, a.hi * b.lo, a.hi * b.hi};
            lo = *std::min_element(c, c + 4);
            hi = *std::max_element(c, c + 4);
            ok = std::llabs(a.lo) < (1ll << 31) && std::llabs(a.hi) < (1ll << 31) && std::llabs(b.lo) < (1ll << 31) &&
                 std::llabs(b.hi) < (1ll << 31);
            break;
          }
          case B_DIV:
            ok = b.lo == b.hi && b.lo > 0 && a.lo >= 0;
            if (ok) {
              lo = a.lo / b.lo;
              hi = a.hi / b.lo;
            }
            break;
          default: ok = false;
        }
        if (ok && lo >= INT32_MIN && hi <= INT32_MAX) {
          k.ranged = true;
          k.lo = lo;
          k.hi = hi;
        }
      }
    }
  }
};

// ===================================================================== text helpers
static std::string lit(const KN& k) {
  char b[96];
  switch (k.dt) {
    case DT_F32: {
      float v = (float)k.f;
      if (std::isnan(v)) return "__int_as_float(0x7fc00000)";
      if (std::isinf(v)) return v > 0 ? "__int_as_float(0x7f800000)" : "__int_as_float((int)0xff800000)";
      snprintf(b, sizeof b, "(%af)", (double)v);
      return b;
    }
    case DT_F64: {
      double v = k.f;
      if (std::isnan(v)) return "__longlong_as_double(0x7ff8000000000000LL)";
      if (std::isinf(v)) return v > 0 ? "__longlong_as_double(0x7ff0000000000000LL)" : "__longlong_as_double((long long)0xfff0000000000000ULL)";
      snprintf(b, sizeof b, "(%a)", v);
      return b;
    }
    case DT_I32:
      if (k.iv == INT32_MIN) return "(-2147483647 - 1)";
      snprintf(b, sizeof b, "(%" PRId64 ")", k.iv);
      return b;
    case DT_I64:
      if (k.iv == INT64_MIN) return "(-9223372036854775807LL - 1LL)";
      snprintf(b, sizeof b, "(%" PRId64 "LL)", k.iv);
      return b;
    case DT_BOOL: return k.iv ? "true" : "false";
  }
  return "0";
}

// The reference's emitted spellings (lib/backend_cuda/emit.ml:58-159): integer
// add/sub/mul/neg wrap through the unsigned type, shift counts are masked and
// Shr is logical, float math keeps its single-precision name for F32.
static std::string bin_text(Dt dt, int op, const std::string& a, const std::string& b) {
  const bool i32 = dt == DT_I32, i64 = dt == DT_I64;
  const char* u = i32 ? "unsigned int" : "unsigned long long";
  const char* s = i32 ? "int" : "long long";
  auto wrapping = [&](const char* sym) {
    if (i32 || i64) return std::string("((") + s + ")((" + u + ")(" + a + ") " + sym + " (" + u + ")(" + b + ")))";
    return "(" + a + " " + sym + " " + b + ")";
  };
  switch (op) {
    case B_ADD: return wrapping("+");
    case B_SUB: return wrapping("-");
    case B_MUL: return wrapping("*");
    case B_DIV: return "(" + a + " / " + b + ")";
    case B_MIN:
      if (dt == DT_F32) return "fminf(" + a + ", " + b + ")";
      if (dt == DT_F64) return "fmin(" + a + ", " + b + ")";
      return "((" + a + " < " + b + ") ? " + a + " : " + b + ")";
    case B_MAX:
      if (dt == DT_F32) return "fmaxf(" + a + ", " + b + ")";
      if (dt == DT_F64) return "fmax(" + a + ", " + b + ")";
      return "((" + a + " > " + b + ") ? " + a + " : " + b + ")";
    case B_AND: return "(" + a + " & " + b + ")";
    case B_OR: return "(" + a + " | " + b + ")";
    case B_XOR: return "(" + a + " ^ " + b + ")";
    case B_SHL:
    case B_SHR: {
      const char* sym = op == B_SHL ? "<<" : ">>";
      const char* mask = i32 ? "31" : "63";
      return std::string("((") + s + ")((" + u + ")(" + a + ") " + sym + " ((" + b + ") & " + mask + ")))";
    }
  }
  return "0";
}

static std::string neg_text(Dt dt, const std::string& a) {
  if (dt == DT_I32) return "((int)(0u - (unsigned int)(" + a + ")))";
  if (dt == DT_I64) return "((long long)(0ull - (unsigned long long)(" + a + ")))";
  return "(-(" + a + "))";
}

static std::string un_text(Dt dt, int op, const std::string& a) {
  const bool f32 = dt == DT_F32;
  auto m = [&](const char* f, const char* d) { return std::string(f32 ? f : d) + "(" + a + ")"; };
  switch (op) {
    case U_NEG: return neg_text(dt, a);
    case U_SQRT: return m("sqrtf", "sqrt");
    case U_EXP: return m("expf", "exp");
    case U_LOG: return m("logf", "log");
    case U_ABS:
      if (is_float(dt)) return m("fabsf", "fabs");
      return "((" + a + " < 0) ? " + neg_text(dt, a) + " : " + a + ")";
    case U_SIN: return m("sinf", "sin");
    case U_COS: return m("cosf", "cos");
    case U_ERF: return m("erff", "erf");
    case U_ERFINV: return m("erfinvf", "erfinv");
  }
  return "0";
}

// Casts follow the interpreter (cudacaml_backend_interp.ml:198-237): floats
// go to integers through int64 truncation, 64-bit integers reach F32 through
// double, integers narrow by wrapping, booleans are 0/1.
static std::string cast_text(Dt from, Dt to, const std::string& a) {
  if (from == to) return a;
  if (to == DT_BOOL) return "((" + a + ") != 0)";
  if (from == DT_BOOL) {
    if (to == DT_F32) return "((" + a + ") ? 1.0f : 0.0f)";
    if (to == DT_F64) return "((" + a + ") ? 1.0 : 0.0)";
    return std::string("((") + a + ") ? (" + dt_ctype(to) + ")1 : (" + dt_ctype(to) + ")0)";
  }
  if (is_float(from)) {
    if (to == DT_F32) return "((float)(" + a + "))";
    if (to == DT_F64) return "((double)(" + a + "))";
    if (to == DT_I64) return "((long long)(" + a + "))";
    return "((int)(unsigned int)(unsigned long long)(long long)(" + a + "))";
  }
  // integer source
  if (to == DT_F32) return from == DT_I64 ? "((float)(double)(" + a + "))" : "((float)(" + a + "))";
  if (to == DT_F64) return "((double)(" + a + "))";
  if (to == DT_I32) return "((int)(unsigned int)(unsigned long long)(" + a + "))";
  return "((long long)(" + a + "))";
}

static const char* cmp_sym(int op) {
  static const char* s[] = {"==", "!=", "<", "<=", ">", ">="};
  return s[op];
}

// ===================================================================== emitter
struct Emitter {
  const KCtx& c;
  std::ostringstream& o;
  std::string ind = "    ";
  std::string index_text = "i";
  std::string suffix;
  std::unordered_map<int, std::string> name;
  std::unordered_map<int, std::string> direct;  // buffer -> lane expression
  std::unordered_map<int, std::string> direct_node;  // LOAD node -> lane expression
  std::vector<std::string> redval;               // REDVAL slot -> name
  std::string arg_names[2] = {"a", "b"};

  Emitter(const KCtx& cc, std::ostringstream& oo) : c(cc), o(oo) {}

  // I64 value that is the zero extension of an I32 value: text of the I32.
  bool zext32(int id, std::string& out) {
    const KN& k = c.n[id];
    if (k.op == K_CONST && k.dt == DT_I64 && k.iv >= 0 && k.iv <= 0xFFFFFFFFLL) {
      KN t = k;
      t.dt = DT_I32;
      t.iv = (int64_t)(int32_t)(uint32_t)k.iv;
      out = lit(t);
      return true;
    }
    if (k.op == K_BIN && k.sub == B_AND && k.dt == DT_I64) {  // either operand order (AND is commutative)
      for (int s = 0; s < 2; ++s) {
        const int m = s ? k.a : k.b, v = s ? k.b : k.a;
        if (c.n[m].op == K_CONST && c.n[m].iv == 0xFFFFFFFFLL && c.n[v].op == K_CAST && c.n[c.n[v].a].dt == DT_I32) {
          out = val(c.n[v].a);
          return true;
        }
      }
    }
    return false;
  }
  // SHR(MUL(zext a, zext b), 32) in I64
  bool mulhi_operands(int id, std::string& a, std::string& b) {
    const KN& s = c.n[id];
    if (!(s.op == K_BIN && s.sub == B_SHR && s.dt == DT_I64 && c.n[s.b].op == K_CONST && c.n[s.b].iv == 32)) return false;
    const KN& m = c.n[s.a];
    if (!(m.op == K_BIN && m.sub == B_MUL && m.dt == DT_I64)) return false;
    return zext32(m.a, a) && zext32(m.b, b);
  }

  // Philox's mulhilo uses the high and the low word of one 32x32 product:
  // the high word through the __umulhi spelling below, the low word as an I32
  // multiply of the same operands. Such a pair is computed once, as a 64-bit
  // product that both words are read from.
  std::string opkey(int id) const {  // an I32 operand: a constant by value, any other node by id
    const KN& x = c.n[id];
    return x.op == K_CONST ? "c" + std::to_string(x.iv) : "n" + std::to_string(id);
  }
  bool zext32_key(int id, std::string& key) const {
    const KN& k = c.n[id];
    if (k.op == K_CONST && k.dt == DT_I64 && k.iv >= 0 && k.iv <= 0xFFFFFFFFLL) {
      key = "c" + std::to_string((int64_t)(int32_t)(uint32_t)k.iv);
      return true;
    }
    if (k.op == K_BIN && k.sub == B_AND && k.dt == DT_I64)
      for (int s = 0; s < 2; ++s) {
        const int m = s ? k.a : k.b, v = s ? k.b : k.a;
        if (c.n[m].op == K_CONST && c.n[m].iv == 0xFFFFFFFFLL && c.n[v].op == K_CAST && c.n[c.n[v].a].dt == DT_I32) {
          key = opkey(c.n[v].a);
          return true;
        }
      }
    return false;
  }
  static std::string pair_key(std::string a, std::string b) {
    if (b < a) std::swap(a, b);
    return a + "*" + b;
  }
  bool hi_key(int id, std::string& key) const {  // id: the I32 cast of SHR(MUL(zext a, zext b), 32)
    const KN& k = c.n[id];
    if (!(k.op == K_CAST && k.dt == DT_I32 && k.sub == 0)) return false;
    const KN& s = c.n[k.a];
    if (!(s.op == K_BIN && s.sub == B_SHR && s.dt == DT_I64 && c.n[s.b].op == K_CONST && c.n[s.b].iv == 32)) return false;
    const KN& m = c.n[s.a];
    std::string ka, kb;
    if (!(m.op == K_BIN && m.sub == B_MUL && m.dt == DT_I64 && zext32_key(m.a, ka) && zext32_key(m.b, kb))) return false;
    key = pair_key(ka, kb);
    return true;
  }
  bool lo_key(int id, std::string& key) const {
    const KN& k = c.n[id];
    if (!(k.op == K_BIN && k.sub == B_MUL && k.dt == DT_I32)) return false;
    key = pair_key(opkey(k.a), opkey(k.b));
    return true;
  }
  bool scanned = false;
  std::set<std::string> his, los;
  std::unordered_map<std::string, std::string> wide;  // pair -> name of the 64-bit product
  bool paired(const std::string& key) {
    if (!scanned) {
      scanned = true;
      for (int i = 0; i < (int)c.n.size(); ++i) {
        std::string kk;
        if (hi_key(i, kk)) his.insert(kk);
        if (lo_key(i, kk)) los.insert(kk);
      }
    }
    return his.count(key) && los.count(key);
  }
  std::string wide_product(const std::string& key, const std::string& a, const std::string& b) {
    auto it = wide.find(key);
    if (it != wide.end()) return it->second;
    const std::string nm = "w" + std::to_string(wide.size()) + suffix;
    o << ind << "const unsigned long long " << nm << " = (unsigned long long)(unsigned int)(" << a << ") * (unsigned int)(" << b
      << ");\n";
    wide[key] = nm;
    return nm;
  }

  std::string val(int id) {
    auto it = name.find(id);
    if (it != name.end()) return it->second;
    const KN& k = c.n[id];
    std::string e;
    std::string pk;
    if (lo_key(id, pk) && paired(pk)) {
      const std::string a = val(k.a), b = val(k.b);
      e = "((int)(unsigned int)" + wide_product(pk, a, b) + ")";
    } else if (hi_key(id, pk) && paired(pk)) {
      std::string ua, ub;
      mulhi_operands(k.a, ua, ub);
      e = "((int)(" + wide_product(pk, ua, ub) + " >> 32))";
    }
    if (!e.empty()) {
      std::string nm = "v" + std::to_string(id) + suffix;
      o << ind << "const int " << nm << " = " << e << ";\n";
      name[id] = nm;
      return nm;
    }
    switch (k.op) {
      case K_CONST: return lit(k);
      case K_INDEX: return index_text;
      case K_ARG: return arg_names[k.iv];
      case K_REDVAL: return redval.at(k.iv);
      case K_LOAD: {
        auto dn = direct_node.find(id);
        if (dn != direct_node.end()) {
          e = dn->second;
          break;
        }
        auto d = direct.find(k.buf);
        if (d != direct.end() && k.a == c.index_node) {
          e = d->second;
        } else {
          e = "p.b" + std::to_string(k.buf) + "[" + val(k.a) + "]";
        }
        break;
      }
      case K_CHECK:
        e = "ccb::checked_index(" + val(k.a) + ", " + std::to_string(k.iv) + "LL, p.err, ccb::ERR_GATHER_OOB)";
        break;
      case K_BIN: e = bin_text(k.dt, k.sub, val(k.a), val(k.b)); break;
      case K_UN: e = un_text(k.dt, k.sub, val(k.a)); break;
      case K_CMP: e = "(" + val(k.a) + " " + cmp_sym(k.sub) + " " + val(k.b) + ")"; break;
      case K_LOGIC: e = "(" + val(k.a) + (k.sub == 0 ? " && " : " || ") + val(k.b) + ")"; break;
      case K_NOT: e = "(!" + val(k.a) + ")"; break;
      case K_SELECT: e = "(" + val(k.a) + " ? " + val(k.b) + " : " + val(k.c) + ")"; break;
      case K_FMA: e = "fma(" + val(k.a) + ", " + val(k.b) + ", " + val(k.c) + ")"; break;
      case K_CAST: {
        if (k.sub == 1) {  // the word read as unsigned
          e = "((double)(unsigned int)(" + val(k.a) + "))";
          break;
        }
        // (int)(((u64)zext(a) * (u64)zext(b)) >> 32) is the high word of the
        // 32x32 product: spell it __umulhi so it maps to one multiply.
        std::string ua, ub;
        if (k.dt == DT_I32 && mulhi_operands(k.a, ua, ub)) {
          e = "((int)__umulhi((unsigned int)(" + ua + "), (unsigned int)(" + ub + ")))";
          break;
        }
        e = cast_text(c.n[k.a].dt, k.dt, val(k.a));
        break;
      }
    }
    std::string nm = "v" + std::to_string(id) + suffix;
    o << ind << "const " << dt_ctype(k.dt) << " " << nm << " = " << e << ";\n";
    name[id] = nm;
    return nm;
  }
};

// ===================================================================== lowering
namespace {

enum GKind { G_MAPRED, G_SCAN_FLAT, G_SCAN_ROWS, G_RED_ROWS, G_SCATTER, G_MATMUL, G_MATMUL_TC, G_TRANSPOSE };

struct Red {
  int t = -1;           // output tensor
  int64_t elem = 0;     // element of t this accumulator produces
  Dt dt = DT_F32;
  int comb_t = -1;      // tensor whose fn2 is the combiner (-1: plain add)
  int init = -1;        // KNode in the group's ctx (constant)
  int var = -1;         // accumulated element value
  int inv = -1;         // invariant factor applied after the pass (-1: none)
};

struct Group {
  int kind = G_MAPRED;
  int64_t domain = 0;
  KCtx ctx;
  std::vector<std::pair<int, int>> stores;  // (tensor, value KNode)
  std::vector<Red> reds;
  std::vector<std::pair<int, int>> tails;   // (tensor, value KNode)
  int root = -1;
  int val = -1, val2 = -1;  // single-root kinds: source / index KNodes
  int64_t rows = 0, n = 0;  // rows kernels
  int mm_a = -1, mm_b = -1; // matmul operand KNodes (built with INDEX = flat operand index)
  KCtx ctx_b;               // matmul: B operand
  int epi = -1;             // tensor-core product or scan: the map pass run in its stores
  int fused_into = -1;      // map pass / transpose: the group that runs it
  int tstore = -1;          // row scan: the transpose group whose output it writes directly
  int tpost = -1;           // row scan with tstore: the map pass over the transpose it also runs
  int tload = -1;           // row scan whose tstore is a map pass over the inlined transpose: its LOAD node
};

struct JoinFail {};

class Lowerer {
 public:
  const GGraph& g;
  std::vector<int> uses;
  std::vector<char> is_out, mat;
  std::vector<int> group_of;
  std::vector<Group> groups;

  explicit Lowerer(const GGraph& gg) : g(gg) {}

  // A product with a tiny inner dimension (LSM's X . beta, K = 3 or 4) is an
  // element-wise dot product: it fuses into its consumer like a map instead
  // of costing a tiled launch. Ascending k, as both reference backends sum.
  static constexpr int64_t kSmallK = 8;
  bool small_k(int t) const {
    const GTensor& x = g.ts[t];
    return x.kind == T_MATMUL && g.ts[x.dep0].shape.size() == 2 && g.ts[x.dep0].shape[1] <= kSmallK;
  }

  // ------------------------------------------------------------ tensor-core operands
  // An F32 product with enough work runs on the tcgen05 tensor cores. Its
  // operands must then be plain views of buffers: each operand is traced
  // through reshapes and index-affine gathers (Dsl.transpose is one,
  // lib/ir/dsl.ml:167-182) to the tensor it reads, which is materialised,
  // and the trace must end in row-major or transposed order.
  struct TcInfo {
    bool on = false;
    int va = -1, vb = -1;       // tensors read for A and B
    bool a_mn = false, b_mn = false;  // A stored [K][M]; B stored [K][N]
  };
  std::vector<TcInfo> tc;

  // a*r + b*c + k over r in [0,R), c in [0,C).
  struct Aff {
    bool ok = false;
    int64_t a = 0, b = 0, k = 0;
  };
  static void aff_range(const Aff& f, int64_t R, int64_t C, int64_t& lo, int64_t& hi) {
    const int64_t ea = f.a * (R - 1), eb = f.b * (C - 1);
    lo = f.k + std::min<int64_t>(0, ea) + std::min<int64_t>(0, eb);
    hi = f.k + std::max<int64_t>(0, ea) + std::max<int64_t>(0, eb);
  }
  static bool int_dt(Dt d) { return d == DT_I32 || d == DT_I64; }

  // The value of integer element function `e` (Arg 0 and Index bound to
  // `arg`) as an affine form, exact over the whole (r, c) domain, or !ok.
  Aff aff_expr(int e, const Aff& arg, int64_t R, int64_t C, std::unordered_map<int, Aff>& memo) const {
    auto it = memo.find(e);
    if (it != memo.end()) return it->second;
    const GExpr& x = g.ex[e];
    Aff r;
    switch (x.kind) {
      case E_CONST:
        if (int_dt(x.dt)) {
          r.ok = true;
          r.k = x.i;
        }
        break;
      case E_ARG:
        if (x.i == 0) r = arg;
        break;
      case E_INDEX: r = arg; break;
      case E_CAST:
        if (int_dt(x.dt) && int_dt(g.ex[x.a].dt)) r = aff_expr(x.a, arg, R, C, memo);
        break;
      case E_BINOP: {
        if (!int_dt(x.dt)) break;
        const Aff u = aff_expr(x.a, arg, R, C, memo), v = aff_expr(x.b, arg, R, C, memo);
        if (!u.ok || !v.ok) break;
        const bool uc = u.a == 0 && u.b == 0, vc = v.a == 0 && v.b == 0;
        if (x.op == B_ADD) {
          r = {true, u.a + v.a, u.b + v.b, u.k + v.k};
        } else if (x.op == B_SUB) {
          r = {true, u.a - v.a, u.b - v.b, u.k - v.k};
        } else if (x.op == B_MUL && (uc || vc)) {
          r = uc ? Aff{true, v.a * u.k, v.b * u.k, v.k * u.k} : Aff{true, u.a * v.k, u.b * v.k, u.k * v.k};
        } else if (x.op == B_DIV && vc && v.k > 0) {
          // non-negative numerator: truncation is floor; one coordinate must
          // pass through whole and the rest stay inside [0, d)
          const int64_t d = v.k;
          int64_t lo, hi;
          aff_range(u, R, C, lo, hi);
          if (lo < 0) break;
          const Aff ra{true, u.a, 0, u.k}, rb{true, 0, u.b, u.k};
          int64_t l2, h2;
          if (u.a % d == 0 && u.b % d == 0 && u.k >= 0 && u.k < d) {
            r = {true, u.a / d, u.b / d, 0};
          } else if (u.a % d == 0 && (aff_range(rb, R, C, l2, h2), l2 >= 0 && h2 < d)) {
            r = {true, u.a / d, 0, 0};
          } else if (u.b % d == 0 && (aff_range(ra, R, C, l2, h2), l2 >= 0 && h2 < d)) {
            r = {true, 0, u.b / d, 0};
          }
        }
        break;
      }
      default: break;
    }
    if (r.ok) {  // the element arithmetic must not wrap anywhere on the domain
      int64_t lo, hi;
      aff_range(r, R, C, lo, hi);
      const int64_t lim = x.dt == DT_I32 ? (int64_t(1) << 31) : (int64_t(1) << 62);
      if (lo < -lim || hi >= lim) r.ok = false;
    }
    memo[e] = r;
    return r;
  }

  // Trace operand tensor d (element (r, c) of an R x C operand at flat index
  // C*r + c) through reshapes and affine gathers. Returns the tensor reached
  // and, in f, the flat index of (r, c) in it.
  int peel(int d, int64_t R, int64_t C, Aff& f) const {
    f = Aff{true, C, 1, 0};
    for (int guard = 0; guard < 32; ++guard) {
      const GTensor& x = g.ts[d];
      if (mat[d]) return d;
      if (x.kind == T_RESHAPE) {
        d = x.dep0;
        continue;
      }
      if (x.kind != T_GATHER) return d;
      const GTensor& ix = g.ts[x.dep0];
      Aff nf;
      if (ix.kind == T_IOTA) {
        nf = f;
      } else if (ix.kind == T_MAP && g.ts[ix.dep0].kind == T_IOTA && g.ts[ix.dep0].numel == ix.numel) {
        std::unordered_map<int, Aff> memo;
        nf = aff_expr(ix.body, f, R, C, memo);
      }
      if (!nf.ok) return d;
      int64_t lo, hi;
      aff_range(nf, R, C, lo, hi);
      if (lo < 0 || hi >= g.ts[x.dep1].numel) return d;
      f = nf;
      d = x.dep1;
    }
    return d;
  }

  // A materialised gather that is exactly the transpose of a materialised
  // 2-D buffer (the index is affine, (r, c) -> c*R + r over the [R; C]
  // output): it gets a tiled transpose kernel instead of a strided gather.
  bool transpose_of(int t, int& src) const {
    const GTensor& x = g.ts[t];
    if (x.kind != T_GATHER || x.shape.size() != 2 || (dt_size(x.dt) != 4 && dt_size(x.dt) != 8)) return false;
    const int64_t R = x.shape[0], C = x.shape[1];
    if (R < 1 || C < 1) return false;
    const GTensor& ix = g.ts[x.dep0];
    if (!(ix.kind == T_MAP && g.ts[ix.dep0].kind == T_IOTA && g.ts[ix.dep0].numel == ix.numel && ix.numel == x.numel))
      return false;
    std::unordered_map<int, Aff> memo;
    const Aff f = aff_expr(ix.body, Aff{true, C, 1, 0}, R, C, memo);
    if (!f.ok || f.a != 1 || f.b != R || f.k != 0) return false;
    int d = x.dep1;
    while (g.ts[d].kind == T_RESHAPE && !mat[d]) d = g.ts[d].dep0;
    if (!mat[d] || g.ts[d].numel != R * C || g.ts[d].dt != x.dt) return false;
    src = d;
    return true;
  }

  // Work below this (M*N*K) stays on the exact CUDA-core tile kernel.
  static constexpr int64_t kTcMinWork = int64_t(1) << 21;

  void plan_tensor_core() {
    const int T = (int)g.ts.size();
    tc.assign(T, TcInfo());
    if (g.matmul != MM_TF32) return;
    for (int t = 0; t < T; ++t) {
      const GTensor& x = g.ts[t];
      if (x.kind != T_MATMUL || x.dt != DT_F32 || small_k(t)) continue;
      const GTensor &A = g.ts[x.dep0], &Bt = g.ts[x.dep1];
      if (A.dt != DT_F32 || Bt.dt != DT_F32) continue;
      const int64_t M = x.shape[0], N = x.shape[1], K = A.shape[1];
      if (M * N <= 32 && K >= 2048) continue;  // split-K reduction pass
      if (K < 32 || M * N * K < kTcMinWork || M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) ||
          K >= (int64_t(1) << 31))
        continue;
      TcInfo ti;
      Aff fa, fb;
      ti.va = peel(x.dep0, M, K, fa);
      ti.vb = peel(x.dep1, K, N, fb);
      auto is = [](const Aff& f, int64_t a, int64_t b) { return f.ok && f.a == a && f.b == b && f.k == 0; };
      if (g.ts[ti.va].numel != M * K || g.ts[ti.va].dt != DT_F32 || !(is(fa, K, 1) || is(fa, 1, M))) {
        ti.va = x.dep0;
        fa = Aff{true, K, 1, 0};
      }
      if (g.ts[ti.vb].numel != K * N || g.ts[ti.vb].dt != DT_F32 || !(is(fb, N, 1) || is(fb, 1, K))) {
        ti.vb = x.dep1;
        fb = Aff{true, N, 1, 0};
      }
      ti.a_mn = !is(fa, K, 1);
      ti.b_mn = is(fb, N, 1);
      // TMA: every row pitch a multiple of 16 bytes
      if ((ti.a_mn ? M : K) % 4 != 0 || (ti.b_mn ? N : K) % 4 != 0) continue;
      ti.on = true;
      tc[t] = ti;
      mat[ti.va] = 1;
      mat[ti.vb] = 1;
    }
  }

  // A 4-byte product big enough for matmul_tiled128 re-reads every operand
  // element once per 128-wide tile of the other side, so an operand that is
  // an expression (F32-mode MLP: tanh_like(Z1), dZ1 with its exp) is
  // materialised once, like a tensor-core operand: traced through views to
  // the tensor it reads, which is stored, and the trace's order (row-major
  // or transposed) picks the tile load layout.
  struct SimtInfo {
    bool on = false, a_mn = false, b_km = false;
  };
  std::vector<SimtInfo> simt;
  void plan_simt_operands() {
    const int T = (int)g.ts.size();
    simt.assign(T, SimtInfo());
    for (int t = 0; t < T; ++t) {
      const GTensor& x = g.ts[t];
      if (x.kind != T_MATMUL || dt_size(x.dt) != 4 || small_k(t) || tc[t].on) continue;
      const int64_t M = x.shape[0], N = x.shape[1], K = g.ts[x.dep0].shape[1];
      if ((M * N <= 32 && K >= 2048) || M < 128 || N < 128) continue;
      Aff fa, fb;
      const int va = peel(x.dep0, M, K, fa), vb = peel(x.dep1, K, N, fb);
      auto is = [](const Aff& f, int64_t a, int64_t b) { return f.ok && f.a == a && f.b == b && f.k == 0; };
      SimtInfo si;
      si.on = true;
      if (g.ts[va].numel == M * K && g.ts[va].dt == x.dt && (is(fa, K, 1) || is(fa, 1, M))) {
        mat[va] = 1;
        si.a_mn = !is(fa, K, 1);
      } else {
        mat[x.dep0] = 1;
      }
      if (g.ts[vb].numel == K * N && g.ts[vb].dt == x.dt && (is(fb, N, 1) || is(fb, 1, K))) {
        mat[vb] = 1;
        si.b_km = !is(fb, N, 1);
      } else {
        mat[x.dep1] = 1;
      }
      simt[t] = si;
    }
  }

  void analyse() {
    const int T = (int)g.ts.size();
    uses.assign(T, 0);
    is_out.assign(T, 0);
    mat.assign(T, 0);
    group_of.assign(T, -1);
    for (const auto& t : g.ts) {
      if (t.dep0 >= 0) uses[t.dep0]++;
      if (t.dep1 >= 0) uses[t.dep1]++;
    }
    for (auto& o : g.outputs) is_out[o.second] = 1;
    for (int t = 0; t < T; ++t) {
      const GTensor& x = g.ts[t];
      const bool barrier = x.kind == T_REDUCE || x.kind == T_SCAN || x.kind == T_SCATTER ||
                           (x.kind == T_MATMUL && !small_k(t));
      mat[t] = x.kind == T_PARAM || barrier || is_out[t];
      if (mat[t] && x.dt == DT_BOOL) bad("Value.create: Bool tensors are not storable (node n" + std::to_string(x.uid) + ")");
    }
    plan_tensor_core();
    plan_simt_operands();
  }

  // ------------------------------------------------------------ element builder
  struct Build {
    Lowerer* L;
    int gi;
    KCtx* ctx;
    Group* grp;
    std::map<std::pair<int, int>, int> memo;

    int elem(int t, int idx) {
      auto key = std::make_pair(t, idx);
      auto it = memo.find(key);
      if (it != memo.end()) return it->second;
      int r = elem_uncached(t, idx);
      memo[key] = r;
      return r;
    }

    int elem_uncached(int t, int idx) {
      const GTensor& x = L->g.ts[t];
      if (L->mat[t]) {
        const int gt = L->group_of[t];
        if (x.kind == T_PARAM || (gt >= 0 && gt < gi)) return ctx->load(x.dt, t, idx);
        if (gt == gi && gt >= 0) {
          if (x.kind == T_REDUCE || (x.kind == T_MATMUL && !L->small_k(t))) {
            // A reduction of this very pass: its value exists only after the
            // final fold, so it may appear only in invariant position.
            const KN& ik = ctx->n[idx];
            if (!(ik.ranged && ik.lo == ik.hi)) throw JoinFail();
            for (size_t r = 0; r < grp->reds.size(); ++r)
              if (grp->reds[r].t == t && grp->reds[r].elem == ik.lo) {
                KN k;
                k.op = K_REDVAL;
                k.dt = x.dt;
                k.iv = (int64_t)r;
                return ctx->mk(k);
              }
            throw JoinFail();
          }
          if (x.kind == T_SCAN || x.kind == T_SCATTER) throw JoinFail();
          // element-wise member of this pass: recompute inline
        } else if (x.kind != T_PARAM) {
          throw JoinFail();  // produced by a later kernel
        }
      }
      return inline_node(t, idx);
    }

    int inline_node(int t, int idx) {
      const GTensor& x = L->g.ts[t];
      switch (x.kind) {
        case T_IOTA: return idx;
        case T_MAP: {
          int env[2] = {elem(x.dep0, idx), -1};
          return expr(x.body, env, idx);
        }
        case T_MAP2: {
          int env[2] = {elem(x.dep0, idx), elem(x.dep1, idx)};
          return expr(x.body, env, idx);
        }
        case T_GATHER: {
          const int j = elem(x.dep0, idx);
          KN k;
          k.op = K_CHECK;
          k.dt = DT_I32;
          k.a = j;
          k.iv = L->g.ts[x.dep1].numel;
          int jc = ctx->mk(k);
          if (ctx->n[jc].op == K_CHECK && ctx->n[jc].ranged) jc = j;  // provably in bounds
          return elem(x.dep1, jc);
        }
        case T_RESHAPE: return elem(x.dep0, idx);
        case T_BROADCAST: return elem(x.dep0, ctx->cint(DT_I32, 0));
        case T_MATMUL: {
          if (!L->small_k(t)) break;
          const int64_t N = x.shape[1], K = L->g.ts[x.dep0].shape[1];
          const int row = ctx->bin(DT_I32, B_DIV, idx, ctx->cint(DT_I32, N));
          const int col = ctx->bin(DT_I32, B_SUB, idx, ctx->bin(DT_I32, B_MUL, row, ctx->cint(DT_I32, N)));
          int acc = is_float(x.dt) ? ctx->cfloat(x.dt, 0.0) : ctx->cint(x.dt, 0);
          for (int64_t k = 0; k < K; ++k) {
            const int ia = ctx->bin(DT_I32, B_ADD, ctx->bin(DT_I32, B_MUL, row, ctx->cint(DT_I32, K)), ctx->cint(DT_I32, k));
            const int ib = ctx->bin(DT_I32, B_ADD, ctx->cint(DT_I32, k * N), col);
            acc = ctx->bin(x.dt, B_ADD, acc, ctx->bin(x.dt, B_MUL, elem(x.dep0, ia), elem(x.dep1, ib)));
          }
          return acc;
        }
        default: break;
      }
      throw LowerError(CCB_ERR_INVALID, "lower: node n" + std::to_string(x.uid) + " must be materialised");
    }

    // Instantiate an element function body with its arguments bound.
    int expr(int e, const int env[2], int idx) {
      std::unordered_map<int, int> m;
      std::function<int(int)> go = [&](int id) -> int {
        auto it = m.find(id);
        if (it != m.end()) return it->second;
        const GExpr& x = L->g.ex[id];
        int r = -1;
        switch (x.kind) {
          case E_CONST:
            r = is_float(x.dt) ? ctx->cfloat(x.dt, x.f) : ctx->cint(x.dt, x.i);
            break;
          case E_ARG:
            if (x.i < 0 || x.i > 1 || env[x.i] < 0) bad("lower: unbound Arg " + std::to_string(x.i));
            if (ctx->n[env[x.i]].dt != x.dt) bad("lower: Arg dtype mismatch");
            r = env[x.i];
            break;
          case E_INDEX: r = idx; break;
          case E_BINOP: {
            if (is_float(x.dt) && x.op >= B_AND) bad(std::string("Emit: ") + kBin[x.op] + " on a float dtype");
            if (x.dt == DT_BOOL) bad("Emit: arithmetic on bool");
            const int a = go(x.a), b = go(x.b);
            r = ctx->bin(x.dt, x.op, a, b);
            break;
          }
          case E_UNOP: {
            if (!is_float(x.dt) && x.op != U_NEG && x.op != U_ABS) bad(std::string("Emit: ") + kUn[x.op] + " on a non-float dtype");
            r = ctx->un(x.dt, x.op, go(x.a));
            break;
          }
          case E_CMP: {
            KN k;
            k.op = K_CMP;
            k.dt = DT_BOOL;
            k.sub = x.op;
            k.a = go(x.a);
            k.b = go(x.b);
            r = ctx->mk(k);
            break;
          }
          case E_LOGIC: {
            KN k;
            k.op = K_LOGIC;
            k.dt = DT_BOOL;
            k.sub = x.op;
            k.a = go(x.a);
            k.b = go(x.b);
            r = ctx->mk(k);
            break;
          }
          case E_NOT: {
            KN k;
            k.op = K_NOT;
            k.dt = DT_BOOL;
            k.a = go(x.a);
            r = ctx->mk(k);
            break;
          }
          case E_SELECT: {
            KN k;
            k.op = K_SELECT;
            k.dt = x.dt;
            k.a = go(x.a);
            k.b = go(x.b);
            k.c = go(x.c);
            r = ctx->mk(k);
            break;
          }
          case E_CAST: {
            const int a = go(x.a);
            if (ctx->n[a].dt == x.dt) {
              r = a;
            } else {
              KN k;
              k.op = K_CAST;
              k.dt = x.dt;
              k.a = a;
              r = ctx->mk(k);
            }
            break;
          }
        }
        m[id] = r;
        return r;
      };
      return go(e);
    }
  };

  // ------------------------------------------------------------ factoring
  // e == inv * var where inv holds every part of e that depends on this
  // pass's reductions (and is loop-invariant) and var holds the rest; -1
  // stands for one. Only the late part is pulled out, so constants and other
  // invariants that are available during the pass stay in var.
  std::pair<int, int> factor(KCtx& c, int e) {
    const KN k = c.n[e];
    if (!k.late) return {-1, e};
    if (!k.variant) return {e, -1};
    auto or_one = [&](int v) { return v < 0 ? c.one(k.dt) : v; };
    if (k.op == K_BIN && is_float(k.dt)) {
      if (k.sub == B_MUL) {
        auto fa = factor(c, k.a), fb = factor(c, k.b);
        return {mul_opt(c, k.dt, fa.first, fb.first), mul_opt(c, k.dt, fa.second, fb.second)};
      }
      if (k.sub == B_DIV && !c.n[k.b].variant) {
        auto fa = factor(c, k.a);
        if (c.n[k.b].late) return {c.bin(k.dt, B_DIV, or_one(fa.first), k.b), fa.second};
        return {fa.first, c.bin(k.dt, B_DIV, or_one(fa.second), k.b)};
      }
      if (k.sub == B_ADD || k.sub == B_SUB) {
        auto fa = factor(c, k.a), fb = factor(c, k.b);
        if (fa.first == fb.first && fa.first >= 0) return {fa.first, c.bin(k.dt, k.sub, or_one(fa.second), or_one(fb.second))};
        return {-1, e};
      }
    }
    if (k.op == K_UN && k.sub == U_NEG && is_float(k.dt)) {
      auto fa = factor(c, k.a);
      return {fa.first, c.un(k.dt, U_NEG, or_one(fa.second))};
    }
    if (k.op == K_SELECT && !c.n[k.a].late) {
      auto fa = factor(c, k.b), fb = factor(c, k.c);
      if (fa.first == fb.first && fa.first >= 0) {
        KN s;
        s.op = K_SELECT;
        s.dt = k.dt;
        s.a = k.a;
        s.b = or_one(fa.second);
        s.c = or_one(fb.second);
        return {fa.first, c.mk(s)};
      }
    }
    return {-1, e};
  }

  static void dump(const KCtx& c, int id, int depth) {
    if (depth > 14 || id < 0) return;
    const KN& k = c.n[id];
    fprintf(stderr, "%*s#%d op=%d sub=%d dt=%d late=%d var=%d buf=%d iv=%lld f=%g\n", depth * 2, "", id, k.op, k.sub, (int)k.dt,
            (int)k.late, (int)k.variant, k.buf, (long long)k.iv, k.f);
    if (!k.late) return;
    dump(c, k.a, depth + 1);
    dump(c, k.b, depth + 1);
    dump(c, k.c, depth + 1);
  }

  static int mul_opt(KCtx& c, Dt dt, int x, int y) {
    if (x < 0) return y;
    if (y < 0) return x;
    return c.bin(dt, B_MUL, x, y);
  }

  // Is fn2 of tensor t exactly `add (arg0) (arg1)`? (lib/ad/grad.ml:158-166)
  bool is_plain_add(int t) const {
    const GTensor& x = g.ts[t];
    const GExpr& b = g.ex[x.body];
    if (b.kind != E_BINOP || b.op != B_ADD) return false;
    const GExpr& ea = g.ex[b.a];
    const GExpr& eb = g.ex[b.b];
    return ea.kind == E_ARG && eb.kind == E_ARG && ea.i != eb.i;
  }
  bool init_is_zero(int t) const {
    const GExpr& e = g.ex[g.ts[t].init];
    if (e.kind != E_CONST) return false;
    return is_float(e.dt) ? (e.f == 0.0 && !std::signbit(e.f)) : e.i == 0;
  }

  // ------------------------------------------------------------ joining
  // Try to add root t to MAPRED group gi. On success the group is updated.
  bool try_join(int gi, int t) {
    Group trial = groups[gi];  // copy: a failed join leaves no trace
    Build B{this, gi, &trial.ctx, &trial, {}};
    const GTensor& x = g.ts[t];
    try {
      if (x.kind == T_REDUCE) {
        const int src = x.dep0;
        const int v = B.elem(src, trial.ctx.index());
        Red r;
        r.t = t;
        r.elem = 0;
        r.dt = x.dt;
        r.comb_t = t;
        r.init = init_knode(trial.ctx, t);
        if (!trial.ctx.n[v].late) {
          r.var = v;
        } else {
          if (!is_float(x.dt) || !is_plain_add(t) || !init_is_zero(t)) throw JoinFail();
          auto f = factor(trial.ctx, v);
          if (std::getenv("CCB_DEBUG_LOWER")) {
            fprintf(stderr, "factor n%lld: inv=%d var=%d\n", (long long)x.uid, f.first, f.second);
            dump(trial.ctx, v, 0);
          }
          if (f.first < 0 || (f.second >= 0 && trial.ctx.n[f.second].late)) throw JoinFail();
          r.inv = f.first;
          r.var = f.second < 0 ? trial.ctx.one(x.dt) : f.second;
        }
        if (!trial.reds.empty() && trial.reds[0].dt != x.dt) throw JoinFail();
        trial.reds.push_back(r);
      } else if (x.kind == T_MATMUL && !small_k(t)) {
        // skinny product: one additive accumulator per output cell, INDEX = k
        const GTensor& A = g.ts[x.dep0];
        const int64_t M = x.shape[0], N = x.shape[1], K = A.shape[1];
        if (!trial.reds.empty() && trial.reds[0].dt != x.dt) throw JoinFail();
        const int k = trial.ctx.index();
        for (int64_t i = 0; i < M; ++i)
          for (int64_t j = 0; j < N; ++j) {
            const int ia = trial.ctx.bin(DT_I32, B_ADD, trial.ctx.cint(DT_I32, i * K), k);
            const int ib = trial.ctx.bin(DT_I32, B_ADD, trial.ctx.bin(DT_I32, B_MUL, k, trial.ctx.cint(DT_I32, N)),
                                         trial.ctx.cint(DT_I32, j));
            const int av = B.elem(x.dep0, ia), bv = B.elem(x.dep1, ib);
            const int prod = trial.ctx.bin(x.dt, B_MUL, av, bv);
            if (trial.ctx.n[prod].late) throw JoinFail();
            Red r;
            r.t = t;
            r.elem = i * N + j;
            r.dt = x.dt;
            r.comb_t = -1;
            r.init = is_float(x.dt) ? trial.ctx.cfloat(x.dt, 0.0) : trial.ctx.cint(x.dt, 0);
            r.var = prod;
            trial.reds.push_back(r);
          }
      } else if (x.numel == 1 && !(trial.domain == 1 && trial.reds.empty())) {
        // scalar tail, evaluated in the epilogue
        const int v = B.inline_node(t, trial.ctx.cint(DT_I32, 0));
        trial.tails.push_back({t, v});
      } else {
        if (x.numel != trial.domain) throw JoinFail();
        const int v = B.inline_node(t, trial.ctx.index());
        if (trial.ctx.n[v].late) throw JoinFail();
        trial.stores.push_back({t, v});
      }
    } catch (const JoinFail&) {
      if (std::getenv("CCB_DEBUG_LOWER")) fprintf(stderr, "ccb lower: n%lld cannot join pass %d\n", (long long)x.uid, gi);
      return false;
    }
    if (trial.reds.size() > 64) return false;
    groups[gi] = std::move(trial);
    group_of[t] = gi;
    return true;
  }

  int init_knode(KCtx& c, int t) {
    // The identity, evaluated at index 0 as both backends do.
    Build B{this, -1, &c, nullptr, {}};
    int env[2] = {-1, -1};
    return B.expr(g.ts[t].init, env, c.cint(DT_I32, 0));
  }

  int new_group(int kind, int64_t domain) {
    Group gr;
    gr.kind = kind;
    gr.domain = domain;
    gr.ctx.ilo = 0;
    gr.ctx.ihi = domain > 0 ? domain - 1 : 0;
    groups.push_back(std::move(gr));
    return (int)groups.size() - 1;
  }

  void build_single(int gi, int t) {
    Group& gr = groups[gi];
    group_of[t] = gi;
    gr.root = t;
    const GTensor& x = g.ts[t];
    Build B{this, gi, &gr.ctx, &gr, {}};
    try {
      switch (gr.kind) {
        case G_SCAN_FLAT:
        case G_SCAN_ROWS:
        case G_RED_ROWS:
          gr.val = B.elem(x.dep0, gr.ctx.index());
          break;
        case G_SCATTER:
          gr.val = B.elem(x.dep0, gr.ctx.index());   // index
          gr.val2 = B.elem(x.dep1, gr.ctx.index());  // source
          break;
        case G_MATMUL: {
          gr.ctx.ihi = std::max<int64_t>(0, g.ts[x.dep0].numel - 1);
          gr.ctx_b.ihi = std::max<int64_t>(0, g.ts[x.dep1].numel - 1);
          gr.mm_a = B.elem(x.dep0, gr.ctx.index());
          Build Bb{this, gi, &gr.ctx_b, &gr, {}};
          gr.mm_b = Bb.elem(x.dep1, gr.ctx_b.index());
          break;
        }
      }
    } catch (const JoinFail&) {
      throw LowerError(CCB_ERR_INVALID, "lower: internal: unsatisfied dependency");
    }
    if (gr.ctx.n[gr.val < 0 ? 0 : gr.val].late) bad("lower: internal: late value in a single kernel");
  }

  void group_all() {
    int cur = -1;  // most recent map-reduce group
    for (int t = 0; t < (int)g.ts.size(); ++t) {
      if (!mat[t] || g.ts[t].kind == T_PARAM) continue;
      const GTensor& x = g.ts[t];
      switch (x.kind) {
        case T_IOTA:
        case T_MAP:
        case T_MAP2:
        case T_GATHER:
        case T_RESHAPE:
        case T_BROADCAST: {
          int tsrc = -1;
          if (x.kind == T_GATHER && x.numel >= 4096 && transpose_of(t, tsrc)) {
            const int gi = new_group(G_TRANSPOSE, x.numel);
            groups[gi].root = t;
            groups[gi].val = tsrc;  // the tensor transposed
            group_of[t] = gi;
            break;
          }
          if (cur >= 0 && try_join(cur, t)) break;
          cur = new_group(G_MAPRED, x.numel == 1 ? 1 : x.numel);
          if (!try_join(cur, t)) bad("lower: internal: cannot start a pass");
          break;
        }
        case T_REDUCE: {
          const GTensor& src = g.ts[x.dep0];
          const int64_t n = src.shape.empty() ? 1 : src.shape.back();
          const int64_t rows = x.numel;
          if (rows == 1) {
            if (cur >= 0 && groups[cur].domain == n && try_join(cur, t)) break;
            cur = new_group(G_MAPRED, n);
            if (!try_join(cur, t)) bad("lower: internal: cannot start a reduction");
          } else {
            const int gi = new_group(G_RED_ROWS, rows * n);
            groups[gi].rows = rows;
            groups[gi].n = n;
            build_single(gi, t);
          }
          break;
        }
        case T_SCAN: {
          const GTensor& src = g.ts[x.dep0];
          const int64_t n = src.shape.empty() ? 1 : src.shape.back();
          const int64_t rows = n == 0 ? 0 : src.numel / n;
          const int gi = new_group(rows <= 1 ? G_SCAN_FLAT : G_SCAN_ROWS, src.numel);
          groups[gi].rows = rows;
          groups[gi].n = n;
          build_single(gi, t);
          break;
        }
        case T_SCATTER: {
          const int gi = new_group(G_SCATTER, g.ts[x.dep0].numel);
          build_single(gi, t);
          break;
        }
        case T_MATMUL: {
          const int64_t M = x.shape[0], N = x.shape[1], K = g.ts[x.dep0].shape[1];
          if (tc[t].on) {
            const int gi = new_group(G_MATMUL_TC, M * N);
            groups[gi].root = t;
            group_of[t] = gi;
            break;
          }
          if (small_k(t)) {  // an output: an element-wise store
            if (cur >= 0 && try_join(cur, t)) break;
            cur = new_group(G_MAPRED, x.numel == 1 ? 1 : x.numel);
            if (!try_join(cur, t)) bad("lower: internal: cannot start a pass");
            break;
          }
          if (M * N <= 32 && K >= 2048) {
            if (cur >= 0 && groups[cur].domain == K && try_join(cur, t)) break;
            cur = new_group(G_MAPRED, K);
            if (!try_join(cur, t)) bad("lower: internal: cannot start a split-K product");
          } else {
            const int gi = new_group(G_MATMUL, M * N);
            groups[gi].rows = M;
            groups[gi].n = N;
            build_single(gi, t);
          }
          break;
        }
        default: bad("lower: unexpected node kind");
      }
    }
  }

  // ------------------------------------------------------------ epilogue fusion
  // Does group gi read tensor t?
  bool reads_tensor(int gi, int t) const {
    const Group& gr = groups[gi];
    if (gr.kind == G_MATMUL_TC) return tc[gr.root].va == t || tc[gr.root].vb == t;
    if (gr.kind == G_TRANSPOSE) return gr.val == t;
    for (const KN& k : gr.ctx.n)
      if (k.op == K_LOAD && k.buf == t) return true;
    for (const KN& k : gr.ctx_b.n)
      if (k.op == K_LOAD && k.buf == t) return true;
    return false;
  }

  // A map pass right after a tensor-core product, over the product's
  // elements, storing 4-byte elements and reading nothing but element i of
  // the product, runs in the product's epilogue: the accumulator feeds the
  // element body from registers. The element code is the pass's own, so the
  // results are the bits the separate pass gives. Only products with
  // K >= kEpiMinK fuse: the four epilogue warps drain a tile while the next
  // one accumulates, and a short mainloop leaves them no time for a body. A
  // pass that also reads another tensor stays apart: with one warp per TMEM
  // lane quadrant those loads are latency-bound (measured on the MLP step:
  // dZ1 in the epilogue of the K = 1024 product cost 225 us more than the
  // separate pass).
  //
  // The same holds for a scan whose kernel writes through F::store/store4 (row
  // scans and the 8-byte flat scan): the pass runs on each scanned value as
  // it is stored (LSM's S = S0 exp(cumulative log-increments)).
  static constexpr int64_t kEpiMinK = 2048;
  void fuse_epilogues() {
    for (int gi = 0; gi + 1 < (int)groups.size(); ++gi) {
      Group& mm = groups[gi];
      Group& ep = groups[gi + 1];
      if (ep.kind != G_MAPRED) continue;
      if (mm.kind != G_MATMUL_TC && mm.kind != G_SCAN_ROWS && mm.kind != G_SCAN_FLAT) continue;
      const int t = mm.root;
      if (t < 0) continue;
      const int64_t MN = g.ts[t].numel;
      if (mm.kind == G_MATMUL_TC) {
        if (g.ts[g.ts[t].dep0].shape[1] < kEpiMinK) continue;
      } else if (mm.kind == G_SCAN_ROWS || mm.kind == G_SCAN_FLAT) {
        int srcb = -1;
        if (staged_scan_source(mm, t, srcb)) continue;  // writes its destination directly
      } else {
        continue;
      }
      if (ep.domain != MN || MN >= (1LL << 31) || !ep.reds.empty() || !ep.tails.empty() || ep.stores.empty()) continue;
      bool reads_t = false, ok = true;
      for (const KN& k : ep.ctx.n) {
        if (k.op != K_LOAD) continue;
        if (k.buf != t || k.a != ep.ctx.index_node) ok = false;
        reads_t = true;
      }
      for (auto& st : ep.stores)
        if (g.ts[st.first].numel != MN || (mm.kind == G_MATMUL_TC && dt_size(g.ts[st.first].dt) != 4)) ok = false;
      if (!ok || !reads_t) continue;
      mm.epi = gi + 1;
      ep.fused_into = gi;
    }
  }

  // A short-row scan (warp per row) whose result (after its fused store
  // pass, if any) is read by nothing but a transpose writes the transpose
  // itself, through a shared-memory tile (scan_rows_warp_t): the [rows; n]
  // result is never stored.
  bool expr_uses_index(int e) const {
    if (e < 0) return false;
    const GExpr& x = g.ex[e];
    return x.kind == E_INDEX || expr_uses_index(x.a) || expr_uses_index(x.b) || expr_uses_index(x.c);
  }
  // The next pass's single store is map(f, transpose(t)) with the transpose
  // inlined as a gather of t read nowhere else, and f blind to the index:
  // the LOAD node of t in that pass, else -1.
  int transposed_map_load(int gm, int t) const {
    if (gm >= (int)groups.size() || groups[gm].kind != G_MAPRED) return -1;
    const Group& mp = groups[gm];
    if (!mp.reds.empty() || !mp.tails.empty() || mp.stores.size() != 1) return -1;
    const GTensor& y = g.ts[mp.stores[0].first];
    int src = -1;
    if (y.kind != T_MAP || expr_uses_index(y.body) || mat[y.dep0] || uses[y.dep0] != 1 || !transpose_of(y.dep0, src) ||
        src != t)
      return -1;
    int load = -1;
    for (int k = 0; k < (int)mp.ctx.n.size(); ++k) {
      if (mp.ctx.n[k].op != K_LOAD) continue;
      if (mp.ctx.n[k].buf != t || load >= 0) return -1;
      load = k;
    }
    return load;
  }

  void fuse_transposed_stores() {
    for (int gi = 0; gi < (int)groups.size(); ++gi) {
      Group& sc = groups[gi];
      if (sc.kind != G_SCAN_ROWS || sc.n >= 1024 || sc.rows < 32) continue;
      const int t = sc.root;
      if (sc.epi < 0 && !is_out[t]) {  // the transpose inlined into the next pass
        const int ld = transposed_map_load(gi + 1, t);
        int readers = 0;
        for (int q = 0; q < (int)groups.size(); ++q)
          if (q != gi && reads_tensor(q, t)) ++readers;
        if (ld >= 0 && readers == 1) {
          sc.tstore = gi + 1;
          sc.tload = ld;
          groups[gi + 1].fused_into = gi;
          continue;
        }
      }
      int u = t;
      if (sc.epi >= 0) {
        const Group& ep = groups[sc.epi];
        if (ep.stores.size() != 1 || must_store(gi, sc.epi, t)) continue;
        u = ep.stores[0].first;
      }
      if (is_out[u]) continue;
      int gt = -1, readers = 0;
      for (int q = 0; q < (int)groups.size(); ++q) {
        if (q == gi || q == sc.epi || !reads_tensor(q, u)) continue;
        ++readers;
        if (groups[q].kind == G_TRANSPOSE && groups[q].val == u) gt = q;
      }
      if (gt < 0 || readers != 1) continue;
      sc.tstore = gt;
      groups[gt].fused_into = gi;
      // A map pass right after the transpose that reads only the transposed
      // value at its own element and uses the index for nothing else runs
      // on each value too (LSM: S = S0 exp(.) of the transposed sums).
      const int tt = groups[gt].root;
      const int gm = gt + 1;
      if (gm < (int)groups.size() && groups[gm].kind == G_MAPRED && !is_out[tt]) {
        const Group& mp = groups[gm];
        bool ok = mp.domain == g.ts[tt].numel && mp.reds.empty() && mp.tails.empty() && mp.stores.size() == 1 &&
                  g.ts[mp.stores[0].first].numel == g.ts[tt].numel;
        for (const KN& k : mp.ctx.n) {
          const bool uses_index = k.a == mp.ctx.index_node || k.b == mp.ctx.index_node || k.c == mp.ctx.index_node;
          if (k.op == K_LOAD && !(k.buf == tt && k.a == mp.ctx.index_node)) ok = false;
          if (uses_index && k.op != K_LOAD) ok = false;
        }
        int others = 0;
        for (int q = 0; q < (int)groups.size(); ++q)
          if (q != gm && q != gt && q != gi && reads_tensor(q, tt)) ++others;
        if (ok && others == 0) {
          sc.tpost = gm;
          groups[gm].fused_into = gi;
        }
      }
    }
  }

  // ------------------------------------------------------------ code generation
  Lowered* out = nullptr;
  int sharded_passes = 0;  // reduction passes of a sharded program (at most one)
  std::ostringstream src;
  std::vector<int> node_buf;  // tensor -> buffer index

  int add_buf(const std::string& label, int elem_bytes, int64_t numel, int role, int node, bool zero) {
    BufSpec b;
    b.label = label;
    b.elem_bytes = elem_bytes;
    b.numel = numel;
    b.role = role;
    b.node = node;
    b.zero = zero;
    out->bufs.push_back(b);
    return (int)out->bufs.size() - 1;
  }

  // Fields of P: loaded buffers (const), written buffers, then extras.
  struct Field {
    std::string decl;
    Slot slot;
  };

  static std::set<int> loads_of(const KCtx& c) {
    std::set<int> s;
    for (const KN& k : c.n)
      if (k.op == K_LOAD) s.insert(k.buf);
    return s;
  }

  void emit_struct(const std::vector<Field>& f) {
    src << "  struct P {\n";
    for (auto& x : f)
      if (!x.decl.empty()) src << "    " << x.decl << ";\n";  // an empty decl: a further word of the previous array
    src << "  };\n";
  }

  Field in_field(int t) {
    Field f;
    f.decl = std::string("const ") + dt_ctype(g.ts[t].dt) + "* __restrict__ b" + std::to_string(t);
    f.slot.kind = SL_BUF;
    f.slot.buf = node_buf[t];
    f.slot.access = 0;
    return f;
  }
  Field out_field(int t) {
    Field f;
    f.decl = std::string(dt_ctype(g.ts[t].dt)) + "* __restrict__ o" + std::to_string(t);
    f.slot.kind = SL_BUF;
    f.slot.buf = node_buf[t];
    f.slot.access = 1;
    return f;
  }
  static Field buf_field(const std::string& decl, int buf) {
    Field f;
    f.decl = decl;
    f.slot.kind = SL_BUF;
    f.slot.buf = buf;
    return f;
  }
  static Field i64_field(const std::string& nm, int64_t v) {
    Field f;
    f.decl = "long long " + nm;
    f.slot.kind = SL_I64;
    f.slot.val = v;
    return f;
  }

  // "_<graph name>" restricted to identifier characters: kernels of different
  // graphs are told apart in profiles.
  std::string kname_suffix() const {
    std::string s = "_";
    for (char ch : g.name)
      if (s.size() < 40 && (std::isalnum((unsigned char)ch) || ch == '_')) s += ch;
    return s.size() > 1 ? s : "";
  }

  LaunchSpec& add_launch(const std::string& fn, const std::vector<Field>& fields) {
    LaunchSpec l;
    l.fn = fn;
    for (auto& f : fields) l.slots.push_back(f.slot);
    out->launches.push_back(l);
    OpSpec op;
    op.kind = OP_LAUNCH;
    op.launch = (int)out->launches.size() - 1;
    out->ops.push_back(op);
    out->num_kernels++;
    return out->launches.back();
  }

  // Direct loads: LOAD(buf, INDEX) of 4- or 8-byte elements in the cone of roots.
  std::vector<int> direct_loads(const KCtx& c, const std::vector<int>& roots) {
    std::vector<char> seen(c.n.size(), 0);
    std::set<int> bufs;
    std::function<void(int)> walk = [&](int id) {
      if (id < 0 || seen[id]) return;
      seen[id] = 1;
      const KN& k = c.n[id];
      if (k.op == K_LOAD && k.a == c.index_node && k.dt != DT_BOOL) bufs.insert(k.buf);
      walk(k.a);
      walk(k.b);
      walk(k.c);
    };
    for (int r : roots) walk(r);
    return std::vector<int>(bufs.begin(), bufs.end());
  }

  // A load at index i + u, u uniform over the pass (scalars and constants:
  // LSM's row t of a date-major S at t * n_paths + i), is a contiguous
  // stream. `terms` are u's summands with their signs; u is their wrapping
  // I32 sum, as the element index itself is computed.
  struct OffLoad {
    int id = -1, buf = -1;
    std::vector<std::pair<int, int>> terms;  // (sign, node)
  };
  static int decompose(const KCtx& c, int x, int sign, std::vector<std::pair<int, int>>& terms) {
    if (x == c.index_node) return sign > 0 ? 1 : -100;
    const KN& k = c.n[x];
    if (!k.variant && !k.late) {
      terms.push_back({sign, x});
      return 0;
    }
    if (k.op == K_BIN && k.dt == DT_I32 && (k.sub == B_ADD || k.sub == B_SUB))
      return decompose(c, k.a, sign, terms) + decompose(c, k.b, k.sub == B_ADD ? sign : -sign, terms);
    return -100;
  }
  std::vector<OffLoad> offset_loads(const KCtx& c, const std::vector<int>& roots) {
    std::vector<OffLoad> out;
    std::vector<char> seen(c.n.size(), 0);
    std::function<void(int)> walk = [&](int id) {
      if (id < 0 || seen[id]) return;
      seen[id] = 1;
      const KN& k = c.n[id];
      if (k.op == K_LOAD && k.a != c.index_node && k.dt != DT_BOOL && (dt_size(k.dt) == 4 || dt_size(k.dt) == 8)) {
        int x = k.a;
        if (c.n[x].op == K_CHECK) x = c.n[x].a;
        OffLoad o;
        o.id = id;
        o.buf = k.buf;
        if (c.n[x].dt == DT_I32 && decompose(c, x, 1, o.terms) == 1) out.push_back(o);
      }
      walk(k.a);
      walk(k.b);
      walk(k.c);
    };
    for (int r : roots) walk(r);
    return out;
  }
  // u of an offset load as an int expression (statements emitted by e)
  static std::string uniform_text(Emitter& e, const OffLoad& o) {
    std::string u = "0u";
    for (auto& t : o.terms) u += std::string(t.first > 0 ? " + " : " - ") + "(unsigned)(" + e.val(t.second) + ")";
    return "((int)(" + u + "))";
  }

  void emit_mapred(int gi) {
    Group& gr = groups[gi];
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_mapreduce_" + std::to_string(gi) + kname_suffix();
    const int R = (int)gr.reds.size();
    const Dt acc = R ? gr.reds[0].dt : DT_F32;
    const char* at = dt_ctype(acc);
    // buffers for every output of the pass
    for (auto& s : gr.stores) node_buf[s.first] = add_buf("t" + std::to_string(g.ts[s.first].uid), dt_size(g.ts[s.first].dt), g.ts[s.first].numel, BR_NODE, s.first, false);
    std::set<int> red_t;
    for (auto& r : gr.reds)
      if (!red_t.count(r.t)) {
        red_t.insert(r.t);
        node_buf[r.t] = add_buf("t" + std::to_string(g.ts[r.t].uid), dt_size(g.ts[r.t].dt), g.ts[r.t].numel, BR_NODE, r.t, false);
      }
    for (auto& s : gr.tails) node_buf[s.first] = add_buf("t" + std::to_string(g.ts[s.first].uid), dt_size(g.ts[s.first].dt), 1, BR_NODE, s.first, false);
    const int max_grid = 4096;
    int partials = -1, ticket = -1;
    if (R) {
      partials = add_buf("g" + std::to_string(gi) + "_partials", dt_size(acc), (int64_t)max_grid * R, BR_SCRATCH, -1, false);
      ticket = add_buf("g" + std::to_string(gi) + "_ticket", 4, 1, BR_SCRATCH, -1, true);
    }
    std::vector<int> roots;
    for (auto& s : gr.stores) roots.push_back(s.second);
    for (auto& r : gr.reds) roots.push_back(r.var);
    std::vector<int> direct = direct_loads(gr.ctx, roots);
    const std::vector<OffLoad> offs = offset_loads(gr.ctx, roots);
    // A pass that neither loads nor stores elements (a Monte-Carlo estimator:
    // Philox draws folded into reductions) gains nothing from the 4-wide
    // element path, whose copies of the body (13 with the unrolled and tail
    // loops) overflow the instruction cache: it runs one element at a time
    // (F64 Greeks 2^28 paths: 2.68 -> 2.60 ms).
    const bool scalar_only = direct.empty() && offs.empty() && gr.stores.empty();
    // Sharded program (wire "opt shard"): its one reduction pass walks this
    // rank's slice of the index space and combines the block totals of every
    // rank in its last block (ccb::xrank_combine); passes without reductions
    // only evaluate scalar tails, identically on every rank.
    const int W = g.shard_world;
    const bool sharded = W > 1 && R > 0;
    int64_t xlo = 0, xhi = gr.domain;
    if (W > 1) {
      if (!gr.stores.empty())
        unsupported("shard: pass " + std::to_string(gi) + " stores elements; a sharded program's passes produce scalars only");
      if (sharded) {
        if (!scalar_only)
          unsupported("shard: pass " + std::to_string(gi) +
                      " loads elements by index; only Monte-Carlo estimator passes (reductions of values computed from the "
                      "index, scalar inputs and Rng draws) are sharded");
        if (R > 32) unsupported("shard: a sharded pass exchanges at most 32 reductions, this one has " + std::to_string(R));
        if (++sharded_passes > 1) unsupported("shard: a sharded program has one reduction pass, this one has more");
        xlo = gr.domain * g.shard_rank / W;
        xhi = gr.domain * (g.shard_rank + 1) / W;
      }
    }
    std::vector<Field> fields;
    for (int b : loads_of(gr.ctx)) fields.push_back(in_field(b));
    for (auto& s : gr.stores) fields.push_back(out_field(s.first));
    for (int t : red_t) fields.push_back(out_field(t));
    for (auto& s : gr.tails) fields.push_back(out_field(s.first));
    fields.push_back(buf_field(std::string(at) + "* partials", partials));
    fields.push_back(buf_field("unsigned* ticket", ticket));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", gr.domain));
    if (sharded) {
      for (int q = 0; q < W; ++q) {
        Field f;
        if (q == 0) f.decl = "unsigned long long* xmb[" + std::to_string(W) + "]";
        f.slot.kind = SL_XMB;
        f.slot.val = q;
        fields.push_back(f);
      }
      Field f;
      f.decl = "unsigned long long xepoch";
      f.slot.kind = SL_XEPOCH;
      fields.push_back(f);
    }

    src << "// pass " << gi << ": " << gr.stores.size() << " element stores, " << R << " reductions, " << gr.tails.size()
        << " scalar tails over " << gr.domain << " elements";
    if (sharded) src << ", rank " << g.shard_rank << " of " << W << ": elements [" << xlo << ", " << xhi << ")";
    src << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << at << " acc_t;\n";
    if (sharded)
      src << "  static constexpr int XWORLD = " << W << ", XRANK = " << g.shard_rank << ";\n  static constexpr long long XLO = "
          << xlo << "LL, XHI = " << xhi << "LL;\n";
    src << "  static constexpr int NRED = " << R << ";\n  static constexpr int VEC = " << (scalar_only ? 0 : 1) << ";\n";
    // F64 estimators interleave four elements per iteration (F64 Greeks at
    // 2^28 paths: two instead of one 2.59 -> 2.53 ms; four instead of two
    // 2.508 -> 2.442 ms on one box; eight 2.61 against four 2.436 on
    // another; the F32 pass gained nothing from two or four)
    src << "  static constexpr bool ILP = " << (scalar_only && R > 0 && dt_size(acc) == 8 ? "true" : "false") << ";\n";
    // Passes that stream data keep 4 vector steps in flight; compute-bound
    // passes (Philox Monte Carlo) unroll 2 to keep the body small.
    src << "  static constexpr int UNROLL = " << (direct.empty() && offs.empty() ? 2 : 4) << ";\n";
    src << "  static constexpr bool TAIL = " << (gr.tails.empty() ? "false" : "true") << ";\n";
    // identity / combine
    src << "  static __device__ __forceinline__ acc_t identity(int r) {\n    switch (r) {\n";
    for (int r = 0; r < R; ++r) {
      std::ostringstream tmp;
      Emitter e(gr.ctx, tmp);
      std::string v = e.val(gr.reds[r].init);
      src << "      case " << r << ": {\n" << tmp.str() << "        return " << v << "; }\n";
    }
    src << "    }\n    return acc_t(0);\n  }\n";
    src << "  static __device__ __forceinline__ void init(acc_t* acc) {\n";
    for (int r = 0; r < R; ++r) src << "    acc[" << r << "] = identity(" << r << ");\n";
    src << "  }\n";
    src << "  static __device__ __forceinline__ acc_t combine(int r, acc_t a, acc_t b) {\n    switch (r) {\n";
    for (int r = 0; r < R; ++r) {
      src << "      case " << r << ": {\n";
      if (gr.reds[r].comb_t < 0 || is_plain_add(gr.reds[r].comb_t)) {
        src << "        return " << bin_text(acc, B_ADD, "a", "b") << "; }\n";
      } else {
        src << combine_body(gr.reds[r].comb_t, "        ");
      }
    }
    src << "    }\n    return a;\n  }\n";
    // vec_ok: aligned streams; each offset stream inside its buffer and aligned
    src << "  static __device__ __forceinline__ bool vec_ok(const P& p) {\n    bool ok = true";
    for (int b : direct) src << " && ccb::aligned16(p.b" << b << ")";
    for (auto& s : gr.stores) src << " && ccb::aligned16(p.o" << s.first << ")";
    src << ";\n";
    for (size_t q = 0; q < offs.size(); ++q) {
      Emitter e(gr.ctx, src);
      e.suffix = "_k" + std::to_string(q);
      const std::string u = uniform_text(e, offs[q]);
      src << "    { const long long u = " << u << "; ok = ok && u >= 0 && u + p.n <= " << g.ts[offs[q].buf].numel
          << "LL && ccb::aligned16(p.b" << offs[q].buf << " + u); }\n";
    }
    src << "    return ok;\n  }\n";
    // Reductions of one value with one combiner from one identity (the two
    // halves of a symmetric X^T X, say) are accumulated once.
    std::vector<int> alias(R, -1);
    for (int r = 0; r < R; ++r)
      for (int q = 0; q < r && alias[r] < 0; ++q) {
        const Red &a = gr.reds[q], &b = gr.reds[r];
        auto comb = [&](const Red& x) { return (x.comb_t < 0 || is_plain_add(x.comb_t)) ? -1 : x.comb_t; };
        if (alias[q] < 0 && a.var == b.var && a.init == b.init && a.dt == b.dt && comb(a) == comb(b)) alias[r] = q;
      }
    // elem
    src << "  static __device__ __forceinline__ void elem(const P& p, int i, acc_t* acc) {\n";
    {
      Emitter e(gr.ctx, src);
      for (auto& s : gr.stores) {
        std::string v = e.val(s.second);
        src << "    p.o" << s.first << "[i] = " << v << ";\n";
      }
      for (int r = 0; r < R; ++r) {
        if (alias[r] >= 0) continue;
        std::string v = e.val(gr.reds[r].var);
        src << "    acc[" << r << "] = combine(" << r << ", acc[" << r << "], " << v << ");\n";
      }
      (void)acc;
    }
    src << "  }\n";
    // elem4
    src << "  static __device__ __forceinline__ void elem4(const P& p, int i, acc_t* acc) {\n";
    for (int b : direct) src << "    const ccb::V4<" << dt_ctype(g.ts[b].dt) << "> L" << b << " = ccb::ld4(p.b" << b << " + i);\n";
    for (size_t q = 0; q < offs.size(); ++q) {  // in range and aligned: vec_ok checked
      Emitter e(gr.ctx, src);
      e.suffix = "_k" + std::to_string(q);
      const std::string u = uniform_text(e, offs[q]);
      src << "    const ccb::V4<" << dt_ctype(g.ts[offs[q].buf].dt) << "> K" << q << " = ccb::ld4(p.b" << offs[q].buf
          << " + " << u << " + i);\n";
    }
    for (auto& s : gr.stores) src << "    ccb::V4<" << dt_ctype(g.ts[s.first].dt) << "> S" << s.first << ";\n";
    for (int j = 0; j < 4; ++j) {
      Emitter e(gr.ctx, src);
      e.suffix = "_" + std::to_string(j);
      e.index_text = j == 0 ? "i" : "(i + " + std::to_string(j) + ")";
      for (int b : direct) e.direct[b] = "L" + std::to_string(b) + ".v[" + std::to_string(j) + "]";
      for (size_t q = 0; q < offs.size(); ++q) e.direct_node[offs[q].id] = "K" + std::to_string(q) + ".v[" + std::to_string(j) + "]";
      for (auto& s : gr.stores) {
        std::string v = e.val(s.second);
        src << "    S" << s.first << ".v[" << j << "] = " << v << ";\n";
      }
      for (int r = 0; r < R; ++r) {
        if (alias[r] >= 0) continue;
        std::string v = e.val(gr.reds[r].var);
        src << "    acc[" << r << "] = combine(" << r << ", acc[" << r << "], " << v << ");\n";
      }
    }
    for (auto& s : gr.stores) src << "    ccb::st4(p.o" << s.first << " + i, S" << s.first << ");\n";
    src << "  }\n";
    // epilogue
    src << "  static __device__ __forceinline__ void epilogue(const P& p, const acc_t* res) {\n";
    {
      Emitter e(gr.ctx, src);
      e.index_text = "0";
      for (int r = 0; r < R; ++r) {
        const Red& rd = gr.reds[r];
        std::string fv = "f" + std::to_string(r);
        const std::string rv = "res[" + std::to_string(alias[r] >= 0 ? alias[r] : r) + "]";
        if (rd.inv >= 0) {
          std::string iv = e.val(rd.inv);
          src << "    const acc_t " << fv << " = " << bin_text(acc, B_MUL, iv, rv) << ";\n";
        } else {
          src << "    const acc_t " << fv << " = " << rv << ";\n";
        }
        e.redval.push_back(fv);
        src << "    p.o" << rd.t << "[" << rd.elem << "] = " << fv << ";\n";
      }
      for (auto& s : gr.tails) {
        std::string v = e.val(s.second);
        src << "    p.o" << s.first << "[0] = " << v << ";\n";
      }
    }
    src << "  }\n};\n";
    // Ask for 8 resident blocks (32 registers); the program builder drops the
    // bound for a kernel whose ptxas report shows spills (CCB_MINB_<pass>=1).
    const std::string mb = "CCB_MINB_" + fn.substr(14);
    src << "#ifndef " << mb << "\n#define " << mb << " 8\n#endif\n";
    src << "extern \"C\" __global__ void __launch_bounds__(256, " << mb << ") " << fn << "(const " << F
        << "::P p) { ccb::map_reduce<" << F << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = xhi - xlo;
    l.per_block = 256 * 8;
    l.streams = !scalar_only;
    l.max_grid = R ? max_grid : (1 << 20);
    if (R == 0 && gr.stores.empty()) {
      l.work = 1;  // tails only
    }
  }

  std::string combine_body(int t, const std::string& ind) {
    const GTensor& x = g.ts[t];
    KCtx c;
    std::ostringstream tmp;
    Build B{this, -1, &c, nullptr, {}};
    KN a;
    a.op = K_ARG;
    a.dt = x.dt;
    a.iv = 0;
    KN b = a;
    b.iv = 1;
    int env[2] = {c.mk(a), c.mk(b)};
    const int v = B.expr(x.body, env, c.cint(DT_I32, 0));
    Emitter e(c, tmp);
    e.ind = ind;
    std::string r = e.val(v);
    return tmp.str() + ind + "return " + r + "; }\n";
  }

  // Functor pieces shared by the scan and rows kernels: load/load4 of the
  // source element, identity and combine of the root's fn2.
  void emit_source_access(Group& gr, int t, const std::string& T) {
    const GTensor& x = g.ts[t];
    {
      std::ostringstream tmp;
      KCtx c;
      int iv = init_knode(c, t);
      Emitter e(c, tmp);
      std::string v = e.val(iv);
      src << "  static __device__ __forceinline__ T identity() {\n" << tmp.str() << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ T combine(T a, T b) {\n";
    if (is_plain_add(t))
      src << "    return " << bin_text(x.dt, B_ADD, "a", "b") << "; }\n";
    else
      src << combine_body(t, "    ");
    std::vector<int> direct = direct_loads(gr.ctx, {gr.val});
    src << "  static __device__ __forceinline__ T load(const P& p, long long li) {\n    const int i = (int)li;\n";
    {
      Emitter e(gr.ctx, src);
      std::string v = e.val(gr.val);
      src << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ void load4(const P& p, long long li, T* x) {\n    const int i = (int)li;\n";
    for (int b : direct) src << "    const ccb::V4<" << dt_ctype(g.ts[b].dt) << "> L" << b << " = ccb::ld4(p.b" << b << " + i);\n";
    for (int j = 0; j < 4; ++j) {
      Emitter e(gr.ctx, src);
      e.suffix = "_" + std::to_string(j);
      e.index_text = j == 0 ? "i" : "(i + " + std::to_string(j) + ")";
      for (int b : direct) e.direct[b] = "L" + std::to_string(b) + ".v[" + std::to_string(j) + "]";
      std::string v = e.val(gr.val);
      src << "    x[" << j << "] = " << v << ";\n";
    }
    src << "  }\n";
    src << "  static __device__ __forceinline__ bool vec_ok(const P& p) {\n    return true";
    for (int b : direct) src << " && ccb::aligned16(p.b" << b << ")";
    (void)T;
  }

  // The staged (TMA) flat scan: a 4-byte scan whose source is a buffer read
  // straight at the element index.
  bool staged_scan_source(const Group& gr, int t, int& src_buf) const {
    const GTensor& x = g.ts[t];
    if (gr.kind != G_SCAN_FLAT || dt_size(x.dt) != 4) return false;
    const KN& k = gr.ctx.n[gr.val];
    if (k.op != K_LOAD || k.a != gr.ctx.index_node) return false;
    src_buf = k.buf;
    return true;
  }

  void emit_scan_staged(int gi, int srcb) {
    Group& gr = groups[gi];
    const int t = gr.root;
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_scanstaged_" + std::to_string(gi) + kname_suffix();
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    // 24 KiB tiles (6 strips of 256 x 4 elements): 3 CTAs/SM with the
    // 3-deep ring (2^28 F32: 0.432 ms; 32 KiB tiles at 2 CTAs/SM 0.453,
    // 20 KiB 0.47, 28 KiB 0.48)
    constexpr int strips = 6;
    const int64_t TILE = 1024 * strips;
    const int64_t ntiles = std::max<int64_t>(1, (gr.domain + TILE - 1) / TILE);
    const std::string pre = "g" + std::to_string(gi);
    std::vector<Field> fields;
    fields.push_back(in_field(srcb));
    fields.push_back(out_field(t));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", gr.domain));
    fields.push_back(buf_field("unsigned* tile_counter", add_buf(pre + "_tiles", 4, 1, BR_SCRATCH, -1, true)));
    fields.push_back(buf_field("unsigned* done_counter", add_buf(pre + "_done", 4, 1, BR_SCRATCH, -1, true)));
    fields.push_back(buf_field("unsigned long long* status", add_buf(pre + "_status", 8, ntiles, BR_SCRATCH, -1, true)));
    Field ep;
    ep.decl = "unsigned long long epoch";
    ep.slot.kind = SL_EPOCH;
    fields.push_back(ep);
    src << "// staged flat scan " << gi << " over " << gr.domain << " elements (" << ntiles << " tiles of " << TILE << ")\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n";
    {
      std::ostringstream tmp;
      KCtx c;
      int iv = init_knode(c, t);
      Emitter e(c, tmp);
      std::string v = e.val(iv);
      src << "  static __device__ __forceinline__ T identity() {\n" << tmp.str() << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ T combine(T a, T b) {\n";
    if (is_plain_add(t))
      src << "    return " << bin_text(x.dt, B_ADD, "a", "b") << "; }\n";
    else
      src << combine_body(t, "    ");
    src << "  static __device__ __forceinline__ const T* src(const P& p) { return p.b" << srcb << "; }\n";
    src << "  static __device__ __forceinline__ T* dst(const P& p) { return p.o" << t << "; }\n";
    src << "};\n";
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::scan_flat_staged<" << F
        << ", " << strips << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = ntiles;
    l.per_block = 1;
    l.smem = (int)(3 * TILE * 4 + 64);
  }

  // The staged (TMA) row kernels: a 4-byte row reduction or row scan whose
  // source is a buffer read straight at the element index, over rows of at
  // least 1024 elements and a multiple of 4 (so rows start 16-byte aligned).
  // Opt-in with CCB_ROWS_STAGED=1: on the B200 the register-streaming row
  // kernels are faster (65536 x 4096 F32: reduce_rows 0.157 vs 0.173 ms,
  // scan_rows 0.342 vs 0.358 ms), so they stay the default.
  bool staged_rows_source(const Group& gr, int t, int& src_buf) const {
    const GTensor& x = g.ts[t];
    if ((gr.kind != G_RED_ROWS && gr.kind != G_SCAN_ROWS) || dt_size(x.dt) != 4) return false;
    if (gr.n < 1024 || gr.n % 4 != 0) return false;
    const char* e = std::getenv("CCB_ROWS_STAGED");
    if (!e || e[0] != '1') return false;
    const KN& k = gr.ctx.n[gr.val];
    if (k.op != K_LOAD || k.a != gr.ctx.index_node) return false;
    src_buf = k.buf;
    return true;
  }

  void emit_rows_staged(int gi, int srcb, bool scan) {
    Group& gr = groups[gi];
    const int t = gr.root;
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = std::string(scan ? "ccb_scanrowsstaged_" : "ccb_redrowsstaged_") + std::to_string(gi) + kname_suffix();
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    std::vector<Field> fields;
    fields.push_back(in_field(srcb));
    fields.push_back(out_field(t));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", gr.n));
    fields.push_back(i64_field("rows", gr.rows));
    src << "// staged row " << (scan ? "scan " : "reduction ") << gi << ": " << gr.rows << " rows of " << gr.n << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n";
    {
      std::ostringstream tmp;
      KCtx c;
      int iv = init_knode(c, t);
      Emitter e(c, tmp);
      std::string v = e.val(iv);
      src << "  static __device__ __forceinline__ T identity() {\n" << tmp.str() << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ T combine(T a, T b) {\n";
    if (is_plain_add(t))
      src << "    return " << bin_text(x.dt, B_ADD, "a", "b") << "; }\n";
    else
      src << combine_body(t, "    ");
    src << "  static __device__ __forceinline__ const T* src(const P& p) { return p.b" << srcb << "; }\n";
    if (scan)
      src << "  static __device__ __forceinline__ T* dst(const P& p) { return p.o" << t << "; }\n";
    else
      src << "  static __device__ __forceinline__ void store_row(const P& p, long long r, T v) { p.o" << t << "[r] = v; }\n";
    src << "};\n";
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::rows_staged<" << F
        << ", " << (scan ? "true" : "false") << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = gr.rows;
    l.per_block = 1;
    l.smem = 4 * 16384 + 32;  // ccb::ROW_SMEM: a ring of 4 chunks of 4096 elements and their barriers
  }

  void emit_scan(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root;
    {
      int srcb = -1;
      if (staged_scan_source(gr, t, srcb)) {
        emit_scan_staged(gi, srcb);
        return;
      }
      if (gr.kind == G_SCAN_ROWS && gr.epi < 0 && gr.tstore < 0 && staged_rows_source(gr, t, srcb)) {
        emit_rows_staged(gi, srcb, true);
        return;
      }
    }
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const bool flat = gr.kind == G_SCAN_FLAT;
    const std::string fn = std::string(flat ? "ccb_scan_" : "ccb_scanrows_") + std::to_string(gi) + kname_suffix();
    const int ej = gr.epi;
    // the transposed tensor this scan writes: the transpose itself, or the
    // map pass over it that runs in the same stores
    const int tt = gr.tstore < 0 ? -1
                   : gr.tload >= 0 ? groups[gr.tstore].stores[0].first
                   : gr.tpost >= 0 ? groups[gr.tpost].stores[0].first
                                   : groups[gr.tstore].root;
    const bool store_t = tt < 0 && (ej < 0 || must_store(gi, ej, t));
    if (ej >= 0 && tt < 0)
      for (auto& st : groups[ej].stores)
        node_buf[st.first] = add_buf("t" + std::to_string(g.ts[st.first].uid), dt_size(g.ts[st.first].dt),
                                     g.ts[st.first].numel, BR_NODE, st.first, false);
    if (tt >= 0) node_buf[tt] = add_buf("t" + std::to_string(g.ts[tt].uid), dt_size(g.ts[tt].dt), g.ts[tt].numel, BR_NODE, tt, false);
    if (store_t) node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    const int items = dt_size(x.dt) == 4 ? 16 : 8;
    const int64_t tile = 256 * items;
    const int64_t ntiles = std::max<int64_t>(1, (gr.domain + tile - 1) / tile);
    std::vector<Field> fields;
    for (int b : loads_of(gr.ctx)) fields.push_back(in_field(b));
    if (store_t) fields.push_back(out_field(t));
    if (ej >= 0 && tt < 0)
      for (auto& st : groups[ej].stores) fields.push_back(out_field(st.first));
    if (tt >= 0) fields.push_back(out_field(tt));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", flat ? gr.domain : gr.n));
    fields.push_back(i64_field("rows", gr.rows));
    if (flat) {
      const std::string pre = "g" + std::to_string(gi);
      fields.push_back(buf_field("unsigned* tile_counter", add_buf(pre + "_tiles", 4, 1, BR_SCRATCH, -1, true)));
      if (dt_size(x.dt) == 4) {
        // one packed [epoch | flag | value] word per tile
        fields.push_back(buf_field("unsigned long long* status", add_buf(pre + "_status", 8, ntiles, BR_SCRATCH, -1, true)));
      } else {
        fields.push_back(buf_field("unsigned* flags", add_buf(pre + "_flags", 4, ntiles, BR_SCRATCH, -1, true)));
        fields.push_back(buf_field(std::string(T) + "* aggs", add_buf(pre + "_aggs", dt_size(x.dt), ntiles, BR_SCRATCH, -1, false)));
        fields.push_back(buf_field(std::string(T) + "* incls", add_buf(pre + "_incls", dt_size(x.dt), ntiles, BR_SCRATCH, -1, false)));
      }
      Field ep;
      ep.decl = "unsigned long long epoch";
      ep.slot.kind = SL_EPOCH;
      fields.push_back(ep);
    }
    src << "// " << (flat ? "flat scan" : "row scan") << " " << gi << " over " << gr.domain << " elements";
    if (ej >= 0) src << "; pass " << ej << " in the store" << (store_t ? "" : ", scan not stored");
    if (tt >= 0) src << "; writes the transpose of group " << gr.tstore;
    src << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n  static constexpr int VEC = 1;\n";
    emit_source_access(gr, t, T);
    if (store_t) src << " && ccb::aligned16(p.o" << t << ")";
    if (ej >= 0 && tt < 0)
      for (auto& st : groups[ej].stores) src << " && ccb::aligned16(p.o" << st.first << ")";
    src << ";\n  }\n";
    if (tt >= 0) {
      // value of element i as stored (the fused pass applied), and where the transpose goes
      src << "  typedef " << dt_ctype(g.ts[tt].dt) << " U;\n";
      src << "  static __device__ __forceinline__ U* tout(const P& p) { return p.o" << tt << "; }\n";
      src << "  static __device__ __forceinline__ U value(const P& p, long long li, T v) {\n    const int i = (int)li;\n";
      std::string w = "v";
      if (gr.tload >= 0) {  // the pass over the inlined transpose, its load replaced by v
        const Group& mp = groups[gr.tstore];
        Emitter e(mp.ctx, src);
        e.suffix = "_m";
        e.direct_node[gr.tload] = "v";
        w = e.val(mp.stores[0].second);
      }
      if (ej >= 0) {
        Emitter e(groups[ej].ctx, src);
        e.suffix = "_e";
        e.direct[t] = "v";
        w = e.val(groups[ej].stores[0].second);
      }
      if (gr.tpost >= 0) {
        const Group& mp = groups[gr.tpost];
        Emitter e(mp.ctx, src);
        e.suffix = "_m";
        e.direct[groups[gr.tstore].root] = w;
        w = e.val(mp.stores[0].second);
      }
      src << "    (void)i;\n    return " << w << ";\n  }\n";
    } else if (ej < 0) {
      src << "  static __device__ __forceinline__ void store(const P& p, long long i, T v) { p.o" << t << "[i] = v; }\n";
      src << "  static __device__ __forceinline__ void store4(const P& p, long long i, const T* x) {\n"
          << "    ccb::V4<T> s; s.v[0] = x[0]; s.v[1] = x[1]; s.v[2] = x[2]; s.v[3] = x[3]; ccb::st4(p.o" << t << " + i, s);\n  }\n";
    } else {
      emit_fused_store(groups[ej], t, store_t);
    }
    src << "};\n";
    std::string call;
    if (flat) {
      call = "ccb::scan_flat<" + F + ", " + std::to_string(items) + ">(p);";
    } else if (gr.n >= 1024) {
      call = "ccb::scan_rows_block<" + F + ", " + std::to_string(dt_size(x.dt) == 4 ? 8 : 4) + ">(p);";
    } else if (tt >= 0) {
      call = "ccb::scan_rows_warp_t<" + F + ">(p);";
    } else {
      call = "ccb::scan_rows_warp<" + F + ">(p);";
    }
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { " << call << " }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    if (flat) {
      l.mode = GM_FIXED;
      l.gx = ntiles;
    } else {
      l.mode = GM_PERSISTENT;
      l.work = gr.rows;
      l.per_block = gr.n >= 1024 ? 1 : tt >= 0 ? 32 : 8;
    }
  }

  // With pass ej fused into group gi's stores, gi's own output is written
  // only when it is a graph output or another group reads it.
  bool must_store(int gi, int ej, int t) const {
    if (is_out[t]) return true;
    for (int q = 0; q < (int)groups.size(); ++q)
      if (q != gi && q != ej && reads_tensor(q, t)) return true;
    return false;
  }

  // store/store4 of a scan that runs the fused pass ep on each value v
  // (element i of t) as it is stored.
  void emit_fused_store(const Group& ep, int t, bool store_t) {
    src << "  static __device__ __forceinline__ void store(const P& p, long long li, T v) {\n    const int i = (int)li;\n";
    if (store_t) src << "    p.o" << t << "[i] = v;\n";
    {
      Emitter e(ep.ctx, src);
      e.direct[t] = "v";
      for (auto& st : ep.stores) {
        std::string val = e.val(st.second);
        src << "    p.o" << st.first << "[i] = " << val << ";\n";
      }
    }
    src << "  }\n";
    src << "  static __device__ __forceinline__ void store4(const P& p, long long li, const T* x) {\n    const int i = (int)li;\n";
    if (store_t)
      src << "    { ccb::V4<T> s; s.v[0] = x[0]; s.v[1] = x[1]; s.v[2] = x[2]; s.v[3] = x[3]; ccb::st4(p.o" << t << " + i, s); }\n";
    for (auto& st : ep.stores) src << "    ccb::V4<" << dt_ctype(g.ts[st.first].dt) << "> S" << st.first << ";\n";
    for (int j = 0; j < 4; ++j) {
      Emitter e(ep.ctx, src);
      e.suffix = "_" + std::to_string(j);
      e.index_text = j == 0 ? "i" : "(i + " + std::to_string(j) + ")";
      e.direct[t] = "x[" + std::to_string(j) + "]";
      for (auto& st : ep.stores) {
        std::string val = e.val(st.second);
        src << "    S" << st.first << ".v[" << j << "] = " << val << ";\n";
      }
    }
    for (auto& st : ep.stores) src << "    ccb::st4(p.o" << st.first << " + i, S" << st.first << ");\n";
    src << "  }\n";
  }

  void emit_red_rows(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root;
    {
      int srcb = -1;
      if (staged_rows_source(gr, t, srcb)) {
        emit_rows_staged(gi, srcb, false);
        return;
      }
    }
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_redrows_" + std::to_string(gi) + kname_suffix();
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    std::vector<Field> fields;
    for (int b : loads_of(gr.ctx)) fields.push_back(in_field(b));
    fields.push_back(out_field(t));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", gr.n));
    fields.push_back(i64_field("rows", gr.rows));
    src << "// row reduction " << gi << ": " << gr.rows << " rows of " << gr.n << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n  static constexpr int VEC = 1;\n";
    emit_source_access(gr, t, T);
    src << ";\n  }\n";
    src << "  static __device__ __forceinline__ void store_row(const P& p, long long r, T v) { p.o" << t << "[r] = v; }\n";
    src << "};\n";
    const bool block = gr.n >= 1024;
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::"
        << (block ? "reduce_rows_block" : "reduce_rows_warp") << "<" << F << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = gr.rows;
    l.per_block = block ? 1 : 8;
  }

  void emit_scatter(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root;
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_scatter_" + std::to_string(gi) + kname_suffix();
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    OpSpec z;
    z.kind = OP_ZERO;
    z.buf = node_buf[t];
    out->ops.push_back(z);
    std::vector<Field> fields;
    for (int b : loads_of(gr.ctx)) fields.push_back(in_field(b));
    Field o = out_field(t);
    o.decl = std::string(T) + "* out";
    fields.push_back(o);
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("n", gr.domain));
    fields.push_back(i64_field("m", x.numel));
    src << "// scatter_add " << gi << ": " << gr.domain << " updates into " << x.numel << " bins\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n";
    src << "  static __device__ __forceinline__ int idx(const P& p, long long li) {\n    const int i = (int)li;\n";
    {
      Emitter e(gr.ctx, src);
      std::string v = e.val(gr.val);
      src << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ T val(const P& p, long long li) {\n    const int i = (int)li;\n";
    {
      Emitter e(gr.ctx, src);
      std::string v = e.val(gr.val2);
      src << "    return " << v << ";\n  }\n";
    }
    src << "};\n";
    // 16 KiB of block-private bins (4096 4-byte or 2048 8-byte bins) plus
    // 32 KiB of per-thread copies of the lowest 32 (16) bins. Measured on
    // 2^27 F32 updates: Zipf(1.1) into 2^20 bins 0.34 ms (64 KiB of private
    // bins and no thread copies: 1.09 ms; fewer private bins leave fewer to
    // flush per block), 16 uniform bins 0.23 ms (0.61), 4096 uniform bins
    // 0.29 ms (0.24: the copies cost occupancy).
    const int priv = 16384 / dt_size(x.dt);
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::scatter_add_priv<" << F
        << ", " << priv << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = gr.domain;
    l.per_block = 256 * 16;
    l.smem = (int)((std::min<int64_t>(x.numel, priv) + 256 * (128 / dt_size(x.dt))) * dt_size(x.dt));
  }

  void emit_matmul(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root;
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_matmul_" + std::to_string(gi) + kname_suffix();
    const int64_t M = x.shape[0], N = x.shape[1], K = g.ts[x.dep0].shape[1];
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    std::vector<Field> fields;
    std::set<int> loads = loads_of(gr.ctx);
    for (int b : loads_of(gr.ctx_b)) loads.insert(b);
    for (int b : loads) fields.push_back(in_field(b));
    fields.push_back(out_field(t));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("M", M));
    fields.push_back(i64_field("N", N));
    fields.push_back(i64_field("K", K));
    src << "// matmul " << gi << ": [" << M << "x" << K << "] . [" << K << "x" << N << "]\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n";
    src << "  static __device__ __forceinline__ T a(const P& p, long long r, long long k) {\n    const int i = (int)(r * p.K + k);\n";
    {
      Emitter e(gr.ctx, src);
      std::string v = e.val(gr.mm_a);
      src << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ T b(const P& p, long long k, long long c) {\n    const int i = (int)(k * p.N + c);\n";
    {
      Emitter e(gr.ctx_b, src);
      std::string v = e.val(gr.mm_b);
      src << "    return " << v << ";\n  }\n";
    }
    src << "  static __device__ __forceinline__ void store(const P& p, long long r, long long c, T v) { p.o" << t
        << "[r * p.N + c] = v; }\n";
    // 4-byte products of at least one 128 x 128 tile take the register-
    // blocked kernel; tiles load along the operand's contiguous dimension
    // (a transposed view of a buffer is read along its own rows)
    const bool big = simt[t].on;
    const bool a_mn = big && simt[t].a_mn;
    const bool b_km = big && simt[t].b_km;
    if (big) src << "  static constexpr bool A_MN = " << (a_mn ? "true" : "false") << ", B_KM = " << (b_km ? "true" : "false") << ";\n";
    src << "};\n";
    if (big) {
      src << "extern \"C\" __global__ void __launch_bounds__(256, 2) " << fn << "(const " << F << "::P p) { ccb::matmul_tiled128<"
          << F << ">(p); }\n\n";
    } else {
      src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::matmul_tiled<" << F
          << ">(p); }\n\n";
    }
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_FIXED;
    const int tile = big ? 128 : 64;
    l.gx = std::max<int64_t>(1, (N + tile - 1) / tile);
    l.gy = std::max<int64_t>(1, (M + tile - 1) / tile);
  }

  // F32 product on the tensor cores (ccb::matmul_tc): operands by TMA from
  // the buffers the operand views resolve to.
  void emit_matmul_tc(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root;
    const GTensor& x = g.ts[t];
    const TcInfo& ti = tc[t];
    const std::string F = "F" + std::to_string(gi);
    const int64_t M = x.shape[0], N = x.shape[1], K = g.ts[x.dep0].shape[1];
    // 2-SM pairs (256 x 256 tiles) once both output dimensions fill a pair tile
    const bool pair = M >= 256 && N >= 256;
    const std::string fn = (pair ? "ccb_matmultc2_" : "ccb_matmultc_") + std::to_string(gi) + kname_suffix();
    // with a fused map pass the product itself is stored only when an output
    // or another pass reads it
    const int ej = gr.epi;
    const bool store_c = ej < 0 || must_store(gi, ej, t);
    if (ej >= 0) {
      for (auto& st : groups[ej].stores)
        node_buf[st.first] = add_buf("t" + std::to_string(g.ts[st.first].uid), 4, g.ts[st.first].numel, BR_NODE, st.first, false);
    }
    if (store_c) node_buf[t] = add_buf("t" + std::to_string(x.uid), 4, x.numel, BR_NODE, t, false);
    if (node_buf[ti.va] < 0 || node_buf[ti.vb] < 0) bad("lower: internal: tensor-core operand without a buffer");
    std::vector<Field> fields;
    Field fa, fb;
    fa.decl = "ccb::TmaDesc ta";
    fa.slot.kind = SL_TMAP;
    fa.slot.buf = node_buf[ti.va];
    fa.slot.tbox[0] = 32;
    // MN-major operands with 32-element multiples along MN load a whole tile
    // of 32 x 32 boxes with one 3-D copy: dims {32, K, MN/32}, the 128-byte
    // step between boxes the outermost stride; same shared layout as the
    // 2-D boxes (MLP step 2.46 -> 2.23 ms: its dW products have both operands
    // MN-major, eight 2-D copies per stage and CTA before).
    const bool a3 = ti.a_mn && M % 32 == 0;
    const bool b3 = ti.b_mn && N % 32 == 0;
    // k-step: 64 for pairs (3 stages of 64 KiB: half the stage barriers,
    // copies and commits per flop of 6 x 32 KiB; MLP step 2.23 -> 1.97 ms),
    // 32 for the single-SM kernel
    const int bk = pair ? 64 : 32;
    if (ti.a_mn) {  // A^T stored [K][M]: 32 x 32 boxes, four per 128-row tile
      fa.slot.tdim[0] = M, fa.slot.tdim[1] = K, fa.slot.tstride = M * 4, fa.slot.tbox[1] = bk;
      fa.slot.tswizzle = (int)CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
      if (a3) {
        fa.slot.trank = 3;
        fa.slot.tdim[0] = 32, fa.slot.tdim[2] = M / 32, fa.slot.tstride2 = 128, fa.slot.tbox[2] = 4;
      }
    } else {  // A stored [M][K]: one 32 x 128 box
      fa.slot.tdim[0] = K, fa.slot.tdim[1] = M, fa.slot.tstride = K * 4, fa.slot.tbox[1] = 128;
    }
    fb.decl = "ccb::TmaDesc tb";
    fb.slot.kind = SL_TMAP;
    fb.slot.buf = node_buf[ti.vb];
    fb.slot.tbox[0] = 32;
    if (ti.b_mn) {  // B stored [K][N]: 32 x 32 boxes, eight per 256-column tile
      fb.slot.tdim[0] = N, fb.slot.tdim[1] = K, fb.slot.tstride = N * 4, fb.slot.tbox[1] = bk;
      fb.slot.tswizzle = (int)CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
      if (b3) {
        fb.slot.trank = 3;
        fb.slot.tdim[0] = 32, fb.slot.tdim[2] = N / 32, fb.slot.tstride2 = 128, fb.slot.tbox[2] = pair ? 4 : 8;
      }
    } else {  // B^T stored [N][K]: one 32 x 256 box (32 x 128 per CTA of a pair)
      fb.slot.tdim[0] = K, fb.slot.tdim[1] = N, fb.slot.tstride = K * 4, fb.slot.tbox[1] = pair ? 128 : 256;
    }
    fa.slot.access = fb.slot.access = 0;  // operands are only ever loaded through their maps
    fields.push_back(fa);  // tensor maps first: 64-byte aligned in the block
    fields.push_back(fb);
    if (store_c) fields.push_back(buf_field("float* __restrict__ C", node_buf[t]));
    if (ej >= 0)
      for (auto& st : groups[ej].stores) fields.push_back(out_field(st.first));
    fields.push_back(buf_field("unsigned* err", out->err_buf));
    fields.push_back(i64_field("M", M));
    fields.push_back(i64_field("N", N));
    fields.push_back(i64_field("K", K));
    src << "// matmul " << gi << " on tensor cores (tf32): [" << M << "x" << K << "] . [" << K << "x" << N << "], A "
        << (ti.a_mn ? "MN" : "K") << "-major from n" << g.ts[ti.va].uid << ", B " << (ti.b_mn ? "MN" : "K")
        << "-major from n" << g.ts[ti.vb].uid;
    if (ej >= 0) src << "; pass " << ej << " in the epilogue" << (store_c ? "" : ", product not stored");
    src << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  static constexpr bool A_MN = " << (ti.a_mn ? "true" : "false") << ", B_MN = " << (ti.b_mn ? "true" : "false")
        << ";\n";
    src << "  static constexpr bool EPI = " << (ej >= 0 ? "true" : "false") << ";\n";
    src << "  static constexpr bool A3 = " << (a3 ? "true" : "false") << ", B3 = " << (b3 ? "true" : "false") << ";\n";
    src << "  static constexpr int BK = " << bk << ";\n";
    src << "  static __device__ __forceinline__ bool vec_ok(const P& p) {\n    return true";
    if (store_c) src << " && ccb::aligned16(p.C)";
    if (ej >= 0)
      for (auto& st : groups[ej].stores) src << " && ccb::aligned16(p.o" << st.first << ")";
    src << ";\n  }\n";
    if (ej >= 0) emit_tc_epilogue(groups[ej], t, store_c);
    src << "};\n";
    if (pair) {
      src << "extern \"C\" __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1) " << fn
          << "(const __grid_constant__ " << F << "::P p) { ccb::matmul_tc2<" << F << ">(p); }\n\n";
    } else {
      src << "extern \"C\" __global__ void __launch_bounds__(192, 1) " << fn << "(const __grid_constant__ " << F
          << "::P p) { ccb::matmul_tc<" << F << ">(p); }\n\n";
    }
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = pair ? 2 * ((M + 255) / 256) * ((N + 255) / 256) : ((M + 127) / 128) * ((N + 255) / 256);
    l.per_block = 1;
    l.grid_multiple = pair ? 2 : 1;
    l.block = 192;
    l.smem = 4 * (128 * 32 * 4 + 256 * 32 * 4) + 1024 + 256;
  }

  // epi32(p, i0, v, cnt, vec): the fused map pass over the cnt product
  // entries v[0..cnt) at flat indices i0.. of one row (cnt = 32 and 16-byte
  // aligned bases when vec).
  void emit_tc_epilogue(const Group& ep, int t, bool store_c) {
    src << "  static __device__ __forceinline__ void epi32(const P& p, long long i0, const float* v, int cnt, bool vec) {\n";
    src << "    if (vec && cnt == 32) {\n#pragma unroll\n      for (int k = 0; k < 32; k += 4) {\n";
    src << "        const int i = (int)(i0 + k);\n";
    for (auto& st : ep.stores) src << "        ccb::V4<" << dt_ctype(g.ts[st.first].dt) << "> S" << st.first << ";\n";
    for (int j = 0; j < 4; ++j) {
      Emitter e(ep.ctx, src);
      e.ind = "        ";
      e.suffix = "_" + std::to_string(j);
      e.index_text = j == 0 ? "i" : "(i + " + std::to_string(j) + ")";
      e.direct[t] = "v[k + " + std::to_string(j) + "]";
      for (auto& st : ep.stores) {
        std::string val = e.val(st.second);
        src << "        S" << st.first << ".v[" << j << "] = " << val << ";\n";
      }
    }
    for (auto& st : ep.stores) src << "        ccb::st4(p.o" << st.first << " + i, S" << st.first << ");\n";
    if (store_c) src << "        *(float4*)(p.C + i) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);\n";
    src << "      }\n    } else {\n#pragma unroll\n      for (int k = 0; k < 32; ++k) {\n        if (k >= cnt) break;\n";
    src << "        const int i = (int)(i0 + k);\n";
    {
      Emitter e(ep.ctx, src);
      e.ind = "        ";
      e.direct[t] = "v[k]";
      for (auto& st : ep.stores) {
        std::string val = e.val(st.second);
        src << "        p.o" << st.first << "[i] = " << val << ";\n";
      }
    }
    if (store_c) src << "        p.C[i] = v[k];\n";
    src << "      }\n    }\n  }\n";
  }

  void emit_transpose(int gi) {
    Group& gr = groups[gi];
    const int t = gr.root, srcb = gr.val;
    const GTensor& x = g.ts[t];
    const char* T = dt_ctype(x.dt);
    const std::string F = "F" + std::to_string(gi);
    const std::string fn = "ccb_transpose_" + std::to_string(gi) + kname_suffix();
    node_buf[t] = add_buf("t" + std::to_string(x.uid), dt_size(x.dt), x.numel, BR_NODE, t, false);
    const int64_t R = x.shape[0], C = x.shape[1];  // output [R; C] = transpose of src [C; R]
    std::vector<Field> fields;
    fields.push_back(in_field(srcb));
    fields.push_back(out_field(t));
    fields.push_back(i64_field("rows", C));
    fields.push_back(i64_field("cols", R));
    src << "// transpose " << gi << ": n" << g.ts[srcb].uid << " [" << C << "x" << R << "] -> n" << x.uid << "\n";
    src << "struct " << F << " {\n";
    emit_struct(fields);
    src << "  typedef " << T << " T;\n";
    src << "  static __device__ __forceinline__ const T* src(const P& p) { return p.b" << srcb << "; }\n";
    src << "  static __device__ __forceinline__ T* dst(const P& p) { return p.o" << t << "; }\n";
    src << "};\n";
    src << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const " << F << "::P p) { ccb::transpose_tiles<" << F
        << ">(p); }\n\n";
    LaunchSpec& l = add_launch(fn, fields);
    l.mode = GM_PERSISTENT;
    l.work = ((R + 31) / 32) * ((C + 31) / 32);
    l.per_block = 1;
  }

  // Launch order. The ops of a run execute in one stream, so any order that
  // keeps every buffer hazard (two ops touching one buffer, at least one
  // writing it; the shared error word, only ever OR-ed into, is exempt)
  // computes the same bits. Among the ops whose predecessors have been
  // issued, one that writes a program output goes first (then graph order),
  // so a consumer of that output on another stream -- a gradient's
  // all-reduce, started from the event ccb_program_run_device_events records
  // after the output's last kernel -- overlaps the rest of the program: the
  // MLP step's dW2 product now runs right after dY, ahead of dA1, dZ1, dW1.
  void schedule_ops(Lowered& o) {
    const int n = (int)o.ops.size();
    std::vector<std::vector<std::pair<int, int>>> use(n);  // (buffer, access)
    for (int i = 0; i < n; ++i) {
      const OpSpec& op = o.ops[i];
      if (op.kind == OP_ZERO) {
        use[i].push_back({op.buf, 1});
        continue;
      }
      for (const Slot& sl : o.launches[op.launch].slots)
        if ((sl.kind == SL_BUF || sl.kind == SL_TMAP) && sl.buf >= 0 && sl.buf != o.err_buf) use[i].push_back({sl.buf, sl.access});
    }
    std::set<int> out_bufs;
    for (const IOSpec& io : o.outputs) out_bufs.insert(io.buf);
    std::vector<int> npred(n, 0), prio(n, 0);
    std::vector<std::vector<int>> succ(n);
    for (int j = 0; j < n; ++j) {
      for (auto& u : use[j])
        if (u.second != 0 && out_bufs.count(u.first)) prio[j] = 1;
      for (int i = 0; i < j; ++i) {
        bool dep = false;
        for (auto& a : use[i])
          for (auto& b : use[j])
            if (a.first == b.first && (a.second != 0 || b.second != 0)) dep = true;
        if (dep) {
          succ[i].push_back(j);
          ++npred[j];
        }
      }
    }
    std::vector<OpSpec> order;
    std::vector<char> done(n, 0);
    for (int k = 0; k < n; ++k) {
      int pick = -1;
      for (int i = 0; i < n; ++i)
        if (!done[i] && npred[i] == 0 && (pick < 0 || prio[i] > prio[pick])) pick = i;
      done[pick] = 1;
      order.push_back(o.ops[pick]);
      for (int j : succ[pick]) --npred[j];
    }
    o.ops = order;
  }

  void generate(Lowered& o) {
    out = &o;
    o.name = g.name;
    o.shard_rank = g.shard_rank;
    o.shard_world = g.shard_world;
    node_buf.assign(g.ts.size(), -1);
    o.err_buf = add_buf("err", 4, 1, BR_SCRATCH, -1, true);
    // params first, in graph order (lib/lower/lower.ml:977-987)
    std::set<std::string> seen;
    for (int t = 0; t < (int)g.ts.size(); ++t) {
      const GTensor& x = g.ts[t];
      if (x.kind != T_PARAM) continue;
      if (seen.count(x.name)) bad("Graph.create: two Param nodes named " + x.name);
      seen.insert(x.name);
      if (x.dt == DT_BOOL) bad("param " + x.name + ": Bool tensors are not storable");
      node_buf[t] = add_buf("p_" + x.name, dt_size(x.dt), x.numel, BR_PARAM, t, false);
      IOSpec io;
      io.name = x.name;
      io.dt = x.dt;
      io.shape = x.shape;
      io.buf = node_buf[t];
      io.bytes = x.numel * dt_size(x.dt);
      o.params.push_back(io);
    }
    src << "// generated by cudacaml-b200 for sm_100a: " << g.name << "\n#include \"ccb_skel.cuh\"\n\n";
    for (int gi = 0; gi < (int)groups.size(); ++gi) {
      if (g.shard_world > 1 && groups[gi].kind != G_MAPRED)
        unsupported("shard: a sharded program is one Monte-Carlo estimator pass (and scalar tails); pass " + std::to_string(gi) +
                    " is a scan, row reduction, scatter, product or transpose");
      switch (groups[gi].kind) {
        case G_MAPRED:
          if (groups[gi].fused_into < 0) emit_mapred(gi);
          break;
        case G_SCAN_FLAT:
        case G_SCAN_ROWS: emit_scan(gi); break;
        case G_RED_ROWS: emit_red_rows(gi); break;
        case G_SCATTER: emit_scatter(gi); break;
        case G_MATMUL: emit_matmul(gi); break;
        case G_MATMUL_TC: emit_matmul_tc(gi); break;
        case G_TRANSPOSE:
          if (groups[gi].fused_into < 0) emit_transpose(gi);
          break;
      }
    }
    if (g.shard_world > 1 && sharded_passes == 0) unsupported("shard: the program has no reduction pass to shard");
    for (auto& op : g.outputs) {
      const GTensor& x = g.ts[op.second];
      IOSpec io;
      io.name = op.first;
      io.dt = x.dt;
      io.shape = x.shape;
      io.buf = node_buf[op.second];
      io.bytes = x.numel * dt_size(x.dt);
      if (io.buf < 0) bad("lower: internal: output " + op.first + " has no buffer");
      o.outputs.push_back(io);
    }
    o.source = src.str();
    schedule_ops(o);
    // plan text
    std::ostringstream pt;
    for (size_t b = 0; b < o.bufs.size(); ++b) {
      const BufSpec& s = o.bufs[b];
      pt << "alloc " << s.label << " " << (s.role == BR_PARAM ? "param" : s.role == BR_NODE ? "node" : "scratch") << " "
         << s.numel << "x" << s.elem_bytes << "B" << (s.zero ? " zero" : "") << "\n";
    }
    for (auto& p : o.params) pt << "upload " << p.name << " -> " << o.bufs[p.buf].label << "\n";
    for (auto& op : o.ops) {
      if (op.kind == OP_ZERO) pt << "zero " << o.bufs[op.buf].label << "\n";
      else pt << "launch " << o.launches[op.launch].fn << "\n";
    }
    for (auto& p : o.outputs) pt << "download " << o.bufs[p.buf].label << " -> " << p.name << "\n";
    o.plan_text = pt.str();
  }
};

}  // namespace

int lower_graph(const GGraph& g, Lowered& out) {
  try {
    Lowerer L(g);
    L.analyse();
    L.group_all();
    L.fuse_epilogues();
    L.fuse_transposed_stores();
    L.generate(out);
  } catch (const LowerError& e) {
    return fail(e.code, e.what());
  } catch (const std::exception& e) {
    return fail(CCB_ERR_INVALID, std::string("lower: ") + e.what());
  }
  return CCB_OK;
}

}  // namespace ccb
