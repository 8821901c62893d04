// ORACLE -- test infrastructure only. Nothing in the product (cudacaml_b200/,
// libccb.so) links, loads or calls this file; only tests/, the smoke check and
// bench.py's cpu_baseline leg do, and only as the checker.
//
// A C++ restatement of CUDACaml's pure-OCaml reference interpreter,
// lib/backend_interp/cudacaml_backend_interp.ml, over the graph wire format of
// cudacaml_b200/wire.py. It follows the interpreter's semantics exactly:
//   * every F32 result is computed in double and rounded to single precision
//     (round_f32, cudacaml_backend_interp.ml:36, 61, 160);
//   * integers wrap, shift counts are masked, Shr is logical (ml:63-91);
//   * erfinv is Giles' single-precision polynomial plus two Newton steps on
//     libm erf (ml:98-143); exp/log/sin/cos/erf are glibc libm, which is what
//     OCaml's Stdlib binds;
//   * casts go through double (floats) or int64 (integers) (ml:198-237);
//   * Reduce/Scan/Scatter_add/Matmul are strictly sequential folds in ascending
//     index order (ml:335-433); Gather/Scatter_add are bounds-checked (ml:371-406);
//   * every tensor node is evaluated once and memoised by uid (ml:296-307).
// Element functions are evaluated lazily (Select evaluates only the branch it
// takes, ml:255-256) with a per-element memo over the expression DAG.
//
// Build: see oracle/Makefile (g++ -O2 -ffp-contract=off, no fast-math).
#include <cctype>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

enum Dt { F32 = 0, F64 = 1, I32 = 2, I64 = 3, BOOLT = 4 };

Dt parse_dt(const std::string& s) {
  if (s == "f32") return F32;
  if (s == "f64") return F64;
  if (s == "i32") return I32;
  if (s == "i64") return I64;
  if (s == "bool") return BOOLT;
  throw std::runtime_error("oracle: unknown dtype " + s);
}
const char* dt_name(Dt d) {
  static const char* n[] = {"f32", "f64", "i32", "i64", "bool"};
  return n[d];
}
int dt_size(Dt d) { return (d == F32 || d == I32) ? 4 : (d == BOOLT ? 1 : 8); }
bool is_float(Dt d) { return d == F32 || d == F64; }

// One scalar: floats in f (an F32 value is always exactly representable),
// integers and booleans in i (I32 sign-extended).
struct S {
  double f = 0.0;
  int64_t i = 0;
};

double round_f32(double x) { return (double)(float)x; }

// OCaml's Float.min / Float.max (stdlib float.ml): NaN-propagating, and
// min(-0, +0) = -0, max(-0, +0) = +0.
double ocaml_fmin(double x, double y) {
  if (y > x || (!std::signbit(y) && std::signbit(x))) return std::isnan(y) ? y : x;
  return std::isnan(x) ? x : y;
}
double ocaml_fmax(double x, double y) {
  if (y > x || (!std::signbit(y) && std::signbit(x))) return std::isnan(x) ? x : y;
  return std::isnan(y) ? y : x;
}

// Giles, "Approximating the erfinv function" (GPU Computing Gems, 2010),
// single-precision branch, as the interpreter uses it for its starting point
// (cudacaml_backend_interp.ml:100-126), then two Newton steps (128-143).
double erfinv_guess(double x) {
  double w = -std::log((1.0 - x) * (1.0 + x));
  double p;
  if (w < 5.0) {
    w = w - 2.5;
    p = 2.81022636e-08;
    p = 3.43273939e-07 + p * w;
    p = -3.5233877e-06 + p * w;
    p = -4.39150654e-06 + p * w;
    p = 0.00021858087 + p * w;
    p = -0.00125372503 + p * w;
    p = -0.00417768164 + p * w;
    p = 0.246640727 + p * w;
    p = 1.50140941 + p * w;
  } else {
    w = std::sqrt(w) - 3.0;
    p = -0.000200214257;
    p = 0.000100950558 + p * w;
    p = 0.00134934322 + p * w;
    p = -0.00367342844 + p * w;
    p = 0.00573950773 + p * w;
    p = -0.0076224613 + p * w;
    p = 0.00943887047 + p * w;
    p = 1.00167406 + p * w;
    p = 2.83297682 + p * w;
  }
  return p * x;
}

double ocaml_erfinv(double x) {
  static const double two_over_sqrt_pi = 2.0 / std::sqrt(M_PI);
  if (std::isnan(x)) return x;
  if (x == 1.0) return INFINITY;
  if (x == -1.0) return -INFINITY;
  if (std::fabs(x) > 1.0) return NAN;
  if (x == 0.0) return x;
  double y = erfinv_guess(x);
  for (int k = 0; k < 2; ++k) {
    double d = two_over_sqrt_pi * std::exp(-(y * y));
    if (d != 0.0) y = y - (std::erf(y) - x) / d;
  }
  return y;
}

// Int64.of_float on amd64 (cvttsd2si): truncation, and the "integer
// indefinite" value for NaN and out-of-range inputs.
int64_t ocaml_int64_of_float(double x) {
  if (std::isnan(x) || x >= 9223372036854775808.0 || x < -9223372036854775808.0) return INT64_MIN;
  return (int64_t)x;
}
int64_t wrap32(int64_t v) { return (int64_t)(int32_t)(uint32_t)(uint64_t)v; }

struct ExprNode {
  Dt dt;
  std::string kind, op;
  int a = -1, b = -1, c = -1;  // child expression indices
  S cval;
  int argi = 0;
};

struct TensorNode {
  int64_t uid;
  Dt dt;
  std::vector<int64_t> shape;
  std::string kind, name;
  std::vector<int> deps;  // indices into tensors
  int arg0 = -1, arg1 = -1, body = -1, init = -1;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

struct Value {
  Dt dt;
  std::vector<int64_t> shape;
  std::vector<uint8_t> bytes;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  void alloc() { bytes.assign((size_t)numel() * dt_size(dt), 0); }
  S get(int64_t k) const {
    S s;
    const uint8_t* p = bytes.data();
    switch (dt) {
      case F32: s.f = ((const float*)p)[k]; break;
      case F64: s.f = ((const double*)p)[k]; break;
      case I32: s.i = ((const int32_t*)p)[k]; break;
      case I64: s.i = ((const int64_t*)p)[k]; break;
      default: throw std::runtime_error("oracle: bool value");
    }
    return s;
  }
  void set(int64_t k, S s) {
    uint8_t* p = bytes.data();
    switch (dt) {
      case F32: ((float*)p)[k] = (float)s.f; break;
      case F64: ((double*)p)[k] = s.f; break;
      case I32: ((int32_t*)p)[k] = (int32_t)s.i; break;
      case I64: ((int64_t*)p)[k] = s.i; break;
      default: throw std::runtime_error("oracle: bool value");
    }
  }
};

struct Graph {
  std::string name;
  std::vector<ExprNode> exprs;
  std::vector<TensorNode> tensors;
  std::vector<std::pair<std::string, int>> outputs;
  // run results
  std::vector<Value> results;
  std::string last_error;
};

// ---------------------------------------------------------------- parsing
// A name is one token on the wire with '%', whitespace and control bytes
// written as %XX and the empty name as a lone '%'; decode it back to the
// caller's bytes.
std::string wire_name(const std::string& s) {
  if (s == "%") return std::string();
  std::string out;
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i] != '%') {
      out += s[i];
      continue;
    }
    if (i + 2 >= s.size() || !std::isxdigit((unsigned char)s[i + 1]) || !std::isxdigit((unsigned char)s[i + 2]))
      throw std::runtime_error("oracle: bad %XX escape in name " + s);
    out += (char)std::stoi(s.substr(i + 1, 2), nullptr, 16);
    i += 2;
  }
  return out;
}

void parse(Graph& g, const char* text) {
  std::istringstream in(text);
  std::string line;
  std::unordered_map<int64_t, int> eidx, tidx;
  bool header = false, ended = false;
  auto E = [&](int64_t id) {
    auto it = eidx.find(id);
    if (it == eidx.end()) throw std::runtime_error("oracle: unknown expression id " + std::to_string(id));
    return it->second;
  };
  auto T = [&](int64_t id) {
    auto it = tidx.find(id);
    if (it == tidx.end()) throw std::runtime_error("oracle: unknown tensor id " + std::to_string(id));
    return it->second;
  };
  while (std::getline(in, line)) {
    if (line.empty()) continue;
    std::istringstream ls(line);
    std::string tag;
    ls >> tag;
    if (tag == "ccbgraph") {
      header = true;
    } else if (tag == "name") {
      ls >> g.name;
      g.name = wire_name(g.name);
    } else if (tag == "e") {
      int64_t id;
      std::string dts, kind;
      ls >> id >> dts >> kind;
      ExprNode n;
      n.dt = parse_dt(dts);
      n.kind = kind;
      if (kind == "const") {
        std::string v;
        ls >> v;
        if (is_float(n.dt)) {
          uint64_t bits = std::stoull(v, nullptr, 16);
          std::memcpy(&n.cval.f, &bits, 8);
        } else {
          n.cval.i = std::stoll(v);
        }
      } else if (kind == "arg") {
        ls >> n.argi;
      } else if (kind == "index") {
      } else if (kind == "binop" || kind == "cmp" || kind == "logic") {
        int64_t a, b;
        ls >> n.op >> a >> b;
        n.a = E(a);
        n.b = E(b);
      } else if (kind == "unop") {
        int64_t a;
        ls >> n.op >> a;
        n.a = E(a);
      } else if (kind == "not" || kind == "cast") {
        int64_t a;
        ls >> a;
        n.a = E(a);
      } else if (kind == "select") {
        int64_t c, a, b;
        ls >> c >> a >> b;
        n.a = E(c);
        n.b = E(a);
        n.c = E(b);
      } else {
        throw std::runtime_error("oracle: unknown expression kind " + kind);
      }
      eidx[id] = (int)g.exprs.size();
      g.exprs.push_back(n);
    } else if (tag == "t") {
      TensorNode t;
      std::string dts;
      int rank;
      ls >> t.uid >> dts >> rank;
      t.dt = parse_dt(dts);
      t.shape.resize(rank);
      for (int k = 0; k < rank; ++k) ls >> t.shape[k];
      ls >> t.kind;
      int64_t a, b, x, y, z, w;
      if (t.kind == "param") {
        ls >> t.name;
        t.name = wire_name(t.name);
      } else if (t.kind == "iota") {
      } else if (t.kind == "map") {
        ls >> a >> x >> z;
        t.deps = {T(a)};
        t.arg0 = E(x);
        t.body = E(z);
      } else if (t.kind == "map2") {
        ls >> a >> b >> x >> y >> z;
        t.deps = {T(a), T(b)};
        t.arg0 = E(x);
        t.arg1 = E(y);
        t.body = E(z);
      } else if (t.kind == "reduce" || t.kind == "scan") {
        ls >> a >> x >> y >> z >> w;
        t.deps = {T(a)};
        t.arg0 = E(x);
        t.arg1 = E(y);
        t.body = E(z);
        t.init = E(w);
      } else if (t.kind == "gather" || t.kind == "scatter_add" || t.kind == "matmul") {
        ls >> a >> b;
        t.deps = {T(a), T(b)};
      } else if (t.kind == "reshape" || t.kind == "broadcast") {
        ls >> a;
        t.deps = {T(a)};
      } else {
        throw std::runtime_error("oracle: unknown tensor kind " + t.kind);
      }
      tidx[t.uid] = (int)g.tensors.size();
      g.tensors.push_back(t);
    } else if (tag == "o") {
      std::string nm;
      int64_t id;
      ls >> nm >> id;
      g.outputs.push_back({wire_name(nm), T(id)});
    } else if (tag == "end") {
      ended = true;
    } else {
      throw std::runtime_error("oracle: bad line: " + line);
    }
  }
  if (!header || !ended) throw std::runtime_error("oracle: truncated graph text");
}

// ------------------------------------------------------ scalar semantics
S binop(Dt d, const std::string& op, S x, S y) {
  S r;
  if (is_float(d)) {
    double a = x.f, b = y.f, v;
    if (op == "add") v = a + b;
    else if (op == "sub") v = a - b;
    else if (op == "mul") v = a * b;
    else if (op == "div") v = a / b;
    else if (op == "min") v = ocaml_fmin(a, b);
    else if (op == "max") v = ocaml_fmax(a, b);
    else throw std::invalid_argument("Backend_interp: " + op + " on a float dtype");
    r.f = (d == F32) ? round_f32(v) : v;
    return r;
  }
  if (d == I32 || d == I64) {
    const bool w32 = (d == I32);
    const int64_t a = x.i, b = y.i;
    const uint64_t ua = (uint64_t)a, ub = (uint64_t)b;
    int64_t v;
    if (op == "add") v = (int64_t)(ua + ub);
    else if (op == "sub") v = (int64_t)(ua - ub);
    else if (op == "mul") v = (int64_t)(ua * ub);
    else if (op == "div") {
      if (b == 0) throw std::domain_error("Division_by_zero");
      if (w32) v = (a == INT32_MIN && b == -1) ? INT32_MIN : a / b;
      else v = (a == INT64_MIN && b == -1) ? INT64_MIN : a / b;
    } else if (op == "min") v = a < b ? a : b;
    else if (op == "max") v = a > b ? a : b;
    else if (op == "bit_and") v = a & b;
    else if (op == "bit_or") v = a | b;
    else if (op == "bit_xor") v = a ^ b;
    else if (op == "shl") {
      v = w32 ? (int64_t)(int32_t)((uint32_t)a << (b & 31)) : (int64_t)(ua << (b & 63));
    } else if (op == "shr") {
      v = w32 ? (int64_t)(int32_t)((uint32_t)a >> (b & 31)) : (int64_t)(ua >> (b & 63));
    } else throw std::invalid_argument("Backend_interp: unknown binop " + op);
    r.i = w32 ? wrap32(v) : v;
    return r;
  }
  throw std::invalid_argument("Backend_interp: binop on bool");
}

S unop(Dt d, const std::string& op, S x) {
  S r;
  if (is_float(d)) {
    double a = x.f, v;
    if (op == "neg") v = -a;
    else if (op == "sqrt") v = std::sqrt(a);
    else if (op == "exp") v = std::exp(a);
    else if (op == "log") v = std::log(a);
    else if (op == "abs") v = std::fabs(a);
    else if (op == "sin") v = std::sin(a);
    else if (op == "cos") v = std::cos(a);
    else if (op == "erf") v = std::erf(a);
    else if (op == "erfinv") v = ocaml_erfinv(a);
    else throw std::invalid_argument("Backend_interp: unknown unop " + op);
    r.f = (d == F32) ? round_f32(v) : v;
    return r;
  }
  if (d == I32 || d == I64) {
    const bool w32 = (d == I32);
    int64_t a = x.i, v;
    if (op == "neg") v = (int64_t)(0 - (uint64_t)a);
    else if (op == "abs") v = a >= 0 ? a : (int64_t)(0 - (uint64_t)a);
    else throw std::invalid_argument(std::string("Backend_interp: ") + op + " on " + dt_name(d));
    r.i = w32 ? wrap32(v) : v;
    return r;
  }
  throw std::invalid_argument("Backend_interp: unop on bool");
}

bool cmp(Dt d, const std::string& op, S x, S y) {
  if (is_float(d)) {
    double a = x.f, b = y.f;
    if (op == "eq") return a == b;
    if (op == "ne") return a != b;
    if (op == "lt") return a < b;
    if (op == "le") return a <= b;
    if (op == "gt") return a > b;
    if (op == "ge") return a >= b;
  } else {
    int64_t a = x.i, b = y.i;
    if (op == "eq") return a == b;
    if (op == "ne") return a != b;
    if (op == "lt") return a < b;
    if (op == "le") return a <= b;
    if (op == "gt") return a > b;
    if (op == "ge") return a >= b;
  }
  throw std::invalid_argument("Backend_interp: unknown comparison " + op);
}

S cast(Dt from, Dt to, S x) {
  if (from == to) return x;
  S r;
  if (is_float(from)) {  // of_float
    double v = x.f;
    switch (to) {
      case F32: r.f = round_f32(v); break;
      case F64: r.f = v; break;
      case I32: r.i = wrap32(ocaml_int64_of_float(v)); break;
      case I64: r.i = ocaml_int64_of_float(v); break;
      case BOOLT: r.i = (v != 0.0); break;
    }
    return r;
  }
  if (from == I32 || from == I64) {  // of_int64
    int64_t v = x.i;
    switch (to) {
      case F32: r.f = round_f32((double)v); break;
      case F64: r.f = (double)v; break;
      case I32: r.i = wrap32(v); break;
      case I64: r.i = v; break;
      case BOOLT: r.i = (v != 0); break;
    }
    return r;
  }
  // of_bool
  switch (to) {
    case F32:
    case F64: r.f = x.i ? 1.0 : 0.0; break;
    default: r.i = x.i ? 1 : 0; break;
  }
  return r;
}

// ------------------------------------------------------ element functions
// Lazy, memoised evaluation of one element function over the expression DAG.
struct Evaluator {
  const std::vector<ExprNode>& ex;
  std::vector<S> val;
  std::vector<uint64_t> gen;
  uint64_t cur = 0;
  S env[2];
  int nenv = 0;
  int64_t index = 0;
  int arg_dt[2] = {-1, -1};
  explicit Evaluator(const std::vector<ExprNode>& e) : ex(e), val(e.size()), gen(e.size(), 0) {}

  void begin(int64_t idx, int n, const S* args, const Dt* dts) {
    ++cur;
    index = idx;
    nenv = n;
    for (int k = 0; k < n; ++k) {
      env[k] = args[k];
      arg_dt[k] = dts[k];
    }
  }
  S eval(int e) {
    if (gen[e] == cur) return val[e];
    const ExprNode& n = ex[e];
    S r;
    if (n.kind == "const") {
      r = n.cval;
    } else if (n.kind == "arg") {
      if (n.argi >= nenv) throw std::invalid_argument("Backend_interp: Arg " + std::to_string(n.argi) + " is unbound");
      if (arg_dt[n.argi] != n.dt) throw std::invalid_argument("Backend_interp: Arg dtype mismatch");
      r = env[n.argi];
    } else if (n.kind == "index") {
      r.i = wrap32(index);
    } else if (n.kind == "binop") {
      S a = eval(n.a), b = eval(n.b);
      r = binop(n.dt, n.op, a, b);
    } else if (n.kind == "unop") {
      r = unop(n.dt, n.op, eval(n.a));
    } else if (n.kind == "cmp") {
      S a = eval(n.a), b = eval(n.b);
      r.i = cmp(ex[n.a].dt, n.op, a, b);
    } else if (n.kind == "logic") {
      // OCaml's && and || short-circuit (ml:252-253).
      bool a = eval(n.a).i != 0;
      if (n.op == "and") r.i = a ? (eval(n.b).i != 0) : 0;
      else r.i = a ? 1 : (eval(n.b).i != 0);
    } else if (n.kind == "not") {
      r.i = !(eval(n.a).i != 0);
    } else if (n.kind == "select") {
      r = (eval(n.a).i != 0) ? eval(n.b) : eval(n.c);
    } else if (n.kind == "cast") {
      r = cast(ex[n.a].dt, n.dt, eval(n.a));
    } else {
      throw std::runtime_error("oracle: bad expression kind");
    }
    val[e] = r;
    gen[e] = cur;
    return r;
  }
};

int64_t row_length(const std::vector<int64_t>& shape) { return shape.empty() ? 1 : shape.back(); }

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t k = 0; k < s.size(); ++k) r += (k ? "," : "") + std::to_string(s[k]);
  return r + "]";
}

void run(Graph& g, const std::map<std::string, const Value*>& inputs, std::vector<Value>& vals) {
  vals.assign(g.tensors.size(), Value());
  Evaluator ev(g.exprs);
  for (size_t ti = 0; ti < g.tensors.size(); ++ti) {
    const TensorNode& t = g.tensors[ti];
    Value& out = vals[ti];
    out.dt = t.dt;
    out.shape = t.shape;
    const int64_t N = t.numel();
    if (t.kind == "param") {
      auto it = inputs.find(t.name);
      if (it == inputs.end()) throw std::invalid_argument("Backend_interp: missing input \"" + t.name + "\"");
      const Value* v = it->second;
      if (v->dt != t.dt)
        throw std::invalid_argument("Backend_interp: input \"" + t.name + "\" has dtype " + dt_name(v->dt) +
                                    ", expected " + dt_name(t.dt));
      if (v->shape != t.shape)
        throw std::invalid_argument("Backend_interp: input \"" + t.name + "\" has shape " + shape_str(v->shape) +
                                    ", expected " + shape_str(t.shape));
      out = *v;
      continue;
    }
    if (t.dt == BOOLT) throw std::invalid_argument("Value.create: Bool tensors are not storable");
    out.alloc();
    if (t.kind == "iota") {
      for (int64_t i = 0; i < N; ++i) {
        S s;
        s.i = wrap32(i);
        out.set(i, s);
      }
    } else if (t.kind == "map") {
      const Value& src = vals[t.deps[0]];
      Dt dts[1] = {src.dt};
      for (int64_t i = 0; i < N; ++i) {
        S a = src.get(i);
        ev.begin(i, 1, &a, dts);
        out.set(i, ev.eval(t.body));
      }
    } else if (t.kind == "map2") {
      const Value& va = vals[t.deps[0]];
      const Value& vb = vals[t.deps[1]];
      Dt dts[2] = {va.dt, vb.dt};
      for (int64_t i = 0; i < N; ++i) {
        S a[2] = {va.get(i), vb.get(i)};
        ev.begin(i, 2, a, dts);
        out.set(i, ev.eval(t.body));
      }
    } else if (t.kind == "reduce") {
      const Value& src = vals[t.deps[0]];
      const int64_t n = row_length(src.shape);
      const int64_t rows = N;
      Dt dts[2] = {src.dt, src.dt};
      for (int64_t r = 0; r < rows; ++r) {
        ev.begin(0, 0, nullptr, dts);
        S acc = ev.eval(t.init);
        for (int64_t j = 0; j < n; ++j) {
          const int64_t i = r * n + j;
          S a[2] = {acc, src.get(i)};
          ev.begin(i, 2, a, dts);
          acc = ev.eval(t.body);
        }
        out.set(r, acc);
      }
    } else if (t.kind == "scan") {
      const Value& src = vals[t.deps[0]];
      const int64_t n = row_length(src.shape);
      const int64_t rows = n == 0 ? 0 : src.numel() / n;
      Dt dts[2] = {src.dt, src.dt};
      for (int64_t r = 0; r < rows; ++r) {
        ev.begin(0, 0, nullptr, dts);
        S acc = ev.eval(t.init);
        for (int64_t j = 0; j < n; ++j) {
          const int64_t i = r * n + j;
          S a[2] = {acc, src.get(i)};
          ev.begin(i, 2, a, dts);
          acc = ev.eval(t.body);
          out.set(i, acc);
        }
      }
    } else if (t.kind == "gather") {
      const Value& idx = vals[t.deps[0]];
      const Value& src = vals[t.deps[1]];
      const int64_t n = src.numel();
      for (int64_t i = 0; i < N; ++i) {
        const int64_t j = idx.get(i).i;
        if (j < 0 || j >= n)
          throw std::invalid_argument("Backend_interp: gather index out of bounds: " + std::to_string(j) + " at " +
                                      std::to_string(i) + " (source has " + std::to_string(n) + " elements)");
        out.set(i, src.get(j));
      }
    } else if (t.kind == "scatter_add") {
      const Value& idx = vals[t.deps[0]];
      const Value& src = vals[t.deps[1]];
      const int64_t m = N;
      for (int64_t i = 0; i < src.numel(); ++i) {
        const int64_t j = idx.get(i).i;
        if (j < 0 || j >= m)
          throw std::invalid_argument("Backend_interp: scatter_add index out of bounds: " + std::to_string(j) +
                                      " at " + std::to_string(i) + " (output has " + std::to_string(m) + " elements)");
        out.set(j, binop(t.dt, "add", out.get(j), src.get(i)));
      }
    } else if (t.kind == "matmul") {
      const Value& va = vals[t.deps[0]];
      const Value& vb = vals[t.deps[1]];
      const int64_t k = row_length(va.shape);
      const int64_t n = row_length(t.shape);
      const int64_t rows = n == 0 ? 0 : N / n;
      S zero = cast(I64, t.dt, S());
      for (int64_t i = 0; i < rows; ++i)
        for (int64_t j = 0; j < n; ++j) {
          S acc = zero;
          for (int64_t p = 0; p < k; ++p)
            acc = binop(t.dt, "add", acc, binop(t.dt, "mul", va.get(i * k + p), vb.get(p * n + j)));
          out.set(i * n + j, acc);
        }
    } else if (t.kind == "reshape") {
      const Value& src = vals[t.deps[0]];
      for (int64_t i = 0; i < N; ++i) out.set(i, src.get(i));
    } else if (t.kind == "broadcast") {
      const Value& src = vals[t.deps[0]];
      S x = src.get(0);
      for (int64_t i = 0; i < N; ++i) out.set(i, x);
    } else {
      throw std::runtime_error("oracle: unknown tensor kind " + t.kind);
    }
  }
}

void set_err(char* err, int errlen, const std::string& m) {
  if (err && errlen > 0) {
    std::strncpy(err, m.c_str(), errlen - 1);
    err[errlen - 1] = 0;
  }
}

}  // namespace

// ------------------------------------------------------------- C-ABI
extern "C" {

void* ccbo_load(const char* text, char* err, int errlen) {
  auto g = std::make_unique<Graph>();
  try {
    parse(*g, text);
  } catch (const std::exception& e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
  return g.release();
}

void ccbo_free(void* h) { delete (Graph*)h; }

// dtypes: 0 f32, 1 f64, 2 i32, 3 i64. Returns 0 on success, 1 on an
// Invalid_argument-class error, 2 on Division_by_zero, 3 otherwise.
int ccbo_run(void* h, int n_inputs, const char** names, const int* dtypes, const int* ranks,
             const long long* dims, const void** data, char* err, int errlen) {
  Graph& g = *(Graph*)h;
  std::vector<Value> ins(n_inputs);
  std::map<std::string, const Value*> by_name;
  const long long* dp = dims;
  for (int k = 0; k < n_inputs; ++k) {
    Value& v = ins[k];
    v.dt = (Dt)dtypes[k];
    v.shape.assign(dp, dp + ranks[k]);
    dp += ranks[k];
    v.alloc();
    if (!v.bytes.empty()) std::memcpy(v.bytes.data(), data[k], v.bytes.size());
    by_name[names[k]] = &v;
  }
  std::vector<Value> vals;
  try {
    run(g, by_name, vals);
  } catch (const std::invalid_argument& e) {
    set_err(err, errlen, e.what());
    return 1;
  } catch (const std::domain_error& e) {
    set_err(err, errlen, e.what());
    return 2;
  } catch (const std::exception& e) {
    set_err(err, errlen, e.what());
    return 3;
  }
  g.results.clear();
  for (auto& o : g.outputs) g.results.push_back(vals[o.second]);
  return 0;
}

int ccbo_num_outputs(void* h) { return (int)((Graph*)h)->outputs.size(); }
const char* ccbo_output_name(void* h, int i) { return ((Graph*)h)->outputs[i].first.c_str(); }
int ccbo_output_dtype(void* h, int i) { return (int)((Graph*)h)->results[i].dt; }
int ccbo_output_rank(void* h, int i) { return (int)((Graph*)h)->results[i].shape.size(); }
long long ccbo_output_dim(void* h, int i, int k) { return ((Graph*)h)->results[i].shape[k]; }
const void* ccbo_output_data(void* h, int i) { return ((Graph*)h)->results[i].bytes.data(); }
long long ccbo_output_bytes(void* h, int i) { return (long long)((Graph*)h)->results[i].bytes.size(); }

// Philox-4x32-10 on raw words, for the known-answer tests. Written here in
// plain integer C so the KATs pin the constants independently of the graph
// path (test/unit/test_rng.ml:73-86 in the reference).
void ccbo_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c[4] = {ctr_in[0], ctr_in[1], ctr_in[2], ctr_in[3]};
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 1; r <= 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n1 = lo1, n2 = hi0 ^ c[3] ^ k1, n3 = lo0;
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    if (r < 10) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
  }
  for (int k = 0; k < 4; ++k) out[k] = c[k];
}

double ccbo_erfinv(double x) { return ocaml_erfinv(x); }
}
