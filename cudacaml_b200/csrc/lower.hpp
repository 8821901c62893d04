// Graph wire format -> kernels + host plan.
//
// The replacement of the reference compiler: lib/lower/fusion.ml (which nodes
// own a buffer), lib/lower/lower.ml (per-root kernels and the host plan) and
// lib/backend_cuda/emit.ml (CUDA text). It targets the skeletons of skel.cuh.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace ccb {

enum Dt : int { DT_F32 = 0, DT_F64 = 1, DT_I32 = 2, DT_I64 = 3, DT_BOOL = 4 };
int dt_size(Dt d);
const char* dt_name(Dt d);
const char* dt_ctype(Dt d);

// Expression and tensor kinds of the wire format (lib/ir/expr.ml, lib/ir/tensor.ml).
enum EKind { E_CONST, E_ARG, E_INDEX, E_BINOP, E_UNOP, E_CMP, E_LOGIC, E_NOT, E_SELECT, E_CAST };
enum TKind { T_PARAM, T_IOTA, T_MAP, T_MAP2, T_REDUCE, T_SCAN, T_GATHER, T_SCATTER, T_MATMUL, T_RESHAPE, T_BROADCAST };
enum BinOp { B_ADD, B_SUB, B_MUL, B_DIV, B_MIN, B_MAX, B_AND, B_OR, B_XOR, B_SHL, B_SHR };
enum UnOp { U_NEG, U_SQRT, U_EXP, U_LOG, U_ABS, U_SIN, U_COS, U_ERF, U_ERFINV };
enum CmpOp { C_EQ, C_NE, C_LT, C_LE, C_GT, C_GE };

struct GExpr {
  Dt dt;
  int kind;
  int op = 0;
  int a = -1, b = -1, c = -1;
  double f = 0.0;   // float constant (exact double of the wire)
  int64_t i = 0;    // integer / bool constant, or Arg position
};

struct GTensor {
  int64_t uid;
  Dt dt;
  std::vector<int64_t> shape;
  int kind;
  std::string name;  // params
  int dep0 = -1, dep1 = -1;
  int arg0 = -1, arg1 = -1, body = -1, init = -1;
  int64_t numel = 1;
};

enum MatmulMode { MM_F32 = 0, MM_TF32 = 1 };

struct GGraph {
  std::string name;
  int matmul = MM_F32;  // wire "opt matmul": precision of F32 products
  // wire "opt shard <rank> <world>": this rank's slice of the program's one
  // Monte-Carlo estimator pass, combined across the world in its last block
  int shard_rank = 0, shard_world = 1;
  std::vector<GExpr> ex;
  std::vector<GTensor> ts;
  std::vector<std::pair<std::string, int>> outputs;
};

// Status code (CCB_*) and message through ccb::fail on error.
int parse_graph(const char* text, GGraph& g);

// ------------------------------------------------------------ lowered program
enum BufRole { BR_PARAM = 0, BR_NODE = 1, BR_SCRATCH = 2 };
struct BufSpec {
  std::string label;
  int elem_bytes = 4;
  int64_t numel = 0;
  int role = BR_SCRATCH;
  int node = -1;      // tensor index for params and nodes
  bool zero = false;  // zero-filled once at allocation
};

// SL_TMAP: a 128-byte TMA tensor map (16 words, 64-byte aligned in the
// parameter block) over buffer `buf`, 2-D fp32, swizzle `tswizzle`: inner
// extent tdim[0], outer tdim[1], outer stride tstride bytes, box tbox[0] x
// tbox[1]. The executor encodes it against the buffer the run binds.
// SL_XMB: the mailbox of rank `val` of a sharded program (as bound by
// ccb_program_bind_peers); SL_XEPOCH: the program's cross-rank epoch of this
// run (1, 2, 3, ... per run, the same on every rank).
enum SlotKind { SL_BUF = 0, SL_I64 = 1, SL_EPOCH = 2, SL_TMAP = 3, SL_XMB = 4, SL_XEPOCH = 5 };
struct Slot {
  int kind = SL_BUF;
  int buf = -1;
  // how the kernel uses `buf` (SL_BUF, SL_TMAP): 0 reads it, 1 writes it,
  // 2 both or unknown; the launch scheduler keeps every hazard it implies
  int access = 2;
  int64_t val = 0;
  int64_t tdim[3] = {0, 0, 1};
  int64_t tstride = 0, tstride2 = 0;  // bytes between dim-1 / dim-2 steps
  int tbox[3] = {0, 0, 1};
  int trank = 2;
  int tswizzle = 3;  // CUtensorMapSwizzle: 3 = 128B, 4 = 128B with 32-byte atoms
};

enum GridMode { GM_FIXED = 0, GM_PERSISTENT = 1 };
struct LaunchSpec {
  std::string fn;
  int mode = GM_FIXED;
  int64_t gx = 1, gy = 1;
  int64_t work = 0;            // persistent: work items
  int64_t per_block = 1;       // persistent: items one block iteration covers
  int64_t max_grid = 1 << 30;  // persistent: cap (scratch is sized for it)
  int block = 256;
  int smem = 0;  // dynamic shared memory bytes
  int grid_multiple = 1;  // persistent grids: the grid is a multiple of this (cluster size)
  // map-reduce passes that stream element data: after a spill relaxes their
  // bound, one more resident block is tried (latency hiding pays for
  // streams; an instruction-bound estimator runs faster at its own occupancy)
  bool streams = false;
  std::vector<Slot> slots;
};

enum OpKind { OP_LAUNCH = 0, OP_ZERO = 1 };
struct OpSpec {
  int kind = OP_LAUNCH;
  int launch = -1;
  int buf = -1;
};

struct IOSpec {
  std::string name;
  Dt dt;
  std::vector<int64_t> shape;
  int buf = -1;
  int64_t bytes = 0;
};

struct Lowered {
  std::string name;
  std::string source;
  std::vector<BufSpec> bufs;
  std::vector<LaunchSpec> launches;
  std::vector<OpSpec> ops;
  std::vector<IOSpec> params, outputs;
  int err_buf = -1;
  int num_kernels = 0;
  int shard_rank = 0, shard_world = 1;  // see GGraph
  std::string plan_text;
};

int lower_graph(const GGraph& g, Lowered& out);

}  // namespace ccb
