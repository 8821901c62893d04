// Compiled programs: NVRTC + module load + per-lane buffer pools, and the
// stream-ordered execution of the host plan. Replaces the reference's
// Backend_cuda.compile_on (lib/backend_cuda/cudacaml_backend_cuda.ml:30-43) and
// Executor (lib/backend_cuda/executor.ml:72-244).
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <unordered_map>

#include "common.hpp"
#include "lower.hpp"

namespace ccb {
void live_add(long long d);
}

namespace {
using namespace ccb;

struct Lane {
  CUstream stream = nullptr;
  CUevent done = nullptr;
  std::vector<CUdeviceptr> bufs;
  unsigned* host_err = nullptr;  // pinned slot the error word is copied to
  bool err_pending = false;      // resident runs since the last copy of the word
  uint64_t epoch = 0;
  // Encoded tensor maps, keyed by (launch, slot), with the base they encode.
  std::unordered_map<int64_t, std::pair<CUdeviceptr, CUtensorMap>> tmaps;
};

struct Program {
  Lowered L;
  int device = -1;
  CUmodule mod = nullptr;
  std::vector<CUfunction> fns;
  std::vector<unsigned> gx, gy;
  std::vector<Lane> lanes;
  int num_launch_ops = 0;
  // Sharded programs: every rank's mailbox as this rank addresses it, and the
  // cross-rank epoch of the last run (ccb_program_bind_peers resets it).
  std::vector<CUdeviceptr> peers;
  uint64_t xepoch = 0;
};

// Words of one mailbox slot of a sharded program (flag + 32 values) and the
// whole mailbox of a world: ccb::XSLOT_WORDS in the skeleton header.
constexpr int kXslotWords = 33;
size_t mailbox_bytes(int world) { return (size_t)2 * world * kXslotWords * sizeof(uint64_t); }

// The device error word of a lane accumulates over runs until a check
// reports it; then it is cleared, so a chain of runs checked once reports any
// error raised anywhere in the chain. Runs with host buffers copy the word to
// the lane's pinned slot as their last step; device-resident runs only mark
// it pending (no copy between their kernels). An explicit check (`fresh`)
// always reads the word once `stream` has drained, which also covers runs
// replayed from a captured graph.
int lane_check(Program& P, int lane, CUstream stream, bool fresh) {
  Lane& lnp = P.lanes[lane];
  if (lnp.err_pending || fresh) {
    const Driver& d = driver();
    CCB_CU(d.cuMemcpyDtoHAsync(lnp.host_err, lnp.bufs[P.L.err_buf], 4, stream));
    CCB_CU(d.cuStreamSynchronize(stream));
    lnp.err_pending = false;
  }
  const unsigned e = *P.lanes[lane].host_err;
  if (e == 0) return CCB_OK;
  {
    const Driver& d = driver();
    Lane& ln = P.lanes[lane];
    CCB_CU(d.cuMemsetD8Async(ln.bufs[P.L.err_buf], 0, 4, ln.stream));
    CCB_CU(d.cuStreamSynchronize(ln.stream));
  }
  std::string m = "device check failed:";
  if (e & 1u) m += " gather index out of bounds;";
  if (e & 2u) m += " scatter_add index out of bounds;";
  if (e & 4u) m += " scan look-back wait gave up (bounded spin exhausted);";
  if (e & 8u) m += " bulk-copy (TMA) wait gave up (bounded spin exhausted);";
  if (e & 16u) m += " tensor-core pipeline wait gave up (bounded spin exhausted);";
  if (e & 32u) m += " cross-rank combine gave up: a peer rank did not publish its totals (bounded wait);";
  *P.lanes[lane].host_err = 0;
  return fail(CCB_ERR_DEVICE_CHECK, m);
}

int64_t buf_bytes(const BufSpec& b) { return b.numel * (int64_t)b.elem_bytes; }

int destroy(Program* P) {
  if (!P) return CCB_OK;
  if (P->device >= 0 && driver().ok && ensure_context(P->device) == CCB_OK) {
    const Driver& d = driver();
    for (Lane& l : P->lanes) {
      if (l.stream) d.cuStreamSynchronize(l.stream);
      for (CUdeviceptr b : l.bufs)
        if (b) {
          d.cuMemFree(b);
          live_add(-1);
        }
      if (l.host_err) d.cuMemFreeHost(l.host_err);
      if (l.done) d.cuEventDestroy(l.done);
      if (l.stream) d.cuStreamDestroy(l.stream);
    }
    if (P->mod) d.cuModuleUnload(P->mod);
  }
  delete P;
  return CCB_OK;
}

// The TMA tensor map of slot `sl` over the buffer at `base`, encoded once per
// (lane, launch, slot, base). A base that is not 16-byte aligned cannot be
// described to the copy engine and is rejected.
int tensor_map(Lane& ln, int64_t key, const Slot& sl, CUdeviceptr base, const CUtensorMap*& out) {
  auto it = ln.tmaps.find(key);
  if (it != ln.tmaps.end() && it->second.first == base) {
    out = &it->second.second;
    return CCB_OK;
  }
  if (base & 15)
    return fail(CCB_ERR_INVALID, "tensor-core matmul operand at a device address that is not 16-byte aligned");
  CUtensorMap m;
  const cuuint64_t dims[3] = {(cuuint64_t)sl.tdim[0], (cuuint64_t)sl.tdim[1], (cuuint64_t)sl.tdim[2]};
  const cuuint64_t strides[2] = {(cuuint64_t)sl.tstride, (cuuint64_t)sl.tstride2};
  const cuuint32_t box[3] = {(cuuint32_t)sl.tbox[0], (cuuint32_t)sl.tbox[1], (cuuint32_t)sl.tbox[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  CCB_CU(driver().cuTensorMapEncodeTiled(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)sl.trank, (void*)base, dims, strides,
                                         box, estr,
                                         CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)sl.tswizzle,
                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  auto& slot = ln.tmaps[key];
  slot.first = base;
  slot.second = m;
  out = &slot.second;
  return CCB_OK;
}

// Issue one run on `stream`: uploads (host runs), zero fills and launches,
// downloads (host runs) and the error-word readback.
int issue(Program& P, int lane, const void* const* h_in, void* const* h_out, const void* const* d_in, void* const* d_out,
          CUstream stream, CUevent const* out_events = nullptr) {
  const Driver& d = driver();
  Lane& ln = P.lanes[lane];
  std::vector<CUdeviceptr> ptr = ln.bufs;
  std::vector<char> overridden(ptr.size(), 0);
  if (d_in) {
    for (size_t i = 0; i < P.L.params.size(); ++i) {
      ptr[P.L.params[i].buf] = (CUdeviceptr)d_in[i];
      overridden[P.L.params[i].buf] = 1;
    }
  }
  // Resident outputs are written in place; an output whose buffer is already
  // bound (a param, or a second name for one node) is copied afterwards.
  std::vector<std::pair<CUdeviceptr, int>> copies;  // (dst, buf)
  if (d_out) {
    for (size_t j = 0; j < P.L.outputs.size(); ++j) {
      const int b = P.L.outputs[j].buf;
      if (overridden[b]) {
        copies.push_back({(CUdeviceptr)d_out[j], b});
      } else {
        ptr[b] = (CUdeviceptr)d_out[j];
        overridden[b] = 1;
      }
    }
  }
  if (h_in) {
    for (size_t i = 0; i < P.L.params.size(); ++i) {
      const IOSpec& p = P.L.params[i];
      if (p.bytes) CCB_CU(d.cuMemcpyHtoDAsync(ptr[p.buf], h_in[i], p.bytes, stream));
    }
  }
  // Under stream capture the launch arguments are frozen into the graph; a
  // flat scan's per-run epoch would then repeat on every replay.
  CUstreamCaptureStatus cs = CU_STREAM_CAPTURE_STATUS_NONE;
  CCB_CU(d.cuStreamIsCapturing(stream, &cs));
  const bool capturing = cs != CU_STREAM_CAPTURE_STATUS_NONE;
  if (capturing)
    for (const LaunchSpec& l : P.L.launches)
      for (const Slot& sl : l.slots) {
        if (sl.kind == SL_EPOCH)
          return fail(CCB_ERR_INVALID, "graph capture: " + l.fn + " (a flat scan) cannot be replayed from a graph");
        if (sl.kind == SL_XEPOCH)
          return fail(CCB_ERR_INVALID, "graph capture: " + l.fn + " (a sharded pass) cannot be replayed from a graph");
      }
  if (P.L.shard_world > 1) {
    if ((int)P.peers.size() != P.L.shard_world)
      return fail(CCB_ERR_INVALID, "sharded program (rank " + std::to_string(P.L.shard_rank) + " of " +
                                       std::to_string(P.L.shard_world) + "): ccb_program_bind_peers has not been called");
    ++P.xepoch;
  }
  ln.epoch = ln.epoch % ((1u << 30) - 2) + 1;
  // output j's event goes right after the last op that references its
  // buffer (no later op touches it); outputs copied out after the launches
  // get theirs after the copies
  std::vector<std::vector<int>> ev_at(P.L.ops.size());
  std::vector<int> ev_end;
  if (out_events) {
    for (size_t j = 0; j < P.L.outputs.size(); ++j) {
      if (!out_events[j]) continue;
      const int b = P.L.outputs[j].buf;
      bool copied = false;
      for (auto& c : copies)
        if (c.second == b && c.first == (CUdeviceptr)(d_out ? d_out[j] : nullptr)) copied = true;
      int last = -1;
      for (size_t o = 0; o < P.L.ops.size(); ++o) {
        const OpSpec& op = P.L.ops[o];
        if (op.kind == OP_ZERO) {
          if (op.buf == b) last = (int)o;
          continue;
        }
        for (const Slot& sl : P.L.launches[op.launch].slots)
          if ((sl.kind == SL_BUF || sl.kind == SL_TMAP) && sl.buf == b) last = (int)o;
      }
      if (copied || last < 0)
        ev_end.push_back((int)j);
      else
        ev_at[last].push_back((int)j);
    }
  }
  std::vector<uint64_t> blk;
  for (size_t oi = 0; oi < P.L.ops.size(); ++oi) {
    const OpSpec& op = P.L.ops[oi];
    if (op.kind == OP_ZERO) {
      const int64_t n = buf_bytes(P.L.bufs[op.buf]);
      if (n) CCB_CU(d.cuMemsetD8Async(ptr[op.buf], 0, n, stream));
      for (int j : ev_at[oi]) CCB_CU(d.cuEventRecord(out_events[j], stream));
      continue;
    }
    const LaunchSpec& l = P.L.launches[op.launch];
    blk.clear();
    for (size_t s = 0; s < l.slots.size(); ++s) {
      const Slot& sl = l.slots[s];
      if (sl.kind == SL_TMAP) {
        const CUtensorMap* m = nullptr;
        CCB_TRY(tensor_map(ln, op.launch * 64 + (int64_t)s, sl, ptr[sl.buf], m));
        const uint64_t* w = reinterpret_cast<const uint64_t*>(m);
        blk.insert(blk.end(), w, w + 16);
        continue;
      }
      switch (sl.kind) {
        case SL_BUF: blk.push_back((uint64_t)ptr[sl.buf]); break;
        case SL_I64: blk.push_back((uint64_t)sl.val); break;
        case SL_XMB: blk.push_back((uint64_t)P.peers[sl.val]); break;
        case SL_XEPOCH: blk.push_back(P.xepoch); break;
        default: blk.push_back(ln.epoch); break;
      }
    }
    blk.resize((blk.size() + 7) & ~(size_t)7, 0);  // a block with tensor maps is padded to 64 bytes
    void* args[] = {blk.data()};
    CCB_CU(d.cuLaunchKernel(P.fns[op.launch], P.gx[op.launch], P.gy[op.launch], 1, l.block, 1, 1, (unsigned)l.smem, stream,
                            args, nullptr));
    for (int j : ev_at[oi]) CCB_CU(d.cuEventRecord(out_events[j], stream));
  }
  for (auto& c : copies) {
    const int64_t n = buf_bytes(P.L.bufs[c.second]);
    if (n) CCB_CU(d.cuMemcpyDtoDAsync(c.first, ptr[c.second], n, stream));
  }
  for (int j : ev_end) CCB_CU(d.cuEventRecord(out_events[j], stream));
  if (h_out) {
    for (size_t j = 0; j < P.L.outputs.size(); ++j) {
      const IOSpec& o = P.L.outputs[j];
      if (o.bytes) CCB_CU(d.cuMemcpyDtoHAsync(h_out[j], ptr[o.buf], o.bytes, stream));
    }
  }
  if (h_in || h_out) {
    CCB_CU(d.cuMemcpyDtoHAsync(ln.host_err, ln.bufs[P.L.err_buf], 4, stream));
    ln.err_pending = false;
  } else {
    ln.err_pending = true;
  }
  if (!capturing) CCB_CU(d.cuEventRecord(ln.done, stream));
  return CCB_OK;
}

Program* as_prog(ccb_program_t p) { return static_cast<Program*>(p); }

// Compile with the occupancy bound the generator asked for (8 resident
// blocks of 256 threads: 32 registers), load, and recompile without the bound
// any map-reduce pass whose loaded function uses local memory (spills or
// register arrays that did not fit). The local size is read from the loaded
// function, not from a compiler log. CCB_MINB=<n> in the environment forces
// one bound for every pass (a tuning aid).
int compile_tuned(const Lowered& L, CUmodule& mod, std::vector<std::string>& relaxed) {
  const Driver& d = driver();
  const std::string name = L.name.empty() ? "ccb" : L.name;
  std::vector<std::string> opts;
  std::string cubin, log;
  if (const char* f = std::getenv("CCB_MINB")) {
    for (const auto& l : L.launches)
      if (l.fn.rfind("ccb_mapreduce_", 0) == 0) opts.push_back("-DCCB_MINB_" + l.fn.substr(14) + "=" + f);
    CCB_TRY(nvrtc_compile_opts(L.source, name, opts, cubin, log));
    CCB_CU(d.cuModuleLoadData(&mod, cubin.data()));
    return CCB_OK;
  }
  CCB_TRY(nvrtc_compile_opts(L.source, name, opts, cubin, log));
  CCB_CU(d.cuModuleLoadData(&mod, cubin.data()));
  for (const auto& l : L.launches) {
    if (l.fn.rfind("ccb_mapreduce_", 0) != 0) continue;
    CUfunction f;
    CCB_CU(d.cuModuleGetFunction(&f, mod, l.fn.c_str()));
    int local = 0;
    CCB_CU(d.cuFuncGetAttribute(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f));
    if (local > 0) relaxed.push_back(l.fn);
  }
  if (relaxed.empty()) return CCB_OK;
  std::vector<std::string> base = opts;
  for (const auto& fn : relaxed) opts.push_back("-DCCB_MINB_" + fn.substr(14) + "=1");
  d.cuModuleUnload(mod);
  mod = nullptr;
  CCB_TRY(nvrtc_compile_opts(L.source, name, opts, cubin, log));
  CCB_CU(d.cuModuleLoadData(&mod, cubin.data()));
  // Without the bound a pass runs at the occupancy its registers allow; one
  // more resident block per SM often fits without local memory (the LSM date
  // pass: 138 registers, 1 block/SM, unbounded; 128 registers, 2 blocks/SM,
  // no spills, with the bound 2: LSM price 5.86 -> 5.52 ms). Try that level
  // for every relaxed pass that streams element data and keep it where
  // nothing spills. Monte-Carlo estimators, bound by instruction issue, keep
  // their own occupancy (F64 Greeks with two elements per iteration: 2.59 ms
  // at 5 blocks/SM against 2.54 at 4, on one box).
  std::vector<int> level(relaxed.size(), 1);
  std::vector<std::string> up = base;
  bool any = false;
  for (size_t r = 0; r < relaxed.size(); ++r) {
    bool streams = false;
    for (const auto& l : L.launches)
      if (l.fn == relaxed[r]) streams = l.streams;
    if (!streams) {
      up.push_back("-DCCB_MINB_" + relaxed[r].substr(14) + "=1");
      continue;
    }
    CUfunction f;
    CCB_CU(d.cuModuleGetFunction(&f, mod, relaxed[r].c_str()));
    int occ = 1;
    d.cuOccupancyMaxActiveBlocksPerMultiprocessor(&occ, f, 256, 0);
    const int next = std::max(1, occ) + 1;
    if (next < 8) {
      level[r] = next;
      any = true;
    }
    up.push_back("-DCCB_MINB_" + relaxed[r].substr(14) + "=" + std::to_string(level[r]));
  }
  if (!any) return CCB_OK;
  std::string cubin2, log2;
  CUmodule mod2 = nullptr;
  CCB_TRY(nvrtc_compile_opts(L.source, name, up, cubin2, log2));
  CCB_CU(d.cuModuleLoadData(&mod2, cubin2.data()));
  std::vector<char> keep(relaxed.size(), 0);
  int kept = 0;
  for (size_t r = 0; r < relaxed.size(); ++r) {
    if (level[r] == 1) continue;
    CUfunction f;
    int local = 0;
    CCB_CU(d.cuModuleGetFunction(&f, mod2, relaxed[r].c_str()));
    CCB_CU(d.cuFuncGetAttribute(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f));
    keep[r] = local == 0;
    kept += keep[r];
  }
  if (kept == 0) {
    d.cuModuleUnload(mod2);
    return CCB_OK;
  }
  int raised = 0;
  for (size_t r = 0; r < relaxed.size(); ++r) raised += level[r] > 1;
  d.cuModuleUnload(mod);
  mod = mod2;
  if (kept == raised) return CCB_OK;
  std::vector<std::string> mixed = base;  // some passes spill one level up: those stay unbounded
  for (size_t r = 0; r < relaxed.size(); ++r)
    mixed.push_back("-DCCB_MINB_" + relaxed[r].substr(14) + "=" + std::to_string(keep[r] ? level[r] : 1));
  d.cuModuleUnload(mod);
  mod = nullptr;
  CCB_TRY(nvrtc_compile_opts(L.source, name, mixed, cubin, log));
  CCB_CU(d.cuModuleLoadData(&mod, cubin.data()));
  return CCB_OK;
}

int need_device(Program* P) {
  if (!P) return fail(CCB_ERR_INVALID, "null program");
  if (P->device < 0) return fail(CCB_ERR_INVALID, "program was lowered without a device (ccb_program_lower)");
  return ensure_context(P->device);
}

int check_lane(Program* P, int lane) {
  if (lane < 0 || lane >= (int)P->lanes.size())
    return fail(CCB_ERR_INVALID, "lane " + std::to_string(lane) + " out of range (" + std::to_string(P->lanes.size()) + " lanes)");
  return CCB_OK;
}

}  // namespace

extern "C" {

int ccb_program_lower(const char* graph, ccb_program_t* prog) {
  if (!graph || !prog) return fail(CCB_ERR_INVALID, "ccb_program_lower: null argument");
  GGraph g;
  CCB_TRY(parse_graph(graph, g));
  auto P = std::make_unique<Program>();
  CCB_TRY(lower_graph(g, P->L));
  for (auto& op : P->L.ops)
    if (op.kind == OP_LAUNCH) P->num_launch_ops++;
  *prog = P.release();
  return CCB_OK;
}

int ccb_program_create(const char* graph, int device, int lanes, ccb_program_t* prog) {
  if (lanes < 1) return fail(CCB_ERR_INVALID, "Backend_cuda.compile_on: streams must be >= 1");
  ccb_program_t h = nullptr;
  CCB_TRY(ccb_program_lower(graph, &h));
  Program* P = as_prog(h);
  int rc = ensure_context(device);
  if (rc != CCB_OK) {
    destroy(P);
    return rc;
  }
  P->device = device;
  const Driver& d = driver();
  auto cleanup = [&](int code) {
    destroy(P);
    return code;
  };
  std::vector<std::string> relaxed;
  rc = compile_tuned(P->L, P->mod, relaxed);
  if (rc != CCB_OK) return cleanup(rc);
  if (std::getenv("CCB_DEBUG_TUNE"))
    for (const auto& fn : relaxed) fprintf(stderr, "ccb tune %s: bound relaxed (local memory at 8 blocks/SM)\n", fn.c_str());
  CUresult r;
  int sms = 0;
  CUdevice dev;
  d.cuDeviceGet(&dev, device);
  d.cuDeviceGetAttribute(&sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev);
  for (auto& l : P->L.launches) {
    CUfunction f;
    r = d.cuModuleGetFunction(&f, P->mod, l.fn.c_str());
    if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuModuleGetFunction"));
    P->fns.push_back(f);
    int64_t gx = l.gx, gy = l.gy;
    int static_smem = 0;
    d.cuFuncGetAttribute(&static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, f);
    if (static_smem + l.smem > 48 * 1024) {  // above the default limit: opt in
      r = d.cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, l.smem);
      if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuFuncSetAttribute(max dynamic shared memory)"));
    }
    if (l.mode == GM_PERSISTENT) {
      int occ = 1;
      d.cuOccupancyMaxActiveBlocksPerMultiprocessor(&occ, f, l.block, (size_t)l.smem);
      const int64_t cap = std::min<int64_t>(l.max_grid, (int64_t)std::max(1, sms) * std::max(1, occ));
      const int64_t want = (l.work + l.per_block - 1) / std::max<int64_t>(1, l.per_block);
      gx = std::max<int64_t>(1, std::min(want, cap));
      gy = 1;
      if (l.grid_multiple > 1) gx = std::max<int64_t>(l.grid_multiple, gx / l.grid_multiple * l.grid_multiple);
    }
    if (gx > 0x7fffffff || gy > 65535) return cleanup(fail(CCB_ERR_UNSUPPORTED, "launch grid too large for " + l.fn));
    if (std::getenv("CCB_DEBUG_TUNE")) {
      int regs = 0;
      d.cuFuncGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, f);
      fprintf(stderr, "ccb grid %s: %lld x %lld, %d registers\n", l.fn.c_str(), (long long)gx, (long long)gy, regs);
    }
    P->gx.push_back((unsigned)gx);
    P->gy.push_back((unsigned)gy);
  }
  P->lanes.resize(lanes);
  for (Lane& ln : P->lanes) {
    r = d.cuStreamCreate(&ln.stream, CU_STREAM_NON_BLOCKING);
    if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuStreamCreate"));
    r = d.cuEventCreate(&ln.done, CU_EVENT_DISABLE_TIMING);
    if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuEventCreate"));
    r = d.cuMemHostAlloc((void**)&ln.host_err, 64, CU_MEMHOSTALLOC_PORTABLE);
    if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuMemHostAlloc"));
    *ln.host_err = 0;
    ln.bufs.assign(P->L.bufs.size(), 0);
    for (size_t b = 0; b < P->L.bufs.size(); ++b) {
      const int64_t n = std::max<int64_t>(buf_bytes(P->L.bufs[b]), 16);
      r = d.cuMemAlloc(&ln.bufs[b], (size_t)n);
      if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, ("cuMemAlloc (" + P->L.bufs[b].label + ")").c_str()));
      live_add(1);
      if (P->L.bufs[b].zero) {
        r = d.cuMemsetD8Async(ln.bufs[b], 0, (size_t)n, ln.stream);
        if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuMemsetD8Async"));
      }
    }
    r = d.cuStreamSynchronize(ln.stream);
    if (r != CUDA_SUCCESS) return cleanup(cu_fail(r, "cuStreamSynchronize"));
  }
  *prog = P;
  return CCB_OK;
}

int ccb_program_destroy(ccb_program_t prog) { return destroy(as_prog(prog)); }

int ccb_program_source(ccb_program_t prog, const char** source) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *source = as_prog(prog)->L.source.c_str();
  return CCB_OK;
}

int ccb_program_device(ccb_program_t prog, int* device) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *device = as_prog(prog)->device;
  return CCB_OK;
}

int ccb_program_num_kernels(ccb_program_t prog, int* n) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *n = as_prog(prog)->L.num_kernels;
  return CCB_OK;
}

int ccb_program_num_launches(ccb_program_t prog, int* n) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *n = as_prog(prog)->num_launch_ops;
  return CCB_OK;
}

int ccb_program_plan(ccb_program_t prog, const char** text) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *text = as_prog(prog)->L.plan_text.c_str();
  return CCB_OK;
}

int ccb_program_num_params(ccb_program_t prog, int* n) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *n = (int)as_prog(prog)->L.params.size();
  return CCB_OK;
}

int ccb_program_param(ccb_program_t prog, int i, const char** name, int* dtype, int* rank, const long long** dims) {
  Program* P = as_prog(prog);
  if (!P || i < 0 || i >= (int)P->L.params.size()) return fail(CCB_ERR_INVALID, "ccb_program_param: bad index");
  const IOSpec& s = P->L.params[i];
  *name = s.name.c_str();
  *dtype = (int)s.dt;
  *rank = (int)s.shape.size();
  *dims = (const long long*)s.shape.data();
  return CCB_OK;
}

int ccb_program_num_outputs(ccb_program_t prog, int* n) {
  if (!prog) return fail(CCB_ERR_INVALID, "null program");
  *n = (int)as_prog(prog)->L.outputs.size();
  return CCB_OK;
}

int ccb_program_output(ccb_program_t prog, int i, const char** name, int* dtype, int* rank, const long long** dims) {
  Program* P = as_prog(prog);
  if (!P || i < 0 || i >= (int)P->L.outputs.size()) return fail(CCB_ERR_INVALID, "ccb_program_output: bad index");
  const IOSpec& s = P->L.outputs[i];
  *name = s.name.c_str();
  *dtype = (int)s.dt;
  *rank = (int)s.shape.size();
  *dims = (const long long*)s.shape.data();
  return CCB_OK;
}

int ccb_program_enqueue(ccb_program_t prog, int lane, const void* const* inputs, void* const* outputs) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  return issue(*P, lane, inputs, outputs, nullptr, nullptr, P->lanes[lane].stream);
}

int ccb_program_wait(ccb_program_t prog, int lane) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  CCB_CU(driver().cuEventSynchronize(P->lanes[lane].done));
  return lane_check(*P, lane, P->lanes[lane].stream, false);
}

int ccb_program_run(ccb_program_t prog, const void* const* inputs, void* const* outputs) {
  CCB_TRY(ccb_program_enqueue(prog, 0, inputs, outputs));
  return ccb_program_wait(prog, 0);
}

int ccb_program_run_device(ccb_program_t prog, int lane, const void* const* inputs, void* const* outputs,
                           ccb_stream_t stream) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  if (!P->L.params.empty() && !inputs) return fail(CCB_ERR_INVALID, "run_device: inputs required");
  if (!outputs) return fail(CCB_ERR_INVALID, "run_device: outputs required");
  return issue(*P, lane, nullptr, nullptr, inputs, outputs, stream ? (CUstream)stream : P->lanes[lane].stream);
}

int ccb_program_run_device_events(ccb_program_t prog, int lane, const void* const* inputs, void* const* outputs,
                                  ccb_stream_t stream, ccb_event_t const* output_events) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  if (!P->L.params.empty() && !inputs) return fail(CCB_ERR_INVALID, "run_device: inputs required");
  if (!outputs) return fail(CCB_ERR_INVALID, "run_device: outputs required");
  return issue(*P, lane, nullptr, nullptr, inputs, outputs, stream ? (CUstream)stream : P->lanes[lane].stream,
               reinterpret_cast<CUevent const*>(output_events));
}

int ccb_program_check(ccb_program_t prog, int lane, ccb_stream_t stream) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  const CUstream s = stream ? (CUstream)stream : P->lanes[lane].stream;
  CCB_CU(driver().cuStreamSynchronize(s));
  return lane_check(*P, lane, s, true);
}

int ccb_program_shard(ccb_program_t prog, int* rank, int* world) {
  Program* P = as_prog(prog);
  if (!P || !rank || !world) return fail(CCB_ERR_INVALID, "ccb_program_shard: null argument");
  *rank = P->L.shard_rank;
  *world = P->L.shard_world;
  return CCB_OK;
}

int ccb_program_mailbox_bytes(ccb_program_t prog, size_t* bytes) {
  Program* P = as_prog(prog);
  if (!P || !bytes) return fail(CCB_ERR_INVALID, "ccb_program_mailbox_bytes: null argument");
  *bytes = P->L.shard_world > 1 ? mailbox_bytes(P->L.shard_world) : 0;
  return CCB_OK;
}

int ccb_program_bind_peers(ccb_program_t prog, void* const* mailboxes, int nranks) {
  Program* P = as_prog(prog);
  if (!P || !mailboxes) return fail(CCB_ERR_INVALID, "ccb_program_bind_peers: null argument");
  if (P->L.shard_world < 2) return fail(CCB_ERR_INVALID, "ccb_program_bind_peers: the program is not sharded");
  if (nranks != P->L.shard_world)
    return fail(CCB_ERR_INVALID, "ccb_program_bind_peers: " + std::to_string(nranks) + " mailboxes for a world of " +
                                     std::to_string(P->L.shard_world));
  std::vector<CUdeviceptr> v(nranks);
  for (int q = 0; q < nranks; ++q) {
    if (!mailboxes[q]) return fail(CCB_ERR_INVALID, "ccb_program_bind_peers: mailbox of rank " + std::to_string(q) + " is null");
    if ((uintptr_t)mailboxes[q] & 7)
      return fail(CCB_ERR_INVALID, "ccb_program_bind_peers: mailbox of rank " + std::to_string(q) + " is not 8-byte aligned");
    v[q] = (CUdeviceptr)mailboxes[q];
  }
  P->peers = v;
  P->xepoch = 0;
  return CCB_OK;
}

int ccb_program_lane_stream(ccb_program_t prog, int lane, ccb_stream_t* stream) {
  Program* P = as_prog(prog);
  CCB_TRY(need_device(P));
  CCB_TRY(check_lane(P, lane));
  *stream = P->lanes[lane].stream;
  return CCB_OK;
}

}  // extern "C"
