// The runtime half of the C-ABI: devices and primary contexts, memory,
// streams, events, NVRTC modules, launches and NCCL. It replaces the
// reference's cudajit-based lib/runtime (device.ml, buffer.ml, stream.ml,
// event.ml, jit.ml, launch.ml, pinned.ml) with direct driver-API calls.
#include <atomic>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.hpp"

namespace ccb {

namespace {
thread_local std::string g_last_error;
thread_local int g_current = -1;
std::atomic<long long> g_live{0};
std::mutex g_ctx_mu;
std::vector<CUcontext> g_ctx;  // primary context per ordinal (retained once)
bool g_inited = false;
int g_init_status = CCB_OK;
std::once_flag g_init_once;
#include "skel_embed.inc"
}  // namespace

const char* skeleton_header() { return kSkelHeader; }

void live_add(long long d) { g_live += d; }

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cu_fail(CUresult r, const char* what) {
  const char* s = nullptr;
  if (driver().ok && driver().cuGetErrorString) driver().cuGetErrorString(r, &s);
  return fail(CCB_ERR_DRIVER, std::string(what) + ": " + (s ? s : "CUDA error ") + " (" + std::to_string((int)r) + ")");
}

int ensure_driver() {
  std::call_once(g_init_once, [] {
    const Driver& d = driver();
    if (!d.ok) {
      g_init_status = CCB_ERR_NO_DEVICE;
      return;
    }
    if (d.cuInit(0) != CUDA_SUCCESS) {
      g_init_status = CCB_ERR_NO_DEVICE;
      return;
    }
    int n = 0;
    if (d.cuDeviceGetCount(&n) != CUDA_SUCCESS || n <= 0) {
      g_init_status = CCB_ERR_NO_DEVICE;
      return;
    }
    g_ctx.assign(n, nullptr);
    g_inited = true;
  });
  if (g_init_status != CCB_OK) {
    const Driver& d = driver();
    return fail(CCB_ERR_NO_DEVICE, d.ok ? "no CUDA device" : "no CUDA driver: " + d.why);
  }
  return CCB_OK;
}

int ensure_context(int ordinal) {
  CCB_TRY(ensure_driver());
  const Driver& d = driver();
  CUcontext ctx = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    if (ordinal < 0 || ordinal >= (int)g_ctx.size())
      return fail(CCB_ERR_NO_DEVICE, "device ordinal " + std::to_string(ordinal) + " out of range (" +
                                         std::to_string(g_ctx.size()) + " devices)");
    if (!g_ctx[ordinal]) {
      CUdevice dev;
      CCB_CU(d.cuDeviceGet(&dev, ordinal));
      CCB_CU(d.cuDevicePrimaryCtxRetain(&g_ctx[ordinal], dev));
    }
    ctx = g_ctx[ordinal];
  }
  CCB_CU(d.cuCtxSetCurrent(ctx));
  g_current = ordinal;
  return CCB_OK;
}

int current_device() { return g_current < 0 ? 0 : g_current; }

// Make sure some context is current: device 0 unless the thread picked one.
static int ensure_current() { return ensure_context(current_device()); }

int nvrtc_compile(const std::string& source, const std::string& name, std::string& cubin, std::string& log) {
  return nvrtc_compile_opts(source, name, {}, cubin, log);
}

int nvrtc_compile_opts(const std::string& source, const std::string& name, const std::vector<std::string>& extra,
                       std::string& cubin, std::string& log) {
  const Nvrtc& r = nvrtc();
  if (!r.ok) return fail(CCB_ERR_COMPILE, "NVRTC unavailable: " + r.why);
  nvrtcProgram prog;
  const char* hdr_src[] = {skeleton_header()};
  const char* hdr_name[] = {"ccb_skel.cuh"};
  nvrtcResult rc = r.nvrtcCreateProgram(&prog, source.c_str(), (name + ".cu").c_str(), 1, hdr_src, hdr_name);
  if (rc != NVRTC_SUCCESS) return fail(CCB_ERR_COMPILE, std::string("nvrtcCreateProgram: ") + r.nvrtcGetErrorString(rc));
  std::vector<const char*> opts = {"--gpu-architecture=sm_100a", "-std=c++17", "-lineinfo", "--fmad=true"};
  for (auto& e : extra) opts.push_back(e.c_str());
  rc = r.nvrtcCompileProgram(prog, (int)opts.size(), opts.data());
  size_t lsz = 0;
  r.nvrtcGetProgramLogSize(prog, &lsz);
  log.assign(lsz, '\0');
  if (lsz) r.nvrtcGetProgramLog(prog, &log[0]);
  while (!log.empty() && log.back() == '\0') log.pop_back();
  if (rc != NVRTC_SUCCESS) {
    r.nvrtcDestroyProgram(&prog);
    return fail(CCB_ERR_COMPILE, "nvrtc: " + std::string(r.nvrtcGetErrorString(rc)) + "\n" + log);
  }
  size_t csz = 0;
  r.nvrtcGetCUBINSize(prog, &csz);
  cubin.assign(csz, '\0');
  r.nvrtcGetCUBIN(prog, &cubin[0]);
  r.nvrtcDestroyProgram(&prog);
  return CCB_OK;
}

}  // namespace ccb

using namespace ccb;

extern "C" {

const char* ccb_last_error(void) { return g_last_error.c_str(); }
const char* ccb_version(void) { return "ccb 0.1 sm_100a"; }

int ccb_available(void) {
  if (!driver().ok) return 0;
  return ensure_driver() == CCB_OK ? 1 : 0;
}

int ccb_init(void) { return ensure_context(current_device()); }

int ccb_device_count(int* count) {
  CCB_TRY(ensure_driver());
  CCB_CU(driver().cuDeviceGetCount(count));
  return CCB_OK;
}

int ccb_set_device(int ordinal) { return ensure_context(ordinal); }

int ccb_get_device(int* ordinal) {
  *ordinal = current_device();
  return CCB_OK;
}

int ccb_device_info(int ordinal, ccb_device_info_t* info) {
  CCB_TRY(ensure_driver());
  const Driver& d = driver();
  int n = 0;
  CCB_CU(d.cuDeviceGetCount(&n));
  if (ordinal < 0 || ordinal >= n) return fail(CCB_ERR_NO_DEVICE, "no device " + std::to_string(ordinal));
  CUdevice dev;
  CCB_CU(d.cuDeviceGet(&dev, ordinal));
  std::memset(info, 0, sizeof(*info));
  CCB_CU(d.cuDeviceGetName(info->name, sizeof(info->name) - 1, dev));
  CCB_CU(d.cuDeviceGetAttribute(&info->cc_major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, dev));
  CCB_CU(d.cuDeviceGetAttribute(&info->cc_minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, dev));
  CCB_CU(d.cuDeviceGetAttribute(&info->multiprocessors, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev));
  size_t total = 0;
  CCB_CU(d.cuDeviceTotalMem(&total, dev));
  info->total_memory_bytes = (long long)total;
  return CCB_OK;
}

int ccb_device_synchronize(void) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuCtxSynchronize());
  return CCB_OK;
}

int ccb_malloc(size_t bytes, void** dptr) {
  CCB_TRY(ensure_current());
  CUdeviceptr p = 0;
  CCB_CU(driver().cuMemAlloc(&p, bytes == 0 ? 1 : bytes));
  *dptr = (void*)p;
  g_live++;
  return CCB_OK;
}

int ccb_free(void* dptr) {
  if (!dptr) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemFree((CUdeviceptr)dptr));
  g_live--;
  return CCB_OK;
}

int ccb_live_count(long long* count) {
  *count = g_live.load();
  return CCB_OK;
}

int ccb_memcpy_h2d(void* dst, const void* src, size_t bytes, ccb_stream_t s) {
  if (!bytes) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemcpyHtoDAsync((CUdeviceptr)dst, src, bytes, (CUstream)s));
  return CCB_OK;
}

int ccb_memcpy_d2h(void* dst, const void* src, size_t bytes, ccb_stream_t s) {
  if (!bytes) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemcpyDtoHAsync(dst, (CUdeviceptr)src, bytes, (CUstream)s));
  return CCB_OK;
}

int ccb_memcpy_d2d(void* dst, const void* src, size_t bytes, ccb_stream_t s) {
  if (!bytes) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemcpyDtoDAsync((CUdeviceptr)dst, (CUdeviceptr)src, bytes, (CUstream)s));
  return CCB_OK;
}

int ccb_memset_d8(void* dst, unsigned char v, size_t bytes, ccb_stream_t s) {
  if (!bytes) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemsetD8Async((CUdeviceptr)dst, v, bytes, (CUstream)s));
  return CCB_OK;
}

int ccb_host_alloc(size_t bytes, void** hptr) {
  CCB_TRY(ensure_current());
  void* p = nullptr;
  CCB_CU(driver().cuMemHostAlloc(&p, bytes == 0 ? 1 : bytes, CU_MEMHOSTALLOC_PORTABLE));
  std::memset(p, 0, bytes);
  *hptr = p;
  return CCB_OK;
}

int ccb_host_free(void* hptr) {
  if (!hptr) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuMemFreeHost(hptr));
  return CCB_OK;
}

// ---------------------------------------------------------------- peer memory
int ccb_ipc_mem_handle(void* dptr, unsigned char handle[64]) {
  if (!dptr || !handle) return fail(CCB_ERR_INVALID, "ccb_ipc_mem_handle: null pointer");
  CCB_TRY(ensure_current());
  CUipcMemHandle h;
  CCB_CU(driver().cuIpcGetMemHandle(&h, (CUdeviceptr)dptr));
  std::memcpy(handle, h.reserved, 64);
  return CCB_OK;
}

int ccb_ipc_mem_open(const unsigned char handle[64], void** dptr) {
  if (!dptr || !handle) return fail(CCB_ERR_INVALID, "ccb_ipc_mem_open: null pointer");
  CCB_TRY(ensure_current());
  CUipcMemHandle h;
  std::memcpy(h.reserved, handle, 64);
  CUdeviceptr p = 0;
  CCB_CU(driver().cuIpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS));
  *dptr = (void*)p;
  return CCB_OK;
}

int ccb_ipc_mem_close(void* dptr) {
  if (!dptr) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuIpcCloseMemHandle((CUdeviceptr)dptr));
  return CCB_OK;
}

int ccb_peer_access_enable(int peer) {
  CCB_TRY(ensure_current());
  const int self = current_device();
  if (peer == self) return CCB_OK;
  CCB_TRY(ensure_context(peer));  // retain the peer's primary context
  CUcontext peer_ctx = nullptr;
  CCB_CU(driver().cuCtxGetCurrent(&peer_ctx));
  CCB_TRY(ensure_context(self));
  CUdevice a, b;
  CCB_CU(driver().cuDeviceGet(&a, self));
  CCB_CU(driver().cuDeviceGet(&b, peer));
  int can = 0;
  CCB_CU(driver().cuDeviceCanAccessPeer(&can, a, b));
  if (!can) return fail(CCB_ERR_UNSUPPORTED, "device " + std::to_string(self) + " cannot access device " + std::to_string(peer));
  const CUresult r = driver().cuCtxEnablePeerAccess(peer_ctx, 0);
  if (r != CUDA_SUCCESS && r != CUDA_ERROR_PEER_ACCESS_ALREADY_ENABLED) return cu_fail(r, "cuCtxEnablePeerAccess");
  return CCB_OK;
}

int ccb_stream_create(ccb_stream_t* s) {
  CCB_TRY(ensure_current());
  CUstream st;
  CCB_CU(driver().cuStreamCreate(&st, CU_STREAM_NON_BLOCKING));
  *s = st;
  return CCB_OK;
}

int ccb_stream_destroy(ccb_stream_t s) {
  if (!s) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuStreamDestroy((CUstream)s));
  return CCB_OK;
}

int ccb_stream_synchronize(ccb_stream_t s) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuStreamSynchronize((CUstream)s));
  return CCB_OK;
}

int ccb_stream_query(ccb_stream_t s, int* idle) {
  CCB_TRY(ensure_current());
  CUresult r = driver().cuStreamQuery((CUstream)s);
  if (r == CUDA_SUCCESS) {
    *idle = 1;
    return CCB_OK;
  }
  if (r == CUDA_ERROR_NOT_READY) {
    *idle = 0;
    return CCB_OK;
  }
  return cu_fail(r, "cuStreamQuery");
}

int ccb_event_create(ccb_event_t* e) {
  CCB_TRY(ensure_current());
  CUevent ev;
  CCB_CU(driver().cuEventCreate(&ev, CU_EVENT_DEFAULT));
  *e = ev;
  return CCB_OK;
}

int ccb_event_destroy(ccb_event_t e) {
  if (!e) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuEventDestroy((CUevent)e));
  return CCB_OK;
}

int ccb_event_record(ccb_event_t e, ccb_stream_t s) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuEventRecord((CUevent)e, (CUstream)s));
  return CCB_OK;
}

int ccb_event_synchronize(ccb_event_t e) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuEventSynchronize((CUevent)e));
  return CCB_OK;
}

int ccb_event_elapsed_ms(ccb_event_t a, ccb_event_t b, float* ms) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuEventElapsedTime(ms, (CUevent)a, (CUevent)b));
  return CCB_OK;
}

int ccb_stream_wait_event(ccb_stream_t s, ccb_event_t e) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuStreamWaitEvent((CUstream)s, (CUevent)e, 0));
  return CCB_OK;
}

int ccb_graph_begin(ccb_stream_t s) {
  CCB_TRY(ensure_current());
  if (!s) return fail(CCB_ERR_INVALID, "graph_begin: the legacy default stream cannot be captured");
  CCB_CU(driver().cuStreamBeginCapture((CUstream)s, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL));
  return CCB_OK;
}

int ccb_graph_end(ccb_stream_t s, ccb_graph_t* graph) {
  CCB_TRY(ensure_current());
  if (!graph) return fail(CCB_ERR_INVALID, "graph_end: null output");
  const Driver& d = driver();
  CUgraph g = nullptr;
  CCB_CU(d.cuStreamEndCapture((CUstream)s, &g));
  CUgraphExec e = nullptr;
  const CUresult r = d.cuGraphInstantiateWithFlags(&e, g, 0);
  d.cuGraphDestroy(g);
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuGraphInstantiateWithFlags");
  *graph = e;
  return CCB_OK;
}

int ccb_graph_launch(ccb_graph_t graph, ccb_stream_t s) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuGraphLaunch((CUgraphExec)graph, (CUstream)s));
  return CCB_OK;
}

int ccb_graph_destroy(ccb_graph_t graph) {
  if (!graph) return CCB_OK;
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuGraphExecDestroy((CUgraphExec)graph));
  return CCB_OK;
}

static char* dup_string(const std::string& s) {
  char* p = (char*)std::malloc(s.size() + 1);
  std::memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

void ccb_free_string(char* s) { std::free(s); }

int ccb_nvrtc_check(const char* source, const char* name, size_t* cubin_bytes, char** log) {
  std::string cubin, lg;
  int rc = nvrtc_compile(source, name ? name : "ccb", cubin, lg);
  if (log) *log = dup_string(lg);
  if (cubin_bytes) *cubin_bytes = cubin.size();
  return rc;
}

int ccb_module_compile(const char* source, const char* name, ccb_module_t* mod, char** log) {
  std::string cubin, lg;
  int rc = nvrtc_compile(source, name ? name : "ccb", cubin, lg);
  if (log) *log = dup_string(lg);
  if (rc != CCB_OK) return rc;
  CCB_TRY(ensure_current());
  CUmodule m;
  CCB_CU(driver().cuModuleLoadData(&m, cubin.data()));
  *mod = m;
  return CCB_OK;
}

int ccb_module_unload(ccb_module_t mod) {
  CCB_TRY(ensure_current());
  CCB_CU(driver().cuModuleUnload((CUmodule)mod));
  return CCB_OK;
}

int ccb_module_get_function(ccb_module_t mod, const char* name, ccb_function_t* fn) {
  CCB_TRY(ensure_current());
  CUfunction f;
  CCB_CU(driver().cuModuleGetFunction(&f, (CUmodule)mod, name));
  *fn = f;
  return CCB_OK;
}

// The kernel's parameter count, from the loaded function's own metadata:
// cuFuncGetParamInfo answers for every index below the count and refuses the
// first one past it.
static int param_count(CUfunction f, int* count) {
  const Driver& d = driver();
  int k = 0;
  for (;; ++k) {
    size_t off = 0, sz = 0;
    if (d.cuFuncGetParamInfo(f, (size_t)k, &off, &sz) != CUDA_SUCCESS) break;
    if (k > 4096) return fail(CCB_ERR_DRIVER, "cuFuncGetParamInfo: parameter count not found");
  }
  *count = k;
  return CCB_OK;
}

int ccb_launch(ccb_function_t fn, unsigned gx, unsigned gy, unsigned gz, unsigned bx, unsigned by, unsigned bz,
               unsigned smem, ccb_stream_t s, void** args, int nargs) {
  CCB_TRY(ensure_current());
  if (!fn) return fail(CCB_ERR_INVALID, "ccb_launch: null function");
  if (nargs < 0 || (nargs > 0 && !args)) return fail(CCB_ERR_INVALID, "ccb_launch: bad argument block");
  int want = 0;
  CCB_TRY(param_count((CUfunction)fn, &want));
  if (want != nargs)
    return fail(CCB_ERR_INVALID, "ccb_launch: the kernel takes " + std::to_string(want) + " arguments, " +
                                     std::to_string(nargs) + " given");
  CCB_CU(driver().cuLaunchKernel((CUfunction)fn, gx, gy, gz, bx, by, bz, smem, (CUstream)s, args, nullptr));
  return CCB_OK;
}

// ---------------------------------------------------------------- NCCL
static int nccl_fail(ncclResult_t r, const char* what) {
  return fail(CCB_ERR_NCCL, std::string(what) + ": " + nccl().ncclGetErrorString(r));
}
#define CCB_NCCL(call)                                         \
  do {                                                         \
    ncclResult_t _r = (call);                                  \
    if (_r != ncclSuccess) return nccl_fail(_r, #call);        \
  } while (0)

static int need_nccl() {
  if (!nccl().ok) return fail(CCB_ERR_NCCL, "NCCL unavailable: " + nccl().why);
  return CCB_OK;
}

int ccb_comm_init_all(int ndev, const int* devices, ccb_comm_t* comms) {
  CCB_TRY(need_nccl());
  for (int i = 0; i < ndev; ++i) CCB_TRY(ensure_context(devices[i]));
  std::vector<ncclComm_t> cs(ndev);
  CCB_NCCL(nccl().ncclCommInitAll(cs.data(), ndev, devices));
  for (int i = 0; i < ndev; ++i) comms[i] = cs[i];
  return CCB_OK;
}

int ccb_comm_unique_id(unsigned char id[128]) {
  CCB_TRY(need_nccl());
  ncclUniqueId u;
  CCB_NCCL(nccl().ncclGetUniqueId(&u));
  static_assert(sizeof(u) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id, &u, 128);
  return CCB_OK;
}

int ccb_comm_init_rank(int nranks, const unsigned char id[128], int rank, ccb_comm_t* comm) {
  CCB_TRY(need_nccl());
  CCB_TRY(ensure_current());
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclComm_t c;
  CCB_NCCL(nccl().ncclCommInitRank(&c, nranks, u, rank));
  *comm = c;
  return CCB_OK;
}

int ccb_comm_destroy(ccb_comm_t comm) {
  CCB_TRY(need_nccl());
  CCB_NCCL(nccl().ncclCommDestroy((ncclComm_t)comm));
  return CCB_OK;
}

int ccb_allreduce(ccb_comm_t comm, const void* send, void* recv, size_t count, int dtype, int op, ccb_stream_t s) {
  CCB_TRY(need_nccl());
  ncclDataType_t t;
  switch (dtype) {
    case 0: t = ncclFloat32; break;
    case 1: t = ncclFloat64; break;
    case 2: t = ncclInt32; break;
    case 3: t = ncclInt64; break;
    default: return fail(CCB_ERR_INVALID, "ccb_allreduce: bad dtype code " + std::to_string(dtype));
  }
  ncclRedOp_t o;
  switch (op) {
    case 0: o = ncclSum; break;
    case 1: o = ncclMax; break;
    case 2: o = ncclMin; break;
    default: return fail(CCB_ERR_INVALID, "ccb_allreduce: bad op code " + std::to_string(op));
  }
  CCB_NCCL(nccl().ncclAllReduce(send, recv, count, t, o, (ncclComm_t)comm, (cudaStream_t)s));
  return CCB_OK;
}

int ccb_group_start(void) {
  CCB_TRY(need_nccl());
  CCB_NCCL(nccl().ncclGroupStart());
  return CCB_OK;
}

int ccb_group_end(void) {
  CCB_TRY(need_nccl());
  CCB_NCCL(nccl().ncclGroupEnd());
  return CCB_OK;
}

}  // extern "C"
