#include <cstdlib>
#include "dyn.hpp"

#include <dlfcn.h>

#include <mutex>
#include <vector>

namespace ccb {
namespace {

void* open_first(const std::vector<const char*>& names, std::string& why) {
  for (const char* n : names) {
    if (void* h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) return h;
  }
  const char* e = dlerror();
  why = std::string("cannot open ") + names.front() + (e ? std::string(": ") + e : std::string());
  return nullptr;
}

template <class T>
bool sym(void* h, T& fp, const char* name, std::string& why) {
  fp = reinterpret_cast<T>(dlsym(h, name));
  if (!fp) {
    why = std::string("missing symbol ") + name;
    return false;
  }
  return true;
}

}  // namespace

const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = open_first({"libcuda.so.1", "libcuda.so"}, d.why);
    if (!h) return;
    bool ok = true;
    // Versioned driver symbols: the _v2 spellings are what cuda.h's macros map
    // the plain names to, so resolve those.
#define S(field, name) ok = ok && sym(h, d.field, name, d.why);
    S(cuInit, "cuInit")
    S(cuDriverGetVersion, "cuDriverGetVersion")
    S(cuDeviceGetCount, "cuDeviceGetCount")
    S(cuDeviceGet, "cuDeviceGet")
    S(cuDeviceGetName, "cuDeviceGetName")
    S(cuDeviceGetAttribute, "cuDeviceGetAttribute")
    S(cuDeviceTotalMem, "cuDeviceTotalMem_v2")
    S(cuDevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain")
    S(cuCtxSetCurrent, "cuCtxSetCurrent")
    S(cuCtxGetCurrent, "cuCtxGetCurrent")
    S(cuCtxSynchronize, "cuCtxSynchronize")
    S(cuMemAlloc, "cuMemAlloc_v2")
    S(cuMemFree, "cuMemFree_v2")
    S(cuMemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2")
    S(cuMemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2")
    S(cuMemcpyDtoDAsync, "cuMemcpyDtoDAsync_v2")
    S(cuMemsetD8Async, "cuMemsetD8Async")
    S(cuMemsetD32Async, "cuMemsetD32Async")
    S(cuMemHostAlloc, "cuMemHostAlloc")
    S(cuMemFreeHost, "cuMemFreeHost")
    S(cuStreamCreate, "cuStreamCreate")
    S(cuStreamDestroy, "cuStreamDestroy_v2")
    S(cuStreamSynchronize, "cuStreamSynchronize")
    S(cuStreamQuery, "cuStreamQuery")
    S(cuStreamWaitEvent, "cuStreamWaitEvent")
    S(cuEventCreate, "cuEventCreate")
    S(cuEventDestroy, "cuEventDestroy_v2")
    S(cuEventRecord, "cuEventRecord")
    S(cuEventSynchronize, "cuEventSynchronize")
    S(cuEventElapsedTime, "cuEventElapsedTime")
    S(cuModuleLoadData, "cuModuleLoadData")
    S(cuModuleUnload, "cuModuleUnload")
    S(cuModuleGetFunction, "cuModuleGetFunction")
    S(cuLaunchKernel, "cuLaunchKernel")
    S(cuFuncGetParamInfo, "cuFuncGetParamInfo")
    S(cuIpcGetMemHandle, "cuIpcGetMemHandle")
    S(cuIpcOpenMemHandle, "cuIpcOpenMemHandle_v2")
    S(cuIpcCloseMemHandle, "cuIpcCloseMemHandle")
    S(cuDeviceCanAccessPeer, "cuDeviceCanAccessPeer")
    S(cuCtxEnablePeerAccess, "cuCtxEnablePeerAccess")
    S(cuFuncSetAttribute, "cuFuncSetAttribute")
    S(cuFuncGetAttribute, "cuFuncGetAttribute")
    S(cuOccupancyMaxActiveBlocksPerMultiprocessor, "cuOccupancyMaxActiveBlocksPerMultiprocessor")
    S(cuGetErrorString, "cuGetErrorString")
    S(cuPointerGetAttribute, "cuPointerGetAttribute")
    S(cuTensorMapEncodeTiled, "cuTensorMapEncodeTiled")
    S(cuStreamBeginCapture, "cuStreamBeginCapture_v2")
    S(cuStreamEndCapture, "cuStreamEndCapture")
    S(cuStreamIsCapturing, "cuStreamIsCapturing")
    S(cuGraphInstantiateWithFlags, "cuGraphInstantiateWithFlags")
    S(cuGraphLaunch, "cuGraphLaunch")
    S(cuGraphExecDestroy, "cuGraphExecDestroy")
    S(cuGraphDestroy, "cuGraphDestroy")
#undef S
    d.ok = ok;
  });
  return d;
}

const Nvrtc& nvrtc() {
  static Nvrtc r;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = open_first({"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"}, r.why);
    if (!h) return;
    bool ok = true;
#define S(name) ok = ok && sym(h, r.name, #name, r.why);
    S(nvrtcCreateProgram)
    S(nvrtcDestroyProgram)
    S(nvrtcCompileProgram)
    S(nvrtcGetProgramLogSize)
    S(nvrtcGetProgramLog)
    S(nvrtcGetCUBINSize)
    S(nvrtcGetCUBIN)
    S(nvrtcGetErrorString)
    S(nvrtcVersion)
#undef S
    r.ok = ok;
  });
  return r;
}

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    // One NCCL per process: a copy already loaded (by the host application,
    // e.g. the framework that drives the other ranks) is used as it is, then
    // the one CCB_NCCL_LIB names, then the loader's default. Loading a second,
    // different libnccl.so.2 first would bind the application's later NCCL
    // users to it.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h)
      if (const char* lib = std::getenv("CCB_NCCL_LIB")) h = dlopen(lib, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = open_first({"libnccl.so.2", "libnccl.so"}, n.why);
    if (!h) return;
    bool ok = true;
#define S(name) ok = ok && sym(h, n.name, #name, n.why);
    S(ncclGetUniqueId)
    S(ncclCommInitRank)
    S(ncclCommInitAll)
    S(ncclCommDestroy)
    S(ncclAllReduce)
    S(ncclGroupStart)
    S(ncclGroupEnd)
    S(ncclGetErrorString)
#undef S
    n.ok = ok;
  });
  return n;
}

}  // namespace ccb
