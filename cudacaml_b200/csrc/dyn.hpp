// Lazily opened CUDA driver, NVRTC and NCCL entry points.
//
// libccb.so links none of the three: it dlopen()s them on first use, so the
// library (and every symbol in include/ccb.h) loads on a machine with no GPU
// driver, and a CPU-only test can still check exports and run NVRTC.
#pragma once
#include <cuda.h>
#include <nccl.h>
#include <nvrtc.h>

#include <string>

namespace ccb {

struct Driver {
  bool ok = false;
  std::string why;
#define CCB_DRV(name) decltype(&::name) name = nullptr;
  CCB_DRV(cuInit)
  CCB_DRV(cuDriverGetVersion)
  CCB_DRV(cuDeviceGetCount)
  CCB_DRV(cuDeviceGet)
  CCB_DRV(cuDeviceGetName)
  CCB_DRV(cuDeviceGetAttribute)
  CCB_DRV(cuDeviceTotalMem)
  CCB_DRV(cuDevicePrimaryCtxRetain)
  CCB_DRV(cuCtxSetCurrent)
  CCB_DRV(cuCtxGetCurrent)
  CCB_DRV(cuCtxSynchronize)
  CCB_DRV(cuMemAlloc)
  CCB_DRV(cuMemFree)
  CCB_DRV(cuMemcpyHtoDAsync)
  CCB_DRV(cuMemcpyDtoHAsync)
  CCB_DRV(cuMemcpyDtoDAsync)
  CCB_DRV(cuMemsetD8Async)
  CCB_DRV(cuMemsetD32Async)
  CCB_DRV(cuMemHostAlloc)
  CCB_DRV(cuMemFreeHost)
  CCB_DRV(cuStreamCreate)
  CCB_DRV(cuStreamDestroy)
  CCB_DRV(cuStreamSynchronize)
  CCB_DRV(cuStreamQuery)
  CCB_DRV(cuStreamWaitEvent)
  CCB_DRV(cuEventCreate)
  CCB_DRV(cuEventDestroy)
  CCB_DRV(cuEventRecord)
  CCB_DRV(cuEventSynchronize)
  CCB_DRV(cuEventElapsedTime)
  CCB_DRV(cuModuleLoadData)
  CCB_DRV(cuModuleUnload)
  CCB_DRV(cuModuleGetFunction)
  CCB_DRV(cuLaunchKernel)
  CCB_DRV(cuFuncGetParamInfo)
  CCB_DRV(cuIpcGetMemHandle)
  CCB_DRV(cuIpcOpenMemHandle)
  CCB_DRV(cuIpcCloseMemHandle)
  CCB_DRV(cuDeviceCanAccessPeer)
  CCB_DRV(cuCtxEnablePeerAccess)
  CCB_DRV(cuFuncSetAttribute)
  CCB_DRV(cuFuncGetAttribute)
  CCB_DRV(cuOccupancyMaxActiveBlocksPerMultiprocessor)
  CCB_DRV(cuGetErrorString)
  CCB_DRV(cuPointerGetAttribute)
  CCB_DRV(cuTensorMapEncodeTiled)
  CCB_DRV(cuStreamBeginCapture)
  CCB_DRV(cuStreamEndCapture)
  CCB_DRV(cuStreamIsCapturing)
  CCB_DRV(cuGraphInstantiateWithFlags)
  CCB_DRV(cuGraphLaunch)
  CCB_DRV(cuGraphExecDestroy)
  CCB_DRV(cuGraphDestroy)
#undef CCB_DRV
};

struct Nvrtc {
  bool ok = false;
  std::string why;
#define CCB_RTC(name) decltype(&::name) name = nullptr;
  CCB_RTC(nvrtcCreateProgram)
  CCB_RTC(nvrtcDestroyProgram)
  CCB_RTC(nvrtcCompileProgram)
  CCB_RTC(nvrtcGetProgramLogSize)
  CCB_RTC(nvrtcGetProgramLog)
  CCB_RTC(nvrtcGetCUBINSize)
  CCB_RTC(nvrtcGetCUBIN)
  CCB_RTC(nvrtcGetErrorString)
  CCB_RTC(nvrtcVersion)
#undef CCB_RTC
};

struct Nccl {
  bool ok = false;
  std::string why;
#define CCB_NC(name) decltype(&::name) name = nullptr;
  CCB_NC(ncclGetUniqueId)
  CCB_NC(ncclCommInitRank)
  CCB_NC(ncclCommInitAll)
  CCB_NC(ncclCommDestroy)
  CCB_NC(ncclAllReduce)
  CCB_NC(ncclGroupStart)
  CCB_NC(ncclGroupEnd)
  CCB_NC(ncclGetErrorString)
#undef CCB_NC
};

// Each returns the table, loading it on first use (thread-safe). Check .ok.
const Driver& driver();
const Nvrtc& nvrtc();
const Nccl& nccl();

}  // namespace ccb
