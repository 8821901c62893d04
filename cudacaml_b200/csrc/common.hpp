// Status codes, the thread-local error message, and driver-call helpers shared
// by the runtime, the program executor and the NCCL wrappers.
#pragma once
#include <string>
#include <vector>

#include "../../include/ccb.h"
#include "dyn.hpp"

namespace ccb {

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cu_fail(CUresult r, const char* what);

// cuInit once; CCB_ERR_NO_DEVICE when there is no driver or no device.
int ensure_driver();
// Retain device `ordinal`'s primary context and make it current on this thread.
int ensure_context(int ordinal);
int current_device();

// NVRTC: compile `source` to an sm_100a CUBIN with the skeleton header on
// the include path. Returns CCB_OK or CCB_ERR_COMPILE (log in `log`).
int nvrtc_compile(const std::string& source, const std::string& name, std::string& cubin, std::string& log);
int nvrtc_compile_opts(const std::string& source, const std::string& name, const std::vector<std::string>& extra,
                       std::string& cubin, std::string& log);

const char* skeleton_header();

}  // namespace ccb

#define CCB_CU(call)                                              \
  do {                                                            \
    CUresult _ccb_r = (call);                                     \
    if (_ccb_r != CUDA_SUCCESS) return ::ccb::cu_fail(_ccb_r, #call); \
  } while (0)

#define CCB_TRY(expr)              \
  do {                             \
    int _ccb_s = (expr);           \
    if (_ccb_s != CCB_OK) return _ccb_s; \
  } while (0)
