// ccb_sum_f32_noalloc: the flat F32 sum (the map_reduce skeleton, the same
// single-pass kernel a `reduce add` graph lowers to) for callers that cannot
// allocate device memory.
//
// Who cannot allocate: code running where cudaMalloc is unavailable or
// forbidden -- inside a CUDA graph being captured by someone else's framework,
// in a real-time or signal-safe path that must not take the driver's
// allocation locks, under a memory pool that the host application owns and
// has fully reserved, or in a plugin that is given device pointers but no
// allocator. The regular path (ccb_program_create) allocates its reduction
// scratch (block partials and a ticket) per program; this entry point instead
// keeps that scratch in one file-scope __device__ array, so a call allocates
// nothing: no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits and sharing:
//  * the scratch holds at most kMaxBlocks (4096) block partials, so the grid
//    is capped at 4096 blocks; n may be anything from 0 to 2^31 - 1 elements
//    (element indices are int32, as in the graph IR) and larger n is rejected;
//  * every GPU that loads this library holds the array (16 KiB + 256 B) until
//    the process exits;
//  * all calls on one device share the array and it keeps the last call's
//    contents: each call clears the ticket first (cudaMemsetAsync, which does
//    not allocate), and two calls that overlap on the GPU (different streams,
//    no ordering between them) race on it and produce wrong sums;
//  * the first call on a device does the set-up for that device
//    (cudaGetSymbolAddress of the array and an occupancy query); make that
//    first call before any stream capture begins;
//  * the device address found at set-up is kept for the life of the process:
//    after a reset of a device's primary context (cudaDeviceReset,
//    cuDevicePrimaryCtxReset) it is stale, so do not call this entry point on
//    a device whose context was reset since its first call.
// Errors are reported like every other entry point of the library: an int
// status and the message of ccb_last_error() on the calling thread.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "ccb_skel.cuh"

namespace ccb {
void set_error(const std::string& msg);  // the library's thread-local message (runtime.cpp)
}

namespace {

constexpr int kMaxBlocks = 4096;
constexpr int kBlock = 256;

// [0, kMaxBlocks) float partials, then the last-block ticket. A sum reads
// no data-dependent index and waits on nothing, so it has no error word.
struct Scratch {
  float partials[kMaxBlocks];
  unsigned ticket;
};
static __device__ __align__(256) Scratch g_scratch;

struct FSum {
  struct P {
    const float* __restrict__ x;
    float* __restrict__ out;
    float* partials;
    unsigned* ticket;
    long long n;
  };
  typedef float acc_t;
  static constexpr int NRED = 1;
  static constexpr int VEC = 1;
  static constexpr int UNROLL = 4;
  static constexpr bool ILP = false;
  static constexpr bool TAIL = false;
  static __device__ __forceinline__ acc_t identity(int) { return 0.0f; }
  static __device__ __forceinline__ void init(acc_t* acc) { acc[0] = 0.0f; }
  static __device__ __forceinline__ acc_t combine(int, acc_t a, acc_t b) { return a + b; }
  static __device__ __forceinline__ bool vec_ok(const P& p) { return ccb::aligned16(p.x); }
  static __device__ __forceinline__ void elem(const P& p, int i, acc_t* acc) { acc[0] = acc[0] + p.x[i]; }
  static __device__ __forceinline__ void elem4(const P& p, int i, acc_t* acc) {
    const ccb::V4<float> v = ccb::ld4(p.x + i);
    acc[0] = acc[0] + v.v[0];
    acc[0] = acc[0] + v.v[1];
    acc[0] = acc[0] + v.v[2];
    acc[0] = acc[0] + v.v[3];
  }
  static __device__ __forceinline__ void epilogue(const P& p, const acc_t* res) { p.out[0] = res[0]; }
};

__global__ void __launch_bounds__(kBlock) ccb_sum_f32_noalloc_kernel(const FSum::P p) { ccb::map_reduce<FSum>(p); }

struct DeviceSetup {
  bool ready = false;
  Scratch* scratch = nullptr;  // device address of g_scratch on this device
  int max_grid = 1;
};
constexpr int kMaxDevices = 64;
DeviceSetup g_setup[kMaxDevices];
std::mutex g_mu;

// Status codes as in ccb.h: CCB_ERR_INVALID 1, CCB_ERR_NO_DEVICE 2, CCB_ERR_DRIVER 3.
int fail(int code, const std::string& m) {
  ccb::set_error(m);
  return code;
}

// Once per device, with that device current: resolve the array's device
// address (host code only ever sees the symbol's host-side stand-in) and size
// the grid.
int setup(int dev, DeviceSetup** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSetup& s = g_setup[dev];
  if (!s.ready) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess) return fail(3, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    int sms = 0, occ = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(3, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ccb_sum_f32_noalloc_kernel, kBlock, 0);
    if (e != cudaSuccess) return fail(3, std::string("cudaOccupancyMaxActiveBlocksPerMultiprocessor: ") + cudaGetErrorString(e));
    s.scratch = static_cast<Scratch*>(ptr);
    s.max_grid = sms * (occ > 0 ? occ : 1);
    if (s.max_grid > kMaxBlocks) s.max_grid = kMaxBlocks;
    if (s.max_grid < 1) s.max_grid = 1;
    s.ready = true;
  }
  *out = &s;
  return 0;
}

}  // namespace

extern "C" {

int ccb_sum_f32_noalloc(const float* x, long long n, float* out, void* stream) {
  if (n < 0 || n > 2147483647LL)
    return fail(1, "ccb_sum_f32_noalloc: n = " + std::to_string(n) + " is outside [0, 2^31 - 1] (int32 element indices)");
  if (!out || (n > 0 && !x)) return fail(1, "ccb_sum_f32_noalloc: null pointer");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(2, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(2, "ccb_sum_f32_noalloc: device ordinal out of range");
  DeviceSetup* s = nullptr;
  int rc = setup(dev, &s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The ticket must start at zero; the array keeps whatever the last call left.
  e = cudaMemsetAsync(&s->scratch->ticket, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) return fail(3, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  FSum::P p;
  p.x = x;
  p.out = out;
  p.partials = s->scratch->partials;
  p.ticket = &s->scratch->ticket;
  p.n = n;
  long long want = (n + (long long)kBlock * 8 - 1) / ((long long)kBlock * 8);
  if (want < 1) want = 1;
  const int grid = (int)(want < s->max_grid ? want : s->max_grid);
  ccb_sum_f32_noalloc_kernel<<<grid, kBlock, 0, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(3, std::string("launch: ") + cudaGetErrorString(e));
  return 0;
}

}  // extern "C"
