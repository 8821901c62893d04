// ccb_xrank_sum: the sum of a few scalars across the ranks of one box, each
// rank on its own GPU, over NVLink peer memory -- the recombination step of a
// Monte-Carlo run split by counter range (the four results of the Greeks
// graph), without a library collective.
//
// Every rank owns a mailbox in its own HBM and holds a device pointer to every
// other rank's mailbox (an IPC mapping across processes, or a peer-enabled
// allocation in one process). A call with epoch e (identical on every rank,
// strictly increasing from 1) is one tiny kernel per rank: lane q writes this
// rank's values into slot [e & 1][rank] of rank q's mailbox, publishes them
// with a system-scope release store of e into the slot's flag, then lane q
// polls slot [e & 1][q] of the local mailbox with system-scope acquire loads
// until it reads e, and each value is summed over the ranks in rank order, so
// every rank gets the same bits. Slots alternate between two halves by epoch
// parity: a rank can only write epoch e + 2 after every rank has finished
// epoch e + 1, hence after every rank has read epoch e.
//
// Waits are bounded: a peer that never publishes makes the wait give up after
// kXrankSpin polls, raise bit kErrXrank in the caller's error word and leave
// `out` untouched; the kernel returns and the context stays usable.
//
// Mailboxes must be zero-filled and every rank must have finished zeroing its
// own before any rank's first call (a zeroing that lands after a peer's write
// would erase it).
#include <cuda_runtime.h>

#include <string>

namespace ccb {
void set_error(const std::string& msg);  // the library's thread-local message (runtime.cpp)
}

namespace {

constexpr int kMaxRanks = 16;
constexpr int kMaxValues = 8;
constexpr int kSlotWords = 1 + kMaxValues;  // flag (epoch) + values, 8 bytes each
constexpr unsigned kXrankSpin = 1u << 22;
constexpr unsigned kErrXrank = 32u;

struct XP {
  unsigned long long* mb[kMaxRanks];  // mailbox of rank q, as this rank addresses it
  const void* in;
  void* out;
  unsigned* err;
  unsigned long long epoch;
  int nranks, rank, count, dtype;
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long load_bits(const void* in, int dtype, int k) {
  switch (dtype) {
    case 0: return (unsigned long long)__float_as_uint(static_cast<const float*>(in)[k]);
    case 1: return (unsigned long long)__double_as_longlong(static_cast<const double*>(in)[k]);
    case 2: return (unsigned long long)(unsigned)static_cast<const int*>(in)[k];
    default: return (unsigned long long)static_cast<const long long*>(in)[k];
  }
}

__global__ void __launch_bounds__(32) ccb_xrank_sum_kernel(const XP p) {
  const int lane = threadIdx.x;
  const size_t half = (size_t)(p.epoch & 1ull) * p.nranks * kSlotWords;
  // publish this rank's values in every rank's mailbox
  for (int q = lane; q < p.nranks; q += 32) {
    unsigned long long* slot = p.mb[q] + half + (size_t)p.rank * kSlotWords;
    for (int k = 0; k < p.count; ++k) slot[1 + k] = load_bits(p.in, p.dtype, k);
    __threadfence_system();
    st_release_sys(slot, p.epoch);
  }
  // wait, bounded, for every rank's values in the local mailbox
  bool ok = true;
  for (int q = lane; q < p.nranks; q += 32) {
    const unsigned long long* flag = p.mb[p.rank] + half + (size_t)q * kSlotWords;
    unsigned it = 0;
    while (ld_acquire_sys(flag) != p.epoch) {
      if (++it > kXrankSpin) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) atomicOr(p.err, kErrXrank);
    return;
  }
  // value k summed over the ranks in rank order; each lane acquires the flag
  // of every slot it reads
  if (lane < p.count) {
    double sd = 0.0;
    float sf = 0.0f;
    long long si = 0;
    for (int q = 0; q < p.nranks; ++q) {
      const unsigned long long* slot = p.mb[p.rank] + half + (size_t)q * kSlotWords;
      (void)ld_acquire_sys(slot);
      const unsigned long long b = *(volatile const unsigned long long*)(slot + 1 + lane);
      switch (p.dtype) {
        case 0: sf = sf + __uint_as_float((unsigned)b); break;
        case 1: sd = sd + __longlong_as_double((long long)b); break;
        case 2: si = (long long)(int)((unsigned)si + (unsigned)b); break;
        default: si = (long long)((unsigned long long)si + b); break;
      }
    }
    switch (p.dtype) {
      case 0: static_cast<float*>(p.out)[lane] = sf; break;
      case 1: static_cast<double*>(p.out)[lane] = sd; break;
      case 2: static_cast<int*>(p.out)[lane] = (int)si; break;
      default: static_cast<long long*>(p.out)[lane] = si; break;
    }
  }
}

int fail(int code, const std::string& m) {
  ccb::set_error(m);
  return code;
}

}  // namespace

extern "C" {

int ccb_xrank_mailbox_bytes(int nranks, size_t* bytes) {
  if (nranks < 1 || nranks > kMaxRanks || !bytes)
    return fail(1, "ccb_xrank_mailbox_bytes: nranks must be in [1, " + std::to_string(kMaxRanks) + "]");
  *bytes = (size_t)2 * nranks * kSlotWords * sizeof(unsigned long long);
  return 0;
}

int ccb_xrank_sum(const void* in, void* out, int count, int dtype, int nranks, int rank, void* const* mailboxes,
                  unsigned long long epoch, unsigned* err, void* stream) {
  if (count < 1 || count > kMaxValues)
    return fail(1, "ccb_xrank_sum: count = " + std::to_string(count) + " is outside [1, " + std::to_string(kMaxValues) + "]");
  if (dtype < 0 || dtype > 3) return fail(1, "ccb_xrank_sum: dtype code " + std::to_string(dtype) + " (0 f32, 1 f64, 2 i32, 3 i64)");
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return fail(1, "ccb_xrank_sum: rank " + std::to_string(rank) + " of " + std::to_string(nranks) + " (at most " +
                       std::to_string(kMaxRanks) + " ranks)");
  if (epoch == 0) return fail(1, "ccb_xrank_sum: epochs start at 1 (a zero-filled mailbox reads as epoch 0)");
  if (!in || !out || !mailboxes || !err) return fail(1, "ccb_xrank_sum: null pointer");
  XP p = {};
  for (int q = 0; q < nranks; ++q) {
    if (!mailboxes[q]) return fail(1, "ccb_xrank_sum: mailbox of rank " + std::to_string(q) + " is null");
    p.mb[q] = static_cast<unsigned long long*>(mailboxes[q]);
  }
  p.in = in;
  p.out = out;
  p.err = err;
  p.epoch = epoch;
  p.nranks = nranks;
  p.rank = rank;
  p.count = count;
  p.dtype = dtype;
  ccb_xrank_sum_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(3, std::string("ccb_xrank_sum launch: ") + cudaGetErrorString(e));
  return 0;
}

}  // extern "C"
