// ccb_skel.cuh -- the hand-written sm_100a kernel skeletons.
//
// Lowering (lower.cpp) emits, per kernel, one functor struct `F` that carries
// the fused scalar body of a CUDACaml graph (element loads, the inlined
// element expression, stores, reduction combiners) and instantiates one of
// the skeletons below with it. The skeletons own everything that is not the
// body: loop structure, 128-bit vectorised access, warp-shuffle reductions
// and scans, the single-pass last-block reduction, decoupled look-back,
// per-row scheduling, atomics, the tiled product.
//
// They replace the per-node kernel templates of the reference compiler
// (lib/lower/lower.ml:232-958) and its fixed geometry (lib/lower/schedule.ml).
// The file is compiled by NVRTC for sm_100a only; it uses builtins and no
// standard headers.
//
// Safety: every wait is bounded (a look-back gives up after a fixed number of
// polls and raises ERR_LOOKBACK in the program's error word), and every
// data-dependent index is checked (a bad gather or scatter index raises
// ERR_GATHER_OOB / ERR_SCATTER_OOB and is clamped or skipped instead of
// being dereferenced). No kernel traps.
#pragma once

namespace ccb {

typedef unsigned long long u64;
typedef long long i64;

enum : unsigned { ERR_GATHER_OOB = 1u, ERR_SCATTER_OOB = 2u, ERR_LOOKBACK = 4u };
constexpr unsigned FULL = 0xffffffffu;
// Poll limits of the bounded waits. A translation unit may set smaller ones
// before including this header (the tests that make a wait run out do).
#ifndef CCB_LOOKBACK_SPIN_LIMIT
#define CCB_LOOKBACK_SPIN_LIMIT (1u << 21)
#endif
#ifndef CCB_MBAR_SPIN_LIMIT
#define CCB_MBAR_SPIN_LIMIT (1u << 22)
#endif
constexpr unsigned LOOKBACK_SPIN_LIMIT = CCB_LOOKBACK_SPIN_LIMIT;

__device__ __forceinline__ void raise_error(unsigned* err, unsigned code) { atomicOr(err, code); }

// A bounds-checked element index: out-of-range indices raise `code` and read
// element 0 instead (the reference device kernel would read out of bounds).
__device__ __forceinline__ int checked_index(int j, long long n, unsigned* err, unsigned code) {
  if ((unsigned)j >= (unsigned long long)n) {
    raise_error(err, code);
    return 0;
  }
  return j;
}

// ---------------------------------------------------------------- vectors
template <class T>
struct __align__(16) V4 {
  T v[4];
};
template <class T>
__device__ __forceinline__ V4<T> ld4(const T* p) {
  return *reinterpret_cast<const V4<T>*>(p);
}
template <class T>
__device__ __forceinline__ void st4(T* p, const V4<T>& x) {
  *reinterpret_cast<V4<T>*>(p) = x;
}
__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<u64>(p) & 15ull) == 0; }

template <class T>
__device__ __forceinline__ T ld_cg(const T* p) {
  return __ldcg(p);
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned* p) { return *(const volatile unsigned*)p; }
__device__ __forceinline__ void st_volatile(unsigned* p, unsigned v) { *(volatile unsigned*)p = v; }

// ---------------------------------------------------------------- warp/block reductions
// Increasing shuffle offsets keep lane order: lane 0 ends with
// v0 (+) v1 (+) ... (+) v31, so a merely associative combiner is respected.
template <class F, class T>
__device__ __forceinline__ T warp_reduce(int r, T v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = F::combine(r, v, __shfl_down_sync(FULL, v, o));
  return v;
}

// ---------------------------------------------------------------- sharded passes
// A Monte-Carlo estimator pass compiled for rank XRANK of XWORLD GPUs of one
// box walks only its slice [XLO, XHI) of the index space (Philox counters are
// the global element index, so the slices together draw exactly the unsplit
// program's numbers). Its last block then combines the block totals of all
// ranks over NVLink peer memory before the scalar tails run, so every rank
// ends with the unsplit program's outputs (up to the summation order) and no
// collective follows the kernel.
//
// Mailboxes: rank q owns one in its own HBM, [2 halves][XWORLD ranks]
// [XSLOT_WORDS u64] (flag = epoch, then the values as 64-bit patterns); P
// carries every rank's as this rank addresses it (xmb[q]: an IPC mapping or a
// peer-enabled allocation) and the run's epoch (xepoch, the same on every
// rank, 1, 2, 3, ... per run). Warp 0 of the last block: lane q writes this
// rank's totals into slot [e & 1][XRANK] of rank q's mailbox, fences at system
// scope and release-stores e into the slot's flag; lane q then polls slot
// [e & 1][q] of the local mailbox (acquire, system scope) until it reads e;
// value r is folded over the ranks in rank order with the pass's own
// combiner, so every rank computes the same bits. Halves alternate by epoch
// parity: a rank writes epoch e + 2 only after every rank published e + 1,
// i.e. after every rank finished reading epoch e. The wait is bounded: after
// XRANK_SPIN polls it raises ERR_XRANK and the scalar tails are skipped (the
// outputs keep their old contents); the kernel returns.
constexpr unsigned ERR_XRANK = 32u;
constexpr int XSLOT_WORDS = 33;  // flag + at most 32 reductions
#ifndef CCB_XRANK_SPIN_LIMIT
#define CCB_XRANK_SPIN_LIMIT (1u << 22)
#endif

template <class...>
using void_t = void;
template <class F, class = void>
struct Shard {
  static constexpr int WORLD = 1, RANK = 0;
  static constexpr long long LO = 0, HI = -1;  // HI < 0: the whole index space [0, n)
};
template <class F>
struct Shard<F, void_t<decltype(F::XWORLD)>> {
  static constexpr int WORLD = F::XWORLD, RANK = F::XRANK;
  static constexpr long long LO = F::XLO, HI = F::XHI;
};

__device__ __forceinline__ void st_release_sys_u64(u64* p, u64 v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ u64 ld_acquire_sys_u64(const u64* p) {
  u64 v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
template <class T>
__device__ __forceinline__ u64 to_bits64(T v) {
  union {
    T t;
    u64 u;
  } x;
  x.u = 0;
  x.t = v;
  return x.u;
}
template <class T>
__device__ __forceinline__ T from_bits64(u64 u) {
  union {
    T t;
    u64 u;
  } x;
  x.u = u;
  return x.t;
}

// Warp 0 of the last block of a sharded pass; tot[r] holds this rank's total
// of reduction r on entry and the all-rank total on a true return.
template <class F, class T>
__device__ __forceinline__ bool xrank_combine(const typename F::P& p, T (*tot)[33]) {
  constexpr int R = F::NRED, W = Shard<F>::WORLD, ME = Shard<F>::RANK;
  static_assert(R <= XSLOT_WORDS - 1, "a sharded pass exchanges at most 32 reductions");
  static_assert(W <= 32, "at most 32 ranks");
  const int lane = threadIdx.x & 31;
  const u64 e = p.xepoch;
  const u64 half = (e & 1ull) * (u64)W * XSLOT_WORDS;
  if (lane < W) {
    u64* slot = p.xmb[lane] + half + (u64)ME * XSLOT_WORDS;
#pragma unroll
    for (int r = 0; r < R; ++r) slot[1 + r] = to_bits64(tot[r][32]);
    __threadfence_system();
    st_release_sys_u64(slot, e);
  }
  bool ok = true;
  if (lane < W) {
    const u64* flag = p.xmb[ME] + half + (u64)lane * XSLOT_WORDS;
    unsigned it = 0;
    while (ld_acquire_sys_u64(flag) != e) {
      if (++it > CCB_XRANK_SPIN_LIMIT) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  if (!__all_sync(FULL, ok)) {
    if (lane == 0) raise_error(p.err, ERR_XRANK);
    return false;
  }
  // every flag reads e; each lane acquires the slots it reads itself
  for (int r = lane; r < R; r += 32) {
    const u64* box = p.xmb[ME] + half;
    (void)ld_acquire_sys_u64(box);
    T v = from_bits64<T>(*(volatile const u64*)(box + 1 + r));
    for (int q = 1; q < W; ++q) {
      (void)ld_acquire_sys_u64(box + (u64)q * XSLOT_WORDS);
      v = F::combine(r, v, from_bits64<T>(*(volatile const u64*)(box + (u64)q * XSLOT_WORDS + 1 + r)));
    }
    tot[r][32] = v;
  }
  return true;
}

// ---------------------------------------------------------------- map / map-reduce
// F provides:
//   struct P { ...; long long n; acc_t* partials; unsigned* ticket; unsigned* err; }
//   typedef acc_t; static constexpr int NRED, VEC, UNROLL; static constexpr bool TAIL;
//   init(acc_t*), identity(r), combine(r,a,b), elem(p,i,acc), elem4(p,i,acc),
//   vec_ok(p), epilogue(p, const acc_t* res)
// and, for a sharded pass, XWORLD, XRANK, XLO, XHI and P::xmb[XWORLD], P::xepoch.
template <class F>
__device__ __forceinline__ void reduce_finish(const typename F::P& p, typename F::acc_t* acc) {
  typedef typename F::acc_t T;
  constexpr int R = F::NRED;
  __shared__ T sh[R][33];
  __shared__ int am_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    T v = warp_reduce<F>(r, acc[r]);
    if (lane == 0) sh[r][warp] = v;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      T v = lane < nw ? sh[r][lane] : F::identity(r);
      v = warp_reduce<F>(r, v);
      if (lane == 0) p.partials[(u64)blockIdx.x * R + r] = v;
    }
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(p.ticket, 1u);
    am_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!am_last) return;
  // Last block: every partial is published. Fold them in a fixed order
  // (thread t takes blocks t, t+B, ... ascending, then the ordered tree), so
  // the result is reproducible for a given grid. The partials of KB blocks
  // are loaded before any is combined, so their L2 round trips overlap: this
  // fold is the serial tail of every launch (one round trip instead of KB).
  __threadfence();
  constexpr int WORDS = R * (int)(sizeof(T) / 4);
  constexpr int KB = WORDS >= 32 ? 1 : (32 / WORDS > 8 ? 8 : 32 / WORDS);
  const unsigned G = gridDim.x;
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = F::identity(r);
  for (unsigned b0 = threadIdx.x; b0 < G; b0 += KB * blockDim.x) {
    T x[KB][R];
#pragma unroll
    for (int k = 0; k < KB; ++k) {
      const unsigned b = b0 + k * blockDim.x;
#pragma unroll
      for (int r = 0; r < R; ++r) x[k][r] = b < G ? ld_cg(&p.partials[(u64)b * R + r]) : F::identity(r);
    }
#pragma unroll
    for (int k = 0; k < KB; ++k) {
      if (b0 + k * blockDim.x < G) {
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = F::combine(r, acc[r], x[k][r]);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    T v = warp_reduce<F>(r, acc[r]);
    if (lane == 0) sh[r][warp] = v;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      T v = lane < nw ? sh[r][lane] : F::identity(r);
      v = warp_reduce<F>(r, v);
      if (lane == 0) sh[r][32] = v;
    }
  }
  __syncthreads();
  bool combined = true;
  if constexpr (Shard<F>::WORLD > 1) {
    __shared__ int xok;
    if (warp == 0) {
      const bool ok = xrank_combine<F>(p, sh);
      if (lane == 0) xok = ok;
    }
    __syncthreads();
    combined = xok != 0;
  }
  if (threadIdx.x == 0) {
    if (combined) {
      T res[R];
#pragma unroll
      for (int r = 0; r < R; ++r) res[r] = sh[r][32];
      F::epilogue(p, res);
    }
    *p.ticket = 0u;  // ready for the next launch
    __threadfence();
  }
}

template <class F>
__device__ __forceinline__ void map_reduce(const typename F::P& p) {
  typedef typename F::acc_t T;
  constexpr int R = F::NRED;
  T acc[R > 0 ? R : 1];
  F::init(acc);
  // Indices are unsigned: n < 2^31 (element indices are int32) and a
  // grid-stride step adds far less than 2^31, so `i + step` never wraps
  // before the bound check. A signed index would overflow past INT_MAX for n
  // near 2^31 and pass `i < n` with a negative value.
  // A sharded pass walks its slice [LO, HI) of the global index space.
  static_assert(Shard<F>::WORLD == 1 || (F::VEC == 0 && R > 0), "only estimator passes are sharded");
  const unsigned n = Shard<F>::HI < 0 ? (unsigned)p.n : (unsigned)Shard<F>::HI;
  const unsigned tid = (unsigned)Shard<F>::LO + blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned nth = gridDim.x * blockDim.x;
  if (F::VEC && F::vec_ok(p)) {
    constexpr unsigned U = F::UNROLL;
    const unsigned n4 = n >> 2;
    unsigned g = tid;
    for (; g + (U - 1) * nth < n4; g += U * nth) {
#pragma unroll
      for (unsigned u = 0; u < U; ++u) F::elem4(p, (int)((g + u * nth) << 2), acc);
    }
    for (; g < n4; g += nth) F::elem4(p, (int)(g << 2), acc);
    for (unsigned i = (n4 << 2) + tid; i < n; i += nth) F::elem(p, (int)i, acc);
  } else if constexpr (F::VEC == 0 && F::ILP) {
    // four independent elements per iteration: four dependency chains for
    // the scheduler (F64 Greeks at 2^28 paths, four instead of two: 2.508 ->
    // 2.442 ms on one box); each thread still folds its elements in
    // ascending order, so the bits do not change
    unsigned i = tid;
    for (; i + 3 * nth < n; i += 4 * nth) {
      F::elem(p, (int)i, acc);
      F::elem(p, (int)(i + nth), acc);
      F::elem(p, (int)(i + 2 * nth), acc);
      F::elem(p, (int)(i + 3 * nth), acc);
    }
    for (; i < n; i += nth) F::elem(p, (int)i, acc);
  } else {
    for (unsigned i = tid; i < n; i += nth) F::elem(p, (int)i, acc);
  }
  if constexpr (R > 0) {
    reduce_finish<F>(p, acc);
  } else if constexpr (F::TAIL) {
    if (blockIdx.x == 0 && threadIdx.x == 0) F::epilogue(p, acc);
  }
}

// ---------------------------------------------------------------- block scan helpers
// Inclusive warp scan, order preserving (earlier lanes on the left).
template <class F, class T>
__device__ __forceinline__ T warp_scan_incl(T v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v = F::combine(y, v);
  }
  return v;
}

// Block-wide exclusive scan of one value per thread. Returns the exclusive
// prefix of this thread; *total receives the block total. BLOCK threads.
template <class F, int BLOCK, class T>
__device__ __forceinline__ T block_scan_excl(T v, T* total, T* s_warp /* [BLOCK/32 + 1] */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = BLOCK / 32;
  T incl = warp_scan_incl<F>(v, lane);
  T excl_in_warp = __shfl_up_sync(FULL, incl, 1);
  if (lane == 0) excl_in_warp = F::identity();
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T w = lane < NW ? s_warp[lane] : F::identity();
    w = warp_scan_incl<F>(w, lane);
    if (lane < NW) s_warp[lane] = w;
  }
  __syncthreads();
  const T warp_prefix = warp == 0 ? F::identity() : s_warp[warp - 1];
  *total = s_warp[NW - 1];
  return warp == 0 ? excl_in_warp : F::combine(warp_prefix, excl_in_warp);
}

// ---------------------------------------------------------------- single-pass flat scan
// Decoupled look-back (Merrill & Garland, "Single-pass Parallel Prefix Scan
// with Decoupled Look-back", 2016). Tiles are claimed in launch order through
// p.tile_counter, so a tile only ever waits on tiles that are already running.
// Status words carry the launch epoch, so no clearing pass is needed between
// launches. Each poll inspects LB_WINDOWS x 32 predecessors. One window is
// fastest on the B200: the nearest inclusive prefix is usually within 32
// tiles, and every further status word polled is L2 traffic that the tile
// streams wait behind (2^28 F32: 4 windows 0.494 ms, 2 0.471, 1 0.455).
//
// 4-byte T: one 64-bit status word per tile, [epoch:30 | flag:2 | value:32],
// written and read with single relaxed 64-bit accesses (no fence needed:
// flag and value arrive together). 8-byte T: a 32-bit [epoch | flag] word plus
// separate aggregate / inclusive arrays, ordered with fences.
//
// F provides T, identity(), combine(a,b), load(p,i), load4(p,i,T*),
// store(p,i,v), store4(p,i,const T*), vec_ok(p); P provides n, tile_counter,
// status (u64, 4-byte T) or flags + aggs + incls (8-byte T), epoch, err.
constexpr int LB_WINDOWS = 1;

__device__ __forceinline__ u64 ld_relaxed_u64(const u64* p) {
  u64 v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(u64* p, u64 v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
template <class T>
__device__ __forceinline__ unsigned to_bits32(T v) {
  union {
    T t;
    unsigned u;
  } x;
  x.t = v;
  return x.u;
}
template <class T>
__device__ __forceinline__ T from_bits32(unsigned u) {
  union {
    T t;
    unsigned u;
  } x;
  x.u = u;
  return x.t;
}

// Fold one window of 32 predecessors (lane l = tile pred - l, older to the
// left) into prefix; returns true when an inclusive prefix ended the walk.
template <class F>
__device__ __forceinline__ bool fold_window(typename F::T v, bool is_p, typename F::T& prefix, int lane) {
  typedef typename F::T T;
  const unsigned pmask = __ballot_sync(FULL, is_p);
  const int stop = pmask ? __ffs(pmask) - 1 : 31;
  if (lane > stop) v = F::identity();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_down_sync(FULL, v, o);
    v = F::combine(y, v);
  }
  prefix = F::combine(__shfl_sync(FULL, v, 0), prefix);
  return pmask != 0;
}

template <class F>
__device__ __forceinline__ typename F::T lookback(const typename F::P& p, unsigned tile, typename F::T agg, int lane) {
  typedef typename F::T T;
  T prefix = F::identity();
  unsigned spins = 0;
  if constexpr (sizeof(T) == 4) {
    const u64 ep = (u64)p.epoch << 34;
    const u64 FA = 1ull << 32, FP = 2ull << 32;
    if (tile == 0) {
      if (lane == 0) st_relaxed_u64(&p.status[0], ep | FP | to_bits32(agg));
      return prefix;
    }
    if (lane == 0) st_relaxed_u64(&p.status[tile], ep | FA | to_bits32(agg));
    long long pred = (long long)tile - 1;
    const u64 sentinel = ep | FP | to_bits32(F::identity());
    while (true) {
      u64 s[LB_WINDOWS];
#pragma unroll
      for (int j = 0; j < LB_WINDOWS; ++j) {
        const long long idx = pred - lane - 32 * j;
        s[j] = idx >= 0 ? ld_relaxed_u64(&p.status[idx]) : sentinel;
      }
      while (true) {
        bool ok = true;
#pragma unroll
        for (int j = 0; j < LB_WINDOWS; ++j) ok = ok && (s[j] >> 34) == (u64)p.epoch && ((s[j] >> 32) & 3u) != 0;
        if (__all_sync(FULL, ok)) break;
        if (++spins > LOOKBACK_SPIN_LIMIT) {
          if (lane == 0) raise_error(p.err, ERR_LOOKBACK);
          return F::identity();
        }
        __nanosleep(16);
#pragma unroll
        for (int j = 0; j < LB_WINDOWS; ++j) {
          const long long idx = pred - lane - 32 * j;
          const bool vj = (s[j] >> 34) == (u64)p.epoch && ((s[j] >> 32) & 3u) != 0;
          if (!vj && idx >= 0) s[j] = ld_relaxed_u64(&p.status[idx]);
        }
      }
      bool done = false;
#pragma unroll
      for (int j = 0; j < LB_WINDOWS; ++j) {
        if (!done) done = fold_window<F>(from_bits32<T>((unsigned)s[j]), ((s[j] >> 32) & 3u) == 2u, prefix, lane);
      }
      if (done) break;
      pred -= 32 * LB_WINDOWS;
    }
    if (lane == 0) st_relaxed_u64(&p.status[tile], ep | FP | to_bits32(F::combine(prefix, agg)));
    return prefix;
  } else {
    const unsigned ep = ((unsigned)p.epoch) << 2;
    if (tile == 0) {
      if (lane == 0) {
        p.incls[0] = agg;
        __threadfence();
        st_volatile(&p.flags[0], ep | 2u);
      }
      return prefix;
    }
    if (lane == 0) {
      p.aggs[tile] = agg;
      __threadfence();
      st_volatile(&p.flags[tile], ep | 1u);
    }
    long long pred = (long long)tile - 1;
    while (true) {
      unsigned f[LB_WINDOWS];
      while (true) {
        bool ok = true;
#pragma unroll
        for (int j = 0; j < LB_WINDOWS; ++j) {
          const long long idx = pred - lane - 32 * j;
          f[j] = idx >= 0 ? ld_volatile(&p.flags[idx]) : (ep | 2u);
          ok = ok && (f[j] & ~3u) == ep && (f[j] & 3u) != 0u;
        }
        if (__all_sync(FULL, ok)) break;
        if (++spins > LOOKBACK_SPIN_LIMIT) {
          if (lane == 0) raise_error(p.err, ERR_LOOKBACK);
          return F::identity();
        }
        __nanosleep(16);
      }
      __threadfence();
      bool done = false;
#pragma unroll
      for (int j = 0; j < LB_WINDOWS; ++j) {
        if (!done) {
          const long long idx = pred - lane - 32 * j;
          T v = F::identity();
          if (idx >= 0) v = ((f[j] & 3u) == 2u) ? ld_cg(&p.incls[idx]) : ld_cg(&p.aggs[idx]);
          done = fold_window<F>(v, (f[j] & 3u) == 2u, prefix, lane);
        }
      }
      if (done) break;
      pred -= 32 * LB_WINDOWS;
    }
    if (lane == 0) {
      p.incls[tile] = F::combine(prefix, agg);
      __threadfence();
      st_volatile(&p.flags[tile], ep | 2u);
    }
    return prefix;
  }
}

template <class F, int ITEMS>
__device__ __forceinline__ void scan_flat(const typename F::P& p) {
  typedef typename F::T T;
  constexpr int BLOCK = 256;
  constexpr long long TILE = (long long)BLOCK * ITEMS;
  __shared__ unsigned s_tile;
  __shared__ T s_warp[BLOCK / 32 + 1];
  __shared__ T s_prefix;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.tile_counter, 1u);
  __syncthreads();
  const unsigned tile = s_tile;
  const long long n = p.n;
  const long long base = (long long)tile * TILE + (long long)threadIdx.x * ITEMS;
  T x[ITEMS];
  const bool full_vec = F::VEC && base + ITEMS <= n && F::vec_ok(p);
  if (full_vec) {
#pragma unroll
    for (int k = 0; k < ITEMS; k += 4) F::load4(p, base + k, &x[k]);
  } else {
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) x[k] = (base + k < n) ? F::load(p, base + k) : F::identity();
  }
#pragma unroll
  for (int k = 1; k < ITEMS; ++k) x[k] = F::combine(x[k - 1], x[k]);
  T total;
  const T excl = block_scan_excl<F, BLOCK>(x[ITEMS - 1], &total, s_warp);
  if ((threadIdx.x >> 5) == 0) {
    const T prefix = lookback<F>(p, tile, total, threadIdx.x & 31);
    if (threadIdx.x == 0) s_prefix = prefix;
  }
  __syncthreads();
  const T pre = F::combine(s_prefix, excl);
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) x[k] = F::combine(pre, x[k]);
  if (full_vec) {
#pragma unroll
    for (int k = 0; k < ITEMS; k += 4) F::store4(p, base + k, &x[k]);
  } else {
#pragma unroll
    for (int k = 0; k < ITEMS; ++k)
      if (base + k < n) F::store(p, base + k, x[k]);
  }
  // The block holding the last ticket runs after every other block has taken
  // its ticket, so it can rearm the counter for the next launch.
  if (threadIdx.x == 0 && tile == gridDim.x - 1) atomicExch(p.tile_counter, 0u);
}

// ---------------------------------------------------------------- staged flat scan (TMA)
// Persistent single-pass scan of a 4-byte source buffer. Each CTA keeps three
// tiles of STRIPS x 4 KiB (the lowering uses 6: 24 KiB, 3 CTAs per SM) in
// flight in shared memory: one arriving by a 1-D bulk async
// copy (cp.async.bulk, the TMA engine; never multicast), one whose aggregate
// it publishes, and one it finishes. Publishing tile k's aggregate before
// walking back for tile k-1 gives every predecessor a full iteration to
// publish, so the walk rarely waits; the walk itself overlaps the next bulk
// load. Tiles are claimed dynamically in order (forward progress as in
// scan_flat). The tile aggregate folds each thread's strided chunks, i.e. it
// assumes a commutative combiner, as the reference's device reduction does;
// the scanned values themselves are combined in order.
// F provides T (4 bytes), identity(), combine(a,b), src(p), dst(p); P provides
// n, tile_counter, done_counter, status, epoch, err.
constexpr unsigned ERR_TMA = 8u;
constexpr unsigned MBAR_SPIN_LIMIT = CCB_MBAR_SPIN_LIMIT;

__device__ __forceinline__ unsigned smem_u32(const void* ptr) { return (unsigned)__cvta_generic_to_shared(ptr); }
__device__ __forceinline__ void mbar_init(u64* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(u64* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, u64* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ bool mbar_try_wait(u64* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for a bulk copy; on timeout raise ERR_TMA and keep waiting, again
// bounded, so the copy in flight lands before the CTA moves on.
__device__ __forceinline__ void mbar_wait(u64* bar, unsigned parity, unsigned* err) {
  for (unsigned it = 0; it < MBAR_SPIN_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return;
  if (threadIdx.x == 0) raise_error(err, ERR_TMA);
  for (unsigned it = 0; it < MBAR_SPIN_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return;
}

template <class F>
__device__ __forceinline__ void publish_aggregate(const typename F::P& p, unsigned tile, typename F::T agg) {
  const u64 ep = (u64)p.epoch << 34;
  st_relaxed_u64(&p.status[tile], ep | (tile == 0 ? (2ull << 32) : (1ull << 32)) | to_bits32(agg));
}

// Walk back from `tile` (whose aggregate is published) to the nearest
// inclusive prefix; publish tile's own inclusive prefix; return the exclusive
// prefix. Warp-wide.
template <class F>
__device__ __forceinline__ typename F::T walk_back(const typename F::P& p, unsigned tile, typename F::T agg, int lane) {
  typedef typename F::T T;
  T prefix = F::identity();
  if (tile == 0) return prefix;
  const u64 ep = (u64)p.epoch << 34;
  const u64 sentinel = ep | (2ull << 32) | to_bits32(F::identity());
  long long pred = (long long)tile - 1;
  unsigned spins = 0;
  while (true) {
    u64 s[LB_WINDOWS];
#pragma unroll
    for (int j = 0; j < LB_WINDOWS; ++j) {
      const long long idx = pred - lane - 32 * j;
      s[j] = idx >= 0 ? ld_relaxed_u64(&p.status[idx]) : sentinel;
    }
    bool done = false;
#pragma unroll
    for (int j = 0; j < LB_WINDOWS; ++j) {
      if (done) break;
      // this window must be fully published before it can be folded
      while (!__all_sync(FULL, (s[j] >> 34) == (u64)p.epoch && ((s[j] >> 32) & 3u) != 0)) {
        if (++spins > LOOKBACK_SPIN_LIMIT) {
          if (lane == 0) raise_error(p.err, ERR_LOOKBACK);
          return F::identity();
        }
        __nanosleep(16);
        const long long idx = pred - lane - 32 * j;
        if (idx >= 0) s[j] = ld_relaxed_u64(&p.status[idx]);
      }
      done = fold_window<F>(from_bits32<T>((unsigned)s[j]), ((s[j] >> 32) & 3u) == 2u, prefix, lane);
    }
    if (done) break;
    pred -= 32 * LB_WINDOWS;
  }
  if (lane == 0) st_relaxed_u64(&p.status[tile], ep | (2ull << 32) | to_bits32(F::combine(prefix, agg)));
  return prefix;
}

template <class F, int STRIPS>
__device__ __forceinline__ void scan_flat_staged(const typename F::P& p) {
  typedef typename F::T T;
  static_assert(sizeof(T) == 4, "staged scan is for 4-byte element types");
  constexpr int BLOCK = 256, NBUF = 3, STRIP = BLOCK * 4, TILE = STRIP * STRIPS;
  constexpr int NW = BLOCK / 32;
  constexpr int NE = STRIPS * NW, PER = (NE + 31) / 32;  // chunk totals, PER per lane in the fold
  static_assert(NE <= 32 * 4, "at most 4 chunk totals per lane");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* buf = reinterpret_cast<T*>(smem_raw);
  u64* bars = reinterpret_cast<u64*>(smem_raw + (size_t)NBUF * TILE * sizeof(T));
  __shared__ int s_tile[NBUF];
  __shared__ int s_tma[NBUF];
  __shared__ T s_ws[STRIPS * NW];   // warp totals per strip, (strip, warp) order
  __shared__ T s_off[STRIPS * NW];  // their exclusive prefixes within the tile
  __shared__ T s_prefix;
  const long long n = p.n;
  const long long ntiles = (n + TILE - 1) / TILE;
  const T* src = F::src(p);
  T* dst = F::dst(p);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool src_aligned = aligned16(src);
  const bool dst_aligned = aligned16(dst);
  // The phase parity of each ring buffer's barrier, one bit per buffer in a
  // register (an array indexed by k % NBUF would live in local memory).
  unsigned parity = 0u;

  // thread 0: claim the next tile into buffer b and start its bulk load
  auto claim = [&](int b) {
    const unsigned t = atomicAdd(p.tile_counter, 1u);
    const bool ok = (long long)t < ntiles;
    s_tile[b] = ok ? (int)t : -1;
    s_tma[b] = 0;
    if (ok) {
      const long long base = (long long)t * TILE;
      if (src_aligned && base + TILE <= n) {
        s_tma[b] = 1;
        fence_proxy_async_smem();
        mbar_expect_tx(&bars[b], TILE * (unsigned)sizeof(T));
        bulk_load(buf + (size_t)b * TILE, src + base, TILE * (unsigned)sizeof(T), &bars[b]);
      }
    }
  };

  if (tid == 0) {
    for (int b = 0; b < NBUF; ++b) mbar_init(&bars[b], 1);
    mbar_fence_init();
    claim(0);
    claim(1);
  }
  __syncthreads();

  // Thread tid owns chunk (strip s, tid): elements [s*STRIP + 4*tid, +4) of
  // the tile, so chunk order (s, tid) is element order.
  T agg_prev = F::identity();
  T off_prev[STRIPS];
#pragma unroll
  for (int sI = 0; sI < STRIPS; ++sI) off_prev[sI] = F::identity();
  for (int k = 0;; ++k) {
    const int bc = k % NBUF;               // tile k: scan offsets + aggregate
    const int bp = (k + NBUF - 1) % NBUF;  // tile k-1: prefix + store
    const int tc = s_tile[bc];
    const int tp = k > 0 ? s_tile[bp] : -1;
    if (tc < 0 && tp < 0) break;
    T agg_cur = F::identity();
    T off_cur[STRIPS];
    if (tc >= 0) {
      const long long base = (long long)tc * TILE;
      T* b = buf + (size_t)bc * TILE;
      if (s_tma[bc]) {
        mbar_wait(&bars[bc], (parity >> bc) & 1u, p.err);
        parity ^= 1u << bc;
      } else {
        for (int e = tid; e < TILE; e += BLOCK) b[e] = (base + e < n) ? src[base + e] : F::identity();
        __syncthreads();
      }
      T excl_w[STRIPS];
#pragma unroll
      for (int sI = 0; sI < STRIPS; ++sI) {
        const V4<T> v = *reinterpret_cast<const V4<T>*>(b + sI * STRIP + 4 * tid);
        const T tot = F::combine(F::combine(F::combine(v.v[0], v.v[1]), v.v[2]), v.v[3]);
        const T incl = warp_scan_incl<F>(tot, lane);
        T ex = __shfl_up_sync(FULL, incl, 1);
        excl_w[sI] = lane == 0 ? F::identity() : ex;
        if (lane == 31) s_ws[sI * NW + warp] = incl;
      }
      __syncthreads();
      if (warp == 0) {
        // NE warp totals in (strip, warp) order, PER consecutive ones per lane
        T w[PER];
        T part = F::identity();
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          const int e = PER * lane + q;
          w[q] = e < NE ? s_ws[e] : F::identity();
          part = F::combine(part, w[q]);
        }
        const T incl = warp_scan_incl<F>(part, lane);
        T ex = __shfl_up_sync(FULL, incl, 1);
        if (lane == 0) ex = F::identity();
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          const int e = PER * lane + q;
          if (e < NE) s_off[e] = ex;
          ex = F::combine(ex, w[q]);
        }
        if (lane == 31) publish_aggregate<F>(p, (unsigned)tc, incl);
        agg_cur = __shfl_sync(FULL, incl, 31);
      }
      __syncthreads();
#pragma unroll
      for (int sI = 0; sI < STRIPS; ++sI) off_cur[sI] = F::combine(s_off[sI * NW + warp], excl_w[sI]);
    }
    if (tp >= 0) {
      if (warp == 0) {
        const T pre = walk_back<F>(p, (unsigned)tp, agg_prev, lane);
        if (lane == 0) s_prefix = pre;
      }
      __syncthreads();
      const T carry = s_prefix;
      const long long base = (long long)tp * TILE;
      const T* b = buf + (size_t)bp * TILE;
#pragma unroll
      for (int sI = 0; sI < STRIPS; ++sI) {
        const int e0 = sI * STRIP + 4 * tid;
        V4<T> v = *reinterpret_cast<const V4<T>*>(b + e0);
        const T pre = F::combine(carry, off_prev[sI]);
        v.v[0] = F::combine(pre, v.v[0]);
#pragma unroll
        for (int q = 1; q < 4; ++q) v.v[q] = F::combine(v.v[q - 1], v.v[q]);
        const long long g = base + e0;
        if (dst_aligned && g + 4 <= n) {
          st4(dst + g, v);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (g + q < n) dst[g + q] = v.v[q];
        }
      }
    }
    // buffer bp is free (or was never used): claim tile k+2 into it
    __syncthreads();
    if (tid == 0) claim((k + 2) % NBUF);
    __syncthreads();
    agg_prev = agg_cur;
#pragma unroll
    for (int sI = 0; sI < STRIPS; ++sI) off_prev[sI] = off_cur[sI];
  }
  // the last CTA out rearms the counters for the next launch
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.done_counter, 1u) == gridDim.x - 1) {
      *p.tile_counter = 0u;
      *p.done_counter = 0u;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------- staged rows (TMA)
// Row reduction and row scan over [rows; n] of a 4-byte source buffer read at
// the element index, n a multiple of 4 (so every row starts 16-byte aligned
// when the buffer does). Each CTA walks its rows (blockIdx.x, + gridDim.x,
// ...) as one sequence of chunks of up to ROW_STRIPS x 1024 elements; thread
// 0 keeps ROW_RING chunks in flight by 1-D bulk copies (cp.async.bulk, the
// TMA engine, never multicast), so the next row's first chunks are already
// arriving while a row finishes. A chunk is consumed as strips of 1024
// elements, thread t owning elements [4t, 4t + 4) of each strip (conflict-free
// 16-byte shared reads). If the buffer is not 16-byte aligned the CTA stages
// the chunks with plain loads instead. Every wait is bounded (ERR_TMA).
// F provides T, identity(), combine(a,b), src(p); reductions store_row(p,r,v),
// scans dst(p); P provides n, rows, err.
constexpr int ROW_STRIPS = 4, ROW_RING = 4;
constexpr int ROW_CHUNK = ROW_STRIPS * 1024;
constexpr unsigned ROW_SMEM = ROW_RING * ROW_CHUNK * 4 + ROW_RING * 8;

template <class F, bool SCAN>
__device__ __forceinline__ void rows_staged(const typename F::P& p) {
  typedef typename F::T T;
  static_assert(sizeof(T) == 4, "staged rows are for 4-byte element types");
  constexpr int BLOCK = 256, C = ROW_CHUNK, NB = ROW_RING, NW = BLOCK / 32;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  u64* bars = reinterpret_cast<u64*>(smem_raw + (size_t)NB * C * sizeof(T));
  __shared__ T s_w[ROW_STRIPS * NW];  // warp totals per strip, (strip, warp) order
  __shared__ T s_red[NW];
  __shared__ T s_tot;  // a scanned chunk's total
  static_assert(ROW_STRIPS * NW == 32, "one warp total per lane in the offset scan");
  const long long n = p.n, rows = p.rows;
  const T* src = F::src(p);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long cpr = (n + C - 1) / C;  // chunks per row
  const long long mine = (long long)blockIdx.x < rows ? (rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const long long total = mine * cpr;
  const bool tma = aligned16(src);
  struct Chunk {
    long long row, c0;
    int cnt;
  };
  auto where = [&](long long q) {  // chunk q of this CTA's sequence
    Chunk k;
    k.row = blockIdx.x + (q / cpr) * (long long)gridDim.x;
    k.c0 = (q % cpr) * (long long)C;
    const long long left = n - k.c0;
    k.cnt = (int)(left < C ? left : C);
    return k;
  };
  auto issue = [&](long long q) {  // thread 0 only
    const Chunk k = where(q);
    const long long row = k.row, c0 = k.c0;
    const int cnt = k.cnt;
    const int b = (int)(q % NB);
    fence_proxy_async_smem();
    mbar_expect_tx(&bars[b], (unsigned)cnt * 4u);
    bulk_load(ring + (size_t)b * C, src + row * n + c0, (unsigned)cnt * 4u, &bars[b]);
  };
  if (tid == 0) {
    for (int b = 0; b < NB; ++b) mbar_init(&bars[b], 1);
    mbar_fence_init();
    if (tma)
      for (long long q = 0; q < total && q < NB; ++q) issue(q);
  }
  __syncthreads();
  unsigned parity = 0u;  // one phase bit per ring buffer
  T acc = F::identity(), carry = F::identity();
  for (long long q = 0; q < total; ++q) {
    const Chunk k = where(q);
    const long long row = k.row, c0 = k.c0;
    const int cnt = k.cnt;
    const int b = (int)(q % NB);
    T* buf = ring + (size_t)b * C;
    if (tma) {
      mbar_wait(&bars[b], (parity >> b) & 1u, p.err);
      parity ^= 1u << b;
    } else {
      for (int e = tid; e < cnt; e += BLOCK) buf[e] = src[row * n + c0 + e];
      __syncthreads();
    }
    if constexpr (!SCAN) {
#pragma unroll
      for (int sI = 0; sI < ROW_STRIPS; ++sI) {
        const int e = sI * 1024 + 4 * tid;
        if (e < cnt) {
          const V4<T> v = *reinterpret_cast<const V4<T>*>(buf + e);
          acc = F::combine(acc, v.v[0]);
          acc = F::combine(acc, v.v[1]);
          acc = F::combine(acc, v.v[2]);
          acc = F::combine(acc, v.v[3]);
        }
      }
    } else {
      // strip scan: thread totals -> warp scans -> (strip, warp) offsets
      V4<T> v[ROW_STRIPS];
      T excl[ROW_STRIPS];
#pragma unroll
      for (int sI = 0; sI < ROW_STRIPS; ++sI) {
        const int e = sI * 1024 + 4 * tid;
        if (e < cnt) {
          v[sI] = *reinterpret_cast<const V4<T>*>(buf + e);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) v[sI].v[k] = F::identity();
        }
#pragma unroll
        for (int k = 1; k < 4; ++k) v[sI].v[k] = F::combine(v[sI].v[k - 1], v[sI].v[k]);
        const T incl = warp_scan_incl<F>(v[sI].v[3], lane);
        T ex = __shfl_up_sync(FULL, incl, 1);
        excl[sI] = lane == 0 ? F::identity() : ex;
        if (lane == 31) s_w[sI * NW + warp] = incl;
      }
      __syncthreads();
      if (warp == 0) {  // the 32 warp totals in (strip, warp) order, one per lane
        const T incl = warp_scan_incl<F>(s_w[lane], lane);
        T ex = __shfl_up_sync(FULL, incl, 1);
        if (lane == 0) ex = F::identity();
        s_w[lane] = ex;
        if (lane == 31) s_tot = incl;
      }
      __syncthreads();
      const T chunk_total = s_tot;
      T* dst = F::dst(p) + row * n + c0;
      const bool vec = aligned16(dst);
#pragma unroll
      for (int sI = 0; sI < ROW_STRIPS; ++sI) {
        const int e = sI * 1024 + 4 * tid;
        const T pre = F::combine(carry, F::combine(s_w[sI * NW + warp], excl[sI]));
        V4<T> o;
#pragma unroll
        for (int k = 0; k < 4; ++k) o.v[k] = F::combine(pre, v[sI].v[k]);
        if (e + 4 <= cnt && vec) {
          st4(dst + e, o);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (e + k < cnt) dst[e + k] = o.v[k];
        }
      }
      carry = F::combine(carry, chunk_total);
    }
    __syncthreads();  // every thread is done with buf (and with s_w)
    if (tma && tid == 0 && q + NB < total) issue(q + NB);
    if (c0 + cnt >= n) {  // the row's last chunk
      if constexpr (!SCAN) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) acc = F::combine(acc, __shfl_down_sync(FULL, acc, o));
        if (lane == 0) s_red[warp] = acc;
        __syncthreads();
        if (warp == 0) {
          T r = lane < NW ? s_red[lane] : F::identity();
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) r = F::combine(r, __shfl_down_sync(FULL, r, o));
          if (lane == 0) F::store_row(p, row, r);
        }
        __syncthreads();
        acc = F::identity();
      } else {
        carry = F::identity();
      }
    }
  }
}

// ---------------------------------------------------------------- transpose
// A materialised Dsl.transpose of a buffer: src [rows; cols] -> dst
// [cols; rows], in 32 x 32 tiles staged through shared memory so that both
// the reads (rows of src) and the writes (rows of dst) are coalesced.
// Persistent grid over tiles. F provides T, src(p), dst(p); P provides
// rows, cols.
template <class F>
__device__ __forceinline__ void transpose_tiles(const typename F::P& p) {
  typedef typename F::T T;
  __shared__ T tile[32][33];
  const long long rows = p.rows, cols = p.cols;
  const long long tr = (rows + 31) / 32, tcn = (cols + 31) / 32;
  const T* src = F::src(p);
  T* dst = F::dst(p);
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (long long t = blockIdx.x; t < tr * tcn; t += gridDim.x) {
    const long long r0 = (t / tcn) * 32, c0 = (t % tcn) * 32;
#pragma unroll
    for (int k = ty; k < 32; k += 8) {
      const long long r = r0 + k, c = c0 + tx;
      if (r < rows && c < cols) tile[k][tx] = src[r * cols + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = ty; k < 32; k += 8) {
      const long long c = c0 + k, r = r0 + tx;
      if (c < cols && r < rows) dst[c * rows + r] = tile[tx][k];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- rows
// Row kernels over [rows; n] (last axis). F provides T, identity(),
// combine(a,b), load(p,i), load4(p,i,T*), vec_ok(p) and, for reductions,
// store_row(p,r,v); for scans store(p,i,v), store4(p,i,const T*).
template <class F>
__device__ __forceinline__ void reduce_rows_block(const typename F::P& p) {
  typedef typename F::T T;
  __shared__ T sh[33];
  const long long n = p.n;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const bool vec = F::VEC && (n & 3) == 0 && F::vec_ok(p);
  for (long long row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const long long base = row * n;
    T acc = F::identity();
    if (vec) {
      long long j = (long long)threadIdx.x * 4;
      const long long step = (long long)blockDim.x * 4;
      for (; j + step < n; j += 2 * step) {
        T a[4], b[4];
        F::load4(p, base + j, a);
        F::load4(p, base + j + step, b);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc = F::combine(acc, a[k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc = F::combine(acc, b[k]);
      }
      if (j < n) {
        T a[4];
        F::load4(p, base + j, a);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc = F::combine(acc, a[k]);
      }
    } else {
      for (long long j = threadIdx.x; j < n; j += blockDim.x) acc = F::combine(acc, F::load(p, base + j));
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) acc = F::combine(acc, __shfl_down_sync(FULL, acc, o));
    if (lane == 0) sh[warp] = acc;
    __syncthreads();
    if (warp == 0) {
      T v = lane < nw ? sh[lane] : F::identity();
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) v = F::combine(v, __shfl_down_sync(FULL, v, o));
      if (lane == 0) F::store_row(p, row, v);
    }
    __syncthreads();
  }
}

template <class F>
__device__ __forceinline__ void reduce_rows_warp(const typename F::P& p) {
  typedef typename F::T T;
  const long long n = p.n;
  const int lane = threadIdx.x & 31;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long row = wid; row < p.rows; row += nwarps) {
    const long long base = row * n;
    T acc = F::identity();
    for (long long j = lane; j < n; j += 32) acc = F::combine(acc, F::load(p, base + j));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) acc = F::combine(acc, __shfl_down_sync(FULL, acc, o));
    if (lane == 0) F::store_row(p, row, acc);
  }
}

// One block per row; the row is walked in chunks of BLOCK*ITEMS with a carry.
template <class F, int ITEMS>
__device__ __forceinline__ void scan_rows_block(const typename F::P& p) {
  typedef typename F::T T;
  constexpr int BLOCK = 256;
  __shared__ T s_warp[BLOCK / 32 + 1];
  const long long n = p.n;
  const bool vec = F::VEC && (n & 3) == 0 && F::vec_ok(p);
  for (long long row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const long long rbase = row * n;
    T carry = F::identity();
    for (long long c0 = 0; c0 < n; c0 += (long long)BLOCK * ITEMS) {
      const long long j0 = c0 + (long long)threadIdx.x * ITEMS;
      T x[ITEMS];
      const bool fv = vec && j0 + ITEMS <= n;
      if (fv) {
#pragma unroll
        for (int k = 0; k < ITEMS; k += 4) F::load4(p, rbase + j0 + k, &x[k]);
      } else {
#pragma unroll
        for (int k = 0; k < ITEMS; ++k) x[k] = (j0 + k < n) ? F::load(p, rbase + j0 + k) : F::identity();
      }
#pragma unroll
      for (int k = 1; k < ITEMS; ++k) x[k] = F::combine(x[k - 1], x[k]);
      T total;
      const T excl = block_scan_excl<F, BLOCK>(x[ITEMS - 1], &total, s_warp);
      const T pre = F::combine(carry, excl);
#pragma unroll
      for (int k = 0; k < ITEMS; ++k) x[k] = F::combine(pre, x[k]);
      if (fv) {
#pragma unroll
        for (int k = 0; k < ITEMS; k += 4) F::store4(p, rbase + j0 + k, &x[k]);
      } else {
#pragma unroll
        for (int k = 0; k < ITEMS; ++k)
          if (j0 + k < n) F::store(p, rbase + j0 + k, x[k]);
      }
      carry = F::combine(carry, total);
      __syncthreads();
    }
  }
}

// One warp per row, for rows shorter than a block's chunk.
template <class F>
__device__ __forceinline__ void scan_rows_warp(const typename F::P& p) {
  typedef typename F::T T;
  const long long n = p.n;
  const int lane = threadIdx.x & 31;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long row = wid; row < p.rows; row += nwarps) {
    const long long rbase = row * n;
    T carry = F::identity();
    for (long long c0 = 0; c0 < n; c0 += 32) {
      const long long j = c0 + lane;
      T x = j < n ? F::load(p, rbase + j) : F::identity();
      T incl = warp_scan_incl<F>(x, lane);
      T v = F::combine(carry, incl);
      if (j < n) F::store(p, rbase + j, v);
      carry = __shfl_sync(FULL, v, 31);
    }
  }
}

// Row scan whose result is only needed transposed (LSM's S, read date by
// date): a block owns 32 consecutive rows, warp w scans rows w, w+8, w+16,
// w+24 in 32-column chunks, each chunk's values (through F::value, the fused
// store pass if any) go to a shared 32 x 33 tile, and the block writes the
// chunk's 32 columns as rows of the [n; rows] output, 32 consecutive rows of
// 4 or 8 bytes each. F provides T, U (output element), identity, combine,
// load(p, i), value(p, i, v), tout(p); P provides n (row length), rows.
template <class F>
__device__ __forceinline__ void scan_rows_warp_t(const typename F::P& p) {
  typedef typename F::T T;
  typedef typename F::U U;
  __shared__ U tile[32][33];
  const long long n = p.n, rows = p.rows;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  U* out = F::tout(p);
  for (long long row0 = (long long)blockIdx.x * 32; row0 < rows; row0 += (long long)gridDim.x * 32) {
    T carry[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) carry[q] = F::identity();
    for (long long c0 = 0; c0 < n; c0 += 32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = warp + 8 * q;
        const long long row = row0 + r, j = c0 + lane;
        const bool in = row < rows && j < n;
        const T x = in ? F::load(p, row * n + j) : F::identity();
        const T v = F::combine(carry[q], warp_scan_incl<F>(x, lane));
        if (in) tile[lane][r] = F::value(p, row * n + j, v);
        carry[q] = __shfl_sync(FULL, v, 31);
      }
      __syncthreads();
      for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
        const int c = e >> 5, r = e & 31;
        const long long row = row0 + r, col = c0 + c;
        if (row < rows && col < n) out[col * rows + row] = tile[c][r];
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- scatter_add
// out is zero-filled by the executor (a memset) before this runs; every
// element lands through an atomic add. F provides T, idx(p,i), val(p,i);
// P provides n (source elements), m (output elements), out, err.
//
// Each thread loads SCATTER_BATCH (index, value) pairs, a grid stride apart,
// before issuing their atomics, so that many loads are in flight per thread.
constexpr int SCATTER_BATCH = 8;

template <class F>
__device__ __forceinline__ void scatter_add(const typename F::P& p) {
  typedef typename F::T T;
  const long long n = p.n;
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += nth * SCATTER_BATCH) {
    int j[SCATTER_BATCH];
    T v[SCATTER_BATCH];
#pragma unroll
    for (int u = 0; u < SCATTER_BATCH; ++u) {
      const long long i = i0 + u * nth;
      j[u] = i < n ? F::idx(p, i) : 0;
      v[u] = i < n ? F::val(p, i) : T(0);
    }
#pragma unroll
    for (int u = 0; u < SCATTER_BATCH; ++u) {
      if (i0 + u * nth >= n) break;
      if ((unsigned)j[u] >= (unsigned long long)p.m) {
        raise_error(p.err, ERR_SCATTER_OOB);
        continue;
      }
      atomicAdd(&p.out[j[u]], v[u]);
    }
  }
}

// Privatised scatter_add in three tiers. The lowest LANE bins (128 bytes of
// them) are kept per thread in shared memory, bin b of thread t at
// b * 256 + t, so each lane owns a bank and a plain read-modify-write needs
// no atomic: a shared floating-point atomic retries for every lane that hit
// the same bin, and skewed distributions (Zipf puts 43% of its mass on the
// first 32 of 2^20 bins) collide inside a warp on most updates. Bins up to
// PRIV accumulate in a block-wide shared histogram with shared atomics; the
// rest go straight to global atomics. At the end each block sums its thread
// copies and flushes its non-zero private bins with one global atomic per
// bin. Each thread loads SCATTER_BATCH (index, value) pairs, a grid stride
// apart, before their updates. Persistent grid of 256-thread blocks; dynamic
// shared memory of (min(m, PRIV) + 256 * LANE) * sizeof(T) bytes.
template <class F, int PRIV>
__device__ __forceinline__ void scatter_add_priv(const typename F::P& p) {
  typedef typename F::T T;
  constexpr int LANE = 128 / (int)sizeof(T), NWARP = 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sh = reinterpret_cast<T*>(smem_raw);
  const long long n = p.n, m = p.m;
  const int priv = (int)(m < PRIV ? m : PRIV);
  const int lb = priv < LANE ? priv : LANE;
  T* lanes = sh + priv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = tid; b < priv; b += blockDim.x) sh[b] = T(0);
  for (int b = 0; b < LANE; ++b) lanes[b * 256 + tid] = T(0);
  __syncthreads();
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long i0 = (long long)blockIdx.x * blockDim.x + tid; i0 < n; i0 += nth * SCATTER_BATCH) {
    int j[SCATTER_BATCH];
    T v[SCATTER_BATCH];
#pragma unroll
    for (int u = 0; u < SCATTER_BATCH; ++u) {
      const long long i = i0 + u * nth;
      j[u] = i < n ? F::idx(p, i) : 0;
      v[u] = i < n ? F::val(p, i) : T(0);
    }
#pragma unroll
    for (int u = 0; u < SCATTER_BATCH; ++u) {
      if (i0 + u * nth >= n) break;
      if ((unsigned)j[u] >= (unsigned long long)m) {
        raise_error(p.err, ERR_SCATTER_OOB);
        continue;
      }
      if (j[u] < lb)
        lanes[j[u] * 256 + tid] += v[u];
      else if (j[u] < priv)
        atomicAdd(&sh[j[u]], v[u]);
      else
        atomicAdd(&p.out[j[u]], v[u]);
    }
  }
  __syncthreads();
  // bins [0, lb): warp w sums bins w, w + 8, ... over the 256 thread copies
  for (int b = warp; b < lb; b += NWARP) {
    T sum = T(0);
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += lanes[b * 256 + 32 * k + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_down_sync(FULL, sum, o);
    if (lane == 0) sh[b] = sum;
  }
  __syncthreads();
  for (int b = tid; b < priv; b += blockDim.x) {
    const T v = sh[b];
    if (v != T(0)) atomicAdd(&p.out[b], v);
  }
}

// ---------------------------------------------------------------- matmul (CUDA cores)
// C[M,N] = A[M,K] . B[K,N], row-major, each output accumulated in ascending k
// (the reference's contract, lib/ir/tensor.ml:35-40). 64x64 output tile per
// 256-thread block, 4x4 outputs per thread, K staged 16 at a time through
// shared memory. F provides T, a(p,row,k), b(p,k,col), store(p,row,col,v);
// P provides M, N, K.
template <class F>
__device__ __forceinline__ void matmul_tiled(const typename F::P& p) {
  typedef typename F::T T;
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ T As[BK][BM + 1];
  __shared__ T Bs[BK][BN + 1];
  const long long M = p.M, N = p.N, K = p.K;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const long long row0 = (long long)blockIdx.y * BM, col0 = (long long)blockIdx.x * BN;
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
  for (long long k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + e * 256;  // 0..1023
      const int ar = idx >> 4, ak = idx & 15;   // A tile: 64 rows x 16 k
      const long long gr = row0 + ar, gk = k0 + ak;
      As[ak][ar] = (gr < M && gk < K) ? F::a(p, gr, gk) : T(0);
      const int bk = idx >> 6, bc = idx & 63;   // B tile: 16 k x 64 cols
      const long long gk2 = k0 + bk, gc = col0 + bc;
      Bs[bk][bc] = (gk2 < K && gc < N) ? F::b(p, gk2, gc) : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      T a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const long long r = row0 + ty + 16 * i, c = col0 + tx + 16 * j;
      if (r < M && c < N) F::store(p, r, c, acc[i][j]);
    }
}

// C[M,N] = A[M,K] . B[K,N] for 4-byte T on the CUDA cores, each output still
// accumulated in ascending k: 128 x 128 output tile per 256-thread block,
// 8 x 8 outputs per thread (rows ty*4+i and 64+ty*4+i, columns tx*4+j and
// 64+tx*4+j, read as 16-byte fragments), K staged 8 at a time in two
// shared buffers (the next step's elements are loaded into registers while
// this one is multiplied). Tiles are loaded along the operand's contiguous
// dimension: F::A_MN when A is a transposed view (a(r,k) = At[k][r]),
// F::B_KM when B is one (b(k,c) = Bt[c][k]); rows of the shared tiles are
// padded to 132 elements so the transposing stores hit distinct banks.
template <class F>
__device__ __forceinline__ void matmul_tiled128(const typename F::P& p) {
  typedef typename F::T T;
  static_assert(sizeof(T) == 4, "4-byte elements");
  constexpr int BM = 128, BN = 128, BK = 8, LD = BM + 4;
  __shared__ __align__(16) T As[2][BK][LD];
  __shared__ __align__(16) T Bs[2][BK][LD];
  const long long M = p.M, N = p.N, K = p.K;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const long long row0 = (long long)blockIdx.y * BM, col0 = (long long)blockIdx.x * BN;
  T ra[4], rb[4];
  // element q of this thread's share of a k-step: (row or column, k)
  auto a_rc = [&](int q, int& r, int& k) {
    const int e = tid + 256 * q;
    if (F::A_MN) { r = e & 127; k = e >> 7; } else { r = e >> 3; k = e & 7; }
  };
  auto b_rc = [&](int q, int& c, int& k) {
    const int e = tid + 256 * q;
    if (F::B_KM) { c = e >> 3; k = e & 7; } else { c = e & 127; k = e >> 7; }
  };
  auto load = [&](long long k0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int r, k, c, kb;
      a_rc(q, r, k);
      ra[q] = (row0 + r < M && k0 + k < K) ? F::a(p, row0 + r, k0 + k) : T(0);
      b_rc(q, c, kb);
      rb[q] = (col0 + c < N && k0 + kb < K) ? F::b(p, k0 + kb, col0 + c) : T(0);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int r, k, c, kb;
      a_rc(q, r, k);
      As[buf][k][r] = ra[q];
      b_rc(q, c, kb);
      Bs[buf][kb][c] = rb[q];
    }
  };
  T acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = T(0);
  const int steps = (int)((K + BK - 1) / BK);
  load(0);
  stash(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int buf = s & 1;
    if (s + 1 < steps) load((long long)(s + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      T a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      memcpy(a, &a0, 16);
      memcpy(a + 4, &a1, 16);
      memcpy(b, &b0, 16);
      memcpy(b + 4, &b1, 16);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += a[i] * b[j];
    }
    if (s + 1 < steps) stash(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long r = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long c = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (r < M && c < N) F::store(p, r, c, acc[i][j]);
    }
  }
}

// ------------------------------------------------------------------------
// F32 matmul on the tcgen05 tensor cores (kind::tf32), persistent.
//
// One CTA per SM owns 128x256 output tiles in turn. Warp 0 (one thread) is
// the TMA producer: per 32-wide k-step it loads the A tile (128 x 32) and
// the B tile (256 x 32) into a 4-deep ring of 48 KiB stages, 128-byte
// swizzled. Warp 1 (one thread) issues tcgen05.mma (M=128, N=256, K=8, four
// per stage) into one of two TMEM accumulators of 256 fp32 columns, and
// releases each stage with tcgen05.commit. Warps 2-5 drain the finished
// accumulator (tcgen05.ld, 32 columns at a time, one TMEM lane quadrant per
// warp) into global memory while the next tile accumulates in the other
// buffer. Loads are plain TMA (no cluster multicast).
//
// Operands arrive as views of materialised row-major buffers: A is K-major
// (A[r][k] at r*K+k) or MN-major (at k*M+r); B is MN-major (B[k][c] at
// k*N+c) or K-major (at c*K+k). K-major tiles are loaded with the 128-byte
// swizzle, MN-major tiles with the 128-byte swizzle of 32-byte atoms. Out-of-range tile rows and k-steps read as
// zero (TMA fill), so any M, N, K >= 1 is exact in shape; stores are masked.
//
// Numerics: TF32 operands (10 explicit mantissa bits), FP32 accumulation.
// Bound used by the tests: |C - C_exact| <= (2^-9 + K*2^-23) * sum_k |A||B|.
//
// F provides P (first fields: TmaDesc ta, tb; then C, err, M, N, K) and the
// constants A_MN, B_MN.
struct alignas(64) TmaDesc {
  unsigned long long w[16];
};

namespace tc {
constexpr int BM = 128, BN = 256, BK = 32, STAGES = 4, THREADS = 192;
constexpr unsigned A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr unsigned SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr unsigned TMEM_COLS = 2 * BN;
constexpr int GROUP_M = 16;  // tile raster: 16 M-tiles per band for L2 reuse
constexpr unsigned ERR_TC_WAIT = 16u;

__device__ __forceinline__ void wait(u64* bar, unsigned parity, unsigned* err) {
  for (unsigned it = 0; it < MBAR_SPIN_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return;
  raise_error(err, ERR_TC_WAIT);
  for (unsigned it = 0; it < MBAR_SPIN_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return;
}
__device__ __forceinline__ void arrive(u64* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(unsigned dst, const TmaDesc* map, int x, int y, u64* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(unsigned dst, const TmaDesc* map, int x, int y, int z, u64* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, version 1 (sm_100). Layout 2 is the
// 128-byte swizzle with 16-byte atoms (K-major operands); layout 1 the
// 128-byte swizzle with 32-byte atoms, the only one UMMA accepts for
// MN-major 32-bit operands.
constexpr unsigned LAYOUT_SW128 = 2u, LAYOUT_SW128_BASE32B = 1u;
__device__ __forceinline__ u64 sdesc(unsigned saddr, unsigned lbo, unsigned sbo, unsigned layout) {
  return (u64)((saddr >> 4) & 0x3FFFu) | ((u64)((lbo >> 4) & 0x3FFFu) << 16) | ((u64)((sbo >> 4) & 0x3FFFu) << 32) |
         (1ull << 46) | ((u64)layout << 61);
}
// K-major tile: 128-byte rows, 8-row groups 1024 bytes apart; k-step kk
// (8 tf32 = 32 bytes) starts kk*32 bytes into the swizzle atom.
__device__ __forceinline__ u64 desc_k(unsigned tile, int kk) { return sdesc(tile + kk * 32u, 16u, 1024u, LAYOUT_SW128); }
// MN-major tile: 32-element (128-byte) rows along MN, one row per k; 4-row
// atoms 512 bytes apart (SBO) and 32-element MN blocks 4096 bytes apart (LBO);
// k-step kk covers rows 8kk..8kk+7.
__device__ __forceinline__ u64 desc_mn(unsigned tile, int kk, unsigned lbo = 4096u) {
  return sdesc(tile + kk * 1024u, lbo, 512u, LAYOUT_SW128_BASE32B);
}
__device__ __forceinline__ void mma(unsigned d, u64 a, u64 b, unsigned idesc, unsigned accumulate) {
  const unsigned z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
__device__ __forceinline__ void commit(u64* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void ld32(unsigned taddr, float* v) {
  unsigned r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 32 accumulator columns of one row (cnt of them valid) at flat index
// i0 of the product, or hand them to the fused map pass (F::EPI).
template <class F>
__device__ __forceinline__ void store32(const typename F::P& p, long long i0, const float* v, int cnt, bool vec) {
  if constexpr (F::EPI) {
    F::epi32(p, i0, v, cnt, vec);
  } else {
    float* dst = p.C + i0;
    if (vec && cnt == 32) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) *(float4*)(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < cnt) dst[i] = v[i];
    }
  }
}

__device__ __forceinline__ void tile_of(long long t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const long long band = (long long)GROUP_M * tiles_n;
  const int first = (int)(t / band) * GROUP_M;
  const int rows = min(tiles_m - first, GROUP_M);
  const int r = (int)(t % band);
  tm = first + r % rows;
  tn = r / rows;
}
}  // namespace tc

template <class F>
__device__ __forceinline__ void matmul_tc(const typename F::P& p) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char ccb_tc_smem[];
  const unsigned raw = smem_u32(ccb_tc_smem);
  const unsigned pad = (1024u - (raw & 1023u)) & 1023u;
  unsigned char* base = ccb_tc_smem + pad;
  const unsigned sbase = raw + pad;
  u64* full = (u64*)(base + STAGES * STAGE_BYTES);
  u64* empty = full + STAGES;
  u64* accf = empty + STAGES;
  u64* acce = accf + 2;
  unsigned* tslot = (unsigned*)(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long M = p.M, N = p.N, K = p.K;
  const int tiles_m = (int)((M + BM - 1) / BM), tiles_n = (int)((N + BN - 1) / BN);
  const long long ntiles = (long long)tiles_m * tiles_n;
  const int KT = (int)((K + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const unsigned tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      unsigned stage = 0, phase = 0;
      for (long long t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int tm, tn;
        tile_of(t, tiles_m, tiles_n, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int ks = 0; ks < KT; ++ks) {
          wait(&empty[stage], phase ^ 1u, p.err);
          const unsigned sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES;
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          const int k0 = ks * BK;
          if (F::A_MN) {
            if constexpr (F::A3) {
              tma_load_3d(sa, &p.ta, 0, k0, m0 / 32, &full[stage]);
            } else {
#pragma unroll
              for (int g = 0; g < BM / 32; ++g) tma_load_2d(sa + g * 4096u, &p.ta, m0 + 32 * g, k0, &full[stage]);
            }
          } else {
            tma_load_2d(sa, &p.ta, k0, m0, &full[stage]);
          }
          if (F::B_MN) {
            if constexpr (F::B3) {
              tma_load_3d(sb, &p.tb, 0, k0, n0 / 32, &full[stage]);
            } else {
#pragma unroll
              for (int g = 0; g < BN / 32; ++g) tma_load_2d(sb + g * 4096u, &p.tb, n0 + 32 * g, k0, &full[stage]);
            }
          } else {
            tma_load_2d(sb, &p.tb, k0, n0, &full[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const unsigned idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((F::A_MN ? 1u : 0u) << 15) | ((F::B_MN ? 1u : 0u) << 16) |
                             ((unsigned)(BN >> 3) << 17) | ((unsigned)(BM >> 4) << 24);
      unsigned stage = 0, phase = 0;
      int it = 0;
      for (long long t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const unsigned ab = it & 1, aph = (it >> 1) & 1;
        wait(&acce[ab], aph ^ 1u, p.err);
        fence_after();
        const unsigned d = tmem + ab * BN;
        for (int ks = 0; ks < KT; ++ks) {
          wait(&full[stage], phase, p.err);
          fence_after();
          const unsigned sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const u64 a = F::A_MN ? desc_mn(sa, kk) : desc_k(sa, kk);
            const u64 b = F::B_MN ? desc_mn(sb, kk) : desc_k(sb, kk);
            mma(d, a, b, idesc, (ks | kk) != 0 ? 1u : 0u);
          }
          commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        commit(&accf[ab]);
      }
    }
  } else {  // epilogue: warps 2..5, TMEM lane quadrant warp % 4
    const int q = warp & 3;
    const bool vec = (N % 4 == 0) && F::vec_ok(p);
    int it = 0;
    for (long long t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      int tm, tn;
      tile_of(t, tiles_m, tiles_n, tm, tn);
      const long long row = (long long)tm * BM + q * 32 + lane;
      const long long n0 = (long long)tn * BN;
      const unsigned ab = it & 1, aph = (it >> 1) & 1;
      wait(&accf[ab], aph, p.err);
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the polls
      fence_after();
      for (int c = 0; c < BN && n0 + c < N; c += 32) {
        float v[32];
        __syncwarp();
        ld32(tmem + ((unsigned)(q * 32) << 16) + ab * BN + c, v);
        if (row < M) store32<F>(p, row * N + n0 + c, v, N - n0 - c < 32 ? (int)(N - n0 - c) : 32, vec);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) arrive(&acce[ab]);
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  __syncwarp();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------------
// F32 matmul on the tcgen05 tensor cores, 2-SM pairs (cta_group::2).
//
// A cluster of two CTAs on two SMs owns 256 x 256 output tiles in turn.
// Each CTA stages its own 128 rows of A and 128 columns of B per 32-wide
// k-step (32 KiB, a 6-deep ring); one thread of the even CTA (the leader)
// issues tcgen05.mma.cta_group::2 (M=256, N=256, K=8), which reads both
// CTAs' shared memory and accumulates each CTA's 128 rows x 256 columns in
// its own TMEM (two 256-column buffers, as in matmul_tc). Per SM this moves
// two thirds of the operand bytes of a 128 x 256 single-SM tile for the same
// flops. Both CTAs' TMA copies (plain loads, no cluster multicast) complete
// on the leader's stage barrier; the leader's commits release the stage in
// both CTAs (a commit to each CTA's barrier, addressed through mapa); both
// CTAs' epilogue warps release an accumulator to the leader.
// Same operand views, bounds handling and numerics as matmul_tc.
namespace tc2 {
constexpr int BM = 256, BN = 256, HALF = 128, THREADS = 192;
constexpr unsigned RING_BYTES = 6u * 32768u;  // the stage ring: 6 x 32 KiB or 3 x 64 KiB
constexpr unsigned TMEM_COLS = 2 * BN;

__device__ __forceinline__ unsigned cta_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of `local` in CTA `rank` of this cluster.
__device__ __forceinline__ unsigned peer_addr(const void* local, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void tma_load_2d(unsigned dst, const TmaDesc* map, int x, int y, unsigned bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(unsigned dst, const TmaDesc* map, int x, int y, int z, unsigned bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void mma(unsigned d, u64 a, u64 b, unsigned idesc, unsigned accumulate) {
  const unsigned z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z));
}
// Arrive on barrier `bar` of both CTAs once the MMAs issued so far complete.
__device__ __forceinline__ void commit_both(u64* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer_addr(bar, 0)) : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer_addr(bar, 1)) : "memory");
}
__device__ __forceinline__ void arrive_leader(u64* bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(peer_addr(bar, 0)) : "memory");
}
}  // namespace tc2

template <class F>
__device__ __forceinline__ void matmul_tc2(const typename F::P& p) {
  using namespace tc2;
  // k-step of BK (32 or 64): a stage holds this CTA's 128 rows of A and 128
  // columns of B over BK; K-major operands come as BK/32 boxes 32 wide (the
  // 128-byte swizzle span), MN-major ones as one 3-D copy (or 2-D boxes) of
  // 32-element MN blocks BK rows deep.
  constexpr int BK = F::BK;
  constexpr unsigned A_BYTES = HALF * BK * 4, B_BYTES = HALF * BK * 4, STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int STAGES = (int)(RING_BYTES / STAGE_BYTES);
  constexpr unsigned KCHUNK = HALF * 32 * 4;  // one 32-wide K-major box: 16 KiB
  constexpr unsigned MNBLK = 32 * BK * 4;     // one 32-element MN block: 4 or 8 KiB
  extern __shared__ __align__(1024) unsigned char ccb_tc_smem[];
  const unsigned raw = smem_u32(ccb_tc_smem);
  const unsigned pad = (1024u - (raw & 1023u)) & 1023u;
  unsigned char* base = ccb_tc_smem + pad;
  const unsigned sbase = raw + pad;
  u64* full = (u64*)(base + STAGES * STAGE_BYTES);
  u64* empty = full + STAGES;
  u64* accf = empty + STAGES;
  u64* acce = accf + 2;
  unsigned* tslot = (unsigned*)(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned rank = cta_rank();
  const bool leader = rank == 0;
  const long long M = p.M, N = p.N, K = p.K;
  const int tiles_m = (int)((M + BM - 1) / BM), tiles_n = (int)((N + BN - 1) / BN);
  const long long ntiles = (long long)tiles_m * tiles_n;
  const int KT = (int)((K + BK - 1) / BK);
  const long long pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (+ both CTAs' bytes)
      mbar_init(&empty[s], 1);  // the leader's commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);  // the leader's commit
      mbar_init(&acce[b], 8);  // four epilogue warps of each CTA (used in the leader)
    }
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc::fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc::fence_after();
  const unsigned tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer (both CTAs)
      unsigned stage = 0, phase = 0;
      for (long long t = pair; t < ntiles; t += npairs) {
        int tm, tn;
        tc::tile_of(t, tiles_m, tiles_n, tm, tn);
        const int m0 = tm * BM + (int)rank * HALF, n0 = tn * BN + (int)rank * HALF;
        for (int ks = 0; ks < KT; ++ks) {
          tc::wait(&empty[stage], phase ^ 1u, p.err);
          const unsigned sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES;
          const unsigned fb = peer_addr(&full[stage], 0);
          if (leader) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&full[stage])),
                         "r"(2u * STAGE_BYTES)
                         : "memory");
          }
          const int k0 = ks * BK;
          if constexpr (F::A_MN) {
            if constexpr (F::A3) {
              tma_load_3d(sa, &p.ta, 0, k0, m0 / 32, fb);
            } else {
#pragma unroll
              for (int g = 0; g < HALF / 32; ++g) tma_load_2d(sa + g * MNBLK, &p.ta, m0 + 32 * g, k0, fb);
            }
          } else {
#pragma unroll
            for (int c = 0; c < BK / 32; ++c) tma_load_2d(sa + c * KCHUNK, &p.ta, k0 + 32 * c, m0, fb);
          }
          if constexpr (F::B_MN) {
            if constexpr (F::B3) {
              tma_load_3d(sb, &p.tb, 0, k0, n0 / 32, fb);
            } else {
#pragma unroll
              for (int g = 0; g < HALF / 32; ++g) tma_load_2d(sb + g * MNBLK, &p.tb, n0 + 32 * g, k0, fb);
            }
          } else {
#pragma unroll
            for (int c = 0; c < BK / 32; ++c) tma_load_2d(sb + c * KCHUNK, &p.tb, k0 + 32 * c, n0, fb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issuer: one thread of the pair
      const unsigned idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((F::A_MN ? 1u : 0u) << 15) | ((F::B_MN ? 1u : 0u) << 16) |
                             ((unsigned)(BN >> 3) << 17) | ((unsigned)(BM >> 4) << 24);
      unsigned stage = 0, phase = 0;
      int it = 0;
      for (long long t = pair; t < ntiles; t += npairs, ++it) {
        const unsigned ab = it & 1, aph = (it >> 1) & 1;
        tc::wait(&acce[ab], aph ^ 1u, p.err);
        tc::fence_after();
        const unsigned d = tmem + ab * BN;
        for (int ks = 0; ks < KT; ++ks) {
          tc::wait(&full[stage], phase, p.err);
          tc::fence_after();
          const unsigned sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const u64 a = F::A_MN ? tc::desc_mn(sa, kk, MNBLK) : tc::desc_k(sa + (kk >> 2) * KCHUNK, kk & 3);
            const u64 b = F::B_MN ? tc::desc_mn(sb, kk, MNBLK) : tc::desc_k(sb + (kk >> 2) * KCHUNK, kk & 3);
            mma(d, a, b, idesc, (ks | kk) != 0 ? 1u : 0u);
          }
          commit_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        commit_both(&accf[ab]);
      }
    }
  } else {  // epilogue: warps 2..5 of each CTA, TMEM lane quadrant warp % 4
    const int q = warp & 3;
    const bool vec = (N % 4 == 0) && F::vec_ok(p);
    int it = 0;
    for (long long t = pair; t < ntiles; t += npairs, ++it) {
      int tm, tn;
      tc::tile_of(t, tiles_m, tiles_n, tm, tn);
      const long long row = (long long)tm * BM + (long long)rank * HALF + q * 32 + lane;
      const long long n0 = (long long)tn * BN;
      const unsigned ab = it & 1, aph = (it >> 1) & 1;
      tc::wait(&accf[ab], aph, p.err);
      __syncwarp();
      tc::fence_after();
      for (int c = 0; c < BN && n0 + c < N; c += 32) {
        float v[32];
        __syncwarp();
        tc::ld32(tmem + ((unsigned)(q * 32) << 16) + ab * BN + c, v);
        if (row < M) tc::store32<F>(p, row * N + n0 + c, v, N - n0 - c < 32 ? (int)(N - n0 - c) : 32, vec);
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&acce[ab]);
    }
  }
  tc::fence_before();
  __syncthreads();
  cluster_sync();  // the pair is done with both TMEM allocations
  tc::fence_after();
  __syncwarp();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

}  // namespace ccb
