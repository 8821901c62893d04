/* ccb.h -- the C-ABI of libccb.so, the B200-native execution backend for
 * CUDACaml graphs.
 *
 * Every entry point takes plain pointers, sizes and opaque handles, returns an
 * int status (CCB_OK = 0) and, on failure, leaves a message readable through
 * ccb_last_error() on the calling thread. The reference's OCaml runtime binds
 * the CUDA driver and NVRTC through the third-party `cudajit` package; each
 * group below names the reference interface (file:line in sinj3d/CUDACaml)
 * that its functions replace, so an OCaml `ctypes` binding can swap one for
 * the other. libccb.so opens libcuda.so.1, libnvrtc and libnccl lazily, so it
 * loads on a machine without a GPU; only the calls that need a device fail.
 */
#ifndef CCB_H
#define CCB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
enum {
  CCB_OK = 0,
  CCB_ERR_INVALID = 1,     /* caller mistake: Invalid_argument on the OCaml side */
  CCB_ERR_NO_DEVICE = 2,   /* no driver, no device, or an ordinal out of range   */
  CCB_ERR_DRIVER = 3,      /* a CUDA driver call failed                           */
  CCB_ERR_COMPILE = 4,     /* NVRTC rejected the generated source                 */
  CCB_ERR_NCCL = 5,        /* an NCCL call failed                                  */
  CCB_ERR_DEVICE_CHECK = 6,/* a kernel raised its error word (index out of bounds,
                              a bounded wait ran out); the message says which     */
  CCB_ERR_UNSUPPORTED = 7  /* a graph feature this backend does not lower         */
};

/* Message of the last failing call on this thread ("" if none).
 * Replaces the exception text cudajit raises (lib/runtime/jit.ml:16-23). */
const char* ccb_last_error(void);
/* Library version string, e.g. "ccb 0.1 sm_100a". */
const char* ccb_version(void);

/* ---------------------------------------------------------------- devices
 * Replaces lib/runtime/device.mli (available/init/count/with_device/info). */
typedef struct {
  char name[256];
  int cc_major, cc_minor;     /* compute capability, (10, 0) on B200 */
  int multiprocessors;
  long long total_memory_bytes;
} ccb_device_info_t;

int ccb_available(void);                     /* 1 if a driver and >= 1 device; never fails  */
int ccb_init(void);                          /* cuInit + primary context of device 0         */
int ccb_device_count(int* count);
int ccb_set_device(int ordinal);             /* primary context current on this thread       */
int ccb_get_device(int* ordinal);
int ccb_device_info(int ordinal, ccb_device_info_t* info);
int ccb_device_synchronize(void);

/* ---------------------------------------------------------------- memory
 * Replaces lib/runtime/buffer.mli (alloc/free/upload/download/copy_device,
 * live_count) and lib/runtime/pinned.mli (page-locked host memory). All act
 * on the current device. A 0-byte request still returns a valid pointer
 * (lib/runtime/buffer.ml:16-18). */
typedef void* ccb_stream_t;   /* NULL = the legacy default stream */
typedef void* ccb_event_t;

int ccb_malloc(size_t bytes, void** dptr);
int ccb_free(void* dptr);
int ccb_live_count(long long* count);        /* allocations minus frees */
int ccb_memcpy_h2d(void* dst, const void* src, size_t bytes, ccb_stream_t s);   /* async on s */
int ccb_memcpy_d2h(void* dst, const void* src, size_t bytes, ccb_stream_t s);   /* async on s */
int ccb_memcpy_d2d(void* dst, const void* src, size_t bytes, ccb_stream_t s);   /* async on s */
int ccb_memset_d8(void* dst, unsigned char v, size_t bytes, ccb_stream_t s);
int ccb_host_alloc(size_t bytes, void** hptr);   /* pinned, portable, zero-filled */
int ccb_host_free(void* hptr);

/* ---------------------------------------------------------------- streams/events
 * Replaces lib/runtime/stream.mli and lib/runtime/event.mli. */
int ccb_stream_create(ccb_stream_t* s);      /* non-blocking (lib/runtime/stream.ml:13-15) */
int ccb_stream_destroy(ccb_stream_t s);
int ccb_stream_synchronize(ccb_stream_t s);
int ccb_stream_query(ccb_stream_t s, int* idle);
int ccb_event_create(ccb_event_t* e);
int ccb_event_destroy(ccb_event_t e);
int ccb_event_record(ccb_event_t e, ccb_stream_t s);
int ccb_event_synchronize(ccb_event_t e);
int ccb_event_elapsed_ms(ccb_event_t start, ccb_event_t end, float* ms);
int ccb_stream_wait_event(ccb_stream_t s, ccb_event_t e);

/* ---------------------------------------------------------------- modules
 * Replaces lib/runtime/jit.mli and lib/runtime/launch.mli: NVRTC for sm_100a
 * with the skeleton header on the include path, cuModuleLoadData, and a
 * launch that takes a by-value argument block (Launch.run's `args` list,
 * lib/runtime/launch.ml:9-13): `args[i]` points at the value of parameter i
 * and `nargs` is the list's length, checked against the kernel's own
 * parameter count (CCB_ERR_INVALID when they differ, before any launch). */
typedef void* ccb_module_t;
typedef void* ccb_function_t;
int ccb_module_compile(const char* source, const char* name, ccb_module_t* mod, char** log);
int ccb_module_unload(ccb_module_t mod);
int ccb_module_get_function(ccb_module_t mod, const char* name, ccb_function_t* fn);
int ccb_launch(ccb_function_t fn, unsigned gx, unsigned gy, unsigned gz, unsigned bx, unsigned by,
               unsigned bz, unsigned smem, ccb_stream_t s, void** args, int nargs);
/* Compile source to an sm_100a CUBIN without loading it (works without a GPU). */
int ccb_nvrtc_check(const char* source, const char* name, size_t* cubin_bytes, char** log);
void ccb_free_string(char* s);

/* ---------------------------------------------------------------- programs
 * One compiled graph: the replacement of lib/lower (Fusion.plan, Lower.program),
 * lib/backend_cuda/emit.ml (Emit.program), lib/runtime/jit.ml (Jit.compile) and
 * lib/backend_cuda/executor.ml (Executor.create_on/run_async/run/run_resident).
 *
 * `graph` is the text wire format (cudacaml_b200/wire.py documents it).
 * A program is compiled for one device and owns `lanes` executors, each with
 * its own non-blocking stream and buffer pool (compile_with ~streams,
 * lib/backend_cuda/cudacaml_backend_cuda.mli:28). */
typedef void* ccb_program_t;

int ccb_program_create(const char* graph, int device, int lanes, ccb_program_t* prog);
/* Lower and emit only: no device needed. `source` is owned by the program. */
int ccb_program_lower(const char* graph, ccb_program_t* prog);
int ccb_program_destroy(ccb_program_t prog);                      /* Backend_cuda.release */
int ccb_program_source(ccb_program_t prog, const char** source);  /* Backend_cuda.source  */
int ccb_program_device(ccb_program_t prog, int* device);          /* Backend_cuda.device_of */
/* Structure, for tests: kernels emitted, launches per run, plan text. */
int ccb_program_num_kernels(ccb_program_t prog, int* n);
int ccb_program_num_launches(ccb_program_t prog, int* n);
int ccb_program_plan(ccb_program_t prog, const char** text);

/* Params and outputs in graph order. dtype codes: 0 f32, 1 f64, 2 i32, 3 i64. */
int ccb_program_num_params(ccb_program_t prog, int* n);
int ccb_program_param(ccb_program_t prog, int i, const char** name, int* dtype, int* rank,
                      const long long** dims);
int ccb_program_num_outputs(ccb_program_t prog, int* n);
int ccb_program_output(ccb_program_t prog, int i, const char** name, int* dtype, int* rank,
                       const long long** dims);

/* Host in, host out. `inputs[i]` is the host storage of param i (graph param
 * order), `outputs[j]` receives output j. enqueue issues the uploads, the
 * launches and the downloads on lane `lane`'s stream and returns at once
 * (Executor.run_async, lib/backend_cuda/executor.ml:109-165); the host
 * buffers must stay alive until ccb_program_wait(lane) returns. wait blocks,
 * then checks the lane's device error word. run = enqueue + wait on lane 0. */
int ccb_program_enqueue(ccb_program_t prog, int lane, const void* const* inputs, void* const* outputs);
int ccb_program_wait(ccb_program_t prog, int lane);
int ccb_program_run(ccb_program_t prog, const void* const* inputs, void* const* outputs);

/* Device in, device out, zero-copy (Executor.run_resident,
 * lib/backend_cuda/executor.ml:181-244): kernels read `inputs[i]` and write
 * `outputs[j]` (caller-owned device pointers of the exact byte size) directly.
 * Issued on `stream` (NULL: the lane's own stream); it does not synchronise.
 * ccb_program_check then synchronises that stream and reads the error word
 * (runs with host buffers copy it as their last step; device runs do not).
 * A lane's error word accumulates over runs until a wait or check reports it
 * (and clears it), so a chain of device runs checked once reports an error
 * raised anywhere in the chain. */
int ccb_program_run_device(ccb_program_t prog, int lane, const void* const* inputs,
                           void* const* outputs, ccb_stream_t stream);
/* As ccb_program_run_device, and for each output j whose output_events[j] is
 * not NULL, records that event on `stream` as soon as output j is final (after
 * the last kernel that touches its buffer), so another stream can start on it
 * (an all-reduce of one gradient while the next one is computed). No
 * counterpart in the reference. */
int ccb_program_run_device_events(ccb_program_t prog, int lane, const void* const* inputs,
                                  void* const* outputs, ccb_stream_t stream,
                                  ccb_event_t const* output_events);
int ccb_program_check(ccb_program_t prog, int lane, ccb_stream_t stream);
/* Kernel launches per run (for the bench's gpu_launches count). */
int ccb_program_lane_stream(ccb_program_t prog, int lane, ccb_stream_t* stream);

/* ---------------------------------------------------------------- sharded programs
 * Replaces the recombination half of Multi (lib/backend_cuda/multi.ml:95-109,
 * mean_scalar of per-device results on the host) for Monte-Carlo estimators.
 * A graph lowered with the wire option `opt shard <rank> <world>` (one process
 * or one device per rank, each rank on its own GPU of one box) is the unsplit
 * graph: its one reduction pass walks only this rank's slice
 * [n*rank/world, n*(rank+1)/world) of the index space -- Philox counters are
 * the global element index, so the slices draw exactly the unsplit program's
 * numbers -- and its last block sums the block totals of every rank in rank
 * order over NVLink peer memory before the scalar tails run. Every rank's
 * outputs are then the unsplit program's (up to summation order), the same
 * bits on every rank, with no collective after the kernel. Programs with
 * element loads or stores, scans, products or more than one reduction pass
 * are refused (CCB_ERR_UNSUPPORTED).
 *
 * ccb_program_mailbox_bytes: bytes of one rank's mailbox (0 if not sharded).
 * ccb_program_bind_peers: mailboxes[q] is rank q's mailbox as this rank
 * addresses it (its own allocation, an IPC mapping from ccb_ipc_mem_open, or
 * a peer allocation after ccb_peer_access_enable), 8-byte aligned; every
 * owner zero-fills its mailbox before any rank's first run after binding,
 * and every rank runs the program the same number of times in the same
 * order, one run at a time. The ranks wait on each other inside the kernel,
 * so a thread that drives several ranks issues every rank's run before it
 * waits on any (a run whose outputs are pageable host memory blocks the
 * issuing thread until its download is done). A run before binding is
 * CCB_ERR_INVALID; a run under stream capture is refused. A peer that never runs makes the bounded
 * wait give up: ccb_program_check / wait report CCB_ERR_DEVICE_CHECK and the
 * scalar outputs keep their previous contents. No counterpart in the
 * reference. */
int ccb_program_shard(ccb_program_t prog, int* rank, int* world);
int ccb_program_mailbox_bytes(ccb_program_t prog, size_t* bytes);
int ccb_program_bind_peers(ccb_program_t prog, void* const* mailboxes, int nranks);

/* ---------------------------------------------------------------- CUDA graphs
 * No counterpart in the reference (its executor launches every kernel from
 * the host). Work issued on `s` between ccb_graph_begin and ccb_graph_end
 * (program runs with ccb_program_run_device, copies, memsets, events) is
 * captured instead of run and instantiated once; ccb_graph_launch replays it
 * with one launch. Pointers and sizes are fixed at capture; device-resident
 * runs copy no error word, so ccb_program_check after a replay reports errors
 * raised in it. A run of a program with a flat scan is refused while
 * capturing (its look-back tags status words with a per-run epoch, which a
 * replay would repeat). Nothing that synchronises may be issued meanwhile. */
typedef void* ccb_graph_t;
int ccb_graph_begin(ccb_stream_t s);
int ccb_graph_end(ccb_stream_t s, ccb_graph_t* graph);
int ccb_graph_launch(ccb_graph_t graph, ccb_stream_t s);
int ccb_graph_destroy(ccb_graph_t graph);

/* ---------------------------------------------------------------- no-allocation sum
 * No counterpart in the reference. For callers that cannot allocate device
 * memory (inside someone else's stream capture, under an application-owned
 * memory pool, in a real-time path that must not take the driver's
 * allocation locks, or in a plugin handed device pointers but no allocator):
 * the flat F32 sum that a `reduce add` graph lowers to, with its reduction
 * scratch in one file-scope __device__ array instead of an allocation.
 * out[0] = sum of x[0..n). Allocates nothing; issued on `stream` (a
 * cudaStream_t, NULL = legacy default) on the current device, not
 * synchronised. n must be in [0, 2^31 - 1]. The scratch (4096 block partials
 * plus a ticket, about 16 KiB) is held by every GPU that loads the library
 * until exit and is shared by all calls on a device: calls that overlap on
 * the GPU race and give wrong sums. The first call on a device does that
 * device's set-up (it finds the array's device address once and keeps it);
 * make it before any stream capture, and do not call the entry point on a
 * device whose primary context was reset since then (cudaDeviceReset): the
 * kept address is stale. Errors: CCB_ERR_INVALID, CCB_ERR_NO_DEVICE,
 * CCB_ERR_DRIVER, with the message in ccb_last_error(). */
int ccb_sum_f32_noalloc(const float* x, long long n, float* out, void* stream);

/* ---------------------------------------------------------------- peer memory and the cross-rank sum
 * New: the reference has no collective (lib/backend_cuda/multi.ml:51-109
 * combines per-device results on the host). A rank exports a device
 * allocation of its own with ccb_ipc_mem_handle (64 opaque bytes, cuIpc),
 * another process of the same box maps it with ccb_ipc_mem_open (peer access
 * over NVLink enabled lazily) and unmaps it with ccb_ipc_mem_close. In one
 * process, ccb_peer_access_enable(peer) lets the current device read and
 * write `peer`'s allocations directly. */
int ccb_ipc_mem_handle(void* dptr, unsigned char handle[64]);
int ccb_ipc_mem_open(const unsigned char handle[64], void** dptr);
int ccb_ipc_mem_close(void* dptr);
int ccb_peer_access_enable(int peer);
/* out[k] = sum over ranks r = 0..nranks-1, in rank order, of rank r's in[k],
 * k < count <= 8, dtype codes as above, for ranks on distinct GPUs of one box:
 * one 32-thread kernel per rank on `stream` writes this rank's values into
 * every rank's mailbox over peer memory and sums what the local mailbox
 * receives (so every rank gets the same bits). mailboxes[q] is rank q's
 * mailbox as this rank addresses it (ccb_xrank_mailbox_bytes(nranks) bytes,
 * zero-filled by its owner before any rank's first call), nranks <= 16.
 * `epoch` is the same on every rank for one sum and increases from 1 with
 * every call. A peer that never publishes makes the bounded wait give up:
 * bit 32 is raised in the device word *err and `out` is left untouched. Two
 * ranks must never share one GPU (their kernels wait on each other). No
 * counterpart in the reference. */
int ccb_xrank_mailbox_bytes(int nranks, size_t* bytes);
int ccb_xrank_sum(const void* in, void* out, int count, int dtype, int nranks, int rank, void* const* mailboxes,
                  unsigned long long epoch, unsigned* err, void* stream);

/* ---------------------------------------------------------------- NCCL
 * New: the reference has no collective (lib/backend_cuda/multi.ml:51-109
 * combines on the host). Multi recombines per-device partial results with an
 * all-reduce over NVLink. dtype codes as above; op 0 = sum, 1 = max, 2 = min. */
typedef void* ccb_comm_t;
int ccb_comm_init_all(int ndev, const int* devices, ccb_comm_t* comms);  /* one process, ndev comms */
int ccb_comm_unique_id(unsigned char id[128]);
int ccb_comm_init_rank(int nranks, const unsigned char id[128], int rank, ccb_comm_t* comm);
int ccb_comm_destroy(ccb_comm_t comm);
int ccb_allreduce(ccb_comm_t comm, const void* send, void* recv, size_t count, int dtype, int op,
                  ccb_stream_t s);
int ccb_group_start(void);
int ccb_group_end(void);

#ifdef __cplusplus
}
#endif
#endif /* CCB_H */
