(* Ccb: ctypes bindings for every entry point of include/ccb.h (libccb.so).

   NOT BUILT HERE: the build image has no OCaml toolchain. This is the module
   a maintainer adds as lib/runtime/ccb.ml. It binds libccb.so the way the
   reference already binds the CUDA driver for page-locked memory
   (lib/runtime/pinned.ml:14-24: Dl.dlopen + Foreign.foreign, opened lazily
   so the module loads on a machine without the library), and it replaces
   every cudajit call of lib/runtime and lib/backend_cuda.

   Error convention: every function returns an int status (0 = ok) and
   leaves a message in ccb_last_error on the calling thread. [check] turns
   caller mistakes (status 1) into Invalid_argument and everything else
   into Failure, which is what the reference raises today
   (lib/runtime/jit.ml:16-23, lib/backend_cuda/executor.mli:28-31). *)

open Ctypes

let lib = lazy (Dl.dlopen ~filename:"libccb.so" ~flags:[ Dl.RTLD_NOW; Dl.RTLD_GLOBAL ])
let fn name t = lazy (Foreign.foreign ~from:(Lazy.force lib) name t)
let ( !! ) = Lazy.force

(* Status codes (include/ccb.h) *)
let ok = 0
let err_invalid = 1
let err_no_device = 2
let err_driver = 3
let err_compile = 4
let err_nccl = 5
let err_device_check = 6
let err_unsupported = 7

(* Opaque handles: streams, events, modules, functions, programs, graphs and
   communicators are all void* on the C side. *)
type handle = unit ptr

let handle : handle typ = ptr void

(* ---------------------------------------------------------------- status *)
let last_error_ = fn "ccb_last_error" (void @-> returning string)
let version_ = fn "ccb_version" (void @-> returning string)
let last_error () = !!last_error_ ()
let version () = !!version_ ()

let check what rc =
  if rc = ok then ()
  else if rc = err_invalid then invalid_arg (what ^ ": " ^ last_error ())
  else failwith (what ^ ": " ^ last_error ())

(* ---------------------------------------------------------------- devices
   Replaces lib/runtime/device.mli. *)
type device_info

let device_info : device_info structure typ = structure "ccb_device_info_t"
let di_name = field device_info "name" (array 256 char)
let di_cc_major = field device_info "cc_major" int
let di_cc_minor = field device_info "cc_minor" int
let di_multiprocessors = field device_info "multiprocessors" int
let di_total_memory_bytes = field device_info "total_memory_bytes" llong
let () = seal device_info

let available = fn "ccb_available" (void @-> returning int)
let init = fn "ccb_init" (void @-> returning int)
let device_count = fn "ccb_device_count" (ptr int @-> returning int)
let set_device = fn "ccb_set_device" (int @-> returning int)
let get_device = fn "ccb_get_device" (ptr int @-> returning int)
let device_info_ = fn "ccb_device_info" (int @-> ptr device_info @-> returning int)
let device_synchronize = fn "ccb_device_synchronize" (void @-> returning int)

(* ---------------------------------------------------------------- memory
   Replaces lib/runtime/buffer.mli and lib/runtime/pinned.mli. *)
let malloc = fn "ccb_malloc" (size_t @-> ptr (ptr void) @-> returning int)
let free = fn "ccb_free" (ptr void @-> returning int)
let live_count = fn "ccb_live_count" (ptr llong @-> returning int)
let memcpy_h2d = fn "ccb_memcpy_h2d" (ptr void @-> ptr void @-> size_t @-> handle @-> returning int)
let memcpy_d2h = fn "ccb_memcpy_d2h" (ptr void @-> ptr void @-> size_t @-> handle @-> returning int)
let memcpy_d2d = fn "ccb_memcpy_d2d" (ptr void @-> ptr void @-> size_t @-> handle @-> returning int)
let memset_d8 = fn "ccb_memset_d8" (ptr void @-> uchar @-> size_t @-> handle @-> returning int)
let host_alloc = fn "ccb_host_alloc" (size_t @-> ptr (ptr void) @-> returning int)
let host_free = fn "ccb_host_free" (ptr void @-> returning int)

(* ---------------------------------------------------------------- streams/events
   Replaces lib/runtime/stream.mli and lib/runtime/event.mli. *)
let stream_create = fn "ccb_stream_create" (ptr handle @-> returning int)
let stream_destroy = fn "ccb_stream_destroy" (handle @-> returning int)
let stream_synchronize = fn "ccb_stream_synchronize" (handle @-> returning int)
let stream_query = fn "ccb_stream_query" (handle @-> ptr int @-> returning int)
let event_create = fn "ccb_event_create" (ptr handle @-> returning int)
let event_destroy = fn "ccb_event_destroy" (handle @-> returning int)
let event_record = fn "ccb_event_record" (handle @-> handle @-> returning int)
let event_synchronize = fn "ccb_event_synchronize" (handle @-> returning int)
let event_elapsed_ms = fn "ccb_event_elapsed_ms" (handle @-> handle @-> ptr float @-> returning int)
let stream_wait_event = fn "ccb_stream_wait_event" (handle @-> handle @-> returning int)

(* ---------------------------------------------------------------- modules
   Replaces lib/runtime/jit.mli and lib/runtime/launch.mli. Strings the
   library allocates (compile logs) are returned as char* and released with
   ccb_free_string. *)
let module_compile =
  fn "ccb_module_compile" (string @-> string @-> ptr handle @-> ptr (ptr char) @-> returning int)

let module_unload = fn "ccb_module_unload" (handle @-> returning int)
let module_get_function = fn "ccb_module_get_function" (handle @-> string @-> ptr handle @-> returning int)

let launch =
  fn "ccb_launch"
    (handle @-> uint @-> uint @-> uint @-> uint @-> uint @-> uint @-> uint @-> handle @-> ptr (ptr void) @-> int
   @-> returning int)

let nvrtc_check = fn "ccb_nvrtc_check" (string @-> string @-> ptr size_t @-> ptr (ptr char) @-> returning int)
let free_string = fn "ccb_free_string" (ptr char @-> returning void)

(* ---------------------------------------------------------------- programs
   Replaces Lower/Emit/Jit/Executor (lib/lower, lib/backend_cuda). *)
let program_create = fn "ccb_program_create" (string @-> int @-> int @-> ptr handle @-> returning int)
let program_lower = fn "ccb_program_lower" (string @-> ptr handle @-> returning int)
let program_destroy = fn "ccb_program_destroy" (handle @-> returning int)
let program_source = fn "ccb_program_source" (handle @-> ptr string @-> returning int)
let program_device = fn "ccb_program_device" (handle @-> ptr int @-> returning int)
let program_num_kernels = fn "ccb_program_num_kernels" (handle @-> ptr int @-> returning int)
let program_num_launches = fn "ccb_program_num_launches" (handle @-> ptr int @-> returning int)
let program_plan = fn "ccb_program_plan" (handle @-> ptr string @-> returning int)
let program_num_params = fn "ccb_program_num_params" (handle @-> ptr int @-> returning int)

let program_param =
  fn "ccb_program_param"
    (handle @-> int @-> ptr string @-> ptr int @-> ptr int @-> ptr (ptr llong) @-> returning int)

let program_num_outputs = fn "ccb_program_num_outputs" (handle @-> ptr int @-> returning int)

let program_output =
  fn "ccb_program_output"
    (handle @-> int @-> ptr string @-> ptr int @-> ptr int @-> ptr (ptr llong) @-> returning int)

let program_enqueue =
  fn "ccb_program_enqueue" (handle @-> int @-> ptr (ptr void) @-> ptr (ptr void) @-> returning int)

let program_wait = fn "ccb_program_wait" (handle @-> int @-> returning int)
let program_run = fn "ccb_program_run" (handle @-> ptr (ptr void) @-> ptr (ptr void) @-> returning int)

let program_run_device =
  fn "ccb_program_run_device" (handle @-> int @-> ptr (ptr void) @-> ptr (ptr void) @-> handle @-> returning int)

let program_run_device_events =
  fn "ccb_program_run_device_events"
    (handle @-> int @-> ptr (ptr void) @-> ptr (ptr void) @-> handle @-> ptr handle @-> returning int)

let program_check = fn "ccb_program_check" (handle @-> int @-> handle @-> returning int)
let program_lane_stream = fn "ccb_program_lane_stream" (handle @-> int @-> ptr handle @-> returning int)

(* ---------------------------------------------------------------- sharded programs (no reference counterpart:
   lib/backend_cuda/multi.ml:95-109 averages per-device results on the host) *)
let program_shard = fn "ccb_program_shard" (handle @-> ptr int @-> ptr int @-> returning int)
let program_mailbox_bytes = fn "ccb_program_mailbox_bytes" (handle @-> ptr size_t @-> returning int)
let program_bind_peers = fn "ccb_program_bind_peers" (handle @-> ptr (ptr void) @-> int @-> returning int)

(* ---------------------------------------------------------------- CUDA graphs (no reference counterpart) *)
let graph_begin = fn "ccb_graph_begin" (handle @-> returning int)
let graph_end = fn "ccb_graph_end" (handle @-> ptr handle @-> returning int)
let graph_launch = fn "ccb_graph_launch" (handle @-> handle @-> returning int)
let graph_destroy = fn "ccb_graph_destroy" (handle @-> returning int)

(* ---------------------------------------------------------------- allocation-free sum (no reference counterpart) *)
let sum_f32_noalloc = fn "ccb_sum_f32_noalloc" (ptr float @-> llong @-> ptr float @-> handle @-> returning int)

(* ---------------------------------------------------------------- peer memory and the cross-rank sum
   (no reference counterpart) *)
let ipc_mem_handle = fn "ccb_ipc_mem_handle" (ptr void @-> ptr uchar @-> returning int)
let ipc_mem_open = fn "ccb_ipc_mem_open" (ptr uchar @-> ptr (ptr void) @-> returning int)
let ipc_mem_close = fn "ccb_ipc_mem_close" (ptr void @-> returning int)
let peer_access_enable = fn "ccb_peer_access_enable" (int @-> returning int)
let xrank_mailbox_bytes = fn "ccb_xrank_mailbox_bytes" (int @-> ptr size_t @-> returning int)

let xrank_sum =
  fn "ccb_xrank_sum"
    (ptr void @-> ptr void @-> int @-> int @-> int @-> int @-> ptr (ptr void) @-> ullong @-> ptr uint @-> handle
   @-> returning int)

(* ---------------------------------------------------------------- NCCL (no reference counterpart:
   lib/backend_cuda/multi.ml:51-109 combines on the host) *)
let comm_init_all = fn "ccb_comm_init_all" (int @-> ptr int @-> ptr handle @-> returning int)
let comm_unique_id = fn "ccb_comm_unique_id" (ptr uchar @-> returning int)
let comm_init_rank = fn "ccb_comm_init_rank" (int @-> ptr uchar @-> int @-> ptr handle @-> returning int)
let comm_destroy = fn "ccb_comm_destroy" (handle @-> returning int)

let allreduce =
  fn "ccb_allreduce" (handle @-> ptr void @-> ptr void @-> size_t @-> int @-> int @-> handle @-> returning int)

let group_start = fn "ccb_group_start" (void @-> returning int)
let group_end = fn "ccb_group_end" (void @-> returning int)

(* dtype codes of the C-ABI: 0 f32, 1 f64, 2 i32, 3 i64 *)
let dtype_code : type a. a Cudacaml_ir.Dtype.t -> int = function
  | Cudacaml_ir.Dtype.F32 -> 0
  | Cudacaml_ir.Dtype.F64 -> 1
  | Cudacaml_ir.Dtype.I32 -> 2
  | Cudacaml_ir.Dtype.I64 -> 3
  | Cudacaml_ir.Dtype.Bool -> invalid_arg "Ccb.dtype_code: Bool tensors are not storable"

(* ---------------------------------------------------------------- small helpers *)

(* A fresh out-parameter of type [t], the call, then its value. *)
let out t f =
  let p = allocate_n t ~count:1 in
  f p;
  !@p

let get_int what f = out int (fun p -> check what (f p))
let get_handle what f = out handle (fun p -> check what (f p))

let count () = get_int "ccb_device_count" !!device_count
let current () = get_int "ccb_get_device" !!get_device
let use d = check "ccb_set_device" (!!set_device d)

(* Device.with_device: make [d] current for [f], restore the previous one. *)
let with_device d f =
  let prev = current () in
  use d;
  Fun.protect ~finally:(fun () -> use prev) f

type info = { name : string; compute_capability : int * int; multiprocessors : int; total_memory_bytes : int }

let info_of d =
  let s = make device_info in
  check "ccb_device_info" (!!device_info_ d (addr s));
  let raw = getf s di_name in
  let chars = CArray.to_list raw in
  let rec upto acc = function [] -> List.rev acc | '\000' :: _ -> List.rev acc | c :: r -> upto (c :: acc) r in
  {
    name = String.of_seq (List.to_seq (upto [] chars));
    compute_capability = (getf s di_cc_major, getf s di_cc_minor);
    multiprocessors = getf s di_multiprocessors;
    total_memory_bytes = Int64.to_int (Signed.LLong.to_int64 (getf s di_total_memory_bytes));
  }
