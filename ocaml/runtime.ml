(* The runtime layer over libccb.so: Device, Buffer, Stream, Event, Pinned.

   NOT BUILT HERE: the build image has no OCaml toolchain. These modules
   replace lib/runtime/{device,buffer,stream,event,pinned}.ml, keeping their
   .mli signatures (lib/runtime/*.mli) except the cudajit-typed seams
   ([Buffer.unsafe_ptr], [Stream.unsafe_stream]), which now return the raw
   pointer libccb.so takes (a [unit Ctypes.ptr]). Jit and Launch are not
   needed by the backend any more (libccb.so compiles and launches whole
   programs); [Ccb.module_compile] / [Ccb.launch] remain for tools that want
   a hand-written kernel. *)

open Cudacaml_ir

let ( !! ) = Lazy.force

module Device = struct
  let available () = try !!Ccb.available () = 1 with _ -> false
  let init () = Ccb.check "ccb_init" (!!Ccb.init ())
  let synchronize () = Ccb.check "ccb_device_synchronize" (!!Ccb.device_synchronize ())
  let count () = Ccb.count ()

  (* The device a [with_device] has made current; 0 outside one. *)
  let current_ = ref 0
  let current () = !current_

  let with_device d f =
    let prev = !current_ in
    Ccb.use d;
    current_ := d;
    Fun.protect
      ~finally:(fun () ->
        Ccb.use prev;
        current_ := prev)
      f

  type info = Ccb.info = {
    name : string;
    compute_capability : int * int;
    multiprocessors : int;
    total_memory_bytes : int;
  }

  let info_of d = Ccb.info_of d
  let info () = info_of 0
  let name () = (info ()).name

  let info_to_string i =
    Printf.sprintf "device: %s\ncompute: sm_%d%d\nmultiprocessors: %d\nmemory_mib: %d\n" i.name
      (fst i.compute_capability) (snd i.compute_capability) i.multiprocessors (i.total_memory_bytes / 1048576)
end

module Stream = struct
  type t = Ccb.handle

  let default : t = Ctypes.null

  let create () = Ccb.get_handle "ccb_stream_create" !!Ccb.stream_create
  let synchronize s = Ccb.check "ccb_stream_synchronize" (!!Ccb.stream_synchronize s)
  let is_idle s = Ccb.get_int "ccb_stream_query" (!!Ccb.stream_query s) = 1
  let unsafe_stream (s : t) = s
end

module Event = struct
  (* A record, so the finaliser that destroys the driver event is attached
     to a heap block that lives exactly as long as the event is reachable. *)
  type t = { h : Ccb.handle }

  let record s =
    let h = Ccb.get_handle "ccb_event_create" !!Ccb.event_create in
    Ccb.check "ccb_event_record" (!!Ccb.event_record h s);
    let e = { h } in
    Gc.finalise (fun e -> ignore (!!Ccb.event_destroy e.h)) e;
    e

  let wait s e = Ccb.check "ccb_stream_wait_event" (!!Ccb.stream_wait_event s e.h)
  let synchronize e = Ccb.check "ccb_event_synchronize" (!!Ccb.event_synchronize e.h)

  let elapsed_ms ~start ~stop =
    Ccb.out Ctypes.float (fun p -> Ccb.check "ccb_event_elapsed_ms" (!!Ccb.event_elapsed_ms start.h stop.h p))
end

(* Host storage of a [Value] as a void pointer (Bigarray data, never moved
   by the GC). *)
let host_ptr (Value.P v) =
  match Value.raw v with
  | Value.Raw a -> Ctypes.to_voidp (Ctypes.bigarray_start Ctypes.array1 a)

let host_bytes (Value.P v) = Value.byte_size v

module Buffer = struct
  type t = { ptr : unit Ctypes.ptr; bytes : int; mutable live : bool }

  let alloc ~bytes =
    let p = Ccb.out (Ctypes.ptr Ctypes.void) (fun p ->
                Ccb.check "ccb_malloc" (!!Ccb.malloc (Unsigned.Size_t.of_int bytes) p)) in
    { ptr = p; bytes; live = true }

  let free b =
    if b.live then begin
      b.live <- false;
      Ccb.check "ccb_free" (!!Ccb.free b.ptr)
    end

  let byte_size b = b.bytes

  let live_count () =
    Int64.to_int (Signed.LLong.to_int64 (Ccb.out Ctypes.llong (fun p -> Ccb.check "ccb_live_count" (!!Ccb.live_count p))))

  let same_size what v b =
    if host_bytes v <> b.bytes then
      invalid_arg (Printf.sprintf "%s: %d host bytes, %d device bytes" what (host_bytes v) b.bytes)

  let upload_async v b ~stream =
    same_size "Buffer.upload" v b;
    Ccb.check "ccb_memcpy_h2d" (!!Ccb.memcpy_h2d b.ptr (host_ptr v) (Unsigned.Size_t.of_int b.bytes) stream)

  let download_async b v ~stream =
    same_size "Buffer.download" v b;
    Ccb.check "ccb_memcpy_d2h" (!!Ccb.memcpy_d2h (host_ptr v) b.ptr (Unsigned.Size_t.of_int b.bytes) stream)

  let upload v b =
    upload_async v b ~stream:Stream.default;
    Stream.synchronize Stream.default

  let download b v =
    download_async b v ~stream:Stream.default;
    Stream.synchronize Stream.default

  let copy_device ~dst ~src ~stream =
    if dst.bytes <> src.bytes then invalid_arg "Buffer.copy_device: sizes differ";
    Ccb.check "ccb_memcpy_d2d" (!!Ccb.memcpy_d2d dst.ptr src.ptr (Unsigned.Size_t.of_int src.bytes) stream)

  let unsafe_ptr b = b.ptr
end

(* Page-locked host memory from ccb_host_alloc (cuMemHostAlloc, PORTABLE,
   zero-filled), freed by a finaliser on the Bigarray that views it, as
   lib/runtime/pinned.ml:76-108 does. *)
module Pinned = struct
  let owned : (nativeint, unit) Hashtbl.t = Hashtbl.create 64

  let alloc_bytes n =
    Ccb.out (Ctypes.ptr Ctypes.void) (fun p ->
        Ccb.check "ccb_host_alloc" (!!Ccb.host_alloc (Unsigned.Size_t.of_int (max n 1)) p))

  let own p a =
    let key = Ctypes.raw_address_of_ptr p in
    Hashtbl.replace owned key ();
    Gc.finalise
      (fun _ ->
        Hashtbl.remove owned key;
        ignore (!!Ccb.host_free p))
      a

  let alloc : type a. a Dtype.t -> Shape.t -> a Value.t =
   fun dtype shape ->
    let n = Shape.numel shape in
    let p = alloc_bytes (n * Dtype.size_in_bytes dtype) in
    let raw : a Value.raw =
      match dtype with
      | Dtype.F32 ->
          let a = Ctypes.(bigarray_of_ptr array1 n Bigarray.Float32 (from_voidp float p)) in
          own p a;
          Value.Raw a
      | Dtype.F64 ->
          let a = Ctypes.(bigarray_of_ptr array1 n Bigarray.Float64 (from_voidp double p)) in
          own p a;
          Value.Raw a
      | Dtype.I32 ->
          let a = Ctypes.(bigarray_of_ptr array1 n Bigarray.Int32 (from_voidp int32_t p)) in
          own p a;
          Value.Raw a
      | Dtype.I64 ->
          let a = Ctypes.(bigarray_of_ptr array1 n Bigarray.Int64 (from_voidp int64_t p)) in
          own p a;
          Value.Raw a
      | Dtype.Bool -> invalid_arg "Pinned.alloc: Bool tensors are not storable"
    in
    Value.of_raw dtype shape raw

  let of_value v =
    let c = alloc (Value.dtype v) (Value.shape v) in
    for i = 0 to Value.numel v - 1 do
      Value.set c i (Value.get v i)
    done;
    c

  let is_pinned v = Hashtbl.mem owned (Ctypes.raw_address_of_ptr (host_ptr (Value.P v)))
end
