(* Program: compiled graphs on libccb.so -- the body of
   Cudacaml_backend_cuda (lib/backend_cuda/cudacaml_backend_cuda.mli:6-84),
   kept in its own module so that Multi can use it without a cycle.

   NOT BUILT HERE: the build image has no OCaml toolchain. The graph crosses
   the C-ABI once as text (Wire.to_wire); libccb.so lowers it to the sm_100a
   skeletons, compiles it with NVRTC and owns one executor (stream + buffer
   pool) per lane. The Python mirror of this module is
   cudacaml_b200/backend_cuda.py, which the repository's tests exercise call
   for call. *)

open Cudacaml_ir
open Cudacaml_runtime

let name = "cuda"
let ( !! ) = Lazy.force

type io = { io_name : string; io_dtype : Dtype.packed; io_shape : Shape.t }

type compiled = {
  prog : Ccb.handle;
  device : int;
  streams : int;
  params : io list;  (** in the order ccb_program_enqueue takes them *)
  outputs : io list;
  mutable next : int;
  mutable released : bool;
}

let dtype_of_code = function
  | 0 -> Dtype.P Dtype.F32
  | 1 -> Dtype.P Dtype.F64
  | 2 -> Dtype.P Dtype.I32
  | 3 -> Dtype.P Dtype.I64
  | k -> failwith (Printf.sprintf "libccb: unknown dtype code %d" k)

(* Params and outputs as the program reports them (ccb_program_param /
   ccb_program_output): name, dtype code, rank, dims. *)
let ios prog count get =
  let n = Ccb.get_int "ccb_program_num_*" (count prog) in
  List.init n (fun i ->
      let nm = Ctypes.allocate Ctypes.string "" in
      let dt = Ctypes.allocate Ctypes.int 0 and rank = Ctypes.allocate Ctypes.int 0 in
      let dims = Ctypes.allocate (Ctypes.ptr Ctypes.llong) (Ctypes.from_voidp Ctypes.llong Ctypes.null) in
      Ccb.check "ccb_program_param/output" (get prog i nm dt rank dims);
      let r = Ctypes.( !@ ) rank in
      let d = Ctypes.( !@ ) dims in
      let shape =
        Shape.of_dims
          (List.init r (fun k -> Int64.to_int (Signed.LLong.to_int64 (Ctypes.( !@ ) (Ctypes.( +@ ) d k)))))
      in
      { io_name = Ctypes.( !@ ) nm; io_dtype = dtype_of_code (Ctypes.( !@ ) dt); io_shape = shape })

let source graph =
  let h = Ccb.get_handle "ccb_program_lower" (!!Ccb.program_lower (Wire.to_wire graph)) in
  Fun.protect
    ~finally:(fun () -> ignore (!!Ccb.program_destroy h))
    (fun () -> Ccb.out Ctypes.string (fun p -> Ccb.check "ccb_program_source" (!!Ccb.program_source h p)))

let release c =
  if not c.released then begin
    c.released <- true;
    Ccb.check "ccb_program_destroy" (!!Ccb.program_destroy c.prog)
  end

(* ?shard:(rank, world): rank [rank] of a sharded Monte-Carlo program
   (include/ccb.h, sharded programs); bind_peers before its first run. *)
let compile_on ~device ?(streams = 1) ?shard graph =
  if streams < 1 then invalid_arg "Backend_cuda.compile_on: streams must be >= 1";
  let prog =
    Ccb.get_handle "ccb_program_create" (!!Ccb.program_create (Wire.to_wire ?shard graph) device streams)
  in
  let c =
    {
      prog;
      device;
      streams;
      params = ios prog !!Ccb.program_num_params !!Ccb.program_param;
      outputs = ios prog !!Ccb.program_num_outputs !!Ccb.program_output;
      next = 0;
      released = false;
    }
  in
  Gc.finalise (fun c -> try release c with _ -> ()) c;
  c

let mailbox_bytes c =
  Unsigned.Size_t.to_int
    (Ccb.out Ctypes.size_t (fun p -> Ccb.check "ccb_program_mailbox_bytes" (!!Ccb.program_mailbox_bytes c.prog p)))

(* Every rank's mailbox as this rank addresses it, in rank order; each owner
   zero-fills its own before any rank's first run. *)
let bind_peers c (mailboxes : unit Ctypes.ptr list) =
  let arr = Ctypes.CArray.of_list (Ctypes.ptr Ctypes.void) mailboxes in
  Ccb.check "ccb_program_bind_peers"
    (!!Ccb.program_bind_peers c.prog (Ctypes.CArray.start arr) (List.length mailboxes))

let compile_with ~streams graph = compile_on ~device:0 ~streams graph
let compile graph = compile_on ~device:0 graph
let device_of c = c.device

let live c = if c.released then failwith "Backend_cuda.run: compiled program has been released"

(* Every param present with its dtype and shape before a byte moves
   (lib/backend_cuda/executor.ml:14-21). *)
let bind c inputs =
  List.map
    (fun io ->
      match List.assoc_opt io.io_name inputs with
      | None -> invalid_arg ("Executor.run: missing input " ^ io.io_name)
      | Some (Value.P v as p) ->
          if Dtype.packed_name io.io_dtype <> Dtype.name (Value.dtype v) then
            invalid_arg (Printf.sprintf "Executor.run: input %s has dtype %s, expected %s" io.io_name
                           (Dtype.name (Value.dtype v)) (Dtype.packed_name io.io_dtype));
          if not (Shape.equal (Value.shape v) io.io_shape) then
            invalid_arg (Printf.sprintf "Executor.run: input %s has shape %s, expected %s" io.io_name
                           (Shape.to_string (Value.shape v)) (Shape.to_string io.io_shape));
          p)
    c.params

let fresh_outputs c =
  List.map (fun io -> match io.io_dtype with Dtype.P d -> (io.io_name, Value.P (Value.create d io.io_shape))) c.outputs

(* Host storage of a [Value] (Bigarray data, never moved by the GC). *)
let host_ptr (Value.P v) =
  match Value.raw v with Value.Raw a -> Ctypes.to_voidp (Ctypes.bigarray_start Ctypes.array1 a)

let ptr_array vs = Ctypes.CArray.(start (of_list (Ctypes.ptr Ctypes.void) (List.map host_ptr vs)))

type job = { jc : compiled; lane : int; keep : Value.packed list; outs : (string * Value.packed) list;
             mutable done_ : bool }

let run_async c ~inputs =
  live c;
  let ins = bind c inputs in
  let outs = fresh_outputs c in
  let lane = c.next in
  c.next <- (c.next + 1) mod c.streams;
  Ccb.check "ccb_program_enqueue"
    (!!Ccb.program_enqueue c.prog lane (ptr_array ins) (ptr_array (List.map snd outs)));
  { jc = c; lane; keep = ins; outs; done_ = false }

let wait j =
  if not j.done_ then begin
    Ccb.check "ccb_program_wait" (!!Ccb.program_wait j.jc.prog j.lane);
    j.done_ <- true
  end;
  ignore (Sys.opaque_identity j.keep);
  j.outs

let run c ~inputs =
  live c;
  let ins = bind c inputs in
  let outs = fresh_outputs c in
  Ccb.check "ccb_program_run" (!!Ccb.program_run c.prog (ptr_array ins) (ptr_array (List.map snd outs)));
  ignore (Sys.opaque_identity ins);
  outs

(* ------------------------------------------------------------------ *)
(* Device-resident values                                              *)
(* ------------------------------------------------------------------ *)

type resident = { buf : Buffer.t; dtype : Dtype.packed; shape : Shape.t }

let upload (Value.P v as p) =
  Device.init ();
  let buf = Buffer.alloc ~bytes:(Value.byte_size v) in
  Buffer.upload p buf;
  { buf; dtype = Dtype.P (Value.dtype v); shape = Value.shape v }

let download r =
  let v = match r.dtype with Dtype.P d -> Value.P (Value.create d r.shape) in
  Buffer.download r.buf v;
  v

let free_resident r = Buffer.free r.buf

(* Zero-copy on the residents' pointers; outputs are freshly allocated
   residents the caller owns. issue_resident only issues the run on lane 0
   (check synchronises and reads the lane's device error word); run_resident
   does both. The ranks of a sharded program wait on each other inside the
   kernel, so Multi issues every device's run before it checks any. *)
let issue_resident c ~inputs =
  live c;
  Device.with_device c.device (fun () ->
      let ins =
        List.map
          (fun io ->
            match List.assoc_opt io.io_name inputs with
            | None -> invalid_arg ("Executor.run_resident: missing input " ^ io.io_name)
            | Some r ->
                let want = match io.io_dtype with Dtype.P d -> Shape.numel io.io_shape * Dtype.size_in_bytes d in
                if Buffer.byte_size r.buf <> want then
                  invalid_arg (Printf.sprintf "Executor.run_resident: input %s has %d bytes, expected %d" io.io_name
                                 (Buffer.byte_size r.buf) want);
                Buffer.unsafe_ptr r.buf)
          c.params
      in
      let outs =
        List.map
          (fun io ->
            let bytes = match io.io_dtype with Dtype.P d -> Shape.numel io.io_shape * Dtype.size_in_bytes d in
            (io.io_name, { buf = Buffer.alloc ~bytes; dtype = io.io_dtype; shape = io.io_shape }))
          c.outputs
      in
      let arr l = Ctypes.CArray.(start (of_list (Ctypes.ptr Ctypes.void) l)) in
      Ccb.check "ccb_program_run_device"
        (!!Ccb.program_run_device c.prog 0 (arr ins)
           (arr (List.map (fun (_, r) -> Buffer.unsafe_ptr r.buf) outs))
           Stream.default);
      outs)

let check c =
  Device.with_device c.device (fun () -> Ccb.check "ccb_program_check" (!!Ccb.program_check c.prog 0 Stream.default))

let run_resident c ~inputs =
  let outs = issue_resident c ~inputs in
  check c;
  outs
