(* Multi over libccb.so: data-parallel runs across the GPUs of one box,
   behind the reference's signature (lib/backend_cuda/multi.mli:14-64) plus
   optional additions.

   NOT BUILT HERE: the build image has no OCaml toolchain. This file replaces
   lib/backend_cuda/multi.ml. Its Python mirror is cudacaml_b200/multi.py,
   which the repository's CPU (gloo, world size 2) and GPU (two B200s, NCCL)
   tests exercise.

   Additions, all optional:
   - [?counter_key]: split a Monte-Carlo graph by Philox counter range with
     the same seed (device d draws counters [d*n/D, (d+1)*n/D)) instead of
     asking the caller to reseed each device (multi.mli:39-44);
   - [?split]: slice only the named inputs by rows;
   - [allreduce_sum]: recombine whole outputs on the devices with NCCL
     (ccb_allreduce inside ccb_group_start/end) over NVLink;
   - [allreduce_mean]: recombine scalar outputs with the cross-device sum
     over NVLink peer memory (ccb_xrank_sum);
   - [?sharded]: compile the unsplit graph on every device as one rank of a
     sharded Monte-Carlo program (ccb_program_bind_peers): device i walks
     paths [i*n/D, (i+1)*n/D) and the kernel's last block combines all
     devices' totals over NVLink, so every device's outputs are already the
     whole run's. *)

open Cudacaml_ir
open Cudacaml_runtime
module B = Program

let ( !! ) = Lazy.force
let ctr_base = "__ctr_base"

(* Device i of d's share of n paths: (first path, count). Rng counters are
   I32 flat indices, so the whole range must stay below 2^31. *)
let path_range ~n ~d i =
  if d <= 0 || i < 0 || i >= d then invalid_arg (Printf.sprintf "Multi: device %d of %d" i d);
  if n mod d <> 0 then invalid_arg (Printf.sprintf "Multi.create: n = %d is not divisible by %d devices" n d);
  if n > 1 lsl 31 then invalid_arg (Printf.sprintf "Multi: %d paths exceed the I32 counter range (2^31)" n);
  (i * (n / d), n / d)

(* Rewrite every Rng.u32 counter [map2 f (iota s) (broadcast s key)]
   (lib/rng/rng.ml:49-59) whose leading dimension is [rows] to count from the
   scalar parameter [__ctr_base] times the draw's elements per path. *)
let offset_counters ~key ~rows (g : Graph.t) : Graph.t =
  let base = Dsl.scalar ctr_base Dtype.I32 in
  let memo : (int, Tensor.packed) Hashtbl.t = Hashtbl.create 256 in
  let cast_as : type a b. a Tensor.t -> b Tensor.t -> b Tensor.t =
   fun like x -> match Dtype.equal like.Tensor.dtype x.Tensor.dtype with Some Dtype.Equal -> x | None -> assert false
  in
  let is_key_broadcast : type b. b Tensor.t -> bool =
   fun k ->
    match k.Tensor.node with
    | Tensor.Broadcast (_, p) -> ( match p.Tensor.node with Tensor.Param n -> n = key | _ -> false)
    | _ -> false
  in
  let rec go : type a. a Tensor.t -> a Tensor.t =
   fun t ->
    let k = Uid.to_int t.Tensor.uid in
    match Hashtbl.find_opt memo k with
    | Some (Tensor.P t') -> cast_as t t'
    | None ->
        let t' = rebuild t in
        Hashtbl.add memo k (Tensor.P t');
        t'
  and rebuild : type a. a Tensor.t -> a Tensor.t =
   fun t ->
    let mk node = Tensor.make t.Tensor.dtype t.Tensor.shape node in
    match t.Tensor.node with
    | Tensor.Param _ | Tensor.Iota -> t
    | Tensor.Map (f, a) ->
        let a' = go a in
        if a' == a then t else mk (Tensor.Map (f, a'))
    | Tensor.Map2 (f, a, b) -> (
        let counter =
          match (a.Tensor.node, Dtype.equal a.Tensor.dtype Dtype.I32) with
          | Tensor.Iota, Some Dtype.Equal
            when is_key_broadcast b
                 && (match Shape.dims a.Tensor.shape with r :: _ -> r = rows | [] -> false) ->
              let per_path = List.fold_left ( * ) 1 (List.tl (Shape.dims a.Tensor.shape)) in
              let start =
                if per_path = 1 then base
                else Dsl.map (fun v -> Dsl.mul v (Dsl.const Dtype.I32 (Int32.of_int per_path))) base
              in
              let shifted = Dsl.map2 Dsl.add a (Dsl.broadcast a.Tensor.shape start) in
              Some (mk (Tensor.Map2 (f, cast_as a shifted, b)))
          | _ -> None
        in
        match counter with
        | Some t' -> t'
        | None ->
            let a' = go a and b' = go b in
            if a' == a && b' == b then t else mk (Tensor.Map2 (f, a', b')))
    | Tensor.Reduce (f, init, a) ->
        let a' = go a in
        if a' == a then t else mk (Tensor.Reduce (f, init, a'))
    | Tensor.Scan (f, init, a) ->
        let a' = go a in
        if a' == a then t else mk (Tensor.Scan (f, init, a'))
    | Tensor.Gather (i, a) ->
        let i' = go i and a' = go a in
        if i' == i && a' == a then t else mk (Tensor.Gather (i', a'))
    | Tensor.Scatter_add (i, a, s) ->
        let i' = go i and a' = go a in
        if i' == i && a' == a then t else mk (Tensor.Scatter_add (i', a', s))
    | Tensor.Matmul (a, b) ->
        let a' = go a and b' = go b in
        if a' == a && b' == b then t else mk (Tensor.Matmul (a', b'))
    | Tensor.Reshape (s, a) ->
        let a' = go a in
        if a' == a then t else mk (Tensor.Reshape (s, a'))
    | Tensor.Broadcast (s, a) ->
        let a' = go a in
        if a' == a then t else mk (Tensor.Broadcast (s, a'))
  in
  Graph.create ~name:(Graph.name g) ~outputs:(List.map (fun (n, Tensor.P t) -> (n, Tensor.P (go t))) (Graph.outputs g))

type t = {
  slots : (int * B.compiled) array;  (** (ordinal, program) *)
  n : int;
  per : int;
  counter : bool;
  split : string list option;
  sharded : bool;
  mailboxes : (int * Buffer.t) array;  (** sharded: (ordinal, mailbox) per device *)
  mutable comms : Ccb.handle array option;
  mutable released : bool;
}

let release t =
  if not t.released then begin
    t.released <- true;
    Array.iter (fun (_, c) -> B.release c) t.slots;
    Array.iter (fun (d, b) -> Device.with_device d (fun () -> Buffer.free b)) t.mailboxes;
    Option.iter (Array.iter (fun h -> ignore (!!Ccb.comm_destroy h))) t.comms;
    t.comms <- None
  end

let create ~devices ~n ?counter_key ?split ?(sharded = false) build =
  let d = List.length devices in
  if d = 0 then invalid_arg "Multi.create: devices must not be empty";
  if n mod d <> 0 then invalid_arg (Printf.sprintf "Multi.create: n = %d is not divisible by %d devices" n d);
  if sharded && (counter_key <> None || split <> None) then
    invalid_arg "Multi.create: a sharded Multi splits the index space itself (no counter_key, no split)";
  if sharded && List.length (List.sort_uniq compare devices) <> d then
    invalid_arg "Multi.create: a sharded Multi needs distinct devices (its ranks wait on each other)";
  if counter_key <> None then ignore (path_range ~n ~d 0);
  let per = n / d in
  let sharded = sharded && d > 1 in
  let slots =
    Array.of_list
      (List.mapi
         (fun i ordinal ->
           if sharded then (ordinal, B.compile_on ~device:ordinal ~shard:(i, d) (build ~n))
           else
             let g = build ~n:per in
             let g = match counter_key with Some key -> offset_counters ~key ~rows:per g | None -> g in
             (ordinal, B.compile_on ~device:ordinal g))
         devices)
  in
  let mailboxes =
    if not sharded then [||]
    else begin
      let bytes = B.mailbox_bytes (snd slots.(0)) in
      let ords = Array.of_list devices in
      let boxes =
        Array.map
          (fun dv ->
            Device.with_device dv (fun () ->
                Array.iter (fun q -> if q <> dv then Ccb.check "ccb_peer_access_enable" (!!Ccb.peer_access_enable q)) ords;
                let b = Buffer.alloc ~bytes in
                Ccb.check "ccb_memset_d8"
                  (!!Ccb.memset_d8 (Buffer.unsafe_ptr b) (Unsigned.UChar.of_int 0) (Unsigned.Size_t.of_int bytes) Stream.default);
                Device.synchronize ();
                (dv, b)))
          ords
      in
      let ptrs = Array.to_list (Array.map (fun (_, b) -> Buffer.unsafe_ptr b) boxes) in
      Array.iter (fun (_, c) -> B.bind_peers c ptrs) slots;
      boxes
    end
  in
  let t = { slots; n; per; counter = counter_key <> None; split; sharded; mailboxes; comms = None; released = false } in
  Gc.finalise (fun t -> try release t with _ -> ()) t;
  t

let leading_dim (Value.P v) = match Shape.dims (Value.shape v) with d :: _ -> Some d | [] -> None

(* Rows [i*per, (i+1)*per) of a value whose leading dimension is n: a
   Bigarray sub-view, no host copy. *)
let slice ~index ~per (Value.P v) =
  let dims = Shape.dims (Value.shape v) in
  let row = List.fold_left ( * ) 1 (List.tl dims) in
  match Value.raw v with
  | Value.Raw a ->
      let sub = Bigarray.Array1.sub a (index * per * row) (per * row) in
      Value.P (Value.of_raw (Value.dtype v) (Shape.of_dims (per :: List.tl dims)) (Value.Raw sub))

let splits t name v =
  match t.split with
  | Some names ->
      if List.mem name names && leading_dim v <> Some t.n then
        invalid_arg (Printf.sprintf "Multi.run: input %s does not have leading dimension %d" name t.n);
      List.mem name names
  | None -> leading_dim v = Some t.n

let inputs_for t i inputs =
  if t.sharded then inputs else
  let ins = List.map (fun (name, v) -> if splits t name v then (name, slice ~index:i ~per:t.per v) else (name, v)) inputs in
  if t.counter then
    let first, _ = path_range ~n:t.n ~d:(Array.length t.slots) i in
    ins @ [ (ctr_base, Value.P (Value.of_list Dtype.I32 Shape.scalar [ Int32.of_int first ])) ]
  else ins

let run_per_device t ~inputs =
  if t.released then failwith "Multi.run: this Multi.t has been released";
  if t.sharded then begin
    (* every device's run is issued before any is waited on: a sharded
       kernel's last block waits for all devices' totals *)
    let issued =
      Array.mapi
        (fun i (d, c) ->
          Device.with_device d (fun () ->
              let ins = List.map (fun (nm, v) -> (nm, B.upload v)) (inputs i) in
              (ins, B.issue_resident c ~inputs:ins)))
        t.slots
    in
    Array.to_list
      (Array.mapi
         (fun i (ins, outs) ->
           let d, c = t.slots.(i) in
           B.check c;
           Device.with_device d (fun () ->
               let vals = List.map (fun (nm, r) -> (nm, B.download r)) outs in
               List.iter (fun (_, r) -> B.free_resident r) (ins @ outs);
               vals))
         issued)
  end
  else
    let jobs = Array.mapi (fun i (_, c) -> B.run_async c ~inputs:(inputs i)) t.slots in
    Array.to_list (Array.map B.wait jobs)

let run t ~inputs = run_per_device t ~inputs:(fun i -> inputs_for t i inputs)

let concat vs =
  match vs with
  | [] -> invalid_arg "Multi.concat: no values to concatenate"
  | Value.P first :: _ ->
      let rest = match Shape.dims (Value.shape first) with [] -> invalid_arg "Multi.concat: a rank-0 value has no leading axis" | _ :: r -> r in
      let lead =
        List.fold_left
          (fun acc (Value.P v) ->
            match (Dtype.equal (Value.dtype v) (Value.dtype first), Shape.dims (Value.shape v)) with
            | Some Dtype.Equal, d :: r when r = rest -> acc + d
            | _ -> invalid_arg "Multi.concat: dtype or trailing shape mismatch")
          0 vs
      in
      let out = Value.create (Value.dtype first) (Shape.of_dims (lead :: rest)) in
      let k = ref 0 in
      List.iter
        (fun (Value.P v) ->
          match Dtype.equal (Value.dtype v) (Value.dtype first) with
          | Some Dtype.Equal ->
              for j = 0 to Value.numel v - 1 do
                Value.set out !k (Value.get v j);
                incr k
              done
          | None -> assert false)
        vs;
      Value.P out

let scalar_float (Value.P v) =
  if Value.numel v <> 1 then invalid_arg "Multi.mean_scalar: not a scalar";
  match Value.dtype v with
  | Dtype.F32 -> Value.get v 0
  | Dtype.F64 -> Value.get v 0
  | Dtype.I32 -> Int32.to_float (Value.get v 0)
  | Dtype.I64 -> Int64.to_float (Value.get v 0)
  | Dtype.Bool -> invalid_arg "Multi.mean_scalar: a bool output has no mean"

let mean_scalar = function
  | [] -> invalid_arg "Multi.mean_scalar: no values to average"
  | vs -> List.fold_left (fun acc v -> acc +. scalar_float v) 0.0 vs /. float_of_int (List.length vs)

(* Run every device resident, then one grouped NCCL all-reduce (sum) per
   named output, on the devices; the sums are read back from the first
   device. Needs distinct ordinals (NCCL puts one rank on each GPU). *)
let allreduce_sum t ~names ~inputs =
  if t.released then failwith "Multi.run: this Multi.t has been released";
  let ords = Array.map fst t.slots in
  if List.length (List.sort_uniq compare (Array.to_list ords)) <> Array.length ords then
    invalid_arg "Multi.allreduce: NCCL needs distinct devices; use mean_scalar for repeats";
  let d = Array.length t.slots in
  let comms =
    match t.comms with
    | Some c -> c
    | None ->
        let devs = Ctypes.CArray.of_list Ctypes.int (Array.to_list ords) in
        let hs = Ctypes.CArray.make Ccb.handle d in
        Ccb.check "ccb_comm_init_all" (!!Ccb.comm_init_all d (Ctypes.CArray.start devs) (Ctypes.CArray.start hs));
        let c = Array.of_list (Ctypes.CArray.to_list hs) in
        t.comms <- Some c;
        c
  in
  let per_dev =
    Array.mapi
      (fun i (_, c) ->
        let ins = List.map (fun (n, v) -> (n, B.upload v)) (inputs_for t i inputs) in
        let outs = B.run_resident c ~inputs:ins in
        List.iter (fun (_, r) -> B.free_resident r) ins;
        outs)
      t.slots
  in
  List.iter
    (fun name ->
      Ccb.check "ccb_group_start" (!!Ccb.group_start ());
      Array.iteri
        (fun i (ordinal, _) ->
          let r = List.assoc name per_dev.(i) in
          let count = Shape.numel r.B.shape in
          let code = match r.B.dtype with Dtype.P dt -> Ccb.dtype_code dt in
          Device.with_device ordinal (fun () ->
              let p = Buffer.unsafe_ptr r.B.buf in
              Ccb.check "ccb_allreduce"
                (!!Ccb.allreduce comms.(i) p p (Unsigned.Size_t.of_int count) code 0 Stream.default)))
        t.slots;
      Ccb.check "ccb_group_end" (!!Ccb.group_end ()))
    names;
  Array.iter (fun (ordinal, _) -> Device.with_device ordinal Device.synchronize) t.slots;
  let result =
    List.map (fun name -> (name, Device.with_device (fst t.slots.(0)) (fun () -> B.download (List.assoc name per_dev.(0))))) names
  in
  Array.iteri
    (fun i (ordinal, _) -> Device.with_device ordinal (fun () -> List.iter (fun (_, r) -> B.free_resident r) per_dev.(i)))
    t.slots;
  result

(* Scalar outputs are recombined over NVLink peer memory instead: one
   mailbox per device (zero-filled before any device's first sum), peer
   access between the devices, then per named output one ccb_xrank_sum per
   device (a 32-thread kernel; every device gets the same bits). *)
type peer = { boxes : unit Ctypes.ptr Ctypes.CArray.t; errs : Buffer.t array; owned : Buffer.t array;
              mutable epoch : int }

let peers : (int list, peer) Hashtbl.t = Hashtbl.create 4

let peer_of ords =
  let key = Array.to_list ords in
  match Hashtbl.find_opt peers key with
  | Some p -> p
  | None ->
      let n = Array.length ords in
      let bytes = Ccb.out Ctypes.size_t (fun p -> Ccb.check "ccb_xrank_mailbox_bytes" (!!Ccb.xrank_mailbox_bytes n p)) in
      let bytes = Unsigned.Size_t.to_int bytes in
      let owned, errs =
        Array.split
          (Array.map
             (fun d ->
               Device.with_device d (fun () ->
                   Array.iter (fun q -> if q <> d then Ccb.check "ccb_peer_access_enable" (!!Ccb.peer_access_enable q)) ords;
                   let b = Buffer.alloc ~bytes and e = Buffer.alloc ~bytes:4 in
                   Ccb.check "ccb_memset_d8" (!!Ccb.memset_d8 (Buffer.unsafe_ptr b) (Unsigned.UChar.of_int 0) (Unsigned.Size_t.of_int bytes) Stream.default);
                   Ccb.check "ccb_memset_d8" (!!Ccb.memset_d8 (Buffer.unsafe_ptr e) (Unsigned.UChar.of_int 0) (Unsigned.Size_t.of_int 4) Stream.default);
                   Device.synchronize ();
                   (b, e)))
             ords)
      in
      let boxes = Ctypes.CArray.of_list (Ctypes.ptr Ctypes.void) (Array.to_list (Array.map Buffer.unsafe_ptr owned)) in
      let p = { boxes; errs; owned; epoch = 0 } in
      Hashtbl.add peers key p;
      p

let allreduce_mean t ~names ~inputs =
  if t.released then failwith "Multi.run: this Multi.t has been released";
  if t.sharded then
    (* every device's outputs are already the whole run's *)
    let outs = List.hd (run t ~inputs) in
    List.map (fun name -> (name, scalar_float (List.assoc name outs))) names
  else
  let ords = Array.map fst t.slots in
  if List.length (List.sort_uniq compare (Array.to_list ords)) <> Array.length ords then
    invalid_arg "Multi.allreduce: a cross-device sum needs distinct devices; use mean_scalar for repeats";
  let n = Array.length ords in
  let pe = peer_of ords in
  let per_dev =
    Array.mapi
      (fun i (_, c) ->
        let ins = List.map (fun (nm, v) -> (nm, B.upload v)) (inputs_for t i inputs) in
        let outs = B.run_resident c ~inputs:ins in
        List.iter (fun (_, r) -> B.free_resident r) ins;
        outs)
      t.slots
  in
  List.iter
    (fun name ->
      pe.epoch <- pe.epoch + 1;
      Array.iteri
        (fun i ordinal ->
          let r = List.assoc name per_dev.(i) in
          if Shape.numel r.B.shape <> 1 then invalid_arg ("Multi.allreduce_mean: output " ^ name ^ " is not a scalar");
          let code = match r.B.dtype with Dtype.P dt -> Ccb.dtype_code dt in
          Device.with_device ordinal (fun () ->
              let p = Buffer.unsafe_ptr r.B.buf in
              Ccb.check "ccb_xrank_sum"
                (!!Ccb.xrank_sum p p 1 code n i (Ctypes.CArray.start pe.boxes) (Unsigned.ULLong.of_int pe.epoch)
                   (Ctypes.from_voidp Ctypes.uint (Buffer.unsafe_ptr pe.errs.(i))) Stream.default)))
        ords)
    names;
  Array.iter (fun d -> Device.with_device d Device.synchronize) ords;
  Array.iteri
    (fun i d ->
      Device.with_device d (fun () ->
          let w = Value.create Dtype.I32 (Shape.of_dims [ 1 ]) in
          Buffer.download pe.errs.(i) (Value.P w);
          if Int32.logand (Value.get w 0) 32l <> 0l then failwith "Multi.allreduce_mean: a peer did not publish (bounded wait gave up)"))
    ords;
  let result =
    List.map
      (fun name ->
        (name, scalar_float (Device.with_device ords.(0) (fun () -> B.download (List.assoc name per_dev.(0)))) /. float_of_int n))
      names
  in
  Array.iteri (fun i d -> Device.with_device d (fun () -> List.iter (fun (_, r) -> B.free_resident r) per_dev.(i))) ords;
  result
