(* Wire.to_wire: a Graph.t as the text libccb.so's ccb_program_create and
   ccb_program_lower parse (include/ccb.h; the format is documented in
   cudacaml_b200/wire.py, whose printer this one matches line for line).

   NOT BUILT HERE: the build image has no OCaml toolchain. This is the module
   a maintainer adds as lib/backend_cuda/wire.ml, next to the reference's
   Emit, written against the reference's own IR (lib/ir/expr.ml,
   lib/ir/tensor.ml, lib/ir/graph.mli). The Python printer is exercised by
   every test of this repository; this one prints the same lines for the same
   graph (names may differ only in which non-ASCII characters are escaped,
   and both spellings decode to the same name).

   Layout of the text:
     ccbgraph 1
     name <graph name>
     opt matmul tf32                      only when allow_tf32 is set
     opt shard <rank> <world>             only for ~shard:(rank, world) with world > 1
     e <eid> <dtype> <expression node>    post-order, each shared node once
     t <tid> <dtype> <rank> <dims> <kind> <operands>   Graph.topological_order
     o <output name> <tid>                Graph.outputs order
     end *)

open Cudacaml_ir

(* F32 products on the tcgen05 tensor cores (TF32 operands, F32
   accumulation) when set; the reference's F32 arithmetic otherwise. *)
let allow_tf32 = ref false

let dt (type a) (d : a Dtype.t) = Dtype.name d

let binop_name : Expr.binop -> string = function
  | Expr.Add -> "add"
  | Expr.Sub -> "sub"
  | Expr.Mul -> "mul"
  | Expr.Div -> "div"
  | Expr.Min -> "min"
  | Expr.Max -> "max"
  | Expr.Bit_and -> "bit_and"
  | Expr.Bit_or -> "bit_or"
  | Expr.Bit_xor -> "bit_xor"
  | Expr.Shl -> "shl"
  | Expr.Shr -> "shr"

let unop_name : Expr.unop -> string = function
  | Expr.Neg -> "neg"
  | Expr.Sqrt -> "sqrt"
  | Expr.Exp -> "exp"
  | Expr.Log -> "log"
  | Expr.Abs -> "abs"
  | Expr.Sin -> "sin"
  | Expr.Cos -> "cos"
  | Expr.Erf -> "erf"
  | Expr.Erfinv -> "erfinv"

let cmp_name : Expr.cmp -> string = function
  | Expr.Eq -> "eq"
  | Expr.Ne -> "ne"
  | Expr.Lt -> "lt"
  | Expr.Le -> "le"
  | Expr.Gt -> "gt"
  | Expr.Ge -> "ge"

let logic_name : Expr.logic -> string = function Expr.And -> "and" | Expr.Or -> "or"

(* Names are one token: '%', whitespace and control bytes as %XX (per byte,
   so UTF-8 passes through unchanged), the empty name as a lone %. *)
let wire_name n =
  if n = "" then "%"
  else begin
    let b = Buffer.create (String.length n + 8) in
    String.iter
      (fun c ->
        let k = Char.code c in
        if c = '%' || c = ' ' || c = '\t' || c = '\n' || c = '\r' || c = '\011' || c = '\012' || k < 0x20
           || k = 0x7f
        then Printf.bprintf b "%%%02X" k
        else Buffer.add_char b c)
      n;
    Buffer.contents b
  end

(* Float constants travel as the bits of the OCaml float (an IEEE double),
   F32 ones included: the receiver rounds to F32 exactly as Emit's literals
   do. *)
let const_text : type a. a Dtype.t -> a -> string =
 fun d v ->
  match d with
  | Dtype.F32 -> Printf.sprintf "%016Lx" (Int64.bits_of_float v)
  | Dtype.F64 -> Printf.sprintf "%016Lx" (Int64.bits_of_float v)
  | Dtype.I32 -> Int32.to_string v
  | Dtype.I64 -> Int64.to_string v
  | Dtype.Bool -> if v then "1" else "0"

let to_wire ?shard (g : Graph.t) : string =
  let b = Buffer.create 8192 in
  let line fmt = Printf.kbprintf (fun b -> Buffer.add_char b '\n') b fmt in
  let seen : (int, unit) Hashtbl.t = Hashtbl.create 1024 in
  let eid (e : _ Expr.t) = Uid.to_int e.Expr.uid in
  (* Post-order, each shared node once (the [seen] table); the recursion is
     as deep as the expression, a few hundred nodes for Philox-10. *)
  let rec ex : type a. a Expr.t -> unit =
   fun e ->
    if not (Hashtbl.mem seen (eid e)) then begin
      let id = eid e and d = dt e.Expr.dtype in
      (match e.Expr.node with
      | Expr.Const v -> line "e %d %s const %s" id d (const_text e.Expr.dtype v)
      | Expr.Arg i -> line "e %d %s arg %d" id d i
      | Expr.Index -> line "e %d i32 index" id
      | Expr.Binop (op, x, y) ->
          ex x;
          ex y;
          line "e %d %s binop %s %d %d" id d (binop_name op) (eid x) (eid y)
      | Expr.Unop (op, x) ->
          ex x;
          line "e %d %s unop %s %d" id d (unop_name op) (eid x)
      | Expr.Cmp (op, x, y) ->
          ex x;
          ex y;
          line "e %d bool cmp %s %d %d" id (cmp_name op) (eid x) (eid y)
      | Expr.Logic (op, x, y) ->
          ex x;
          ex y;
          line "e %d bool logic %s %d %d" id (logic_name op) (eid x) (eid y)
      | Expr.Not x ->
          ex x;
          line "e %d bool not %d" id (eid x)
      | Expr.Select (c, x, y) ->
          ex c;
          ex x;
          ex y;
          line "e %d %s select %d %d %d" id d (eid c) (eid x) (eid y)
      | Expr.Cast (x, _) ->
          ex x;
          line "e %d %s cast %d" id d (eid x));
      Hashtbl.replace seen id ()
    end
  in
  let tid (Tensor.P t) = Uid.to_int t.Tensor.uid in
  let head (Tensor.P t) =
    let dims = Shape.dims t.Tensor.shape in
    Printf.sprintf "t %d %s %d%s" (Uid.to_int t.Tensor.uid) (dt t.Tensor.dtype) (List.length dims)
      (String.concat "" (List.map (fun k -> " " ^ string_of_int k) dims))
  in
  let tensor (Tensor.P t as p) =
    let h = head p in
    match t.Tensor.node with
    | Tensor.Param n -> line "%s param %s" h (wire_name n)
    | Tensor.Iota -> line "%s iota" h
    | Tensor.Map (f, a) ->
        ex f.Expr.arg1;
        ex f.Expr.body1;
        line "%s map %d %d %d" h (tid (Tensor.P a)) (eid f.Expr.arg1) (eid f.Expr.body1)
    | Tensor.Map2 (f, a, c) ->
        ex f.Expr.arg_a;
        ex f.Expr.arg_b;
        ex f.Expr.body2;
        line "%s map2 %d %d %d %d %d" h (tid (Tensor.P a)) (tid (Tensor.P c)) (eid f.Expr.arg_a)
          (eid f.Expr.arg_b) (eid f.Expr.body2)
    | Tensor.Reduce (f, init, a) ->
        ex f.Expr.arg_a;
        ex f.Expr.arg_b;
        ex f.Expr.body2;
        ex init;
        line "%s reduce %d %d %d %d %d" h (tid (Tensor.P a)) (eid f.Expr.arg_a) (eid f.Expr.arg_b)
          (eid f.Expr.body2) (eid init)
    | Tensor.Scan (f, init, a) ->
        ex f.Expr.arg_a;
        ex f.Expr.arg_b;
        ex f.Expr.body2;
        ex init;
        line "%s scan %d %d %d %d %d" h (tid (Tensor.P a)) (eid f.Expr.arg_a) (eid f.Expr.arg_b)
          (eid f.Expr.body2) (eid init)
    | Tensor.Gather (i, a) -> line "%s gather %d %d" h (tid (Tensor.P i)) (tid (Tensor.P a))
    | Tensor.Scatter_add (i, a, _) -> line "%s scatter_add %d %d" h (tid (Tensor.P i)) (tid (Tensor.P a))
    | Tensor.Matmul (a, c) -> line "%s matmul %d %d" h (tid (Tensor.P a)) (tid (Tensor.P c))
    | Tensor.Reshape (_, a) -> line "%s reshape %d" h (tid (Tensor.P a))
    | Tensor.Broadcast (_, a) -> line "%s broadcast %d" h (tid (Tensor.P a))
  in
  line "ccbgraph 1";
  line "name %s" (wire_name (Graph.name g));
  if !allow_tf32 then line "opt matmul tf32";
  (match shard with Some (r, w) when w > 1 -> line "opt shard %d %d" r w | _ -> ());
  List.iter tensor (Graph.topological_order g);
  List.iter (fun (n, p) -> line "o %s %d" (wire_name n) (tid p)) (Graph.outputs g);
  line "end";
  Buffer.contents b
