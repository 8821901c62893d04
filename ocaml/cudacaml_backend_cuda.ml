(* Cudacaml_backend_cuda over libccb.so, behind the reference's unchanged
   signature (lib/backend_cuda/cudacaml_backend_cuda.mli:6-84).

   NOT BUILT HERE: the build image has no OCaml toolchain. This file replaces
   lib/backend_cuda/cudacaml_backend_cuda.ml; everything it exports comes from
   Program (compile, run, source, release, compile_with, compile_on,
   device_of, run_async/wait, resident/upload/download/free_resident,
   run_resident) and Multi.

   One value of the .mli has no meaning any more: [executor] (the reference's
   Kernel_ir-plan executor) raises Invalid_argument. [Emit], [Mangle] and
   [Executor] stay exported, unchanged, for tooling that prints the
   reference's own kernels; nothing on the compile or run path uses them. *)

include Program
module Emit = Emit
module Mangle = Mangle
module Executor = Executor
module Multi = Multi

let executor _ =
  invalid_arg "Backend_cuda.executor: libccb.so runs whole programs; there is no Kernel_ir executor"
