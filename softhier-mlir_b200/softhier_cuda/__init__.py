"""Host side of the B200 softhier-ops library.

  lib        ctypes binding of libsh_ops_cuda.so (include/sh_ops.h + include/sh_ops_cuda.h)
  runtime    device arena / stream plumbing (torch allocates, the library computes)
  dialect    parser for the softhier dialect text the reference frontends emit
  emit_cuda  lowering of a dialect module to one library call per op (C source or an in-process program)
  encoder    batched SigLIP encoder driver (data-parallel across GPUs) on the C ABI
  summa      2-D block-distributed SUMMA GEMM across GPUs (NCCL panel broadcasts + the tcgen05 GEMM)
"""
