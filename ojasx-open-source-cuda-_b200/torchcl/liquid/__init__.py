"""Dispatch decisions of the reference's torchcl.liquid package, reduced to the
one the GEMM path needs (which precision a matmul runs in)."""
