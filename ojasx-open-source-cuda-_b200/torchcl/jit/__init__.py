"""Fusion front end (the reference's torchcl.jit)."""
