"""Kernel launchers (the reference's torchcl.ops)."""
