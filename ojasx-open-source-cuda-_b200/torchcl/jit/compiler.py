"""Elementwise fusion — the reference's JITCompiler (torchcl/jit/compiler.py:55-231).

The reference generates OpenCL source for `out[i] = u_n(...u_1(a[i] op b[i]))`
and compiles it at run time.  On B200 the same expression is evaluated by one
ahead-of-time sm_100a kernel (ojx_elementwise) driven by an op-code list, and the
GEMM-adjacent case (a lazy matmul followed by add/sub/mul/div and unary ops) never
reaches this module: api.py folds it into the GEMM's epilogue.

Supported op names and formulas are the reference's (_UNARY_OPS / _BINARY_OPS).
Buffers are device addresses (CLBuffer.buffer); dtypes default to float32.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from torchcl import _lib as L
from torchcl.jit.cache import get_kernel_cache
from torchcl.ops.engine import ojx_dtype
from torchcl.runtime.context import get_queue

# Formulas, for reference; the device code in csrc/epilogue.cuh implements them.
_UNARY_OPS = {
    "relu": "fmax(x, 0)", "sigmoid": "1 / (1 + exp(-x))", "tanh": "tanh(x)", "neg": "-x",
    "abs": "fabs(x)", "exp": "exp(x)", "log": "log(x)", "sqrt": "sqrt(x)",
    "silu": "x / (1 + exp(-x))",
    "gelu": "x * 0.5 * (1 + tanh(0.7978845608 * (x + 0.044715 * x * x * x)))",
    "square": "x * x",
}
_BINARY_OPS = {"add": "a + b", "sub": "a - b", "mul": "a * b", "div": "a / b"}


def _build_plan(chain):
    """(binary op or None, unary names) -> (ctypes op-code array, number of unary ops)."""
    _, ops = chain
    for op in ops:
        if op not in _UNARY_OPS:
            raise ValueError(f"Unknown unary op for fusion: {op}")
    if len(ops) > L.MAX_UNARY:
        raise ValueError(f"at most {L.MAX_UNARY} fused unary ops")
    codes = [L.UNARY[o] for o in ops]
    return (ctypes.c_int32 * max(1, len(codes)))(*codes), len(codes)


class JITCompiler:
    def __init__(self) -> None:
        self._cache = get_kernel_cache()

    def _plan(self, binary_op, ops: Sequence[str]):
        return self._cache.plan_for((binary_op, tuple(ops)), _build_plan)

    def fuse_elementwise_chain(self, ops: Sequence[str], n: int, input_buffers: list,
                               output_buffer, dtypes=(torch.float32, torch.float32)) -> None:
        """out[i] = ops[-1](...ops[0](in[i])) (compiler.py:64-97)."""
        codes, n_codes = self._plan(None, ops)
        din, dout = dtypes
        L.check(L.lib().ojx_elementwise(int(output_buffer), ojx_dtype(dout), int(input_buffers[0]),
                                        ojx_dtype(din), None, 0, 0, codes, n_codes, int(n),
                                        get_queue()), "fuse_elementwise_chain")

    def fuse_binary_then_unary(self, binary_op: str, unary_ops: Sequence[str], n: int, a_buf,
                               b_buf, out_buf,
                               dtypes=(torch.float32, torch.float32, torch.float32)) -> None:
        """out[i] = unary_ops(a[i] binary_op b[i]) (compiler.py:99-133)."""
        if binary_op not in _BINARY_OPS:
            raise ValueError(f"Unknown binary op for fusion: {binary_op}")
        codes, n_codes = self._plan(binary_op, unary_ops)
        da, db, dout = dtypes
        L.check(L.lib().ojx_elementwise(int(out_buf), ojx_dtype(dout), int(a_buf), ojx_dtype(da),
                                        int(b_buf), ojx_dtype(db), L.BINARY[binary_op], codes,
                                        n_codes, int(n), get_queue()), "fuse_binary_then_unary")


_global_jit: JITCompiler | None = None


def get_jit_compiler() -> JITCompiler:
    global _global_jit
    if _global_jit is None:
        _global_jit = JITCompiler()
    return _global_jit
