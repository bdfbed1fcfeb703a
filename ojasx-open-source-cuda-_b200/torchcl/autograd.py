"""Autograd functions of the GEMM path — replaces MatmulFunction and
LinearFunction of torchcl/autograd.py (:277-314, :355-412).

Same classes, `apply` signatures and saved state.  What changes is the backward:
the reference materialises B^T, A^T and grad_output^T with transpose kernels
(autograd.py:301-311, 396-401) before running plain GEMMs; here every gradient
is ONE GEMM that reads the stored operand transposed through its descriptor
(op(A) / op(B) flags of ojx_gemm), and the bias gradient is ojx_sum_columns.

    forward  Matmul   C  = A @ B                       one GEMM
    backward Matmul   dA = dC @ B^T      (B read transposed)
                      dB = A^T @ dC      (A read transposed)
    forward  Linear   Y  = X @ W^T + b                 one GEMM, bias in the epilogue
    backward Linear   dX = dY @ W
                      dW = dY^T @ X      (dY read transposed)
                      db = dY.sum(0)     (column sums, fp32 accumulation)

Tensors keep their dtype (float32 via 3xTF32, bfloat16 / float16 via the tcgen05
f16 kernel; gradients of bf16 tensors are bf16).  Inputs may be device handles or
CPU tensors (uploaded).  The reference's other autograd functions (activations,
layer norm, cross entropy, convolution) are outside the GEMM path this package
replaces.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from torchcl.api import _get_buf, _get_dtype, _get_shape, _wrap_output, is_opencl_tensor, to_opencl
from torchcl.ops.engine import get_engine


def _dev(t):
    return t if is_opencl_tensor(t) else to_opencl(t)


def _alloc(shape: tuple, dtype: torch.dtype = torch.float32):
    """Allocate a device buffer and its handle (autograd.py:33-38)."""
    engine = get_engine()
    buf = engine.allocate_output(shape, dtype)
    return _wrap_output(buf, shape, dtype), buf


class MatmulFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        a, b = _dev(a), _dev(b)
        (M, K), (K2, N) = _get_shape(a), _get_shape(b)
        if K != K2:
            raise ValueError(f"matmul dimension mismatch: {(M, K)} @ {(K2, N)}")
        dt = _get_dtype(a)
        out, out_buf = _alloc((M, N), dt)
        get_engine().gemm(_get_buf(a), _get_buf(b), out_buf, M, N, K, dtype_a=dt,
                          dtype_b=_get_dtype(b), dtype_c=dt)
        ctx.save_for_backward(a, b)
        ctx._M, ctx._N, ctx._K = M, N, K
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        a, b = ctx.saved_tensors
        g = _dev(grad_output)
        M, N, K = ctx._M, ctx._N, ctx._K
        eng = get_engine()
        da_t, db_t, dg = _get_dtype(a), _get_dtype(b), _get_dtype(g)
        # dA[M, K] = dC[M, N] @ B^T  (B stored [K, N]: read as op(B) = B^T)
        grad_a, ga_buf = _alloc((M, K), da_t)
        eng.gemm(_get_buf(g), _get_buf(b), ga_buf, M, K, N, dtype_a=dg, dtype_b=db_t,
                 dtype_c=da_t, trans_b=True)
        # dB[K, N] = A^T @ dC  (A stored [M, K]: read as op(A) = A^T)
        grad_b, gb_buf = _alloc((K, N), db_t)
        eng.gemm(_get_buf(a), _get_buf(g), gb_buf, K, N, M, dtype_a=da_t, dtype_b=dg,
                 dtype_c=db_t, trans_a=True)
        return grad_a, grad_b


class LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor,
                bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        x, weight = _dev(x), _dev(weight)
        if bias is not None:
            bias = _dev(bias)
        x_shape, w_shape = _get_shape(x), _get_shape(weight)
        K = int(x_shape[-1])
        M = int(math.prod(x_shape[:-1])) if len(x_shape) > 1 else 1
        N, K2 = int(w_shape[0]), int(w_shape[1])
        if K != K2:
            raise ValueError(f"Linear dimension mismatch: input {x_shape}, weight {w_shape}")
        dt = _get_dtype(x)
        out_shape = tuple(x_shape[:-1]) + (N,)
        out, out_buf = _alloc(out_shape, dt)
        get_engine().gemm(_get_buf(x), _get_buf(weight), out_buf, M, N, K, dtype_a=dt,
                          dtype_b=_get_dtype(weight), dtype_c=dt, trans_b=True,
                          operand=_get_buf(bias) if bias is not None else None,
                          operand_kind="row" if bias is not None else None,
                          operand_dtype=_get_dtype(bias) if bias is not None else None)
        ctx.save_for_backward(x, weight, bias)
        ctx._x_shape = x_shape
        ctx._M, ctx._N, ctx._K = M, N, K
        ctx._has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, weight, bias = ctx.saved_tensors
        g = _dev(grad_output)
        M, N, K = ctx._M, ctx._N, ctx._K
        eng = get_engine()
        dx_t, dw_t, dg = _get_dtype(x), _get_dtype(weight), _get_dtype(g)
        # dX[M, K] = dY[M, N] @ W[N, K]
        grad_x, gx_buf = _alloc(ctx._x_shape, dx_t)
        eng.gemm(_get_buf(g), _get_buf(weight), gx_buf, M, K, N, dtype_a=dg, dtype_b=dw_t,
                 dtype_c=dx_t)
        # dW[N, K] = dY^T @ X  (dY stored [M, N]: read as op(A) = dY^T)
        grad_w, gw_buf = _alloc((N, K), dw_t)
        eng.gemm(_get_buf(g), _get_buf(x), gw_buf, N, K, M, dtype_a=dg, dtype_b=dx_t,
                 dtype_c=dw_t, trans_a=True)
        grad_bias = None
        if ctx._has_bias:
            db_t = _get_dtype(bias)
            grad_bias, gb_buf = _alloc((N,), db_t)
            eng.run_sum_columns(_get_buf(g), gb_buf, M, N, dtype_in=dg, dtype_out=db_t)
        return grad_x, grad_w, grad_bias


__all__ = ["MatmulFunction", "LinearFunction"]
