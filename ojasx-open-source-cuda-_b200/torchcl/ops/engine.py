"""Compute engine — replaces torchcl/ops/engine.py (OpenCLEngine) for the GEMM
hot path.  Kernel selection and launch geometry live in libojx (ojx_gemm picks
the tcgen05 tile GEMM, the 3xTF32 GEMM, the skinny split-K GEMM or the SIMT GEMM);
this class converts tensors to buffers and fills the GEMM descriptor.

Method names and arguments follow the reference (engine.py:46-83, 156-255,
332-392) so existing callers keep working.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from torchcl import _lib as L
from torchcl.runtime.context import get_queue
from torchcl.runtime.memory import CLBuffer, get_buffer_pool, note_use

_TORCH_TO_OJX = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16}
_OJX_TO_TORCH = {v: k for k, v in _TORCH_TO_OJX.items()}
_ITEMSIZE = {L.F32: 4, L.BF16: 2, L.F16: 2}


def ojx_dtype(dt) -> int:
    """ojx dtype code of a torch dtype, numpy dtype or None (fp32)."""
    if dt is None:
        return L.F32
    if isinstance(dt, torch.dtype):
        if dt not in _TORCH_TO_OJX:
            raise ValueError(f"unsupported dtype {dt}; the GEMM path takes float32, bfloat16, float16")
        return _TORCH_TO_OJX[dt]
    nd = np.dtype(dt)
    if nd == np.float32:
        return L.F32
    if nd == np.float16:
        return L.F16
    raise ValueError(f"unsupported dtype {dt}")


def torch_dtype(code: int) -> torch.dtype:
    return _OJX_TO_TORCH[code]


def _unary_codes(ops) -> list[int]:
    codes = []
    for op in ops or ():
        if op not in L.UNARY:
            raise ValueError(f"Unknown unary op for fusion: {op}")
        codes.append(L.UNARY[op])
    if len(codes) > L.MAX_UNARY:
        raise ValueError(f"at most {L.MAX_UNARY} fused unary ops")
    return codes


class OpenCLEngine:
    """Tensor <-> buffer conversion and kernel launches on the current stream."""

    def __init__(self) -> None:
        self._pool = get_buffer_pool()
        self.last_route = None

    # ── tensor <-> buffer ────────────────────────────────────────────
    def tensor_to_buffer(self, tensor: torch.Tensor) -> CLBuffer:
        t = tensor.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        t = t.contiguous()
        ojx_dtype(t.dtype)
        return self._pool.host_to_device(t)

    def buffer_to_tensor(self, cl_buf: CLBuffer, shape: tuple, dtype: torch.dtype = torch.float32
                         ) -> torch.Tensor:
        out = torch.empty(tuple(shape), dtype=dtype)
        nbytes = out.numel() * out.element_size()
        if nbytes:
            self._pool.copy_to_host(cl_buf, out.data_ptr(), nbytes)
        return out

    def allocate_output(self, shape: tuple, dtype=torch.float32) -> CLBuffer:
        numel = math.prod(int(d) for d in shape) if shape else 1
        code = ojx_dtype(dtype)
        return self._pool.allocate(numel * _ITEMSIZE[code], dtype, tuple(shape))

    def free_buffer(self, cl_buf: CLBuffer) -> None:
        self._pool.free(cl_buf)

    # ── GEMM ─────────────────────────────────────────────────────────
    def gemm(self, a_buf, b_buf, out_buf, M: int, N: int, K: int, *, dtype_a=None, dtype_b=None,
             dtype_c=None, trans_a=False, trans_b=False, lda=0, ldb=0, ldc=0, operand=None,
             operand_kind=None, operand_dtype=None, ld_operand=0, binary="add",
             operand_is_lhs=False, unary=(), fp32_mode=L.FP32_AUTO, flags=0, stream=None,
             batch=None, stride_a=0, stride_b=0, stride_c=0, stride_operand=0) -> str:
        """One fused GEMM: out = unary(...(bin(op(A) @ op(B), operand))).  With `batch`,
        `batch` problems whose operands are stride_* elements apart (ojx_gemm_batched)."""
        d = self._desc(a_buf, b_buf, out_buf, M, N, K, dtype_a=dtype_a, dtype_b=dtype_b,
                       dtype_c=dtype_c, trans_a=trans_a, trans_b=trans_b, lda=lda, ldb=ldb,
                       ldc=ldc, operand=operand, operand_kind=operand_kind,
                       operand_dtype=operand_dtype, ld_operand=ld_operand, binary=binary,
                       operand_is_lhs=operand_is_lhs, unary=unary, fp32_mode=fp32_mode,
                       flags=flags)
        q = get_queue() if stream is None else stream
        lib = L.lib()
        if batch is None:
            L.check(lib.ojx_gemm(ctypes.byref(d), q), "gemm")
        else:
            L.check(lib.ojx_gemm_batched(ctypes.byref(d), int(batch), int(stride_a), int(stride_b),
                                         int(stride_c), int(stride_operand), q), "gemm_batched")
        self.last_route = L.ROUTES.get(lib.ojx_last_route(), "?")
        return self.last_route

    def gemm_host_io(self, host_a: int, b_buf, host_c: int, dev_a, dev_c, M: int, N: int, K: int,
                     **kw) -> str:
        """The same fused GEMM with A and C in (pinned) host memory: ojx_gemm_host_io
        uploads A in row chunks into dev_a, runs each chunk's GEMM into dev_c and
        downloads it to host_c while the next chunk uploads, all ordered after the
        work already queued on the current stream.  Returns the route."""
        d = self._desc(host_a, b_buf, host_c, M, N, K, **kw)
        lib = L.lib()
        L.check(lib.ojx_gemm_host_io(ctypes.byref(d), _addr(dev_a), _addr(dev_c), 0, get_queue()),
                "gemm_host_io")
        self.last_route = L.ROUTES.get(lib.ojx_last_route(), "?")
        return self.last_route

    def _desc(self, a_buf, b_buf, out_buf, M: int, N: int, K: int, *, dtype_a=None, dtype_b=None,
              dtype_c=None, trans_a=False, trans_b=False, lda=0, ldb=0, ldc=0, operand=None,
              operand_kind=None, operand_dtype=None, ld_operand=0, binary="add",
              operand_is_lhs=False, unary=(), fp32_mode=L.FP32_AUTO, flags=0) -> L.GemmDesc:
        d = L.GemmDesc()
        d.M, d.N, d.K = int(M), int(N), int(K)
        d.dtype_a = ojx_dtype(dtype_a if dtype_a is not None else getattr(a_buf, "dtype", None))
        d.dtype_b = ojx_dtype(dtype_b if dtype_b is not None else getattr(b_buf, "dtype", None))
        d.dtype_c = ojx_dtype(dtype_c if dtype_c is not None else getattr(out_buf, "dtype", None))
        d.trans_a, d.trans_b = int(bool(trans_a)), int(bool(trans_b))
        d.lda, d.ldb, d.ldc = int(lda), int(ldb), int(ldc)
        d.a = _addr(a_buf)
        d.b = _addr(b_buf)
        d.c = _addr(out_buf)
        if operand is not None and operand_kind is not None:
            d.operand = _addr(operand)
            d.operand_kind = {"row": L.OPERAND_ROW, "full": L.OPERAND_FULL}[operand_kind]
            d.dtype_operand = ojx_dtype(operand_dtype if operand_dtype is not None
                                        else getattr(operand, "dtype", None))
            d.ld_operand = int(ld_operand)
            if binary not in L.BINARY:
                raise ValueError(f"Unknown binary op for fusion: {binary}")
            d.binary_op = L.BINARY[binary]
            d.operand_is_lhs = int(bool(operand_is_lhs))
        codes = _unary_codes(unary)
        d.n_unary = len(codes)
        for i, c in enumerate(codes):
            d.unary[i] = c
        d.fp32_mode = int(fp32_mode)
        d.flags = int(flags)
        return d

    def run_matmul(self, a_buf, b_buf, out_buf, M, N, K, use_tiled: bool = True) -> None:
        """C[M,N] = A[M,K] @ B[K,N] (engine.py:156-185)."""
        self.gemm(a_buf, b_buf, out_buf, M, N, K)

    def run_matmul_bias(self, a_buf, b_buf, bias_buf, out_buf, M, N, K) -> None:
        """C = A @ B + bias[N] with the bias fused into the store (engine.py:187-215)."""
        self.gemm(a_buf, b_buf, out_buf, M, N, K, operand=bias_buf, operand_kind="row")

    def run_matmul_fp16(self, a_buf, b_buf, out_buf, M, N, K, use_tiled: bool = True) -> None:
        """Half operands, fp32 accumulate, half result (engine.py:217-255)."""
        self.gemm(a_buf, b_buf, out_buf, M, N, K, dtype_a=torch.float16, dtype_b=torch.float16,
                  dtype_c=torch.float16)

    def run_linear(self, a_buf, b_buf, bias_buf, out_buf, M, N, K, use_tiled: bool = True) -> None:
        """C[M,N] = A[M,K] @ B[N,K]^T (+ bias[N]) (engine.py:351-392), B read transposed in place."""
        self.gemm(a_buf, b_buf, out_buf, M, N, K, trans_b=True,
                  operand=bias_buf, operand_kind="row" if bias_buf is not None else None)

    def run_transpose(self, a_buf, out_buf, M, N, dtype=None) -> None:
        """out[N,M] = a[M,N]^T (engine.py:332-349)."""
        code = ojx_dtype(dtype if dtype is not None else getattr(a_buf, "dtype", None))
        L.check(L.lib().ojx_transpose(_addr(out_buf), _addr(a_buf), int(M), int(N), code,
                                      get_queue()), "transpose")

    def run_fill(self, out_buf, value: float, n: int, dtype=None) -> None:
        code = ojx_dtype(dtype if dtype is not None else getattr(out_buf, "dtype", None))
        L.check(L.lib().ojx_fill(_addr(out_buf), float(value), int(n), code, get_queue()), "fill")

    def run_cast(self, out_buf, dtype_out, in_buf, dtype_in, n: int) -> None:
        L.check(L.lib().ojx_cast(_addr(out_buf), ojx_dtype(dtype_out), _addr(in_buf),
                                 ojx_dtype(dtype_in), int(n), get_queue()), "cast")

    def run_fused_attention(self, Q, K, V, Out, B: int, H: int, M: int, N: int, D: int,
                            scale: float, is_causal: bool = False, dtype=None,
                            max_keys: int = 0, composed: bool = False) -> str:
        """Out = softmax(scale * Q K^T) V per (batch, head) (engine.py:755-773): one
        fused tcgen05 kernel for bf16/fp16 with head dim 64/128, else two batched
        GEMMs around a row-softmax kernel.  Returns the route."""
        code = ojx_dtype(dtype if dtype is not None else getattr(Q, "dtype", None))
        L.check(L.lib().ojx_attention(_addr(Out), _addr(Q), _addr(K), _addr(V), code, int(B), int(H),
                                      int(M), int(N), int(D), float(scale), int(bool(is_causal)),
                                      int(max_keys), L.ATTN_FLAG_COMPOSED if composed else 0,
                                      get_queue()), "fused_attention")
        self.last_route = L.ROUTES.get(L.lib().ojx_last_route(), "?")
        return self.last_route

    def run_sum_columns(self, input_buf, out_buf, rows: int, cols: int, dtype_in=None,
                        dtype_out=None) -> None:
        """out[cols] = input[rows, cols].sum(0) in fp32 (engine.py:807-822)."""
        L.check(L.lib().ojx_sum_columns(
            _addr(out_buf), ojx_dtype(dtype_out if dtype_out is not None else getattr(out_buf, "dtype", None)),
            _addr(input_buf), ojx_dtype(dtype_in if dtype_in is not None else getattr(input_buf, "dtype", None)),
            int(rows), int(cols), 0, get_queue()), "sum_columns")

    def run_elementwise(self, out_buf, a_buf, b_buf, binary, unary, n: int, dtype_out=None,
                        dtype_a=None, dtype_b=None) -> None:
        """out[i] = unary(...(a[i] op b[i])) — the JIT's fused elementwise kernel."""
        codes = _unary_codes(unary)
        arr = (ctypes.c_int32 * max(1, len(codes)))(*codes)
        if b_buf is not None and binary not in L.BINARY:
            raise ValueError(f"Unknown binary op for fusion: {binary}")
        L.check(L.lib().ojx_elementwise(
            _addr(out_buf), ojx_dtype(dtype_out if dtype_out is not None else getattr(out_buf, "dtype", None)),
            _addr(a_buf), ojx_dtype(dtype_a if dtype_a is not None else getattr(a_buf, "dtype", None)),
            _addr(b_buf) if b_buf is not None else None,
            ojx_dtype(dtype_b if dtype_b is not None else getattr(b_buf, "dtype", None)) if b_buf is not None else 0,
            L.BINARY[binary] if b_buf is not None else 0, arr, len(codes), int(n), get_queue()),
            "elementwise")


def _addr(buf) -> int | None:
    if buf is None:
        return None
    if isinstance(buf, CLBuffer):
        note_use(buf)  # a graph being captured must keep this buffer
        return buf.buffer
    return int(buf)


_global_engine: OpenCLEngine | None = None


def get_engine() -> OpenCLEngine:
    global _global_engine
    if _global_engine is None:
        _global_engine = OpenCLEngine()
    return _global_engine
