"""Shared helpers of the GPU parity tests: run one fused GEMM through libojx's
C-ABI (torchcl.ops.engine -> ojx_gemm) on host inputs, and the matching oracle call."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

CODES = {torch.float32: O.F32, torch.bfloat16: O.BF16, torch.float16: O.F16}


def host_bits(t: torch.Tensor) -> np.ndarray:
    """Host array the oracle reads: float32 values, or 16-bit patterns for bf16/fp16."""
    t = t.contiguous()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def as_f32(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.float32:
        return x
    if dtype == torch.bfloat16:
        return O.bf16_to_f32(x)
    return x.view(np.float16).astype(np.float32)


def randn(seed: int, shape, dtype=torch.float32, scale=1.0, uniform=False) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    if uniform:
        t = torch.rand(*shape, generator=g) * 2 - 1
    else:
        t = torch.randn(*shape, generator=g)
    return (t * scale).to(dtype)


def run_gemm(A, B, *, trans_a=False, trans_b=False, operand=None, kind=None, binary="add",
             lhs=False, unary=(), fp32_mode=0, flags=0, out_dtype=None):
    """(C as a CPU tensor, route name) for epilogue(op(A) @ op(B)) on the device."""
    from torchcl.ops.engine import get_engine
    eng = get_engine()
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    out_dtype = out_dtype or A.dtype
    a_buf, b_buf = eng.tensor_to_buffer(A), eng.tensor_to_buffer(B)
    op_buf = eng.tensor_to_buffer(operand) if operand is not None else None
    out = eng.allocate_output((M, N), out_dtype)
    try:
        route = eng.gemm(a_buf, b_buf, out, M, N, K, dtype_a=A.dtype, dtype_b=B.dtype,
                         dtype_c=out_dtype, trans_a=trans_a, trans_b=trans_b, operand=op_buf,
                         operand_kind=kind, operand_dtype=operand.dtype if operand is not None else None,
                         binary=binary, operand_is_lhs=lhs, unary=unary, fp32_mode=fp32_mode,
                         flags=flags)
        C = eng.buffer_to_tensor(out, (M, N), out_dtype)
    finally:
        for b in (a_buf, b_buf, op_buf, out):
            if b is not None:
                eng.free_buffer(b)
    return C, route


def oracle_gemm(A, B, *, trans_a=False, trans_b=False, operand=None, kind=None, binary="add",
                lhs=False, unary=(), out_dtype=None, fused=False, rows=None):
    out_dtype = out_dtype or A.dtype
    C = O.gemm(host_bits(A), host_bits(B), dtype_a=CODES[A.dtype], dtype_b=CODES[B.dtype],
               dtype_c=CODES[out_dtype], trans_a=trans_a, trans_b=trans_b,
               operand=host_bits(operand) if operand is not None else None, operand_kind=kind,
               operand_dtype=CODES[operand.dtype] if operand is not None else O.F32,
               binary=binary, operand_is_lhs=lhs, unary=unary, fused=fused, rows=rows)
    return as_f32(C, out_dtype)


def oracle_cols(A, B, cols, *, trans_a=False, trans_b=False, operand=None, kind=None,
                binary="add", unary=(), out_dtype=None):
    out_dtype = out_dtype or A.dtype
    C = O.gemm_cols(host_bits(A), host_bits(B), cols, dtype_a=CODES[A.dtype],
                    dtype_b=CODES[B.dtype], dtype_c=CODES[out_dtype], trans_a=trans_a,
                    trans_b=trans_b, operand=host_bits(operand) if operand is not None else None,
                    operand_kind=kind,
                    operand_dtype=CODES[operand.dtype] if operand is not None else O.F32,
                    binary=binary, unary=unary)
    return as_f32(C, out_dtype)


def rel_l2(x, ref) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-30))


def assert_fp32_parity(C, ref, A, B, trans_a=False, trans_b=False):
    """north_star fp32 bar: rel-L2 <= 1e-5 and max-abs <= 1e-4 * ||A||_F ||B||_F / sqrt(M N)."""
    M = A.shape[1] if trans_a else A.shape[0]
    N = B.shape[0] if trans_b else B.shape[1]
    scale = float(A.double().norm() * B.double().norm()) / np.sqrt(M * N)
    C = np.asarray(C, dtype=np.float64)
    r = rel_l2(C, ref)
    m = float(np.abs(C - ref).max()) if C.size else 0.0
    assert r <= 1e-5, f"rel-L2 {r:.3e} > 1e-5"
    assert m <= 1e-4 * scale, f"max-abs {m:.3e} > 1e-4 * {scale:.3e}"
    return r, m


def assert_half_parity(C, ref, tol=1e-2):
    """north_star bf16/fp16 bar: rel-L2 <= 1e-2 against the fp32-accumulating oracle."""
    r = rel_l2(C, ref)
    assert r <= tol, f"rel-L2 {r:.3e} > {tol}"
    return r


# ── device-resident operands (the BASELINE-size parity tests) ──────────────────

def device_gemm(A, B, C, *, trans_a=False, trans_b=False, bias=None, unary=(), fp32_mode=0,
                flags=0) -> str:
    """C = unary(op(A) @ op(B) + bias[N]) through ojx_gemm on torch CUDA tensors, on
    torch's current stream; returns the route the library took."""
    import ctypes
    from torchcl import _lib as L
    lib = L.lib()
    code = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16}
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    d = L.GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.dtype_a, d.dtype_b, d.dtype_c = code[A.dtype], code[B.dtype], code[C.dtype]
    d.trans_a, d.trans_b = int(trans_a), int(trans_b)
    d.a, d.b, d.c = A.data_ptr(), B.data_ptr(), C.data_ptr()
    if bias is not None:
        d.operand, d.dtype_operand = bias.data_ptr(), code[bias.dtype]
        d.operand_kind, d.binary_op = L.OPERAND_ROW, L.BINARY["add"]
    d.n_unary = len(unary)
    for i, u in enumerate(unary):
        d.unary[i] = L.UNARY[u]
    d.fp32_mode, d.flags = fp32_mode, flags
    L.check(lib.ojx_gemm(ctypes.byref(d), torch.cuda.current_stream().cuda_stream), "ojx_gemm")
    route = L.ROUTES.get(lib.ojx_last_route())
    torch.cuda.synchronize()
    L.check(lib.ojx_poll_device_error(), "device error")
    return route


def sample_indices(n_total: int, n: int, seed: int) -> np.ndarray:
    """n distinct indices of [0, n_total), sorted, from a seeded generator (all of
    them when n >= n_total)."""
    if n >= n_total:
        return np.arange(n_total, dtype=np.int64)
    return np.sort(np.random.default_rng(seed).choice(n_total, size=n, replace=False)).astype(np.int64)


def sampled_parity(A, B, C, *, trans_a=False, trans_b=False, bias=None, unary=(), n=64,
                   seed=0):
    """(gpu, oracle, rows, cols) for n seeded complete rows and n complete columns of C.

    A, B, C and bias are device tensors.  The oracle computes the sampled rows from
    op(A)[rows, :] and the whole of op(B), and the sampled columns from the whole of
    op(A) and op(B)[:, cols] (each element is the same ascending-k dot product as in
    the full product).  gpu and oracle are the concatenated samples, fp32."""
    M, N = C.shape
    rows = sample_indices(M, n, seed)
    cols = sample_indices(N, n, seed + 1)
    rt, ct = torch.from_numpy(rows).to(C.device), torch.from_numpy(cols).to(C.device)
    a_rows = (A[:, rt].t() if trans_a else A[rt]).contiguous().cpu()
    b_cols = (B[ct].t() if trans_b else B[:, ct]).contiguous().cpu()
    A_h, B_h = A.cpu(), B.cpu()
    bias_h = bias.cpu() if bias is not None else None
    kind = "row" if bias is not None else None
    ref_r = oracle_gemm(a_rows, B_h, trans_b=trans_b, operand=bias_h, kind=kind, unary=unary,
                        out_dtype=C.dtype)
    ref_c = oracle_gemm(A_h, b_cols, trans_a=trans_a,
                        operand=bias_h[torch.from_numpy(cols)] if bias_h is not None else None,
                        kind=kind, unary=unary, out_dtype=C.dtype)
    got_r = C[rt].float().cpu().numpy()
    got_c = C[:, ct].float().cpu().numpy()
    gpu = np.concatenate([got_r.ravel(), got_c.ravel()])
    ref = np.concatenate([ref_r.ravel(), ref_c.ravel()])
    return gpu, ref, rows, cols


def fp32_scale(A, B, M: int, N: int) -> float:
    """||A||_F ||B||_F / sqrt(M N) of an [M, N] product (the north_star max-abs scale)."""
    return float(A.double().norm() * B.double().norm()) / float(np.sqrt(M * N))
