"""ctypes front end of the CPU checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module, as the checker or as the timed CPU baseline; the torchcl package never does.

* `gemm(...)` / `gemm_cols(...)` / `elementwise(...)` / `cast(...)`: the C++ restatement
  in ojx_oracle.cpp of torchcl/kernels/matmul.cl + torchcl/jit/compiler.py semantics.
* `RefKernels`: the reference's own OpenCL C kernels compiled for the host
  (oracle/_ref, built by build_oracle.py when the reference tree is present).

Array arguments are numpy arrays; bf16 and fp16 travel as uint16 bit patterns
(numpy has no bf16) and are labelled by the dtype codes below.
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent

F32, BF16, F16 = 0, 1, 2
UNARY = {"relu": 1, "sigmoid": 2, "tanh": 3, "neg": 4, "abs": 5, "exp": 6, "log": 7, "sqrt": 8,
         "silu": 9, "gelu": 10, "square": 11}
BINARY = {"add": 1, "sub": 2, "mul": 3, "div": 4}
OPERAND = {None: 0, "row": 1, "full": 2}

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_i = ctypes.c_int


def _load(path: pathlib.Path) -> ctypes.CDLL:
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run python oracle/build_oracle.py)")
    return ctypes.CDLL(str(path))


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        from oracle.build_oracle import ORACLE_LIB
        _lib = _load(ORACLE_LIB)
        _lib.oracle_gemm.argtypes = [_i64, _i64, _i64, _i, _i, _i, _i, _i, _p, _i64, _p, _i64, _p,
                                     _i64, _p, _i, _i, _i64, _i, _i, _p, _i, _i, _i, _p, _i64]
        _lib.oracle_gemm_cols.argtypes = [_i64, _i64, _i64, _i, _i, _i, _i, _i, _p, _i64, _p, _i64,
                                          _p, _p, _i, _i, _i64, _i, _i, _p, _i, _i, _i, _p, _i64]
        _lib.oracle_elementwise.argtypes = [_p, _i, _p, _i, _p, _i, _i, _p, _i, _i64]
        _lib.oracle_cast.argtypes = [_p, _i, _p, _i, _i64]
        _lib.oracle_sum_columns.argtypes = [_p, _p, _i, _i64, _i64, _i64, _i64]
        _lib.oracle_attention.argtypes = [_p, _p, _p, _p, _i, _i64, _i64, _i64, _i64,
                                          ctypes.c_float, _i, _i64]
    return _lib


def _ptr(x) -> int | None:
    return None if x is None else x.ctypes.data


def _np_for(dt: int):
    return np.float32 if dt == F32 else np.uint16


def _unary_arr(unary):
    codes = np.array([UNARY[u] if isinstance(u, str) else int(u) for u in (unary or [])] or [0],
                     dtype=np.int32)
    return codes, len(unary or [])


def gemm(a: np.ndarray, b: np.ndarray, *, dtype_a=F32, dtype_b=F32, dtype_c=F32, trans_a=False,
         trans_b=False, operand: np.ndarray | None = None, operand_kind=None, operand_dtype=F32,
         binary="add", operand_is_lhs=False, unary=(), fused=False, threads=0,
         rows: np.ndarray | None = None) -> np.ndarray:
    """C = epilogue(op(A) @ op(B)); a/b are 2-D arrays in their stored layout."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    M, K = (a.shape[1], a.shape[0]) if trans_a else a.shape
    Kb, N = (b.shape[1], b.shape[0]) if trans_b else b.shape
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    c = np.zeros((M, N), dtype=_np_for(dtype_c))
    if operand is not None:
        operand = np.ascontiguousarray(operand)
    codes, n_un = _unary_arr(unary)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    rc = lib().oracle_gemm(M, N, K, dtype_a, dtype_b, dtype_c, int(trans_a), int(trans_b),
                           _ptr(a), a.shape[1], _ptr(b), b.shape[1], _ptr(c), N,
                           _ptr(operand), OPERAND[operand_kind], operand_dtype,
                           N if operand_kind == "full" else 0, BINARY.get(binary, 0),
                           int(operand_is_lhs), _ptr(codes), n_un, int(fused), threads,
                           _ptr(rows_arr), 0 if rows_arr is None else len(rows_arr))
    if rc:
        raise RuntimeError("oracle_gemm failed")
    return c


def gemm_cols(a, b, cols, *, dtype_a=F32, dtype_b=F32, dtype_c=F32, trans_a=False, trans_b=False,
              operand=None, operand_kind=None, operand_dtype=F32, binary="add",
              operand_is_lhs=False, unary=(), fused=False, threads=0) -> np.ndarray:
    """Columns `cols` of epilogue(op(A) @ op(B)) as an [M, len(cols)] array."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    M, K = (a.shape[1], a.shape[0]) if trans_a else a.shape
    N = b.shape[0] if trans_b else b.shape[1]
    cols = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.zeros((M, len(cols)), dtype=_np_for(dtype_c))
    if operand is not None:
        operand = np.ascontiguousarray(operand)
    codes, n_un = _unary_arr(unary)
    rc = lib().oracle_gemm_cols(M, N, K, dtype_a, dtype_b, dtype_c, int(trans_a), int(trans_b),
                                _ptr(a), a.shape[1], _ptr(b), b.shape[1], _ptr(out),
                                _ptr(operand), OPERAND[operand_kind], operand_dtype,
                                N if operand_kind == "full" else 0, BINARY.get(binary, 0),
                                int(operand_is_lhs), _ptr(codes), n_un, int(fused), threads,
                                _ptr(cols), len(cols))
    if rc:
        raise RuntimeError("oracle_gemm_cols failed")
    return out


def elementwise(a, b=None, *, binary=None, unary=(), dtype_a=F32, dtype_b=F32, dtype_out=F32):
    a = np.ascontiguousarray(a)
    out = np.zeros(a.shape, dtype=_np_for(dtype_out))
    bb = None if b is None else np.ascontiguousarray(b)
    codes, n_un = _unary_arr(unary)
    lib().oracle_elementwise(_ptr(out), dtype_out, _ptr(a), dtype_a, _ptr(bb), dtype_b,
                             BINARY.get(binary, 0) if binary else 0, _ptr(codes), n_un, a.size)
    return out


def cast(x: np.ndarray, dtype_in: int, dtype_out: int) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.zeros(x.shape, dtype=_np_for(dtype_out))
    lib().oracle_cast(_ptr(out), dtype_out, _ptr(x), dtype_in, x.size)
    return out


def sum_columns(x: np.ndarray, dtype_in: int = F32, block: int = 0) -> np.ndarray:
    """fp32 column sums of a [rows, cols] array (float32 values or 16-bit patterns).
    block=0 is the reference kernel's order; block=64 the GPU kernel's."""
    x = np.ascontiguousarray(x)
    rows, cols = x.shape
    out = np.zeros(cols, dtype=np.float32)
    lib().oracle_sum_columns(_ptr(out), _ptr(x), dtype_in, rows, cols, cols, block)
    return out


def attention(q, k, v, scale=None, causal=False, dtype: int = F32, max_keys: int = 2048):
    """[..., M, D] x [..., N, D] attention in the reference kernel's order
    (fp32 values or 16-bit patterns); max_keys=2048 keeps the reference's key cap,
    0 keeps every key."""
    q, k, v = (np.ascontiguousarray(x) for x in (q, k, v))
    *lead, M, D = q.shape
    N = k.shape[-2]
    BH = int(np.prod(lead)) if lead else 1
    if scale is None:
        scale = D ** -0.5
    out = np.zeros((BH, M, D), dtype=np.float32)
    lib().oracle_attention(_ptr(out), _ptr(q), _ptr(k), _ptr(v), dtype, BH, M, N, D,
                           float(scale), int(bool(causal)), int(max_keys))
    return out.reshape(*lead, M, D)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (round to nearest even)."""
    return cast(np.asarray(x, dtype=np.float32), F32, BF16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class RefKernels:
    """The reference's matmul/activation/elementwise/precision kernels built for the host."""

    def __init__(self, variant: str = "nofma"):
        from oracle.build_oracle import REF_LIBS
        self.variant = variant
        L = _load(REF_LIBS[variant])
        f32p = ctypes.POINTER(ctypes.c_float)
        for name in ("ref_matmul_reg_tiled_f32", "ref_matmul_naive_f32", "ref_matmul_tiled_f32"):
            getattr(L, name).argtypes = [_p, _p, _p, _i, _i, _i]
        for name in ("ref_matmul_reg_tiled_bias_f32", "ref_matmul_bias_f32"):
            getattr(L, name).argtypes = [_p, _p, _p, _p, _i, _i, _i]
        L.ref_linear_forward_tiled_f32.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i]
        L.ref_transpose_f32.argtypes = [_p, _p, _i, _i]
        L.ref_matmul_tiled_fp16.argtypes = [_p, _p, _p, _i, _i, _i]
        L.ref_activation.argtypes = [ctypes.c_char_p, _p, _p, _i]
        L.ref_binary.argtypes = [ctypes.c_char_p, _p, _p, _p, _i]
        L.ref_unary.argtypes = [ctypes.c_char_p, _p, _p, _i]
        L.ref_pack_fp32_to_fp16.argtypes = [_p, _p, _i]
        L.ref_unpack_fp16_to_fp32.argtypes = [_p, _p, _i]
        L.ref_sum_columns_f32.argtypes = [_p, _p, _i, _i]
        L.ref_matmul_batched_strided_f32.argtypes = [_p, _p, _p, _i, _i, _i, _i]
        L.ref_flash_attention_f32.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _i, ctypes.c_float, _i]
        del f32p
        self.L = L

    @staticmethod
    def available(variant: str = "nofma") -> bool:
        from oracle.build_oracle import REF_LIBS
        return REF_LIBS[variant].exists()

    def matmul(self, A, B, kernel="reg_tiled", bias=None):
        A = np.ascontiguousarray(A, dtype=np.float32)
        B = np.ascontiguousarray(B, dtype=np.float32)
        M, K = A.shape
        N = B.shape[1]
        C = np.zeros((M, N), dtype=np.float32)
        if bias is None:
            getattr(self.L, f"ref_matmul_{kernel}_f32")(_ptr(A), _ptr(B), _ptr(C), M, N, K)
        else:
            bias = np.ascontiguousarray(bias, dtype=np.float32)
            name = "ref_matmul_reg_tiled_bias_f32" if kernel == "reg_tiled" else "ref_matmul_bias_f32"
            getattr(self.L, name)(_ptr(A), _ptr(B), _ptr(bias), _ptr(C), M, N, K)
        return C

    def bmm(self, A, B):
        A = np.ascontiguousarray(A, dtype=np.float32)
        B = np.ascontiguousarray(B, dtype=np.float32)
        batch, M, K = A.shape
        N = B.shape[2]
        C = np.zeros((batch, M, N), dtype=np.float32)
        self.L.ref_matmul_batched_strided_f32(_ptr(A), _ptr(B), _ptr(C), batch, M, N, K)
        return C

    def attention(self, q, k, v, scale=None, causal=False):
        q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
        B, H, M, D = q.shape
        N = k.shape[2]
        if scale is None:
            scale = D ** -0.5
        out = np.zeros_like(q)
        self.L.ref_flash_attention_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, M, N, D,
                                       float(scale), int(bool(causal)))
        return out

    def sum_columns(self, X):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        out = np.zeros(cols, dtype=np.float32)
        self.L.ref_sum_columns_f32(_ptr(X), _ptr(out), rows, cols)
        return out

    def linear(self, A, W, bias=None):
        A = np.ascontiguousarray(A, dtype=np.float32)
        W = np.ascontiguousarray(W, dtype=np.float32)
        M, K = A.shape
        N = W.shape[0]
        C = np.zeros((M, N), dtype=np.float32)
        b = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else A
        self.L.ref_linear_forward_tiled_f32(_ptr(A), _ptr(W), _ptr(b), _ptr(C), M, N, K,
                                            int(bias is not None))
        return C

    def transpose(self, A):
        A = np.ascontiguousarray(A, dtype=np.float32)
        M, N = A.shape
        out = np.zeros((N, M), dtype=np.float32)
        self.L.ref_transpose_f32(_ptr(A), _ptr(out), M, N)
        return out

    def matmul_fp16(self, A16, B16):
        A16 = np.ascontiguousarray(A16, dtype=np.uint16)
        B16 = np.ascontiguousarray(B16, dtype=np.uint16)
        M, K = A16.shape
        N = B16.shape[1]
        C = np.zeros((M, N), dtype=np.uint16)
        self.L.ref_matmul_tiled_fp16(_ptr(A16), _ptr(B16), _ptr(C), M, N, K)
        return C

    def activation(self, name, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros_like(x)
        if self.L.ref_activation(name.encode(), _ptr(x), _ptr(out), x.size):
            raise ValueError(name)
        return out

    def binary(self, name, a, b):
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        out = np.zeros_like(a)
        if self.L.ref_binary(name.encode(), _ptr(a), _ptr(b), _ptr(out), a.size):
            raise ValueError(name)
        return out

    def unary(self, name, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros_like(x)
        if self.L.ref_unary(name.encode(), _ptr(x), _ptr(out), x.size):
            raise ValueError(name)
        return out

    def pack_fp16(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.shape, dtype=np.uint16)
        self.L.ref_pack_fp32_to_fp16(_ptr(x), _ptr(out), x.size)
        return out
