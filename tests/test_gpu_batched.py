"""Batched GEMM (ojx_gemm_batched, blas.bmm): the reference's blas.bmm
(torchcl/blas/__init__.py:123-150, winograd_gemm.cl:91-119), checked problem by
problem against the oracle GEMM, plus the reference's own bmm test and golden
output, and the one-launch property."""
import numpy as np
import pytest
import torch

import torchcl
import torchcl.blas as blas
from torchcl import _lib as L
from torchcl.ops.engine import get_engine

from gpu_helpers import assert_fp32_parity, assert_half_parity, oracle_gemm, randn

pytestmark = pytest.mark.gpu


def _run(A, B, *, trans_a=False, trans_b=False, shared_b=False, bias=None, bias_per_batch=False,
         unary=(), out_dtype=None):
    """C[b] for every b through one ojx_gemm_batched call; A is [batch, ...], B is
    [batch, ...] (or one matrix when shared_b)."""
    eng = get_engine()
    batch = A.shape[0]
    M = A.shape[2] if trans_a else A.shape[1]
    K = A.shape[1] if trans_a else A.shape[2]
    Bm = B if shared_b else B[0]
    N = Bm.shape[0] if trans_b else Bm.shape[1]
    out_dtype = out_dtype or A.dtype
    a, b = eng.tensor_to_buffer(A), eng.tensor_to_buffer(B)
    op = eng.tensor_to_buffer(bias) if bias is not None else None
    c = eng.allocate_output((batch, M, N), out_dtype)
    n0 = L.lib().ojx_kernel_launch_count()
    route = eng.gemm(a, b, c, M, N, K, dtype_a=A.dtype, dtype_b=B.dtype, dtype_c=out_dtype,
                     trans_a=trans_a, trans_b=trans_b, operand=op,
                     operand_kind="row" if bias is not None else None,
                     operand_dtype=bias.dtype if bias is not None else None, unary=unary,
                     batch=batch, stride_a=M * K, stride_b=0 if shared_b else K * N,
                     stride_c=M * N, stride_operand=N if bias_per_batch else 0)
    launches = L.lib().ojx_kernel_launch_count() - n0
    C = eng.buffer_to_tensor(c, (batch, M, N), out_dtype)
    return C, route, launches


def _check_each(C, A, B, *, trans_a=False, trans_b=False, shared_b=False, bias=None,
                bias_per_batch=False, unary=()):
    for i in range(A.shape[0]):
        Bi = B if shared_b else B[i]
        bi = None if bias is None else (bias[i] if bias_per_batch else bias)
        ref = oracle_gemm(A[i], Bi, trans_a=trans_a, trans_b=trans_b, operand=bi,
                          kind="row" if bi is not None else None, unary=unary, out_dtype=C.dtype)
        if C.dtype == torch.float32:
            assert_fp32_parity(C[i].numpy(), ref, A[i], Bi, trans_a=trans_a, trans_b=trans_b)
        else:
            assert_half_parity(C[i].float().numpy(), ref)


@pytest.mark.parametrize("batch,M,N,K", [(4, 256, 256, 128), (3, 200, 136, 72), (16, 64, 64, 64),
                                         (2, 1, 512, 256), (40, 128, 1024, 64)])
@pytest.mark.parametrize("trans_a,trans_b", [(False, False), (True, False), (False, True)])
def test_bf16_batched_one_launch(batch, M, N, K, trans_a, trans_b):
    A = randn(batch * 10 + M, (batch, K, M) if trans_a else (batch, M, K), torch.bfloat16)
    B = randn(batch * 10 + N, (batch, N, K) if trans_b else (batch, K, N), torch.bfloat16, scale=0.1)
    C, route, launches = _run(A, B, trans_a=trans_a, trans_b=trans_b)
    aligned = (M * 2) % 16 == 0 if trans_a else (K * 2) % 16 == 0
    aligned = aligned and ((K * 2) % 16 == 0 if trans_b else (N * 2) % 16 == 0) and (N * 2) % 16 == 0
    if aligned and (M * K * 2) % 16 == 0 and (K * N * 2) % 16 == 0:
        assert route == "tc_f16" and launches == 1, (route, launches)
    _check_each(C, A, B, trans_a=trans_a, trans_b=trans_b)


def test_bf16_batched_shared_weight_and_bias_epilogue():
    batch, M, N, K = 6, 192, 320, 256
    A = randn(1, (batch, M, K), torch.bfloat16)
    W = randn(2, (K, N), torch.bfloat16, scale=0.05)  # one weight for every problem
    bias = randn(3, (batch, N), torch.bfloat16, scale=0.1)  # one bias row per problem
    C, route, launches = _run(A, W, shared_b=True, bias=bias, bias_per_batch=True, unary=("gelu",))
    assert route == "tc_f16" and launches == 1
    _check_each(C, A, W, shared_b=True, bias=bias, bias_per_batch=True, unary=("gelu",))
    b1 = bias[0]  # shared bias
    C, _, _ = _run(A, W, shared_b=True, bias=b1, unary=("silu",))
    _check_each(C, A, W, shared_b=True, bias=b1, unary=("silu",))


@pytest.mark.parametrize("batch,M,N,K", [(4, 96, 80, 72), (3, 300, 128, 33)])
def test_fp32_batched_3xtf32(batch, M, N, K):
    A, B = randn(5, (batch, M, K)), randn(6, (batch, K, N))
    C, route, launches = _run(A, B, unary=("relu",))
    assert route == "tc_3xtf32" and launches == 3  # two operand splits + one GEMM
    _check_each(C, A, B, unary=("relu",))


def test_batched_fallback_loops_problems():
    """Strides that break 16-byte alignment (K = 7 in bf16) take one launch per problem."""
    A, B = randn(7, (3, 20, 7), torch.bfloat16), randn(8, (3, 7, 9), torch.bfloat16)
    C, route, launches = _run(A, B)
    assert launches == 3
    _check_each(C, A, B)


def test_batched_rejects_overlapping_outputs():
    eng = get_engine()
    a = eng.allocate_output((2, 16, 16), torch.float32)
    with pytest.raises(ValueError):
        eng.gemm(a, a, a, 16, 16, 16, batch=2, stride_a=256, stride_b=256, stride_c=100)


def test_ojas_blas_bmm_reference():
    """tests/test_ojas_blas.py:55-66"""
    torch.manual_seed(42)
    A = torch.randn(4, 32, 64)
    B = torch.randn(4, 64, 32)
    expected = torch.bmm(A, B)
    out_cl = blas.bmm(A, B)
    diff = (torchcl.to_cpu(out_cl) - expected).abs().max().item()
    assert diff < 1e-3, f"Difference too high in Batched GEMM: {diff}"


def test_bmm_golden_through_public_api(golden_dir):
    rec = np.load(golden_dir / "bmm_42.npz")
    A, B = torch.from_numpy(rec["A"]), torch.from_numpy(rec["B"])
    n0 = L.lib().ojx_kernel_launch_count()
    got = torchcl.to_cpu(blas.bmm(A, B)).numpy()
    assert L.lib().ojx_kernel_launch_count() - n0 == 3  # 3xTF32: one batched GEMM (+ 2 splits)
    ref = rec["C_nofma"]  # the reference kernel's own output
    for i in range(4):
        assert_fp32_parity(got[i], ref[i], A[i], B[i])


def test_bmm_bf16_and_shared_rhs():
    A = randn(9, (5, 48, 96), torch.bfloat16)
    B = randn(10, (96, 40), torch.bfloat16, scale=0.1)
    got = torchcl.to_cpu(blas.bmm(torchcl.to_opencl(A), torchcl.to_opencl(B)))
    ref = torch.matmul(A.float(), B.float())
    assert ((got.float() - ref).norm() / ref.norm()).item() < 1e-2
