"""Training-side GEMMs: MatmulFunction / LinearFunction forward and backward
(the reference's torchcl/autograd.py:277-314, 355-412), OpenCLLinear
(torchcl/nn.py:58-119) and the bias-gradient column sums (reduction.cl:170-181).
Every gradient GEMM reads its transposed operand through the descriptor, so each
is checked against the oracle's GEMM with the same transpose flags."""
import types

import numpy as np
import pytest
import torch

import torchcl
from torchcl import _lib as L
from torchcl.autograd import LinearFunction, MatmulFunction
from torchcl.nn import OpenCLLinear

from gpu_helpers import assert_fp32_parity, assert_half_parity, host_bits, oracle_gemm, randn
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CODES = {torch.float32: O.F32, torch.bfloat16: O.BF16, torch.float16: O.F16}


def _ctx(saved, **attrs):
    """Stand-in for the autograd context, as the reference's tests build one
    (tests/test_autograd.py:108-118)."""
    ctx = types.SimpleNamespace(**attrs)
    ctx.saved_tensors = saved
    ctx.save_for_backward = lambda *t: setattr(ctx, "saved_tensors", t)
    return ctx


def _np(t):
    return torchcl.to_cpu(t).float().numpy()


def _check(got, ref, A=None, B=None, trans_a=False, trans_b=False):
    if got.dtype == torch.float32:
        assert_fp32_parity(got.numpy(), ref, A, B, trans_a=trans_a, trans_b=trans_b)
    else:
        assert_half_parity(got.float().numpy(), ref)


@pytest.mark.parametrize("rows,cols", [(0, 5), (1, 1), (63, 300), (64, 64), (65, 129),
                                       (1000, 4097), (8192, 1024)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sum_columns_matches_oracle(rows, cols, dtype):
    X = randn(rows + cols, (rows, cols), dtype)
    xd = torchcl.to_opencl(X) if rows else None
    from torchcl.ops.engine import get_engine
    eng = get_engine()
    ob = eng.allocate_output((cols,), torch.float32)
    eng.run_sum_columns(torchcl.api._get_buf(xd) if rows else None, ob, rows, cols,
                        dtype_in=dtype, dtype_out=torch.float32)
    out = eng.buffer_to_tensor(ob, (cols,), torch.float32).numpy()
    bits = host_bits(X) if rows else np.zeros((0, cols), np.float32 if dtype == torch.float32 else np.uint16)
    blocked = O.sum_columns(bits, CODES[dtype], block=64)
    # same summation order as the oracle's blocked restatement: bit-exact
    np.testing.assert_array_equal(out.view(np.uint32), blocked.view(np.uint32))
    if rows:
        seq = O.sum_columns(bits, CODES[dtype])  # the reference kernel's order
        assert np.linalg.norm(out - seq) <= 1e-5 * max(np.linalg.norm(seq), 1e-30)


def test_sum_columns_bf16_output_and_reference_fixture(golden_dir):
    rec = np.load(golden_dir / "sum_columns_257x300.npz")
    X = torch.from_numpy(rec["X"])
    from torchcl.ops.engine import get_engine
    eng = get_engine()
    xb = eng.tensor_to_buffer(X)
    ob = eng.allocate_output((300,), torch.bfloat16)
    eng.run_sum_columns(xb, ob, 257, 300, dtype_in=torch.float32, dtype_out=torch.bfloat16)
    got = eng.buffer_to_tensor(ob, (300,), torch.bfloat16).float().numpy()
    ref = rec["S_nofma"]  # the reference kernel's own column sums
    assert np.abs(got - ref).max() <= 2 ** -7 * np.abs(ref).max()


def test_matmul_autograd_reference():
    """tests/test_autograd.py:83-91"""
    m1_cpu, m2_cpu = torch.randn(16, 32), torch.randn(32, 8)
    result_cl = MatmulFunction.apply(torchcl.to_opencl(m1_cpu), torchcl.to_opencl(m2_cpu))
    assert torch.allclose(torchcl.to_cpu(result_cl), m1_cpu @ m2_cpu, atol=1e-2)


@pytest.mark.parametrize("M,N,K", [(16, 8, 32), (256, 320, 384), (130, 50, 70), (1, 300, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_matmul_function_backward(M, N, K, dtype):
    A, B = randn(1, (M, K), dtype), randn(2, (K, N), dtype, scale=0.1)
    G = randn(3, (M, N), dtype)
    a, b = torchcl.to_opencl(A), torchcl.to_opencl(B)
    ctx = _ctx(())
    C = MatmulFunction.forward(ctx, a, b)
    _check(torchcl.to_cpu(C), oracle_gemm(A, B), A, B)
    gA, gB = MatmulFunction.backward(ctx, torchcl.to_opencl(G))
    _check(torchcl.to_cpu(gA), oracle_gemm(G, B, trans_b=True), G, B, trans_b=True)
    _check(torchcl.to_cpu(gB), oracle_gemm(A, G, trans_a=True), A, G, trans_a=True)
    if dtype == torch.float32:  # and against torch's own autograd
        At, Bt = A.clone().requires_grad_(), B.clone().requires_grad_()
        (At @ Bt).backward(G)
        assert torch.allclose(torchcl.to_cpu(gA), At.grad, rtol=1e-4, atol=1e-4)
        assert torch.allclose(torchcl.to_cpu(gB), Bt.grad, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [(64, 96, 128), (200, 300, 136), (8, 1000, 256), (1024, 512, 768)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_linear_function_forward_backward(M, N, K, dtype):
    X, W = randn(4, (M, K), dtype), randn(5, (N, K), dtype, scale=0.05)
    bias, G = randn(6, (N,), dtype, scale=0.1), randn(7, (M, N), dtype)
    ctx = _ctx(())
    Y = LinearFunction.forward(ctx, torchcl.to_opencl(X), torchcl.to_opencl(W), torchcl.to_opencl(bias))
    _check(torchcl.to_cpu(Y), oracle_gemm(X, W, trans_b=True, operand=bias, kind="row"), X, W,
           trans_b=True)
    gX, gW, gb = LinearFunction.backward(ctx, torchcl.to_opencl(G))
    _check(torchcl.to_cpu(gX), oracle_gemm(G, W), G, W)
    _check(torchcl.to_cpu(gW), oracle_gemm(G, X, trans_a=True), G, X, trans_a=True)
    sums = O.sum_columns(host_bits(G), CODES[dtype], block=64)
    if dtype == torch.float32:
        np.testing.assert_array_equal(_np(gb).view(np.uint32), sums.view(np.uint32))
    else:  # bf16 gradient: the fp32 sums rounded once
        np.testing.assert_array_equal(host_bits(torchcl.to_cpu(gb)), O.bf16_bits(sums))


def test_linear_function_through_torch_autograd():
    """loss.backward()-style use: torch.autograd.grad drives LinearFunction.backward."""
    X = torch.randn(32, 64, requires_grad=True)
    W = (torch.randn(48, 64) * 0.1).requires_grad_()
    b = torch.randn(48, requires_grad=True)
    Y = LinearFunction.apply(X, W, b)
    G = torch.randn(32, 48)
    gx, gw, gb = torch.autograd.grad(Y, (X, W, b), grad_outputs=torchcl.to_opencl(G))
    Xr, Wr, br = (t.detach().clone().requires_grad_() for t in (X, W, b))
    torch.nn.functional.linear(Xr, Wr, br).backward(G)
    for got, ref in ((gx, Xr.grad), (gw, Wr.grad), (gb, br.grad)):
        assert torch.allclose(torchcl.to_cpu(got), ref, rtol=1e-4, atol=1e-4)


def test_opencl_linear_module():
    torch.manual_seed(0)
    layer = OpenCLLinear(96, 40)
    x = torch.randn(24, 96)
    y = torchcl.to_cpu(layer(torchcl.to_opencl(x)))
    ref = torch.nn.functional.linear(x, layer.weight.data, layer.bias.data)
    assert torch.allclose(y, ref, rtol=1e-4, atol=1e-4)
    n0 = L.lib().ojx_kernel_launch_count()
    layer(torchcl.to_opencl(x))
    assert L.lib().ojx_kernel_launch_count() - n0 <= 3  # one GEMM (3xTF32: two operand splits + GEMM)
    with pytest.raises(ValueError):
        layer(torchcl.to_opencl(torch.randn(4, 95)))
