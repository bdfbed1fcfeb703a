"""End to end through the public API with the overlapped host pipeline.

torchcl.to_opencl of a pinned host tensor defers its upload; torchcl.to_cpu of a
lazy GEMM on it then runs upload, fused GEMM and download chunk by chunk
(ojx_gemm_host_io).  The result must equal the device-resident path's bit for bit
(same kernels, rows processed independently) and the oracle within the bars, and
both handles must hold their device data afterwards."""
import numpy as np
import pytest
import torch

from gpu_helpers import assert_fp32_parity, assert_half_parity, oracle_gemm, randn

pytestmark = pytest.mark.gpu


def _pinned(t):
    return t.contiguous().pin_memory()


@pytest.mark.parametrize("dtype,shape,act", [
    (torch.bfloat16, (2048, 1536, 1024), "relu"),   # 8 row chunks of 256
    (torch.float16, (1000, 264, 520), "silu"),      # 8 chunks of 128 rows, the last ragged
    (torch.float32, (1200, 264, 136), "gelu"),      # 3xTF32, 5 chunks of 256 rows
])
def test_pinned_gemm_to_cpu_matches_device_path(dtype, shape, act, monkeypatch):
    import torchcl
    monkeypatch.setattr(torchcl.api, "DEFERRED_UPLOAD_MIN_BYTES", 0)  # defer every pinned upload
    M, N, K = shape
    A = randn(1, (M, K), dtype)
    W = randn(2, (K, N), dtype, scale=0.05)
    bias = randn(3, (N,), dtype, scale=0.1)
    w, b = torchcl.to_opencl(W), torchcl.to_opencl(bias)
    f = getattr(torchcl, act)
    a = torchcl.to_opencl(_pinned(A))
    assert getattr(torchcl.api._elem(a), "_torchcl_host", None) is not None  # deferred
    n0 = torchcl._lib.lib().ojx_kernel_launch_count()
    got = torchcl.to_cpu(f(torchcl.add(torchcl.matmul(a, w), b)))
    assert got.is_pinned()
    assert torchcl._lib.lib().ojx_kernel_launch_count() > n0
    eager = torchcl.to_cpu(f(torchcl.add(torchcl.matmul(torchcl.to_opencl(A), w), b)))
    assert torch.equal(got, eager)
    ref = oracle_gemm(A, W, operand=bias, kind="row", unary=(act,))
    if dtype == torch.float32:
        assert_fp32_parity(got.numpy(), ref, A, W)
    else:
        assert_half_parity(got.float().numpy(), ref, tol=4e-3)
    # the deferred handle now holds A on the device
    assert torch.equal(torchcl.to_cpu(a), A)


def test_deferred_handle_used_by_other_ops_uploads_once():
    import torchcl
    A = randn(4, (1024, 512), torch.float32)
    a = torchcl.to_opencl(_pinned(A))
    r = torchcl.to_cpu(torchcl.relu(a))          # elementwise consumer: plain upload
    assert torch.equal(r, torch.relu(A))
    W = randn(5, (512, 256), torch.float32, scale=0.1)
    got = torchcl.to_cpu(torchcl.matmul(a, torchcl.to_opencl(W)))  # already uploaded: eager GEMM
    ref = oracle_gemm(A, W)
    assert_fp32_parity(got.numpy(), ref, A, W)


def test_small_or_pageable_tensors_upload_at_once():
    import torchcl
    small = _pinned(torch.ones(16, 16))
    h = torchcl.to_opencl(small)
    assert getattr(torchcl.api._elem(h), "_torchcl_host", None) is None
    big = torch.ones(1024, 512)
    h2 = torchcl.to_opencl(big)
    assert getattr(torchcl.api._elem(h2), "_torchcl_host", None) is None
    assert np.array_equal(torchcl.to_cpu(h2).numpy(), big.numpy())
