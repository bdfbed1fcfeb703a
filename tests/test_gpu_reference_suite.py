"""The reference's own hot-path tests, ported onto the B200 torchcl (same seeds,
shapes and tolerances; file:line of the reference test in each docstring), plus
the reference's golden outputs replayed through the public API."""
import gc

import numpy as np
import pytest
import torch

import torchcl
import torchcl.blas as blas
from torchcl import _lib as L
from torchcl.jit.cache import get_kernel_cache
from torchcl.jit.compiler import get_jit_compiler
from torchcl.jit.tuner import get_auto_tuner
from torchcl.runtime.memory import get_buffer_pool

pytestmark = pytest.mark.gpu


def test_baseline_arithmetic():
    """tests/test_cuda_correctness_baseline.py:12-31"""
    torch.manual_seed(101)
    a_cpu = torch.randn(10000)
    b_cpu = torch.randn(10000) + 2.0
    a_cl, b_cl = torchcl.to_opencl(a_cpu), torchcl.to_opencl(b_cpu)
    for name, cpu_fn, cl_fn, tol in [("add", torch.add, torchcl.add, 1e-5),
                                     ("sub", torch.sub, torchcl.sub, 1e-5),
                                     ("mul", torch.mul, torchcl.mul, 1e-5),
                                     ("div", torch.div, torchcl.div, 1e-4)]:
        diff = (cpu_fn(a_cpu, b_cpu) - torchcl.to_cpu(cl_fn(a_cl, b_cl))).abs().max().item()
        assert diff < tol, name


def test_baseline_activations():
    """tests/test_cuda_correctness_baseline.py:34-51"""
    torch.manual_seed(202)
    x_cpu = torch.randn(10000)
    x_cl = torchcl.to_opencl(x_cpu)
    for name, cpu_fn, cl_fn, tol in [
            ("relu", torch.relu, torchcl.relu, 1e-6),
            ("sigmoid", torch.sigmoid, torchcl.sigmoid, 1e-5),
            ("tanh", torch.tanh, torchcl.tanh_, 1e-5),
            ("gelu", lambda x: torch.nn.functional.gelu(x, approximate="tanh"), torchcl.gelu, 1e-5),
            ("silu", torch.nn.functional.silu, torchcl.silu, 1e-5)]:
        diff = (cpu_fn(x_cpu) - torchcl.to_cpu(cl_fn(x_cl))).abs().max().item()
        assert diff < tol, f"{name}: {diff}"


def test_baseline_matrix_ops():
    """tests/test_cuda_correctness_baseline.py:54-69"""
    torch.manual_seed(303)
    A_cpu, B_cpu = torch.randn(64, 128), torch.randn(128, 64)
    A_cl, B_cl = torchcl.to_opencl(A_cpu), torchcl.to_opencl(B_cpu)
    assert (torch.matmul(A_cpu, B_cpu) - torchcl.to_cpu(torchcl.matmul(A_cl, B_cl))).abs().max() < 1e-4
    assert (A_cpu.t() - torchcl.to_cpu(torchcl.transpose(A_cl))).abs().max() < 1e-6


def test_baseline_streams_and_events():
    """tests/test_cuda_correctness_baseline.py:118-136"""
    s1, s2 = torchcl.Stream(), torchcl.Stream()
    e1, e2 = torchcl.Event(), torchcl.Event()
    e1.record(s1)
    with torchcl.stream(s1):
        a = torchcl.to_opencl(torch.randn(256, 256))
        b = torchcl.matmul(a, a)
        b_buf = torchcl.api._get_buf(b)  # launch it on s1
    with torchcl.stream(s2):
        s2.wait_stream(s1)
        c = torchcl.relu(b)
        torchcl.api._get_buf(c)
    e2.record(s2)
    s2.synchronize()
    assert e1.elapsed_time(e2) >= 0.0
    assert b_buf is not None


def test_ojas_blas_gemm_fused():
    """tests/test_ojas_blas.py:11-23"""
    torch.manual_seed(42)
    A, B, bias = torch.randn(64, 128), torch.randn(128, 64), torch.randn(64)
    out = torchcl.to_cpu(blas.gemm(A, B, bias=bias, activation="relu"))
    assert (out - torch.relu(A @ B + bias)).abs().max().item() < 1e-3


def test_ojas_blas_bmm():
    """tests/test_ojas_blas.py:55-66"""
    torch.manual_seed(42)
    A, B = torch.randn(4, 32, 64), torch.randn(4, 64, 32)
    out = torchcl.to_cpu(blas.bmm(A, B))
    assert (out - torch.bmm(A, B)).abs().max().item() < 1e-3


def test_fused_unary_chains():
    """tests/test_jit.py:15-45"""
    jit, pool = get_jit_compiler(), get_buffer_pool()
    n = 1024
    x = np.random.randn(n).astype(np.float32)
    x_buf, out_buf = pool.host_to_device(x), pool.allocate(n * 4)
    for ops, expected in [(["sigmoid", "relu"], np.maximum(0, 1.0 / (1.0 + np.exp(-x)))),
                          (["neg", "exp"], np.exp(-x)), (["tanh", "abs"], np.abs(np.tanh(x)))]:
        jit.fuse_elementwise_chain(ops, n, [x_buf.buffer], out_buf.buffer)
        assert np.allclose(pool.device_to_host(out_buf, np.float32, (n,)), expected, atol=1e-3)
    pool.free(x_buf)
    pool.free(out_buf)


def test_fused_binary_unary():
    """tests/test_jit.py:48-72"""
    jit, pool = get_jit_compiler(), get_buffer_pool()
    n = 1024
    a, b = np.random.randn(n).astype(np.float32), np.random.randn(n).astype(np.float32)
    a_buf, b_buf, out_buf = pool.host_to_device(a), pool.host_to_device(b), pool.allocate(n * 4)
    jit.fuse_binary_then_unary("add", ["relu"], n, a_buf.buffer, b_buf.buffer, out_buf.buffer)
    assert np.allclose(pool.device_to_host(out_buf, np.float32, (n,)), np.maximum(0, a + b), atol=1e-3)
    jit.fuse_binary_then_unary("mul", ["sigmoid"], n, a_buf.buffer, b_buf.buffer, out_buf.buffer)
    assert np.allclose(pool.device_to_host(out_buf, np.float32, (n,)), 1 / (1 + np.exp(-(a * b))), atol=1e-3)
    for buf in (a_buf, b_buf, out_buf):
        pool.free(buf)


def test_autotuner_and_kernel_cache():
    """tests/test_jit.py:75-98"""
    tuner = get_auto_tuner()
    wg = tuner.optimal_workgroup_1d(100000)
    assert wg > 0 and (wg & (wg - 1)) == 0
    assert tuner.optimal_tile_size(512, 512, 512) in (4, 8, 16)
    jit, pool, cache = get_jit_compiler(), get_buffer_pool(), get_kernel_cache()
    n = 512
    x_buf = pool.host_to_device(np.random.randn(n).astype(np.float32))
    out_buf = pool.allocate(n * 4)
    hits = cache.stats()["hits"]
    jit.fuse_elementwise_chain(["sigmoid", "relu"], n, [x_buf.buffer], out_buf.buffer)
    jit.fuse_elementwise_chain(["sigmoid", "relu"], n, [x_buf.buffer], out_buf.buffer)
    assert cache.stats()["hits"] >= hits + 1
    pool.free(x_buf)
    pool.free(out_buf)


def test_jit_integration():
    """tests/test_jit_integration.py:11-47"""
    torch.manual_seed(42)
    a, b = torch.randn(128, 128), torch.randn(128, 128)
    res = torchcl.to_cpu(torchcl.relu(torchcl.add(torchcl.to_opencl(a), torchcl.to_opencl(b))))
    assert (res - torch.relu(a + b)).abs().max().item() < 1e-4
    cache = get_jit_compiler()._cache
    a2, b2 = torch.randn(128, 128), torch.randn(128, 128)
    hits = cache.stats()["hits"]
    res2 = torchcl.to_cpu(torchcl.relu(torchcl.add(torchcl.to_opencl(a2), torchcl.to_opencl(b2))))
    assert (res2 - torch.relu(a2 + b2)).abs().max().item() < 1e-4
    assert cache.stats()["hits"] > hits


def test_mixed_precision_matmul():
    """tests/test_mixed_precision_flow.py:7-51 (fp16 route forced through the dispatcher)"""
    from torchcl.liquid.cost_model import KernelConfig
    from torchcl.liquid.dispatch import get_dispatcher
    dispatcher = get_dispatcher()
    original = dispatcher.dispatch
    dispatcher.dispatch = lambda op, *a, **k: KernelConfig(256, 16, "tiled", "half")
    try:
        a_cpu, b_cpu = torch.randn(32, 32), torch.randn(32, 32)
        res = torchcl.to_cpu(torchcl.matmul(torchcl.to_opencl(a_cpu), torchcl.to_opencl(b_cpu)))
        assert res.dtype == torch.float32
        assert torch.allclose(res, a_cpu @ b_cpu, atol=5e-2, rtol=1e-2)
    finally:
        dispatcher.dispatch = original


def test_smoke_data_movement_and_creation():
    """tests/test_smoke.py:13-35"""
    a = torch.randn(100, 100)
    a_cl = torchcl.to_opencl(a)
    assert torch.allclose(torchcl.to_cpu(a_cl), a, atol=1e-4)
    assert torchcl.is_opencl_tensor(a_cl) is True and torchcl.is_opencl_tensor(a) is False
    assert torch.allclose(torchcl.to_cpu(torchcl.zeros(3, 3)), torch.zeros(3, 3))
    assert torch.allclose(torchcl.to_cpu(torchcl.ones(4, 4)), torch.ones(4, 4))
    assert torch.allclose(torchcl.to_cpu(torchcl.full(2, 3, fill_value=7.0)), torch.full((2, 3), 7.0))
    assert torchcl.to_cpu(torchcl.randn(5, 5)).shape == (5, 5)


def test_smoke_matrix_operations():
    """tests/test_smoke.py:73-103"""
    m1, m2 = torch.randn(64, 128), torch.randn(128, 32)
    out = torchcl.to_cpu(torchcl.matmul(torchcl.to_opencl(m1), torchcl.to_opencl(m2)))
    assert torch.allclose(out, m1 @ m2, atol=1e-2)
    m3 = torch.randn(16, 32)
    assert torch.allclose(torchcl.to_cpu(torchcl.transpose(torchcl.to_opencl(m3))), m3.T, atol=1e-4)
    big_a, big_b = torch.randn(512, 512), torch.randn(512, 512)
    r = torchcl.matmul(torchcl.to_opencl(big_a), torchcl.to_opencl(big_b))
    torchcl.synchronize()
    assert torch.allclose(torchcl.to_cpu(r), big_a @ big_b, atol=0.5)


def test_shadow_buffer_gc():
    """tests/test_memory_leak.py:10-35"""
    gc.collect()
    initial = len(torchcl.api._opencl_buffers)

    def allocate_tensors():
        for _ in range(50):
            t = torchcl.randn(10, 10)
            assert getattr(t, "_torchcl_id") in torchcl.api._opencl_buffers

    allocate_tensors()
    gc.collect()
    assert len(torchcl.api._opencl_buffers) == initial


@pytest.mark.parametrize("name", ["baseline_matmul_303", "blas_gemm_bias_relu_42", "cfg1_512_bias_relu",
                                  "ragged_33x65x47", "naive_bias_4x256x300"])
def test_reference_golden_through_public_api(golden_dir, name):
    """The reference's own outputs (its kernels, compiled for the host) vs torchcl on B200."""
    rec = dict(np.load(golden_dir / f"{name}.npz"))
    A, B = torch.from_numpy(rec["A"]), torch.from_numpy(rec["B"])
    act = str(rec["meta"][1])
    bias = torch.from_numpy(rec["bias"]) if "bias" in rec else None
    out = torchcl.to_cpu(blas.gemm(A, B, bias=bias, activation=act or None))
    ref = rec["C_nofma"].astype(np.float64)
    C = out.numpy().astype(np.float64)
    rel = np.linalg.norm(C - ref) / np.linalg.norm(ref)
    scale = float(A.double().norm() * B.double().norm()) / np.sqrt(C.size)
    assert rel <= 1e-5 and np.abs(C - ref).max() <= 1e-4 * scale


def test_fused_gemm_chain_is_one_launch():
    """relu(add(matmul(A, B), bias)) on bf16 is a single kernel (the reference needs two)."""
    torch.manual_seed(5)
    A = torchcl.to_opencl(torch.randn(256, 512).to(torch.bfloat16))
    B = torchcl.to_opencl(torch.randn(512, 384).to(torch.bfloat16))
    bias = torchcl.to_opencl(torch.randn(384).to(torch.bfloat16))
    out = torchcl.relu(torchcl.add(torchcl.matmul(A, B), bias))
    lib = L.lib()
    before = lib.ojx_kernel_launch_count()
    torchcl.api._get_buf(out)
    assert lib.ojx_kernel_launch_count() - before == 1
    ref = torch.relu(torchcl.to_cpu(A).float() @ torchcl.to_cpu(B).float() + torchcl.to_cpu(bias).float())
    got = torchcl.to_cpu(out).float()
    assert torch.linalg.norm(got - ref) / torch.linalg.norm(ref) < 4e-3


def test_transposed_views_and_linear():
    torch.manual_seed(6)
    A, W, b = torch.randn(96, 80), torch.randn(112, 80), torch.randn(112)
    Ad, Wd, bd = torchcl.to_opencl(A), torchcl.to_opencl(W), torchcl.to_opencl(b)
    out = torchcl.to_cpu(torchcl.silu(torchcl.linear(Ad, Wd, bd)))
    assert torch.allclose(out, torch.nn.functional.silu(A @ W.T + b), atol=1e-4)
    out2 = torchcl.to_cpu(torchcl.matmul(torchcl.transpose(Wd), torchcl.transpose(torchcl.transpose(Wd))))
    assert torch.allclose(out2, W.T @ W, atol=1e-3)


def test_ojasx_tensor_dispatch():
    torch.manual_seed(7)
    A, B, bias = torch.randn(40, 24), torch.randn(24, 16), torch.randn(16)
    Ad, Bd, bd = torchcl.to_opencl(A), torchcl.to_opencl(B), torchcl.to_opencl(bias)
    out = torch.relu(torch.addmm(bd, Ad, Bd))
    assert torch.allclose(torchcl.to_cpu(out), torch.relu(torch.addmm(bias, A, B)), atol=1e-4)
    out2 = torch.mm(Ad, Bd)
    assert torch.allclose(torchcl.to_cpu(out2), A @ B, atol=1e-4)
