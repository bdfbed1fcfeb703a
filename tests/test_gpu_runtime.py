"""Runtime layer on the device: caching pool statistics and evict-and-retry under
an injected cudaMalloc failure, the bounded-wait timeout path (no GPU fault: the
producer warp is silenced so the consumer's bounded wait expires and the kernel
returns), and kernel-launch accounting."""
import ctypes

import pytest
import torch

import torchcl
from torchcl import _lib as L
from torchcl.runtime.memory import get_buffer_pool

from gpu_helpers import assert_half_parity, oracle_gemm, randn, run_gemm

pytestmark = pytest.mark.gpu


def test_pool_reuse_and_stats():
    torchcl.init_opencl()
    pool = get_buffer_pool()
    s0 = pool.get_stats()
    a = pool.allocate(3000)
    assert a.capacity == 4096 and a.buffer % 256 == 0
    pool.free(a)
    b = pool.allocate(2500)  # same bin -> the freed block comes back
    assert b.buffer == a.buffer
    s1 = pool.get_stats()
    assert s1["reuse_count"] >= s0["reuse_count"] + 1
    assert s1["active_bytes"] - s0["active_bytes"] == 4096
    pool.free(b)
    assert pool.get_stats()["cached_bytes"] >= 4096


def test_pool_evict_and_retry_then_oom():
    torchcl.init_opencl()
    pool = get_buffer_pool()
    lib = L.lib()
    pool.empty_cache()  # no cached block may satisfy the requests below
    cached = pool.allocate(1 << 20)
    pool.free(cached)  # something to evict
    ev0 = pool.get_stats()["evictions"]
    lib.ojx_pool_debug_fail_next(1)  # first cudaMalloc fails, the retry after eviction succeeds
    buf = pool.allocate(3 << 20)
    assert pool.get_stats()["evictions"] == ev0 + 1
    assert pool.get_stats()["cached_bytes"] == 0
    pool.free(buf)
    lib.ojx_pool_debug_fail_next(2)  # both attempts fail -> MemoryError, like memory.py:111-115
    with pytest.raises(MemoryError):
        pool.allocate(5 << 20)
    lib.ojx_pool_debug_fail_next(0)
    ok = pool.allocate(5 << 20)  # the pool is usable afterwards
    pool.free(ok)


def test_bounded_wait_times_out_and_context_survives():
    torchcl.init_opencl()
    lib = L.lib()
    M, N, K = 256, 256, 256
    A = randn(1, (M, K), torch.bfloat16)
    B = randn(2, (K, N), torch.bfloat16)
    L.check(lib.ojx_poll_device_error())
    lib.ojx_set_wait_budget(2_000_000)  # about a millisecond
    try:
        lib.ojx_debug_silence_producer_once()
        # reading the result back synchronises and reports the expired wait
        with pytest.raises(L.TimeoutError_):
            run_gemm(A, B, flags=0x2)
        L.check(lib.ojx_poll_device_error())  # the error word was read and cleared
    finally:
        lib.ojx_set_wait_budget(4_000_000_000)
    # the same context keeps working
    C, route = run_gemm(A, B, flags=0x2)
    assert_half_parity(C.float().numpy(), oracle_gemm(A, B), tol=4e-3)
    L.check(lib.ojx_poll_device_error())


def test_skinny_timeout_path():
    torchcl.init_opencl()
    lib = L.lib()
    X = randn(3, (4, 512), torch.bfloat16)
    W = randn(4, (512, 1024), torch.bfloat16)
    lib.ojx_set_wait_budget(2_000_000)
    try:
        lib.ojx_debug_silence_producer_once()
        with pytest.raises(L.TimeoutError_):
            run_gemm(X, W)
        assert L.ROUTES[lib.ojx_last_route()] == "skinny"
    finally:
        lib.ojx_set_wait_budget(4_000_000_000)
    C, _ = run_gemm(X, W)
    assert_half_parity(C.float().numpy(), oracle_gemm(X, W), tol=4e-3)


def test_skinny_tagged_poll_times_out_and_context_survives():
    """The finishing CTA of a tagged skinny launch waits (bounded) for the other
    contributors' epoch-tagged partials.  With the contributors silenced, every
    finisher's poll must expire: the launch reports OJX_ERR_TIMEOUT and the next
    launch, with a new epoch, computes the right result."""
    torchcl.init_opencl()
    lib = L.lib()
    X = randn(7, (4, 4096), torch.bfloat16)  # cfg4's shape: 3 contributors per group, tagged
    W = randn(8, (4096, 14336), torch.bfloat16, scale=0.02)
    L.check(lib.ojx_poll_device_error())
    lib.ojx_set_wait_budget(2_000_000)  # about a millisecond
    try:
        lib.ojx_debug_silence_skinny_contributors_once()
        with pytest.raises(L.TimeoutError_):
            run_gemm(X, W)
        assert L.ROUTES[lib.ojx_last_route()] == "skinny"
        L.check(lib.ojx_poll_device_error())
    finally:
        lib.ojx_set_wait_budget(4_000_000_000)
    C, _ = run_gemm(X, W)
    assert_half_parity(C.float().numpy(), oracle_gemm(X, W), tol=4e-3)
    L.check(lib.ojx_poll_device_error())


def test_launch_counter_and_device_info():
    info = torchcl.get_device_info()
    assert info["max_compute_units"] >= 100 and "sm_10" in info["version"]
    lib = L.lib()
    n0 = lib.ojx_kernel_launch_count()
    A = randn(5, (128, 64), torch.bfloat16)
    B = randn(6, (64, 128), torch.bfloat16)
    run_gemm(A, B, flags=0x2)
    assert lib.ojx_kernel_launch_count() == n0 + 1


@pytest.mark.parametrize("M,N,K,dtype,chunk", [(1000, 512, 256, torch.bfloat16, 256),
                                               (4096, 1024, 512, torch.bfloat16, 0),
                                               (700, 384, 200, torch.float32, 128),
                                               (8, 2048, 1024, torch.bfloat16, 0)])
def test_gemm_host_io_matches_device_gemm(M, N, K, dtype, chunk):
    """ojx_gemm_host_io (host A and C, rows in overlapped chunks) gives exactly the
    device-resident GEMM's output: every row's accumulation is the same."""
    torchcl.init_opencl()
    lib = L.lib()
    A = randn(1, (M, K), dtype)
    W = randn(2, (K, N), dtype, scale=0.05)
    bias = randn(3, (N,), dtype, scale=0.1)
    es = A.element_size()
    dev = torch.device("cuda", 0)
    Wd, bd = W.to(dev), bias.to(dev)
    Ad = torch.empty(M, K, dtype=dtype, device=dev)
    Cd = torch.empty(M, N, dtype=dtype, device=dev)
    ha, hc = ctypes.c_void_p(), ctypes.c_void_p()
    L.check(lib.ojx_host_alloc(M * K * es, ctypes.byref(ha)))
    L.check(lib.ojx_host_alloc(M * N * es, ctypes.byref(hc)))
    try:
        ctypes.memmove(ha.value, A.contiguous().data_ptr(), M * K * es)
        code = L.BF16 if dtype == torch.bfloat16 else L.F32
        d = L.GemmDesc()
        d.M, d.N, d.K = M, N, K
        d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = code
        d.b, d.operand = Wd.data_ptr(), bd.data_ptr()
        d.operand_kind, d.binary_op = L.OPERAND_ROW, L.BINARY["add"]
        d.n_unary, d.unary[0] = 1, L.UNARY["relu"]
        d.a, d.c = ha.value, hc.value
        L.check(lib.ojx_gemm_host_io(ctypes.byref(d), Ad.data_ptr(), Cd.data_ptr(), chunk, None))
        L.check(lib.ojx_synchronize())
        got = torch.empty(M, N, dtype=dtype)
        ctypes.memmove(got.data_ptr(), hc.value, M * N * es)
        # the same GEMM on device-resident operands
        Ad2 = A.to(dev)
        Cd2 = torch.empty(M, N, dtype=dtype, device=dev)
        d.a, d.c = Ad2.data_ptr(), Cd2.data_ptr()
        L.check(lib.ojx_gemm(ctypes.byref(d), None))
        L.check(lib.ojx_synchronize())
        assert torch.equal(got, Cd2.cpu())
        ref = oracle_gemm(A, W, operand=bias, kind="row", unary=("relu",))
        if dtype == torch.bfloat16:
            assert_half_parity(got.float().numpy(), ref)
    finally:
        lib.ojx_host_free(ha.value)
        lib.ojx_host_free(hc.value)


def test_gemm_host_io_rejects_strided_operands():
    torchcl.init_opencl()
    lib = L.lib()
    d = L.GemmDesc()
    d.M, d.N, d.K = 64, 64, 64
    d.a = d.b = d.c = 16
    d.lda = 128
    assert lib.ojx_gemm_host_io(ctypes.byref(d), 16, 16, 0, None) == L.OJX_ERR_INVALID
