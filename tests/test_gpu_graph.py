"""Graph capture and replay (torchcl.jit.graph_runner, the reference's
torchcl/jit/graph_runner.py): every route recorded through the public API,
replayed with fresh inputs written in place, and compared bit for bit with the
same step dispatched directly (the kernels are deterministic), plus the oracle
for the values themselves."""
import ctypes
import gc

import numpy as np
import pytest
import torch

import torchcl
from torchcl import _lib as L
from torchcl import api, blas
from torchcl.jit.graph_runner import capture_graph, get_active_capture_graph
from torchcl.runtime.memory import get_buffer_pool

from gpu_helpers import assert_fp32_parity, assert_half_parity, oracle_gemm, randn

pytestmark = pytest.mark.gpu


def _refresh(handle, t: torch.Tensor) -> None:
    """Overwrite a device tensor's buffer in place (inputs of a captured graph)."""
    get_buffer_pool().host_to_device(t.contiguous(), cl_buf=api._get_buf(handle))


@pytest.mark.parametrize("M,N,K,dtype,act,route", [
    (512, 512, 512, torch.float32, "relu", "tc_3xtf32"),     # cfg1 shape
    (256, 1024, 512, torch.bfloat16, "silu", "tc_f16"),
    (1, 14336, 4096, torch.bfloat16, "silu", "skinny"),       # cfg4 decode, M=1
    (16, 3000, 1024, torch.bfloat16, "gelu", "skinny"),
    (8, 300, 200, torch.float32, "tanh", "simt"),
])
def test_replay_matches_dispatch(M, N, K, dtype, act, route):
    scale = 0.02 if dtype != torch.float32 else 1.0
    A0 = randn(1, (M, K), dtype)
    W = randn(2, (K, N), dtype, scale=scale)
    bias = randn(3, (N,), dtype, scale=0.1)
    a, w, b = torchcl.to_opencl(A0), torchcl.to_opencl(W), torchcl.to_opencl(bias)
    with capture_graph("t") as cg:
        assert get_active_capture_graph() is cg
        out = blas.gemm(a, w, bias=b, activation=act)
    assert get_active_capture_graph() is None
    assert len(cg) >= 1
    names = " ".join(c.kernel for c in cg.commands)
    want = {"tc_3xtf32": "tc_gemm_kernel", "tc_f16": "tc_gemm_kernel",
            "skinny": "skinny_gemm_kernel", "simt": "simt_gemm_kernel"}[route]
    assert want in names, names
    # the block ran the graph once: `out` holds the first result
    first = torchcl.to_cpu(out)
    direct = torchcl.to_cpu(blas.gemm(a, w, bias=b, activation=act))
    assert torch.equal(first, direct)
    for i in range(3):  # new inputs each replay; the skinny counters must start clean every time
        Ai = randn(10 + i, (M, K), dtype)
        _refresh(a, Ai)
        cg.replay()
        got = torchcl.to_cpu(out)
        direct = torchcl.to_cpu(blas.gemm(a, w, bias=b, activation=act))
        assert torch.equal(got, direct), f"replay {i}"
        ref = oracle_gemm(Ai, W, operand=bias, kind="row", unary=(act,), out_dtype=dtype)
        if dtype == torch.float32:
            assert_fp32_parity(got.numpy(), ref, Ai, W)
        else:
            assert_half_parity(got.float().numpy(), ref)
    cg.close()


def test_replay_counts_its_kernels_and_uses_one_host_call():
    a = torchcl.to_opencl(randn(4, (256, 512), torch.bfloat16))
    w = torchcl.to_opencl(randn(5, (512, 768), torch.bfloat16, scale=0.05))
    with capture_graph() as cg:
        y1 = torchcl.relu(torchcl.matmul(a, w))
        y2 = torchcl.add(torchcl.matmul(a, w), y1)       # full [M, N] operand folded
        y3 = torchcl.sigmoid(torchcl.mul(y1, y2))        # elementwise chain
    assert len(cg) == 3, [c.kernel for c in cg.commands]
    assert "elementwise" in cg.commands[2].kernel
    n0 = L.lib().ojx_kernel_launch_count()
    cg.replay()
    torchcl.synchronize()
    assert L.lib().ojx_kernel_launch_count() - n0 == 3
    A, Wt = torchcl.to_cpu(a).float(), torchcl.to_cpu(w).float()
    r1 = torch.relu(A @ Wt)
    r3 = torch.sigmoid(r1 * (A @ Wt + r1))
    got = torchcl.to_cpu(y3).float()
    assert (got - r3).norm() / r3.norm() < 1e-2
    cg.close()


def test_fp32_graph_keeps_its_own_scratch():
    """A later, larger 3xTF32 GEMM on the default stream grows that stream's
    workspace; the graph's scratch is its own, so the replay is unaffected."""
    A = randn(6, (384, 256))
    W = randn(7, (256, 320))
    a, w = torchcl.to_opencl(A), torchcl.to_opencl(W)
    with capture_graph() as cg:
        out = torchcl.gelu(torchcl.matmul(a, w))
    first = torchcl.to_cpu(out)
    big = torchcl.matmul(torchcl.to_opencl(randn(8, (1024, 2048))), torchcl.to_opencl(randn(9, (2048, 1024))))
    torchcl.to_cpu(big)
    cg.replay()
    assert torch.equal(torchcl.to_cpu(out), first)
    cg.close()


def test_graph_buffers_stay_reserved_until_close():
    a = torchcl.to_opencl(randn(11, (128, 256), torch.bfloat16))
    w = torchcl.to_opencl(randn(12, (256, 256), torch.bfloat16, scale=0.05))
    with capture_graph() as cg:
        out = torchcl.relu(torchcl.matmul(a, w))
    addr = api._get_buf(out).buffer
    del out
    gc.collect()
    # the output's block is not handed out again while the graph lives
    pool = get_buffer_pool()
    grabbed = [pool.allocate(128 * 256 * 2, torch.bfloat16) for _ in range(8)]
    assert addr not in {g.buffer for g in grabbed}
    for g in grabbed:
        pool.free(g)
    cg.replay()
    torchcl.synchronize()
    cg.close()


def test_capture_rejects_host_transfers_and_closes_cleanly():
    a = torchcl.to_opencl(randn(13, (64, 64)))
    with pytest.raises(RuntimeError, match="captured"):
        with capture_graph():
            torchcl.to_cpu(torchcl.matmul(a, a))
    assert get_active_capture_graph() is None
    # the library keeps working after the aborted capture
    got = torchcl.to_cpu(torchcl.relu(torchcl.matmul(a, a)))
    A = torchcl.to_cpu(a)
    ref = torch.relu(A @ A)
    assert (got - ref).abs().max() < 1e-3


def test_capture_begin_rejects_legacy_stream():
    assert L.lib().ojx_graph_capture_begin(None) == L.OJX_ERR_INVALID
