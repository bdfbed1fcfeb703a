"""Back-to-back skinny (decode) GEMMs on one stream, each reading what the one
before it wrote: the launches overlap through programmatic dependent launch, so
these tests check that every dependent read still sees the previous kernel's
output (the reference's decode path is torchcl/kernels/matmul.cl:346-385 via
torchcl/ops/engine.py:166-179; here it is the skinny route of ojx_gemm)."""
import ctypes

import numpy as np
import pytest
import torch

from torchcl import _lib as L

from gpu_helpers import host_bits, oracle_gemm, rel_l2

pytestmark = pytest.mark.gpu


def _desc(x, w, c, bias, act):
    d = L.GemmDesc()
    d.M, d.K = x.shape
    d.N = w.shape[1]
    d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = L.BF16
    d.a, d.b, d.c = x.data_ptr(), w.data_ptr(), c.data_ptr()
    if bias is not None:
        d.operand, d.operand_kind, d.binary_op = bias.data_ptr(), L.OPERAND_ROW, L.BINARY["add"]
    if act:
        d.n_unary, d.unary[0] = 1, L.UNARY[act]
    return d


def _launch(d, stream):
    lib = L.lib()
    L.check(lib.ojx_gemm(ctypes.byref(d), stream.cuda_stream), "ojx_gemm")
    assert L.ROUTES[lib.ojx_last_route()] == "skinny"


def _chain(xs, ws, bs, cs, stream, sync_each):
    for x, w, b, c in zip(xs, ws, bs, cs):
        _launch(_desc(x, w, c, b, "silu"), stream)
        if sync_each:
            torch.cuda.synchronize()
    torch.cuda.synchronize()


@pytest.mark.parametrize("M", [1, 16])
def test_layer_chain_reads_each_previous_output(M):
    """x_{i+1} = silu(x_i @ W_i + b_i) for 8 layers, queued without a host wait."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(100 + M)
    H, layers = 2048, 8
    ws = [(torch.randn(H, H, device=dev, generator=g) * 0.03).bfloat16() for _ in range(layers)]
    bs = [(torch.randn(H, device=dev, generator=g) * 0.1).bfloat16() for _ in range(layers)]
    x0 = torch.randn(M, H, device=dev, generator=g).bfloat16()
    stream = torch.cuda.current_stream(dev)
    outs = {}
    for sync_each in (False, True):
        cs = [torch.full((M, H), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(layers)]
        _chain([x0] + cs[:-1], ws, bs, cs, stream, sync_each)
        outs[sync_each] = [c.cpu() for c in cs]
    for i in range(layers):  # deterministic kernels: overlapped == serialised, bit for bit
        assert torch.equal(outs[False][i], outs[True][i]), f"layer {i}"
    xin = x0.cpu()
    for i in range(layers):  # and each layer matches the oracle on the input it was given
        ref = oracle_gemm(xin, ws[i].cpu(), operand=bs[i].cpu(), kind="row", unary=("silu",))
        got = outs[False][i].float().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, ref) <= 1e-2, (i, rel_l2(got, ref))
        xin = outs[False][i]


def test_weight_written_by_the_previous_launch():
    """The second GEMM's W is the first GEMM's output: the W tiles it prefetches
    into L2 before its dependency wait must not hand it stale values."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    K0, N = 4096, 6144
    x0 = torch.randn(16, K0, device=dev, generator=g).bfloat16()
    w0 = (torch.randn(K0, N, device=dev, generator=g) * 0.02).bfloat16()
    x1 = torch.randn(16, 16, device=dev, generator=g).bfloat16()
    stream = torch.cuda.current_stream(dev)
    for trial in range(3):
        c1 = torch.full((16, N), float(trial + 1), device=dev, dtype=torch.bfloat16)
        c2 = torch.empty(16, N, device=dev, dtype=torch.bfloat16)
        _launch(_desc(x0, w0, c1, None, None), stream)
        _launch(_desc(x1, c1, c2, None, None), stream)  # W of this launch = C of the last
        torch.cuda.synchronize()
        ref = oracle_gemm(x1.cpu(), c1.cpu())
        got = c2.float().cpu().numpy()
        assert rel_l2(got, ref) <= 1e-2, (trial, rel_l2(got, ref))
        # the stale contents (every element = trial + 1) would give rows of a constant sum
        stale = oracle_gemm(x1.cpu(), torch.full((16, N), float(trial + 1)).bfloat16())
        assert rel_l2(got, stale) > 0.5


def test_skinny_after_a_torch_kernel_sees_its_writes():
    """A plain kernel (torch's) writes X; the skinny launch that follows reads it."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(9)
    w = (torch.randn(4096, 14336, device=dev, generator=g) * 0.02).bfloat16()
    b = (torch.randn(14336, device=dev, generator=g) * 0.1).bfloat16()
    x = torch.zeros(4, 4096, device=dev, dtype=torch.bfloat16)
    c = torch.empty(4, 14336, device=dev, dtype=torch.bfloat16)
    src = torch.randn(4, 4096, device=dev, generator=g).bfloat16()
    stream = torch.cuda.current_stream(dev)
    x.copy_(src * 2)
    _launch(_desc(x, w, c, b, "silu"), stream)
    torch.cuda.synchronize()
    ref = oracle_gemm(x.cpu(), w.cpu(), operand=b.cpu(), kind="row", unary=("silu",))
    assert rel_l2(c.float().cpu().numpy(), ref) <= 1e-2
    assert np.array_equal(host_bits(x.cpu()), host_bits((src * 2).cpu()))
