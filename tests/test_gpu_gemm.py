"""GPU parity of every GEMM route against the oracle on identical seeded inputs.

Bars (north_star): fp32 rel-L2 <= 1e-5 and max-abs <= 1e-4 * ||A|| ||B|| / sqrt(MN);
bf16/fp16 rel-L2 <= 1e-2 against the fp32-accumulating oracle (and a tighter
4e-3 where the only difference is accumulation order plus one bf16 rounding).
The FFMA route accumulates k in ascending order with one fma per step, exactly
like the oracle's fused variant, so it must match that variant bit for bit when
the epilogue has no transcendental function.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import (assert_fp32_parity, assert_half_parity, oracle_gemm, randn, rel_l2,
                         run_gemm)

pytestmark = pytest.mark.gpu

HALF = [torch.bfloat16, torch.float16]
TRANS = [(False, False), (True, False), (False, True), (True, True)]


def _operands(seed, M, N, K, dtype, ta, tb, scale_b=1.0):
    A = randn(seed, (K, M) if ta else (M, K), dtype)
    B = randn(seed + 1, (N, K) if tb else (K, N), dtype, scale=scale_b)
    return A, B


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("ta,tb", TRANS)
@pytest.mark.parametrize("shape", [(128, 256, 64), (200, 136, 72), (129, 264, 520),
                                   (512, 512, 512), (1024, 768, 1024)])
def test_tc_half_layouts(dtype, ta, tb, shape):
    M, N, K = shape
    A, B = _operands(sum(shape), M, N, K, dtype, ta, tb)
    C, route = run_gemm(A, B, trans_a=ta, trans_b=tb, flags=0x2)  # no skinny route
    # TMA needs 16-byte row strides: lda = M (A stored transposed) or K, ldb = K or N
    lda, ldb = (M if ta else K), (K if tb else N)
    assert route == ("tc_f16" if lda % 8 == 0 and ldb % 8 == 0 else "simt")
    ref = oracle_gemm(A, B, trans_a=ta, trans_b=tb)
    assert_half_parity(C.float().numpy(), ref, tol=4e-3)


@pytest.mark.parametrize("unary", [(), ("relu",), ("gelu",), ("silu",), ("sigmoid",), ("tanh",),
                                   ("gelu", "square", "neg"), ("abs", "sqrt", "log", "exp")])
def test_tc_bf16_bias_epilogue(unary):
    M, N, K = 256, 384, 256
    A, B = _operands(7, M, N, K, torch.bfloat16, False, False)
    bias = randn(9, (N,), torch.float32, scale=0.1)
    C, route = run_gemm(A, B, operand=bias, kind="row", unary=unary)
    assert route == "tc_f16"
    ref = oracle_gemm(A, B, operand=bias, kind="row", unary=unary)
    assert_half_parity(C.float().numpy(), ref, tol=4e-3)


@pytest.mark.parametrize("binary", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("lhs", [False, True])
def test_tc_bf16_full_operand(binary, lhs):
    M, N, K = 192, 256, 128
    A, B = _operands(11, M, N, K, torch.bfloat16, False, True)
    X = randn(13, (M, N), torch.float32) + (3.0 if binary == "div" else 0.0)
    C, route = run_gemm(A, B, trans_b=True, operand=X, kind="full", binary=binary, lhs=lhs,
                        unary=("tanh",), out_dtype=torch.float32)
    assert route == "tc_f16"
    ref = oracle_gemm(A, B, trans_b=True, operand=X, kind="full", binary=binary, lhs=lhs,
                      unary=("tanh",), out_dtype=torch.float32)
    assert rel_l2(C.numpy(), ref) < 1e-4  # fp32 output: only accumulation order differs


@pytest.mark.parametrize("shape", [(1, 7, 31), (7, 33, 65), (33, 65, 127), (129, 1, 7)])
def test_unaligned_shapes_route_to_simt(shape):
    M, N, K = shape
    A, B = _operands(17, M, N, K, torch.bfloat16, False, False)
    C, route = run_gemm(A, B, unary=("relu",))
    assert route == "simt"
    ref = oracle_gemm(A, B, unary=("relu",))
    assert_half_parity(C.float().numpy(), ref, tol=4e-3)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_skinny_cfg4_full_size(M):
    """X[M,4096] @ W[4096,14336] + bias, SiLU, bf16."""
    K, N = 4096, 14336
    X = randn(3, (M, K), torch.bfloat16)
    W = randn(4, (K, N), torch.bfloat16, scale=0.02)
    bias = torch.zeros(N, dtype=torch.bfloat16)
    C, route = run_gemm(X, W, operand=bias, kind="row", unary=("silu",))
    assert route == "skinny"
    ref = oracle_gemm(X, W, operand=bias, kind="row", unary=("silu",))
    assert_half_parity(C.float().numpy(), ref, tol=4e-3)


@pytest.mark.parametrize("shape,tb", [((3, 1000, 320), False), ((16, 384, 4160), True),
                                      ((1, 136, 64), False), ((9, 2048, 8192), False)])
def test_skinny_ragged_and_repeat(shape, tb):
    M, N, K = shape
    X, W = _operands(21, M, N, K, torch.bfloat16, False, tb, scale_b=0.05)
    bias = randn(23, (N,), torch.bfloat16, scale=0.1)
    ref = oracle_gemm(X, W, trans_b=tb, operand=bias, kind="row", unary=("gelu",))
    for _ in range(2):  # second launch reuses the arrival counters of the first
        C, route = run_gemm(X, W, trans_b=tb, operand=bias, kind="row", unary=("gelu",))
        assert route == "skinny"
        assert_half_parity(C.float().numpy(), ref, tol=4e-3)


@pytest.mark.parametrize("shape,tb", [((1, 14336, 4096), False), ((4, 14336, 4096), False),
                                      ((16, 14336, 4096), False), ((3, 1000, 320), False),
                                      ((16, 384, 4160), True), ((9, 2048, 8192), False),
                                      ((5, 65536, 128), False)])
def test_skinny_handoffs_agree(shape, tb):
    """The tagged hand-off (a group's last contributor polls the others' epoch-tagged
    partials) and the arrival-counter hand-off sum the same partials in the same order:
    bit-identical outputs, twice in a row (the second launch meets the first one's
    tags and counters), and both within the bf16 bar of the oracle.  The last shape
    has more units per CTA than k blocks per group, where only the counter applies."""
    from torchcl._lib import FLAG_SKINNY_COUNTER
    M, N, K = shape
    X, W = _operands(41, M, N, K, torch.bfloat16, False, tb, scale_b=0.05)
    bias = randn(43, (N,), torch.bfloat16, scale=0.1)
    ref = oracle_gemm(X, W, trans_b=tb, operand=bias, kind="row", unary=("silu",))
    outs = []
    for flags in (0, FLAG_SKINNY_COUNTER, 0, FLAG_SKINNY_COUNTER):
        C, route = run_gemm(X, W, trans_b=tb, operand=bias, kind="row", unary=("silu",), flags=flags)
        assert route == "skinny"
        outs.append(C.view(torch.int16))
    for C in outs[1:]:
        assert torch.equal(C, outs[0])
    assert_half_parity(outs[0].view(torch.bfloat16).float().numpy(), ref, tol=4e-3)


def test_skinny_matches_tile_route():
    M, N, K = 16, 1024, 2048
    X, W = _operands(31, M, N, K, torch.bfloat16, False, False)
    C1, r1 = run_gemm(X, W)
    C2, r2 = run_gemm(X, W, flags=0x2)
    assert (r1, r2) == ("skinny", "tc_f16")
    assert rel_l2(C1.float().numpy(), C2.float().numpy()) < 4e-3


@pytest.mark.parametrize("ta,tb", TRANS)
@pytest.mark.parametrize("shape", [(512, 512, 512), (333, 517, 259), (100, 7, 3), (1024, 1024, 1024)])
def test_fp32_3xtf32(ta, tb, shape):
    M, N, K = shape
    A, B = _operands(41 + M, M, N, K, torch.float32, ta, tb)
    bias = randn(43, (N,), torch.float32, scale=0.1)
    C, route = run_gemm(A, B, trans_a=ta, trans_b=tb, operand=bias, kind="row",
                        unary=("gelu",), fp32_mode=1)
    assert route == "tc_3xtf32"
    ref = oracle_gemm(A, B, trans_a=ta, trans_b=tb, operand=bias, kind="row", unary=("gelu",))
    assert_fp32_parity(C.numpy(), ref, A, B, ta, tb)


@pytest.mark.parametrize("shape", [(64, 128, 64), (512, 512, 512), (33, 65, 31), (1, 300, 17)])
@pytest.mark.parametrize("unary", [(), ("relu",)])
def test_fp32_ffma_bit_exact(shape, unary):
    M, N, K = shape
    A, B = _operands(51, M, N, K, torch.float32, False, False)
    bias = randn(53, (N,), torch.float32)
    C, route = run_gemm(A, B, operand=bias, kind="row", unary=unary, fp32_mode=2)
    assert route == "simt"
    ref = oracle_gemm(A, B, operand=bias, kind="row", unary=unary, fused=True)
    np.testing.assert_array_equal(C.numpy(), ref)


def test_fp32_auto_routes():
    A, B = _operands(61, 64, 64, 64, torch.float32, False, False)
    assert run_gemm(A, B)[1] == "tc_3xtf32"
    A, B = _operands(61, 8, 64, 64, torch.float32, False, False)
    assert run_gemm(A, B)[1] == "simt"


def test_output_canaries_and_ldc():
    """A GEMM into the interior of a padded buffer touches nothing outside it."""
    from torchcl.ops.engine import get_engine
    eng = get_engine()
    M, N, K, ldc = 130, 200, 96, 264
    A, B = _operands(71, M, N, K, torch.bfloat16, False, False)
    host = torch.full((M + 2, ldc), 12345.0, dtype=torch.bfloat16)
    a, b, c = eng.tensor_to_buffer(A), eng.tensor_to_buffer(B), eng.tensor_to_buffer(host)
    es = 2
    eng.gemm(a, b, c.buffer + (ldc + 8) * es, M, N, K, dtype_a=torch.bfloat16,
             dtype_b=torch.bfloat16, dtype_c=torch.bfloat16, ldc=ldc, unary=("relu",))
    out = eng.buffer_to_tensor(c, (M + 2, ldc), torch.bfloat16)
    for buf in (a, b, c):
        eng.free_buffer(buf)
    ref = oracle_gemm(A, B, unary=("relu",))
    inner = out[1:M + 1, 8:8 + N].float().numpy()
    assert_half_parity(inner, ref, tol=4e-3)
    mask = torch.ones_like(out, dtype=torch.bool)
    mask[1:M + 1, 8:8 + N] = False
    assert bool((out[mask] == 12345.0).all())


def test_empty_and_zero_k():
    A = torch.zeros(5, 0, dtype=torch.bfloat16)
    B = torch.zeros(0, 8, dtype=torch.bfloat16)
    bias = randn(81, (8,), torch.float32)
    C, route = run_gemm(A, B, operand=bias, kind="row", unary=("relu",), out_dtype=torch.float32)
    np.testing.assert_allclose(C.numpy(), np.broadcast_to(np.maximum(bias.numpy(), 0), (5, 8)))
