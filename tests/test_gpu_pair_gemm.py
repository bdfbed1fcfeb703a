"""The CTA-pair instance of the tcgen05 GEMM (cta_group::2, clusters of 2 CTAs,
256 x 256 tiles: each CTA loads 128 rows of A and half of the tile's B columns, and
the pair leader's MMAs read both CTAs' shared memory).

It is taken on request (OJX_GEMM_FLAG_PAIR) for unbatched bf16/fp16 problems with A
row-major whose 256 x 256 tiles fill every pair at least once.  Each case runs it and
the default one-CTA kernel on the same inputs.  Both are compared with the oracle; the
two kernels sum every element's k-steps in the same order, so their results must
match bit for bit.  The shapes cover ragged K, ragged N (the second CTA's half of
the last column tile partly past N), ragged M (the second CTA's 128 rows of the last
row tile entirely past M), both B layouts and both 16-bit types."""
import pytest
import torch

from gpu_helpers import assert_half_parity, oracle_gemm, randn, run_gemm

pytestmark = pytest.mark.gpu

PAIR = 0x8


@pytest.mark.parametrize("M,N,K,dtype,tb,unary", [
    (2048, 2560, 512, torch.bfloat16, False, ("relu",)),
    (2304, 2304, 1000, torch.float16, True, ("silu",)),
    (2200, 2504, 520, torch.bfloat16, False, ("gelu",)),
    (2100, 2504, 136, torch.bfloat16, True, ()),
])
def test_pair_kernel_matches_one_cta_kernel_and_oracle(M, N, K, dtype, tb, unary):
    from torchcl import _lib as L
    lib = L.lib()
    A = randn(M, (M, K), dtype)
    B = randn(N, (N, K) if tb else (K, N), dtype, scale=0.05)
    bias = randn(K, (N,), torch.float32, scale=0.1)
    n0 = lib.ojx_kernel_launch_count()
    C2, r2 = run_gemm(A, B, trans_b=tb, operand=bias, kind="row", unary=unary, flags=PAIR)
    C1, r1 = run_gemm(A, B, trans_b=tb, operand=bias, kind="row", unary=unary)
    assert (r1, r2) == ("tc_f16", "tc_f16")
    assert lib.ojx_kernel_launch_count() - n0 == 2
    ref = oracle_gemm(A, B, trans_b=tb, operand=bias, kind="row", unary=unary)
    assert_half_parity(C2.float().numpy(), ref, tol=4e-3)
    assert torch.equal(C2.view(torch.int16), C1.view(torch.int16))


def test_pair_kernel_into_a_padded_output():
    """ldc > N and an offset start: the pair's TMA stores write exactly the block."""
    from torchcl.ops.engine import get_engine
    eng = get_engine()
    M, N, K, ldc = 2048, 2560, 256, 2600
    A = randn(3, (M, K), torch.bfloat16)
    B = randn(4, (K, N), torch.bfloat16, scale=0.05)
    host = torch.full((M + 1, ldc), 7.0, dtype=torch.bfloat16)
    a, b, c = eng.tensor_to_buffer(A), eng.tensor_to_buffer(B), eng.tensor_to_buffer(host)
    route = eng.gemm(a, b, c.buffer + (ldc + 16) * 2, M, N, K, dtype_a=torch.bfloat16,
                     dtype_b=torch.bfloat16, dtype_c=torch.bfloat16, ldc=ldc, flags=PAIR)
    out = eng.buffer_to_tensor(c, (M + 1, ldc), torch.bfloat16)
    for buf in (a, b, c):
        eng.free_buffer(buf)
    assert route == "tc_f16"
    ref = oracle_gemm(A, B)
    assert_half_parity(out[1:, 16:16 + N].float().numpy(), ref, tol=4e-3)
    mask = torch.ones_like(out, dtype=torch.bool)
    mask[1:, 16:16 + N] = False
    assert bool((out[mask] == 7.0).all())
