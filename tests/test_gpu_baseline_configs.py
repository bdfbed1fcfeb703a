"""GPU parity at the BASELINE configurations' own shapes, on the inputs bench.py times.

Each case regenerates a config's seeded inputs on the device with bench.make_inputs
(the same generator calls, so the same A, W and bias the benchmark line is quoted
on), runs the fused GEMM through the C-ABI (ojx_gemm) and compares it with the
oracle (the reference's ascending-k fp32 accumulation, then the epilogue):

* up to 4096^3 over the whole of C;
* above that over 64 seeded complete rows and 64 seeded complete columns of C
  (the oracle computes those from the matching slices of the operands).

Bars (north_star): fp32 rel-L2 <= 1e-5 and max-abs <= 1e-4 * ||A||_F ||B||_F / sqrt(MN);
bf16 rel-L2 <= 1e-2 against the fp32-accumulating oracle.
Configs: cfg1 fp32 relu(A@B + bias) 512^3; cfg2 fp32 gelu_tanh(A@B + bias) at 1024,
2048, 4096 and 8192 with the A^T@B and A@B^T variants; cfg3 bf16 FFN silu(X@W)
8192x4096x11008; cfg4 bf16 skinny silu(X@W + bias) M in {1, 4, 16}; cfg5 bf16
relu(A@W + bias) 32768^3 (8 GB of device memory: A, W and C of 2 GB each plus the
fp32 draw).
"""
import numpy as np
import pytest
import torch

import bench
from gpu_helpers import (assert_fp32_parity, device_gemm, fp32_scale, oracle_gemm, rel_l2,
                         sampled_parity)

pytestmark = pytest.mark.gpu

FULL_LIMIT = 4096  # whole-matrix comparison up to this size, sampled above it


def _inputs(name, **over):
    cfg = dict(bench.CONFIGS[name])
    cfg.update(over)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    A, W, bias = bench.make_inputs(cfg, dev)
    return cfg, A, W, bias


def _check(cfg, A, B, C, bias, ta, tb, route, expect_route):
    M, N = C.shape
    unary = (cfg["act"],)
    assert route == expect_route, (route, expect_route)
    if max(cfg["M"], cfg["N"], cfg["K"]) <= FULL_LIMIT:
        got = C.float().cpu().numpy()
        ref = oracle_gemm(A.cpu(), B.cpu(), trans_a=ta, trans_b=tb, operand=bias.cpu(), kind="row",
                          unary=unary)
        sample = "whole C"
    else:
        got, ref, rows, cols = sampled_parity(A, B, C, trans_a=ta, trans_b=tb, bias=bias,
                                              unary=unary, n=64, seed=cfg["seed"])
        sample = f"{len(rows)} rows + {len(cols)} columns of C"
    err = rel_l2(got, ref)
    mx = float(np.abs(got.astype(np.float64) - ref).max())
    print(f"{cfg['desc']} ta={ta} tb={tb}: rel-L2 {err:.3e}, max-abs {mx:.3e} over {sample}")
    if C.dtype == torch.float32:
        scale = fp32_scale(A, B, M, N)
        assert err <= 1e-5, f"rel-L2 {err:.3e} > 1e-5 ({sample})"
        assert mx <= 1e-4 * scale, f"max-abs {mx:.3e} > 1e-4 * {scale:.3e} ({sample})"
    else:
        assert err <= 1e-2, f"rel-L2 {err:.3e} > 1e-2 ({sample})"
    return err


def test_cfg1_fp32_512():
    cfg, A, W, bias = _inputs("cfg1")
    C = torch.empty(cfg["M"], cfg["N"], device=A.device, dtype=torch.float32)
    route = device_gemm(A, W, C, bias=bias, unary=(cfg["act"],))
    _check(cfg, A, W, C, bias, False, False, route, "tc_3xtf32")
    # the same problem on the FFMA route is bit-exact to the oracle's one-fma-per-step variant
    route = device_gemm(A, W, C, bias=bias, unary=(cfg["act"],), fp32_mode=2)
    assert route == "simt"
    ref = oracle_gemm(A.cpu(), W.cpu(), operand=bias.cpu(), kind="row", unary=(cfg["act"],),
                      fused=True)
    np.testing.assert_array_equal(C.cpu().numpy(), ref)


@pytest.mark.parametrize("size", [1024, 2048, 4096, 8192])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True)])
def test_cfg2_fp32_sweep(size, ta, tb):
    """A, B ~ U(-1,1), bias ~ N(0, 0.1), gelu_tanh; the transposed variants read the same
    square buffers as A^T (stored [K, M]) or B^T (stored [N, K])."""
    cfg, A, B, bias = _inputs("cfg2", M=size, N=size, K=size)
    C = torch.empty(size, size, device=A.device, dtype=torch.float32)
    route = device_gemm(A, B, C, trans_a=ta, trans_b=tb, bias=bias, unary=(cfg["act"],))
    _check(cfg, A, B, C, bias, ta, tb, route, "tc_3xtf32")


def test_cfg3_bf16_ffn():
    cfg, X, W, bias = _inputs("cfg3")
    C = torch.empty(cfg["M"], cfg["N"], device=X.device, dtype=torch.bfloat16)
    route = device_gemm(X, W, C, bias=bias, unary=(cfg["act"],))
    _check(cfg, X, W, C, bias, False, False, route, "tc_f16")


@pytest.mark.parametrize("m", [1, 4, 16])
def test_cfg4_bf16_skinny(m):
    cfg, X, W, bias = _inputs("cfg4", M=m)
    C = torch.empty(m, cfg["N"], device=X.device, dtype=torch.bfloat16)
    route = device_gemm(X, W, C, bias=bias, unary=(cfg["act"],))
    _check(cfg, X, W, C, bias, False, False, route, "skinny")


def test_cfg5_bf16_32768():
    cfg, A, W, bias = _inputs("cfg5")
    C = torch.empty(cfg["M"], cfg["N"], device=A.device, dtype=torch.bfloat16)
    route = device_gemm(A, W, C, bias=bias, unary=(cfg["act"],))
    _check(cfg, A, W, C, bias, False, False, route, "tc_f16")
    del A, W, C
    torch.cuda.empty_cache()
