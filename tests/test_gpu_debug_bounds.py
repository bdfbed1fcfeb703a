"""The bounds-checking build (libojx_debug.so, OJX_DEBUG_BOUNDS=1) on odd shapes.

In that build every TMA tile origin and every epilogue store of the GEMM and
attention kernels is checked on the device before it is issued; a failure is
recorded in the device error word and read back by ojx_poll_device_error as
OJX_ERR_BOUNDS with the site and coordinates.  The shapes below are the ragged
ones the SURVEY's race/sanitizer plan names (M, N, K in {1, 7, 31, 33, 65, 127,
129} and non-multiples of the tiles), on every route: tcgen05 bf16/fp16 tiles with
both operand majors, the skinny split-K route, 3xTF32, the SIMT route, batched
GEMMs and fused attention.  Each result is compared with the oracle and no check
may fire.  The library is chosen when it is first loaded, so the cases run in a
child process with the variable set."""
import os
import pathlib
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = pathlib.Path(__file__).resolve().parents[1]

CHILD = r'''
import ctypes, sys
import numpy as np, torch
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/ojasx-open-source-cuda-_b200", sys.argv[1] + "/tests"]
from torchcl import _lib as L
assert L.DEBUG_BOUNDS and L.LIB_PATH.name == "libojx_debug.so"
lib = L.lib()
assert lib.ojx_debug_bounds_enabled() == 1
L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
from gpu_helpers import oracle_gemm, randn, rel_l2, run_gemm, assert_fp32_parity

cases = [  # (M, N, K, dtype, trans_a, trans_b, route)
    (33, 136, 72, torch.bfloat16, False, False, "tc_f16"),
    (129, 264, 520, torch.float16, False, True, "tc_f16"),
    (136, 72, 200, torch.bfloat16, True, False, "tc_f16"),   # A^T stored [K, M]: M % 8 == 0
    (200, 1000, 136, torch.bfloat16, True, True, "tc_f16"),
    (1, 136, 72, torch.bfloat16, False, False, "skinny"),
    (7, 1000, 320, torch.bfloat16, False, True, "skinny"),
    (16, 264, 4160, torch.float16, False, False, "skinny"),
    (33, 65, 31, torch.float32, False, False, "tc_3xtf32"),
    (129, 127, 33, torch.float32, True, True, "tc_3xtf32"),
    (2100, 2504, 520, torch.bfloat16, False, True, "tc_f16"),  # CTA pairs (flag 0x8), ragged
    (31, 7, 65, torch.bfloat16, False, False, "simt"),
    (7, 33, 1, torch.float32, False, False, "simt"),
]
for M, N, K, dt, ta, tb, want in cases:
    A = randn(M + N, (K, M) if ta else (M, K), dt)
    B = randn(K + 1, (N, K) if tb else (K, N), dt, scale=0.1)
    bias = randn(N, (N,), dt, scale=0.1)
    C, route = run_gemm(A, B, trans_a=ta, trans_b=tb, operand=bias, kind="row", unary=("gelu",),
                        fp32_mode=1 if want == "tc_3xtf32" else 0, flags=0x8 if M > 2000 else 0)
    assert route == want, (M, N, K, route, want)
    L.check(lib.ojx_poll_device_error(), f"{(M, N, K)} {route}")
    ref = oracle_gemm(A, B, trans_a=ta, trans_b=tb, operand=bias, kind="row", unary=("gelu",))
    if dt == torch.float32:
        assert_fp32_parity(C.numpy(), ref, A, B, ta, tb)
    else:
        assert rel_l2(C.float().numpy(), ref) <= 4e-3, (M, N, K, route)
    print("ok", M, N, K, route, flush=True)

# batched (rank-3 maps) and fused attention
import torchcl
torchcl.init_opencl(device_index=0)
A = randn(5, (3, 33, 72), torch.bfloat16); B = randn(6, (3, 72, 136), torch.bfloat16, scale=0.1)
got = torchcl.to_cpu(torchcl.blas.bmm(A, B)).float()
ref = torch.bmm(A.float(), B.float())
assert rel_l2(got.numpy(), ref.numpy()) <= 4e-3
L.check(lib.ojx_poll_device_error(), "bmm")
for (Bq, H, Mq, Nk, D, causal) in [(1, 2, 129, 65, 64, False), (2, 1, 200, 200, 128, True)]:
    q, k, v = (randn(s, (Bq, H, n, D), torch.bfloat16) for s, n in ((7, Mq), (8, Nk), (9, Nk)))
    out = torchcl.to_cpu(torchcl.fused_attention(torchcl.to_opencl(q), torchcl.to_opencl(k),
                                                 torchcl.to_opencl(v), is_causal=causal)).float()
    L.check(lib.ojx_poll_device_error(), "attention")
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           is_causal=causal)
    assert rel_l2(out.numpy(), ref.numpy()) <= 2e-2, (Mq, Nk, D)
    print("ok attention", Mq, Nk, D, flush=True)
print("ALL OK")
'''


def test_debug_bounds_build_on_ragged_shapes():
    env = dict(os.environ, OJX_DEBUG_BOUNDS="1")
    res = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], capture_output=True, text=True,
                         env=env, timeout=600)
    assert res.returncode == 0 and "ALL OK" in res.stdout, res.stdout[-3000:] + res.stderr[-3000:]
