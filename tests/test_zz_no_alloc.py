"""ojx_gemm_skinny_noalloc: the decode GEMM for callers that must not have the
library allocate device memory (engines that reserve the GPU's memory up front,
loops where an allocation could synchronise the device).  Called through the
C-ABI and compared with the regular entry point, ojx_gemm (whose skinny route
takes its scratch from a cudaMalloc-grown workspace), on two calls in a row, so
the second call runs on the scratch contents the first one left behind.

This file is collected last on purpose; it must also pass on its own in a fresh
process (it initialises the device itself)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _upload(lib, L, t: torch.Tensor) -> int:
    t = t.contiguous()
    nbytes = t.numel() * t.element_size()
    p = ctypes.c_void_p()
    L.check(lib.ojx_malloc(nbytes, ctypes.byref(p), None), "ojx_malloc")
    L.check(lib.ojx_memcpy_h2d(p.value, t.data_ptr(), nbytes, None), "h2d")
    return p.value


def _download(lib, L, ptr: int, shape, dtype) -> torch.Tensor:
    out = torch.empty(shape, dtype=dtype)
    L.check(lib.ojx_memcpy_d2h(out.data_ptr(), ptr, out.numel() * out.element_size(), None), "d2h")
    L.check(lib.ojx_synchronize(), "sync")
    L.check(lib.ojx_poll_device_error(), "device error")
    return out


@pytest.mark.parametrize("M,N,K,trans_b", [(16, 14336, 4096, False), (1, 1000, 320, True),
                                           (7, 4096, 2048, False)])
def test_noalloc_matches_regular_entry_point_twice(M, N, K, trans_b):
    import sys
    import pathlib
    repo = pathlib.Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "ojasx-open-source-cuda-_b200")]
    from torchcl import _lib as L

    lib = L.lib()
    L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
    g = torch.Generator().manual_seed(M * 7 + N + K)
    X = torch.randn(M, K, generator=g).bfloat16()
    W = (torch.randn((N, K) if trans_b else (K, N), generator=g) * 0.02).bfloat16()
    bias = (torch.randn(N, generator=g) * 0.1).bfloat16()
    px, pw, pb = _upload(lib, L, X), _upload(lib, L, W), _upload(lib, L, bias)
    out = []
    for _ in range(3):
        p = ctypes.c_void_p()
        L.check(lib.ojx_malloc(M * N * 2, ctypes.byref(p), None), "ojx_malloc")
        out.append(p.value)

    def desc(c_ptr):
        d = L.GemmDesc()
        d.M, d.N, d.K = M, N, K
        d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = L.BF16
        d.trans_b = int(trans_b)
        d.a, d.b, d.c = px, pw, c_ptr
        d.operand, d.operand_kind, d.binary_op = pb, L.OPERAND_ROW, L.BINARY["add"]
        d.n_unary, d.unary[0] = 1, L.UNARY["silu"]
        return d

    try:
        L.check(lib.ojx_gemm(ctypes.byref(desc(out[0])), None), "ojx_gemm")
        assert L.ROUTES[lib.ojx_last_route()] == "skinny"
        ref = _download(lib, L, out[0], (M, N), torch.bfloat16).float().numpy()
        for i in (1, 2):  # two calls in a row on the shared scratch array
            L.check(lib.ojx_gemm_skinny_noalloc(ctypes.byref(desc(out[i])), None), "noalloc")
            got = _download(lib, L, out[i], (M, N), torch.bfloat16).float().numpy()
            rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
            assert rel <= 4e-3, f"call {i}: rel-L2 {rel:.3e}"
    finally:
        for ptr in [px, pw, pb] + out:
            lib.ojx_free(ptr)


def test_noalloc_rejects_problems_beyond_its_scratch():
    import sys
    import pathlib
    repo = pathlib.Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "ojasx-open-source-cuda-_b200")]
    from torchcl import _lib as L

    lib = L.lib()
    L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
    p = ctypes.c_void_p()
    L.check(lib.ojx_malloc(1 << 16, ctypes.byref(p), None), "ojx_malloc")
    try:
        d = L.GemmDesc()
        d.M, d.N, d.K = 16, 1 << 20, 64  # 4096 column groups: far more partial slots than fit
        d.dtype_a = d.dtype_b = d.dtype_c = L.BF16
        d.a = d.b = d.c = p.value  # never read: the size check comes first
        assert lib.ojx_gemm_skinny_noalloc(ctypes.byref(d), None) == L.OJX_ERR_INVALID
        assert "scratch" in L.last_error()
    finally:
        lib.ojx_free(p.value)
