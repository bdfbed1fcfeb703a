"""The C-ABI library: it loads, exports every symbol include/ojx.h declares, and
validates arguments on the host before touching a device (CPU only)."""
import ctypes
import pathlib
import re

import pytest

from torchcl import _lib as L

REPO = pathlib.Path(__file__).resolve().parents[1]


def _declared_functions() -> list[str]:
    text = (REPO / "include" / "ojx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ojx_\w+)\s*\(", text, flags=re.M)))


def test_library_built_and_loads():
    assert L.LIB_PATH.exists(), "run python ojasx-open-source-cuda-_b200/build.py"
    assert L.lib().ojx_abi_version() == 1


def test_exports_every_declared_symbol():
    declared = _declared_functions()
    assert len(declared) >= 38
    so = ctypes.CDLL(str(L.LIB_PATH))
    missing = [name for name in declared if not hasattr(so, name)]
    assert not missing, missing
    # the Python binding covers the whole header too
    assert sorted(L.exported_symbols()) == declared


def test_pool_bin_policy():
    cap = ctypes.c_size_t()
    lib = L.lib()

    def bin_of(n):
        assert lib.ojx_pool_bin_size(n, ctypes.byref(cap)) == 0
        return cap.value

    assert bin_of(0) == 512 and bin_of(1) == 512 and bin_of(512) == 512
    assert bin_of(513) == 1024 and bin_of(4096) == 4096 and bin_of(4097) == 8192
    assert bin_of(64 << 20) == 64 << 20
    two_mb = 2 << 20
    assert bin_of((64 << 20) + 1) == (64 << 20) + two_mb
    big = 32768 * 32768 * 2
    assert bin_of(big) == big and bin_of(big + 1) == big + two_mb


def test_gemm_rejects_bad_descriptors_without_device():
    lib = L.lib()
    assert lib.ojx_gemm(None, None) == L.OJX_ERR_INVALID
    d = L.GemmDesc()
    d.M, d.N, d.K = -1, 4, 4
    assert lib.ojx_gemm(ctypes.byref(d), None) == L.OJX_ERR_INVALID
    assert "negative" in L.last_error()
    d.M = 4
    d.n_unary = 9
    assert lib.ojx_gemm(ctypes.byref(d), None) == L.OJX_ERR_INVALID
    d.n_unary = 1
    d.unary[0] = 99
    assert lib.ojx_gemm(ctypes.byref(d), None) == L.OJX_ERR_INVALID
    d.unary[0] = L.UNARY["relu"]
    d.operand_kind = L.OPERAND_ROW  # operand pointer missing
    assert lib.ojx_gemm(ctypes.byref(d), None) == L.OJX_ERR_INVALID
    d.operand_kind = 0
    d.M = 0  # empty problem: nothing to do, no device needed
    assert lib.ojx_gemm(ctypes.byref(d), None) == L.OJX_OK
    assert lib.ojx_elementwise(None, 0, None, 0, None, 0, 0, None, 0, -1, None) == L.OJX_ERR_INVALID
    assert lib.ojx_set_wait_budget(0) == L.OJX_ERR_INVALID


def test_status_maps_to_reference_exceptions():
    with pytest.raises(ValueError):
        L.check(L.OJX_ERR_INVALID)
    with pytest.raises(MemoryError):
        L.check(L.OJX_ERR_OOM)
    with pytest.raises(RuntimeError):
        L.check(L.OJX_ERR_CUDA)
    with pytest.raises(L.TimeoutError_):
        L.check(L.OJX_ERR_TIMEOUT)
    L.check(L.OJX_OK)


def test_desc_layout_matches_header():
    # ojx_gemm_desc: 3 int64, 4+2 int32, 4 int64, 4 pointers, 4 int32, int32[8], 2 int32
    assert ctypes.sizeof(L.GemmDesc) == 3 * 8 + 6 * 4 + 4 * 8 + 4 * 8 + 4 * 4 + 8 * 4 + 2 * 4
    assert L.GemmDesc.lda.offset == 48 and L.GemmDesc.a.offset == 80
