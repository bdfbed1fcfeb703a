"""The oracle restatement against the reference's own outputs (CPU only).

Golden vectors in tests/golden/ were produced by tests/golden/make_golden.py from
the OjasX reference itself: its OpenCL C kernels (matmul.cl, activation.cl,
precision.cl) and its JIT-generated kernels, compiled for the host.  Bit-exact
agreement is required.  When the reference tree is present (development
container), the live reference build in oracle/_ref is also compared on fresh
random shapes.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

GEMM_CASES = ["baseline_matmul_303", "blas_gemm_bias_relu_42", "cfg1_512_bias_relu",
              "ragged_33x65x47", "naive_bias_4x256x300", "linear_40x72x56"]
JIT_CASES = ["unary_sigmoid_relu", "unary_neg_exp", "unary_tanh_abs", "unary_gelu",
             "unary_silu_square", "binary_add_relu", "binary_mul_sigmoid", "binary_sub_gelu",
             "binary_div_tanh", "binary_add_silu"]


def _load(golden_dir, name):
    return dict(np.load(golden_dir / f"{name}.npz"))


def _oracle_for(rec, fused):
    kernel, act = (str(x) for x in rec["meta"])
    unary = [act] if act else []
    bias = rec.get("bias")
    kw = dict(operand=bias, operand_kind="row" if bias is not None else None, unary=unary,
              fused=fused)
    if kernel == "linear":
        return O.gemm(rec["A"], rec["B"], trans_b=True, **kw)
    return O.gemm(rec["A"], rec["B"], **kw)


@pytest.mark.parametrize("name", GEMM_CASES)
def test_gemm_golden_nofma_bit_exact(golden_dir, oracle_lib, name):
    rec = _load(golden_dir, name)
    np.testing.assert_array_equal(_oracle_for(rec, fused=False), rec["C_nofma"])


@pytest.mark.parametrize("name", [c for c in GEMM_CASES if c != "naive_bias_4x256x300"])
def test_gemm_golden_fma_bit_exact(golden_dir, oracle_lib, name):
    # The host build of matmul_naive_f32 with -ffp-contract=fast does not fuse every
    # step of its k loop, so it is not a one-fma-per-step reference; it is left out.
    rec = _load(golden_dir, name)
    np.testing.assert_array_equal(_oracle_for(rec, fused=True), rec["C_fma"])


def test_gemm_golden_close_to_float64(golden_dir, oracle_lib):
    rec = _load(golden_dir, "baseline_matmul_303")
    exact = rec["A"].astype(np.float64) @ rec["B"].astype(np.float64)
    assert np.abs(rec["C_nofma"] - exact).max() < 1e-4  # tests/test_cuda_correctness_baseline.py:62


def test_fp16_golden(golden_dir, oracle_lib):
    rec = _load(golden_dir, "fp16_tiled_32")
    out = O.gemm(rec["A16"], rec["B16"], dtype_a=O.F16, dtype_b=O.F16, dtype_c=O.F16)
    np.testing.assert_array_equal(out, rec["C16_nofma"])


@pytest.mark.parametrize("name", ["sum_columns_257x300", "sum_columns_1024x96"])
def test_sum_columns_golden_bit_exact(golden_dir, oracle_lib, name):
    """reduction.cl:170-181: the oracle's column sums in the reference's order."""
    rec = _load(golden_dir, name)
    out = O.sum_columns(rec["X"])
    np.testing.assert_array_equal(out.view(np.uint32), rec["S_nofma"].view(np.uint32))
    np.testing.assert_array_equal(out.view(np.uint32), rec["S_fma"].view(np.uint32))
    # the GPU kernel's blocked order stays within the fp32 bar of the reference's
    blocked = O.sum_columns(rec["X"], block=64)
    assert np.linalg.norm(blocked - out) <= 1e-6 * np.linalg.norm(out)


def test_bmm_golden_bit_exact(golden_dir, oracle_lib):
    """winograd_gemm.cl:91-119 (blas.bmm): the oracle GEMM per batch entry."""
    rec = _load(golden_dir, "bmm_42")
    out = np.stack([O.gemm(rec["A"][i], rec["B"][i]) for i in range(rec["A"].shape[0])])
    np.testing.assert_array_equal(out.view(np.uint32), rec["C_nofma"].view(np.uint32))
    assert np.abs(out - rec["C_fma"]).max() < 1e-4


@pytest.mark.parametrize("name", ["attention_2x4x32x32x64", "attention_2x4x16x16x32",
                                  "attention_causal_1x2x40x40x48", "attention_1x1x5x2100x32"])
def test_attention_golden_bit_exact(golden_dir, oracle_lib, name):
    """flash_attention.cl:8-187: the oracle's attention in the reference's order."""
    rec = _load(golden_dir, name)
    out = O.attention(rec["q"], rec["k"], rec["v"], causal=bool(rec["causal"]))
    np.testing.assert_array_equal(out.view(np.uint32), rec["out_nofma"].view(np.uint32))
    assert np.abs(out - rec["out_fma"]).max() < 1e-5


def test_transpose_golden(golden_dir):
    rec = _load(golden_dir, "transpose_16x32")
    np.testing.assert_array_equal(rec["A"].T, rec["T_nofma"])


@pytest.mark.parametrize("act", ["relu", "sigmoid", "tanh", "gelu", "silu"])
def test_activation_golden(golden_dir, oracle_lib, act):
    rec = _load(golden_dir, "activations_202")
    x = rec["x"]
    np.testing.assert_array_equal(O.elementwise(x, unary=[act]), rec[f"{act}_nofma"])
    # and the reference's own tolerance against torch (tests/test_cuda_correctness_baseline.py:34-51)
    tx = torch.from_numpy(x)
    ref = {"relu": torch.relu, "sigmoid": torch.sigmoid, "tanh": torch.tanh,
           "gelu": lambda t: torch.nn.functional.gelu(t, approximate="tanh"),
           "silu": torch.nn.functional.silu}[act](tx).numpy()
    tol = 1e-6 if act == "relu" else 1e-5
    assert np.abs(rec[f"{act}_nofma"] - ref).max() < tol


@pytest.mark.parametrize("name", JIT_CASES)
def test_jit_golden(golden_dir, oracle_lib, name):
    inp = _load(golden_dir, "jit_inputs")
    rec = _load(golden_dir, name)
    binop, ops = (str(x) for x in rec["meta"])
    out = O.elementwise(inp["a"], inp["b"] if binop else None, binary=binop or None,
                        unary=ops.split(","))
    np.testing.assert_array_equal(out, rec["out_nofma"])


@pytest.mark.skipif(not O.RefKernels.available("nofma"),
                    reason="oracle/_ref not built (reference tree absent)")
@pytest.mark.parametrize("shape", [(1, 1, 1), (7, 31, 33), (65, 129, 127), (31, 300, 16),
                                   (128, 64, 200)])
def test_live_reference_bit_exact(oracle_lib, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 1000 + N + K)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    R = O.RefKernels("nofma")
    for kern in ("reg_tiled", "tiled", "naive"):
        np.testing.assert_array_equal(O.gemm(A, B), R.matmul(A, B, kern))
    np.testing.assert_array_equal(O.gemm(A, B, operand=bias, operand_kind="row"),
                                  R.matmul(A, B, "reg_tiled", bias=bias))
    W = np.ascontiguousarray(B.T)
    np.testing.assert_array_equal(O.gemm(A, W, trans_b=True, operand=bias, operand_kind="row"),
                                  R.linear(A, W, bias))
    RF = O.RefKernels("fma")
    np.testing.assert_array_equal(O.gemm(A, B, fused=True), RF.matmul(A, B, "reg_tiled"))


def test_oracle_transposes_and_epilogue(oracle_lib):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((37, 53), dtype=np.float32)
    B = rng.standard_normal((53, 29), dtype=np.float32)
    X = rng.standard_normal((37, 29), dtype=np.float32)
    base = O.gemm(A, B)
    np.testing.assert_array_equal(O.gemm(np.ascontiguousarray(A.T), B, trans_a=True), base)
    np.testing.assert_array_equal(O.gemm(A, np.ascontiguousarray(B.T), trans_b=True), base)
    out = O.gemm(A, B, operand=X, operand_kind="full", binary="sub", operand_is_lhs=True,
                 unary=["tanh", "abs"])
    np.testing.assert_array_equal(out, O.elementwise(X, base, binary="sub", unary=["tanh", "abs"]))
    rows = np.array([0, 5, 36])
    part = O.gemm(A, B, rows=rows)
    np.testing.assert_array_equal(part[rows], base[rows])
    cols = np.array([1, 28])
    np.testing.assert_array_equal(O.gemm_cols(A, B, cols), base[:, cols])


def test_oracle_bf16_extension(oracle_lib):
    rng = np.random.default_rng(4)
    A = rng.standard_normal((16, 64), dtype=np.float32)
    B = rng.standard_normal((64, 24), dtype=np.float32)
    Ab, Bb = O.bf16_bits(A), O.bf16_bits(B)
    out = O.bf16_to_f32(O.gemm(Ab, Bb, dtype_a=O.BF16, dtype_b=O.BF16, dtype_c=O.BF16))
    ref = (torch.from_numpy(O.bf16_to_f32(Ab)).double() @ torch.from_numpy(O.bf16_to_f32(Bb)).double())
    rel = np.linalg.norm(out - ref.numpy()) / np.linalg.norm(ref.numpy())
    assert rel < 4e-3
    # bf16 conversion matches torch's round-to-nearest-even
    np.testing.assert_array_equal(Ab, torch.from_numpy(A).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
