"""Generate the golden fixtures in tests/golden/ from the OjasX reference itself.

    python tests/golden/make_golden.py [--ref-root <OjasX checkout>]

Run in the development container (the reference tree is not present on GPU boxes;
the fixtures it writes are committed).  Two sources of truth are used:

1. The reference's OpenCL C kernels (torchcl/kernels/matmul.cl, activation.cl,
   precision.cl, reduction.cl, winograd_gemm.cl, flash_attention.cl), compiled for the host by oracle/build_oracle.py through
   oracle/ref_harness/clshim.h and launched with torchcl/ops/engine.py's geometry.
2. The reference's JIT code generator: torchcl.jit.compiler.JITCompiler is imported
   from the reference tree (with a stand-in `pyopencl` module, since pyopencl is not
   installed; the generator itself never touches it), its
   `_generate_fused_unary_source` / `_generate_fused_binary_unary_source` produce the
   OpenCL source text, and that text is compiled through the same shim.  The
   generated source is only kept in a temporary directory.

Each case stores seeded inputs and the outputs of both host builds: "nofma"
(-ffp-contract=off) and "fma" (-ffp-contract=fast), the two ends of what an OpenCL
compiler may do with `sum += a * b`.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import pathlib
import sys
import tempfile
import types

import numpy as np

REPO = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from oracle import build_oracle  # noqa: E402
from oracle.oracle import RefKernels  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent


def _torch_randn(seed: int, *shape) -> np.ndarray:
    import torch
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).numpy()


def gemm_cases(R: dict) -> dict:
    cases = {}
    # tests/test_cuda_correctness_baseline.py:54-69 (seed 303, 64x128 @ 128x64)
    A, B = _torch_randn(303, 64, 128), _torch_randn(304, 128, 64)
    cases["baseline_matmul_303"] = dict(kernel="reg_tiled", A=A, B=B)
    # tests/test_ojas_blas.py:11-23 (seed 42, gemm + bias + relu)
    A, B, bias = _torch_randn(42, 64, 128), _torch_randn(43, 128, 64), _torch_randn(44, 64)
    cases["blas_gemm_bias_relu_42"] = dict(kernel="reg_tiled", A=A, B=B, bias=bias, act="relu")
    # BASELINE config 1 shape at reduced K (512 x 512 @ 512 x 512 + bias, relu)
    A, B, bias = _torch_randn(0, 512, 512), _torch_randn(1, 512, 512), _torch_randn(2, 512)
    cases["cfg1_512_bias_relu"] = dict(kernel="reg_tiled", A=A, B=B, bias=bias, act="relu")
    # ragged shapes through the register-tiled and naive kernels
    A, B = _torch_randn(5, 33, 65), _torch_randn(6, 65, 47)
    cases["ragged_33x65x47"] = dict(kernel="reg_tiled", A=A, B=B)
    A, B, bias = _torch_randn(7, 4, 256), _torch_randn(8, 256, 300), _torch_randn(9, 300)
    cases["naive_bias_4x256x300"] = dict(kernel="naive", A=A, B=B, bias=bias, act="silu")
    # linear_forward_tiled_f32: A[M,K] @ W[N,K]^T + bias
    A, W, bias = _torch_randn(10, 40, 72), _torch_randn(11, 56, 72), _torch_randn(12, 56)
    cases["linear_40x72x56"] = dict(kernel="linear", A=A, B=W, bias=bias)
    out = {}
    for name, c in cases.items():
        rec = {k: v for k, v in c.items() if isinstance(v, np.ndarray)}
        for variant, rk in R.items():
            if c["kernel"] == "linear":
                C = rk.linear(c["A"], c["B"], c.get("bias"))
            else:
                C = rk.matmul(c["A"], c["B"], c["kernel"], bias=c.get("bias"))
            if c.get("act"):
                C = rk.activation(c["act"], C)
            rec[f"C_{variant}"] = C
        rec["meta"] = np.array([c["kernel"], c.get("act") or ""])
        out[name] = rec
    # matmul_tiled_fp16 (tests/test_mixed_precision_flow.py:7-51 shape 32^3)
    A, B = _torch_randn(50, 32, 32), _torch_randn(51, 32, 32)
    rk = R["nofma"]
    A16, B16 = rk.pack_fp16(A), rk.pack_fp16(B)
    out["fp16_tiled_32"] = dict(A16=A16, B16=B16, **{f"C16_{v}": r.matmul_fp16(A16, B16)
                                                     for v, r in R.items()},
                                meta=np.array(["fp16", ""]))
    # transpose_f32 (tests/test_smoke.py:73-82 shape 16x32)
    X = _torch_randn(60, 16, 32)
    out["transpose_16x32"] = dict(A=X, T_nofma=R["nofma"].transpose(X), meta=np.array(["transpose", ""]))
    return out


def batched_cases(R: dict) -> dict:
    # tests/test_ojas_blas.py:55-66 (torch.manual_seed(42); A [4,32,64], B [4,64,32]) through
    # winograd_gemm.cl:91-119 matmul_batched_strided_f32, as blas.bmm launches it.
    import torch
    torch.manual_seed(42)
    A = torch.randn(4, 32, 64).numpy()
    B = torch.randn(4, 64, 32).numpy()
    return {"bmm_42": dict(A=A, B=B, **{f"C_{v}": r.bmm(A, B) for v, r in R.items()},
                           meta=np.array(["bmm", ""]))}


def attention_cases(R: dict) -> dict:
    # flash_attention.cl:8-187 through engine.py:755-773: the shapes of
    # tests/test_fused_attention.py:9 and tests/test_cuda_correctness_baseline.py:108-111,
    # a causal ragged case, and N > 2048 (the kernel's score buffer keeps 2048 keys).
    out = {}
    for seed, (B, H, M, N, D), causal in ((80, (2, 4, 32, 32, 64), False), (81, (2, 4, 16, 16, 32), False),
                                          (82, (1, 2, 40, 40, 48), True), (83, (1, 1, 5, 2100, 32), False)):
        q, k, v = _torch_randn(seed, B, H, M, D), _torch_randn(seed + 100, B, H, N, D), \
            _torch_randn(seed + 200, B, H, N, D)
        name = f"attention{'_causal' if causal else ''}_{B}x{H}x{M}x{N}x{D}"
        out[name] = dict(q=q, k=k, v=v, causal=np.array(causal),
                         **{f"out_{v_}": r.attention(q, k, v, causal=causal) for v_, r in R.items()},
                         meta=np.array(["attention", ""]))
    return out


def reduction_cases(R: dict) -> dict:
    # reduction.cl:170-181 sum_columns_f32: the bias gradient of LinearFunction.backward
    # (torchcl/autograd.py:404-408), on a ragged and a taller gradient.
    out = {}
    for seed, rows, cols in ((70, 257, 300), (71, 1024, 96)):
        X = _torch_randn(seed, rows, cols)
        out[f"sum_columns_{rows}x{cols}"] = dict(
            X=X, **{f"S_{v}": r.sum_columns(X) for v, r in R.items()},
            meta=np.array(["sum_columns", ""]))
    return out


def activation_cases(R: dict) -> dict:
    # tests/test_cuda_correctness_baseline.py:34-51 (seed 202, 10 000 randn)
    x = _torch_randn(202, 10000)
    rec = {"x": x}
    for v, rk in R.items():
        for name in ("relu", "sigmoid", "tanh", "gelu", "silu"):
            rec[f"{name}_{v}"] = rk.activation(name, x)
    return {"activations_202": rec}


def _import_reference_jit(ref_root: str):
    """Import torchcl.jit.compiler from the reference with a stand-in pyopencl."""
    stub = types.ModuleType("pyopencl")

    class _Anything:
        def __getattr__(self, name):
            return _Anything()

        def __call__(self, *a, **k):
            return _Anything()

    for attr in ("Buffer", "Kernel", "Program", "Context", "CommandQueue", "Event", "Device",
                 "Platform", "mem_flags", "device_type", "command_queue_properties",
                 "profiling_info", "event_info", "command_execution_status", "LocalMemory",
                 "MemoryError", "RuntimeError", "enqueue_copy", "get_platforms"):
        setattr(stub, attr, _Anything())
    stub.MemoryError = MemoryError
    stub.RuntimeError = RuntimeError
    stub.get_platforms = lambda: []
    sys.modules["pyopencl"] = stub
    saved = [m for m in list(sys.modules) if m == "torchcl" or m.startswith("torchcl.")]
    for m in saved:
        del sys.modules[m]
    sys.path.insert(0, ref_root)
    try:
        comp = importlib.import_module("torchcl.jit.compiler")
        return comp.JITCompiler.__new__(comp.JITCompiler)
    finally:
        sys.path.remove(ref_root)


def jit_cases(ref_root: str) -> dict:
    gen = _import_reference_jit(ref_root)
    n = 1024
    a, b = _torch_randn(70, n), _torch_randn(71, n)
    chains = {
        "unary_sigmoid_relu": (None, ["sigmoid", "relu"]),
        "unary_neg_exp": (None, ["neg", "exp"]),
        "unary_tanh_abs": (None, ["tanh", "abs"]),
        "unary_gelu": (None, ["gelu"]),
        "unary_silu_square": (None, ["silu", "square"]),
        "binary_add_relu": ("add", ["relu"]),
        "binary_mul_sigmoid": ("mul", ["sigmoid"]),
        "binary_sub_gelu": ("sub", ["gelu"]),
        "binary_div_tanh": ("div", ["tanh"]),
        "binary_add_silu": ("add", ["silu"]),
    }
    out = {"jit_inputs": {"a": a, "b": b}}
    with tempfile.TemporaryDirectory() as td:
        td = pathlib.Path(td)
        for name, (binop, ops) in chains.items():
            src = (gen._generate_fused_binary_unary_source(binop, ops) if binop
                   else gen._generate_fused_unary_source(ops))
            cl = td / f"{name}.cl"
            cl.write_text(src)
            rec = {"meta": np.array([binop or "", ",".join(ops)])}
            for variant, fma in (("nofma", False), ("fma", True)):
                so = build_oracle.build_ref_jit(cl, binop is not None, td / f"{name}_{variant}.so", fma)
                L = ctypes.CDLL(str(so))
                L.ref_jit_run.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
                o = np.zeros(n, dtype=np.float32)
                L.ref_jit_run(a.ctypes.data, b.ctypes.data if binop else None, o.ctypes.data, n)
                rec[f"out_{variant}"] = o
            out[name] = rec
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=build_oracle.DEFAULT_REF_ROOT)
    ap.add_argument("--only", default=None, help="write only the fixtures of one group "
                    "(gemm, activation, reduction, batched, attention, jit)")
    args = ap.parse_args()
    build_oracle.build_oracle()
    if not build_oracle.build_ref(args.ref_root):
        raise SystemExit(f"reference tree not found at {args.ref_root}")
    R = {"nofma": RefKernels("nofma"), "fma": RefKernels("fma")}
    groups = {"gemm": lambda: gemm_cases(R), "activation": lambda: activation_cases(R),
              "reduction": lambda: reduction_cases(R), "batched": lambda: batched_cases(R),
              "attention": lambda: attention_cases(R),
              "jit": lambda: jit_cases(args.ref_root)}
    fixtures = {}
    for name, make in groups.items():
        if args.only in (None, name):
            fixtures.update(make())
    for name, rec in fixtures.items():
        np.savez_compressed(OUT / f"{name}.npz", **rec)
    print(f"wrote {len(fixtures)} fixtures to {OUT}")


if __name__ == "__main__":
    main()
