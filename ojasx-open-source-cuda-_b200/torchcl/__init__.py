"""torchcl on NVIDIA B200 (sm_100a).

Drop-in for the OjasX `torchcl` GEMM path: the same Python surface (to_opencl /
to_cpu handles, lazy elementwise ops, matmul, transpose, blas.gemm, streams and
events) backed by libojx.so — hand-written tcgen05/TMA/TMEM GEMM kernels with the
bias/activation epilogue fused before the single store, a split-K skinny kernel
for decode shapes, a caching cudaMalloc pool and CUDA streams.

The device is initialised on first use (not at import), so the package imports on
machines without a GPU; any device call there raises RuntimeError.
"""
__version__ = "0.2.0"

from torchcl.runtime.context import (
    init_opencl, init, get_device_info, get_context, get_queue, get_device, synchronize,
    is_available,
)
from torchcl.runtime.stream import Stream, Event, stream, current_stream, default_stream
from torchcl.api import (
    to_opencl, to_cpu, is_opencl_tensor,
    zeros, zeros_like, ones, ones_like, full, randn,
    add, sub, mul, div, neg, abs_, exp, log, sqrt, square,
    relu, sigmoid, tanh_, gelu, silu,
    matmul, transpose, linear, fused_attention,
)
from torchcl import blas  # noqa: E402

__all__ = [
    "get_device_info", "is_available", "synchronize", "init_opencl", "init",
    "to_opencl", "to_cpu", "is_opencl_tensor",
    "zeros", "zeros_like", "ones", "ones_like", "full", "randn",
    "add", "sub", "mul", "div", "neg", "abs_", "exp", "log", "sqrt", "square",
    "relu", "sigmoid", "tanh_", "gelu", "silu",
    "matmul", "transpose", "linear", "fused_attention", "blas",
    "Stream", "Event", "stream", "current_stream", "default_stream",
]
