"""TorchCL public API on the B200 GEMM engine.

Same surface as the reference's torchcl/api.py (to_opencl / to_cpu /
is_opencl_tensor / synchronize, zeros/ones/full/randn, lazy elementwise ops,
matmul, transpose) and the same device-tensor handle scheme: a CPU placeholder
tensor tagged with `_torchcl_id/_torchcl_shape/_torchcl_dtype`, whose buffer
lives in the weak map `_opencl_buffers` and returns to the pool when the handle
is garbage collected (api.py:29-79, 182-189).

What changes is the lazy graph (api.py:88-161):
  * `matmul` returns a *lazy GEMM* node instead of launching at once.
  * `add/sub/mul/div(gemm, X)` with X of shape [M, N] (or a [N] / [1, N] row
    bias) folds X into the GEMM epilogue, and unary ops on a lazy GEMM append to
    its epilogue chain (up to 8).  Materialising the node is ONE kernel launch
    with one store — the reference needs a GEMM launch plus the JIT's fused
    elementwise launch (jit/compiler.py:99-133) that re-reads C.
  * `transpose` returns a lazy transposed view; a GEMM consumes it through its
    descriptor (no copy), anything else materialises it with one transpose kernel.
  * every other lazy chain is executed by the fused elementwise kernel, exactly
    as the reference's `_create_lazy_unary/_create_lazy_binary` chains.
A node is a value: folding creates a new handle and leaves the old one lazy, so
materialising the old handle later computes its own (epilogue-free) GEMM.
Inputs may be float32, bfloat16 or float16; a GEMM returns its input dtype.
"""
from __future__ import annotations

import math
import threading
import weakref
from typing import Any

import numpy as np
import torch

from torchcl import _lib as L
from torchcl.ops.engine import get_engine, ojx_dtype
from torchcl.runtime.context import synchronize as _sync
from torchcl.runtime.memory import CLBuffer, get_buffer_pool, note_use

_opencl_buffers = weakref.WeakValueDictionary()
_buffer_lock = threading.RLock()
_tensor_id_counter = 0
_id_lock = threading.RLock()  # reentrant: a GC finalizer may run while it is held

_NOT_ON_DEVICE = "This tensor is not on the OpenCL device. Use torchcl.to_opencl(tensor) first."


def _cleanup_buffer(cl_buf: CLBuffer) -> None:
    try:
        get_buffer_pool().free(cl_buf)
    except Exception:
        pass


def _next_id() -> int:
    global _tensor_id_counter
    with _id_lock:
        _tensor_id_counter += 1
        return _tensor_id_counter


def _make_handle(shape: tuple, dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, int]:
    """A placeholder carrying the device tensor's identity, shape and dtype.

    The reference allocates torch.empty(shape) on the host (api.py:46-53); here the
    placeholder is a single element expanded to `shape`, so a 32768x32768 device
    tensor does not also cost 4 GiB of host memory.
    """
    shape = tuple(int(d) for d in shape)
    handle = torch.empty((), dtype=dtype).expand(shape) if shape else torch.empty((), dtype=dtype)
    tid = _next_id()
    handle._torchcl_id = tid
    handle._torchcl_shape = shape
    handle._torchcl_dtype = dtype
    return handle, tid


def _elem(t):
    return t._elem if hasattr(t, "_elem") else t


def _wrap(handle: torch.Tensor):
    from torchcl.tensor import OjasXTensor
    return OjasXTensor(handle)


def _is_lazy(tensor) -> bool:
    return getattr(_elem(tensor), "_lazy_inputs", None) is not None


def _lazy_type(tensor) -> str | None:
    return getattr(_elem(tensor), "_lazy_op_type", None) if _is_lazy(tensor) else None


def _get_shape(tensor) -> tuple:
    e = _elem(tensor)
    s = getattr(e, "_torchcl_shape", None)
    return s if s is not None else tuple(e.shape)


def _get_dtype(tensor) -> torch.dtype:
    e = _elem(tensor)
    d = getattr(e, "_torchcl_dtype", None)
    return d if d is not None else e.dtype


def _get_buf(tensor) -> CLBuffer:
    """The device buffer of a handle, materialising a lazy node (or finishing a
    deferred upload) first."""
    e = _elem(tensor)
    tid = getattr(e, "_torchcl_id", None)
    if tid is not None:
        with _buffer_lock:
            buf = _opencl_buffers.get(tid)
        if buf is None and getattr(e, "_torchcl_host", None) is not None:
            buf = _finish_upload(e)
        if buf is None and _is_lazy(e):
            materialize_lazy_tensor(e)
            buf = _opencl_buffers[tid]
        if buf is not None:
            note_use(buf)  # a graph being captured must keep this buffer
            return buf
    raise ValueError(_NOT_ON_DEVICE)


def _wrap_output(cl_buf: CLBuffer, shape: tuple, dtype: torch.dtype = torch.float32):
    handle, tid = _make_handle(shape, dtype)
    with _buffer_lock:
        _opencl_buffers[tid] = cl_buf
    weakref.finalize(handle, _cleanup_buffer, cl_buf)
    return _wrap(handle)


def is_opencl_tensor(tensor: Any) -> bool:
    if tensor is None or not isinstance(tensor, torch.Tensor):
        return False
    e = _elem(tensor)
    tid = getattr(e, "_torchcl_id", None)
    if tid is None:
        return False
    with _buffer_lock:
        return (tid in _opencl_buffers or _is_lazy(e)
                or getattr(e, "_torchcl_host", None) is not None)


# ── lazy nodes ───────────────────────────────────────────────────────────

# Lazy nodes created while a graph is captured (weak references, creation order);
# torchcl.jit.graph_runner materialises the live ones before the capture ends.
_capture_lazy: list | None = None


def _new_lazy(shape, dtype, op_type: str, inputs: list, **attrs):
    handle, _ = _make_handle(shape, dtype)
    handle._lazy_inputs = inputs
    handle._lazy_op_type = op_type
    handle._lazy_ops = list(attrs.pop("ops", []))
    for k, v in attrs.items():
        setattr(handle, k, v)
    if _capture_lazy is not None:
        _capture_lazy.append(weakref.ref(handle))
    return _wrap(handle)


def _create_lazy_unary(op_name: str, a):
    if op_name not in L.UNARY:
        raise ValueError(f"Unknown unary op for fusion: {op_name}")
    ae = _elem(a)
    shape, dtype = _get_shape(ae), _get_dtype(ae)
    kind = _lazy_type(ae)
    if kind == "gemm" and len(ae._lazy_ops) < L.MAX_UNARY:
        # fold into the GEMM epilogue
        return _new_lazy(shape, dtype, "gemm", list(ae._lazy_inputs), ops=ae._lazy_ops + [op_name],
                         _lazy_gemm=dict(ae._lazy_gemm))
    if kind in ("unary", "binary_then_unary") and len(ae._lazy_ops) < L.MAX_UNARY:
        attrs = {"ops": ae._lazy_ops + [op_name]}
        if kind == "binary_then_unary":
            attrs["_lazy_binary_op"] = ae._lazy_binary_op
        return _new_lazy(shape, dtype, kind, list(ae._lazy_inputs), **attrs)
    if _is_lazy(ae):
        materialize_lazy_tensor(ae)
    return _new_lazy(shape, dtype, "unary", [ae], ops=[op_name])


def _operand_kind_for(operand_shape: tuple, out_shape: tuple) -> str | None:
    M, N = out_shape
    if tuple(operand_shape) == (M, N):
        return "full"
    if tuple(operand_shape) in ((N,), (1, N)):
        return "row"
    return None


def _fold_into_gemm(op_name: str, gemm_e, other_e, lhs: bool):
    g = gemm_e._lazy_gemm
    if g.get("operand") is not None or gemm_e._lazy_ops:
        return None
    kind = _operand_kind_for(_get_shape(other_e), _get_shape(gemm_e))
    if kind is None:
        return None
    if _is_lazy(other_e):
        materialize_lazy_tensor(other_e)
    ng = dict(g)
    ng.update(operand=other_e, operand_kind=kind, binary=op_name, operand_is_lhs=lhs)
    return _new_lazy(_get_shape(gemm_e), _get_dtype(gemm_e), "gemm", list(gemm_e._lazy_inputs),
                     ops=[], _lazy_gemm=ng)


def _create_lazy_binary(op_name: str, a, b):
    if op_name not in L.BINARY:
        raise ValueError(f"Unknown binary op for fusion: {op_name}")
    ae, be = _elem(a), _elem(b)
    if _lazy_type(ae) == "gemm":
        r = _fold_into_gemm(op_name, ae, be, lhs=False)
        if r is not None:
            return r
    if _lazy_type(be) == "gemm":
        r = _fold_into_gemm(op_name, be, ae, lhs=True)
        if r is not None:
            return r
    if _is_lazy(ae):
        materialize_lazy_tensor(ae)
    if _is_lazy(be):
        materialize_lazy_tensor(be)
    sa, sb = _get_shape(ae), _get_shape(be)
    if math.prod(sa) != math.prod(sb):
        # The reference reads b[i] for every i < numel(a) (jit/compiler.py:190-193), which
        # is out of bounds when b is smaller; that case is rejected here.
        raise ValueError(f"elementwise {op_name}: shapes {sa} and {sb} differ in size")
    return _new_lazy(sa, _get_dtype(ae), "binary_then_unary", [ae, be], ops=[],
                     _lazy_binary_op=op_name)


def _gemm_source(t) -> tuple[Any, bool]:
    """(stored handle, transposed?) of a GEMM input; lazy transposes become a flag."""
    e = _elem(t)
    if _lazy_type(e) == "transpose":
        return e._lazy_inputs[0], True
    return e, False


def _materialize_gemm(e) -> CLBuffer:
    engine = get_engine()
    g = e._lazy_gemm
    a_src, ta = _gemm_source(e._lazy_inputs[0])
    b_src, tb = _gemm_source(e._lazy_inputs[1])
    a_buf, b_buf = _get_buf(a_src), _get_buf(b_src)
    M, N = _get_shape(e)
    K = g["K"]
    dtype = _get_dtype(e)
    operand = g.get("operand")
    op_buf = _get_buf(operand) if operand is not None else None
    op_dtype = _get_dtype(operand) if operand is not None else None
    kw = dict(trans_a=ta, trans_b=tb, operand=op_buf, operand_kind=g.get("operand_kind"),
              operand_dtype=op_dtype, binary=g.get("binary", "add"),
              operand_is_lhs=g.get("operand_is_lhs", False), unary=e._lazy_ops,
              fp32_mode=g.get("fp32_mode", L.FP32_AUTO))
    if g.get("precision") == "half" and dtype == torch.float32:
        # The reference's forced-fp16 route (api.py:449-461): pack to half, half GEMM,
        # unpack to fp32.  Here: cast kernels + the tcgen05 f16 GEMM.
        pool = get_buffer_pool()
        ka = M * K
        a16 = pool.allocate(ka * 2, torch.float16)
        b16 = pool.allocate(K * N * 2, torch.float16)
        c16 = pool.allocate(M * N * 2, torch.float16)
        engine.run_cast(a16, torch.float16, a_buf, _get_dtype(a_src), ka)
        engine.run_cast(b16, torch.float16, b_buf, _get_dtype(b_src), K * N)
        engine.gemm(a16, b16, c16, M, N, K, dtype_a=torch.float16, dtype_b=torch.float16,
                    dtype_c=torch.float16, **kw)
        out = engine.allocate_output((M, N), torch.float32)
        engine.run_cast(out, torch.float32, c16, torch.float16, M * N)
        for tmp in (a16, b16, c16):
            pool.free(tmp)
        return out
    out = engine.allocate_output((M, N), dtype)
    engine.gemm(a_buf, b_buf, out, M, N, K, dtype_a=_get_dtype(a_src), dtype_b=_get_dtype(b_src),
                dtype_c=dtype, **kw)
    return out


def materialize_lazy_tensor(tensor) -> None:
    e = _elem(tensor)
    with _buffer_lock:
        if e._torchcl_id in _opencl_buffers:
            return
    kind = e._lazy_op_type
    engine = get_engine()
    shape, dtype = _get_shape(e), _get_dtype(e)
    if kind == "gemm":
        out_buf = _materialize_gemm(e)
    elif kind == "transpose":
        src = e._lazy_inputs[0]
        sbuf = _get_buf(src)
        r, c = _get_shape(src)
        out_buf = engine.allocate_output(shape, dtype)
        engine.run_transpose(sbuf, out_buf, r, c, dtype=dtype)
    else:
        for inp in e._lazy_inputs:
            if _is_lazy(inp):
                materialize_lazy_tensor(inp)
        from torchcl.jit.compiler import get_jit_compiler
        jit = get_jit_compiler()
        n = int(np.prod(shape)) if shape else 1
        out_buf = engine.allocate_output(shape, dtype)
        if kind == "unary":
            src = e._lazy_inputs[0]
            jit.fuse_elementwise_chain(e._lazy_ops, n, [_get_buf(src).buffer], out_buf.buffer,
                                       dtypes=(_get_dtype(src), dtype))
        elif kind == "binary_then_unary":
            a, b = e._lazy_inputs
            jit.fuse_binary_then_unary(e._lazy_binary_op, e._lazy_ops, n, _get_buf(a).buffer,
                                       _get_buf(b).buffer, out_buf.buffer,
                                       dtypes=(_get_dtype(a), _get_dtype(b), dtype))
        else:
            raise RuntimeError(f"unknown lazy node {kind}")
    with _buffer_lock:
        _opencl_buffers[e._torchcl_id] = out_buf
    weakref.finalize(e, _cleanup_buffer, out_buf)


# ── data movement ───────────────────────────────────────────────────────

# A pinned host tensor of at least this many bytes is uploaded when its data is
# first needed (see to_opencl) rather than at once.
DEFERRED_UPLOAD_MIN_BYTES = 1 << 20


def to_opencl(tensor: torch.Tensor):
    """Copy a CPU tensor (float32 / bfloat16 / float16) to the device.

    A pageable tensor is copied at once, as the reference does (api.py:210-217).
    A contiguous pinned tensor (torch's pin_memory) of 1 MiB or more is instead read
    when its device data is first needed, which lets to_cpu() of a GEMM on it
    overlap the upload, the GEMM and the download chunk by chunk.  Such a tensor
    follows torch's non_blocking contract: leave it unmodified until the handle
    has been used (or torchcl.synchronize() has returned)."""
    if is_opencl_tensor(tensor):
        return tensor
    t = tensor.detach()
    if (t.device.type == "cpu" and t.is_contiguous() and _pinned(t)
            and t.numel() * t.element_size() >= DEFERRED_UPLOAD_MIN_BYTES
            and t.dtype in (torch.float32, torch.bfloat16, torch.float16)):
        handle, _ = _make_handle(tuple(t.shape), t.dtype)
        handle._torchcl_host = t
        return _wrap(handle)
    cl_buf = get_engine().tensor_to_buffer(tensor)
    return _wrap_output(cl_buf, tuple(tensor.shape), tensor.dtype)


def _pinned(t: torch.Tensor) -> bool:
    try:
        return bool(t.is_pinned())
    except RuntimeError:  # torch without a usable CUDA runtime: nothing is pinned
        return False


def _finish_upload(e) -> CLBuffer:
    """Upload a deferred handle's host tensor now (blocking) and register the buffer."""
    with _buffer_lock:
        buf = _opencl_buffers.get(e._torchcl_id)
        host = getattr(e, "_torchcl_host", None)
        if buf is not None or host is None:
            return buf
        buf = get_engine().tensor_to_buffer(host)
        _attach(e, buf)
        return buf


def _attach(e, cl_buf: CLBuffer) -> None:
    """Make cl_buf the device buffer of handle e (which had none)."""
    with _buffer_lock:
        _opencl_buffers[e._torchcl_id] = cl_buf
        if getattr(e, "_torchcl_host", None) is not None:
            e._torchcl_host = None
    weakref.finalize(e, _cleanup_buffer, cl_buf)


def _host_io_plan(e):
    """(A handle, B handle) when e is a lazy GEMM that to_cpu can run with A read
    from the host: A a deferred (pinned) upload used untransposed, B on the device
    or uploadable, no forced-half route, 16-bit or fp32 output.  Else None."""
    if _lazy_type(e) != "gemm" or len(_get_shape(e)) != 2:
        return None
    with _buffer_lock:
        if e._torchcl_id in _opencl_buffers:
            return None
    g = e._lazy_gemm
    if g.get("precision") == "half" and _get_dtype(e) == torch.float32:
        return None  # the forced fp16 route of fp32 inputs (casts around a half GEMM)
    a_src, ta = _gemm_source(e._lazy_inputs[0])
    if ta or getattr(a_src, "_torchcl_host", None) is None:
        return None
    return a_src, e._lazy_inputs[1]


def _to_cpu_host_io(e, a_src) -> torch.Tensor:
    """to_cpu of a lazy GEMM whose A waits in pinned host memory: one
    ojx_gemm_host_io call uploads A in row chunks, runs each chunk's fused GEMM and
    downloads each finished chunk into a pinned output while the next one uploads.
    A's handle keeps the uploaded copy and the node keeps its device result, as if
    both had been materialised."""
    engine = get_engine()
    pool = get_buffer_pool()
    g = e._lazy_gemm
    b_src, tb = _gemm_source(e._lazy_inputs[1])
    b_buf = _get_buf(b_src)
    operand = g.get("operand")
    op_buf = _get_buf(operand) if operand is not None else None
    M, N = _get_shape(e)
    K = g["K"]
    dtype = _get_dtype(e)
    host_a = a_src._torchcl_host
    try:
        out = torch.empty((M, N), dtype=dtype, pin_memory=True)
    except RuntimeError:
        out = torch.empty((M, N), dtype=dtype)
    dev_a = pool.allocate(host_a.numel() * host_a.element_size(), host_a.dtype, tuple(host_a.shape))
    dev_c = engine.allocate_output((M, N), dtype)
    try:
        engine.gemm_host_io(host_a.data_ptr(), b_buf, out.data_ptr(), dev_a, dev_c, M, N, K,
                            dtype_a=host_a.dtype, dtype_b=_get_dtype(b_src), dtype_c=dtype,
                            trans_b=tb, operand=op_buf, operand_kind=g.get("operand_kind"),
                            operand_dtype=_get_dtype(operand) if operand is not None else None,
                            binary=g.get("binary", "add"),
                            operand_is_lhs=g.get("operand_is_lhs", False), unary=e._lazy_ops,
                            fp32_mode=g.get("fp32_mode", L.FP32_AUTO))
        _sync()
    except Exception:
        pool.free(dev_a)
        pool.free(dev_c)
        raise
    _attach(a_src, dev_a)
    _attach(e, dev_c)
    return out


def to_cpu(tensor):
    """Copy a device tensor back to a CPU torch tensor (materialising it first).

    For a lazy GEMM whose A is a deferred pinned upload (to_opencl of a pinned
    tensor), the upload, the fused GEMM and the download run as one overlapped
    pipeline, and the result is returned in pinned memory."""
    if tensor is None:
        return None
    e = _elem(tensor)
    if not is_opencl_tensor(e):
        return tensor
    plan = _host_io_plan(e)
    if plan is not None:
        return _to_cpu_host_io(e, plan[0])
    return get_engine().buffer_to_tensor(_get_buf(e), _get_shape(e), _get_dtype(e))


def synchronize() -> None:
    _sync()


# ── creation ────────────────────────────────────────────────────────────

def _shape_args(shape):
    if len(shape) == 1 and isinstance(shape[0], (tuple, list, torch.Size)):
        return tuple(shape[0])
    return tuple(shape)


def full(*shape, fill_value: float, dtype: torch.dtype = torch.float32):
    shape = _shape_args(shape)
    engine = get_engine()
    buf = engine.allocate_output(shape, dtype)
    engine.run_fill(buf, fill_value, math.prod(shape) if shape else 1, dtype=dtype)
    return _wrap_output(buf, shape, dtype)


def zeros(*shape, dtype: torch.dtype = torch.float32):
    return full(*shape, fill_value=0.0, dtype=dtype)


def ones(*shape, dtype: torch.dtype = torch.float32):
    return full(*shape, fill_value=1.0, dtype=dtype)


def zeros_like(tensor, dtype: torch.dtype | None = None):
    return zeros(_get_shape(tensor), dtype=dtype or _get_dtype(tensor))


def ones_like(tensor, dtype: torch.dtype | None = None):
    return ones(_get_shape(tensor), dtype=dtype or _get_dtype(tensor))


def randn(*shape, dtype: torch.dtype = torch.float32):
    return to_opencl(torch.randn(*_shape_args(shape), dtype=dtype))


# ── elementwise (lazy) ──────────────────────────────────────────────────

def _require(*ts):
    for t in ts:
        if not is_opencl_tensor(t):
            raise ValueError(_NOT_ON_DEVICE)


def add(a, b):
    _require(a, b)
    return _create_lazy_binary("add", a, b)


def sub(a, b):
    _require(a, b)
    return _create_lazy_binary("sub", a, b)


def mul(a, b):
    _require(a, b)
    return _create_lazy_binary("mul", a, b)


def div(a, b):
    _require(a, b)
    return _create_lazy_binary("div", a, b)


def _unary_api(name):
    def fn(a):
        _require(a)
        return _create_lazy_unary(name, a)
    fn.__name__ = name
    return fn


neg = _unary_api("neg")
abs_ = _unary_api("abs")
exp = _unary_api("exp")
log = _unary_api("log")
sqrt = _unary_api("sqrt")
relu = _unary_api("relu")
sigmoid = _unary_api("sigmoid")
tanh_ = _unary_api("tanh")
gelu = _unary_api("gelu")
silu = _unary_api("silu")
square = _unary_api("square")


# ── matrix ops ──────────────────────────────────────────────────────────

def matmul(a, b):
    """C = A @ B as a lazy GEMM node (api.py:427-469 validation and dtype routing).

    fp32 inputs give an fp32 result (3xTF32 on tcgen05, or FFMA for small M);
    bf16/fp16 inputs give a bf16/fp16 result with fp32 accumulation.
    """
    _require(a, b)
    a_shape, b_shape = _get_shape(a), _get_shape(b)
    if len(a_shape) != 2 or len(b_shape) != 2:
        raise ValueError(f"matmul requires 2D tensors, got {a_shape} and {b_shape}")
    M, K = a_shape
    K2, N = b_shape
    if K != K2:
        raise ValueError(f"matmul dimension mismatch: {a_shape} @ {b_shape}")
    da, db = _get_dtype(a), _get_dtype(b)
    if da != db:
        raise ValueError(f"matmul dtype mismatch: {da} @ {db}")
    ojx_dtype(da)
    from torchcl.liquid.dispatch import get_dispatcher
    config = get_dispatcher().dispatch("matmul", a)
    ae, be = _elem(a), _elem(b)
    if _lazy_type(ae) not in (None, "transpose"):
        materialize_lazy_tensor(ae)
    if _lazy_type(be) not in (None, "transpose"):
        materialize_lazy_tensor(be)
    g = {"K": int(K), "precision": config.precision}
    return _new_lazy((M, N), da, "gemm", [ae, be], ops=[], _lazy_gemm=g)


def transpose(a):
    """A^T as a lazy view (api.py:472-482); consumed by GEMMs without a copy."""
    _require(a)
    shape = _get_shape(a)
    if len(shape) != 2:
        raise ValueError(f"transpose requires 2D tensor, got {shape}")
    ae = _elem(a)
    if _lazy_type(ae) == "transpose":
        return _wrap(ae._lazy_inputs[0])
    if _is_lazy(ae):
        materialize_lazy_tensor(ae)
    return _new_lazy((shape[1], shape[0]), _get_dtype(ae), "transpose", [ae])


def fused_attention(q, k, v, scale: float | None = None, is_causal: bool = False,
                    max_keys: int | None = None, composed: bool = False):
    """Scaled dot-product attention (api.py:667-695): Q [B, H, M, D], K and V
    [B, H, N, D] -> [B, H, M, D] in Q's dtype.  `max_keys=2048` reproduces the
    reference kernel, which only sees the first 2048 keys (flash_attention.cl:6);
    the default uses every key.  `composed=True` forces the GEMM + softmax + GEMM
    path where the fused kernel would run (tests compare the two)."""
    for t in (q, k, v):
        if not is_opencl_tensor(t):
            raise ValueError(_NOT_ON_DEVICE)
    qs, ks, vs = _get_shape(q), _get_shape(k), _get_shape(v)
    if len(qs) != 4 or len(ks) != 4 or ks != vs or qs[:2] != ks[:2] or qs[3] != ks[3]:
        raise ValueError(f"fused_attention: shapes {qs}, {ks}, {vs} do not match [B,H,M,D] / [B,H,N,D]")
    dt = _get_dtype(q)
    if _get_dtype(k) != dt or _get_dtype(v) != dt:
        raise ValueError("fused_attention: q, k and v must share a dtype")
    B, H, M, D = qs
    N = ks[2]
    if scale is None:
        scale = D ** -0.5
    engine = get_engine()
    out = engine.allocate_output((B, H, M, D), dt)
    engine.run_fused_attention(_get_buf(q), _get_buf(k), _get_buf(v), out, B, H, M, N, D, scale,
                               is_causal=is_causal, dtype=dt, max_keys=max_keys or 0,
                               composed=composed)
    return _wrap_output(out, (B, H, M, D), dt)


def linear(x, weight, bias=None):
    """x @ weight^T (+ bias) — the reference's run_linear (engine.py:351-392) as one GEMM."""
    out = matmul(x, transpose(weight))
    return add(out, bias) if bias is not None else out
