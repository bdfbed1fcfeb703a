"""OjasXTensor — the wrapper subclass the reference returns from every op
(torchcl/tensor.py:95-144), with its ATen routing (tensor.py:39-90) reduced to the
GEMM path: aten.mm / addmm / linear-shaped calls and the elementwise ops that fold
into a GEMM epilogue run on the device; any other ATen op runs on the CPU and the
result is copied back, as the reference's execute_on_cpu does.  There is no
silent CPU fallback for a GEMM: a device error raises.
"""
from __future__ import annotations

import torch

import torchcl.api as api

aten = torch.ops.aten


def _unwrap(x):
    return x._elem if isinstance(x, OjasXTensor) else x


def _gelu(x, approximate="none"):
    if approximate != "tanh":
        return NotImplemented
    return api.gelu(x)


def _addmm(bias, m1, m2, beta=1, alpha=1):
    if beta != 1 or alpha != 1:
        return NotImplemented
    return api.add(api.matmul(m1, m2), bias)


def _binary(fn):
    def op(a, b, alpha=1):
        if alpha != 1 or not isinstance(b, torch.Tensor) or not isinstance(a, torch.Tensor):
            return NotImplemented
        return fn(a, b)
    return op


def _transpose(a, d0=0, d1=1):
    if sorted((d0 % 2, d1 % 2)) != [0, 1] or len(api._get_shape(a)) != 2:
        return NotImplemented
    return api.transpose(a)


DISPATCH_TABLE = {
    aten.mm.default: api.matmul,
    aten.addmm.default: _addmm,
    aten.t.default: api.transpose,
    aten.transpose.int: _transpose,
    aten.add.Tensor: _binary(api.add),
    aten.sub.Tensor: _binary(api.sub),
    aten.mul.Tensor: lambda a, b: api.mul(a, b) if isinstance(b, torch.Tensor) else NotImplemented,
    aten.div.Tensor: lambda a, b: api.div(a, b) if isinstance(b, torch.Tensor) else NotImplemented,
    aten.neg.default: api.neg,
    aten.abs.default: api.abs_,
    aten.exp.default: api.exp,
    aten.log.default: api.log,
    aten.sqrt.default: api.sqrt,
    aten.relu.default: api.relu,
    aten.sigmoid.default: api.sigmoid,
    aten.tanh.default: api.tanh_,
    aten.gelu.default: _gelu,
    aten.silu.default: api.silu,
}


def execute_on_cpu(func, *args, **kwargs):
    """Run an ATen op the device path does not cover on CPU copies (tensor.py:61-78)."""
    def to_host(x):
        return api.to_cpu(x._elem) if isinstance(x, OjasXTensor) else x

    cpu_args = torch.utils._pytree.tree_map(to_host, args)
    cpu_kwargs = torch.utils._pytree.tree_map(to_host, kwargs)
    res = func(*cpu_args, **cpu_kwargs)

    def to_dev(x):
        if isinstance(x, torch.Tensor) and x.dtype in (torch.float32, torch.bfloat16, torch.float16):
            return OjasXTensor(api._elem(api.to_opencl(x.contiguous())))
        return x

    return torch.utils._pytree.tree_map(to_dev, res)


def dispatch_op(func, *args, **kwargs):
    fn = DISPATCH_TABLE.get(func)
    if fn is not None:
        res = fn(*args, **kwargs)
        if res is not NotImplemented:
            return res
    return execute_on_cpu(func, *args, **kwargs)


class OjasXTensor(torch.Tensor):
    """A device-tensor handle visible to PyTorch as a tensor of the right shape."""

    @staticmethod
    def __new__(cls, elem):
        if isinstance(elem, cls):
            return elem
        size = tuple(getattr(elem, "_torchcl_shape", elem.size()))
        strides, acc = [], 1
        for d in reversed(size):
            strides.append(acc)
            acc *= max(int(d), 1)
        r = torch.Tensor._make_wrapper_subclass(cls, size, strides=tuple(reversed(strides)),
                                                storage_offset=0, dtype=elem.dtype,
                                                layout=elem.layout, device=torch.device("cpu"),
                                                requires_grad=elem.requires_grad)
        r._elem = elem
        return r

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        return dispatch_op(func, *args, **(kwargs or {}))

    def __getattr__(self, name):
        if name in ("_torchcl_id", "_torchcl_shape", "_torchcl_dtype", "_lazy_inputs",
                    "_lazy_op_type", "_lazy_binary_op", "_lazy_ops", "_lazy_gemm"):
            return getattr(self._elem, name)
        raise AttributeError(f"'{type(self).__name__}' object has no attribute '{name}'")

    def __repr__(self):
        return f"OjasXTensor(shape={tuple(self.shape)}, dtype={self.dtype}, device='opencl')"
