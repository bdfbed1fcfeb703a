"""Layers of the GEMM path — replaces OpenCLLinear of torchcl/nn.py:58-119.

Same constructor (in_features, out_features, bias; Kaiming-uniform weights as
torch.nn.Linear), same lazy upload of the parameters on the first forward.  The
reference's forward materialises weight^T with a transpose kernel, runs a GEMM,
then adds the bias with a third launch (nn.py:104-118); here the forward is one
GEMM that reads the [out, in] weight transposed through its descriptor and adds
the bias in the epilogue (LinearFunction).
"""
from __future__ import annotations

import math

import torch
from torch import nn

from torchcl.api import _get_shape, is_opencl_tensor, to_opencl
from torchcl.autograd import LinearFunction


class OpenCLLinear(nn.Module):
    """output = input @ weight.T + bias on the device."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        k = 1.0 / math.sqrt(in_features)
        self.weight = nn.Parameter(torch.empty(out_features, in_features).uniform_(-k, k))
        self.bias = nn.Parameter(torch.empty(out_features).uniform_(-k, k)) if bias else None
        self._weight_gpu = None
        self._bias_gpu = None

    def _ensure_on_gpu(self) -> None:
        """Upload weight and bias on first use (nn.py:83-89)."""
        if self._weight_gpu is None or not is_opencl_tensor(self._weight_gpu):
            self._weight_gpu = to_opencl(self.weight.data)
        if self.bias is not None and (self._bias_gpu is None or not is_opencl_tensor(self._bias_gpu)):
            self._bias_gpu = to_opencl(self.bias.data)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._ensure_on_gpu()
        x_shape = _get_shape(x) if is_opencl_tensor(x) else tuple(x.shape)
        if len(x_shape) != 2:
            raise ValueError(f"OpenCLLinear expects 2D input, got shape {x_shape}")
        if x_shape[1] != self.in_features:
            raise ValueError(f"Expected input feature size {self.in_features}, got {x_shape[1]}")
        return LinearFunction.apply(x, self._weight_gpu, self._bias_gpu)


__all__ = ["OpenCLLinear"]
