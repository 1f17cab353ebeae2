"""Adam for the example fits (MLXDiffRastExamples/Adam.swift), as one fused
CUDA pass per step (dr_adam_step) that updates the parameter in place."""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _lib as L
from .ops import _ctx, _f32, _ptr


class Adam:
    """Adam.swift:9-44: state m, v (zeros) and the step count t on the
    instance; bias-corrected update with PyTorch's defaults.  `step` updates
    `param` in place (and returns it); `mask`, if given, multiplies the
    gradient first, as the examples do with their x/y-only position masks."""

    def __init__(self, shape, learning_rate: float = 1e-2, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, device: Optional[torch.device] = None):
        self.learning_rate = float(learning_rate)
        self.beta1, self.beta2, self.eps = float(beta1), float(beta2), float(eps)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.m = torch.zeros(tuple(shape), dtype=torch.float32, device=dev)
        self.v = torch.zeros(tuple(shape), dtype=torch.float32, device=dev)
        self.t = 0

    def bias_corrections(self):
        """(1 - beta1^t, 1 - beta2^t) in float32, as the reference's Float pow."""
        b1, b2, t = np.float32(self.beta1), np.float32(self.beta2), np.float32(self.t)
        return float(np.float32(1) - np.power(b1, t)), float(np.float32(1) - np.power(b2, t))

    def step(self, param: torch.Tensor, grad: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if tuple(param.shape) != tuple(self.m.shape) or tuple(grad.shape) != tuple(self.m.shape):
            raise ValueError(f"adam: param/grad shape must be {tuple(self.m.shape)}")
        if not (param.is_contiguous() and param.dtype == torch.float32):
            raise ValueError("adam: param must be a contiguous float32 tensor (updated in place)")
        g = _f32(grad, "grad")
        mk = _f32(mask.expand_as(param), "mask") if mask is not None else None
        self.t += 1
        c1, c2 = self.bias_corrections()
        c = _ctx(param)
        L.check(L.lib().dr_adam_step(c, _ptr(param), _ptr(g), _ptr(mk), _ptr(self.m), _ptr(self.v), param.numel(),
                                     self.learning_rate, self.beta1, self.beta2, self.eps, c1, c2), c, "adam")
        return param
