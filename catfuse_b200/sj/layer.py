"""Multi-step aware layer wrappers: in step_mode 'm' the [T, B] leading dims
are folded into the batch for the wrapped stateless layer."""
from __future__ import annotations

import torch
import torch.nn as nn

from .base import StepModule


class _SeqMixin(StepModule):
    def _init_step(self, step_mode):
        self._step_mode = step_mode

    def forward(self, x):
        if self.step_mode == "s":
            return super().forward(x)
        T, B = x.shape[:2]
        y = super().forward(x.flatten(0, 1))
        return y.reshape(T, B, *y.shape[1:])


class Conv2d(_SeqMixin, nn.Conv2d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.Conv2d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class BatchNorm2d(_SeqMixin, nn.BatchNorm2d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.BatchNorm2d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class BatchNorm1d(_SeqMixin, nn.BatchNorm1d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.BatchNorm1d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class Linear(_SeqMixin, nn.Linear):
    def __init__(self, *args, step_mode="s", **kw):
        nn.Linear.__init__(self, *args, **kw)
        self._init_step(step_mode)

    def forward(self, x):  # Linear is shape-agnostic over leading dims
        return nn.Linear.forward(self, x)


class MaxPool2d(_SeqMixin, nn.MaxPool2d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.MaxPool2d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class AvgPool2d(_SeqMixin, nn.AvgPool2d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.AvgPool2d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class AdaptiveAvgPool2d(_SeqMixin, nn.AdaptiveAvgPool2d):
    def __init__(self, *args, step_mode="s", **kw):
        nn.AdaptiveAvgPool2d.__init__(self, *args, **kw)
        self._init_step(step_mode)


class Flatten(_SeqMixin, nn.Flatten):
    def __init__(self, *args, step_mode="s", **kw):
        nn.Flatten.__init__(self, *args, **kw)
        self._init_step(step_mode)
