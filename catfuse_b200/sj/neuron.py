"""Leaky integrate-and-fire neuron with SpikingJelly's ``LIFNode`` semantics.

charge:  decay_input: h = v + (x - (v - v_reset)) / tau
         otherwise  : h = v - (v - v_reset) / tau + x       (v_reset = 0 when soft)
fire:    s = heaviside(h - v_threshold)
reset:   hard: v = s ? v_reset : h        soft (v_reset None): v = h - s * v_threshold
"""
from __future__ import annotations

import torch

from .base import MemoryModule
from .surrogate import Sigmoid


class BaseNode(MemoryModule):
    def __init__(self, v_threshold=1.0, v_reset=0.0, surrogate_function=None, detach_reset=False,
                 step_mode="s", backend="torch", store_v_seq=False):
        super().__init__()
        self.v_threshold = v_threshold
        self.v_reset = v_reset
        self.register_memory("v", 0.0 if v_reset is None else v_reset)
        self.surrogate_function = surrogate_function or Sigmoid()
        self.detach_reset = detach_reset
        self.step_mode = step_mode
        self.backend = backend
        self.store_v_seq = store_v_seq

    def _init_v(self, x):
        if not isinstance(self.v, torch.Tensor) or self.v.shape != x.shape or self.v.device != x.device:
            self.v = torch.full_like(x, float(self.v))

    def _charge(self, x):
        raise NotImplementedError

    def single_step_forward(self, x):
        self._init_v(x)
        h = self._charge(x)
        s = (h >= self.v_threshold).to(x.dtype)
        if self.v_reset is None:
            self.v = h - s * self.v_threshold
        else:
            self.v = torch.where(s.bool(), torch.full_like(h, float(self.v_reset)), h)
        return s

    def multi_step_forward(self, x_seq):
        out = []
        v_seq = []
        for t in range(x_seq.shape[0]):
            out.append(self.single_step_forward(x_seq[t]))
            if self.store_v_seq:
                v_seq.append(self.v)
        if self.store_v_seq:
            self.v_seq = torch.stack(v_seq)
        return torch.stack(out)


class LIFNode(BaseNode):
    def __init__(self, tau=2.0, decay_input=True, v_threshold=1.0, v_reset=0.0,
                 surrogate_function=None, detach_reset=False, step_mode="s", backend="torch",
                 store_v_seq=False):
        if tau <= 1.0:
            raise ValueError("tau must be > 1")
        super().__init__(v_threshold, v_reset, surrogate_function, detach_reset, step_mode, backend,
                         store_v_seq)
        self.tau = tau
        self.decay_input = decay_input

    def _charge(self, x):
        vr = 0.0 if self.v_reset is None else self.v_reset
        if self.decay_input:
            return self.v + (x - (self.v - vr)) / self.tau
        return self.v - (self.v - vr) / self.tau + x

    def extra_repr(self):
        return (f"v_threshold={self.v_threshold}, v_reset={self.v_reset}, tau={self.tau}, "
                f"decay_input={self.decay_input}, step_mode={self.step_mode}")


def is_lif(m) -> bool:
    """True for this package's LIFNode or SpikingJelly's."""
    if isinstance(m, LIFNode):
        return True
    try:
        from spikingjelly.activation_based import neuron as _sjn  # type: ignore
        return isinstance(m, _sjn.LIFNode)
    except Exception:
        return False
