"""Stateful-module base (SpikingJelly ``activation_based.base`` contract):
modules with a ``step_mode`` ('s' single step on [B, ...], 'm' multi-step on
[T, B, ...]) and registered memories that ``reset()`` restores."""
from __future__ import annotations

import copy

import torch.nn as nn


class StepModule:
    def supported_step_mode(self):
        return ("s", "m")

    @property
    def step_mode(self):
        return self._step_mode

    @step_mode.setter
    def step_mode(self, value):
        if value not in self.supported_step_mode():
            raise ValueError(f"step_mode must be one of {self.supported_step_mode()}, got {value}")
        self._step_mode = value


class MemoryModule(nn.Module, StepModule):
    def __init__(self):
        super().__init__()
        self._memories = {}
        self._memories_rv = {}
        self._step_mode = "s"

    def register_memory(self, name: str, value):
        self._memories[name] = value
        self._memories_rv[name] = copy.deepcopy(value)

    def reset(self):
        for k in self._memories:
            self._memories[k] = copy.deepcopy(self._memories_rv[k])

    def __getattr__(self, name):
        mem = self.__dict__.get("_memories")
        if mem is not None and name in mem:
            return mem[name]
        return super().__getattr__(name)

    def __setattr__(self, name, value):
        mem = self.__dict__.get("_memories")
        if mem is not None and name in mem:
            mem[name] = value
        else:
            super().__setattr__(name, value)

    def single_step_forward(self, x, *args, **kwargs):
        raise NotImplementedError

    def multi_step_forward(self, x_seq, *args, **kwargs):
        return __import__("torch").stack(
            [self.single_step_forward(x_seq[t], *args, **kwargs) for t in range(x_seq.shape[0])])

    def forward(self, *args, **kwargs):
        if self.step_mode == "s":
            return self.single_step_forward(*args, **kwargs)
        return self.multi_step_forward(*args, **kwargs)
