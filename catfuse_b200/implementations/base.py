"""Implementation contract for one Conv->(BN)->LIF operator sigma.

Mirrors ``catfuse/implementations/base.py``: the frozen topology
(:class:`ConvLIFSpec`, ``:33-56``), the runtime params with a pre-folded BN
(:class:`ConvLIFParams`, ``:59-85``), the analytic HBM cost record
(:class:`IOCost`, ``:88-136``), the :class:`Implementation` ABC
(``:143-243``), the StaticZero short-circuit (``:250-308``) and the schedule
algebra of the four primitive transforms (TimeBlock, BatchFold, StreamFuse,
StateCarry) with its typing rules (``:319-483``).

B200 note: every implementation here runs the same fused sm_100a kernel, so
the bit-exactness contract between implementations holds literally (sparse
chunk skipping adds exact zeros); they differ in the HBM bytes they move.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn


@dataclass(frozen=True)
class ConvLIFSpec:
    in_channels: int
    out_channels: int
    kernel_size: int
    stride: int
    padding: int
    has_conv_bias: bool
    has_bn: bool
    tau: float
    v_threshold: float
    v_reset: Optional[float]
    decay_input: bool = True
    bn_eps: float = 1e-5

    def output_hw(self, h_in: int, w_in: int):
        h = (h_in + 2 * self.padding - self.kernel_size) // self.stride + 1
        w = (w_in + 2 * self.padding - self.kernel_size) // self.stride + 1
        return h, w

    def lif_config(self):
        from ..ops import LIFConfig
        return LIFConfig(self.tau, self.v_threshold, self.v_reset, self.decay_input)


class ConvLIFParams:
    """References to the pattern's tensors; BN already folded:
    bn_scale = gamma / sqrt(var + eps), bn_bias = beta - mean * bn_scale."""
    __slots__ = ("weight", "bias", "bn_scale", "bn_bias")

    def __init__(self, weight, bias, bn_scale, bn_bias):
        self.weight = weight
        self.bias = bias
        self.bn_scale = bn_scale
        self.bn_bias = bn_bias


@dataclass(frozen=True)
class IOCost:
    """Analytic HBM bytes of one forward, per tensor."""
    x_load: int
    w_load: int
    z_io: int
    v_io: int
    spike_write: int
    schedule: str
    num_blocks: int

    @property
    def intermediate_io(self) -> int:
        return self.z_io + self.v_io

    @property
    def total(self) -> int:
        return self.x_load + self.w_load + self.z_io + self.v_io + self.spike_write

    def as_dict(self) -> dict:
        return {"x_load": self.x_load, "w_load": self.w_load, "z_io": self.z_io,
                "v_io": self.v_io, "spike_write": self.spike_write,
                "intermediate_io": self.intermediate_io, "total": self.total,
                "schedule": self.schedule, "num_blocks": self.num_blocks}


class Implementation(nn.Module, ABC):
    """One element of Impl(sigma)."""

    name: str = "<unset>"

    @abstractmethod
    def forward(self, x: torch.Tensor, spec: ConvLIFSpec, params: ConvLIFParams,
                state) -> torch.Tensor:
        """x [T, B, C_in, H, W] fp32 CUDA -> spikes [T, B, C_out, H_out, W_out] fp32."""

    @abstractmethod
    def analytic_io_cost(self, spec: ConvLIFSpec, T: int, B: int, H_in: int, W_in: int,
                         K: int = None, *, dtype_bytes: int = 4) -> IOCost:
        ...

    @abstractmethod
    def schedule_decomposition(self, spec: ConvLIFSpec, T: int,
                               K: int = None) -> "ScheduleDecomposition":
        ...

    def reset_caches(self) -> None:
        pass


def folded_affine(spec: ConvLIFSpec, params: ConvLIFParams):
    """(scale, shift) of z' = acc*scale + shift for the kernel epilogue; scale
    None means 1.  A conv bias is folded as shift = bn_bias + bias*bn_scale."""
    if spec.has_bn:
        scale = params.bn_scale.detach().float().contiguous()
        shift = params.bn_bias.detach().float()
        if spec.has_conv_bias and params.bias is not None:
            shift = shift + params.bias.detach().float() * scale
        return scale, shift.contiguous()
    if spec.has_conv_bias and params.bias is not None:
        return None, params.bias.detach().float().contiguous()
    return None, None


def static_zero_forward(spec: ConvLIFSpec, params: ConvLIFParams, T: int, B: int, H_out: int,
                        W_out: int, device, state, lif_sequential_fn=None) -> torch.Tensor:
    """x == 0 everywhere: conv(0) = bias, so z = BN(bias) per channel; the LIF
    still evolves v.  Runs the sm_100a affine-LIF kernel with z absent."""
    from .. import ops
    _, shift = folded_affine(spec, params)
    if shift is None:
        shift = torch.zeros(spec.out_channels, dtype=torch.float32, device=device)
    v_in = state.get(shape=(B, spec.out_channels, H_out, W_out), device=device,
                     dtype=torch.float32)
    spikes, v_out = ops.bn_lif(None, None, shift.to(device), shape=(T, B, spec.out_channels,
                               H_out, W_out), v0=v_in, lif=spec.lif_config(), device=device)
    state.set(v_out)
    return spikes


# ---------------------------------------------------------------------------
# schedule algebra
# ---------------------------------------------------------------------------
TSI_OPS = frozenset({"Conv", "BN", "Linear", "Add", "Pool"})
CSR_OPS = frozenset({"LIF", "PSN"})
TGO_OPS = frozenset({"Attention", "GroupNorm", "LayerNorm"})


@dataclass(frozen=True)
class ScheduleTransform:
    primitive: str
    args: tuple

    @classmethod
    def TimeBlock(cls, K: int):
        return cls("TimeBlock", (int(K),))

    @classmethod
    def BatchFold(cls, op: str):
        return cls("BatchFold", (str(op),))

    @classmethod
    def StreamFuse(cls, u: str, v: str):
        return cls("StreamFuse", (str(u), str(v)))

    @classmethod
    def StateCarry(cls, op: str):
        return cls("StateCarry", (str(op),))

    def __str__(self) -> str:
        if self.primitive == "TimeBlock":
            return f"TimeBlock(K={self.args[0]})"
        if self.primitive == "StreamFuse":
            return f"StreamFuse({self.args[0]}, {self.args[1]})"
        if self.primitive in ("BatchFold", "StateCarry"):
            return f"{self.primitive}({self.args[0]})"
        return f"{self.primitive}{self.args}"

    def check_typing(self):
        p, a = self.primitive, self.args
        kind = lambda op: "CSR" if op in CSR_OPS else ("TSI" if op in TSI_OPS else "unknown/TGO")
        if p == "TimeBlock":
            if len(a) != 1:
                return [f"TimeBlock takes 1 arg, got {len(a)}"]
            return [] if a[0] >= 1 else [f"TimeBlock(K) requires K >= 1, got {a[0]}"]
        if p == "BatchFold":
            if len(a) != 1:
                return [f"BatchFold takes 1 arg, got {len(a)}"]
            return [] if a[0] in TSI_OPS else [
                f"BatchFold({a[0]}) ILLEGAL — op must be TSI; {a[0]} is {kind(a[0])}"]
        if p == "StreamFuse":
            if len(a) != 2:
                return [f"StreamFuse takes 2 args, got {len(a)}"]
            errs = []
            if a[0] not in TSI_OPS:
                errs.append(f"StreamFuse({a[0]}, {a[1]}) ILLEGAL — u={a[0]} must be TSI")
            if a[1] not in CSR_OPS:
                errs.append(f"StreamFuse({a[0]}, {a[1]}) ILLEGAL — v={a[1]} must be CSR")
            return errs
        if p == "StateCarry":
            if len(a) != 1:
                return [f"StateCarry takes 1 arg, got {len(a)}"]
            return [] if a[0] in CSR_OPS else [
                f"StateCarry({a[0]}) ILLEGAL — op must be CSR; {a[0]} is {kind(a[0])}"]
        return [f"Unknown primitive '{p}'"]


@dataclass(frozen=True)
class ScheduleDecomposition:
    transforms: tuple
    form: str
    description: str = ""

    def __str__(self) -> str:
        return " ∘ ".join(str(t) for t in reversed(self.transforms))

    def verify(self):
        errors = []
        for i, t in enumerate(self.transforms):
            for e in t.check_typing():
                errors.append(f"transform[{i}] {t}: {e}")
        prims = [t.primitive for t in self.transforms]
        if "TimeBlock" not in prims:
            errors.append("Missing TimeBlock — a schedule must be chunked "
                          "(use TimeBlock(K=T) for the single-block case)")
        sf = {t.args[1] for t in self.transforms if t.primitive == "StreamFuse" and len(t.args) == 2}
        sc = {t.args[0] for t in self.transforms if t.primitive == "StateCarry" and len(t.args) == 1}
        for v in sorted(sf - sc):
            errors.append(f"StreamFuse(_, {v}) without StateCarry({v}) — the CSR state of {v} "
                          f"must be carried at block boundaries")
        if self.form not in ("form_1", "form_2", "form_3", "custom"):
            errors.append(f"unknown form '{self.form}'")
        return (len(errors) == 0, errors)
