"""CTF pattern library: fused-module wrappers that replace matched
SpikingJelly subgraphs (reference: ``catfuse/patterns.py``).

Same classes, constructor arguments, ``from_sj_modules`` / ``from_sj_block``
classmethods, ``forward(x[T, B, ...])`` contract and ``reset()`` behaviour as
the reference; each forward runs the sm_100a kernels of this package:

  PartialFusionConvLIF        Conv -> LIF                  (fused tcgen05 kernel)
  PartialFusionConvBNLIF      Conv -> BN -> LIF            (DenseKeep)
  PartialFusionConvBNAddLIF   Conv -> BN -> +identity -> LIF
  FusedLinearLIF              Linear -> LIF                (1x1 conv on tokens)
  FusedAddBNLIF               Add -> BN -> LIF             (affine-LIF kernel)
  FusedAddLIF / FusedAvgPoolLIF
  CTFSEWBasicBlock / CTFSpikingBasicBlock / CTFSEWBottleneck / CTFSpikingBottleneck
  STFusionConvBNLIF           Conv -> BN -> LIF with runtime EGD (SparseFlow)

Every pattern also exposes ``native_conv()`` (where it is a convolution) so
:mod:`catfuse_b200.network` can chain patterns without leaving the kernels'
[B, H, W, T, C] fp16 layout.
"""
from __future__ import annotations

import math

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .implementations import ConvLIFParams, ConvLIFSpec, DenseKeep, SparseFlow
from .implementations.base import folded_affine
from .implementations._fused import _WeightCache, check_input
from .sj.base import MemoryModule as _SJMemoryModule
from .state import StateBuffer

try:  # recognise real SpikingJelly modules when installed
    from spikingjelly.activation_based.base import MemoryModule as _RealSJMemoryModule  # type: ignore
    _BASES = (_RealSJMemoryModule,)
except Exception:  # pragma: no cover - SJ is optional
    _BASES = (_SJMemoryModule,)


def _first(v):
    return v[0] if isinstance(v, (tuple, list)) else v


def _lif_attrs(lif):
    tau = float(getattr(lif, "tau", 2.0))
    v_th = float(getattr(lif, "v_threshold", 1.0))
    vr = getattr(lif, "v_reset", 0.0)
    v_reset = None if vr is None else float(vr)
    decay_input = bool(getattr(lif, "decay_input", True))
    return tau, v_th, v_reset, decay_input


class NativeConv:
    """What a fused conv pattern contributes to a native network plan."""

    def __init__(self, owner, spec: ConvLIFSpec, params: ConvLIFParams):
        self.owner = owner
        self.spec = spec
        self.params = params

    def packed(self, device, precision: str = "fp16"):
        caches = self.owner.__dict__.setdefault("_native_caches", {})
        cache = caches.setdefault(precision, _WeightCache())
        return cache.get(self.spec, self.params, device, precision)


class CTFPattern(*_BASES):
    """Base class: multi-step ([T, B, ...]) fused pattern whose CSR state lives
    in registered :class:`StateBuffer` objects; ``reset()`` clears them."""

    policy_row: Optional[int] = None

    def __init__(self):
        super().__init__()
        self._catfuse_states: list = []
        try:
            self.step_mode = "m"
        except Exception:
            pass

    def _register_state(self, state) -> None:
        if not isinstance(state, StateBuffer):
            raise TypeError(f"_register_state expects a StateBuffer, got {type(state).__name__}")
        if not hasattr(self, "_catfuse_states") or self._catfuse_states is None:
            self._catfuse_states = []
        self._catfuse_states.append(state)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    @classmethod
    def from_sj_modules(cls, *sj_modules, **kwargs):
        raise NotImplementedError

    def reset(self):
        for state in getattr(self, "_catfuse_states", []):
            state.reset()

    def single_step_forward(self, x, *args):
        return self.forward(x, *args)

    def multi_step_forward(self, x_seq, *args):
        return self.forward(x_seq, *args)

    def __call__(self, *args, **kwargs):
        # Bypass SJ's step-mode dispatch: patterns are always multi-step.
        return nn.Module.__call__(self, *args, **kwargs)


# ---------------------------------------------------------------------------
# Conv patterns
# ---------------------------------------------------------------------------

class _ConvPatternMixin:
    """Shared plumbing for conv patterns that own weight + raw BN params."""

    def _conv_spec(self, has_bn: bool, has_bias: bool) -> ConvLIFSpec:
        return ConvLIFSpec(self.in_channels, self.out_channels, self.kernel_size, self.stride,
                           self.padding, has_bias, has_bn, float(self.tau),
                           float(self.v_threshold),
                           None if self.v_reset is None else float(self.v_reset),
                           bool(getattr(self, "decay_input", True)),
                           float(getattr(self, "bn_eps", 1e-5)))


class PartialFusionConvLIF(CTFPattern, _ConvPatternMixin):
    """Conv -> LIF (no BN).  As in the reference kernel
    (``catfuse/kernels/partial_fusion_conv_lif_impl.py``), v starts from 0 on
    every call (no state carried across calls)."""

    policy_row = 1

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, tau: float = 2.0, v_threshold: float = 1.0,
                 v_reset: float = 0.0):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_size, self.stride, self.padding = kernel_size, stride, padding
        self.tau, self.v_threshold, self.v_reset = tau, v_threshold, v_reset
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels, kernel_size, kernel_size))
        nn.init.kaiming_normal_(self.weight)
        self.conv_bias = None
        self._impl = DenseKeep()

    def _spec_params(self):
        spec = self._conv_spec(False, self.conv_bias is not None)
        return spec, ConvLIFParams(self.weight, self.conv_bias, None, None)

    def native_conv(self):
        return NativeConv(self, *self._spec_params())

    def forward(self, x):
        squeeze = x.dim() == 4
        if squeeze:
            x = x.unsqueeze(0)
        spec, params = self._spec_params()
        out = self._impl.forward(x, spec, params, StateBuffer())
        return out.squeeze(0) if squeeze else out

    @classmethod
    def from_sj_modules(cls, sj_conv, sj_lif):
        tau, v_th, v_reset, _ = _lif_attrs(sj_lif)
        inst = cls(sj_conv.in_channels, sj_conv.out_channels, _first(sj_conv.kernel_size),
                   _first(sj_conv.stride), _first(sj_conv.padding), tau, v_th,
                   0.0 if v_reset is None else v_reset)
        inst.v_reset = v_reset
        inst.weight.data.copy_(sj_conv.weight.data)
        if sj_conv.bias is not None:
            inst.conv_bias = nn.Parameter(sj_conv.bias.data.clone())
        return inst


class PartialFusionConvBNLIF(CTFPattern, _ConvPatternMixin):
    """Conv -> BN -> LIF with StateCarry through a StateBuffer (DenseKeep).

    Unlike the reference (``catfuse/patterns.py:296-331``), a conv bias copied
    from the SJ conv is applied (folded into the BN shift)."""

    policy_row = 2

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, tau: float = 2.0, v_threshold: float = 1.0,
                 v_reset: float = 0.0, bn_eps: float = 1e-5):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_size, self.stride, self.padding = kernel_size, stride, padding
        self.tau, self.v_threshold, self.v_reset, self.bn_eps = tau, v_threshold, v_reset, bn_eps
        self.decay_input = True
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels, kernel_size, kernel_size))
        self.bn_weight = nn.Parameter(torch.ones(out_channels))
        self.bn_bias = nn.Parameter(torch.zeros(out_channels))
        self.register_buffer("running_mean", torch.zeros(out_channels))
        self.register_buffer("running_var", torch.ones(out_channels))
        nn.init.kaiming_normal_(self.weight)
        self.conv_bias = None
        self.state = StateBuffer()
        self._register_state(self.state)
        self.spec = self._conv_spec(True, False)
        self._impl = DenseKeep()
        self._params = None
        self._params_key = None

    def _ensure_params(self):
        def tag(t):
            return None if t is None else (id(t), t._version)
        key = (tag(self.weight), tag(self.bn_weight), tag(self.bn_bias), tag(self.running_mean),
               tag(self.running_var), tag(self.conv_bias))
        if self._params_key == key and self._params is not None:
            return self._params
        with torch.no_grad():
            inv_std = torch.rsqrt(self.running_var + self.bn_eps)
            bn_scale = (self.bn_weight * inv_std).detach()
            bn_bias = (self.bn_bias - self.running_mean * bn_scale).detach()
        self.spec = self._conv_spec(True, self.conv_bias is not None)
        self._params = ConvLIFParams(self.weight, self.conv_bias, bn_scale, bn_bias)
        self._params_key = key
        return self._params

    def native_conv(self):
        params = self._ensure_params()
        return NativeConv(self, self.spec, params)

    def forward(self, x):
        params = self._ensure_params()
        if x.dim() == 4:
            return self._impl.forward(x.unsqueeze(0), self.spec, params, self.state).squeeze(0)
        return self._impl.forward(x, self.spec, params, self.state)

    @classmethod
    def from_sj_modules(cls, sj_conv, sj_bn, sj_lif):
        tau, v_th, v_reset, decay_input = _lif_attrs(sj_lif)
        inst = cls(sj_conv.in_channels, sj_conv.out_channels, _first(sj_conv.kernel_size),
                   _first(sj_conv.stride), _first(sj_conv.padding), tau, v_th,
                   0.0 if v_reset is None else v_reset, sj_bn.eps)
        inst.v_reset = v_reset
        inst.decay_input = decay_input
        inst.weight.data.copy_(sj_conv.weight.data)
        if sj_conv.bias is not None:
            inst.conv_bias = nn.Parameter(sj_conv.bias.data.clone())
        inst.bn_weight.data.copy_(sj_bn.weight.data)
        inst.bn_bias.data.copy_(sj_bn.bias.data)
        inst.running_mean.data.copy_(sj_bn.running_mean.data)
        inst.running_var.data.copy_(sj_bn.running_var.data)
        inst.spec = inst._conv_spec(True, inst.conv_bias is not None)
        return inst


class PartialFusionConvBNAddLIF(PartialFusionConvBNLIF):
    """Conv -> BN -> (+ identity) -> LIF, the second half of a standard Spiking
    ResNet block.  As in the reference kernel
    (``catfuse/kernels/partial_fusion_conv_bn_add_lif_impl.py:76-123``) v starts
    at 0 on every call.  The identity is added in fp32 inside the kernel
    epilogue after a rounding to fp16 at the kernel boundary."""

    policy_row = 9

    def forward(self, x, identity):
        squeeze = x.dim() == 4
        if squeeze:
            x, identity = x.unsqueeze(0), identity.unsqueeze(0)
        check_input(x, self.spec)
        params = self._ensure_params()
        T, B, _, H, W = x.shape
        Ho, Wo = self.spec.output_hw(H, W)
        wp, scale, shift = self.__dict__.setdefault("_wcache", _WeightCache()).get(
            self.spec, params, x.device)
        xp = ops.pack_tbchw(x.contiguous(), wp.shape[-1])
        idp = ops.pack_tbchw(identity.contiguous(), self.out_channels)
        out = ops.conv_bn_lif(xp, wp, scale, shift, self.stride, self.padding, identity=idp,
                              res_mode="add_pre", lif=self.spec.lif_config())
        out = ops.unpack_bhwtc(out)
        return out.squeeze(0) if squeeze else out


class STFusionConvBNLIF(CTFPattern, _ConvPatternMixin):
    """Spatio-temporal fused Conv -> BN -> LIF with a SparseFlow backend and the
    runtime execution-grounded dispatch (EGD) of
    ``catfuse/sparseflow/ops/st_fusion_conv_bn_lif.py:91-565``.

    ``egd="device"`` (default): the dispatch is per tile on the GPU — the
    prescan marks each tile's active channel chunks and the fused kernel skips
    the rest (an all-zero tile is StaticZero); no host synchronisation.
    ``egd="host"``: the reference's rule — count nonzeros, read the count on
    the host, and route sparsity > 0.7 (or nnz == 0) to SparseFlow, else to
    DenseKeep.  Both produce identical spikes."""

    policy_row = "STFusionConvBNLIF"

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, stride: int = 1,
                 padding: int = 1, bias: bool = True, bn_scale: Optional[torch.Tensor] = None,
                 bn_bias: Optional[torch.Tensor] = None, tau: float = 2.0,
                 v_threshold: float = 1.0, v_reset: Optional[float] = 0.0,
                 decay_input: bool = True, K: int = 4, threshold: float = 1e-6,
                 egd: str = "device"):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_size, self.stride, self.padding = kernel_size, stride, padding
        self.K = K
        self.tau, self.v_threshold, self.v_reset = float(tau), float(v_threshold), v_reset
        self.decay_input = decay_input
        self.threshold = threshold
        self.egd = egd
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels, kernel_size, kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        if bn_scale is not None:
            self.register_buffer("bn_scale", bn_scale.clone())
            self.register_buffer("bn_bias_folded", bn_bias.clone())
        else:
            self.register_buffer("bn_scale", None)
            self.register_buffer("bn_bias_folded", None)
        self.state = StateBuffer()
        self._register_state(self.state)
        self.spec = ConvLIFSpec(in_channels, out_channels, kernel_size, stride, padding,
                                bias is True, bn_scale is not None, float(tau), float(v_threshold),
                                v_reset, bool(decay_input))
        self._impl_dense = DenseKeep()
        self._impl_sparse = SparseFlow()
        self._params = None
        self._params_key = None
        self.last_dispatch = None

    def _ensure_params(self):
        key = (id(self.weight), id(self.bias), id(self.bn_scale), id(self.bn_bias_folded))
        if self._params_key == key and self._params is not None:
            return self._params
        self._params = ConvLIFParams(self.weight, self.bias, self.bn_scale, self.bn_bias_folded)
        self._params_key = key
        return self._params

    def native_conv(self):
        return NativeConv(self, self.spec, self._ensure_params())

    @classmethod
    def from_sj_modules(cls, conv, bn, lif, K: int = 4, threshold: float = 1e-6):
        bn.eval()
        inv_std = 1.0 / torch.sqrt(bn.running_var + bn.eps)
        scale = inv_std if bn.weight is None else bn.weight * inv_std
        shift = -bn.running_mean * scale if bn.bias is None else bn.bias - bn.running_mean * scale
        tau, v_th, v_reset, decay_input = _lif_attrs(lif)
        m = cls(conv.in_channels, conv.out_channels, _first(conv.kernel_size), _first(conv.stride),
                _first(conv.padding), conv.bias is not None, scale.detach(), shift.detach(), tau,
                v_th, v_reset, decay_input, K, threshold)
        m.weight.data.copy_(conv.weight.data)
        if conv.bias is not None:
            m.bias.data.copy_(conv.bias.data)
        return m

    def _dense_forward(self, x):
        return self._impl_dense.forward(x, self.spec, self._ensure_params(), self.state)

    def _batchfold_forward(self, x):
        return self._impl_sparse.forward(x, self.spec, self._ensure_params(), self.state)

    def forward(self, x):
        squeeze = x.dim() == 4
        if squeeze:
            x = x.unsqueeze(0)
        if self.egd == "host":
            from .policy import EGD_SPARSITY_THRESHOLD
            nnz = int(torch.count_nonzero(x).item())
            sparsity = 1.0 - nnz / max(x.numel(), 1)
            if nnz == 0 or sparsity > EGD_SPARSITY_THRESHOLD:
                self.last_dispatch = "StaticZero" if nnz == 0 else "SparseFlow"
                out = self._batchfold_forward(x)
            else:
                self.last_dispatch = "DenseKeep"
                out = self._dense_forward(x)
        else:
            # device-side EGD: the prescan's tile masks feed the kernel, which
            # counts the active (tile, chunk) pairs and runs the masks or the
            # dense schedule (calibrated threshold of the hardware profile);
            # no host synchronisation.  dispatch_decision() reads it back.
            from .hardware import detect_hardware
            frac = detect_hardware().egd_max_active_frac
            self._egd_stats = {}
            out = self._impl_sparse.forward(x, self.spec, self._ensure_params(), self.state,
                                            stats=self._egd_stats,
                                            egd_max_active_frac=frac if frac >= 0 else 1.0)
            self._egd_frac = frac if frac >= 0 else 1.0
            self.last_dispatch = "EGD(device)"
        return out.squeeze(0) if squeeze else out

    def dispatch_decision(self) -> Optional[str]:
        """What the device-side EGD of the last forward chose: "StaticZero"
        (no active chunk), "SparseFlow" (masks ran) or "DenseKeep" (reads the
        tile masks back: synchronises)."""
        st = getattr(self, "_egd_stats", None)
        if not st or "tile_mask" not in st:
            return self.last_dispatch
        from . import ops
        mask = st["tile_mask"]
        cin_p = ops.pad16(self.in_channels)
        n_kx = cin_p // ops.conv_chunk(cin_p, False)   # device-dispatch masks: dense chunk
        bits = (1 << n_kx) - 1
        active = sum(bin(int(m) & bits).count("1") for m in mask.cpu().tolist())
        if active == 0:
            return "StaticZero"
        limit = math.floor(self._egd_frac * mask.numel() * n_kx)
        return "SparseFlow" if active <= limit else "DenseKeep"

    def extra_repr(self):
        s = f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, K={self.K}"
        if self.bn_scale is not None:
            s += ", bn=folded"
        return s + f", tau={self.tau}, v_th={self.v_threshold}"


# ---------------------------------------------------------------------------
# Linear / elementwise patterns
# ---------------------------------------------------------------------------

class FusedLinearLIF(CTFPattern):
    """Linear -> LIF over x[T, B, ..., C_in]; the linear is a 1x1 convolution
    over the tokens on the tensor cores with the LIF in the epilogue; v carried
    in a StateBuffer.  ``weight_io`` keeps the reference's [in, out] layout."""

    policy_row = 4

    def __init__(self, in_features: int, out_features: int, tau: float = 2.0,
                 v_threshold: float = 1.0, v_reset: float = 0.0):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.tau, self.v_threshold, self.v_reset = tau, v_threshold, v_reset
        self.weight_io = nn.Parameter(torch.empty(in_features, out_features))
        nn.init.kaiming_normal_(self.weight_io.T)
        self.bias = None
        # folded BN1d affine: buffers, so that .to(device) moves them with the weights
        self.register_buffer("bn_scale", None)
        self.register_buffer("bn_shift", None)
        self.state = StateBuffer()
        self._register_state(self.state)

    def _spec(self):
        return ConvLIFSpec(self.in_features, self.out_features, 1, 1, 0, self.bias is not None,
                           self.bn_scale is not None, float(self.tau), float(self.v_threshold),
                           None if self.v_reset is None else float(self.v_reset))

    def _params(self):
        w = self.weight_io.t().reshape(self.out_features, self.in_features, 1, 1)
        return ConvLIFParams(w, self.bias, self.bn_scale, self.bn_shift)

    def forward(self, x):
        squeeze = x.dim() == 2
        if squeeze:
            x = x.unsqueeze(0)
        T, B = x.shape[:2]
        tok = x.shape[2:-1]
        L = 1
        for d in tok:
            L *= int(d)
        # [T, B, L, C] -> [T, B, C, L, 1] for the packer
        x5 = x.reshape(T, B, L, self.in_features).permute(0, 1, 3, 2).unsqueeze(-1)
        from .implementations._fused import fused_forward
        cache = self.__dict__.setdefault("_wcache", _WeightCache())
        spec = self._spec()
        out = fused_forward(x5.contiguous(), spec, self._params(), self.state, cache, sparse=False)
        out = out.squeeze(-1).permute(0, 1, 3, 2).reshape(T, B, *tok, self.out_features)
        return out.squeeze(0) if squeeze else out

    @classmethod
    def from_sj_modules(cls, sj_linear, sj_lif, sj_bn=None):
        tau, v_th, v_reset, _ = _lif_attrs(sj_lif)
        inst = cls(sj_linear.in_features, sj_linear.out_features, tau, v_th,
                   0.0 if v_reset is None else v_reset)
        inst.v_reset = v_reset
        inst.weight_io.data.copy_(sj_linear.weight.data.T)
        if sj_linear.bias is not None:
            inst.bias = nn.Parameter(sj_linear.bias.data.clone())
        if sj_bn is not None:  # Linear -> BN1d -> LIF (folded into the epilogue)
            inv_std = torch.rsqrt(sj_bn.running_var + sj_bn.eps)
            scale = sj_bn.weight.data * inv_std
            inst.bn_scale = scale.clone()
            inst.bn_shift = (sj_bn.bias.data - sj_bn.running_mean * scale).clone()
        return inst


class FusedAddBNLIF(CTFPattern):
    """Add -> BN -> LIF: z = (a + x) * scale + shift, LIF with v carried."""

    policy_row = 6

    def __init__(self, num_features: int, tau: float = 2.0, v_threshold: float = 1.0,
                 v_reset: float = 0.0, bn_eps: float = 1e-5):
        super().__init__()
        self.num_features = num_features
        self.tau, self.v_threshold, self.v_reset, self.bn_eps = tau, v_threshold, v_reset, bn_eps
        self.bn_weight = nn.Parameter(torch.ones(num_features))
        self.bn_bias = nn.Parameter(torch.zeros(num_features))
        self.register_buffer("running_mean", torch.zeros(num_features))
        self.register_buffer("running_var", torch.ones(num_features))
        self.state = StateBuffer()
        self._register_state(self.state)

    def forward(self, a, x):
        inv_std = torch.rsqrt(self.running_var + self.bn_eps)
        scale = (self.bn_weight * inv_std).detach().contiguous()
        shift = (self.bn_bias - self.running_mean * scale).detach().contiguous()
        z = (a + x).contiguous()
        v0 = self.state.tensor if self.state.is_initialized else None
        lif = ops.LIFConfig(self.tau, self.v_threshold, self.v_reset)
        s, vT = ops.bn_lif(z.float(), scale, shift, v0=v0, lif=lif)
        self.state.set(vT)
        return s

    @classmethod
    def from_sj_modules(cls, sj_bn, sj_lif):
        tau, v_th, v_reset, _ = _lif_attrs(sj_lif)
        inst = cls(sj_bn.num_features, tau, v_th, 0.0 if v_reset is None else v_reset, sj_bn.eps)
        inst.v_reset = v_reset
        inst.bn_weight.data.copy_(sj_bn.weight.data)
        inst.bn_bias.data.copy_(sj_bn.bias.data)
        inst.running_mean.data.copy_(sj_bn.running_mean.data)
        inst.running_var.data.copy_(sj_bn.running_var.data)
        return inst


class FusedAddLIF(CTFPattern):
    """Add -> LIF (``catfuse/kernels/add_lif.py``): z = x1 + x2, v carried."""

    policy_row = 5

    def __init__(self, tau: float = 2.0, v_threshold: float = 1.0, v_reset: float = 0.0):
        super().__init__()
        self.tau, self.v_threshold, self.v_reset = tau, v_threshold, v_reset
        self.state = StateBuffer()
        self._register_state(self.state)

    def forward(self, x1, x2):
        v0 = self.state.tensor if self.state.is_initialized else None
        s, vT = ops.add_lif(x1.float().contiguous(), x2.float().contiguous(), v0=v0,
                            lif=ops.LIFConfig(self.tau, self.v_threshold, self.v_reset))
        self.state.set(vT)
        return s

    @classmethod
    def from_sj_modules(cls, sj_lif):
        tau, v_th, v_reset, _ = _lif_attrs(sj_lif)
        return cls(tau, v_th, v_reset)


class FusedAvgPoolLIF(CTFPattern):
    """k x k average pool -> LIF (``catfuse/kernels/avgpool_lif.py``), v carried."""

    policy_row = 7

    def __init__(self, kernel_size: int = 2, tau: float = 2.0, v_threshold: float = 1.0,
                 v_reset: float = 0.0):
        super().__init__()
        self.kernel_size = kernel_size
        self.tau, self.v_threshold, self.v_reset = tau, v_threshold, v_reset
        self.state = StateBuffer()
        self._register_state(self.state)

    def forward(self, x):
        v0 = self.state.tensor if self.state.is_initialized else None
        s, vT = ops.avgpool_lif(x.float().contiguous(), self.kernel_size, v0=v0,
                                lif=ops.LIFConfig(self.tau, self.v_threshold, self.v_reset))
        self.state.set(vT)
        return s

    @classmethod
    def from_sj_modules(cls, sj_pool, sj_lif):
        tau, v_th, v_reset, _ = _lif_attrs(sj_lif)
        return cls(_first(sj_pool.kernel_size), tau, v_th, v_reset)


# ---------------------------------------------------------------------------
# ResNet blocks
# ---------------------------------------------------------------------------

def _sew(identity, out, cnf):
    if cnf == "ADD":
        return identity + out
    if cnf == "AND":
        return identity * out
    if cnf == "IAND":
        return identity * (1.0 - out)
    raise NotImplementedError(f"Unknown cnf: {cnf}")


class CTFSEWBasicBlock(CTFPattern):
    """SEW BasicBlock: two Conv-BN-LIF, optional Conv-BN-LIF downsample, and
    the spike-level combine ``g(identity, out)``."""

    def __init__(self, fused_first, fused_second, fused_downsample, cnf):
        super().__init__()
        self.fused_first = fused_first
        self.fused_second = fused_second
        self.fused_downsample = fused_downsample
        self.cnf = cnf

    def forward(self, x):
        out = self.fused_second(self.fused_first(x))
        identity = self.fused_downsample(x) if self.fused_downsample is not None else x
        return _sew(identity, out, self.cnf)

    @classmethod
    def from_sj_block(cls, b):
        ds = None
        if b.downsample is not None:
            ds = PartialFusionConvBNLIF.from_sj_modules(b.downsample[0], b.downsample[1],
                                                        b.downsample_sn)
        return cls(PartialFusionConvBNLIF.from_sj_modules(b.conv1, b.bn1, b.sn1),
                   PartialFusionConvBNLIF.from_sj_modules(b.conv2, b.bn2, b.sn2), ds, b.cnf)


class _ConvBN(nn.Module):
    """Conv -> BN without LIF (the standard Spiking ResNet downsample), on the
    fused kernel's z-only epilogue."""

    def __init__(self, weight, scale, shift, stride, padding):
        super().__init__()
        self.weight = nn.Parameter(weight.clone())
        self.register_buffer("bn_scale", scale.clone())
        self.register_buffer("bn_shift", shift.clone())
        self.stride, self.padding = stride, padding
        k = weight.shape[-1]
        self.spec = ConvLIFSpec(weight.shape[1], weight.shape[0], k, stride, padding, False, True,
                                2.0, 1.0, 0.0)

    def params(self):
        return ConvLIFParams(self.weight, None, self.bn_scale, self.bn_shift)

    def native_conv(self):
        return NativeConv(self, self.spec, self.params())

    def forward(self, x):
        check_input(x, self.spec)
        wp, scale, shift = self.__dict__.setdefault("_wcache", _WeightCache()).get(
            self.spec, self.params(), x.device)
        xp = ops.pack_tbchw(x.contiguous(), wp.shape[-1])
        out = ops.conv_bn_lif(xp, wp, scale, shift, self.stride, self.padding, res_mode="z_only")
        return ops.unpack_bhwtc(out)


def _fold(bn):
    inv_std = torch.rsqrt(bn.running_var + bn.eps)
    scale = bn.weight * inv_std
    return scale.detach(), (bn.bias - bn.running_mean * scale).detach()


class CTFSpikingBasicBlock(CTFPattern):
    """Standard Spiking ResNet BasicBlock: Conv-BN-LIF, then Conv-BN + identity
    -> LIF (add before the LIF); the downsample is Conv-BN without LIF."""

    def __init__(self, fused_first, fused_second_add, downsample_conv_weight=None,
                 downsample_bn_scale=None, downsample_bn_bias=None, downsample_stride=1,
                 downsample_padding=0):
        super().__init__()
        self.fused_first = fused_first
        self.fused_second_add = fused_second_add
        self.has_downsample = downsample_conv_weight is not None
        self.downsample = (_ConvBN(downsample_conv_weight, downsample_bn_scale, downsample_bn_bias,
                                   downsample_stride, downsample_padding)
                           if self.has_downsample else None)

    def forward(self, x):
        out = self.fused_first(x)
        identity = self.downsample(x) if self.has_downsample else x
        return self.fused_second_add(out, identity)

    @classmethod
    def from_sj_block(cls, b):
        first = PartialFusionConvBNLIF.from_sj_modules(b.conv1, b.bn1, b.sn1)
        second = PartialFusionConvBNAddLIF.from_sj_modules(b.conv2, b.bn2, b.sn2)
        if b.downsample is not None:
            c, bn = b.downsample[0], b.downsample[1]
            scale, shift = _fold(bn)
            return cls(first, second, c.weight.data, scale, shift, _first(c.stride),
                       _first(c.padding))
        return cls(first, second)


class CTFSEWBottleneck(CTFPattern):
    def __init__(self, fused_first, fused_middle, fused_last, fused_downsample, cnf):
        super().__init__()
        self.fused_first, self.fused_middle, self.fused_last = fused_first, fused_middle, fused_last
        self.fused_downsample = fused_downsample
        self.cnf = cnf

    def forward(self, x):
        out = self.fused_last(self.fused_middle(self.fused_first(x)))
        identity = self.fused_downsample(x) if self.fused_downsample is not None else x
        return _sew(identity, out, self.cnf)

    @classmethod
    def from_sj_block(cls, b):
        ds = None
        if b.downsample is not None:
            ds = PartialFusionConvBNLIF.from_sj_modules(b.downsample[0], b.downsample[1],
                                                        b.downsample_sn)
        return cls(PartialFusionConvBNLIF.from_sj_modules(b.conv1, b.bn1, b.sn1),
                   PartialFusionConvBNLIF.from_sj_modules(b.conv2, b.bn2, b.sn2),
                   PartialFusionConvBNLIF.from_sj_modules(b.conv3, b.bn3, b.sn3), ds, b.cnf)


class CTFSpikingBottleneck(CTFPattern):
    def __init__(self, fused_first, fused_middle, fused_last_add, downsample_conv_weight=None,
                 downsample_bn_scale=None, downsample_bn_bias=None, downsample_stride=1,
                 downsample_padding=0):
        super().__init__()
        self.fused_first, self.fused_middle = fused_first, fused_middle
        self.fused_last_add = fused_last_add
        self.has_downsample = downsample_conv_weight is not None
        self.downsample = (_ConvBN(downsample_conv_weight, downsample_bn_scale, downsample_bn_bias,
                                   downsample_stride, downsample_padding)
                           if self.has_downsample else None)

    def forward(self, x):
        out = self.fused_middle(self.fused_first(x))
        identity = self.downsample(x) if self.has_downsample else x
        return self.fused_last_add(out, identity)

    @classmethod
    def from_sj_block(cls, b):
        first = PartialFusionConvBNLIF.from_sj_modules(b.conv1, b.bn1, b.sn1)
        middle = PartialFusionConvBNLIF.from_sj_modules(b.conv2, b.bn2, b.sn2)
        last = PartialFusionConvBNAddLIF.from_sj_modules(b.conv3, b.bn3, b.sn3)
        if b.downsample is not None:
            c, bn = b.downsample[0], b.downsample[1]
            scale, shift = _fold(bn)
            return cls(first, middle, last, c.weight.data, scale, shift, _first(c.stride),
                       _first(c.padding))
        return cls(first, middle, last)


class FusedSSA(CTFPattern):
    """Spikformer spiking self-attention block over x[T, B, N, C]:
    q/k/v = Linear->BN1d->LIF (fused tensor-core linear), the attention core
    (q kᵀ · scale) v with its attention LIF in one kernel (``ops.ssa_lif``:
    exact integer arithmetic on the spikes, membrane carried over T), then
    proj = Linear->BN1d->LIF.  Mirrors SSA.forward of the reference
    (models/spikformer_github.py:138-158); every LIF keeps its membrane in a
    StateBuffer (StateCarry across calls) and ``reset()`` clears them all."""

    policy_row = 4

    def __init__(self, q, k, v, proj, heads: int, attn_tau: float = 2.0,
                 attn_v_threshold: float = 1.0, attn_v_reset: Optional[float] = 0.0,
                 scale: Optional[float] = None):
        super().__init__()
        self.q, self.k, self.v, self.proj = q, k, v, proj
        self.heads = int(heads)
        dim = q.out_features
        if dim % self.heads:
            raise ValueError("dim must be a multiple of heads")
        self.scale = float((dim // self.heads) ** -0.5 if scale is None else scale)
        self.attn_lif = ops.LIFConfig(tau=attn_tau, v_threshold=attn_v_threshold,
                                      v_reset=attn_v_reset)
        self.attn_state = StateBuffer()
        self._register_state(self.attn_state)

    def reset(self):
        super().reset()
        for m in (self.q, self.k, self.v, self.proj):
            m.reset()

    def forward(self, x):
        if x.dim() != 4 or not x.is_cuda:
            raise ValueError("FusedSSA expects a CUDA tensor x[T, B, N, C]")
        T, B, N, C = x.shape
        qs, ks, vs = self.q(x), self.k(x), self.v(x)          # [T, B, N, C] spikes
        to_bntc = lambda s: s.permute(1, 2, 0, 3).to(torch.float16).contiguous()
        v_att = self.attn_state.get((B, N, C), x.device)
        y = ops.ssa_lif(to_bntc(qs), to_bntc(ks), to_bntc(vs), self.heads, self.scale,
                        v_in=v_att, v_out=v_att, lif=self.attn_lif)
        self.attn_state.set(v_att)
        return self.proj(y.permute(2, 0, 1, 3).float())

    @classmethod
    def from_sj_modules(cls, sj_ssa):
        """From a reference-style SSA module with q/q_bn/q_lif, k/..., v/...,
        attn_lif, proj/proj_bn/proj_lif and num_heads."""
        def lin(name):
            return FusedLinearLIF.from_sj_modules(getattr(sj_ssa, name),
                                                  getattr(sj_ssa, name + "_lif"),
                                                  getattr(sj_ssa, name + "_bn", None))
        tau, v_th, v_reset, _ = _lif_attrs(sj_ssa.attn_lif)
        return cls(lin("q"), lin("k"), lin("v"), lin("proj"), sj_ssa.num_heads, tau, v_th,
                   v_reset, getattr(sj_ssa, "scale", None))


PATTERN_REGISTRY = {
    "PartialFusionConvLIF": PartialFusionConvLIF,
    "PartialFusionConvBNLIF": PartialFusionConvBNLIF,
    "PartialFusionConvBNAddLIF": PartialFusionConvBNAddLIF,
    "FusedLinearLIF": FusedLinearLIF,
    "FusedAddBNLIF": FusedAddBNLIF,
    "FusedAddLIF": FusedAddLIF,
    "FusedAvgPoolLIF": FusedAvgPoolLIF,
    "CTFSEWBasicBlock": CTFSEWBasicBlock,
    "CTFSpikingBasicBlock": CTFSpikingBasicBlock,
    "CTFSEWBottleneck": CTFSEWBottleneck,
    "CTFSpikingBottleneck": CTFSpikingBottleneck,
    "STFusionConvBNLIF": STFusionConvBNLIF,
    "FusedSSA": FusedSSA,
}

__all__ = list(PATTERN_REGISTRY) + ["CTFPattern", "PATTERN_REGISTRY", "NativeConv"]
