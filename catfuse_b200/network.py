"""Native network executor for rewritten spiking ResNets.

After the rewrite, a SEW / Spiking ResNet is a chain of fused conv patterns.
Running them one by one through their module ``forward`` would convert
layouts at every boundary; :class:`CTFNetwork` instead compiles the chain into
a :class:`NetworkPlan` — one pack kernel, one fused Conv->BN->LIF launch per
conv layer (the SEW residual combine fused into the epilogue of the block's
second conv), an optional max-pool, and the avgpool+fc head — over static
buffers in the kernels' [B, H, W, T, C] fp16 layout, captured into a CUDA
graph per input shape.  The rewritten module tree stays attached (state
dicts, routing stats, module-level use).

Membrane state: every LIF layer owns a v buffer [B, H, W, C] fp32 in the plan.
After ``reset()`` (``functional.reset_net``) the next forward starts from
v = 0 (the kernels skip the read); otherwise v_T of the previous forward is
carried in (StateCarry), as SpikingJelly does.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn as nn

from . import ops
from .ops import LIFConfig
from .patterns import (CTFSEWBasicBlock, CTFSpikingBasicBlock, PartialFusionConvBNLIF,
                       STFusionConvBNLIF, _ConvBN)
from .sj.neuron import is_lif


class UnsupportedTopology(ValueError):
    pass


# Network operand precision: "fp16" (fp16 weights, the reference GPU path's
# operand precision: TF32 cuDNN / fp16 StreamFuse), "split" (hi + lo weights
# and stem input everywhere) or "fp32" (fp32-faithful: the real-valued stem as
# hi + lo, every spike layer that the channel-major kernel runs with exact
# integer weight planes, the rest split).
NETWORK_PRECISIONS = ("fp16", "split", "fp32")


@dataclass
class ConvStep:
    name: str
    native: object                # patterns.NativeConv
    src: int                      # activation buffer index
    dst: int
    identity: Optional[int] = None
    res_mode: str = "none"
    lif: Optional[LIFConfig] = None   # None: z-only (Conv+BN branch)
    sparse: bool = False
    # filled at build time
    v: Optional[torch.Tensor] = None
    mask: Optional[torch.Tensor] = None
    wp: Optional[torch.Tensor] = None
    scale: Optional[torch.Tensor] = None
    shift: Optional[torch.Tensor] = None
    stride: int = 0               # launch geometry (differs from spec for im2col)
    pad: int = 0
    im2col: bool = False
    prec: str = "fp16"            # operand precision of this launch (ops.PRECISIONS)
    # dual launch: this conv also computes `dual` (the block's downsample) in
    # the same kernel (concatenated weight rows); the partner is skipped
    dual: Optional["ConvStep"] = None
    fused: bool = False
    dual_wp: Optional[torch.Tensor] = None
    dual_scale: Optional[torch.Tensor] = None
    dual_shift: Optional[torch.Tensor] = None


@dataclass
class PoolStep:
    src: int
    dst: int
    k: int
    s: int
    p: int


@dataclass
class Graphable:
    steps: List[object] = field(default_factory=list)


def _native_of(m):
    if hasattr(m, "native_conv"):
        return m.native_conv()
    raise UnsupportedTopology(f"{type(m).__name__} is not a fused conv pattern")


def _lif_of(m) -> LIFConfig:
    return LIFConfig(float(m.tau), float(m.v_threshold),
                     None if m.v_reset is None else float(m.v_reset),
                     bool(getattr(m, "decay_input", True)))


def _stem_pattern(model):
    c = model.conv1
    if isinstance(c, (PartialFusionConvBNLIF, STFusionConvBNLIF)):
        return c
    if isinstance(c, nn.Conv2d) and isinstance(model.bn1, nn.BatchNorm2d) and is_lif(model.sn1):
        return PartialFusionConvBNLIF.from_sj_modules(c, model.bn1, model.sn1).to(c.weight.device)
    raise UnsupportedTopology("stem is not Conv-BN-LIF")


def _block_parts(b):
    """-> (kind, first, second, downsample, cnf) with fused patterns."""
    if isinstance(b, CTFSEWBasicBlock):
        return "sew", b.fused_first, b.fused_second, b.fused_downsample, b.cnf
    if isinstance(b, CTFSpikingBasicBlock):
        return "spiking", b.fused_first, b.fused_second_add, b.downsample, None
    if type(b).__name__ == "BasicBlock":
        first, second = b.conv1, b.conv2
        if not hasattr(first, "native_conv") or not hasattr(second, "native_conv"):
            raise UnsupportedTopology("block convs are not fused")
        ds = None
        if getattr(b, "downsample", None) is not None:
            ds = b.downsample[0] if isinstance(b.downsample, nn.Sequential) else b.downsample
            if not hasattr(ds, "native_conv"):
                raise UnsupportedTopology("downsample is not fused")
        if getattr(b, "cnf", None) is None:
            raise UnsupportedTopology("un-rewritten standard Spiking BasicBlock")
        return "sew", first, second, ds, b.cnf
    raise UnsupportedTopology(f"unsupported block {type(b).__name__}")


class NetworkPlan:
    """Kernel launch list + static buffers for one input shape."""

    def __init__(self, model: nn.Module, T: int, B: int, H: int, W: int, device,
                 use_sparse: bool = False, precision: str = "fp16"):
        if precision not in NETWORK_PRECISIONS:
            raise ValueError(f"precision must be one of {NETWORK_PRECISIONS}")
        self.precision = precision
        hi_lo = precision != "fp16"   # real-valued stem input carried as hi + lo
        self.T, self.B, self.H, self.W = T, B, H, W
        self.device = torch.device(device)
        self.steps = []
        self.shapes = []  # activation buffer shapes (B, H, W, T, C)
        stem = _stem_pattern(model)
        cin = stem.in_channels
        self.in_channels = cin
        self.x_in = torch.zeros((T, B, cin, H, W), dtype=torch.float32, device=self.device)
        sspec = _native_of(stem).spec
        k0 = sspec.kernel_size
        # A stem with few input channels runs as a 1x1 convolution over an
        # im2col-packed input (one K chunk per tile instead of k*k taps).
        # (hi + lo precision: the parts of the real-valued input side by side,
        # for any kernel size)
        kk_mult = 2 if hi_lo else 1
        # (few input channels, e.g. images: a k x k stem over 3 channels would
        # otherwise run k*k tiny K=16 chunks per tile)
        self.im2col = k0 > 1 and (hi_lo or cin <= 8)
        if self.im2col:
            ho0, wo0 = sspec.output_hw(H, W)
            self.shapes.append((B, ho0, wo0, T, ops.pad16(kk_mult * cin * k0 * k0)))
        else:
            self.shapes.append((B, H, W, T, ops.pad16(cin)))
        self.stem_geom = (k0, sspec.stride, sspec.padding)
        cur = 0

        def add_conv(name, pat, src, identity=None, res_mode="none", lif=True):
            nat = _native_of(pat)
            spec = nat.spec
            b_, h_, w_, t_, c_ = self.shapes[src]
            ho, wo = spec.output_hw(h_, w_)
            self.shapes.append((b_, ho, wo, t_, spec.out_channels))
            dst = len(self.shapes) - 1
            sparse = use_sparse and isinstance(pat, STFusionConvBNLIF)
            if precision == "fp16":
                prec = "fp16"
            elif precision == "fp32" and ops.planes_ok(spec.out_channels, c_):
                prec, sparse = "planes", False   # the plane mode runs dense
            else:
                prec, sparse = "split", False    # device EGD runs fp16 weights
            self.steps.append(ConvStep(name, nat, src, dst, identity, res_mode,
                                       _lif_of(pat) if lif else None, sparse, prec=prec))
            return dst

        pairs = []   # (conv1, downsample) steps of SEW blocks
        if self.im2col:
            b_, h_, w_, t_, c_ = self.shapes[0]
            self.shapes.append((b_, h_, w_, t_, sspec.out_channels))
            self.steps.append(ConvStep("stem", _native_of(stem), 0, 1, None, "none", _lif_of(stem),
                                       False, stride=1, pad=0, im2col=True,
                                       prec="split" if hi_lo else "fp16"))
            cur = 1
        else:
            cur = add_conv("stem", stem, cur)
        mp = getattr(model, "maxpool", None)
        if isinstance(mp, nn.MaxPool2d):
            k = mp.kernel_size if isinstance(mp.kernel_size, int) else mp.kernel_size[0]
            s = mp.stride if isinstance(mp.stride, int) else mp.stride[0]
            p = mp.padding if isinstance(mp.padding, int) else mp.padding[0]
            b_, h_, w_, t_, c_ = self.shapes[cur]
            self.shapes.append((b_, (h_ + 2 * p - k) // s + 1, (w_ + 2 * p - k) // s + 1, t_, c_))
            self.steps.append(PoolStep(cur, len(self.shapes) - 1, k, s, p))
            cur = len(self.shapes) - 1
        elif mp is not None and not isinstance(mp, nn.Identity):
            raise UnsupportedTopology(f"unsupported pooling {type(mp).__name__}")

        for li in range(1, 5):
            stage = getattr(model, f"layer{li}")
            for bi, blk in enumerate(stage):
                kind, first, second, ds, cnf = _block_parts(blk)
                nm = f"layer{li}.{bi}"
                x_in = cur
                h1 = add_conv(nm + ".conv1", first, x_in)
                if kind == "sew":
                    ident = add_conv(nm + ".downsample", ds, x_in) if ds is not None else x_in
                    if ds is not None:
                        pairs.append((self.steps[-2], self.steps[-1]))
                    cur = add_conv(nm + ".conv2", second, h1, ident, cnf)
                else:
                    ident = x_in
                    if ds is not None:
                        ident = add_conv(nm + ".downsample", ds, x_in, lif=False)
                    cur = add_conv(nm + ".conv2", second, h1, ident, "add_pre")
        self.final = cur
        fc = model.fc
        if not isinstance(fc, nn.Linear):
            raise UnsupportedTopology("classifier is not Linear")
        self.fc_w = fc.weight.detach().float().contiguous().to(self.device)
        self.fc_b = None if fc.bias is None else fc.bias.detach().float().contiguous().to(self.device)
        self.logits = torch.zeros((T, B, fc.out_features), dtype=torch.float32, device=self.device)
        self.acts = [torch.zeros(s, dtype=torch.float16, device=self.device) for s in self.shapes]
        for st in self.steps:
            if isinstance(st, ConvStep):
                st.wp, st.scale, st.shift = st.native.packed(self.device, st.prec)
                if st.im2col:
                    w0 = st.native.params.weight.detach().to(self.device)
                    if st.prec == "split":
                        st.wp, pre = ops.im2col_weight_split(w0, self.shapes[0][-1])
                        _, sc0, _ = st.native.packed(self.device, "fp16")
                        base = (torch.ones(w0.shape[0], dtype=torch.float32, device=self.device)
                                if sc0 is None else sc0.float())
                        st.scale = (base / pre).contiguous()
                    else:
                        st.wp = ops.im2col_weight(w0, self.shapes[0][-1])
                else:
                    st.stride, st.pad = st.native.spec.stride, st.native.spec.padding
                b_, ho, wo, t_, co = self.shapes[st.dst]
                if st.lif is not None:
                    st.v = torch.zeros((b_, ho, wo, co), dtype=torch.float32, device=self.device)
                if st.sparse:
                    cin_p = self.shapes[st.src][-1]
                    g = ops.conv_geometry(t_, b_, ho, wo, co, cin_p, st.stride, True)
                    st.mask = torch.zeros(g["n_mtiles"], dtype=torch.int32, device=self.device)
        for first, ds in pairs:
            self._try_dual(first, ds)
        from .hardware import detect_hardware
        frac = detect_hardware().egd_max_active_frac
        self.egd_frac = frac if frac >= 0 else 1.0
        self.fresh = True
        self._graphs = {}

    def _try_dual(self, first: ConvStep, ds: ConvStep) -> None:
        """Run a SEW block's 1x1 stride-s downsample in the launch of its 3x3
        stride-s first conv (same input; the downsample's weights at the
        centre tap) when both are plain fp16 LIF convs on the channel-major
        kernel."""
        fs, dsp = first.native.spec, ds.native.spec
        c1, c2 = fs.out_channels, dsp.out_channels
        cin_p = self.shapes[first.src][-1]
        ok = (first.prec == ds.prec == "fp16" and not first.sparse and not ds.sparse
              and first.lif is not None and ds.lif is not None and first.lif == ds.lif
              and first.identity is None and ds.identity is None
              and fs.kernel_size == 3 and fs.padding == 1 and dsp.kernel_size == 1
              and dsp.padding == 0 and fs.stride == dsp.stride and first.src == ds.src
              and (c1 + c2) % 128 == 0 and c1 % 128 == 0 and ops.planes_ok(c1 + c2, cin_p))
        if not ok:
            return
        dev = self.device
        w1 = first.native.params.weight.detach().float().to(dev)
        w2 = ds.native.params.weight.detach().float().to(dev)
        w = torch.zeros((c1 + c2, w1.shape[1], 3, 3), dtype=torch.float32, device=dev)
        w[:c1] = w1
        w[c1:, :, 1, 1] = w2[:, :, 0, 0]
        first.dual_wp = ops.pack_conv_weight(w, cin_p)
        parts = []
        for st, c in ((first, c1), (ds, c2)):
            sc = torch.ones(c, device=dev) if st.scale is None else st.scale.float()
            sh = torch.zeros(c, device=dev) if st.shift is None else st.shift.float()
            parts.append((sc, sh))
        first.dual_scale = torch.cat([parts[0][0], parts[1][0]]).contiguous()
        first.dual_shift = torch.cat([parts[0][1], parts[1][1]]).contiguous()
        first.dual = ds
        ds.fused = True

    def conv_launch(self, st: ConvStep, fresh: bool) -> None:
        """The kernel launch of one conv step (nothing for a step whose work
        rides in its partner's dual launch)."""
        if st.fused:
            return
        if st.dual is not None:
            ds = st.dual
            ops.conv_bn_lif_dual(self.acts[st.src], st.dual_wp, st.dual_scale, st.dual_shift,
                                 st.native.spec.out_channels, st.stride, st.pad,
                                 v_in=None if fresh else st.v, v_out=st.v, out=self.acts[st.dst],
                                 v_in2=None if fresh else ds.v, v_out2=ds.v,
                                 out2=self.acts[ds.dst], lif=st.lif)
            return
        spec = st.native.spec
        if st.sparse:
            ops.prescan_conv_tiles(self.acts[st.src], spec.out_channels, spec.kernel_size,
                                   spec.kernel_size, spec.stride, spec.padding,
                                   mask_out=st.mask, egd=True)
        ident = self.acts[st.identity] if st.identity is not None else None
        if st.lif is None:
            ops.conv_bn_lif(self.acts[st.src], st.wp, st.scale, st.shift, st.stride,
                            st.pad, res_mode="z_only", out=self.acts[st.dst],
                            precision=st.prec)
        else:
            ops.conv_bn_lif(self.acts[st.src], st.wp, st.scale, st.shift, st.stride,
                            st.pad, identity=ident,
                            res_mode=st.res_mode if ident is not None else "none",
                            v_in=None if fresh else st.v, v_out=st.v,
                            tile_mask=st.mask if st.sparse else None, lif=st.lif,
                            out=self.acts[st.dst], precision=st.prec,
                            egd_max_active_frac=self.egd_frac if st.sparse else None)

    # ---- execution ---------------------------------------------------------
    def launches(self) -> int:
        n = 2  # pack + head
        for st in self.steps:
            if isinstance(st, ConvStep) and st.fused:
                continue
            n += 1 + (1 if isinstance(st, ConvStep) and st.sparse else 0)
        return n

    def pack_input(self):
        if self.im2col:
            k, s_, p_ = self.stem_geom
            pack = ops.pack_im2col_split if self.precision != "fp16" else ops.pack_im2col
            pack(self.x_in, k, s_, p_, self.shapes[0][-1], out=self.acts[0])
        else:
            ops.pack_tbchw(self.x_in, self.shapes[0][-1], out=self.acts[0])

    def run_eager(self, fresh: bool):
        self.pack_input()
        for st in self.steps:
            if isinstance(st, PoolStep):
                ops.maxpool_bhwtc(self.acts[st.src], st.k, st.s, st.p, out=self.acts[st.dst])
            else:
                self.conv_launch(st, fresh)
        ops.avgpool_fc(self.acts[self.final], self.fc_w, self.fc_b, out=self.logits)

    def run(self, use_graph: bool = True):
        fresh = self.fresh
        if not use_graph:
            self.run_eager(fresh)
        else:
            g = self._graphs.get(fresh)
            if g is None:
                # warm up on a side stream (the graph-capture protocol), then capture
                s = torch.cuda.Stream(device=self.device)
                s.wait_stream(torch.cuda.current_stream(self.device))
                saved = [st.v.clone() for st in self.steps if isinstance(st, ConvStep) and st.v is not None]
                with torch.cuda.stream(s):
                    self.run_eager(fresh)
                torch.cuda.current_stream(self.device).wait_stream(s)
                i = 0
                for st in self.steps:
                    if isinstance(st, ConvStep) and st.v is not None:
                        st.v.copy_(saved[i])
                        i += 1
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.run_eager(fresh)
                self._graphs[fresh] = g
            g.replay()
        self.fresh = False
        return self.logits

    def layer_states(self):
        """{layer name: v_T in the reference layout [B, C, H, W]}."""
        out = {}
        for st in self.steps:
            if isinstance(st, ConvStep) and st.v is not None:
                out[st.name] = ops.v_to_nchw(st.v)
        return out


class CTFNetwork(nn.Module):
    """Wraps a rewritten spiking ResNet; ``forward(x[T, B, C, H, W])`` runs the
    native plan and returns logits [T, B, classes] (fp32)."""

    #: When true, every forward reads the device error word of the bounded
    #: waits (one stream synchronisation) and raises CatfuseNativeError if a
    #: wait expired; the test suite turns it on.
    check_errors = False

    def __init__(self, model: nn.Module, use_graph: bool = True, use_sparse: bool = True,
                 precision: str = "fp16"):
        super().__init__()
        if precision not in NETWORK_PRECISIONS:
            raise ValueError(f"precision must be one of {NETWORK_PRECISIONS}")
        self.model = model
        self.use_graph = use_graph
        self.use_sparse = use_sparse
        self.precision = precision
        self._plans = {}
        self._fresh = True
        # validate now (raises UnsupportedTopology)
        _stem_pattern(model)
        for li in range(1, 5):
            for blk in getattr(model, f"layer{li}"):
                _block_parts(blk)

    def reset(self):
        self._fresh = True
        for p in self._plans.values():
            p.fresh = True

    def plan_for(self, x: torch.Tensor) -> NetworkPlan:
        T, B, C, H, W = x.shape
        key = (T, B, C, H, W, x.device)
        p = self._plans.get(key)
        if p is None:
            p = NetworkPlan(self.model, T, B, H, W, x.device, self.use_sparse, self.precision)
            self._plans[key] = p
        return p

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 5:
            raise ValueError("expected x[T, B, C, H, W]")
        if not x.is_cuda:
            raise RuntimeError("CTFNetwork runs on an sm_100 GPU only (CPU tensor given)")
        p = self.plan_for(x)
        if self._fresh:
            p.fresh = True
            self._fresh = False
        p.x_in.copy_(x)
        out = p.run(self.use_graph).clone()
        if self.check_errors:
            # synchronises: raises if a bounded device wait expired in this forward
            ops.check_device_error()
        return out
