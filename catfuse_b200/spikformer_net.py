"""Native executor for a rewritten Spikformer (SPS tokenizer + spiking
self-attention blocks + token-mean head).

The whole forward runs as one CUDA graph of sm_100a kernels over static
buffers in the [B, H, W, T, C] fp16 layout; the 64 tokens of the 8x8 SPS map
are the pixels of that map, so every Linear -> BN1d -> LIF is a 1x1 fused
conv on the token map and ``cf_ssa_lif`` reads q, k, v as [B, N, T, C]:

* SPS: im2col stem conv0 (3 -> embed/8; output channels padded to a
  multiple of 32 with zero weights and zero affine, which never spike),
  conv1, conv2 + 3x3/2 max-pool, conv3 + max-pool, rpe conv whose epilogue
  adds the pooled features (SEW ADD after the LIF);
* each block: q, k, v (1x1 fused conv + BN1d + LIF), the attention core +
  attention LIF (``cf_ssa_lif``), proj with the residual add in its epilogue,
  fc1, fc2 with the residual add;
* head: token mean -> pre-head LIF -> linear (``cf_token_mean_lif_fc``).

Residual sums are spike counts (integers <= 2 * depth + 2), exact in fp16.
Membrane state: one v buffer per LIF layer; after ``reset()`` the next
forward starts from v = 0, otherwise v_T is carried in (StateCarry).
Reference model: ``models/spikformer_github.py:57-329``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn as nn

from . import ops
from .implementations.base import folded_affine
from .ops import LIFConfig
from .sj.neuron import is_lif


class UnsupportedSpikformer(ValueError):
    pass


def is_spikformer(model: nn.Module) -> bool:
    return all(hasattr(model, a) for a in ("patch_embed", "blocks", "pre_head_lif", "head"))


def _lif_cfg(m) -> LIFConfig:
    return LIFConfig(float(getattr(m, "tau", 2.0)), float(m.v_threshold),
                     None if m.v_reset is None else float(m.v_reset),
                     bool(getattr(m, "decay_input", True)))


def _conv_parts(mod, name):
    """(weight [Cout, Cin, k, k] fp32, scale or None, shift or None, LIFConfig,
    stride, pad) of a fused conv / linear pattern after the rewrite."""
    if hasattr(mod, "native_conv"):
        nat = mod.native_conv()
        spec, params = nat.spec, nat.params
    elif hasattr(mod, "_spec") and hasattr(mod, "_params"):   # FusedLinearLIF
        spec, params = mod._spec(), mod._params()
    else:
        raise UnsupportedSpikformer(f"{name} ({type(mod).__name__}) is not a fused pattern")
    scale, shift = folded_affine(spec, params)
    return (params.weight.detach().float(), scale, shift, spec.lif_config(), spec.stride,
            spec.padding)


@dataclass
class _Conv:
    name: str
    src: int
    dst: int
    w: torch.Tensor              # [Cout_buf, Cin_buf, k, k] fp32 (padded)
    scale: Optional[torch.Tensor]
    shift: Optional[torch.Tensor]
    lif: LIFConfig
    stride: int
    pad: int
    identity: Optional[int] = None
    prec: str = "fp16"
    im2col: bool = False
    # built
    wp: Optional[torch.Tensor] = None
    v: Optional[torch.Tensor] = None


@dataclass
class _Pool:
    src: int
    dst: int


@dataclass
class _SSA:
    name: str
    q: int
    k: int
    v: int
    dst: int
    heads: int
    scale: float
    lif: LIFConfig
    vstate: Optional[torch.Tensor] = None


def _pad_to(c: int, m: int) -> int:
    return (c + m - 1) // m * m


class SpikformerPlan:
    """Launch list + static buffers of one input shape."""

    def __init__(self, model: nn.Module, T: int, B: int, H: int, W: int, device,
                 precision: str = "fp16"):
        from .network import NETWORK_PRECISIONS
        if precision not in NETWORK_PRECISIONS:
            raise ValueError(f"precision must be one of {NETWORK_PRECISIONS}")
        self.T, self.B, self.H, self.W = T, B, H, W
        self.device = torch.device(device)
        self.precision = precision
        hi_lo = precision != "fp16"
        self.shapes: List[tuple] = []
        self.steps: List[object] = []
        pe = model.patch_embed

        def new_buf(b, h, w, c):
            self.shapes.append((b, h, w, T, c))
            return len(self.shapes) - 1

        def choose_prec(cout, cin_p):
            if precision == "fp16":
                return "fp16"
            if precision == "fp32" and ops.planes_ok(cout, cin_p):
                return "planes"
            return "split"

        # ---- SPS ----------------------------------------------------------
        w0, sc0, sh0, lif0, s0, p0 = _conv_parts(pe.conv0, "patch_embed.conv0")
        cin = w0.shape[1]
        k0 = w0.shape[2]
        Kp = ops.pad16((2 if hi_lo else 1) * cin * k0 * k0)
        self.stem_geom = (k0, s0, p0)
        Ho, Wo = (H + 2 * p0 - k0) // s0 + 1, (W + 2 * p0 - k0) // s0 + 1
        self.in_channels = cin
        x0 = new_buf(B, Ho, Wo, Kp)
        cur_c = w0.shape[0]
        cbuf = _pad_to(cur_c, 32)
        y = new_buf(B, Ho, Wo, cbuf)
        self.steps.append(_Conv("patch_embed.conv0", x0, y, w0, sc0, sh0, lif0, 1, 0,
                                prec="split" if hi_lo else "fp16", im2col=True))
        h, w = Ho, Wo
        for i in (1, 2, 3):
            wi, sci, shi, lifi, si, pi = _conv_parts(getattr(pe, f"conv{i}"), f"patch_embed.conv{i}")
            cin_buf = self.shapes[y][-1]
            ho, wo = (h + 2 * pi - wi.shape[2]) // si + 1, (w + 2 * pi - wi.shape[3]) // si + 1
            cout = wi.shape[0]
            dst = new_buf(B, ho, wo, _pad_to(cout, 32))
            self.steps.append(_Conv(f"patch_embed.conv{i}", y, dst, wi, sci, shi, lifi, si, pi,
                                    prec=choose_prec(_pad_to(cout, 32), cin_buf)))
            y, h, w = dst, ho, wo
            if i in (2, 3):
                pool = getattr(pe, f"pool{i}")
                if not isinstance(pool, nn.MaxPool2d) or pool.kernel_size not in (3, (3, 3)):
                    raise UnsupportedSpikformer("SPS pools must be 3x3/2 max-pools")
                h2, w2 = (h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1
                dst = new_buf(B, h2, w2, self.shapes[y][-1])
                self.steps.append(_Pool(y, dst))
                y, h, w = dst, h2, w2
        feat = y
        wr, scr, shr, lifr, sr, pr = _conv_parts(pe.rpe_conv, "patch_embed.rpe_conv")
        C = wr.shape[0]
        tok = new_buf(B, h, w, C)
        self.steps.append(_Conv("patch_embed.rpe_conv", feat, tok, wr, scr, shr, lifr, sr, pr,
                                identity=feat, prec=choose_prec(C, self.shapes[feat][-1])))
        self.N = h * w
        self.dim = C
        x = tok
        # ---- encoder blocks ------------------------------------------------
        for bi, blk in enumerate(model.blocks):
            a, m = blk.attn, blk.mlp
            pre = f"blocks.{bi}."
            qkv = []
            for n in ("q", "k", "v"):
                wn, scn, shn, lifn, _, _ = _conv_parts(getattr(a, n), pre + "attn." + n)
                dst = new_buf(B, h, w, C)
                self.steps.append(_Conv(pre + "attn." + n, x, dst, wn.reshape(C, C, 1, 1), scn,
                                        shn, lifn, 1, 0, prec=choose_prec(C, C)))
                qkv.append(dst)
            if not is_lif(a.attn_lif):
                raise UnsupportedSpikformer("attn_lif must be a LIF node")
            att = new_buf(B, h, w, C)
            self.steps.append(_SSA(pre + "attn.attn_lif", qkv[0], qkv[1], qkv[2], att,
                                   int(a.num_heads), float(getattr(a, "scale", (C // a.num_heads) ** -0.5)),
                                   _lif_cfg(a.attn_lif)))
            wp_, scp, shp, lifp, _, _ = _conv_parts(a.proj, pre + "attn.proj")
            x1 = new_buf(B, h, w, C)
            self.steps.append(_Conv(pre + "attn.proj", att, x1, wp_.reshape(C, C, 1, 1), scp, shp,
                                    lifp, 1, 0, identity=x, prec=choose_prec(C, C)))
            w1, sc1, sh1, lif1, _, _ = _conv_parts(m.fc1, pre + "mlp.fc1")
            hid = w1.shape[0]
            hb = new_buf(B, h, w, hid)
            self.steps.append(_Conv(pre + "mlp.fc1", x1, hb, w1.reshape(hid, C, 1, 1), sc1, sh1,
                                    lif1, 1, 0, prec=choose_prec(hid, C)))
            w2, sc2, sh2, lif2, _, _ = _conv_parts(m.fc2, pre + "mlp.fc2")
            x2 = new_buf(B, h, w, C)
            self.steps.append(_Conv(pre + "mlp.fc2", hb, x2, w2.reshape(C, hid, 1, 1), sc2, sh2,
                                    lif2, 1, 0, identity=x1, prec=choose_prec(C, hid)))
            x = x2
        self.final = x
        if not is_lif(model.pre_head_lif) or not isinstance(model.head, nn.Linear):
            raise UnsupportedSpikformer("head must be LIF -> Linear")
        self.head_lif = _lif_cfg(model.pre_head_lif)
        self.head_w = model.head.weight.detach().float().contiguous().to(self.device)
        self.head_b = (None if model.head.bias is None
                       else model.head.bias.detach().float().contiguous().to(self.device))
        self.head_v = torch.zeros((B, C), dtype=torch.float32, device=self.device)
        self.logits = torch.zeros((T, B, self.head_w.shape[0]), dtype=torch.float32,
                                  device=self.device)
        self.x_in = torch.zeros((T, B, cin, H, W), dtype=torch.float32, device=self.device)
        self.acts = [torch.zeros(s, dtype=torch.float16, device=self.device) for s in self.shapes]
        for st in self.steps:
            if isinstance(st, _Conv):
                self._build_conv(st)
            elif isinstance(st, _SSA):
                st.vstate = torch.zeros((B, self.N, C), dtype=torch.float32, device=self.device)
        self.fresh = True
        self._graphs = {}

    # ---- weight preparation --------------------------------------------------
    def _build_conv(self, st: _Conv):
        dev = self.device
        b_, ho, wo, t_, cout_buf = self.shapes[st.dst]
        cin_buf = self.shapes[st.src][-1]
        w = st.w.to(dev)
        cout, cin = w.shape[0], w.shape[1]
        scale = (torch.ones(cout, device=dev) if st.scale is None else st.scale.to(dev).float())
        shift = (torch.zeros(cout, device=dev) if st.shift is None else st.shift.to(dev).float())
        if cout_buf > cout:   # padded output channels: zero weights, zero affine -> no spikes
            w = torch.cat([w, torch.zeros((cout_buf - cout, *w.shape[1:]), device=dev)], 0)
            scale = torch.cat([scale, torch.zeros(cout_buf - cout, device=dev)])
            shift = torch.cat([shift, torch.zeros(cout_buf - cout, device=dev)])
        if st.im2col:
            if st.prec == "split":
                st.wp, pre = ops.im2col_weight_split(w, cin_buf)
                scale = scale / pre
            else:
                st.wp = ops.im2col_weight(w, cin_buf)
        else:
            if cin_buf > cin:  # padded input channels of the buffer carry zeros
                w = torch.cat([w, torch.zeros((w.shape[0], cin_buf - cin, *w.shape[2:]),
                                              device=dev)], 1)
            if st.prec == "planes":
                st.wp, pre = ops.pack_conv_weight_planes(w, cin_buf)
                scale = scale / pre
            elif st.prec == "split":
                st.wp, pre = ops.pack_conv_weight_split(w, cin_buf)
                scale = scale / pre
            else:
                st.wp = ops.pack_conv_weight(w, cin_buf)
        st.scale = scale.contiguous()
        st.shift = shift.contiguous()
        st.v = torch.zeros((b_, ho, wo, cout_buf), dtype=torch.float32, device=dev)

    # ---- execution -----------------------------------------------------------
    def launches(self) -> int:
        return 2 + len(self.steps)

    def pack_input(self):
        k, s_, p_ = self.stem_geom
        pack = ops.pack_im2col_split if self.precision != "fp16" else ops.pack_im2col
        pack(self.x_in, k, s_, p_, self.shapes[0][-1], out=self.acts[0])

    def run_eager(self, fresh: bool):
        self.pack_input()
        for st in self.steps:
            if isinstance(st, _Pool):
                ops.maxpool_bhwtc(self.acts[st.src], 3, 2, 1, out=self.acts[st.dst])
            elif isinstance(st, _SSA):
                q, k, v, o = (self.acts[i] for i in (st.q, st.k, st.v, st.dst))
                B_, h, w, T_, C = q.shape
                view = lambda t: t.view(B_, h * w, T_, C)
                ops.ssa_lif(view(q), view(k), view(v), st.heads, st.scale,
                            v_in=None if fresh else st.vstate, v_out=st.vstate, lif=st.lif,
                            out=view(o))
            else:
                ident = self.acts[st.identity] if st.identity is not None else None
                ops.conv_bn_lif(self.acts[st.src], st.wp, st.scale, st.shift,
                                1 if st.im2col else st.stride, 0 if st.im2col else st.pad,
                                identity=ident, res_mode="add" if ident is not None else "none",
                                v_in=None if fresh else st.v, v_out=st.v, lif=st.lif,
                                out=self.acts[st.dst], precision=st.prec)
        fin = self.acts[self.final]
        B_, h, w, T_, C = fin.shape
        ops.token_mean_lif_fc(fin.view(B_, h * w, T_, C), self.head_w, self.head_b,
                              v_in=None if fresh else self.head_v, v_out=self.head_v,
                              lif=self.head_lif, out=self.logits)

    def run(self, use_graph: bool = True):
        fresh = self.fresh
        if not use_graph:
            self.run_eager(fresh)
        else:
            g = self._graphs.get(fresh)
            if g is None:
                states = ([st.v for st in self.steps if isinstance(st, _Conv)]
                          + [st.vstate for st in self.steps if isinstance(st, _SSA)] + [self.head_v])
                saved = [t.clone() for t in states]
                s = torch.cuda.Stream(device=self.device)
                s.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(s):
                    self.run_eager(fresh)
                torch.cuda.current_stream(self.device).wait_stream(s)
                for t, c in zip(states, saved):
                    t.copy_(c)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.run_eager(fresh)
                self._graphs[fresh] = g
            g.replay()
        self.fresh = False
        return self.logits

    def layer_spikes(self):
        """{reference LIF name: spikes [T, B, ...]} of every LIF layer of the
        last forward (residual outputs minus their identity; SPS maps as
        [T, B, C, H, W], tokens as [T, B, N, C])."""
        out = {}
        for st in self.steps:
            if isinstance(st, _Pool):
                continue
            y = self.acts[st.dst]
            if isinstance(st, _Conv) and st.identity is not None:
                y = y - self.acts[st.identity]
            B_, h, w, T_, Cb = y.shape
            if st.name.startswith("patch_embed"):
                c = st.w.shape[0] if isinstance(st, _Conv) else Cb
                key = st.name.replace("conv", "lif").replace("rpe_lif", "rpe_lif")
                if st.name.endswith("rpe_conv"):
                    key = "patch_embed.rpe_lif"
                out[key] = y[..., :c].permute(3, 0, 4, 1, 2).float().cpu()
            else:
                out[st.name] = y.reshape(B_, h * w, T_, Cb).permute(2, 0, 1, 3).float().cpu()
        return out


class CTFSpikformer(nn.Module):
    """Wraps a rewritten Spikformer; ``forward(x[T, B, 3, H, W])`` runs the
    native plan and returns logits [T, B, classes] (fp32)."""

    #: When true, every forward reads the device error word of the bounded
    #: waits (one stream synchronisation) and raises CatfuseNativeError if a
    #: wait expired; the test suite turns it on.
    check_errors = False

    def __init__(self, model: nn.Module, use_graph: bool = True, precision: str = "fp16"):
        super().__init__()
        if not is_spikformer(model):
            raise UnsupportedSpikformer("not a Spikformer")
        self.model = model
        self.use_graph = use_graph
        self.precision = precision
        self._plans = {}
        self._fresh = True

    def reset(self):
        self._fresh = True
        for p in self._plans.values():
            p.fresh = True

    def plan_for(self, x: torch.Tensor) -> SpikformerPlan:
        T, B, C, H, W = x.shape
        key = (T, B, C, H, W, x.device)
        p = self._plans.get(key)
        if p is None:
            p = SpikformerPlan(self.model, T, B, H, W, x.device, self.precision)
            self._plans[key] = p
        return p

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 4:
            x = x.unsqueeze(0).repeat(int(getattr(self.model, "T", 4)), 1, 1, 1, 1)
        if x.dim() != 5:
            raise ValueError("expected x[T, B, C, H, W]")
        if not x.is_cuda:
            raise RuntimeError("CTFSpikformer runs on an sm_100 GPU only (CPU tensor given)")
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


__all__ = ["SpikformerPlan", "CTFSpikformer", "is_spikformer", "UnsupportedSpikformer"]
