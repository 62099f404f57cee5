"""Tensor-level wrappers around the C ABI.

Every function takes CUDA tensors, checks shapes/dtypes/contiguity, passes raw
pointers and the current CUDA stream to the library, and returns new tensors
(or writes the provided ``out`` tensors).  Nothing here computes on the CPU:
a CPU tensor or a missing library raises.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import (FMT_BITS, FMT_F16, FMT_F32, FMT_U8, RES_ADD_POST, RES_ADD_PRE,
                   RES_AND_POST, RES_IAND_POST, RES_NONE, RES_Z_ONLY, CatfuseNativeError)

__all__ = [
    "LIFConfig", "ssa_lif", "lif_fwd", "bn_lif", "add_lif", "avgpool_lif", "pack_tbchw", "unpack_bhwtc",
    "v_to_nhwc", "v_to_nchw", "pack_im2col", "im2col_weight", "pack_conv_weight", "conv_bn_lif", "linear_bn_lif",
    "conv_geometry", "prescan", "prescan_conv_tiles", "conv_chunk", "avgpool_fc", "maxpool_bhwtc",
    "pad16", "SPIKE_FORMATS", "RES_MODES", "PRECISIONS", "pack_conv_weight_split",
    "pack_im2col_split", "im2col_weight_split", "split_prescale", "check_device_error",
    "set_wait_limit", "token_mean_lif_fc", "conv_bn_lif_dual",
]

# Operand precision of the fused conv: "fp16" = fp16 weights (spikes are exact
# in fp16); "split" = weights (and a real-valued stem input) carried as fp16
# hi + lo parts, two MMAs per chunk into the same fp32 accumulator; "planes" =
# weights quantised to 29-bit integers as three fp16 digit planes in separate
# accumulators, exact accumulation for integer activations (spike counts).
PRECISIONS = ("fp16", "split", "planes")
WEIGHT_PARTS = {"fp16": 1, "split": 2, "planes": 3}


def planes_ok(Cout: int, Cin_p: int) -> bool:
    """The integer-plane mode runs on the channel-major kernel only."""
    return Cout % 128 == 0 or (Cout % 64 == 0 and Cin_p >= 64)

SPIKE_FORMATS = {torch.float32: FMT_F32, torch.float16: FMT_F16, torch.uint8: FMT_U8,
                 "bits": FMT_BITS}
RES_MODES = {None: RES_NONE, "none": RES_NONE, "add": RES_ADD_POST, "ADD": RES_ADD_POST,
             "and": RES_AND_POST, "AND": RES_AND_POST, "iand": RES_IAND_POST,
             "IAND": RES_IAND_POST, "add_pre": RES_ADD_PRE, "z_only": RES_Z_ONLY}


@dataclass(frozen=True)
class LIFConfig:
    """SpikingJelly LIFNode parameters.  ``v_reset=None`` = soft reset."""
    tau: float = 2.0
    v_threshold: float = 1.0
    v_reset: Optional[float] = 0.0
    decay_input: bool = True

    def args(self):
        hard = self.v_reset is not None
        return (float(self.tau), float(self.v_threshold),
                float(self.v_reset) if hard else 0.0, int(hard), int(bool(self.decay_input)))


_DEFAULT_LIF = LIFConfig()


def pad16(c: int) -> int:
    return (int(c) + 15) // 16 * 16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, dtype=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise CatfuseNativeError(f"{name} must be a CUDA tensor (no CPU path exists)",
                                 _lib.CF_ERR_INVALID_ARG)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return t


def _zfmt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return FMT_F32
    if t.dtype == torch.float16:
        return FMT_F16
    raise TypeError(f"expected fp32 or fp16, got {t.dtype}")


def _alloc_spikes(T: int, shape, fmt, device):
    n = 1
    for d in shape:
        n *= int(d)
    if fmt == "bits":
        if n % 32:
            raise ValueError("bit-packed spikes need N % 32 == 0")
        return torch.empty((T, n // 32), dtype=torch.int32, device=device)
    return torch.empty((T, *shape), dtype=fmt, device=device)


# ---------------------------------------------------------------------------
# LIF family (reference layout [T, ...])
# ---------------------------------------------------------------------------

def lif_fwd(z: torch.Tensor, v0: Optional[torch.Tensor] = None, lif: LIFConfig = _DEFAULT_LIF,
            spike_dtype=torch.float32, store_v: bool = True):
    """Multi-step LIF over z[T, ...] -> (spikes[T, ...], v_T[...])."""
    _need(z, "z")
    T = z.shape[0]
    inner = tuple(z.shape[1:])
    N = z[0].numel() if T else 0
    if v0 is not None:
        _need(v0, "v0", torch.float32)
        if v0.numel() != N:
            raise ValueError("v0 must have N elements")
    s = _alloc_spikes(T, inner, spike_dtype, z.device)
    vT = torch.empty(inner, dtype=torch.float32, device=z.device) if store_v else None
    _lib.call("cf_lif_fwd", z.data_ptr(), _zfmt(z), _ptr(v0), s.data_ptr(),
              SPIKE_FORMATS[spike_dtype], _ptr(vT), T, N, *lif.args(), _stream())
    return s, vT


def bn_lif(z: Optional[torch.Tensor], scale: Optional[torch.Tensor], shift: Optional[torch.Tensor],
           shape=None, identity: Optional[torch.Tensor] = None, v0: Optional[torch.Tensor] = None,
           lif: LIFConfig = _DEFAULT_LIF, spike_dtype=torch.float32, store_v: bool = True,
           device=None):
    """Per-channel affine (+identity) + LIF over z[T, B, C, *spatial].

    ``z=None`` is the StaticZero case (z' = shift); then ``shape`` gives
    (T, B, C, *spatial)."""
    if z is not None:
        _need(z, "z")
        shape = tuple(z.shape)
        device = z.device
    if shape is None or len(shape) < 3:
        raise ValueError("need z or shape=(T, B, C, ...)")
    T, B, C = shape[0], shape[1], shape[2]
    HW = 1
    for d in shape[3:]:
        HW *= int(d)
    device = device if device is not None else (shift.device if shift is not None else None)
    for t, n in ((scale, "scale"), (shift, "shift")):
        if t is not None:
            _need(t, n, torch.float32)
            if t.numel() != C:
                raise ValueError(f"{n} must have C={C} elements")
    if identity is not None:
        _need(identity, "identity")
        if tuple(identity.shape) != tuple(shape):
            raise ValueError("identity must match z's shape")
    if v0 is not None:
        _need(v0, "v0", torch.float32)
    s = _alloc_spikes(T, shape[1:], spike_dtype, device)
    vT = torch.empty(shape[1:], dtype=torch.float32, device=device) if store_v else None
    _lib.call("cf_bn_lif", _ptr(z), _zfmt(z) if z is not None else FMT_F32, _ptr(scale),
              _ptr(shift), _ptr(identity), _zfmt(identity) if identity is not None else FMT_F32,
              _ptr(v0), s.data_ptr(), SPIKE_FORMATS[spike_dtype], _ptr(vT), T, B, C, HW,
              *lif.args(), _stream())
    return s, vT


def add_lif(x1: torch.Tensor, x2: torch.Tensor, v0: Optional[torch.Tensor] = None,
            lif: LIFConfig = _DEFAULT_LIF, spike_dtype=torch.float32):
    _need(x1, "x1", torch.float32)
    _need(x2, "x2", torch.float32)
    if x1.shape != x2.shape:
        raise ValueError("x1 and x2 must have the same shape")
    T = x1.shape[0]
    N = x1[0].numel() if T else 0
    if v0 is not None:
        _need(v0, "v0", torch.float32)
    s = _alloc_spikes(T, tuple(x1.shape[1:]), spike_dtype, x1.device)
    vT = torch.empty(tuple(x1.shape[1:]), dtype=torch.float32, device=x1.device)
    _lib.call("cf_add_lif", x1.data_ptr(), x2.data_ptr(), _ptr(v0), s.data_ptr(),
              SPIKE_FORMATS[spike_dtype], vT.data_ptr(), T, N, *lif.args(), _stream())
    return s, vT


def avgpool_lif(x: torch.Tensor, k: int = 2, v0: Optional[torch.Tensor] = None,
                lif: LIFConfig = _DEFAULT_LIF, spike_dtype=torch.float32):
    """k x k / stride k average pool over x[T,B,C,H,W] then LIF."""
    _need(x, "x", torch.float32)
    T, B, C, H, W = x.shape
    if H % k or W % k:
        raise ValueError("H and W must be multiples of k")
    if v0 is not None:
        _need(v0, "v0", torch.float32)
    s = torch.empty((T, B, C, H // k, W // k), dtype=spike_dtype, device=x.device)
    vT = torch.empty((B, C, H // k, W // k), dtype=torch.float32, device=x.device)
    _lib.call("cf_avgpool_lif", x.data_ptr(), _ptr(v0), s.data_ptr(), SPIKE_FORMATS[spike_dtype],
              vT.data_ptr(), T, B, C, H, W, int(k), *lif.args(), _stream())
    return s, vT


# ---------------------------------------------------------------------------
# layouts
# ---------------------------------------------------------------------------

def pack_tbchw(x: torch.Tensor, Cp: Optional[int] = None, out: Optional[torch.Tensor] = None):
    """x[T,B,C,H,W] (fp32/fp16) -> [B,H,W,T,Cp] fp16."""
    _need(x, "x")
    T, B, C, H, W = x.shape
    Cp = pad16(C) if Cp is None else int(Cp)
    if out is None:
        out = torch.empty((B, H, W, T, Cp), dtype=torch.float16, device=x.device)
    else:
        _need(out, "out", torch.float16)
    _lib.call("cf_pack_tbchw", x.data_ptr(), _zfmt(x), out.data_ptr(), T, B, C, H, W, Cp, _stream())
    return out


def pack_im2col(x: torch.Tensor, k: int, stride: int, pad: int, Kp: Optional[int] = None,
                out: Optional[torch.Tensor] = None):
    """x[T,B,C,H,W] -> im2col [B,Ho,Wo,T,Kp] fp16 (q = (kh*k+kw)*C + c)."""
    _need(x, "x")
    T, B, C, H, W = x.shape
    Kp = pad16(k * k * C) if Kp is None else int(Kp)
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    if out is None:
        out = torch.empty((B, Ho, Wo, T, Kp), dtype=torch.float16, device=x.device)
    _lib.call("cf_pack_im2col", x.data_ptr(), _zfmt(x), out.data_ptr(), T, B, C, H, W, k, stride,
              pad, Kp, _stream())
    return out


def im2col_weight(w: torch.Tensor, Kp: Optional[int] = None) -> torch.Tensor:
    """w[Cout,Cin,k,k] -> [Cout,1,1,Kp] fp16 matching pack_im2col's q order
    (one-time weight preparation)."""
    Cout, Cin, kh, kw = w.shape
    Kp = pad16(kh * kw * Cin) if Kp is None else int(Kp)
    flat = w.detach().float().permute(0, 2, 3, 1).reshape(Cout, kh * kw * Cin)
    out = torch.zeros((Cout, Kp), dtype=torch.float32, device=w.device)
    out[:, :flat.shape[1]] = flat
    return out.half().reshape(Cout, 1, 1, Kp).contiguous()


def unpack_bhwtc(y: torch.Tensor, C: Optional[int] = None, dtype=torch.float32,
                 out: Optional[torch.Tensor] = None):
    """y[B,H,W,T,C'] fp16 -> [T,B,C,H,W] (the first C channels; requires C' == C)."""
    _need(y, "y", torch.float16)
    B, H, W, T, Cy = y.shape
    C = Cy if C is None else int(C)
    if C != Cy:
        raise ValueError("unpack expects the channel dimension to equal C")
    if out is None:
        out = torch.empty((T, B, C, H, W), dtype=dtype, device=y.device)
    _lib.call("cf_unpack_bhwtc", y.data_ptr(), out.data_ptr(), _zfmt(out), T, B, C, H, W, _stream())
    return out


def v_to_nhwc(v: torch.Tensor, out: Optional[torch.Tensor] = None):
    _need(v, "v", torch.float32)
    B, C, H, W = v.shape
    if out is None:
        out = torch.empty((B, H, W, C), dtype=torch.float32, device=v.device)
    _lib.call("cf_v_layout", v.data_ptr(), out.data_ptr(), B, C, H, W, 1, _stream())
    return out


def v_to_nchw(v: torch.Tensor, out: Optional[torch.Tensor] = None):
    _need(v, "v", torch.float32)
    B, H, W, C = v.shape
    if out is None:
        out = torch.empty((B, C, H, W), dtype=torch.float32, device=v.device)
    _lib.call("cf_v_layout", v.data_ptr(), out.data_ptr(), B, C, H, W, 0, _stream())
    return out


def split_prescale(w: torch.Tensor) -> float:
    """Power of two that brings max|w| to [2^13, 2^14): the lo parts of the
    split weights then stay clear of the fp16 subnormal range."""
    m = float(w.detach().abs().max()) if w.numel() else 0.0
    if m == 0.0 or m != m:
        return 1.0
    import math
    e = math.frexp(m)[1]  # m = f * 2^e, 0.5 <= f < 1
    return float(2.0 ** (14 - e))


def pack_conv_weight_split(w: torch.Tensor, Cin_p: Optional[int] = None,
                           prescale: Optional[float] = None):
    """w[Cout,Cin,KH,KW] -> (wp2[Cout,KH,KW,2*Cin_p] fp16 = hi | lo per tap, prescale).

    The conv computes acc = x * (w * prescale); pass scale / prescale as the
    epilogue scale (exact: prescale is a power of two)."""
    w = w.detach().float().contiguous()
    _need(w, "w", torch.float32)
    Cout, Cin, KH, KW = w.shape
    Cin_p = pad16(Cin) if Cin_p is None else int(Cin_p)
    prescale = split_prescale(w) if prescale is None else float(prescale)
    out = torch.empty((Cout, KH, KW, 2 * Cin_p), dtype=torch.float16, device=w.device)
    _lib.call("cf_pack_conv_weight_split", w.data_ptr(), out.data_ptr(), Cout, Cin, KH, KW, Cin_p,
              prescale, _stream())
    return out, prescale


def pack_im2col_split(x: torch.Tensor, k: int, stride: int, pad: int, Kp: Optional[int] = None,
                      out: Optional[torch.Tensor] = None):
    """x[T,B,C,H,W] -> [B,Ho,Wo,T,Kp] fp16 with hi parts at q < k*k*C and the
    rounding remainders (lo) at q + k*k*C."""
    _need(x, "x")
    T, B, C, H, W = x.shape
    Kp = pad16(2 * k * k * C) if Kp is None else int(Kp)
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    if out is None:
        out = torch.empty((B, Ho, Wo, T, Kp), dtype=torch.float16, device=x.device)
    _lib.call("cf_pack_im2col_split", x.data_ptr(), _zfmt(x), out.data_ptr(), T, B, C, H, W, k,
              stride, pad, Kp, _stream())
    return out


def im2col_weight_split(w: torch.Tensor, Kp: Optional[int] = None):
    """Weights for pack_im2col_split inputs: the row [w, w, 0...] (hi and lo
    input parts both meet the full weight), split into hi | lo.
    -> (wp2[Cout,1,1,2*Kp] fp16, prescale)."""
    Cout, Cin, kh, kw = w.shape
    KK = kh * kw * Cin
    Kp = pad16(2 * KK) if Kp is None else int(Kp)
    flat = w.detach().float().permute(0, 2, 3, 1).reshape(Cout, KK)
    row = torch.zeros((Cout, Kp), dtype=torch.float32, device=w.device)
    row[:, :KK] = flat
    row[:, KK:2 * KK] = flat
    return pack_conv_weight_split(row.reshape(Cout, Kp, 1, 1), Kp)


def planes_prescale(w: torch.Tensor) -> float:
    """Power of two with max|w| * prescale in [2^27, 2^28)."""
    m = float(w.detach().abs().max()) if w.numel() else 0.0
    if m == 0.0 or m != m:
        return 1.0
    import math
    e = math.frexp(m)[1]
    return float(2.0 ** (28 - e))


def pack_conv_weight_planes(w: torch.Tensor, Cin_p: Optional[int] = None,
                            prescale: Optional[float] = None):
    """w[Cout,Cin,KH,KW] -> (wq[Cout,KH,KW,3*Cin_p] fp16 digit planes, prescale):
    q = rint(w * prescale) = q2 * 2^20 + q1 * 2^10 + q0, planes q2 | q1 | q0 per tap."""
    w = w.detach().float().contiguous()
    _need(w, "w", torch.float32)
    Cout, Cin, KH, KW = w.shape
    Cin_p = pad16(Cin) if Cin_p is None else int(Cin_p)
    prescale = planes_prescale(w) if prescale is None else float(prescale)
    out = torch.empty((Cout, KH, KW, 3 * Cin_p), dtype=torch.float16, device=w.device)
    _lib.call("cf_pack_conv_weight_planes", w.data_ptr(), out.data_ptr(), Cout, Cin, KH, KW, Cin_p,
              prescale, _stream())
    return out, prescale


def pack_conv_weight(w: torch.Tensor, Cin_p: Optional[int] = None):
    """w[Cout,Cin,KH,KW] -> [Cout,KH,KW,Cin_p] fp16 (zero padded)."""
    w = w.detach().float().contiguous()
    _need(w, "w", torch.float32)
    Cout, Cin, KH, KW = w.shape
    Cin_p = pad16(Cin) if Cin_p is None else int(Cin_p)
    out = torch.empty((Cout, KH, KW, Cin_p), dtype=torch.float16, device=w.device)
    _lib.call("cf_pack_conv_weight", w.data_ptr(), out.data_ptr(), Cout, Cin, KH, KW, Cin_p, _stream())
    return out


# ---------------------------------------------------------------------------
# fused conv / linear on tcgen05
# ---------------------------------------------------------------------------

def conv_geometry(T, B, Ho, Wo, Cout, Cin_p=64, stride=1, sparse=False, planes=False):
    """Tile geometry cf_conv_bn_lif uses for this output shape and input width
    (the per-tile mask buffer of the sparse path has n_mtiles entries)."""
    import ctypes
    buf = (ctypes.c_int32 * 6)()
    flags = (1 if sparse else 0) | (2 if planes else 0)
    _lib.call("cf_conv_geometry_ex", T, B, Ho, Wo, Cout, Cin_p, stride, flags, buf)
    return dict(TP=buf[0], Wb=buf[1], Hb=buf[2], Bb=buf[3], n_mtiles=buf[4], BN=buf[5])


def conv_chunk(Cin_p: int, sparse: bool) -> int:
    rc = _lib.load().cf_conv_chunk(int(Cin_p), int(bool(sparse)))
    if rc < 0:
        _lib.check(rc, "cf_conv_chunk")
    return rc


def conv_bn_lif(x: torch.Tensor, wp: torch.Tensor, scale: Optional[torch.Tensor],
                shift: Optional[torch.Tensor], stride: int = 1, pad: int = 1,
                identity: Optional[torch.Tensor] = None, res_mode=None,
                v_in: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None,
                tile_mask: Optional[torch.Tensor] = None, lif: LIFConfig = _DEFAULT_LIF,
                out: Optional[torch.Tensor] = None, precision: str = "fp16",
                egd_max_active_frac: Optional[float] = None):
    """Fused conv+BN+LIF on x[B,H,W,T,Cin_p] fp16 with wp[Cout,KH,KW,Cin_p] fp16
    (precision "fp16"), split weights wp[Cout,KH,KW,2*Cin_p] from
    pack_conv_weight_split (precision "split") or digit planes
    wp[Cout,KH,KW,3*Cin_p] from pack_conv_weight_planes (precision "planes");
    for the last two the scale is already divided by the prescale.
    ``egd_max_active_frac`` (with ``tile_mask``): decide on the device whether
    the masks run (at most that fraction of (tile, chunk) pairs active) or
    the launch runs dense; the result is identical either way.

    Returns out[B,Ho,Wo,T,Cout] fp16.  v_out (if given) receives v_T in
    [B,Ho,Wo,Cout] fp32; v_in may alias v_out."""
    _need(x, "x", torch.float16)
    _need(wp, "wp", torch.float16)
    if precision not in PRECISIONS:
        raise ValueError(f"precision must be one of {PRECISIONS}")
    B, H, W, T, Cin_p = x.shape
    Cout, KH, KW, Cw = wp.shape
    if Cw != WEIGHT_PARTS[precision] * Cin_p:
        raise ValueError(f"weight channels {Cw} do not match activation Cin_p {Cin_p} "
                         f"at precision {precision!r}")
    Ho = (H + 2 * pad - KH) // stride + 1
    Wo = (W + 2 * pad - KW) // stride + 1
    mode = RES_MODES[res_mode] if not isinstance(res_mode, int) else res_mode
    for t, n in ((scale, "scale"), (shift, "shift")):
        if t is not None:
            _need(t, n, torch.float32)
    if identity is not None:
        _need(identity, "identity", torch.float16)
        if tuple(identity.shape) != (B, Ho, Wo, T, Cout):
            raise ValueError("identity must be [B,Ho,Wo,T,Cout] fp16")
    for t, n in ((v_in, "v_in"), (v_out, "v_out")):
        if t is not None:
            _need(t, n, torch.float32)
            if tuple(t.shape) != (B, Ho, Wo, Cout):
                raise ValueError(f"{n} must be [B,Ho,Wo,Cout] fp32")
    if tile_mask is not None:
        _need(tile_mask, "tile_mask", torch.int32)
    if out is None:
        out = torch.empty((B, Ho, Wo, T, Cout), dtype=torch.float16, device=x.device)
    else:
        _need(out, "out", torch.float16)
    if precision == "planes":
        if tile_mask is not None:
            raise ValueError("the integer-plane mode runs dense only (no tile mask)")
        _lib.call("cf_conv_bn_lif_planes", x.data_ptr(), wp.data_ptr(), _ptr(scale), _ptr(shift),
                  _ptr(identity), mode, _ptr(v_in), _ptr(v_out), out.data_ptr(),
                  T, B, H, W, Cin_p, Cout, KH, KW, stride, pad, *lif.args(), _stream())
        return out
    if egd_max_active_frac is not None:
        if tile_mask is None or precision != "fp16":
            raise ValueError("the device dispatch needs a tile mask and fp16 weights")
        _lib.call("cf_conv_bn_lif_egd", x.data_ptr(), wp.data_ptr(), _ptr(scale), _ptr(shift),
                  _ptr(identity), mode, _ptr(v_in), _ptr(v_out), out.data_ptr(),
                  _ptr(tile_mask), T, B, H, W, Cin_p, Cout, KH, KW, stride, pad, *lif.args(),
                  float(egd_max_active_frac), _stream())
        return out
    fn = "cf_conv_bn_lif_split" if precision == "split" else "cf_conv_bn_lif"
    _lib.call(fn, x.data_ptr(), wp.data_ptr(), _ptr(scale), _ptr(shift),
              _ptr(identity), mode, _ptr(v_in), _ptr(v_out), out.data_ptr(), _ptr(tile_mask),
              T, B, H, W, Cin_p, Cout, KH, KW, stride, pad, *lif.args(), _stream())
    return out


def linear_bn_lif(x: torch.Tensor, w: torch.Tensor, scale=None, shift=None, identity=None,
                  res_mode=None, v_in=None, v_out=None, lif: LIFConfig = _DEFAULT_LIF, out=None):
    """x[B,L,T,Cin_p] fp16, w[Cout,Cin_p] fp16 -> out[B,L,T,Cout] fp16."""
    _need(x, "x", torch.float16)
    _need(w, "w", torch.float16)
    B, L, T, Cin_p = x.shape
    Cout = w.shape[0]
    mode = RES_MODES[res_mode] if not isinstance(res_mode, int) else res_mode
    if out is None:
        out = torch.empty((B, L, T, Cout), dtype=torch.float16, device=x.device)
    _lib.call("cf_linear_bn_lif", x.data_ptr(), w.data_ptr(), _ptr(scale), _ptr(shift),
              _ptr(identity), mode, _ptr(v_in), _ptr(v_out), out.data_ptr(), T, B, L, Cin_p, Cout,
              *lif.args(), _stream())
    return out



def ssa_lif(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int,
            scale: Optional[float] = None, v_in=None, v_out=None, lif: LIFConfig = _DEFAULT_LIF,
            out=None):
    """Spiking self-attention + attention LIF on token spikes q, k, v [B,N,T,C] fp16
    (layout of linear_bn_lif) -> spikes [B,N,T,C] fp16; scale defaults to
    head_dim ** -0.5; v_in / v_out [B,N,C] fp32 carry the attention LIF state."""
    for t_, n_ in ((q, "q"), (k, "k"), (v, "v")):
        _need(t_, n_, torch.float16)
    B, N, T, C = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape")
    if scale is None:
        scale = (C // heads) ** -0.5
    if out is None:
        out = torch.empty_like(q)
    _lib.call("cf_ssa_lif", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
              _ptr(v_in), _ptr(v_out), T, B, N, C, heads, float(scale), *lif.args(), _stream())
    return out

# ---------------------------------------------------------------------------
# prescan
# ---------------------------------------------------------------------------

def prescan(x: torch.Tensor, k: int, stride: int, pad: int, BH: int, BW: int, GS: int,
            threshold: float = 1e-6, count_nnz: bool = True):
    """Reference-geometry prescan over x[N,C,H,W] -> (ag_mask int32, tile_class
    int32, nnz int64[1] or None)."""
    _need(x, "x")
    N, C, H, W = x.shape
    fmt = {torch.float32: FMT_F32, torch.float16: FMT_F16, torch.uint8: FMT_U8}[x.dtype]
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    GH, GW = -(-Ho // BH), -(-Wo // BW)
    ag = torch.empty(N * GH * GW, dtype=torch.int32, device=x.device)
    cls = torch.empty_like(ag)
    nnz = torch.zeros(1, dtype=torch.int64, device=x.device) if count_nnz else None
    _lib.call("cf_prescan", x.data_ptr(), fmt, ag.data_ptr(), cls.data_ptr(), _ptr(nnz), N, C, H,
              W, Ho, Wo, k, stride, pad, BH, BW, GS, float(threshold), _stream())
    return ag, cls, nnz


def prescan_conv_tiles(x: torch.Tensor, Cout: int, KH: int, KW: int, stride: int, pad: int,
                       mask_out: Optional[torch.Tensor] = None,
                       nnz_out: Optional[torch.Tensor] = None, egd: bool = False):
    """Conv-tile prescan over x[B,H,W,T,Cin_p] fp16 -> per-M-tile chunk mask
    (the chunk of masked launches, or with ``egd`` the dense chunk that the
    device-dispatch launches use)."""
    _need(x, "x", torch.float16)
    B, H, W, T, Cin_p = x.shape
    Ho = (H + 2 * pad - KH) // stride + 1
    Wo = (W + 2 * pad - KW) // stride + 1
    g = conv_geometry(T, B, Ho, Wo, Cout, Cin_p, stride, True)
    chunk = conv_chunk(Cin_p, not egd)
    if mask_out is None:
        mask_out = torch.empty(g["n_mtiles"], dtype=torch.int32, device=x.device)
    if nnz_out is not None:
        _need(nnz_out, "nnz_out", torch.int64)
    _lib.call("cf_prescan_conv_tiles", x.data_ptr(), mask_out.data_ptr(), _ptr(nnz_out), T, B, H, W,
              Cin_p, Cout, KH, KW, stride, pad, chunk, _stream())
    return mask_out


def maxpool_bhwtc(x: torch.Tensor, k: int, stride: int, pad: int,
                  out: Optional[torch.Tensor] = None):
    """Max pool over x[B,H,W,T,C] fp16 (k, stride, pad) -> [B,Ho,Wo,T,C]."""
    _need(x, "x", torch.float16)
    B, H, W, T, C = x.shape
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    if out is None:
        out = torch.empty((B, Ho, Wo, T, C), dtype=torch.float16, device=x.device)
    _lib.call("cf_maxpool_bhwtc", x.data_ptr(), out.data_ptr(), B, H, W, T, C, k, stride, pad,
              _stream())
    return out


def avgpool_fc(x: torch.Tensor, fc_w: torch.Tensor, fc_b: Optional[torch.Tensor],
               out: Optional[torch.Tensor] = None):
    """x[B,H,W,T,C] fp16 -> logits[T,B,K] fp32."""
    _need(x, "x", torch.float16)
    _need(fc_w, "fc_w", torch.float32)
    B, H, W, T, C = x.shape
    K = fc_w.shape[0]
    if out is None:
        out = torch.empty((T, B, K), dtype=torch.float32, device=x.device)
    _lib.call("cf_avgpool_fc", x.data_ptr(), fc_w.data_ptr(), _ptr(fc_b), out.data_ptr(), T, B, H,
              W, C, K, _stream())
    return out


# ---------------------------------------------------------------------------
# bounded device-side waits
# ---------------------------------------------------------------------------

def check_device_error(stream: Optional[int] = None) -> None:
    """Raise CatfuseNativeError(CF_ERR_DEVICE_TIMEOUT) if a bounded wait inside
    a fused conv launch expired since the last check (synchronises the stream;
    the error word is cleared by the read)."""
    import ctypes
    code = ctypes.c_int32(0)
    rc = _lib.load().cf_check_device_error(_stream() if stream is None else stream,
                                           ctypes.byref(code))
    _lib.check(rc, f"device-side wait expired (site {code.value})")


def set_wait_limit(max_polls: int = 0) -> None:
    """Bound on the polls of every device-side wait of later conv launches
    (0 restores the default of 2^24 polls)."""
    _lib.call("cf_set_wait_limit", int(max_polls))


def token_mean_lif_fc(x: torch.Tensor, fc_w: torch.Tensor, fc_b: Optional[torch.Tensor],
                      v_in: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None,
                      lif: LIFConfig = _DEFAULT_LIF, out: Optional[torch.Tensor] = None):
    """Spikformer head over tokens x[B,N,T,C] fp16: token mean -> LIF -> fc.
    -> logits[T,B,K] fp32; v_in / v_out [B,C] fp32 carry the LIF state."""
    _need(x, "x", torch.float16)
    _need(fc_w, "fc_w", torch.float32)
    B, N, T, C = x.shape
    K = fc_w.shape[0]
    if out is None:
        out = torch.empty((T, B, K), dtype=torch.float32, device=x.device)
    _lib.call("cf_token_mean_lif_fc", x.data_ptr(), _ptr(v_in), _ptr(v_out), fc_w.data_ptr(),
              _ptr(fc_b), out.data_ptr(), T, B, N, C, K, *lif.args(), _stream())
    return out


def conv_bn_lif_dual(x: torch.Tensor, wp: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                     Cout1: int, stride: int, pad: int, v_in=None, v_out=None, out=None,
                     v_in2=None, v_out2=None, out2=None, lif: LIFConfig = _DEFAULT_LIF):
    """Two convs over x[B,H,W,T,Cin_p] in one launch (cf_conv_bn_lif_dual):
    weight rows [0, Cout1) -> out, [Cout1, Cout) -> out2.  Returns (out, out2)."""
    _need(x, "x", torch.float16)
    _need(wp, "wp", torch.float16)
    B, H, W, T, Cin_p = x.shape
    Cout, KH, KW, Cw = wp.shape
    if Cw != Cin_p:
        raise ValueError("weight / activation channel mismatch")
    Ho = (H + 2 * pad - KH) // stride + 1
    Wo = (W + 2 * pad - KW) // stride + 1
    if out is None:
        out = torch.empty((B, Ho, Wo, T, Cout1), dtype=torch.float16, device=x.device)
    if out2 is None:
        out2 = torch.empty((B, Ho, Wo, T, Cout - Cout1), dtype=torch.float16, device=x.device)
    _lib.call("cf_conv_bn_lif_dual", x.data_ptr(), wp.data_ptr(), _ptr(scale), _ptr(shift),
              _ptr(v_in), _ptr(v_out), out.data_ptr(), _ptr(v_in2), _ptr(v_out2), out2.data_ptr(),
              int(Cout1), T, B, H, W, Cin_p, Cout, KH, KW, stride, pad, *lif.args(), _stream())
    return out, out2
