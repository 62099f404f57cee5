"""Shared driver of the fused sm_100a Conv->BN->LIF kernel for the
Implementation classes (DenseKeep, SparseFlow).

Boundary work per call: pack x[T,B,C,H,W] into the kernel layout
[B,H,W,T,Cin_p] fp16 (exact for spikes), run the kernel, unpack the spikes to
the reference layout fp32 and keep v_T in the StateBuffer (in the kernel
layout; converted lazily if someone reads it).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from .base import ConvLIFParams, ConvLIFSpec, folded_affine

KERNEL_TIME_BLOCK = 8   # time steps per kernel launch (TMEM tile = 16 px x 8 steps)


class _WeightCache:
    """Packed fp16 weight + folded affine, keyed on tensor identity and version."""

    def __init__(self):
        self.key = None
        self.wp = None
        self.scale = None
        self.shift = None

    def reset(self):
        self.key = None
        self.wp = self.scale = self.shift = None

    def get(self, spec: ConvLIFSpec, params: ConvLIFParams, device, precision: str = "fp16"):
        """-> (packed weight, epilogue scale, epilogue shift) for ``precision``
        ("fp16": wp[Cout,KH,KW,Cin_p]; "split": hi | lo weights, "planes":
        integer digit planes, each with the scale divided by the power-of-two
        prescale of the packing)."""
        def tag(t):
            return None if t is None else (id(t), t.data_ptr(), t._version, t.device)
        key = (tag(params.weight), tag(params.bias), tag(params.bn_scale), tag(params.bn_bias),
               device, precision)
        if key != self.key:
            w = params.weight.detach().to(device)
            scale, shift = folded_affine(spec, params)
            self.shift = None if shift is None else shift.to(device)
            if precision in ("split", "planes"):
                pack = (ops.pack_conv_weight_split if precision == "split"
                        else ops.pack_conv_weight_planes)
                self.wp, pre = pack(w, ops.pad16(spec.in_channels))
                base = (torch.ones(spec.out_channels, dtype=torch.float32, device=device)
                        if scale is None else scale.to(device).float())
                self.scale = (base / pre).contiguous()
            else:
                self.wp = ops.pack_conv_weight(w, ops.pad16(spec.in_channels))
                self.scale = None if scale is None else scale.to(device)
            self.key = key
        return self.wp, self.scale, self.shift


def check_input(x: torch.Tensor, spec: ConvLIFSpec):
    if x.dim() != 5:
        raise ValueError(f"expected x[T, B, C, H, W], got {tuple(x.shape)}")
    if x.shape[2] != spec.in_channels:
        raise ValueError(f"expected {spec.in_channels} input channels, got {x.shape[2]}")
    if not x.is_cuda:
        raise RuntimeError("the fused Conv-BN-LIF path runs on an sm_100 GPU only (CPU tensor given)")


def fused_forward(x: torch.Tensor, spec: ConvLIFSpec, params: ConvLIFParams, state,
                  cache: _WeightCache, sparse: bool, out_dtype=torch.float32,
                  stats: Optional[dict] = None, precision: str = "fp16",
                  egd_max_active_frac: Optional[float] = None) -> torch.Tensor:
    """``sparse``: prescan + masked conv; with ``egd_max_active_frac`` the
    kernel decides on the device whether the masks run (EGD)."""
    check_input(x, spec)
    T, B, Cin, H, W = x.shape
    Ho, Wo = spec.output_hw(H, W)
    Cout = spec.out_channels
    dev = x.device
    wp, scale, shift = cache.get(spec, params, dev, precision)
    xp = ops.pack_tbchw(x.contiguous(), ops.pad16(spec.in_channels))
    v_in = state.get_native((B, Cout, Ho, Wo), dev)
    v_out = torch.empty((B, Ho, Wo, Cout), dtype=torch.float32, device=dev)
    mask = None
    if sparse:
        nnz = torch.zeros(1, dtype=torch.int64, device=dev) if stats is not None else None
        mask = ops.prescan_conv_tiles(xp, Cout, spec.kernel_size, spec.kernel_size, spec.stride,
                                      spec.padding, nnz_out=nnz,
                                      egd=egd_max_active_frac is not None)
        if stats is not None:
            stats["nnz"] = nnz
            stats["tile_mask"] = mask
    out = ops.conv_bn_lif(xp, wp, scale, shift, spec.stride, spec.padding, v_in=v_in,
                          v_out=v_out, tile_mask=mask, lif=spec.lif_config(), precision=precision,
                          egd_max_active_frac=egd_max_active_frac if sparse else None)
    state.set_native(v_out)
    return ops.unpack_bhwtc(out, dtype=out_dtype)


def fused_io_cost(spec: ConvLIFSpec, T, B, H_in, W_in, dtype_bytes, schedule):
    from .base import IOCost
    Ho, Wo = spec.output_hw(H_in, W_in)
    kk = spec.kernel_size * spec.kernel_size
    nblocks = -(-T // KERNEL_TIME_BLOCK)
    return IOCost(
        x_load=T * B * H_in * W_in * spec.in_channels * dtype_bytes,
        w_load=spec.out_channels * spec.in_channels * kk * 2,
        z_io=0,
        v_io=2 * nblocks * B * Ho * Wo * spec.out_channels * 4,
        spike_write=T * B * Ho * Wo * spec.out_channels * dtype_bytes,
        schedule=schedule, num_blocks=nblocks)
