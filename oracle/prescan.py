"""Receptive-field prescan restatement (numpy, bit-exact integer output).

Semantics of the reference cascade ``_prescan_2d_impl``
(``catfuse/sparseflow/prescan.py:153-189``): per channel group the abs-max
(``:32-45``), a max-pool with the conv's (k, s, p) — i.e. the max over each
valid output pixel's receptive field —, a ceil-mode max-pool over each
BH x BW output tile, ``> threshold``, bit-packing of the groups (``:48-54``)
and the tile class 0 / 1 / 2 (``:57-109``).  Geometry helpers follow
``choose_group_size`` / ``_select_tile_sizes``
(``catfuse/sparseflow/sparse_conv2d_kernel.py:64-84``).
"""
from __future__ import annotations

import numpy as np


def choose_group_size(c_in: int) -> int:
    gs = 16 if c_in <= 128 else 32
    while -(-c_in // gs) > 32:
        gs *= 2
    return gs


def select_tile_sizes(h: int, w: int):
    return (8, 16) if h * w >= 3136 else (8, 8)


def prescan_rf(x, k, stride, pad, BH, BW, GS, threshold=1e-6):
    """x: [N, C, H, W] -> (ag_mask int32 [N*GH*GW], tile_class int32 [...],
    nnz int)."""
    x = np.asarray(x)
    N, C, H, W = x.shape
    G = -(-C // GS)
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    GH, GW = -(-Ho // BH), -(-Wo // BW)
    xp = np.zeros((N, G * GS, H, W), np.float32)
    xp[:, :C] = np.abs(x.astype(np.float32))
    gmax = xp.reshape(N, G, GS, H, W).max(axis=2)           # [N, G, H, W]
    # max over each output pixel's receptive field (padding ignored)
    rf = np.full((N, G, Ho, Wo), -np.inf, np.float32)
    for kh in range(k):
        for kw in range(k):
            for oh in range(Ho):
                ih = oh * stride - pad + kh
                if ih < 0 or ih >= H:
                    continue
                iws = np.arange(Wo) * stride - pad + kw
                ok = (iws >= 0) & (iws < W)
                if not ok.any():
                    continue
                rf[:, :, oh, ok] = np.maximum(rf[:, :, oh, ok], gmax[:, :, ih, iws[ok]])
    # ceil-mode tile max
    tile = np.full((N, G, GH, GW), -np.inf, np.float32)
    for gh in range(GH):
        for gw in range(GW):
            blk = rf[:, :, gh * BH:(gh + 1) * BH, gw * BW:(gw + 1) * BW]
            tile[:, :, gh, gw] = blk.reshape(N, G, -1).max(axis=2)
    active = tile > np.float32(threshold)                     # [N, G, GH, GW]
    active = active.transpose(0, 2, 3, 1).reshape(-1, G)
    weights = (np.uint64(1) << np.arange(G, dtype=np.uint64))
    mask = (active.astype(np.uint64) * weights).sum(axis=1).astype(np.uint64)
    ag = (mask & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.int32)
    all_mask = np.uint64((1 << G) - 1)
    cls = np.where(mask == 0, 0, np.where(mask == all_mask, 2, 1)).astype(np.int32)
    nnz = int(np.count_nonzero(x))
    return ag, cls, nnz
