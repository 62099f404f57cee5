"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is available; these stand in for them).

* config 0: one Conv3x3->BN->LIF layer, T=4, B=32, 128->128, 32x32, input
  spikes Bernoulli(0.1), Kaiming-normal weights, eval-mode BN statistics
  mean~N(0,0.1), var~U(0.5,1.5), gamma~U(0.8,1.2), beta~N(0,0.1);
* config 2: block-structured spikes for the SparseFlow sweep: 8x8 spatial x
  32-channel blocks, each all-zero with probability s, else Bernoulli(0.3).

One ``torch.Generator`` per tensor, seeded 0, 1, 2, ... in the order listed.
"""
from __future__ import annotations

import math

import torch

CONFIG0 = dict(T=4, B=32, C=128, H=32, W=32, p=0.1)
CONFIG2 = dict(T=4, B=32, C=256, H=28, W=28, sparsities=(0.8, 0.9, 0.95, 0.99, 1.0))


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def bernoulli_spikes(shape, p: float, seed: int = 0) -> torch.Tensor:
    return (torch.rand(shape, generator=_gen(seed)) < p).float()


def kaiming_conv_weight(cout: int, cin: int, k: int, seed: int = 1) -> torch.Tensor:
    """Kaiming-normal (fan_in, gain sqrt(2)) conv weight [cout, cin, k, k]."""
    std = math.sqrt(2.0 / (cin * k * k))
    return torch.randn((cout, cin, k, k), generator=_gen(seed)) * std


def bn_stats(c: int, seed: int = 2):
    """(mean, var, gamma, beta) with the distributions of config 0."""
    mean = torch.randn(c, generator=_gen(seed)) * 0.1
    var = torch.rand(c, generator=_gen(seed + 1)) + 0.5
    gamma = torch.rand(c, generator=_gen(seed + 2)) * 0.4 + 0.8
    beta = torch.randn(c, generator=_gen(seed + 3)) * 0.1
    return mean, var, gamma, beta


def fold_bn(mean, var, gamma, beta, eps: float = 1e-5):
    """Eval-mode BN as an affine: scale = gamma / sqrt(var + eps),
    shift = beta - mean * scale (fp32)."""
    scale = (gamma.float() / torch.sqrt(var.float() + eps)).float()
    shift = (beta.float() - mean.float() * scale).float()
    return scale, shift


def config0(T=None, B=None, C=None, H=None, W=None):
    """-> (x[T,B,C,H,W] fp32 {0,1}, w[C,C,3,3], scale[C], shift[C])."""
    c = dict(CONFIG0)
    for k, v in (("T", T), ("B", B), ("C", C), ("H", H), ("W", W)):
        if v is not None:
            c[k] = v
    x = bernoulli_spikes((c["T"], c["B"], c["C"], c["H"], c["W"]), c["p"], seed=0)
    w = kaiming_conv_weight(c["C"], c["C"], 3, seed=1)
    scale, shift = fold_bn(*bn_stats(c["C"], seed=2))
    return x, w, scale, shift


def block_sparse_spikes(T, B, C, H, W, s: float, seed: int = 0, block_hw: int = 8,
                        block_c: int = 32, p_active: float = 0.3) -> torch.Tensor:
    """Config 2 input: blocks of block_hw x block_hw pixels x block_c channels,
    each all-zero with probability s, else Bernoulli(p_active) inside."""
    g = _gen(seed)
    nb = (T, B, -(-C // block_c), -(-H // block_hw), -(-W // block_hw))
    keep = (torch.rand(nb, generator=g) >= s).float()
    keep = (keep.repeat_interleave(block_c, 2).repeat_interleave(block_hw, 3)
            .repeat_interleave(block_hw, 4))[:, :, :C, :H, :W]
    return keep * (torch.rand((T, B, C, H, W), generator=g) < p_active).float()
