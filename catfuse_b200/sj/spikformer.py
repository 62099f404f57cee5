"""Spikformer-style spiking transformer in the layout of the reference's
``models/spikformer_github.py`` (module and attribute names kept, so the
rewrite rules of ``substitute_sf`` and the native plan find the same
``X / X_bn / X_lif`` triples): SPS tokenizer (conv0..conv3 + BN + LIF,
max-pools after conv2 and conv3, relative position embedding conv with a
residual), ``depth`` encoder blocks (spiking self-attention + MLP, each with a
residual add of spike counts), token mean -> pre-head LIF -> linear head.

Every tensor is multi-step: images [T, B, C, H, W], tokens [T, B, N, C].
SpikingJelly itself is not installable here; LIF nodes are this package's
multi-step ``LIFNode`` (tau 2, v_th 1, hard reset to 0, decay_input).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .neuron import LIFNode


def _lif(v_threshold: float = 1.0) -> LIFNode:
    return LIFNode(tau=2.0, v_threshold=v_threshold, detach_reset=True, step_mode="m")


def _linear_bn(x, lin: nn.Linear, bn: nn.BatchNorm1d):
    """x[T, B, N, C] -> BN1d(Linear(x)) over the feature axis, [T, B, N, C']."""
    y = lin(x)
    T, B, N, C = y.shape
    y = bn(y.reshape(T * B * N, C))
    return y.reshape(T, B, N, C)


class MLP(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, v_threshold: float = 1.0):
        super().__init__()
        self.fc1, self.fc1_bn, self.fc1_lif = nn.Linear(dim, hidden_dim), nn.BatchNorm1d(hidden_dim), _lif(v_threshold)
        self.fc2, self.fc2_bn, self.fc2_lif = nn.Linear(hidden_dim, dim), nn.BatchNorm1d(dim), _lif(v_threshold)

    def forward(self, x):
        y = self.fc1_lif(_linear_bn(x, self.fc1, self.fc1_bn))
        return self.fc2_lif(_linear_bn(y, self.fc2, self.fc2_bn))


class SSA(nn.Module):
    def __init__(self, dim: int, num_heads: int, v_threshold: float = 1.0):
        super().__init__()
        if dim % num_heads:
            raise ValueError("dim must be a multiple of num_heads")
        self.dim, self.num_heads = dim, num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        for n in ("q", "k", "v", "proj"):
            setattr(self, n, nn.Linear(dim, dim))
            setattr(self, n + "_bn", nn.BatchNorm1d(dim))
            setattr(self, n + "_lif", _lif(v_threshold))
        self.attn_lif = _lif(v_threshold)

    def forward(self, x):
        T, B, N, C = x.shape
        h, d = self.num_heads, self.head_dim
        q, k, v = (getattr(self, n + "_lif")(_linear_bn(x, getattr(self, n), getattr(self, n + "_bn")))
                   for n in ("q", "k", "v"))
        split = lambda t: t.reshape(T, B, N, h, d).permute(0, 1, 3, 2, 4)   # [T, B, h, N, d]
        attn = split(q) @ split(k).transpose(-2, -1) * self.scale
        y = (attn @ split(v)).transpose(2, 3).reshape(T, B, N, C)
        y = self.attn_lif(y)
        return self.proj_lif(_linear_bn(y, self.proj, self.proj_bn))


class Block(nn.Module):
    def __init__(self, dim: int, num_heads: int, mlp_ratio: float = 4.0, v_threshold: float = 1.0):
        super().__init__()
        self.attn = SSA(dim, num_heads, v_threshold)
        self.mlp = MLP(dim, int(dim * mlp_ratio), v_threshold)

    def forward(self, x):
        x = x + self.attn(x)
        return x + self.mlp(x)


class SPS(nn.Module):
    def __init__(self, in_channels: int, embed_dim: int, v_threshold: float = 1.0):
        super().__init__()
        widths = (embed_dim // 8, embed_dim // 4, embed_dim // 2, embed_dim)
        cin = in_channels
        for i, c in enumerate(widths):
            setattr(self, f"conv{i}", nn.Conv2d(cin, c, 3, 1, 1, bias=False))
            setattr(self, f"bn{i}", nn.BatchNorm2d(c))
            setattr(self, f"lif{i}", _lif(v_threshold))
            cin = c
        self.pool2 = nn.MaxPool2d(3, 2, 1)
        self.pool3 = nn.MaxPool2d(3, 2, 1)
        self.rpe_conv = nn.Conv2d(embed_dim, embed_dim, 3, 1, 1, bias=False)
        self.rpe_bn = nn.BatchNorm2d(embed_dim)
        self.rpe_lif = _lif(v_threshold)

    @staticmethod
    def _fold(fn, x):
        T, B = x.shape[:2]
        y = fn(x.flatten(0, 1))
        return y.reshape(T, B, *y.shape[1:])

    def _cbl(self, i, x):
        conv, bn, lif = getattr(self, f"conv{i}"), getattr(self, f"bn{i}"), getattr(self, f"lif{i}")
        return lif(self._fold(lambda t: bn(conv(t)), x))

    def forward(self, x):
        y = self._cbl(0, x)
        y = self._cbl(1, y)
        y = self._fold(self.pool2, self._cbl(2, y))
        feat = self._fold(self.pool3, self._cbl(3, y))
        y = self.rpe_lif(self._fold(lambda t: self.rpe_bn(self.rpe_conv(t)), feat)) + feat
        return y.flatten(-2).transpose(-1, -2)          # [T, B, N, C]


class Spikformer(nn.Module):
    def __init__(self, img_size: int = 32, in_channels: int = 3, num_classes: int = 10,
                 embed_dim: int = 384, num_heads: int = 12, mlp_ratio: float = 4.0,
                 depth: int = 4, T: int = 4, v_threshold: float = 1.0):
        super().__init__()
        self.T = T
        self.img_size = img_size
        self.num_classes = num_classes
        self.patch_embed = SPS(in_channels, embed_dim, v_threshold)
        self.blocks = nn.ModuleList([Block(embed_dim, num_heads, mlp_ratio, v_threshold)
                                     for _ in range(depth)])
        self.pre_head_lif = _lif(v_threshold)
        self.head = nn.Linear(embed_dim, num_classes)

    def forward(self, x):
        if x.dim() == 4:
            x = x.unsqueeze(0).repeat(self.T, 1, 1, 1, 1)
        y = self.patch_embed(x)
        for blk in self.blocks:
            y = blk(y)
        return self.head(self.pre_head_lif(y.mean(dim=2)))


def build_spikformer_cifar(embed_dim: int = 384, num_heads: int = 12, mlp_ratio: float = 4.0,
                           depth: int = 4, num_classes: int = 10, T: int = 4) -> Spikformer:
    """The benchmark configuration: embed 384, 12 heads, MLP ratio 4, 4 blocks,
    32x32 images -> 8x8 = 64 tokens."""
    return Spikformer(32, 3, num_classes, embed_dim, num_heads, mlp_ratio, depth, T)


__all__ = ["Spikformer", "SPS", "SSA", "MLP", "Block", "build_spikformer_cifar"]
