"""Eval-mode BatchNorm fold (reference: ``catfuse/patterns.py:321-324`` and
``catfuse/kernels/partial_fusion_conv_bn_lif_impl.py:185-204``):
scale = gamma * rsqrt(var + eps), shift = beta - mean * scale."""
from __future__ import annotations

import torch


def fold_bn(gamma, beta, mean, var, eps=1e-5):
    gamma, beta, mean, var = (torch.as_tensor(a, dtype=torch.float32) for a in (gamma, beta, mean, var))
    inv_std = torch.rsqrt(var + eps)
    scale = gamma * inv_std
    shift = beta - mean * scale
    return scale, shift
