"""Spikformer forward on the CPU (test infrastructure: the checker of the
native Spikformer plan, never the product path).

Restates ``SpikformerGithub.forward`` of the reference
(``models/spikformer_github.py``): SPS tokenizer (``:181-254``: conv0..conv3
-> BN -> LIF with max-pools after conv2 and conv3, rpe conv -> BN -> LIF plus
the pooled features), encoder blocks (``:162-178``: x + SSA(x), then x +
MLP(x)), SSA (``:138-158``: q/k/v = Linear -> BN1d -> LIF, attn_lif on
(q k^T * scale) v per head, proj = Linear -> BN1d -> LIF), MLP (``:76-90``),
token mean -> pre_head_lif -> head (``:311-329``).  BN is eval-mode; LIF is
SpikingJelly's multi-step LIFNode (tau 2, v_th 1, hard reset 0, decay_input)
from v = 0.  ``dtype`` float64 gives the high-precision reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .nets import _lif


def _bn(z, p, name, channel_dim):
    shape = [1] * z.dim()
    shape[channel_dim] = -1
    inv = 1.0 / torch.sqrt(p[name + ".running_var"] + 1e-5)
    return ((z - p[name + ".running_mean"].view(shape)) * inv.view(shape) * p[name + ".weight"].view(shape)
            + p[name + ".bias"].view(shape))


def _conv_bn_lif(x, p, conv, bn, record=None, tag=None):
    T, B = x.shape[:2]
    z = F.conv2d(x.reshape(T * B, *x.shape[2:]), p[conv + ".weight"], None, 1, 1)
    z = _bn(z, p, bn, 1).reshape(T, B, *z.shape[1:])
    s, v = _lif(z)
    if record is not None:
        record.append((tag, s, v))
    return s


def _linear_bn_lif(x, p, name, record=None, tag=None):
    z = F.linear(x, p[name + ".weight"], p[name + ".bias"])
    s, v = _lif(_bn(z, p, name + "_bn", -1))
    if record is not None:
        record.append((tag or name, s, v))
    return s


def _pool(x):
    T, B = x.shape[:2]
    y = F.max_pool2d(x.reshape(T * B, *x.shape[2:]), 3, 2, 1)
    return y.reshape(T, B, *y.shape[1:])


def spikformer_forward(x, p, num_heads, depth, record=None, dtype=torch.float32):
    """x: [T, B, 3, H, W] -> logits [T, B, K]; ``record`` collects
    (name, spikes, v_T) of every LIF layer in forward order."""
    x = torch.as_tensor(x).to(dtype)
    p = {k: (v.to(dtype) if torch.is_floating_point(v) else v) for k, v in p.items()}
    pe = "patch_embed."
    y = _conv_bn_lif(x, p, pe + "conv0", pe + "bn0", record, pe + "lif0")
    y = _conv_bn_lif(y, p, pe + "conv1", pe + "bn1", record, pe + "lif1")
    y = _pool(_conv_bn_lif(y, p, pe + "conv2", pe + "bn2", record, pe + "lif2"))
    feat = _pool(_conv_bn_lif(y, p, pe + "conv3", pe + "bn3", record, pe + "lif3"))
    y = _conv_bn_lif(feat, p, pe + "rpe_conv", pe + "rpe_bn", record, pe + "rpe_lif") + feat
    T, B, C = y.shape[:3]
    x = y.flatten(-2).transpose(-1, -2)           # [T, B, N, C]
    N = x.shape[2]
    h = num_heads
    d = C // h
    for i in range(depth):
        a = f"blocks.{i}.attn."
        q, k, v = (_linear_bn_lif(x, p, a + n, record) for n in ("q", "k", "v"))
        split = lambda t: t.reshape(T, B, N, h, d).permute(0, 1, 3, 2, 4)
        att = (split(q) @ split(k).transpose(-2, -1)) * (d ** -0.5)
        z = (att @ split(v)).transpose(2, 3).reshape(T, B, N, C)
        s, vv = _lif(z)
        if record is not None:
            record.append((a + "attn_lif", s, vv))
        x = x + _linear_bn_lif(s, p, a + "proj", record)
        m = f"blocks.{i}.mlp."
        hdn = _linear_bn_lif(x, p, m + "fc1", record)
        x = x + _linear_bn_lif(hdn, p, m + "fc2", record)
    s, vv = _lif(x.mean(dim=2))
    if record is not None:
        record.append(("pre_head_lif", s, vv))
    return F.linear(s, p["head.weight"], p["head.bias"])
