"""SEW-ResNet-18 and Spiking-ResNet-18 multi-step forward on the CPU (fp32).

Topologies as described by the reference: the CIFAR-shape SEW-ResNet-18
(``experiments/_helpers.py:69-111``: 3x3/s1 stem with 64 channels, no
max-pool, four stages 64/128/256/512 of two BasicBlocks, cnf ADD), the SEW
BasicBlock (``catfuse/patterns.py:676-715``: out = sn2(bn2(conv2(sn1(bn1(
conv1(x)))))); identity = x or downsample_sn(downsample(x)); out = identity
+ out) and the standard Spiking BasicBlock (``catfuse/patterns.py:748-754``:
add before the second LIF, no LIF on the downsample).  The classifier is
avgpool -> flatten(2) -> fc over [T, B, ...].  BN uses eval-mode
``F.batch_norm``; LIF is SpikingJelly's multi-step LIFNode (tau=2,
v_th=1, v_reset=0, decay_input, hard reset) starting from v=0.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

STAGES = (64, 128, 256, 512)


def _lif(z, tau=2.0, vth=1.0, vr=0.0):
    v = torch.zeros_like(z[0])
    out = torch.empty_like(z)
    for t in range(z.shape[0]):
        v = v + (z[t] - (v - vr)) / tau
        s = v >= vth
        out[t] = s.to(z.dtype)
        v = torch.where(s, torch.full_like(v, vr), v)
    return out, v


def _conv_bn(x, p, conv, bn, stride, pad):
    T, B = x.shape[:2]
    z = F.conv2d(x.reshape(T * B, *x.shape[2:]), p[conv + ".weight"], None, stride, pad)
    z = F.batch_norm(z, p[bn + ".running_mean"], p[bn + ".running_var"], p[bn + ".weight"],
                     p[bn + ".bias"], False, 0.0, 1e-5)
    return z.reshape(T, B, *z.shape[1:])


def make_resnet18_params(num_classes=10, stem="cifar", seed=0, in_ch=3):
    """Seeded random weights in SpikingJelly/torchvision naming.

    Conv weights: Kaiming-normal (fan_in, gain sqrt(2)); BN eval stats:
    mean ~ N(0, 0.1), var ~ U(0.5, 1.5), gamma ~ U(0.8, 1.2), beta ~ N(0, 0.1);
    fc: U(-1/sqrt(512), 1/sqrt(512)).  One generator, fixed draw order."""
    g = torch.Generator().manual_seed(seed)
    p = {}

    def conv(name, cout, cin, k):
        p[name + ".weight"] = torch.randn(cout, cin, k, k, generator=g) * math.sqrt(2.0 / (cin * k * k))

    def bn(name, c):
        p[name + ".weight"] = torch.rand(c, generator=g) * 0.4 + 0.8
        p[name + ".bias"] = torch.randn(c, generator=g) * 0.1
        p[name + ".running_mean"] = torch.randn(c, generator=g) * 0.1
        p[name + ".running_var"] = torch.rand(c, generator=g) + 0.5

    if stem == "cifar":
        conv("conv1", 64, in_ch, 3)
    else:
        conv("conv1", 64, in_ch, 7)
    bn("bn1", 64)
    cin = 64
    for si, c in enumerate(STAGES):
        for bi in range(2):
            pre = f"layer{si + 1}.{bi}"
            stride = 2 if (bi == 0 and si > 0) else 1
            conv(pre + ".conv1", c, cin, 3); bn(pre + ".bn1", c)
            conv(pre + ".conv2", c, c, 3); bn(pre + ".bn2", c)
            if stride != 1 or cin != c:
                conv(pre + ".downsample.0", c, cin, 1); bn(pre + ".downsample.1", c)
            cin = c
    bound = 1.0 / math.sqrt(512)
    p["fc.weight"] = (torch.rand(num_classes, 512, generator=g) * 2 - 1) * bound
    p["fc.bias"] = (torch.rand(num_classes, generator=g) * 2 - 1) * bound
    return p


def _resnet18_forward(x, p, sew, stem, record=None, branch_dtype=None, dtype=torch.float32):
    x = torch.as_tensor(x).to(dtype)
    p = {k: (v.to(dtype) if torch.is_floating_point(v) else v) for k, v in p.items()}
    if stem == "cifar":
        z = _conv_bn(x, p, "conv1", "bn1", 1, 1)
    else:
        z = _conv_bn(x, p, "conv1", "bn1", 2, 3)
    s, v = _lif(z)
    if record is not None:
        record.append(("sn1", s, v))
    if stem != "cifar":
        T, B = s.shape[:2]
        s = F.max_pool2d(s.reshape(T * B, *s.shape[2:]), 3, 2, 1).reshape(T, B, 64, *(
            (d + 2 - 3) // 2 + 1 for d in s.shape[3:]))
    out = s
    cin = 64
    for si, c in enumerate(STAGES):
        for bi in range(2):
            pre = f"layer{si + 1}.{bi}"
            stride = 2 if (bi == 0 and si > 0) else 1
            xin = out
            s1, v1 = _lif(_conv_bn(xin, p, pre + ".conv1", pre + ".bn1", stride, 1))
            if record is not None:
                record.append((pre + ".sn1", s1, v1))
            z2 = _conv_bn(s1, p, pre + ".conv2", pre + ".bn2", 1, 1)
            has_ds = (pre + ".downsample.0.weight") in p
            if sew:
                s2, v2 = _lif(z2)
                if record is not None:
                    record.append((pre + ".sn2", s2, v2))
                if has_ds:
                    sd, vd = _lif(_conv_bn(xin, p, pre + ".downsample.0", pre + ".downsample.1", stride, 0))
                    if record is not None:
                        record.append((pre + ".downsample_sn", sd, vd))
                    ident = sd
                else:
                    ident = xin
                out = ident + s2
            else:
                ident = (_conv_bn(xin, p, pre + ".downsample.0", pre + ".downsample.1", stride, 0)
                         if has_ds else xin)
                if has_ds and branch_dtype is not None:   # storage precision of the branch
                    ident = ident.to(branch_dtype).to(z2.dtype)
                s2, v2 = _lif(z2 + ident)
                if record is not None:
                    record.append((pre + ".sn2", s2, v2))
                out = s2
            cin = c
    T, B = out.shape[:2]
    pooled = out.mean(dim=(3, 4))                     # [T, B, 512]
    return F.linear(pooled, p["fc.weight"], p["fc.bias"])  # [T, B, K]


def sew_resnet18_forward(x, p, stem="cifar", record=None, dtype=torch.float32):
    """x: [T, B, 3, H, W] -> logits [T, B, K].  ``dtype`` float64 gives the
    high-precision reference against which fp32 paths are measured."""
    return _resnet18_forward(x, p, True, stem, record, None, dtype)


def spiking_resnet18_forward(x, p, stem="imagenet", record=None, branch_dtype=None,
                             dtype=torch.float32):
    """``branch_dtype`` rounds the Conv-BN downsample branch to that type before
    the residual add (to mirror a kernel that stores the branch in fp16);
    ``dtype`` float64 gives the high-precision reference."""
    return _resnet18_forward(x, p, False, stem, record, branch_dtype, dtype)
