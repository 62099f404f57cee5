"""Spiking ResNet model builders with SpikingJelly's module naming.

SEW-ResNet (spike-element-wise residual: ``out = g(identity, sn2(...))`` with
cnf ADD / AND / IAND, and an LIF after the downsample) and the standard
Spiking ResNet (residual added before the second LIF, no LIF on the
downsample).  Attribute names follow SJ / torchvision so that state dicts and
the CATFuse rewrite rules (``conv{i}/bn{i}/sn{i}``, ``downsample`` +
``downsample_sn``) apply unchanged.  ``build_sew_resnet18_cifar`` applies the
CIFAR stem adaptation the reference's experiments use (3x3/s1 stem, no
max-pool).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import functional, layer
from .neuron import LIFNode


def _sew_fn(x, y, cnf):
    if cnf == "ADD":
        return x + y
    if cnf == "AND":
        return x * y
    if cnf == "IAND":
        return x * (1.0 - y)
    raise NotImplementedError(cnf)


def conv3x3(cin, cout, stride=1):
    return layer.Conv2d(cin, cout, 3, stride, 1, bias=False)


def conv1x1(cin, cout, stride=1):
    return layer.Conv2d(cin, cout, 1, stride, 0, bias=False)


class _SEWBasicBlock(nn.Module):
    expansion = 1

    def __init__(self, inplanes, planes, stride=1, downsample=None, cnf="ADD", spiking_neuron=LIFNode,
                 **neuron_kw):
        super().__init__()
        self.conv1 = conv3x3(inplanes, planes, stride)
        self.bn1 = layer.BatchNorm2d(planes)
        self.sn1 = spiking_neuron(**neuron_kw)
        self.conv2 = conv3x3(planes, planes)
        self.bn2 = layer.BatchNorm2d(planes)
        self.sn2 = spiking_neuron(**neuron_kw)
        self.downsample = downsample
        if downsample is not None:
            self.downsample_sn = spiking_neuron(**neuron_kw)
        self.stride = stride
        self.cnf = cnf

    def forward(self, x):
        identity = x
        out = self.sn1(self.bn1(self.conv1(x)))
        out = self.sn2(self.bn2(self.conv2(out)))
        if self.downsample is not None:
            identity = self.downsample_sn(self.downsample(x))
        return _sew_fn(identity, out, self.cnf)


class _SpikingBasicBlock(nn.Module):
    expansion = 1

    def __init__(self, inplanes, planes, stride=1, downsample=None, spiking_neuron=LIFNode,
                 **neuron_kw):
        super().__init__()
        self.conv1 = conv3x3(inplanes, planes, stride)
        self.bn1 = layer.BatchNorm2d(planes)
        self.sn1 = spiking_neuron(**neuron_kw)
        self.conv2 = conv3x3(planes, planes)
        self.bn2 = layer.BatchNorm2d(planes)
        self.sn2 = spiking_neuron(**neuron_kw)
        self.downsample = downsample
        self.stride = stride

    def forward(self, x):
        identity = x
        out = self.sn1(self.bn1(self.conv1(x)))
        out = self.bn2(self.conv2(out))
        if self.downsample is not None:
            identity = self.downsample(x)
        out = out + identity
        return self.sn2(out)


# The CATFuse rewrite recognises blocks by class name ("BasicBlock") and the
# presence of `cnf` (SEW) — the names SpikingJelly uses.
class BasicBlock(_SEWBasicBlock):
    pass


class SpikingBasicBlock(_SpikingBasicBlock):
    pass


SpikingBasicBlock.__name__ = "BasicBlock"
SpikingBasicBlock.__qualname__ = "BasicBlock"


class _ResNet(nn.Module):
    def __init__(self, block, layers, num_classes=1000, sew=True, cnf="ADD",
                 spiking_neuron=LIFNode, **neuron_kw):
        super().__init__()
        self.inplanes = 64
        self._sew = sew
        self._cnf = cnf
        self._neuron = spiking_neuron
        self._neuron_kw = neuron_kw
        self.conv1 = layer.Conv2d(3, 64, 7, 2, 3, bias=False)
        self.bn1 = layer.BatchNorm2d(64)
        self.sn1 = spiking_neuron(**neuron_kw)
        self.maxpool = layer.MaxPool2d(3, 2, 1)
        self.layer1 = self._make_layer(block, 64, layers[0])
        self.layer2 = self._make_layer(block, 128, layers[1], 2)
        self.layer3 = self._make_layer(block, 256, layers[2], 2)
        self.layer4 = self._make_layer(block, 512, layers[3], 2)
        self.avgpool = layer.AdaptiveAvgPool2d((1, 1))
        self.fc = layer.Linear(512 * block.expansion, num_classes)
        for m in self.modules():
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            elif isinstance(m, nn.BatchNorm2d):
                nn.init.ones_(m.weight)
                nn.init.zeros_(m.bias)

    def _make_layer(self, block, planes, blocks, stride=1):
        downsample = None
        if stride != 1 or self.inplanes != planes * block.expansion:
            downsample = nn.Sequential(conv1x1(self.inplanes, planes * block.expansion, stride),
                                       layer.BatchNorm2d(planes * block.expansion))
        kw = dict(spiking_neuron=self._neuron, **self._neuron_kw)
        if self._sew:
            kw["cnf"] = self._cnf
        layers = [block(self.inplanes, planes, stride, downsample, **kw)]
        self.inplanes = planes * block.expansion
        for _ in range(1, blocks):
            layers.append(block(self.inplanes, planes, **kw))
        return nn.Sequential(*layers)

    def forward(self, x):
        x = self.sn1(self.bn1(self.conv1(x)))
        x = self.maxpool(x)
        x = self.layer4(self.layer3(self.layer2(self.layer1(x))))
        x = self.avgpool(x)
        step_mode = getattr(self.sn1, "step_mode", "s")
        x = torch.flatten(x, 2) if step_mode == "m" else torch.flatten(x, 1)
        return self.fc(x)


class SEWResNet(_ResNet):
    def __init__(self, block, layers, num_classes=1000, cnf="ADD", spiking_neuron=LIFNode, **kw):
        super().__init__(block, layers, num_classes, True, cnf, spiking_neuron, **kw)


class SpikingResNet(_ResNet):
    def __init__(self, block, layers, num_classes=1000, spiking_neuron=LIFNode, **kw):
        super().__init__(block, layers, num_classes, False, None, spiking_neuron, **kw)


def sew_resnet18(pretrained=False, num_classes=1000, cnf="ADD", spiking_neuron=LIFNode, **kw):
    kw.pop("surrogate_function", None)
    kw.pop("detach_reset", None)
    return SEWResNet(BasicBlock, [2, 2, 2, 2], num_classes, cnf, spiking_neuron, **kw)


def spiking_resnet18(pretrained=False, num_classes=1000, spiking_neuron=LIFNode, **kw):
    kw.pop("surrogate_function", None)
    kw.pop("detach_reset", None)
    return SpikingResNet(SpikingBasicBlock, [2, 2, 2, 2], num_classes, spiking_neuron, **kw)


def build_sew_resnet18_cifar(num_classes=10, tau=2.0, v_threshold=1.0):
    """SEW-ResNet-18 with the CIFAR stem (3x3/s1/p1, 64 ch, no max-pool), cnf
    ADD, LIF(tau, v_threshold), multi-step, eval mode."""
    net = sew_resnet18(num_classes=num_classes, cnf="ADD", spiking_neuron=LIFNode, tau=tau,
                       v_threshold=v_threshold)
    net.conv1 = layer.Conv2d(3, 64, 3, 1, 1, bias=False)
    net.maxpool = nn.Identity()
    functional.set_step_mode(net, "m")
    return net.eval()


def build_spiking_resnet18_imagenet(num_classes=1000, tau=2.0, v_threshold=1.0):
    net = spiking_resnet18(num_classes=num_classes, spiking_neuron=LIFNode, tau=tau,
                           v_threshold=v_threshold)
    functional.set_step_mode(net, "m")
    return net.eval()


def load_params(net: nn.Module, params: dict) -> nn.Module:
    """Load a {name: tensor} dict in SJ/torchvision naming (missing BN
    ``num_batches_tracked`` entries are fine)."""
    missing, unexpected = net.load_state_dict(params, strict=False)
    missing = [k for k in missing if not k.endswith("num_batches_tracked")]
    if missing or unexpected:
        raise KeyError(f"parameter mismatch: missing={missing[:5]} unexpected={unexpected[:5]}")
    return net


@torch.no_grad()
def init_random_(net: nn.Module, seed: int = 0) -> nn.Module:
    """Seeded random init for benchmarking without a checkpoint: Kaiming-normal
    conv weights (fan_in), BN eval statistics mean ~ N(0, 0.1),
    var ~ U(0.5, 1.5), gamma ~ U(0.8, 1.2), beta ~ N(0, 0.1) (the BN setting of
    the single-layer benchmark config), default Linear init."""
    g = torch.Generator().manual_seed(seed)
    for m in net.modules():
        if isinstance(m, nn.Conv2d):
            fan_in = m.in_channels * m.kernel_size[0] * m.kernel_size[1] // m.groups
            m.weight.copy_(torch.randn(m.weight.shape, generator=g) * (2.0 / fan_in) ** 0.5)
            if m.bias is not None:
                m.bias.zero_()
        elif isinstance(m, (nn.BatchNorm2d, nn.BatchNorm1d)):
            c = m.num_features
            m.weight.copy_(torch.rand(c, generator=g) * 0.4 + 0.8)
            m.bias.copy_(torch.randn(c, generator=g) * 0.1)
            m.running_mean.copy_(torch.randn(c, generator=g) * 0.1)
            m.running_var.copy_(torch.rand(c, generator=g) + 0.5)
        elif isinstance(m, nn.Linear):
            bound = 1.0 / m.in_features ** 0.5
            m.weight.copy_((torch.rand(m.weight.shape, generator=g) * 2 - 1) * bound)
            if m.bias is not None:
                m.bias.copy_((torch.rand(m.bias.shape, generator=g) * 2 - 1) * bound)
    return net


@torch.no_grad()
def calibrate_bn_(net: nn.Module, x_seq: torch.Tensor) -> nn.Module:
    """Set every BatchNorm's running statistics to the batch statistics of one
    forward over ``x_seq`` (what training would converge to), keeping its
    affine gamma/beta.  With random weights and random BN statistics the
    spiking activity of a deep SNN dies out after a few layers; calibrated
    statistics keep per-layer firing rates in the range of a trained network,
    so benchmarks exercise representative (dense) work."""
    bns = [m for m in net.modules() if isinstance(m, (nn.BatchNorm2d, nn.BatchNorm1d))]
    saved = [(m.momentum, m.training) for m in bns]
    for m in bns:
        m.momentum = 1.0
        m.train()
    functional.reset_net(net)
    net(x_seq)
    functional.reset_net(net)
    for m, (mom, tr) in zip(bns, saved):
        m.momentum = mom
        m.train(tr)
    return net
