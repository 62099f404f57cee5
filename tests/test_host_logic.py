"""Host-side logic of the drop-in API (CPU only): policy, hardware profile,
StateBuffer, schedule algebra, I/O cost model, the SJ-compatible modules, the
graph rewrite and the no-CPU-fallback guarantee."""
import pytest
import torch
import torch.nn as nn

import oracle
from catfuse_b200 import hardware, policy
from catfuse_b200.implementations import (ConvLIFSpec, DenseKeep, ScheduleDecomposition,
                                          ScheduleTransform, SparseFlow)
from catfuse_b200.sj import functional, layer, neuron, zoo
from catfuse_b200.state import StateBuffer


def test_policy_table_and_formulas():
    assert policy.io_ratio_partial_fusion(4) == pytest.approx((3 + 0.5) / 7)
    assert policy.io_ratio_full_fusion(8) == pytest.approx((1 + 0.25) / 5)
    v100 = hardware.V100_PCIE_32GB
    # the reference thresholds under the V100 profile
    assert policy.classify_shape_regime(256, 256, 8, 8, 3, v100) == "memory_bound"
    assert policy.classify_shape_regime(64, 64, 32, 32, 3, v100) == "compute_bound"
    assert policy.classify_shape_regime(512, 512, 56, 56, 3, v100) == "compute_bound"
    assert policy.classify_shape_regime(64, 64, 32, 32, 1, v100) == "memory_bound"
    r = policy.get_policy("Conv3x3_BN_LIF", 256, 256, 8, 8, 3, T=4, hwprof=v100)
    assert r.spatial_backend == policy.SpatialBackend.SPARSE_FLOW and r.K == 8
    # B200 calibration: the shape stays memory-bound but routes to DenseKeep
    b200 = hardware.B200
    r = policy.get_policy("Conv3x3_BN_LIF", 256, 256, 8, 8, 3, T=4, hwprof=b200)
    assert r.spatial_backend == policy.SpatialBackend.DENSE_KEEP and r.K == 8
    assert 0.0 < b200.egd_max_active_frac < 1.0
    r = policy.get_policy("Linear_LIF", T=6)
    assert r.K == 6 and r.spatial_backend == policy.SpatialBackend.DENSE_KEEP
    r = policy.get_policy("Unknown_Pattern", 64, 64, 8, 8, 3, T=2)
    assert r.K == 2
    assert policy.optimal_K(4) == 4 and policy.optimal_K(16, "compute_bound") == 8


def test_hardware_profiles():
    assert hardware._BY_SM[(10, 0)] is hardware.B200
    assert hardware.B200.sm_count == 148 and hardware.B200.sm_capability == 100
    prof = hardware.detect_hardware()
    assert isinstance(prof, hardware.HardwareProfile)


def test_state_buffer_semantics():
    sb = StateBuffer()
    assert not sb.is_initialized and sb.tensor is None
    v = sb.get((2, 3), "cpu")
    assert torch.equal(v, torch.zeros(2, 3))
    sb.set(torch.ones(2, 3, requires_grad=True))
    assert not sb.tensor.requires_grad
    assert torch.equal(sb.get((2, 3), "cpu"), torch.ones(2, 3))
    assert torch.equal(sb.get((4,), "cpu"), torch.zeros(4))  # shape change -> zeros
    sb.reset()
    assert not sb.is_initialized
    assert sb.get_native((1, 2, 3, 4), "cpu") is None       # fresh: kernels skip v0


def test_schedule_algebra_and_io_cost():
    spec = ConvLIFSpec(64, 64, 3, 1, 1, False, True, 2.0, 1.0, 0.0)
    for impl in (DenseKeep(), SparseFlow()):
        d = impl.schedule_decomposition(spec, T=4)
        ok, errs = d.verify()
        assert ok, errs
        c = impl.analytic_io_cost(spec, T=4, B=2, H_in=8, W_in=8)
        assert c.z_io == 0 and c.total > 0 and c.as_dict()["total"] == c.total
    bad = ScheduleDecomposition((ScheduleTransform.BatchFold("LIF"),
                                 ScheduleTransform.StreamFuse("Conv", "LIF")), "form_2")
    ok, errs = bad.verify()
    assert not ok and len(errs) == 3   # BatchFold(CSR), no TimeBlock, StreamFuse w/o StateCarry
    assert str(ScheduleDecomposition((ScheduleTransform.StateCarry("LIF"),
                                      ScheduleTransform.TimeBlock(4)), "form_2")) == \
        "TimeBlock(K=4) ∘ StateCarry(LIF)"
    assert spec.output_hw(32, 32) == (32, 32)


def test_sj_lif_node_matches_oracle():
    x = torch.randn(6, 2, 5, generator=torch.Generator().manual_seed(0)) * 1.5
    for vr, decay in ((0.0, True), (None, True), (0.0, False)):
        n = neuron.LIFNode(tau=2.5, v_reset=vr, decay_input=decay, step_mode="m")
        s = n(x)
        s_o, v_o = oracle.lif_multistep(x.numpy(), None, 2.5, 1.0, vr, hard_reset=vr is not None,
                                        decay_input=decay)
        assert (s.numpy() == s_o).all() and (n.v.numpy() == v_o).all()
        functional.reset_net(n)
        assert n.v == (0.0 if vr is None else vr)


def test_substitute_sew_resnet18_routing():
    from catfuse_b200.substitute import substitute, substitute_sf
    from catfuse_b200.patterns import PartialFusionConvBNLIF, STFusionConvBNLIF, CTFSEWBasicBlock
    net = zoo.init_random_(zoo.build_sew_resnet18_cifar())
    # the reference's thresholds (V100 profile): 6 memory-bound sites -> SparseFlow
    m, st = substitute_sf(net, T=4, hwprof=hardware.V100_PCIE_32GB)
    assert st["total_lif_nodes"] == 20 and st["fused_lif_nodes"] == 20
    assert st["coverage_pct"] == 100.0
    assert isinstance(m.conv1, PartialFusionConvBNLIF) and isinstance(m.bn1, nn.Identity)
    assert isinstance(m.layer4[1].conv2, STFusionConvBNLIF)
    assert st["patterns_matched"]["STFusionConvBNLIF"] == 6
    # the calibrated B200 profile keeps every site on DenseKeep ...
    mb, stb = substitute_sf(net, T=4, hwprof=hardware.B200)
    assert "STFusionConvBNLIF" not in stb["patterns_matched"]
    # ... unless SparseFlow is forced (then the native plan runs the device EGD)
    mf, stf = substitute_sf(net, T=4, force_sparse=True, hwprof=hardware.B200)
    assert stf["patterns_matched"]["STFusionConvBNLIF"] > 6
    assert isinstance(m.layer2[0].downsample[0], PartialFusionConvBNLIF)
    names = [r["name"] for r in st["routing"]]
    assert len(names) == len(set(names)) == 20
    m2, st2 = substitute(net)
    assert st2["patterns_matched"] == {"CTFSEWBasicBlock": 8} and st2["fused_lif_nodes"] == 19
    assert isinstance(m2.layer1[0], CTFSEWBasicBlock)
    # the input model is not modified
    assert isinstance(net.conv1, nn.Conv2d)


def test_substitute_spiking_resnet_keeps_add_before_lif():
    from catfuse_b200.substitute import substitute_sf
    from catfuse_b200.patterns import CTFSpikingBasicBlock
    net = zoo.init_random_(zoo.build_spiking_resnet18_imagenet(num_classes=10))
    m, st = substitute_sf(net, T=4)
    assert all(isinstance(b, CTFSpikingBasicBlock) for l in (m.layer1, m.layer2, m.layer3, m.layer4)
               for b in l)
    assert st["fused_lif_nodes"] == st["total_lif_nodes"] == 17


def test_substitute_sequential_and_linear_bn():
    from catfuse_b200.substitute import substitute, substitute_sf
    from catfuse_b200.patterns import FusedLinearLIF, PartialFusionConvBNLIF, PartialFusionConvLIF
    seq = nn.Sequential(layer.Conv2d(3, 32, 3, 1, 1), layer.BatchNorm2d(32), neuron.LIFNode(),
                        layer.Conv2d(32, 32, 3, 1, 1), neuron.LIFNode(),
                        nn.Flatten(2), layer.Linear(32, 32), layer.BatchNorm1d(32), neuron.LIFNode(),
                        layer.Linear(32, 10), neuron.LIFNode())
    m, st = substitute(nn.Sequential(seq))
    kinds = [type(c).__name__ for c in m[0]]
    assert kinds == ["PartialFusionConvBNLIF", "PartialFusionConvLIF", "Flatten", "FusedLinearLIF",
                     "FusedLinearLIF"]
    assert st["fused_lif_nodes"] == st["total_lif_nodes"] == 4
    fl = m[0][3]
    assert fl.bn_scale is not None  # BN1d folded, not dropped

    class Tok(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = layer.Linear(16, 32)
            self.fc1_bn = layer.BatchNorm1d(32)
            self.fc1_lif = neuron.LIFNode()
            self.proj = layer.Conv2d(8, 32, 3, 1, 1)
            self.proj_bn = layer.BatchNorm2d(32)
            self.proj_lif = neuron.LIFNode()
    m, st = substitute_sf(Tok(), T=4)
    assert isinstance(m.fc1, FusedLinearLIF) and isinstance(m.proj, PartialFusionConvBNLIF)
    assert st["fused_lif_nodes"] == 2


def test_no_cpu_fallback():
    from catfuse_b200 import optimize, ops
    from catfuse_b200.patterns import PartialFusionConvBNLIF
    from catfuse_b200._lib import CatfuseNativeError
    with pytest.raises((CatfuseNativeError, RuntimeError)):
        ops.pack_tbchw(torch.zeros(1, 1, 3, 4, 4))
    pat = PartialFusionConvBNLIF(16, 32, 3, 1, 1)
    with pytest.raises(RuntimeError):
        pat(torch.zeros(2, 1, 16, 8, 8))
    net = zoo.init_random_(zoo.build_sew_resnet18_cifar())
    model, stats = optimize(net, device=None, T=4)
    assert stats["native_plan"]
    with pytest.raises(RuntimeError):
        model(torch.zeros(4, 1, 3, 32, 32))


def test_shard_bounds():
    from catfuse_b200.distributed import shard_bounds
    for B, W in ((64, 8), (10, 3), (3, 4)):
        spans = [shard_bounds(B, r, W) for r in range(W)]
        assert spans[0][0] == 0 and spans[-1][1] == B
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [h - l for l, h in spans]
        assert max(sizes) - min(sizes) <= 1
