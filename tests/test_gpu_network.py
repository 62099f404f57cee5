"""GPU tests of the rewritten networks and the module-level patterns, called
through the public API (optimize / patterns) and checked against the oracle."""
import numpy as np
import pytest
import torch

import oracle
from lif_parity import check_lif_parity, lif_trace

pytestmark = pytest.mark.gpu


def _sew_net(B=8, seed=0):
    from catfuse_b200.sj import zoo
    net = zoo.init_random_(zoo.build_sew_resnet18_cifar(), seed)
    g = torch.Generator().manual_seed(100 + seed)
    x = torch.randn(B, 3, 32, 32, generator=g).unsqueeze(0).repeat(4, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, x)
    return net.eval(), x


def _teacher_forced_layers(plan, dev):
    """Every fused conv layer of the plan checked against the oracle fed with
    the plan's own input activation (fp16 operands, fp32 accumulation)."""
    from catfuse_b200 import ops
    from catfuse_b200.network import ConvStep
    worst = 0.0
    for st in plan.steps:
        if not isinstance(st, ConvStep):
            continue
        spec = st.native.spec
        C = plan.shapes[st.src][-1]
        if getattr(st, "im2col", False):   # stem fed from the im2col-packed input
            x = plan.x_in.cpu().half().float()
        else:
            x = ops.unpack_bhwtc(plan.acts[st.src]).cpu()[:, :, :spec.in_channels]
        y = ops.unpack_bhwtc(plan.acts[st.dst]).cpu().numpy()
        w = st.native.params.weight.detach().float().cpu()
        scale = None if st.scale is None else st.scale.cpu()
        shift = None if st.shift is None else st.shift.cpu()
        z = oracle.conv.conv_z(x, w, scale, shift, spec.stride, spec.padding,
                               operand_dtype=torch.float16).numpy()
        if st.lif is None:
            assert np.abs(y - z).max() <= 2e-3 * max(1.0, np.abs(z).max()), st.name
            continue
        ident = None
        if st.identity is not None:
            ident = ops.unpack_bhwtc(plan.acts[st.identity]).cpu().numpy()
        zz = z + ident if (ident is not None and st.res_mode == "add_pre") else z
        s_o, v_o, h = lif_trace(zz.astype(np.float32))
        out_o = s_o
        if ident is not None and st.res_mode in ("ADD", "add"):
            out_o = ident + s_o
        v = ops.v_to_nchw(st.v).cpu().numpy()
        s_got = y - ident if (ident is not None and st.res_mode in ("ADD", "add")) else y
        rate = check_lif_parity(s_got, v, s_o, v_o, h, v_tol=1e-4, near_tol=1e-3,
                                max_flip_rate=1e-4, what=st.name)
        worst = max(worst, rate)
    return worst


def test_sew_resnet18_network_vs_oracle(dev):
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _sew_net()
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    model, stats = optimize(net, device=dev, T=4)
    assert stats["native_plan"] and stats["fused_lif_nodes"] == stats["total_lif_nodes"] == 20
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    plan = model.plan_for(x.to(dev))
    _teacher_forced_layers(plan, dev)
    # End to end against the oracle at the kernel's operand precision (fp16
    # weights and input, fp32 accumulation/BN/LIF): identical spikes, so the
    # logits agree to accumulation-order rounding.
    p16 = {k: (v.half().float() if k.endswith(".weight") and v.dim() == 4 else v)
           for k, v in params.items()}
    ref16 = oracle.sew_resnet18_forward(x.half().float(), p16)
    rel = (logits - ref16).abs().max() / ref16.abs().max()
    assert rel < 1e-3, f"logits rel err vs fp16-operand oracle {rel}"
    assert bool((logits.sum(0).argmax(-1) == ref16.sum(0).argmax(-1)).all())
    # Against the fp32 oracle the spiking dynamics amplify the 10-bit operand
    # rounding layer by layer (each layer alone stays within the per-layer
    # gates checked above); predictions still mostly agree.
    ref = oracle.sew_resnet18_forward(x, params)
    agree = (logits.sum(0).argmax(-1) == ref.sum(0).argmax(-1)).float().mean()
    assert agree >= 0.5, f"argmax agreement with the fp32 oracle {agree}"


def test_network_graph_eager_and_state_carry(dev):
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _sew_net(B=4, seed=1)
    m_graph, _ = optimize(net, device=dev, T=4)
    m_eager, _ = optimize(net, device=dev, T=4, use_graph=False)
    xd = x.to(dev)
    functional.reset_net(m_graph)
    functional.reset_net(m_eager)
    a = m_graph(xd)
    b = m_eager(xd)
    assert torch.equal(a, b)
    # StateCarry: a second call without reset continues the membrane; equal to
    # the last 4 steps of one T=8 call
    a2 = m_graph(xd)
    m8, _ = optimize(net, device=dev, T=8)
    functional.reset_net(m8)
    l8 = m8(torch.cat([xd, xd], 0))
    assert torch.equal(a2, l8[4:])
    assert torch.equal(a, l8[:4])
    # reset -> identical to the first call
    functional.reset_net(m_graph)
    assert torch.equal(m_graph(xd), a)


def test_spiking_resnet18_imagenet_small(dev):
    """Standard Spiking ResNet (add before LIF, 7x7/2 stem + max-pool) at a
    reduced 64x64 input."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional, zoo
    net = zoo.init_random_(zoo.build_spiking_resnet18_imagenet(num_classes=100), 3)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 3, 64, 64, generator=g).unsqueeze(0).repeat(4, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, x)
    net.eval()
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    model, stats = optimize(net, device=dev, T=4)
    assert stats["native_plan"]
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    p16 = {k: (v.half().float() if k.endswith(".weight") and v.dim() == 4 else v)
           for k, v in params.items()}
    # the z-only downsample branch is stored in fp16 before the residual add
    ref = oracle.spiking_resnet18_forward(x.half().float(), p16, branch_dtype=torch.float16)
    rel = (logits - ref).abs().max() / ref.abs().max()
    assert rel < 1e-3, f"logits rel err {rel}"


def test_patterns_module_level(dev):
    from catfuse_b200 import patterns
    from catfuse_b200.sj import layer, neuron
    import torch.nn as nn
    g = torch.Generator().manual_seed(9)
    conv = layer.Conv2d(32, 64, 3, 1, 1, bias=True)
    bn = layer.BatchNorm2d(64)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) * 0.15)
        conv.bias.copy_(torch.randn(64, generator=g) * 0.1)
        bn.running_mean.copy_(torch.randn(64, generator=g) * 0.1)
        bn.running_var.copy_(torch.rand(64, generator=g) + 0.5)
        bn.weight.copy_(torch.rand(64, generator=g) * 0.4 + 0.8)
        bn.bias.copy_(torch.randn(64, generator=g) * 0.1)
    bn.eval()
    lif = neuron.LIFNode(tau=2.0, step_mode="m")
    x = (torch.rand(4, 2, 32, 10, 10, generator=g) < 0.3).float()
    scale, shift = oracle.fold_bn(bn.weight.detach(), bn.bias.detach(), bn.running_mean, bn.running_var)
    shift_b = shift + conv.bias.detach() * scale
    for cls in (patterns.PartialFusionConvBNLIF, patterns.STFusionConvBNLIF):
        m = cls.from_sj_modules(conv, bn, lif).to(dev)
        s1 = m(x.to(dev)).cpu().numpy()
        s2 = m(x.to(dev)).cpu().numpy()   # v carried across calls
        v2 = m.state.tensor.cpu().numpy()
        s_o, v_o, z = oracle.conv_bn_lif(torch.cat([x, x]), conv.weight.detach(), scale, shift_b, 1, 1,
                                         operand_dtype=torch.float16, return_z=True)
        _, _, h = lif_trace(z)
        check_lif_parity(np.concatenate([s1, s2]), v2, s_o, v_o, h, what=cls.__name__)
        m.reset()
        assert np.array_equal(m(x.to(dev)).cpu().numpy(), s1)
    # STFusion: host-side EGD and device-side dispatch agree bit for bit
    st = patterns.STFusionConvBNLIF.from_sj_modules(conv, bn, lif).to(dev)
    xs = x.clone()
    xs[:, :, :, :5] = 0
    a = st(xs.to(dev))
    st.reset()
    st.egd = "host"
    b = st(xs.to(dev))
    assert torch.equal(a, b) and st.last_dispatch in ("SparseFlow", "DenseKeep")
    st.reset()
    z0 = st(torch.zeros_like(xs).to(dev))
    assert st.last_dispatch == "StaticZero"
    s_o, _ = oracle.lif_multistep(np.broadcast_to(shift_b.numpy()[None, None, :, None, None],
                                                  (4, 2, 64, 10, 10)).astype(np.float32))
    assert np.array_equal(z0.cpu().numpy(), s_o)


def test_linear_lif_and_bn_add_lif(dev):
    from catfuse_b200 import patterns
    from catfuse_b200.sj import layer, neuron
    g = torch.Generator().manual_seed(10)
    lin = layer.Linear(96, 64)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(64, 96, generator=g) * 0.2)
        lin.bias.copy_(torch.randn(64, generator=g) * 0.2)
    lif = neuron.LIFNode()
    x = torch.randn(4, 3, 5, 96, generator=g)    # [T, B, tokens, C]
    m = patterns.FusedLinearLIF.from_sj_modules(lin, lif).to(dev)
    s = m(x.to(dev)).cpu().numpy()
    z = (x.half().float() @ lin.weight.detach().half().float().T + lin.bias.detach()).numpy()
    s_o, v_o, h = lif_trace(z)
    check_lif_parity(s, None, s_o, None, h, near_tol=2e-3, what="linear_lif")
    # Conv-BN-Add-LIF (Spiking ResNet second half)
    conv = layer.Conv2d(32, 32, 3, 1, 1, bias=False)
    bn = layer.BatchNorm2d(32).eval()
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) * 0.2)
    pat = patterns.PartialFusionConvBNAddLIF.from_sj_modules(conv, bn, lif).to(dev)
    xs = (torch.rand(4, 2, 32, 8, 8, generator=g) < 0.3).float()
    ident = torch.randn(4, 2, 32, 8, 8, generator=g).half().float()
    out = pat(xs.to(dev), ident.to(dev)).cpu().numpy()
    scale, shift = oracle.fold_bn(bn.weight.detach(), bn.bias.detach(), bn.running_mean, bn.running_var)
    z = oracle.conv.conv_z(xs, conv.weight.detach(), scale, shift, 1, 1, operand_dtype=torch.float16).numpy()
    s_o, v_o, h = lif_trace((z + ident.numpy()).astype(np.float32))
    check_lif_parity(out, None, s_o, None, h, what="conv_bn_add_lif")


def _plan_layer_spikes(plan):
    """{oracle record name: spikes [T,B,C,H,W]} of every LIF layer of a SEW plan
    (the SEW ADD output minus its identity gives the LIF spikes)."""
    from catfuse_b200 import ops
    from catfuse_b200.network import ConvStep
    out = {}
    for st in plan.steps:
        if not isinstance(st, ConvStep) or st.lif is None:
            continue
        y = ops.unpack_bhwtc(plan.acts[st.dst]).cpu()
        if st.identity is not None and st.res_mode in ("ADD", "add"):
            y = y - ops.unpack_bhwtc(plan.acts[st.identity]).cpu()
        name = st.name
        if name == "stem":
            key = "sn1"
        elif name.endswith(".conv1"):
            key = name[:-len(".conv1")] + ".sn1"
        elif name.endswith(".conv2"):
            key = name[:-len(".conv2")] + ".sn2"
        else:
            key = name[:-len(".downsample")] + ".downsample_sn"
        out[key] = y.numpy()
    return out


def _teacher_forced_fp64(plan):
    """Every fused conv layer of an fp32-mode plan against an fp64 restatement
    of the layer (conv, folded BN, LIF all in float64) fed with the plan's own
    input activation: flips only where the fp64 membrane is within 1e-5 of the
    threshold, flip rate <= 1e-4, v within 1e-4."""
    from catfuse_b200 import ops
    from catfuse_b200.network import ConvStep
    worst = 0.0
    for st in plan.steps:
        if not isinstance(st, ConvStep) or st.lif is None:
            continue
        spec = st.native.spec
        if st.im2col:
            x = plan.x_in.cpu().double()
        else:
            x = ops.unpack_bhwtc(plan.acts[st.src]).cpu()[:, :, :spec.in_channels].double()
        _, scale, shift = st.native.packed(plan.device, "fp16")
        w = st.native.params.weight.detach().double().cpu()
        T, B = x.shape[:2]
        z = torch.nn.functional.conv2d(x.reshape(T * B, *x.shape[2:]), w, stride=spec.stride,
                                       padding=spec.padding)
        z = z.reshape(T, B, *z.shape[1:])
        if scale is not None:
            z = z * scale.cpu().double().view(1, 1, -1, 1, 1)
        if shift is not None:
            z = z + shift.cpu().double().view(1, 1, -1, 1, 1)
        y = ops.unpack_bhwtc(plan.acts[st.dst]).cpu().numpy()
        ident = None
        if st.identity is not None:
            ident = ops.unpack_bhwtc(plan.acts[st.identity]).cpu().numpy()
        if ident is not None and st.res_mode == "add_pre":
            z = z + torch.from_numpy(ident).double()
        z = z.numpy()
        v = np.zeros(z.shape[1:])
        s64 = np.zeros_like(z)
        h64 = np.zeros_like(z)
        for t in range(T):
            h = v + (z[t] - v) / 2.0
            s64[t] = h >= 1.0
            h64[t] = h
            v = np.where(h >= 1.0, 0.0, h)
        s_got = y - ident if (ident is not None and st.res_mode in ("ADD", "add")) else y
        vg = ops.v_to_nchw(st.v).cpu().numpy()
        rate = check_lif_parity(s_got, vg, s64, v, h64, v_tol=1e-4, near_tol=1e-5,
                                max_flip_rate=1e-4, what=f"fp32 mode, teacher-forced {st.name}")
        worst = max(worst, rate)
    return worst


@pytest.mark.parametrize("seed", [0, 1])
def test_sew_resnet18_fp32_precision_end_to_end(dev, seed):
    """Config 1 (B=64, T=4) in the fp32-faithful mode (exact integer weight
    planes for the spike layers, hi + lo stem).

    Per layer (teacher-forced, fp64 restatement): the fp32 tolerance -- flips
    only within 1e-5 of the threshold, rate <= 1e-4, v within 1e-4.

    End to end (no teacher forcing) against the fp64 oracle: the T-summed
    classifier argmax agrees on every sample (the reference's gate,
    experiments/exp_40_end_to_end_v2.py:102-166), every layer of stages 1-2
    flips <= 1e-4 of its spikes and every layer <= 1e-3.  A deep spiking
    network amplifies a single threshold coincidence layer by layer (an
    fp32 LIF step and an fp64 one disagree wherever h lands within an fp32
    ulp of v_th), so no fp32 computation stays within 1e-4 of fp64 in the
    last stages for every input: the fp32 CPU oracle itself drifts to
    ~6e-4 at layer 4 on seed 1, which this test prints beside ours."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _sew_net(B=64, seed=seed)
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    model, stats = optimize(net, device=dev, T=4, precision="fp32")
    assert stats["native_plan"]
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    plan = model.plan_for(x.to(dev))
    assert sum(st.prec == "planes" for st in plan.steps if hasattr(st, "prec")) == 19
    _teacher_forced_fp64(plan)
    r64, r32 = [], []
    ref64 = oracle.sew_resnet18_forward(x, params, record=r64, dtype=torch.float64)
    oracle.sew_resnet18_forward(x, params, record=r32)
    got = _plan_layer_spikes(plan)
    assert len(got) == len(r64) == 20
    rows = []
    for (name, s64, _), (_, s32, _) in zip(r64, r32):
        rows.append((name, float((got[name] != s64.numpy()).mean()),
                     float((s32.numpy() != s64.numpy()).mean())))
    for r in rows:
        print("  %-26s flips vs fp64: ours %.2e, fp32 CPU oracle %.2e" % r)
    for name, rate, _ in rows:
        stage = 0 if name == "sn1" else int(name[5])
        assert rate <= (1e-4 if stage <= 2 else 1e-3), f"{name}: flip rate vs fp64 {rate:.2e}"
    agree = (logits.sum(0).argmax(-1) == ref64.sum(0).argmax(-1)).float().mean()
    assert agree == 1.0, f"classifier agreement with fp64 {agree}"
    rel = (logits.double() - ref64).abs().max() / ref64.abs().max()
    print(f"fp32 mode seed {seed}: logits rel err vs fp64 {float(rel):.2e}")


def test_sew_resnet18_fp16_teacher_forced_b64(dev):
    """fp16-operand mode at config 1's batch: every layer, fed its own input,
    meets the per-layer gates against the fp16-operand oracle."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _sew_net(B=64, seed=2)
    model, _ = optimize(net, device=dev, T=4)
    functional.reset_net(model)
    model(x.to(dev))
    plan = model.plan_for(x.to(dev))
    assert _teacher_forced_layers(plan, dev) <= 1e-4


def test_forward_with_k_invariance(dev):
    """SparseFlow.forward_with_k: TimeBlock(K) with v carried through the
    StateBuffer gives the K=T output bit for bit for K in {1, 2, 4, T}
    (the reference's tests/parity_suite_smoke.py:61-117)."""
    from catfuse_b200 import patterns
    from catfuse_b200.sj import layer, neuron
    g = torch.Generator().manual_seed(13)
    conv = layer.Conv2d(64, 128, 3, 1, 1, bias=False)
    bn = layer.BatchNorm2d(128)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) * 0.08)
        bn.running_mean.copy_(torch.randn(128, generator=g) * 0.1)
        bn.running_var.copy_(torch.rand(128, generator=g) + 0.5)
    bn.eval()
    lif = neuron.LIFNode(tau=2.0, step_mode="m")
    T = 8
    x = (torch.rand(T, 2, 64, 12, 12, generator=g) < 0.2).float().to(dev)
    m = patterns.STFusionConvBNLIF.from_sj_modules(conv, bn, lif).to(dev)
    impl = m._impl_sparse
    outs = {}
    for K in (1, 2, 4, T):
        m.reset()
        outs[K] = impl.forward_with_k(x, m.spec, m._ensure_params(), m.state, K=K)
        v = m.state.tensor.clone()
        if K == T:
            vT = v
    for K in (1, 2, 4):
        assert torch.equal(outs[K], outs[T]), f"K={K}"
    assert outs[T].sum() > 0
    # and the dense implementation agrees with the oracle at fp16 operands
    scale, shift = oracle.fold_bn(bn.weight.detach(), bn.bias.detach(), bn.running_mean,
                                  bn.running_var)
    s_o, v_o, z = oracle.conv_bn_lif(x.cpu(), conv.weight.detach(), scale, shift, 1, 1,
                                     operand_dtype=torch.float16, return_z=True)
    _, _, h = lif_trace(z)
    check_lif_parity(outs[T].cpu().numpy(), vT.cpu().numpy(), s_o, v_o, h, what="forward_with_k")


def test_avgpool_fc_head(dev):
    """avgpool -> flatten -> fc over x[B,H,W,T,C] fp16 (the ResNet head)."""
    from catfuse_b200 import ops
    g = torch.Generator().manual_seed(17)
    T, B, C, H, W, K = 4, 5, 512, 4, 4, 10
    x = ((torch.rand(T, B, C, H, W, generator=g) < 0.3).float()
         + (torch.rand(T, B, C, H, W, generator=g) < 0.2).float())   # SEW counts {0,1,2}
    fc_w = torch.randn(K, C, generator=g) * 0.05
    fc_b = torch.randn(K, generator=g) * 0.1
    xp = ops.pack_tbchw(x.to(dev))
    out = ops.avgpool_fc(xp, fc_w.to(dev), fc_b.to(dev)).cpu()
    ref = torch.nn.functional.linear(x.double().mean(dim=(3, 4)), fc_w.double(), fc_b.double())
    assert (out.double() - ref).abs().max() <= 1e-5
    out0 = ops.avgpool_fc(xp, fc_w.to(dev), None).cpu()
    ref0 = torch.nn.functional.linear(x.double().mean(dim=(3, 4)), fc_w.double())
    assert (out0.double() - ref0).abs().max() <= 1e-5


def test_network_device_egd_equals_dense(dev):
    """SEW-ResNet-18 with every 3x3/s1 conv forced onto STFusion: the native
    plan's prescan + device-side EGD gives the same logits bit for bit as the
    dense plan, on inputs whose left half is zero (so some tiles are empty and
    the kernel's choice differs per layer)."""
    from catfuse_b200.network import CTFNetwork
    from catfuse_b200.substitute import substitute_sf
    from catfuse_b200 import hardware
    from catfuse_b200.sj import functional
    net, x = _sew_net(B=8, seed=4)
    x = x.clone()
    x[..., :16] = 0.0
    m, st = substitute_sf(net, T=4, force_sparse=True, hwprof=hardware.B200)
    assert st["patterns_matched"].get("STFusionConvBNLIF", 0) > 6
    m = m.to(dev)
    sparse = CTFNetwork(m, use_sparse=True)
    dense = CTFNetwork(m, use_sparse=False)
    xd = x.to(dev)
    functional.reset_net(sparse)
    functional.reset_net(dense)
    a = sparse(xd)
    b = dense(xd)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    plan = sparse.plan_for(xd)
    assert sum(1 for s in plan.steps if getattr(s, "sparse", False)) > 6


def _spiking_net_224(B, seed):
    from catfuse_b200.sj import zoo
    net = zoo.init_random_(zoo.build_spiking_resnet18_imagenet(num_classes=1000), seed)
    g = torch.Generator().manual_seed(500 + seed)
    x = torch.randn(B, 3, 224, 224, generator=g).unsqueeze(0).repeat(4, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, x)
    return net.eval(), x


def test_spiking_resnet18_224_fp16(dev):
    """Config 3 shape (Spiking ResNet-18, ImageNet stem 7x7/2 + max-pool,
    add-before-LIF blocks, 224x224; B=2 to keep the CPU oracle short): every
    layer, fed its own input, meets the per-layer gates against the oracle at
    the kernel's operand precision.  (End to end, a single near-threshold
    flip among the stem's 1.6 M neurons already cascades through the 16 later
    layers, so the logits are compared per layer rather than at the end.)"""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _spiking_net_224(B=2, seed=5)
    model, stats = optimize(net, device=dev, T=4)
    assert stats["native_plan"]
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    assert torch.isfinite(logits).all()
    plan = model.plan_for(x.to(dev))
    assert plan.shapes[1][1:3] == (112, 112) and plan.shapes[-1][1:3] == (7, 7)
    assert _teacher_forced_layers(plan, dev) <= 1e-4


def test_spiking_resnet18_224_fp32_mode(dev):
    """Config 3 shape in the fp32-faithful mode: every layer, fed its own
    input, against an fp64 restatement of the layer -- flips only within 1e-5
    of the threshold, v within 1e-4 (the z-only downsample branch enters the
    add-before-LIF epilogue from the fp16 activation layout, as the oracle
    restatement reads it)."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _spiking_net_224(B=2, seed=6)
    model, _ = optimize(net, device=dev, T=4, precision="fp32")
    functional.reset_net(model)
    model(x.to(dev))
    plan = model.plan_for(x.to(dev))
    assert _teacher_forced_fp64(plan) <= 1e-4


def test_dual_launch_downsample_bit_identical(dev, monkeypatch):
    """SEW blocks' 1x1/s2 downsample computed inside the first conv's launch
    (cf_conv_bn_lif_dual) gives the same spikes, membranes and logits bit for
    bit as two separate launches."""
    from catfuse_b200 import optimize
    from catfuse_b200.network import ConvStep, NetworkPlan
    from catfuse_b200.sj import functional
    net, x = _sew_net(B=8, seed=3)
    xd = x.to(dev)
    m1, _ = optimize(net, device=dev, T=4)
    functional.reset_net(m1)
    a = m1(xd)
    p1 = m1.plan_for(xd)
    assert sum(1 for st in p1.steps if isinstance(st, ConvStep) and st.dual is not None) == 3
    monkeypatch.setattr(NetworkPlan, "_try_dual", lambda self, f, d: None)
    m2, _ = optimize(net, device=dev, T=4)
    functional.reset_net(m2)
    b = m2(xd)
    p2 = m2.plan_for(xd)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    for s1, s2 in zip(p1.steps, p2.steps):
        if isinstance(s1, ConvStep):
            assert torch.equal(p1.acts[s1.dst], p2.acts[s2.dst]), s1.name
            if s1.v is not None:
                assert torch.equal(s1.v, s2.v), s1.name
