"""Spikformer (config 4: embed 384, 12 heads, MLP ratio 4, 4 blocks, 32x32
images -> 64 tokens, T=4) through optimize() and its native plan, checked
layer by layer against the CPU oracle restatement of the reference model."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _net(B, seed=0, depth=4):
    from catfuse_b200.sj import spikformer, zoo
    net = zoo.init_random_(spikformer.build_spikformer_cifar(depth=depth), seed)
    g = torch.Generator().manual_seed(300 + seed)
    x = torch.randn(B, 3, 32, 32, generator=g).unsqueeze(0).repeat(4, 1, 1, 1, 1)
    zoo.calibrate_bn_(net, x)
    return net.eval(), x


def _compare(got, record, limit):
    rows = []
    for name, s_ref, _ in record:
        if name == "pre_head_lif":
            continue
        g = got[name].numpy()
        r = s_ref.numpy()
        assert g.shape == r.shape, (name, g.shape, r.shape)
        rows.append((name, float((g != r).mean()), float(r.mean())))
    for name, rate, dens in rows:
        print(f"  {name:28s} flips {rate:.2e}  spike rate {dens:.3f}")
    for name, rate, _ in rows:
        assert rate <= limit(name), f"{name}: flip rate {rate:.2e}"
    return rows


def test_spikformer_fp16_vs_oracle(dev):
    """fp16 operands (the reference GPU path's precision): every LIF layer
    against the oracle run at the same operand precision."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _net(B=8)
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    model, stats = optimize(net, device=dev, T=4)
    assert stats["native_plan"] and type(model).__name__ == "CTFSpikformer"
    assert stats["fused_lif_nodes"] >= 4 * 6 + 5
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    plan = model.plan_for(x.to(dev))
    p16 = {k: (v.half().float() if k.endswith(".weight") and v.dim() in (2, 4) and "head" not in k
               and "bn" not in k else v) for k, v in params.items()}
    rec = []
    ref = oracle.spikformer_forward(x.half().float(), p16, 12, 4, record=rec)
    _compare(plan.layer_spikes(), rec, lambda n: 1e-4 if n.startswith("patch") else 1e-3)
    rel = (logits - ref).abs().max() / ref.abs().max().clamp_min(1e-6)
    assert rel < 1e-2, f"logits rel err {rel}"


def test_spikformer_fp32_mode_vs_fp64(dev):
    """fp32-faithful mode (exact integer weight planes, hi + lo stem): every
    LIF layer of the tokenizer and the first block within 1e-4 flips of the
    fp64 oracle, every layer within 1e-3, classifier argmax identical."""
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _net(B=16, seed=1)
    params = {k: v.detach().float() for k, v in net.state_dict().items()}
    model, _ = optimize(net, device=dev, T=4, precision="fp32")
    functional.reset_net(model)
    logits = model(x.to(dev)).cpu()
    plan = model.plan_for(x.to(dev))
    rec = []
    ref = oracle.spikformer_forward(x, params, 12, 4, record=rec, dtype=torch.float64)
    _compare(plan.layer_spikes(), rec,
             lambda n: 1e-4 if (n.startswith("patch") or n.startswith("blocks.0")) else 1e-3)
    agree = (logits.sum(0).argmax(-1) == ref.sum(0).argmax(-1)).float().mean()
    assert agree == 1.0
    rel = (logits.double() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)
    print(f"fp32 mode: logits rel err vs fp64 {float(rel):.2e}")


def test_spikformer_graph_eager_state_carry(dev):
    from catfuse_b200 import optimize
    from catfuse_b200.sj import functional
    net, x = _net(B=2, seed=2, depth=2)
    mg, _ = optimize(net, device=dev, T=4)
    me, _ = optimize(net, device=dev, T=4, use_graph=False)
    xd = x.to(dev)
    functional.reset_net(mg)
    functional.reset_net(me)
    a = mg(xd)
    assert torch.equal(a, me(xd))
    a2 = mg(xd)                      # StateCarry: continues the membranes
    m8, _ = optimize(net, device=dev, T=8)
    functional.reset_net(m8)
    l8 = m8(torch.cat([xd, xd], 0))
    assert torch.equal(a, l8[:4]) and torch.equal(a2, l8[4:])


def test_token_mean_lif_fc(dev):
    from catfuse_b200 import ops
    g = torch.Generator().manual_seed(5)
    T, B, N, C, K = 4, 3, 64, 384, 10
    x = ((torch.rand(B, N, T, C, generator=g) < 0.4).float()
         + (torch.rand(B, N, T, C, generator=g) < 0.4).float() * 3)   # counts {0,1,3,4}
    w = torch.randn(K, C, generator=g) * 0.1
    b = torch.randn(K, generator=g) * 0.1
    v = torch.zeros(B, C, device=dev)
    out = ops.token_mean_lif_fc(x.half().to(dev), w.to(dev), b.to(dev), v_out=v).cpu()
    m = x.mean(dim=1).permute(1, 0, 2)          # [T, B, C]
    s, vT = oracle.lif_multistep(m.numpy())
    ref = torch.from_numpy(s) @ w.T + b
    assert (out - ref).abs().max() <= 1e-5
    assert np.abs(v.cpu().numpy() - vT).max() == 0
