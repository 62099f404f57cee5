"""GPU parity of the fused spiking self-attention + attention LIF kernel
(cf_ssa_lif, through the C ABI) against the CPU oracle: bit-exact against the
exact-integer form, and within the LIF tolerance of the reference's fp32
matmul order."""
import numpy as np
import pytest
import torch

import oracle
from lif_parity import check_lif_parity, lif_trace

pytestmark = pytest.mark.gpu


def _to_bntc(x):  # [T,B,N,C] -> [B,N,T,C] fp16 CUDA
    return torch.from_numpy(np.ascontiguousarray(x.transpose(1, 2, 0, 3))).half().cuda()


@pytest.mark.parametrize("shape", [(4, 3, 64, 384, 12), (2, 2, 37, 64, 2), (5, 1, 16, 96, 4),
                                   (1, 2, 64, 32, 4)])
def test_ssa_lif_vs_oracle(dev, shape):
    from catfuse_b200 import ops
    T, B, N, C, heads = shape
    g = torch.Generator().manual_seed(sum(shape))
    q, k, v = ((torch.rand(T, B, N, C, generator=g) < p).float().numpy() for p in (0.1, 0.1, 0.3))
    v0 = (torch.randn(B, N, C, generator=g) * 0.3).numpy()
    vth = 0.5
    lif = ops.LIFConfig(v_threshold=vth)
    vout = torch.from_numpy(v0).cuda().contiguous()
    out = ops.ssa_lif(_to_bntc(q), _to_bntc(k), _to_bntc(v), heads, v_in=vout, v_out=vout, lif=lif)
    s = out.float().cpu().numpy().transpose(2, 0, 1, 3)
    vT = vout.cpu().numpy()
    s_e, v_e, y = oracle.ssa_lif(q, k, v, heads, v0=v0, form="exact", v_threshold=vth)
    assert np.array_equal(s, s_e), "spikes differ from the exact-integer oracle"
    assert np.array_equal(vT, v_e), "membranes differ from the exact-integer oracle"
    assert 0.005 < s.mean() < 0.97, "degenerate case"
    s_r, v_r, y_r = oracle.ssa_lif(q, k, v, heads, v0=v0, form="reference", v_threshold=vth)
    _, _, h = lif_trace(y_r, v0, vth=vth)
    check_lif_parity(s, vT, s_r, v_r, h, vth=vth, v_tol=1e-4, near_tol=1e-3, max_flip_rate=1e-4,
                     what=f"reference fp32 order {shape}")


def test_ssa_rejects_unsupported(dev):
    from catfuse_b200 import ops
    from catfuse_b200._lib import CatfuseNativeError
    x = torch.zeros(1, 65, 1, 32, dtype=torch.float16, device="cuda")
    with pytest.raises(CatfuseNativeError):
        ops.ssa_lif(x, x, x, 1)


class _RefSSA(torch.nn.Module):
    """Reference-shaped SSA container (attribute names of the reference module)."""

    def __init__(self, dim, heads, vth):
        super().__init__()
        from catfuse_b200.sj import neuron
        self.num_heads = heads
        for n in ("q", "k", "v", "proj"):
            setattr(self, n, torch.nn.Linear(dim, dim))
            bn = torch.nn.BatchNorm1d(dim).eval()
            with torch.no_grad():
                bn.running_mean.normal_(0, 0.1)
                bn.running_var.uniform_(0.5, 1.5)
                bn.weight.uniform_(0.8, 1.2)
                bn.bias.normal_(0, 0.1)
            setattr(self, n + "_bn", bn)
            setattr(self, n + "_lif", neuron.LIFNode(tau=2.0, v_threshold=vth))
        self.attn_lif = neuron.LIFNode(tau=2.0, v_threshold=vth)


def _linear_bn_lif_oracle(x, lin, bn, vth):
    w = lin.weight.detach().half().float()
    z = x.half().float() @ w.T + lin.bias.detach()
    sc = bn.weight.detach() / torch.sqrt(bn.running_var + bn.eps)
    z = z * sc + (bn.bias.detach() - bn.running_mean * sc)
    s, _, h = lif_trace(z.numpy(), vth=vth)
    return s, h


def test_fused_ssa_module(dev):
    from catfuse_b200 import ops, patterns
    torch.manual_seed(3)
    T, B, N, C, heads, vth = 4, 2, 64, 96, 3, 0.5
    ref = _RefSSA(C, heads, vth)
    m = patterns.FusedSSA.from_sj_modules(ref).to(dev)
    x = (torch.rand(T, B, N, C) < 0.3).float() * (1 + (torch.rand(T, B, N, C) < 0.2).float())
    xd = x.to(dev)
    out = m(xd)
    # stage by stage, teacher-forced on the module's own intermediate spikes
    m.reset()
    qs, ks, vs = m.q(xd), m.k(xd), m.v(xd)
    for got, name in ((qs, "q"), (ks, "k"), (vs, "v")):
        s_o, h = _linear_bn_lif_oracle(x, getattr(ref, name), getattr(ref, name + "_bn"), vth)
        check_lif_parity(got.cpu().numpy(), None, s_o, None, h, vth=vth, near_tol=1e-3,
                         max_flip_rate=1e-4, what=f"{name} linear-bn-lif")
    q_, k_, v_ = (t.cpu().numpy() for t in (qs, ks, vs))
    y_e, _, _ = oracle.ssa_lif(q_, k_, v_, heads, v_threshold=vth)
    to_bntc = lambda s: s.permute(1, 2, 0, 3).half().contiguous()
    y = ops.ssa_lif(to_bntc(qs), to_bntc(ks), to_bntc(vs), heads, lif=ops.LIFConfig(v_threshold=vth))
    y = y.permute(2, 0, 1, 3).float()
    assert np.array_equal(y.cpu().numpy(), y_e)
    s_o, h = _linear_bn_lif_oracle(y.cpu(), ref.proj, ref.proj_bn, vth)
    check_lif_parity(out.cpu().numpy(), None, s_o, None, h, vth=vth, near_tol=1e-3,
                     max_flip_rate=1e-4, what="proj linear-bn-lif")
    # StateCarry: a second call continues from the carried membranes; reset restores
    m.reset()
    a = m(xd)
    b2 = m(xd)
    m.reset()
    c = m(xd)
    assert torch.equal(a, c) and torch.equal(a, out)
    assert not torch.equal(a, b2)
