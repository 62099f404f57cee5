"""GPU parity of the bandwidth-bound LIF family against the oracle and the
reference's golden vectors (called through the C ABI)."""
import numpy as np
import pytest
import torch

import oracle
from lif_parity import check_lif_parity, lif_trace

pytestmark = pytest.mark.gpu


def _ops():
    from catfuse_b200 import ops
    return ops


def test_lif_fwd_golden_and_oracle(dev, golden_dir):
    ops = _ops()
    g = np.load(golden_dir / "golden_lif.npz")
    z = torch.from_numpy(g["z"]).to(dev)
    v0 = torch.from_numpy(g["v0"]).to(dev)
    for tau, ks, kv in ((2.0, "spikes", "vT"), (3.0, "spikes_tau3", "vT_tau3")):
        s, vT = ops.lif_fwd(z, v0, ops.LIFConfig(tau=tau))
        s, vT = s.cpu().numpy(), vT.cpu().numpy()
        # bit-exact against the SJ-form oracle
        s_o, v_o = oracle.lif_multistep(g["z"], g["v0"], tau=tau)
        assert np.array_equal(s, s_o)
        assert np.array_equal(vT, v_o)
        # reference Triton kernel form: equal up to 1-ULP charge differences
        _, _, h = lif_trace(g["z"], g["v0"], tau=tau)
        check_lif_parity(s, vT, g[ks], g[kv], h, v_tol=1e-5, near_tol=1e-5, max_flip_rate=1e-3,
                         what=f"golden tau={tau}")


@pytest.mark.parametrize("fmt", [torch.float16, torch.uint8, "bits"])
def test_lif_spike_formats(dev, fmt):
    ops = _ops()
    gen = torch.Generator().manual_seed(1)
    z = (torch.randn(5, 4, 64, 8, generator=gen) * 1.5).to(dev)
    s32, v32 = ops.lif_fwd(z)
    s, v = ops.lif_fwd(z, spike_dtype=fmt)
    assert torch.equal(v, v32)
    if fmt == "bits":
        words = s.cpu().numpy().view(np.uint32)                     # [T, N/32]
        bits = ((words[..., None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(5, -1)
        assert np.array_equal(bits.astype(np.float32), s32.reshape(5, -1).cpu().numpy())
    else:
        assert torch.equal(s.float(), s32)


@pytest.mark.parametrize("hard,decay,tau", [(True, True, 2.0), (False, True, 2.0),
                                            (True, False, 2.0), (False, False, 1.7),
                                            (True, True, 5.0)])
def test_lif_variants_exact(dev, hard, decay, tau):
    ops = _ops()
    gen = torch.Generator().manual_seed(2)
    z = torch.randn(7, 3, 37, generator=gen) * 1.3 + 0.4      # N = 111: scalar path
    v0 = torch.randn(3, 37, generator=gen)
    cfg = ops.LIFConfig(tau=tau, v_threshold=0.8, v_reset=-0.1 if hard else None, decay_input=decay)
    s, vT = ops.lif_fwd(z.to(dev), v0.to(dev), cfg)
    s_o, v_o = oracle.lif_multistep(z.numpy(), v0.numpy(), tau, 0.8, -0.1 if hard else None,
                                    hard_reset=hard, decay_input=decay)
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(vT.cpu().numpy(), v_o)


def test_lif_fp16_input_and_empty(dev):
    ops = _ops()
    gen = torch.Generator().manual_seed(3)
    z = (torch.randn(4, 1024, generator=gen)).half()
    s, vT = ops.lif_fwd(z.to(dev))
    s_o, v_o = oracle.lif_multistep(z.float().numpy())
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(vT.cpu().numpy(), v_o)
    s0, v0 = ops.lif_fwd(torch.empty(0, 16, device=dev))
    assert s0.shape == (0, 16)


def test_bn_lif_golden_static_zero_and_identity(dev, golden_dir):
    ops = _ops()
    g = np.load(golden_dir / "golden_bn_lif.npz")
    z = torch.from_numpy(g["z"]).to(dev)
    sc = torch.from_numpy(g["scale"]).to(dev)
    sh = torch.from_numpy(g["shift"]).to(dev)
    s, vT = ops.bn_lif(z, sc, sh)
    zz = (g["z"] * g["scale"][None, None, :, None, None]).astype(np.float32) + g["shift"][None, None, :, None, None]
    s_o, v_o, h = lif_trace(zz.astype(np.float32))
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(vT.cpu().numpy(), v_o)
    check_lif_parity(s.cpu().numpy(), None, g["spikes"], None, h, near_tol=1e-5, max_flip_rate=1e-3,
                     what="golden bn_lif")
    # StaticZero: z == 0 -> z' = shift
    s0, v0 = ops.bn_lif(None, sc, sh, shape=tuple(z.shape), device=dev)
    z0 = np.broadcast_to(g["shift"][None, None, :, None, None], g["z"].shape).astype(np.float32)
    s0_o, v0_o = oracle.lif_multistep(z0)
    assert np.array_equal(s0.cpu().numpy(), s0_o)
    assert np.array_equal(v0.cpu().numpy(), v0_o)
    # pre-LIF identity (bn_add_lif)
    ident = torch.randn(z.shape, generator=torch.Generator().manual_seed(4))
    s2, v2 = ops.bn_lif(z, sc, sh, identity=ident.to(dev))
    s2_o, v2_o = oracle.lif_multistep((zz + ident.numpy()).astype(np.float32))
    assert np.array_equal(s2.cpu().numpy(), s2_o)
    assert np.array_equal(v2.cpu().numpy(), v2_o)


def test_add_and_avgpool_lif(dev):
    ops = _ops()
    gen = torch.Generator().manual_seed(5)
    x1 = torch.randn(4, 2, 8, 6, 6, generator=gen)
    x2 = torch.randn(4, 2, 8, 6, 6, generator=gen)
    s, vT = ops.add_lif(x1.to(dev), x2.to(dev))
    s_o, v_o = oracle.lif_multistep((x1 + x2).numpy())
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(vT.cpu().numpy(), v_o)
    x = torch.randn(3, 2, 4, 8, 6, generator=gen) * 2
    s, vT = ops.avgpool_lif(x.to(dev), 2)
    xn = x.numpy()
    pooled = ((((xn[..., 0::2, 0::2] + xn[..., 0::2, 1::2]).astype(np.float32) + xn[..., 1::2, 0::2]).astype(np.float32)
               + xn[..., 1::2, 1::2]).astype(np.float32) * np.float32(0.25)).astype(np.float32)
    s_o, v_o = oracle.lif_multistep(pooled)
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(vT.cpu().numpy(), v_o)
