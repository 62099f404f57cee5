"""The CPU oracle pinned against fixtures produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import torch

import oracle
from lif_parity import check_lif_parity, lif_trace


def test_lif_oracle_vs_reference_kernel(golden_dir):
    g = np.load(golden_dir / "golden_lif.npz")
    for tau, ks, kv in ((2.0, "spikes", "vT"), (3.0, "spikes_tau3", "vT_tau3")):
        # the Triton-form restatement reproduces the reference kernel exactly
        s_t, v_t = oracle.lif_multistep_triton_form(g["z"], g["v0"], tau=tau)
        assert np.array_equal(s_t, g[ks])
        assert np.abs(v_t - g[kv]).max() <= 1e-6
        # the SJ form differs only by charge-rounding at the threshold
        s, v, h = lif_trace(g["z"], g["v0"], tau=tau)
        check_lif_parity(s, v, g[ks], g[kv], h, v_tol=1e-5, near_tol=1e-5, max_flip_rate=1e-3)


def test_bn_lif_oracle_vs_reference_kernel(golden_dir):
    g = np.load(golden_dir / "golden_bn_lif.npz")
    z = (g["z"] * g["scale"][None, None, :, None, None]).astype(np.float32) + g["shift"][None, None, :, None, None]
    s, v, h = lif_trace(z.astype(np.float32))
    check_lif_parity(s, None, g["spikes"], None, h, near_tol=1e-5, max_flip_rate=1e-3)


def test_prescan_oracle_bit_exact(golden_dir):
    g = np.load(golden_dir / "golden_prescan.npz")
    for i in range(int(g["n_cases"])):
        c = {k[len(f"c{i}_"):]: g[k] for k in g.files if k.startswith(f"c{i}_")}
        ag, cls, nnz = oracle.prescan_rf(c["x"], int(c["k"]), int(c["s"]), int(c["p"]),
                                         int(c["BH"]), int(c["BW"]), int(c["GS"]))
        assert np.array_equal(ag, c["ag_mask"]), f"case {i}"
        assert np.array_equal(cls, c["tile_class"]), f"case {i}"
        assert nnz == int(np.count_nonzero(c["x"]))
        if "ag_mask_v2" in c:
            assert np.array_equal(ag, c["ag_mask_v2"])
        # geometry helpers
        C = c["x"].shape[1]
        assert oracle.choose_group_size(C) == int(c["GS"])
        assert oracle.select_tile_sizes(int(c["Ho"]), int(c["Wo"])) == (int(c["BH"]), int(c["BW"]))


def test_conv_bn_lif_oracle_vs_reference_paths(golden_dir):
    g = np.load(golden_dir / "golden_conv_bn_lif.npz")
    x = torch.from_numpy(g["x"].astype(np.float32))
    w = torch.from_numpy(g["weight"])
    scale, shift = oracle.fold_bn(g["gamma"], g["beta"], g["mean"], g["var"])
    s, v, z = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, return_z=True)
    _, _, h = lif_trace(z)
    # the reference's own fp32 per-step path
    check_lif_parity(s, v, g["spikes"], g["vT"], h, v_tol=1e-5, near_tol=1e-5, max_flip_rate=1e-4)
    # the StreamFuse kernel (fp16 operands): same operand rounding in the oracle
    s16, v16, z16 = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, operand_dtype=torch.float16,
                                       return_z=True)
    _, _, h16 = lif_trace(z16)
    check_lif_parity(s16, v16, g["sf_spikes"], g["sf_vT"], h16, v_tol=1e-5, near_tol=1e-4,
                     max_flip_rate=1e-4)
    assert g["spikes"].mean() > 0.01


def test_network_oracle_matches_sj_shim():
    """The oracle ResNets equal the SJ-compatible model builders run eagerly."""
    from catfuse_b200.sj import functional, zoo
    p = oracle.make_resnet18_params()
    net = zoo.load_params(zoo.build_sew_resnet18_cifar(), p)
    x = torch.randn(4, 2, 3, 32, 32, generator=torch.Generator().manual_seed(0))
    functional.reset_net(net)
    with torch.no_grad():
        assert torch.equal(net(x), oracle.sew_resnet18_forward(x, p))


def test_ssa_oracle_forms_agree():
    """SSA restatement: the exact-integer form equals a per-head loop of the
    reference's formula in float64, and the fp32 reference order stays within
    a few ulp of it."""
    import torch
    g = torch.Generator().manual_seed(5)
    T, B, N, C, heads = 2, 2, 12, 48, 3
    q, k, v = ((torch.rand(T, B, N, C, generator=g) < 0.3).float().numpy() for _ in range(3))
    _, _, y = oracle.ssa_lif(q, k, v, heads)
    d = C // heads
    sc = np.float32(d ** -0.5)
    for t in range(T):
        for b in range(B):
            for h in range(heads):
                sl = slice(h * d, (h + 1) * d)
                ref = ((q[t, b, :, sl].astype(np.float64) @ k[t, b, :, sl].T.astype(np.float64))
                       @ v[t, b, :, sl].astype(np.float64)) * np.float64(sc)
                assert np.array_equal(y[t, b, :, sl], ref.astype(np.float32))
    _, _, y_r = oracle.ssa_lif(q, k, v, heads, form="reference")
    assert np.abs(y_r - y).max() <= 1e-5 * max(1.0, float(np.abs(y).max()))
