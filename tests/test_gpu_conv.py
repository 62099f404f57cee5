"""GPU parity of the tcgen05 fused Conv -> BN -> LIF kernel (through the C ABI)
against the CPU oracle, the reference's golden vectors, and itself (sparse vs
dense, chunked T vs single block)."""
import numpy as np
import pytest
import torch

import oracle
from catfuse_b200 import workloads
from lif_parity import check_lif_parity, lif_trace

pytestmark = pytest.mark.gpu


def _ops():
    from catfuse_b200 import ops
    return ops


def _case(T, B, Cin, Cout, H, W, k, seed, p=0.25):
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand(T, B, Cin, H, W, generator=g) < p).float()
    w = torch.randn(Cout, Cin, k, k, generator=g) * (2.0 / (Cin * k * k)) ** 0.5 * 1.5
    scale = torch.rand(Cout, generator=g) * 0.4 + 0.8
    shift = torch.randn(Cout, generator=g) * 0.3
    return x, w, scale, shift


def _run(dev, x, w, scale, shift, stride, pad, precision="fp16", **kw):
    ops = _ops()
    T, B, Cin, H, W = x.shape
    Cout = w.shape[0]
    xp = ops.pack_tbchw(x.to(dev))
    if precision == "split":
        wp, pre = ops.pack_conv_weight_split(w.to(dev), xp.shape[-1])
        scale = scale / pre
        kw["precision"] = "split"
    else:
        wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    Ho = (H + 2 * pad - w.shape[2]) // stride + 1
    Wo = (W + 2 * pad - w.shape[3]) // stride + 1
    v_out = torch.empty(B, Ho, Wo, Cout, device=dev)
    out = ops.conv_bn_lif(xp, wp, scale.to(dev), shift.to(dev), stride, pad, v_out=v_out, **kw)
    s = ops.unpack_bhwtc(out).cpu().numpy()
    v = ops.v_to_nchw(v_out).cpu().numpy()
    return s, v, xp


SHAPES = [
    # T, B, Cin, Cout, H, W, k, stride, pad
    (4, 2, 64, 64, 8, 8, 3, 1, 1),
    (4, 4, 128, 128, 16, 16, 3, 1, 1),
    (4, 2, 64, 128, 16, 16, 3, 2, 1),
    (4, 2, 64, 128, 16, 16, 1, 2, 0),
    (4, 2, 3, 64, 32, 32, 3, 1, 1),
    (1, 2, 32, 32, 7, 9, 3, 1, 1),
    (3, 2, 32, 64, 6, 6, 3, 1, 1),
    (2, 3, 48, 96, 10, 6, 3, 1, 1),
    (8, 2, 256, 256, 7, 7, 3, 1, 1),
    (12, 1, 32, 32, 5, 5, 3, 1, 1),
    (4, 2, 16, 64, 15, 15, 7, 2, 3),
    (4, 2, 512, 512, 4, 4, 3, 1, 1),
    # one full output row per tile (single-box receptive-field loads)
    (4, 2, 64, 64, 32, 32, 3, 1, 1),
    (2, 2, 64, 64, 64, 64, 3, 1, 1),
    (4, 3, 64, 32, 32, 32, 3, 1, 1),
    # channel-major kernel (Cout % 128 == 0): N = 256 / 128 pixel-time rows,
    # ragged pixel tiles, T = 1 / 3 / chunked T, several channel tiles
    (12, 1, 32, 128, 5, 5, 3, 1, 1),
    (2, 3, 48, 128, 10, 6, 3, 1, 1),
    (1, 2, 32, 256, 7, 9, 3, 1, 1),
    (3, 1, 64, 384, 9, 9, 3, 2, 1),
    (4, 8, 128, 128, 32, 32, 3, 1, 1),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_bn_lif_vs_oracle(dev, shape):
    T, B, Cin, Cout, H, W, k, st, pad = shape
    x, w, scale, shift = _case(T, B, Cin, Cout, H, W, k, seed=hash(shape) % 1000)
    s, v, _ = _run(dev, x, w, scale, shift, st, pad)
    # same operand precision (fp16 weights, exact spikes): only the fp32
    # accumulation order differs
    s_o, v_o, z = oracle.conv_bn_lif(x, w, scale, shift, st, pad, operand_dtype=torch.float16,
                                     return_z=True)
    _, _, h = lif_trace(z)
    rate = check_lif_parity(s, v, s_o, v_o, h, v_tol=1e-4, near_tol=1e-3, max_flip_rate=1e-4,
                            what=f"fp16-operand oracle {shape}")
    # the fp32 reference (north-star tolerance for the tensor-core path)
    s32, v32, z32 = oracle.conv_bn_lif(x, w, scale, shift, st, pad, return_z=True)
    _, _, h32 = lif_trace(z32)
    check_lif_parity(s, v, s32, v32, h32, v_tol=2e-2, near_tol=2e-2, max_flip_rate=1e-4,
                     what=f"fp32 oracle {shape}")
    assert s.mean() > 0.005, "degenerate case: almost no spikes"


@pytest.mark.parametrize("C", [64, 128])
@pytest.mark.parametrize("mode", ["add", "add_pre", "and", "iand"])
def test_conv_residual_modes(dev, mode, C):
    ops = _ops()
    T, B, H, W = 4, 2, 8, 8
    x, w, scale, shift = _case(T, B, C, C, H, W, 3, seed=11)
    g = torch.Generator().manual_seed(12)
    ident = (torch.rand(T, B, C, H, W, generator=g) < 0.3).float() * (1 + (torch.rand(T, B, C, H, W, generator=g) < 0.3).float())
    idp = ops.pack_tbchw(ident.to(dev))
    s, v, _ = _run(dev, x, w, scale, shift, 1, 1, identity=idp, res_mode=mode)
    out_o, v_o = oracle.conv_bn_lif_residual(x, w, scale, shift, ident, mode, 1, 1,
                                             operand_dtype=torch.float16)
    diff = s != out_o
    assert diff.mean() <= 1e-4, f"{mode}: mismatch rate {diff.mean()}"
    ok = ~diff.any(axis=0)
    assert np.abs(v - v_o)[ok].max() <= 1e-4


@pytest.mark.parametrize("C", [32, 128])
def test_conv_state_carry_and_inplace(dev, C):
    """v_in -> v_out StateCarry; v_in may alias v_out; T-chunked launch equals
    the oracle with v carried."""
    ops = _ops()
    T, B, H, W = 10, 2, 6, 6
    x, w, scale, shift = _case(T, B, C, C, H, W, 3, seed=21)
    g = torch.Generator().manual_seed(22)
    v0 = torch.randn(B, C, H, W, generator=g) * 0.5
    xp = ops.pack_tbchw(x.to(dev))
    wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    v = ops.v_to_nhwc(v0.to(dev).contiguous())
    out = ops.conv_bn_lif(xp, wp, scale.to(dev), shift.to(dev), 1, 1, v_in=v, v_out=v)
    s = ops.unpack_bhwtc(out).cpu().numpy()
    vT = ops.v_to_nchw(v).cpu().numpy()
    s_o, v_o, z = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, v0=v0.numpy(),
                                     operand_dtype=torch.float16, return_z=True)
    _, _, h = lif_trace(z, v0.numpy())
    check_lif_parity(s, vT, s_o, v_o, h, v_tol=1e-4, near_tol=1e-3, what="state carry")


def _conv_tile_mask_oracle(x_bhwtc, geom, KH, KW, st, pad, chunk):
    B, H, W, T, Cp = x_bhwtc.shape
    Ho = (H + 2 * pad - KH) // st + 1
    Wo = (W + 2 * pad - KW) // st + 1
    Wb, Hb, Bb = geom["Wb"], geom["Hb"], geom["Bb"]
    nwt, nht = -(-Wo // Wb), -(-Ho // Hb)
    nbt = -(-B // Bb)
    nz = (x_bhwtc != 0).reshape(B, H, W, T, Cp // chunk, chunk).any(axis=(3, 5))  # [B,H,W,nc]
    masks = []
    for bt in range(nbt):
        for ht in range(nht):
            for wt in range(nwt):
                oh0, oh1 = ht * Hb, min(Ho, ht * Hb + Hb) - 1
                ow0, ow1 = wt * Wb, min(Wo, wt * Wb + Wb) - 1
                r0, r1 = max(0, oh0 * st - pad), min(H, oh1 * st - pad + KH)
                c0, c1 = max(0, ow0 * st - pad), min(W, ow1 * st - pad + KW)
                blk = nz[bt * Bb:(bt + 1) * Bb, r0:r1, c0:c1]
                act = blk.reshape(-1, Cp // chunk).any(axis=0)
                masks.append(int(sum(1 << i for i in np.nonzero(act)[0])))
    return np.array(masks, dtype=np.int64)


@pytest.mark.parametrize("sparsity", workloads.CONFIG2["sparsities"])
def test_sparse_masks_and_bit_identity(dev, sparsity):
    """SparseFlow at the config-2 shape ([4, 32, 256, 28, 28], 8x8x32 zero
    blocks): the conv-tile prescan masks are exact, the masked conv matches
    the oracle, and it is bit-identical to the unmasked launch of the same
    geometry (every chunk enabled) -- skipped chunks add exact zeros."""
    ops = _ops()
    c = workloads.CONFIG2
    T, B, C, H, W = c["T"], c["B"], c["C"], c["H"], c["W"]
    x = workloads.block_sparse_spikes(T, B, C, H, W, sparsity, seed=31)
    _, w, scale, shift = _case(1, 1, C, C, 1, 1, 3, seed=32)
    xp = ops.pack_tbchw(x.to(dev))
    wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    nnz = torch.zeros(1, dtype=torch.int64, device=dev)
    mask = ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, nnz_out=nnz)
    assert int(nnz.item()) == int((x != 0).sum())
    geom = ops.conv_geometry(T, B, H, W, C, xp.shape[-1], 1, True)
    chunk = ops.conv_chunk(xp.shape[-1], True)
    m_o = _conv_tile_mask_oracle(xp.cpu().numpy(), geom, 3, 3, 1, 1, chunk)
    assert np.array_equal(mask.cpu().numpy().astype(np.int64) & 0xFFFFFFFF, m_o)
    sc, sh = scale.to(dev), shift.to(dev)
    sparse = ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, tile_mask=mask)
    full = torch.full_like(mask, -1)  # every chunk of every tile: same geometry, no skipping
    unmasked = ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, tile_mask=full)
    torch.cuda.synchronize()
    assert torch.equal(sparse, unmasked)
    s_o, _ = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, operand_dtype=torch.float16)
    sp = ops.unpack_bhwtc(sparse).cpu().numpy()
    assert (sp != s_o).mean() <= 1e-4
    if sparsity == 1.0:
        # StaticZero: z = shift everywhere
        s_z, _ = oracle.conv_bn_lif(torch.zeros_like(x), w, scale, shift, 1, 1)
        assert np.array_equal(sp, s_z)


def test_config0_exact(dev):
    """Config 0 exactly: T=4, B=32, 128->128, 32x32, Bernoulli(0.1) spikes,
    Kaiming weights, BN statistics of the stated distributions."""
    x, w, scale, shift = workloads.config0()
    s, v, _ = _run(dev, x, w, scale, shift, 1, 1)
    s_o, v_o, z = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, operand_dtype=torch.float16,
                                     return_z=True)
    _, _, h = lif_trace(z)
    check_lif_parity(s, v, s_o, v_o, h, v_tol=1e-4, near_tol=1e-3, max_flip_rate=1e-4,
                     what="config 0, fp16-operand oracle")
    s32, v32, z32 = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, return_z=True)
    _, _, h32 = lif_trace(z32)
    check_lif_parity(s, v, s32, v32, h32, v_tol=2e-2, near_tol=2e-2, max_flip_rate=1e-4,
                     what="config 0, fp32 oracle")
    # the extended-precision (split-weight) path meets the fp32 tolerance
    ss, vs, _ = _run(dev, x, w, scale, shift, 1, 1, precision="split")
    check_lif_parity(ss, vs, s32, v32, h32, v_tol=1e-4, near_tol=1e-4, max_flip_rate=1e-4,
                     what="config 0, split precision vs fp32 oracle")
    assert s32.mean() > 1e-3


SPLIT_SHAPES = [
    (4, 2, 64, 64, 8, 8, 3, 1, 1),          # pixel-major kernel
    (4, 2, 64, 32, 32, 32, 3, 1, 1),        # pixel-major, resident weights, halo box
    (4, 4, 128, 128, 16, 16, 3, 1, 1),      # channel-major, kh-box
    (4, 2, 64, 128, 16, 16, 3, 2, 1),       # channel-major, stride 2
    (4, 2, 64, 128, 16, 16, 1, 2, 0),       # 1x1 downsample
    (4, 2, 512, 512, 4, 4, 3, 1, 1),        # kw-group stages
    (12, 1, 32, 128, 5, 5, 3, 1, 1),        # chunked T
]


@pytest.mark.parametrize("shape", SPLIT_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_split_precision_vs_fp32(dev, shape):
    """Split (hi + lo) weights: fp32-faithful -- v within 1e-4 of the fp32
    oracle and flips only within 1e-4 of the threshold."""
    T, B, Cin, Cout, H, W, k, st, pad = shape
    x, w, scale, shift = _case(T, B, Cin, Cout, H, W, k, seed=hash(shape) % 997)
    s, v, _ = _run(dev, x, w, scale, shift, st, pad, precision="split")
    s32, v32, z32 = oracle.conv_bn_lif(x, w, scale, shift, st, pad, return_z=True)
    _, _, h32 = lif_trace(z32)
    check_lif_parity(s, v, s32, v32, h32, v_tol=1e-4, near_tol=1e-4, max_flip_rate=1e-4,
                     what=f"split vs fp32 {shape}")
    assert s.mean() > 0.005


def test_split_sparse_equals_split_dense_geometry(dev):
    """Split weights with a tile mask walk hi and lo chunks of the active
    activation chunks only; equal to the all-chunks launch bit for bit."""
    ops = _ops()
    T, B, C, H, W = 4, 4, 256, 14, 14
    x = workloads.block_sparse_spikes(T, B, C, H, W, 0.9, seed=41)
    _, w, scale, shift = _case(1, 1, C, C, 1, 1, 3, seed=42)
    xp = ops.pack_tbchw(x.to(dev))
    wp2, pre = ops.pack_conv_weight_split(w.to(dev), xp.shape[-1])
    sc = (scale / pre).to(dev)
    mask = ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1)
    a = ops.conv_bn_lif(xp, wp2, sc, shift.to(dev), 1, 1, tile_mask=mask, precision="split")
    b = ops.conv_bn_lif(xp, wp2, sc, shift.to(dev), 1, 1, tile_mask=torch.full_like(mask, -1),
                        precision="split")
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_split_weight_pack(dev):
    """hi + lo reproduces w * prescale to 22 bits; hi is fp16(w * prescale)."""
    ops = _ops()
    g = torch.Generator().manual_seed(5)
    w = torch.randn(32, 20, 3, 3, generator=g) * 0.05
    wp2, pre = ops.pack_conv_weight_split(w.to(dev), 32)
    wp2 = wp2.cpu().float().reshape(32, 3, 3, 2, 32)
    ref = (w * pre).permute(0, 2, 3, 1)
    assert torch.equal(wp2[..., 0, :20], ref.half().float())
    rec = wp2[..., 0, :20] + wp2[..., 1, :20]
    assert (rec - ref).abs().max() <= ref.abs().max() * 2.0 ** -21
    assert wp2[..., 20:].abs().max() == 0
    assert 2.0 ** 13 <= float((w * pre).abs().max()) < 2.0 ** 14


def test_conv_golden_reference(dev, golden_dir):
    """Reference outputs: the fp32 CPU per-step path and the StreamFuse
    Triton kernel (interpreter) on the same seeded inputs."""
    g = np.load(golden_dir / "golden_conv_bn_lif.npz")
    x = torch.from_numpy(g["x"].astype(np.float32))
    w = torch.from_numpy(g["weight"])
    scale, shift = oracle.fold_bn(g["gamma"], g["beta"], g["mean"], g["var"])
    s, v, _ = _run(dev, x, w, scale, shift, 1, 1)
    _, _, z32 = oracle.conv_bn_lif(x, w, scale, shift, 1, 1, return_z=True)
    _, _, h = lif_trace(z32)
    check_lif_parity(s, v, g["spikes"], g["vT"], h, v_tol=2e-2, near_tol=2e-2, max_flip_rate=1e-4,
                     what="golden fp32 reference path")
    check_lif_parity(s, v, g["sf_spikes"], g["sf_vT"], h, v_tol=2e-2, near_tol=2e-2,
                     max_flip_rate=1e-4, what="golden StreamFuse kernel")


@pytest.mark.parametrize("shape", [(4, 2, 3, 32, 32, 3, 1, 1, 32), (2, 3, 5, 9, 7, 3, 2, 1, 48),
                                   (1, 2, 2, 6, 6, 5, 1, 2, 64)])
def test_im2col_pack(dev, shape):
    """Stem im2col pack: y[b,ho,wo,t,q] = x[t,b,c,ho*s-p+kh,wo*s-p+kw], q = (kh*k+kw)*C+c,
    zero outside the image and for q >= k*k*C (exact: fp16 of the fp32 input)."""
    ops = _ops()
    T, B, C, H, W, k, s, p, Kp = shape
    g = torch.Generator().manual_seed(7)
    x = torch.randn(T, B, C, H, W, generator=g)
    y = ops.pack_im2col(x.to(dev), k, s, p, Kp).cpu()
    cols = torch.nn.functional.unfold(x.reshape(T * B, C, H, W), k, padding=p, stride=s)
    Ho = (H + 2 * p - k) // s + 1
    Wo = (W + 2 * p - k) // s + 1
    # unfold rows are (c, kh, kw); the pack orders q as (kh, kw, c)
    cols = cols.reshape(T, B, C, k * k, Ho, Wo).permute(1, 4, 5, 0, 3, 2).reshape(B, Ho, Wo, T, k * k * C)
    ref = torch.zeros(B, Ho, Wo, T, Kp)
    ref[..., :k * k * C] = cols
    assert torch.equal(y, ref.half())


@pytest.mark.parametrize("shape", [(4, 2, 3, 32, 32, 3, 1, 1), (2, 3, 3, 17, 13, 7, 2, 3)])
def test_im2col_split_stem(dev, shape):
    """Split stem: the im2col pack carries the real-valued input as hi + lo and
    the weight row [w, w] as hi + lo; the conv then meets the fp32 oracle at
    the fp32 tolerance."""
    ops = _ops()
    T, B, C, H, W, k, s_, p = shape
    g = torch.Generator().manual_seed(9)
    x = torch.randn(T, B, C, H, W, generator=g)
    y = ops.pack_im2col_split(x.to(dev), k, s_, p).cpu().float()
    KK = k * k * C
    hi = ops.pack_im2col(x.to(dev), k, s_, p, y.shape[-1]).cpu().float()
    assert torch.equal(y[..., :KK], hi[..., :KK])
    # hi + lo reproduces the fp32 input to 22 bits
    Ho_ = (H + 2 * p - k) // s_ + 1
    Wo_ = (W + 2 * p - k) // s_ + 1
    cols = torch.nn.functional.unfold(x.reshape(T * B, C, H, W), k, padding=p, stride=s_)
    cols = cols.reshape(T, B, C, k * k, Ho_, Wo_).permute(1, 4, 5, 0, 3, 2).reshape(B, Ho_, Wo_, T, KK)
    err = (y[..., :KK] + y[..., KK:2 * KK] - cols).abs()
    assert (err <= cols.abs() * 2.0 ** -21 + 2.0 ** -24).all()
    Cout = 64
    w = torch.randn(Cout, C, k, k, generator=g) * (2.0 / KK) ** 0.5
    scale = torch.rand(Cout, generator=g) * 0.4 + 0.8
    shift = torch.randn(Cout, generator=g) * 0.3
    wp2, pre = ops.im2col_weight_split(w.to(dev), y.shape[-1])
    yd = ops.pack_im2col_split(x.to(dev), k, s_, p, y.shape[-1])
    Bq, Ho, Wo = yd.shape[0], yd.shape[1], yd.shape[2]
    v = torch.empty(Bq, Ho, Wo, Cout, device=dev)
    out = ops.conv_bn_lif(yd, wp2, (scale / pre).to(dev), shift.to(dev), 1, 0, v_out=v,
                          precision="split")
    sg = ops.unpack_bhwtc(out).cpu().numpy()
    vg = ops.v_to_nchw(v).cpu().numpy()
    s32, v32, z32 = oracle.conv_bn_lif(x, w, scale, shift, s_, p, return_z=True)
    _, _, h32 = lif_trace(z32)
    check_lif_parity(sg, vg, s32, v32, h32, v_tol=1e-4, near_tol=1e-4, max_flip_rate=1e-4,
                     what=f"split stem {shape}")


PLANE_SHAPES = [
    # B, Cin, Cout, H, W, k, stride, pad
    (8, 64, 64, 32, 32, 3, 1, 1),      # M=64 channel-major tiles
    (8, 128, 128, 16, 16, 3, 1, 1),    # kh-box stages
    (4, 512, 512, 4, 4, 3, 1, 1),      # kw-group stages, K = 4608
    (4, 64, 128, 16, 16, 3, 2, 1),     # stride 2
    (4, 64, 128, 16, 16, 1, 2, 0),     # 1x1 downsample
    (3, 96, 256, 9, 7, 3, 1, 1),       # ragged tiles, Cin_p not a multiple of 64
]


@pytest.mark.parametrize("shape", PLANE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_planes_exact_accumulation(dev, shape):
    """Integer weight planes: the convolution equals the fp64 convolution with
    the quantised weight q / prescale, rounded once to fp32 -- bit for bit.
    Read through the membrane: T=1, v0=0, no spikes, so v = z / 2 exactly."""
    ops = _ops()
    B, Cin, Cout, H, W, k, st, pad = shape
    g = torch.Generator().manual_seed(sum(shape))
    x = ((torch.rand(1, B, Cin, H, W, generator=g) < 0.3).float()
         + (torch.rand(1, B, Cin, H, W, generator=g) < 0.2).float())   # counts {0,1,2}
    w = torch.randn(Cout, Cin, k, k, generator=g) * (2.0 / (Cin * k * k)) ** 0.5
    xp = ops.pack_tbchw(x.to(dev))
    wq, pre = ops.pack_conv_weight_planes(w.to(dev), xp.shape[-1])
    # the planes reproduce q = rint(w * prescale) exactly
    planes = wq.cpu().double().reshape(Cout, k, k, 3, -1)[..., :Cin]
    q = planes[..., 0, :] * 2.0 ** 20 + planes[..., 1, :] * 2.0 ** 10 + planes[..., 2, :]
    assert torch.equal(q, torch.round((w.double() * pre)).permute(0, 2, 3, 1))
    assert planes.abs().max() <= 512
    Ho = (H + 2 * pad - k) // st + 1
    Wo = (W + 2 * pad - k) // st + 1
    v = torch.empty(B, Ho, Wo, Cout, device=dev)
    lif = ops.LIFConfig(2.0, 1e30, 0.0, True)
    sc = torch.full((Cout,), 1.0 / pre, device=dev)
    ops.conv_bn_lif(xp, wq, sc, torch.zeros(Cout, device=dev), st, pad, v_out=v, lif=lif,
                    precision="planes")
    z = (ops.v_to_nchw(v).cpu() * 2).double()
    qw = q.permute(0, 3, 1, 2) / pre
    z64 = torch.nn.functional.conv2d(x[0].double(), qw, stride=st, padding=pad)
    assert torch.equal(z, z64.float().double())


@pytest.mark.parametrize("shape", [(4, 4, 128, 128, 16, 16, 3, 1, 1), (4, 2, 64, 64, 32, 32, 3, 1, 1),
                                   (12, 1, 64, 128, 6, 6, 3, 1, 1)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("mode", ["none", "add", "add_pre"])
def test_conv_planes_vs_fp32_oracle(dev, shape, mode):
    """Full Conv->BN->LIF in the plane mode (residual modes, chunked T) at the
    fp32 tolerance: v within 1e-4, flips only within 1e-5 of the threshold."""
    ops = _ops()
    T, B, Cin, Cout, H, W, k, st, pad = shape
    x, w, scale, shift = _case(T, B, Cin, Cout, H, W, k, seed=sum(shape) + len(mode))
    g = torch.Generator().manual_seed(3)
    xp = ops.pack_tbchw(x.to(dev))
    wq, pre = ops.pack_conv_weight_planes(w.to(dev), xp.shape[-1])
    kw = {}
    ident = None
    if mode != "none":
        ident = (torch.rand(T, B, Cout, H, W, generator=g) < 0.3).float()
        kw = dict(identity=ops.pack_tbchw(ident.to(dev)), res_mode=mode)
    v = torch.empty(B, H, W, Cout, device=dev)
    out = ops.conv_bn_lif(xp, wq, (scale / pre).to(dev), shift.to(dev), st, pad, v_out=v,
                          precision="planes", **kw)
    got = ops.unpack_bhwtc(out).cpu().numpy()
    vg = ops.v_to_nchw(v).cpu().numpy()
    if mode == "none":
        s32, v32, z32 = oracle.conv_bn_lif(x, w, scale, shift, st, pad, return_z=True)
        ref = s32
    else:
        ref, v32 = oracle.conv_bn_lif_residual(x, w, scale, shift, ident, mode, st, pad)
        z32 = oracle.conv.conv_z(x, w, scale, shift, st, pad).numpy()
        if mode == "add_pre":
            z32 = (z32 + ident.numpy()).astype(np.float32)
        got = got - ident.numpy() if mode == "add" else got
        ref = ref - ident.numpy() if mode == "add" else ref
    _, _, h32 = lif_trace(z32)
    check_lif_parity(got, vg, ref, v32, h32, v_tol=1e-4, near_tol=1e-5, max_flip_rate=1e-4,
                     what=f"planes {mode} {shape}")


@pytest.mark.parametrize("sparsity", [0.0, 0.9, 0.99, 1.0])
def test_device_egd_dispatch_bit_identical(dev, sparsity):
    """Device-side EGD: whatever the kernel decides (masks or dense), the
    result equals the plain masked launch and the dense launch of the same
    geometry bit for bit, at thresholds that force either choice."""
    ops = _ops()
    T, B, C, H, W = 4, 8, 256, 28, 28
    x = workloads.block_sparse_spikes(T, B, C, H, W, sparsity, seed=51)
    _, w, scale, shift = _case(1, 1, C, C, 1, 1, 3, seed=52)
    xp = ops.pack_tbchw(x.to(dev))
    wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    sc, sh = scale.to(dev), shift.to(dev)
    mask = ops.prescan_conv_tiles(xp, C, 3, 3, 1, 1, egd=True)   # dense-chunk masks
    ref = ops.conv_bn_lif(xp, wp, sc, sh, 1, 1)                  # dense launch, same chunk
    for frac in (0.0, 0.3, 1.0):
        got = ops.conv_bn_lif(xp, wp, sc, sh, 1, 1, tile_mask=mask, egd_max_active_frac=frac)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), frac
    # the masks of the dense chunk match the oracle
    geom = ops.conv_geometry(T, B, H, W, C, xp.shape[-1], 1, True)
    m_o = _conv_tile_mask_oracle(xp.cpu().numpy(), geom, 3, 3, 1, 1, ops.conv_chunk(xp.shape[-1], False))
    assert np.array_equal(mask.cpu().numpy().astype(np.int64) & 0xFFFFFFFF, m_o)
