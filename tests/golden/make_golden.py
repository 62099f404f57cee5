"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the reference checkout (read-only) and Triton:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref /path/to/CATFuse

The reference needs SpikingJelly only for a base class at import time; a
throw-away stub package providing ``spikingjelly.activation_based.base.
MemoryModule`` (an ``nn.Module``) and an empty ``neuron.LIFNode`` is written to
a temporary directory and put on ``sys.path`` for the duration of this script.
Triton kernels run on CPU tensors under ``TRITON_INTERPRET=1``; autotuned
kernels are called through ``.fn`` with an explicit config.

Every case uses seeded generators so the fixtures are reproducible.  Output:
``golden_<name>.npz`` files next to this script, each holding inputs and the
reference outputs.  The script never writes anywhere else.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

_SJ_STUB = {
    "spikingjelly/__init__.py": "",
    "spikingjelly/activation_based/__init__.py": "",
    "spikingjelly/activation_based/base.py": (
        "import torch.nn as nn\n"
        "class MemoryModule(nn.Module):\n"
        "    def __init__(self):\n"
        "        super().__init__()\n"
        "        self.step_mode = 's'\n"
        "    def reset(self):\n"
        "        pass\n"
    ),
    "spikingjelly/activation_based/neuron.py": "class LIFNode:\n    pass\n",
    "spikingjelly/activation_based/functional.py": "",
}


def _install_stub() -> str:
    d = tempfile.mkdtemp(prefix="sjstub_")
    for rel, src in _SJ_STUB.items():
        p = Path(d) / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(src)
    sys.path.insert(0, d)
    return d


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def bernoulli(shape, p, seed):
    return (torch.rand(shape, generator=_gen(seed)) < p).float()


def block_sparse(T, B, C, H, W, block_hw, block_c, s_zero, p_in, seed):
    """Block-structured spikes: each (block_hw x block_hw x block_c) block is
    all-zero with probability s_zero, else Bernoulli(p_in) inside."""
    g = _gen(seed)
    nb_h, nb_w, nb_c = -(-H // block_hw), -(-W // block_hw), -(-C // block_c)
    keep = (torch.rand((T, B, nb_c, nb_h, nb_w), generator=g) >= s_zero).float()
    keep = keep.repeat_interleave(block_c, 2).repeat_interleave(block_hw, 3).repeat_interleave(block_hw, 4)
    keep = keep[:, :, :C, :H, :W]
    inner = (torch.rand((T, B, C, H, W), generator=g) < p_in).float()
    return keep * inner


def bn_params(C, seed):
    g = _gen(seed)
    mean = torch.randn(C, generator=g) * 0.1
    var = torch.rand(C, generator=g) + 0.5
    gamma = torch.rand(C, generator=g) * 0.4 + 0.8
    beta = torch.randn(C, generator=g) * 0.1
    return gamma, beta, mean, var


def kaiming(shape, seed):
    g = _gen(seed)
    fan_in = shape[1] * shape[2] * shape[3]
    return torch.randn(shape, generator=g) * (2.0 / fan_in) ** 0.5


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    _install_stub()
    sys.path.insert(0, args.ref)

    from catfuse.sparseflow.lif_seq_kernel import lif_sequential
    from catfuse.sparseflow.fast_prescan_v2 import fast_spike_prescan_2d_v2
    from catfuse.sparseflow.prescan import build_rf_prescan_metadata
    from catfuse.sparseflow.sparse_conv2d_kernel import choose_group_size, _select_tile_sizes
    from catfuse.sparseflow.streamfuse_kernel import sparse_streamfuse_conv3x3_bn_lif
    from catfuse.sparseflow.ops.st_fusion_conv_bn_lif import STFusionConvBNLIF, _fold_bn_params
    from catfuse.kernels.partial_fusion_conv_bn_lif_impl import _bn_lif_state_carry_kernel
    import torch.nn as nn

    class _LIF:  # attribute holder read by from_sj_modules
        tau, v_threshold, v_reset, decay_input = 2.0, 1.0, 0.0, True

    # ---- 1. multi-step LIF (Triton lif_sequential, interpreter) -------------
    T, shape = 6, (2, 8, 5, 7)
    z = torch.randn((T,) + shape, generator=_gen(100)) * 0.8 + 0.3
    v0 = torch.randn(shape, generator=_gen(101)) * 0.5
    s, vT = lif_sequential(z, v0, tau=2.0, v_threshold=1.0, v_reset=0.0)
    # tau = 3 exercises the true-division path
    s3, vT3 = lif_sequential(z, v0, tau=3.0, v_threshold=1.0, v_reset=0.0)
    np.savez_compressed(HERE / "golden_lif.npz", z=z.numpy(), v0=v0.numpy(),
                        spikes=s.numpy(), vT=vT.numpy(), spikes_tau3=s3.numpy(), vT_tau3=vT3.numpy())

    # ---- 2. BN + LIF state-carry kernel (partial fusion, interpreter) --------
    Tb, Bb, Cb, Hb, Wb = 4, 2, 16, 6, 6
    zb = torch.randn((Tb, Bb, Cb, Hb, Wb), generator=_gen(200)) * 1.2
    gamma, beta, mean, var = bn_params(Cb, 201)
    inv_std = torch.rsqrt(var + 1e-5)
    scale = (gamma * inv_std).contiguous()
    shift = (beta - mean * scale).contiguous()
    sb = torch.empty_like(zb)
    N = Bb * Cb * Hb * Wb
    _bn_lif_state_carry_kernel[(-(-N // 1024),)](
        zb, sb, scale, shift, Tb, N, Cb, Hb * Wb, 1.0 / 2.0, 1.0 - 1.0 / 2.0, 1.0, BLOCK_N=1024)
    np.savez_compressed(HERE / "golden_bn_lif.npz", z=zb.numpy(), scale=scale.numpy(),
                        shift=shift.numpy(), spikes=sb.numpy())

    # ---- 3. prescan: torch cascade and Triton v2 -----------------------------
    cases = []
    for (Np, C, H, W, k, st, p, seed, sparsity) in [
        (4, 64, 14, 14, 3, 1, 1, 300, 0.97),
        (3, 256, 28, 28, 3, 1, 1, 301, 0.99),
        (2, 96, 17, 13, 3, 2, 1, 302, 0.9),
        (2, 512, 7, 7, 1, 1, 0, 303, 0.95),
        (2, 64, 12, 12, 3, 1, 1, 304, 1.0),
        (2, 128, 20, 20, 3, 1, 1, 305, 0.9),
        (2, 32, 10, 10, 3, 1, 1, 306, 0.3),
    ]:
        x = block_sparse(1, Np, C, H, W, 4, 16, sparsity, 0.3, seed)[0]
        Ho = (H + 2 * p - k) // st + 1
        Wo = (W + 2 * p - k) // st + 1
        BH, BW = _select_tile_sizes(Ho, Wo)
        GS = choose_group_size(C)
        G = -(-C // GS)
        tc, ag = build_rf_prescan_metadata(
            x.permute(0, 2, 3, 1), (Ho, Wo), (k, k), st, p, (BH, BW), GS, G, 1e-6)
        entry = dict(x=x.numpy().astype(np.uint8), k=k, s=st, p=p, BH=BH, BW=BW, GS=GS,
                     Ho=Ho, Wo=Wo, ag_mask=ag.numpy(), tile_class=tc.numpy())
        if st == 1:
            tc2, ag2 = fast_spike_prescan_2d_v2(x, Ho, Wo, kernel_size=k, stride=st, padding=p,
                                                block_h=BH, block_w=BW, group_size_c=GS)
            entry["ag_mask_v2"] = ag2.numpy()
            entry["tile_class_v2"] = tc2.numpy()
        cases.append(entry)
    flat = {}
    for i, e in enumerate(cases):
        for key, val in e.items():
            flat[f"c{i}_{key}"] = np.asarray(val)
    flat["n_cases"] = np.asarray(len(cases))
    np.savez_compressed(HERE / "golden_prescan.npz", **flat)

    # ---- 4. Conv3x3 -> BN -> LIF ---------------------------------------------
    # (a) the reference's own fp32 CPU path (STFusionConvBNLIF's pure-PyTorch
    #     per-step fallback, SpikingJelly charge form), v carried over T;
    # (b) the fused StreamFuse Triton kernel under the interpreter (fp16
    #     operands, fp32 accumulation, Triton LIF form).
    T4, B4, Ci, Co, H4, W4 = 3, 2, 32, 64, 8, 8
    x4 = bernoulli((T4, B4, Ci, H4, W4), 0.5, 400)
    conv = nn.Conv2d(Ci, Co, 3, 1, 1, bias=False)
    with torch.no_grad():
        conv.weight.copy_(kaiming((Co, Ci, 3, 3), 401))
    bn = nn.BatchNorm2d(Co)
    g4, b4, m4, v4 = bn_params(Co, 402)
    with torch.no_grad():
        bn.weight.copy_(g4); bn.bias.copy_(b4)
        bn.running_mean.copy_(m4); bn.running_var.copy_(v4)
    bn.eval()
    mod = STFusionConvBNLIF.from_sj_modules(conv, bn, _LIF(), K=T4)
    v = torch.zeros(B4, Co, H4, W4)
    outs = []
    with torch.no_grad():
        for t in range(T4):
            sp, v = mod._fallback_forward_single(x4[t], v)
            outs.append(sp)
    ref_spikes = torch.stack(outs)
    ref_vT = v.clone()
    # StreamFuse kernel
    scale4, shift4 = _fold_bn_params(bn)
    w_cl = conv.weight.detach().half().permute(0, 2, 3, 1).contiguous()
    GH = -(-H4 // 8); GW = -(-W4 // 16)
    sf_spikes = torch.empty(T4 * B4, Co, H4, W4)
    sf_vT = torch.empty(B4, Co, H4, W4)
    dummy = torch.empty(1)
    GSC = choose_group_size(Ci)
    sparse_streamfuse_conv3x3_bn_lif.fn[(B4 * GH * GW, -(-Co // 64))](
        x4.reshape(T4 * B4, Ci, H4, W4).contiguous(), w_cl, dummy,
        scale4.float().contiguous(), shift4.float().contiguous(),
        torch.zeros(B4, Co, H4, W4), sf_spikes, sf_vT, T4, B4,
        C_IN=Ci, C_OUT=Co, H=H4, W=W4, H_OUT=H4, W_OUT=W4, GH=GH, GW=GW,
        HAS_BIAS=False, HAS_BN=True, DECAY=0.5, RECIP_TAU=0.5, V_TH=1.0,
        HAS_V_RESET=True, V_RESET=0.0, GROUP_SIZE_C=GSC, NUM_GROUPS=-(-Ci // GSC), BLOCK_N=64)
    np.savez_compressed(
        HERE / "golden_conv_bn_lif.npz", x=x4.numpy().astype(np.uint8),
        weight=conv.weight.detach().numpy(), gamma=g4.numpy(), beta=b4.numpy(),
        mean=m4.numpy(), var=v4.numpy(), spikes=ref_spikes.numpy(), vT=ref_vT.numpy(),
        sf_spikes=sf_spikes.reshape(T4, B4, Co, H4, W4).numpy(), sf_vT=sf_vT.numpy())
    print("wrote:", sorted(p.name for p in HERE.glob("golden_*.npz")))


if __name__ == "__main__":
    main()
