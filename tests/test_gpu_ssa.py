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
