"""cf_prescan (the reference-geometry receptive-field prescan) against the
fixtures produced by the reference's own prescan code and against the numpy
oracle at the config-2 shape; masks, tile classes and nnz must be bit-exact.
Mirrors the reference's tests/test_11_fast_prescan.py:30-41,90-95
(Triton masks == torch masks, bit for bit)."""
import numpy as np
import pytest
import torch

import oracle
from catfuse_b200 import ops, workloads

pytestmark = pytest.mark.gpu


def _cases(golden_dir):
    g = np.load(golden_dir / "golden_prescan.npz")
    for i in range(int(g["n_cases"])):
        yield i, {k[len(f"c{i}_"):]: g[k] for k in g.files if k.startswith(f"c{i}_")}


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.uint8])
def test_prescan_vs_reference_golden(dev, golden_dir, dtype):
    n = 0
    for i, c in _cases(golden_dir):
        x = torch.from_numpy(c["x"].astype(np.float32))
        if dtype == torch.uint8 and not torch.all((x == 0) | (x == 1)):
            continue  # u8 holds spikes only
        ag, cls, nnz = ops.prescan(x.to(dtype).to(dev), int(c["k"]), int(c["s"]), int(c["p"]),
                                   int(c["BH"]), int(c["BW"]), int(c["GS"]))
        torch.cuda.synchronize()
        assert np.array_equal(ag.cpu().numpy(), c["ag_mask"]), f"case {i} ag_mask"
        assert np.array_equal(cls.cpu().numpy(), c["tile_class"]), f"case {i} tile_class"
        assert int(nnz.item()) == int(np.count_nonzero(c["x"])), f"case {i} nnz"
        if "ag_mask_v2" in c:  # the reference's Triton prescan v2 agrees too
            assert np.array_equal(ag.cpu().numpy(), c["ag_mask_v2"])
        n += 1
    assert n >= 5


@pytest.mark.parametrize("s", workloads.CONFIG2["sparsities"])
def test_prescan_config2_vs_oracle(dev, s):
    c = workloads.CONFIG2
    T, B, C, H, W = c["T"], c["B"], c["C"], c["H"], c["W"]
    x = workloads.block_sparse_spikes(T, B, C, H, W, s, seed=7)
    xn = x.reshape(T * B, C, H, W)
    GS = oracle.choose_group_size(C)
    BH, BW = oracle.select_tile_sizes(H, W)
    ag_o, cls_o, nnz_o = oracle.prescan_rf(xn.numpy(), 3, 1, 1, BH, BW, GS)
    for dtype in (torch.float32, torch.float16, torch.uint8):
        ag, cls, nnz = ops.prescan(xn.to(dtype).to(dev).contiguous(), 3, 1, 1, BH, BW, GS)
        torch.cuda.synchronize()
        assert np.array_equal(ag.cpu().numpy(), ag_o), (s, dtype)
        assert np.array_equal(cls.cpu().numpy(), cls_o), (s, dtype)
        assert int(nnz.item()) == nnz_o
    if s == 1.0:
        assert (cls_o == 0).all() and nnz_o == 0


def test_prescan_edge_shapes(dev):
    """Ragged maps (tiles hanging over the edge), stride 2, k=1, a single
    channel group, an all-zero input and an all-ones input."""
    g = torch.Generator().manual_seed(3)
    cases = [((3, 48, 9, 11), 3, 1, 1), ((2, 96, 15, 15), 3, 2, 1), ((2, 64, 10, 10), 1, 1, 0),
             ((1, 16, 8, 8), 3, 1, 1), ((2, 256, 7, 7), 3, 1, 1)]
    for shape, k, s, p in cases:
        N, C, H, W = shape
        for fill in ("rand", "zero", "ones"):
            if fill == "rand":
                x = (torch.rand(shape, generator=g) < 0.02).float()
            elif fill == "zero":
                x = torch.zeros(shape)
            else:
                x = torch.ones(shape)
            Ho = (H + 2 * p - k) // s + 1
            Wo = (W + 2 * p - k) // s + 1
            GS = oracle.choose_group_size(C)
            BH, BW = oracle.select_tile_sizes(Ho, Wo)
            ag_o, cls_o, nnz_o = oracle.prescan_rf(x.numpy(), k, s, p, BH, BW, GS)
            ag, cls, nnz = ops.prescan(x.to(dev), k, s, p, BH, BW, GS)
            torch.cuda.synchronize()
            assert np.array_equal(ag.cpu().numpy(), ag_o), (shape, fill)
            assert np.array_equal(cls.cpu().numpy(), cls_o), (shape, fill)
            assert int(nnz.item()) == nnz_o
