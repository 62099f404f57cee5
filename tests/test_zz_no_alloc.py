"""cf_conv_bn_lif_egd_noalloc: the SparseFlow conv for callers that cannot
allocate device memory (a host framework whose allocator owns the GPU and
hands the library only the tensors of a call).  Its tile masks live in a
fixed array inside the library, so the caller passes only inputs and outputs.

Checked through the C ABI against the allocating path (cf_prescan_conv_tiles
into a caller-owned mask, then cf_conv_bn_lif_egd): bit-identical spikes and
membranes on two calls in a row with different inputs, so the second call
cannot lean on masks the first one left behind.  Also checks that a shape
needing more masks than the fixed array holds is refused.  Kept in its own
file, collected last."""
import pytest
import torch

from catfuse_b200 import workloads

pytestmark = pytest.mark.gpu


def _inputs(dev, sparsity, seed, T=4, B=8, C=128, H=28, W=28):
    from catfuse_b200 import ops
    g = torch.Generator().manual_seed(seed)
    x = workloads.block_sparse_spikes(T, B, C, H, W, sparsity, seed=seed)
    w = torch.randn(C, C, 3, 3, generator=g) * (2.0 / (C * 9)) ** 0.5 * 1.5
    scale = (torch.rand(C, generator=g) * 0.4 + 0.8).to(dev)
    shift = (torch.randn(C, generator=g) * 0.3).to(dev)
    xp = ops.pack_tbchw(x.to(dev))
    wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    v0 = (torch.rand(B, H, W, C, generator=g) * 0.5).to(dev)
    return xp, wp, scale, shift, v0


def _noalloc(xp, wp, scale, shift, v0, frac):
    from catfuse_b200 import _lib, ops
    B, H, W, T, Cin_p = xp.shape
    Cout = wp.shape[0]
    out = torch.empty(B, H, W, T, Cout, dtype=torch.float16, device=xp.device)
    v_out = torch.empty(B, H, W, Cout, dtype=torch.float32, device=xp.device)
    _lib.call("cf_conv_bn_lif_egd_noalloc", xp.data_ptr(), wp.data_ptr(), scale.data_ptr(),
              shift.data_ptr(), None, 0, v0.data_ptr(), v_out.data_ptr(), out.data_ptr(),
              T, B, H, W, Cin_p, Cout, 3, 3, 1, 1, *ops.LIFConfig().args(), float(frac),
              ops._stream())
    return out, v_out


def _allocating(xp, wp, scale, shift, v0, frac):
    from catfuse_b200 import ops
    Cout = wp.shape[0]
    mask = ops.prescan_conv_tiles(xp, Cout, 3, 3, 1, 1, egd=True)
    v_out = torch.empty_like(v0)
    out = ops.conv_bn_lif(xp, wp, scale, shift, 1, 1, v_in=v0, v_out=v_out, tile_mask=mask,
                          egd_max_active_frac=frac)
    return out, v_out


@pytest.mark.parametrize("frac", [0.0, 0.5, 1.0])
def test_noalloc_matches_allocating_path_twice(dev, frac):
    # two different inputs back to back: the denser one first, so stale masks
    # from call 1 would wrongly enable chunks in call 2 if they survived
    for sparsity, seed in ((0.8, 71), (0.99, 72)):
        args = _inputs(dev, sparsity, seed)
        got, vg = _noalloc(*args, frac)
        ref, vr = _allocating(*args, frac)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (frac, sparsity)
        assert torch.equal(vg, vr), (frac, sparsity)


def test_noalloc_refuses_shapes_beyond_the_fixed_array(dev):
    from catfuse_b200 import _lib, ops
    # 64 x 512 x 512 output pixels x 4 steps needs far more than 65536 M tiles;
    # the size check runs before any pointer is touched
    lib = _lib.load()
    rc = lib.cf_conv_bn_lif_egd_noalloc(16, 16, None, None, None, 0, None, None, 16,
                                        4, 64, 512, 512, 128, 128, 3, 3, 1, 1,
                                        *ops.LIFConfig().args(), 0.5, None)
    assert rc == _lib.CF_ERR_UNSUPPORTED
    assert "fixed mask array" in _lib.last_error()
