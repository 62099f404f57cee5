"""The bounded-wait expiry path of the fused conv kernel, exercised without a
GPU fault: a test hook makes CTA 0's producers skip their first load, so the
consumer's wait for it can never complete; with a short wait limit it gives
up, records its site in the device error word and the kernel ends early.
The host then reads CF_ERR_DEVICE_TIMEOUT, the word is cleared, and the next
normal launch on the same context is correct."""
import pytest
import torch

from catfuse_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _inputs(dev, C):
    g = torch.Generator().manual_seed(77)
    x = (torch.rand(4, 2, C, 16, 16, generator=g) < 0.3).float()
    w = torch.randn(C, C, 3, 3, generator=g) * (2.0 / (C * 9)) ** 0.5 * 1.5
    xp = ops.pack_tbchw(x.to(dev))
    wp = ops.pack_conv_weight(w.to(dev), xp.shape[-1])
    scale = (torch.rand(C, generator=g) * 0.4 + 0.8).to(dev)
    shift = (torch.randn(C, generator=g) * 0.3).to(dev)
    return xp, wp, scale, shift


@pytest.mark.parametrize("C", [32, 128])   # pixel-major and channel-major kernels
def test_wait_expiry_reports_timeout_and_recovers(dev, C):
    lib = _lib.load()
    xp, wp, scale, shift = _inputs(dev, C)
    ref = ops.conv_bn_lif(xp, wp, scale, shift, 1, 1)
    ops.check_device_error()            # clean before the test
    try:
        ops.set_wait_limit(1 << 12)
        assert lib.cf_test_arm_stalled_load(1) == _lib.CF_OK
        ops.conv_bn_lif(xp, wp, scale, shift, 1, 1)   # the launch itself succeeds
        with pytest.raises(_lib.CatfuseNativeError) as err:
            ops.check_device_error()
        assert err.value.code == _lib.CF_ERR_DEVICE_TIMEOUT
        assert "site" in str(err.value)
    finally:
        lib.cf_test_arm_stalled_load(0)
        ops.set_wait_limit(0)
    ops.check_device_error()            # the read cleared the word
    again = ops.conv_bn_lif(xp, wp, scale, shift, 1, 1)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)
    ops.check_device_error()
