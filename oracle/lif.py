"""Multi-step LIF restatement (numpy fp32, one rounding per operation).

Follows:
* the SpikingJelly charge/fire/reset form the reference documents as
  bit-exact to SJ (``tests/check_lif_parity.py:16-22``,
  ``catfuse/implementations/dense_keep.py:143-155``,
  ``catfuse/sparseflow/ops/st_fusion_conv_bn_lif.py:425-445`` for the
  soft-reset and ``decay_input=False`` forms);
* the Triton kernel form ``v*decay + z/tau + v_reset/tau``
  (``catfuse/sparseflow/lif_seq_kernel.py:37-43``) for cross-checks of the
  reference's own kernel outputs.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def lif_multistep(z, v0=None, tau=2.0, v_threshold=1.0, v_reset=0.0,
                  hard_reset=True, decay_input=True):
    """z: [T, ...] -> (spikes [T, ...] fp32 in {0,1}, v_T [...] fp32).

    ``v_reset=None`` (or hard_reset=False) selects the soft reset
    ``v -= s * v_threshold`` and charges as if v_reset were 0.
    """
    z = np.asarray(z, dtype=f32)
    soft = (v_reset is None) or (not hard_reset)
    vr = f32(0.0 if soft else v_reset)
    tau = f32(tau)
    vth = f32(v_threshold)
    v = np.zeros(z.shape[1:], f32) if v0 is None else np.array(v0, dtype=f32, copy=True)
    out = np.empty_like(z)
    for t in range(z.shape[0]):
        if decay_input:
            h = (v + (z[t] - (v - vr)) / tau).astype(f32)
        else:
            h = ((v - (v - vr) / tau) + z[t]).astype(f32)
        s = h >= vth
        if soft:
            v = np.where(s, (h - vth).astype(f32), h).astype(f32)
        else:
            v = np.where(s, vr, h).astype(f32)
        out[t] = s
    return out, v


def lif_multistep_triton_form(z, v0=None, tau=2.0, v_threshold=1.0, v_reset=0.0):
    """The reference Triton kernel's arithmetic (hard reset):
    v = v*(1-1/tau) + z*(1/tau) + v_reset*(1/tau)."""
    z = np.asarray(z, dtype=f32)
    decay = f32(1.0 - 1.0 / tau)
    rt = f32(1.0 / tau)
    vr = f32(v_reset)
    v = np.zeros(z.shape[1:], f32) if v0 is None else np.array(v0, dtype=f32, copy=True)
    out = np.empty_like(z)
    for t in range(z.shape[0]):
        v = ((v * decay + z[t] * rt).astype(f32) + vr * rt).astype(f32)
        s = v >= f32(v_threshold)
        v = np.where(s, vr, v).astype(f32)
        out[t] = s
    return out, v
