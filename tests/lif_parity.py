"""Parity helpers shared by the tests: spike/membrane comparison with the
tolerances of the north-star contract (v within v_tol; spike flips at most
max_flip_rate of the elements and only where the reference membrane is within
near_tol of the threshold)."""
from __future__ import annotations

import numpy as np


def lif_trace(z, v0=None, tau=2.0, vth=1.0, vr=0.0, hard=True, decay_input=True):
    """Oracle LIF that also returns the pre-fire membrane h[t]."""
    z = np.asarray(z, np.float32)
    f32 = np.float32
    v = np.zeros(z.shape[1:], f32) if v0 is None else np.array(v0, f32, copy=True)
    hs = np.empty_like(z)
    ss = np.empty_like(z)
    for t in range(z.shape[0]):
        if decay_input:
            h = (v + (z[t] - (v - f32(vr))) / f32(tau)).astype(f32)
        else:
            h = ((v - (v - f32(vr)) / f32(tau)) + z[t]).astype(f32)
        s = h >= f32(vth)
        v = np.where(s, f32(vr), h).astype(f32) if hard else np.where(s, h - f32(vth), h).astype(f32)
        hs[t] = h
        ss[t] = s
    return ss, v, hs


def check_lif_parity(s_got, v_got, s_ref, v_ref, h_ref, vth=1.0, v_tol=1e-4, near_tol=1e-3,
                     max_flip_rate=1e-4, what=""):
    s_got = np.asarray(s_got, np.float32)
    s_ref = np.asarray(s_ref, np.float32)
    T = s_ref.shape[0]
    mism = s_got != s_ref                                   # [T, ...]
    n = s_ref.size
    rate = mism.sum() / max(n, 1)
    assert rate <= max_flip_rate, f"{what}: spike flip rate {rate:.3e} > {max_flip_rate:.1e}"
    # the first mismatch of every neuron must sit near the threshold
    any_m = mism.any(axis=0)
    if any_m.any():
        first = np.argmax(mism, axis=0)
        idx = np.nonzero(any_m)
        h_at = h_ref[(first[idx],) + idx]
        far = np.abs(h_at - vth) >= near_tol
        assert not far.any(), (f"{what}: {int(far.sum())} flips away from threshold, "
                               f"max |h-vth| = {np.abs(h_at - vth).max():.3e}")
    if v_got is not None:
        ok = ~any_m
        dv = np.abs(np.asarray(v_got, np.float32) - np.asarray(v_ref, np.float32))[ok]
        if dv.size:
            assert dv.max() <= v_tol, f"{what}: max |dv| = {dv.max():.3e} > {v_tol}"
    return rate
