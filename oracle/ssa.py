"""Spiking self-attention (Spikformer SSA core) restatement — test
infrastructure only (checker for the CUDA path, never shipped or measured).

Follows SSA.forward of the reference (models/spikformer_github.py:147-153):
per head ``attn = (q @ k^T) * scale``, ``y = attn @ v``, heads merged, then
``attn_lif`` (SpikingJelly multi-step LIF, oracle/lif.py).

Two arithmetic forms:
* ``exact``: q, k, v are {0,1}, so (q @ k^T) @ v is an integer matrix; y is
  that integer times scale rounded once to fp32 (float64 product of an
  integer <= 2^11 and an fp32 scale is exact) — the form the kernel computes;
* ``reference``: the reference's order in fp32 torch (attn rounded, then a
  float32 matmul), for a tolerance-based cross-check.
"""
from __future__ import annotations

import numpy as np
import torch

from .lif import lif_multistep


def ssa_lif(q, k, v, heads, scale=None, v0=None, form="exact", tau=2.0, v_threshold=1.0,
            v_reset=0.0, hard_reset=True, decay_input=True):
    """q, k, v: [T, B, N, C] {0,1} -> (spikes [T,B,N,C] fp32, v_T [B,N,C], y [T,B,N,C])."""
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32); v = np.asarray(v, np.float32)
    T, B, N, C = q.shape
    d = C // heads
    scale = np.float32(d ** -0.5 if scale is None else scale)

    def split(x):  # [T,B,N,C] -> [T,B,h,N,d]
        return x.reshape(T, B, N, heads, d).transpose(0, 1, 3, 2, 4)

    qh, kh, vh = split(q), split(k), split(v)
    if form == "exact":
        o = np.matmul(np.matmul(qh.astype(np.float64), kh.transpose(0, 1, 2, 4, 3).astype(np.float64)),
                      vh.astype(np.float64))
        y = (o * np.float64(scale)).astype(np.float32)
    else:
        tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(a)) for a in (qh, kh, vh))
        attn = torch.matmul(tq, tk.transpose(-2, -1)) * float(scale)
        y = torch.matmul(attn, tv).numpy()
    y = y.transpose(0, 1, 3, 2, 4).reshape(T, B, N, C)
    s, vT = lif_multistep(y, v0, tau, v_threshold, v_reset, hard_reset, decay_input)
    return s, vT, y
