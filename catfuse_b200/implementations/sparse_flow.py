"""SparseFlow on B200: prescan (per-M-tile mask of active input channel
chunks) followed by the fused tcgen05 Conv->BN->LIF kernel that walks only
the active chunks; tiles with an empty mask issue no MMA (StaticZero per
tile).

Replaces ``SparseFlow`` (``catfuse/implementations/sparse_flow.py:186-328``)
and its ``sparse_streamfuse_conv3x3_bn_lif`` kernel
(``catfuse/sparseflow/streamfuse_kernel.py:32-187``).  Unlike the reference,
any kernel size and stride is supported, and the result equals DenseKeep's
exactly (skipped chunks contribute exact zeros).
"""
from __future__ import annotations

import torch

from .base import (Implementation, ScheduleDecomposition, ScheduleTransform)
from ._fused import KERNEL_TIME_BLOCK, _WeightCache, fused_forward, fused_io_cost


class SparseFlow(Implementation):
    name = "SparseFlow"

    def __init__(self):
        super().__init__()
        self._cache = _WeightCache()
        self.last_stats = None

    def reset_caches(self) -> None:
        self._cache.reset()

    def forward(self, x, spec, params, state, stats=None, egd_max_active_frac=None):
        return fused_forward(x, spec, params, state, self._cache, sparse=True, stats=stats,
                             egd_max_active_frac=egd_max_active_frac)

    def forward_with_k(self, x, spec, params, state, K=None):
        """TimeBlock(K): chunks of K steps, v carried through the StateBuffer;
        the output is identical for every K."""
        T = x.shape[0]
        K = T if K is None else max(1, min(int(K), int(T)))
        if K >= T:
            return self.forward(x, spec, params, state)
        return torch.cat([self.forward(x[s:s + K].contiguous(), spec, params, state)
                          for s in range(0, T, K)], dim=0)

    def analytic_io_cost(self, spec, T, B, H_in, W_in, K=None, *, dtype_bytes=4):
        K = T if K is None else max(1, min(int(K), int(T)))
        c = fused_io_cost(spec, T, B, H_in, W_in, dtype_bytes,
                          f"TimeBlock({K})∘StreamFuse(Conv,LIF)∘StateCarry(LIF) — prescan-masked tcgen05")
        nblocks = -(-T // min(K, KERNEL_TIME_BLOCK))
        Ho, Wo = spec.output_hw(H_in, W_in)
        from .base import IOCost
        return IOCost(c.x_load * 2, c.w_load, 0, 2 * nblocks * B * Ho * Wo * spec.out_channels * 4,
                      c.spike_write, c.schedule, nblocks)

    def schedule_decomposition(self, spec, T, K=None):
        K = T if K is None else max(1, min(int(K), int(T)))
        return ScheduleDecomposition(
            transforms=(ScheduleTransform.StateCarry("LIF"), ScheduleTransform.StreamFuse("Conv", "LIF"),
                        ScheduleTransform.TimeBlock(K)),
            form="form_2",
            description=f"SparseFlow (sm_100a): TimeBlock(K={K}) ∘ StreamFuse(Conv, LIF) ∘ StateCarry(LIF)")

    def __repr__(self):
        return f"SparseFlow(cached={'yes' if self._cache.wp is not None else 'no'})"
