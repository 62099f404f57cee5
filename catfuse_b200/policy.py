"""Spatio-temporal policy: per fusible pattern, the TimeBlock size K and the
spatial backend (DenseKeep / SparseFlow / StaticZero).

API and formulas follow the reference (``catfuse/policy.py:28-279``):
``SpatialBackend``, ``PolicyRow``, the I/O-ratio model, ``optimal_K``,
``classify_shape_regime``, ``build_default_policy_table`` and
``get_policy``.  Thresholds come from a :class:`HardwareProfile` (default:
the B200 profile) instead of being fixed to V100.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


class SpatialBackend:
    DENSE_KEEP = "DenseKeep"
    SPARSE_FLOW = "SparseFlow"
    STATIC_ZERO = "StaticZero"


@dataclass
class PolicyRow:
    pattern: str
    shape_regime: str
    K: int
    spatial_backend: str
    fusion_mode: str
    io_ratio: Optional[float] = None

    def __repr__(self):
        return (f"PolicyRow({self.pattern}, {self.shape_regime}, K={self.K}, "
                f"spatial={self.spatial_backend}, fusion={self.fusion_mode}, io={self.io_ratio})")


# Runtime EGD: sparsity above this routes a Conv-BN-LIF call to SparseFlow
# (reference: catfuse/sparseflow/ops/st_fusion_conv_bn_lif.py:519).
EGD_SPARSITY_THRESHOLD = 0.7


def io_ratio_partial_fusion(K: int) -> float:
    """Conv output z round-trips HBM: (3 + 2/K) / 7."""
    return (3.0 + 2.0 / K) / 7.0


def io_ratio_full_fusion(K: int) -> float:
    """z stays on chip (StreamFuse): (1 + 2/K) / 5."""
    return (1.0 + 2.0 / K) / 5.0


def _hw(hwprof):
    if hwprof is None:
        from .hardware import DEFAULT as hwprof
    return hwprof


def optimal_K(T: int, regime: str = "memory_bound", hwprof=None) -> int:
    hw = _hw(hwprof)
    if regime == "compute_bound":
        return min(hw.default_K_compute_bound, T)
    return min(hw.default_K_memory_bound, T)


def classify_shape_regime(C_in: int, C_out: int, H: int, W: int, kernel_size: int = 3,
                          hwprof=None) -> str:
    hw = _hw(hwprof)
    sf_C, sf_H = hw.sf_threshold_C, hw.sf_threshold_H
    if kernel_size == 1:
        return "memory_bound"
    if C_in >= sf_C and H <= sf_H:
        return "memory_bound"
    if C_in <= sf_C // 2:
        return "compute_bound"
    if H >= sf_H * 2:
        return "compute_bound"
    return "memory_bound"


def build_default_policy_table():
    # On B200 every Conv-BN-LIF row is realised by the same fused tcgen05
    # kernel ("full_tcgen05"); DenseKeep vs SparseFlow only toggles the
    # prescan-driven chunk skipping.
    t = {}
    t[("Conv3x3_BN_LIF", "compute_bound")] = PolicyRow(
        "Conv3x3_BN_LIF", "compute_bound", 4, SpatialBackend.DENSE_KEEP, "full_tcgen05",
        io_ratio_full_fusion(4))
    t[("Conv3x3_BN_LIF", "memory_bound")] = PolicyRow(
        "Conv3x3_BN_LIF", "memory_bound", 8, SpatialBackend.SPARSE_FLOW, "full_tcgen05",
        io_ratio_full_fusion(8))
    t[("Conv1x1_LIF", "memory_bound")] = PolicyRow(
        "Conv1x1_LIF", "memory_bound", 8, SpatialBackend.SPARSE_FLOW, "full_tcgen05",
        io_ratio_full_fusion(8))
    for pat in ("Linear_LIF", "Add_LIF", "Add_BN_LIF", "AvgPool_LIF"):
        t[(pat, "all")] = PolicyRow(pat, "all", 0, SpatialBackend.DENSE_KEEP, "full_cuda", None)
    return t


_DEFAULT_TABLE = None


def get_policy(pattern: str, C_in: int = 0, C_out: int = 0, H: int = 0, W: int = 0,
               kernel_size: int = 3, T: int = 16, hwprof=None) -> PolicyRow:
    global _DEFAULT_TABLE
    if _DEFAULT_TABLE is None:
        _DEFAULT_TABLE = build_default_policy_table()
    if pattern in ("Linear_LIF", "Add_LIF", "Add_BN_LIF", "AvgPool_LIF"):
        regime = "all"
    else:
        regime = classify_shape_regime(C_in, C_out, H, W, kernel_size, hwprof)
    row = _DEFAULT_TABLE.get((pattern, regime))
    if (row is not None and row.spatial_backend == SpatialBackend.SPARSE_FLOW
            and not getattr(_hw(hwprof), "sparseflow_routing", True)):
        row = PolicyRow(row.pattern, row.shape_regime, row.K, SpatialBackend.DENSE_KEEP,
                        row.fusion_mode, row.io_ratio)
    if row is not None:
        if row.K == 0:
            return PolicyRow(row.pattern, row.shape_regime, T, row.spatial_backend, row.fusion_mode,
                             row.io_ratio)
        return row
    K = min(4, T)
    return PolicyRow(pattern, regime, K, SpatialBackend.DENSE_KEEP, "full_tcgen05",
                     io_ratio_full_fusion(K))


__all__ = ["SpatialBackend", "PolicyRow", "EGD_SPARSITY_THRESHOLD", "io_ratio_partial_fusion",
           "io_ratio_full_fusion", "optimal_K", "classify_shape_regime",
           "build_default_policy_table", "get_policy"]
