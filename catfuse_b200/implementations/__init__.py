"""Implementation hierarchy (reference: ``catfuse/implementations/__init__.py``)."""
from .base import (Implementation, ConvLIFSpec, ConvLIFParams, IOCost, ScheduleTransform,
                   ScheduleDecomposition, TSI_OPS, CSR_OPS, TGO_OPS, static_zero_forward,
                   folded_affine)
from .dense_keep import DenseKeep
from .sparse_flow import SparseFlow

_SPARSEFLOW_AVAILABLE = True

__all__ = ["Implementation", "ConvLIFSpec", "ConvLIFParams", "IOCost", "ScheduleTransform",
           "ScheduleDecomposition", "TSI_OPS", "CSR_OPS", "TGO_OPS", "DenseKeep", "SparseFlow",
           "static_zero_forward", "folded_affine"]
