"""HardwareProfile — per-GPU thresholds for the policy (reference:
``catfuse/hardware.py:23-179``), with a B200 profile registered for sm_100.

The B200 profile holds the nominal HBM figure and SM count.  On B200 the
fused tcgen05 kernel serves DenseKeep, SparseFlow and StaticZero alike, so
the SparseFlow thresholds only decide where the prescan pass pays for
itself, and the runtime dispatch (EGD) is decided on the device from the
prescan's tile masks: ``egd_max_active_frac`` is the largest fraction of
active (tile, channel chunk) pairs for which the masked launch beats the
dense one, calibrated on B200 with ``python -m catfuse_b200.hbm_bench``
(config-2 sweep: masked time is linear in the active fraction; the value is
the crossover with the dense launch, prescan included).  Profiles without a
calibration keep the reference's element-sparsity rule (> 0.7 -> SparseFlow).
``sparseflow_routing`` decides whether the shape policy sends memory-bound
convs to SparseFlow at all (off on B200, see the profile's comment).
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass


@dataclass(frozen=True)
class HardwareProfile:
    arch_name: str
    sm_version: tuple
    hbm_bandwidth_gbps: float
    l2_size_mb: float
    sm_count: int
    sf_threshold_C: int
    sf_threshold_H: int
    default_K_memory_bound: int
    default_K_compute_bound: int
    notes: str = ""
    egd_max_active_frac: float = -1.0   # < 0: no device calibration (host rule)
    # Static routing: whether memory-bound conv shapes go to SparseFlow
    # (STFusionConvBNLIF, prescan + runtime EGD) at all.
    sparseflow_routing: bool = True

    @property
    def sm_capability(self) -> int:
        return self.sm_version[0] * 10 + self.sm_version[1]


V100_PCIE_32GB = HardwareProfile("V100 PCIe 32GB", (7, 0), 900.0, 6.0, 80, 256, 14, 8, 4,
                                 "reference project default")
V100_SXM_32GB = HardwareProfile("V100 SXM 32GB", (7, 0), 900.0, 6.0, 80, 256, 14, 8, 4)
A100_40GB = HardwareProfile("A100 40GB", (8, 0), 1555.0, 40.0, 108, 128, 28, 8, 4)
A100_80GB = HardwareProfile("A100 80GB", (8, 0), 2039.0, 40.0, 108, 128, 28, 8, 4)


B200 = HardwareProfile(
    arch_name="B200",
    sm_version=(10, 0),
    hbm_bandwidth_gbps=7700.0,
    l2_size_mb=126.0,
    sm_count=148,
    sf_threshold_C=256,
    sf_threshold_H=14,
    # The fused kernel runs up to 8 time steps per launch (one TMEM tile holds
    # 128/8 pixels x 8 steps); longer T is chunked with v carried in HBM.
    default_K_memory_bound=8,
    default_K_compute_bound=8,
    notes="sm_100a tcgen05 path; thresholds route the prescan, not the conv kernel",
    egd_max_active_frac=0.5,
    # Calibrated off: on B200 the prescan costs ~20 % of a dense 256-channel
    # conv and the masked launch only wins below ~50 % active (tile, chunk)
    # pairs; a 64-channel chunk of a 64-pixel x 4-step tile (plus halo) is
    # empty only at per-element spike densities of ~1e-4, far below the 1-20 %
    # of spiking ResNets, so every ResNet conv stays on DenseKeep.  SparseFlow
    # (with the device EGD) remains available through force_sparse.
    sparseflow_routing=False,
)

DEFAULT = B200

_BY_SM = {
    (7, 0): V100_PCIE_32GB,
    (8, 0): A100_40GB,
    (10, 0): B200,
}

_WARNED = set()


def detect_hardware() -> HardwareProfile:
    try:
        import torch
        if not torch.cuda.is_available():
            return DEFAULT
        dev = torch.cuda.current_device()
        cap = torch.cuda.get_device_capability(dev)
        if cap in _BY_SM:
            return _BY_SM[cap]
        if cap not in _WARNED:
            warnings.warn(f"catfuse_b200.hardware: unknown device sm_{cap[0]}{cap[1]}; using "
                          f"{DEFAULT.arch_name}")
            _WARNED.add(cap)
        return DEFAULT
    except Exception:
        return DEFAULT


__all__ = ["HardwareProfile", "V100_PCIE_32GB", "V100_SXM_32GB", "A100_40GB", "A100_80GB", "B200",
           "DEFAULT", "detect_hardware"]
