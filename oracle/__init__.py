"""CPU oracle for the multi-step SNN inference hot path (TEST INFRASTRUCTURE).

This package restates, on the CPU, the reference algorithm of every kernel on
the path (SpikingJelly multi-step LIF semantics as reproduced by CATFuse, the
BN fold, Conv->BN->LIF, the receptive-field prescan, the SEW / Spiking
ResNet-18 forward and the Spikformer forward).  It exists only to CHECK the CUDA path:

* only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
  / reference arm may import it;
* the product package ``catfuse_b200`` never imports it and has no CPU
  fallback.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against fixtures produced by running the reference's own code
(``tests/golden/make_golden.py``: Triton kernels under ``TRITON_INTERPRET=1``
and the reference's pure-PyTorch per-step path).
"""
from .lif import lif_multistep, lif_multistep_triton_form
from .bn import fold_bn
from .conv import conv_bn_lif, conv_bn_lif_residual
from .prescan import prescan_rf, choose_group_size, select_tile_sizes
from .ssa import ssa_lif
from .nets import sew_resnet18_forward, spiking_resnet18_forward, make_resnet18_params
from .spikformer import spikformer_forward

__all__ = [
    "lif_multistep", "lif_multistep_triton_form", "fold_bn", "conv_bn_lif",
    "conv_bn_lif_residual", "prescan_rf", "choose_group_size", "select_tile_sizes",
    "sew_resnet18_forward", "spiking_resnet18_forward", "make_resnet18_params", "ssa_lif",
    "spikformer_forward",
]
