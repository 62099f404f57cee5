"""SpikingJelly-compatible building blocks (activation_based API subset).

CATFuse rewrites SpikingJelly (SJ) models.  SJ is an optional dependency:
when ``spikingjelly`` is importable its classes are recognised as well, but
this package carries the subset that the hot path needs so that models can be
built and rewritten without it — ``base.MemoryModule``, ``neuron.LIFNode``
(multi-step, torch backend), ``functional.reset_net`` /
``functional.set_step_mode``, the multi-step ``layer`` wrappers, a
``surrogate`` placeholder (inference only), and a model zoo with the SEW /
Spiking ResNet topologies (``zoo``).  These modules are the *unoptimised*
model a user hands to :func:`catfuse_b200.optimize`; they run eagerly in
PyTorch.
"""
from . import base, functional, layer, neuron, surrogate  # noqa: F401
