"""catfuse_b200 — B200-native (sm_100a) multi-step SNN inference hot path.

A drop-in for CATFuse's inference path: ``optimize(sj_model)`` rewrites a
SpikingJelly-style model into fused patterns (``patterns``), routed by the
StaticZero / SparseFlow / DenseKeep policy (``policy``), whose kernels are the
hand-written sm_100a CUDA kernels of ``libcatfuse_sm100.so`` reached through
its C ABI (``include/catfuse_b200.h``).  There is no CPU fallback.
"""
from __future__ import annotations

__version__ = "0.1.0"


def optimize(model, device="cuda:0", policy=None, T=16, use_sparseflow=True, native=True,
             use_graph=True, precision="fp16"):
    """Rewrite ``model`` into fused CTF patterns.  Returns ``(model, stats)``.

    Reference: ``catfuse/__init__.py:9-13`` (there ``device`` and ``policy``
    are ignored).  Here ``device`` moves the rewritten model (when CUDA is
    available), ``policy`` may be a :class:`~catfuse_b200.hardware.HardwareProfile`
    overriding the routing thresholds, and — for spiking ResNets — ``native``
    wraps the result in :class:`~catfuse_b200.network.CTFNetwork`, which runs
    the whole forward as one CUDA graph of fused kernels without leaving the
    kernels' layout between layers.  ``precision`` selects the conv operand
    precision of the native plan: "fp16" (fp16 weights; spikes are exact) or
    "split" (weights and the stem input as fp16 hi + lo pairs, fp32-faithful,
    twice the tensor-core work).
    """
    import torch
    from .substitute import substitute, substitute_sf
    if use_sparseflow:
        new_model, stats = substitute_sf(model, T=T, hwprof=policy)
    else:
        new_model, stats = substitute(model)
    if device is not None and torch.cuda.is_available():
        new_model = new_model.to(device)
    stats["native_plan"] = False
    if native:
        from .spikformer_net import CTFSpikformer, is_spikformer
        if is_spikformer(new_model):
            net = CTFSpikformer(new_model, use_graph=use_graph, precision=precision)
            stats["native_plan"] = True
            return net, stats
        from .network import CTFNetwork, UnsupportedTopology
        try:
            # STFusion sites keep their runtime dispatch inside the native plan:
            # prescan + device-side EGD (SparseFlow / DenseKeep / StaticZero)
            net = CTFNetwork(new_model, use_graph=use_graph, use_sparse=use_sparseflow,
                             precision=precision)
            stats["native_plan"] = True
            return net, stats
        except UnsupportedTopology as e:
            stats["native_plan_reason"] = str(e)
    return new_model, stats


__all__ = ["optimize", "__version__"]
