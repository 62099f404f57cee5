"""Conv -> BN -> (residual) -> multi-step LIF on the CPU (fp32).

Reference path: ``STFusionConvBNLIF._fallback_forward_single``
(``catfuse/sparseflow/ops/st_fusion_conv_bn_lif.py:425-445``) applied per time
step with v carried (StateCarry), which is also the math of
``partial_fusion_conv_bn_lif`` (``catfuse/kernels/partial_fusion_conv_bn_lif_impl.py:215-268``)
and ``PartialFusionConvBNAddLIF`` (``catfuse/patterns.py:394-486``) for the
pre-LIF residual; the SEW post-LIF combine follows ``CTFSEWBasicBlock.forward``
(``catfuse/patterns.py:700-715``).  The convolution is BatchFolded over T
(``catfuse/implementations/dense_keep.py:122-128``).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .lif import lif_multistep


def conv_z(x, weight, scale=None, shift=None, stride=1, pad=1, conv_bias=None,
           operand_dtype=None):
    """z[T,B,Cout,Ho,Wo] = BN(conv(x)) with BN as z*scale + shift.

    ``operand_dtype=torch.float16`` rounds x and the weights to fp16 first
    (the tensor-core operand precision), accumulation stays fp32."""
    x = torch.as_tensor(x, dtype=torch.float32)
    w = torch.as_tensor(weight, dtype=torch.float32)
    if operand_dtype is not None:
        x = x.to(operand_dtype).float()
        w = w.to(operand_dtype).float()
    T, B = x.shape[:2]
    z = F.conv2d(x.reshape(T * B, *x.shape[2:]), w,
                 None if conv_bias is None else torch.as_tensor(conv_bias, dtype=torch.float32),
                 stride=stride, padding=pad)
    if scale is not None:
        z = z * torch.as_tensor(scale, dtype=torch.float32).view(1, -1, 1, 1)
    if shift is not None:
        z = z + torch.as_tensor(shift, dtype=torch.float32).view(1, -1, 1, 1)
    return z.reshape(T, B, *z.shape[1:])


def conv_bn_lif(x, weight, scale=None, shift=None, stride=1, pad=1, v0=None,
                tau=2.0, v_threshold=1.0, v_reset=0.0, hard_reset=True,
                decay_input=True, conv_bias=None, operand_dtype=None, return_z=False):
    z = conv_z(x, weight, scale, shift, stride, pad, conv_bias, operand_dtype)
    s, vT = lif_multistep(z.numpy(), None if v0 is None else np.asarray(v0, np.float32),
                          tau, v_threshold, v_reset, hard_reset, decay_input)
    if return_z:
        return s, vT, z.numpy()
    return s, vT


def conv_bn_lif_residual(x, weight, scale, shift, identity, mode, stride=1, pad=1,
                         v0=None, tau=2.0, v_threshold=1.0, v_reset=0.0,
                         operand_dtype=None):
    """mode: 'add_pre' (z += identity before the LIF), or the SEW combines
    'add' / 'and' / 'iand' applied to the LIF spikes."""
    z = conv_z(x, weight, scale, shift, stride, pad, None, operand_dtype).numpy()
    ident = np.asarray(identity, np.float32)
    if mode == "add_pre":
        z = (z + ident).astype(np.float32)
    s, vT = lif_multistep(z, v0, tau, v_threshold, v_reset)
    if mode == "add":
        out = ident + s
    elif mode == "and":
        out = ident * s
    elif mode == "iand":
        out = ident * (1.0 - s)
    else:
        out = s
    return out.astype(np.float32), vT
