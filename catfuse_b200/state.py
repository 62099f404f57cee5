"""StateBuffer — lazily initialised membrane state carried across forward calls.

Same contract as the reference (``catfuse/state.py:26-98``): ``get`` returns
the current tensor, allocating zeros when uninitialised or when shape /
device / dtype differ; ``set`` stores a detached tensor; ``reset`` drops it so
the next ``get`` starts from zeros (``functional.reset_net`` semantics).

B200 addition: the fused kernels keep v in the pixel-major layout
``[B, H, W, C]``.  A buffer may hold the state in that layout (``set_native``)
and converts to the reference layout ``[B, C, H, W]`` only when a caller asks
through ``get``/``tensor``; ``is_zero`` tells the kernels that v0 == 0 so they
can skip reading it.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


class StateBuffer:
    __slots__ = ("_v", "_native", "_native_shape")

    def __init__(self):
        self._v: Optional[torch.Tensor] = None
        self._native: Optional[torch.Tensor] = None     # [B, H, W, C] fp32
        self._native_shape: Optional[Tuple[int, ...]] = None  # reference shape

    # ---- reference API ------------------------------------------------------
    def get(self, shape, device, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        target_shape = torch.Size(shape)
        target_device = torch.device(device) if not isinstance(device, torch.device) else device
        self._materialize()
        if (self._v is None or self._v.shape != target_shape or self._v.device != target_device
                or self._v.dtype != dtype):
            self._v = torch.zeros(target_shape, device=target_device, dtype=dtype)
            self._native = None
        return self._v

    def set(self, v: torch.Tensor) -> None:
        self._v = v.detach()
        self._native = None
        self._native_shape = None

    def reset(self) -> None:
        self._v = None
        self._native = None
        self._native_shape = None

    @property
    def is_initialized(self) -> bool:
        return self._v is not None or self._native is not None

    @property
    def tensor(self) -> Optional[torch.Tensor]:
        self._materialize()
        return self._v

    def __repr__(self) -> str:
        t = self.tensor
        if t is None:
            return "StateBuffer(uninitialized)"
        return f"StateBuffer(shape={tuple(t.shape)}, device={t.device}, dtype={t.dtype})"

    # ---- native-layout access used by the fused kernels ----------------------
    def set_native(self, v_bhwc: torch.Tensor) -> None:
        """Store v in the kernels' [B, H, W, C] layout."""
        B, H, W, C = v_bhwc.shape
        self._native = v_bhwc.detach()
        self._native_shape = (B, C, H, W)
        self._v = None

    def get_native(self, shape_bchw, device) -> Optional[torch.Tensor]:
        """v in [B, H, W, C] for the kernels, or None when v0 == 0 (fresh)."""
        B, C, H, W = shape_bchw
        device = torch.device(device)
        if self._native is not None and self._native_shape == tuple(shape_bchw) \
                and self._native.device == device:
            return self._native
        if self._v is not None and tuple(self._v.shape) == tuple(shape_bchw) \
                and self._v.device == device:
            from .ops import v_to_nhwc
            return v_to_nhwc(self._v.float().contiguous())
        return None

    def _materialize(self) -> None:
        if self._native is not None and self._v is None:
            from .ops import v_to_nchw
            self._v = v_to_nchw(self._native)
            self._native = None
            self._native_shape = None
