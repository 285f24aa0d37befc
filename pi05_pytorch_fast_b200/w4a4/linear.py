"""W4A4Linear: drop-in for nn.Linear on the B200 W4A4 path.

Same constructor arguments, buffers, checks and forward contract as the
reference's ``pi05_fast/w4a4/linear.py:10-59`` (``packed`` int32 buffer,
empty fp16 ``weight`` dtype marker, optional bias, fragment-major flag).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .extension import int4_gemm, int4_gemm_tiled
from .pack import pack_linear_weight, should_rotate


class W4A4Linear(nn.Module):
    """Runtime INT4 activations x packed INT4 weights, fp16 out."""

    def __init__(
        self,
        packed: torch.Tensor,
        bias: torch.Tensor | None = None,
        rotate: bool | None = None,
        in_features: int | None = None,
        preshuffled: bool = False,
    ):
        super().__init__()
        if packed.dim() != 2:
            raise ValueError("packed weight must be [N, K/8+1]")
        self.out_features = int(packed.shape[0])
        self.in_features = int(in_features or (packed.shape[1] - 1) * 8)
        if packed.shape[1] < self.in_features // 8 + 1:
            raise ValueError("packed weight row is too short for in_features")
        self.rotate = should_rotate(self.in_features, rotate)
        self.preshuffled = bool(preshuffled)
        if self.preshuffled and packed.shape[1] != self.in_features // 8 + 9:
            raise ValueError("preshuffled weight must use the K/8+9 marker stride")
        self.register_buffer("packed", packed.to(torch.int32), persistent=True)
        # Callers read ``proj.weight.dtype``: keep an empty fp16 marker.
        self.register_buffer("weight", torch.empty(0, dtype=torch.float16, device=packed.device),
                             persistent=False)
        if bias is None:
            self.register_parameter("bias", None)
        else:
            self.bias = nn.Parameter(bias.detach().clone(), requires_grad=False)

    @classmethod
    def from_linear(cls, linear: nn.Linear, rotate: bool | None = None) -> "W4A4Linear":
        bias = None if linear.bias is None else linear.bias.detach()
        return cls(pack_linear_weight(linear.weight, rotate=rotate), bias=bias, rotate=rotate,
                   in_features=linear.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xh = x if x.dtype == torch.float16 else x.to(torch.float16)
        xh = xh if xh.is_contiguous() else xh.contiguous()
        op = int4_gemm_tiled if self.preshuffled else int4_gemm
        y = op(xh, self.packed)
        if y.dtype != x.dtype:
            y = y.to(x.dtype)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y

    def extra_repr(self) -> str:
        return (f"in={self.in_features}, out={self.out_features}, rotate={self.rotate}, "
                f"preshuffled={self.preshuffled}")
