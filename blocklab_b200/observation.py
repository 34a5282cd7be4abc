"""RGBA8 -> float32 NCHW observation conversion (reference
src/environment/CudaObservation.cu:13-44, ``convertRgba8ToFloatNchw``)."""
from __future__ import annotations

from typing import Optional

import torch

from . import _native as N
from ._native import check


def convert_rgba8_to_float_nchw(rgba8: torch.Tensor, out: Optional[torch.Tensor] = None,
                                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """(N, H, W, 4) uint8 CUDA tensor -> (N, 3, H, W) float32, value * (1/255), alpha dropped."""
    if rgba8.device.type != "cuda" or rgba8.dtype != torch.uint8 or rgba8.dim() != 4 or rgba8.shape[-1] != 4:
        raise ValueError("rgba8 must be a (N, H, W, 4) uint8 CUDA tensor")
    rgba8 = rgba8.contiguous()
    n, h, w, _ = rgba8.shape
    if out is None:
        out = torch.empty((n, 3, h, w), dtype=torch.float32, device=rgba8.device)
    elif out.shape != (n, 3, h, w) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous (N, 3, H, W) float32 tensor")
    s = stream if stream is not None else torch.cuda.current_stream(rgba8.device)
    check(N.lib.blk_convert_rgba8_to_float_nchw(rgba8.data_ptr(), out.data_ptr(), n, w, h, int(s.cuda_stream)))
    return out
