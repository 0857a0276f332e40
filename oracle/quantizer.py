"""The HF quantize-dequantize path on the CPU (test oracle and timed CPU baseline only).

Restates ``rotate_quantize`` (``mla_quant/quantizer.py:102-124``) in the reference's
cast order: ``R_eff = R.to(bf16).float()``; ``rot = x.float() @ R_eff`` (torch CPU FP32
GEMM, TF32 off, "highest" precision as ``mla_quant/numerics.py:7-22`` sets it); the
Lloyd INT2 quantize-dequantize of ``codec.qdq`` with the HF scalars
(``quantizer.py:31-35``); ``.to(bf16)``; ``.float() @ R_effᵀ``; ``.to(bf16)``; rows
under the high-precision mask return the input unchanged.
"""

from __future__ import annotations

import numpy as np

from . import codec
from .writer import bf16_round


def rotate_quantize(latent: np.ndarray, rotation: np.ndarray, threshold: float, gain: float,
                    mask: np.ndarray | None = None) -> np.ndarray:
    """``latent`` FP32 ``[n, D]`` holding BF16 values -> FP32 ``[n, D]`` holding BF16 values."""
    import torch

    torch.set_float32_matmul_precision("highest")
    x = np.ascontiguousarray(latent, np.float32)
    reff = torch.from_numpy(np.ascontiguousarray(rotation, np.float32)).to(torch.bfloat16).float()
    rot = (torch.from_numpy(x) @ reff).numpy()
    deq = bf16_round(codec.qdq(rot, *codec.hf_scalars(threshold, gain)))
    restored = bf16_round((torch.from_numpy(deq) @ reff.T).numpy())
    if mask is None:
        return restored
    return np.where(np.asarray(mask, bool)[:, None], x, restored)
