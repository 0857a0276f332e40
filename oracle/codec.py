"""Numpy restatement of the OSCAR Lloyd INT2 codec (test oracle only).

Reference: ``mla_quant/oscar.py:120-144`` (``oscar_lloyd_int2_qdq``)::

    mean  = groups.mean(-1)
    std   = sqrt(mean((x - mean)^2) + 1e-8)
    n     = (x - mean) / std
    code  = [n >= -t] + [n >= 0] + [n >= t]                 in {0, 1, 2, 3}
    scale = (span / 3) * g * std                            span = C3 - C0
    zero  = -C0 / (span / 3) - mean / scale
    deq   = (code - zero) * scale

PyTorch semantics that the restatement keeps (checked against torch 2.11):

* ``tensor >= python_float`` compares against the scalar rounded to FP32;
* ``python_float * tensor`` rounds the scalar to FP32 first, then multiplies in FP32;
* ``(span / 3.0) * gain`` and ``-C0 / (span / 3.0)`` are evaluated in Python double
  before that rounding;
* ``diff.pow(2)`` is ``diff * diff`` (no fused multiply-add anywhere).

The only freedom is the order of the two 128-element FP32 sums.  torch's CPU order
is ISA-dependent, so the oracle fixes one order that the CUDA kernels reproduce
exactly (``group_sum`` below).  Against the reference the result differs by at most
an ULP or two in ``mean``/``std``, which can flip a code only when ``n`` lies within
that distance of a threshold; the golden tests measure that fraction.
"""

from __future__ import annotations

import numpy as np

# mla_quant/oscar.py:104-111
LLOYD_MAX_THRESHOLDS = (-0.9810652732849121, 0.0, 0.9810652732849121)
LLOYD_MAX_CENTROIDS = (
    -1.5095585584640503,
    -0.4527800381183624,
    0.4527800381183624,
    1.5095585584640503,
)
LLOYD_MAX_STRETCH = 1.16
SPAN = LLOYD_MAX_CENTROIDS[3] - LLOYD_MAX_CENTROIDS[0]
SPAN3 = SPAN / 3.0
ZERO_CONST = -LLOYD_MAX_CENTROIDS[0] / SPAN3
GROUP = 128
EPS = np.float32(1e-08)
INV_GROUP = np.float32(1.0 / GROUP)


def hf_scalars(threshold: float, gain: float) -> tuple[np.float32, np.float32, np.float32]:
    """(t32, scale_factor32, zero_const32) as the HF quantizer path forms them.

    ``LearnedRotationQuantizer.quantize_layer`` wraps the manifest floats in FP32
    tensors (``quantizer.py:308-309``); ``oscar_lloyd_hard`` reads them back as Python
    floats and swaps an FP32(1.16) gain for the double 1.16 (``quantizer.py:31-35``).
    """
    t = float(np.float32(threshold))
    g32 = np.float32(gain)
    g = LLOYD_MAX_STRETCH if g32 == np.float32(LLOYD_MAX_STRETCH) else float(g32)
    return np.float32(t), np.float32(SPAN3 * g), np.float32(ZERO_CONST)


def serving_scalars(threshold: float, gain: float) -> tuple[np.float32, np.float32, np.float32]:
    """(t32, scale_factor32, zero_const32) as the serving writer forms them.

    ``load_layer_quantizers`` returns the manifest values as Python floats
    (``rolaq_mla.py:41-53``) and the writer passes ``(-t, 0, t)`` and ``gain`` as
    kernel constants (``mla_fused_writer.py:158-164``): the gain is never rounded to
    FP32 before the double product with ``span / 3``.
    """
    return np.float32(threshold), np.float32(SPAN3 * float(gain)), np.float32(ZERO_CONST)


def group_sum(v: np.ndarray) -> np.ndarray:
    """FP32 sum over the last axis (length 128) in the kernels' fixed order.

    Eight running sums ``acc[k] += v[8*i + k]`` for ``i = 0..15``, then the tree
    ``((a0+a1)+(a2+a3)) + ((a4+a5)+(a6+a7))``.
    """
    assert v.dtype == np.float32 and v.shape[-1] == GROUP
    acc = np.zeros(v.shape[:-1] + (8,), np.float32)
    for i in range(GROUP // 8):
        acc = acc + v[..., 8 * i : 8 * i + 8]
    a = acc
    return ((a[..., 0] + a[..., 1]) + (a[..., 2] + a[..., 3])) + (
        (a[..., 4] + a[..., 5]) + (a[..., 6] + a[..., 7])
    )


def encode(x: np.ndarray, t32, scale_factor32, zero_const32=np.float32(ZERO_CONST)):
    """Rotated FP32 rows ``[n, D]`` -> (codes uint8 ``[n, D]``, scale ``[n, NG]``, zero ``[n, NG]``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    if d % GROUP:
        raise ValueError("latent width must be a multiple of 128")
    g = x.reshape(n, d // GROUP, GROUP)
    mean = group_sum(g) * INV_GROUP
    diff = g - mean[..., None]
    var = group_sum(diff * diff) * INV_GROUP
    std = np.sqrt(var + EPS)
    nrm = diff / std[..., None]
    t = np.float32(t32)
    codes = (
        (nrm >= -t).astype(np.uint8) + (nrm >= np.float32(0)).astype(np.uint8) + (nrm >= t).astype(np.uint8)
    )
    scale = np.float32(scale_factor32) * std
    zero = np.float32(zero_const32) - mean / scale
    return codes.reshape(n, d), scale.astype(np.float32), zero.astype(np.float32)


def dequant(codes: np.ndarray, scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    """``(code - zero) * scale`` in FP32, group-wise (``oscar.py:144``)."""
    n, d = codes.shape
    c = codes.reshape(n, d // GROUP, GROUP).astype(np.float32)
    out = (c - zero[..., None]) * scale[..., None]
    return out.reshape(n, d).astype(np.float32)


def qdq(x: np.ndarray, t32, scale_factor32, zero_const32=np.float32(ZERO_CONST)) -> np.ndarray:
    """Full quantize-dequantize of rotated FP32 rows (``oscar_lloyd_int2_qdq``)."""
    codes, scale, zero = encode(x, t32, scale_factor32, zero_const32)
    return dequant(codes, scale, zero)


# ---- OSCAR's uniform min/max INT2 baseline ------------------------------------------


def encode_uniform(x: np.ndarray):
    """Rotated FP32 rows ``[n, D]`` -> (codes ``[n, D]``, scale ``[n, NG]``, minimum ``[n, NG]``).

    Restates ``uniform_int2_qdq`` (``mla_quant/oscar.py:91-101``): per 128-group
    ``scale = (max - min) / 3`` where ``|max - min| > 1e-8`` (the scalar rounded to FP32),
    else 1; ``code = clamp(round((x - min) / scale), 0, 3)`` with round-half-to-even
    (``torch.round``, ``np.rint``); every operation in FP32.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    g = x.reshape(n, d // GROUP, GROUP)
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    rng = mx - mn
    scale = np.where(np.abs(rng) > np.float32(1e-08), rng / np.float32(3.0), np.float32(1.0)).astype(np.float32)
    q = (g - mn[..., None]) / scale[..., None]
    codes = np.clip(np.rint(q), 0, 3).astype(np.uint8)
    return codes.reshape(n, d), scale, mn.astype(np.float32)


def uniform_qdq(x: np.ndarray) -> np.ndarray:
    """``codes * scale + min`` in FP32 (the reference's reconstruction)."""
    codes, scale, mn = encode_uniform(x)
    n, d = codes.shape
    c = codes.reshape(n, d // GROUP, GROUP).astype(np.float32)
    return (c * scale[..., None] + mn[..., None]).reshape(n, d).astype(np.float32)


def uniform_params(scale: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """The cache's (scale, zero) of the uniform codec: zero = FP32(-min / scale), so that
    the reader's ``(code - zero) * scale`` reconstructs ``code * scale + min``."""
    return params_array(scale, (-mn / scale).astype(np.float32))


# ---- packed byte layout (this build's cache format) -------------------------------
# Code of latent element j lives in byte j // 4 of the slot's row, bits 2*(j % 4).


def pack(codes: np.ndarray) -> np.ndarray:
    """uint8 codes ``[n, D]`` -> packed bytes ``[n, D // 4]``."""
    n, d = codes.shape
    c = codes.reshape(n, d // 4, 4).astype(np.uint8)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def unpack(packed: np.ndarray, d: int) -> np.ndarray:
    """packed bytes ``[n, D // 4]`` -> uint8 codes ``[n, D]``."""
    p = packed.reshape(packed.shape[0], d // 4).astype(np.uint8)
    out = np.stack([(p >> (2 * k)) & 3 for k in range(4)], axis=-1)
    return out.reshape(p.shape[0], d).astype(np.uint8)


def params_array(scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    """(scale, zero) -> FP32 ``[n, NG, 2]`` as stored per slot."""
    return np.stack([scale, zero], axis=-1).astype(np.float32)


def rotate_reference(x_bf16_as_f32: np.ndarray, rotation_f32: np.ndarray) -> np.ndarray:
    """``x.float() @ R.to(bf16).float()`` with the reference FP32 GEMM (torch CPU).

    ``quantizer.py:117-118`` / ``mla_fused_writer.py:142-147``.  Uses torch with TF32
    off and "highest" precision (``numerics.py:7-22``).  Inputs must already hold
    BF16-representable values.
    """
    import torch

    torch.set_float32_matmul_precision("highest")
    xt = torch.from_numpy(np.ascontiguousarray(x_bf16_as_f32, np.float32))
    r = torch.from_numpy(np.ascontiguousarray(rotation_f32, np.float32)).to(torch.bfloat16).float()
    return (xt @ r).numpy()
