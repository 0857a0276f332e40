"""General packed writer for already-rotated rows (drop-in for the upstream
``sglang/QuantKernel/mla_latent_int2.py`` entry points the reference patches).

``scatter_pack_rows`` keeps the patched signature and check of
``deployment/patches/rolaq_sglang.patch:9-34``; the codec runs in
``rolaq_scatter_pack_rows``: the learned / default Lloyd INT2 codec, or with
``lloyd_max=False`` OSCAR's uniform min/max INT2 baseline (``mla_quant/oscar.py:91-101``).
Only 2-bit storage is built; other widths raise ``NotImplementedError``.
"""

from __future__ import annotations

import torch

from . import ops

# Lloyd-Max INT2 constants under the upstream names (values: mla_quant/oscar.py:104-111)
_LM_THRESHOLDS = ops.LLOYD_MAX_THRESHOLDS
_LM_CENTROIDS = ops.LLOYD_MAX_CENTROIDS
_LM_SPAN = ops.SPAN
_LM_RATIO = ops.LLOYD_MAX_STRETCH


def scatter_pack_rows(x, slots, codes_buf, params_buf, group_size, lloyd_max, bits=2, quantizer_params=None):
    """Quantize ``x`` (``[n, D]``, rotated frame) into ``codes/params`` at ``slots``."""
    if quantizer_params is not None and (not lloyd_max or bits != 2):
        raise ValueError("Learned threshold/gain require the INT2 Lloyd writer")
    if bits != 2:
        raise NotImplementedError("only 2-bit packed storage is implemented")
    if group_size != 128:
        raise ValueError("group_size must be 128")
    n = x.shape[0]
    if n == 0:
        return
    x = x.contiguous().to(torch.float32)
    if lloyd_max:
        threshold, gain = quantizer_params if quantizer_params is not None else (_LM_THRESHOLDS[2], _LM_RATIO)
        codec = ops.codec_serving(threshold, gain)
    else:
        codec = ops.codec_uniform()
    ops.scatter_pack_rows(x, slots.contiguous(), codes_buf, params_buf, codec)
