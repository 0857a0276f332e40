"""General packed writer for already-rotated rows (drop-in for the upstream
``sglang/QuantKernel/mla_latent_int2.py`` entry points the reference patches).

``scatter_pack_rows`` keeps the patched signature and check of
``deployment/patches/rolaq_sglang.patch:9-34``; the codec runs in
``rolaq_scatter_pack_rows``.  Only the Lloyd INT2 codec is implemented; the OSCAR
uniform min/max baseline (``lloyd_max=False``) is rejected.
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
    if not lloyd_max or bits != 2:
        raise NotImplementedError("only the Lloyd-Max INT2 codec is implemented")
    if group_size != 128:
        raise ValueError("group_size must be 128")
    n = x.shape[0]
    if n == 0:
        return
    x = x.contiguous().to(torch.float32)
    threshold, gain = quantizer_params if quantizer_params is not None else (_LM_THRESHOLDS[2], _LM_RATIO)
    ops.scatter_pack_rows(x, slots.contiguous(), codes_buf, params_buf, ops.codec_serving(threshold, gain))
