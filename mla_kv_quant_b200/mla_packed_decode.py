"""Packed-INT2 MLA decode reader (stands in for the upstream
``srt/layers/attention/triton_ops/mla_packed_decode.py``).

``prepare_gf_splits`` keeps the reference's helper (``rolaq_sglang.patch:81-92``).
``packed_mla_decode_gf_fwd`` takes the role of the upstream function of that name
(called at ``rolaq_sglang.patch:51-111``): split-KV attention over the INT2 pages
plus one split over the BF16 window rows, merged by log-sum-exp.  Its argument list
is this build's own (the upstream signature is not vendored): queries
``[B, H, D + Dr]`` in the rotated frame, a 64-token page table, ``seq_lens``, the
softmax scale, the number of INT2 splits, and optional scratch ``attn_logits``
``[B, H, S + 1, D]`` / ``attn_lse`` ``[B, H, S + 1]`` that the caller may preallocate
(as the reference does for CUDA-graph capture).
"""

from __future__ import annotations

import torch

from . import ops


def prepare_gf_splits(splits, quant, merge):
    """``quant = max(splits - 1, 1)``, ``merge = quant + 1`` in one launch."""
    ops.prepare_gf_splits(splits, quant, merge)


def packed_mla_decode_gf_fwd(q, pool, layer_id, page_table, seq_lens, sm_scale, num_kv_splits,
                             attn_logits=None, attn_lse=None, out=None, out_lse=None, err=None):
    """Decode attention for one layer; returns ``out`` ``[B, H, D]`` BF16 (rotated frame)."""
    d = pool.kv_lora_rank
    if q.dim() == 2:
        q = q.view(q.shape[0], -1, d + pool.qk_rope_head_dim)
    b, h, _ = q.shape
    s = int(num_kv_splits)
    if attn_logits is None:
        attn_logits = torch.empty(b, h, s + 1, d, dtype=torch.float32, device=q.device)
    if attn_lse is None:
        attn_lse = torch.empty(b, h, s + 1, dtype=torch.float32, device=q.device)
    if out is None:
        out = torch.empty(b, h, d, dtype=torch.bfloat16, device=q.device)
    ops.packed_decode(q, pool.layer_view(layer_id), page_table, seq_lens, sm_scale, s, attn_logits, attn_lse, out,
                      out_lse=out_lse, err=err)
    return out


packed_mla_decode = packed_mla_decode_gf_fwd
