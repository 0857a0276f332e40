"""Decode writer plugin (drop-in for ``deployment/sglang/QuantKernel/mla_fused_writer.py``).

``try_fast_decode_store`` keeps the reference's contract: it returns whether it
handled the write, so the caller's fallback path stays in charge otherwise.  The
reference ran ``c = c_kv.float() @ R`` as an FP32 cuBLAS GEMM and then one Triton
launch (the Lloyd codec) or ``scatter_pack_rows`` + ``_aux`` (any other codec); here
one sm_100a launch (``rolaq_fused_write``) does the rotation on tcgen05, the codec
(learned / default Lloyd, or OSCAR's uniform min/max when the pool runs without
Lloyd-Max), the packed scatter, the BF16 ``k_pe`` store and the s4r16 ring stores.
A layer without a rotation is written unrotated (``c = c_kv``, the reference's
``mla_fused_writer.py:146-149``): the identity matrix as the tcgen05 operand gives
``c`` exactly.
"""

from __future__ import annotations

import torch

from . import ops

_SUPPORTED = {(512, 64), (256, 32)}


def try_fast_decode_store(pool, layer_id, loc, c_kv, k_pe):
    """Return whether the decode write was handled (``mla_fused_writer.py:110-224``)."""
    meta = pool._fb_window_meta
    n = c_kv.numel() // pool.kv_lora_rank
    if (
        n <= 0
        or (pool.kv_lora_rank, pool.qk_rope_head_dim) not in _SUPPORTED
        or not pool._latent_windows
        or not meta
        or meta.get("fallback")
        or not meta["is_decode"]
        or meta["seq_lens"] is None
        or meta["req_pool_indices"] is None
        or meta["seq_lens"].numel() != n
        or meta["req_pool_indices"].numel() != n
        or pool._selfcheck_budget > 0
        or pool._audit_budget > 0
        or pool._bits != 2  # only 2-bit packed storage is built; the caller's path takes the rest
    ):
        return False
    loc64 = loc.reshape(-1).to(torch.int64)
    pool._write_loc = loc64
    ops.fused_write(
        c_kv.reshape(-1, pool.kv_lora_rank),
        k_pe.reshape(-1, pool.qk_rope_head_dim),
        loc64,
        pool.write_rotation_t(layer_id),
        pool.codec(layer_id),
        pool.layer_view(layer_id),
        seq_lens=meta["seq_lens"],
        req_idx=meta["req_pool_indices"],
    )
    return True
