"""Decode-backend shim: the packed-pool branch of SGLang's ``TritonAttnBackend``.

The reference's backend (``deployment/patches/rolaq_sglang.patch:51-72``) hands the
packed reader the request -> token map of the batch (``req_to_token_pool.req_to_token``,
``req_pool_indices``, ``seq_lens``) and per-batch scratch (``attn_logits`` / ``attn_lse``)
sized for the largest captured batch.  This reader takes 64-token pages instead, so
``init_forward_metadata`` turns the token map into a page table once per batch (one
launch, ``rolaq_page_table_from_req_to_token``, no host sync: capturable), and
``forward_decode`` runs the packed decode for one layer with preallocated scratch.
Every buffer is allocated in ``__init__``, none per batch or per layer.

The split count follows the batch, as the reference's per-batch
``forward_metadata.num_kv_splits`` under a ``max_kv_splits`` bound does
(``deployment/patches/rolaq_sglang.patch:51-72, 98-111``): the
scratch holds ``max_batch * (num_kv_splits + 1)`` partials per head, and a batch of ``b``
requests takes ``ops.default_num_splits(b, max_context_len)`` splits within that room, so one
long request is spread over the SMs instead of the few CTAs ``max_batch``'s count gives it.
An explicit ``num_kv_splits`` fixes the count for every batch.
"""

from __future__ import annotations

import math

import torch

from . import ops
from .mla_packed_decode import packed_mla_decode_gf_fwd


class PackedMLADecodeBackend:
    def __init__(self, pool, num_heads: int, max_batch: int, max_context_len: int, sm_scale: float,
                 num_kv_splits: int | None = None):
        self.pool = pool
        self.num_heads = num_heads
        self.sm_scale = float(sm_scale)
        self.max_batch = max_batch
        self.max_context_len = max_context_len
        self.max_pages = math.ceil(max_context_len / ops.PAGE)
        d, dr = pool.kv_lora_rank, pool.qk_rope_head_dim
        self.fixed_splits = bool(num_kv_splits)
        # sink + recent BF16 window rows of the pool (s4r16 unless it says otherwise)
        self.window_rows = getattr(pool, "_win_p", 4) + getattr(pool, "_win_r", 16)
        self.num_kv_splits = num_kv_splits or ops.default_num_splits(max_batch, max_context_len, latent_dim=d,
                                                                     rope_dim=dr, heads=num_heads,
                                                                     window_rows=self.window_rows)
        dev = pool.device
        self.page_table = torch.full((max_batch, self.max_pages), -1, dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.attn_logits = torch.empty(max_batch, num_heads, self.num_kv_splits + 1, d, dtype=torch.float32,
                                       device=dev)
        self.attn_lse = torch.empty(max_batch, num_heads, self.num_kv_splits + 1, dtype=torch.float32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.batch = 0
        self.splits = self.num_kv_splits

    def splits_for(self, batch: int) -> int:
        """KV splits for a batch of ``batch`` requests: the fixed count, or the default count for
        ``batch`` x ``max_context_len`` bounded by the partials the scratch holds per request."""
        if self.fixed_splits or batch <= 0:
            return self.num_kv_splits
        room = self.max_batch * (self.num_kv_splits + 1) // batch - 1
        s = ops.default_num_splits(batch, self.max_context_len, latent_dim=self.pool.kv_lora_rank,
                                   rope_dim=self.pool.qk_rope_head_dim, heads=self.num_heads,
                                   window_rows=self.window_rows)
        return max(1, min(s, room))

    def init_forward_metadata(self, req_to_token: torch.Tensor, req_pool_indices: torch.Tensor,
                              seq_lens: torch.Tensor) -> None:
        """Once per decode batch: the batch's page table and int32 lengths from the token map
        (``forward_batch.req_to_token_pool.req_to_token``, ``req_pool_indices``, ``seq_lens``).
        A page whose tokens are not one aligned run of 64 slots is marked absent and
        ``DEV_BAD_PAGE`` is set in ``self.err``."""
        b = req_pool_indices.numel()
        if b > self.max_batch:
            raise ValueError(f"batch {b} exceeds max_batch {self.max_batch}")
        if req_to_token.shape[1] < self.max_pages * ops.PAGE:
            raise ValueError("req_to_token rows are shorter than max_context_len rounded to pages")
        ops.page_table_from_req_to_token(req_to_token, req_pool_indices, seq_lens, self.page_table[:b],
                                         self.seq_lens[:b], err=self.err)
        self.batch = b
        self.splits = self.splits_for(b)

    def forward_decode(self, q: torch.Tensor, layer_id: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """One layer's decode attention: ``q`` ``[B, H * (D + Dr)]`` or ``[B, H, D + Dr]`` (rotated
        frame) -> ``[B, H, D]`` BF16."""
        b = self.batch
        d, dr = self.pool.kv_lora_rank, self.pool.qk_rope_head_dim
        q = q.view(b, self.num_heads, d + dr)
        h, parts = self.num_heads, self.splits + 1
        logits = self.attn_logits.view(-1)[: b * h * parts * d].view(b, h, parts, d)
        lse = self.attn_lse.view(-1)[: b * h * parts].view(b, h, parts)
        return packed_mla_decode_gf_fwd(q, self.pool, layer_id, self.page_table[:b], self.seq_lens[:b],
                                        self.sm_scale, self.splits, attn_logits=logits, attn_lse=lse, out=out,
                                        err=self.err)
