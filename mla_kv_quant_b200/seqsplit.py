"""Sequence-split decode of long requests across the GPUs of one node.

Each rank owns one contiguous, page-aligned slice of every request's positions
(and the cache pages of that slice).  It runs the packed decode kernel restricted
to its slice (``token_range``) and merges its own splits into one FP32 partial
``(o, lse)`` per (request, head); the ranks exchange those partials with one NCCL ``all_gather_into_tensor`` of
``B * H * (D + 4) * 4`` bytes per rank, about 33 KB for one DeepSeek-V2-Lite request.  Every rank then merges the ``world`` partials
with the same LSE kernel and holds the full output.

The reference serves one GPU only (``deployment/serve.py:135-136``); this module
is the multi-GPU extension the packed path's sharding needs.  No kernel reads
another GPU's memory: the partials cross NVLink through NCCL.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import ops


def rank_token_range(seq_len: int, world: int, rank: int, page: int = ops.PAGE) -> tuple[int, int]:
    """Contiguous page-aligned slice ``[start, end)`` of ``seq_len`` positions for ``rank``."""
    pages = (seq_len + page - 1) // page
    per = (pages + world - 1) // world
    start = min(seq_len, rank * per * page)
    end = min(seq_len, (rank + 1) * per * page)
    return start, end


def gather_merge(o_local: torch.Tensor, lse_local: torch.Tensor, group=None,
                 merge: Callable[[torch.Tensor, torch.Tensor], tuple[torch.Tensor, torch.Tensor]] | None = None):
    """All-gather per-rank partials ``o [rows, D]`` (FP32 or BF16) / ``lse [rows]`` and
    LSE-merge them.

    One collective: each rank packs its rows as ``[o (D) | lse | pad]`` (D + 4 floats, so
    rows stay 16-byte aligned) and a single ``all_gather_into_tensor`` moves them; the
    merge reads strided views of the gathered buffer.
    ``merge(parts_o [world, rows, D], parts_lse [world, rows]) -> (out, lse)``; the
    default is the CUDA merge kernel (``rolaq_merge_partials``) writing FP32.
    """
    world = dist.get_world_size(group)
    rows, d = o_local.shape
    packed = torch.zeros(rows, d + 4, dtype=torch.float32, device=o_local.device)
    packed[:, :d] = o_local  # FP32 or BF16 partials
    packed[:, d] = lse_local
    flat = torch.empty(world * rows, d + 4, dtype=torch.float32, device=o_local.device)
    dist.all_gather_into_tensor(flat, packed, group=group)
    parts = flat.view(world, rows, d + 4)
    parts_o = parts[:, :, :d]
    parts_lse = parts[:, :, d]
    if merge is not None:
        return merge(parts_o, parts_lse)
    out = torch.empty(rows, d, dtype=torch.float32, device=o_local.device)
    lse = torch.empty(rows, dtype=torch.float32, device=o_local.device)
    ops.merge_partials(parts_o, parts_lse, out_f32=out, out_lse=lse)
    return out, lse


class SequenceSplitDecoder:
    """Decode attention for requests whose pages are spread over the ranks of ``group``."""

    def __init__(self, pool, group=None):
        self.pool = pool
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def local_partial(self, q, layer_id, page_table, seq_lens, sm_scale, num_splits, token_range):
        """This rank's slice: its split partials LSE-merged in FP32, ``(o [B*H, D], lse [B*H])``.
        The partial stays FP32 through the exchange, so the final output is rounded to BF16
        once, after the cross-rank merge."""
        b, h, _ = q.shape
        d = self.pool.kv_lora_rank
        parts = num_splits + 1
        part_o = torch.empty(b, h, parts, d, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(b, h, parts, dtype=torch.float32, device=q.device)
        scratch = torch.empty(b, h, d, dtype=torch.bfloat16, device=q.device)
        ops.packed_decode(q, self.pool.layer_view(layer_id), page_table, seq_lens, sm_scale, num_splits, part_o,
                          part_lse, scratch, token_range=token_range)
        o = torch.empty(b * h, d, dtype=torch.float32, device=q.device)
        lse = torch.empty(b * h, dtype=torch.float32, device=q.device)
        ops.merge_partials(part_o.view(b * h, parts, d).transpose(0, 1), part_lse.view(b * h, parts).t(), out_f32=o,
                           out_lse=lse)
        return o, lse

    def decode(self, q, layer_id, page_table, seq_lens_host: list[int], seq_lens, sm_scale, num_splits=4):
        """``q [B, H, D + Dr]`` -> ``out [B, H, D]`` BF16 on every rank."""
        b, h, _ = q.shape
        rng = torch.tensor([rank_token_range(int(L), self.world, self.rank) for L in seq_lens_host],
                           dtype=torch.int32, device=q.device)
        o, lse = self.local_partial(q, layer_id, page_table, seq_lens, sm_scale, num_splits, rng)
        out, _ = gather_merge(o, lse, self.group)
        return out.view(b, h, -1).to(torch.bfloat16)
