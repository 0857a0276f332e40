"""Sequence-split decode of long requests across the GPUs of one node.

Each rank owns one contiguous, page-aligned slice of every request's positions (and the
cache pages of that slice).  It runs the packed decode kernel restricted to its slice
(``token_range``) and merges its own splits into one FP32 partial ``(o, lse)`` per
(request, head): ``B * H * (D + 4) * 4`` bytes per rank, about 33 KB for one
DeepSeek-V2-Lite request.  The ranks exchange those partials in one of two ways.
``PeerExchange`` has the merging kernel store them into every rank's receive buffer over
NVLink (CUDA IPC mappings) and a bounded wait collect them.  Otherwise one NCCL
``all_gather_into_tensor`` moves them.  Every rank then merges the ``world`` partials with
the same LSE kernel and holds the full output.  Without a process group the decoder runs
on one GPU holding the whole request.

The reference serves one GPU only (``deployment/serve.py:135-136``); this module is the
multi-GPU extension the packed path's sharding needs.  No kernel reads another GPU's
memory: the exchange writes to peers and reads its own receive buffer.
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


def _distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


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
    world = dist.get_world_size(group) if _distributed() else 1  # no process group: one rank
    rows, d = o_local.shape
    packed = torch.zeros(rows, d + 4, dtype=torch.float32, device=o_local.device)
    packed[:, :d] = o_local  # FP32 or BF16 partials
    packed[:, d] = lse_local
    if world > 1:
        flat = torch.empty(world * rows, d + 4, dtype=torch.float32, device=o_local.device)
        dist.all_gather_into_tensor(flat, packed, group=group)
    else:
        flat = packed
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

    def __init__(self, pool, group=None, exchange: "PeerExchange | None" = None):
        """``exchange``: a :class:`PeerExchange` of the same group moves the partials over NVLink
        peer memory; without one they go through one NCCL all-gather."""
        self.pool = pool
        self.group = group
        self.world = dist.get_world_size(group) if _distributed() else 1  # no process group: one GPU
        self.rank = dist.get_rank(group) if _distributed() else 0
        self.exchange = exchange

    def local_partial(self, q, layer_id, page_table, seq_lens, sm_scale, num_splits, token_range):
        """This rank's slice: its split partials LSE-merged in FP32, ``(o [B*H, D], lse [B*H])``.
        The partial stays FP32 through the exchange, so the final output is rounded to BF16
        once, after the cross-rank merge."""
        b, h, _ = q.shape
        d = self.pool.kv_lora_rank
        parts = num_splits + 1
        part_o = torch.empty(b, h, parts, d, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(b, h, parts, dtype=torch.float32, device=q.device)
        ops.packed_decode(q, self.pool.layer_view(layer_id), page_table, seq_lens, sm_scale, num_splits, part_o,
                          part_lse, None, token_range=token_range)  # the partials only: merged below in FP32
        o = torch.empty(b * h, d, dtype=torch.float32, device=q.device)
        lse = torch.empty(b * h, dtype=torch.float32, device=q.device)
        ops.merge_partials(part_o.view(b * h, parts, d).transpose(0, 1), part_lse.view(b * h, parts).t(), out_f32=o,
                           out_lse=lse)
        return o, lse

    def decode(self, q, layer_id, page_table, seq_lens_host: list[int], seq_lens, sm_scale,
               num_splits: int | None = None):
        """``q [B, H, D + Dr]`` -> ``out [B, H, D]`` BF16 on every rank.  ``num_splits`` (INT2
        splits per request of this rank's slice) defaults to ``ops.default_num_splits`` for
        the batch and the longest slice of this rank."""
        b, h, _ = q.shape
        ranges = [rank_token_range(int(L), self.world, self.rank) for L in seq_lens_host]
        if num_splits is None:
            longest = max([e - s for s, e in ranges] + [1])
            num_splits = ops.default_num_splits(b, longest, latent_dim=self.pool.kv_lora_rank,
                                                rope_dim=self.pool.qk_rope_head_dim, heads=h,
                                                window_rows=getattr(self.pool, "_win_p", 4)
                                                + getattr(self.pool, "_win_r", 16))
        rng = torch.tensor(ranges, dtype=torch.int32, device=q.device)
        if self.exchange is not None:
            d = self.pool.kv_lora_rank
            part_o = torch.empty(b, h, num_splits + 1, d, dtype=torch.float32, device=q.device)
            part_lse = torch.empty(b, h, num_splits + 1, dtype=torch.float32, device=q.device)
            ops.packed_decode(q, self.pool.layer_view(layer_id), page_table, seq_lens, sm_scale, num_splits, part_o,
                              part_lse, None, token_range=rng)  # the partials only: the push merges them
            out = torch.empty(b, h, d, dtype=torch.bfloat16, device=q.device)
            self.exchange.exchange(part_o, part_lse, out_bf16=out)
            return out
        o, lse = self.local_partial(q, layer_id, page_table, seq_lens, sm_scale, num_splits, rng)
        out, _ = gather_merge(o, lse, self.group)
        return out.view(b, h, -1).to(torch.bfloat16)


class PeerExchange:
    """The sequence-split exchange over NVLink peer memory (``rolaq_peer_merge_push`` /
    ``rolaq_peer_wait_merge``), in place of the NCCL all-gather of :func:`gather_merge`.

    Every rank owns one receive buffer (``rolaq_device_alloc``) mapped into every other rank
    with CUDA IPC; the kernel that merges a rank's splits writes the rank's FP32 partial
    straight into all of them and flags it, and the final merge waits (bounded) for every
    rank's flag.  Construction is collective (one ``all_gather_object`` of the IPC handles and
    a barrier); :meth:`close` is collective too.  ``rows`` bounds ``batch * heads``."""

    def __init__(self, rows: int, latent_dim: int, group=None, device: torch.device | None = None):
        import ctypes

        from . import _lib

        self.group = group
        self._dist = dist.is_available() and dist.is_initialized()  # a single rank needs no process group
        self.world = dist.get_world_size(group) if self._dist else 1
        self.rank = dist.get_rank(group) if self._dist else 0
        self.rows, self.d = rows, latent_dim
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nbytes = lib.rolaq_peer_recv_bytes(self.world, rows, latent_dim)
        if nbytes <= 0:
            raise ValueError(f"no exchange for latent_dim {latent_dim}, rows {rows}")
        own = ctypes.c_void_p()
        _lib.call("rolaq_device_alloc", nbytes, ctypes.byref(own))
        self._own = own.value
        handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
        _lib.call("rolaq_ipc_get_handle", self._own, handle)
        handles: list = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened, ptrs = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            _lib.call("rolaq_ipc_open", (ctypes.c_char * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h), ctypes.byref(p))
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=dev)  # addresses as seen by this process
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        if self.world > 1:
            dist.barrier(group)  # every rank holds every mapping before any push

    def exchange(self, part_o: torch.Tensor, part_lse: torch.Tensor, out_bf16: torch.Tensor | None = None,
                 out_f32: torch.Tensor | None = None, out_lse: torch.Tensor | None = None,
                 err: torch.Tensor | None = None) -> None:
        """``part_o [B, H, parts, D]`` / ``part_lse [B, H, parts]`` (a token-range decode's
        split partials, contiguous) -> the merged output of all ranks, ``[B, H, D]``."""
        from . import _lib

        b, h, parts, d = part_o.shape
        rows = b * h
        if d != self.d or rows > self.rows or not part_o.is_contiguous() or not part_lse.is_contiguous():
            raise ValueError("partials must be contiguous [B, H, parts, D] with B * H <= rows")
        if part_o.dtype != torch.float32 or part_lse.dtype != torch.float32 or tuple(part_lse.shape) != (b, h, parts):
            raise ValueError("part_o / part_lse must be float32 [B, H, parts, D] / [B, H, parts]")
        dev = self.peers.device
        for name, t, dt, n in (("part_o", part_o, None, None), ("out_bf16", out_bf16, torch.bfloat16, rows * d),
                               ("out_f32", out_f32, torch.float32, rows * d), ("out_lse", out_lse, torch.float32, rows)):
            if t is None:
                continue
            if t.device != dev:
                raise ValueError(f"{name} must be on {dev}")
            if dt is not None and (t.dtype != dt or t.numel() != n or not t.is_contiguous()):
                raise ValueError(f"{name} must be contiguous {dt} with {n} elements")
        _lib.call("rolaq_peer_merge_push", part_o.data_ptr(), part_lse.data_ptr(), parts, rows, d,
                  self.peers.data_ptr(), self.world, self.rank, self.state.data_ptr(), _lib.stream_ptr())
        _lib.call("rolaq_peer_wait_merge", self._own, self.world, rows, d, self.state.data_ptr(),
                  _lib.ptr(out_bf16), _lib.ptr(out_f32), _lib.ptr(out_lse), _lib.ptr(err), _lib.stream_ptr())

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's, once no rank writes."""
        from . import _lib

        if self._own is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(self.group)
        for p in self._opened:
            _lib.call("rolaq_ipc_close", p)
        self._opened = []
        if self.world > 1:
            dist.barrier(self.group)
        _lib.call("rolaq_device_free", self._own)
        self._own = None
