"""Fused cache writer semantics (test oracle only).

Restates what one call of the reference decode writer leaves in the pool
(``deployment/sglang/QuantKernel/mla_fused_writer.py:54-107`` = the upstream
``_scatter_pack_kernel`` codec plus ``_aux`` at ``:16-51``):

* codes/params of every row are written to ``codes[slot]`` / ``params[slot]``;
* ``rope[slot] = k_pe`` for ``slot > 0``;
* a protected row (``pos < P`` or ``pos >= seq - W``, valid request, ``slot > 0``)
  stores its rotated latent in BF16 at ring row ``r``, sets ``owners[r] = slot`` and
  ``rows[slot] = r``; other rows with ``slot > 0`` set ``rows[slot] = -1``.

Decode calls have no explicit positions: ``pos = seq - 1`` (``mla_fused_writer.py:40``).
"""

from __future__ import annotations

import numpy as np

from . import codec
from .window import ring_row


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 bit patterns (uint16), round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


class Pool:
    """One layer of the packed cache plus the shared slot/ring maps, as numpy arrays."""

    def __init__(self, num_slots: int, d: int, dr: int, max_reqs: int, sink: int, recent: int):
        self.d, self.dr = d, dr
        self.sink, self.recent, self.max_reqs = sink, recent, max_reqs
        self.num_slots = num_slots
        self.ring_rows = 1 + max_reqs * (sink + recent)
        self.codes = np.zeros((num_slots, d // 4), np.uint8)
        self.params = np.zeros((num_slots, d // codec.GROUP, 2), np.float32)
        self.rope = np.zeros((num_slots, dr), np.uint16)  # bf16 bits
        self.hp = np.zeros((self.ring_rows, d), np.uint16)  # bf16 bits
        self.rows = np.full((num_slots,), -1, np.int32)
        self.owners = np.zeros((self.ring_rows,), np.int32)


def write(pool: Pool, rotated: np.ndarray, kpe_bits: np.ndarray, slots, seq_lens, req_idx,
          t32, scale_factor32, positions=None, zero_const32=np.float32(codec.ZERO_CONST)):
    """Apply one writer call to ``pool`` (in place).  ``rotated`` is FP32 ``[n, D]``."""
    slots = np.asarray(slots, np.int64)
    codes, scale, zero = codec.encode(rotated, t32, scale_factor32, zero_const32)
    packed = codec.pack(codes)
    prm = codec.params_array(scale, zero)
    ok = (slots >= 0) & (slots < pool.num_slots)
    pool.codes[slots[ok]] = packed[ok]
    pool.params[slots[ok]] = prm[ok]
    live = ok & (slots > 0)
    pool.rope[slots[live]] = kpe_bits[live]
    if seq_lens is None or req_idx is None:
        return
    seq = np.asarray(seq_lens, np.int64)
    req = np.asarray(req_idx, np.int64)
    pos = seq - 1 if positions is None else np.asarray(positions, np.int64)
    keep = ((pos < pool.sink) | (pos >= seq - pool.recent)) & (req >= 0) & (req < pool.max_reqs) & live
    ring = ring_row(req, pos, pool.sink, pool.recent)
    hp_bits = bf16_bits(rotated)
    for i in np.nonzero(live)[0]:
        if keep[i]:
            pool.hp[ring[i]] = hp_bits[i]
            pool.owners[ring[i]] = slots[i]
            pool.rows[slots[i]] = ring[i]
        else:
            pool.rows[slots[i]] = -1
