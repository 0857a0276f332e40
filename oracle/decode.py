"""Absorbed MLA decode attention over the packed INT2 cache (test oracle only).

Restates the math of the reference serving read path:

* queries arrive in the rotated latent frame: ``q_nope_out = q_nope @ (W_kc R)``
  because ``fold_read_rotation`` folded ``R`` into ``W_b``
  (``deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71``,
  ``deployment/patches/rolaq_sglang.patch:225-232, 261-270``), so
  ``q = [q_lat (D) | q_pe (Dr)]``;
* the key of a token is ``[c_hat | k_pe]`` and its value is ``c_hat``, where ``c_hat``
  is the INT2-dequantized rotated latent, or the BF16 ring row for window tokens
  whose ring row still belongs to them (``hp_row_of_slot`` / ``hp_owner_of_row``,
  ``mla_fused_writer.py:49-51``);
* ``out = softmax(q . k * sm_scale) @ v`` per head, left in the rotated frame
  (``rolaq_sglang.patch:243-248``: the un-rotation is folded into ``w_vc``);
* split-KV partials ``(lse, o)`` are merged by log-sum-exp
  (``rolaq_sglang.patch:81-111``).
"""

from __future__ import annotations

import numpy as np

from . import codec
from .writer import bf16_to_f32

PAGE = 64


def token_slots(page_table_row: np.ndarray, seq_len: int) -> np.ndarray:
    pos = np.arange(seq_len, dtype=np.int64)
    return page_table_row[pos // PAGE].astype(np.int64) * PAGE + pos % PAGE


def latent_rows(pool, slots: np.ndarray, seq_len: int, dtype=np.float64, use_window=True) -> np.ndarray:
    """Keys/values ``c_hat`` of one request's tokens, ``[seq_len, D]``."""
    d = pool.d
    codes = codec.unpack(pool.codes[slots], d)
    prm = pool.params[slots]
    lat = codec.dequant(codes, prm[..., 0], prm[..., 1]).astype(dtype)
    if use_window and (pool.sink or pool.recent):
        pos = np.arange(seq_len)
        prot = (pos < pool.sink) | (pos >= seq_len - pool.recent)
        for p in np.nonzero(prot)[0]:
            s = slots[p]
            r = int(pool.rows[s])
            if r >= 0 and int(pool.owners[r]) == int(s):
                lat[p] = bf16_to_f32(pool.hp[r]).astype(dtype)
    return lat


def attend(q: np.ndarray, lat: np.ndarray, pe: np.ndarray, sm_scale: float):
    """One request: q ``[H, D+Dr]`` -> (out ``[H, D]``, lse ``[H]``) in q's dtype."""
    d = lat.shape[1]
    if lat.shape[0] == 0:
        return np.zeros((q.shape[0], d), q.dtype), np.full((q.shape[0],), -np.inf, q.dtype)
    s = (q[:, :d] @ lat.T + q[:, d:] @ pe.T) * sm_scale
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    out = (p @ lat) / l
    return out, (m + np.log(l))[:, 0]


def decode(pool, q_bits: np.ndarray, page_table: np.ndarray, seq_lens, sm_scale: float,
           dtype=np.float64, requests=None):
    """Reference output for every request: (out ``[B, H, D]``, lse ``[B, H]``)."""
    q = bf16_to_f32(q_bits).astype(dtype)
    b_all = q.shape[0]
    reqs = range(b_all) if requests is None else requests
    out = np.zeros((b_all, q.shape[1], pool.d), dtype)
    lse = np.full((b_all, q.shape[1]), -np.inf, dtype)
    for b in reqs:
        L = int(seq_lens[b])
        slots = token_slots(page_table[b], L)
        lat = latent_rows(pool, slots, L, dtype)
        pe = bf16_to_f32(pool.rope[slots]).astype(dtype)
        out[b], lse[b] = attend(q[b], lat, pe, sm_scale)
    return out, lse


def merge(parts_o: np.ndarray, parts_lse: np.ndarray):
    """LSE merge over axis 0: parts_o ``[S, ..., D]`` (normalised), parts_lse ``[S, ...]``."""
    m = np.max(parts_lse, axis=0)
    safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(parts_lse - safe)
    den = w.sum(axis=0)
    num = (w[..., None] * parts_o).sum(axis=0)
    out = np.where(den[..., None] > 0, num / np.where(den > 0, den, 1)[..., None], 0.0)
    lse = np.where(den > 0, safe + np.log(np.where(den > 0, den, 1)), -np.inf)
    return out, lse
