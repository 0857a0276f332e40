"""Sink/recent window rules (test oracle only).

* ``target_state`` restates ``FakeQuantizedDynamicCache._target_window_state``
  (``mla_quant/cache.py:775-800``): 0 = padding, 1 = BF16 (first ``sink`` valid or
  last ``recent`` valid tokens), 2 = INT2.
* ``ring_row`` restates the ring placement of the fused writer's ``_aux``
  (``deployment/sglang/QuantKernel/mla_fused_writer.py:36-51``).
* ``protected`` is the per-position window test that both rules share for an
  unpadded request of length ``seq_len``.
"""

from __future__ import annotations

import numpy as np

# mla_quant/common.py:16
WINDOWS = {"nowin": (0, 0), "s4r8": (4, 8), "s4r16": (4, 16)}


def target_state(valid: np.ndarray, sink: int, recent: int) -> np.ndarray:
    """valid bool ``[B, L]`` -> uint8 state ``[B, L]``."""
    valid = np.asarray(valid, bool)
    state = valid.astype(np.uint8) * 2
    if sink:
        from_start = np.cumsum(valid.astype(np.int64), axis=-1)
        sink_mask = valid & (from_start <= sink)
    else:
        sink_mask = np.zeros_like(valid)
    if recent:
        from_end = np.cumsum(valid[:, ::-1].astype(np.int64), axis=-1)[:, ::-1]
        recent_mask = valid & (from_end <= recent)
    else:
        recent_mask = np.zeros_like(valid)
    state[sink_mask | recent_mask] = 1
    return state


def protected(pos, seq_len, sink: int, recent: int):
    """True where position ``pos`` of a length-``seq_len`` request is kept in BF16."""
    pos = np.asarray(pos)
    return (pos < sink) | (pos >= np.asarray(seq_len) - recent)


def ring_row(req, pos, sink: int, recent: int):
    """Ring index ``1 + req*(P+W) + (pos < P ? pos : P + (pos-P) mod W)``.

    Row 0 of the ring is never used (it backs CUDA-graph padding).
    """
    req = np.asarray(req, np.int64)
    pos = np.asarray(pos, np.int64)
    w = max(recent, 1)
    inner = np.where(pos < sink, pos, sink + np.maximum(pos - sink, 0) % w)
    return 1 + req * (sink + recent) + inner
