"""The sink/recent window lifecycle of the HF fake-quantized latent cache, on the GPU.

Restates, for the learned latent quantizer (``LearnedRotationQuantizer``) and the
``nope`` component, what ``FakeQuantizedDynamicCache.update`` does in the reference
(``mla_quant/cache.py:1007-1060``):

* every token has a target state per append (``_target_window_state``, ``cache.py:
  775-800``): 0 = padding, 1 = high precision (the first ``sink`` valid tokens of the row or
  its last ``recent`` valid tokens), 2 = quantized;
* appended rows whose target is 2 are quantize-dequantized on arrival; rows in the window
  stay as given (``_apply_window_to_new``, ``cache.py:819-845``: the selected rows of all
  batch elements go to the quantizer in one call);
* a row that leaves the recent window (state 1 -> 2) is quantize-dequantized then, once
  (``_requantize_rows``, ``cache.py:949-965``); a state never goes back from 2 to 1
  (``target = max(target, old_state)``).

The quantize-dequantize itself is ``LearnedRotationQuantizer.quantize_layer`` (the tcgen05
rotation, the Lloyd INT2 codec and the un-rotation of this package).  Counters follow the
reference's window statistics (``transitions_hp_to_quantized``, ``requantized_rows``).
"""

from __future__ import annotations

import torch


class WindowedLatentCache:
    def __init__(self, quantizer, sink_tokens: int = 4, recent_tokens: int = 16,
                 pad_mask: torch.Tensor | None = None):
        self.quantizer = quantizer
        self.sink_tokens = int(sink_tokens)
        self.recent_tokens = int(recent_tokens)
        self.pad_mask = pad_mask  # [B, T] bool, True = real token (left padding), or None
        self.keys: dict[int, torch.Tensor] = {}
        self.row_state: dict[int, torch.Tensor] = {}
        self.stats = {"transitions_hp_to_quantized": 0, "requantized_rows": 0, "updates": 0}

    def get_seq_length(self, layer_idx: int = 0) -> int:
        k = self.keys.get(layer_idx)
        return 0 if k is None else int(k.shape[-2])

    def _valid(self, full_len: int, batch: int, device) -> torch.Tensor:
        """``cache.py:760-772``: all valid, or the last ``full_len`` columns of the pad mask."""
        m = self.pad_mask
        if m is None or m.shape[0] != batch or m.shape[1] < full_len:
            return torch.ones(batch, full_len, dtype=torch.bool, device=device)
        return m[:, -full_len:].to(device=device, dtype=torch.bool)

    def target_state(self, full_len: int, batch: int, device) -> torch.Tensor:
        """``cache.py:775-800``: uint8 ``[B, full_len]`` (0 pad, 1 high precision, 2 quantized)."""
        valid = self._valid(full_len, batch, device)
        state = valid.to(torch.uint8) * 2
        mark = torch.zeros_like(valid)
        if self.sink_tokens:
            mark |= valid & (valid.to(torch.int64).cumsum(-1) <= self.sink_tokens)
        if self.recent_tokens:
            mark |= valid & (valid.flip(-1).to(torch.int64).cumsum(-1).flip(-1) <= self.recent_tokens)
        state.masked_fill_(mark, 1)
        return state

    def _qdq_rows(self, tensor: torch.Tensor, layer_idx: int, mask: torch.Tensor) -> torch.Tensor:
        """Quantize-dequantize the rows of ``tensor`` ``[B, ..., L, D]`` selected by ``mask``
        ``[B, L]``, all batch elements in one quantizer call (``cache.py:831-845``)."""
        b, length, d = tensor.shape[0], tensor.shape[-2], tensor.shape[-1]
        head_shape = tensor.shape[1:-2]
        expanded = mask.reshape(b, *[1] * len(head_shape), length).expand(tensor.shape[:-1]).reshape(-1)
        flat = tensor.reshape(-1, d)
        selected = flat[expanded]
        if selected.numel() == 0:
            return tensor
        quantized = self.quantizer.quantize_layer(selected.reshape(-1, d), layer_idx, "nope")
        out = flat.clone()
        out[expanded] = quantized.reshape(-1, d)
        return out.reshape_as(tensor)

    def update(self, latent: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Append ``latent`` ``[B, ..., L_new, D]`` to the layer and return the whole cached
        latent with the window rules applied (``cache.py:1007-1060``)."""
        past = self.keys.get(layer_idx)
        past_len = 0 if past is None else int(past.shape[-2])
        new_len = int(latent.shape[-2])
        full_len = past_len + new_len
        batch = int(latent.shape[0])
        target = self.target_state(full_len, batch, latent.device)
        latent = self._qdq_rows(latent, layer_idx, target[:, past_len:full_len] == 2)
        keys = latent if past is None else torch.cat([past, latent], dim=-2)
        old = self.row_state.get(layer_idx)
        if old is not None and past_len > 0:
            if old.shape[0] != batch or old.shape[1] < past_len:
                raise RuntimeError(f"sink/recent row state shape does not match the cache: "
                                   f"state={tuple(old.shape)} batch={batch} past_len={past_len}")
            target[:, :past_len] = torch.maximum(target[:, :past_len], old[:, :past_len])
            transition = (old[:, :past_len] == 1) & (target[:, :past_len] == 2)
            full = torch.cat([transition, torch.zeros(batch, new_len, dtype=torch.bool, device=keys.device)], -1)
            keys = self._qdq_rows(keys, layer_idx, full)
            count = int(transition.sum().item())
            self.stats["transitions_hp_to_quantized"] += count
            self.stats["requantized_rows"] += count
        self.keys[layer_idx] = keys
        self.row_state[layer_idx] = target
        self.stats["updates"] += 1
        return keys
