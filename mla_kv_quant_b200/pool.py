"""Paged packed-INT2 MLA latent pool (the on-device format the writer and reader share).

Stands in for the upstream ``_PackedLatentMixin`` pool whose attributes the
reference writer reads (``deployment/sglang/QuantKernel/mla_fused_writer.py:117-191``)
and whose allocation and accounting the reference patch changes
(``deployment/patches/rolaq_sglang.patch:115-188``).  Per layer:

    c_codes[li]   uint8 [size, D/4]      4 codes per byte, element j at byte j/4, bits 2(j%4)
    c_params[li]  f32   [size, D/128, 2] (scale, zero)
    rope_buf[li]  bf16  [size, Dr]
    hp_c[li]      bf16  [1 + max_reqs*(P+W), D]  rotated latents of window tokens

and, shared by all layers, ``hp_row_of_slot`` int32 [size] and ``hp_owner_of_row``
int32 [ring rows].  ``size`` is a multiple of the 64-token page; slot 0 is reserved
for CUDA-graph padding.
"""

from __future__ import annotations

import torch

from . import ops
from .envs import envs
from .rolaq_mla import load_layer_quantizers


class PackedLatentPool:
    def __init__(
        self,
        size: int,
        layer_num: int,
        kv_lora_rank: int = 512,
        qk_rope_head_dim: int = 64,
        max_reqs: int = 64,
        sink: int = 4,
        recent: int = 16,
        device: str | torch.device = "cuda",
        rotations: dict[int, torch.Tensor] | None = None,
        quantizer_params: list | None = None,
        start_layer: int = 0,
        lloyd_max: bool = True,
        bits: int = 2,
        group_size: int = 128,
    ):
        if size % ops.PAGE:
            raise ValueError(f"pool size must be a multiple of {ops.PAGE} slots")
        if kv_lora_rank % group_size or group_size != 128:
            raise ValueError("kv_lora_rank must be a multiple of the 128 group")
        if quantizer_params is not None and (not lloyd_max or bits != 2):
            raise ValueError("RoLaQ requires SGLANG_LLOYD_MAX=1 and INT2 packed storage")
        self.size = size
        self.layer_num = layer_num
        self.start_layer = start_layer
        self.kv_lora_rank = kv_lora_rank
        self.qk_rope_head_dim = qk_rope_head_dim
        self.dtype = torch.bfloat16
        self.device = torch.device(device)
        self._max_reqs = max_reqs
        self._win_p = sink
        self._win_r = recent
        self._latent_windows = (sink + recent) > 0
        self._lloyd_max = lloyd_max
        self._bits = bits
        self._group_size = group_size
        self._selfcheck_budget = 0
        self._audit_budget = 0
        self._fb_window_meta = None
        self._rolaq_fused_decode_write = bool(envs.SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE.get())
        d, dr, ng = kv_lora_rank, qk_rope_head_dim, kv_lora_rank // group_size
        ring = 1 + max_reqs * (sink + recent)
        dev = self.device
        self._codes = torch.zeros(layer_num, size, d // 4, dtype=torch.uint8, device=dev)
        self._params = torch.zeros(layer_num, size, ng, 2, dtype=torch.float32, device=dev)
        self._rope = torch.zeros(layer_num, size, dr, dtype=torch.bfloat16, device=dev)
        self._hp = torch.zeros(layer_num, ring, d, dtype=torch.bfloat16, device=dev)
        self.c_codes = list(self._codes.unbind(0))
        self.c_params = list(self._params.unbind(0))
        self.rope_buf = list(self._rope.unbind(0))
        self.hp_c = list(self._hp.unbind(0))
        self.hp_row_of_slot = torch.full((size,), -1, dtype=torch.int32, device=dev)
        self.hp_owner_of_row = torch.zeros(ring, dtype=torch.int32, device=dev)
        self.rotations = dict(rotations or {})
        self._rolaq_quantizers = list(quantizer_params) if quantizer_params is not None else [None] * layer_num
        self._rot_t: dict[int, tuple[int, torch.Tensor]] = {}
        self._identity_t: torch.Tensor | None = None

    # ---- construction from the reference's environment flags ---------------------------
    @classmethod
    def from_env(cls, size: int, layer_num: int, **kw):
        """Read the artifact paths and window sizes the reference server sets
        (``deployment/serve.py:95-122``, ``rolaq_sglang.patch:41-47, 123-133``)."""
        import torch as _t

        rotation_path = envs.SGLANG_OSCAR_MLA_KV_ROTATION_PATH.get()
        quantizer_path = envs.SGLANG_ROLAQ_MLA_QUANTIZER_PATH.get()
        lloyd = bool(envs.SGLANG_LLOYD_MAX.get())
        bits = int(envs.SGLANG_OSCAR_MLA_KV_BITS.get())
        group = int(envs.SGLANG_OSCAR_MLA_KV_GROUP_SIZE.get())
        sink = int(envs.SGLANG_MIXED_KV_PREFIX_TOKENS.get())
        recent = int(envs.SGLANG_MIXED_KV_RECENT_TOKENS.get())
        if not rotation_path:
            raise ValueError("Packed MLA latent storage needs a rotation path (SGLANG_OSCAR_MLA_KV_ROTATION_PATH)")
        start = kw.pop("start_layer", 0)
        layer_ids = list(range(start, start + layer_num))
        rotations = {
            i: _t.load(f"{rotation_path}/layer_{i}.pt", map_location="cpu", weights_only=True) for i in layer_ids
        }
        d = kw.get("kv_lora_rank", 512)
        if quantizer_path and (not lloyd or bits != 2):
            raise ValueError("RoLaQ requires SGLANG_LLOYD_MAX=1 and INT2 packed storage")
        params = load_layer_quantizers(quantizer_path, rotation_path, group, d, layer_ids)
        return cls(size, layer_num, sink=sink, recent=recent, rotations=rotations, quantizer_params=params,
                   start_layer=start, lloyd_max=lloyd, bits=bits, group_size=group, **kw)

    # ---- rotation access used by the writer (mla_fused_writer.py:137-147) ----------------
    def latent_rotation(self, layer_id: int, local: bool = True) -> torch.Tensor | None:
        """The artifact's FP32 rotation of ``layer_id`` (global layer id)."""
        return self.rotations.get(layer_id)

    def write_rotation_t(self, layer_id: int) -> torch.Tensor:
        """``bf16(R)^T`` on the pool device, cached per layer (the tcgen05 B operand).  A
        layer without a rotation gets the identity: the writer then stores ``c = c_kv``
        exactly (BF16 values times 1 accumulate exactly in FP32), as the reference's
        writer does without a rotation (``mla_fused_writer.py:146-149``)."""
        r = self.latent_rotation(layer_id)
        if r is None:
            if self._identity_t is None:
                self._identity_t = torch.eye(self.kv_lora_rank, dtype=torch.bfloat16, device=self.device)
            return self._identity_t
        cached = self._rot_t.get(layer_id)
        if cached is None or cached[0] != id(r):
            rt = r.to(device=self.device, dtype=torch.bfloat16).t().contiguous()
            cached = (id(r), rt)
            self._rot_t[layer_id] = cached
        return cached[1]

    def layer_view(self, layer_id: int) -> ops.LayerView:
        li = layer_id - self.start_layer
        return ops.LayerView(self.c_codes[li], self.c_params[li], self.rope_buf[li], self.hp_c[li],
                             self.hp_row_of_slot, self.hp_owner_of_row, self._win_p, self._win_r, self._max_reqs)

    def codec(self, layer_id: int):
        """Serving-path codec of a layer: the learned Lloyd scalars, the Lloyd-Max defaults,
        or OSCAR's uniform min/max codec when the pool runs without Lloyd-Max."""
        if not self._lloyd_max:
            return ops.codec_uniform()
        li = layer_id - self.start_layer
        params = self._rolaq_quantizers[li]
        if params is None:
            return ops.codec_serving(ops.LLOYD_MAX_THRESHOLDS[2], ops.LLOYD_MAX_STRETCH)
        return ops.codec_serving(params[0], params[1])

    # ---- window metadata for one forward (the reference's _fb_window_meta) ---------------
    def set_window_meta(self, is_decode: bool, seq_lens: torch.Tensor | None, req_pool_indices: torch.Tensor | None,
                        fallback: bool = False) -> None:
        self._fb_window_meta = {"is_decode": is_decode, "seq_lens": seq_lens, "req_pool_indices": req_pool_indices,
                                "fallback": fallback}

    # ---- writes ------------------------------------------------------------------------------
    def set_kv_buffer(self, layer_id: int, loc: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor,
                      positions: torch.Tensor | None = None) -> None:
        """Write new latents (``rolaq_sglang.patch:149-164``): the fused decode writer
        when enabled and applicable, else the fused writer with explicit positions
        (prefill) through the same tcgen05 kernel."""
        if self._rolaq_fused_decode_write:
            from .mla_fused_writer import try_fast_decode_store

            if try_fast_decode_store(self, layer_id, loc, c_kv, k_pe):
                return
        meta = self._fb_window_meta or {}
        view = self.layer_view(layer_id)
        x = c_kv.reshape(-1, self.kv_lora_rank)
        pe = k_pe.reshape(-1, self.qk_rope_head_dim)
        ops.fused_write(x, pe, loc.reshape(-1).to(torch.int64), self.write_rotation_t(layer_id), self.codec(layer_id),
                        view, seq_lens=meta.get("seq_lens"), req_idx=meta.get("req_pool_indices"),
                        positions=positions)

    # ---- accounting (rolaq_sglang.patch:166-188) ------------------------------------------
    def cell_size_bytes(self) -> int:
        """Bytes per token slot over all layers, plus the shared 4-byte ring map entry."""
        d, dr = self.kv_lora_rank, self.qk_rope_head_dim
        per_layer = d // 4 + (d // self._group_size) * 8 + dr * 2
        return per_layer * self.layer_num + 4

    def fixed_overhead_bytes(self) -> int:
        """The BF16 window arena: (1 + max_reqs*(P+W)) rows per layer plus owner entries."""
        ring = 1 + self._max_reqs * (self._win_p + self._win_r)
        return ring * (self.kv_lora_rank * 2 * self.layer_num + 4)

    def get_kv_size_bytes(self) -> int:
        return self.cell_size_bytes() * self.size + self.fixed_overhead_bytes()
