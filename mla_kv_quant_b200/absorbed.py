"""The absorbed-MLA projections on either side of the packed decode (drop-in for the
DeepSeek MLA forward's ``torch.bmm`` calls that ``deployment/patches/rolaq_sglang.patch``
wraps around the packed reader).

With the read rotation folded into the ``kv_b_proj`` weight (``fold_read_rotation``,
``deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71``, applied by the weight loader at
``rolaq_sglang.patch:261-270``) the decode's query is ``[q_nope @ W_kc', q_pe]`` and its
output ``o`` needs only ``o @ W_vc'`` (``rolaq_sglang.patch:205-248``): no rotation runs at
decode time.  ``absorb_query`` builds the query (the bmm and the concat in one launch) and
``project_output`` applies ``W_vc'``, both on tcgen05 with FP32 accumulation.
"""

from __future__ import annotations

import torch

from . import ops


def split_absorbed_weights(w: torch.Tensor, heads: int, qk_nope_head_dim: int, v_head_dim: int):
    """``kv_b_proj`` weight ``[H * (Dn + Dv), D]`` (after ``fold_read_rotation``) -> ``(w_kc, w_vc)``
    in the layouts SGLang's DeepSeek loader keeps for its bmm: ``w_kc`` stored ``[H, D, Dn]``
    and ``w_vc`` stored ``[H, Dv, D]``, each contiguous (the reduced dimension last)."""
    d = w.shape[-1]
    w3 = w.view(heads, qk_nope_head_dim + v_head_dim, d)
    w_kc = w3[:, :qk_nope_head_dim, :].transpose(1, 2).contiguous()
    w_vc = w3[:, qk_nope_head_dim:, :].contiguous()
    return w_kc, w_vc


def absorb_query(q_nope: torch.Tensor, q_pe: torch.Tensor | None, w_kc: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``[q_nope @ w_kc^T | q_pe]`` per head: ``[B, H, Dn]``, ``[B, H, Dr]`` -> ``[B, H, D + Dr]`` BF16."""
    b, h, _ = q_nope.shape
    dr = 0 if q_pe is None else q_pe.shape[-1]
    if out is None:
        out = torch.empty(b, h, w_kc.shape[1] + dr, dtype=torch.bfloat16, device=q_nope.device)
    ops.absorb_query(q_nope, q_pe, w_kc, out)
    return out


def project_output(o: torch.Tensor, w_vc: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``o @ w_vc^T`` per head: ``[B, H, D]`` -> ``[B, H, Dv]`` BF16."""
    b, h, _ = o.shape
    if out is None:
        out = torch.empty(b, h, w_vc.shape[1], dtype=torch.bfloat16, device=o.device)
    ops.project_output(o, w_vc, out)
    return out
