"""The absorbed-query and output-projection kernels against an FP32 torch composition of
the same BF16 operands (the reference's torch.bmm path, deployment/patches/
rolaq_sglang.patch:205-248): BF16 outputs within half a BF16 ulp of the FP32 value plus
1e-4 of the row's scale (accumulation order), for the DeepSeek-V2-Lite and MiniCPM3 shapes,
batches below, at and above one 128-row tile."""

import numpy as np
import pytest
import torch

from mla_kv_quant_b200 import absorbed, synth
from mla_kv_quant_b200.rolaq_mla import fold_read_rotation

pytestmark = pytest.mark.gpu


def _close(out, ref, scale):
    ref = ref.double().cpu().numpy()
    got = out.double().cpu().numpy()
    half_ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 8)
    assert np.max(np.abs(got - ref) - half_ulp - 1e-4 * scale) <= 0


@pytest.mark.parametrize("b,h,dn,d,dr,dv", [(64, 16, 128, 512, 64, 128), (128, 40, 64, 256, 32, 64),
                                              (3, 16, 128, 512, 64, 128), (200, 16, 128, 512, 64, 128)])
def test_absorbed_projections_match_fp32(b, h, dn, d, dr, dv):
    dev = "cuda"
    w = (synth.normal_bf16((h * (dn + dv), d), seed=5, device=dev).float() * 0.05).to(torch.bfloat16)
    w_kc, w_vc = absorbed.split_absorbed_weights(w, h, dn, dv)
    q_nope = synth.normal_bf16((b, h, dn), seed=6, device=dev)
    q_pe = synth.normal_bf16((b, h, dr), seed=7, device=dev)
    q = absorbed.absorb_query(q_nope, q_pe, w_kc)
    o = synth.normal_bf16((b, h, d), seed=8, device=dev)
    y = absorbed.project_output(o, w_vc)
    torch.cuda.synchronize()
    ref_q = torch.einsum("bhk,hnk->bhn", q_nope.float(), w_kc.float())
    scale_q = float((q_nope.float().abs().sum(-1).max() * w_kc.float().abs().max()).item())
    _close(q[..., :d], ref_q, scale_q)
    assert torch.equal(q[..., d:], q_pe)
    ref_y = torch.einsum("bhe,hve->bhv", o.float(), w_vc.float())
    scale_y = float((o.float().abs().sum(-1).max() * w_vc.float().abs().max()).item())
    _close(y, ref_y, scale_y)


def test_absorbed_query_in_rotated_frame(tmp_path):
    """With the read rotation folded into the weight, the absorbed query equals the rotated
    query of the unfolded weight (rolaq_mla.py:56-71): (q_nope W_kc) R up to BF16 rounding."""
    from mla_kv_quant_b200.artifacts import write_synthetic_artifact

    h, dn, dv, d = 4, 128, 128, 512
    r = synth.rotation(d, seed=9)
    write_synthetic_artifact(tmp_path, {0: r}, {0: (0.8, 1.0)}, {"model_type": "deepseek_v2"})
    w = (synth.normal_bf16((h * (dn + dv), d), seed=10).float() * 0.05).to(torch.bfloat16)
    wf = fold_read_rotation(w.cuda(), 0, str(tmp_path))
    w_kc, _ = absorbed.split_absorbed_weights(wf, h, dn, dv)
    q_nope = synth.normal_bf16((8, h, dn), seed=11, device="cuda")
    q = absorbed.absorb_query(q_nope, None, w_kc)
    w_kc0, _ = absorbed.split_absorbed_weights(w.cuda(), h, dn, dv)
    ref = torch.einsum("bhk,hnk->bhn", q_nope.float(), w_kc0.float()) @ r.cuda().to(torch.bfloat16).float()
    rel = (q.float() - ref).norm() / ref.norm()
    assert rel.item() < 1e-2
