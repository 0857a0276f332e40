"""The LSE merge of many partials (16 or more: a long request with many KV splits, or one slice
of a sequence-split request), which spreads each row over 128-column chunks and the partials
over a CTA's warps.  Checked against the oracle's merge (FP64) and, through the decode call,
against the oracle's decode; the split merge inside the decode call, the generic merge and the
peer exchange's merge give bit-identical FP32 results on the same partials."""

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, bits, cosine, fill_requests
from mla_kv_quant_b200 import ops, synth
from mla_kv_quant_b200.seqsplit import PeerExchange
from oracle import decode as odecode

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("parts,rows,d", [(129, 16, 512), (33, 40, 256), (16, 3, 200), (300, 2, 512)])
def test_merge_many_parts_matches_oracle(parts, rows, d):
    rng = np.random.default_rng(parts + rows)
    o = rng.standard_normal((parts, rows, d)).astype(np.float32)
    lse = (rng.standard_normal((parts, rows)) * 3).astype(np.float32)
    lse[1::7, 0] = -np.inf  # empty splits: their values are garbage and must not be read
    o[1::7, 0] = np.nan
    lse[:, rows - 1] = -np.inf  # a row with no tokens at all
    out = torch.full((rows, d), float("nan"), device="cuda")
    out16 = torch.full((rows, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    out_lse = torch.full((rows,), float("nan"), device="cuda")
    po, pl = torch.from_numpy(o).cuda(), torch.from_numpy(lse).cuda()
    ops.merge_partials(po, pl, out_f32=out, out_lse=out_lse)
    ops.merge_partials(po, pl, out_bf16=out16)
    torch.cuda.synchronize()
    # an empty split weighs 0: the oracle takes its values as 0 (0 * NaN would poison its sum)
    o_ref = np.where(np.isneginf(lse)[..., None], 0.0, o.astype(np.float64))
    ref, ref_lse = odecode.merge(o_ref, lse.astype(np.float64))
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 1e-5
    fin = np.isfinite(ref_lse)
    assert np.allclose(out_lse.cpu().numpy()[fin], ref_lse[fin], atol=1e-5)
    assert np.all(got[rows - 1] == 0) and np.isneginf(out_lse.cpu().numpy()[rows - 1])
    assert torch.equal(out16, out.to(torch.bfloat16))


@pytest.mark.parametrize("d,dr,h,splits", [(512, 64, 16, 40), (256, 32, 40, 20)])
def test_decode_long_request_many_splits(d, dr, h, splits):
    """One request of 12,000 tokens over `splits` INT2 splits (one wave: the window split runs
    first and the split merge is the many-partials one), against the FP64 oracle; the decode
    call's BF16 output is its FP32 merge rounded, and equals the generic merge's."""
    seq_lens = [12000]
    pages = (seq_lens[0] + 63) // 64
    g = torch.Generator().manual_seed(101)
    pt = (torch.randperm(pages, generator=g) + 1).to(torch.int32).reshape(1, pages).cuda()
    pool = GpuPool(64 * (pages + 1), d, dr, max_reqs=1, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=102), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=103)
    q = synth.normal_bf16((1, h, d + dr), seed=104, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    sm = 1.0 / np.sqrt(192.0 if d == 512 else 96.0)
    part_o = torch.empty(1, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(1, h, splits + 1, device="cuda")
    out = torch.full((1, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((1, h), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, sm, splits, part_o, part_lse, out, out_lse=lse, err=err)
    o32 = torch.empty(h, d, device="cuda")
    lse32 = torch.empty(h, device="cuda")
    ops.merge_partials(part_o.view(h, splits + 1, d).transpose(0, 1), part_lse.view(h, splits + 1).t(), out_f32=o32,
                       out_lse=lse32)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out.view(h, d), o32.to(torch.bfloat16))
    assert torch.equal(lse.view(h), lse32)
    ref, ref_lse = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm)
    f = o32.cpu().numpy()
    assert np.abs(f - ref[0]).max() <= 2e-2
    assert cosine(out.float().cpu().numpy()[0], ref[0]) >= 0.9995
    assert np.allclose(lse32.cpu().numpy(), ref_lse[0], atol=2e-3)


def test_peer_exchange_many_parts_equals_generic_merge():
    """The exchange's push merges many partials like the generic merge (the NCCL path's local
    merge): on one rank the exchanged FP32 output is bit-identical to it."""
    d, h, parts = 512, 16, 33
    rng = np.random.default_rng(7)
    o = torch.from_numpy(rng.standard_normal((1, h, parts, d)).astype(np.float32)).cuda()
    lse = torch.from_numpy((rng.standard_normal((1, h, parts)) * 2).astype(np.float32)).cuda()
    lse[0, 3, ::5] = float("-inf")
    ref = torch.empty(h, d, device="cuda")
    ref_lse = torch.empty(h, device="cuda")
    ops.merge_partials(o.view(h, parts, d).transpose(0, 1), lse.view(h, parts).t(), out_f32=ref, out_lse=ref_lse)
    xch = PeerExchange(h, d)
    try:
        out32 = torch.full((1, h, d), float("nan"), device="cuda")
        out_lse = torch.full((h,), float("nan"), device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        for _ in range(2):
            xch.exchange(o, lse, out_f32=out32, out_lse=out_lse, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
    finally:
        xch.close()
    assert torch.equal(out32.view(h, d), ref)
    assert torch.equal(out_lse, ref_lse)
