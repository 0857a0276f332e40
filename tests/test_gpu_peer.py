"""The sequence-split exchange over peer memory (``PeerExchange``): on one GPU the rank
exchanges with itself (the same kernels, its own receive buffer as the only peer), and the
result must equal the local LSE merge of the same split partials; with two or more GPUs the
bench's ``--mode seqsplit`` compares it with the NCCL all-gather path."""

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, bits, fill_requests
from mla_kv_quant_b200 import ops, synth
from mla_kv_quant_b200.seqsplit import PeerExchange
from oracle import decode as odecode

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d,dr,h", [(512, 64, 16), (256, 32, 40)])
def test_peer_exchange_single_rank_equals_local_merge(d, dr, h):
    seq_lens = [900, 257, 64]
    b = len(seq_lens)
    g = torch.Generator().manual_seed(81)
    pages = 15
    pt = (torch.randperm(b * pages, generator=g) + 1).to(torch.int32).reshape(b, pages).cuda()
    pool = GpuPool(64 * (b * pages + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=82), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=83)
    q = synth.normal_bf16((b, h, d + dr), seed=84, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    sm = 0.07
    parts = 4
    part_o = torch.empty(b, h, parts, d, device="cuda")
    part_lse = torch.empty(b, h, parts, device="cuda")
    scratch = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, sm, parts - 1, part_o, part_lse, scratch)
    ref32 = torch.empty(b * h, d, device="cuda")
    ref_lse = torch.empty(b * h, device="cuda")
    ops.merge_partials(part_o.view(b * h, parts, d).transpose(0, 1), part_lse.view(b * h, parts).t(), out_f32=ref32,
                       out_lse=ref_lse)
    xch = PeerExchange(b * h, d)
    try:
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        for step in range(3):  # both parities of the receive buffer, and a reused state
            out = torch.full((b, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
            out32 = torch.full((b, h, d), float("nan"), device="cuda")
            lse = torch.full((b * h,), float("nan"), device="cuda")
            xch.exchange(part_o, part_lse, out_bf16=out, out_f32=out32, out_lse=lse, err=err)
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            assert int(xch.state[0].item()) == step + 1
            # one partial per rank: the merge of a single partial is the partial itself
            assert torch.allclose(out32.view(b * h, d), ref32, rtol=1e-6, atol=1e-6), step
            assert torch.allclose(lse, ref_lse, rtol=1e-6, atol=1e-6)
            assert torch.equal(out, out32.to(torch.bfloat16))  # the BF16 output is the FP32 result rounded
    finally:
        xch.close()
    # and the merged result is the decode the oracle computes
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm)
    assert np.abs(ref32.view(b, h, d).cpu().numpy() - ref).max() <= 2e-2


def test_partials_only_decode_matches_merged_call():
    """``packed_decode(out=None)`` writes the same split partials the merged call merges: the
    exchange of those partials (one rank) equals the merged call's output."""
    d, dr, h = 512, 64, 16
    seq_lens = [1300, 90]
    b = len(seq_lens)
    g = torch.Generator().manual_seed(91)
    pages = 21
    pt = (torch.randperm(b * pages, generator=g) + 1).to(torch.int32).reshape(b, pages).cuda()
    pool = GpuPool(64 * (b * pages + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=92), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=93)
    q = synth.normal_bf16((b, h, d + dr), seed=94, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    parts = 3
    merged = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, 0.07, parts - 1, torch.empty(b, h, parts, d, device="cuda"),
                      torch.empty(b, h, parts, device="cuda"), merged)
    part_o = torch.full((b, h, parts, d), float("nan"), device="cuda")
    part_lse = torch.full((b, h, parts), float("nan"), device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, 0.07, parts - 1, part_o, part_lse, None)
    xch = PeerExchange(b * h, d)
    try:
        out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
        xch.exchange(part_o, part_lse, out_bf16=out)
        torch.cuda.synchronize()
    finally:
        xch.close()
    assert torch.isfinite(part_lse).all() or (part_lse == float("-inf")).any()
    diff = (out.float() - merged.float()).abs()
    assert float(diff.max()) <= 2 ** -8 * float(merged.float().abs().max()), float(diff.max())


def test_peer_wait_gives_up_when_no_rank_pushes():
    """A rank whose peers never push: the merge's wait ends after its bound (~2 s) with
    ROLAQ_DEV_PEER_TIMEOUT in err and a zero output, and the context stays usable.  The
    missing push is made on the host: the step counter is moved past every flag."""
    from mla_kv_quant_b200 import _lib

    d, rows = 512, 8
    xch = PeerExchange(rows, d)
    try:
        xch.state[0] = 5  # a step no rank has flagged
        out = torch.full((rows, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.call("rolaq_peer_wait_merge", xch._own, xch.world, rows, d, xch.state.data_ptr(), out.data_ptr(), None,
                  None, err.data_ptr(), _lib.stream_ptr())
        torch.cuda.synchronize()
        assert int(err.item()) & _lib.DEV_PEER_TIMEOUT
        assert torch.equal(out.float(), torch.zeros(rows, d, device="cuda"))
        # the device still answers
        assert float(torch.ones(4, device="cuda").sum().item()) == 4.0
    finally:
        xch.state[0] = 0
        xch.close()


def test_sequence_split_decoder_on_one_gpu():
    """``SequenceSplitDecoder`` without a process group (one GPU holds the whole request),
    through both exchanges, on the default split count of its slice: the two outputs are
    identical and equal the merged decode call's within BF16 rounding of its weights."""
    from mla_kv_quant_b200.mla_packed_decode import packed_mla_decode_gf_fwd
    from mla_kv_quant_b200.pool import PackedLatentPool
    from mla_kv_quant_b200.seqsplit import SequenceSplitDecoder

    d, dr, h, L = 512, 64, 16, 12000
    n = (L + 63) // 64
    pool = PackedLatentPool(64 * (n + 2), 1, max_reqs=1, rotations={0: synth.rotation(d, 11)})
    g = torch.Generator().manual_seed(12)
    pt = (torch.randperm(n + 1, generator=g)[:n] + 1).to(torch.int32).reshape(1, n).cuda()
    pos = torch.arange(L, device="cuda")
    slots = pt[0, pos // 64] * 64 + pos % 64
    pool.set_window_meta(False, torch.full((L,), L, dtype=torch.int32, device="cuda"),
                         torch.zeros(L, dtype=torch.int64, device="cuda"))
    pool.set_kv_buffer(0, slots.long(), synth.latents(L, d, seed=13, device="cuda"),
                       synth.normal_bf16((L, dr), seed=14, device="cuda"), positions=pos.int())
    q = synth.normal_bf16((1, h, d + dr), seed=15, device="cuda")
    sl = torch.tensor([L], dtype=torch.int32, device="cuda")
    splits = ops.default_num_splits(1, L)
    assert splits + 1 >= 16  # the slice's splits take the many-partials merge
    out_nccl = SequenceSplitDecoder(pool).decode(q, 0, pt, [L], sl, 0.07)
    xch = PeerExchange(h, d)
    try:
        out_peer = SequenceSplitDecoder(pool, exchange=xch).decode(q, 0, pt, [L], sl, 0.07)
        torch.cuda.synchronize()
    finally:
        xch.close()
    ref = packed_mla_decode_gf_fwd(q, pool, 0, pt, sl, 0.07, splits)
    torch.cuda.synchronize()
    assert torch.equal(out_peer, out_nccl)
    diff = (out_peer.float() - ref.float()).abs()
    assert float(diff.max()) <= 2 ** -8 * float(ref.float().abs().max()), float(diff.max())
