"""Packed decode attention against the oracle (FP64) over the same pool contents.

Tolerance (north star: max-abs <= 2e-2, cosine >= 0.9995), applied per request to
* the kernel's FP32 result (its partials LSE-merged to FP32): max-abs <= 2e-2;
* the BF16 output: max-abs <= 2e-2 + half a BF16 ulp of the reference value (the
  output format alone rounds |v| in [8, 16) by up to 0.031), cosine >= 0.9995.
"""

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, bits, cosine, fill_requests
from mla_kv_quant_b200 import _lib, ops, synth
from oracle import decode as odecode
from oracle import writer as owriter

pytestmark = pytest.mark.gpu

SHAPES = [(512, 64, 16), (256, 32, 40), (512, 64, 8), (256, 32, 16)]


def _setup(d, dr, seq_lens, max_pages=None, seed=0, sink=4, recent=16, row_gain=None):
    b = len(seq_lens)
    mp = max_pages or max(1, max((L + 63) // 64 for L in seq_lens))
    g = torch.Generator().manual_seed(seed)
    total = b * mp
    perm = (torch.randperm(total, generator=g) + 1).to(torch.int32)
    pt = perm.reshape(b, mp).cuda()
    pool = GpuPool(64 * (total + 1), d, dr, max_reqs=b, sink=sink, recent=recent)
    r = synth.rotation(d, seed=seed + 5)
    codec = ops.codec_serving(0.85, synth.signal_gain(0.85))
    fill_requests(pool, seq_lens, pt, r, codec, seed=seed, row_gain=row_gain)
    return pool, pt


def half_ulp_bf16(v):
    e = np.floor(np.log2(np.maximum(np.abs(v), 1e-30)))
    return np.exp2(e - 8)


def fp32_result(part_o, part_lse):
    b, h, parts, d = part_o.shape
    o = torch.empty(b * h, d, device="cuda")
    ops.merge_partials(part_o.view(b * h, parts, d).transpose(0, 1), part_lse.view(b * h, parts).t(), out_f32=o)
    torch.cuda.synchronize()
    return o.view(b, h, d).cpu().numpy()


def _check(out, ref, seq_lens, out32=None):
    for b, L in enumerate(seq_lens):
        o = out[b].float().cpu().numpy()
        if L == 0:
            assert np.all(o == 0)
            continue
        if out32 is not None:
            e32 = np.max(np.abs(out32[b] - ref[b]))
            assert e32 <= 2e-2, f"request {b}: FP32 max-abs {e32}"
        excess = np.abs(o - ref[b]) - half_ulp_bf16(ref[b])
        assert np.max(excess) <= 2e-2, f"request {b}: BF16 max-abs beyond output rounding {np.max(excess)}"
        assert cosine(o, ref[b]) >= 0.9995


@pytest.mark.parametrize("d,dr,h", SHAPES)
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_decode_matches_oracle(d, dr, h, splits):
    seq_lens = [1, 19, 20, 21, 64, 65, 700, 1500]
    pool, pt = _setup(d, dr, seq_lens, seed=h + splits)
    b = len(seq_lens)
    q = synth.normal_bf16((b, h, d + dr), seed=3, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    part_o = torch.empty(b, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(b, h, splits + 1, device="cuda")
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(b, h, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    sm = 1.0 / np.sqrt(192.0)
    ops.packed_decode(q, pool.view(), pt, sl, sm, splits, part_o, part_lse, out, out_lse=lse, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref, ref_lse = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm)
    _check(out, ref, seq_lens, fp32_result(part_o, part_lse))
    assert np.allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


@pytest.mark.parametrize("direction", ["rising", "falling"])
@pytest.mark.parametrize("d,dr,h", [(512, 64, 16), (256, 32, 40)])
def test_decode_drifting_scales_and_scores(direction, d, dr, h):
    """Group scales and scores that drift 2^6 along the sequence: the kernel's running
    reference max and per-group weight scale both move many times inside a split."""
    seq_lens = [3000, 2200]

    def gain(L):
        x = torch.arange(L, dtype=torch.float64) / L
        return torch.exp2(6.0 * (x if direction == "rising" else 1.0 - x))

    pool, pt = _setup(d, dr, seq_lens, seed=21, row_gain=gain)
    b = len(seq_lens)
    q = synth.normal_bf16((b, h, d + dr), seed=4, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    splits = 2
    part_o = torch.empty(b, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(b, h, splits + 1, device="cuda")
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    sm = 0.02  # keeps the softmax from collapsing onto a single token at the largest gain
    ops.packed_decode(q, pool.view(), pt, sl, sm, splits, part_o, part_lse, out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm)
    o32 = fp32_result(part_o, part_lse)
    for i in range(b):
        scale = max(1.0, float(np.abs(ref[i]).max()))
        assert np.abs(o32[i] - ref[i]).max() <= 2e-2 * scale
        assert cosine(o32[i], ref[i]) >= 0.9995


def test_decode_zero_length_and_window_only():
    d, dr, h = 512, 64, 16
    seq_lens = [0, 3, 20]
    pool, pt = _setup(d, dr, seq_lens, max_pages=2)
    q = synth.normal_bf16((3, h, d + dr), seed=1, device="cuda")
    out = torch.empty(3, h, d, dtype=torch.bfloat16, device="cuda")
    part_o = torch.empty(3, h, 5, d, device="cuda")
    part_lse = torch.empty(3, h, 5, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, 0.07, 4, part_o, part_lse, out)
    torch.cuda.synchronize()
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, 0.07)
    _check(out, ref, seq_lens)


def test_decode_ring_row_ownership_fallback():
    """A window token whose ring row was taken over by another slot is read from INT2."""
    d, dr, h = 512, 64, 16
    seq_lens = [300]
    pool, pt = _setup(d, dr, seq_lens)
    pos = 299
    slot = int(pt[0, pos // 64]) * 64 + pos % 64
    r = int(pool.rows[slot])
    pool.owners[r] = 1  # stolen
    q = synth.normal_bf16((1, h, d + dr), seed=4, device="cuda")
    out = torch.empty(1, h, d, dtype=torch.bfloat16, device="cuda")
    ops.packed_decode(q, pool.view(), pt, torch.tensor(seq_lens, dtype=torch.int32, device="cuda"), 0.07, 2,
                      torch.empty(1, h, 3, d, device="cuda"), torch.empty(1, h, 3, device="cuda"), out)
    torch.cuda.synchronize()
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, 0.07)
    _check(out, ref, seq_lens)


def test_decode_token_range_partials_merge_to_full():
    """Two slices decoded separately and LSE-merged equal the whole (sequence split)."""
    d, dr, h = 512, 64, 16
    seq_lens = [1000, 333]
    pool, pt = _setup(d, dr, seq_lens, seed=9)
    b = 2
    q = synth.normal_bf16((b, h, d + dr), seed=2, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    full = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    full_lse = torch.empty(b, h, device="cuda")
    fpo, fpl = torch.empty(b, h, 4, d, device="cuda"), torch.empty(b, h, 4, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, 0.07, 3, fpo, fpl, full, out_lse=full_lse)
    full32 = fp32_result(fpo, fpl)
    outs, lses = [], []
    for lo_hi in ([[0, 512], [0, 128]], [[512, 1000], [128, 333]]):
        rng = torch.tensor(lo_hi, dtype=torch.int32, device="cuda")
        part_o = torch.empty(b, h, 4, d, device="cuda")
        part_lse = torch.empty(b, h, 4, device="cuda")
        scratch = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
        ops.packed_decode(q, pool.view(), pt, sl, 0.07, 3, part_o, part_lse, scratch, token_range=rng)
        o = torch.empty(b * h, d, device="cuda")
        l = torch.empty(b * h, device="cuda")
        ops.merge_partials(part_o.view(b * h, 4, d).transpose(0, 1), part_lse.view(b * h, 4).t(), out_f32=o,
                           out_lse=l)
        outs.append(o)
        lses.append(l)
    merged = torch.empty(b * h, d, device="cuda")
    ops.merge_partials(torch.stack(outs), torch.stack(lses), out_f32=merged)
    torch.cuda.synchronize()
    # Both results against the FP64 oracle (the decode tolerance), then against each other.
    # Slicing the sequence moves the tile (and segment) boundaries that the attention weights
    # are quantised against: two E4M3 terms carry a weight to 2^-8 of itself, so the two FP32
    # results agree to 2^-8 of the largest dequantised value a weight multiplies, not bit for bit.
    merged_np = merged.view(b, h, d).cpu().numpy()
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, 0.07)
    for i in range(b):
        e_full = np.abs(full32[i] - ref[i]).max()
        e_merged = np.abs(merged_np[i] - ref[i]).max()
        print(f"request {i}: full vs oracle {e_full:.3g}, slices vs oracle {e_merged:.3g}, "
              f"max |ref| {np.abs(ref[i]).max():.3g}")
        assert e_full <= 2e-2 and e_merged <= 2e-2
    diff = np.abs(merged_np - full32).max()
    print(f"slices vs full: {diff:.3g}")
    assert diff <= 1e-2


def test_decode_bad_page_is_reported():
    d, dr, h = 512, 64, 16
    pool, pt = _setup(d, dr, [200])
    pt = pt.clone()
    pt[0, 1] = 10_000  # outside the pool
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(1, h, d, dtype=torch.bfloat16, device="cuda")
    q = synth.normal_bf16((1, h, d + dr), seed=1, device="cuda")
    ops.packed_decode(q, pool.view(), pt, torch.tensor([200], dtype=torch.int32, device="cuda"), 0.07, 2,
                      torch.empty(1, h, 3, d, device="cuda"), torch.empty(1, h, 3, device="cuda"), out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEV_BAD_PAGE
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("d,dr,h", [(512, 64, 16), (256, 32, 40)])
@pytest.mark.parametrize("bad_page", [0, 4])
def test_decode_bad_window_page_is_masked(d, dr, h, bad_page):
    """A window page outside the pool is reported, and its rows take no weight: the output
    equals the oracle's attention over the remaining tokens (page 0 holds the sink rows,
    page 4 the recent rows of a 300-token request)."""
    L = 300
    pool, pt = _setup(d, dr, [L], seed=13)
    opool = pool.to_oracle()
    pt_ok = pt.cpu().numpy()
    pt = pt.clone()
    pt[0, bad_page] = 10_000  # outside the pool
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(1, h, d, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(1, h, device="cuda")
    q = synth.normal_bf16((1, h, d + dr), seed=1, device="cuda")
    sm = 1.0 / np.sqrt(192.0)
    ops.packed_decode(q, pool.view(), pt, torch.tensor([L], dtype=torch.int32, device="cuda"), sm, 2,
                      torch.empty(1, h, 3, d, device="cuda"), torch.empty(1, h, 3, device="cuda"), out, out_lse=lse,
                      err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEV_BAD_PAGE
    # the oracle over the tokens whose page is valid
    slots = odecode.token_slots(pt_ok[0], L)
    lat = odecode.latent_rows(opool, slots, L)
    pe = owriter.bf16_to_f32(opool.rope[slots]).astype(np.float64)
    keep = np.arange(L) // 64 != bad_page
    qf = owriter.bf16_to_f32(bits(q)).astype(np.float64)[0]
    ref, ref_lse = odecode.attend(qf, lat[keep], pe[keep], sm)
    o = out[0].float().cpu().numpy()
    assert np.max(np.abs(o - ref) - half_ulp_bf16(ref)) <= 2e-2
    assert cosine(o, ref) >= 0.9995
    assert np.allclose(lse[0].cpu().numpy(), ref_lse, atol=2e-3)


def test_merge_partials_matches_oracle():
    rng = np.random.default_rng(0)
    parts, rows, d = 5, 7, 512
    o = rng.standard_normal((parts, rows, d)).astype(np.float32)
    lse = rng.standard_normal((parts, rows)).astype(np.float32) * 3
    lse[1, 2] = -np.inf
    lse[:, 4] = -np.inf  # all parts empty
    out = torch.empty(rows, d, device="cuda")
    out_lse = torch.empty(rows, device="cuda")
    ops.merge_partials(torch.from_numpy(o).cuda(), torch.from_numpy(lse).cuda(), out_f32=out, out_lse=out_lse)
    torch.cuda.synchronize()
    ref, ref_lse = odecode.merge(o.astype(np.float64), lse.astype(np.float64))
    assert np.allclose(out.cpu().numpy(), ref, atol=1e-5)
    fin = np.isfinite(ref_lse)
    assert np.allclose(out_lse.cpu().numpy()[fin], ref_lse[fin], atol=1e-5)
    assert np.all(out.cpu().numpy()[4] == 0) and np.isneginf(out_lse.cpu().numpy()[4])
