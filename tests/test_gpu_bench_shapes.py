"""Parity at the shapes the benchmark times.

* Writer, config 1: 8 requests x 16384 tokens = 131072 rows in one launch.  The
  persistent tcgen05 grid (one CTA per SM, four groups) then runs ~28 row tiles per
  CTA, so every TMEM accumulator, every epilogue warp set and many mbarrier phase
  flips are exercised.  Codes/params are bit-exact against the oracle codec on the
  kernel's own FP32 rotation; against the reference FP32 GEMM rotation at most 1e-4
  of the codes differ (rounding ties); k_pe, ring rows and maps equal the oracle
  writer's.
* Decode, config 2: 64 requests x 16384 tokens with the benchmark's default split
  count and with 9 splits (15 / 14 tiles per CTA), through the caller-scratch and the static-scratch entry points, a seeded
  subset of 8 requests against the FP64 oracle with the decode tests' tolerance: the
  kernel's FP32 result (its partials merged in FP32) within max-abs 2e-2, the BF16 output
  within 2e-2 plus half a BF16 ulp of the value (the output format's own rounding),
  cosine >= 0.9995; the static-scratch output equals the caller-scratch output.
"""

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, bits, cosine, fill_requests, oracle_scalars, rotate_cpu
from mla_kv_quant_b200 import ops, synth
from oracle import codec as ocodec
from oracle import decode as odecode
from oracle import writer as owriter

pytestmark = pytest.mark.gpu

CTX = 16384


def test_writer_config1_every_tile_slot_and_phase():
    d, dr, reqs = 512, 64, 8
    n = reqs * CTX
    pt, num_slots = synth.page_table(reqs, CTX, seed=41, device="cuda")
    pool = GpuPool(num_slots, d, dr, max_reqs=reqs)
    x = synth.latents(n, d, seed=42, device="cuda")
    pe = synth.normal_bf16((n, dr), seed=43, device="cuda")
    r = synth.rotation(d, seed=44)
    rt = r.to(torch.bfloat16).t().contiguous().cuda()
    pos = torch.arange(CTX, device="cuda").repeat(reqs)
    req = torch.arange(reqs, device="cuda").repeat_interleave(CTX)
    slots = (pt[req, pos // 64].long() * 64 + pos % 64).contiguous()
    seq = torch.full((n,), CTX, dtype=torch.int32, device="cuda")
    codec = ops.codec_serving(0.78, synth.signal_gain(0.78))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fused_write(x, pe, slots, rt, codec, pool.view(), seq_lens=seq, req_idx=req, positions=pos.to(torch.int32),
                    err=err)
    rot = torch.empty(n, d, device="cuda")
    ops.rotate_rows(x, rt, out_f32=rot)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    s = slots.cpu().numpy()
    rot_np = rot.cpu().numpy()
    oc, osc, oze = ocodec.encode(rot_np, *oracle_scalars(codec))
    assert np.array_equal(pool.codes.cpu().numpy()[s], ocodec.pack(oc))
    assert np.array_equal(pool.params.cpu().numpy()[s], ocodec.params_array(osc, oze))
    # k_pe, ring rows, maps: the oracle writer applied to the same rotated rows
    opool = owriter.Pool(num_slots, d, dr, reqs, 4, 16)
    t32, sf32, z32 = oracle_scalars(codec)
    owriter.write(opool, rot_np, bits(pe), s, seq.cpu().numpy(), req.cpu().numpy(), t32, sf32,
                  positions=pos.cpu().numpy(), zero_const32=z32)
    assert np.array_equal(bits(pool.rope), opool.rope)
    assert np.array_equal(bits(pool.hp), opool.hp)
    assert np.array_equal(pool.rows.cpu().numpy(), opool.rows)
    assert np.array_equal(pool.owners.cpu().numpy(), opool.owners)
    # against the reference FP32 GEMM rotation: codes differ only at rounding ties
    rc, _, _ = ocodec.encode(rotate_cpu(x, r), *oracle_scalars(codec))
    got = ocodec.unpack(pool.codes.cpu().numpy()[s], d)
    assert np.mean(got != rc) <= 1e-4


@pytest.fixture(scope="module")
def config2_pool():
    d, dr, b = 512, 64, 64
    seq_lens = [CTX] * b
    g = torch.Generator().manual_seed(51)
    pages = CTX // 64
    pt = (torch.randperm(b * pages, generator=g) + 1).to(torch.int32).reshape(b, pages).cuda()
    pool = GpuPool(64 * (b * pages + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=52), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=53)
    return pool, pt, seq_lens


@pytest.mark.parametrize("which", ["default", "nine"])
def test_decode_config2_default_splits(config2_pool, which):
    import ctypes

    from mla_kv_quant_b200 import _lib

    pool, pt, seq_lens = config2_pool
    d, dr, h = 512, 64, 16
    b = len(seq_lens)
    # the bench's split count, and 9 (15 / 14 tiles per split: many tiles per CTA)
    splits = ops.default_num_splits(b, CTX) if which == "default" else 9
    q = synth.normal_bf16((b, h, d + dr), seed=54, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = torch.full((b, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((b, h), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    sm = 1.0 / np.sqrt(192.0)
    part_o = torch.empty(b, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(b, h, splits + 1, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, sm, splits, part_o, part_lse, out, out_lse=lse, err=err)
    o32 = torch.empty(b * h, d, device="cuda")
    ops.merge_partials(part_o.view(b * h, splits + 1, d).transpose(0, 1), part_lse.view(b * h, splits + 1).t(),
                       out_f32=o32)
    # the static-scratch entry point, called through the C ABI, on the same inputs
    lib = _lib.load()
    cs = pool.view().c_struct()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out_s = torch.full_like(out, float("nan"))
    lse_s = torch.full_like(lse, float("nan"))
    rc = lib.rolaq_packed_decode_static(q.data_ptr(), q.stride(0), q.stride(1), b, h, ctypes.byref(cs),
                                        pt.data_ptr(), pt.stride(0), pt.shape[1], sl.data_ptr(), None, sm, splits,
                                        out_s.data_ptr(), out_s.stride(0), out_s.stride(1), lse_s.data_ptr(),
                                        err.data_ptr(), stream)
    assert rc == 0, lib.rolaq_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out_s, out) and torch.equal(lse_s, lse)
    sub = sorted(np.random.default_rng(55).choice(b, size=8, replace=False).tolist())
    ref, ref_lse = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm, requests=sub)
    o = out.float().cpu().numpy()
    f = o32.view(b, h, d).cpu().numpy()
    for i in sub:
        e32 = np.abs(f[i] - ref[i]).max()
        print(f"splits {splits} request {i}: FP32 max-abs {e32:.4g}, max |ref| {np.abs(ref[i]).max():.3g}")
        assert e32 <= 2e-2, f"request {i}: FP32 max-abs {e32}"
        half_ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref[i]), 1e-30))) - 8)
        assert np.max(np.abs(o[i] - ref[i]) - half_ulp) <= 2e-2, f"request {i}"
        assert cosine(o[i], ref[i]) >= 0.9995
    assert np.allclose(lse.cpu().numpy()[sub], ref_lse[sub], atol=2e-3)


@pytest.mark.parametrize("which", ["default", "many"])
def test_decode_minicpm3_shape_default_splits(which):
    """The MiniCPM3-4B shape (D = 256, Dr = 32, H = 40, softmax scale 1/sqrt(64 + 32)) on
    the tcgen05 kernel: 8 requests x 8192 tokens with the default split count (one wave:
    the window split runs first) and with 32 splits (two waves: separate window and merge
    launches), every request against the FP64 oracle."""
    d, dr, h, b, ctx = 256, 32, 40, 8, 8192
    seq_lens = [ctx] * b
    g = torch.Generator().manual_seed(61)
    pages = ctx // 64
    pt = (torch.randperm(b * pages, generator=g) + 1).to(torch.int32).reshape(b, pages).cuda()
    pool = GpuPool(64 * (b * pages + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=62), ops.codec_serving(0.9, synth.signal_gain(0.9)),
                  seed=63)
    splits = ops.default_num_splits(b, ctx, latent_dim=d, rope_dim=dr, heads=h) if which == "default" else 32
    q = synth.normal_bf16((b, h, d + dr), seed=64, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    sm = 1.0 / np.sqrt(96.0)
    part_o = torch.empty(b, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(b, h, splits + 1, device="cuda")
    ops.packed_decode(q, pool.view(), pt, sl, sm, splits, part_o, part_lse, out, err=err)
    o32 = torch.empty(b * h, d, device="cuda")
    ops.merge_partials(part_o.view(b * h, splits + 1, d).transpose(0, 1), part_lse.view(b * h, splits + 1).t(),
                       out_f32=o32)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm)
    o = out.float().cpu().numpy()
    f = o32.view(b, h, d).cpu().numpy()
    for i in range(b):
        assert np.abs(f[i] - ref[i]).max() <= 2e-2, f"request {i}"
        half_ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref[i]), 1e-30))) - 8)
        assert np.max(np.abs(o[i] - ref[i]) - half_ulp) <= 2e-2, f"request {i}"
        assert cosine(o[i], ref[i]) >= 0.9995



def test_decode_window_ctas_loop_over_chunks():
    """B = 128 with one split (the Moonlight layout): the INT2 grid leaves 20 SMs, so each
    window CTA serves two chunks of requests while the INT2 kernel runs; a seeded subset of
    requests against the FP64 oracle."""
    d, dr, h, b, ctx = 512, 64, 16, 128, 640
    seq_lens = [ctx - 7 * (i % 5) for i in range(b)]
    g = torch.Generator().manual_seed(71)
    pages = (ctx + 63) // 64
    pt = (torch.randperm(b * pages, generator=g) + 1).to(torch.int32).reshape(b, pages).cuda()
    pool = GpuPool(64 * (b * pages + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=72), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=73)
    q = synth.normal_bf16((b, h, d + dr), seed=74, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = torch.full((b, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    sm = 1.0 / np.sqrt(192.0)
    ops.packed_decode(q, pool.view(), pt, sl, sm, 1, torch.empty(b, h, 2, d, device="cuda"),
                      torch.empty(b, h, 2, device="cuda"), out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    sub = sorted(np.random.default_rng(75).choice(b, size=10, replace=False).tolist() + [0, b - 1])
    ref, _ = odecode.decode(pool.to_oracle(), bits(q), pt.cpu().numpy(), seq_lens, sm, requests=sub)
    o = out.float().cpu().numpy()
    for i in sub:
        half_ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref[i]), 1e-30))) - 8)
        assert np.max(np.abs(o[i] - ref[i]) - half_ulp) <= 2e-2, f"request {i}"
        assert cosine(o[i], ref[i]) >= 0.9995
