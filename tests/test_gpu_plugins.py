"""Reference-facing entry points on the GPU: the serving writer plugin through the
pool, the reader, the HF quantizer API and the loader's read-rotation fold."""

import json

import numpy as np
import pytest
import torch

from gpu_helpers import bits, cosine, oracle_scalars
from mla_kv_quant_b200 import ops, synth
from mla_kv_quant_b200.mla_fused_writer import try_fast_decode_store
from mla_kv_quant_b200.mla_packed_decode import packed_mla_decode_gf_fwd, prepare_gf_splits
from mla_kv_quant_b200.pool import PackedLatentPool
from mla_kv_quant_b200.quantizer import LearnedRotationQuantizer, rotate_quantize
from mla_kv_quant_b200.rolaq_mla import fold_read_rotation
from oracle import codec as ocodec
from oracle import decode as odecode
from oracle import writer as owriter

pytestmark = pytest.mark.gpu


def _oracle_pool(pool, li):
    p = owriter.Pool(pool.size, pool.kv_lora_rank, pool.qk_rope_head_dim, pool._max_reqs, pool._win_p, pool._win_r)
    p.codes = pool.c_codes[li].cpu().numpy()
    p.params = pool.c_params[li].cpu().numpy()
    p.rope = bits(pool.rope_buf[li])
    p.hp = bits(pool.hp_c[li])
    p.rows = pool.hp_row_of_slot.cpu().numpy()
    p.owners = pool.hp_owner_of_row.cpu().numpy()
    return p


def test_decode_steps_through_pool_plugin(monkeypatch):
    """Prefill 3 requests, then 40 decode steps through try_fast_decode_store (the
    recent window wraps twice); the pool must equal the oracle's after every step and
    the reader must match the oracle decode at the end."""
    monkeypatch.setenv("SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE", "1")
    layers, d, dr, h = 2, 512, 64, 16
    rot = {i: synth.rotation(d, 100 + i) for i in range(layers)}
    params = [(0.8, synth.signal_gain(0.8)), None]  # layer 1 falls back to the Lloyd-Max defaults
    pool = PackedLatentPool(64 * 24, layers, max_reqs=4, rotations=rot, quantizer_params=params)
    g = torch.Generator().manual_seed(0)
    pages = (torch.randperm(23, generator=g) + 1).to(torch.int32)
    pt = pages[:21].reshape(3, 7).cuda()
    lens = [5, 100, 300]
    oracle = [_oracle_pool(pool, li) for li in range(layers)]

    def slot_of(b, p):
        return int(pt[b, p // 64]) * 64 + p % 64

    def write(li, c_kv, k_pe, slots, seq, req, positions, decode):
        pool.set_window_meta(decode, seq, req)
        if decode:
            assert try_fast_decode_store(pool, li, slots, c_kv, k_pe)
        else:
            pool.set_kv_buffer(li, slots, c_kv, k_pe, positions=positions)
        codec = pool.codec(li)
        # the oracle codec runs on the kernel's own FP32 rotation (shared MMA order)
        gpu_rot = torch.empty(c_kv.shape[0], d, device="cuda")
        ops.rotate_rows(c_kv, pool.write_rotation_t(li), out_f32=gpu_rot)
        owriter.write(oracle[li], gpu_rot.cpu().numpy(), bits(k_pe), slots.cpu().numpy(), seq.cpu().numpy(),
                      req.cpu().numpy(), *oracle_scalars(codec)[:2],
                      positions=None if positions is None else positions.cpu().numpy())

    # prefill
    for b, L in enumerate(lens):
        for li in range(layers):
            x = synth.latents(L, d, seed=10 * b + li, device="cuda")
            pe = synth.normal_bf16((L, dr), seed=10 * b + li + 5, device="cuda")
            slots = torch.tensor([slot_of(b, p) for p in range(L)], device="cuda")
            write(li, x, pe, slots, torch.full((L,), L, dtype=torch.int32, device="cuda"),
                  torch.full((L,), b, dtype=torch.int64, device="cuda"), torch.arange(L, device="cuda"), False)
    # decode steps
    for step in range(40):
        lens = [L + 1 for L in lens]
        slots = torch.tensor([slot_of(b, L - 1) for b, L in enumerate(lens)], device="cuda")
        seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
        req = torch.arange(3, device="cuda")
        for li in range(layers):
            x = synth.latents(3, d, seed=1000 + 7 * step + li, device="cuda")
            pe = synth.normal_bf16((3, dr), seed=2000 + step + li, device="cuda")
            write(li, x, pe, slots, seq, req, None, True)
    torch.cuda.synchronize()
    for li in range(layers):
        got = _oracle_pool(pool, li)
        for name in ("codes", "params", "rope", "hp", "rows", "owners"):
            assert np.array_equal(getattr(got, name), getattr(oracle[li], name)), (li, name)
    # reader through the plugin entry point, with caller-provided scratch
    q = synth.normal_bf16((3, h, d + dr), seed=77, device="cuda")
    splits = torch.tensor([4, 4, 4], dtype=torch.int32, device="cuda")
    quant, merge = torch.empty_like(splits), torch.empty_like(splits)
    prepare_gf_splits(splits, quant, merge)
    ns = int(quant.max())
    out = packed_mla_decode_gf_fwd(q, pool, 1, pt, torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                   1 / np.sqrt(192), ns, attn_logits=torch.empty(3, h, ns + 1, d, device="cuda"),
                                   attn_lse=torch.empty(3, h, ns + 1, device="cuda"))
    torch.cuda.synchronize()
    ref, _ = odecode.decode(oracle[1], bits(q), pt.cpu().numpy(), lens, 1 / np.sqrt(192))
    for b in range(3):
        o = out[b].float().cpu().numpy()
        half_ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref[b]), 1e-30))) - 8)
        assert np.max(np.abs(o - ref[b]) - half_ulp) <= 2e-2 and cosine(o, ref[b]) >= 0.9995


def test_try_fast_decode_store_guards():
    pool = PackedLatentPool(64 * 2, 1, rotations={0: synth.rotation(512, 1)})
    x = synth.latents(2, 512, seed=1, device="cuda")
    pe = synth.normal_bf16((2, 64), seed=2, device="cuda")
    loc = torch.tensor([1, 2], device="cuda")
    assert not try_fast_decode_store(pool, 0, loc, x, pe)  # no window metadata
    pool.set_window_meta(False, torch.tensor([3, 3], device="cuda"), torch.tensor([0, 0], device="cuda"))
    assert not try_fast_decode_store(pool, 0, loc, x, pe)  # prefill is not the decode writer's job
    pool.set_window_meta(True, torch.tensor([3], device="cuda"), torch.tensor([0, 0], device="cuda"))
    assert not try_fast_decode_store(pool, 0, loc, x, pe)  # metadata does not match the rows
    pool.set_window_meta(True, torch.tensor([3, 4], device="cuda"), torch.tensor([0, 1], device="cuda"))
    pool._audit_budget = 1
    assert not try_fast_decode_store(pool, 0, loc, x, pe)
    pool._audit_budget = 0
    assert try_fast_decode_store(pool, 0, loc, x, pe)


@pytest.mark.parametrize("d", [512, 256])
def test_rotate_quantize_matches_reference_golden(golden_dir, d):
    z = np.load(golden_dir / "rotate.npz")
    lat = torch.from_numpy(z[f"lat{d}"].view(np.int16)).view(torch.bfloat16).reshape(1, -1, d).cuda()
    r = torch.from_numpy(z[f"r{d}"])
    t, g = z[f"tg{d}"]
    for key, mask in ((f"out_plain{d}", None), (f"out_masked{d}", torch.from_numpy(z[f"mask{d}"]))):
        ref = torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16).float().numpy().reshape(-1, d)
        out = rotate_quantize(lat, r, 128, "oscar_lloyd", torch.tensor(t, dtype=torch.float32),
                              torch.tensor(g, dtype=torch.float32), high_precision_mask=mask)
        o = out.float().cpu().numpy().reshape(-1, d)
        assert np.mean(o == ref) >= 0.97
        assert np.max(np.abs(o - ref)) <= 2e-2 * max(1.0, np.abs(ref).max())
        assert cosine(o, ref) >= 0.9995


def test_learned_quantizer_matches_reference_golden(golden_dir):
    z = np.load(golden_dir / "artifact.npz")
    ref_json = json.loads((golden_dir / "artifact.json").read_text())
    q = LearnedRotationQuantizer(golden_dir / "artifact_d256")
    lat = torch.from_numpy(z["lat"].view(np.int16)).view(torch.bfloat16).cuda()

    def cmp(out, key):
        ref = torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16).float().numpy()
        o = out.float().cpu().numpy()
        assert o.shape == ref.shape
        assert np.mean(o == ref) >= 0.97 and cosine(o, ref) >= 0.9995

    cmp(q.quantize_layer(lat, 0, "nope"), "q0")
    cmp(q.quantize_layer(lat, 1, "nope"), "q1")
    cmp(q.quantize_layer(lat[:, -1:], 1, "nope"), "q1_decode")
    mask = torch.zeros(40, dtype=torch.bool)
    mask[:4] = True
    mask[-16:] = True
    q.high_precision_mask = mask
    cmp(q.quantize_layer(lat, 0, "nope"), "q0_masked")
    assert q.layer_calls == ref_json["layer_calls"]
    assert q.call_count == ref_json["call_count"] and q.element_count == ref_json["element_count"]
    assert [list(s) for s in q.first_shapes] == ref_json["first_shapes"]


def test_fold_read_rotation_matches_reference_golden(golden_dir):
    z = np.load(golden_dir / "artifact.npz")
    w = torch.from_numpy(z["w"].view(np.int16)).view(torch.bfloat16)
    ref = torch.from_numpy(z["w_folded1"].view(np.int16)).view(torch.bfloat16).float()
    out_cpu = fold_read_rotation(w, 1, golden_dir / "artifact_d256")
    out_gpu = fold_read_rotation(w.cuda(), 1, golden_dir / "artifact_d256")
    assert out_cpu.device.type == "cpu" and out_gpu.is_cuda
    assert torch.equal(out_cpu, out_gpu.cpu())
    diff = (out_cpu.float() - ref).abs()
    # accumulation order only: identical except one-ulp BF16 rounding flips
    assert (diff == 0).float().mean() >= 0.97
    assert torch.all(diff <= ref.abs() * 2 ** -7 + 1e-6)


@pytest.mark.parametrize("lloyd_max", [True, False])
def test_decode_write_unrotated_and_uniform(monkeypatch, lloyd_max):
    """The writer plugin handles what the reference's handles (mla_fused_writer.py:
    142-149, 194-224): a layer without a rotation is stored as c = c_kv, and a pool
    without Lloyd-Max stores OSCAR's uniform min/max codes; both return True."""
    monkeypatch.setenv("SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE", "1")
    d, dr, b = 512, 64, 5
    rot = {0: synth.rotation(d, 7)}  # layer 1 has no rotation
    pool = PackedLatentPool(64 * 8, 2, max_reqs=b, rotations=rot, lloyd_max=lloyd_max)
    slots = torch.tensor([70, 130, 200, 260, 333], device="cuda")
    seq = torch.tensor([9, 30, 64, 65, 200], dtype=torch.int32, device="cuda")
    req = torch.arange(b, device="cuda")
    pool.set_window_meta(True, seq, req)
    for li in range(2):
        x = synth.latents(b, d, seed=li + 3, device="cuda")
        pe = synth.normal_bf16((b, dr), seed=li + 4, device="cuda")
        assert try_fast_decode_store(pool, li, slots, x, pe)
        torch.cuda.synchronize()
        if li == 1:
            c = x.float().cpu().numpy()  # unrotated: exactly the BF16 input
        else:
            rot_gpu = torch.empty(b, d, device="cuda")
            ops.rotate_rows(x, pool.write_rotation_t(li), out_f32=rot_gpu)
            c = rot_gpu.cpu().numpy()
        s = slots.cpu().numpy()
        if lloyd_max:
            oc, osc, oze = ocodec.encode(c, *oracle_scalars(pool.codec(li)))
            prm = ocodec.params_array(osc, oze)
        else:
            oc, osc, omn = ocodec.encode_uniform(c)
            prm = ocodec.uniform_params(osc, omn)
        assert np.array_equal(pool.c_codes[li].cpu().numpy()[s], ocodec.pack(oc))
        assert np.array_equal(pool.c_params[li].cpu().numpy()[s], prm)
        assert np.array_equal(bits(pool.rope_buf[li])[s], bits(pe))


def test_backend_shim_from_req_to_token():
    """The decode-backend shim builds the page table from SGLang's token map and decodes
    exactly what the reader gives with the explicit page table; a page whose tokens are not
    one aligned run of 64 slots is reported and skipped."""
    from mla_kv_quant_b200.backend import PackedMLADecodeBackend

    d, dr, h = 512, 64, 16
    lens = [300, 64, 1, 777]
    b = len(lens)
    pool = PackedLatentPool(64 * 60, 1, max_reqs=8, rotations={0: synth.rotation(d, 3)})
    g = torch.Generator().manual_seed(4)
    pages = (torch.randperm(59, generator=g) + 1).to(torch.int32)
    mp = 13
    pt = pages[: b * mp].reshape(b, mp).cuda()
    req_idx = torch.tensor([5, 0, 7, 2], device="cuda")  # pool rows of the requests
    req_to_token = torch.zeros(8, 64 * 16, dtype=torch.int32, device="cuda")
    for i, L in enumerate(lens):
        pos = torch.arange(L, device="cuda")
        slots = pt[i, pos // 64] * 64 + pos % 64
        req_to_token[req_idx[i], :L] = slots.int()
        x = synth.latents(L, d, seed=i, device="cuda")
        pe = synth.normal_bf16((L, dr), seed=10 + i, device="cuda")
        pool.set_window_meta(False, torch.full((L,), L, dtype=torch.int32, device="cuda"),
                             torch.full((L,), int(req_idx[i]), dtype=torch.int64, device="cuda"))
        pool.set_kv_buffer(0, slots.long(), x, pe, positions=pos.int())
    seq = torch.tensor(lens, dtype=torch.int64, device="cuda")
    be = PackedMLADecodeBackend(pool, h, max_batch=8, max_context_len=64 * 16, sm_scale=0.07, num_kv_splits=3)
    be.init_forward_metadata(req_to_token, req_idx, seq)
    q = synth.normal_bf16((b, h, d + dr), seed=9, device="cuda")
    got = be.forward_decode(q.view(b, -1), 0)
    ref = packed_mla_decode_gf_fwd(q, pool, 0, pt, seq.int(), 0.07, 3)
    torch.cuda.synchronize()
    assert int(be.err.item()) == 0
    for i, L in enumerate(lens):
        n = (L + 63) // 64
        assert torch.equal(be.page_table[i, :n].cpu(), pt[i, :n].cpu())
        assert bool((be.page_table[i, n:] == -1).all())
    assert torch.equal(got, ref)
    # a request whose second page is not one aligned run of slots
    req_to_token[req_idx[0], 64 + 5] += 1
    be.init_forward_metadata(req_to_token, req_idx, seq)
    torch.cuda.synchronize()
    assert int(be.err.item()) & 2  # DEV_BAD_PAGE
    assert int(be.page_table[0, 1].item()) == -1 and int(be.page_table[0, 0].item()) == int(pt[0, 0].item())


def test_backend_shim_single_long_request_takes_more_splits():
    """A shim sized for 64 requests decodes a batch of one 12,000-token request on the split
    count of a one-request batch (64 splits, not max_batch's 2), inside the same scratch, bit
    for bit as the reader with that count, and within the decode tolerance of the oracle."""
    from mla_kv_quant_b200.backend import PackedMLADecodeBackend

    d, dr, h, L = 512, 64, 16, 12000
    n = (L + 63) // 64
    pool = PackedLatentPool(64 * (n + 2), 1, max_reqs=1, rotations={0: synth.rotation(d, 5)})
    g = torch.Generator().manual_seed(6)
    pt = (torch.randperm(n + 1, generator=g)[:n] + 1).to(torch.int32).reshape(1, n).cuda()
    pos = torch.arange(L, device="cuda")
    slots = pt[0, pos // 64] * 64 + pos % 64
    req_to_token = torch.zeros(1, 16384, dtype=torch.int32, device="cuda")
    req_to_token[0, :L] = slots.int()
    pool.set_window_meta(False, torch.full((L,), L, dtype=torch.int32, device="cuda"),
                         torch.zeros(L, dtype=torch.int64, device="cuda"))
    pool.set_kv_buffer(0, slots.long(), synth.latents(L, d, seed=7, device="cuda"),
                       synth.normal_bf16((L, dr), seed=8, device="cuda"), positions=pos.int())
    be = PackedMLADecodeBackend(pool, h, max_batch=64, max_context_len=16384, sm_scale=0.07)
    req_idx = torch.zeros(1, dtype=torch.int64, device="cuda")
    seq = torch.tensor([L], dtype=torch.int64, device="cuda")
    be.init_forward_metadata(req_to_token, req_idx, seq)
    assert be.num_kv_splits == 2 and be.splits == 64
    q = synth.normal_bf16((1, h, d + dr), seed=9, device="cuda")
    got = be.forward_decode(q.view(1, -1), 0)
    ref = packed_mla_decode_gf_fwd(q, pool, 0, pt, seq.int(), 0.07, 64)
    torch.cuda.synchronize()
    assert int(be.err.item()) == 0
    assert torch.equal(got, ref)
    want, _ = odecode.decode(_oracle_pool(pool, 0), bits(q), pt.cpu().numpy(), [L], 0.07)
    o = got.float().cpu().numpy()[0]
    assert np.max(np.abs(o - want[0]) - np.exp2(np.floor(np.log2(np.maximum(np.abs(want[0]), 1e-30))) - 8)) <= 2e-2
    assert cosine(o, want[0]) >= 0.9995


def test_hf_window_lifecycle_on_gpu(golden_dir):
    """The HF path's s4r16 window on the GPU: a 30-token prefill and 25 decode steps (batch 2,
    the second row left-padded by 3, the pad mask growing with the sequence as HF passes it).
    The row states and the number of rows re-quantized on leaving the window follow the
    oracle's window rules step by step; window rows are their BF16 input bit for bit; every
    quantized row equals the CPU oracle's rotate_quantize of its own input (quantized once,
    never twice), up to rounding ties of the FP32 rotation."""
    from mla_kv_quant_b200.hf_window import WindowedLatentCache
    from oracle import quantizer as oquant
    from oracle import window as owindow

    q = LearnedRotationQuantizer(golden_dir / "artifact_d256")
    d, b, pre, steps, pad = 256, 2, 30, 25, 3
    total = pre + steps
    pad_mask = np.ones((b, total), bool)
    pad_mask[1, :pad] = False
    cache = WindowedLatentCache(q, 4, 16)
    x = synth.latents(b * total, d, seed=3, device="cuda").view(b, 1, total, d)
    expect_state, expect_moves = None, 0
    for lo, hi in [(0, pre)] + [(t, t + 1) for t in range(pre, total)]:
        cache.pad_mask = torch.from_numpy(pad_mask[:, :hi]).cuda()
        keys = cache.update(x[:, :, lo:hi], 1)
        tgt = owindow.target_state(pad_mask[:, :hi], 4, 16)
        if expect_state is not None:
            tgt[:, :lo] = np.maximum(tgt[:, :lo], expect_state)
            expect_moves += int(((expect_state == 1) & (tgt[:, :lo] == 2)).sum())
        expect_state = tgt
        assert np.array_equal(cache.row_state[1].cpu().numpy(), expect_state)
    torch.cuda.synchronize()
    assert cache.stats["requantized_rows"] == expect_moves > 0
    keys, xin = keys.cpu(), x.cpu()
    window = torch.from_numpy(expect_state == 1)
    quant = torch.from_numpy(expect_state == 2)
    assert torch.equal(keys[:, 0][window], xin[:, 0][window])
    rows = xin[:, 0][quant].float().numpy()
    ref = oquant.rotate_quantize(rows, q.rotations[1].numpy(), q.params[1][0], q.params[1][1])
    got = keys[:, 0][quant].float().numpy()
    assert np.mean(got == ref) > 0.99 and np.max(np.abs(got - ref)) < 0.05 * np.abs(ref).max()
