"""The tcgen05 fused writer against the oracle and a plain FP32 reference.

* The rotation GEMM agrees with the FP32 GEMM of the same BF16 operands to
  accumulation-order rounding.
* The codec stage is bit-exact: codes/params equal the oracle codec applied to the
  kernel's own FP32 rotation (rolaq_rotate_rows shares the MMA and its order).
* Against the reference rotation (torch FP32 GEMM) codes differ only at rounding
  ties: <= 1e-4 of all codes.
* k_pe, ring rows and slot<->ring maps equal the oracle writer's.
"""

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, bits, f32_of_bf16, oracle_scalars, rotate_cpu
from mla_kv_quant_b200 import _lib, ops, synth
from oracle import codec as ocodec
from oracle import writer as owriter

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d", [512, 256])
@pytest.mark.parametrize("n", [1, 64, 129, 1000])
def test_rotate_rows_matches_fp32_gemm(d, n):
    x = synth.latents(n, d, seed=n, device="cuda")
    r = synth.rotation(d, seed=d + 1)
    rt = r.to(torch.bfloat16).t().contiguous().cuda()
    out32 = torch.empty(n, d, device="cuda")
    out16 = torch.empty(n, d, dtype=torch.bfloat16, device="cuda")
    ops.rotate_rows(x, rt, out_f32=out32, out_bf16=out16)
    torch.cuda.synchronize()
    ref = rotate_cpu(x, r)
    err = np.abs(out32.cpu().numpy() - ref)
    scale = np.abs(f32_of_bf16(x)).max(axis=1, keepdims=True) * np.sqrt(d)
    assert np.all(err <= 1e-5 * scale)
    assert torch.equal(out16.cpu(), out32.cpu().to(torch.bfloat16))


@pytest.mark.parametrize("d,dr", [(512, 64), (256, 32)])
@pytest.mark.parametrize("n", [1, 64, 129, 1000])
def test_fused_write_codec_bit_exact(d, dr, n):
    num_slots = 64 * ((n + 63) // 64 + 2)
    pool = GpuPool(num_slots, d, dr, max_reqs=4)
    x = synth.latents(n, d, seed=7 + n, device="cuda")
    pe = synth.normal_bf16((n, dr), seed=9, device="cuda")
    r = synth.rotation(d, seed=3)
    rt = r.to(torch.bfloat16).t().contiguous().cuda()
    slots = (torch.randperm(num_slots - 1, generator=torch.Generator().manual_seed(n))[:n] + 1).cuda()
    codec = ops.codec_serving(0.83, synth.signal_gain(0.83))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fused_write(x, pe, slots, rt, codec, pool.view(), err=err)
    rot = torch.empty(n, d, device="cuda")
    ops.rotate_rows(x, rt, out_f32=rot)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    s = slots.cpu().numpy()
    oc, osc, oze = ocodec.encode(rot.cpu().numpy(), *oracle_scalars(codec))
    assert np.array_equal(pool.codes.cpu().numpy()[s], ocodec.pack(oc))
    assert np.array_equal(pool.params.cpu().numpy()[s], ocodec.params_array(osc, oze))
    assert np.array_equal(bits(pool.rope)[s], bits(pe))
    # against the reference FP32 GEMM: only rounding ties may flip
    rc, rsc, _ = ocodec.encode(rotate_cpu(x, r), *oracle_scalars(codec))
    got = ocodec.unpack(pool.codes.cpu().numpy()[s], d)
    assert np.mean(got != rc) <= 1e-4
    assert np.allclose(pool.params.cpu().numpy()[s][..., 0], rsc, rtol=1e-5)


@pytest.mark.parametrize("mode", ["decode", "prefill"])
def test_fused_write_window_stores(mode):
    d, dr, max_reqs = 512, 64, 6
    pool = GpuPool(64 * 40, d, dr, max_reqs=max_reqs)
    opool = pool.to_oracle()
    r = synth.rotation(d, seed=11)
    rt = r.to(torch.bfloat16).t().contiguous().cuda()
    codec = ops.codec_serving(0.9, synth.signal_gain(0.9))
    g = torch.Generator().manual_seed(0)
    steps = 3 if mode == "decode" else 1
    for step in range(steps):
        if mode == "decode":
            # one new token per request (ids 0..5), one request id outside the ring
            # (6 >= max_reqs) and one CUDA-graph padding row at slot 0
            n = 8
            seq = torch.tensor([5, 17, 20, 21, 37, 1, 9, 9], dtype=torch.int32) + step
            req = torch.tensor([0, 1, 2, 3, 4, 5, 6, 0], dtype=torch.int64)
            slots = torch.randperm(64 * 40 - 1, generator=g)[:n] + 1
            slots[7] = 0
            pos = None
        else:
            n = 300
            L = 300
            seq = torch.full((n,), L, dtype=torch.int32)
            req = torch.full((n,), 2, dtype=torch.int64)
            pos = torch.arange(n, dtype=torch.int32)
            slots = torch.randperm(64 * 40 - 1, generator=g)[:n] + 1
        x = synth.latents(n, d, seed=step, device="cuda")
        pe = synth.normal_bf16((n, dr), seed=step + 50, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        ops.fused_write(x, pe, slots.cuda(), rt, codec, pool.view(), seq_lens=seq.cuda(), req_idx=req.cuda(),
                        positions=None if pos is None else pos.cuda(), err=err)
        rot = torch.empty(n, d, device="cuda")
        ops.rotate_rows(x, rt, out_f32=rot)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        owriter.write(opool, rot.cpu().numpy(), bits(pe), slots.numpy(), seq.numpy(), req.numpy(),
                      *oracle_scalars(codec)[:2], positions=None if pos is None else pos.numpy())
    got = pool.to_oracle()
    assert np.array_equal(got.codes, opool.codes)
    assert np.array_equal(got.params, opool.params)
    assert np.array_equal(got.rope, opool.rope)
    assert np.array_equal(got.rows, opool.rows)
    assert np.array_equal(got.owners, opool.owners)
    assert np.array_equal(got.hp, opool.hp)


def test_fused_write_bad_slot_flag():
    d, dr = 256, 32
    pool = GpuPool(128, d, dr, max_reqs=1)
    x = synth.latents(3, d, seed=1, device="cuda")
    pe = synth.normal_bf16((3, dr), seed=2, device="cuda")
    rt = synth.rotation(d, 1).to(torch.bfloat16).t().contiguous().cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fused_write(x, pe, torch.tensor([5, 500, 6], device="cuda"), rt, ops.codec_serving(0.9, 1.0), pool.view(),
                    err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEV_BAD_SLOT
    written = pool.codes.cpu().numpy().any(axis=1)
    assert written[5] and written[6] and written.sum() == 2


def test_fused_write_rejects_bad_arguments():
    d, dr = 512, 64
    pool = GpuPool(128, d, dr, max_reqs=1)
    x = synth.latents(4, d, seed=1, device="cuda")
    pe = synth.normal_bf16((4, dr), seed=2, device="cuda")
    rt = synth.rotation(d, 1).to(torch.bfloat16).t().contiguous().cuda()
    with pytest.raises(ValueError):
        ops.fused_write(x[:, :256], pe, torch.arange(4, device="cuda"), rt, ops.codec_serving(0.9, 1.0), pool.view())
    with pytest.raises(_lib.RolaqError, match="finite and > 0"):
        ops.fused_write(x, pe, torch.arange(4, device="cuda"), rt, _lib.Codec(0.0, 1.0, 1.5), pool.view())


@pytest.mark.parametrize("side", ["at", "above", "below"])
@pytest.mark.parametrize("sign", [1, -1])
def test_fused_write_codes_at_quotient_boundaries(side, sign):
    """The threshold sits exactly on a normalised value that many elements share (and one
    FP32 step either side of it).  With the identity rotation the kernel's rotated rows are
    the BF16 inputs, so these elements are decided by the writer's exact quotient bounds
    ([n >= t] with n == t must hold, with n one step below t must not)."""
    d, dr, n = 512, 64, 256
    rng = np.random.default_rng(11)
    base = (rng.integers(-3, 4, size=(n, d)) * np.exp2(rng.integers(-3, 4, size=(n, 1)))).astype(np.float32)
    x = torch.from_numpy(base).to(torch.bfloat16)  # small integers times powers of two: exact
    g = base.reshape(n, d // 128, 128)
    mean = ocodec.group_sum(g) * ocodec.INV_GROUP
    diff = g - mean[..., None]
    std = np.sqrt(ocodec.group_sum(diff * diff) * ocodec.INV_GROUP + ocodec.EPS)
    nrm = diff / std[..., None]
    cand = nrm[(sign * nrm > 0.55) & (sign * nrm < 1.45)]
    vals, counts = np.unique(cand, return_counts=True)
    t = np.float32(abs(vals[np.argmax(counts)]))
    t = {"at": t, "above": np.nextafter(t, np.float32(np.inf)), "below": np.nextafter(t, np.float32(-np.inf))}[side]
    assert np.sum(np.abs(nrm) == np.float32(abs(vals[np.argmax(counts)]))) >= 8  # the boundary is populated

    num_slots = 64 * (n // 64 + 2)
    pool = GpuPool(num_slots, d, dr, max_reqs=4)
    slots = (torch.arange(n) + 64).cuda()
    rt = torch.eye(d, dtype=torch.bfloat16, device="cuda")
    codec = ops.codec_serving(float(t), synth.signal_gain(0.85))
    assert np.float32(codec.threshold) == t
    pe = synth.normal_bf16((n, dr), seed=1, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fused_write(x.cuda(), pe, slots, rt, codec, pool.view(), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    oc, osc, oze = ocodec.encode(base, *oracle_scalars(codec))
    s = slots.cpu().numpy()
    assert np.array_equal(pool.codes.cpu().numpy()[s], ocodec.pack(oc))
    assert np.array_equal(pool.params.cpu().numpy()[s], ocodec.params_array(osc, oze))
