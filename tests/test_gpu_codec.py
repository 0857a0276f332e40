"""CUDA codec kernels against the oracle: bit-exact codes and params."""

import numpy as np
import pytest
import torch

from mla_kv_quant_b200 import _lib, ops
from oracle import codec as ocodec

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    g = torch.Generator().manual_seed(seed)
    s = torch.exp(0.5 * torch.randn(d, generator=g))
    x = torch.randn(n, d, generator=g) * s
    x[0] = 0.75  # constant groups
    x[1, ::2], x[1, 1::2] = 1.0, -1.0  # exact +-1 groups
    x[2] = torch.arange(d) * 0.01 - 1.0
    x[3] *= 1e-3
    return x.float()


@pytest.mark.parametrize("d", [512, 256])
@pytest.mark.parametrize("slots64", [True, False])
def test_scatter_pack_bit_exact(d, slots64):
    n, num_slots = 300, 1024
    x = _rows(n, d, seed=d)
    g = torch.Generator().manual_seed(5)
    slots = torch.randperm(num_slots, generator=g)[:n]
    codec = ops.codec_serving(0.87, 1.04)
    codes = torch.zeros(num_slots, d // 4, dtype=torch.uint8, device="cuda")
    params = torch.zeros(num_slots, d // 128, 2, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = slots.cuda().to(torch.int64 if slots64 else torch.int32)
    ops.scatter_pack_rows(x.cuda(), s, codes, params, codec, err=err)
    torch.cuda.synchronize()
    oc, osc, oze = ocodec.encode(x.numpy(), np.float32(codec.threshold), np.float32(codec.scale_factor),
                                 np.float32(codec.zero_const))
    got_codes = codes.cpu().numpy()[slots.numpy()]
    got_params = params.cpu().numpy()[slots.numpy()]
    assert np.array_equal(got_codes, ocodec.pack(oc))
    assert np.array_equal(got_params, ocodec.params_array(osc, oze))
    assert int(err.item()) == 0
    # untouched slots stay zero
    untouched = np.setdiff1d(np.arange(num_slots), slots.numpy())
    assert not codes.cpu().numpy()[untouched].any()


def test_scatter_pack_bad_slot_reported_not_written():
    d = 512
    x = _rows(4, d, seed=1).cuda()
    codes = torch.zeros(16, d // 4, dtype=torch.uint8, device="cuda")
    params = torch.zeros(16, 4, 2, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    slots = torch.tensor([1, 16, -3, 2], dtype=torch.int64, device="cuda")
    ops.scatter_pack_rows(x, slots, codes, params, ops.codec_serving(0.9, 1.0), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEV_BAD_SLOT
    written = codes.cpu().numpy().any(axis=1)
    assert written[1] and written[2] and written.sum() == 2


@pytest.mark.parametrize("d", [512, 256])
def test_dequant_matches_oracle(d):
    x = _rows(200, d, seed=3)
    codec = ops.codec_hf(0.8, 1.01)
    codes = torch.zeros(200, d // 4, dtype=torch.uint8, device="cuda")
    params = torch.zeros(200, d // 128, 2, dtype=torch.float32, device="cuda")
    ops.scatter_pack_rows(x.cuda(), torch.arange(200, device="cuda"), codes, params, codec)
    out32 = torch.empty(200, d, device="cuda")
    out16 = torch.empty(200, d, dtype=torch.bfloat16, device="cuda")
    ops.dequant_rows(codes, params, out_f32=out32, out_bf16=out16)
    perm = torch.randperm(200, generator=torch.Generator().manual_seed(2))[:50]
    sel = torch.empty(50, d, device="cuda")
    ops.dequant_rows(codes, params, slots=perm.cuda(), out_f32=sel)
    torch.cuda.synchronize()
    ref = ocodec.qdq(x.numpy(), np.float32(codec.threshold), np.float32(codec.scale_factor))
    assert np.array_equal(out32.cpu().numpy(), ref)
    assert torch.equal(out16.cpu(), torch.from_numpy(ref).to(torch.bfloat16))
    assert np.array_equal(sel.cpu().numpy(), ref[perm.numpy()])


def test_prepare_gf_splits():
    s = torch.tensor([0, 1, 2, 5, 129], dtype=torch.int32, device="cuda")
    q = torch.empty_like(s)
    m = torch.empty_like(s)
    ops.prepare_gf_splits(s, q, m)
    assert q.tolist() == [1, 1, 1, 4, 128]
    assert m.tolist() == [2, 2, 2, 5, 129]


def _uniform_rows(n, d, seed):
    x = _rows(n, d, seed)
    x[4] = torch.tensor([0.0, 0.5, 1.5, 2.5, 3.0, 1.0, 2.0, 0.25]).repeat(d // 8)  # scale 1: exact .5 ties
    x[5] = x[4] - 7.0
    return x


@pytest.mark.parametrize("d", [512, 256])
def test_scatter_pack_uniform_bit_exact(d):
    """OSCAR's uniform min/max codec (lloyd_max=False) through the scatter-pack kernel."""
    from mla_kv_quant_b200.mla_latent_int2 import scatter_pack_rows

    n, num_slots = 300, 1024
    x = _uniform_rows(n, d, seed=d + 1)
    slots = torch.randperm(num_slots, generator=torch.Generator().manual_seed(6))[:n]
    codes = torch.zeros(num_slots, d // 4, dtype=torch.uint8, device="cuda")
    params = torch.zeros(num_slots, d // 128, 2, dtype=torch.float32, device="cuda")
    scatter_pack_rows(x.cuda(), slots.cuda().to(torch.int32), codes, params, 128, lloyd_max=False)
    torch.cuda.synchronize()
    oc, osc, omn = ocodec.encode_uniform(x.numpy())
    s = slots.numpy()
    assert np.array_equal(codes.cpu().numpy()[s], ocodec.pack(oc))
    assert np.array_equal(params.cpu().numpy()[s], ocodec.uniform_params(osc, omn))


@pytest.mark.parametrize("d", [512, 256])
@pytest.mark.parametrize("n", [64, 1000])
def test_fused_write_uniform_bit_exact(d, n):
    """The fused writer with the uniform codec (n = 64: the SIMT small-batch kernel; 1000:
    the tcgen05 kernel) against the oracle codec on the kernel's own FP32 rotation."""
    from mla_kv_quant_b200 import synth

    x = synth.latents(n, d, seed=n + d, device="cuda")
    rt = synth.rotation(d, seed=7).to(torch.bfloat16).t().contiguous().cuda()
    codes = torch.zeros(n + 64, d // 4, dtype=torch.uint8, device="cuda")
    params = torch.zeros(n + 64, d // 128, 2, dtype=torch.float32, device="cuda")
    slots = torch.arange(64, 64 + n, device="cuda")
    ops.encode_rows(x, rt, ops.codec_uniform(), codes, params, slots=slots)
    rot = torch.empty(n, d, device="cuda")
    ops.rotate_rows(x, rt, out_f32=rot)
    torch.cuda.synchronize()
    oc, osc, omn = ocodec.encode_uniform(rot.cpu().numpy())
    assert np.array_equal(codes.cpu().numpy()[64:], ocodec.pack(oc))
    assert np.array_equal(params.cpu().numpy()[64:], ocodec.uniform_params(osc, omn))
