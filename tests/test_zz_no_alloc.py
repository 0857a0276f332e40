"""rolaq_packed_decode_static (split partials in the library's fixed device array) against
rolaq_packed_decode (caller scratch), both called through the C ABI.

The file sorts last so that the GPU case also runs after every other decode call of the
session has used the same device; it passes on its own as well.
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import GpuPool, fill_requests
from mla_kv_quant_b200 import _lib, ops, synth


def test_static_decode_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    cap = lib.rolaq_packed_decode_static_capacity()
    assert cap == 8 << 20
    cache = _lib.LayerCache()
    cache.latent_dim, cache.rope_dim = 512, 64
    # 65535 x 16 x 2 x 513 floats > capacity: rejected before any CUDA call
    rc = lib.rolaq_packed_decode_static(None, 0, 0, 65535, 16, ctypes.byref(cache), None, 0, 1, None, None, 0.1, 1,
                                        None, 0, 0, None, None, None)
    assert rc == _lib.ROLAQ_EINVAL
    assert b"static decode scratch" in lib.rolaq_last_error()


@pytest.mark.gpu
def test_static_decode_matches_caller_scratch_twice():
    lib = _lib.load()
    d, dr, h = 512, 64, 16
    seq_lens = [700, 64, 1, 1500, 0, 333]
    b = len(seq_lens)
    mp = max(1, max((L + 63) // 64 for L in seq_lens))
    g = torch.Generator().manual_seed(3)
    pt = (torch.randperm(b * mp, generator=g) + 1).to(torch.int32).reshape(b, mp).cuda()
    pool = GpuPool(64 * (b * mp + 1), d, dr, max_reqs=b, sink=4, recent=16)
    fill_requests(pool, seq_lens, pt, synth.rotation(d, seed=8), ops.codec_serving(0.85, synth.signal_gain(0.85)),
                  seed=5)
    q = synth.normal_bf16((b, h, d + dr), seed=6, device="cuda")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    splits, sm = 3, 1.0 / np.sqrt(192.0)
    cs = pool.view().c_struct()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert (splits + 1) * b * h * (d + 1) <= lib.rolaq_packed_decode_static_capacity()

    part_o = torch.empty(b, h, splits + 1, d, device="cuda")
    part_lse = torch.empty(b, h, splits + 1, device="cuda")
    out_ref = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    lse_ref = torch.empty(b, h, device="cuda")
    rc = lib.rolaq_packed_decode(q.data_ptr(), q.stride(0), q.stride(1), b, h, ctypes.byref(cs), pt.data_ptr(),
                                 pt.stride(0), pt.shape[1], sl.data_ptr(), None, sm, splits, part_o.data_ptr(),
                                 part_lse.data_ptr(), out_ref.data_ptr(), out_ref.stride(0), out_ref.stride(1),
                                 lse_ref.data_ptr(), err.data_ptr(), stream)
    assert rc == 0, lib.rolaq_last_error()

    for _ in range(2):  # two calls in a row reuse the same static scratch
        out = torch.full_like(out_ref, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        rc = lib.rolaq_packed_decode_static(q.data_ptr(), q.stride(0), q.stride(1), b, h, ctypes.byref(cs),
                                            pt.data_ptr(), pt.stride(0), pt.shape[1], sl.data_ptr(), None, sm, splits,
                                            out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
                                            err.data_ptr(), stream)
        assert rc == 0, lib.rolaq_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        # same kernels on the same inputs: equal up to the decode tolerance (in practice bit for bit)
        assert torch.isfinite(out.float()).all()
        assert (out.float() - out_ref.float()).abs().max().item() <= 1e-6
        ok = torch.isfinite(lse_ref)
        assert torch.equal(ok, torch.isfinite(lse))
        assert (lse[ok] - lse_ref[ok]).abs().max().item() <= 1e-6
