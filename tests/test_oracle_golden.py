"""The CPU oracle against golden vectors produced by the reference itself.

Fixtures: tests/golden/make_golden.py ran mla_quant.oscar.oscar_lloyd_int2_qdq,
quantize_learned and rotate_quantize (noforit/mla_kv_quant) on seeded inputs.
"""

import numpy as np
import pytest

from oracle import codec, decode, quantizer, window, writer


def _flips(ours, ref, scale):
    """Elements whose value differs by more than a quarter code step (a code flip)."""
    step = np.repeat(scale, codec.GROUP, axis=1)
    return np.abs(ours - ref) > 0.25 * step


@pytest.mark.parametrize("style", ["direct", "hf"])
def test_codec_matches_reference(golden_dir, style):
    z = np.load(golden_dir / "codec.npz")
    x = z["x"]
    total = flips = 0
    for k, (t, g) in enumerate(z["pairs"]):
        scal = codec.serving_scalars(t, g) if style == "direct" else codec.hf_scalars(t, g)
        c, sc, ze = codec.encode(x, *scal)
        ours = codec.dequant(c, sc, ze)
        ref = z[style][k]
        f = _flips(ours, ref, sc)
        flips += int(f.sum())
        total += f.size
        # away from code flips the values agree to a few FP32 ulps of the group scale
        tol = 8 * np.finfo(np.float32).eps * (np.abs(ref) + np.repeat(sc, codec.GROUP, axis=1))
        assert np.all(np.abs(ours - ref)[~f] <= tol[~f])
    # the reference's own tie fraction bound (north star: <= 1e-4); observed 0
    assert flips / total <= 1e-4


def test_hf_scalar_gain_substitution():
    # FP32(1.16) is replaced by the double 1.16 (quantizer.py:33-34)
    t32, sf, _ = codec.hf_scalars(0.98, np.float32(1.16))
    assert sf == np.float32(codec.SPAN3 * 1.16)
    _, sf2, _ = codec.hf_scalars(0.98, 1.0000001)
    assert sf2 == np.float32(codec.SPAN3 * float(np.float32(1.0000001)))


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    c = rng.integers(0, 4, size=(17, 512), dtype=np.uint8)
    p = codec.pack(c)
    assert p.shape == (17, 128)
    assert np.array_equal(codec.unpack(p, 512), c)
    # bit layout: element j at byte j // 4, bits 2 * (j % 4)
    one = np.zeros((1, 512), np.uint8)
    one[0, 5] = 3
    assert codec.pack(one)[0, 1] == 3 << 2


def test_constant_group_edge_case():
    x = np.full((2, 128), 3.25, np.float32)
    c, sc, ze = codec.encode(x, *codec.serving_scalars(0.9, 1.0))
    assert np.all(c == 2)  # n = 0 -> [n >= -t] + [n >= 0]
    assert np.allclose(sc, np.float32(codec.SPAN3) * np.sqrt(np.float32(1e-8)))


@pytest.mark.parametrize("d", [512, 256])
def test_rotate_quantize_restatement(golden_dir, d):
    import torch

    z = np.load(golden_dir / "rotate.npz")
    r = z[f"r{d}"]
    lat = writer.bf16_to_f32(z[f"lat{d}"].reshape(-1, d))
    t, g = z[f"tg{d}"]
    restored = quantizer.rotate_quantize(lat, r, t, g)
    ref = writer.bf16_to_f32(z[f"out_plain{d}"].reshape(-1, d))
    # identical except where a ULP of mean/std moved a BF16 rounding
    assert np.mean(restored == ref) > 0.99
    assert np.max(np.abs(restored - ref)) < 0.05 * np.max(np.abs(ref))
    mask = z[f"mask{d}"]
    masked = quantizer.rotate_quantize(lat, r, t, g, mask=mask)
    refm = writer.bf16_to_f32(z[f"out_masked{d}"].reshape(-1, d))
    assert np.array_equal(masked[mask], refm[mask])


def test_window_state_and_ring():
    valid = np.ones((2, 30), bool)
    valid[1, :5] = False  # left padding
    st = window.target_state(valid, 4, 16)
    assert list(st[0, :4]) == [1] * 4 and list(st[0, 4:14]) == [2] * 10 and list(st[0, 14:]) == [1] * 16
    assert list(st[1, :5]) == [0] * 5 and list(st[1, 5:9]) == [1] * 4
    # ring: sinks map to 1 + req*20 + pos, recents wrap modulo 16
    assert window.ring_row(3, 2, 4, 16) == 1 + 60 + 2
    assert window.ring_row(3, 4, 4, 16) == 1 + 60 + 4
    assert window.ring_row(3, 20, 4, 16) == 1 + 60 + 4  # (20 - 4) % 16 == 0
    assert window.ring_row(0, 19, 4, 16) == 1 + 4 + 15


def test_oracle_writer_and_decode_small():
    rng = np.random.default_rng(1)
    d, dr, h = 256, 32, 4
    pool = writer.Pool(num_slots=64 * 4, d=d, dr=dr, max_reqs=2, sink=4, recent=16)
    L = 100
    pt = np.array([[1, 3]], np.int32)
    slots = decode.token_slots(pt[0], L)
    x = rng.standard_normal((L, d)).astype(np.float32)
    kpe = writer.bf16_bits(rng.standard_normal((L, dr)).astype(np.float32))
    writer.write(pool, x, kpe, slots, np.full(L, L), np.zeros(L, np.int64), *codec.serving_scalars(0.9, 1.05)[:2],
                 positions=np.arange(L))
    # window rows hold the BF16 rotated latent and belong to their slots
    for p in list(range(4)) + list(range(L - 16, L)):
        r = pool.rows[slots[p]]
        assert r >= 0 and pool.owners[r] == slots[p]
    assert pool.rows[slots[50]] == -1
    q = writer.bf16_bits(rng.standard_normal((1, h, d + dr)).astype(np.float32))
    out, lse = decode.decode(pool, q, pt, [L], 0.1)
    # the split/merge identity: two halves merged equal the whole
    qf = writer.bf16_to_f32(q).astype(np.float64)[0]
    lat = decode.latent_rows(pool, slots, L)
    pe = writer.bf16_to_f32(pool.rope[slots]).astype(np.float64)
    o1, l1 = decode.attend(qf, lat[:37], pe[:37], 0.1)
    o2, l2 = decode.attend(qf, lat[37:], pe[37:], 0.1)
    om, lm = decode.merge(np.stack([o1, o2]), np.stack([l1, l2]))
    assert np.allclose(om, out[0]) and np.allclose(lm, lse[0])


def test_uniform_codec_restatement(golden_dir):
    """OSCAR's uniform min/max INT2 codec: the restated codes reconstruct the reference's
    ``uniform_int2_qdq`` output bit for bit, ties to even included."""
    z = np.load(golden_dir / "uniform.npz")
    x, deq = z["x"], z["deq"]
    assert np.array_equal(codec.uniform_qdq(x), deq)
    codes, scale, mn = codec.encode_uniform(x)
    ties = codes[24, :8]  # (0, .5, 1.5, 2.5, 3, 1, 2, .25) with scale 1: halves go to even
    assert list(ties) == [0, 0, 2, 2, 3, 1, 2, 0]
    assert np.all(scale[26] == 1.0) and np.all(codes[26] == 0)  # constant group
