"""Host-side logic of the drop-in modules (no GPU needed)."""

import json
import shutil

import numpy as np
import pytest
import torch

from mla_kv_quant_b200 import ops, rolaq_mla, synth
from mla_kv_quant_b200.envs import envs
from mla_kv_quant_b200.pool import PackedLatentPool
from mla_kv_quant_b200.quantizer import LearnedRotationQuantizer, rotate_quantize
from mla_kv_quant_b200.seqsplit import rank_token_range
from oracle import codec as ocodec


def test_learned_quantizer_loads_golden_artifact(golden_dir):
    q = LearnedRotationQuantizer(golden_dir / "artifact_d256")
    ref = json.loads((golden_dir / "artifact.json").read_text())
    meta = q.metadata()
    meta.pop("rotation_dir")
    assert meta == ref["metadata"]
    assert q.width == 256 and q.family == "oscar_lloyd"
    assert q.layer_calls == {"0": {"prefill": 0, "decode": 0}, "1": {"prefill": 0, "decode": 0}}


def _copy_artifact(golden_dir, tmp_path):
    dst = tmp_path / "art"
    shutil.copytree(golden_dir / "artifact_d256", dst)
    return dst


def test_learned_quantizer_rejects_bad_artifacts(golden_dir, tmp_path):
    art = _copy_artifact(golden_dir, tmp_path)
    m = json.loads((art / "manifest.json").read_text())
    bad = dict(m, recipe="other")
    (art / "manifest.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="not a learned rotation artifact"):
        LearnedRotationQuantizer(art)
    bad = json.loads(json.dumps(m))
    bad["layers"]["0"]["sha256"] = "0" * 64
    (art / "manifest.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="hash mismatch"):
        LearnedRotationQuantizer(art)
    bad = json.loads(json.dumps(m))
    bad["layers"]["1"]["param1"] = 1.5  # gain outside [0.8, 1.3]
    (art / "manifest.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="out of bounds"):
        LearnedRotationQuantizer(art)
    bad = dict(m, windows=True)
    (art / "manifest.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="window lifecycle"):
        LearnedRotationQuantizer(art)


def test_quantize_layer_validation_and_no_cpu_fallback(golden_dir):
    q = LearnedRotationQuantizer(golden_dir / "artifact_d256")
    x = torch.zeros(1, 4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="nope only"):
        q.quantize_layer(x, 0, "rope")
    with pytest.raises(ValueError, match="invalid MLA latent"):
        q.quantize_layer(torch.zeros(1, 4, 128, dtype=torch.bfloat16), 0, "nope")
    with pytest.raises(ValueError, match="missing learned rotation"):
        q.quantize_layer(x, 7, "nope")
    with pytest.raises(ValueError, match="CUDA tensors only"):
        q.quantize_layer(x, 0, "nope")
    with pytest.raises(ValueError, match="high precision mask shape"):
        rotate_quantize(x, torch.eye(256), 128, "oscar_lloyd", 0.9, 1.0, high_precision_mask=torch.ones(3, dtype=torch.bool))
    # an all-True mask returns the input untouched without any device work
    assert rotate_quantize(x, torch.eye(256), 128, "oscar_lloyd", 0.9, 1.0,
                           high_precision_mask=torch.ones(4, dtype=torch.bool)) is x


def test_serving_loader_matches_reference(golden_dir):
    ref = json.loads((golden_dir / "artifact.json").read_text())
    art = str(golden_dir / "artifact_d256")
    got = rolaq_mla.load_layer_quantizers(art, art, 128, 256, [0, 1])
    assert [list(x) for x in got] == ref["load_layer_quantizers"]
    assert rolaq_mla.load_layer_quantizers("", art, 128, 256, [0, 1]) == [None, None]
    with pytest.raises(ValueError, match="same artifact"):
        rolaq_mla.load_layer_quantizers(art, str(golden_dir), 128, 256, [0])
    with pytest.raises(ValueError, match="cache dimensions"):
        rolaq_mla.load_layer_quantizers(art, art, 128, 512, [0])


def test_codec_scalars_match_oracle():
    for t, g in [(0.9810652732849121, 1.16), (0.83, 1.0123), (0.5, 0.8), (1.5, 1.3)]:
        hf = ops.codec_hf(t, g)
        ht, hsf, hz = ocodec.hf_scalars(t, g)
        assert (np.float32(hf.threshold), np.float32(hf.scale_factor), np.float32(hf.zero_const)) == (ht, hsf, hz)
        sv = ops.codec_serving(t, g)
        st, ssf, sz = ocodec.serving_scalars(t, g)
        assert (np.float32(sv.threshold), np.float32(sv.scale_factor), np.float32(sv.zero_const)) == (st, ssf, sz)


def test_pool_accounting_matches_reference_formula():
    pool = PackedLatentPool(size=64 * 10, layer_num=27, max_reqs=8, device="cpu")
    # per token: codes D/4 + params 8*NG + k_pe 2*Dr per layer, + one int32 ring-map entry
    assert pool.cell_size_bytes() == (128 + 32 + 128) * 27 + 4
    assert pool.fixed_overhead_bytes() == (1 + 8 * 20) * (512 * 2 * 27 + 4)
    assert pool.get_kv_size_bytes() == pool.cell_size_bytes() * 640 + pool.fixed_overhead_bytes()
    assert len(pool.c_codes) == 27 and tuple(pool.c_codes[0].shape) == (640, 128)
    with pytest.raises(ValueError, match="multiple of 64"):
        PackedLatentPool(size=100, layer_num=1, device="cpu")
    with pytest.raises(ValueError, match="SGLANG_LLOYD_MAX"):
        PackedLatentPool(size=64, layer_num=1, device="cpu", quantizer_params=[(0.9, 1.0)], lloyd_max=False)


def test_env_flags(monkeypatch):
    monkeypatch.setenv("SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE", "1")
    monkeypatch.setenv("SGLANG_MIXED_KV_RECENT_TOKENS", "8")
    assert envs.SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE.get() is True
    assert envs.SGLANG_MIXED_KV_RECENT_TOKENS.get() == 8
    monkeypatch.delenv("SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE")
    assert envs.SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE.get() is False


def test_backend_split_count_follows_the_batch():
    """The decode-backend shim sizes its scratch for max_batch x (num_kv_splits + 1) partials
    per head and gives a smaller batch more splits within that room; an explicit
    num_kv_splits stays fixed."""
    from types import SimpleNamespace

    from mla_kv_quant_b200.backend import PackedMLADecodeBackend

    pool = SimpleNamespace(kv_lora_rank=512, qk_rope_head_dim=64, device=torch.device("cpu"))
    be = PackedMLADecodeBackend(pool, 16, max_batch=64, max_context_len=16384, sm_scale=0.07)
    assert be.num_kv_splits == ops.default_num_splits(64, 16384) == 2
    assert be.splits_for(64) == 2
    assert be.splits_for(1) == ops.default_num_splits(1, 16384) == 64
    for b in range(1, 65):
        s = be.splits_for(b)
        assert 1 <= s and b * (s + 1) <= 64 * (2 + 1)
    fixed = PackedMLADecodeBackend(pool, 16, max_batch=8, max_context_len=1024, sm_scale=0.07, num_kv_splits=3)
    assert fixed.splits_for(1) == fixed.splits_for(8) == 3


def test_split_heuristics_and_ranges():
    s = ops.default_num_splits(64, 16384)
    assert 1 <= s <= 64
    assert ops.default_num_splits(1, 100) == 1
    # the benchmarked shapes: B64 x 16K and B128 x 8K one wave, window split first; B64 x 32K
    # (a 4(a) rank) four waves; one 128K request on 128 splits
    assert ops.default_num_splits(64, 16384) == 2
    assert ops.default_num_splits(128, 8192, latent_dim=256, rope_dim=32, heads=40) == 1
    assert ops.default_num_splits(64, 32768) == 9
    assert ops.default_num_splits(1, 131072) == 128
    # a few long requests: never one full wave of many splits with no SM left for the window
    # split (B2 x 128K: 74 splits measured 62.4 us, 73 splits 47.1)
    for b, ctx in ((2, 131072), (2, 65536), (4, 65536), (4, 131072), (4, 32768)):
        s = ops.default_num_splits(b, ctx)
        free = 148 - b * s
        assert free >= 1 and free * 2 * 4 >= b, (b, ctx, s)
    for L in (1, 63, 64, 65, 4097, 131072):
        for world in (1, 2, 3, 8):
            ranges = [rank_token_range(L, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == L
            for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
                assert a1 == b0 and (a0 % 64 == 0 or a0 == L)
            assert sum(e - s for s, e in ranges) == L


def test_synth_distributions():
    p = synth.layer_params(27)
    assert all(0.7 <= t <= 1.0 and 0.8 <= g <= 1.3 for t, g in p)
    r = synth.rotation(64, 1)
    assert torch.allclose(r.double().T @ r.double(), torch.eye(64, dtype=torch.float64), atol=1e-6)
    pt, slots = synth.page_table(3, 130)
    assert pt.shape == (3, 3) and int(pt.min()) >= 1 and slots == (3 * 3 + 1) * 64
    assert len(set(pt.flatten().tolist())) == 9


def _fake_checkpoint(tmp_path):
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.make_fake_checkpoint(tmp_path / "fake-minicpm3")


def test_checkpoint_fingerprint_matches_reference(golden_dir, tmp_path):
    from mla_kv_quant_b200.artifacts import checkpoint_fingerprint

    ckpt = _fake_checkpoint(tmp_path)
    assert checkpoint_fingerprint(ckpt) == json.loads((golden_dir / "fingerprint.json").read_text())


def test_validate_config_checks_the_checkpoint(tmp_path):
    from types import SimpleNamespace

    from mla_kv_quant_b200.artifacts import checkpoint_fingerprint, write_synthetic_artifact

    ckpt = _fake_checkpoint(tmp_path)
    rots = {i: synth.rotation(256, 60 + i) for i in range(2)}
    write_synthetic_artifact(tmp_path / "art", rots, {0: (0.8, 1.0), 1: (0.9, 1.1)}, checkpoint_fingerprint(ckpt))
    q = LearnedRotationQuantizer(tmp_path / "art")
    cfg = SimpleNamespace(model_type="minicpm3", num_hidden_layers=2, kv_lora_rank=256, qk_rope_head_dim=32,
                          _name_or_path=str(ckpt))
    q.validate_config(cfg)
    with pytest.raises(ValueError, match="model mismatch: kv_lora_rank"):
        q.validate_config(SimpleNamespace(**dict(vars(cfg), kv_lora_rank=512)))
    (ckpt / "model-00002-of-00002.safetensors").write_bytes(b"\x00" * 10)
    with pytest.raises(ValueError, match="shard names/sizes differ"):
        q.validate_config(SimpleNamespace(**vars(cfg)))
