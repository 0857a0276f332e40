"""Generate the golden fixtures in this folder by running the reference itself.

Run once, in a container where the reference (noforit/mla_kv_quant) is checked out:

    python tests/golden/make_golden.py --reference /path/to/mla_kv_quant

It imports the reference's own ``mla_quant`` and ``deployment/sglang/srt/mem_cache``
modules on the CPU, with ``configure_reference_numerics()`` applied, and records
their outputs on seeded inputs.  Nothing here is used at test time except the files
it writes; the tests never import the reference.

Fixtures written:

* ``fingerprint.json`` -- ``local_checkpoint_fingerprint`` (``mla_quant/artifacts.py:43-58``)
  of the fake checkpoint ``make_fake_checkpoint`` builds.
* ``uniform.npz``   -- ``uniform_int2_qdq`` (``mla_quant/oscar.py:91-101``), OSCAR's
  uniform min/max INT2 baseline, on seeded rows plus exact-tie and constant groups.
* ``codec.npz``     -- ``oscar_lloyd_int2_qdq`` (``mla_quant/oscar.py:120-144``) on
  seeded FP32 rows for several (threshold, gain) pairs, plus the HF-path scalar
  handling through ``quantize_learned`` (``mla_quant/quantizer.py:31-35, 73-82``).
* ``rotate.npz``    -- ``rotate_quantize`` (``mla_quant/quantizer.py:102-124``) on BF16
  latents with an s4r16 high-precision mask, D = 512 and D = 256.
* ``artifact_d256/`` -- a two-layer v2 learned artifact (manifest + ``layer_{i}.pt``),
  and ``artifact.npz`` / ``artifact.json``: ``LearnedRotationQuantizer.quantize_layer``
  outputs, ``metadata()``, ``layer_calls``; the serving loader's
  ``load_layer_quantizers`` values and ``fold_read_rotation`` output
  (``deployment/sglang/srt/mem_cache/rolaq_mla.py:16-71``).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def orthogonal(d: int, seed: int) -> np.ndarray:
    import torch

    g = torch.Generator().manual_seed(seed)
    a = torch.randn(d, d, generator=g, dtype=torch.float64)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r))[None, :]
    return q.float().numpy()


def latents(n: int, d: int, seed: int) -> np.ndarray:
    """N(0,1) x per-channel lognormal(0, 0.5), 8 outlier channels x10."""
    import torch

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    s = torch.exp(0.5 * torch.randn(d, generator=g))
    idx = torch.randperm(d, generator=g)[:8]
    s[idx] *= 10.0
    return (x * s).to(torch.bfloat16).float().numpy()


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def signal_gain(t: float) -> float:
    # mla_quant/train.py:21-29, evaluated for a scalar threshold
    centers = [-1.5095585584640503 + i * (3.0191171169281006) / 3 for i in range(4)]
    phi0 = 1 / math.sqrt(2 * math.pi)
    phi_t = math.exp(-t * t / 2) * phi0
    inner, outer = abs(centers[1]), abs(centers[3])
    return 1 / (2 * (inner * (phi0 - phi_t) + outer * phi_t))


def make_fake_checkpoint(root: Path) -> Path:
    """A local checkpoint directory with fixed bytes: config.json, a safetensors index
    naming two shards, and the shards (sizes are all that the fingerprint reads).  The
    tests rebuild the same directory with this function."""
    root.mkdir(parents=True, exist_ok=True)
    config = {"model_type": "minicpm3", "num_hidden_layers": 2, "kv_lora_rank": 256, "qk_rope_head_dim": 32,
              "hidden_size": 2560}
    (root / "config.json").write_text(json.dumps(config, indent=2, sort_keys=True) + "\n")
    index = {"metadata": {"total_size": 3000},
             "weight_map": {"a.weight": "model-00001-of-00002.safetensors",
                            "b.weight": "model-00002-of-00002.safetensors",
                            "c.weight": "model-00001-of-00002.safetensors"}}
    (root / "model.safetensors.index.json").write_text(json.dumps(index, indent=2, sort_keys=True) + "\n")
    (root / "model-00001-of-00002.safetensors").write_bytes(bytes(range(256)) * 7)
    (root / "model-00002-of-00002.safetensors").write_bytes(b"\x5a" * 1208)
    return root


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of noforit/mla_kv_quant")
    ap.add_argument("--only", choices=["uniform", "fingerprint"], default=None, help="write only this fixture")
    args = ap.parse_args()
    ref = Path(args.reference).resolve()
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "deployment" / "sglang" / "srt" / "mem_cache"))
    import torch
    from mla_quant.numerics import configure_reference_numerics
    from mla_quant.oscar import oscar_lloyd_int2_qdq
    from mla_quant.quantizer import (
        LearnedRotationQuantizer,
        NUMERICS,
        RECIPE,
        FORMAT_VERSION,
        quantize_learned,
        rotate_quantize,
    )
    import rolaq_mla

    configure_reference_numerics()
    torch.manual_seed(0)

    # ---- checkpoint fingerprint of a fake local checkpoint (mla_quant/artifacts.py:43-58) ----
    if args.only in (None, "fingerprint"):
        import tempfile

        from mla_quant.artifacts import local_checkpoint_fingerprint

        with tempfile.TemporaryDirectory() as tmp:
            ckpt = make_fake_checkpoint(Path(tmp) / "fake-minicpm3")
            fp = local_checkpoint_fingerprint(ckpt)
        (HERE / "fingerprint.json").write_text(json.dumps(fp, indent=2, sort_keys=True) + "\n")
        if args.only == "fingerprint":
            print("wrote fingerprint.json to", HERE)
            return

    # ---- uniform min/max baseline codec (mla_quant/oscar.py:91-101) ----------------------
    from mla_quant.oscar import uniform_int2_qdq

    xu = latents(24, 512, seed=3)
    ties = np.tile(np.float32([0.0, 0.5, 1.5, 2.5, 3.0, 1.0, 2.0, 0.25]), (1, 64))  # scale 1: exact .5 ties
    neg = ties - np.float32(7.0)
    xu = np.concatenate(
        [xu, ties, neg, np.full((1, 512), -2.5, np.float32), (np.arange(512, dtype=np.float32)[None, :] * 0.003)], 0
    ).astype(np.float32)
    np.savez_compressed(HERE / "uniform.npz", x=xu, deq=uniform_int2_qdq(torch.from_numpy(xu), 128).numpy())
    if args.only == "uniform":
        print("wrote uniform.npz to", HERE)
        return

    # ---- codec --------------------------------------------------------------------
    x = latents(40, 512, seed=0)
    x = np.concatenate(
        [
            x,
            np.full((1, 512), 0.75, np.float32),  # constant groups: std = sqrt(1e-8)
            np.tile(np.float32([1.0, -1.0]), (1, 256)),  # exact +-1 groups
            (np.arange(512, dtype=np.float32)[None, :] - 200.0) * np.float32(0.01),  # ramp
        ],
        0,
    ).astype(np.float32)
    xt = torch.from_numpy(x)
    pairs = [
        (0.9810652732849121, 1.16),
        (0.85, signal_gain(0.85)),
        (0.7, signal_gain(0.7)),
        (1.0, signal_gain(1.0)),
        (0.5, 0.8),
        (1.5, 1.3),
    ]
    direct = np.stack([oscar_lloyd_int2_qdq(xt, 128, t, g).numpy() for t, g in pairs])
    # HF path: FP32 tensors read back as Python floats, FP32(1.16) swapped for 1.16
    hf = np.stack(
        [
            quantize_learned(
                xt, 128, "oscar_lloyd", torch.tensor(t, dtype=torch.float32), torch.tensor(g, dtype=torch.float32)
            ).numpy()
            for t, g in pairs
        ]
    )
    np.savez_compressed(
        HERE / "codec.npz", x=x, pairs=np.array(pairs, np.float64), direct=direct, hf=hf
    )

    # ---- rotate_quantize ----------------------------------------------------------
    rot = {}
    for d, n, seed in ((512, 64, 11), (256, 48, 12)):
        r = orthogonal(d, seed)
        lat = torch.from_numpy(latents(n, d, seed=seed + 100)).to(torch.bfloat16).reshape(1, n, d)
        t = 0.83
        g = signal_gain(t)
        mask = torch.zeros(n, dtype=torch.bool)
        mask[:4] = True
        mask[-16:] = True
        out_masked = rotate_quantize(
            lat, torch.from_numpy(r), 128, "oscar_lloyd",
            torch.tensor(t, dtype=torch.float32), torch.tensor(g, dtype=torch.float32),
            high_precision_mask=mask,
        )
        out_plain = rotate_quantize(
            lat, torch.from_numpy(r), 128, "oscar_lloyd",
            torch.tensor(t, dtype=torch.float32), torch.tensor(g, dtype=torch.float32),
        )
        rot[f"r{d}"] = r
        rot[f"lat{d}"] = bf16_bits(lat)
        rot[f"mask{d}"] = mask.numpy()
        rot[f"out_masked{d}"] = bf16_bits(out_masked)
        rot[f"out_plain{d}"] = bf16_bits(out_plain)
        rot[f"tg{d}"] = np.array([t, g], np.float64)
    np.savez_compressed(HERE / "rotate.npz", **rot)

    # ---- v2 artifact, HF quantizer and serving loader --------------------------------
    art = HERE / "artifact_d256"
    art.mkdir(exist_ok=True)
    layers = {}
    params = [(0.8, signal_gain(0.8)), (0.9810652732849121, 1.16)]
    for i, (t, g) in enumerate(params):
        r = torch.from_numpy(orthogonal(256, 40 + i)).contiguous()
        path = art / f"layer_{i}.pt"
        torch.save(r, path)
        layers[str(i)] = {
            "file": path.name,
            "sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
            "param0": float(t),
            "param1": float(g),
        }
    manifest = {
        "format_version": FORMAT_VERSION,
        "recipe": RECIPE,
        "numerics": NUMERICS,
        "family": "oscar_lloyd",
        "train_part": "joint",
        "mla_output_weight": 0.0,
        "group_size": 128,
        "components": ["nope"],
        "windows": False,
        "model": {
            "model_type": "minicpm3",
            "num_hidden_layers": 2,
            "kv_lora_rank": 256,
            "qk_rope_head_dim": 32,
        },
        "layers": layers,
        "calibration": {"note": "synthetic golden artifact"},
    }
    (art / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")

    q = LearnedRotationQuantizer(art)
    lat = torch.from_numpy(latents(40, 256, seed=7)).to(torch.bfloat16).reshape(1, 40, 256)
    outs = {
        "lat": bf16_bits(lat),
        "q0": bf16_bits(q.quantize_layer(lat, 0, "nope")),
        "q1": bf16_bits(q.quantize_layer(lat, 1, "nope")),
        "q1_decode": bf16_bits(q.quantize_layer(lat[:, -1:], 1, "nope")),
    }
    mask = torch.zeros(40, dtype=torch.bool)
    mask[:4] = True
    mask[-16:] = True
    q.high_precision_mask = mask
    outs["q0_masked"] = bf16_bits(q.quantize_layer(lat, 0, "nope"))
    meta = q.metadata()
    meta.pop("rotation_dir")
    loader = rolaq_mla.load_layer_quantizers(str(art), str(art), 128, 256, [0, 1])
    w = torch.from_numpy(latents(2 * (128 + 128), 256, seed=9)).to(torch.bfloat16)
    outs["w"] = bf16_bits(w)
    outs["w_folded1"] = bf16_bits(rolaq_mla.fold_read_rotation(w, 1, str(art)))
    np.savez_compressed(HERE / "artifact.npz", **outs)
    (HERE / "artifact.json").write_text(
        json.dumps(
            {
                "metadata": meta,
                "layer_calls": q.layer_calls,
                "call_count": q.call_count,
                "element_count": q.element_count,
                "first_shapes": [list(s) for s in q.first_shapes],
                "load_layer_quantizers": loader,
            },
            indent=2,
        )
        + "\n"
    )
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
