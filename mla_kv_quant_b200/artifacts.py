"""Read side of the RoLaQ v2 learned artifact, plus a writer for synthetic artifacts.

Format (``mla_quant/quantizer.py:155-215``): ``manifest.json`` with
``format_version = 2``, ``recipe``, ``numerics``, ``family = "oscar_lloyd"``,
``group_size = 128``, ``components = ["nope"]``, ``windows = false``, ``model``
{model_type, num_hidden_layers, kv_lora_rank, qk_rope_head_dim, ...} and
``layers`` {i: {file, sha256, param0 (threshold), param1 (gain)}}; one
``layer_{i}.pt`` FP32 ``[D, D]`` rotation per layer.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from pathlib import Path
from typing import Any

import torch

FORMAT_VERSION = 2
RECIPE = "learned_shared_latent_rotation_quantizer_v2"
NUMERICS = "fp32_rotation_bf16_roundtrip_fp32_qdq_input_dtype_roundtrip_fp32_inverse_input_dtype"
CONFIG_FIELDS = ("model_type", "num_hidden_layers", "kv_lora_rank", "qk_rope_head_dim")


def sha256_file(path: str | Path) -> str:
    digest = hashlib.sha256()
    with Path(path).open("rb") as handle:
        for chunk in iter(lambda: handle.read(1024 * 1024), b""):
            digest.update(chunk)
    return digest.hexdigest()


def atomic_write_json(path: str | Path, value) -> None:
    """Atomically replace a JSON file (``mla_quant/artifacts.py:19-33``)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, temporary = tempfile.mkstemp(prefix=f".{path.name}.", dir=path.parent)
    try:
        with os.fdopen(fd, "w") as handle:
            json.dump(value, handle, ensure_ascii=False, indent=2, allow_nan=False)
            handle.write("\n")
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(temporary, path)
    finally:
        if os.path.exists(temporary):
            os.unlink(temporary)


def checkpoint_identity(model_path: str | Path) -> dict[str, Any]:
    """Config/index hashes of a local checkpoint (``mla_quant/oscar.py:26-43``)."""
    root = Path(model_path).expanduser().resolve()
    config_path = root / "config.json"
    if not config_path.is_file():
        raise ValueError(f"OSCAR requires a local model directory with config.json: {root}")
    config = json.loads(config_path.read_text())
    index = root / "model.safetensors.index.json"
    return {
        "checkpoint_name": root.name,
        "config_sha256": sha256_file(config_path),
        "weight_index_sha256": sha256_file(index) if index.exists() else None,
        **{key: config.get(key) for key in CONFIG_FIELDS},
    }


def local_checkpoint_fingerprint(model_path: str | Path) -> dict:
    """Identity plus shard sizes (``mla_quant/artifacts.py:43-58``)."""
    root = Path(model_path).expanduser().resolve()
    identity = checkpoint_identity(root)
    index = root / "model.safetensors.index.json"
    if index.is_file():
        names = sorted(set(json.loads(index.read_text())["weight_map"].values()))
    else:
        names = [p.name for p in sorted(root.glob("*.safetensors"))]
        if not names:
            names = [p.name for p in sorted(root.glob("pytorch_model*.bin"))]
    identity["weight_files"] = {name: {"size": (root / name).stat().st_size} for name in names}
    identity["weight_identity_policy"] = "config_index_sha256_and_shard_size"
    return identity


def write_synthetic_artifact(output_dir: str | Path, rotations: dict[int, torch.Tensor],
                             params: dict[int, tuple[float, float]], model: dict[str, Any],
                             calibration: dict[str, Any] | None = None) -> dict[str, Any]:
    """Write a v2 artifact for seeded synthetic rotations (benchmarks and tests).

    Same files and manifest fields the reference loader reads; the checkpoint
    fingerprint fields are whatever ``model`` holds (no checkpoint is needed).
    """
    root = Path(output_dir)
    root.mkdir(parents=True, exist_ok=True)
    layers = {}
    for layer in sorted(rotations):
        r = rotations[layer].detach().cpu().float().contiguous()
        path = root / f"layer_{layer}.pt"
        torch.save(r, path)
        t, g = params[layer]
        layers[str(layer)] = {"file": path.name, "sha256": sha256_file(path), "param0": float(t),
                              "param1": float(g)}
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
        "model": dict(model),
        "layers": layers,
        "calibration": calibration or {"source": "synthetic"},
    }
    atomic_write_json(root / "manifest.json", manifest)
    return manifest
