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
from pathlib import Path
from typing import Any

import torch

FORMAT_VERSION = 2
RECIPE = "learned_shared_latent_rotation_quantizer_v2"
NUMERICS = "fp32_rotation_bf16_roundtrip_fp32_qdq_input_dtype_roundtrip_fp32_inverse_input_dtype"
CONFIG_FIELDS = ("model_type", "num_hidden_layers", "kv_lora_rank", "qk_rope_head_dim")


def sha256_file(path: str | Path) -> str:
    """Hex SHA-256 of a file's bytes (the manifest's per-layer ``sha256``)."""
    with open(path, "rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def _write_json_replacing(path: Path, value) -> None:
    """Write ``value`` as indented JSON next to ``path``, then rename it over ``path``
    (readers never see a half-written manifest)."""
    path.parent.mkdir(parents=True, exist_ok=True)
    staged = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    staged.write_text(json.dumps(value, ensure_ascii=False, indent=2, allow_nan=False) + "\n")
    os.replace(staged, path)


def _shard_sizes(root: Path) -> dict[str, dict[str, int]]:
    """{shard file: {"size": bytes}} of a local checkpoint: the shards a safetensors index
    names, else every ``*.safetensors`` file, else every ``pytorch_model*.bin`` file."""
    index = root / "model.safetensors.index.json"
    if index.is_file():
        shards = set(json.loads(index.read_text())["weight_map"].values())
    else:
        shards = {p.name for p in root.glob("*.safetensors")} or {p.name for p in root.glob("pytorch_model*.bin")}
    return {name: {"size": (root / name).stat().st_size} for name in sorted(shards)}


def checkpoint_fingerprint(model_path: str | Path) -> dict[str, Any]:
    """The checkpoint identity a v2 manifest records under ``model`` and that
    ``LearnedRotationQuantizer.validate_config`` compares (``mla_quant/quantizer.py:
    266-289``): hashes of ``config.json`` and of the safetensors index (None without
    one), the shard sizes, and the config fields ``CONFIG_FIELDS``."""
    root = Path(model_path).expanduser().resolve()
    config_file = root / "config.json"
    if not config_file.is_file():
        raise ValueError(f"OSCAR requires a local model directory with config.json: {root}")
    index = root / "model.safetensors.index.json"
    config = json.loads(config_file.read_text())
    fingerprint: dict[str, Any] = {field: config.get(field) for field in CONFIG_FIELDS}
    fingerprint.update(
        checkpoint_name=root.name,
        config_sha256=sha256_file(config_file),
        weight_index_sha256=sha256_file(index) if index.exists() else None,
        weight_files=_shard_sizes(root),
        weight_identity_policy="config_index_sha256_and_shard_size",
    )
    return fingerprint


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
    _write_json_replacing(root / "manifest.json", manifest)
    return manifest
