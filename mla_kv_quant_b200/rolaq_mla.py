"""Frozen RoLaQ parameters for the packed cache (drop-in for
``deployment/sglang/srt/mem_cache/rolaq_mla.py``).

The cache format is INT2 codes plus FP32 (scale, zero) per 128-group; only the
writer's threshold and gain come from the learned artifact.
"""

import hashlib
import json
import math
from functools import lru_cache
from pathlib import Path

import torch

from . import ops


@lru_cache(maxsize=8)
def load_manifest(path):
    """Validate a v2 learned artifact (``rolaq_mla.py:16-38``)."""
    root = Path(path).resolve()
    manifest = json.loads((root / "manifest.json").read_text())
    if manifest.get("recipe") != "learned_shared_latent_rotation_quantizer_v2":
        raise ValueError("RoLaQ requires a frozen v2 learned artifact")
    if manifest.get("family") != "oscar_lloyd":
        raise ValueError("The packed RoLaQ writer currently supports oscar_lloyd only")
    if manifest.get("components") != ["nope"] or manifest.get("group_size") != 128:
        raise ValueError("Expected content-only, group-128 RoLaQ artifact")
    count = manifest["model"]["num_hidden_layers"]
    if set(manifest["layers"]) != {str(i) for i in range(count)}:
        raise ValueError("RoLaQ artifact must cover every decoder layer")
    for layer, item in manifest["layers"].items():
        if item["file"] != f"layer_{int(layer)}.pt":
            raise ValueError("Unexpected rotation filename")
        data = (root / item["file"]).read_bytes()
        if hashlib.sha256(data).hexdigest() != item["sha256"]:
            raise ValueError(f"RoLaQ rotation hash mismatch: layer {layer}")
        t, gain = item["param0"], item["param1"]
        if not (math.isfinite(t) and math.isfinite(gain) and t > 0 and gain > 0):
            raise ValueError(f"Invalid quantizer parameters at layer {layer}")
    return manifest


def load_layer_quantizers(path, rotation_path, group_size, width, layer_ids):
    """Per-layer ``(threshold, gain)`` or ``None`` entries (``rolaq_mla.py:41-53``)."""
    if not path:
        return [None for _ in layer_ids]
    if Path(path).resolve() != Path(rotation_path).resolve():
        raise ValueError("Learned quantizer and rotations must come from the same artifact")
    manifest = load_manifest(path)
    if manifest["group_size"] != group_size or manifest["model"]["kv_lora_rank"] != width:
        raise ValueError("RoLaQ artifact does not match the cache dimensions")
    result = []
    for layer in layer_ids:
        item = manifest["layers"][str(layer)]
        result.append((float(item["param0"]), float(item["param1"])))
    return result


def fold_read_rotation(weight, layer_id, rotation_path):
    """Return ``W_b @ R`` for absorbed readers (``rolaq_mla.py:56-71``).

    ``W_b`` is ``[heads * (key_dim + value_dim), latent_dim]`` BF16; the product runs
    on the tcgen05 rotation kernel (BF16 operands, FP32 accumulation, BF16 result),
    the same arithmetic as ``(weight.float() @ R.bf16().float()).bf16()``.  CPU
    weights are folded on the current CUDA device and returned on the CPU.
    """
    if weight.dtype != torch.bfloat16:
        raise ValueError("Read-rotation absorption is validated for BF16 weights only")
    path = Path(rotation_path) / f"layer_{layer_id}.pt"
    rotation = torch.load(path, map_location="cpu", weights_only=True)
    if rotation.shape != (weight.shape[-1], weight.shape[-1]):
        raise ValueError("Read-rotation shape mismatch")
    if not torch.cuda.is_available():
        raise RuntimeError("fold_read_rotation runs on the sm_100a rotation kernel and needs a CUDA device")
    dev = weight.device if weight.is_cuda else torch.device("cuda", torch.cuda.current_device())
    w = weight.to(dev).contiguous()
    rt = rotation.to(device=dev, dtype=torch.bfloat16).t().contiguous()  # out[o] = sum_k w[k] * R[k][o]
    out = torch.empty_like(w)
    ops.rotate_rows(w, rt, out_bf16=out)
    return out if weight.is_cuda else out.cpu()
