"""Drop-in for the HF quantize-dequantize API of ``mla_quant/quantizer.py``.

Same names, arguments, validation and error messages as the reference inference
path (``quantizer.py:73-124, 136-152, 218-331``); the arithmetic runs in the sm_100a
kernels of librolaq_b200.so:

    rotate (tcgen05, BF16 x BF16 -> FP32)  ->  Lloyd INT2 codec  ->  dequant to the
    input dtype  ->  un-rotate (tcgen05)  ->  input dtype

Only CUDA tensors on an sm_100 device are accepted, and only BF16 latents (the dtype
MLA models cache): the kernels stage BF16 operands for the tensor cores.  The
training path of the reference (``_LloydSTE``, gradients through the quantizer) is
calibration-time code and is not provided.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Any

import torch

from . import ops
from .artifacts import FORMAT_VERSION, NUMERICS, RECIPE, sha256_file

LLOYD_BOUNDS = ((0.5, 1.5), (0.8, 1.3))
QUANT_FAMILIES = ("oscar_lloyd",)


def _validate_parameters(family, first, second):
    """``quantizer.py:136-142``."""
    if family not in QUANT_FAMILIES:
        raise ValueError(f"unknown quant family {family!r}")
    for value, (lo, hi) in zip((first, second), LLOYD_BOUNDS):
        if not math.isfinite(value) or not lo - 1e-06 <= value <= hi + 1e-06:
            raise ValueError("quantizer parameter non-finite or out of bounds")


def _validate_rotation(rotation, width, layer):
    """``quantizer.py:145-152``."""
    if rotation.dtype != torch.float32 or rotation.shape != (width, width):
        raise ValueError(f"layer {layer} requires a square FP32 rotation")
    if not torch.isfinite(rotation).all():
        raise ValueError(f"layer {layer} rotation contains non-finite values")
    residual = (rotation.double().T @ rotation.double() - torch.eye(width, dtype=torch.float64)).abs().max().item()
    if residual > 1e-05:
        raise ValueError(f"layer {layer} rotation not orthogonal, residual={residual}")


def _normalize_high_precision_mask(mask: torch.Tensor, latent: torch.Tensor) -> torch.Tensor:
    """Accept [seq], [batch, seq] or exactly latent.shape[:-1] (``quantizer.py:85-99``)."""
    mask = mask.to(device=latent.device, dtype=torch.bool)
    expected = tuple(latent.shape[:-1])
    if mask.ndim == 1 and len(expected) > 1:
        mask = mask.reshape(*[1] * (len(expected) - 1), mask.shape[0])
    elif mask.ndim == 2 and len(expected) == 3:
        mask = mask.unsqueeze(1)
    try:
        mask = torch.broadcast_to(mask, expected)
    except RuntimeError as error:
        raise ValueError(f"high precision mask shape {tuple(mask.shape)} does not match {expected}") from error
    return mask


def _scalar(v) -> float:
    return float(v.detach()) if isinstance(v, torch.Tensor) else float(v)


class _Rotation:
    """Device copies of one effective rotation: R_eff (BF16, [k][o]) and its transpose."""

    def __init__(self, rotation: torch.Tensor, device: torch.device):
        eff = rotation.to(device=device, dtype=torch.bfloat16)
        self.r = eff.contiguous()  # un-rotation weight: out[o] = sum_k x[k] * R[o][k]
        self.rt = eff.t().contiguous()  # rotation weight: out[o] = sum_k x[k] * R[k][o]


def _qdq_rotated(latent2d: torch.Tensor, rot: _Rotation, codec) -> torch.Tensor:
    """rotate -> codec -> dequant (BF16) -> un-rotate (BF16), rows of ``latent2d``."""
    n, d = latent2d.shape
    dev = latent2d.device
    codes = torch.empty(n, d // 4, dtype=torch.uint8, device=dev)
    params = torch.empty(n, d // 128, 2, dtype=torch.float32, device=dev)
    ops.encode_rows(latent2d, rot.rt, codec, codes, params)
    deq = torch.empty(n, d, dtype=torch.bfloat16, device=dev)
    ops.dequant_rows(codes, params, out_bf16=deq)
    out = torch.empty(n, d, dtype=torch.bfloat16, device=dev)
    ops.rotate_rows(deq, rot.r, out_bf16=out)
    return out


def quantize_learned(values, group_size, family, first, second, temperature=None):
    """Hard Lloyd INT2 QDQ of already-rotated FP32 values (``quantizer.py:73-82``)."""
    if family != "oscar_lloyd":
        raise ValueError("only the official OSCAR affine-grid family is supported")
    if torch.is_grad_enabled() and (
        getattr(first, "requires_grad", False) or getattr(second, "requires_grad", False) or values.requires_grad
    ):
        raise ValueError("the straight-through training path is calibration-time code and is not provided")
    if int(group_size) != 128:
        raise ValueError("group_size must be 128")
    codec = ops.codec_hf(_scalar(first), _scalar(second))
    shape = values.shape
    x = values.reshape(-1, shape[-1]).float().contiguous()
    n, d = x.shape
    codes = torch.empty(n, d // 4, dtype=torch.uint8, device=x.device)
    params = torch.empty(n, d // 128, 2, dtype=torch.float32, device=x.device)
    ops.scatter_pack_rows(x, torch.arange(n, dtype=torch.int64, device=x.device), codes, params, codec)
    out = torch.empty(n, d, dtype=torch.float32, device=x.device)
    ops.dequant_rows(codes, params, out_f32=out)
    return out.reshape(shape)


def rotate_quantize(
    latent: torch.Tensor,
    rotation: torch.Tensor,
    group_size: int,
    family: str,
    first: torch.Tensor,
    second: torch.Tensor,
    temperature: torch.Tensor | None = None,
    high_precision_mask: torch.Tensor | None = None,
) -> torch.Tensor:
    """OSCAR cast order, with optional rows returned unquantized (``quantizer.py:102-124``)."""
    if high_precision_mask is not None:
        high_precision_mask = _normalize_high_precision_mask(high_precision_mask, latent)
        if bool(high_precision_mask.all()):
            return latent
    if family != "oscar_lloyd":
        raise ValueError("only the official OSCAR affine-grid family is supported")
    if int(group_size) != 128:
        raise ValueError("group_size must be 128")
    if latent.dtype != torch.bfloat16:
        raise ValueError("the tcgen05 quantizer path takes BF16 latents")
    rot = rotation if isinstance(rotation, _Rotation) else _Rotation(rotation, latent.device)
    codec = ops.codec_hf(_scalar(first), _scalar(second))
    d = latent.shape[-1]
    restored = _qdq_rotated(latent.reshape(-1, d).contiguous(), rot, codec).reshape(latent.shape)
    if high_precision_mask is None:
        return restored
    return torch.where(high_precision_mask.unsqueeze(-1), latent, restored)


class LearnedRotationQuantizer:
    """Inference quantizer over a v2 artifact (``quantizer.py:218-331``)."""

    def __init__(self, artifact_dir: str | Path):
        self.root = Path(artifact_dir).expanduser().resolve()
        path = self.root / "manifest.json"
        self.manifest = json.loads(path.read_text())
        self.manifest_sha256 = sha256_file(path)
        if (self.manifest.get("format_version"), self.manifest.get("recipe")) != (FORMAT_VERSION, RECIPE):
            raise ValueError("not a learned rotation artifact")
        if self.manifest.get("numerics") != NUMERICS:
            raise ValueError("learned artifact numerical recipe mismatch")
        if self.manifest.get("group_size") != 128 or self.manifest.get("components") != ["nope"]:
            raise ValueError("learned artifact must be nope-only group 128")
        self.family = self.manifest["family"]
        self.width = int(self.manifest["model"]["kv_lora_rank"])
        self.group_size = 128
        if self.width <= 0 or self.width % self.group_size:
            raise ValueError("latent width is incompatible with group size")
        count = int(self.manifest["model"]["num_hidden_layers"])
        if set(self.manifest["layers"]) != {str(i) for i in range(count)}:
            raise ValueError("learned artifact has missing or unexpected layers")
        if self.manifest.get("windows") is not False:
            raise ValueError("window lifecycle is not supported by this artifact")
        self.rotations = {}
        self.params = {}
        for layer, record in self.manifest["layers"].items():
            if record["file"] != f"layer_{int(layer)}.pt":
                raise ValueError("unexpected learned rotation filename")
            file = self.root / record["file"]
            if sha256_file(file) != record["sha256"]:
                raise ValueError(f"learned rotation hash mismatch at layer {layer}")
            rotation = torch.load(file, map_location="cpu", weights_only=True)
            _validate_rotation(rotation, self.width, layer)
            _validate_parameters(self.family, record["param0"], record["param1"])
            self.rotations[int(layer)] = rotation
            self.params[int(layer)] = (float(record["param0"]), float(record["param1"]))
        self._cache: dict[tuple[int, str, torch.dtype], _Rotation] = {}
        self.high_precision_mask: torch.Tensor | None = None
        self.layer_calls = {str(i): {"prefill": 0, "decode": 0} for i in self.rotations}
        self.call_count = 0
        self.element_count = 0
        self.first_shapes: list[tuple[int, ...]] = []
        self._validated_configs: list[Any] = []

    def validate_config(self, config: Any) -> None:
        """``quantizer.py:266-289``."""
        from .artifacts import checkpoint_fingerprint
        from .numerics import validate_artifact_numerics

        validate_artifact_numerics(self.manifest)
        if any(config is previous for previous in self._validated_configs):
            return
        expected = self.manifest["model"]
        for key in ("model_type", "num_hidden_layers", "kv_lora_rank", "qk_rope_head_dim"):
            if getattr(config, key, None) != expected[key]:
                raise ValueError(f"learned artifact model mismatch: {key}")
        model_path = getattr(config, "_name_or_path", "")
        if not model_path:
            raise ValueError("learned artifact validation needs the model checkpoint path")
        actual = checkpoint_fingerprint(model_path)
        identity_fields = ["config_sha256", "weight_index_sha256"]
        if "weight_files" in expected:
            sizes = lambda record: {name: value["size"] for name, value in record.items()}  # noqa: E731
            if sizes(actual["weight_files"]) != sizes(expected["weight_files"]):
                raise ValueError("learned artifact shard names/sizes differ from the checkpoint")
        if any(actual.get(key) != expected.get(key) for key in identity_fields):
            raise ValueError("learned artifact belongs to a different checkpoint")
        self._validated_configs.append(config)

    def quantize_layer(self, tensor: torch.Tensor, layer_idx: int, component: str) -> torch.Tensor:
        """``quantizer.py:291-315``."""
        if component != "nope":
            raise ValueError("learned rotation quantizes nope only")
        if tensor.ndim < 2 or tensor.shape[-1] != self.width or (not tensor.is_floating_point()):
            raise ValueError("invalid MLA latent shape or dtype")
        if layer_idx not in self.rotations:
            raise ValueError(f"missing learned rotation for layer {layer_idx}")
        key = (layer_idx, str(tensor.device), tensor.dtype)
        if key not in self._cache:
            if tensor.dtype != torch.bfloat16:
                raise ValueError("the tcgen05 quantizer path takes BF16 latents")
            self._cache[key] = _Rotation(self.rotations[layer_idx], tensor.device)
        phase = "decode" if tensor.shape[-2] == 1 else "prefill"
        self.layer_calls[str(layer_idx)][phase] += 1
        self.call_count += 1
        self.element_count += tensor.numel()
        if len(self.first_shapes) < 4:
            self.first_shapes.append(tuple(tensor.shape))
        first, second = self.params[layer_idx]
        mask = self.high_precision_mask
        if mask is not None and mask.shape[-1] != tensor.shape[-2]:
            mask = mask[..., -tensor.shape[-2]:]
        return rotate_quantize(tensor, self._cache[key], self.group_size, self.family, first, second,
                               high_precision_mask=mask)

    def metadata(self) -> dict[str, Any]:
        """``quantizer.py:317-331``."""
        return {
            "recipe": self.manifest["recipe"],
            "family": self.family,
            "train_part": self.manifest.get("train_part"),
            "mla_output_weight": self.manifest.get("mla_output_weight"),
            "rotation_dir": str(self.root),
            "manifest_sha256": self.manifest_sha256,
            "rotation_hashes": {layer: record["sha256"] for layer, record in self.manifest["layers"].items()},
            "calibration": self.manifest.get("calibration", {}),
            "numerics": self.manifest.get("numerics"),
            "components": ["nope"],
        }
