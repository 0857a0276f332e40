"""Seeded synthetic inputs with the shapes and value distributions of the benchmark
configurations (no dataset or checkpoint is involved).

* latents: N(0, 1) per element x a per-channel lognormal(0, 0.5) scale, with 8 seeded
  outlier channels x10, rounded to BF16;
* rotations: Q of a seeded Gaussian QR (FP64), sign-fixed by diag(R), stored FP32;
* per-layer threshold t ~ U[0.7, 1.0] with gain g = signal_gain(t), the legal
  (t, g) pairs of the calibration (``mla_quant/train.py:21-29``);
* k_pe and queries: N(0, 1) in BF16;
* page tables: a seeded permutation of 64-token pages, page 0 never used.
"""

from __future__ import annotations

import math

import torch

OSCAR_LLOYD_CENTERS = tuple(-1.5095585584640503 + i * 3.0191171169281006 / 3 for i in range(4))


def signal_gain(t: float) -> float:
    """``1 / signal_response(t)`` (``mla_quant/train.py:21-29``) for a scalar t."""
    phi0 = 1 / math.sqrt(2 * math.pi)
    phi_t = math.exp(-t * t / 2) * phi0
    inner, outer = abs(OSCAR_LLOYD_CENTERS[1]), abs(OSCAR_LLOYD_CENTERS[3])
    return 1 / (2 * (inner * (phi0 - phi_t) + outer * phi_t))


def rotation(d: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(d, d, generator=g, dtype=torch.float64)
    q, r = torch.linalg.qr(a)
    return (q * torch.sign(torch.diagonal(r))[None, :]).float().contiguous()


def layer_params(layers: int, seed: int = 2) -> list[tuple[float, float]]:
    g = torch.Generator().manual_seed(seed)
    ts = (0.7 + 0.3 * torch.rand(layers, generator=g, dtype=torch.float64)).tolist()
    return [(t, signal_gain(t)) for t in ts]


def channel_scale(d: int, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    s = torch.exp(0.5 * torch.randn(d, generator=g))
    s[torch.randperm(d, generator=g)[:8]] *= 10.0
    return s.to(device)


def latents(n: int, d: int, seed: int, device="cpu", scale: torch.Tensor | None = None) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    s = channel_scale(d, seed + 7919, device) if scale is None else scale
    return (torch.randn(n, d, generator=g, device=device) * s).to(torch.bfloat16)


def normal_bf16(shape, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=device).to(torch.bfloat16)


def page_table(batch: int, ctx: int, seed: int = 4, spare_pages: int = 0, device="cpu"):
    """Random page assignment; returns (page_table int32 [B, pages], num_slots)."""
    pages = (ctx + 63) // 64
    total = batch * pages + spare_pages
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(total, generator=g) + 1  # page 0 is never used
    return perm[: batch * pages].reshape(batch, pages).to(torch.int32).to(device), (total + 1) * 64
