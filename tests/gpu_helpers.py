"""Shared set-up for the -m gpu parity tests: seeded pools written by the CUDA
writer, and their mirror in the oracle's numpy pool."""

from __future__ import annotations

import numpy as np
import torch

from mla_kv_quant_b200 import ops, synth
from oracle import codec as ocodec
from oracle import writer as owriter


def bits(t: torch.Tensor) -> np.ndarray:
    """BF16 tensor -> uint16 bit patterns (numpy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32_of_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy()


class GpuPool:
    """One layer's cache on the GPU plus the shared maps."""

    def __init__(self, num_slots, d, dr, max_reqs, sink=4, recent=16, device="cuda"):
        self.d, self.dr, self.sink, self.recent, self.max_reqs = d, dr, sink, recent, max_reqs
        ring = 1 + max_reqs * (sink + recent)
        self.codes = torch.zeros(num_slots, d // 4, dtype=torch.uint8, device=device)
        self.params = torch.zeros(num_slots, d // 128, 2, dtype=torch.float32, device=device)
        self.rope = torch.zeros(num_slots, dr, dtype=torch.bfloat16, device=device)
        self.hp = torch.zeros(ring, d, dtype=torch.bfloat16, device=device)
        self.rows = torch.full((num_slots,), -1, dtype=torch.int32, device=device)
        self.owners = torch.zeros(ring, dtype=torch.int32, device=device)

    def view(self):
        return ops.LayerView(self.codes, self.params, self.rope, self.hp, self.rows, self.owners, self.sink,
                             self.recent, self.max_reqs)

    def to_oracle(self) -> owriter.Pool:
        p = owriter.Pool(self.codes.shape[0], self.d, self.dr, self.max_reqs, self.sink, self.recent)
        p.codes = self.codes.cpu().numpy()
        p.params = self.params.cpu().numpy()
        p.rope = bits(self.rope)
        p.hp = bits(self.hp)
        p.rows = self.rows.cpu().numpy()
        p.owners = self.owners.cpu().numpy()
        return p


def fill_requests(pool: GpuPool, seq_lens, page_table: torch.Tensor, rotation: torch.Tensor, codec, seed=0,
                  positions_mode=True, row_gain=None):
    """Prefill every request with seeded latents through the fused writer.

    ``row_gain(L) -> [L]`` (optional) multiplies each token's latent and rope rows, e.g.
    to make group scales and scores drift along the sequence.
    Returns the BF16 inputs (c_kv, k_pe) per request for oracle checks.
    """
    dev = pool.codes.device
    rt = rotation.to(device=dev, dtype=torch.bfloat16).t().contiguous()
    inputs = []
    scale = synth.channel_scale(pool.d, 1234, dev)
    for b, L in enumerate(seq_lens):
        if L == 0:
            inputs.append(None)
            continue
        c_kv = synth.latents(L, pool.d, seed + 17 * b, dev, scale=scale)
        k_pe = synth.normal_bf16((L, pool.dr), seed + 31 * b + 5, dev)
        if row_gain is not None:
            gain = row_gain(L).to(dev).float()[:, None]
            c_kv = (c_kv.float() * gain).to(torch.bfloat16)
            k_pe = (k_pe.float() * gain).to(torch.bfloat16)
        pos = torch.arange(L, device=dev)
        slots = (page_table[b, pos // 64].long() * 64 + pos % 64).contiguous()
        seq = torch.full((L,), L, dtype=torch.int32, device=dev)
        req = torch.full((L,), b, dtype=torch.int64, device=dev)
        ops.fused_write(c_kv, k_pe, slots, rt, codec, pool.view(), seq_lens=seq, req_idx=req,
                        positions=pos.to(torch.int32) if positions_mode else None)
        inputs.append((c_kv, k_pe, slots))
    torch.cuda.synchronize()
    return inputs


def oracle_scalars(codec):
    return np.float32(codec.threshold), np.float32(codec.scale_factor), np.float32(codec.zero_const)


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def rotate_cpu(x_bf16: torch.Tensor, rotation: torch.Tensor) -> np.ndarray:
    """The reference FP32 GEMM on the CPU (oracle.codec.rotate_reference)."""
    return ocodec.rotate_reference(f32_of_bf16(x_bf16), rotation.cpu().numpy())
