"""Torch-tensor wrappers of the C ABI entry points (one function per entry point).

Every function validates shapes/dtypes/devices, passes raw pointers and the
current CUDA stream, and raises on a non-OK status.  Nothing here allocates unless
an output argument is omitted, in which case a fresh tensor is returned.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

# mla_quant/oscar.py:104-111 -- Lloyd-Max INT2 constants
LLOYD_MAX_THRESHOLDS = (-0.9810652732849121, 0.0, 0.9810652732849121)
LLOYD_MAX_CENTROIDS = (-1.5095585584640503, -0.4527800381183624, 0.4527800381183624, 1.5095585584640503)
LLOYD_MAX_STRETCH = 1.16
SPAN = LLOYD_MAX_CENTROIDS[3] - LLOYD_MAX_CENTROIDS[0]
GROUP_SIZE = 128
PAGE = 64


def _f32(x: float) -> float:
    return float(torch.tensor(x, dtype=torch.float32))


def codec_hf(threshold: float, gain: float) -> _lib.Codec:
    """Codec scalars as the HF quantize-dequantize path forms them.

    ``quantize_layer`` wraps the manifest values in FP32 tensors and
    ``oscar_lloyd_hard`` reads them back, swapping an FP32(1.16) gain for the double
    1.16 (mla_quant/quantizer.py:31-35, 307-309); the products with ``span / 3`` are
    Python doubles rounded to FP32 where they meet the FP32 tensors
    (mla_quant/oscar.py:141-143).
    """
    t = _f32(threshold)
    g32 = _f32(gain)
    g = LLOYD_MAX_STRETCH if g32 == _f32(LLOYD_MAX_STRETCH) else g32
    return _lib.Codec(t, _f32(SPAN / 3.0 * g), _f32(-LLOYD_MAX_CENTROIDS[0] / (SPAN / 3.0)))


def codec_serving(threshold: float, gain: float) -> _lib.Codec:
    """Codec scalars as the serving writer forms them: the manifest doubles go
    straight into the kernel constants (deployment/sglang/QuantKernel/
    mla_fused_writer.py:158-164, deployment/patches/rolaq_sglang.patch:22-33)."""
    return _lib.Codec(_f32(threshold), _f32(SPAN / 3.0 * float(gain)), _f32(-LLOYD_MAX_CENTROIDS[0] / (SPAN / 3.0)))


def codec_uniform() -> _lib.Codec:
    """OSCAR's uniform min/max INT2 codec (``mla_quant/oscar.py:91-101``), the writer's
    baseline when the pool runs without Lloyd-Max (``mla_fused_writer.py:194-224``)."""
    return _lib.Codec(0.0, 0.0, 0.0, _lib.CODEC_UNIFORM)


def _check(t: torch.Tensor, name: str, dtype=None, ndim=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    _lib.require_device(t)


def _index(t: torch.Tensor | None, name: str):
    if t is None:
        return None, 0
    if t.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"{name} must be int32 or int64")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    _lib.require_device(t)
    return t.data_ptr(), int(t.dtype == torch.int64)


def _err_ptr(err: torch.Tensor | None):
    if err is None:
        return None
    if err.dtype != torch.int32 or err.numel() < 1:
        raise TypeError("err must be an int32 tensor with at least one element")
    return err.data_ptr()


class LayerView:
    """The pool tensors of one layer, as the C ABI's ``rolaq_layer_cache``."""

    def __init__(self, codes, params, rope, hp=None, rows=None, owners=None, sink=0, recent=0, max_reqs=0):
        self.codes, self.params, self.rope = codes, params, rope
        self.hp, self.rows, self.owners = hp, rows, owners
        self.sink, self.recent, self.max_reqs = int(sink), int(recent), int(max_reqs)
        d = codes.shape[-1] * 4
        if codes.dtype != torch.uint8 or codes.dim() != 2:
            raise TypeError("codes must be uint8 [slots, D/4]")
        if params.dtype != torch.float32 or tuple(params.shape) != (codes.shape[0], d // GROUP_SIZE, 2):
            raise TypeError("params must be float32 [slots, D/128, 2]")
        if rope.dtype != torch.bfloat16 or rope.dim() != 2 or rope.shape[0] != codes.shape[0]:
            raise TypeError("rope must be bfloat16 [slots, Dr]")
        for t in (codes, params, rope, hp, rows, owners):
            if t is not None and not t.is_contiguous():
                raise ValueError("pool tensors must be contiguous")
        if hp is not None and (hp.dtype != torch.bfloat16 or hp.shape[-1] != d):
            raise TypeError("hp must be bfloat16 [ring_rows, D]")
        if rows is not None and (rows.dtype != torch.int32 or rows.shape[0] != codes.shape[0]):
            raise TypeError("rows must be int32 [slots]")
        if owners is not None and owners.dtype != torch.int32:
            raise TypeError("owners must be int32 [ring_rows]")
        self.latent_dim = d
        self.rope_dim = rope.shape[1]
        self.num_slots = codes.shape[0]
        self.num_ring_rows = 0 if hp is None else hp.shape[0]

    def c_struct(self) -> _lib.LayerCache:
        return _lib.LayerCache(
            _lib.ptr(self.codes), _lib.ptr(self.params), _lib.ptr(self.rope), _lib.ptr(self.hp),
            _lib.ptr(self.rows), _lib.ptr(self.owners), self.num_slots, self.num_ring_rows, self.latent_dim,
            self.rope_dim, self.sink, self.recent, self.max_reqs,
        )


def scatter_pack_rows(x: torch.Tensor, slots: torch.Tensor, codes: torch.Tensor, params: torch.Tensor,
                      codec: _lib.Codec, err: torch.Tensor | None = None) -> None:
    """``rolaq_scatter_pack_rows``: rotated FP32 rows -> codes/params at ``slots``."""
    _check(x, "x", torch.float32, 2)
    if x.stride(1) != 1:
        raise ValueError("x rows must be contiguous")
    sp, s64 = _index(slots, "slots")
    if slots.numel() != x.shape[0]:
        raise ValueError("slots must have one entry per row")
    _lib.call("rolaq_scatter_pack_rows", x.data_ptr(), x.stride(0), sp, s64, x.shape[0], x.shape[1], GROUP_SIZE,
              codec, codes.data_ptr(), params.data_ptr(), codes.shape[0], _err_ptr(err), _lib.stream_ptr())


def write_aux(c: torch.Tensor, k_pe: torch.Tensor, slots: torch.Tensor, view: LayerView, seq_lens=None,
              req_idx=None, positions=None, err=None) -> None:
    """``rolaq_write_aux``: k_pe, ring rows and slot/ring maps from rotated FP32 rows."""
    _check(c, "c", torch.float32, 2)
    _check(k_pe, "k_pe", torch.bfloat16, 2)
    if slots.dtype != torch.int64:
        raise TypeError("slots must be int64")
    sq, sq64 = _index(seq_lens, "seq_lens")
    rq, rq64 = _index(req_idx, "req_idx")
    po, po64 = _index(positions, "positions")
    cs = view.c_struct()
    _lib.call("rolaq_write_aux", c.data_ptr(), c.stride(0), k_pe.data_ptr(), k_pe.stride(0), slots.data_ptr(),
              sq, sq64, rq, rq64, po, po64, c.shape[0], ctypes.byref(cs), _err_ptr(err), _lib.stream_ptr())


def fused_write(c_kv: torch.Tensor, k_pe: torch.Tensor, slots: torch.Tensor, rot_t: torch.Tensor,
                codec: _lib.Codec, view: LayerView, seq_lens=None, req_idx=None, positions=None, err=None) -> None:
    """``rolaq_fused_write``: tcgen05 rotation + codec + scatter + k_pe + window stores."""
    _check(c_kv, "c_kv", torch.bfloat16, 2)
    _check(k_pe, "k_pe", torch.bfloat16, 2)
    _check(rot_t, "rot_t", torch.bfloat16, 2)
    if c_kv.stride(1) != 1 or k_pe.stride(1) != 1 or not rot_t.is_contiguous():
        raise ValueError("c_kv/k_pe rows and rot_t must be contiguous")
    if slots.dtype != torch.int64 or not slots.is_contiguous():
        raise TypeError("slots must be contiguous int64")
    n = c_kv.shape[0]
    if k_pe.shape[0] != n or slots.numel() != n:
        raise ValueError("c_kv, k_pe and slots must have the same number of rows")
    if c_kv.shape[1] != view.latent_dim or k_pe.shape[1] != view.rope_dim:
        raise ValueError("c_kv / k_pe widths do not match the cache")
    if tuple(rot_t.shape) != (view.latent_dim, view.latent_dim):
        raise ValueError("rot_t must be [D, D]")
    sq, sq64 = _index(seq_lens, "seq_lens")
    rq, rq64 = _index(req_idx, "req_idx")
    po, po64 = _index(positions, "positions")
    cs = view.c_struct()
    _lib.call("rolaq_fused_write", c_kv.data_ptr(), c_kv.stride(0), k_pe.data_ptr(), k_pe.stride(0),
              slots.data_ptr(), sq, sq64, rq, rq64, po, po64, n, rot_t.data_ptr(), codec, ctypes.byref(cs),
              _err_ptr(err), _lib.stream_ptr())


def encode_rows(x: torch.Tensor, rot_t: torch.Tensor, codec: _lib.Codec, codes: torch.Tensor,
                params: torch.Tensor, slots: torch.Tensor | None = None) -> None:
    """``rolaq_fused_write`` without k_pe or window stores: BF16 rows -> rotated ->
    codes/params at ``slots`` (default: row i -> slot i)."""
    _check(x, "x", torch.bfloat16, 2)
    _check(rot_t, "rot_t", torch.bfloat16, 2)
    if x.stride(1) != 1 or not rot_t.is_contiguous():
        raise ValueError("x rows and rot_t must be contiguous")
    n, d = x.shape
    if codes.dtype != torch.uint8 or tuple(codes.shape[1:]) != (d // 4,) or not codes.is_contiguous():
        raise ValueError("codes must be contiguous uint8 [slots, D/4]")
    if params.dtype != torch.float32 or tuple(params.shape[1:]) != (d // GROUP_SIZE, 2) or not params.is_contiguous():
        raise ValueError("params must be contiguous float32 [slots, D/128, 2]")
    if slots is None:
        if codes.shape[0] < n:
            raise ValueError("codes has fewer slots than rows")
        slots = torch.arange(n, dtype=torch.int64, device=x.device)
    elif slots.dtype != torch.int64 or slots.numel() != n:
        raise ValueError("slots must be int64 with one entry per row")
    cs = _lib.LayerCache(codes.data_ptr(), params.data_ptr(), None, None, None, None, codes.shape[0], 0, d, 0, 0, 0, 0)
    _lib.call("rolaq_fused_write", x.data_ptr(), x.stride(0), None, 0, slots.data_ptr(), None, 0, None, 0, None, 0,
              n, rot_t.data_ptr(), codec, ctypes.byref(cs), None, _lib.stream_ptr())


def rotate_rows(x: torch.Tensor, w: torch.Tensor, out_f32: torch.Tensor | None = None,
                out_bf16: torch.Tensor | None = None) -> None:
    """``rolaq_rotate_rows``: out[i, o] = sum_k x[i, k] * w[o, k] on tcgen05 (FP32 accumulate)."""
    _check(x, "x", torch.bfloat16, 2)
    _check(w, "w", torch.bfloat16, 2)
    if x.stride(1) != 1 or not w.is_contiguous():
        raise ValueError("x rows and w must be contiguous")
    out = out_f32 if out_f32 is not None else out_bf16
    if out is None:
        raise ValueError("give out_f32 and/or out_bf16")
    if out_f32 is not None and out_bf16 is not None and out_f32.stride(0) != out_bf16.stride(0):
        raise ValueError("out_f32 and out_bf16 must share the row stride")
    _lib.call("rolaq_rotate_rows", x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], w.data_ptr(),
              _lib.ptr(out_f32), _lib.ptr(out_bf16), out.stride(0), _lib.stream_ptr())


def dequant_rows(codes: torch.Tensor, params: torch.Tensor, slots: torch.Tensor | None = None, n: int | None = None,
                 out_f32: torch.Tensor | None = None, out_bf16: torch.Tensor | None = None,
                 err: torch.Tensor | None = None) -> None:
    """``rolaq_dequant_rows``."""
    _check(codes, "codes", torch.uint8, 2)
    sp, s64 = _index(slots, "slots")
    rows = slots.numel() if slots is not None else (codes.shape[0] if n is None else n)
    out = out_f32 if out_f32 is not None else out_bf16
    if out is None:
        raise ValueError("give out_f32 and/or out_bf16")
    _lib.call("rolaq_dequant_rows", codes.data_ptr(), params.data_ptr(), sp, s64, rows, codes.shape[1] * 4,
              codes.shape[0], _lib.ptr(out_f32), _lib.ptr(out_bf16), out.stride(0), _err_ptr(err),
              _lib.stream_ptr())


def prepare_gf_splits(splits: torch.Tensor, quant: torch.Tensor, merge: torch.Tensor) -> None:
    """``rolaq_prepare_gf_splits`` (deployment/patches/rolaq_sglang.patch:81-92)."""
    for name, t in (("splits", splits), ("quant", quant), ("merge", merge)):
        _check(t, name, torch.int32)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if quant.numel() < splits.numel() or merge.numel() < splits.numel():
        raise ValueError("quant/merge too small")
    _lib.call("rolaq_prepare_gf_splits", splits.data_ptr(), quant.data_ptr(), merge.data_ptr(), splits.numel(),
              _lib.stream_ptr())


def packed_decode(q: torch.Tensor, view: LayerView, page_table: torch.Tensor, seq_lens: torch.Tensor,
                  sm_scale: float, num_splits: int, part_o: torch.Tensor, part_lse: torch.Tensor,
                  out: torch.Tensor | None, out_lse: torch.Tensor | None = None, err: torch.Tensor | None = None,
                  token_range: torch.Tensor | None = None) -> None:
    """``rolaq_packed_decode``: q [B, H, D+Dr] bf16 -> out [B, H, D] bf16 (rotated frame).
    ``out=None`` writes only the split partials (``part_o``, ``part_lse``; the window split's
    at index ``num_splits``) for a caller that merges them itself."""
    _check(q, "q", torch.bfloat16, 3)
    if out is not None:
        _check(out, "out", torch.bfloat16, 3)
    _check(page_table, "page_table", torch.int32, 2)
    _check(seq_lens, "seq_lens", torch.int32, 1)
    b, h, w = q.shape
    if w != view.latent_dim + view.rope_dim or q.stride(2) != 1:
        raise ValueError("q must be [B, H, D + Dr] with contiguous rows")
    if out is not None and (tuple(out.shape) != (b, h, view.latent_dim) or out.stride(2) != 1):
        raise ValueError("out must be [B, H, D] with contiguous rows")
    if page_table.shape[0] < b or page_table.stride(1) != 1 or seq_lens.numel() < b:
        raise ValueError("page_table / seq_lens too small")
    parts = num_splits + 1
    if part_o.dtype != torch.float32 or part_o.numel() < b * h * parts * view.latent_dim or not part_o.is_contiguous():
        raise ValueError("part_o must be contiguous float32 with B*H*(num_splits+1)*D elements")
    if part_lse.dtype != torch.float32 or part_lse.numel() < b * h * parts or not part_lse.is_contiguous():
        raise ValueError("part_lse must be contiguous float32 with B*H*(num_splits+1) elements")
    if token_range is not None:
        _check(token_range, "token_range", torch.int32, 2)
        if token_range.shape[0] < b or token_range.shape[1] != 2 or not token_range.is_contiguous():
            raise ValueError("token_range must be contiguous int32 [B, 2]")
    if out_lse is not None and (out_lse.dtype != torch.float32 or out_lse.numel() < b * h):
        raise ValueError("out_lse must be float32 with B*H elements")
    cs = view.c_struct()
    _lib.call("rolaq_packed_decode", q.data_ptr(), q.stride(0), q.stride(1), b, h, ctypes.byref(cs),
              page_table.data_ptr(), page_table.stride(0), page_table.shape[1], seq_lens.data_ptr(),
              _lib.ptr(token_range), float(sm_scale), int(num_splits), part_o.data_ptr(), part_lse.data_ptr(),
              _lib.ptr(out), out.stride(0) if out is not None else 0, out.stride(1) if out is not None else 0,
              _lib.ptr(out_lse), _err_ptr(err), _lib.stream_ptr())


def merge_partials(part_o: torch.Tensor, part_lse: torch.Tensor, out_bf16: torch.Tensor | None = None,
                   out_f32: torch.Tensor | None = None, out_lse: torch.Tensor | None = None) -> None:
    """``rolaq_merge_partials`` for partials laid out [parts, rows, D] / [parts, rows]."""
    _check(part_o, "part_o", torch.float32, 3)
    _check(part_lse, "part_lse", torch.float32, 2)
    parts, rows, d = part_o.shape
    out = out_bf16 if out_bf16 is not None else out_f32
    ld = out.stride(-2) if out is not None else d
    _lib.call("rolaq_merge_partials", part_o.data_ptr(), part_o.stride(1), part_o.stride(0), part_lse.data_ptr(),
              part_lse.stride(1), part_lse.stride(0), parts, rows, d, _lib.ptr(out_bf16), _lib.ptr(out_f32), ld,
              _lib.ptr(out_lse), _lib.stream_ptr())


def _window_rpc(latent_dim: int, rope_dim: int, window_rows: int) -> int:
    """Requests one window CTA stages at a time (``window_rpc`` in ``csrc/window.cu``)."""
    if window_rows <= 0:
        return 8
    per_req = window_rows * (latent_dim + rope_dim) * 4 + 2 * 32 * 8 + 4
    rpc = min((200 * 1024) // per_req, (12 * 512) // (window_rows * (latent_dim + rope_dim) // 8))
    return max(1, min(rpc, 8))


def default_num_splits(batch: int, max_ctx: int, sm_count: int = 148, ctas_per_sm: int | None = None,
                       latent_dim: int = 512, rope_dim: int = 64, heads: int = 16, window_rows: int = 20) -> int:
    """Pick the number of INT2 KV splits per request: the count that minimises
    ``waves * (tiles per split + 3)``, where a wave is ``sm_count * ctas_per_sm`` CTAs, a tile is
    128 tokens and the 3 is a CTA's fixed cost (set-up, query conversion, epilogue) in tiles,
    fitted to split-count sweeps on B200 (B64 x 16K: 2 splits; B128 x 8K: 1).  Ties go to
    fewer splits.  The tcgen05 kernel (every built shape) holds one CTA per SM.

    A one-wave grid of 15 or more splits that leaves too few SMs for the window split to run
    beside it (``window_first_fits`` in ``csrc/window.cu``; ``window_rows`` = sink + recent)
    costs 5 tiles more: the window split and the merge then follow the INT2 grid, and the
    merge spreads the many splits of few requests over few CTAs.  Measured on B200, one call:
    B2 x 128K, 74 splits 62.4 us against 73 splits 47.1; B4 x 64K, 37 splits 56.0 against
    36 splits 45.8."""
    tc = {(512, 64, 16), (512, 64, 8), (256, 32, 40), (256, 32, 16)}
    if ctas_per_sm is None:
        ctas_per_sm = 1 if (latent_dim, rope_dim, heads) in tc else 2
    tiles = max(1, math.ceil(max_ctx / (2 * PAGE)))
    slots = sm_count * ctas_per_sm
    rpc = _window_rpc(latent_dim, rope_dim, window_rows)
    best, best_cost = 1, float("inf")
    for s in range(1, min(tiles, 128) + 1):
        tps = math.ceil(tiles / s)
        if tps < 2 and s > 1:
            break
        waves = math.ceil(batch * s / slots)
        cost = waves * (tps + 3)
        if (latent_dim, rope_dim, heads) in tc and waves == 1 and s + 1 >= 16:
            free = sm_count - batch * s
            if not (free >= 1 and free * 2 * rpc >= batch):
                cost += 5
        if cost < best_cost:
            best, best_cost = s, cost
    return best


def absorb_query(q_nope: torch.Tensor, q_pe: torch.Tensor | None, w_kc: torch.Tensor, q_out: torch.Tensor,
                 err: torch.Tensor | None = None) -> None:
    """``rolaq_absorb_query``: ``q_out[..., :D] = q_nope @ w_kc[h]^T`` per head, ``q_out[..., D:] = q_pe``.

    q_nope ``[B, H, Dn]``, q_pe ``[B, H, Dr]`` (or None), w_kc ``[H, D, Dn]`` contiguous,
    q_out ``[B, H, D + Dr]``; all BF16 with contiguous rows."""
    _check(q_nope, "q_nope", torch.bfloat16, 3)
    _check(w_kc, "w_kc", torch.bfloat16, 3)
    _check(q_out, "q_out", torch.bfloat16, 3)
    b, h, dn = q_nope.shape
    hh, d, dn2 = w_kc.shape
    if hh != h or dn2 != dn or not w_kc.is_contiguous():
        raise ValueError("w_kc must be contiguous [H, D, Dn]")
    dr = 0 if q_pe is None else q_pe.shape[2]
    if q_pe is not None:
        _check(q_pe, "q_pe", torch.bfloat16, 3)
        if tuple(q_pe.shape[:2]) != (b, h) or q_pe.stride(2) != 1:
            raise ValueError("q_pe must be [B, H, Dr] with contiguous rows")
    if tuple(q_out.shape) != (b, h, d + dr) or q_out.stride(2) != 1 or q_nope.stride(2) != 1:
        raise ValueError("q_out must be [B, H, D + Dr]; rows contiguous")
    _lib.call("rolaq_absorb_query", q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1), _lib.ptr(q_pe),
              0 if q_pe is None else q_pe.stride(0), 0 if q_pe is None else q_pe.stride(1), w_kc.data_ptr(), b, h, dn,
              d, dr, q_out.data_ptr(), q_out.stride(0), q_out.stride(1), _err_ptr(err), _lib.stream_ptr())


def project_output(o: torch.Tensor, w_vc: torch.Tensor, out: torch.Tensor, err: torch.Tensor | None = None) -> None:
    """``rolaq_project_output``: ``out[b, h] = o[b, h] @ w_vc[h]^T``; o ``[B, H, D]``, w_vc ``[H, Dv, D]``
    contiguous, out ``[B, H, Dv]``; BF16, contiguous rows."""
    _check(o, "o", torch.bfloat16, 3)
    _check(w_vc, "w_vc", torch.bfloat16, 3)
    _check(out, "out", torch.bfloat16, 3)
    b, h, d = o.shape
    hh, dv, d2 = w_vc.shape
    if hh != h or d2 != d or not w_vc.is_contiguous():
        raise ValueError("w_vc must be contiguous [H, Dv, D]")
    if tuple(out.shape) != (b, h, dv) or out.stride(2) != 1 or o.stride(2) != 1:
        raise ValueError("out must be [B, H, Dv]; rows contiguous")
    _lib.call("rolaq_project_output", o.data_ptr(), o.stride(0), o.stride(1), w_vc.data_ptr(), b, h, d, dv,
              out.data_ptr(), out.stride(0), out.stride(1), _err_ptr(err), _lib.stream_ptr())


def page_table_from_req_to_token(req_to_token: torch.Tensor, req_pool_indices: torch.Tensor, seq_lens: torch.Tensor,
                                 page_table: torch.Tensor, seq_lens_out: torch.Tensor | None = None,
                                 err: torch.Tensor | None = None) -> None:
    """``rolaq_page_table_from_req_to_token``: the reader's 64-token page table (and int32
    lengths) from SGLang's ``req_to_token`` map, one launch, no host sync."""
    _check(req_to_token, "req_to_token", torch.int32, 2)
    _check(page_table, "page_table", torch.int32, 2)
    if req_to_token.stride(1) != 1 or page_table.stride(1) != 1:
        raise ValueError("req_to_token / page_table rows must be contiguous")
    rp, r64 = _index(req_pool_indices, "req_pool_indices")
    sp, s64 = _index(seq_lens, "seq_lens")
    b = req_pool_indices.numel()
    if seq_lens.numel() < b or page_table.shape[0] < b:
        raise ValueError("seq_lens / page_table have fewer rows than req_pool_indices")
    max_pages = min(page_table.shape[1], req_to_token.shape[1] // PAGE)
    if seq_lens_out is not None and (seq_lens_out.dtype != torch.int32 or seq_lens_out.numel() < b):
        raise ValueError("seq_lens_out must be int32 with one entry per request")
    _lib.call("rolaq_page_table_from_req_to_token", req_to_token.data_ptr(), req_to_token.stride(0), rp, r64, sp,
              s64, b, max_pages, page_table.data_ptr(), page_table.stride(0), _lib.ptr(seq_lens_out), _err_ptr(err),
              _lib.stream_ptr())
