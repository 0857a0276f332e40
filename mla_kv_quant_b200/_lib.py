"""ctypes binding of librolaq_b200.so (the C ABI in include/rolaq_b200.h).

The library is loaded from ``mla_kv_quant_b200/_lib/`` (built by
``python -m mla_kv_quant_b200.build``).  There is no fallback: if the library is
missing every entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "librolaq_b200.so"

ROLAQ_OK = 0
ROLAQ_EINVAL = -1
ROLAQ_EUNSUPPORTED = -2
ROLAQ_ECUDA = -3

CODEC_LLOYD = 0
CODEC_UNIFORM = 1

DEV_BAD_SLOT = 1
DEV_BAD_PAGE = 2
DEV_TIMEOUT = 4
DEV_BAD_REQ = 8
DEV_PEER_TIMEOUT = 16
IPC_HANDLE_BYTES = 64

EXPORTS = (
    "rolaq_version",
    "rolaq_last_error",
    "rolaq_check_device",
    "rolaq_scatter_pack_rows",
    "rolaq_write_aux",
    "rolaq_fused_write",
    "rolaq_rotate_rows",
    "rolaq_dequant_rows",
    "rolaq_prepare_gf_splits",
    "rolaq_packed_decode",
    "rolaq_packed_decode_static_capacity",
    "rolaq_packed_decode_static",
    "rolaq_merge_partials",
    "rolaq_absorb_query",
    "rolaq_project_output",
    "rolaq_page_table_from_req_to_token",
    "rolaq_peer_recv_bytes",
    "rolaq_peer_merge_push",
    "rolaq_peer_wait_merge",
    "rolaq_device_alloc",
    "rolaq_device_free",
    "rolaq_ipc_get_handle",
    "rolaq_ipc_open",
    "rolaq_ipc_close",
)


class LayerCache(ctypes.Structure):
    """``rolaq_layer_cache``."""

    _fields_ = [
        ("codes", ctypes.c_void_p),
        ("params", ctypes.c_void_p),
        ("rope", ctypes.c_void_p),
        ("hp", ctypes.c_void_p),
        ("rows", ctypes.c_void_p),
        ("owners", ctypes.c_void_p),
        ("num_slots", ctypes.c_int64),
        ("num_ring_rows", ctypes.c_int64),
        ("latent_dim", ctypes.c_int32),
        ("rope_dim", ctypes.c_int32),
        ("sink", ctypes.c_int32),
        ("recent", ctypes.c_int32),
        ("max_reqs", ctypes.c_int64),
    ]


class Codec(ctypes.Structure):
    """``rolaq_codec``."""

    _fields_ = [
        ("threshold", ctypes.c_float),
        ("scale_factor", ctypes.c_float),
        ("zero_const", ctypes.c_float),
        ("family", ctypes.c_int32),
    ]


class RolaqError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
F32 = ctypes.c_float
INT = ctypes.c_int

_SIGS = {
    "rolaq_version": (INT, []),
    "rolaq_last_error": (ctypes.c_char_p, []),
    "rolaq_check_device": (INT, []),
    "rolaq_scatter_pack_rows": (INT, [P, I64, P, INT, I64, I32, I32, Codec, P, P, I64, P, P]),
    "rolaq_write_aux": (INT, [P, I64, P, I64, P, P, INT, P, INT, P, INT, I64, ctypes.POINTER(LayerCache), P, P]),
    "rolaq_fused_write": (
        INT,
        [P, I64, P, I64, P, P, INT, P, INT, P, INT, I64, P, Codec, ctypes.POINTER(LayerCache), P, P],
    ),
    "rolaq_rotate_rows": (INT, [P, I64, I64, I32, P, P, P, I64, P]),
    "rolaq_dequant_rows": (INT, [P, P, P, INT, I64, I32, I64, P, P, I64, P, P]),
    "rolaq_prepare_gf_splits": (INT, [P, P, P, I64, P]),
    "rolaq_packed_decode": (
        INT,
        [P, I64, I64, I32, I32, ctypes.POINTER(LayerCache), P, I64, I32, P, P, F32, I32, P, P, P, I64, I64, P, P, P],
    ),
    "rolaq_packed_decode_static_capacity": (I64, []),
    "rolaq_packed_decode_static": (
        INT,
        [P, I64, I64, I32, I32, ctypes.POINTER(LayerCache), P, I64, I32, P, P, F32, I32, P, I64, I64, P, P, P],
    ),
    "rolaq_merge_partials": (INT, [P, I64, I64, P, I64, I64, I32, I64, I32, P, P, I64, P, P]),
    "rolaq_page_table_from_req_to_token": (INT, [P, I64, P, INT, P, INT, I64, I32, P, I64, P, P, P]),
    "rolaq_absorb_query": (INT, [P, I64, I64, P, I64, I64, P, I32, I32, I32, I32, I32, P, I64, I64, P, P]),
    "rolaq_project_output": (INT, [P, I64, I64, P, I32, I32, I32, I32, P, I64, I64, P, P]),
    "rolaq_peer_recv_bytes": (I64, [I32, I64, I32]),
    "rolaq_peer_merge_push": (INT, [P, P, I32, I64, I32, P, I32, I32, P, P]),
    "rolaq_peer_wait_merge": (INT, [P, I32, I64, I32, P, P, P, P, P, P]),
    "rolaq_device_alloc": (INT, [I64, ctypes.POINTER(ctypes.c_void_p)]),
    "rolaq_device_free": (INT, [P]),
    "rolaq_ipc_get_handle": (INT, [P, P]),
    "rolaq_ipc_open": (INT, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "rolaq_ipc_close": (INT, [P]),
}


def load(path: Path | str | None = None):
    """Load (once) and return the ctypes library object."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m mla_kv_quant_b200.build` "
                "(the packed-INT2 path has no CPU or Python fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != ROLAQ_OK:
        raise RolaqError(name, rc, lib.rolaq_last_error().decode(errors="replace"))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_checked_devices: set[int] = set()


def require_device(t: torch.Tensor) -> None:
    """Raise unless ``t`` lives on an sm_100 CUDA device the library supports."""
    if not t.is_cuda:
        raise ValueError("the packed-INT2 kernels run on CUDA tensors only (no CPU fallback)")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if idx in _checked_devices:
        return
    with torch.cuda.device(idx):
        call("rolaq_check_device")
    _checked_devices.add(idx)
