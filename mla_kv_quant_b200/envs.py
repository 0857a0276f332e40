"""Environment flags the reference serving stack reads for this path.

Names and defaults follow ``deployment/patches/rolaq_sglang.patch:41-47`` (the RoLaQ
flags) and the OSCAR flags ``deployment/serve.py:95-122`` sets.  Tunables of the
kernels (splits, pages per CTA) are function arguments, never environment reads.
"""

from __future__ import annotations

import os


class _Env:
    def __init__(self, name: str, default, kind):
        self.name, self.default, self.kind = name, default, kind

    def get(self):
        raw = os.environ.get(self.name)
        if raw is None or raw == "":
            return self.default
        if self.kind is bool:
            return raw.strip().lower() in ("1", "true", "yes", "on")
        return self.kind(raw)


class _Envs:
    SGLANG_ROLAQ_MLA_QUANTIZER_PATH = _Env("SGLANG_ROLAQ_MLA_QUANTIZER_PATH", "", str)
    SGLANG_ROLAQ_MLA_ABSORB_READ_ROTATIONS = _Env("SGLANG_ROLAQ_MLA_ABSORB_READ_ROTATIONS", False, bool)
    SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE = _Env("SGLANG_ROLAQ_MLA_FUSED_DECODE_WRITE", False, bool)
    SGLANG_OSCAR_MLA_KV_ROTATION_PATH = _Env("SGLANG_OSCAR_MLA_KV_ROTATION_PATH", "", str)
    SGLANG_OSCAR_MLA_KV_PACKED = _Env("SGLANG_OSCAR_MLA_KV_PACKED", False, bool)
    SGLANG_OSCAR_MLA_KV_BITS = _Env("SGLANG_OSCAR_MLA_KV_BITS", 2, int)
    SGLANG_OSCAR_MLA_KV_GROUP_SIZE = _Env("SGLANG_OSCAR_MLA_KV_GROUP_SIZE", 128, int)
    SGLANG_LLOYD_MAX = _Env("SGLANG_LLOYD_MAX", False, bool)
    SGLANG_MIXED_KV_PREFIX_TOKENS = _Env("SGLANG_MIXED_KV_PREFIX_TOKENS", 4, int)
    SGLANG_MIXED_KV_RECENT_TOKENS = _Env("SGLANG_MIXED_KV_RECENT_TOKENS", 16, int)


envs = _Envs()
