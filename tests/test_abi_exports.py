"""The C ABI library loads and exports every symbol include/rolaq_b200.h declares.

Only host-side paths are exercised here (argument validation that returns before
any launch); the compute paths are covered by the -m gpu tests.
"""

import ctypes
import re
from pathlib import Path

import pytest

from mla_kv_quant_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "rolaq_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|int64_t|const char\*)\s+(rolaq_\w+)\(", text, flags=re.M)))


def test_header_lists_every_binding():
    assert declared() == sorted(_lib.EXPORTS)


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from mla_kv_quant_b200 import build

        build.build()
    return _lib.load()


def test_library_exports_all_symbols(lib):
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.rolaq_version() == 10000


def test_validation_returns_status_without_launching(lib):
    codec = _lib.Codec(0.9, 1.0, 1.5)
    rc = lib.rolaq_scatter_pack_rows(None, 512, None, 1, -1, 512, 128, codec, None, None, 1, None, None)
    assert rc == _lib.ROLAQ_EINVAL and b"n < 0" in lib.rolaq_last_error()
    rc = lib.rolaq_scatter_pack_rows(None, 512, None, 1, 4, 512, 64, codec, None, None, 1, None, None)
    assert rc == _lib.ROLAQ_EUNSUPPORTED and b"group_size" in lib.rolaq_last_error()
    cache = _lib.LayerCache()
    cache.latent_dim = 384
    rc = lib.rolaq_packed_decode(None, 0, 0, 1, 16, ctypes.byref(cache), None, 0, 1, None, None, 0.1, 4, None, None,
                                 None, 0, 0, None, None, None)
    assert rc == _lib.ROLAQ_EUNSUPPORTED and b"latent_dim" in lib.rolaq_last_error()
    rc = lib.rolaq_merge_partials(None, 0, 0, None, 0, 0, 0, 1, 512, None, None, 0, None, None)
    assert rc == _lib.ROLAQ_EINVAL
    rc = lib.rolaq_prepare_gf_splits(None, None, None, 0, None)
    assert rc == _lib.ROLAQ_OK  # empty input is a no-op


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU or Python fallback"):
        _lib.load(tmp_path / "librolaq_b200.so")
