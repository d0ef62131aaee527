"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, and its host-only entry points behave (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

from synapcore_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "sckv.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^SCKV_API\s+[^(]*?\b(sckv_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_header_symbols():
    lib = N.load()
    declared = _declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(N.EXPORTED_SYMBOLS)


def test_version_and_status_strings():
    lib = N.load()
    assert b"sm_100a" in lib.sckv_version()
    assert N.status_string(N.SCKV_ERR_BOUNDS) == "index out of bounds"
    assert N.status_string(N.SCKV_ERR_POOL_EXHAUSTED) == "page pool exhausted"


@pytest.mark.parametrize("dtype,expect_scale", [(N.DTYPE_F16, 0), (N.DTYPE_INT8, 1), (N.DTYPE_FP8_E4M3, 1)])
def test_required_bytes_matches_layout(dtype, expect_scale):
    L, H, D, P = 16, 16, 128, 64
    data, scales, alloc = N.required_bytes(L, H, D, 16, P, dtype)
    el = 2 if dtype == N.DTYPE_F16 else 1
    assert data == L * P * 2 * H * 16 * D * el
    if dtype == N.DTYPE_INT8:
        assert scales == L * P * 2 * H * 16 * 2
    elif dtype == N.DTYPE_FP8_E4M3:
        assert scales == L * P * 2 * H * 4
    else:
        assert scales == 0
    assert alloc >= P * (4 + 8 + 4 + 4)


def test_reference_page_bytes():
    """fp16 all-layer page of the OLMoE shape = 2,097,152 bytes
    (tests/test_p1_2_paged_kv_cache.py:125 of the reference)."""
    data, _, _ = N.required_bytes(16, 16, 128, 16, 1, N.DTYPE_F16)
    assert data == 2097152
    data8, sc8, _ = N.required_bytes(16, 16, 128, 16, 1, N.DTYPE_INT8)
    assert data8 + sc8 == 1064960


def test_invalid_geometry_rejected():
    with pytest.raises(N.SCKVError):
        N.required_bytes(16, 16, 128, 8, 64, N.DTYPE_F16)  # page_tokens must be 16
    with pytest.raises(N.SCKVError):
        N.required_bytes(16, 16, 100, 16, 64, N.DTYPE_F16)  # head_dim % 16
    with pytest.raises(N.SCKVError):
        N.required_bytes(16, 16, 128, 16, 64, 9)
