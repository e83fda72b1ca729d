"""The C-ABI library: built, loadable, exports every symbol the header declares, and rejects
bad arguments on the host before any launch (no GPU needed for these calls)."""
import ctypes
import re
from pathlib import Path

import pytest

from lagunalab_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "laguna_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(lg_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "lg_router_topk" in names and "lg_q8_decode_attention" in names
    assert "lg_moe_experts" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    h = ctypes.CDLL(str(_lib.LIB_PATH))
    for n in declared():
        assert hasattr(h, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_header_enum_values_match_the_binding():
    text = HEADER.read_text()
    values = {}
    for body in re.findall(r"enum\s*\{([^}]*)\}", text):
        for name, val in re.findall(r"(LG_\w+)\s*=\s*(-?\d+)", body):
            values[name] = int(val)
    for name in ("LG_SCORE_SIGMOID", "LG_SCORE_SOFTMAX", "LG_PATH_AUTO", "LG_PATH_GEMV",
                 "LG_PATH_TENSOR", "LG_MOE_GEMV_MAX_ROWS"):
        assert values[name] == getattr(_lib, name), name


def test_abi_version_and_no_error():
    assert _lib.lib().lg_abi_version() == 2
    assert isinstance(_lib.lib().lg_last_error(), bytes)


def test_workspace_sizes_are_host_only_and_monotone():
    L = _lib.lib()
    a = L.lg_moe_workspace_bytes(16, 2048, 1024, 128, 8, 1024)
    b = L.lg_moe_workspace_bytes(4096, 2048, 1024, 128, 8, 1024)
    assert 0 < a < b and a % 256 == 0
    assert L.lg_q8_decode_workspace_bytes(1, 32, 4, 82671) > 0


def _fake(n=1):
    return ctypes.c_void_p(0x1000 * n)  # never dereferenced: the checks fail first


def test_q8_rejects_head_dim_and_group():
    with pytest.raises(ValueError, match="head_dim"):
        _lib.call("lg_q8_decode_attention", _fake(), 1, 8, 2, 64, _fake(), _fake(), _fake(),
                  _fake(), _fake(), _fake(), 256, 10, 0.1, _fake(), _fake(), 1 << 20, None)
    with pytest.raises(ValueError, match="too many"):
        _lib.call("lg_q8_decode_attention", _fake(), 1, 34, 2, 128, _fake(), _fake(), _fake(),
                  _fake(), _fake(), _fake(), 256, 10, 0.1, _fake(), _fake(), 1 << 20, None)
    with pytest.raises(ValueError, match="n"):
        _lib.call("lg_q8_decode_attention", _fake(), 1, 8, 2, 128, _fake(), _fake(), _fake(),
                  _fake(), _fake(), _fake(), 256, 0, 0.1, _fake(), _fake(), 1 << 20, None)


def test_router_rejects_unsupported_sizes():
    args = lambda E, k, H=2048: (_fake(), 4, H, _fake(), None, None, 0, None, E, k, 1, 0,
                                 _fake(), _fake(), _fake(), None, None)
    with pytest.raises(ValueError, match="256"):
        _lib.call("lg_router_topk", *args(300, 8))
    with pytest.raises(ValueError, match="k="):
        _lib.call("lg_router_topk", *args(8, 9))
    with pytest.raises(ValueError, match="multiple of 64"):
        _lib.call("lg_router_topk", *args(8, 2, H=100))


def test_experts_reject_non_4bit_and_small_workspace():
    z = [_fake()] * 9
    with pytest.raises(ValueError, match="4-bit"):
        _lib.call("lg_moe_experts", _fake(), 4, 2048, 1024, 8, 2, _fake(), _fake(), 1.0, *z,
                  0, *([None] * 9), 64, 8, 0, _fake(), _fake(), 1 << 30, None)
    with pytest.raises(_lib.LagunaError) as e:
        _lib.call("lg_moe_experts", _fake(), 4, 2048, 1024, 8, 2, _fake(), _fake(), 1.0, *z,
                  0, *([None] * 9), 64, 4, 0, _fake(), _fake(), 16, None)
    assert e.value.code == _lib.LG_ERR_WORKSPACE


def test_quantize_rejects_bad_geometry():
    with pytest.raises(ValueError, match="multiple of group_size"):
        _lib.call("lg_quantize_rows", _fake(), 0, 1, 1, 4, 100, 0, 0, 100, 8, 64, _fake(),
                  _fake(), _fake(), 4, 0, None)
    with pytest.raises(ValueError, match="capacity"):
        _lib.call("lg_quantize_rows", _fake(), 0, 1, 1, 4, 128, 0, 0, 128, 8, 64, _fake(),
                  _fake(), _fake(), 3, 0, None)
