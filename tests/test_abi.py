"""The C ABI: libxencb.so loads without a GPU and exports exactly what include/xencb.h declares.
CPU only; no compute entry point is called here (they need a CUDA device)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from kv_skill_v2_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "xencb.h"


def declared() -> list:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"XENCB_API\s+[\w\s\*]+?\b(xencb_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "xencb_read_decode" in names and "xencb_route" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(N.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), f"{name} declared in xencb.h but not exported"


def test_binding_table_matches_header():
    assert sorted(N.SIGNATURES) == declared()


def test_host_only_entry_points():
    L = N.lib()
    assert L.xencb_abi_version() == N.ABI_VERSION
    assert L.xencb_route_k(4, 64) == 4 and L.xencb_route_k(0, 64) == 64 and L.xencb_route_k(64, 64) == 64
    assert isinstance(L.xencb_last_error(), bytes)
    before = N.launch_count()
    assert before >= 0
    assert L.xencb_route_k(4, 64) == 4 and N.launch_count() == before  # host-only calls launch nothing
    # prepared 3xF16 weights: a 256-byte head, then per 128-row band and 64-column block a 32 KiB tile pair
    for n, k in [(2048, 4096), (200, 520), (128, 64), (44, 40), (1, 8)]:
        pairs = -(-n // 128) * -(-k // 64)
        assert L.xencb_weights_prep_bytes(n, k) == 256 + pairs * 2 * 128 * 64 * 2
    assert L.xencb_weights_prep_bytes(0, 64) == 0 and L.xencb_weights_prep_bytes(64, 0) == 0


def test_header_constants_match_binding():
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define (XENCB_\w+) (\d+)u?", text))
    assert int(consts["XENCB_F32"]) == N.F32 and int(consts["XENCB_F16"]) == N.F16 and int(consts["XENCB_BF16"]) == N.BF16
    assert int(consts["XENCB_EINVAL"]) == N.EINVAL and int(consts["XENCB_ABI_VERSION"]) == N.ABI_VERSION
    assert int(consts["XENCB_PIN_RMS"]) == N.PIN_RMS and int(consts["XENCB_PIN_L2"]) == N.PIN_L2


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "LIB_PATH", tmp_path / "libxencb.so")
    monkeypatch.setattr(N, "_lib", None)
    with pytest.raises(N.NativeMissing):
        N.lib()
