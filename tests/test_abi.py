"""The C ABI without a GPU: the library loads, exports every entry point include/otq.h declares,
and the Python binding declares exactly those (no compute call is made here)."""
import ctypes
import re

import pytest

from conftest import ROOT
from opentpu_b200 import _lib as L

HEADER = ROOT / "include" / "otq.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"OTQ_API\s+[\w\s\*]+?\b(otq_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "otq_mm" in names and "otq_qmm" in names and "otq_quantize_rows" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    if not L.LIB_PATH.exists():
        pytest.fail(f"{L.LIB_PATH} is not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(str(L.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header():
    assert sorted(L.SIGNATURES) == declared()


def test_status_strings_without_a_device():
    lib = L.load()
    assert lib.otq_version().decode().startswith("libotq")
    for st in (0, -1, -2, -3, -4, -5):
        assert lib.otq_status_string(st)
    with pytest.raises(ValueError):
        L.check(L.ERR_ARG, "x")
    with pytest.raises(RuntimeError):
        L.check(L.ERR_DEVICE, "x")


def test_flag_and_format_codes_are_the_references():
    # opentpu/isa.py:21,26-27,30
    assert L.FMT == {"int8": 0, "int4": 1, "fp4": 2, "nvfp4": 3}
    assert (L.MM_UNIT, L.MM_ACC, L.MM_ASCALE, L.MM_RSC) == (1, 2, 8, 0x80)
    text = HEADER.read_text()
    for name, val in (("OTQ_MM_UNIT", "0x1"), ("OTQ_MM_RSC", "0x80"), ("OTQ_FMT_NVFP4", "3")):
        assert re.search(rf"#define {name} {val}\b", text)


def test_qact_planes_size_without_a_device():
    """otq_qact_planes_bytes is arithmetic only: 9 Mp + 3 Mp K bytes, Mp = M rounded up to 128;
    K must be whole 32-element groups (and at most 65536)."""
    lib = L.load()
    for M, K in ((1, 32), (128, 1024), (129, 2048), (512, 11008), (0, 64)):
        Mp = -(-M // 128) * 128
        assert lib.otq_qact_planes_bytes(M, K) == 9 * Mp + 3 * Mp * K
    for M, K in ((4, 48), (4, 0), (-1, 64), (4, 65568)):
        assert lib.otq_qact_planes_bytes(M, K) < 0
