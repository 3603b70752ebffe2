"""CPU checks of the C ABI: the library loads and exports every declared symbol."""

from __future__ import annotations

import ctypes
import os
import re

from copy_on_write_sdm_b200 import _lib
from tests.conftest import ROOT


def header_symbols() -> list[str]:
    text = open(os.path.join(ROOT, "include", "cow_sdm.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cow_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(header_symbols()) == set(_lib.exported_symbols())


def test_host_only_entry_points():
    lib = _lib.load()
    assert lib.cow_abi_version() == 1
    assert lib.cow_last_error() == b"no error"
    # scratch sizing: per-pool header (8 pools x 8 B) + one flag per bank slot (pools padded to 4-bank tiles, + one tile per pool), one per 128-bank group
    assert lib.cow_decode_scratch_bytes(64 * 7, 7) == 64 + 8 * (4 * (112 + 7) + 448 // 128 + 7)
    assert lib.cow_scan_blocks(0) == 8
    assert lib.cow_scan_blocks(2048) == 9


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    assert lib.cow_decode_step(None, None, 1, 4, 16, 1, 0, None, 0, None) == _lib.ERR_INVALID
    pool = _lib.CowPool()
    step = _lib.CowStep()
    # width 130 is not a multiple of 4 -> unsupported before anything launches
    pool.width = 130
    pool.slab_dtype = _lib.F32
    scratch = ctypes.create_string_buffer(64)
    assert lib.cow_decode_step(ctypes.byref(pool), ctypes.byref(step), 1, 4, 16, 1, 0,
                               ctypes.addressof(scratch), 64, None) == _lib.ERR_UNSUPPORTED
    assert lib.cow_grow(None, None, 0, None, None, 0, 4, 0, None, None, None) == _lib.ERR_INVALID
