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


def test_multi_pool_and_host_step_entry_points_reject_bad_arguments():
    lib = _lib.load()
    pools = (_lib.CowPool * 2)()
    for p in pools:
        p.banks, p.slots, p.width, p.capacity = 4, 8, 128, 16
    counts = (ctypes.c_int64 * 2)(2, 0)
    # workspace sizes: masks rounded to 16 bytes + scan header per pool
    assert lib.cow_release_workspace_bytes(pools, counts, 2) > 0
    assert lib.cow_release_workspace_bytes(pools, counts, 0) == -1
    assert lib.cow_release_workspace_bytes(pools, counts, _lib.MAX_LAYERS + 1) == -1
    assert lib.cow_retain_workspace_bytes(pools, 2) == 2 * 16
    assert lib.cow_append_workspace_bytes(pools, 2) > 0
    assert lib.cow_pack_workspace_bytes(-1, 1) == -1
    assert lib.cow_validate_workspace_bytes(pools, 2) == 2 * 4 * 20
    # a workspace that is too small (or missing) is rejected before anything launches
    ws = ctypes.create_string_buffer(16)
    ptrs = (ctypes.c_void_p * 2)(None, None)
    out = ctypes.create_string_buffer(8)
    assert lib.cow_release_layers(pools, ptrs, counts, 2, None, 0, out, None) == _lib.ERR_INVALID
    assert lib.cow_retain_layers(pools, ptrs, counts, 2, ptrs, ptrs, ws, 0, out, None) == _lib.ERR_INVALID
    assert lib.cow_validate_layers(pools, 2, ws, 16, out, None) == _lib.ERR_INVALID
    assert lib.cow_pack_apply_layers(pools, 0, ws, 16, None) == _lib.ERR_INVALID
    assert lib.cow_prefill_recurrence_layers(pools, None, 2, 4, 4, 16, 1, 0, None) == _lib.ERR_INVALID
    # resolved-route prefill: records of (4 + 3*4 + 3*16) words per (bank, token), 8 banks, 4 tokens
    assert lib.cow_prefill_workspace_bytes(pools, 2, 4, 4, 16) == 8 * 4 * 64 * 4
    assert lib.cow_prefill_workspace_bytes(pools, 2, 4, 0, 16) == -1
    assert lib.cow_prefill_recurrence_layers_ws(pools, None, 2, 4, 4, 16, 1, 0, ws, 16, None) == _lib.ERR_INVALID
    # direct cohort admission: workspace per pool = scan flags + two row lists
    assert lib.cow_admit_prefix_workspace_bytes(2, 8, 2) > 0
    assert lib.cow_admit_prefix_workspace_bytes(-1, 8, 1) == -1
    assert lib.cow_admit_prefix_workspace_bytes(2, 8, _lib.MAX_LAYERS + 1) == -1
    assert lib.cow_admit_prefix_layers(pools, None, None, 2, 2, None, ws, 16, None) == _lib.ERR_INVALID
    # host-to-host steps: negative sizes, missing buffers or events
    assert lib.cow_decode_step_host(pools, None, 1, 4, 16, 1, 0, None, 0, None, None, -1, None, None, 0,
                                    None) == _lib.ERR_INVALID
    assert lib.cow_decode_step_host_overlapped(pools, None, 1, 4, 16, 1, 0, None, 0, ws, ws, 16, ws, ws, 16,
                                               None, None, None, None, None, None) == _lib.ERR_INVALID


def test_readout_entry_rejects_bad_arguments():
    lib = _lib.load()
    ws = ctypes.create_string_buffer(16)
    p = [ws] * 5
    # missing output
    assert lib.cow_readout_mlp_step(*p, 1e-6, *[ws] * 6, 1e-5, ws, ws, 1, 1, 64, 2, 256, None,
                                    None) == _lib.ERR_INVALID
    # width not a multiple of heads
    assert lib.cow_readout_mlp_step(*p, 1e-6, *[ws] * 6, 1e-5, ws, ws, 1, 1, 65, 2, 256, ws,
                                    None) == _lib.ERR_INVALID
    # wider than the compiled kernel
    assert lib.cow_readout_mlp_step(*p, 1e-6, *[ws] * 6, 1e-5, ws, ws, 1, 1, 1024, 2, 256, ws,
                                    None) == _lib.ERR_UNSUPPORTED


def test_attention_entry_rejects_bad_arguments():
    lib = _lib.load()
    ws = ctypes.create_string_buffer(64)
    out = ctypes.create_string_buffer(64)

    def call(width, heads, hidden, cap, dst):
        return lib.cow_attention_mlp_decode(ws, ws, ws, ws, 1e-5, ws, ws, ws, ws, cap, ws, ws, 1e-5, ws, ws, 1,
                                            width, heads, hidden, dst, None)
    assert call(64, 2, 256, 8, None) == _lib.ERR_INVALID  # missing output
    assert call(64, 3, 256, 8, out) == _lib.ERR_INVALID  # width not a multiple of heads
    assert call(64, 2, 256, 0, out) == _lib.ERR_INVALID  # empty cache
    assert call(64, 2, 256, 8, ws) == _lib.ERR_INVALID  # output aliasing the residual input
    assert call(1024, 2, 256, 8, out) == _lib.ERR_UNSUPPORTED  # wider than the compiled kernel
    assert call(128, 4, 512, 1 << 20, out) == _lib.ERR_UNSUPPORTED  # scores beyond shared memory


def test_growth_in_place_and_piped_step_reject_bad_arguments():
    lib = _lib.load()
    ws = ctypes.create_string_buffer(64)
    # a shrinking, negative or missing-buffer growth is rejected before any launch
    assert lib.cow_grow_in_place(ws, 8, 4, ws, ws, None) == _lib.ERR_INVALID
    assert lib.cow_grow_in_place(ws, -1, 4, ws, ws, None) == _lib.ERR_INVALID
    assert lib.cow_grow_in_place(None, 4, 8, ws, ws, None) == _lib.ERR_INVALID
    assert lib.cow_grow_in_place(ws, 4, 8, None, ws, None) == _lib.ERR_INVALID
    assert lib.cow_grow_in_place(ws, 4, 1 << 32, ws, ws, None) == _lib.ERR_INVALID
    # no descriptor, and a descriptor without buffers or events
    assert lib.cow_decode_step_host_piped(None, ws, None) == _lib.ERR_INVALID
    desc = _lib.CowHostPipeline()
    assert lib.cow_decode_step_host_piped(ctypes.addressof(desc), ws, None) == _lib.ERR_INVALID
