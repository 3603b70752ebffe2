"""ctypes binding of ``libcowsdm.so`` (the C ABI declared in ``include/cow_sdm.h``).

There is no CPU fallback: if the library is missing or a CUDA device is not
available, every operation raises.  Tensors cross the boundary as raw
pointers; the library never allocates (torch's caching allocator owns every
buffer) and never synchronises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_int32, c_int64, c_void_p

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcowsdm.so")

# return codes / dtype codes / status bits (mirrors include/cow_sdm.h)
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE, ERR_SCRATCH_LIMIT = 0, 1, 2, 3, 4, 5
NOALLOC_SCRATCH_BYTES = 1 << 20
F32, BF16, F16 = 0, 1, 2
I32, I64 = 0, 1
ST_SLAB_EXHAUSTED = 0x1
ST_INDEX_RANGE = 0x2
ST_DUPLICATE_WRITE = 0x4
ST_WAIT_TIMEOUT = 0x8
ST_TEMPLATE_RANGE = 0x10
ST_BAD_BANK_LIST = 0x20
ST_DISCARD_LIVE = 0x40
ST_MULTI_OWNER = 0x100
ST_FREE_DUPLICATE = 0x200
ST_NOT_COVERED = 0x400
ST_ROW_RANGE = 0x800
ST_MAP_FULL = 0x1000
MAP_DENSE, MAP_HASH = 0, 1
MAX_LAYERS, MAX_WRITES, MAX_READS, MAX_WIDTH = 8, 32, 256, 512

_DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
_INDEX_CODE = {torch.int32: I32, torch.int64: I64}


class CowPool(ctypes.Structure):
    _fields_ = [
        ("m0", c_void_p),
        ("templates", c_void_p),
        ("slab", c_void_p),
        ("map", c_void_p),
        ("free_rows", c_void_p),
        ("free_count", c_void_p),
        ("status", c_void_p),
        ("banks", c_int64),
        ("slots", c_int64),
        ("width", c_int64),
        ("capacity", c_int64),
        ("template_count", c_int64),
        ("slab_dtype", c_int32),
        ("map_kind", c_int32),
        ("table_slots", c_int64),
        ("free_mirror", c_void_p),
    ]


class CowStep(ctypes.Structure):
    _fields_ = [
        ("write_indices", c_void_p),
        ("write_weights", c_void_p),
        ("values", c_void_p),
        ("input_gate", c_void_p),
        ("erase_gate", c_void_p),
        ("forget_log_gate", c_void_p),
        ("read_indices", c_void_p),
        ("read_weights", c_void_p),
        ("output", c_void_p),
        ("first_touch", c_void_p),
    ]


class CowHostPipeline(ctypes.Structure):
    _fields_ = [
        ("pools", POINTER(CowPool)),
        ("steps", POINTER(CowStep)),
        ("layers", c_int32),
        ("writes", c_int32),
        ("reads", c_int32),
        ("index_dtype", c_int32),
        ("act_dtype", c_int32),
        ("_pad", c_int32),
        ("scan_scratch", c_void_p),
        ("scratch_bytes", c_int64),
        ("device_inputs", c_void_p),
        ("input_bytes", c_int64),
        ("host_outputs", c_void_p),
        ("device_outputs", c_void_p),
        ("output_bytes", c_int64),
        ("h2d_stream", c_void_p),
        ("d2h_stream", c_void_p),
        ("h2d_done", c_void_p),
        ("computed", c_void_p),
        ("d2h_done", c_void_p),
    ]


P = c_void_p
_SIGNATURES = {
    "cow_abi_version": (c_int32, []),
    "cow_last_error": (c_char_p, []),
    "cow_decode_scratch_bytes": (c_int64, [c_int64, c_int32]),
    "cow_decode_step": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int32, c_int32,
                                  c_int32, c_int32, P, c_int64, P]),
    "cow_decode_step_checked": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int32, c_int32,
                                          c_int32, c_int32, P, c_int64, P, POINTER(c_int32)]),
    "cow_decode_step_noalloc": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int32, c_int32,
                                          c_int32, c_int32, P]),
    "cow_decode_step_host": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int32, c_int32, c_int32,
                                       c_int32, P, c_int64, P, P, c_int64, P, P, c_int64, P]),
    "cow_decode_step_host_piped": (c_int32, [P, P, P]),
    "cow_decode_step_host_mapped": (c_int32, [P, P, P, P]),
    "cow_register_host_range": (c_int32, [P, c_int64]),
    "cow_hash_from_dense": (c_int32, [P, c_int64, c_int64, P, c_int64, P, P]),
    "cow_hash_to_dense": (c_int32, [P, c_int64, c_int64, P, c_int64, P, P]),
    "cow_hash_max_live": (c_int32, [P, c_int64, c_int64, P, P]),
    "cow_unregister_host_range": (c_int32, [P]),
    "cow_decode_step_host_overlapped": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int32, c_int32,
                                                  c_int32, c_int32, P, c_int64, P, P, c_int64, P, P, c_int64,
                                                  P, P, P, P, P, P]),
    "cow_dense_step": (c_int32, [POINTER(c_void_p), POINTER(c_int64), POINTER(CowStep), c_int32,
                                 c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, P]),
    "cow_init_pool": (c_int32, [POINTER(CowPool), P]),
    "cow_scan_blocks": (c_int64, [c_int64]),
    "cow_prefill_mark": (c_int32, [P, c_int32, c_int64, c_int64, c_int32, c_int64, P, P, P]),
    "cow_mask_to_map": (c_int32, [P, c_int64, P, P]),
    "cow_pack_count": (c_int32, [P, c_int64, P, P]),
    "cow_pack_apply": (c_int32, [P, c_int64, P, POINTER(CowPool), P, P]),
    "cow_copy_rows": (c_int32, [P, c_int32, P, P, c_int32, P, c_int64, c_int64, c_int32, P, P,
                                c_int64, P]),
    "cow_prefill_recurrence": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int64, c_int32,
                                         c_int32, c_int32, c_int32, P]),
    "cow_prefill_recurrence_layers": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int64, c_int32,
                                                c_int32, c_int32, c_int32, P]),
    "cow_prefill_workspace_bytes": (c_int64, [POINTER(CowPool), c_int32, c_int64, c_int32, c_int32]),
    "cow_prefill_recurrence_layers_ws": (c_int32, [POINTER(CowPool), POINTER(CowStep), c_int32, c_int64, c_int32,
                                                   c_int32, c_int32, c_int32, P, c_int64, P]),
    "cow_grow": (c_int32, [P, P, c_int64, P, P, c_int64, c_int64, c_int32, P, P, P]),
    "cow_grow_in_place": (c_int32, [P, c_int64, c_int64, P, P, P]),
    "cow_release": (c_int32, [POINTER(CowPool), P, c_int64, P, P, P, P]),
    "cow_repack": (c_int32, [POINTER(CowPool), P, P, P, c_int64, P, P, P]),
    "cow_append": (c_int32, [POINTER(CowPool), POINTER(CowPool), P, P, P, P, P]),
    "cow_retain": (c_int32, [POINTER(CowPool), P, c_int64, P, P, P, P, P]),
    "cow_validate": (c_int32, [POINTER(CowPool), P, P, P]),
    "cow_materialize": (c_int32, [POINTER(CowPool), P, c_int32, P]),
    "cow_controller_step": (c_int32, [P, P, P, ctypes.c_float, P, P, P, P, c_int64, c_int64, c_int32, c_int32,
                                      c_int32, c_int32, c_int32, P, P, P, P, P, P, P, P, P]),
    "cow_readout_mlp_step": (c_int32, [P, P, P, P, P, ctypes.c_float, P, P, P, P, P, P, ctypes.c_float, P, P,
                                       c_int64, c_int64, c_int32, c_int32, c_int32, P, P]),
    "cow_attention_mlp_decode": (c_int32, [P, P, P, P, ctypes.c_float, P, P, P, P, c_int64, P, P, ctypes.c_float,
                                           P, P, c_int64, c_int32, c_int32, c_int32, P, P]),
    "cow_route_controller": (c_int32, [P, P, P, P, P, P, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32,
                                       P, P, P, P, P, P, P]),
    "cow_release_workspace_bytes": (c_int64, [POINTER(CowPool), P, c_int32]),
    "cow_release_layers": (c_int32, [POINTER(CowPool), P, P, c_int32, P, c_int64, P, P]),
    "cow_retain_workspace_bytes": (c_int64, [POINTER(CowPool), c_int32]),
    "cow_retain_layers": (c_int32, [POINTER(CowPool), P, P, c_int32, P, P, P, c_int64, P, P]),
    "cow_append_workspace_bytes": (c_int64, [POINTER(CowPool), c_int32]),
    "cow_append_count_layers": (c_int32, [POINTER(CowPool), POINTER(CowPool), c_int32, P, c_int64, P, P]),
    "cow_append_layers": (c_int32, [POINTER(CowPool), POINTER(CowPool), c_int32, P, P, c_int64, P]),
    "cow_pack_workspace_bytes": (c_int64, [c_int64, c_int32]),
    "cow_prefill_mark_count_layers": (c_int32, [P, P, c_int32, c_int64, c_int64, c_int32, c_int32, c_int64, P,
                                                c_int32, P, c_int64, P, P]),
    "cow_pack_apply_layers": (c_int32, [POINTER(CowPool), c_int32, P, c_int64, P]),
    "cow_admit_prefix_workspace_bytes": (c_int64, [c_int64, c_int64, c_int32]),
    "cow_admit_prefix_layers": (c_int32, [POINTER(CowPool), P, P, c_int64, c_int32, P, P, c_int64, P]),
    "cow_validate_workspace_bytes": (c_int64, [POINTER(CowPool), c_int32]),
    "cow_validate_layers": (c_int32, [POINTER(CowPool), c_int32, P, c_int64, P, P]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library (once).  Raises if it was never built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m copy_on_write_sdm_b200._build` "
                "(this package has no CPU or Triton fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    if rc in (ERR_INVALID, ERR_UNSUPPORTED):
        kind = "invalid argument" if rc == ERR_INVALID else "unsupported shape"
        raise ValueError(f"{what}: {kind} (libcowsdm code {rc})")
    if rc == ERR_SCRATCH_LIMIT:
        raise ValueError(f"{what}: more banks than the fixed no-alloc scratch holds "
                         f"({NOALLOC_SCRATCH_BYTES} bytes); use the scratch-taking entry point")
    if rc == ERR_CUDA:
        msg = load().cow_last_error().decode()
        raise RuntimeError(f"{what}: CUDA error: {msg}")
    raise RuntimeError(f"{what}: libcowsdm error {rc}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"unsupported floating dtype {dtype}") from None


def index_code(dtype: torch.dtype) -> int:
    try:
        return _INDEX_CODE[dtype]
    except KeyError:
        raise ValueError(f"unsupported index dtype {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(
            f"{what} must be a CUDA tensor: the packed copy-on-write SDM path runs only "
            "through the sm_100a kernels (no CPU fallback)"
        )


_STATUS_TEXT = [
    (ST_SLAB_EXHAUSTED, "SDM COW physical slab is exhausted"),
    (ST_INDEX_RANGE, "SDM route index lies outside the logical table"),
    (ST_DUPLICATE_WRITE, "one SDM step cannot write one logical slot twice"),
    (ST_WAIT_TIMEOUT, "a bounded inter-block wait in the decode scan gave up"),
    (ST_TEMPLATE_RANGE, "template index lies outside shared initial memory"),
    (ST_BAD_BANK_LIST, "released bank index is invalid or duplicated"),
    (ST_DISCARD_LIVE, "discarded SDM banks must be released before compaction"),
    (ST_MULTI_OWNER, "one physical SDM row has multiple logical owners"),
    (ST_FREE_DUPLICATE, "free SDM row stack contains duplicates"),
    (ST_MAP_FULL, "a hashed SDM map table has no room for a first touch"),
    (ST_NOT_COVERED, "active and free SDM rows do not partition the slab"),
    (ST_ROW_RANGE, "active and free SDM rows do not partition the slab"),
]


def status_text(bits: int) -> str:
    return "; ".join(text for bit, text in _STATUS_TEXT if bits & bit) or "ok"
