"""B200-native packed copy-on-write Sparse Delta Memory serving.

Drop-in for the reference's ``copy_on_write_sdm`` serving path: the same
``PackedSDMCopyOnWriteState`` / ``packed_sdm_cow_step`` /
``dense_sdm_sparse_step`` API, backed by hand-written sm_100a CUDA kernels in
``libcowsdm.so`` (C ABI: ``include/cow_sdm.h``).  There is no CPU or Triton
path: operations on CPU tensors raise.
"""

from .allocator import (
    PackedSDMCopyOnWriteState,
    SDMCopyOnWriteStep,
    dense_sdm_sparse_step,
    dense_sdm_sparse_step_layers,
    packed_sdm_cow_step,
    packed_sdm_cow_step_layers,
)
from .session import DecodeSession

__all__ = [
    "DecodeSession",
    "PackedSDMCopyOnWriteState",
    "SDMCopyOnWriteStep",
    "dense_sdm_sparse_step",
    "dense_sdm_sparse_step_layers",
    "packed_sdm_cow_step",
    "packed_sdm_cow_step_layers",
]
