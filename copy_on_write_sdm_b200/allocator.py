"""Packed copy-on-write SDM state on B200: the drop-in for the reference's allocator.

Public surface (same names, arguments, errors and tensor fields as the
reference's ``copy_on_write_sdm/allocator.py``):

* ``PackedSDMCopyOnWriteState`` (allocator.py:477-1096): ``allocate``,
  ``from_dense_overlay``, ``grow_capacity``, ``prepare_step_capacity``,
  ``trim_capacity``, ``append_banks_from``, ``retain_banks``, ``release``,
  ``materialize_dense``, ``allocated_rows_tensor``, ``storage_bytes``,
  ``used_bytes``, ``validate_invariants``; plus the sparse prefill handoff
  ``from_prefix_routes`` that replaces the dense ``[B,T,N,D]`` recurrence;
* ``packed_sdm_cow_step`` (allocator.py:1382-1526) and
  ``dense_sdm_sparse_step`` (allocator.py:1529-1633);
* ``packed_sdm_cow_step_layers`` / ``dense_sdm_sparse_step_layers``: one launch
  for several independent pools (the synthetic multi-layer screen).

Every device operation runs through ``libcowsdm.so`` (sm_100a).  The state's
``overflow_flag`` is the library's 32-bit status word: 0 means healthy, any
set bit is an error that ``validate_invariants`` (and every checked call)
turns into the reference's exception.  Row-placement order is the
reference's deterministic CPU order, so maps and free stacks are bit-exact.
"""

from __future__ import annotations

import contextlib
import ctypes
import math
import os
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from . import _lib

_BACKENDS = ("auto", "cuda", "triton")


def _tensor_bytes(tensor: torch.Tensor) -> int:
    return tensor.numel() * tensor.element_size()


@dataclass(frozen=True)
class SDMCopyOnWriteStep:
    """Diagnostics for one packed SDM decode step (allocator.py:468-474)."""

    first_touches_by_sequence: torch.Tensor
    repeated_writes_by_sequence: torch.Tensor
    allocated_rows_after_step: torch.Tensor


# --------------------------------------------------------------------------
# per-device scratch (scan flags of the decode step, lifecycle scratch)
# --------------------------------------------------------------------------

_DECODE_SCRATCH: dict[int, torch.Tensor] = {}
# Buffers that decode_scratch replaced.  A CUDA graph that captured a decode
# launch keeps the scratch address it was captured with, so a replaced buffer
# must never go back to the caching allocator: it stays here for the life of
# the process (a few KB to a few MB per device in all).
_RETIRED_DECODE_SCRATCH: list[torch.Tensor] = []
_M0_CACHE: dict[tuple, torch.Tensor] = {}


def decode_scratch(device: torch.device, total_banks: int, layers: int) -> torch.Tensor:
    """Zero-initialised look-back scratch of the fused decode step, one per device.

    Every decode launch tags its scan flags with one launch epoch and advances
    it once all its pools are closed, so one buffer serves any sequence of
    launches on one stream, whatever their pool layouts, including launches
    captured in CUDA graphs.  When a larger launch needs more bytes the buffer
    is replaced (at least doubling) and the old one is kept alive, so graphs
    that captured it stay valid.  Decode launches that could overlap on the
    GPU (different streams) must pass their own ``scratch=`` buffer.
    """
    need = int(_lib.load().cow_decode_scratch_bytes(total_banks, layers))
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _DECODE_SCRATCH.get(key)
    if buf is None or buf.numel() < need:
        size = max(need, 4096, 0 if buf is None else 2 * buf.numel())
        if buf is not None:
            _RETIRED_DECODE_SCRATCH.append(buf)
        buf = torch.zeros(size, dtype=torch.uint8, device=device)
        _DECODE_SCRATCH[key] = buf
    return buf


def new_decode_scratch(device: torch.device, total_banks: int, layers: int) -> torch.Tensor:
    """A private zero-filled decode scratch buffer for one owner (a session or
    a captured graph), sized for ``layers`` pools of ``total_banks`` banks."""
    need = int(_lib.load().cow_decode_scratch_bytes(total_banks, layers))
    return torch.zeros(max(need, 4096), dtype=torch.uint8, device=device)


def _scan_scratch(device: torch.device, n: int) -> torch.Tensor:
    blocks = int(_lib.load().cow_scan_blocks(n))
    return torch.zeros(blocks + 8, dtype=torch.int32, device=device)


@contextlib.contextmanager
def dense_maps(states: Sequence[PackedSDMCopyOnWriteState]):
    """Lifecycle operations work on the dense map: hashed pools among ``states``
    are expanded for the duration and hashed again afterwards (tables of at
    least their previous size, larger if a bank now holds more slots)."""
    hashed = [(st, st.map_table_slots) for st in states if st.map_table_slots]
    for st, _ in hashed:
        st.use_dense_map()
    try:
        yield
    finally:
        for st, t in hashed:
            live = int((st.logical_to_physical >= 0).sum(dim=1).max()) if st.banks else 0
            st.use_hash_map(max(t, st._table_slots_for(live)))


def _on_dense_maps(pick):
    """Run a lifecycle operation with the hashed pools that ``pick(args)`` names
    expanded to dense maps."""
    def wrap(fn):
        def inner(*args, **kwargs):
            states = pick(*args, **kwargs)
            if not any(st.map_table_slots for st in states):
                return fn(*args, **kwargs)
            with dense_maps(states):
                return fn(*args, **kwargs)
        inner.__name__, inner.__doc__, inner.__wrapped__ = fn.__name__, fn.__doc__, fn
        return inner
    return wrap


# --------------------------------------------------------------------------
# the state
# --------------------------------------------------------------------------


# Process-wide counters of pool assignments: [any field, tensor fields].  A
# runtime that caches proofs or descriptors over a set of pools compares one
# integer per step instead of one counter per pool (a change to any pool
# anywhere invalidates its cache, which is conservative).
POOL_EPOCHS = [0, 0]

_TENSOR_FIELDS = frozenset({"shared_initial_memory", "template_indices", "values", "logical_to_physical",
                            "free_rows", "free_count", "overflow_flag", "_m0_f32"})


@dataclass
class PackedSDMCopyOnWriteState:
    """One shared slab backing several independent logical SDM tables.

    Fields and meaning follow the reference (allocator.py:477-505):
    ``shared_initial_memory [H,N,D]`` (``M0``), ``template_indices [banks]``,
    ``values [C,D]`` (the pooled slab), ``logical_to_physical [banks,N]``
    (int32, -1 = shared), ``free_rows [C]`` (int32 stack), ``free_count`` and
    ``overflow_flag`` (0-d int32; here the library's status bit word).
    """

    shared_initial_memory: torch.Tensor
    template_indices: torch.Tensor
    values: torch.Tensor
    logical_to_physical: torch.Tensor
    free_rows: torch.Tensor
    free_count: torch.Tensor
    overflow_flag: torch.Tensor
    capacity_is_proven: bool = False
    proven_maximum_additional_allocations: int = 0
    growth_quantum_rows: int = 0
    growth_events: int = 0
    growth_rows_added: int = 0
    growth_rows_copied: int = 0
    slab_rows_moved: int = 0
    # Hashed logical map (not in the reference): when map_table_slots > 0,
    # logical_to_physical holds [banks, map_table_slots] int64 open-addressing
    # tables ((slot << 32) | row, -1 empty) and hashed_slots is N.
    map_table_slots: int = 0
    hashed_slots: int = 0
    _m0_f32: torch.Tensor | None = field(default=None, repr=False, compare=False)

    def __setattr__(self, name: str, value) -> None:
        # Caches in DecodeSession and GraphedDecode compare these counters: one
        # counts replaced tensors (descriptors), one every assignment (proofs).
        object.__setattr__(self, name, value)
        d = self.__dict__
        d["_mutations"] = d.get("_mutations", 0) + 1
        POOL_EPOCHS[0] += 1
        if name in _TENSOR_FIELDS:
            d["_tensor_version"] = d.get("_tensor_version", 0) + 1
            POOL_EPOCHS[1] += 1
            # a slab or stack replaced other than by growth releases the growth reserve
            store = d.get("_slab_store")
            if store is not None and name in ("values", "free_rows") \
                    and value.data_ptr() != store[0 if name == "values" else 1].data_ptr():
                del d["_slab_store"]

    # ---------------- construction ----------------

    @staticmethod
    def _normalise_m0(shared_initial_memory: torch.Tensor) -> torch.Tensor:
        if shared_initial_memory.ndim == 2:
            shared_initial_memory = shared_initial_memory.unsqueeze(0)
        if shared_initial_memory.ndim != 3:
            raise ValueError("shared initial memory must be [H,N,D] or [N,D]")
        return shared_initial_memory

    @staticmethod
    def _m0_float(m0: torch.Tensor) -> torch.Tensor:
        # The kernels read M0 as float32; bf16/fp16 -> fp32 is exact, so the
        # arithmetic equals the reference's ``M0[...].float()``.  One copy is
        # shared by every pool built from the same (unmodified) parameter.
        if m0.dtype == torch.float32 and m0.is_contiguous() and m0.data_ptr() % 16 == 0:
            return m0
        key = (m0.data_ptr(), m0._version, m0.dtype, tuple(m0.shape), str(m0.device))
        hit = _M0_CACHE.get(key)
        if hit is None:
            if len(_M0_CACHE) >= 64:
                _M0_CACHE.pop(next(iter(_M0_CACHE)))
            hit = _M0_CACHE[key] = m0.detach().float().contiguous().clone()
        return hit

    @classmethod
    def allocate(
        cls,
        shared_initial_memory: torch.Tensor,
        *,
        banks: int,
        capacity_rows: int,
        template_indices: torch.Tensor | None = None,
        state_dtype: torch.dtype = torch.float32,
        growth_quantum_rows: int = 0,
    ) -> "PackedSDMCopyOnWriteState":
        """Allocate an empty shared slab (allocator.py:507-586)."""

        shared_initial_memory = cls._normalise_m0(shared_initial_memory)
        templates, slots, width = shared_initial_memory.shape
        if banks <= 0 or capacity_rows <= 0:
            raise ValueError("banks and physical capacity must be positive")
        if growth_quantum_rows < 0:
            raise ValueError("SDM growth quantum cannot be negative")
        if state_dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError("SDM COW state must use float16, bfloat16, or float32")
        device = shared_initial_memory.device
        _lib.require_cuda(shared_initial_memory, "shared initial memory")
        if template_indices is None:
            if templates != 1:
                raise ValueError("multiple initial-memory templates require explicit mapping")
            template_indices = torch.zeros(banks, device=device, dtype=torch.int64)
        elif (
            template_indices.shape != (banks,)
            or template_indices.dtype not in (torch.int32, torch.int64)
            or template_indices.device != device
        ):
            raise ValueError("template indices must be integer [B] on the state device")
        else:
            template_indices = template_indices.to(torch.int64)
        lo, hi = torch.aminmax(template_indices)
        if int(lo) < 0 or int(hi) >= templates:
            raise ValueError("template index lies outside shared initial memory")
        return cls._empty(
            shared_initial_memory,
            template_indices.contiguous(),
            banks=banks,
            capacity_rows=capacity_rows,
            state_dtype=state_dtype,
            growth_quantum_rows=growth_quantum_rows,
            init=True,
        )

    @classmethod
    def _empty(cls, m0, templates, *, banks, capacity_rows, state_dtype, growth_quantum_rows, init,
               m0_f32=None, mapping=None):
        device = m0.device
        _, slots, width = m0.shape
        state = cls(
            shared_initial_memory=m0,
            template_indices=templates,
            values=torch.empty(capacity_rows, width, device=device, dtype=state_dtype),
            logical_to_physical=(mapping if mapping is not None
                                 else torch.empty(banks, slots, device=device, dtype=torch.int32)),
            free_rows=torch.empty(capacity_rows, device=device, dtype=torch.int32),
            free_count=torch.empty((), device=device, dtype=torch.int32),
            overflow_flag=torch.zeros((), device=device, dtype=torch.int32),
            growth_quantum_rows=growth_quantum_rows,
            _m0_f32=m0_f32 if m0_f32 is not None else cls._m0_float(m0),
        )
        if init:
            state._call("cow_init_pool", ctypes.byref(state._pool()), state._stream())
        return state

    @classmethod
    @torch.no_grad()
    def from_dense_overlay(
        cls,
        shared_initial_memory: torch.Tensor,
        dense_memory: torch.Tensor,
        active_slots: torch.Tensor,
        *,
        template_indices: torch.Tensor,
        capacity_rows: int | None = None,
        state_dtype: torch.dtype = torch.float32,
        maximum_future_allocations: int | None = None,
        growth_quantum_rows: int = 0,
    ) -> "PackedSDMCopyOnWriteState":
        """Pack an exact full-prefix state into a first-write overlay (allocator.py:589-690).

        Active rows take physical rows ``0..A-1`` in ``nonzero()`` order; the
        free stack is ``arange(A, C)``.
        """

        shared_initial_memory = cls._normalise_m0(shared_initial_memory)
        if dense_memory.ndim != 3:
            raise ValueError("SDM handoff memory must be [H,N,D] and [B,N,D]")
        banks, slots, width = dense_memory.shape
        if (
            active_slots.shape != (banks, slots)
            or active_slots.dtype != torch.bool
            or active_slots.device != dense_memory.device
            or shared_initial_memory.device != dense_memory.device
            or shared_initial_memory.shape[1:] != (slots, width)
        ):
            raise ValueError("SDM handoff state and active-slot mask do not align")
        if template_indices.shape != (banks,) or template_indices.device != dense_memory.device:
            raise ValueError("SDM handoff template indices must be [B] on device")
        _lib.require_cuda(dense_memory, "dense SDM memory")
        if growth_quantum_rows < 0:
            raise ValueError("SDM growth quantum cannot be negative")
        lib = _lib.load()
        device = dense_memory.device
        stream = _lib.stream_of(device)
        mapping = torch.empty(banks, slots, device=device, dtype=torch.int32)
        active = active_slots.contiguous()
        _lib.check(lib.cow_mask_to_map(active.data_ptr(), active.numel(), mapping.data_ptr(), stream),
                   "cow_mask_to_map")
        return cls._pack_layout(
            shared_initial_memory, mapping, template_indices,
            capacity_rows=capacity_rows, state_dtype=state_dtype,
            maximum_future_allocations=maximum_future_allocations,
            growth_quantum_rows=growth_quantum_rows,
            row_source=("dense", dense_memory.contiguous()),
        )

    @classmethod
    @torch.no_grad()
    def from_prefix_routes(
        cls,
        shared_initial_memory: torch.Tensor,
        write_indices: torch.Tensor,
        write_weights: torch.Tensor,
        values: torch.Tensor,
        input_gate: torch.Tensor,
        forget_log_gate: torch.Tensor,
        read_indices: torch.Tensor,
        read_weights: torch.Tensor,
        *,
        template_indices: torch.Tensor,
        erase_gate: torch.Tensor | None = None,
        capacity_rows: int | None = None,
        state_dtype: torch.dtype = torch.float32,
        maximum_future_allocations: int | None = None,
        growth_quantum_rows: int = 0,
    ) -> tuple["PackedSDMCopyOnWriteState", torch.Tensor]:
        """Sparse prefill handoff: run the prefix recurrence on written rows only.

        Inputs are per bank and token: indices/weights ``[banks,T,W|R]``,
        values ``[banks,T,D]``, gates ``[banks,T]``.  The reference computes
        the dense terminal table with the full recurrence (sdm.py:1174-1199,
        storing ``[B,T,N,D]``) and packs its hard-write union with
        ``from_dense_overlay`` (inference.py:314-366).  A slot no prefix token
        writes never leaves ``M0``, so the packed layout is built first (rows
        ``0..A-1`` in ``nonzero()`` order, filled from ``M0``) and the
        recurrence then runs in place on those rows.  Returns the state and
        the prefix readings ``[banks,T,D]`` (the reference's readings).
        """

        states, readings = from_prefix_routes_layers(
            [shared_initial_memory],
            [dict(write_indices=write_indices, write_weights=write_weights, values=values,
                  input_gate=input_gate, forget_log_gate=forget_log_gate, read_indices=read_indices,
                  read_weights=read_weights, erase_gate=erase_gate)],
            template_indices=template_indices, capacity_rows=capacity_rows, state_dtype=state_dtype,
            maximum_future_allocations=maximum_future_allocations,
            growth_quantum_rows=growth_quantum_rows)
        return states[0], readings[0]

    @classmethod
    def _pack_layout(cls, m0, mapping, template_indices, *, capacity_rows, state_dtype,
                     maximum_future_allocations, growth_quantum_rows, row_source, validate=True):
        """nonzero()-order layout of ``mapping >= 0`` (allocator.py:624-689)."""
        device = mapping.device
        scan = _scan_scratch(device, mapping.numel())
        _lib.check(_lib.load().cow_pack_count(mapping.data_ptr(), mapping.numel(), scan.data_ptr(),
                                              _lib.stream_of(device)), "cow_pack_count")
        templates = template_indices.to(torch.int64).contiguous()
        active_count, lo, hi = _read_counts_and_range([scan[0]], templates)
        _check_template_range(lo, hi, m0)
        state = cls._pack_finish(m0, mapping, templates, scan, active_count[0], capacity_rows=capacity_rows,
                                 state_dtype=state_dtype, maximum_future_allocations=maximum_future_allocations,
                                 growth_quantum_rows=growth_quantum_rows, row_source=row_source)
        if validate:
            state.validate_invariants()
        return state

    @classmethod
    def _pack_state(cls, m0, mapping, templates, active_count, *, capacity_rows, state_dtype,
                    maximum_future_allocations, growth_quantum_rows):
        """Capacity choice and tensors of a packed pool holding ``active_count`` live
        rows (allocator.py:624-689); the caller fills map, stack and rows."""
        banks, slots = mapping.shape
        if capacity_rows is None and growth_quantum_rows:
            q = growth_quantum_rows
            selected = max(q, ((active_count + q - 1) // q) * q)
        else:
            selected = banks * slots if capacity_rows is None else capacity_rows
        if selected < active_count:
            raise ValueError("SDM physical capacity is smaller than the prefill working set")
        if maximum_future_allocations is not None:
            if maximum_future_allocations < 0:
                raise ValueError("maximum future allocations cannot be negative")
            possible = min(maximum_future_allocations, banks * slots - active_count)
            if selected - active_count < possible:
                raise ValueError("SDM physical capacity cannot cover the declared decode trace")
        else:
            possible = 0
        state = cls._empty(m0, templates, banks=banks, capacity_rows=selected,
                           state_dtype=state_dtype, growth_quantum_rows=growth_quantum_rows,
                           init=False, mapping=mapping)
        state.capacity_is_proven = maximum_future_allocations is not None
        state.proven_maximum_additional_allocations = possible
        return state

    @classmethod
    def _pack_finish(cls, m0, mapping, templates, scan, active_count, *, capacity_rows, state_dtype,
                     maximum_future_allocations, growth_quantum_rows, row_source):
        """Size and build the packed pool once ``cow_pack_count`` has run on ``mapping``."""
        lib = _lib.load()
        device = mapping.device
        stream = _lib.stream_of(device)
        banks, slots = mapping.shape
        n = banks * slots
        state = cls._pack_state(m0, mapping, templates, active_count, capacity_rows=capacity_rows,
                                state_dtype=state_dtype, maximum_future_allocations=maximum_future_allocations,
                                growth_quantum_rows=growth_quantum_rows)
        src_index = torch.empty(max(active_count, 1), device=device, dtype=torch.int32)
        pool = state._pool()
        _lib.check(lib.cow_pack_apply(mapping.data_ptr(), n, src_index.data_ptr(), ctypes.byref(pool),
                                      scan.data_ptr(), stream), "cow_pack_apply")
        kind, source = row_source
        sdt = _lib.dtype_code(state_dtype)
        if active_count:
            if kind == "dense":
                _lib.check(lib.cow_copy_rows(state.values.data_ptr(), sdt, None, source.data_ptr(),
                                             _lib.dtype_code(source.dtype), src_index.data_ptr(),
                                             active_count, m0.shape[2], 0, None, None, slots, stream),
                           "cow_copy_rows")
            else:
                _lib.check(lib.cow_copy_rows(state.values.data_ptr(), sdt, None, None, 0,
                                             src_index.data_ptr(), active_count, m0.shape[2], 1,
                                             state._m0_f32.data_ptr(), templates.data_ptr(), slots,
                                             stream), "cow_copy_rows")
        return state

    # ---------------- plumbing ----------------

    def _stream(self) -> int:
        return _lib.stream_of(self.values.device)

    def _pool(self) -> _lib.CowPool:
        m0 = self._m0_f32
        return _lib.CowPool(
            m0.data_ptr(), self.template_indices.data_ptr(), self.values.data_ptr(),
            self.logical_to_physical.data_ptr(), self.free_rows.data_ptr(),
            self.free_count.data_ptr(), self.overflow_flag.data_ptr(),
            self.banks, self.slots, self.width, self.capacity_rows, m0.shape[0],
            _lib.dtype_code(self.values.dtype), _lib.MAP_HASH if self.map_table_slots else _lib.MAP_DENSE,
            self.map_table_slots,
        )

    # ---------------- hashed logical map ----------------

    # Tables are sized so that no bank's table is more than this full.
    HASH_MAX_LOAD = 0.7

    @classmethod
    def _table_slots_for(cls, live: int) -> int:
        need = max(4, math.ceil(live / cls.HASH_MAX_LOAD))
        return 1 << (need - 1).bit_length()

    @torch.no_grad()
    def use_hash_map(self, table_slots: int | None = None, *, headroom_rows_per_bank: int = 0) -> int:
        """Replace the dense ``[banks, N]`` map by per-bank hashed tables (no
        counterpart in the reference, whose README names a sparse map as future
        work).  ``table_slots`` (a power of two) defaults to the smallest size
        that keeps every bank at most 70 % full with ``headroom_rows_per_bank``
        more rows.  Growth pools keep their tables within that load through
        ``prepare_step_capacity``; fixed pools must declare the rows a bank may
        still gain as headroom.  Decode reads the tables directly; lifecycle
        operations expand them to the dense map for their duration.  Returns
        the table size; synchronises once."""
        if headroom_rows_per_bank < 0:
            raise ValueError("hash map headroom cannot be negative")
        if self.map_table_slots:
            if table_slots is None or table_slots == self.map_table_slots:
                return self.map_table_slots
            self.use_dense_map()
        lib = _lib.load()
        mapping = self.logical_to_physical
        live = int((mapping >= 0).sum(dim=1).max()) if self.banks else 0
        t = table_slots if table_slots is not None else self._table_slots_for(live + headroom_rows_per_bank)
        if t < 4 or t & (t - 1) or t <= live:
            raise ValueError("hash map table size must be a power of two above the live slots of every bank")
        tables = torch.empty(self.banks, t, dtype=torch.int64, device=mapping.device)
        status = torch.zeros((), dtype=torch.int32, device=mapping.device)
        _lib.check(lib.cow_hash_from_dense(mapping.data_ptr(), self.banks, self.slots, tables.data_ptr(), t,
                                           status.data_ptr(), self._stream()), "cow_hash_from_dense")
        if int(status):
            raise RuntimeError(f"hash map build failed: {_lib.status_text(int(status))}")
        slots = self.slots
        self.hashed_slots = slots
        self.logical_to_physical = tables
        self.map_table_slots = t
        self.__dict__["_hash_live"] = live  # largest live count of a bank at the last exact count
        return t

    @torch.no_grad()
    def use_dense_map(self) -> None:
        """Expand hashed tables back to the reference's dense ``[banks, N]`` int32 map."""
        if not self.map_table_slots:
            return
        lib = _lib.load()
        tables = self.logical_to_physical
        mapping = torch.empty(self.banks, self.hashed_slots, dtype=torch.int32, device=tables.device)
        status = torch.zeros((), dtype=torch.int32, device=tables.device)
        _lib.check(lib.cow_hash_to_dense(tables.data_ptr(), self.banks, self.map_table_slots, mapping.data_ptr(),
                                         self.hashed_slots, status.data_ptr(), self._stream()), "cow_hash_to_dense")
        self.map_table_slots = 0
        self.logical_to_physical = mapping
        self.hashed_slots = 0
        if int(status):
            raise RuntimeError(f"hash map expansion failed: {_lib.status_text(int(status))}")

    def hash_max_live(self) -> int:
        """Largest number of private slots of any bank (hashed pools; synchronises)."""
        out = torch.empty((), dtype=torch.int32, device=self.values.device)
        self._call("cow_hash_max_live", self.logical_to_physical.data_ptr(), self.banks, self.map_table_slots,
                   out.data_ptr(), self._stream())
        return int(out)

    def _hash_room(self, per_bank: int) -> int:
        """Rows every bank may still gain within the load limit, after rehashing to
        larger tables when fewer than ``per_bank`` remain (hashed pools)."""
        limit = int(self.map_table_slots * self.HASH_MAX_LOAD)
        live = self.hash_max_live()
        if live + per_bank > limit:
            self.use_hash_map(self._table_slots_for(live + max(per_bank, live // 2)))
            limit = int(self.map_table_slots * self.HASH_MAX_LOAD)
        self.__dict__["_hash_live"] = live
        return limit - live

    @staticmethod
    def _call(name: str, *args) -> None:
        _lib.check(getattr(_lib.load(), name)(*args), name)

    # ---------------- lifecycle ----------------

    @torch.no_grad()
    def grow_capacity(self, minimum_capacity_rows: int) -> int:
        """Grow the slab by whole quanta; row IDs stay stable (allocator.py:692-744).

        The slab is stored with a reserve behind ``capacity_rows``, so most growths
        only extend the views and push the new row ids (``cow_grow_in_place``); the
        allocator state after each growth is the reference's.  ``growth_rows_copied``
        counts what the reference copies; ``slab_rows_moved`` what this one did."""

        if minimum_capacity_rows <= self.capacity_rows:
            return 0
        quantum = self.growth_quantum_rows
        if quantum <= 0:
            raise ValueError("SDM COW slab growth is disabled")
        selected = ((minimum_capacity_rows + quantum - 1) // quantum) * quantum
        old_capacity = self.capacity_rows
        added = selected - old_capacity
        store = self.__dict__.get("_slab_store")
        if (store is not None and store[0].data_ptr() == self.values.data_ptr()
                and store[1].data_ptr() == self.free_rows.data_ptr() and store[0].shape[0] >= selected):
            # Inside the reserve: the rows exist already; only their ids join the
            # free stack, in the order the copying growth gives them.
            self._call("cow_grow_in_place", self.free_rows.data_ptr(), old_capacity, selected,
                       self.free_count.data_ptr(), self.overflow_flag.data_ptr(), self._stream())
            self.values = store[0][:selected]
            self.free_rows = store[1][:selected]
        else:
            # A new slab with a reserve behind it (a quarter of the capacity, at most
            # 1 GiB of rows, at least one quantum), so that the following growths
            # copy nothing; old rows are copied once here.
            row_bytes = self.width * self.values.element_size()
            extra = max(quantum, min(selected // 4, (1 << 30) // max(row_bytes, 1)))
            reserve = selected + ((extra + quantum - 1) // quantum) * quantum
            device = self.values.device
            values = torch.empty(reserve, self.width, device=device, dtype=self.values.dtype)
            free_rows = torch.empty(reserve, device=device, dtype=self.free_rows.dtype)
            self._call("cow_grow", self.values.data_ptr(), self.free_rows.data_ptr(), old_capacity,
                       values.data_ptr(), free_rows.data_ptr(), selected, self.width,
                       _lib.dtype_code(self.values.dtype), self.free_count.data_ptr(),
                       self.overflow_flag.data_ptr(), self._stream())
            self.__dict__["_slab_store"] = (values, free_rows)
            self.values = values[:selected]
            self.free_rows = free_rows[:selected]
            self.slab_rows_moved += old_capacity
        self.proven_maximum_additional_allocations += added
        self.growth_events += 1
        self.growth_rows_added += added
        self.growth_rows_copied += old_capacity
        return added

    @torch.no_grad()
    def prepare_step_capacity(self, maximum_new_rows: int) -> int:
        """Pessimistic host-side proof for one fused step (allocator.py:746-774).

        Charges every possible W-way first touch until the next occasional
        ``free_count`` reconciliation, so the decode kernel never meets an
        empty free stack.
        """

        if maximum_new_rows < 0:
            raise ValueError("maximum new SDM rows cannot be negative")
        if self.growth_quantum_rows <= 0:
            if not self.capacity_is_proven:
                raise ValueError("SDM COW capacity has no decode proof")
            return 0
        if self.proven_maximum_additional_allocations < maximum_new_rows:
            free_rows = int(self.free_count.item())
            if free_rows < maximum_new_rows:
                self.grow_capacity(self.capacity_rows + maximum_new_rows - free_rows)
                free_rows = int(self.free_count.item())
            if self.map_table_slots and self.banks:
                # Hashed map: the proof also never covers more steps than the
                # fullest bank's table absorbs (one step adds at most
                # maximum_new_rows / banks rows to a bank).
                per_bank = -(-maximum_new_rows // self.banks)
                room = self._hash_room(per_bank)
                free_rows = min(free_rows, room // max(per_bank, 1) * maximum_new_rows)
            self.proven_maximum_additional_allocations = free_rows
        self.proven_maximum_additional_allocations -= maximum_new_rows
        self.capacity_is_proven = True
        return self.capacity_rows

    @torch.no_grad()
    @_on_dense_maps(lambda self, *_, **__: [self])
    def trim_capacity(self, *, headroom_rows: int = 0) -> int:
        """Repack live rows to ``0..A-1`` in ``nonzero()`` order (allocator.py:776-840)."""

        if headroom_rows < 0:
            raise ValueError("SDM trim headroom cannot be negative")
        quantum = self.growth_quantum_rows
        if quantum <= 0:
            raise ValueError("SDM COW slab trimming requires copy-on-write capacity")
        lib = _lib.load()
        stream = self._stream()
        device = self.values.device
        n = self.banks * self.slots
        scan = _scan_scratch(device, n)
        _lib.check(lib.cow_pack_count(self.logical_to_physical.data_ptr(), n, scan.data_ptr(), stream),
                   "cow_pack_count")
        active_count = int(scan[0])
        selected = max(quantum, ((active_count + headroom_rows + quantum - 1) // quantum) * quantum)
        if selected >= self.capacity_rows:
            return 0
        values = torch.empty(selected, self.width, device=device, dtype=self.values.dtype)
        mapping = torch.empty_like(self.logical_to_physical)
        free_rows = torch.empty(selected, device=device, dtype=self.free_rows.dtype)
        src_rows = torch.empty(max(active_count, 1), device=device, dtype=torch.int32)
        pool = self._pool()
        _lib.check(lib.cow_repack(ctypes.byref(pool), mapping.data_ptr(), values.data_ptr(),
                                  free_rows.data_ptr(), selected, src_rows.data_ptr(), scan.data_ptr(),
                                  stream), "cow_repack")
        sdt = _lib.dtype_code(self.values.dtype)
        if active_count:
            _lib.check(lib.cow_copy_rows(values.data_ptr(), sdt, None, self.values.data_ptr(), sdt,
                                         src_rows.data_ptr(), active_count, self.width, 0, None, None,
                                         self.slots, stream), "cow_copy_rows")
        removed = self.capacity_rows - selected
        self.values = values
        self.logical_to_physical = mapping
        self.free_rows = free_rows
        self.capacity_is_proven = False
        self.proven_maximum_additional_allocations = selected - active_count
        return removed

    @torch.no_grad()
    def append_banks_from(self, other: "PackedSDMCopyOnWriteState") -> int:
        """Admit another cohort's banks; copy only live rows (allocator.py:842-915)."""

        return append_layers([self], [other])[0]

    def _append_check(self, other: "PackedSDMCopyOnWriteState") -> None:
        if (
            other.slots != self.slots
            or other.width != self.width
            or other.values.device != self.values.device
            or other.values.dtype != self.values.dtype
            or other.shared_initial_memory.shape != self.shared_initial_memory.shape
        ):
            raise ValueError("admitted SDM banks do not match the destination pool")
        if (
            other.shared_initial_memory.data_ptr() != self.shared_initial_memory.data_ptr()
            and not torch.equal(other.shared_initial_memory, self.shared_initial_memory)
        ):
            raise ValueError("admitted SDM banks use different learned initial memory")

    def _append_commit(self, other: "PackedSDMCopyOnWriteState", admitted: torch.Tensor, active_count: int,
                       free_count: int) -> None:
        """Extend map and templates after the rows moved.  ``free_count`` is the
        free count the pop started from (after any growth)."""
        self.logical_to_physical = torch.cat((self.logical_to_physical, admitted), dim=0).contiguous()
        self.template_indices = torch.cat((self.template_indices, other.template_indices), dim=0).contiguous()
        if self.growth_quantum_rows:
            # free_count on the device is now free_count - active_count
            self.proven_maximum_additional_allocations = min(
                self.proven_maximum_additional_allocations, free_count - active_count
            )
        else:
            self.capacity_is_proven = False
            self.proven_maximum_additional_allocations = 0

    @torch.no_grad()
    def retain_banks(self, bank_indices: torch.Tensor) -> None:
        """Compact already-released banks; live rows do not move (allocator.py:917-943)."""

        retain_layers([self], [bank_indices])

    @staticmethod
    def _retain_check(bits: int) -> None:
        if bits & _lib.ST_BAD_BANK_LIST:
            raise ValueError("retained bank index is invalid or duplicated")
        if bits & _lib.ST_DISCARD_LIVE:
            raise ValueError("discarded SDM banks must be released before compaction")

    def _retain_commit(self, pending, bits: int) -> None:
        self._retain_check(bits)
        self.logical_to_physical, self.template_indices = pending[0], pending[1]

    @property
    def banks(self) -> int:
        return self.logical_to_physical.shape[0]

    @property
    def slots(self) -> int:
        return self.hashed_slots if self.map_table_slots else self.logical_to_physical.shape[1]

    @property
    def width(self) -> int:
        return self.values.shape[1]

    @property
    def capacity_rows(self) -> int:
        return self.values.shape[0]

    def allocated_rows_tensor(self) -> torch.Tensor:
        """Device-resident number of live physical rows (allocator.py:960-963)."""

        return self.free_count.new_tensor(self.capacity_rows) - self.free_count

    def storage_bytes(self) -> dict[str, int]:
        """Retained tensor storage, shared model state separate (allocator.py:965-982)."""

        private = {
            "value_slab_reserved": _tensor_bytes(self.values),
            "logical_to_physical": _tensor_bytes(self.logical_to_physical),
            "free_row_stack": _tensor_bytes(self.free_rows),
            "free_count": _tensor_bytes(self.free_count),
            "overflow_flag": _tensor_bytes(self.overflow_flag),
            "template_indices": _tensor_bytes(self.template_indices),
        }
        private["private_allocator_reserved_total"] = sum(private.values())
        shared = _tensor_bytes(self.shared_initial_memory)
        if self._m0_f32 is not None and self._m0_f32.data_ptr() != self.shared_initial_memory.data_ptr():
            # float32 copy of a bf16/fp16 M0 read by the kernels (shared, model-wide)
            shared += _tensor_bytes(self._m0_f32)
        private["shared_initial_memory"] = shared
        private["including_shared_initial_memory"] = private["private_allocator_reserved_total"] + shared
        return private

    def used_bytes(self) -> dict[str, int]:
        """Live-row bytes plus resident metadata (allocator.py:984-1002); synchronises."""

        allocated = int(self.allocated_rows_tensor().item())
        live_values = allocated * self.width * self.values.element_size()
        metadata = (
            _tensor_bytes(self.logical_to_physical)
            + _tensor_bytes(self.free_rows)
            + _tensor_bytes(self.free_count)
            + _tensor_bytes(self.overflow_flag)
            + _tensor_bytes(self.template_indices)
        )
        return {
            "allocated_rows": allocated,
            "live_value_bytes": live_values,
            "allocator_metadata_bytes": metadata,
            "private_live_total": live_values + metadata,
        }

    @torch.no_grad()
    @_on_dense_maps(lambda self, *_, **__: [self])
    def materialize_dense(self) -> torch.Tensor:
        """Effective ``[banks,N,D]`` table for validation, never serving (allocator.py:1004-1017)."""

        out = torch.empty(self.banks, self.slots, self.width, device=self.values.device,
                          dtype=self.values.dtype)
        pool = self._pool()
        self._call("cow_materialize", ctypes.byref(pool), out.data_ptr(),
                   _lib.dtype_code(self.values.dtype), self._stream())
        return out

    @torch.no_grad()
    @_on_dense_maps(lambda self, *_, **__: [self])
    def release(self, bank_indices: torch.Tensor) -> torch.Tensor:
        """Release whole banks; rows return to the stack at ``old_free + rank`` (allocator.py:1019-1068).

        Invalid or repeated bank indices release nothing and set the status
        word (the reference's asynchronous device assertion).
        """

        if (
            bank_indices.ndim != 1
            or bank_indices.dtype not in (torch.int32, torch.int64)
            or bank_indices.device != self.values.device
        ):
            raise ValueError("released bank indices must be integer [S] on device")
        if bank_indices.numel() == 0:
            return self.free_count.new_zeros(())
        indices = bank_indices.to(torch.int64).contiguous()
        device = self.values.device
        mask = torch.empty(max(self.banks, 1), device=device, dtype=torch.int32)
        scan = _scan_scratch(device, indices.numel() * self.slots)
        released = torch.empty((), device=device, dtype=torch.int32)
        pool = self._pool()
        self._call("cow_release", ctypes.byref(pool), indices.data_ptr(), indices.numel(),
                   mask.data_ptr(), scan.data_ptr(), released.data_ptr(), self._stream())
        return released

    @torch.no_grad()
    def validate_invariants(self) -> dict[str, Any]:
        """Live rows and the free stack partition ``[0, C)`` (allocator.py:1070-1096); synchronises."""

        return validate_layers([self])[0]

    def _validate_result(self, flag: int, bits: int, free: int) -> dict[str, Any]:
        if flag & _lib.ST_SLAB_EXHAUSTED:
            raise AssertionError("SDM COW allocator recorded a slab overflow")
        if flag:
            raise AssertionError(f"SDM COW allocator recorded an error: {_lib.status_text(flag)}")
        if bits & _lib.ST_MULTI_OWNER:
            raise AssertionError("one physical SDM row has multiple logical owners")
        if bits & _lib.ST_FREE_DUPLICATE:
            raise AssertionError("free SDM row stack contains duplicates")
        if bits & (_lib.ST_NOT_COVERED | _lib.ST_ROW_RANGE):
            raise AssertionError("active and free SDM rows do not partition the slab")
        return {
            "capacity_rows": self.capacity_rows,
            "allocated_rows": self.capacity_rows - free,
            "free_rows": free,
            "exact_partition": True,
        }

    def status(self) -> int:
        """Synchronously read the device status word (0 = healthy)."""

        return int(self.overflow_flag.item())


# --------------------------------------------------------------------------
# several pools at once (the SDM layers of one serving batch)
# --------------------------------------------------------------------------


def _read_counts_and_range(values: torch.Tensor | Sequence[torch.Tensor], templates: torch.Tensor | None):
    """One host synchronisation for device integers (a vector or several 0-d
    tensors) and, optionally,
    the (min, max) of a template-index vector.  Returns ``(ints, lo, hi)``."""
    if isinstance(values, torch.Tensor):
        parts = [values.reshape(-1).to(torch.int64)]
        k = values.numel()
    else:
        parts = [torch.stack([v.reshape(()).to(torch.int64) for v in values])] if values else []
        k = len(values)
    if templates is not None and templates.numel():
        lo, hi = torch.aminmax(templates)
        parts.append(torch.stack((lo, hi)))
    host = torch.cat(parts).tolist() if parts else []
    if templates is not None and templates.numel():
        return host[:k], host[k], host[k + 1]
    return host[:k], None, None


def _check_template_range(lo, hi, m0: torch.Tensor) -> None:
    if lo is not None and (lo < 0 or hi >= m0.shape[0]):
        raise ValueError("template index lies outside shared initial memory")


_WORKSPACE: dict[int, torch.Tensor] = {}
# The prefill walks its prefix on routes resolved beforehand by a parallel pass
# (cow_prefill_recurrence_layers_ws); COW_PREFILL_RESOLVED=0 selects the walk
# that resolves each token's routes itself, for comparisons.
_PREFILL_RESOLVED = os.environ.get("COW_PREFILL_RESOLVED", "1") != "0"


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device scratch of the multi-pool lifecycle calls (stream-ordered reuse)."""
    if nbytes < 0:
        raise ValueError("invalid pools for a multi-pool lifecycle call")
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes + nbytes // 4, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACE[key] = buf
    return buf


def _chunks(n: int):
    for a in range(0, n, _lib.MAX_LAYERS):
        yield a, min(n, a + _lib.MAX_LAYERS)


def _pool_array(states) -> ctypes.Array:
    return (_lib.CowPool * len(states))(*[st._pool() for st in states])


def _ptrs(tensors) -> ctypes.Array:
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() if t is not None and t.numel() else None
                                              for t in tensors])


def _bank_list(bank_indices: torch.Tensor, device, what: str) -> torch.Tensor:
    if (
        bank_indices.ndim != 1
        or bank_indices.dtype not in (torch.int32, torch.int64)
        or bank_indices.device != device
    ):
        raise ValueError(f"{what} bank indices must be integer [S] on device")
    return bank_indices.to(torch.int64).contiguous()


@torch.no_grad()
@_on_dense_maps(lambda states: list(states))
def validate_layers(states: Sequence[PackedSDMCopyOnWriteState]) -> list[dict[str, Any]]:
    """``validate_invariants`` of several pools: one call per 8 pools, one host synchronisation."""
    if not states:
        return []
    lib = _lib.load()
    device = states[0].values.device
    stream = _lib.stream_of(device)
    outs = []
    for a, b in _chunks(len(states)):
        pools = _pool_array(states[a:b])
        ws = _workspace(device, lib.cow_validate_workspace_bytes(pools, b - a))
        out = torch.empty(3 * (b - a), dtype=torch.int32, device=device)
        _lib.check(lib.cow_validate_layers(pools, b - a, ws.data_ptr(), ws.numel(), out.data_ptr(), stream),
                   "cow_validate_layers")
        outs.append(out)
    host = torch.cat(outs).tolist()
    return [st._validate_result(*host[3 * i:3 * i + 3]) for i, st in enumerate(states)]


@torch.no_grad()
@_on_dense_maps(lambda states, *_: list(states))
def release_layers(states: Sequence[PackedSDMCopyOnWriteState], bank_indices: Sequence[torch.Tensor]) -> int:
    """``release`` on several pools: one call per 8 pools, one host synchronisation
    for the total count."""
    if len(states) != len(bank_indices):
        raise ValueError("one bank list per pool")
    if not states:
        return 0
    lib = _lib.load()
    device = states[0].values.device
    stream = _lib.stream_of(device)
    idx = [_bank_list(b, st.values.device, "released") for st, b in zip(states, bank_indices)]
    released = torch.empty(len(states), dtype=torch.int32, device=device)
    for a, b in _chunks(len(states)):
        pools = _pool_array(states[a:b])
        counts = (ctypes.c_int64 * (b - a))(*[t.numel() for t in idx[a:b]])
        ws = _workspace(device, lib.cow_release_workspace_bytes(pools, counts, b - a))
        _lib.check(lib.cow_release_layers(pools, _ptrs(idx[a:b]), counts, b - a, ws.data_ptr(), ws.numel(),
                                          released[a:].data_ptr(), stream), "cow_release_layers")
    return sum(released.tolist())


@torch.no_grad()
@_on_dense_maps(lambda states, *_: list(states))
def retain_layers(states: Sequence[PackedSDMCopyOnWriteState], bank_indices: Sequence[torch.Tensor]) -> None:
    """``retain_banks`` on several pools: one call per 8 pools, one host
    synchronisation.  Nothing changes unless every pool's selection is valid."""
    if len(states) != len(bank_indices):
        raise ValueError("one bank list per pool")
    if not states:
        return
    lib = _lib.load()
    device = states[0].values.device
    stream = _lib.stream_of(device)
    idx = [_bank_list(b, st.values.device, "retained") for st, b in zip(states, bank_indices)]
    maps = [torch.empty(t.numel(), st.slots, device=device, dtype=torch.int32) for st, t in zip(states, idx)]
    templates = [torch.empty(t.numel(), device=device, dtype=torch.int64) for t in idx]
    status = torch.empty(len(states), dtype=torch.int32, device=device)
    for a, b in _chunks(len(states)):
        pools = _pool_array(states[a:b])
        counts = (ctypes.c_int64 * (b - a))(*[t.numel() for t in idx[a:b]])
        ws = _workspace(device, lib.cow_retain_workspace_bytes(pools, b - a))
        _lib.check(lib.cow_retain_layers(pools, _ptrs(idx[a:b]), counts, b - a, _ptrs(maps[a:b]),
                                         _ptrs(templates[a:b]), ws.data_ptr(), ws.numel(),
                                         status[a:].data_ptr(), stream), "cow_retain_layers")
    bits = status.tolist()
    for x in bits:
        PackedSDMCopyOnWriteState._retain_check(x)
    for st, m, t, x in zip(states, maps, templates, bits):
        st._retain_commit((m, t, None), x)


@torch.no_grad()
@_on_dense_maps(lambda states, others: [*states, *others])
def append_layers(states: Sequence[PackedSDMCopyOnWriteState],
                  others: Sequence[PackedSDMCopyOnWriteState]) -> list[int]:
    """``append_banks_from`` on several pools: one host synchronisation (plus the
    slab growth the reference does when a pool lacks free rows)."""
    if len(states) != len(others):
        raise ValueError("one admitted pool per destination pool")
    if not states:
        return []
    for st, o in zip(states, others):
        st._append_check(o)
    lib = _lib.load()
    device = states[0].values.device
    stream = _lib.stream_of(device)
    admitted = []
    for a, b in _chunks(len(states)):
        dst, oth = states[a:b], others[a:b]
        other_pools = _pool_array(oth)
        ws = _workspace(device, lib.cow_append_workspace_bytes(other_pools, b - a))
        counts = torch.empty(2 * (b - a), dtype=torch.int32, device=device)
        _lib.check(lib.cow_append_count_layers(_pool_array(dst), other_pools, b - a, ws.data_ptr(), ws.numel(),
                                               counts.data_ptr(), stream), "cow_append_count_layers")
        host = counts.tolist()
        frees = []
        for i, st in enumerate(dst):
            active, free = host[2 * i], host[2 * i + 1]
            if free < active:
                free += st.grow_capacity(st.capacity_rows + active - free)
            frees.append(free)
        maps = [torch.empty(o.banks, st.slots, device=device, dtype=torch.int32) for st, o in zip(dst, oth)]
        _lib.check(lib.cow_append_layers(_pool_array(dst), other_pools, b - a, _ptrs(maps), ws.data_ptr(),
                                         ws.numel(), stream), "cow_append_layers")
        for i, (st, o, m) in enumerate(zip(dst, oth, maps)):
            st._append_commit(o, m, host[2 * i], frees[i])
            admitted.append(host[2 * i])
    return admitted


def _prefix_steps(shared_initial_memories, prefixes, template_indices):
    """Validated step arguments of several pools' prefixes (one set of shapes
    and dtypes for all): ``(m0s, steps, (banks, T, W, R, width, slots, index
    code, activation code))``."""
    n = len(prefixes)
    if len(shared_initial_memories) != n or not 1 <= n <= _lib.MAX_LAYERS:
        raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per prefill")
    m0s, steps, shape = [], [], None
    for m0, x in zip(shared_initial_memories, prefixes):
        m0 = PackedSDMCopyOnWriteState._normalise_m0(m0)
        write_indices, read_indices = x["write_indices"], x["read_indices"]
        erase_gate = x.get("erase_gate")
        if write_indices.ndim != 3 or read_indices.ndim != 3:
            raise ValueError("prefix routes must be [banks,T,K]")
        banks, time, writes = write_indices.shape
        reads = read_indices.shape[2]
        width, slots = m0.shape[2], m0.shape[1]
        if (
            x["write_weights"].shape != write_indices.shape
            or x["read_weights"].shape != read_indices.shape
            or read_indices.shape[:2] != (banks, time)
            or x["values"].shape != (banks, time, width)
            or x["input_gate"].shape != (banks, time)
            or x["forget_log_gate"].shape != (banks, time)
            or (erase_gate is not None and erase_gate.shape != (banks, time))
            or template_indices.shape != (banks,)
        ):
            raise ValueError("SDM prefix routes, values and gates do not align")
        if time <= 0:
            raise ValueError("prefill requires at least one token")
        _lib.require_cuda(write_indices, "prefix write indices")
        step = _StepArgs.make(write_indices.reshape(banks * time, writes),
                              x["write_weights"].reshape(banks * time, writes),
                              x["values"].reshape(banks * time, width),
                              x["input_gate"].reshape(-1), x["forget_log_gate"].reshape(-1),
                              read_indices.reshape(banks * time, reads),
                              x["read_weights"].reshape(banks * time, reads),
                              None if erase_gate is None else erase_gate.reshape(-1),
                              collect=False)
        key = (banks, time, writes, reads, width, slots, step.idx_code, step.act_code)
        if shape is not None and key != shape:
            raise ValueError("pools prefilled together must share banks, T, W, R, width and dtypes")
        shape = key
        m0s.append(m0)
        steps.append(step)
    return m0s, steps, shape


@torch.no_grad()
def from_prefix_routes_layers(
    shared_initial_memories: Sequence[torch.Tensor],
    prefixes: Sequence[dict],
    *,
    template_indices: torch.Tensor,
    capacity_rows: int | None = None,
    state_dtype: torch.dtype = torch.float32,
    maximum_future_allocations: int | None = None,
    growth_quantum_rows: int = 0,
) -> tuple[list[PackedSDMCopyOnWriteState], list[torch.Tensor]]:
    """Sparse prefill handoff of up to 8 independent pools (``from_prefix_routes``
    per pool) in one set of launches with two host synchronisations.

    ``prefixes[l]`` holds pool l's ``write_indices``, ``write_weights``,
    ``values``, ``input_gate``, ``forget_log_gate``, ``read_indices``,
    ``read_weights`` and optionally ``erase_gate`` (shapes ``[banks,T,W|R]``,
    ``[banks,T,D]``, ``[banks,T]``); every pool has the same banks, T, W, R,
    width and dtypes and uses ``template_indices``.
    """
    n = len(prefixes)
    if len(shared_initial_memories) != n or not 1 <= n <= _lib.MAX_LAYERS:
        raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per prefill")
    lib = _lib.load()
    m0s, steps, shape = _prefix_steps(shared_initial_memories, prefixes, template_indices)
    banks, time, writes, reads, width, slots, idx_code, act_code = shape
    device = steps[0].widx.device
    stream = _lib.stream_of(device)
    templates = template_indices.to(torch.int64).contiguous()
    maps = [torch.empty(banks, slots, device=device, dtype=torch.int32) for _ in range(n)]
    ws = _workspace(device, lib.cow_pack_workspace_bytes(banks * slots, n))
    out = torch.empty(2 * n, device=device, dtype=torch.int32)
    _lib.check(lib.cow_prefill_mark_count_layers(_ptrs([st.widx for st in steps]), _ptrs([st.ridx for st in steps]),
                                                 idx_code, banks, time, writes, reads,
                                                 slots, _ptrs(maps), n, ws.data_ptr(), ws.numel(), out.data_ptr(),
                                                 stream), "cow_prefill_mark_count_layers")
    host, lo, hi = _read_counts_and_range(out, templates)
    for l in range(n):
        if host[2 * l]:
            raise ValueError(_lib.status_text(host[2 * l]))
    _check_template_range(lo, hi, m0s[0])
    states = [PackedSDMCopyOnWriteState._pack_state(
        m0s[l], maps[l], templates, host[2 * l + 1], capacity_rows=capacity_rows, state_dtype=state_dtype,
        maximum_future_allocations=maximum_future_allocations, growth_quantum_rows=growth_quantum_rows)
        for l in range(n)]
    pools = _pool_array(states)
    _lib.check(lib.cow_pack_apply_layers(pools, n, ws.data_ptr(), ws.numel(), stream), "cow_pack_apply_layers")
    structs = (_lib.CowStep * n)(*[step.struct for step in steps])
    if _PREFILL_RESOLVED:
        rws = _workspace(device, lib.cow_prefill_workspace_bytes(pools, n, time, writes, reads))
        _lib.check(lib.cow_prefill_recurrence_layers_ws(pools, structs, n, time, writes, reads, idx_code, act_code,
                                                        rws.data_ptr(), rws.numel(), stream),
                   "cow_prefill_recurrence_layers_ws")
    else:
        _lib.check(lib.cow_prefill_recurrence_layers(pools, structs, n, time, writes, reads, idx_code, act_code,
                                                     stream), "cow_prefill_recurrence_layers")
    # Route errors met during the walk are ValueErrors (as in the reference's
    # prefill); anything else is an invariant failure.
    vws = _workspace(device, lib.cow_validate_workspace_bytes(pools, n))
    vout = torch.empty(3 * n, device=device, dtype=torch.int32)
    _lib.check(lib.cow_validate_layers(pools, n, vws.data_ptr(), vws.numel(), vout.data_ptr(), stream),
               "cow_validate_layers")
    flat = vout.tolist()
    for l in range(n):
        if flat[3 * l]:
            raise ValueError(_lib.status_text(flat[3 * l]))
    for l, st in enumerate(states):
        st._validate_result(*flat[3 * l:3 * l + 3])
    return states, [step.output.reshape(banks, time, width) for step in steps]


@torch.no_grad()
@_on_dense_maps(lambda states, *_a, **_k: list(states))
def admit_prefix_routes_layers(states: Sequence[PackedSDMCopyOnWriteState], prefixes: Sequence[dict], *,
                               template_indices: torch.Tensor) -> list[torch.Tensor]:
    """Prefill a cohort and admit it into ``states`` (one live pool per layer) in one
    set of launches, without pools of its own: the same maps, free stacks,
    rows, growth and readings as ``from_prefix_routes_layers`` (with the live
    pools' growth quantum) followed by ``append_layers``.

    Every marked slot of the cohort pops the live pool's free stack in
    ``nonzero()`` order (the order in which appending the packed cohort pops
    it, allocator.py:884-896), its row is filled from ``M0`` and the prefix
    walk runs on the admitted banks in place.  Routes and templates are checked
    before anything changes (one host synchronisation, which also reads the
    free counts for growth).  Returns the readings ``[banks, T, width]`` per pool.
    """
    n = len(states)
    if len(prefixes) != n or not 1 <= n <= _lib.MAX_LAYERS:
        raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per admission")
    lib = _lib.load()
    m0s, steps, shape = _prefix_steps([st.shared_initial_memory for st in states], prefixes, template_indices)
    banks, time, writes, reads, width, slots, idx_code, act_code = shape
    for st in states:
        if st.slots != slots or st.width != width:
            raise ValueError("admitted SDM banks do not match the destination pool")
    if banks == 0:
        return [step.output.reshape(0, time, width) for step in steps]
    device = states[0].values.device
    stream = _lib.stream_of(device)
    templates = template_indices.to(torch.int64).contiguous()
    marks = [torch.empty(banks, slots, device=device, dtype=torch.int32) for _ in range(n)]
    ws = _workspace(device, max(lib.cow_pack_workspace_bytes(banks * slots, n),
                                lib.cow_admit_prefix_workspace_bytes(banks, slots, n)))
    out = torch.empty(2 * n, device=device, dtype=torch.int32)
    _lib.check(lib.cow_prefill_mark_count_layers(_ptrs([st.widx for st in steps]), _ptrs([st.ridx for st in steps]),
                                                 idx_code, banks, time, writes, reads,
                                                 slots, _ptrs(marks), n, ws.data_ptr(), ws.numel(), out.data_ptr(),
                                                 stream), "cow_prefill_mark_count_layers")
    # One read for the mark status (write and read route checks), the live
    # counts and the free counts.
    frees_dev = torch.stack([st.free_count.reshape(()) for st in states]).to(torch.int64)
    host, lo, hi = _read_counts_and_range(torch.cat((out.to(torch.int64), frees_dev)), templates)
    for l in range(n):
        if host[2 * l]:
            raise ValueError(_lib.status_text(host[2 * l]))
    _check_template_range(lo, hi, m0s[0])
    frees = []
    for l, st in enumerate(states):
        active, free = host[2 * l + 1], host[2 * n + l]
        if free < active:
            free += st.grow_capacity(st.capacity_rows + active - free)
        frees.append(free)
    admitted = [torch.empty(banks, slots, device=device, dtype=torch.int32) for _ in range(n)]
    _lib.check(lib.cow_admit_prefix_layers(_pool_array(states), _ptrs(marks), templates.data_ptr(), banks, n,
                                           _ptrs(admitted), ws.data_ptr(), ws.numel(), stream),
               "cow_admit_prefix_layers")
    old_banks = []
    for l, st in enumerate(states):
        old_banks.append(st.banks)
        st.logical_to_physical = torch.cat((st.logical_to_physical, admitted[l]), dim=0).contiguous()
        st.template_indices = torch.cat((st.template_indices, templates), dim=0).contiguous()
        active = host[2 * l + 1]
        if st.growth_quantum_rows:
            st.proven_maximum_additional_allocations = min(st.proven_maximum_additional_allocations,
                                                           frees[l] - active)
        else:
            st.capacity_is_proven = False
            st.proven_maximum_additional_allocations = 0
    # The walk on the admitted banks: each pool seen from its first admitted bank.
    pools = _pool_array(states)
    for l in range(n):
        pools[l].map += old_banks[l] * slots * 4
        pools[l].templates += old_banks[l] * 8
        pools[l].banks = banks
    structs = (_lib.CowStep * n)(*[step.struct for step in steps])
    rws = _workspace(device, lib.cow_prefill_workspace_bytes(pools, n, time, writes, reads))
    _lib.check(lib.cow_prefill_recurrence_layers_ws(pools, structs, n, time, writes, reads, idx_code, act_code,
                                                    rws.data_ptr(), rws.numel(), stream),
               "cow_prefill_recurrence_layers_ws")
    return [step.output.reshape(banks, time, width) for step in steps]


# --------------------------------------------------------------------------
# step arguments
# --------------------------------------------------------------------------


class _StepArgs:
    """Validated, contiguous, same-dtype views of one step's routes + its output."""

    __slots__ = ("widx", "ww", "values", "in_g", "er_g", "fl_g", "ridx", "rw", "output", "first",
                 "struct", "idx_code", "act_code", "writes", "reads", "_keep")

    @classmethod
    def make(cls, write_indices, write_weights, values, input_gate, forget_log_gate, read_indices,
             read_weights, erase_gate, *, collect: bool, output: torch.Tensor | None = None):
        self = cls()
        act = values.dtype
        if act not in (torch.float32, torch.bfloat16, torch.float16):
            raise ValueError("SDM step values must be float32, bfloat16 or float16")

        def prep(t: torch.Tensor) -> torch.Tensor:
            t = t if t.dtype == act else t.to(act)
            t = t.contiguous()
            if t.data_ptr() % 16:
                t = t.clone()
            return t

        idx_dtype = write_indices.dtype
        if idx_dtype not in (torch.int32, torch.int64) or read_indices.dtype not in (torch.int32, torch.int64):
            raise ValueError("SDM route indices must be int32 or int64")
        self.widx = write_indices.contiguous()
        self.ridx = read_indices.contiguous() if read_indices.dtype == idx_dtype else read_indices.to(idx_dtype).contiguous()
        self.ww, self.values, self.in_g, self.fl_g, self.rw = (
            prep(write_weights), prep(values), prep(input_gate), prep(forget_log_gate), prep(read_weights))
        self.er_g = self.in_g if erase_gate is None else prep(erase_gate)
        self.output = output if output is not None else torch.empty_like(self.values)
        self.writes = self.widx.shape[-1]
        self.reads = self.ridx.shape[-1]
        self.first = (torch.empty(self.widx.shape, device=self.widx.device, dtype=torch.uint8)
                      if collect else None)
        self.idx_code = _lib.index_code(idx_dtype)
        self.act_code = _lib.dtype_code(act)
        self.struct = _lib.CowStep(
            self.widx.data_ptr(), self.ww.data_ptr(), self.values.data_ptr(), self.in_g.data_ptr(),
            self.er_g.data_ptr(), self.fl_g.data_ptr(), self.ridx.data_ptr(), self.rw.data_ptr(),
            self.output.data_ptr(), _lib.ptr(self.first),
        )
        return self


def _validate_indices(indices, *, name, banks, device):
    if (
        indices.ndim != 2
        or indices.shape[0] != banks
        or indices.shape[1] <= 0
        or indices.dtype not in (torch.int32, torch.int64)
        or indices.device != device
    ):
        raise ValueError(f"{name} indices must be integer [B,K] on device")


def _validate_step(banks, width, device, write_indices, write_weights, values, input_gate,
                   forget_log_gate, read_indices, read_weights, erase_gate):
    _validate_indices(write_indices, name="write", banks=banks, device=device)
    _validate_indices(read_indices, name="read", banks=banks, device=device)
    if (
        write_weights.shape != write_indices.shape
        or read_weights.shape != read_indices.shape
        or values.shape != (banks, width)
    ):
        raise ValueError("SDM route weights and values do not align")
    tensors = (write_weights, values, input_gate, forget_log_gate, read_weights) + (
        () if erase_gate is None else (erase_gate,))
    if any(t.device != device for t in tensors):
        raise ValueError("SDM COW step tensors must share one device")
    effective_erase = input_gate if erase_gate is None else erase_gate
    if input_gate.shape != (banks,):
        raise ValueError("native SDM input gate must be [B]")
    if effective_erase.shape != input_gate.shape or forget_log_gate.shape != input_gate.shape:
        raise ValueError("SDM input, erase, and forget gates must align")
    if write_indices.shape[1] > _lib.MAX_WRITES or read_indices.shape[1] > _lib.MAX_READS:
        raise ValueError(
            f"this build supports W <= {_lib.MAX_WRITES} and R <= {_lib.MAX_READS} routes per step")
    if width % 4 or width > _lib.MAX_WIDTH:
        raise ValueError(f"this build supports widths that are multiples of 4 up to {_lib.MAX_WIDTH}")


def _check_backend(backend: str) -> None:
    if backend == "torch":
        raise ValueError(
            "backend='torch' (the reference's CPU path) does not exist in this build: "
            "packed SDM runs only through the sm_100a kernels")
    if backend not in _BACKENDS:
        raise ValueError("allocator backend must be auto or cuda")


@torch.no_grad()
def packed_sdm_cow_step_layers(
    states: Sequence[PackedSDMCopyOnWriteState],
    steps: Sequence[dict],
    *,
    validate_routes: bool = False,
    collect_diagnostics: bool = False,
    outputs: Sequence[torch.Tensor] | None = None,
    scratch: torch.Tensor | None = None,
) -> list[torch.Tensor]:
    """One fused launch for several independent pools (e.g. all SDM layers of a
    synthetic screen).  ``steps[l]`` holds the keyword arguments of
    ``packed_sdm_cow_step`` for ``states[l]``.  Same semantics per pool as
    ``packed_sdm_cow_step``; returns the readings.
    """

    if len(states) != len(steps) or not 1 <= len(states) <= _lib.MAX_LAYERS:
        raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per launch")
    lib = _lib.load()
    args = []
    for i, (state, st) in enumerate(zip(states, steps)):
        _lib.require_cuda(state.values, "SDM COW state")
        erase = st.get("erase_gate")
        _validate_step(state.banks, state.width, state.values.device, st["write_indices"],
                       st["write_weights"], st["values"], st["input_gate"], st["forget_log_gate"],
                       st["read_indices"], st["read_weights"], erase)
        args.append(_StepArgs.make(st["write_indices"], st["write_weights"], st["values"],
                                   st["input_gate"], st["forget_log_gate"], st["read_indices"],
                                   st["read_weights"], erase, collect=collect_diagnostics,
                                   output=None if outputs is None else outputs[i]))
    a0 = args[0]
    for a, s in zip(args, states):
        if (a.writes, a.reads, a.idx_code, a.act_code) != (a0.writes, a0.reads, a0.idx_code, a0.act_code) \
                or s.width != states[0].width or s.values.dtype != states[0].values.dtype:
            raise ValueError("pools fused into one launch must share width, W, R and dtypes")
    n = len(states)
    pools = (_lib.CowPool * n)(*[s._pool() for s in states])
    structs = (_lib.CowStep * n)(*[a.struct for a in args])
    device = states[0].values.device
    total_banks = sum(s.banks for s in states)
    if scratch is None:
        scratch = decode_scratch(device, total_banks, n)
    _lib.check(lib.cow_decode_step(pools, structs, n, a0.writes, a0.reads, a0.idx_code, a0.act_code,
                                   scratch.data_ptr(), scratch.numel(), _lib.stream_of(device)),
               "cow_decode_step")
    if validate_routes or any(not s.capacity_is_proven for s in states):
        for s in states:
            bits = s.status()
            if bits:
                raise ValueError(_lib.status_text(bits))
    if collect_diagnostics:
        return [a.output for a in args], [a.first for a in args]
    return [a.output for a in args]


@torch.no_grad()
def packed_sdm_cow_step(
    state: PackedSDMCopyOnWriteState,
    write_indices: torch.Tensor,
    write_weights: torch.Tensor,
    values: torch.Tensor,
    input_gate: torch.Tensor,
    forget_log_gate: torch.Tensor,
    read_indices: torch.Tensor,
    read_weights: torch.Tensor,
    *,
    erase_gate: torch.Tensor | None = None,
    backend: str = "auto",
    validate_routes: bool = True,
    collect_diagnostics: bool = True,
    scratch: torch.Tensor | None = None,
) -> tuple[torch.Tensor, SDMCopyOnWriteStep | None]:
    """One exact sparse SDM write + read through the packed overlay (allocator.py:1382-1526).

    One fused kernel launch.  With ``validate_routes`` (or when the capacity
    is not proven) the call synchronises once to turn device status bits
    (bad index, repeated write, exhausted slab) into ``ValueError``.
    ``scratch`` (not in the reference's signature) is an optional owner-held
    look-back buffer (``new_decode_scratch``); the per-device one otherwise.
    """

    _check_backend(backend)
    _lib.require_cuda(state.values, "SDM COW state")
    steps = [dict(write_indices=write_indices, write_weights=write_weights, values=values,
                  input_gate=input_gate, forget_log_gate=forget_log_gate, read_indices=read_indices,
                  read_weights=read_weights, erase_gate=erase_gate)]
    result = packed_sdm_cow_step_layers([state], steps, validate_routes=validate_routes,
                                        collect_diagnostics=collect_diagnostics, scratch=scratch)
    if not collect_diagnostics:
        return result[0], None
    outputs, firsts = result
    first_by_sequence = firsts[0].sum(dim=-1)
    return outputs[0], SDMCopyOnWriteStep(
        first_touches_by_sequence=first_by_sequence,
        repeated_writes_by_sequence=(write_indices.shape[1] - first_by_sequence),
        allocated_rows_after_step=state.allocated_rows_tensor(),
    )


@torch.no_grad()
def dense_sdm_sparse_step_layers(
    memories: Sequence[torch.Tensor], steps: Sequence[dict], *,
    outputs: Sequence[torch.Tensor] | None = None,
) -> list[torch.Tensor]:
    """Dense-table control over several independent tables in one launch."""

    if len(memories) != len(steps) or not 1 <= len(memories) <= _lib.MAX_LAYERS:
        raise ValueError(f"between 1 and {_lib.MAX_LAYERS} tables per launch")
    lib = _lib.load()
    args = []
    for i, (mem, st) in enumerate(zip(memories, steps)):
        if mem.ndim != 3:
            raise ValueError("dense SDM memory must be [B,N,D]")
        _lib.require_cuda(mem, "dense SDM memory")
        if not mem.is_contiguous():
            raise ValueError("dense SDM memory must be contiguous")
        banks, _, width = mem.shape
        erase = st.get("erase_gate")
        _validate_step(banks, width, mem.device, st["write_indices"], st["write_weights"], st["values"],
                       st["input_gate"], st["forget_log_gate"], st["read_indices"], st["read_weights"], erase)
        args.append(_StepArgs.make(st["write_indices"], st["write_weights"], st["values"], st["input_gate"],
                                   st["forget_log_gate"], st["read_indices"], st["read_weights"], erase,
                                   collect=False, output=None if outputs is None else outputs[i]))
    a0 = args[0]
    m0 = memories[0]
    for a, m in zip(args, memories):
        if (a.writes, a.reads, a.idx_code, a.act_code) != (a0.writes, a0.reads, a0.idx_code, a0.act_code) \
                or m.shape[1:] != m0.shape[1:] or m.dtype != m0.dtype:
            raise ValueError("tables fused into one launch must share shape, W, R and dtypes")
    n = len(memories)
    mem_ptrs = (ctypes.c_void_p * n)(*[m.data_ptr() for m in memories])
    banks = (ctypes.c_int64 * n)(*[m.shape[0] for m in memories])
    structs = (_lib.CowStep * n)(*[a.struct for a in args])
    _lib.check(lib.cow_dense_step(mem_ptrs, banks, structs, n, m0.shape[1], m0.shape[2],
                                  _lib.dtype_code(m0.dtype), a0.writes, a0.reads, a0.idx_code,
                                  a0.act_code, _lib.stream_of(m0.device)), "cow_dense_step")
    return [a.output for a in args]


@torch.no_grad()
def dense_sdm_sparse_step(
    memory: torch.Tensor,
    write_indices: torch.Tensor,
    write_weights: torch.Tensor,
    values: torch.Tensor,
    input_gate: torch.Tensor,
    forget_log_gate: torch.Tensor,
    read_indices: torch.Tensor,
    read_weights: torch.Tensor,
    *,
    erase_gate: torch.Tensor | None = None,
    backend: str = "auto",
    validate_routes: bool = True,
) -> torch.Tensor:
    """Mutate one dense table with the same sparse routes (allocator.py:1529-1633).

    The benchmark control: same math, no map, no allocation.
    """

    _check_backend(backend)
    if memory.ndim != 3:
        raise ValueError("dense SDM memory must be [B,N,D]")
    steps = [dict(write_indices=write_indices, write_weights=write_weights, values=values,
                  input_gate=input_gate, forget_log_gate=forget_log_gate, read_indices=read_indices,
                  read_weights=read_weights, erase_gate=erase_gate)]
    if validate_routes:
        n = memory.shape[1]
        bad = ((write_indices < 0) | (write_indices >= n)).any() | ((read_indices < 0) | (read_indices >= n)).any()
        if write_indices.shape[1] > 1:
            ordered = write_indices.sort(dim=-1).values
            bad = bad | (ordered[:, 1:] == ordered[:, :-1]).any()
        if bool(bad):
            raise ValueError("SDM route index lies outside the logical table or repeats a write")
    return dense_sdm_sparse_step_layers([memory], steps)[0]
