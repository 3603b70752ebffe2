"""Serving-state checkpoints and request migration.

A checkpoint holds a set of live requests of a ``FaithfulSDMDecodeState``:
for every SDM layer the request banks' private rows and where they sit in the
logical tables, plus the dense K/V caches and positions.  It is the packed
cohort that ``append_banks_from`` / ``FaithfulSDMDecodeState.admit`` already
take (allocator.py:842-915, inference.py:161-206), so restoring a checkpoint
is an admission: a request can move to another GPU, or a serving process can
stop and resume its live requests, without replaying the prefix.

Per SDM layer the private state of the selected banks is stored compactly:

* ``live``: int64 ``[A]``, the flat ``bank * N + slot`` index of every slot
  that owns a private row, in ``nonzero()`` order of the selected banks'
  ``[S*H, N]`` map (bank = request * H + head, requests in the given order);
* ``rows``: ``[A, D]`` in the slab dtype, row ``k`` belonging to ``live[k]``;
* ``templates``: int64 ``[S*H]``.

Restoring places row ``k`` at physical row ``k`` (the map becomes
``map.flat[live] = arange(A)``) and fills the free stack with
``arange(A, C)`` -- the layout ``from_dense_overlay`` gives a prefilled cohort
(allocator.py:624-689).  Shared ``M0`` is not stored: it belongs to the model.

File format (``save`` / ``load``): the 8-byte magic ``COWSDMC1``, a
little-endian uint64 header length, a UTF-8 JSON header (format version,
layout, positions, per-layer shapes and dtypes, byte offsets), then the raw
little-endian tensor bytes, each starting on a 64-byte boundary.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from typing import Sequence

import torch

from . import _lib
from .allocator import PackedSDMCopyOnWriteState, dense_maps, validate_layers
from .inference import FaithfulSDMDecodeState, _banks_per_state

MAGIC = b"COWSDMC1"
FORMAT_VERSION = 1
_ALIGN = 64
_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
           "int32": torch.int32, "int64": torch.int64, "bool": torch.bool}


def _dtype_name(dtype: torch.dtype) -> str:
    for k, v in _DTYPES.items():
        if v == dtype:
            return k
    raise ValueError(f"unsupported checkpoint dtype {dtype}")


@dataclass
class LayerCheckpoint:
    """Private state of the checkpointed banks of one SDM pool."""

    live: torch.Tensor        # int64 [A] flat bank*N+slot, nonzero() order
    rows: torch.Tensor        # [A, D] slab dtype
    templates: torch.Tensor   # int64 [S*H]
    slots: int
    growth_quantum_rows: int


@dataclass
class ServingCheckpoint:
    """Live requests of a ``FaithfulSDMDecodeState`` (see the module docstring)."""

    layout: str
    capacity: int
    activation_dtype: torch.dtype
    positions: torch.Tensor                   # int64 [S]
    sdm_layer_positions: tuple[int, ...]
    layers: list[LayerCheckpoint]
    dense_keys: list[torch.Tensor] = field(default_factory=list)    # [S, heads, capacity, head_width]
    dense_values: list[torch.Tensor] = field(default_factory=list)

    @property
    def requests(self) -> int:
        return int(self.positions.numel())

    def live_rows(self) -> int:
        return sum(int(l.live.numel()) for l in self.layers)

    def nbytes(self) -> int:
        ts = [self.positions] + [t for l in self.layers for t in (l.live, l.rows, l.templates)]
        ts += list(self.dense_keys) + list(self.dense_values)
        return sum(t.numel() * t.element_size() for t in ts)

    def to(self, device) -> "ServingCheckpoint":
        return ServingCheckpoint(
            layout=self.layout, capacity=self.capacity, activation_dtype=self.activation_dtype,
            positions=self.positions.to(device), sdm_layer_positions=self.sdm_layer_positions,
            layers=[LayerCheckpoint(l.live.to(device), l.rows.to(device), l.templates.to(device), l.slots,
                                    l.growth_quantum_rows) for l in self.layers],
            dense_keys=[t.to(device) for t in self.dense_keys], dense_values=[t.to(device) for t in self.dense_values])

    # ---------------- file format ----------------

    def save(self, path) -> None:
        tensors, meta = [], {"layers": [], "dense_keys": [], "dense_values": []}

        def put(t: torch.Tensor) -> dict:
            t = t.detach().to("cpu").contiguous()
            tensors.append(t)
            return {"index": len(tensors) - 1, "dtype": _dtype_name(t.dtype), "shape": list(t.shape)}

        meta["positions"] = put(self.positions)
        for l in self.layers:
            meta["layers"].append({"live": put(l.live), "rows": put(l.rows), "templates": put(l.templates),
                                   "slots": l.slots, "growth_quantum_rows": l.growth_quantum_rows})
        meta["dense_keys"] = [put(t) for t in self.dense_keys]
        meta["dense_values"] = [put(t) for t in self.dense_values]
        blobs = [t.view(torch.uint8).reshape(-1).numpy().tobytes() if t.numel() else b"" for t in tensors]
        offsets, off = [], 0
        for b in blobs:
            off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
            offsets.append(off)
            off += len(b)
        header = {"format_version": FORMAT_VERSION, "layout": self.layout, "capacity": self.capacity,
                  "activation_dtype": _dtype_name(self.activation_dtype),
                  "sdm_layer_positions": list(self.sdm_layer_positions), "tensors": meta,
                  "offsets": offsets, "sizes": [len(b) for b in blobs], "byteorder": "little"}
        hb = json.dumps(header, sort_keys=True).encode()
        with open(path, "wb") as f:
            f.write(MAGIC)
            f.write(struct.pack("<Q", len(hb)))
            f.write(hb)
            base = f.tell()
            for o, b in zip(offsets, blobs):
                f.seek(base + o)
                f.write(b)

    @classmethod
    def load(cls, path) -> "ServingCheckpoint":
        with open(path, "rb") as f:
            data = f.read()
        if data[:8] != MAGIC:
            raise ValueError("not an SDM serving checkpoint")
        (hlen,) = struct.unpack("<Q", data[8:16])
        header = json.loads(data[16:16 + hlen].decode())
        if header.get("format_version") != FORMAT_VERSION:
            raise ValueError(f"unsupported checkpoint format version {header.get('format_version')}")
        base = 16 + hlen
        offsets, sizes = header["offsets"], header["sizes"]

        def get(d: dict) -> torch.Tensor:
            i = d["index"]
            dtype = _DTYPES[d["dtype"]]
            raw = bytearray(data[base + offsets[i]: base + offsets[i] + sizes[i]])
            if len(raw) != sizes[i]:
                raise ValueError("truncated SDM serving checkpoint")
            flat = torch.frombuffer(raw, dtype=torch.uint8) if sizes[i] else torch.empty(0, dtype=torch.uint8)
            return flat.view(dtype).reshape(d["shape"]).clone()

        t = header["tensors"]
        layers = [LayerCheckpoint(get(l["live"]), get(l["rows"]), get(l["templates"]), int(l["slots"]),
                                  int(l["growth_quantum_rows"])) for l in t["layers"]]
        return cls(layout=header["layout"], capacity=int(header["capacity"]),
                   activation_dtype=_DTYPES[header["activation_dtype"]], positions=get(t["positions"]),
                   sdm_layer_positions=tuple(header["sdm_layer_positions"]), layers=layers,
                   dense_keys=[get(d) for d in t["dense_keys"]], dense_values=[get(d) for d in t["dense_values"]])


# --------------------------------------------------------------------------
# export / restore
# --------------------------------------------------------------------------


@torch.no_grad()
def export_requests(state: FaithfulSDMDecodeState, sequence_indices: Sequence[int] | torch.Tensor, *,
                    device: torch.device | str | None = "cpu") -> ServingCheckpoint:
    """Checkpoint the live requests ``sequence_indices`` (in that order); ``state`` is unchanged.

    ``device=None`` keeps the tensors on the state's GPU (direct migration to
    another GPU then copies them peer to peer in ``restore_requests``).
    """
    idx = torch.as_tensor(sequence_indices, dtype=torch.int64, device=state.device).reshape(-1)
    if idx.numel() == 0:
        raise ValueError("no requests to checkpoint")
    host = idx.tolist()
    if (min(host) < 0 or max(host) >= state.batch or len(set(host)) != len(host)
            or not bool(state.active_sequences[idx].all())):
        raise ValueError("checkpointed request is invalid, duplicated, or inactive")
    heads = [state._heads(st, state.batch) for st in state.sdm_states]
    layers = []
    with dense_maps(state.sdm_states):  # hashed pools export through their dense form
        for st, banks in zip(state.sdm_states, _banks_per_state(idx, heads)):
            sub = st.logical_to_physical.index_select(0, banks).reshape(-1)
            live = torch.nonzero(sub >= 0).reshape(-1)
            rows = st.values.index_select(0, sub.index_select(0, live).to(torch.int64))
            layers.append(LayerCheckpoint(live, rows, st.template_indices.index_select(0, banks), st.slots,
                                          st.growth_quantum_rows))
    ckpt = ServingCheckpoint(
        layout=state.layout, capacity=state.capacity, activation_dtype=state.activation_dtype,
        positions=state.current_positions().index_select(0, idx), sdm_layer_positions=state.sdm_layer_positions,
        layers=layers, dense_keys=[t.index_select(0, idx) for t in state.dense_keys],
        dense_values=[t.index_select(0, idx) for t in state.dense_values])
    return ckpt if device is None else ckpt.to(device)


@torch.no_grad()
def restore_requests(ckpt: ServingCheckpoint, shared_initial_memories: Sequence[torch.Tensor], *,
                     capacity_rows: Sequence[int | None] | None = None) -> FaithfulSDMDecodeState:
    """Rebuild the checkpointed requests as a cohort on the device of
    ``shared_initial_memories`` (one ``M0`` per SDM layer, the model's).  Admit
    it into a live state with ``FaithfulSDMDecodeState.admit``.

    Each pool holds the checkpointed rows at ``0..A-1`` and ``arange(A, C)``
    on its free stack, ``C`` = ``capacity_rows[l]`` or ``A`` rounded up to the
    growth quantum (at least one quantum; ``A`` without a quantum).
    """
    if len(shared_initial_memories) != len(ckpt.layers):
        raise ValueError("one shared initial memory per checkpointed SDM layer")
    device = shared_initial_memories[0].device
    _lib.require_cuda(shared_initial_memories[0], "shared initial memory")
    states = []
    for l, (m0, lay) in enumerate(zip(shared_initial_memories, ckpt.layers)):
        m0 = PackedSDMCopyOnWriteState._normalise_m0(m0)
        banks = int(lay.templates.numel())
        active = int(lay.live.numel())
        if (m0.shape[1] != lay.slots or lay.rows.ndim != 2 or lay.rows.shape[0] != active
                or lay.rows.shape[1] != m0.shape[2] or m0.device != device):
            raise ValueError("checkpoint does not match the shared initial memory")
        want = None if capacity_rows is None else capacity_rows[l]
        q = lay.growth_quantum_rows
        if want is None:
            cap = max(q, (active + q - 1) // q * q) if q else max(active, 1)
        else:
            cap = int(want)
        if cap < active:
            raise ValueError("restored SDM capacity is smaller than the checkpointed rows")
        templates = lay.templates.to(device=device, dtype=torch.int64)
        lo, hi = (int(v) for v in torch.aminmax(templates)) if banks else (0, 0)
        if banks and (lo < 0 or hi >= m0.shape[0]):
            raise ValueError("template index lies outside shared initial memory")
        mapping = torch.full((banks, lay.slots), -1, dtype=torch.int32, device=device)
        live = lay.live.to(device)
        if active and (int(live.min()) < 0 or int(live.max()) >= banks * lay.slots
                       or not bool((live[1:] > live[:-1]).all())):
            raise ValueError("checkpoint live slots must be increasing flat indices inside the banks")
        mapping.view(-1).index_copy_(0, live, torch.arange(active, dtype=torch.int32, device=device))
        st = PackedSDMCopyOnWriteState._empty(m0, templates, banks=banks, capacity_rows=cap,
                                              state_dtype=lay.rows.dtype, growth_quantum_rows=q, init=False,
                                              mapping=mapping)
        if active:
            st.values[:active].copy_(lay.rows.to(device))
        st.free_rows[: cap - active].copy_(torch.arange(active, cap, dtype=torch.int32, device=device))
        st.free_count.fill_(cap - active)
        st.capacity_is_proven = False
        st.proven_maximum_additional_allocations = 0
        states.append(st)
    validate_layers(states)
    positions = ckpt.positions.to(device=device, dtype=torch.int64)
    uniform = bool((positions == positions[0]).all())
    return FaithfulSDMDecodeState(
        layout=ckpt.layout, position=int(positions.max()), capacity=ckpt.capacity,
        activation_dtype=ckpt.activation_dtype,
        active_sequences=torch.ones(ckpt.requests, dtype=torch.bool, device=device),
        sdm_layer_positions=tuple(ckpt.sdm_layer_positions), sdm_states=tuple(states),
        dense_keys=tuple(t.to(device) for t in ckpt.dense_keys),
        dense_values=tuple(t.to(device) for t in ckpt.dense_values),
        positions=None if uniform else positions)


@torch.no_grad()
def migrate_requests(source: FaithfulSDMDecodeState, sequence_indices: Sequence[int], destination:
                     FaithfulSDMDecodeState, *, release_source: bool = True) -> int:
    """Move live requests from ``source`` into ``destination`` (any GPU):
    checkpoint, restore next to ``destination``'s pools, admit; then release and
    compact them at the source.  Returns the number of requests moved."""
    ckpt = export_requests(source, sequence_indices, device=None)
    m0s = [st.shared_initial_memory for st in destination.sdm_states]
    cohort = restore_requests(ckpt.to(destination.device), m0s)
    moved = destination.admit(cohort)
    if release_source:
        source.release_and_compact(list(sequence_indices))
    return moved
