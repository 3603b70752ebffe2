"""Serving lifecycle over packed SDM pools: prefill handoff, decode, release,
survivor compaction, admission and trimming (reference ``copy_on_write_sdm/
inference.py``).

Differences from the reference, by design:

* the prefill runs the sparse prefix kernel (``from_prefix_routes``): only
  written rows are ever materialised, so there is no ``[B,T,N,D]`` states
  tensor and no ``N <= 1024`` limit;
* every packed step is one fused sm_100a launch with the reference's
  deterministic row-placement order.

Everything else -- fields, method names, argument meaning, errors and the
``storage_bytes`` keys -- follows the reference.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Sequence

import torch
from torch import nn

from .allocator import (PackedSDMCopyOnWriteState, admit_prefix_routes_layers, append_layers, dense_sdm_sparse_step,
                        packed_sdm_cow_step,
                        release_layers, retain_layers)
from .sdm import SparseDeltaMemory

if TYPE_CHECKING:
    from .model import SDMDecoderStack


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _banks_of(requests: torch.Tensor, heads: int) -> torch.Tensor:
    """Bank ids ``request*H + h`` of the given requests, request-major."""
    return (requests[:, None] * heads + torch.arange(heads, device=requests.device)[None, :]).reshape(-1)


def _banks_per_state(requests: torch.Tensor, heads: Sequence[int],
                     host: Sequence[int] | None = None) -> list[torch.Tensor]:
    """``_banks_of`` for every pool, computed once per distinct head count;
    from the host copy of ``requests`` (one small copy, no kernels) when given."""
    cache: dict[int, torch.Tensor] = {}
    for h in heads:
        if h not in cache:
            cache[h] = (_banks_of(requests, h) if host is None else
                        torch.tensor([r * h + j for r in host for j in range(h)], dtype=torch.int64)
                        .to(requests.device))
    return [cache[h] for h in heads]


@dataclass
class FaithfulSDMDecodeState:
    """Retained state of one batch of independent requests (reference inference.py:26-276).

    ``sdm_states`` holds one packed pool per "B" layer (shared ``M0``, private
    rows in the slab); ``dense_keys`` / ``dense_values`` are the fixed-capacity
    K/V caches of the "A" layers.  ``positions`` is ``None`` while every
    request sits at ``position``; after an admission of a cohort at a
    different position it holds one position per request.
    """

    layout: str
    position: int
    capacity: int
    activation_dtype: torch.dtype
    active_sequences: torch.Tensor
    sdm_layer_positions: tuple[int, ...]
    sdm_states: tuple[PackedSDMCopyOnWriteState, ...]
    dense_keys: tuple[torch.Tensor, ...]
    dense_values: tuple[torch.Tensor, ...]
    positions: torch.Tensor | None = None

    @property
    def batch(self) -> int:
        return self.active_sequences.numel()

    @property
    def device(self) -> torch.device:
        return self.active_sequences.device

    @property
    def dtype(self) -> torch.dtype:
        return self.activation_dtype

    def current_positions(self) -> torch.Tensor:
        if self.positions is not None:
            return self.positions
        return torch.full((self.batch,), self.position, device=self.device, dtype=torch.int64)

    def _heads(self, state: PackedSDMCopyOnWriteState, batch: int) -> int:
        if batch == 0:
            if state.banks != 0:
                raise AssertionError("empty serving batch retained SDM banks")
            return 0
        if state.banks % batch:
            raise AssertionError("SDM serving banks do not divide by batch")
        return state.banks // batch

    def _active_host(self) -> list[bool]:
        """``active_sequences`` as a host list, read from the device only when the
        tensor was replaced or changed in place since this object last knew it."""
        act = self.active_sequences
        cached = self.__dict__.get("_active_of")
        if cached is not None and cached[0] is act and cached[1] == act._version:
            return cached[2]
        host = act.tolist()
        self.__dict__["_active_of"] = (act, act._version, host)  # holds the tensor: its identity stays unique
        return host

    def _set_active(self, tensor: torch.Tensor, host: list[bool]) -> None:
        self.active_sequences = tensor
        self.__dict__["_active_of"] = (tensor, tensor._version, host)

    @torch.no_grad()
    def release(self, sequence_indices: torch.Tensor | Sequence[int] | None = None) -> int:
        """Return the private rows of finished requests to every layer's pool (inference.py:71-114)."""
        active = self._active_host()
        if sequence_indices is None:
            host = [i for i, a in enumerate(active) if a]
            chosen = torch.tensor(host, dtype=torch.int64).to(self.device)
        elif isinstance(sequence_indices, torch.Tensor):
            chosen = sequence_indices.to(device=self.device, dtype=torch.int64)
            host = chosen.tolist() if chosen.ndim == 1 else None
        else:  # a host sequence: checked on the host, copied to the device once
            flat = torch.as_tensor(sequence_indices, dtype=torch.int64)
            host = flat.tolist() if flat.ndim == 1 else None
            chosen = flat.to(self.device)
        if chosen.ndim != 1:
            raise ValueError("released sequence indices must be a vector")
        if chosen.numel() == 0:
            return 0
        if (min(host) < 0 or max(host) >= self.batch or len(set(host)) != len(host)
                or not all(active[i] for i in host)):
            raise ValueError("released sequence is invalid, duplicated, or inactive")
        total = release_layers(self.sdm_states,
                               _banks_per_state(chosen, [self._heads(st, self.batch) for st in self.sdm_states], host))
        self.active_sequences[chosen] = False
        after = list(active)
        for i in host:
            after[i] = False
        self._set_active(self.active_sequences, after)
        return total

    @torch.no_grad()
    def compact(self) -> torch.Tensor:
        """Drop released request slots; live rows stay where they are (inference.py:116-159)."""
        before = self.batch
        kept = [i for i, a in enumerate(self._active_host()) if a]
        if len(kept) == before:
            # Nothing was released: every gather below would be the identity,
            # so only the checks and the position update remain.
            keep = torch.arange(before, device=self.device)
            for state in self.sdm_states:
                self._heads(state, before)
            if not before:
                self.position = 0
            elif self.positions is not None:
                self.position = self._max_position()
            return keep
        keep = torch.tensor(kept, dtype=torch.int64).to(self.device)
        if before:
            retain_layers(self.sdm_states,
                          _banks_per_state(keep, [self._heads(st, before) for st in self.sdm_states], kept))
        self.dense_keys = tuple(t[keep].contiguous() for t in self.dense_keys)
        self.dense_values = tuple(t[keep].contiguous() for t in self.dense_values)
        if self.positions is not None:
            self.positions = self.positions[keep].contiguous()
        self._set_active(torch.ones(keep.numel(), device=self.device, dtype=torch.bool), [True] * keep.numel())
        # With one shared position the survivors keep it; otherwise the
        # largest survivor position (one read).
        self.position = (self._max_position() if self.positions is not None else self.position) \
            if keep.numel() else 0
        return keep

    @torch.no_grad()
    def admit(self, incoming: "FaithfulSDMDecodeState") -> int:
        """Move a prefilled cohort into this state's pools (inference.py:161-206)."""
        self.compact()
        incoming.compact()
        compatible = (
            self.layout == incoming.layout and self.capacity == incoming.capacity
            and self.activation_dtype == incoming.activation_dtype and self.device == incoming.device
            and self.sdm_layer_positions == incoming.sdm_layer_positions
            and len(self.sdm_states) == len(incoming.sdm_states)
            and len(self.dense_keys) == len(incoming.dense_keys)
        )
        if not compatible:
            raise ValueError("admitted faithful-SDM state is incompatible")
        append_layers(self.sdm_states, incoming.sdm_states)
        self.dense_keys = tuple(torch.cat(p, dim=0).contiguous() for p in zip(self.dense_keys, incoming.dense_keys))
        self.dense_values = tuple(torch.cat(p, dim=0).contiguous()
                                  for p in zip(self.dense_values, incoming.dense_values))
        total = self.batch + incoming.batch
        if self.positions is None and incoming.positions is None and self.batch and incoming.batch:
            # Both sides hold one position each: known on the host.
            if self.position != incoming.position:
                self.positions = torch.cat((self.current_positions(), incoming.current_positions())).contiguous()
                self.position = max(self.position, incoming.position)
            self._set_active(torch.ones(total, device=self.device, dtype=torch.bool), [True] * total)
            return incoming.batch
        merged = torch.cat((self.current_positions(), incoming.current_positions())).contiguous()
        self._set_active(torch.ones(merged.numel(), device=self.device, dtype=torch.bool), [True] * total)
        if merged.numel():
            # all positions equal <=> min == max; one read for both
            lo, hi = torch.stack((merged.min(), merged.max())).tolist()
            if lo == hi:
                self.position, self.positions = lo, None
            else:
                self.positions = merged
                self.position = hi
        else:
            self.positions = merged
        return incoming.batch

    @torch.no_grad()
    def admit_prefix(self, prefixes: Sequence[dict], *, template_indices: torch.Tensor) -> list[torch.Tensor]:
        """Prefill a cohort of requests from its SDM prefix routes and admit it in one
        step, without pools of its own: the same state as prefilling the cohort
        (``from_prefix_routes_layers``) and calling ``admit`` with it.

        ``prefixes[l]`` holds SDM layer l's ``[banks, T, ...]`` routes, values
        and gates (as for ``from_prefix_routes``); ``template_indices`` gives each
        admitted bank's head.  Every request of the cohort sits at position T.
        Only batches without attention layers (no K/V caches to extend) take
        this path.  Returns each SDM layer's readings ``[banks, T, width]``.
        """
        if self.dense_keys or self.dense_values:
            raise ValueError("batches with attention layers admit prefilled cohorts through admit()")
        if len(prefixes) != len(self.sdm_states):
            raise ValueError("one prefix per SDM layer")
        self.compact()
        heads = self._heads(self.sdm_states[0], self.batch) if self.batch else None
        banks, time = prefixes[0]["write_indices"].shape[:2]
        if heads is None:
            if template_indices.numel() == 0:
                heads = 1
            else:
                heads = int(template_indices.max().item()) + 1 if banks else 1
        if banks % heads:
            raise ValueError("admitted SDM banks do not divide by the batch's heads")
        readings = admit_prefix_routes_layers(self.sdm_states, prefixes, template_indices=template_indices)
        incoming = banks // heads
        before = self.batch
        total = before + incoming
        if before == 0:
            self.position, self.positions = time, None
        elif self.positions is None and self.position == time:
            pass
        else:
            cohort = torch.full((incoming,), time, device=self.device, dtype=torch.int64)
            self.positions = torch.cat((self.current_positions(), cohort)).contiguous()
            self.position = max(self.position, time)
        self._set_active(torch.ones(total, device=self.device, dtype=torch.bool), [True] * total)
        return readings

    def _max_position(self) -> int:
        """``int(positions.max())``, read again only when the positions tensor was
        replaced or changed in place since the last read."""
        pos = self.positions
        cached = self.__dict__.get("_max_position_of")
        if cached is not None and cached[0] is pos and cached[1] == pos._version:
            return cached[2]
        value = int(pos.max().item())
        self.__dict__["_max_position_of"] = (pos, pos._version, value)  # holds the tensor: its identity stays unique
        return value

    @torch.no_grad()
    def trim_sdm_pools(self, *, headroom_rows: int = 0) -> int:
        return sum(state.trim_capacity(headroom_rows=headroom_rows) for state in self.sdm_states)

    @torch.no_grad()
    def release_and_compact(self, sequence_indices=None, *, trim: bool = False, trim_headroom_rows: int = 0) -> int:
        released = self.release(sequence_indices)
        self.compact()
        if trim:
            self.trim_sdm_pools(headroom_rows=trim_headroom_rows)
        return released

    def storage_bytes(self) -> dict[str, int]:
        """Private live/reserved SDM state, shared M0 and dense K/V (inference.py:233-276 keys)."""
        live_values = metadata = reserved = shared = logical = 0
        for state in self.sdm_states:
            used, stored = state.used_bytes(), state.storage_bytes()
            live_values += used["live_value_bytes"]
            metadata += used["allocator_metadata_bytes"]
            reserved += stored["private_allocator_reserved_total"]
            shared += _nbytes(state.shared_initial_memory)
            logical += state.banks * state.slots * state.width * 4
        caches = (*self.dense_keys, *self.dense_values)
        kv_allocated = sum(_nbytes(t) for t in caches)
        kv_live = sum(t[:, :, : self.position].numel() * t.element_size() for t in caches)
        lifecycle = _nbytes(self.active_sequences) + (0 if self.positions is None else _nbytes(self.positions))
        return {
            "sdm_private_value_live": live_values,
            "sdm_private_allocator_metadata": metadata,
            "sdm_private_live_total": live_values + metadata,
            "sdm_private_reserved_total": reserved,
            "sdm_logical_dense_fp32": logical,
            "sdm_shared_initial_memory": shared,
            "dense_kv_live": kv_live,
            "dense_kv_allocated": kv_allocated,
            "lifecycle": lifecycle,
            "per_user_live_total_excluding_shared": live_values + metadata + kv_live + lifecycle,
            "total_reserved_excluding_shared": reserved + kv_allocated + lifecycle,
        }


def _check_controller(module) -> None:
    if not isinstance(module, SparseDeltaMemory):
        raise TypeError("packed serving requires the native SDM controller")


def _kv_cache(key: torch.Tensor, value: torch.Tensor, capacity: int):
    """Fixed-capacity K/V cache (reference inference.py:293-306), zero-filled.

    The per-request-position decode attends over ``max(position)+1`` cache
    slots and masks the unwritten ones; masking cannot neutralise NaN/Inf
    bit patterns left in uninitialised memory, so unwritten slots hold 0.
    """
    batch, heads, time, hw = key.shape
    if value.shape != key.shape or capacity < time:
        raise ValueError("dense prefill cache capacity is invalid")
    kc = key.new_zeros(batch, heads, capacity, hw)
    vc = value.new_zeros(batch, heads, capacity, hw)
    kc[:, :, :time].copy_(key)
    vc[:, :, :time].copy_(value)
    return kc, vc


@torch.no_grad()
def prefill_faithful_sdm_stack(stack: "SDMDecoderStack", tokens: torch.Tensor, *, capacity: int | None = None,
                               sdm_capacity_rows: int | Sequence[int] | None = None,
                               sdm_growth_quantum_rows: int = 0):
    """Full prefix through the stack; every "B" layer hands its written rows to a pool (inference.py:369-456).

    Pool sizing follows the reference's ``_pack_prefill_layer``
    (inference.py:353-366): with a growth quantum the pool holds the written
    rows rounded up to whole quanta; without one it is proven for the whole
    remaining trace, ``B*H*W*(capacity - T)`` first touches.
    """
    if tokens.ndim != 3 or tokens.shape[-1] != stack.width:
        raise ValueError(f"tokens must be [B,T,{stack.width}]")
    if stack.training:
        raise ValueError("faithful SDM prefill requires stack.eval()")
    batch, time, _ = tokens.shape
    if time <= 0:
        raise ValueError("prefill requires at least one token")
    cap = time if capacity is None else capacity
    if cap < time:
        raise ValueError("prefill capacity is shorter than the prefix")
    if sdm_growth_quantum_rows < 0:
        raise ValueError("SDM growth quantum cannot be negative")
    b_layers = tuple(i for i, kind in enumerate(stack.layout) if kind == "B")
    if isinstance(sdm_capacity_rows, Sequence) and not isinstance(sdm_capacity_rows, (str, bytes)):
        per_layer = tuple(int(v) for v in sdm_capacity_rows)
        if len(per_layer) != len(b_layers):
            raise ValueError("SDM capacities must contain one value per B layer")
    else:
        per_layer = (sdm_capacity_rows,) * len(b_layers)

    keys, values, pools = [], [], []
    for i, kind in enumerate(stack.layout):
        if kind == "A":
            block = stack.attention_layers[str(i)]
            attended, k, v = block.attention.prefill_with_cache(tokens)
            tokens = tokens + attended
            tokens = tokens + block.mlp(tokens)
            kc, vc = _kv_cache(k, v, cap)
            keys.append(kc)
            values.append(vc)
            continue
        module = stack.sdm_layers[str(i)]
        _check_controller(module)
        future = None if sdm_growth_quantum_rows else batch * module.memory_heads * module.writes * (cap - time)
        mixed, pool = module.prefill(tokens, capacity_rows=per_layer[len(pools)],
                                     maximum_future_allocations=future,
                                     growth_quantum_rows=sdm_growth_quantum_rows)
        tokens = tokens + mixed
        tokens = tokens + stack.sdm_mlps[str(i)](tokens)
        pools.append(pool)
    return tokens, FaithfulSDMDecodeState(
        layout=stack.layout, position=time, capacity=cap, activation_dtype=tokens.dtype,
        active_sequences=torch.ones(batch, device=tokens.device, dtype=torch.bool),
        sdm_layer_positions=b_layers, sdm_states=tuple(pools), dense_keys=tuple(keys),
        dense_values=tuple(values))


def _one_token(module: SparseDeltaMemory, tokens: torch.Tensor):
    _check_controller(module)
    if tokens.shape != (tokens.shape[0], 1, module.width):
        raise ValueError("faithful SDM decode requires one token")
    return module.controller(tokens)


def _step_kwargs(step) -> dict:
    return dict(write_indices=step.write_indices[:, 0], write_weights=step.write_weights[:, 0],
                values=step.values[:, 0], input_gate=step.input_gate[:, 0],
                forget_log_gate=step.forget_log_gate[:, 0], read_indices=step.read_indices[:, 0],
                read_weights=step.read_weights[:, 0])


@torch.no_grad()
def _decode_faithful_sdm_layer(module: SparseDeltaMemory, tokens: torch.Tensor,
                               state: PackedSDMCopyOnWriteState, *, backend: str = "auto",
                               mlp: nn.Module | None = None) -> torch.Tensor:
    """One token through one SDM layer and its pool (inference.py:538-566).  Returns the
    layer's mixed output; with ``mlp`` given, the residual stream after the layer and
    that MLP block (inference.py:655-661) instead."""
    step = _one_token(module, tokens)
    if state.banks != tokens.shape[0] * module.memory_heads:
        raise ValueError("packed SDM banks do not match batch and memory heads")
    if state.growth_quantum_rows:
        state.prepare_step_capacity(state.banks * module.writes)
    reading, _ = packed_sdm_cow_step(state, **_step_kwargs(step), backend=backend, validate_routes=False,
                                     collect_diagnostics=False)
    if mlp is not None:
        return module.finish_residual(tokens, step.normalized, reading[:, None], mlp)
    return module.finish(step.normalized, reading[:, None])


@torch.no_grad()
def _decode_faithful_sdm_layer_dense(module: SparseDeltaMemory, tokens: torch.Tensor, memory: torch.Tensor, *,
                                     backend: str = "auto") -> torch.Tensor:
    """Dense-table control with the same controller (inference.py:569-598)."""
    step = _one_token(module, tokens)
    if memory.shape != (tokens.shape[0] * module.memory_heads, module.slots, module.head_width):
        raise ValueError("dense SDM memory does not match batch and controller")
    reading = dense_sdm_sparse_step(memory, **_step_kwargs(step), backend=backend, validate_routes=False)
    return module.finish(step.normalized, reading[:, None])


@torch.no_grad()
def decode_faithful_sdm_stack(stack: "SDMDecoderStack", tokens: torch.Tensor,
                              state: FaithfulSDMDecodeState) -> torch.Tensor:
    """Consume one token per request through K/V caches and packed pools (inference.py:601-669)."""
    if tokens.shape != (state.batch, 1, stack.width):
        raise ValueError(f"decode tokens must be [{state.batch},1,{stack.width}]")
    if stack.training:
        raise ValueError("faithful SDM decode requires stack.eval()")
    if state.layout != stack.layout:
        raise ValueError("decode state layout does not match the stack")
    if tokens.device != state.device or tokens.dtype != state.dtype:
        raise ValueError("decode tokens do not match state device and dtype")
    positions = state.current_positions()
    if state.positions is None:
        if state.position >= state.capacity:
            raise ValueError("decode state has reached its fixed capacity")
        where: int | torch.Tensor = state.position
    else:
        if bool((positions >= state.capacity).any()):
            raise ValueError("decode state has reached its fixed capacity")
        where = positions
    if not bool(state.active_sequences.all()):
        raise ValueError("released requests must be removed before further decode")
    n_b, n_a = stack.layout.count("B"), stack.layout.count("A")
    if (len(state.sdm_states) != n_b or len(state.sdm_layer_positions) != n_b
            or len(state.dense_keys) != n_a or len(state.dense_values) != n_a):
        raise ValueError("decode state does not match the stack")
    a_i = b_i = 0
    for i, kind in enumerate(stack.layout):
        if kind == "A":
            block = stack.attention_layers[str(i)]
            tokens = block.decode_residual(tokens, state.dense_keys[a_i], state.dense_values[a_i], where)
            a_i += 1
            continue
        if state.sdm_layer_positions[b_i] != i:
            raise ValueError("SDM decode layer ordering is inconsistent")
        tokens = _decode_faithful_sdm_layer(stack.sdm_layers[str(i)], tokens, state.sdm_states[b_i],
                                            mlp=stack.sdm_mlps[str(i)])
        b_i += 1
    if state.positions is None:
        state.position += 1
    else:
        positions.add_(1)
        state.positions = positions
        state.position = int(positions.max().item())
    return tokens
