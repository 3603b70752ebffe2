"""Generate golden vectors by running the REFERENCE implementation on CPU.

Run from the repository root in a container where the reference project is
available (it is not shipped with this repository):

    PYTHONPATH=<path to copy-on-write-sdm> python tests/golden/make_golden.py

Every case drives the reference's own public API (``PackedSDMCopyOnWriteState``,
``packed_sdm_cow_step(backend="torch")``, ``dense_sdm_sparse_step``, the
lifecycle methods and ``serial_gated_delta_recurrence``) on seeded inputs and
stores inputs and outputs as ``.npz`` files next to this script.  The tests
read only the ``.npz`` files, so they run where the reference is absent.

Recorded environment: torch version and seeds are stored in each file under
``meta_*`` keys.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

from copy_on_write_sdm.allocator import (  # noqa: E402  (reference package)
    PackedSDMCopyOnWriteState,
    dense_sdm_sparse_step,
    packed_sdm_cow_step,
)
from copy_on_write_sdm.sdm import serial_gated_delta_recurrence  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().copy()


def _routes(g: torch.Generator, banks: int, slots: int, k: int) -> torch.Tensor:
    return torch.stack([torch.randperm(slots, generator=g)[:k] for _ in range(banks)])


def _step_inputs(g: torch.Generator, banks: int, slots: int, width: int, W: int, R: int):
    return dict(
        write_indices=_routes(g, banks, slots, W),
        write_weights=torch.softmax(torch.randn(banks, W, generator=g), dim=-1),
        values=torch.randn(banks, width, generator=g),
        input_gate=torch.rand(banks, generator=g),
        forget_log_gate=-torch.rand(banks, generator=g),
        read_indices=_routes(g, banks, slots, R),
        read_weights=torch.softmax(torch.randn(banks, R, generator=g), dim=-1),
    )


def _snapshot(prefix: str, st: PackedSDMCopyOnWriteState, out: dict) -> None:
    fc = int(st.free_count)
    active = st.logical_to_physical >= 0
    bank, slot = active.nonzero(as_tuple=True)
    out[f"{prefix}map"] = _np(st.logical_to_physical)
    out[f"{prefix}free_stack"] = _np(st.free_rows[:fc])
    out[f"{prefix}free_count"] = np.int64(fc)
    out[f"{prefix}capacity"] = np.int64(st.capacity_rows)
    out[f"{prefix}live_rows"] = _np(st.values[st.logical_to_physical[bank, slot].long()])
    out[f"{prefix}templates"] = _np(st.template_indices)
    out[f"{prefix}counters"] = np.array(
        [
            st.growth_events,
            st.growth_rows_added,
            st.growth_rows_copied,
            st.proven_maximum_additional_allocations,
            int(st.capacity_is_proven),
        ],
        dtype=np.int64,
    )


def _save(name: str, out: dict, seed: int) -> None:
    out["meta_torch"] = np.array(torch.__version__)
    out["meta_seed"] = np.int64(seed)
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def decode_trace(name, *, seed, banks, slots, width, W, R, steps, capacity, heads=1):
    """Packed steps from ``allocate`` with the dense control on the same routes."""
    g = torch.Generator().manual_seed(seed)
    m0 = 0.02 * torch.randn(heads, slots, width, generator=g)
    templates = torch.arange(heads).repeat(banks // heads)
    st = PackedSDMCopyOnWriteState.allocate(
        m0, banks=banks, capacity_rows=capacity, template_indices=templates
    )
    dense = m0[templates].clone()
    out = {"m0": _np(m0), "templates": _np(templates), "capacity0": np.int64(capacity)}
    keys = ("write_indices", "write_weights", "values", "input_gate", "forget_log_gate",
            "read_indices", "read_weights")
    rec = {k: [] for k in keys}
    readings, dense_readings, maps, free_counts, first = [], [], [], [], []
    for _ in range(steps):
        x = _step_inputs(g, banks, slots, width, W, R)
        for k in keys:
            rec[k].append(_np(x[k]))
        d = dense_sdm_sparse_step(dense, **x, backend="torch")
        r, diag = packed_sdm_cow_step(st, **x, backend="torch")
        assert torch.equal(d, r)
        assert torch.equal(dense, st.materialize_dense())
        readings.append(_np(r))
        dense_readings.append(_np(d))
        maps.append(_np(st.logical_to_physical))
        free_counts.append(int(st.free_count))
        first.append(_np(diag.first_touches_by_sequence))
    for k in keys:
        out[f"in_{k}"] = np.stack(rec[k])
    out["readings"] = np.stack(readings)
    out["dense_readings"] = np.stack(dense_readings)
    out["maps"] = np.stack(maps)
    out["free_counts"] = np.array(free_counts, dtype=np.int64)
    out["first_by_bank"] = np.stack(first)
    if dense.numel() <= 65536:
        out["final_dense"] = _np(dense)
    _snapshot("final_", st, out)
    st.validate_invariants()
    _save(name, out, seed)


def lifecycle_trace(name, *, seed=5):
    """Growth, release, compaction, admission and trim on a two-template pool."""
    heads, slots, width, W, R = 2, 16, 8, 3, 5
    g = torch.Generator().manual_seed(seed)
    m0 = torch.randn(heads, slots, width, generator=g)
    requests = 3
    banks = requests * heads
    templates = torch.arange(heads).repeat(requests)
    quantum = 8
    st = PackedSDMCopyOnWriteState.allocate(
        m0, banks=banks, capacity_rows=quantum, template_indices=templates,
        growth_quantum_rows=quantum,
    )
    out = {"m0": _np(m0), "templates": _np(templates), "quantum": np.int64(quantum)}
    ops = []

    def step(tag, nb):
        x = _step_inputs(g, nb, slots, width, W, R)
        st.prepare_step_capacity(nb * W)
        r, _ = packed_sdm_cow_step(st, **x, backend="torch", collect_diagnostics=False)
        for k, v in x.items():
            out[f"{tag}_in_{k}"] = _np(v)
        out[f"{tag}_reading"] = _np(r)
        _snapshot(f"{tag}_", st, out)
        st.validate_invariants()
        ops.append(tag)

    for i in range(4):
        step(f"s{i}", banks)
    # Release request 1 (banks 2, 3) in descending bank order to pin push order.
    rel = torch.tensor([3, 2])
    out["release_banks"] = _np(rel)
    out["release_count"] = np.int64(int(st.release(rel)))
    _snapshot("rel_", st, out)
    ops.append("rel")
    keep = torch.tensor([0, 1, 4, 5])
    st.retain_banks(keep)
    out["retain_banks"] = _np(keep)
    _snapshot("ret_", st, out)
    ops.append("ret")
    # Admit a cohort of 2 requests packed from a dense overlay.
    nb2 = 2 * heads
    dense2 = torch.randn(nb2, slots, width, generator=g)
    active2 = torch.rand(nb2, slots, generator=g) < 0.3
    t2 = torch.arange(heads).repeat(2)
    other = PackedSDMCopyOnWriteState.from_dense_overlay(
        m0, dense2, active2, template_indices=t2, growth_quantum_rows=quantum
    )
    out["cohort_dense"] = _np(dense2)
    out["cohort_active"] = _np(active2)
    out["cohort_templates"] = _np(t2)
    _snapshot("other_", other, out)
    out["adm_count"] = np.int64(st.append_banks_from(other))
    _snapshot("adm_", st, out)
    st.validate_invariants()
    ops.append("adm")
    for i in range(4, 6):
        step(f"s{i}", st.banks)
    # Release a middle request, then trim with headroom.
    st.release(torch.tensor([4, 5]))
    st.retain_banks(torch.tensor([0, 1, 2, 3, 6, 7]))
    out["trim_removed"] = np.int64(st.trim_capacity(headroom_rows=3))
    _snapshot("trim_", st, out)
    st.validate_invariants()
    ops.append("trim")
    step("s6", st.banks)
    out["materialized"] = _np(st.materialize_dense())
    out["ops"] = np.array(ops)
    _save(name, out, seed)


def prefill_handoff(name, *, seed=3):
    """Reference prefill: dense serial recurrence + ``from_dense_overlay`` of the write union."""
    B, H, T, slots, width, W, R = 2, 2, 24, 64, 16, 4, 8
    banks = B * H
    g = torch.Generator().manual_seed(seed)
    m0 = 0.05 * torch.randn(H, slots, width, generator=g)
    templates = torch.arange(H).repeat(B)
    widx = torch.stack([_routes(g, banks, slots, W) for _ in range(T)], dim=1)
    ridx = torch.stack([_routes(g, banks, slots, R) for _ in range(T)], dim=1)
    ww = torch.softmax(torch.randn(banks, T, W, generator=g), dim=-1)
    rw = torch.softmax(torch.randn(banks, T, R, generator=g), dim=-1)
    values = torch.randn(banks, T, width, generator=g)
    in_g = torch.rand(banks, T, generator=g)
    fl = -torch.rand(banks, T, generator=g)
    write_routes = torch.zeros(banks, T, slots).scatter(-1, widx, ww)
    read_routes = torch.zeros(banks, T, slots).scatter(-1, ridx, rw)
    readings, final_memory, _ = serial_gated_delta_recurrence(
        m0[templates], write_routes, values, in_g, fl, read_routes
    )
    active = torch.zeros(banks, slots, dtype=torch.bool).scatter(
        1, widx.reshape(banks, T * W), True
    )
    quantum = 32
    st = PackedSDMCopyOnWriteState.from_dense_overlay(
        m0, final_memory, active, template_indices=templates, growth_quantum_rows=quantum
    )
    out = {
        "m0": _np(m0), "templates": _np(templates), "in_write_indices": _np(widx),
        "in_read_indices": _np(ridx), "in_write_weights": _np(ww), "in_read_weights": _np(rw),
        "in_values": _np(values), "in_input_gate": _np(in_g), "in_forget_log_gate": _np(fl),
        "readings": _np(readings), "final_memory": _np(final_memory), "active": _np(active),
        "quantum": np.int64(quantum),
    }
    _snapshot("final_", st, out)
    _save(name, out, seed)


def model_lifecycle(name, *, seed=0):
    """Whole reference model: prefill handoff, decode, release/compact, admit, trim."""
    from copy_on_write_sdm.model import LanguageModel

    torch.manual_seed(seed)
    model = LanguageModel(vocab_size=97, maximum_sequence_length=40, layout="BABB", width=32, heads=2,
                          slots=16, reads=4, writes=2, memory_heads=2, activation_dtype=torch.float32)
    model.initialize_role_keyed(seed)
    model.eval()
    g = torch.Generator().manual_seed(seed + 1)
    out = {f"param_{k}": _np(v) for k, v in model.state_dict().items()}
    prefix = torch.randint(97, (3, 10), generator=g)
    out["prefix"] = _np(prefix)
    with torch.no_grad():
        logits, state = model.prefill(prefix, capacity=24, sdm_growth_quantum_rows=8)
        out["prefill_logits"] = _np(logits)
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"prefill_l{i}_", st, out)
        steps = torch.randint(97, (6, 3, 1), generator=g)
        out["decode_ids"] = _np(steps)
        for t in range(6):
            out[f"decode{t}_logits"] = _np(model.decode(steps[t], state))
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"decoded_l{i}_", st, out)
        out["released_rows"] = np.int64(state.release_and_compact([1]))
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"compact_l{i}_", st, out)
        cohort = torch.randint(97, (2, 4), generator=g)
        out["cohort"] = _np(cohort)
        out["admit_logits"] = _np(model.admit(cohort, state))
        # The reference allocates its K/V caches with torch.empty.  After this
        # admission the per-request-position decode attends over slots that
        # no token wrote (masked with -inf), and NaN bit patterns there turn
        # whole rows into NaN.  Zero the never-written slots so the recorded
        # trajectory is the well-defined one.
        for cache in (*state.dense_keys, *state.dense_values):
            for b, pos in enumerate(state.current_positions().tolist()):
                cache[b, :, pos:].zero_()
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"admit_l{i}_", st, out)
        out["admit_positions"] = _np(state.current_positions())
        steps2 = torch.randint(97, (3, 4, 1), generator=g)
        out["decode2_ids"] = _np(steps2)
        for t in range(3):
            out[f"decode2_{t}_logits"] = _np(model.decode(steps2[t], state))
        out["trimmed_rows"] = np.int64(state.trim_sdm_pools(headroom_rows=4))
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"trim_l{i}_", st, out)
        sb = state.storage_bytes()
        out["storage_keys"] = np.array(sorted(sb))
        out["storage_vals"] = np.array([sb[k] for k in sorted(sb)], dtype=np.int64)
        out["final_positions"] = _np(state.current_positions())
    _save(name, out, seed)


def model_config2(name, *, seed=2):
    """Configuration-2-shaped reference model (vocab 50,257, layout BBBBBBBA,
    width 128, N=256, H=1, top-16/top-4) with seeded weights shared with the
    test (``config2_weights.py``): prefill, then decode steps.  Logits are
    stored for a seeded subset of 4,096 vocabulary columns plus every row's
    argmax (the full logits would be 200 KB per row)."""
    from copy_on_write_sdm.model import LanguageModel

    sys.path.insert(0, HERE)
    from config2_weights import VOCAB, model_kwargs, seeded_params

    model = LanguageModel(**model_kwargs(), activation_dtype=torch.float32)
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict({k: torch.from_numpy(v) for k, v in seeded_params(shapes, seed).items()}, strict=True)
    model.eval()
    g = torch.Generator().manual_seed(seed + 1)
    cols = torch.randperm(VOCAB, generator=g)[:4096].sort().values
    out = {"columns": _np(cols)}

    def keep(prefix, logits):
        flat = logits.reshape(-1, VOCAB)
        out[prefix + "_logits"] = _np(flat[:, cols])
        out[prefix + "_argmax"] = _np(flat.argmax(-1))

    prefix = torch.randint(VOCAB, (2, 12), generator=g)
    out["prefix"] = _np(prefix)
    with torch.no_grad():
        logits, state = model.prefill(prefix, capacity=24, sdm_growth_quantum_rows=64)
        keep("prefill", logits[:, -1:])
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"prefill_l{i}_", st, out)
        steps = torch.randint(VOCAB, (4, 2, 1), generator=g)
        out["decode_ids"] = _np(steps)
        for t in range(4):
            keep(f"decode{t}", model.decode(steps[t], state))
        for i, st in enumerate(state.sdm_states):
            _snapshot(f"decoded_l{i}_", st, out)
    _save(name, out, seed)


def main() -> None:
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    # Configuration 1: H=1, N=256, D=128, top-16/top-4, seed 0, B=1, prefix 16 + 32 decode.
    decode_trace("cfg1_decode", seed=0, banks=1, slots=256, width=128, W=4, R=16,
                 steps=48, capacity=256)
    # Reference unit-test shape (tests/test_allocator.py:14-27): B=3, N=16, D=8.
    decode_trace("small_decode", seed=11, banks=3, slots=16, width=8, W=2, R=4,
                 steps=6, capacity=48)
    # Multi-bank, multi-template trace at a configuration-3-like bank count.
    decode_trace("multibank_decode", seed=7, banks=64, slots=64, width=32, W=4, R=16,
                 steps=12, capacity=64 * 64, heads=4)
    lifecycle_trace("lifecycle")
    prefill_handoff("prefill_handoff")
    model_lifecycle("model_lifecycle")
    model_config2("model_config2")


if __name__ == "__main__":
    sys.exit(main())
