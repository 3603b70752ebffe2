"""Pin the CPU oracle against golden vectors produced by the reference itself.

Allocator state (maps, free stacks, counts, counters) must match bit for bit;
slab rows and readouts within 1e-5 abs / 1e-5 rel (FP32).
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import cow_oracle as O
from tests.conftest import GOLDEN

ATOL = 1e-5
RTOL = 1e-5
STEP_KEYS = ("write_indices", "write_weights", "values", "input_gate", "forget_log_gate",
             "read_indices", "read_weights")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def assert_state(st: O.OracleState, g: dict, prefix: str) -> None:
    np.testing.assert_array_equal(st.logical_to_physical, g[f"{prefix}map"])
    np.testing.assert_array_equal(st.free_stack(), g[f"{prefix}free_stack"])
    assert st.free_count == int(g[f"{prefix}free_count"])
    assert st.capacity_rows == int(g[f"{prefix}capacity"])
    np.testing.assert_array_equal(st.template_indices, g[f"{prefix}templates"])
    np.testing.assert_allclose(st.live_rows(), g[f"{prefix}live_rows"], atol=ATOL, rtol=RTOL)
    counters = [st.growth_events, st.growth_rows_added, st.growth_rows_copied,
                st.proven_maximum_additional_allocations, int(st.capacity_is_proven)]
    np.testing.assert_array_equal(counters, g[f"{prefix}counters"])


@pytest.mark.parametrize("name", ["cfg1_decode", "small_decode", "multibank_decode"])
def test_decode_trace(name):
    g = load(name)
    banks = g["templates"].shape[0]
    st = O.allocate(g["m0"], banks=banks, capacity_rows=int(g["capacity0"]),
                    template_indices=g["templates"])
    dense = g["m0"][g["templates"]].copy()
    steps = g["readings"].shape[0]
    for t in range(steps):
        x = {k: g[f"in_{k}"][t] for k in STEP_KEYS}
        reading, first = O.packed_step(st, **x)
        d_reading = O.dense_step(dense, **x)
        np.testing.assert_allclose(reading, g["readings"][t], atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(d_reading, g["dense_readings"][t], atol=ATOL, rtol=RTOL)
        np.testing.assert_array_equal(st.logical_to_physical, g["maps"][t])
        assert st.free_count == g["free_counts"][t]
        np.testing.assert_array_equal(first.sum(axis=1), g["first_by_bank"][t])
    assert_state(st, g, "final_")
    if "final_dense" in g:
        np.testing.assert_allclose(dense, g["final_dense"], atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(O.materialize_dense(st), g["final_dense"], atol=ATOL, rtol=RTOL)
    O.validate_invariants(st)


def test_lifecycle_trace():
    g = load("lifecycle")
    q = int(g["quantum"])
    st = O.allocate(g["m0"], banks=g["templates"].shape[0], capacity_rows=q,
                    template_indices=g["templates"], growth_quantum_rows=q)
    W = g["s0_in_write_indices"].shape[1]

    def step(tag):
        x = {k: g[f"{tag}_in_{k}"] for k in STEP_KEYS}
        O.prepare_step_capacity(st, st.banks * W)
        r, _ = O.packed_step(st, **x)
        np.testing.assert_allclose(r, g[f"{tag}_reading"], atol=ATOL, rtol=RTOL)
        assert_state(st, g, f"{tag}_")
        O.validate_invariants(st)

    for i in range(4):
        step(f"s{i}")
    assert O.release(st, g["release_banks"]) == int(g["release_count"])
    assert_state(st, g, "rel_")
    O.retain_banks(st, g["retain_banks"])
    assert_state(st, g, "ret_")
    other = O.from_dense_overlay(g["m0"], g["cohort_dense"], g["cohort_active"],
                                 template_indices=g["cohort_templates"], growth_quantum_rows=q)
    assert_state(other, g, "other_")
    assert O.append_banks_from(st, other) == int(g["adm_count"])
    assert_state(st, g, "adm_")
    for i in range(4, 6):
        step(f"s{i}")
    O.release(st, [4, 5])
    O.retain_banks(st, [0, 1, 2, 3, 6, 7])
    assert O.trim_capacity(st, headroom_rows=3) == int(g["trim_removed"])
    assert_state(st, g, "trim_")
    step("s6")
    np.testing.assert_allclose(O.materialize_dense(st), g["materialized"], atol=ATOL, rtol=RTOL)


def test_sparse_prefill_matches_dense_recurrence_handoff():
    g = load("prefill_handoff")
    st, readings = O.sparse_prefill(
        g["m0"], g["templates"], g["in_write_indices"], g["in_write_weights"], g["in_values"],
        g["in_input_gate"], g["in_forget_log_gate"], g["in_read_indices"], g["in_read_weights"],
        growth_quantum_rows=int(g["quantum"]),
    )
    np.testing.assert_allclose(readings, g["readings"], atol=ATOL, rtol=RTOL)
    assert_state(st, g, "final_")
    np.testing.assert_allclose(O.materialize_dense(st), g["final_memory"], atol=ATOL, rtol=RTOL)
    np.testing.assert_array_equal(st.logical_to_physical >= 0, g["active"])


def test_overflow_and_errors_raise():
    st = O.allocate(np.zeros((1, 8, 4), np.float32), banks=2, capacity_rows=3)
    x = dict(write_indices=[[0, 1], [2, 3]], write_weights=np.full((2, 2), 0.5, np.float32),
             values=np.ones((2, 4), np.float32), input_gate=np.ones(2, np.float32),
             forget_log_gate=np.zeros(2, np.float32), read_indices=[[0], [1]],
             read_weights=np.ones((2, 1), np.float32))
    with pytest.raises(ValueError):
        O.packed_step(st, **x)
    with pytest.raises(ValueError):
        O.grow_capacity(st, 10)
    with pytest.raises(ValueError):
        O.release(st, [0, 0])
