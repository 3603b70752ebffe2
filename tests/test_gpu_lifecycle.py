"""GPU parity of the allocator lifecycle: growth, release, compaction,
admission, trimming and the prefill handoff (golden traces from the reference)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

ATOL = 1e-5
RTOL = 1e-5
KEYS = ("write_indices", "write_weights", "values", "input_gate", "forget_log_gate",
        "read_indices", "read_weights")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def cu(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def assert_golden_state(st, g, prefix):
    np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), g[f"{prefix}map"])
    fc = int(st.free_count)
    assert fc == int(g[f"{prefix}free_count"])
    np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), g[f"{prefix}free_stack"])
    assert st.capacity_rows == int(g[f"{prefix}capacity"])
    np.testing.assert_array_equal(st.template_indices.cpu().numpy(), g[f"{prefix}templates"])
    mp = st.logical_to_physical.cpu().numpy()
    b, s = np.nonzero(mp >= 0)
    np.testing.assert_allclose(st.values.cpu().numpy()[mp[b, s]], g[f"{prefix}live_rows"], atol=ATOL, rtol=RTOL)
    counters = [st.growth_events, st.growth_rows_added, st.growth_rows_copied,
                st.proven_maximum_additional_allocations, int(st.capacity_is_proven)]
    np.testing.assert_array_equal(counters, g[f"{prefix}counters"])


def test_golden_lifecycle(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    g = load("lifecycle")
    q = int(g["quantum"])
    m0 = cu(g["m0"], dev)
    st = PackedSDMCopyOnWriteState.allocate(m0, banks=g["templates"].shape[0], capacity_rows=q,
                                            template_indices=cu(g["templates"], dev), growth_quantum_rows=q)
    W = g["s0_in_write_indices"].shape[1]

    def step(tag):
        x = {k: cu(g[f"{tag}_in_{k}"], dev) for k in KEYS}
        st.prepare_step_capacity(st.banks * W)
        r, _ = packed_sdm_cow_step(st, **x, collect_diagnostics=False)
        np.testing.assert_allclose(r.cpu().numpy(), g[f"{tag}_reading"], atol=ATOL, rtol=RTOL)
        assert_golden_state(st, g, f"{tag}_")
        st.validate_invariants()

    for i in range(4):
        step(f"s{i}")
    assert int(st.release(cu(g["release_banks"], dev))) == int(g["release_count"])
    assert_golden_state(st, g, "rel_")
    st.retain_banks(cu(g["retain_banks"], dev))
    assert_golden_state(st, g, "ret_")
    other = PackedSDMCopyOnWriteState.from_dense_overlay(
        m0, cu(g["cohort_dense"], dev), cu(g["cohort_active"], dev),
        template_indices=cu(g["cohort_templates"], dev), growth_quantum_rows=q)
    assert_golden_state(other, g, "other_")
    assert st.append_banks_from(other) == int(g["adm_count"])
    assert_golden_state(st, g, "adm_")
    st.validate_invariants()
    for i in range(4, 6):
        step(f"s{i}")
    st.release(torch.tensor([4, 5], device=dev))
    st.retain_banks(torch.tensor([0, 1, 2, 3, 6, 7], device=dev))
    assert st.trim_capacity(headroom_rows=3) == int(g["trim_removed"])
    assert_golden_state(st, g, "trim_")
    st.validate_invariants()
    step("s6")
    np.testing.assert_allclose(st.materialize_dense().cpu().numpy(), g["materialized"], atol=ATOL, rtol=RTOL)


def test_golden_prefill_handoff_sparse(dev):
    """Sparse prefill (no [B,T,N,D] states) == reference dense recurrence + from_dense_overlay."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    g = load("prefill_handoff")
    st, readings = PackedSDMCopyOnWriteState.from_prefix_routes(
        cu(g["m0"], dev), cu(g["in_write_indices"], dev), cu(g["in_write_weights"], dev),
        cu(g["in_values"], dev), cu(g["in_input_gate"], dev), cu(g["in_forget_log_gate"], dev),
        cu(g["in_read_indices"], dev), cu(g["in_read_weights"], dev),
        template_indices=cu(g["templates"], dev), growth_quantum_rows=int(g["quantum"]))
    np.testing.assert_allclose(readings.cpu().numpy(), g["readings"], atol=ATOL, rtol=RTOL)
    assert_golden_state(st, g, "final_")
    np.testing.assert_allclose(st.materialize_dense().cpu().numpy(), g["final_memory"], atol=ATOL, rtol=RTOL)


def test_golden_prefill_handoff_dense_overlay(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    g = load("prefill_handoff")
    st = PackedSDMCopyOnWriteState.from_dense_overlay(
        cu(g["m0"], dev), cu(g["final_memory"], dev), cu(g["active"], dev),
        template_indices=cu(g["templates"], dev), growth_quantum_rows=int(g["quantum"]))
    assert_golden_state(st, g, "final_")


def test_release_edge_cases(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    rng = np.random.default_rng(2)
    banks, slots, width = 6, 32, 16
    m0 = rng.standard_normal((1, slots, width)).astype(np.float32)
    dense = rng.standard_normal((banks, slots, width)).astype(np.float32)
    active = rng.random((banks, slots)) < 0.4
    active[3] = False  # a bank with no private rows
    tmpl = np.zeros(banks, np.int64)
    st = PackedSDMCopyOnWriteState.from_dense_overlay(cu(m0, dev), cu(dense, dev), cu(active, dev),
                                                      template_indices=cu(tmpl, dev), growth_quantum_rows=16)
    ref = O.from_dense_overlay(m0, dense, active, template_indices=tmpl, growth_quantum_rows=16)
    assert int(st.release(torch.empty(0, dtype=torch.int64, device=dev))) == 0
    for sel in ([5, 0], [3], [1, 2, 4]):
        assert int(st.release(torch.tensor(sel, device=dev))) == O.release(ref, sel)
        np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), ref.logical_to_physical)
        fc = int(st.free_count)
        assert fc == ref.free_count
        np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), ref.free_stack())
        st.validate_invariants()
    # everything released: trimming returns to one quantum
    assert st.trim_capacity() == O.trim_capacity(ref)
    assert st.capacity_rows == ref.capacity_rows == 16
    # a bad bank list releases nothing and is reported by validate_invariants
    st.release(torch.tensor([1, 1], device=dev))
    with pytest.raises(AssertionError, match="invalid or duplicated"):
        st.validate_invariants()


def test_retain_errors(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    m0 = torch.zeros(1, 8, 4, device=dev)
    dense = torch.ones(3, 8, 4, device=dev)
    active = torch.zeros(3, 8, dtype=torch.bool, device=dev)
    active[1, 2] = True
    st = PackedSDMCopyOnWriteState.from_dense_overlay(m0, dense, active,
                                                      template_indices=torch.zeros(3, dtype=torch.int64, device=dev))
    with pytest.raises(ValueError, match="released before compaction"):
        st.retain_banks(torch.tensor([0, 2], device=dev))
    with pytest.raises(ValueError, match="invalid or duplicated"):
        st.retain_banks(torch.tensor([0, 0], device=dev))
    st.retain_banks(torch.tensor([1], device=dev))
    assert st.banks == 1 and int((st.logical_to_physical >= 0).sum()) == 1
    st.validate_invariants()
