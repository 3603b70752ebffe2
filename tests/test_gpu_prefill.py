"""GPU parity of the resolved-route prefill walk (cow_prefill_recurrence_layers_ws).

The walk that reads routes resolved by a parallel pass must give the same
rows, maps and status bits as the walk that resolves each token itself, bit
for bit, and the same readings (bit for bit on the one-warp walk, within the
test tolerance where a block of warps per bank sums partial readouts),
whether the prefix fits one chunk of records or needs several; both are pinned to the
oracle's sparse prefill (the reference's dense recurrence restricted to
written rows, sdm.py:474-529 and allocator.py:589-690).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

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


def prefix(rng, banks, tokens, slots, width, writes, reads):
    routes = lambda k: np.stack([O.uniform_routes(rng, banks, slots, k) for _ in range(tokens)], 1)
    return dict(write_indices=routes(writes),
                write_weights=O.softmax(rng.standard_normal((banks, tokens, writes), dtype=np.float32)),
                values=rng.standard_normal((banks, tokens, width), dtype=np.float32),
                input_gate=rng.random((banks, tokens), dtype=np.float32),
                forget_log_gate=-rng.random((banks, tokens), dtype=np.float32),
                read_indices=routes(reads),
                read_weights=O.softmax(rng.standard_normal((banks, tokens, reads), dtype=np.float32)))


def run(m0s, xs, templates, dev, quantum, state_dtype=torch.float32):
    from copy_on_write_sdm_b200.allocator import from_prefix_routes_layers

    states, reads = from_prefix_routes_layers(
        [cu(m, dev) for m in m0s], [{k: cu(x[k], dev) for k in KEYS} for x in xs],
        template_indices=cu(templates, dev), growth_quantum_rows=quantum, state_dtype=state_dtype)
    torch.cuda.synchronize(dev)
    return states, reads


def with_path(monkeypatch, resolved: bool, chunk_tokens: int | None = None):
    """Select the prefill walk; ``chunk_tokens`` caps the resolved walk's
    workspace at that many tokens of records, so longer prefixes run in chunks."""
    from copy_on_write_sdm_b200 import _lib, allocator

    monkeypatch.setattr(allocator, "_PREFILL_RESOLVED", resolved)
    if chunk_tokens is not None:
        lib = _lib.load()
        real = lib.cow_prefill_recurrence_layers_ws

        def capped(pools, steps, n, time, writes, reads, idx, act, ws, ws_bytes, stream):
            per_token = sum(pools[i].banks for i in range(n)) * (((4 + 3 * writes + 3 * reads) + 3) // 4 * 4) * 4
            return real(pools, steps, n, time, writes, reads, idx, act, ws, per_token * chunk_tokens, stream)

        monkeypatch.setattr(lib, "cow_prefill_recurrence_layers_ws", capped)


@pytest.mark.parametrize("slots,width,writes,reads,tokens,state_dtype", [
    (256, 128, 4, 16, 40, torch.float32),   # the serving shape (f32 rows, W <= 4, R <= 32)
    (512, 64, 8, 24, 17, torch.float32),    # W <= 8 variant, narrow rows
    (128, 256, 12, 40, 9, torch.bfloat16),  # wide routes (R > 32), two chunks per row, bf16 slab
])
def test_resolved_walk_matches_per_token_walk_and_oracle(dev, monkeypatch, slots, width, writes, reads, tokens,
                                                         state_dtype):
    rng = np.random.default_rng(slots + width + reads)
    heads, requests, layers = 2, 5, 3
    banks = heads * requests
    templates = np.tile(np.arange(heads), requests)
    m0s = [(0.02 * rng.standard_normal((heads, slots, width))).astype(np.float32) for _ in range(layers)]
    xs = [prefix(rng, banks, tokens, slots, width, writes, reads) for _ in range(layers)]
    quantum = banks * writes

    with_path(monkeypatch, False)
    old_states, old_reads = run(m0s, xs, templates, dev, quantum, state_dtype)
    results = {}
    for chunk in (None, 1, 7):
        with_path(monkeypatch, True, chunk)
        results[chunk] = run(m0s, xs, templates, dev, quantum, state_dtype)
    # Cohorts of the serving shape walk with a block of warps per bank, whose
    # partial readouts are summed in another order: readings within tolerance,
    # rows and maps bit-identical.  Other shapes: everything bit-identical.
    split = state_dtype == torch.float32 and width <= 128 and writes <= 4 and reads <= 32
    for chunk, (states, reads_) in results.items():
        for l in range(layers):
            if split:
                torch.testing.assert_close(reads_[l], old_reads[l], atol=ATOL, rtol=RTOL)
            else:
                assert torch.equal(reads_[l], old_reads[l]), f"readings differ (chunk {chunk}, layer {l})"
            assert torch.equal(states[l].logical_to_physical, old_states[l].logical_to_physical)
            live = states[l].logical_to_physical[states[l].logical_to_physical >= 0].long()
            assert torch.equal(states[l].values[live], old_states[l].values[live]), f"rows differ (chunk {chunk})"
    if state_dtype != torch.float32:
        return
    states, reads_ = results[None]
    for l in range(layers):
        x = xs[l]
        ref, ref_read = O.sparse_prefill(m0s[l], templates, *(x[k] for k in KEYS), growth_quantum_rows=quantum)
        np.testing.assert_allclose(reads_[l].cpu().numpy(), ref_read, atol=ATOL, rtol=RTOL)
        np.testing.assert_array_equal(states[l].logical_to_physical.cpu().numpy(), ref.logical_to_physical)
        mp = states[l].logical_to_physical.cpu().numpy()
        b, s = np.nonzero(mp >= 0)
        np.testing.assert_allclose(states[l].values.cpu().numpy()[mp[b, s]], ref.live_rows(), atol=ATOL, rtol=RTOL)


def test_resolved_walk_reports_route_errors_like_per_token_walk(dev, monkeypatch):
    """A repeated write address at one token is a ValueError with the same text on both walks."""
    rng = np.random.default_rng(9)
    heads, banks, slots, width, tokens = 1, 4, 64, 32, 12
    templates = np.zeros(banks, np.int64)
    m0s = [(0.02 * rng.standard_normal((heads, slots, width))).astype(np.float32)]
    x = prefix(rng, banks, tokens, slots, width, 4, 16)
    x["write_indices"][2, 7, 1] = x["write_indices"][2, 7, 0]
    messages = []
    for resolved in (False, True):
        with_path(monkeypatch, resolved, 3 if resolved else None)
        with pytest.raises(ValueError) as err:
            run(m0s, [x], templates, dev, banks * 4)
        messages.append(str(err.value))
    assert messages[0] == messages[1]


def _decode_state(states, requests, position):
    from copy_on_write_sdm_b200.inference import FaithfulSDMDecodeState

    return FaithfulSDMDecodeState(
        layout="B" * len(states), position=position, capacity=0, activation_dtype=torch.float32,
        active_sequences=torch.ones(requests, dtype=torch.bool, device=states[0].values.device),
        sdm_layer_positions=tuple(range(len(states))), sdm_states=tuple(states), dense_keys=(), dense_values=())


@pytest.mark.parametrize("quantum", [16, 4096])  # 16: the admission grows every pool
def test_admit_prefix_matches_prefill_then_admit(dev, quantum):
    """admit_prefix (the cohort prefilled straight into the live pools) leaves the
    same maps, free stacks, rows, growth counters, positions and readings as
    prefilling the cohort into pools of its own and admitting them."""
    from copy_on_write_sdm_b200.allocator import from_prefix_routes_layers

    rng = np.random.default_rng(31 + quantum)
    heads, live, cohort, layers, slots, width, W, R = 2, 6, 3, 3, 256, 128, 4, 16
    m0s = [(0.02 * rng.standard_normal((heads, slots, width))).astype(np.float32) for _ in range(layers)]
    warm = [prefix(rng, live * heads, 12, slots, width, W, R) for _ in range(layers)]
    new = [prefix(rng, cohort * heads, 9, slots, width, W, R) for _ in range(layers)]
    live_t = np.tile(np.arange(heads), live)
    new_t = np.tile(np.arange(heads), cohort)
    pair = []
    for _ in range(2):
        states, _ = run(m0s, warm, live_t, dev, quantum)
        state = _decode_state(states, live, 12)
        state.release_and_compact([1, 4])
        pair.append(state)
    a, b = pair
    cohort_states, want = run(m0s, new, new_t, dev, quantum)
    a.admit(_decode_state(cohort_states, cohort, 9))
    got = b.admit_prefix([{k: cu(x[k], dev) for k in KEYS} for x in new], template_indices=cu(new_t, dev))
    torch.cuda.synchronize(dev)
    for l in range(layers):
        assert torch.equal(got[l], want[l])
        p, q = a.sdm_states[l], b.sdm_states[l]
        assert torch.equal(p.logical_to_physical, q.logical_to_physical)
        assert torch.equal(p.template_indices, q.template_indices)
        fp = int(p.free_count)
        assert fp == int(q.free_count) and torch.equal(p.free_rows[:fp], q.free_rows[:fp])
        assert p.capacity_rows == q.capacity_rows
        assert (p.growth_events, p.growth_rows_added, p.proven_maximum_additional_allocations) == \
            (q.growth_events, q.growth_rows_added, q.proven_maximum_additional_allocations)
        live_rows = p.logical_to_physical[p.logical_to_physical >= 0].long()
        assert torch.equal(p.values[live_rows], q.values[live_rows])
        q.validate_invariants()
    if quantum == 16:
        assert b.sdm_states[0].growth_events > 0
    assert a.batch == b.batch == live - 2 + cohort
    assert torch.equal(a.current_positions(), b.current_positions()) and a.position == b.position


def test_admit_prefix_refuses_bad_routes_without_changing_the_pools(dev):
    from copy_on_write_sdm_b200.allocator import from_prefix_routes_layers  # noqa: F401

    rng = np.random.default_rng(77)
    heads, slots, width = 1, 64, 32
    m0s = [(0.02 * rng.standard_normal((heads, slots, width))).astype(np.float32)]
    states, _ = run(m0s, [prefix(rng, 4, 5, slots, width, 4, 16)], np.zeros(4, np.int64), dev, 64)
    state = _decode_state(states, 4, 5)
    before = (state.sdm_states[0].logical_to_physical.clone(), int(state.sdm_states[0].free_count))
    for bad in ("read", "write"):
        x = prefix(rng, 2, 3, slots, width, 4, 16)
        if bad == "read":
            x["read_indices"][1, 2, 5] = slots
        else:
            x["write_indices"][0, 1, 2] = x["write_indices"][0, 1, 0]
        with pytest.raises(ValueError):
            state.admit_prefix([{k: cu(x[k], dev) for k in KEYS}], template_indices=cu(np.zeros(2, np.int64), dev))
        assert torch.equal(state.sdm_states[0].logical_to_physical, before[0])
        assert int(state.sdm_states[0].free_count) == before[1] and state.batch == 4
