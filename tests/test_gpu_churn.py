"""GPU parity of a continuous-batching churn trace (configuration 5 shape).

N=4096 slots, D=128, H=4, two pools, six live requests with short lengths so
that completions happen every few steps.  Every step runs the serving order
of the churn benchmark: ``release_and_compact`` of finished requests, sparse
prefill + ``admit`` of a cohort of the same size, an occasional trim,
``prepare_step_capacity`` (growth by whole one-step quanta) and one fused
decode launch over both pools.  The oracle replays the same trace with the
same inputs; maps, free stacks, counts, capacities and counters must match
bit for bit after every step, readouts within 1e-5 abs / 1e-5 rel.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 1e-5
RTOL = 1e-5
N, D, H, W, R, LAYERS, LIVE = 4096, 128, 4, 4, 16, 2, 6


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def cu(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def prefix_inputs(rng, banks, tokens):
    routes = lambda k: np.stack([O.uniform_routes(rng, banks, N, k) for _ in range(tokens)], 1)
    return dict(write_indices=routes(W),
                write_weights=O.softmax(rng.standard_normal((banks, tokens, W), dtype=np.float32)),
                values=rng.standard_normal((banks, tokens, D), dtype=np.float32),
                input_gate=rng.random((banks, tokens), dtype=np.float32),
                forget_log_gate=-rng.random((banks, tokens), dtype=np.float32),
                read_indices=routes(R),
                read_weights=O.softmax(rng.standard_normal((banks, tokens, R), dtype=np.float32)))


def assert_same(st, ref):
    np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), ref.logical_to_physical)
    fc = int(st.free_count)
    assert fc == ref.free_count
    np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), ref.free_stack())
    assert st.capacity_rows == ref.capacity_rows
    np.testing.assert_array_equal(st.template_indices.cpu().numpy(), ref.template_indices)
    assert (st.growth_events, st.growth_rows_added, st.growth_rows_copied) == \
        (ref.growth_events, ref.growth_rows_added, ref.growth_rows_copied)
    assert st.proven_maximum_additional_allocations == ref.proven_maximum_additional_allocations
    mp = st.logical_to_physical.cpu().numpy()
    b, s = np.nonzero(mp >= 0)
    np.testing.assert_allclose(st.values.cpu().numpy()[mp[b, s]], ref.live_rows(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("quantum_steps,trim_every", [(1, 0), (4, 7)])
def test_churn_trace_matches_oracle(dev, quantum_steps, trim_every):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step_layers
    from copy_on_write_sdm_b200.inference import FaithfulSDMDecodeState

    rng = np.random.default_rng(50 + quantum_steps)
    banks = LIVE * H
    q = O.growth_quantum_rows(banks, W, quantum_steps)
    m0s = [(0.02 * rng.standard_normal((H, N, D))).astype(np.float32) for _ in range(LAYERS)]
    m0s_dev = [cu(m, dev) for m in m0s]

    def cohort(requests, tokens):
        b = requests * H
        templates = np.tile(np.arange(H), requests)
        mine, refs = [], []
        for l in range(LAYERS):
            x = prefix_inputs(rng, b, tokens)
            ref, ref_read = O.sparse_prefill(m0s[l], templates, x["write_indices"], x["write_weights"],
                                             x["values"], x["input_gate"], x["forget_log_gate"],
                                             x["read_indices"], x["read_weights"], growth_quantum_rows=q)
            st, read = PackedSDMCopyOnWriteState.from_prefix_routes(
                m0s_dev[l], *(cu(x[k], dev) for k in ("write_indices", "write_weights", "values", "input_gate",
                                                      "forget_log_gate", "read_indices", "read_weights")),
                template_indices=cu(templates, dev), growth_quantum_rows=q)
            np.testing.assert_allclose(read.cpu().numpy(), ref_read, atol=ATOL, rtol=RTOL)
            assert_same(st, ref)
            mine.append(st)
            refs.append(ref)
        state = FaithfulSDMDecodeState(
            layout="B" * LAYERS, position=tokens, capacity=0, activation_dtype=torch.float32,
            active_sequences=torch.ones(requests, dtype=torch.bool, device=dev),
            sdm_layer_positions=tuple(range(LAYERS)), sdm_states=tuple(mine), dense_keys=(), dense_values=())
        return state, refs

    state, refs = cohort(LIVE, 6)
    remaining = rng.integers(1, 8, size=LIVE)
    completions = trims = 0
    for step in range(40):
        done = np.nonzero(remaining == 0)[0]
        if done.size:
            completions += done.size
            released = (done[:, None] * H + np.arange(H)).reshape(-1)
            got = state.release_and_compact(done.tolist())
            want = 0
            for ref in refs:
                want += O.release(ref, released)
                O.retain_banks(ref, np.setdiff1d(np.arange(ref.banks), released))
            assert got == want
            incoming, incoming_refs = cohort(int(done.size), 3)
            assert state.admit(incoming) == done.size
            for ref, other in zip(refs, incoming_refs):
                O.append_banks_from(ref, other)
            remaining = np.concatenate([remaining[remaining > 0], rng.integers(2, 10, size=done.size)])
        if trim_every and step % trim_every == trim_every - 1:
            trims += 1
            got = state.trim_sdm_pools(headroom_rows=banks)
            assert got == sum(O.trim_capacity(ref, headroom_rows=banks) for ref in refs)
        xs = [O.synthetic_step_inputs(rng, banks, N, D, W, R) for _ in range(LAYERS)]
        for st, ref in zip(state.sdm_states, refs):
            assert st.prepare_step_capacity(banks * W) == O.prepare_step_capacity(ref, banks * W)
        out = packed_sdm_cow_step_layers(state.sdm_states, [{k: cu(v, dev) for k, v in x.items()} for x in xs])
        for l in range(LAYERS):
            want, _ = O.packed_step(refs[l], **xs[l])
            np.testing.assert_allclose(out[l].cpu().numpy(), want, atol=ATOL, rtol=RTOL)
            assert_same(state.sdm_states[l], refs[l])
        remaining = remaining - 1
    assert completions >= 10
    assert trims == (40 // trim_every if trim_every else 0)
    for st, ref in zip(state.sdm_states, refs):
        assert st.growth_events > 0
        st.validate_invariants()
        O.validate_invariants(ref)
