"""CUDA-graph decode (``GraphedDecode``) against the eager ``LanguageModel.decode``.

Two identical states are prefilled from the same prompts; one decodes
eagerly, the other by graph replay.  Allocator state must stay bit-exact
(maps, free stacks, counts, capacities, counters) and logits / slab rows
within 1e-4 / 1e-5 -- the graph attends over the whole K/V cache under a
mask, so only summation order differs.  The trace covers slab growth (a
re-capture), release + compaction + admission at another position
(per-request positions, another re-capture) and plain replays.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda:0")


def same_pools(a, b):
    for x, y in zip(a.sdm_states, b.sdm_states):
        assert torch.equal(x.logical_to_physical, y.logical_to_physical)
        fx, fy = int(x.free_count), int(y.free_count)
        assert fx == fy
        assert torch.equal(x.free_rows[:fx], y.free_rows[:fy])
        assert x.capacity_rows == y.capacity_rows
        assert (x.growth_events, x.growth_rows_added, x.growth_rows_copied,
                x.proven_maximum_additional_allocations) == \
               (y.growth_events, y.growth_rows_added, y.growth_rows_copied,
                y.proven_maximum_additional_allocations)
        mp = x.logical_to_physical
        live = mp[mp >= 0].long()
        torch.testing.assert_close(x.values[live], y.values[live], atol=1e-5, rtol=1e-5)
    assert a.position == b.position
    if a.positions is None:
        assert b.positions is None
    else:
        assert torch.equal(a.positions, b.positions)


@pytest.mark.parametrize("quantum", [0, 16])
def test_graphed_decode_matches_eager(dev, quantum):
    from copy_on_write_sdm_b200.graph import GraphedDecode
    from copy_on_write_sdm_b200.model import LanguageModel

    model = LanguageModel(vocab_size=512, maximum_sequence_length=64, layout="BBAB", width=64, heads=4, slots=64,
                          reads=8, writes=4, memory_heads=2, activation_dtype=torch.float32)
    model.initialize_role_keyed(3)
    model = model.to(dev).eval()
    gen = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 512, (4, 48), generator=gen).to(dev)
    cohort = torch.randint(0, 512, (2, 24), generator=gen).to(dev)

    _, eager = model.prefill(ids[:, :12], capacity=48, sdm_growth_quantum_rows=quantum)
    _, graphed = model.prefill(ids[:, :12], capacity=48, sdm_growth_quantum_rows=quantum)
    runner = GraphedDecode(model, graphed)
    same_pools(eager, graphed)

    def run(ids, t):
        want = model.decode(ids[:, t:t + 1], eager).clone()
        got = runner.step(ids[:, t:t + 1]).clone()
        torch.testing.assert_close(got, want, atol=LOGIT_TOL, rtol=LOGIT_TOL)
        same_pools(eager, graphed)

    for t in range(12, 20):
        run(ids, t)
    # release two requests, compact, admit a cohort prefilled to another position
    for st in (eager, graphed):
        st.release_and_compact([0, 2])
        model.admit(cohort[:, :5], st)
    same_pools(eager, graphed)
    ids = torch.cat([ids[1::2], torch.randint(0, 512, (2, 48), generator=gen).to(dev)], dim=0)
    for t in range(20, 28):
        run(ids, t)
    # Growth pools stay proven: every growth or admission re-captures.  Fixed
    # pools lose their proof on admission and then take the eager checked step.
    assert runner.captures >= (2 if quantum else 1)
    assert runner.replays >= (1 if quantum else 6)
    if quantum:
        assert runner.captures + runner.replays == 16
    for st in graphed.sdm_states:
        st.validate_invariants()
    if quantum:
        assert sum(st.growth_events for st in graphed.sdm_states) > 0
