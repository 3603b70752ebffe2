"""DecodeSession (packed buffers, one launch per step) against the per-call API."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _pools(dev, layers, banks, slots, width, quantum, seed):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    g = torch.Generator().manual_seed(seed)
    return [PackedSDMCopyOnWriteState.allocate((0.02 * torch.randn(1, slots, width, generator=g)).to(dev),
                                               banks=banks, capacity_rows=quantum, growth_quantum_rows=quantum)
            for _ in range(layers)]


def test_snapshot_proofs_keep_growth_where_the_reference_grows(dev):
    """Proofs renewed from background free-count snapshots (no synchronisation)
    leave maps, stacks, capacity and growth events exactly as the reference's
    per-step proof does."""
    from copy_on_write_sdm_b200 import DecodeSession, packed_sdm_cow_step_layers

    layers, banks, slots, width, W, R = 2, 32, 512, 128, 4, 16
    quantum = O.growth_quantum_rows(banks, W, 8)
    ref = _pools(dev, layers, banks, slots, width, quantum, 1)
    new = _pools(dev, layers, banks, slots, width, quantum, 1)
    sess = DecodeSession(new, writes=W, reads=R)
    rng = np.random.default_rng(9)
    for step in range(40):
        xs = [O.synthetic_step_inputs(rng, banks, slots, width, W, R) for _ in range(layers)]
        for l, x in enumerate(xs):
            for k, v in x.items():
                sess.host_views[l][k].copy_(torch.from_numpy(v))
        sess.step_host()
        torch.cuda.synchronize(dev)  # snapshots land before they are needed
        got = sess.host_outputs.clone()
        for p in ref:
            p.prepare_step_capacity(banks * W)
        want = packed_sdm_cow_step_layers(ref, [{k: torch.from_numpy(v).to(dev) for k, v in x.items()} for x in xs])
        torch.cuda.synchronize(dev)
        for l in range(layers):
            np.testing.assert_allclose(got[l].numpy(), want[l].cpu().numpy(), atol=1e-5, rtol=1e-5)
    assert sess.snapshot_proofs > 0
    for p, q in zip(ref, new):
        assert torch.equal(p.logical_to_physical, q.logical_to_physical)
        assert torch.equal(p.free_rows[:int(p.free_count)], q.free_rows[:int(q.free_count)])
        assert p.capacity_rows == q.capacity_rows and p.growth_events == q.growth_events > 0
        q.validate_invariants()


def test_session_matches_per_call_api_through_growth(dev):
    from copy_on_write_sdm_b200 import DecodeSession, packed_sdm_cow_step_layers

    layers, banks, slots, width, W, R = 3, 32, 128, 128, 4, 16
    quantum = O.growth_quantum_rows(banks, W, 2)
    ref = _pools(dev, layers, banks, slots, width, quantum, 1)
    new = _pools(dev, layers, banks, slots, width, quantum, 1)
    sess = DecodeSession(new, writes=W, reads=R)
    rng = np.random.default_rng(4)
    for step in range(12):  # grows several times: pool descriptors are rebuilt
        xs = [O.synthetic_step_inputs(rng, banks, slots, width, W, R) for _ in range(layers)]
        for l, x in enumerate(xs):
            for k, v in x.items():
                sess.host_views[l][k].copy_(torch.from_numpy(v))
        sess.step_host()
        torch.cuda.synchronize(dev)  # the readouts reach host memory asynchronously
        got = sess.host_outputs.clone()
        for p in ref:
            p.prepare_step_capacity(banks * W)
        want = packed_sdm_cow_step_layers(ref, [{k: torch.from_numpy(v).to(dev) for k, v in x.items()} for x in xs])
        torch.cuda.synchronize(dev)
        for l in range(layers):
            np.testing.assert_allclose(got[l].numpy(), want[l].cpu().numpy(), atol=1e-5, rtol=1e-5)
    for p, q in zip(ref, new):
        assert torch.equal(p.logical_to_physical, q.logical_to_physical)
        assert p.capacity_rows == q.capacity_rows and p.growth_events == q.growth_events > 0
        q.validate_invariants()


@pytest.mark.parametrize("index_dtype", [torch.int64, torch.int32])
def test_pipelined_host_steps_match_sequential(dev, index_dtype):
    """step_host_pipelined overlaps copies of neighbouring steps on side streams;
    readouts, maps, stacks and growth must equal the sequential step_host run
    (int64 indices), also when the pipelined session packs int32 indices."""
    from copy_on_write_sdm_b200 import DecodeSession

    layers, banks, slots, width, W, R = 2, 48, 256, 128, 4, 16
    quantum = O.growth_quantum_rows(banks, W, 3)
    seq = DecodeSession(_pools(dev, layers, banks, slots, width, quantum, 7), writes=W, reads=R)
    pipe = DecodeSession(_pools(dev, layers, banks, slots, width, quantum, 7), writes=W, reads=R,
                         index_dtype=index_dtype)
    rng = np.random.default_rng(8)
    steps = 10
    host = torch.empty(steps, seq.step_bytes, dtype=torch.uint8, pin_memory=True)
    phost = torch.empty(steps, pipe.step_bytes, dtype=torch.uint8, pin_memory=True)
    for i in range(steps):
        xs = [O.synthetic_step_inputs(rng, banks, slots, width, W, R) for _ in range(layers)]
        for l, x in enumerate(xs):
            for k, v in x.items():
                seq.host_views[l][k].copy_(torch.from_numpy(v))
                pipe.host_views[l][k].copy_(torch.from_numpy(v))
        host[i].copy_(seq.host_inputs)
        phost[i].copy_(pipe.host_inputs)
    want = []
    for i in range(steps):
        seq.step_host(host[i])
        torch.cuda.synchronize(dev)
        want.append(seq.host_outputs.clone())
    got = []
    pending = []
    for i in range(steps):
        out, ev = pipe.step_host_pipelined(phost[i])
        pending.append((out, ev))
        if len(pending) == 2:  # the buffer of step i-1 is reused by step i+1
            o, e = pending.pop(0)
            e.synchronize()
            got.append(o.clone())
    for o, e in pending:
        e.synchronize()
        got.append(o.clone())
    torch.cuda.synchronize(dev)
    for a, b in zip(want, got):
        if index_dtype == torch.int64:
            assert torch.equal(a, b)
        else:  # int32 indices run another decode kernel variant: 1e-5 as elsewhere
            torch.testing.assert_close(b, a, atol=1e-5, rtol=1e-5)
    for p, q in zip(seq.pools, pipe.pools):
        assert torch.equal(p.logical_to_physical, q.logical_to_physical)
        fp = int(p.free_count)
        assert fp == int(q.free_count) and torch.equal(p.free_rows[:fp], q.free_rows[:fp])
        assert p.growth_events == q.growth_events > 0
        q.validate_invariants()


def test_mapped_host_steps_match_sequential(dev):
    """step_host_mapped: the decode kernel reads the pinned host step and writes
    the readouts to pinned host memory itself.  Readouts, maps, stacks and
    growth must equal the sequential step_host run; pageable memory is refused
    before anything launches."""
    from copy_on_write_sdm_b200 import DecodeSession

    layers, banks, slots, width, W, R = 3, 40, 256, 128, 4, 16
    quantum = O.growth_quantum_rows(banks, W, 3)
    seq = DecodeSession(_pools(dev, layers, banks, slots, width, quantum, 5), writes=W, reads=R)
    mapped = DecodeSession(_pools(dev, layers, banks, slots, width, quantum, 5), writes=W, reads=R)
    rng = np.random.default_rng(6)
    steps = 12
    host = torch.empty(steps, seq.step_bytes, dtype=torch.uint8, pin_memory=True)
    for i in range(steps):
        xs = [O.synthetic_step_inputs(rng, banks, slots, width, W, R) for _ in range(layers)]
        for l, x in enumerate(xs):
            for k, v in x.items():
                seq.host_views[l][k].copy_(torch.from_numpy(v))
        host[i].copy_(seq.host_inputs)
    want = []
    for i in range(steps):
        seq.step_host(host[i])
        torch.cuda.synchronize(dev)
        want.append(seq.host_outputs.clone())
    got, pending = [], []
    for i in range(steps):
        pending.append(mapped.step_host_mapped(host[i]))
        if len(pending) == 2:
            o, e = pending.pop(0)
            e.synchronize()
            got.append(o.clone())
    for o, e in pending:
        e.synchronize()
        got.append(o.clone())
    for a, b in zip(want, got):  # the two paths may pick different decode kernels: 1e-5 as elsewhere
        torch.testing.assert_close(b, a, atol=1e-5, rtol=1e-5)
    for p, q in zip(seq.pools, mapped.pools):
        assert torch.equal(p.logical_to_physical, q.logical_to_physical)
        fp = int(p.free_count)
        assert fp == int(q.free_count) and torch.equal(p.free_rows[:fp], q.free_rows[:fp])
        assert p.growth_events == q.growth_events > 0
        q.validate_invariants()
    pageable = torch.empty(seq.step_bytes, dtype=torch.uint8)
    with pytest.raises(ValueError, match="pinned"):
        mapped.step_host_mapped(pageable)
