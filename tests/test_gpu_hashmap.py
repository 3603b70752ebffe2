"""Hashed logical maps (per-bank open-addressing tables instead of the dense
[banks, N] int32 map).  Row placement never depends on where an entry sits in
a table, so every check here is the dense pool's bar: maps (compared in their
dense form), free stacks and counts bit-exact against the oracle or a dense
twin pool driven through the same calls; rows and readouts within 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 1e-5
RTOL = 1e-5
W, R, WIDTH = 4, 16, 128


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def cu(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def dense_map(st):
    from copy_on_write_sdm_b200.allocator import dense_maps

    with dense_maps([st]):
        return st.logical_to_physical.cpu().numpy()


def same_pool(a, b):
    """a (hashed) and b (dense) hold the same allocator state."""
    ma, mb = dense_map(a), dense_map(b)
    np.testing.assert_array_equal(ma, mb)
    fa, fb = int(a.free_count), int(b.free_count)
    assert fa == fb
    assert torch.equal(a.free_rows[:fa], b.free_rows[:fb])
    assert a.capacity_rows == b.capacity_rows
    live = torch.from_numpy(mb[mb >= 0]).long().to(a.values.device)
    torch.testing.assert_close(a.values[live].float(), b.values[live].float(), atol=ATOL, rtol=RTOL)


def test_round_trip_dense_hash_dense(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    rng = np.random.default_rng(1)
    banks, slots = 300, 4096
    mask = rng.random((banks, slots)) < rng.random((banks, 1)) * 0.05
    dense = rng.standard_normal((banks, slots, 8)).astype(np.float32)
    m0 = (0.02 * rng.standard_normal((1, slots, 8))).astype(np.float32)
    st = PackedSDMCopyOnWriteState.from_dense_overlay(cu(m0, dev), cu(dense, dev), cu(mask, dev),
                                                      template_indices=torch.zeros(banks, dtype=torch.int64,
                                                                                   device=dev))
    want = st.logical_to_physical.cpu().numpy()
    t = st.use_hash_map()
    assert st.map_table_slots == t and t & (t - 1) == 0
    assert int(mask.sum(1).max()) <= 0.7 * t
    assert st.slots == slots and st.banks == banks
    st.use_dense_map()
    np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), want)
    st.use_hash_map(1 << 12)
    assert st.storage_bytes()["logical_to_physical"] == banks * 4096 * 8
    st.validate_invariants()
    np.testing.assert_array_equal(dense_map(st), want)


@pytest.mark.parametrize("banks,layers", [(64, 3), (2048, 1)])
def test_growth_pool_decode_with_rehash_matches_oracle(dev, banks, layers):
    """Tables start at four entries per bank; the capacity proof rehashes them as
    banks fill (several times over the trace) and the trace stays exact."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step_layers

    rng = np.random.default_rng(banks)
    slots = 256
    q = O.growth_quantum_rows(banks, W, 2)
    states, refs = [], []
    for _ in range(layers):
        m0 = (0.02 * rng.standard_normal((1, slots, WIDTH))).astype(np.float32)
        st = PackedSDMCopyOnWriteState.allocate(cu(m0, dev), banks=banks, capacity_rows=q, growth_quantum_rows=q)
        assert st.use_hash_map() == 4
        states.append(st)
        refs.append(O.allocate(m0, banks=banks, capacity_rows=q, growth_quantum_rows=q))
    sizes = set()
    for step in range(24):
        xs = [O.synthetic_step_inputs(rng, banks, slots, WIDTH, W, R) for _ in states]
        for st, r in zip(states, refs):
            st.prepare_step_capacity(banks * W)
            O.prepare_step_capacity(r, banks * W)
            sizes.add(st.map_table_slots)
        wants = [O.packed_step(r, **x)[0] for r, x in zip(refs, xs)]
        gots = packed_sdm_cow_step_layers(states, [{k: cu(v, dev) for k, v in x.items()} for x in xs])
        for got, want in zip(gots, wants):
            np.testing.assert_allclose(got.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
        for st, r in zip(states, refs):
            assert st.status() == 0
            assert int(st.free_count) == r.free_count
    assert len(sizes) >= 3  # rehashed at least twice
    for st, r in zip(states, refs):
        np.testing.assert_array_equal(dense_map(st), r.logical_to_physical)
        fc = int(st.free_count)
        np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), r.free_stack())
        assert st.capacity_rows == r.capacity_rows and st.growth_events == r.growth_events
        st.validate_invariants()


def test_lifecycle_on_hashed_pools_matches_dense_twin(dev):
    """release -> retain -> append -> trim -> decode on a hashed pool and on a
    dense twin: identical allocator state after every operation."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    rng = np.random.default_rng(7)
    banks, slots = 48, 512
    q = O.growth_quantum_rows(banks, W, 4)
    m0 = cu((0.02 * rng.standard_normal((1, slots, WIDTH))).astype(np.float32), dev)

    def make():
        st = PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=q, growth_quantum_rows=q)
        return st

    hashed, dense = make(), make()
    hashed.use_hash_map()

    def step(n):
        for _ in range(n):
            x = {k: cu(v, dev) for k, v in
                 O.synthetic_step_inputs(rng, hashed.banks, slots, WIDTH, W, R).items()}
            outs = []
            for st in (hashed, dense):
                st.prepare_step_capacity(st.banks * W)
                outs.append(packed_sdm_cow_step(st, **x, collect_diagnostics=False)[0])
            torch.testing.assert_close(outs[0], outs[1], atol=ATOL, rtol=RTOL)
        same_pool(hashed, dense)

    step(10)
    idx = torch.tensor([5, 0, 17, 30], device=dev)
    assert int(hashed.release(idx)) == int(dense.release(idx)) > 0
    assert hashed.map_table_slots > 0
    same_pool(hashed, dense)
    keep = torch.tensor([i for i in range(banks) if i not in (5, 0, 17, 30)], device=dev)
    hashed.retain_banks(keep)
    dense.retain_banks(keep)
    same_pool(hashed, dense)
    step(3)
    mask = cu(rng.random((6, slots)) < 0.05, dev)
    cohort = cu(rng.standard_normal((6, slots, WIDTH)).astype(np.float32), dev)
    tmpl = torch.zeros(6, dtype=torch.int64, device=dev)
    for st in (hashed, dense):
        other = PackedSDMCopyOnWriteState.from_dense_overlay(m0, cohort, mask, template_indices=tmpl,
                                                             growth_quantum_rows=q)
        st.append_banks_from(other)
    same_pool(hashed, dense)
    step(3)
    assert hashed.trim_capacity(headroom_rows=8) == dense.trim_capacity(headroom_rows=8)
    same_pool(hashed, dense)
    step(3)
    hashed.validate_invariants()
    torch.testing.assert_close(hashed.materialize_dense(), dense.materialize_dense(), atol=ATOL, rtol=RTOL)


def test_session_on_hashed_pools(dev):
    """DecodeSession over hashed growth pools (proofs renew through the table
    check, never from the mirrored free count) against dense twins."""
    from copy_on_write_sdm_b200 import DecodeSession, PackedSDMCopyOnWriteState

    rng = np.random.default_rng(3)
    layers, banks, slots = 2, 32, 256
    q = O.growth_quantum_rows(banks, W, 2)

    def pools(hashed):
        g = torch.Generator().manual_seed(5)
        out = []
        for _ in range(layers):
            st = PackedSDMCopyOnWriteState.allocate((0.02 * torch.randn(1, slots, WIDTH, generator=g)).to(dev),
                                                    banks=banks, capacity_rows=q, growth_quantum_rows=q)
            if hashed:
                st.use_hash_map()
            out.append(st)
        return out

    a, b = DecodeSession(pools(True), writes=W, reads=R), DecodeSession(pools(False), writes=W, reads=R)
    for _ in range(20):
        xs = [O.synthetic_step_inputs(rng, banks, slots, WIDTH, W, R) for _ in range(layers)]
        for sess in (a, b):
            for l, x in enumerate(xs):
                for k, v in x.items():
                    sess.host_views[l][k].copy_(torch.from_numpy(v))
            sess.step_host()
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(a.host_outputs, b.host_outputs, atol=ATOL, rtol=RTOL)
    for p, r in zip(a.pools, b.pools):
        assert p.map_table_slots > 4
        same_pool(p, r)
        p.validate_invariants()


@pytest.mark.parametrize("slab_dtype,width,w,r", [(torch.bfloat16, 128, 4, 16), (torch.float32, 256, 8, 64),
                                                  (torch.float32, 64, 32, 256)])
def test_hashed_decode_other_variants_match_dense_twin(dev, slab_dtype, width, w, r):
    """Hashed tables under the other compiled decode variants (bf16 slab, wide
    rows, W up to 32, R up to 256) against a dense twin on the same routes."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    rng = np.random.default_rng(width + w)
    banks, slots = 96, 1024
    q = O.growth_quantum_rows(banks, w, 2)
    m0 = cu((0.02 * rng.standard_normal((2, slots, width))).astype(np.float32), dev)
    tmpl = torch.arange(2, device=dev, dtype=torch.int64).repeat(banks // 2)

    def make():
        return PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=q, growth_quantum_rows=q,
                                                  template_indices=tmpl, state_dtype=slab_dtype)

    hashed, dense = make(), make()
    hashed.use_hash_map()
    for _ in range(12):
        x = {k: cu(v, dev) for k, v in O.synthetic_step_inputs(rng, banks, slots, width, w, r).items()}
        outs = []
        for st in (hashed, dense):
            st.prepare_step_capacity(banks * w)
            outs.append(packed_sdm_cow_step(st, **x, collect_diagnostics=False)[0])
        torch.testing.assert_close(outs[0], outs[1], atol=ATOL, rtol=RTOL)
    same_pool(hashed, dense)
    assert hashed.status() == 0 and hashed.map_table_slots > 4
    hashed.validate_invariants()
