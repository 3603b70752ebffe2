"""GPU parity of the fused decode step, the dense control and the error paths.

Bar: maps, free stacks, free counts and first-touch counts bit-exact; slab
rows and readouts within 1e-5 abs / 1e-5 rel (FP32).
"""

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


def cu(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.to(dtype)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def assert_same_state(st, ref, *, live_rows=True):
    np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), ref.logical_to_physical)
    fc = int(st.free_count)
    assert fc == ref.free_count
    np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), ref.free_stack())
    np.testing.assert_array_equal(st.template_indices.cpu().numpy(), ref.template_indices)
    assert st.capacity_rows == ref.capacity_rows
    if live_rows:
        mp = st.logical_to_physical.cpu().numpy()
        b, s = np.nonzero(mp >= 0)
        got = st.values.float().cpu().numpy()[mp[b, s]]
        np.testing.assert_allclose(got, ref.live_rows(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["cfg1_decode", "small_decode", "multibank_decode"])
def test_golden_decode_trace(dev, name):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, dense_sdm_sparse_step, packed_sdm_cow_step

    g = load(name)
    banks = g["templates"].shape[0]
    st = PackedSDMCopyOnWriteState.allocate(cu(g["m0"], dev), banks=banks,
                                            capacity_rows=int(g["capacity0"]),
                                            template_indices=cu(g["templates"], dev))
    dense = cu(g["m0"][g["templates"]], dev).contiguous()
    for t in range(g["readings"].shape[0]):
        x = {k: cu(g[f"in_{k}"][t], dev) for k in KEYS}
        got, diag = packed_sdm_cow_step(st, **x)
        dgot = dense_sdm_sparse_step(dense, **x)
        np.testing.assert_allclose(got.cpu().numpy(), g["readings"][t], atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(dgot.cpu().numpy(), g["dense_readings"][t], atol=ATOL, rtol=RTOL)
        np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), g["maps"][t])
        assert int(st.free_count) == g["free_counts"][t]
        np.testing.assert_array_equal(diag.first_touches_by_sequence.cpu().numpy(), g["first_by_bank"][t])
    fc = int(st.free_count)
    np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), g["final_free_stack"])
    mp = st.logical_to_physical.cpu().numpy()
    b, s = np.nonzero(mp >= 0)
    np.testing.assert_allclose(st.values.cpu().numpy()[mp[b, s]], g["final_live_rows"], atol=ATOL, rtol=RTOL)
    if "final_dense" in g:
        np.testing.assert_allclose(st.materialize_dense().cpu().numpy(), g["final_dense"], atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(dense.cpu().numpy(), g["final_dense"], atol=ATOL, rtol=RTOL)
    st.validate_invariants()


def _random_trace(dev, *, banks, slots, width, W, R, steps, heads=1, seed=0, capacity=None,
                  idx_dtype=torch.int64, layers=1):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step_layers

    rng = np.random.default_rng(seed)
    states, refs = [], []
    for _ in range(layers):
        m0 = (0.02 * rng.standard_normal((heads, slots, width))).astype(np.float32)
        tmpl = np.tile(np.arange(heads), banks // heads)
        cap = capacity or banks * slots
        states.append(PackedSDMCopyOnWriteState.allocate(cu(m0, dev), banks=banks, capacity_rows=cap,
                                                         template_indices=cu(tmpl, dev)))
        states[-1].capacity_is_proven = True
        refs.append(O.allocate(m0, banks=banks, capacity_rows=cap, template_indices=tmpl))
    for _ in range(steps):
        xs = [O.synthetic_step_inputs(rng, banks, slots, width, W, R) for _ in range(layers)]
        wants = [O.packed_step(r, **x)[0] for r, x in zip(refs, xs)]
        steps_dev = []
        for x in xs:
            d = {k: cu(v, dev) for k, v in x.items()}
            d["write_indices"] = d["write_indices"].to(idx_dtype)
            d["read_indices"] = d["read_indices"].to(idx_dtype)
            steps_dev.append(d)
        gots = packed_sdm_cow_step_layers(states, steps_dev)
        for got, want in zip(gots, wants):
            np.testing.assert_allclose(got.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
        for s, r in zip(states, refs):
            np.testing.assert_array_equal(s.logical_to_physical.cpu().numpy(), r.logical_to_physical)
            assert int(s.free_count) == r.free_count
    for s, r in zip(states, refs):
        assert_same_state(s, r)
        s.validate_invariants()


def test_config3_shape_seven_layers_one_launch(dev):
    # Configuration 3 per-layer shape (B=64, H=1, N=256, D=128, top-16/top-4), 7 pools per launch.
    _random_trace(dev, banks=64, slots=256, width=128, W=4, R=16, steps=20, layers=7, seed=3)


def test_many_tiles_lookback_and_int32_indices(dev):
    # 2,048 banks = 512 tiles: exercises multi-hop decoupled look-back.
    _random_trace(dev, banks=2048, slots=64, width=128, W=4, R=16, steps=6, heads=4, seed=5,
                  idx_dtype=torch.int32)


@pytest.mark.parametrize("banks,slots", [(64, 4096), (2500, 256)])
def test_unstaged_map_paths(dev, banks, slots):
    # N > 1024, or more banks than a latency-bound launch: map entries read from HBM.
    _random_trace(dev, banks=banks, slots=slots, width=128, W=4, R=16, steps=5, seed=banks)


def test_ten_thousand_blocks_ticket_order(dev):
    # 40,000 banks = 10,000 blocks: far more than are resident, so tiles are
    # ordered by ticket and the look-back crosses thousands of banks.
    _random_trace(dev, banks=40000, slots=64, width=128, W=4, R=16, steps=3, seed=17)


@pytest.mark.parametrize("width,W,R", [(8, 2, 4), (64, 3, 5), (256, 8, 24), (512, 12, 40), (128, 32, 256)])
def test_shape_variants(dev, width, W, R):
    _random_trace(dev, banks=37, slots=max(64, R), width=width, W=W, R=R, steps=4, seed=width + W)


def test_growth_through_prepare_step_capacity(dev):
    """Quantum growth mid-trace (allocator.py:692-774) keeps maps/stack bit-exact."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    rng = np.random.default_rng(11)
    banks, slots, width, W, R = 16, 256, 128, 4, 16
    q = O.growth_quantum_rows(banks, W, 4)
    m0 = (0.02 * rng.standard_normal((1, slots, width))).astype(np.float32)
    st = PackedSDMCopyOnWriteState.allocate(cu(m0, dev), banks=banks, capacity_rows=q,
                                            growth_quantum_rows=q)
    ref = O.allocate(m0, banks=banks, capacity_rows=q, growth_quantum_rows=q)
    for _ in range(40):
        x = O.synthetic_step_inputs(rng, banks, slots, width, W, R)
        st.prepare_step_capacity(banks * W)
        O.prepare_step_capacity(ref, banks * W)
        want, _ = O.packed_step(ref, **x)
        got, _ = packed_sdm_cow_step(st, **{k: cu(v, dev) for k, v in x.items()},
                                     validate_routes=False, collect_diagnostics=False)
        np.testing.assert_allclose(got.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
    assert st.growth_events == ref.growth_events > 0
    assert st.growth_rows_copied == ref.growth_rows_copied
    # growths inside the reserve move no rows (only the first copies the initial slab)
    assert st.growth_events > 2 and st.slab_rows_moved < st.growth_rows_copied
    assert st.proven_maximum_additional_allocations == ref.proven_maximum_additional_allocations
    assert_same_state(st, ref)
    st.validate_invariants()


def test_low_precision_activations_and_slab(dev):
    """bf16 activations (the reference model's dtype) and a bf16 slab."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    torch.manual_seed(0)
    banks, slots, width, W, R = 8, 64, 128, 4, 16
    m0 = (0.02 * torch.randn(1, slots, width)).to(torch.bfloat16)
    for slab_dtype in (torch.float32, torch.bfloat16):
        st = PackedSDMCopyOnWriteState.allocate(m0.to(dev), banks=banks, capacity_rows=banks * slots,
                                                state_dtype=slab_dtype)
        dense = m0.float().expand(banks, -1, -1).clone().to(slab_dtype)
        for _ in range(5):
            x = dict(
                write_indices=torch.stack([torch.randperm(slots)[:W] for _ in range(banks)]),
                write_weights=torch.softmax(torch.randn(banks, W), -1).bfloat16(),
                values=torch.randn(banks, width).bfloat16(),
                input_gate=torch.rand(banks).bfloat16(),
                forget_log_gate=(-torch.rand(banks)).bfloat16(),
                read_indices=torch.stack([torch.randperm(slots)[:R] for _ in range(banks)]),
                read_weights=torch.softmax(torch.randn(banks, R), -1).bfloat16(),
            )
            # torch fp32 restatement of allocator.py:1582-1633 on the dense table
            b = torch.arange(banks)[:, None]
            cur = dense[b, x["write_indices"]].float() * x["forget_log_gate"].float().exp()[:, None, None]
            ww = x["write_weights"].float()[..., None]
            ret = (ww * cur).sum(1)
            ig = x["input_gate"].float()[:, None]
            delta = ig * x["values"].float() - ig * ret
            dense[b, x["write_indices"]] = (cur + ww * delta[:, None]).to(slab_dtype)
            want = (x["read_weights"].float()[..., None] * dense[b, x["read_indices"]].float()).sum(1)
            got, _ = packed_sdm_cow_step(st, **{k: v.to(dev) for k, v in x.items()})
            assert got.dtype == torch.bfloat16
            tol = 1e-2  # bf16 output rounding (2^-8 relative) on O(1) readouts
            np.testing.assert_allclose(got.float().cpu().numpy(), want.bfloat16().float().numpy(), atol=tol, rtol=tol)
        np.testing.assert_allclose(st.materialize_dense().float().cpu().numpy(), dense.float().numpy(),
                                   atol=1e-5 if slab_dtype == torch.float32 else 1e-2, rtol=1e-5 if slab_dtype == torch.float32 else 1e-2)
        st.validate_invariants()


def test_errors_are_reported_not_trapped(dev):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    banks, slots, width = 2, 16, 8
    m0 = torch.zeros(1, slots, width, device=dev)

    def step_args(widx, ridx):
        return dict(write_indices=torch.tensor(widx, device=dev), write_weights=torch.full((banks, 2), 0.5, device=dev),
                    values=torch.ones(banks, width, device=dev), input_gate=torch.ones(banks, device=dev),
                    forget_log_gate=torch.zeros(banks, device=dev), read_indices=torch.tensor(ridx, device=dev),
                    read_weights=torch.ones(banks, 1, device=dev))

    st = PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=banks * slots)
    with pytest.raises(ValueError, match="outside the logical table"):
        packed_sdm_cow_step(st, **step_args([[0, 99], [1, 2]], [[0], [1]]))
    st = PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=banks * slots)
    with pytest.raises(ValueError, match="write one logical slot twice"):
        packed_sdm_cow_step(st, **step_args([[3, 3], [1, 2]], [[0], [1]]))
    # Unproven, too-small slab: the step reports exhaustion instead of faulting.
    st = PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=3)
    with pytest.raises(ValueError, match="exhausted"):
        packed_sdm_cow_step(st, **step_args([[0, 1], [2, 3]], [[0], [1]]))
    with pytest.raises(AssertionError, match="overflow"):
        st.validate_invariants()
    with pytest.raises(ValueError, match="CPU fallback|sm_100a"):
        packed_sdm_cow_step(st, **step_args([[0, 1], [2, 3]], [[0], [1]]), backend="torch")



def test_two_pass_launch_reports_bad_bank_and_keeps_others_exact(dev):
    """A large launch (prefix pass + decode pass): one bank repeats a write address.

    The bad bank allocates nothing and the step reports it; every other bank's
    placement is exactly the oracle's with that bank contributing no first touches.
    """
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, packed_sdm_cow_step

    rng = np.random.default_rng(21)
    banks, slots, width, W, R = 16384, 64, 128, 4, 16
    m0 = (0.02 * rng.standard_normal((1, slots, width))).astype(np.float32)
    st = PackedSDMCopyOnWriteState.allocate(cu(m0, dev), banks=banks, capacity_rows=banks * slots)
    x = O.synthetic_step_inputs(rng, banks, slots, width, W, R)
    x["write_indices"][1000, 1] = x["write_indices"][1000, 0]
    with pytest.raises(ValueError, match="write one logical slot twice"):
        packed_sdm_cow_step(st, **{k: cu(v, dev) for k, v in x.items()})
    # oracle: the same step with bank 1000 writing slots that are already private
    ref = O.allocate(m0, banks=banks, capacity_rows=banks * slots)
    ok = {k: v.copy() for k, v in x.items()}
    ok["write_indices"][1000] = np.arange(W)
    ref.logical_to_physical[1000, :W] = 0  # pretend private: no first touches for bank 1000
    O.packed_step(ref, **ok)
    ref.logical_to_physical[1000] = -1
    np.testing.assert_array_equal(st.logical_to_physical.cpu().numpy(), ref.logical_to_physical)
    assert int(st.free_count) == ref.free_count
