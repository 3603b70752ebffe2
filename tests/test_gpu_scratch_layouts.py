"""One decode look-back scratch shared by launches of different pool layouts.

The decode kernel's scan flags sit at positions that depend on the layout of
the launch (how many pools, how many banks each).  Every launch tags its flags
with one launch epoch and advances it once all its pools are closed, so a flag
left by an earlier launch of another layout never reads as published.  These
tests run layout sequences that would put such stale flags under a later
launch's scan -- a 2-pool call, a 1-pool call over the same positions, then a
2-pool call on fresh pools whose banks all have first touches -- and hold
every map, free stack and free count bit-exact against the oracle
(allocator.py:1466-1481 pop order), readouts within 1e-5.  The same sequence
runs through the scratch-taking entry point on one torch buffer and through
the one per-device buffer of ``packed_sdm_cow_step``; a captured
``GraphedDecode`` is replayed after a larger launch replaced the per-device
buffer.
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


class PoolSet:
    """``layers`` pools of ``banks`` banks each, on the GPU and in the oracle."""

    def __init__(self, dev, rng, layers, banks, slots):
        from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

        self.banks, self.slots = banks, slots
        self.states, self.refs = [], []
        for _ in range(layers):
            m0 = (0.02 * rng.standard_normal((1, slots, WIDTH))).astype(np.float32)
            st = PackedSDMCopyOnWriteState.allocate(cu(m0, dev), banks=banks, capacity_rows=banks * slots)
            st.capacity_is_proven = True
            self.states.append(st)
            self.refs.append(O.allocate(m0, banks=banks, capacity_rows=banks * slots))

    def step(self, dev, rng, launch):
        xs = [O.synthetic_step_inputs(rng, self.banks, self.slots, WIDTH, W, R) for _ in self.states]
        wants = [O.packed_step(r, **x)[0] for r, x in zip(self.refs, xs)]
        gots = launch(self.states, [{k: cu(v, dev) for k, v in x.items()} for x in xs])
        torch.cuda.synchronize(dev)
        for got, want in zip(gots, wants):
            np.testing.assert_allclose(got.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
        self.check()

    def check(self):
        for s, r in zip(self.states, self.refs):
            np.testing.assert_array_equal(s.logical_to_physical.cpu().numpy(), r.logical_to_physical)
            fc = int(s.free_count)
            assert fc == r.free_count
            np.testing.assert_array_equal(s.free_rows[:fc].cpu().numpy(), r.free_stack())
            assert s.status() == 0


def _scratch_launch(buf):
    from copy_on_write_sdm_b200 import packed_sdm_cow_step_layers

    def launch(states, steps):
        return packed_sdm_cow_step_layers(states, steps, scratch=buf)
    return launch


def _noalloc_launch(dev):
    from copy_on_write_sdm_b200 import _lib, allocator

    lib = _lib.load()

    def launch(states, steps):
        n = len(states)
        args = [allocator._StepArgs.make(x["write_indices"], x["write_weights"], x["values"], x["input_gate"],
                                         x["forget_log_gate"], x["read_indices"], x["read_weights"], None,
                                         collect=False) for x in steps]
        pools = (_lib.CowPool * n)(*[s._pool() for s in states])
        structs = (_lib.CowStep * n)(*[a.struct for a in args])
        _lib.check(lib.cow_decode_step_noalloc(pools, structs, n, W, R, _lib.I64, _lib.F32, _lib.stream_of(dev)),
                   "cow_decode_step_noalloc")
        return [a.output for a in args]
    return launch


def _per_device_launch():
    from copy_on_write_sdm_b200 import packed_sdm_cow_step_layers

    def launch(states, steps):
        return packed_sdm_cow_step_layers(states, steps)
    return launch


def _mixed_layout_rounds(dev, launch, seed):
    rng = np.random.default_rng(seed)
    keep = PoolSet(dev, rng, 2, 256, 64)  # persistent 2-pool layout
    for _ in range(3):
        keep.step(dev, rng, launch)                          # 2 pools x 256 banks
        PoolSet(dev, rng, 1, 512, 64).step(dev, rng, launch)  # 1 pool over the same flag positions
        fresh = PoolSet(dev, rng, 2, 256, 64)                 # every bank has first touches
        fresh.step(dev, rng, launch)
        fresh.step(dev, rng, launch)
        PoolSet(dev, rng, 7, 64, 64).step(dev, rng, launch)   # configuration-3 layout
        PoolSet(dev, rng, 3, 1000, 32).step(dev, rng, launch)  # ragged pools (1000 banks: partial tiles)
    for s in keep.states:
        s.validate_invariants()


def test_mixed_layouts_on_one_scratch_buffer(dev):
    from copy_on_write_sdm_b200 import _lib

    need = _lib.load().cow_decode_scratch_bytes(3000, 3)
    buf = torch.zeros(max(need, 4096), dtype=torch.uint8, device=dev)
    _mixed_layout_rounds(dev, _scratch_launch(buf), seed=11)


def test_mixed_layouts_through_the_per_device_scratch(dev):
    _mixed_layout_rounds(dev, _per_device_launch(), seed=12)


def test_mixed_layouts_through_the_noalloc_entry_point(dev):
    _mixed_layout_rounds(dev, _noalloc_launch(dev), seed=13)


def test_checked_entry_point_reports_status(dev):
    """cow_decode_step_checked: COW_OK on good routes, COW_ERR_DEVICE with the
    status bits on an out-of-range index (reported, not trapped)."""
    import ctypes

    from copy_on_write_sdm_b200 import _lib, allocator

    lib = _lib.load()
    rng = np.random.default_rng(5)
    ps = PoolSet(dev, rng, 1, 64, 64)
    scratch = allocator.new_decode_scratch(dev, 64, 1)
    for bad in (False, True):
        x = O.synthetic_step_inputs(rng, 64, 64, WIDTH, W, R)
        if bad:
            x["read_indices"][3, 0] = 64
        d = {k: cu(v, dev) for k, v in x.items()}
        a = allocator._StepArgs.make(d["write_indices"], d["write_weights"], d["values"], d["input_gate"],
                                     d["forget_log_gate"], d["read_indices"], d["read_weights"], None, collect=False)
        pools = (_lib.CowPool * 1)(ps.states[0]._pool())
        steps = (_lib.CowStep * 1)(a.struct)
        status = ctypes.c_int32(0)
        rc = lib.cow_decode_step_checked(pools, steps, 1, W, R, _lib.I64, _lib.F32, scratch.data_ptr(),
                                         scratch.numel(), _lib.stream_of(dev), ctypes.byref(status))
        if bad:
            assert rc == _lib.ERR_DEVICE and status.value & 0x2
        else:
            assert rc == _lib.OK and status.value == 0
            want = O.packed_step(ps.refs[0], **x)[0]
            np.testing.assert_allclose(a.output.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
            ps.check()


def test_graph_replays_after_the_per_device_scratch_was_replaced(dev):
    """A captured decode keeps its scratch address: a larger launch that replaces
    the per-device buffer, followed by allocations that could reuse freed
    memory, must not disturb later replays (checked against the eager decode)."""
    from copy_on_write_sdm_b200 import allocator
    from copy_on_write_sdm_b200.graph import GraphedDecode
    from copy_on_write_sdm_b200.model import LanguageModel

    torch.backends.cuda.matmul.allow_tf32 = False
    model = LanguageModel(vocab_size=256, maximum_sequence_length=64, layout="BAB", width=64, heads=4, slots=64,
                          reads=8, writes=4, memory_heads=2, activation_dtype=torch.float32)
    model.initialize_role_keyed(4)
    model = model.to(dev).eval()
    gen = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 256, (4, 40), generator=gen).to(dev)
    _, eager = model.prefill(ids[:, :8], capacity=40)
    _, graphed = model.prefill(ids[:, :8], capacity=40)
    runner = GraphedDecode(model, graphed)
    for t in range(8, 11):
        want = model.decode(ids[:, t:t + 1], eager).clone()
        got = runner.step(ids[:, t:t + 1]).clone()
        torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    assert runner.replays >= 1
    # A launch far larger than any before replaces the per-device buffer ...
    old = allocator.decode_scratch(dev, 1, 1)
    rng = np.random.default_rng(3)
    big = PoolSet(dev, rng, 1, old.numel() // 8 + 4096, 16)  # more flags than the buffer holds
    big.step(dev, rng, _per_device_launch())
    assert allocator.decode_scratch(dev, 1, 1).data_ptr() != old.data_ptr()
    # ... and fresh allocations fill whatever memory became free.
    junk = [torch.full((1 << 16,), -1, dtype=torch.int32, device=dev) for _ in range(64)]
    for t in range(11, 16):
        want = model.decode(ids[:, t:t + 1], eager).clone()
        got = runner.step(ids[:, t:t + 1]).clone()
        torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
        for x, y in zip(eager.sdm_states, graphed.sdm_states):
            assert torch.equal(x.logical_to_physical, y.logical_to_physical)
            assert int(x.free_count) == int(y.free_count)
    del junk
