"""The no-alloc decode entry point (cow_decode_step_noalloc) through the C ABI.

It serves callers that cannot allocate device memory when they call in (a
foreign-language host that does not own the process's GPU allocator, or a
serving loop that must not allocate while decoding): its scan scratch is a
fixed array inside the library.  Two identical pools are stepped side by
side, one through cow_decode_step with torch-allocated scratch and one
through cow_decode_step_noalloc, on two calls in a row (the second call runs
on whatever the first left in the shared array); readouts must agree within
the 1e-5 tolerance of the other parity tests and maps / free stacks exactly.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 1e-5
RTOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _pools(dev, layers, banks, slots, width, seed):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(layers):
        m0 = (0.02 * torch.randn(1, slots, width, generator=g)).to(dev)
        out.append(PackedSDMCopyOnWriteState.allocate(m0, banks=banks, capacity_rows=banks * slots))
    return out


def test_noalloc_matches_scratch_entry_point_twice(dev):
    from copy_on_write_sdm_b200 import _lib, allocator

    lib = _lib.load()
    layers, banks, slots, width, W, R = 7, 64, 256, 128, 4, 16
    ref_pools = _pools(dev, layers, banks, slots, width, seed=3)
    new_pools = _pools(dev, layers, banks, slots, width, seed=3)
    rng = np.random.default_rng(9)
    stream = _lib.stream_of(dev)
    scratch = torch.zeros(lib.cow_decode_scratch_bytes(banks * layers, layers), dtype=torch.uint8, device=dev)
    for call in range(2):
        xs = [{k: torch.from_numpy(v).to(dev) for k, v in O.synthetic_step_inputs(rng, banks, slots, width, W, R).items()}
              for _ in range(layers)]
        outs = []
        for pools, noalloc in ((ref_pools, False), (new_pools, True)):
            args = [allocator._StepArgs.make(x["write_indices"], x["write_weights"], x["values"], x["input_gate"],
                                             x["forget_log_gate"], x["read_indices"], x["read_weights"], None,
                                             collect=False) for x in xs]
            c_pools = (_lib.CowPool * layers)(*[p._pool() for p in pools])
            c_steps = (_lib.CowStep * layers)(*[a.struct for a in args])
            if noalloc:
                rc = lib.cow_decode_step_noalloc(c_pools, c_steps, layers, W, R, _lib.I64, _lib.F32, stream)
            else:
                rc = lib.cow_decode_step(c_pools, c_steps, layers, W, R, _lib.I64, _lib.F32,
                                         scratch.data_ptr(), scratch.numel(), stream)
            assert rc == _lib.OK, (call, noalloc, rc)
            outs.append([a.output for a in args])
        torch.cuda.synchronize(dev)
        for a, b in zip(*outs):
            np.testing.assert_allclose(b.cpu().numpy(), a.cpu().numpy(), atol=ATOL, rtol=RTOL)
        for p, q in zip(ref_pools, new_pools):
            assert torch.equal(p.logical_to_physical, q.logical_to_physical)
            assert int(p.free_count) == int(q.free_count) < banks * slots
            fc = int(p.free_count)
            assert torch.equal(p.free_rows[:fc], q.free_rows[:fc])
            assert q.status() == 0
    for q in new_pools:
        q.validate_invariants()


def test_noalloc_rejects_more_banks_than_its_scratch(dev):
    from copy_on_write_sdm_b200 import _lib

    lib = _lib.load()
    pool = _lib.CowPool()
    pool.banks = 200_000  # cow_decode_scratch_bytes(200000, 1) > 1 MiB: rejected before any launch
    pool.width = 128
    step = _lib.CowStep()
    rc = lib.cow_decode_step_noalloc(ctypes.byref(pool), ctypes.byref(step), 1, 4, 16, _lib.I64, _lib.F32,
                                     _lib.stream_of(dev))
    assert rc == _lib.ERR_SCRATCH_LIMIT
    assert lib.cow_decode_scratch_bytes(130_000, 1) <= _lib.NOALLOC_SCRATCH_BYTES
