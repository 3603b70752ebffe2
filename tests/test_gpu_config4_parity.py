"""Decode parity at configuration 4's shape: N=65,536 slots, H=8 heads, Zipf(1.1)
routes over a seeded address permutation, 12,288 banks in one pool.

At this size a launch takes the two-pass path (a first-touch prefix pass, then
the decode pass launched as a programmatic dependent launch), so this is the
placement the configuration-4 roofline is measured on.  The pool starts from a
Zipf prefix: the written-address union of 192 tokens, packed in ``nonzero()``
order (allocator.py:664-685; checked here against the ranking of the mask)
with rows from M0.  The oracle is seeded with that exact state, then both run
8 decode steps of distinct Zipf routes (4 writes, 16 reads).  Every map entry,
the free stack and the free count must be bit-exact against the oracle's pop
order (allocator.py:1466-1481); readouts and live rows within 1e-5 abs / rel.
About 3.2 GB of map plus 1.3 GB of slab on the device and the same on the host.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cow_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 1e-5
RTOL = 1e-5
SLOTS, HEADS, WIDTH, W, R = 65536, 8, 128, 4, 16
REQUESTS, PREFIX, STEPS = 1536, 192, 8


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


class Zipf:
    """Zipf(s) popularity over a seeded permutation of ``n`` addresses."""

    def __init__(self, n, s, gen, device):
        p = torch.arange(1, n + 1, device=device, dtype=torch.float64).pow(-s)
        p /= p.sum()
        self.n = n
        self.cdf = torch.cumsum(p, 0).float()
        self.logp = p.log().float()
        self.perm = torch.randperm(n, generator=gen, device=device)

    def with_replacement(self, shape, gen):
        u = torch.rand(*shape, generator=gen, device=self.cdf.device)
        return self.perm[torch.searchsorted(self.cdf, u).clamp_(max=self.n - 1)]

    def distinct(self, rows, k, gen, chunk=1024):
        out = []
        for r0 in range(0, rows, chunk):
            r = min(chunk, rows - r0)
            g = torch.rand(r, self.n, generator=gen, device=self.cdf.device).clamp_(min=1e-20)
            g.log_().neg_().log_().neg_().add_(self.logp)
            out.append(self.perm[g.topk(k, dim=-1).indices])
        return torch.cat(out)


def _dense_map(st):
    """The pool's logical-to-physical map in the reference's dense form."""
    from copy_on_write_sdm_b200.allocator import dense_maps

    with dense_maps([st]):
        return st.logical_to_physical.cpu().numpy()


@pytest.mark.parametrize("map_kind", ["dense", "hash"])
def test_config4_shape_two_pass_decode_matches_oracle(dev, map_kind):
    """``hash``: the same trace on per-bank hashed tables (sized for the prefix
    plus the trace's first touches); maps compared in their dense form."""
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, _lib, packed_sdm_cow_step_layers

    lib = _lib.load()
    banks = REQUESTS * HEADS
    gen = torch.Generator(device=dev).manual_seed(44)
    zipf = Zipf(SLOTS, 1.1, gen, dev)
    m0 = 0.02 * torch.randn(HEADS, SLOTS, WIDTH, generator=gen, device=dev)
    mapping = torch.full((banks, SLOTS), -1, dtype=torch.int32, device=dev)
    status = torch.zeros((), dtype=torch.int32, device=dev)
    stream = _lib.stream_of(dev)
    for t0 in range(0, PREFIX, 64):
        widx = zipf.with_replacement((banks, 64, W), gen)
        _lib.check(lib.cow_prefill_mark(widx.data_ptr(), _lib.I64, banks, 64, W, SLOTS, mapping.data_ptr(),
                                        status.data_ptr(), stream), "cow_prefill_mark")
    touched = int((mapping >= 0).sum())
    extra = banks * W * STEPS
    templates = torch.arange(HEADS, device=dev, dtype=torch.int64).repeat(REQUESTS)
    st = PackedSDMCopyOnWriteState._pack_layout(
        m0, mapping, templates, capacity_rows=touched + extra, state_dtype=torch.float32,
        maximum_future_allocations=extra, growth_quantum_rows=0, row_source=("m0", None), validate=True)
    del mapping
    # The prefix pack: live slots numbered in nonzero() order, rows = M0, stack arange(A, C).
    mp = st.logical_to_physical.cpu().numpy()
    live = mp >= 0
    assert int(live.sum()) == touched
    np.testing.assert_array_equal(mp[live], np.arange(touched, dtype=np.int32))  # C order = nonzero() order
    assert (mp[~live] == -1).all()
    tmpl = templates.cpu().numpy()
    m0_np = m0.cpu().numpy()
    slab = st.values.cpu().numpy().copy()
    b, s = np.nonzero(live)
    np.testing.assert_array_equal(slab[mp[b, s]], m0_np[tmpl[b], s])
    del b, s, live
    fc = int(st.free_count)
    assert fc == extra
    np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), np.arange(touched, touched + extra))
    ref = O.OracleState(shared_initial_memory=m0_np, template_indices=tmpl, values=slab,
                        logical_to_physical=mp.copy(), free_rows=st.free_rows.cpu().numpy().copy(), free_count=fc)
    if map_kind == "hash":
        t = st.use_hash_map(headroom_rows_per_bank=W * STEPS)
        assert st.storage_bytes()["logical_to_physical"] == banks * t * 8 < banks * SLOTS * 4 // 8
    first_total = 0
    for step in range(STEPS):
        x = dict(write_indices=zipf.distinct(banks, W, gen), read_indices=zipf.distinct(banks, R, gen),
                 write_weights=torch.softmax(torch.randn(banks, W, generator=gen, device=dev), -1),
                 read_weights=torch.softmax(torch.randn(banks, R, generator=gen, device=dev), -1),
                 values=torch.randn(banks, WIDTH, generator=gen, device=dev),
                 input_gate=torch.rand(banks, generator=gen, device=dev),
                 forget_log_gate=-torch.rand(banks, generator=gen, device=dev))
        (got,), (first,) = packed_sdm_cow_step_layers([st], [x], collect_diagnostics=True)
        want, want_first = O.packed_step(ref, **{k: v.cpu().numpy() for k, v in x.items()})
        np.testing.assert_allclose(got.cpu().numpy(), want, atol=ATOL, rtol=RTOL)
        np.testing.assert_array_equal(first.cpu().numpy().astype(bool), want_first)
        first_total += int(want_first.sum())
        assert int(st.free_count) == ref.free_count
        assert st.status() == 0
        if step % 4 == 3:
            np.testing.assert_array_equal(_dense_map(st), ref.logical_to_physical)
            fc = int(st.free_count)
            np.testing.assert_array_equal(st.free_rows[:fc].cpu().numpy(), ref.free_stack())
    # Zipf routes over a 192-token prefix: a mix of private reuse and first touches.
    assert 0 < first_total < banks * W * STEPS
    mp = _dense_map(st)
    b, s = np.nonzero(mp >= 0)
    rows = mp[b, s]
    del b, s
    np.testing.assert_allclose(st.values.cpu().numpy()[rows], ref.values[rows], atol=ATOL, rtol=RTOL)
    st.validate_invariants()
