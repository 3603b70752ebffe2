"""The session's capacity proof on the host, without a GPU.

Every decode launch mirrors each pool's settled free count, tagged with the
launch's epoch, into a page-locked host word.  A proof renewed from that
mirror (mirror - need x launches issued since) is used only when the bound
covers the step; otherwise, or when a pool changed outside the session after
the mirrored launch, the reference's synchronising ``prepare_step_capacity``
runs.  Here a fake "kernel" writes the mirror the way the decode kernel does.
"""

from __future__ import annotations

import numpy as np
import torch

from copy_on_write_sdm_b200.allocator import POOL_EPOCHS


class _Pool:
    """Host stand-in for a pool: the proof fields, a device-like free count and an
    exact ``prepare_step_capacity`` that records each (synchronising) call."""

    def __init__(self, free: int, quantum: int = 64):
        d = self.__dict__
        d["growth_quantum_rows"] = quantum
        d["proven_maximum_additional_allocations"] = 0
        d["capacity_is_proven"] = True
        d["map_table_slots"] = 0
        d["_mutations"] = 0
        self.free_count = torch.tensor(free, dtype=torch.int32)
        self.exact_calls = 0

    def prepare_step_capacity(self, need: int) -> None:
        self.exact_calls += 1
        d = self.__dict__
        d["_mutations"] += 1  # the reference path assigns, which bumps the counters
        POOL_EPOCHS[0] += 1
        d["proven_maximum_additional_allocations"] = int(self.free_count) - need


def make_session(frees, need=4):
    from copy_on_write_sdm_b200.session import DecodeSession

    s = object.__new__(DecodeSession)
    s.pools = [_Pool(f) for f in frees]
    s._pool_dicts = [p.__dict__ for p in s.pools]
    s._need = need
    s._proof_steps, s._proof_key = 0, None
    s._issued, s._mirror_from, s.snapshot_proofs = 0, 0, 0
    s._mirror_np = np.zeros(len(frees), dtype=np.int64)
    return s


def _run(s, steps, pops=4, lag=0):
    """Issue ``steps`` proofs; each step then pops ``pops`` rows from every pool,
    and the launch ``lag`` steps back mirrors its free counts (lag > 0: the host
    runs ahead of the device)."""
    for _ in range(steps):
        epoch = s._issued
        s._prove()
        for l, p in enumerate(s.pools):
            p.free_count -= pops
            hist = p.__dict__.setdefault("_history", [])
            hist.append((epoch, int(p.free_count)))
            if len(hist) > lag:
                at, free = hist[-1 - lag]
                s._mirror_np[l] = (at << 32) | free


def test_mirror_bound_replaces_the_synchronising_read():
    s = make_session([40, 400])
    _run(s, 1)
    assert [p.exact_calls for p in s.pools] == [1, 1]
    _run(s, 12, pops=1, lag=2)  # few first touches: the bounds keep covering the steps
    assert s.snapshot_proofs > 0
    assert [p.exact_calls for p in s.pools] == [1, 1]
    # every pool's proof never exceeds its true free rows
    for p in s.pools:
        assert p.__dict__["proven_maximum_additional_allocations"] <= int(p.free_count)


def test_bound_never_exceeds_the_true_free_rows_when_the_host_runs_ahead():
    s = make_session([200, 60, 1000], need=8)
    for lag in (0, 1, 3, 5):
        _run(s, 20, pops=8, lag=lag)
        for p in s.pools:
            assert p.__dict__["proven_maximum_additional_allocations"] <= int(p.free_count)


def test_insufficient_bound_falls_back_to_the_exact_check():
    s = make_session([9, 9])  # the mirrored bound soon drops below one step's need
    _run(s, 4, pops=4)
    assert all(p.exact_calls >= 2 for p in s.pools)
    assert s.snapshot_proofs == 0


def test_pool_change_outside_the_session_distrusts_older_mirror_values():
    s = make_session([400])
    _run(s, 3, pops=0)
    s.pools[0].__dict__["_mutations"] += 1  # e.g. an admission assigned to the pool
    POOL_EPOCHS[0] += 1
    s._proof_steps = 0  # the proof ran out: the next step takes the slow path
    s.pools[0].__dict__["proven_maximum_additional_allocations"] = 0
    before = s.pools[0].exact_calls
    s._prove()
    assert s._mirror_from == 3
    assert s.pools[0].exact_calls == before + 1  # mirror values of launches 0..2 are not used


def test_unset_mirror_words_are_ignored():
    s = make_session([100, 100])
    assert s._mirror_bounds(5) is None
