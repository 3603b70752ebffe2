"""The session's capacity proof on the host, without a GPU: a proof renewed from a
background free-count snapshot is used only when its lower bound
(snapshot - need x steps issued since) covers the step; otherwise, or after a
pool changed, or once a step decoded on another stream, the reference's
synchronising ``prepare_step_capacity`` runs."""

from __future__ import annotations

import pytest
import torch


class _Pool:
    """Host stand-in for a pool: the proof fields, a device-like free count and an
    exact ``prepare_step_capacity`` that records each (synchronising) call."""

    def __init__(self, free: int, quantum: int = 64):
        d = self.__dict__
        d["growth_quantum_rows"] = quantum
        d["proven_maximum_additional_allocations"] = 0
        d["capacity_is_proven"] = True
        d["_mutations"] = 0
        self.free_count = torch.tensor(free, dtype=torch.int32)
        self.exact_calls = 0

    def prepare_step_capacity(self, need: int) -> None:
        self.exact_calls += 1
        d = self.__dict__
        d["_mutations"] += 1  # the reference path assigns, which bumps the counter
        d["proven_maximum_additional_allocations"] = int(self.free_count) - need


class _Event:
    def record(self, *a):
        pass

    def query(self):
        return True


@pytest.fixture()
def session(monkeypatch):
    from copy_on_write_sdm_b200.session import DecodeSession

    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)

    def make(frees, need=4):
        s = object.__new__(DecodeSession)
        s.pools = [_Pool(f) for f in frees]
        s._need = need
        s._proof_steps, s._proof_key = 0, None
        s._issued, s._snap, s._snapshots, s.snapshot_proofs = 0, None, True, 0
        s._snap_host = torch.empty(len(frees), dtype=torch.int32)
        return s
    return make


def _run(s, steps, pops=4, on_current=True):
    """Issue `steps` proofs; each step then pops `pops` rows from every pool."""
    for _ in range(steps):
        s._prove(on_current=on_current)
        for p in s.pools:
            p.free_count -= pops


def test_snapshot_bound_replaces_the_synchronising_read(session):
    s = session([40, 400])
    _run(s, 1)
    assert [p.exact_calls for p in s.pools] == [1, 1]
    _run(s, 12, pops=1)  # few first touches: the bounds keep covering the steps
    assert s.snapshot_proofs > 0
    # every pool's proof never exceeds its true free rows
    for p in s.pools:
        assert p.__dict__["proven_maximum_additional_allocations"] <= int(p.free_count)


def test_insufficient_bound_falls_back_to_the_exact_check(session):
    s = session([9, 9])  # the snapshot bound soon drops below one step's need
    _run(s, 4, pops=4)
    assert all(p.exact_calls >= 2 for p in s.pools)
    assert s.snapshot_proofs == 0


def test_pool_change_invalidates_a_pending_snapshot(session):
    s = session([40])
    _run(s, 1, pops=0)
    while s._snap is None:
        _run(s, 1, pops=0)
    s.pools[0].__dict__["_mutations"] += 1  # e.g. an admission assigned to the pool
    assert s._snap_bounds() is None


def test_another_stream_turns_snapshots_off(session):
    s = session([400])
    _run(s, 3, pops=0)
    _run(s, 1, pops=0, on_current=False)
    assert s._snapshots is False and s._snap is None
    _run(s, 30, pops=1)
    assert s.snapshot_proofs == 0
