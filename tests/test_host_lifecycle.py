"""Host-side lifecycle bookkeeping that needs no GPU: the maximum request
position and the active-request flags are read from their tensors once and
read again only when a tensor is replaced or changed in place."""

from __future__ import annotations

import torch


def _state(positions):
    from copy_on_write_sdm_b200.inference import FaithfulSDMDecodeState

    n = positions.numel()
    return FaithfulSDMDecodeState(
        layout="B", position=0, capacity=64, activation_dtype=torch.float32,
        active_sequences=torch.ones(n, dtype=torch.bool), sdm_layer_positions=(0,), sdm_states=(),
        dense_keys=(), dense_values=(), positions=positions)


def test_max_position_follows_the_positions_tensor():
    state = _state(torch.tensor([3, 9, 5]))
    assert state._max_position() == 9
    state.positions.add_(1)  # in place: the version moves, so the maximum is read again
    assert state._max_position() == 10
    state.positions = torch.tensor([1, 2])  # replaced
    assert state._max_position() == 2
    state.positions[0] = 40  # indexed in-place write
    assert state._max_position() == 40


def test_max_position_is_cached_while_unchanged(monkeypatch):
    state = _state(torch.tensor([7, 2]))
    assert state._max_position() == 7
    calls = []
    original = torch.Tensor.max

    def counting_max(self, *a, **k):
        calls.append(1)
        return original(self, *a, **k)

    monkeypatch.setattr(torch.Tensor, "max", counting_max)
    assert state._max_position() == 7
    assert not calls


def test_slab_reserve_is_released_when_the_slab_is_replaced():
    """Growth keeps the slab and stack as views of a reserved store; a slab or stack
    replaced any other way (trim, restore) drops that store so its memory is freed."""
    from copy_on_write_sdm_b200.allocator import PackedSDMCopyOnWriteState

    st = PackedSDMCopyOnWriteState(
        shared_initial_memory=torch.zeros(1, 4, 8), template_indices=torch.zeros(2, dtype=torch.int64),
        values=torch.zeros(16, 8), logical_to_physical=torch.full((2, 4), -1, dtype=torch.int32),
        free_rows=torch.arange(16, dtype=torch.int32), free_count=torch.tensor(16, dtype=torch.int32),
        overflow_flag=torch.tensor(0, dtype=torch.int32))
    store = (torch.zeros(32, 8), torch.zeros(32, dtype=torch.int32))
    st.__dict__["_slab_store"] = store
    st.values = store[0][:24]  # growth inside the reserve: same storage, the store stays
    st.free_rows = store[1][:24]
    assert st.__dict__.get("_slab_store") is store and st.capacity_rows == 24
    st.values = torch.zeros(20, 8)  # replaced by other means: the reserve goes
    assert "_slab_store" not in st.__dict__


def test_active_flags_mirror_follows_the_tensor():
    """The host list of active requests is read from the tensor once and again
    only when the tensor is replaced or changed in place."""
    state = _state(torch.tensor([3, 9, 5]))
    assert state._active_host() == [True, True, True]
    state.active_sequences[1] = False  # a caller's in-place write: the version moves
    assert state._active_host() == [True, False, True]
    state.active_sequences = torch.tensor([False, True])  # replaced
    assert state._active_host() == [False, True]


def test_active_flags_mirror_is_not_reread_while_unchanged(monkeypatch):
    state = _state(torch.tensor([1, 2, 3]))
    state._active_host()
    calls = []
    original = torch.Tensor.tolist

    def counting_tolist(self, *a, **k):
        calls.append(1)
        return original(self, *a, **k)

    monkeypatch.setattr(torch.Tensor, "tolist", counting_tolist)
    for _ in range(3):
        assert state._active_host() == [True, True, True]
    assert calls == []


def test_compact_without_releases_keeps_every_request_and_reads_no_flags(monkeypatch):
    state = _state(torch.tensor([4, 6]))
    state._active_host()
    def no_read(self, *a, **k):
        raise AssertionError("the active flags were read again")

    monkeypatch.setattr(torch.Tensor, "tolist", no_read)
    keep = state.compact()
    monkeypatch.undo()
    assert keep.tolist() == [0, 1] and state.position == 6
