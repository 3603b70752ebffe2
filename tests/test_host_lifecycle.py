"""Host-side lifecycle bookkeeping that needs no GPU: the maximum request
position is read from the positions tensor once and read again only when that
tensor is replaced or changed in place."""

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
