"""Serving checkpoint file format on the CPU: save -> load is the identity."""

from __future__ import annotations

import pytest
import torch

from copy_on_write_sdm_b200.checkpoint import MAGIC, LayerCheckpoint, ServingCheckpoint


def _ckpt(rows_dtype):
    g = torch.Generator().manual_seed(0)
    layers = [LayerCheckpoint(live=torch.tensor([3, 7, 64, 200], dtype=torch.int64),
                              rows=torch.randn(4, 16, generator=g).to(rows_dtype),
                              templates=torch.tensor([0, 1], dtype=torch.int64), slots=128, growth_quantum_rows=8),
              LayerCheckpoint(live=torch.empty(0, dtype=torch.int64), rows=torch.empty(0, 16, dtype=rows_dtype),
                              templates=torch.tensor([0, 1], dtype=torch.int64), slots=128, growth_quantum_rows=0)]
    return ServingCheckpoint(layout="BAB", capacity=32, activation_dtype=torch.bfloat16,
                             positions=torch.tensor([11], dtype=torch.int64), sdm_layer_positions=(0, 2),
                             layers=layers, dense_keys=[torch.randn(1, 2, 32, 8, generator=g)],
                             dense_values=[torch.randn(1, 2, 32, 8, generator=g)])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_save_load_round_trip(tmp_path, dtype):
    a = _ckpt(dtype)
    path = tmp_path / "serving.ckpt"
    a.save(path)
    raw = path.read_bytes()
    assert raw[:8] == MAGIC
    b = ServingCheckpoint.load(path)
    assert (b.layout, b.capacity, b.activation_dtype, b.sdm_layer_positions) == \
        (a.layout, a.capacity, a.activation_dtype, a.sdm_layer_positions)
    assert torch.equal(a.positions, b.positions)
    for x, y in zip(a.layers, b.layers):
        assert torch.equal(x.live, y.live) and torch.equal(x.templates, y.templates)
        assert x.rows.dtype == y.rows.dtype and torch.equal(x.rows.view(torch.uint8), y.rows.view(torch.uint8))
        assert (x.slots, x.growth_quantum_rows) == (y.slots, y.growth_quantum_rows)
    for x, y in zip(a.dense_keys + a.dense_values, b.dense_keys + b.dense_values):
        assert torch.equal(x, y)
    assert b.requests == 1 and b.live_rows() == 4 and b.nbytes() == a.nbytes()


def test_rejects_foreign_and_truncated_files(tmp_path):
    p = tmp_path / "x.ckpt"
    p.write_bytes(b"NOTACKPT" + b"\0" * 32)
    with pytest.raises(ValueError):
        ServingCheckpoint.load(p)
    _ckpt(torch.float32).save(p)
    data = p.read_bytes()
    p.write_bytes(data[:-40])
    with pytest.raises(ValueError):
        ServingCheckpoint.load(p)
