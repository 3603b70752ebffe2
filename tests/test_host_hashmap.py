"""Host logic of hashed logical maps, without a GPU: table sizing and the
lifecycle wrapper's bookkeeping."""

from __future__ import annotations

import pytest

from copy_on_write_sdm_b200.allocator import PackedSDMCopyOnWriteState as S
from copy_on_write_sdm_b200.allocator import dense_maps


@pytest.mark.parametrize("live,want", [(0, 4), (1, 4), (2, 4), (3, 8), (5, 8), (6, 16), (5321, 8192),
                                       (5734, 8192), (5735, 16384)])
def test_table_size_keeps_every_bank_at_most_70_percent_full(live, want):
    t = S._table_slots_for(live)
    assert t == want
    assert t & (t - 1) == 0 and t >= 4
    assert live <= S.HASH_MAX_LOAD * t


class _Fake:
    """Stand-in pool with only the fields and methods the wrapper uses."""

    _table_slots_for = S._table_slots_for
    HASH_MAX_LOAD = S.HASH_MAX_LOAD

    def __init__(self, t):
        import torch

        self.map_table_slots = t
        self.calls = []
        self.logical_to_physical = torch.full((3, 16), -1, dtype=torch.int32)
        self.logical_to_physical[1, :9] = 0
        self.banks = 3

    def use_dense_map(self):
        self.calls.append("dense")

    def use_hash_map(self, t):
        self.calls.append(("hash", t))


def test_dense_maps_leaves_dense_pools_alone():
    pools = [_Fake(0), _Fake(0)]
    with dense_maps(pools):
        pass
    assert all(p.calls == [] for p in pools)


def test_dense_maps_expands_then_rebuilds_hashed_pools_even_when_the_operation_fails():
    pools = [_Fake(0), _Fake(8)]
    with pytest.raises(RuntimeError, match="operation failed"):
        with dense_maps(pools):
            assert pools[1].calls == ["dense"]
            raise RuntimeError("operation failed")
    # rebuilt at least as large as before, larger when a bank outgrew it (9 live -> 16)
    assert pools[1].calls == ["dense", ("hash", 16)]
    assert pools[0].calls == []


def test_bench_reports_the_fastest_end_to_end_path():
    import bench

    res = {"h2d": 1, "d2h": 2, "e2e_serial_ms": 30.0, "mapped_device": {}}
    out = bench._e2e_block(640, res, e2e_ms=10.0, e2e_mapped_ms=8.0)
    assert out["path"].startswith("DecodeSession.step_host_mapped")
    assert out["value"] == pytest.approx(640 / 8e-3)
    assert out["pipelined"]["value"] == pytest.approx(640 / 10e-3)
    assert out["h2d_bytes_per_step"] == 1 and out["d2h_bytes_per_step"] == 2
