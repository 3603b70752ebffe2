"""The fused controller kernels against the PyTorch controller: the whole
controller (cow_controller_step) and the route selection alone
(cow_route_controller) give identical addresses, and weights, gates, values
and the normalised tokens within 1e-6 (1e-5 for the fully fused kernel, whose
layer norm and projections sum in their own order)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda:0")


@pytest.mark.parametrize("slots,heads,reads,writes,time", [
    (256, 1, 16, 4, 1), (256, 2, 16, 4, 7), (4096, 4, 16, 4, 3), (65536, 8, 16, 4, 1), (1024, 1, 32, 8, 2),
    (64, 2, 8, 4, 5),
])
@pytest.mark.parametrize("whole", [True, False])
def test_fused_routes_match_torch(dev, slots, heads, reads, writes, time, whole):
    from copy_on_write_sdm_b200.sdm import SparseDeltaMemory

    width = 64 * heads if heads > 1 else 128
    torch.manual_seed(slots + heads + time)
    m = SparseDeltaMemory(width, slots=slots, reads=reads, writes=writes, memory_heads=heads).to(dev).eval()
    tokens = torch.randn(6, time, width, device=dev)
    with torch.no_grad():
        assert m._fused_routes_ok(tokens)
        ntot = 4 * heads * int(slots ** 0.5) + width + 2 * heads
        assert m._fused_controller_ok() == (ntot <= 4096)
        if whole and ntot > 4096:
            pytest.skip("projection wider than the whole-controller kernel; the route kernel covers it")
        if not whole:
            m._fused_controller_ok = lambda: False  # routes fused, projections in PyTorch
        got = m.controller(tokens)
        m._fused_routes_ok = lambda t: False  # the PyTorch path
        want = m.controller(tokens)
    assert torch.equal(got.read_indices, want.read_indices)
    assert torch.equal(got.write_indices, want.write_indices)
    for a, b in ((got.read_weights, want.read_weights), (got.write_weights, want.write_weights),
                 (got.input_gate, want.input_gate), (got.forget_log_gate, want.forget_log_gate),
                 (got.values, want.values), (got.normalized, want.normalized)):
        assert a.shape == b.shape and a.dtype == b.dtype
        tol = 1e-5 if whole else 1e-6
        torch.testing.assert_close(a, b, atol=tol, rtol=tol)
