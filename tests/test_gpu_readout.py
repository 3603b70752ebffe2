"""The fused readout + MLP kernel (cow_readout_mlp_step) against the PyTorch
path it replaces: readings norm, channel gate, output projection, residual add,
then the pre-norm GELU MLP and its residual add, within 1e-5 (both FP32; the
kernel sums its dot products in its own order)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda:0")


@pytest.mark.parametrize("width,heads,batch,time", [
    (128, 2, 16, 1), (64, 4, 3, 5), (256, 8, 2, 1), (512, 4, 4, 2), (96, 3, 1, 1), (128, 1, 37, 1),
    (256, 8, 9, 3),
])
def test_finish_residual_matches_torch(dev, width, heads, batch, time):
    from copy_on_write_sdm_b200.model import ResidualMLP
    from copy_on_write_sdm_b200.sdm import SparseDeltaMemory

    torch.manual_seed(width + heads + time)
    m = SparseDeltaMemory(width, slots=256, reads=8, writes=4, memory_heads=heads).to(dev).eval()
    mlp = ResidualMLP(width).to(dev).eval()
    with torch.no_grad():  # non-trivial norms and biases
        for p in (m.readings_norm.weight, m.readings_norm.bias, mlp.norm.weight, mlp.norm.bias,
                  m.output_gate.bias, m.output_projection.bias):
            p.add_(0.3 * torch.randn_like(p))
    tokens = torch.randn(batch, time, width, device=dev)
    normalized = torch.randn(batch, time, width, device=dev)
    readings = 2.0 * torch.randn(batch * heads, time, width // heads, device=dev) + 0.5
    with torch.no_grad():
        assert m._fused_readout_ok(tokens, normalized, readings, mlp) == (width <= 256)
        got = m._readout_step(tokens, normalized, readings, mlp)  # the kernel, also beyond the dispatch limit
        t1 = tokens + m.finish(normalized, readings)
        want = t1 + mlp(t1)
    assert got.shape == want.shape and got.dtype == want.dtype
    torch.testing.assert_close(got, want, atol=TOL, rtol=TOL)


def test_weight_update_rebuilds_transposed_cache(dev):
    from copy_on_write_sdm_b200.model import ResidualMLP
    from copy_on_write_sdm_b200.sdm import SparseDeltaMemory

    torch.manual_seed(0)
    m = SparseDeltaMemory(128, slots=256, reads=8, writes=4, memory_heads=2).to(dev).eval()
    mlp = ResidualMLP(128).to(dev).eval()
    tokens, normalized = torch.randn(2, 2, 1, 128, device=dev)
    readings = torch.randn(4, 1, 64, device=dev)
    with torch.no_grad():
        m.finish_residual(tokens, normalized, readings, mlp)
        mlp.input.weight.mul_(-1.5)  # in place: the cached transpose must follow
        got = m.finish_residual(tokens, normalized, readings, mlp)
        t1 = tokens + m.finish(normalized, readings)
        want = t1 + mlp(t1)
    torch.testing.assert_close(got, want, atol=TOL, rtol=TOL)


def test_training_mode_takes_the_torch_path(dev):
    from copy_on_write_sdm_b200.model import ResidualMLP
    from copy_on_write_sdm_b200.sdm import SparseDeltaMemory

    m = SparseDeltaMemory(64, slots=64, reads=4, writes=2, memory_heads=2).to(dev)
    mlp = ResidualMLP(64).to(dev)
    x = torch.randn(1, 1, 64, device=dev)
    r = torch.randn(2, 1, 32, device=dev)
    assert not m._fused_readout_ok(x, x, r, mlp)
    assert m.eval()._fused_readout_ok(x, x, r, mlp.eval())
