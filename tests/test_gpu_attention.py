"""The fused dense-attention decode kernel (cow_attention_mlp_decode) against the
PyTorch path it replaces (CausalSelfAttention.decode_with_cache, the residual
adds and the ResidualMLP): block outputs within 1e-5 and the K/V caches equal
after the step (this token's key and value stored at each request's position),
for shared (int) and per-request positions, first and last cache slots."""

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


def _block(width, heads, dev, seed):
    from copy_on_write_sdm_b200.model import DenseAttentionBlock

    torch.manual_seed(seed)
    blk = DenseAttentionBlock(width, heads).to(dev).eval()
    with torch.no_grad():
        for p in (blk.attention.norm.weight, blk.attention.norm.bias, blk.mlp.norm.weight, blk.mlp.norm.bias):
            p.add_(0.3 * torch.randn_like(p))
    return blk


@pytest.mark.parametrize("width,heads,batch,cap,where", [
    (128, 4, 16, 512, "ragged"), (128, 4, 16, 512, 0), (128, 4, 16, 512, 511), (64, 2, 3, 40, "ragged"),
    (256, 8, 5, 100, 57), (96, 3, 2, 17, "ragged"), (128, 1, 4, 64, 63),
])
def test_decode_residual_matches_torch(dev, width, heads, batch, cap, where):
    blk = _block(width, heads, dev, width + cap)
    hw = width // heads
    kc = torch.randn(batch, heads, cap, hw, device=dev)
    vc = torch.randn(batch, heads, cap, hw, device=dev)
    tokens = torch.randn(batch, 1, width, device=dev)
    if where == "ragged":
        position = torch.randint(0, cap, (batch,), device=dev)
        position[0] = cap - 1
        position[-1] = 0
    else:
        position = where
    k1, v1, k2, v2 = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    with torch.no_grad():
        assert blk._fused_decode_ok(tokens, k1, v1)
        got = blk._decode_fused(tokens, k1, v1, position)
        t = tokens + blk.attention.decode_with_cache(tokens, k2, v2, position=position)
        want = t + blk.mlp(t)
    torch.testing.assert_close(got, want, atol=TOL, rtol=TOL)
    torch.testing.assert_close(k1, k2, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(v1, v2, atol=1e-6, rtol=1e-6)


def test_position_outside_cache_is_rejected_or_nan(dev):
    blk = _block(64, 2, dev, 0)
    kc = torch.zeros(2, 2, 8, 32, device=dev)
    vc = torch.zeros_like(kc)
    tokens = torch.randn(2, 1, 64, device=dev)
    with torch.no_grad():
        with pytest.raises(ValueError):
            blk._decode_fused(tokens, kc, vc, 8)
        out = blk._decode_fused(tokens, kc, vc, torch.tensor([3, 8], device=dev))
    assert torch.isnan(out[1]).all() and not torch.isnan(out[0]).any()
    assert kc[1].abs().sum() == 0 and vc[1].abs().sum() == 0  # nothing stored for the bad row
    assert kc[0, :, 3].abs().sum() > 0
