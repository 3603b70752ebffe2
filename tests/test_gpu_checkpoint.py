"""Serving checkpoints on the GPU: a request checkpointed mid-decode, written to
a file, read back and admitted into another live batch decodes exactly as it
would have in its original batch (allocator state bit for bit, logits within
1e-4), and migrate_requests moves requests between live batches."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda:0")


def _model(dev):
    from copy_on_write_sdm_b200.model import LanguageModel

    model = LanguageModel(vocab_size=512, maximum_sequence_length=64, layout="BAB", width=64, heads=4, slots=64,
                          reads=8, writes=4, memory_heads=2, activation_dtype=torch.float32)
    model.initialize_role_keyed(5)
    return model.to(dev).eval()


def _bank_rows(state, request, heads=2):
    """Effective [H, N, D] table of one request in every SDM layer."""
    out = []
    for st in state.sdm_states:
        dense = st.materialize_dense()
        out.append(dense[request * heads:(request + 1) * heads])
    return out


@pytest.mark.parametrize("quantum", [0, 16])
def test_checkpoint_restore_admit_continues_exactly(dev, tmp_path, quantum):
    from copy_on_write_sdm_b200.checkpoint import ServingCheckpoint, export_requests, restore_requests

    model = _model(dev)
    gen = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 512, (4, 40), generator=gen).to(dev)
    other = torch.randint(0, 512, (2, 40), generator=gen).to(dev)
    _, src = model.prefill(ids[:, :10], capacity=48, sdm_growth_quantum_rows=quantum)
    for t in range(10, 14):
        model.decode(ids[:, t:t + 1], src)

    ckpt = export_requests(src, [3, 1])
    path = tmp_path / "two.ckpt"
    ckpt.save(path)
    loaded = ServingCheckpoint.load(path)
    assert loaded.requests == 2 and loaded.live_rows() == ckpt.live_rows() > 0
    m0s = [model.stack.sdm_layers[str(i)].initial_memory for i in src.sdm_layer_positions]
    cohort = restore_requests(loaded, m0s)
    for a, b in zip(_bank_rows(src, 3), _bank_rows(cohort, 0)):
        assert torch.equal(a, b)
    for a, b in zip(_bank_rows(src, 1), _bank_rows(cohort, 1)):
        assert torch.equal(a, b)

    # destination: two other requests at another position, then the restored pair
    # a fixed pool (no growth quantum) must already hold room for the admitted rows
    _, dst = model.prefill(other[:, :7], capacity=48, sdm_growth_quantum_rows=quantum,
                           sdm_capacity_rows=None if quantum else 2048)
    model.decode(other[:, 7:8], dst)
    dst.admit(cohort)
    assert dst.batch == 4
    for t in range(14, 20):
        want = model.decode(ids[:, t:t + 1], src)
        step_ids = torch.cat([other[:, t - 6:t - 5], ids[3:4, t:t + 1], ids[1:2, t:t + 1]], dim=0)
        got = model.decode(step_ids, dst)
        torch.testing.assert_close(got[2], want[3], atol=LOGIT_TOL, rtol=LOGIT_TOL)
        torch.testing.assert_close(got[3], want[1], atol=LOGIT_TOL, rtol=LOGIT_TOL)
    for a, b in zip(_bank_rows(src, 3), _bank_rows(dst, 2)):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)
    for st in (*src.sdm_states, *dst.sdm_states):
        st.validate_invariants()


def test_migrate_requests_moves_and_releases(dev):
    from copy_on_write_sdm_b200.checkpoint import migrate_requests

    model = _model(dev)
    gen = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 512, (3, 30), generator=gen).to(dev)
    _, src = model.prefill(ids[:, :8], capacity=32, sdm_growth_quantum_rows=16)
    _, ref = model.prefill(ids[:, :8], capacity=32, sdm_growth_quantum_rows=16)
    _, dst = model.prefill(ids[:1, :8], capacity=32, sdm_growth_quantum_rows=16)
    live_before = sum(int(st.allocated_rows_tensor()) for st in src.sdm_states)
    assert migrate_requests(src, [2], dst) == 1
    assert src.batch == 2 and dst.batch == 2
    assert sum(int(st.allocated_rows_tensor()) for st in src.sdm_states) < live_before
    for t in range(8, 12):
        want = model.decode(ids[:, t:t + 1], ref)
        got_src = model.decode(ids[:2, t:t + 1], src)
        got_dst = model.decode(torch.cat([ids[:1, t:t + 1], ids[2:3, t:t + 1]]), dst)
        torch.testing.assert_close(got_src, want[:2], atol=LOGIT_TOL, rtol=LOGIT_TOL)
        torch.testing.assert_close(got_dst[1], want[2], atol=LOGIT_TOL, rtol=LOGIT_TOL)
    with pytest.raises(ValueError):
        migrate_requests(src, [5], dst)
