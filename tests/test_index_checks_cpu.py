"""Debug index validation in front of the native kernels (``MESHY_CHECK_INDICES=1``, ``meshy_b200.ops.checks``):
an out-of-range token id, label, KV-cache slot, block-table page, sequence length or expert id raises
``IndexError`` naming the op and the value; valid inputs pass; with the switch off nothing is checked."""

import pytest
import torch

from meshy_b200.ops import checks


@pytest.fixture
def on():
    checks.set_enabled(True)
    yield
    checks.set_enabled(False)


def test_entry_points_reject_bad_indices(on):
    from meshy_b200.ops import decode as D
    from meshy_b200.ops import functional as Fx

    w = torch.randn(50, 8)
    assert Fx.embedding(torch.tensor([0, 49]), w).shape == (2, 8)
    with pytest.raises(IndexError, match="embedding token ids: index 50"):
        Fx.embedding(torch.tensor([3, 50]), w)
    h = torch.randn(4, 8)
    Fx.lm_head_logprobs(h, w, torch.tensor([1, 0, 2, 49]), with_entropy=False)
    with pytest.raises(IndexError, match="LM-head labels: index 77"):
        Fx.lm_head_logprobs(h, w, torch.tensor([1, 2, 3, 77]), with_entropy=False)
    with pytest.raises(IndexError, match="LM-head labels: index -1"):
        Fx.lm_head_logprobs(h, w, torch.tensor([1, -1, 3, 4]), with_entropy=False)
    n_pages, hkv, page, hd = 3, 2, 4, 8
    kc, vc = torch.zeros(n_pages, hkv, page, hd), torch.zeros(n_pages, hkv, page, hd)
    k = torch.randn(2, hkv, hd)
    D.kv_write(k, k, kc, vc, torch.tensor([0, 11]))
    with pytest.raises(IndexError, match="KV-cache slots: index 12"):
        D.kv_write(k, k, kc, vc, torch.tensor([0, 12]))
    q = torch.randn(2, 4, hd)
    bt = torch.tensor([[0, 1, 99], [2, 99, 99]])  # entries past each row's length are never read
    D.paged_attention(q, kc, vc, bt, torch.tensor([8, 3]))
    with pytest.raises(IndexError, match="paged attention block table: index 99"):
        D.paged_attention(q, kc, vc, bt, torch.tensor([9, 3]))
    with pytest.raises(IndexError, match="paged attention sequence lengths"):
        D.paged_attention(q, kc, vc, bt, torch.tensor([13, 3]))
    with pytest.raises(IndexError, match="MoE expert ids"):
        checks.check_range("MoE expert ids", torch.tensor([[0, 8]]), 0, 8)


def test_switch_off_checks_nothing():
    checks.set_enabled(False)
    checks.check_range("x", torch.tensor([5]), 0, 2)  # no error
    assert not checks.enabled()
