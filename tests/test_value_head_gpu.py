"""Fused critic value head + clipped value loss (GPU) against the fp32 PyTorch expression of the same op."""

import pytest
import torch

from meshy_b200.backend.critic.model import value_head_loss
from meshy_b200.backend.vapo import clipped_value_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,D,clip", [(1000, 1536, None), (3000, 2048, 0.2), (5, 256, 0.5)])
def test_value_head_loss_matches_fp32(T, D, clip):
    g = torch.Generator(device="cuda").manual_seed(T)
    h = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(1, D, device="cuda", generator=g) * 0.02).requires_grad_(True)
    b = torch.randn(1, device="cuda", generator=g).requires_grad_(True)
    ret = torch.randn(T, device="cuda", generator=g)
    mask = (torch.rand(T, device="cuda", generator=g) > 0.3).float()
    old = torch.randn(T, device="cuda", generator=g) if clip else None
    denom = float(mask.sum())
    loss, v = value_head_loss(h, w, b, ret, mask, old, clip, denom)
    loss.backward()
    hr = h.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    br = b.detach().clone().requires_grad_(True)
    vr = (hr @ wr.t()).squeeze(-1) + br
    lr = (clipped_value_error(vr, ret, old, clip) * mask).sum() / denom
    lr.backward()
    assert abs(float(loss) - float(lr)) <= 1e-4 * max(1.0, abs(float(lr)))
    assert _rel(v, vr.detach()) < 1e-5
    assert _rel(h.grad, hr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-4
    assert _rel(b.grad, br.grad) < 1e-4
