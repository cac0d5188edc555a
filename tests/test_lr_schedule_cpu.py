"""Learning-rate schedule: constant after warmup unless a recipe opts into decay; ``lr_decay_ratio=None`` is
a linear decay to zero that starts right after warmup (values of the reference's logged curve: 9.9833e-7 at
step 1 and 8.85e-7 at step 69 for lr 1e-6 over 600 steps); warmup ramps; configuration is validated."""

import pytest

from meshy_b200.backend.flat import lr_lambda
from meshy_b200.config import TrainerConfig


def _curve(steps=600, n=70, **kw):
    c = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", steps=steps, lr=1e-6, **kw)
    return [c.lr * lr_lambda(s, warmup=c.warmup_steps, total=c.steps, decay_ratio=c.lr_decay_ratio,
                             decay_type=c.lr_decay_type, min_factor=c.lr_min_factor) for s in range(n)]


def test_constant_by_default():
    assert all(x == pytest.approx(1e-6) for x in _curve())


def test_decay_is_opt_in():
    lrs = _curve(lr_decay_ratio=None)
    assert lrs[1] == pytest.approx(9.9833e-7, rel=1e-4)
    assert lrs[69] == pytest.approx(8.85e-7, rel=1e-4)


def test_warmup_then_tail_decay():
    lrs = _curve(steps=100, n=100, warmup_steps=4, lr_decay_ratio=0.5, lr_decay_type="cosine")
    assert lrs[0] == pytest.approx(1e-6 / 5) and lrs[3] == pytest.approx(4e-6 / 5)
    assert all(x == pytest.approx(1e-6) for x in lrs[4:50])
    assert lrs[75] == pytest.approx(0.5e-6, rel=1e-6) and lrs[99] < 1e-8


def test_validation():
    with pytest.raises(ValueError):
        TrainerConfig(lr_decay_ratio=1.5)
    with pytest.raises(ValueError):
        TrainerConfig(lr_decay_type="step")  # type: ignore[arg-type]
