"""Critic checkpoints: DCP in the reference critic's layout, and optimiser-group migration (CPU).

A critic built without ``optimizer_kwargs`` has one AdamW group (PyTorch defaults); with them it has a decay
group and a no-decay group and those settings are authoritative. A checkpoint moves between the two:
moments and step counts are matched by parameter name, the restoring critic keeps its own grouping and
hyperparameters when they were given explicitly, and takes the saved ones when they were not. After the
restore, the next update equals the update of a critic that never left memory.
"""

import pytest
import torch

from meshy_b200.backend.critic.data import TrajectorySample
from meshy_b200.backend.critic.trainer import CriticTrainer
from meshy_b200.models import get_model_args

ARGS = get_model_args("qwen3", "debugmodel")
EXPLICIT = {"weight_decay": 0.1, "betas": (0.9, 0.98), "eps": 1e-8}


def _critic(explicit: bool, seed=0):
    return CriticTrainer(ARGS, device="cpu", lr=1e-3, warmup_steps=0, max_norm=1.0, seq_len=128,
                         max_tokens_per_micro=256, optimizer_kwargs=dict(EXPLICIT) if explicit else None, seed=seed)


def _window(seed):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(3):
        n = 12 + 5 * i
        toks = torch.randint(0, ARGS.vocab_size, (n,), generator=g)
        mask = torch.zeros(n)
        mask[4:] = 1
        out.append(TrajectorySample(tokens=toks.tolist(), mask=mask.tolist(), reward=float(i % 2)))
    return out


def _train(c, seed):
    samples = _window(seed)
    return c.train_window(samples, list(range(len(samples))))[0]


def _moments(c):
    return (c.flat.master.clone(), c.flat.exp_avg.clone(), c.flat.exp_avg_sq.clone(), c.opt.step_count,
            c.model.value_head.detach().clone(),
            {k: v.clone() for k, v in c.head_opt.state[c.model.value_head].items()})


@pytest.mark.parametrize("saved_explicit", [False, True])
def test_restore_into_grouped_critic_keeps_moments_and_current_groups(tmp_path, saved_explicit):
    src = _critic(saved_explicit)
    for s in range(3):
        _train(src, s)
    path = str(tmp_path / "critic")
    src.save_state(path)
    dst = _critic(True, seed=5)
    dst.load_state(path)
    a, b = _moments(src), _moments(dst)
    for x, y in zip(a[:3], b[:3]):
        assert torch.equal(x, y)
    assert a[3] == b[3] and torch.equal(a[4], b[4])
    for k in ("exp_avg", "exp_avg_sq", "step"):
        assert torch.equal(a[5][k].float(), b[5][k].float()), k
    # the restoring critic keeps its explicit grouping and hyperparameters
    assert dst.grouped and dst.opt.betas == (0.9, 0.98) and dst.opt.weight_decay == 0.1
    assert [g["weight_decay"] for g in dst.head_opt.param_groups] == [0.1, 0.0]
    # next update: identical to a grouped critic that had the same state in memory
    ref = _critic(True, seed=9)
    ref.load_state(path)
    _train(dst, 11)
    _train(ref, 11)
    assert torch.equal(dst.flat.master, ref.flat.master)


def test_implicit_config_takes_the_saved_hyperparameters(tmp_path):
    src = _critic(True)
    _train(src, 0)
    path = str(tmp_path / "critic")
    src.save_state(path)
    dst = _critic(False)
    assert dst.opt.betas == (0.9, 0.999)
    dst.load_state(path)
    assert dst.opt.betas == (0.9, 0.98)


def test_grouped_decay_skips_vectors():
    c = _critic(True)
    decayed = set(c.opt.decay_names)
    assert all(len(s.shape) >= 2 for s in c.flat.slots if s.name in decayed)
    assert any(s.name.endswith("norm") for s in c.flat.slots if s.name not in decayed)
    # with zero gradients only the decay group moves, by exactly (1 - lr * wd)
    before = c.flat.master.clone()
    c.flat.zero_grad()
    c.opt.step(grad_norm=torch.zeros(()))
    for s in c.flat.slots:
        got = c.flat.master[s.offset:s.offset + s.numel]
        want = before[s.offset:s.offset + s.numel] * ((1 - 1e-3 * 0.1) if s.name in decayed else 1.0)
        assert torch.allclose(got, want, atol=1e-7), s.name


def test_missing_moments_fail_the_restore(tmp_path):
    import torch.distributed.checkpoint as dcp

    src = _critic(False)
    _train(src, 0)
    path = str(tmp_path / "critic")
    src.save_state(path)
    # drop one moment from a copy of the checkpoint
    reader = dcp.FileSystemReader(path)
    meta = reader.read_metadata().state_dict_metadata
    full = {}
    for k, m in meta.items():
        if hasattr(m, "size"):
            full[k] = torch.empty(m.size)
    dcp.load(full, checkpoint_id=path, no_dist=True)
    victim = next(k for k in full if k.endswith(".exp_avg_sq"))
    del full[victim]
    broken = str(tmp_path / "broken")
    dcp.save(full, checkpoint_id=broken, no_dist=True)
    with pytest.raises(dcp.api.CheckpointException):
        _critic(True).load_state(broken)
