"""Trainer checkpoints in torchtitan's DCP layout (CPU).

* the fused parameters of every family split into torchtitan's tensors and back exactly, including the
  RoPE row permutation of the Llama-family q / k projections;
* a saved checkpoint carries torchtitan's keys (model FQNs at the top level, the flattened AdamW state under
  ``optimizer.state``, ``train_state.step``) and restores weights, moments and counters;
* two gloo ranks write one checkpoint together (each its share of the parameters) and each reads all of it.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from meshy_b200.models import get_model_args
from meshy_b200.models.titan_names import join_pieces, titan_pieces


def _small(family, flavor):
    """A registry architecture shrunk to a CPU-sized model (same family flags: bias, QK-norm, RoPE layout)."""
    import dataclasses

    args = get_model_args(family, flavor)
    if args.dim <= 512:
        return args
    return dataclasses.replace(args, dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=256,
                               vocab_size=512)


@pytest.mark.parametrize("family,flavor", [("qwen3", "debugmodel"), ("qwen3", "debugmodel_moe"),
                                           ("qwen2_5", "0.5B"), ("minicpm5", "1B"), ("llama3", "debugmodel")])
def test_pieces_round_trip(family, flavor):
    args = _small(family, flavor)
    from meshy_b200.models import build_model

    model = build_model(args, seed=3, device="cpu", dtype=torch.float32)
    names = set()
    for name, p in model.named_parameters():
        pieces = titan_pieces(args, name, p.detach())
        names.update(n for n, _ in pieces)
        back = join_pieces(args, name, [t for _, t in pieces])
        assert torch.equal(back, p.detach()), name
    assert "tok_embeddings.weight" in names and "layers.0.attention.qkv_linear.wq.weight" in names
    assert any(n.startswith("layers.0.feed_forward.w1") or n.startswith("layers.0.moe.experts.w1") for n in names)


def test_llama_rope_rows_match_torchtitan_convention():
    """torchtitan stores q / k rows as interleaved (even, odd) pairs: row 2j of a head is HF row j, row 2j+1
    is HF row j + head_dim / 2."""
    args = _small("minicpm5", "1B")
    hd = args.head_dim
    w = torch.arange(args.qkv_dim, dtype=torch.float32)[:, None].repeat(1, 4)
    (_, wq), _, _ = titan_pieces(args, "layers.0.wqkv", w)
    assert wq[0, 0] == 0 and wq[1, 0] == hd // 2 and wq[2, 0] == 1 and wq[3, 0] == hd // 2 + 1


def _trainer(dp_group=None, seed=0):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.1,
                       max_norm=1.0, dtype="float32")
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=128,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=seed, dp_group=dp_group, timer_enabled=False)


def _batch(seed=0, n=4):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        L = 20 + 3 * i
        mask = torch.zeros(L)
        mask[6:] = 1
        out.append({"tokens": torch.randint(0, 2048, (L,), generator=g), "mask_assistant": mask,
                    "logprobs": -torch.rand(L, generator=g), "advantage": torch.tensor([1.0 - i * 0.5]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def test_save_load_round_trip_with_torchtitan_keys(tmp_path):
    from torch.distributed.checkpoint import FileSystemReader

    t = _trainer()
    t.train_step(_batch())
    t.train_step(_batch(1))
    path = str(tmp_path / "step-2")
    t.save_checkpoint(path, 2)
    keys = set(FileSystemReader(path).read_metadata().state_dict_metadata)
    for k in ("tok_embeddings.weight", "norm.weight", "layers.0.attention.qkv_linear.wq.weight",
              "layers.1.feed_forward.w3.weight", "layers.0.attention.q_norm.weight",
              "optimizer.state.layers.0.feed_forward.w1.weight.exp_avg",
              "optimizer.state.tok_embeddings.weight.exp_avg_sq", "optimizer.state.norm.weight.step",
              "optimizer.param_groups.norm.weight.lr", "train_state.step"):
        assert k in keys, k
    assert not any(k.startswith("model.") for k in keys)  # torchtitan puts model FQNs at the top level
    fresh = _trainer(seed=7)
    assert not torch.equal(fresh.flat.master, t.flat.master)
    fresh.load_checkpoint(path)
    assert torch.equal(fresh.flat.master, t.flat.master)
    assert torch.equal(fresh.flat.exp_avg, t.flat.exp_avg) and torch.equal(fresh.flat.exp_avg_sq, t.flat.exp_avg_sq)
    assert fresh.step == t.step and fresh.optimizer.step_count == t.optimizer.step_count
    # training continues identically from the restored state
    a = t.train_step(_batch(2))["pg_loss"]
    b = fresh.train_step(_batch(2))["pg_loss"]
    assert a == pytest.approx(b, rel=1e-6, abs=1e-7)
    assert torch.allclose(fresh.flat.master, t.flat.master, atol=1e-7)


def _worker(rank, port, path, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        t = _trainer(dp_group=dist.group.WORLD)
        t.train_step(_batch(rank))
        t.save_checkpoint(path, 1)
        fresh = _trainer(dp_group=dist.group.WORLD, seed=9)
        fresh.load_checkpoint(path)
        ok = torch.equal(fresh.flat.master, t.flat.master) and torch.equal(fresh.flat.exp_avg, t.flat.exp_avg)
        files = sorted(f for f in os.listdir(path) if f.endswith(".distcp"))
        q.put((rank, ok, files))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.timeout(300)
def test_two_ranks_write_one_checkpoint(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = str(tmp_path / "step-1")
    ps = [ctx.Process(target=_worker, args=(r, port, path, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, ok, files in res:
        assert ok is True, ok
        assert len(files) == 2, files  # one data file per writing rank
