"""Data-parallel gradient all-reduce overlapped with the backward (gloo, 2 ranks, CPU).

With overlap on, the last micro-batch's backward starts one asynchronous all-reduce per transformer block as
soon as that block's backward is issued, and ``finish`` sums only what is left (embedding, final norm, LM
head). The summed gradients, hence the optimiser steps, must equal those of the reduction done after the
backward in one pass (2 ranks: a + b is exact in either order), with activation checkpointing too, and every
byte of the gradient must be reduced exactly once.
"""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _samples(rank, seed=0, n=4):
    rng = random.Random(seed * 100 + rank)
    out = []
    for i in range(n):
        P, R = rng.randint(3, 9), rng.randint(8, 40)
        toks = [rng.randrange(2048) for _ in range(P + R)]
        out.append({"tokens": torch.tensor(toks), "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(group, ckpt_mode, dtype):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.1,
                       max_norm=0.5, dtype=dtype, activation_checkpoint_mode=ckpt_mode)
    tp = TrainerParamsConfig(mini_batch_size=2, batch_layout="packed", max_tokens_per_micro=64,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=0, dp_group=group, loss_group=group, timer_enabled=False)


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        g = dist.group.WORLD
        out = {}
        for ckpt_mode, dtype in (("none", "float32"), ("full", "float32"), ("none", "bfloat16")):
            res = {}
            for overlap in ("1", "0"):
                os.environ["MESHY_DDP_OVERLAP"] = overlap
                t = _trainer(g, ckpt_mode, dtype)
                assert t.reducer.overlapping == (overlap == "1")
                assert (getattr(t.model, "block_hooks", None) is t.reducer) == (overlap == "1")
                launched = []
                orig = t.reducer.backward_end

                def spy(i, orig=orig, red=t.reducer, launched=launched):
                    n = len(red._works)
                    orig(i)
                    launched.append((i, len(red._works) - n))

                t.reducer.backward_end = spy
                norms = [t.train_step(_samples(rank, s))["grad_norm"] for s in range(2)]
                res[overlap] = (t.flat.master.clone(), norms, t.reducer.last_bytes, launched)
            (w1, n1, b1, l1), (w0, n0, b0, l0) = res["1"], res["0"]
            n_layers = len(t.model.layers)
            full_bytes = t.flat.grad.numel() * t.flat.grad.element_size()
            out[(ckpt_mode, dtype)] = {
                "w_diff": float((w1 - w0).abs().max()), "norms": (n1, n0), "bytes": (b1, b0, full_bytes),
                # the last micro of each mini-batch: every block reduced from its hook, in backward order
                "armed_blocks": [i for i, k in l1 if k > 0], "n_layers": n_layers, "unarmed": l0,
            }
        q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


@pytest.mark.timeout(300)
def test_overlapped_reduction_equals_reduction_after_backward():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for v in res.values():
        assert not isinstance(v, str), v
    for rank in (0, 1):
        for key, o in res[rank].items():
            assert o["w_diff"] == 0.0, (rank, key, o["w_diff"])
            assert o["norms"][0] == o["norms"][1], (rank, key)
            b1, b0, full = o["bytes"]
            assert b1 == b0 == full, (rank, key)  # every byte reduced once, overlapped or not
            L = o["n_layers"]
            # 2 steps x 1 mini-batch each... x2 minis per step: each armed backward walks L-1 .. 0
            armed = o["armed_blocks"]
            assert len(armed) % L == 0 and armed[:L] == list(range(L - 1, -1, -1)), armed
            assert o["unarmed"] == []  # without overlap no boundary is inserted


def test_range_arithmetic_with_skipped_expert_slices():
    """Blocks reduced from their hooks plus what ``finish`` reduces cover every non-skipped element exactly
    once (expert slices that differ per rank are never summed)."""
    from types import SimpleNamespace

    from meshy_b200.parallel.ddp import GradReducer, _subtract

    assert list(_subtract(0, 10, [(2, 4), (6, 7)])) == [(0, 2), (4, 6), (7, 10)]
    assert list(_subtract(3, 5, [(0, 10)])) == [] and list(_subtract(0, 4, [])) == [(0, 4)]
    names = ["embed", "layers.0.wqkv", "layers.0.moe.w13", "layers.0.w2", "layers.1.wqkv", "layers.1.moe.w13",
             "norm", "output"]
    slots, off = [], 0
    for n in names:
        slots.append(SimpleNamespace(name=n, offset=off, numel=10))
        off += 10
    flat = SimpleNamespace(slots=slots, params=[None] * len(slots), grad=None)
    skip = [(s.offset, s.numel) for s in slots if ".moe." in s.name]
    r = GradReducer(flat, None, skip=skip, overlap=True)
    assert {i: (lo, hi) for i, (lo, hi, _) in r._blocks.items()} == {0: (10, 40), 1: (40, 60)}
    covered = []
    for i in (1, 0):  # hooks fire in backward order
        lo, hi, _ = r._blocks[i]
        covered += list(_subtract(lo, hi, r._holes))
    done = sorted((r._blocks[i][0], r._blocks[i][1]) for i in (0, 1))
    for lo, hi in r._ranges(off):
        covered += list(_subtract(lo, hi, done))
    elems = sorted(x for a, b in covered for x in range(a, b))
    want = [x for x in range(off) if not any(o <= x < o + n for o, n in skip)]
    assert elems == want
