"""Tensor-parallel rollout engine on CPU (gloo, 2 ranks).

* engine level: rank 0 drives the replica through :class:`EngineLeader`, rank 1 follows; greedy generations
  equal a single-rank engine's on the same weights (token ids exact, log-probs to fp32 summation order), and
  so do they after a weight update from a full state dict (the replica -> tensor-parallel reshard);
* expert parallelism inside the replica (Qwen3-MoE, ``ep=True``): each rank keeps half of the experts, the
  routed outputs are summed over the ranks, and generations again equal the single-rank engine's;
* server level: ``python -m meshy_b200.rollout.server --tp-size 2`` spawns its follower and answers
  ``/generate`` with the single-card server's tokens; so does a replica over two "nodes" (two server processes,
  ``--nnodes 2 --node-rank 0/1 --dist-init-addr``), the second of which runs only its follower rank;
* service level: an inference replica's server command takes its TP degree from the replica's cards and, over
  several nodes, the node count, this node's index and the master card's rendezvous address.
"""

import os
import socket
import subprocess
import sys
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROMPTS = [[3, 14, 15, 92, 65, 35], [8, 97, 93, 23, 84, 62, 64, 33, 83, 27], [2, 71]]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _engine(group=None, seed=0, flavor="debugmodel", ep=False):
    from meshy_b200.models import get_model_args
    from meshy_b200.rollout.engine import RolloutEngine

    return RolloutEngine(get_model_args("qwen3", flavor), device="cpu", max_running=8, max_seq_len=128,
                         seed=seed, sync_every=4, tp_group=group, ep=ep)


def _run(eng):
    gens = eng.generate(PROMPTS, [12, 7, 20], temperature=0.0, ignore_eos=True)
    return [(g.output_ids, g.output_logprobs) for g in gens]


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from meshy_b200.rollout.spmd import EngineLeader, follow

        g = dist.group.WORLD
        eng = _engine(g)
        assert eng.tp == 2 and eng.local_args.n_heads * 2 == eng.args.n_heads
        if rank == 1:
            follow(eng, g)
            q.put((rank, "ok"))
        else:
            lead = EngineLeader(eng, g)
            out = {"first": _run(lead)}
            # a different model, sent as a full state dict: every rank takes its slices
            from meshy_b200.models import build_model

            other = build_model(eng.args, seed=7, device="cpu", dtype=torch.float32)
            sd = {k: v.detach().clone() for k, v in other.named_parameters()}
            lead.update_weights_from_state_dict(sd, 3)
            out["second"] = _run(lead)
            lead.stop()
            # single-rank references (tp_group=None)
            ref = _engine(None)
            out["ref_first"] = _run(ref)
            ref.update_weights_from_state_dict(sd, 3)
            out["ref_second"] = _run(ref)
            q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


def _same(a, b, tol=1e-4):
    for (ta, la), (tb, lb) in zip(a, b):
        assert ta == tb
        assert max(abs(x - y) for x, y in zip(la, lb)) < tol


def _ep_worker(rank, port, q):
    """Qwen3-MoE replica with attention split over 2 ranks and the experts too (4 of 8 each)."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from meshy_b200.rollout.spmd import EngineLeader, follow

        g = dist.group.WORLD
        eng = _engine(g, flavor="debugmodel_moe", ep=True)
        moe = eng.model.layers[0].moe
        assert moe.w13.shape[0] * 2 == moe.n_experts and moe.expert_offset == rank * moe.n_experts // 2
        if rank == 1:
            follow(eng, g)
            q.put((rank, "ok"))
        else:
            lead = EngineLeader(eng, g)
            out = {"ep": _run(lead)}
            from meshy_b200.models import build_model

            other = build_model(eng.args, seed=7, device="cpu", dtype=torch.float32)
            sd = {k: v.detach().clone() for k, v in other.named_parameters()}
            lead.update_weights_from_state_dict(sd, 2)  # each rank keeps its experts' slices
            out["ep2"] = _run(lead)
            lead.stop()
            ref = _engine(None, flavor="debugmodel_moe")
            out["ref"] = _run(ref)
            ref.update_weights_from_state_dict(sd, 2)
            out["ref2"] = _run(ref)
            q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


@pytest.mark.timeout(300)
def test_tp_ep_moe_engine_matches_single_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ep_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for v in res.values():
        assert not (isinstance(v, str) and v != "ok"), v
    _same(res[0]["ep"], res[0]["ref"])
    _same(res[0]["ep2"], res[0]["ref2"])


@pytest.mark.timeout(300)
def test_tp_engine_matches_single_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for r, v in res.items():
        assert not (isinstance(v, str) and v != "ok"), v
    out = res[0]
    _same(out["first"], out["ref_first"])
    _same(out["second"], out["ref_second"])
    assert out["first"][0][0] != out["second"][0][0] or out["first"][1][0] != out["second"][1][0]


def _server(tp, port, extra=()):
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "meshy_b200.rollout.server", "--model", "qwen3:debugmodel", "--device", "cpu",
           "--port", str(port), "--max-running", "8", "--max-seq-len", "128", "--tp-size", str(tp), *extra]
    return subprocess.Popen(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            start_new_session=True)


def _wait(port, proc, timeout=120):
    import requests

    end = time.time() + timeout
    while time.time() < end:
        assert proc.poll() is None, proc.stdout.read().decode()[-3000:]
        try:
            if requests.get(f"http://127.0.0.1:{port}/health", timeout=2).ok:
                return
        except Exception:
            time.sleep(0.5)
    raise AssertionError("server did not come up")


@pytest.mark.timeout(420)
def test_tp_server_answers_like_single_card_server():
    import requests

    outs = []
    for case in ("tp1", "tp2", "tp2-2nodes"):
        port = _port()
        if case == "tp2-2nodes":
            rdv = f"127.0.0.1:{_port()}"
            procs = [_server(2, port if n == 0 else _port(),
                             ["--nnodes", "2", "--node-rank", str(n), "--dist-init-addr", rdv]) for n in (0, 1)]
        else:
            procs = [_server(1 if case == "tp1" else 2, port)]
        try:
            _wait(port, procs[0])
            assert all(p.poll() is None for p in procs)
            body = {"input_ids": PROMPTS[1], "sampling_params": {"max_new_tokens": 9, "temperature": 0.0,
                                                                 "ignore_eos": True}, "return_logprob": True}
            r = requests.post(f"http://127.0.0.1:{port}/generate", json=body, timeout=120)
            r.raise_for_status()
            outs.append(r.json())
        finally:
            for p in procs:
                os.killpg(p.pid, 15)
            for p in procs:
                p.wait(timeout=30)
    for o in outs[1:]:
        assert outs[0]["output_ids"] == o["output_ids"] and len(o["output_ids"]) == 9
        la = [x[0] for x in outs[0]["meta_info"]["output_token_logprobs"]]
        lb = [x[0] for x in o["meta_info"]["output_token_logprobs"]]
        assert max(abs(x - y) for x, y in zip(la, lb)) < 1e-4


def _service(gpus, me):
    from meshy_b200.config import InferenceServiceConfig
    from meshy_b200.service.inference import InferenceService
    from meshy_b200.service.topology import ServiceInfo

    cfg = InferenceServiceConfig(server_args={"model": "qwen3:debugmodel", "tp_size": 1, "ep_size": len(gpus)})
    info = ServiceInfo("actor_infer-0", "actor_infer", "inference", True, 0, gpus[0].host, 30000, 40000, gpus,
                       False, None, config=cfg)
    return InferenceService(info, None, None, my_gpu=me)


def _flag(cmd, name):
    return cmd[cmd.index(name) + 1] if name in cmd else None


def test_inference_service_command_sets_tp_from_replica_cards():
    from meshy_b200.service.base import GPU

    one = [GPU(r, "10.0.0.1", r, 0) for r in range(4)]
    svc = _service(one, one[2])
    assert svc.is_node_leader is False and svc.is_master is False
    cmd = _service(one, one[0]).command()
    assert _flag(cmd, "--tp-size") == "4" and _flag(cmd, "--ep-size") == "4"  # server_args' tp_size is overridden
    assert _flag(cmd, "--dist-port") == "40000" and "--nnodes" not in cmd
    two = [GPU(r, f"10.0.0.{1 + r // 2}", r % 2, r // 2) for r in range(4)]
    lead0, lead1, other = _service(two, two[0]), _service(two, two[2]), _service(two, two[3])
    assert lead0.is_node_leader and lead1.is_node_leader and not other.is_node_leader
    assert [g.local_rank for g in lead1.node_gpus] == [0, 1]
    c0, c1 = lead0.command(), lead1.command()
    for c, n in ((c0, "0"), (c1, "1")):
        assert _flag(c, "--tp-size") == "4" and _flag(c, "--nnodes") == "2" and _flag(c, "--node-rank") == n
        assert _flag(c, "--dist-init-addr") == "10.0.0.1:40000"


def test_trainer_syncs_through_disk_when_engines_are_on_another_host():
    from types import SimpleNamespace

    from meshy_b200.service.base import GPU
    from meshy_b200.service.training import TrainingService

    def svc(mode, train_hosts, infer_hosts):
        info = SimpleNamespace(config=SimpleNamespace(weight_sync_mode=mode),
                               replica_gpus=[GPU(i, h, i, 0) for i, h in enumerate(train_hosts)])
        infer = [SimpleNamespace(replica_gpus=[GPU(10 + i, h, i, 0)]) for i, h in enumerate(infer_hosts)]
        return SimpleNamespace(info=info, topology=SimpleNamespace(inference_services=lambda: infer))

    assert TrainingService.weight_sync_mode(svc("auto", ["a", "a"], ["a", "a"])) == "auto"
    assert TrainingService.weight_sync_mode(svc("auto", ["a", "a"], ["a", "b"])) == "disk"  # IPC is node-local
    assert TrainingService.weight_sync_mode(svc("device", ["a"], ["b"])) == "device"  # explicit choice stands
