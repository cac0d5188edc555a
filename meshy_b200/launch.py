"""Run launcher: ``python -m meshy_b200.launch --recipe recipe.justrl``.

Same flags and behaviour as the reference's ``scripts/launch.py:39-200``:

* resolves the runtime directory before importing the recipe (a recipe may
  read ``XRL_RUNTIME_DIR`` at import time) and exports the ``XRL_*`` path
  overrides; ``--resume`` requires an explicit ``--runtime-dir``;
* hosts the run's bootstrap store (readiness markers, data-plane endpoint)
  on ``--master-port + 1`` of node 0;
* starts the column-store data plane on node 0 and exports its endpoint;
* starts ONE ``torchrun`` with one ignitor per card (``-m <recipe>``, whose
  ``main()`` runs the :class:`~meshy_b200.service.ignite.Ignitor`);
* forwards SIGINT/SIGTERM to the torchrun process group and tears the data
  plane down on exit.
"""

from __future__ import annotations

import argparse
import importlib
import os
import signal
import subprocess
import sys
import time


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="meshy_b200 service launcher")
    ap.add_argument("--recipe", default="recipe.justrl", help="recipe module path")
    ap.add_argument("--nnodes", type=int, default=1)
    ap.add_argument("--node-rank", type=int, default=0)
    ap.add_argument("--master-addr", default="127.0.0.1")
    ap.add_argument("--master-port", type=int, default=29500)
    ap.add_argument("--nproc-per-node", type=int, default=None,
                    help="cards per node (defaults to the recipe's card count; required for multi-node)")
    ap.add_argument("--runtime-dir", default=None, help="shared runtime dir (default: timestamped)")
    ap.add_argument("--resume", action="store_true",
                    help="continue the run in --runtime-dir from its newest complete global checkpoint")
    ap.add_argument("--checkpoint-dir", default=None, help="weight export directory (default: <runtime>/weights)")
    ap.add_argument("--log-dir", default=None, help="service and engine logs (default: <runtime>/logs)")
    ap.add_argument("--tensorboard-dir", default=None, help="metric event directory (default: <runtime>/tensorboard)")
    ap.add_argument("--trajectory-dir", default=None, help="trajectory JSONL directory (default: <runtime>)")
    return ap


def total_cards(service_groups) -> int:
    """Cards the recipe occupies: colocated groups reuse their target's cards."""
    return sum(g.n_cards for g in service_groups if g.colocate_with is None)


def torchrun_cmd(args, nproc: int) -> list[str]:
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes", str(args.nnodes), "--node-rank",
            str(args.node_rank), "--master-addr", args.master_addr, "--master-port", str(args.master_port),
            "--nproc-per-node", str(nproc), "-m", args.recipe]


def prepare_env(args) -> str:
    runtime = args.runtime_dir or os.environ.get("XRL_RUNTIME_DIR")
    if not runtime:
        if args.resume:
            raise SystemExit("--resume needs --runtime-dir pointing at the run to continue")
        runtime = os.path.abspath(os.path.join(".xrl_runtime", time.strftime("%Y%m%d-%H%M%S")))
    runtime = os.path.abspath(runtime)
    os.environ["XRL_RUNTIME_DIR"] = runtime
    if args.resume:
        from .service.checkpoint import RESUME_ENV

        os.environ[RESUME_ENV] = "1"
    os.makedirs(runtime, exist_ok=True)
    for attr, env in (("checkpoint_dir", "XRL_CHECKPOINT_DIR"), ("log_dir", "XRL_LOG_DIR"),
                      ("tensorboard_dir", "XRL_TENSORBOARD_DIR"), ("trajectory_dir", "XRL_TRAJECTORY_DIR")):
        v = getattr(args, attr)
        if v is not None:
            os.environ[env] = os.path.abspath(v)
    return runtime


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    root = os.getcwd()
    if root not in sys.path:
        sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = os.pathsep.join(filter(None, [root, os.environ.get("PYTHONPATH")]))
    runtime = prepare_env(args)
    recipe = importlib.import_module(args.recipe)
    groups = recipe.SERVICE_GROUPS
    cards = total_cards(groups)
    nproc = args.nproc_per_node or cards
    if nproc <= 0:
        raise SystemExit("the recipe needs no GPU cards; nothing to launch")
    if args.nnodes > 1 and args.nproc_per_node is None:
        raise SystemExit("--nproc-per-node is required with --nnodes > 1")
    if args.nnodes * nproc < cards:
        raise SystemExit(f"recipe needs {cards} cards, launch provides {args.nnodes * nproc}")

    from .service import bootstrap
    from .tq.launch import ColumnStoreCluster, derive_spec

    cluster = None
    if args.node_rank == 0:
        bootstrap.host_store("0.0.0.0" if args.nnodes > 1 else args.master_addr, args.master_port + 1)
        os.environ[bootstrap.ADDR_ENV] = args.master_addr
        cluster = ColumnStoreCluster(derive_spec(groups, runtime))
        cluster.start()
    else:
        os.environ[bootstrap.ADDR_ENV] = args.master_addr
        os.environ[bootstrap.PORT_ENV] = str(args.master_port + 1)
        store = bootstrap.get_store()
        from .tq.launch import ENDPOINT_KEY

        store.wait([ENDPOINT_KEY])
        os.environ["XRL_TQ_ENDPOINTS"] = store.get(ENDPOINT_KEY).decode()

    from .service.base import die_with_parent

    # torchrun gets SIGTERM if this launcher dies without forwarding a signal (SIGKILL, a crash): it then
    # stops its ignitors, whose engines and servers follow them the same way
    proc = subprocess.Popen(torchrun_cmd(args, nproc), env=dict(os.environ), start_new_session=True,
                            preexec_fn=lambda: die_with_parent(signal.SIGTERM))

    def forward(signum, frame):
        try:
            os.killpg(proc.pid, signum)
        except ProcessLookupError:
            pass

    signal.signal(signal.SIGINT, forward)
    signal.signal(signal.SIGTERM, forward)
    try:
        return proc.wait()
    finally:
        if proc.poll() is None:  # leaving on an exception: take the run down with us
            forward(signal.SIGTERM, None)
            try:
                proc.wait(timeout=60)
            except subprocess.TimeoutExpired:
                forward(signal.SIGKILL, None)
        if cluster is not None:
            cluster.stop()


if __name__ == "__main__":
    sys.exit(main())
