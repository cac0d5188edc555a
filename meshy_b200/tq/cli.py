"""Column-store command line (reference ``meshy/transferqueue/cli.py``).

    python -m meshy_b200.tq.cli serve [--host H] [--port P] [--publish-key K]
    python -m meshy_b200.tq.cli info HOST:PORT [--partition P ...]

``serve`` runs a standalone store (the reference's controller + storage units
in one process); ``info`` prints the partitions' row counts of a running one.
"""

from __future__ import annotations

import argparse
import sys


def info_main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="tq-info")
    p.add_argument("endpoint")
    p.add_argument("--partition", action="append", default=None)
    a = p.parse_args(argv)
    from .client import connect

    c = connect(a.endpoint)
    parts = a.partition or ["data.train", "gen_gate"]
    print(f"column store at {a.endpoint}")
    for part in parts:
        print(f"  {part}: {c.num_rows(part)} rows")
    c.close()
    return 0


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in ("serve", "info"):
        print("usage: python -m meshy_b200.tq.cli {serve|info} [args...]", file=sys.stderr)
        return 2
    if argv[0] == "serve":
        from .server import main as serve

        serve(argv[1:])
        return 0
    return info_main(argv[1:])


if __name__ == "__main__":
    sys.exit(main())
