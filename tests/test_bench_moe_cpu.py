"""The MoE layer benchmark (``meshy_b200.bench.moe``) runs on CPU with the debug MoE model and its two arms
agree (the timing itself needs a GPU)."""

import json


def test_moe_bench_runs_on_cpu(capsys):
    from meshy_b200.bench.moe import main

    main(["--device", "cpu", "--model", "qwen3:debugmodel_moe", "--tokens", "48"])
    recs = [json.loads(line) for line in capsys.readouterr().out.splitlines() if line.startswith("{")]
    assert {r.get("impl") for r in recs if "impl" in r} == {"native", "torch"}
    assert [r for r in recs if "max_rel_diff" in r][0]["max_rel_diff"] < 1e-4
