"""The MoE layer and Top-K distillation benchmarks (``meshy_b200.bench.moe`` / ``.distill``) run on CPU with
small shapes and their native and PyTorch arms agree (the timing itself needs a GPU)."""

import json


def test_moe_bench_runs_on_cpu(capsys):
    from meshy_b200.bench.moe import main

    main(["--device", "cpu", "--model", "qwen3:debugmodel_moe", "--tokens", "48"])
    recs = [json.loads(line) for line in capsys.readouterr().out.splitlines() if line.startswith("{")]
    assert {r.get("impl") for r in recs if "impl" in r} == {"native", "torch"}
    assert [r for r in recs if "max_rel_diff" in r][0]["max_rel_diff"] < 1e-4


def test_distill_bench_runs_on_cpu(capsys):
    from meshy_b200.bench.distill import main

    main(["--device", "cpu", "--tokens", "40", "--vocab", "300", "--teacher-dim", "32", "--student-dim", "16"])
    recs = [json.loads(line) for line in capsys.readouterr().out.splitlines() if line.startswith("{")]
    cmp = [r for r in recs if "teacher_ids_equal" in r][0]
    assert cmp["teacher_ids_equal"] == 1.0 and cmp["student_lp_max_abs_diff"] < 1e-4
