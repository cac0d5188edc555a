"""Metric tag hygiene (CPU): a tag is either a scalar or a histogram (histograms live under ``hist/`` even when a
scalar has the same name), and non-finite scalars and histogram values are dropped instead of written."""

import json
import math

from meshy_b200.utils.metrics_adapter import HISTOGRAM_PREFIX, MetricsWriter, read_events


def test_scalar_and_histogram_tags_do_not_collide(tmp_path):
    w = MetricsWriter(str(tmp_path), use_tensorboard=False)
    metrics = {"rollout/advantages": 0.0, "rollout/log_probs": -0.5, "bad": math.nan, "inf": math.inf}
    hist = {"rollout/advantages": [0.1, -0.1], "rollout/log_probs": [-0.4, math.nan], "empty": [math.nan]}
    for step in (1, 2):
        w.write(metrics, step, hist)
    w.close()
    ev = [f for f in tmp_path.iterdir() if f.name.startswith("events.out")][0]
    recs = [r for r in read_events(str(ev)) if r[1]]
    assert [r[0] for r in recs] == [1, 2]
    assert set(recs[0][1]) == {"rollout/advantages", "rollout/log_probs"}  # non-finite scalars dropped
    rows = [json.loads(l) for l in (tmp_path / "metrics.jsonl").read_text().splitlines()]
    assert all(set(r) == {"step", "rollout/advantages", "rollout/log_probs"} for r in rows)
    raw = ev.read_bytes()
    assert (HISTOGRAM_PREFIX + "rollout/advantages").encode() in raw
    assert (HISTOGRAM_PREFIX + "empty").encode() not in raw  # nothing finite to write
