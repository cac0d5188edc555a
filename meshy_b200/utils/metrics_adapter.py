"""Training metrics: rollout statistics, ``perf/*`` gauges and an event writer.

Counterpart of the reference's metrics adapter
(``meshy/backend/titan/metrics.py:36-74,171-322,366-422``):

* :func:`rollout_metrics` — statistics over the *global* batch: response and
  sequence length percentiles, truncation / repetition / mixed-version stamp
  rates, weight staleness against the version being trained, pass rate
  (unshaped reward when the rollout published ``raw_reward``), reward and
  advantage moments, plus histogram series for the ``hist/`` namespace;
* :func:`perf_metrics` — step time, tokens/s/GPU, train and log-prob time,
  actor TFLOP/s (6·N·tokens) and the wait-time ratio;
* :class:`MetricsWriter` — rank-0 writer of TensorBoard event files.  When
  ``torch.utils.tensorboard`` is importable it is used; otherwise the writer
  encodes the event records itself (TFRecord framing with masked CRC-32C,
  ``Event{wall_time, step, Summary{Value{tag, simple_value | histo}}}`` in
  protobuf wire format), so TensorBoard can read the run without the package
  being installed here.  Every record is mirrored to ``metrics.jsonl``.
"""

from __future__ import annotations

import json
import math
import os
import socket
import struct
import time
from typing import Any, Iterable, Sequence

HISTOGRAM_PREFIX = "hist/"
HISTOGRAM_MAX_VALUES = 4096


# ═══════════════════════════════ statistics ══════════════════════════════════

def _field(s: Any, name: str, default=None):
    if isinstance(s, dict):
        return s.get(name, default)
    return getattr(s, name, default)


def _as_list(x) -> list:
    if x is None:
        return []
    if hasattr(x, "tolist"):
        x = x.tolist()
    return list(x) if isinstance(x, (list, tuple)) else [x]


def _percentile(sorted_vals: Sequence[float], q: float) -> float:
    if not sorted_vals:
        return float("nan")
    k = (len(sorted_vals) - 1) * q
    lo, hi = math.floor(k), math.ceil(k)
    if lo == hi:
        return float(sorted_vals[int(k)])
    return float(sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (k - lo))


def _moments(prefix: str, vals: Sequence[float], out: dict) -> None:
    if not vals:
        return
    n = len(vals)
    mean = sum(vals) / n
    var = sum((v - mean) ** 2 for v in vals) / n
    out[f"{prefix}/mean"] = mean
    out[f"{prefix}/std"] = math.sqrt(var)
    out[f"{prefix}/max"] = max(vals)
    out[f"{prefix}/min"] = min(vals)


def rollout_metrics(samples: Sequence[Any], seq_len: int | None = None,
                    current_version: int | None = None) -> tuple[dict[str, float], dict[str, list[float]]]:
    """Batch statistics of rollout rows (dicts or objects with the column names as attributes)."""
    out: dict[str, float] = {}
    hist: dict[str, list[float]] = {}
    if not samples:
        return out, hist
    rewards = [float(v) for s in samples for v in _as_list(_field(s, "reward"))]
    raw = [float(v) for s in samples for v in _as_list(_field(s, "raw_reward"))]
    solve = raw or rewards
    adv = []
    for s in samples:
        a = _field(s, "advantage")
        vals = _as_list(a)
        if vals:
            adv.append(float(vals[0]) if not isinstance(vals[0], list) else float(vals[0][0]))
    resp_lens, seq_lens = [], []
    for s in samples:
        toks = _as_list(_field(s, "tokens"))
        mask = _as_list(_field(s, "mask_assistant")) or _as_list(_field(s, "masks"))
        if toks:
            seq_lens.append(float(len(toks)))
        if mask:
            resp_lens.append(float(sum(1 for m in mask if m)))
    n = len(samples)
    for stamp in ("truncated", "repetition", "mixed_version"):
        vals = [bool(_as_list(_field(s, stamp))[0]) for s in samples if _as_list(_field(s, stamp))]
        if vals:
            out[f"rollout/{stamp}_ratio"] = sum(vals) / len(vals)
    versions = [int(_as_list(_field(s, "weight_version"))[0]) for s in samples
                if _as_list(_field(s, "weight_version"))]
    if versions and current_version is not None:
        stale = [current_version - v for v in versions]
        _moments("rollout/staleness", [float(x) for x in stale], out)
    if solve:
        out["rollout/pass_rate"] = sum(1.0 for r in solve if r > 0.5) / len(solve)
    _moments("rollout/reward", rewards, out)
    if raw:
        _moments("rollout/raw_reward", raw, out)
    _moments("rollout/advantage", adv, out)
    if resp_lens:
        srt = sorted(resp_lens)
        out["rollout/response_lengths"] = sum(resp_lens)
        out["rollout/response_len/mean"] = sum(resp_lens) / len(resp_lens)
        for q, name in ((0.5, "p50"), (0.9, "p90"), (0.99, "p99")):
            out[f"rollout/response_len/{name}"] = _percentile(srt, q)
        out["rollout/response_len/max"] = srt[-1]
        out["rollout/response_len/min"] = srt[0]
        if seq_len:
            out["rollout/clip_ratio"] = sum(1.0 for L in seq_lens if L >= seq_len) / max(1, len(seq_lens))
        hist["response_length"] = resp_lens
    if seq_lens:
        out["rollout/seq_len/mean"] = sum(seq_lens) / len(seq_lens)
        if seq_len:
            out["rollout/seq_len_truncated_ratio"] = sum(1.0 for L in seq_lens if L >= seq_len) / len(seq_lens)
    # the reference's tag names for the same quantities (meshy/backend/titan/metrics.py), so dashboards carry over
    if "rollout/repetition_ratio" in out:
        out["rollout/repetition_frac"] = out["rollout/repetition_ratio"]
    if "rollout/mixed_version_ratio" in out:
        out["rollout/weight_version/mixed_version_ratio"] = out["rollout/mixed_version_ratio"]
    if versions:
        # version spread inside the batch: "stale" means older than the newest version present in the batch
        newest = max(versions)
        out["rollout/weight_version/mean"] = sum(versions) / len(versions)
        out["rollout/weight_version/min"] = float(min(versions))
        out["rollout/weight_version/max"] = float(newest)
        out["rollout/weight_version/median"] = _percentile(sorted(float(v) for v in versions), 0.5)
        out["rollout/weight_version/num_versions"] = float(len(set(versions)))
        out["rollout/weight_version/stale_ratio"] = sum(1.0 for v in versions if v < newest) / len(versions)
    if versions and current_version is not None:
        # lag behind the weights the trainer is about to update
        stale = [current_version - v for v in versions]
        out["rollout/weight_version/staleness_mean"] = sum(stale) / len(stale)
        out["rollout/weight_version/staleness_max"] = float(max(stale))
    if rewards:
        # raw_reward is the unshaped reward when the rollout published one; reward is the shaped value
        out["rollout/raw_reward_mean"] = sum(solve) / len(solve)
        out["rollout/raw_reward"] = out["rollout/raw_reward_mean"]
        out["rollout/rewards"] = sum(rewards) / len(rewards)
    lps = []
    for s in samples:
        lp = _as_list(_field(s, "logprobs"))
        mask = _as_list(_field(s, "mask_assistant")) or _as_list(_field(s, "masks"))
        if lp and mask and len(lp) == len(mask):
            lps.extend(float(x) for x, m in zip(lp, mask) if m)  # sampled tokens only, prompt placeholders out
    if lps:
        out["rollout/log_probs"] = sum(lps) / len(lps)
        hist["rollout/log_probs"] = lps
    if rewards:
        hist["reward"] = rewards
    if adv:
        hist["advantage"] = adv
    out["rollout/num_samples"] = float(n)
    return out, hist


def perf_metrics(result: dict[str, float], total_time: float, tokens: float | None, n_params: float | None,
                 n_gpus: int = 1) -> dict[str, float]:
    total_time = max(float(total_time), 1e-9)
    perf: dict[str, float] = {"perf/step_time": total_time}
    if tokens is not None:
        perf["perf/tokens_per_gpu_per_sec"] = float(tokens) / total_time / max(1, n_gpus)
    timed = [float(v) for k, v in result.items() if k.startswith("time/train/") and isinstance(v, (int, float))]
    train_time = sum(timed)
    old_lp = result.get("time/train/old_logprobs")
    pack = result.get("time/train/pack_batch")
    if pack is not None:
        perf["perf/data_preprocess_time"] = float(pack)
    if old_lp is not None:
        perf["perf/log_probs_time"] = float(old_lp)
    if timed:
        perf["perf/train_time"] = train_time
        if tokens is not None:
            perf["perf/actor_train_tok_per_s"] = float(tokens) / max(train_time, 1e-9)
            if n_params:
                perf["perf/actor_train_tflops"] = 6.0 * float(n_params) * float(tokens) / max(train_time, 1e-9) / 1e12
                if old_lp:
                    perf["perf/log_probs_tflops"] = 2.0 * float(n_params) * float(tokens) / max(float(old_lp), 1e-9) / 1e12
        perf["perf/wait_time_ratio"] = max(0.0, total_time - train_time) / total_time
    return perf


# ═══════════════════════════════ event files ═════════════════════════════════

def _crc32c_table() -> list[int]:
    # CRC-32C (Castagnoli), reflected polynomial 0x82F63B78
    table = []
    for i in range(256):
        c = i
        for _ in range(8):
            c = (c >> 1) ^ 0x82F63B78 if c & 1 else c >> 1
        table.append(c)
    return table


_CRC_TABLE = _crc32c_table()


def crc32c(data: bytes) -> int:
    c = 0xFFFFFFFF
    for b in data:
        c = _CRC_TABLE[(c ^ b) & 0xFF] ^ (c >> 8)
    return c ^ 0xFFFFFFFF


def _masked_crc(data: bytes) -> int:
    # the TFRecord checksum: rotate right by 15 and add a constant
    c = crc32c(data)
    return ((((c >> 15) | (c << 17)) & 0xFFFFFFFF) + 0xA282EAD8) & 0xFFFFFFFF


def _varint(n: int) -> bytes:
    out = bytearray()
    n &= (1 << 64) - 1
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len_field(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _histo_proto(values: Sequence[float]) -> bytes:
    vals = sorted(float(v) for v in values)
    n = len(vals)
    lo, hi = vals[0], vals[-1]
    n_buckets = 30
    edges = [lo + (hi - lo) * (i + 1) / n_buckets for i in range(n_buckets)] if hi > lo else [hi]
    counts = [0.0] * len(edges)
    j = 0
    for v in vals:
        while j < len(edges) - 1 and v > edges[j]:
            j += 1
        counts[j] += 1.0
    msg = (_key(1, 1) + struct.pack("<d", lo) + _key(2, 1) + struct.pack("<d", hi) + _key(3, 1)
           + struct.pack("<d", float(n)) + _key(4, 1) + struct.pack("<d", sum(vals)) + _key(5, 1)
           + struct.pack("<d", sum(v * v for v in vals)))
    msg += _len_field(6, b"".join(struct.pack("<d", e) for e in edges))
    msg += _len_field(7, b"".join(struct.pack("<d", c) for c in counts))
    return msg


def _event(step: int, *, scalars: dict[str, float] | None = None, histos: dict[str, Sequence[float]] | None = None,
           file_version: str | None = None) -> bytes:
    ev = _key(1, 1) + struct.pack("<d", time.time()) + _key(2, 0) + _varint(int(step))
    if file_version is not None:
        ev += _len_field(3, file_version.encode())
    values = b""
    for tag, v in (scalars or {}).items():
        values += _len_field(1, _len_field(1, tag.encode()) + _key(2, 5) + struct.pack("<f", float(v)))
    for tag, vals in (histos or {}).items():
        values += _len_field(1, _len_field(1, tag.encode()) + _len_field(5, _histo_proto(vals)))
    if values:
        ev += _len_field(5, values)
    return ev


def _record(data: bytes) -> bytes:
    header = struct.pack("<Q", len(data))
    return header + struct.pack("<I", _masked_crc(header)) + data + struct.pack("<I", _masked_crc(data))


class MetricsWriter:
    """Rank-0 metric sink: TensorBoard event file + ``metrics.jsonl``; never stops training."""

    def __init__(self, log_dir: str | None, enabled: bool = True, use_tensorboard: bool | None = None):
        self.log_dir = log_dir
        self.enabled = bool(enabled and log_dir)
        self._tb = None
        self._f = None
        self._jsonl = None
        if not self.enabled:
            return
        os.makedirs(log_dir, exist_ok=True)
        if use_tensorboard is not False:
            try:
                from torch.utils.tensorboard import SummaryWriter  # noqa: F401

                self._tb = SummaryWriter(log_dir=log_dir)
            except Exception:
                self._tb = None
        if self._tb is None:
            name = f"events.out.tfevents.{int(time.time())}.{socket.gethostname()}.{os.getpid()}.meshy"
            self._f = open(os.path.join(log_dir, name), "ab")
            self._f.write(_record(_event(0, file_version="brain.Event:2")))
            self._f.flush()
        self._jsonl = open(os.path.join(log_dir, "metrics.jsonl"), "a")

    def write(self, metrics: dict[str, Any], step: int, histograms: dict[str, Iterable[float]] | None = None) -> None:
        if not self.enabled:
            return
        scalars = {k: float(v) for k, v in metrics.items()
                   if isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v))}
        histos = {}
        for name, vals in (histograms or {}).items():
            vals = [float(x) for x in vals if math.isfinite(float(x))]
            if not vals:
                continue
            if len(vals) > HISTOGRAM_MAX_VALUES:
                stride = math.ceil(len(vals) / HISTOGRAM_MAX_VALUES)
                vals = vals[::stride]
            histos[name if name.startswith(HISTOGRAM_PREFIX) else HISTOGRAM_PREFIX + name] = vals
        try:
            if self._tb is not None:
                import torch

                for k, v in scalars.items():
                    self._tb.add_scalar(k, v, global_step=step)
                for k, v in histos.items():
                    self._tb.add_histogram(k, torch.tensor(v), global_step=step)
                self._tb.flush()
            elif self._f is not None:
                self._f.write(_record(_event(step, scalars=scalars, histos=histos)))
                self._f.flush()
            self._jsonl.write(json.dumps({"step": int(step), **scalars}) + "\n")
            self._jsonl.flush()
        except Exception:
            pass

    def close(self) -> None:
        for h in (self._tb, self._f, self._jsonl):
            try:
                if h is not None:
                    h.close()
            except Exception:
                pass


def read_events(path: str) -> list[tuple[int, dict[str, float]]]:
    """Decode the scalar values of an event file written by :class:`MetricsWriter` (tests, tools)."""
    out = []
    with open(path, "rb") as f:
        data = f.read()
    i = 0
    while i + 12 <= len(data):
        (n,) = struct.unpack_from("<Q", data, i)
        (hcrc,) = struct.unpack_from("<I", data, i + 8)
        if hcrc != _masked_crc(data[i:i + 8]):
            raise ValueError("corrupt record header")
        body = data[i + 12:i + 12 + n]
        (dcrc,) = struct.unpack_from("<I", data, i + 12 + n)
        if dcrc != _masked_crc(body):
            raise ValueError("corrupt record body")
        i += 16 + n
        out.append(_decode_event(body))
    return out


def _read_varint(b: bytes, i: int) -> tuple[int, int]:
    shift = n = 0
    while True:
        c = b[i]
        i += 1
        n |= (c & 0x7F) << shift
        shift += 7
        if not c & 0x80:
            return n, i


def _fields(b: bytes):
    i = 0
    while i < len(b):
        key, i = _read_varint(b, i)
        f, w = key >> 3, key & 7
        if w == 0:
            v, i = _read_varint(b, i)
        elif w == 1:
            v = b[i:i + 8]
            i += 8
        elif w == 5:
            v = b[i:i + 4]
            i += 4
        else:
            ln, i = _read_varint(b, i)
            v = b[i:i + ln]
            i += ln
        yield f, w, v


def _decode_event(b: bytes) -> tuple[int, dict[str, float]]:
    step, scalars = 0, {}
    for f, w, v in _fields(b):
        if f == 2:
            step = v
        elif f == 5:
            for f2, _, val in _fields(v):
                if f2 != 1:
                    continue
                tag, sv = None, None
                for f3, w3, x in _fields(val):
                    if f3 == 1:
                        tag = x.decode()
                    elif f3 == 2 and w3 == 5:
                        sv = struct.unpack("<f", x)[0]
                if tag is not None and sv is not None:
                    scalars[tag] = sv
    return step, scalars


__all__ = ["HISTOGRAM_PREFIX", "MetricsWriter", "crc32c", "perf_metrics", "read_events", "rollout_metrics"]
