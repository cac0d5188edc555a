"""Gate-driven GRPO/PPO producer (reference ``meshy/worker/rollout.py:214-731``).

Loop: for each prompt of the (seekable) dataset, acquire a generation slot —
``pacing_window`` W allows ``(gates_seen - 1 + W) * batch_size`` samples to
be started (W=1 lock-step, W>=2 bounded off-policy, None fully async) — then
generate ``group_size`` completions concurrently, score them (reward +
optional shaping, stamps truncated / repetition / mixed_version), optionally
drop zero-variance groups, compute the advantage plug-in (unless a critic owns
it), and append the group's rows to the data partition.  Gate ``N`` arrivals
also drive the rollout's checkpoint shard.
"""

from __future__ import annotations

import asyncio
import time
import copy
import json
import logging
import math
import os
from typing import Any, Callable

import torch

from ..advantage import assign_positive_lm_weights, grpo_advantage, is_zero_variance_group
from ..config import GRPO_TRAINER_FIELDS, GlobalCheckpointConfig
from ..service.registry import resolve_callable
from ..tq.client import Columns
from ..tq.control import GEN_GATE_FIELDS, GEN_GATE_PARTITION, GEN_GATE_TASK
from ..utils.metric import has_repetition
from ..utils.sample import SampleBuilder
from .tq import TQInput, TQOutput, TQWorker

log = logging.getLogger(__name__)

GRPO_FIELDS = tuple(GRPO_TRAINER_FIELDS) + ("positive_lm_weight",)
GRPO_FIELDS_NO_ADVANTAGE = tuple(f for f in GRPO_FIELDS if f != "advantage")
RAW_REWARD_FIELD = "raw_reward"


def sample_to_row(sample, weight_version: int) -> dict:
    raw = getattr(sample, "raw_reward", None)
    return {
        "tokens": torch.tensor(list(sample.tokens), dtype=torch.long),
        "logprobs": torch.tensor(list(sample.logprobs), dtype=torch.float32),
        "mask_assistant": torch.tensor(list(sample.masks), dtype=torch.float32),
        "advantage": torch.tensor(0.0 if sample.advantage is None else float(sample.advantage)),
        "weight_version": torch.tensor(int(weight_version)),
        "reward": torch.tensor(float(sample.reward)),
        "positive_lm_weight": torch.tensor(float(getattr(sample, "positive_lm_weight", 0.0))),
        RAW_REWARD_FIELD: torch.tensor(float(sample.reward if raw is None else raw)),
        "truncated": torch.tensor(int(bool(sample.truncated))),
        "repetition": torch.tensor(int(bool(sample.repetition))),
        "mixed_version": torch.tensor(int(bool(sample.mixed_version))),
    }


class TrajectoryLogger:
    """Append-only JSONL of every finished sample (reference ``rollout.py:162-211``)."""

    def __init__(self, path: str, verbose: bool = False):
        self.path = path
        self.verbose = verbose
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)

    async def write(self, group: list, version: int) -> None:
        lines = []
        for s in group:
            rec = {"timestamp": time.time(), "weight_version": version, "reward": s.reward, "raw_reward": s.raw_reward,
                   "advantage": s.advantage, "finish_reason": s.finish_reason, "truncated": s.truncated,
                   "repetition": s.repetition, "messages": s.messages, "n_tokens": len(s.tokens)}
            if self.verbose:
                rec.update({"tokens": list(s.tokens), "logprobs": list(s.logprobs), "masks": list(s.masks)})
            lines.append(json.dumps(rec, default=str))
        await asyncio.to_thread(self._append, lines)

    def _append(self, lines):
        with open(self.path, "a", encoding="utf-8") as f:
            f.write("\n".join(lines) + "\n")


class RolloutWorker(TQWorker):
    def __init__(self, *, engine, endpoints_ref: str | None, model_path: str, dataset, dataset_kwargs: dict | None,
                 partition_id: str, group_size: int, train_batch_size: int, sampling_params: dict | None,
                 reward, reward_shaping=None, reward_shaping_kwargs: dict | None = None, advantage=None,
                 advantage_kwargs: dict | None = None, filter_zero_std_groups: bool = False,
                 publish_positive_lm_weights: bool = False, oversample_factor: float = 1.0, num_epochs: int = 1,
                 pacing_window: int | str | None = 1, max_running_requests: int = -1, poll_interval: float = 2.0,
                 trajectory_log: str | None = None, verbose_trajectory_log: bool = False,
                 external_advantage: bool = False, checkpoint=None, resume_step: int = 0,
                 state_dir: str | None = None, service_name: str = "rollout", client_factory=None, colocation=None,
                 builder: SampleBuilder | None = None):
        super().__init__()
        if group_size <= 0 or train_batch_size <= 0:
            raise ValueError("group_size and train_batch_size must be positive")
        if num_epochs <= 0:
            raise ValueError("num_epochs must be positive")
        if pacing_window == "auto":
            pacing_window = 1
        if pacing_window is not None and int(pacing_window) < 1:
            raise ValueError("pacing_window must be >= 1, 'auto', or None")
        self.engine = engine
        self.colocation = colocation
        self._colo_request = None
        self.model_path = model_path
        self.builder = builder
        self.dataset_factory = resolve_callable(dataset)
        self.dataset_kwargs = dict(dataset_kwargs or {})
        self.group_size = int(group_size)
        self.train_batch_size = int(train_batch_size)
        self.sampling_params = dict(sampling_params or {})
        self.reward_fn = resolve_callable(reward)
        self.reward_shaping_fn = resolve_callable(reward_shaping) if reward_shaping is not None else None
        self.reward_shaping_kwargs = dict(reward_shaping_kwargs or {})
        self.external_advantage = bool(external_advantage)
        if self.external_advantage:
            if advantage is not None:
                raise ValueError("external_advantage hands the advantage to a critic; drop the advantage callable")
            self.advantage_fn = None
            fields = GRPO_FIELDS_NO_ADVANTAGE
        else:
            self.advantage_fn = grpo_advantage if advantage is None else resolve_callable(advantage)
            fields = GRPO_FIELDS
        if self.reward_shaping_fn is not None:
            fields = fields + (RAW_REWARD_FIELD,)
        self.rollout_fields = tuple(fields)
        self.publish_positive_lm_weights = publish_positive_lm_weights
        self.advantage_kwargs = dict(advantage_kwargs or {})
        self.filter_zero_std_groups = bool(filter_zero_std_groups)
        if oversample_factor < 1.0:
            raise ValueError("oversample_factor must be >= 1")
        self.oversample_factor = float(oversample_factor)
        self.num_epochs = int(num_epochs)
        self.pacing_window = None if pacing_window is None else int(pacing_window)
        self.max_running_requests = int(max_running_requests)
        self.poll_interval = float(poll_interval)
        self.gates_seen = 0
        self.weight_version = 0
        self.samples_started = 0
        self.groups_seen = 0
        self.groups_filtered = 0
        self.checkpoint = GlobalCheckpointConfig.coerce(checkpoint)
        self.resume_step = int(resume_step)
        self.service_name = service_name
        self._state_dir = state_dir
        self._epoch = 0
        self._dataset_index = 0
        self._filtered_at_epoch_start = 0
        self._restore()
        self.trajectory_logger = TrajectoryLogger(trajectory_log, verbose_trajectory_log) if trajectory_log else None
        self.configure_tq(
            endpoints_ref=endpoints_ref, input=None,
            controls={"gen_gate": TQInput(GEN_GATE_PARTITION, tuple(GEN_GATE_FIELDS), 1, GEN_GATE_TASK, True)},
            outputs={"rollouts": TQOutput(self.rollout_fields, new_rows=True, partition=partition_id)},
            poll_interval=poll_interval, client_factory=client_factory)

    # ------------------------------------------------------------------ checkpoint
    @property
    def store(self):
        from ..service.checkpoint import StateStore

        if not self._state_dir:
            raise RuntimeError("rollout checkpointing needs a state_dir")
        return StateStore(self._state_dir)

    def _restore(self) -> None:
        if self.resume_step <= 0:
            return
        p = self.store.payload(self.service_name, self.resume_step)
        if not p:
            raise FileNotFoundError(f"resuming at {self.resume_step} but the rollout shard is missing")
        self._epoch = int(p["epoch"])
        self._dataset_index = int(p["dataset_index"])
        self._filtered_at_epoch_start = int(p["filtered_at_epoch_start"])
        self.groups_seen = int(p["groups_seen"])
        self.groups_filtered = int(p["groups_filtered"])
        self.samples_started = int(p["samples_started"])
        self.weight_version = int(p["weight_version"])
        # the trainer re-publishes a gate AT resume_step (data plane is RAM-only)
        self.gates_seen = self.resume_step

    def _snapshot(self, step: int) -> None:
        self.store.write_meta(self.service_name, step, {
            "epoch": self._epoch, "dataset_index": self._dataset_index,
            "filtered_at_epoch_start": self._filtered_at_epoch_start, "groups_seen": self.groups_seen,
            "groups_filtered": self.groups_filtered, "gates_seen": self.gates_seen,
            "samples_started": self.samples_started, "weight_version": self.weight_version})
        self.store.mark_complete(self.service_name, step)
        self.store.prune(self.service_name, self.checkpoint.keep_latest_k)

    # ------------------------------------------------------------------ pacing
    def generation_budget(self) -> int:
        if self.gates_seen == 0:
            return 0
        return (self.gates_seen - 1 + self.pacing_window) * self.train_batch_size

    async def try_advance_gate(self) -> bool:
        data = await self.read_tq_control("gen_gate")
        if data is None:
            return False
        step = int(data["gate_step"][0].reshape(-1)[0])
        version = int(data["weight_version"][0].reshape(-1)[0])
        if step != self.gates_seen:
            log.warning("gen_gate out of order: expected %d, got %d (v%d)", self.gates_seen, step, version)
        self.gates_seen += 1
        self.weight_version = version
        if self.checkpoint.due(step) and step > self.resume_step:
            self._snapshot(step)
        return True

    async def acquire_generation_slot(self, n: int) -> int:
        if n <= 0:
            raise ValueError("n must be positive")
        while self.gates_seen == 0:
            if self.stopped:
                raise asyncio.CancelledError
            if not await self.try_advance_gate():
                await asyncio.sleep(min(self.poll_interval, 2.0))
        if self.pacing_window is None:
            while await self.try_advance_gate():
                pass
            self.samples_started += n
            return self.weight_version
        while self.samples_started + n > self.generation_budget():
            if self.stopped:
                raise asyncio.CancelledError
            if not await self.try_advance_gate():
                await asyncio.sleep(min(self.poll_interval, 2.0))
        self.samples_started += n
        return self.weight_version

    async def _ensure_colocation(self) -> None:
        if self.colocation is None or self.colocation.owns_gpu:
            return
        if self._colo_request is None:
            from ..service.colocation import SchedulingMode

            self._colo_request = self.colocation.request_gpu(request_id=f"rollout:fallback:{self.gates_seen}",
                                                             kind=SchedulingMode.FALLBACK)
        await asyncio.to_thread(self.colocation.wait_for_grant, self._colo_request)
        self._colo_request = None

    # ------------------------------------------------------------------ groups
    async def rollout_group(self, prompt, version: int) -> list | None:
        await self._ensure_colocation()
        group = [copy.deepcopy(prompt) for _ in range(self.group_size)]

        async def one(s):
            gen = await self.engine.generate(list(s.tokens), sampling_params=self.sampling_params)
            self.builder.append_tokens(s, "assistant", gen.output_ids, gen.output_logprobs)
            s.finish_reason = gen.finish_reason
            s.truncated = gen.finish_reason == "length"
            s.mixed_version = int(getattr(gen, "continuations", 0) or 0) > 0
            s.repetition = has_repetition(s.messages[-1]["content"] if s.messages else "")
            r = float(self.reward_fn(s))
            if self.reward_shaping_fn is not None:
                s.raw_reward = r
                s.reward = float(self.reward_shaping_fn(r, s, **self.reward_shaping_kwargs))
            else:
                s.reward = r
            return s

        group = list(await asyncio.gather(*(one(s) for s in group)))
        if self.publish_positive_lm_weights:
            assign_positive_lm_weights(group)
        self.groups_seen += 1
        if self.filter_zero_std_groups and is_zero_variance_group(group):
            self.groups_filtered += 1
            return None
        if self.advantage_fn is not None:
            out = self.advantage_fn(group, **self.advantage_kwargs)
            if out is not None:
                vals = list(out)
                if len(vals) != len(group):
                    raise ValueError("advantage function result length must match the group")
                for s, v in zip(group, vals):
                    s.advantage = float(v)
        return group

    async def write_group(self, group: list, version: int) -> None:
        rows = [sample_to_row(s, version) for s in group]
        data = Columns.from_rows(rows, self.rollout_fields)
        if self.trajectory_logger is not None:
            await self.trajectory_logger.write(group, version)
        await self.write_tq_output("rollouts", data)

    def _oversample_budget(self, n_prompts):
        if not self.filter_zero_std_groups or self.oversample_factor <= 1.0 or not n_prompts:
            return None
        return int(n_prompts * (self.oversample_factor - 1.0))

    def run(self) -> None:
        asyncio.run(self.run_async())

    async def run_async(self) -> None:
        await self.open_tq()
        try:
            await self._run_rollouts()
        finally:
            await self.close_tq()
            close = getattr(self.engine, "close", None)
            if close is not None:
                try:
                    await close()
                except Exception:
                    pass

    async def _run_rollouts(self) -> None:
        if self.builder is None:
            self.builder = SampleBuilder(self.model_path)
        max_groups = max(1, math.ceil(self.max_running_requests / self.group_size)) \
            if self.max_running_requests > 0 else None
        sem = asyncio.Semaphore(max_groups) if max_groups else None
        tasks: set = set()

        async def execute(prompt, version):
            try:
                g = await self.rollout_group(prompt, version)
                if g is not None:
                    await self.write_group(g, version)
            except Exception as e:  # a failed group is dropped, the run goes on
                log.exception("rollout group failed: %s", e)
            finally:
                if sem is not None:
                    sem.release()

        resuming = self.resume_step > 0
        for epoch in range(self._epoch, self.num_epochs):
            if self.stopped:
                break
            self._epoch = epoch
            ds = self.dataset_factory(**self.dataset_kwargs)
            if resuming:
                ds.seek(self._dataset_index)
            else:
                self._dataset_index = 0
                self._filtered_at_epoch_start = self.groups_filtered
            resuming = False
            budget = self._oversample_budget(getattr(ds, "n_prompts", None))
            while not self.stopped:
                prompts = ds.next_batch(self.builder)
                self._dataset_index = int(getattr(ds, "index", self._dataset_index + len(prompts)))
                if not prompts:
                    break
                if budget is not None and self.groups_filtered - self._filtered_at_epoch_start > budget:
                    break
                for p in prompts:
                    version = await self.acquire_generation_slot(self.group_size)
                    if sem is not None:
                        await sem.acquire()
                    t = asyncio.create_task(execute(p, version))
                    tasks.add(t)
                    t.add_done_callback(tasks.discard)
        if tasks:
            await asyncio.gather(*tasks)
        await self.drain()

    async def drain(self, timeout: float | None = None) -> None:
        """After the last epoch: wait until consumers have cleared every row written to the data
        partition, so the run ends after the final trainer step instead of before it."""
        out = self.tq_outputs.get("rollouts")
        part = out.partition if out is not None else None
        if not part:
            return
        deadline = None if timeout is None else time.monotonic() + timeout
        while not self.stopped:
            n = await self.tq_call(lambda: self._aclient.num_rows(part))
            if n == 0:
                break
            if deadline is not None and time.monotonic() > deadline:
                log.warning("drain: %d rows still unconsumed in %s", n, part)
                return
            await asyncio.sleep(self.poll_interval)
        await self.await_final_weights()

    async def await_final_weights(self, timeout: float | None = None) -> None:
        """After the last step: wait until every engine serves the trainer's final weights. The trainer hands
        them over after clearing its batch (through the card's colocation ring when colocated), so ending the
        run at once would tear the engines down in the middle of that hand-over."""
        timeout = float(os.environ.get("XRL_FINAL_SYNC_TIMEOUT", "60")) if timeout is None else timeout
        versions = getattr(self.engine, "weight_versions", None)
        if versions is None or timeout <= 0:
            return
        while not self.stopped:  # the gates raised since the last generation slot (no snapshot: the run ends)
            data = await self.read_tq_control("gen_gate")
            if data is None:
                break
            self.gates_seen += 1
            self.weight_version = int(data["weight_version"][0].reshape(-1)[0])
        want = self.weight_version
        if want is None:
            return
        deadline = time.monotonic() + timeout
        have = None
        while not self.stopped:
            try:
                have = await asyncio.to_thread(versions)
            except Exception as e:  # noqa: BLE001 - an engine that is down ends the wait at the deadline
                have = repr(e)
            if isinstance(have, list) and all(v is not None and int(v) >= want for v in have):
                return
            if time.monotonic() > deadline:
                log.warning("final weights v%d not on every engine after %.0f s (engines: %s)", want, timeout, have)
                return
            await asyncio.sleep(min(self.poll_interval, 0.5))


__all__ = ["GRPO_FIELDS", "GRPO_FIELDS_NO_ADVANTAGE", "RAW_REWARD_FIELD", "RolloutWorker", "TrajectoryLogger",
           "sample_to_row"]
