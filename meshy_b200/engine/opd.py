"""On-policy distillation engines (reference ``meshy/engine/opd.py:39-143``).

* :class:`StudentTopKEngine` — the actor trainer engine with the
  :class:`~meshy_b200.backend.opd.StudentTopKTrainer` swapped in.
* :class:`OPDTeacherEngine` — a frozen teacher replica: ``score(samples)``
  broadcasts the rows, every rank scores its token-balanced share (packed
  micro-batches under a token budget) and rank 0 gathers per-row Top-K ids and
  log-probs ``[L, K]`` (row ``t`` = the teacher's distribution over token
  ``t + 1``; the last row is zero).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..backend.plan import snake_deal
from ..backend.topk_loss import teacher_topk
from ..models import build_model, get_model_args
from .spmd import SpmdEngine
from .trainer import TrainerEngine


class StudentTopKEngine(TrainerEngine):
    def __init__(self, *a, log_prob_min_clamp: float | None = -10.0, loss_max_clamp: float | None = 10.0, **kw):
        super().__init__(*a, **kw)
        self.clamps = (log_prob_min_clamp, loss_max_clamp)

    def setup(self) -> None:
        from ..backend.opd import StudentTopKTrainer

        if self.world_size > 1 and not torch.distributed.is_initialized():
            self.init_process_group()
        self.trainer = StudentTopKTrainer(self.tc, self.tp, device=self.device,
                                          dp_group=self.compute_group if self.world_size > 1 else None,
                                          log_prob_min_clamp=self.clamps[0], loss_max_clamp=self.clamps[1])
        if self.model_path and os.path.isdir(self.model_path):
            from ..models.hf import load_hf_checkpoint

            self.trainer.flat.load_state_dict(load_hf_checkpoint(self.trainer.model_args, self.model_path))


class OPDTeacherEngine(SpmdEngine):
    def __init__(self, config, **kw):
        super().__init__(**kw)
        self.cfg = config
        self.model = None
        self.weight_version = 0

    def setup(self) -> None:
        super().setup()
        tc = self.cfg.trainer_config
        args = get_model_args(tc.model_name, tc.model_flavor)
        dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.model = build_model(args, device=self.device, dtype=dtype).eval()
        for p in self.model.parameters():
            p.requires_grad_(False)
        if self.cfg.model_path and os.path.isdir(self.cfg.model_path):
            from ..models.hf import load_hf_checkpoint

            sd = load_hf_checkpoint(args, self.cfg.model_path)
            with torch.no_grad():
                for n, p in self.model.named_parameters():
                    p.copy_(sd[n].to(p.dtype))
        self.seq_len = tc.seq_len

    def score(self, samples: list) -> list[tuple[torch.Tensor, torch.Tensor]] | None:
        return self.submit_command("score", samples)

    @torch.no_grad()
    def _score_rows(self, samples, rows) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
        k = int(self.cfg.top_k)
        out = {}
        budget = max(self.seq_len, 8192)
        batch, used = [], 0
        lens = {i: min(len(torch.as_tensor(samples[i]["tokens"]).reshape(-1)), self.seq_len) for i in rows}

        def flush(group):
            if not group:
                return
            d = self.device
            ids = torch.cat([torch.as_tensor(samples[i]["tokens"]).reshape(-1)[:lens[i]].long() for i in group]).to(d)
            pos = torch.cat([torch.arange(lens[i], dtype=torch.int32) for i in group]).to(d)
            cu = torch.tensor([0] + list(torch.tensor([lens[i] for i in group]).cumsum(0).tolist()),
                              dtype=torch.int32, device=d)
            h = self.model.hidden(ids, pos, cu, max(lens[i] for i in group))
            tid, tlp = teacher_topk(h, self.model.output_weight, k)
            off = 0
            for i in group:
                L = lens[i]
                a, b = tid[off:off + L].cpu(), tlp[off:off + L].cpu()
                a[L - 1] = 0
                b[L - 1] = 0.0
                out[i] = (a, b)
                off += L

        for i in rows:
            if used + lens[i] > budget and batch:
                flush(batch)
                batch, used = [], 0
            batch.append(i)
            used += lens[i]
        flush(batch)
        return out

    def cmd_score(self, samples) -> list | None:
        n = len(samples)
        lens = [len(torch.as_tensor(s["tokens"]).reshape(-1)) for s in samples]
        order = sorted(range(n), key=lambda i: (-lens[i], i))
        rows = list(snake_deal(order, self.world_size)[self.rank]) if self.world_size > 1 else list(range(n))
        mine = self._score_rows(samples, rows)
        if self.world_size == 1:
            parts = [mine]
        else:
            parts = [None] * self.world_size if self.rank == 0 else None
            dist.gather_object(mine, parts, dst=0, group=self.control_group)
        if self.rank != 0:
            return None
        allr = {}
        for p in parts:
            allr.update(p)
        return [allr[i] for i in range(n)]

    def on_colocate_acquire(self, grant) -> None:
        pass

    def on_colocate_release(self, target: str) -> None:
        pass


__all__ = ["OPDTeacherEngine", "StudentTopKEngine"]
