"""Paged-KV continuous-batching rollout engine (replaces the reference's SGLang).

Capabilities the reference uses from SGLang (``meshy/engine/sglang.py``) and
how they map here:

* ``/generate`` with ``return_logprob``: :meth:`RolloutEngine.generate` /
  :meth:`submit` + :meth:`step` return output ids, per-token log-probs of the
  sampled tokens and a finish reason (``stop`` / ``length`` / ``abort``);
* ``/pause_generation {mode: abort}`` / ``/continue_generation``:
  :meth:`abort_all`, :meth:`pause`, :meth:`resume`;
* ``/release_memory_occupation`` / ``/resume_memory_occupation`` (tags
  ``kv_cache``, ``weights``): :meth:`release_memory`, :meth:`resume_memory`
  through the VMM pool (:mod:`.memory`), so virtual addresses — and hence
  captured CUDA graphs — survive a hand-off;
* ``/update_weights_from_disk``: :meth:`update_weights_from_disk`; plus the
  device path :meth:`update_weights_from_flat` (one device copy, or done by the
  trainer's optimiser kernel writing straight into :attr:`weight_flat`).

Execution model:

* weights live in one flat bf16 buffer with the trainer's layout;
* the KV cache is ``[layers, 2, pages, kv_heads, page, head_dim]``; a host
  block manager (:mod:`.kv_cache`) hands out pages;
* prefill runs new prompts as one packed varlen forward and writes their KV;
* a decode step (embedding → layers → fused LM-head sampler → row advance) is
  captured once per batch-size bucket in a CUDA graph and replayed; rows that
  finish are compacted away every ``sync_every`` steps, the only host↔device
  synchronisation of the loop.
"""

from __future__ import annotations

import itertools
import math
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from ..models.args import ModelArgs
from ..models.transformer import DecoderLM
from ..ops import decode as D
from ..ops import functional as Fx
from .kv_cache import BlockManager

_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)


@dataclass
class Request:
    rid: Any
    prompt: list[int]
    max_new_tokens: int
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    # engine state
    out_slot: int = -1
    pages: list[int] = field(default_factory=list)
    submitted: float = 0.0


@dataclass
class Generation:
    rid: Any
    prompt_ids: list[int]
    output_ids: list[int]
    output_logprobs: list[float]
    finish_reason: str
    weight_version: int = 0

    @property
    def tokens(self) -> list[int]:
        return self.prompt_ids + self.output_ids


def _bucket(n: int) -> int:
    for b in _BUCKETS:
        if b >= n:
            return b
    return n


class RolloutEngine:
    def __init__(
        self,
        args: ModelArgs,
        *,
        device: str | torch.device = "cpu",
        model: DecoderLM | None = None,
        max_running: int = 256,
        max_total_tokens: int | None = None,
        page_size: int = 64,
        max_seq_len: int | None = None,
        use_cuda_graph: bool = True,
        sync_every: int = 16,
        seed: int = 0,
        eos_token_ids: Sequence[int] = (),
        prefill_chunk_tokens: int = 32768,
        mem_fraction: float = 0.5,
        tp_group=None,
        ep: bool = False,
    ):
        from ..backend.flat import Slot, _align, flatten_module

        self.args = args
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.dtype = torch.bfloat16 if self.cuda else torch.float32
        if model is None:
            from ..models import build_model

            model = build_model(args, seed=seed, device=self.device, dtype=self.dtype)
        # tensor parallelism: this rank keeps its heads and FFN slice of every dense block (the embedding, the
        # norms, the LM head and MoE experts stay whole); the row-parallel outputs are summed over tp_group
        import torch.distributed as dist

        self.tp_group = tp_group if (tp_group is not None and dist.is_initialized()
                                     and dist.get_world_size(tp_group) > 1) else None
        self.tp, self.tp_rank = 1, 0
        self.ep = bool(ep) and self.tp_group is not None  # MoE experts split over the TP ranks too
        self.local_args = args
        self.full_slots = None
        if self.tp_group is not None:
            from ..parallel.tp import local_args, shard_model_tp

            self.tp, self.tp_rank = dist.get_world_size(self.tp_group), dist.get_rank(self.tp_group)
            off, self.full_slots = 0, []
            for name, p in model.named_parameters():  # the trainer's (unsharded) flat layout
                self.full_slots.append(Slot(name, off, p.numel(), tuple(p.shape)))
                off += _align(p.numel())
            shard_model_tp(model, self.tp_group, ep=self.ep)
            self.local_args = local_args(args, self.tp)
        self.model = model.eval()
        for p in self.model.parameters():
            p.requires_grad_(False)
        self.weight_flat, self.weight_slots = flatten_module(self.model, self.dtype, self.device)
        self._vmm = {}
        if self.cuda:
            # weights and KV cache live in virtual-memory regions: releasing them for a colocated trainer
            # frees the physical pages but keeps the addresses, so captured decode graphs stay valid
            from ..ops._ext import ext

            n = self.weight_flat.numel()
            reg = ext().VmmRegion(n * self.weight_flat.element_size(), self.device.index or 0)
            view = reg.view(0, [n], self.weight_flat.dtype)
            view.copy_(self.weight_flat)
            self._vmm["weights"] = reg
            self.weight_flat = view
            self._rebind_weights()
            torch.cuda.empty_cache()
        self.page_size = page_size
        self.max_running = max_running
        self.max_seq_len = min(max_seq_len or args.max_seq_len, args.max_seq_len)
        self.max_pages_per_seq = math.ceil(self.max_seq_len / page_size)
        if max_total_tokens is None:
            if self.cuda:
                free, _ = torch.cuda.mem_get_info(self.device)
                max_total_tokens = int(free * mem_fraction) // max(1, self.local_args.kv_bytes_per_token(2))
            else:
                max_total_tokens = 64 * 1024
        n_pages = max(1, max_total_tokens // page_size)
        self.n_pages = n_pages
        self.blocks = BlockManager(n_pages, page_size)
        self._alloc_kv()
        self.use_cuda_graph = use_cuda_graph and self.cuda
        self.sync_every = max(1, sync_every)
        self.seed = seed
        self.eos = list(eos_token_ids)
        self.prefill_chunk_tokens = prefill_chunk_tokens
        self.weight_version = 0
        self._rid = itertools.count()
        self._gen = torch.Generator(device="cpu").manual_seed(seed)
        self.waiting: list[Request] = []
        self.running: list[Request] = []   # row i <-> running[i]
        self.finished: dict[Any, Generation] = {}
        self.paused = False
        self.lock = threading.RLock()
        self._graphs: dict[int, Any] = {}
        self.stats = {"decode_steps": 0, "prefill_tokens": 0, "decode_tokens": 0, "graph_replays": 0}
        self._init_state()
        self._mega = None
        self._mega_rows = 0
        self.mega_reason = "not on CUDA"
        if self.cuda and self.tp_group is None:
            from .mega import MAX_ROWS, MegaDecoder

            self.mega_reason = MegaDecoder.reason(self.model, self.page_size)
            if self.mega_reason is None:
                self._mega = MegaDecoder(self.model, self.kv, self.device)
                self._mega_rows = MAX_ROWS

    # ------------------------------------------------------------------ memory
    def _alloc_kv(self):
        a = self.local_args  # this rank's KV heads
        shape = [a.n_layers, 2, self.n_pages, a.n_kv_heads, self.page_size, a.head_dim]
        if not self.cuda:
            self.kv = torch.zeros(*shape, dtype=self.dtype, device=self.device)
            return
        from ..ops._ext import ext

        nbytes = math.prod(shape) * torch.empty((), dtype=self.dtype).element_size()
        reg = self._vmm.get("kv_cache") if hasattr(self, "_vmm") else None
        if reg is None:
            reg = ext().VmmRegion(nbytes, self.device.index or 0)
            self._vmm["kv_cache"] = reg
        elif not reg.mapped:
            reg.map()
        self.kv = reg.view(0, shape, self.dtype)
        self.kv.zero_()

    def _init_state(self):
        B, dev = self.max_running, self.device
        R = B  # one output slot per concurrently running request
        self.max_new_cap = self.max_seq_len
        i32, i64 = torch.int32, torch.int64
        self.st = {
            "tok_in": torch.zeros(B, dtype=i64, device=dev),
            "pos": torch.zeros(B, dtype=i32, device=dev),
            "seq_lens": torch.ones(B, dtype=i32, device=dev),
            "gen": torch.zeros(B, dtype=i32, device=dev),
            "max_new": torch.zeros(B, dtype=i32, device=dev),
            "done": torch.ones(B, dtype=i32, device=dev),
            "slot": torch.zeros(B, dtype=i64, device=dev),
            "block_table": torch.zeros(B, self.max_pages_per_seq, dtype=i32, device=dev),
            "req": torch.arange(B, dtype=i32, device=dev),
            # one spare row past the R output slots: a write that must land nowhere goes there
            "out_tok": torch.zeros(R + 1, self.max_new_cap, dtype=i64, device=dev),
            "out_lp": torch.zeros(R + 1, self.max_new_cap, dtype=torch.float32, device=dev),
            "eos": torch.tensor(self.eos, dtype=i64, device=dev),
            "noeos": torch.zeros(0, dtype=i64, device=dev),
            "step": torch.zeros(1, dtype=i64, device=dev),
        }
        self.free_out_slots = list(range(R))
        self._park_rows(0)

    def release_memory(self, tags: Sequence[str] = ("kv_cache", "weights")) -> None:
        """Give GPU memory back for a colocated trainer.

        On CUDA the physical pages of the tagged regions are released while their virtual addresses stay
        reserved, so the captured decode graphs remain valid; weights are parked in pinned host memory
        first (the KV cache is dropped: requests were aborted before a release)."""
        with self.lock:
            if not self.cuda:
                return
            torch.cuda.synchronize(self.device)
            if "weights" in tags and self._vmm["weights"].mapped:
                host = torch.empty(self.weight_flat.shape, dtype=self.weight_flat.dtype, pin_memory=True)
                host.copy_(self.weight_flat)
                self._host_weights = host
                self._vmm["weights"].unmap()
            if "kv_cache" in tags and "kv_cache" in self._vmm and self._vmm["kv_cache"].mapped:
                self._vmm["kv_cache"].unmap()
            torch.cuda.empty_cache()

    def resume_memory(self, tags: Sequence[str] = ("kv_cache", "weights")) -> None:
        with self.lock:
            if not self.cuda:
                return
            if "weights" in tags and not self._vmm["weights"].mapped:
                self._vmm["weights"].map()
                self.weight_flat.copy_(self._host_weights)
                self._host_weights = None
            if "kv_cache" in tags and not self._vmm["kv_cache"].mapped:
                self._alloc_kv()

    def _check_resident(self, tags=("weights", "kv_cache")) -> None:
        """Touching a released region would fault the GPU: refuse on the host instead."""
        for t in tags:
            r = getattr(self, "_vmm", {}).get(t)
            if r is not None and not r.mapped:
                raise RuntimeError(f"{t} memory is released; call resume_memory([{t!r}]) first")

    @property
    def memory_released(self) -> dict:
        return {k: not r.mapped for k, r in getattr(self, "_vmm", {}).items()}

    def _rebind_weights(self):
        for s, p in zip(self.weight_slots, self.model.parameters()):
            p.data = self.weight_flat[s.offset:s.offset + s.numel].view(s.shape)

    # ------------------------------------------------------------------ weights
    def update_weights_from_flat(self, src: torch.Tensor, version: int | None = None) -> None:
        """Device weight sync: ``src`` is a flat buffer in the trainer's layout (with tensor parallelism the
        full model's; this rank takes its slices)."""
        with self.lock:
            self._check_resident(("weights",))
            if self.full_slots is not None:
                self._load_full(lambda s: src[s.offset:s.offset + s.numel].view(s.shape))
                self.weight_version = self.weight_version + 1 if version is None else int(version)
                return
            if src.numel() != self.weight_flat.numel():
                raise ValueError("flat weight layout mismatch")
            if src.dtype == self.weight_flat.dtype:
                self.weight_flat.copy_(src, non_blocking=True)
            elif src.is_cuda and Fx.native(src):
                from ..ops._ext import ext

                ext().cast_copy(src, self.weight_flat)
            else:
                self.weight_flat.copy_(src)
            self.weight_version = self.weight_version + 1 if version is None else int(version)

    def update_weights_from_state_dict(self, sd: dict[str, torch.Tensor], version: int | None = None) -> None:
        with self.lock:
            self._check_resident(("weights",))
            if self.full_slots is not None:
                self._load_full(lambda s: sd[s.name].reshape(s.shape))
            else:
                with torch.no_grad():
                    for s in self.weight_slots:
                        self.weight_flat[s.offset:s.offset + s.numel].copy_(sd[s.name].reshape(-1))
            self.weight_version = self.weight_version + 1 if version is None else int(version)

    @torch.no_grad()
    def _load_full(self, full_of) -> None:
        """Tensor parallelism: every local parameter from its full tensor (``full_of(full_slot)``), sliced for
        this rank -- the replica -> tensor-parallel reshard of a weight sync."""
        from ..parallel.tp import tp_shard_param

        local = {s.name: s for s in self.weight_slots}
        for fs in self.full_slots:
            ls = local[fs.name]
            full = full_of(fs).to(self.weight_flat.device)  # sources may sit on the CPU or another device
            part = tp_shard_param(fs.name, full, self.args, self.tp, self.tp_rank, ep=self.ep)
            self.weight_flat[ls.offset:ls.offset + ls.numel].view(ls.shape).copy_(part)

    def update_weights_from_ipc(self, handles: dict, version: int | None = None) -> bool:
        """``handles``: ``{gpu_uuid: handle}`` of the trainer ranks' published bf16 snapshots; this engine maps the
        one exported on its own GPU (else a visible peer's). Returns whether the handle was local."""
        from .weight_sync import device_uuid, open_ipc_flat, pick_handle

        handle, local, uuid = pick_handle(handles, device_uuid(self.device))
        src = open_ipc_flat(handle, uuid)
        self.update_weights_from_flat(src, version)
        if self.cuda:
            torch.cuda.synchronize(self.device)
        del src
        return local

    def update_weights_from_disk(self, path: str, version: int | None = None) -> None:
        from ..models.hf import load_hf_checkpoint

        self.update_weights_from_state_dict(load_hf_checkpoint(self.args, path), version)

    # ------------------------------------------------------------------ requests
    def submit(self, prompt: Sequence[int], max_new_tokens: int, *, rid=None, temperature=1.0, top_k=-1,
               top_p=1.0, ignore_eos=False) -> Any:
        rid = next(self._rid) if rid is None else rid
        if len(prompt) + max_new_tokens > self.max_seq_len:
            max_new_tokens = max(1, self.max_seq_len - len(prompt))
        req = Request(rid, list(map(int, prompt)), int(max_new_tokens), float(temperature), int(top_k),
                      float(top_p), bool(ignore_eos), submitted=time.time())
        with self.lock:
            self.waiting.append(req)
        return rid

    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int | Sequence[int], *,
                 temperature: float = 1.0, top_k: int = -1, top_p: float = 1.0,
                 ignore_eos: bool = False) -> list[Generation]:
        """Blocking batch generation (the lock-step rollout's call)."""
        if isinstance(max_new_tokens, int):
            max_new_tokens = [max_new_tokens] * len(prompts)
        rids = [self.submit(p, m, temperature=temperature, top_k=top_k, top_p=top_p, ignore_eos=ignore_eos)
                for p, m in zip(prompts, max_new_tokens)]
        self.run_until_idle()
        return [self.finished.pop(r) for r in rids]

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def run_until_idle(self) -> None:
        while self.has_work() and not self.paused:
            self.step()

    @property
    def n_running(self) -> int:
        return len(self.running)

    def loads(self) -> dict[str, int]:
        return {"num_running_reqs": len(self.running), "num_waiting_reqs": len(self.waiting),
                "num_free_pages": self.blocks.num_free}

    # ------------------------------------------------------------------ control
    def pause(self) -> None:
        self.paused = True

    def resume(self) -> None:
        self.paused = False

    def abort_all(self) -> list[Generation]:
        """Finish every running/waiting request now with ``finish_reason='abort'``."""
        with self.lock:
            out = []
            if self.running:
                self._collect(list(range(len(self.running))), reason="abort")
            for req in self.waiting:
                g = Generation(req.rid, req.prompt, [], [], "abort", self.weight_version)
                self.finished[req.rid] = g
            self.waiting.clear()
            for g in self.finished.values():
                if g.finish_reason == "abort":
                    out.append(g)
            return out

    # ------------------------------------------------------------------ scheduling
    def step(self) -> None:
        with self.lock:
            if self.waiting or self.running:
                self._check_resident()
            self._admit()
            if not self.running:
                return
            n = len(self.running)
            self._ensure_pages(range(n), self.sync_every + 1)
            steps = self.sync_every
            for _ in range(steps):
                self._decode_step(n)
            self._sync_finished()

    def _admit(self) -> None:
        if not self.waiting:
            return
        budget = self.prefill_chunk_tokens
        batch: list[Request] = []
        while self.waiting and len(self.running) + len(batch) < self.max_running:
            req = self.waiting[0]
            need = len(req.prompt) + min(req.max_new_tokens, self.sync_every * 2) + 1
            if batch and sum(len(r.prompt) for r in batch) + len(req.prompt) > budget:
                break
            pages = self.blocks.allocate(math.ceil(need / self.page_size))
            if pages is None:
                break
            req.pages = pages
            req.out_slot = self.free_out_slots.pop()
            batch.append(self.waiting.pop(0))
        if batch:
            self._prefill(batch)

    def _ensure_pages(self, rows: Sequence[int], lookahead: int) -> None:
        """Grow page lists so every row can decode ``lookahead`` more tokens."""
        st = self.st
        seq = st["seq_lens"][: len(self.running)].tolist()
        bt_updates = []
        for i in rows:
            req = self.running[i]
            need_tokens = min(seq[i] + lookahead, len(req.prompt) + req.max_new_tokens)
            need = math.ceil(need_tokens / self.page_size)
            if need > len(req.pages):
                new = self.blocks.allocate(need - len(req.pages))
                if new is None:
                    raise RuntimeError("KV cache exhausted; lower max_running or raise max_total_tokens")
                start = len(req.pages)
                req.pages.extend(new)
                bt_updates.append((i, start, new))
        for i, start, new in bt_updates:
            st["block_table"][i, start:start + len(new)] = torch.tensor(new, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def _prefill(self, batch: list[Request]) -> None:
        a, dev, P = self.args, self.device, self.page_size
        lens = [len(r.prompt) for r in batch]
        T = sum(lens)
        toks = torch.tensor([t for r in batch for t in r.prompt], dtype=torch.int64)
        pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens])
        slots = torch.cat([
            torch.tensor(r.pages, dtype=torch.int64).repeat_interleave(P)[:L] * P + torch.arange(L) % P
            for r, L in zip(batch, lens)])
        cu = torch.tensor([0] + list(itertools.accumulate(lens)), dtype=torch.int32)
        toks, pos, slots, cu = (t.to(dev, non_blocking=True) for t in (toks, pos, slots, cu))
        m = self.model
        la = self.local_args
        x = Fx.embedding(toks, m.embed)
        for li, layer in enumerate(m.layers):
            h = Fx.rmsnorm(x, layer.attn_norm, a.norm_eps)
            qkv = Fx.linear(h, layer.wqkv, layer.bqkv)
            q, k, v = D.qkv_rope_to_cache(qkv, pos, layer.q_norm, layer.k_norm, la.n_heads, la.n_kv_heads,
                                          a.head_dim, a.rope_theta, a.norm_eps, self.kv[li, 0], self.kv[li, 1], slots,
                                          keep_kv=True)
            o = Fx.flash_attn_varlen(q, k, v, cu, max(lens))
            x = self._row_parallel(o.reshape(T, la.q_dim), layer.wo, x)
            h = Fx.rmsnorm(x, layer.mlp_norm, a.norm_eps)
            x = self._mlp(layer, h, x)
        last = (cu[1:] - 1).long()
        hl = Fx.rmsnorm(x[last], m.norm, a.norm_eps)
        tok, lp = self._sample_rows(hl, batch)
        self.stats["prefill_tokens"] += T
        # append rows
        st = self.st
        base = len(self.running)
        n = len(batch)
        rows = slice(base, base + n)
        max_new = torch.tensor([r.max_new_tokens for r in batch], dtype=torch.int32)
        req_slots = torch.tensor([r.out_slot for r in batch], dtype=torch.int32)
        plen = torch.tensor(lens, dtype=torch.int32)
        st["req"][rows] = req_slots.to(dev)
        st["max_new"][rows] = max_new.to(dev)
        st["gen"][rows] = 1
        st["tok_in"][rows] = tok
        st["pos"][rows] = plen.to(dev)
        st["seq_lens"][rows] = (plen + 1).to(dev)
        rs = req_slots.to(dev).long()
        st["out_tok"][rs, 0] = tok
        st["out_lp"][rs, 0] = lp
        done = max_new <= 1
        ignore = torch.tensor([r.ignore_eos for r in batch])
        if self.eos:
            hit = torch.isin(tok.cpu(), torch.tensor(self.eos)) & ~ignore
            done = done | hit
        st["done"][rows] = done.to(torch.int32).to(dev)
        bt = torch.zeros(n, self.max_pages_per_seq, dtype=torch.int32)
        for j, r in enumerate(batch):
            bt[j, : len(r.pages)] = torch.tensor(r.pages, dtype=torch.int32)
        st["block_table"][rows] = bt.to(dev)
        pg = torch.tensor([r.pages[L // P] for r, L in zip(batch, lens)], dtype=torch.int64)
        st["slot"][rows] = (pg * P + plen.long() % P).to(dev)
        self.running.extend(batch)

    def _mlp(self, layer, h, x):
        a = self.args
        if layer.moe is None:
            return self._row_parallel(Fx.linear_swiglu(h, layer.w13, a.swiglu_block), layer.w2, x)
        return x + layer.moe(h)

    def _row_parallel(self, h, w, residual):
        """``residual + h @ w.T``; with tensor parallelism ``w`` holds this rank's input columns, and the
        partial products are summed over the TP group in fp32 before the residual is added once."""
        if self.tp_group is None:
            return Fx.linear(h, w, residual=residual)
        import torch.distributed as dist

        if Fx.native(h):
            from ..ops._ext import ext

            y = torch.empty(h.shape[0], w.shape[0], dtype=torch.float32, device=h.device)
            ext().gemm(h, w, y, False, False, None, None, None, Fx.EPI_NONE, False, 0)
        else:
            y = torch.nn.functional.linear(h.float(), w.float())
        dist.all_reduce(y, group=self.tp_group)
        return (residual.float() + y).to(residual.dtype)

    def _sample_rows(self, h, reqs: Sequence[Request]):
        r0 = reqs[0]
        uniform = all(r.temperature == r0.temperature and r.top_k == r0.top_k and r.top_p == r0.top_p
                      for r in reqs)
        w = self.model.output_weight
        if uniform:
            return D.sample(h, w, r0.temperature, top_k=r0.top_k, top_p=r0.top_p, seed=self.seed,
                            step=self.st["step"], generator=self._gen if not self.cuda else None)
        toks, lps = [], []
        for i, r in enumerate(reqs):
            t, l = D.sample(h[i:i + 1], w, r.temperature, top_k=r.top_k, top_p=r.top_p, seed=self.seed,
                            step=self.st["step"], generator=self._gen if not self.cuda else None)
            toks.append(t)
            lps.append(l)
        return torch.cat(toks), torch.cat(lps)

    # ------------------------------------------------------------------ decode
    @torch.no_grad()
    def _decode_hidden(self, b: int, final_split: bool = False):
        """Final normed hidden states ``[b, D]`` of the running rows' next position (writes their K/V).

        Up to 64 rows of an eligible dense model take the whole-step persistent kernel; otherwise one
        kernel per op. ``final_split``: the per-op path may instead return ``(xg, part)``, the final
        RMSNorm's prepared input (see :meth:`_decode_hidden_layers`)."""
        if self._mega is not None and b <= self._mega_rows:
            return self._mega(self.st, b)
        return self._decode_hidden_layers(b, final_split=final_split)

    def _norm_ws(self):
        """Buffers of the split RMSNorm (bf16 g * x and per-tile sums of squares for two norms)."""
        if getattr(self, "_nws", None) is None:
            a = self.args
            tiles = (a.dim + 127) // 128
            self._nws = (torch.empty(self.max_running, a.dim, dtype=self.dtype, device=self.device),
                         torch.zeros(2, tiles, 256, dtype=torch.float32, device=self.device))
        return self._nws

    @torch.no_grad()
    def _decode_hidden_layers(self, b: int, final_split: bool = False):
        """Per-op decode of all layers. With ``final_split`` the last down_proj prepares the final
        RMSNorm like the others (``bf16(g * x)`` and per-tile sums of squares) and, when it could, the
        result is ``(xg [b, D], part)`` for a consumer that applies ``rstd`` itself (the LM-head
        sampler) instead of the normed hidden states."""
        a, m, st = self.args, self.model, self.st
        la = self.local_args
        x = Fx.embedding(st["tok_in"][:b], m.embed)
        pos = st["pos"][:b]
        # RMSNorm split across GEMMs: the residual GEMM producing x writes bf16(g_next * x) and per-tile
        # sums of squares, the consuming GEMM scales its rows by rstd (no normalisation kernels).
        # ``prep`` is the part buffer the next norm can use (None: run the unfused norm).
        # (the split norm needs the whole row-parallel output in one epilogue: off under tensor parallelism)
        split = self.cuda and os.environ.get("MESHY_SPLIT_NORM", "1") != "0" and self.tp_group is None
        fuse_rope = os.environ.get("MESHY_FUSED_QKV_ROPE", "1") != "0"
        xg, parts = self._norm_ws() if split else (None, None)
        prep = None
        L = len(m.layers)
        for li, layer in enumerate(m.layers):
            q = None
            if prep is not None and fuse_rope:
                q = D.qkv_rope_fused(xg[:b], layer.wqkv, layer.bqkv, pos, layer.q_norm, layer.k_norm, a.n_heads,
                                     a.n_kv_heads, a.rope_theta, a.norm_eps, self.kv[li, 0], self.kv[li, 1],
                                     st["slot"][:b], part=prep, d=a.dim)
            if q is None:
                qkv = None
                if prep is not None:
                    qkv = D.linear_norm_scaled(xg[:b], layer.wqkv, layer.bqkv, prep, a.dim, a.norm_eps)
                if qkv is None:
                    qkv = Fx.rmsnorm_linear(x, layer.attn_norm, a.norm_eps, layer.wqkv, layer.bqkv)
                q, _, _ = D.qkv_rope_to_cache(qkv, pos, layer.q_norm, layer.k_norm, la.n_heads, la.n_kv_heads,
                                              a.head_dim, a.rope_theta, a.norm_eps, self.kv[li, 0], self.kv[li, 1],
                                              st["slot"][:b])
            o = D.paged_attention(q, self.kv[li, 0], self.kv[li, 1], st["block_table"][:b], st["seq_lens"][:b],
                                  decode_step=True)
            o = o.reshape(b, la.q_dim)
            prep = None
            if layer.moe is None and split:
                xn = D.linear_norm_prep(o, layer.wo, x, layer.mlp_norm, xg, parts[1])
                if xn is not None:
                    x, prep = xn, parts[1]
            if prep is None:
                x = self._row_parallel(o, layer.wo, x)
            if layer.moe is None:
                act = None
                if prep is not None:
                    act = D.linear_norm_scaled(xg[:b], layer.w13, None, prep, a.dim, a.norm_eps,
                                               swiglu_block=a.swiglu_block)
                if act is None:
                    act = Fx.rmsnorm_linear(x, layer.mlp_norm, a.norm_eps, layer.w13, swiglu_block=a.swiglu_block)
                prep = None
                if split and (li + 1 < L or final_split):
                    g_next = m.layers[li + 1].attn_norm if li + 1 < L else m.norm
                    xn = D.linear_norm_prep(act, layer.w2, x, g_next, xg, parts[0])
                    if xn is not None:
                        x, prep = xn, parts[0]
                if prep is None:
                    x = self._row_parallel(act, layer.w2, x)
            else:
                prep = None
                x = self._mlp(layer, Fx.rmsnorm(x, layer.mlp_norm, a.norm_eps), x)
        if final_split and prep is not None:
            return xg[:b], prep
        return Fx.rmsnorm(x, m.norm, a.norm_eps)

    @torch.no_grad()
    def _decode_body(self, b: int, eos: torch.Tensor):
        m, st, a = self.model, self.st, self.args
        r0 = self.running[0]
        sub = {k: (v[:b] if k not in ("out_tok", "out_lp", "eos", "noeos", "step") else v) for k, v in st.items()}
        sub["eos"] = eos
        # temperature-only sampling of <= 64 rows: LM head + sampler, then merge + row advance (2 kernels)
        fused = (self.cuda and b <= 64 and r0.temperature > 0 and r0.top_k <= 0 and r0.top_p >= 1.0
                 and os.environ.get("MESHY_FUSED_SAMPLER", "1") != "0")
        h = self._decode_hidden(b, final_split=fused)
        part = None
        if isinstance(h, tuple):
            h, part = h
        if fused and D.sample_advance(sub, h, m.output_weight, r0.temperature, seed=self.seed,
                                      page_size=self.page_size, part=part, d=a.dim, eps=a.norm_eps):
            return
        if part is not None:  # undo the split: h = RMSNorm(x) from bf16(g * x) and the row sums of squares
            rstd = torch.rsqrt(part.sum(0)[:b] / a.dim + a.norm_eps)
            h = (h.float() * rstd[:, None]).to(h.dtype)
        tok, lp = D.sample(h, m.output_weight, r0.temperature, top_k=r0.top_k, top_p=r0.top_p, seed=self.seed,
                           step=st["step"], generator=self._gen if not self.cuda else None)
        D.decode_advance(sub, tok, lp, self.page_size)
        st["step"] += 1

    def _decode_step(self, n: int) -> None:
        eos = self.st["eos"] if not all(r.ignore_eos for r in self.running) else self.st["noeos"]
        if not self.use_cuda_graph:
            self._decode_body(n, eos)
        else:
            b = min(_bucket(n), self.max_running)
            key = (b, eos.numel() > 0, self._sampling_key())
            g = self._graphs.get(key)
            if g is None:
                g = self._capture(b, eos)
                self._graphs[key] = g
            g.replay()
            self.stats["graph_replays"] += 1
            self.stats["graph_kernels"] = self.stats.get("graph_kernels", 0) + getattr(g, "n_kernels", 0)
        self.stats["decode_steps"] += 1
        self.stats["decode_tokens"] += n

    def _sampling_key(self):
        r = self.running[0]
        return (r.temperature, r.top_k, r.top_p)

    def _capture(self, b: int, eos: torch.Tensor):
        # rows beyond len(running) are padding: mark them done so advance skips them
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up (allocator, tensor maps)
                saved = {k: v.clone() for k, v in self.st.items()}
                self._decode_body(b, eos)
                for k, v in saved.items():
                    self.st[k].copy_(v)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        saved = {k: v.clone() for k, v in self.st.items()}
        from ..ops._ext import ext

        n0 = ext().launch_count()
        with torch.cuda.graph(g, stream=s):
            self._decode_body(b, eos)
        g.n_kernels = ext().launch_count() - n0
        for k, v in saved.items():
            self.st[k].copy_(v)
        return g

    # ------------------------------------------------------------------ finish
    def _sync_finished(self) -> None:
        n = len(self.running)
        if n == 0:
            return
        if self._mega is not None:
            # the whole-step kernel reports a timed-out wait through the device error word (this is a
            # host sync, like the finish-flag read below)
            from ..ops._ext import ext

            err = int(ext().device_error())
            if err:
                ext().clear_device_error()
                self._mega.reset()
                raise RuntimeError(f"decode kernel reported device error {err} (a bounded wait timed out)")
        done = self.st["done"][:n].tolist()
        rows = [i for i, d in enumerate(done) if d]
        if rows:
            self._collect(rows)

    def _collect(self, rows: list[int], reason: str | None = None) -> None:
        st, n = self.st, len(self.running)
        gen = st["gen"][:n].tolist()
        max_gen = max(gen[i] for i in rows) if rows else 0
        slots = torch.tensor([self.running[i].out_slot for i in rows], dtype=torch.long, device=self.device)
        toks = st["out_tok"].index_select(0, slots)[:, :max_gen].cpu().tolist()
        lps = st["out_lp"].index_select(0, slots)[:, :max_gen].cpu().tolist()
        for j, i in enumerate(rows):
            req = self.running[i]
            g = gen[i]
            out = toks[j][:g]
            fr = reason
            if fr is None:
                fr = "stop" if (not req.ignore_eos and out and out[-1] in self.eos) else "length"
            self.finished[req.rid] = Generation(req.rid, req.prompt, out, lps[j][:g], fr, self.weight_version)
            self.blocks.free(req.pages)
            self.free_out_slots.append(req.out_slot)
        keep = [i for i in range(n) if i not in set(rows)]
        if keep != list(range(len(keep))):
            idx = torch.tensor(keep, dtype=torch.long, device=self.device)
            for k in ("tok_in", "pos", "seq_lens", "gen", "max_new", "done", "slot", "block_table", "req"):
                st[k][: len(keep)] = st[k].index_select(0, idx)
        self._park_rows(len(keep))
        self.running = [self.running[i] for i in keep]

    def _park_rows(self, start: int) -> None:
        """Rows ``>= start`` are idle: done, and their KV write goes to trash page 0."""
        st = self.st
        st["done"][start:] = 1
        st["slot"][start:] = 0
        st["block_table"][start:] = 0
        st["seq_lens"][start:] = 1
        st["pos"][start:] = 0


__all__ = ["Generation", "Request", "RolloutEngine"]
