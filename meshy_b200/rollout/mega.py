"""Whole-step decode through one persistent kernel (``csrc/kernels/decode_mega.cu``).

:class:`MegaDecoder` owns the kernel's workspaces and its per-layer pointer
table for one rollout engine. Calling it runs embedding, every decoder layer
(RMSNorm, QKV, RoPE + KV-cache write, paged attention, o_proj + residual,
RMSNorm, gate/up + SwiGLU, down + residual) and the final RMSNorm for the
first ``b`` running rows in one cooperative launch, and returns the normed
hidden states ``[b, D]`` for the LM-head sampler.

Opt-in (``MESHY_MEGA=1``): on R1-Distill-1.5B it is correct (matches the
per-op path to bf16 accuracy) but still slower than the per-op kernels with
programmatic dependent launch (B200, context 2048: 2.5 ms vs 1.9 ms per step at
1 row, 6.0 ms vs 2.9 ms at 64 rows); its per-phase timeline
(``enable_trace``) shows grid barriers at ~1.4 us but slow phase epilogues.

Eligibility (:meth:`MegaDecoder.reason`): dense blocks (no MoE), head_dim 128,
64-token pages, a GQA group of at most 16 query heads per KV head and at most
8 KV heads, SwiGLU gate/up blocks of 64 rows, at most 64 rows per step, and
per-layer matrices at a uniform stride in the engine's flat weight buffer (the
kernel addresses layer ``l``'s weights as one 3-D TMA tensor).
"""

from __future__ import annotations

import math
import os

import torch

MAX_ROWS = 64


def _split(T: int, KB: int, n: int) -> int:
    """Split-K factor for ``T`` tiles x ``KB`` k-blocks over ``n`` CTAs: the fewest k-blocks on the
    busiest CTA, ties to the smaller split (fewer partial sums). Items longer than 12 k-blocks are
    penalised: one CTA streams one item through a 5-stage ring at well under its share of HBM
    bandwidth (measured: an unsplit 24-block gate/up item took 4x longer than two 12-block ones)."""
    best, best_cost = 1, None
    for s in range(1, min(KB, 32) + 1):
        per = math.ceil(KB / s)
        # every item also pays a fixed epilogue (TMEM drain, partial-sum atomics, tile counter) worth
        # about three k-blocks of streaming
        cost = math.ceil(T * s / n) * (per + 3) + 3 * max(0, per - 12)
        if best_cost is None or cost < best_cost:
            best, best_cost = s, cost
    return best


class MegaDecoder:
    @staticmethod
    def reason(model, page_size: int) -> str | None:
        """Why this model cannot use the whole-step kernel (``None``: it can)."""
        a = model.args
        if os.environ.get("MESHY_MEGA", "0") != "1":
            return "not enabled (MESHY_MEGA=1 turns it on)"
        if any(getattr(blk, "moe", None) is not None for blk in model.layers):
            return "MoE layers"
        if a.head_dim != 128 or page_size != 64:
            return "head_dim 128 and 64-token pages only"
        if a.n_heads % a.n_kv_heads or a.n_heads // a.n_kv_heads > 16 or a.n_kv_heads > 8:
            return "GQA group > 16 or more than 8 KV heads"
        if a.swiglu_block != 64 or a.dim % 128 or a.ffn_dim % 64:
            return "dims do not tile"
        if getattr(model.layers[0], "tp_group", None) is not None:
            return "tensor-parallel blocks"
        names = ("wqkv", "wo", "w13", "w2")
        if len(model.layers) > 1:
            stride = model.layers[1].wqkv.data_ptr() - model.layers[0].wqkv.data_ptr()
            for nm in names:
                ptrs = [getattr(blk, nm).data_ptr() for blk in model.layers]
                if any(q - p != stride for p, q in zip(ptrs, ptrs[1:])):
                    return f"layer weights ({nm}) not at a uniform stride"
        return None

    def __init__(self, model, kv: torch.Tensor, device):
        from ..ops._ext import ext

        self.C = ext()
        self.model = model
        self.kv = kv
        a = model.args
        dev = torch.device(device)
        L = len(model.layers)
        esz = model.layers[0].wqkv.element_size()
        self.layer_stride = ((model.layers[1].wqkv.data_ptr() - model.layers[0].wqkv.data_ptr()) // esz
                             if L > 1 else 0)
        rows = []
        for blk in model.layers:
            def p(t):
                return 0 if t is None else t.data_ptr()
            rows.append([p(blk.attn_norm), p(blk.bqkv), p(blk.q_norm), p(blk.k_norm), p(blk.mlp_norm), 0, 0, 0])
        self.table = torch.tensor(rows, dtype=torch.int64, device=dev)
        self.grid = int(self.C.mega_grid())
        D, F, Hq, Hkv, hd = a.dim, a.ffn_dim, a.n_heads, a.n_kv_heads, a.head_dim
        qkv_dim, q_dim = (Hq + 2 * Hkv) * hd, Hq * hd
        R = MAX_ROWS
        f32, bf = torch.float32, torch.bfloat16
        self.ws = [
            torch.zeros(D * R, dtype=f32, device=dev),                      # x  [D][MP]
            torch.zeros(R, D, dtype=bf, device=dev),                        # xg [MP][D]
            torch.zeros(2 * R, dtype=f32, device=dev),                      # sumsq
            torch.zeros(max(qkv_dim, 2 * F) * R, dtype=f32, device=dev),    # split-K accumulator
            torch.zeros(R * Hq * hd, dtype=bf, device=dev),                 # q
            torch.zeros(int(self.C.mega_apart_floats(self.grid)), dtype=f32, device=dev),
            torch.zeros(R, q_dim, dtype=bf, device=dev),                    # attention output
            torch.zeros(R, F, dtype=bf, device=dev),                        # SwiGLU output
            torch.zeros(R, D, dtype=bf, device=dev),                        # final hidden
            torch.zeros(int(self.C.mega_ctr_words()), dtype=torch.int32, device=dev),
        ]
        n = self.grid
        self.gemm = []
        shapes = ((qkv_dim // 128, D // 64), (D // 128, q_dim // 64), (2 * F // 128, D // 64), (D // 128, F // 64))
        force = os.environ.get("MESHY_MEGA_SPLITS")  # "s_qkv,s_o,s_gu,s_dn" (0 = automatic)
        forced = [int(v) for v in force.split(",")] if force else [0, 0, 0, 0]
        for (T, KB), fs in zip(shapes, forced):
            self.gemm += [T, KB, min(fs, KB) if fs > 0 else _split(T, KB, n)]
        self.scale = 1.0 / math.sqrt(hd)
        #: optional int64 [phases, grid, 8] timeline (global-timer ns: phase start / end per CTA and markers)
        self.trace: torch.Tensor | None = None

    def enable_trace(self) -> torch.Tensor:
        L = len(self.model.layers)
        self.trace = torch.zeros(2 + 5 * L, self.grid, 8, dtype=torch.int64, device=self.table.device)
        return self.trace

    def reset(self) -> None:
        """Clear the counters and accumulators after a step that reported an error."""
        for i in (3, 9):
            self.ws[i].zero_()

    def __call__(self, st: dict, b: int) -> torch.Tensor:
        m, a = self.model, self.model.args
        if not 1 <= b <= MAX_ROWS:
            raise ValueError(f"mega decode takes 1..{MAX_ROWS} rows, got {b}")
        mp = 16 if b <= 16 else (32 if b <= 32 else 64)
        l0 = m.layers[0]
        self.C.mega_decode(self.table, l0.wqkv, l0.wo, l0.w13, l0.w2, int(self.layer_stride), m.embed, m.norm, self.kv,
                           st["tok_in"], st["pos"], st["seq_lens"], st["slot"], st["block_table"], self.ws, b, mp,
                           a.n_heads, a.n_kv_heads, float(a.norm_eps), float(self.scale), float(a.rope_theta),
                           self.gemm, self.grid, self.trace)
        return self.ws[8][:b]


__all__ = ["MAX_ROWS", "MegaDecoder"]
