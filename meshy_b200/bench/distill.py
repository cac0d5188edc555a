"""Top-K on-policy distillation heads at the OPD recipe's shapes: the teacher's top-K over the vocabulary
(Qwen3-8B, width 4096) and the student's log-probabilities of those K ids, forward + backward (Qwen3-1.7B,
width 2048; vocabulary 151,936; K = 8), native kernels against the PyTorch path of the same functions
(``meshy_b200.backend.topk_loss`` under ``torch_baseline``: chunked GEMMs, ``torch.topk`` and ``logsumexp``,
non-reentrant checkpointing of the student's chunks).

Each timed call is preceded by an L2 flush; the LM-head weights (1.2 / 0.6 GB in bf16) exceed L2.

    python -m meshy_b200.bench.distill --tokens 16384
"""

from __future__ import annotations

import argparse
import json

import torch


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=16384)
    p.add_argument("--teacher-dim", type=int, default=4096)
    p.add_argument("--student-dim", type=int, default=2048)
    p.add_argument("--vocab", type=int, default=151936)
    p.add_argument("--k", type=int, default=8)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--device", default="cuda")
    a = p.parse_args(argv)
    from ..backend.topk_loss import gather_logprobs, teacher_topk
    from ..ops import functional as Fx
    from .ops import peaks

    dev = torch.device(a.device)
    cuda = dev.type == "cuda"
    dt = torch.bfloat16 if cuda else torch.float32
    torch.manual_seed(0)
    T, V = a.tokens, a.vocab
    ht = torch.randn(T, a.teacher_dim, device=dev).to(dt)
    wt = (torch.randn(V, a.teacher_dim, device=dev) * 0.02).to(dt)
    hs = torch.randn(T, a.student_dim, device=dev).to(dt).requires_grad_(True)
    ws = (torch.randn(V, a.student_dim, device=dev) * 0.02).to(dt).requires_grad_(True)
    g = torch.randn(T, a.k, device=dev) * 1e-2
    if cuda:  # the trainer's LM-head gradient accumulates into its fp32 flat buffer (native path)
        ws.main_grad = torch.zeros(ws.shape, dtype=torch.float32, device=dev)
    _, peak_tf, src = peaks()
    fl_teacher = 2 * T * V * a.teacher_dim
    fl_student = 3 * 2 * T * V * a.student_dim  # forward GEMM + dgrad + wgrad (the torch path adds a recompute)

    def timed(fn):
        if cuda:
            from .ops import time_op

            return time_op(fn, a.iters, a.warmup)
        import time

        t0 = time.perf_counter()
        fn()
        return (time.perf_counter() - t0) * 1e6

    ids = teacher_topk(ht, wt, a.k)[0]  # the student gathers the same ids in both arms
    res = {}
    for impl in ("native", "torch"):
        with Fx.torch_baseline(impl == "torch"):
            def teach():
                return teacher_topk(ht, wt, a.k)

            def student():
                hs.grad = ws.grad = None
                gather_logprobs(hs, ws, ids).backward(g)

            t_ids, t_lps = teach()
            t_t = timed(teach)
            t_s = timed(student)
            res[impl] = (t_ids, t_lps, gather_logprobs(hs, ws, ids).detach())
        rec = {"bench": "topk_distill", "impl": impl, "tokens": T, "vocab": V, "k": a.k,
               "teacher_topk_us": round(t_t, 1), "teacher_tflops": round(fl_teacher / t_t / 1e6, 1),
               "student_fwd_bwd_us": round(t_s, 1), "student_tflops": round(fl_student / t_s / 1e6, 1)}
        if cuda:
            rec[f"student_frac_of_{src}_bf16_peak"] = round(fl_student / t_s / 1e6 / peak_tf, 3)
        print(json.dumps(rec), flush=True)
    # the PyTorch arm selects from bf16-rounded logits (its GEMM's output type), the native one from fp32
    # logits: near-ties can pick different ids, so the selected values are compared (sorted, tie-insensitive)
    (i0, l0, s0), (i1, l1, s1) = res["native"], res["torch"]
    print(json.dumps({"bench": "topk_distill", "teacher_ids_equal": float((i0 == i1).float().mean()),
                      "teacher_lp_max_abs_diff": float((l0 - l1).abs().max()),
                      "student_lp_max_abs_diff": float((s0 - s1).abs().max())}), flush=True)


if __name__ == "__main__":
    main()
