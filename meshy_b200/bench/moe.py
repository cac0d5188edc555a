"""One MoE layer of Qwen3-30B-A3B (128 experts, top-8, expert width 768, model width 2048): forward and
forward + backward, native kernels against the PyTorch path the reference's trainer takes.

* ``native``: router softmax + top-k kernel, device-side plan and gather, grouped tcgen05 GEMMs (gate/up with
  the SwiGLU epilogue, down), weighted combine; backward through the same kernels (``meshy_b200.ops.moe``),
  the expert weight gradients accumulated into fp32 buffers as the trainer's flat gradient holds them.
* ``torch``: torchtitan's formulation (``TT:torchtitan/models/common/moe.py``): softmax / ``topk`` routing,
  ``argsort`` of the assignments, ``torch._grouped_mm`` over per-expert offsets (no host synchronisation),
  SwiGLU in PyTorch, ``index_add`` combine, autograd for the backward (bf16 weight gradients).

Each timed call is preceded by an L2 flush; the expert weights (1.2 GB in bf16) are larger than L2 anyway.
FLOPs per token: top-k x (2 x D x 2F + 2 x F x D) forward (the router adds 2 x D x E), three times that for
forward + backward.

    python -m meshy_b200.bench.moe --tokens 16384
"""

from __future__ import annotations

import argparse
import json

import torch


def _torch_moe(x, router, w13, w2, top_k: int, norm: bool, block: int):
    from ..ops import reference as ref

    T, D = x.shape
    E = w13.shape[0]
    scores = torch.softmax((x @ router.t()).float(), dim=-1)
    w, e = torch.topk(scores, top_k, dim=-1)
    if norm:
        w = w / w.sum(-1, keepdim=True).clamp(min=1e-20)
    flat_e = e.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    tok = torch.arange(T, device=x.device).repeat_interleave(top_k)[order]
    offs = torch.cumsum(torch.bincount(flat_e, minlength=E), 0).to(torch.int32)
    xs = x[tok]
    h = torch._grouped_mm(xs, w13.transpose(1, 2), offs=offs)
    a = ref.swiglu(h, block)
    y = torch._grouped_mm(a, w2.transpose(1, 2), offs=offs)
    y = y * w.reshape(-1)[order].unsqueeze(-1).to(y.dtype)
    return torch.zeros_like(x).index_add(0, tok, y)


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=16384)
    p.add_argument("--model", default="qwen3:30B-A3B")
    p.add_argument("--impl", nargs="*", default=["native", "torch"])
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--device", default="cuda")
    a = p.parse_args(argv)
    from ..models import get_model_args
    from ..models.moe import MoE
    from .ops import peaks

    name, flavor = a.model.split(":")
    args = get_model_args(name, flavor)
    m = args.moe
    dev = torch.device(a.device)
    cuda = dev.type == "cuda"
    dtype = torch.bfloat16 if cuda else torch.float32
    torch.manual_seed(0)
    layer = MoE(args).to(dev)
    layer.reset_parameters(0.02, 0.02)
    layer = layer.to(dtype)
    if cuda:  # the trainer's expert weight gradients accumulate into its fp32 flat buffer
        for w in (layer.w13, layer.w2):
            w.main_grad = torch.zeros(w.shape, dtype=torch.float32, device=dev)
    x = (torch.randn(a.tokens, args.dim, device=dev) * 0.5).to(dtype).requires_grad_(True)
    dy = torch.randn(a.tokens, args.dim, device=dev).to(dtype) * 1e-2
    _, peak_tf, src = peaks()
    flops_fwd = a.tokens * m.top_k * 6 * args.dim * m.expert_ffn_dim + 2 * a.tokens * args.dim * m.n_experts

    def run(impl):
        if impl == "native":
            return layer(x)
        return _torch_moe(x, layer.router, layer.w13, layer.w2, m.top_k, m.route_norm, args.swiglu_block)

    outs = {}
    for impl in a.impl:
        def fwd():
            with torch.no_grad():
                run(impl)

        def fwd_bwd():
            x.grad = None
            for prm in layer.parameters():
                prm.grad = None
            run(impl).backward(dy)

        if cuda:
            from .ops import time_op

            try:
                t_f = time_op(fwd, a.iters, a.warmup)
                t_fb = time_op(fwd_bwd, a.iters, a.warmup)
            except RuntimeError as e:  # e.g. a grouped GEMM this PyTorch build lacks for the device
                print(json.dumps({"bench": "moe_layer", "impl": impl, "unavailable": str(e).splitlines()[0]}),
                      flush=True)
                continue
        else:  # a CPU run only checks that the bench works
            import time

            t0 = time.perf_counter()
            fwd()
            t_f = (time.perf_counter() - t0) * 1e6
            t0 = time.perf_counter()
            fwd_bwd()
            t_fb = (time.perf_counter() - t0) * 1e6
        with torch.no_grad():
            outs[impl] = run(impl).float()
        rec = {"bench": "moe_layer", "impl": impl, "model": a.model, "tokens": a.tokens, "fwd_us": round(t_f, 1),
               "fwd_bwd_us": round(t_fb, 1), "fwd_tflops": round(flops_fwd / t_f / 1e6, 1),
               "fwd_bwd_tflops": round(3 * flops_fwd / t_fb / 1e6, 1)}
        if cuda:
            rec["fwd_bwd_frac_of_" + src + "_bf16_peak"] = round(3 * flops_fwd / t_fb / 1e6 / peak_tf, 3)
        print(json.dumps(rec), flush=True)
    if len(outs) == 2:
        a_, b_ = outs.values()
        print(json.dumps({"bench": "moe_layer", "max_rel_diff": float((a_ - b_).norm() / b_.norm())}), flush=True)


if __name__ == "__main__":
    main()
