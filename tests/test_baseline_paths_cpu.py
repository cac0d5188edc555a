"""The library comparison baseline's graph-capturable pieces, checked on CPU against the plain PyTorch path.

``_advance_masked`` is the host-sync-free version of the decode row advance that the baseline's captured
decode step runs; it must leave the same state as the reference advance (which selects the live rows with
``nonzero``), including rows that are done and the output slots they must not touch.
"""

import torch

from meshy_b200.ops import decode as D


def _state(seed, B=6, R=6, L=32, pages=4, page=8):
    g = torch.Generator().manual_seed(seed)
    st = {
        "tok_in": torch.randint(0, 100, (B,), generator=g),
        "pos": torch.randint(0, 20, (B,), generator=g).int(),
        "gen": torch.randint(0, 10, (B,), generator=g).int(),
        "max_new": torch.randint(5, 12, (B,), generator=g).int(),
        "done": (torch.rand(B, generator=g) < 0.3).int(),
        "block_table": torch.randint(0, 50, (B, pages), generator=g).int(),
        "req": torch.randperm(R, generator=g)[:B].int(),
        "out_tok": torch.zeros(R + 1, L, dtype=torch.int64),
        "out_lp": torch.zeros(R + 1, L),
        "eos": torch.tensor([7, 9]),
    }
    st["seq_lens"] = st["pos"] + 1
    st["slot"] = torch.zeros(B, dtype=torch.int64)
    tok = torch.randint(0, 12, (B,), generator=g)
    lp = -torch.rand(B, generator=g)
    return st, tok, lp


def test_masked_advance_matches_reference_advance():
    for seed in range(20):
        a, tok, lp = _state(seed)
        b = {k: v.clone() for k, v in a.items()}
        D.decode_advance(a, tok, lp, 8)  # CPU tensors: the reference (nonzero) path
        D._advance_masked(b, tok, lp, 8)
        live = a["done"].numel()
        for k in ("tok_in", "pos", "seq_lens", "gen", "done"):
            assert torch.equal(a[k], b[k]), (seed, k)
        R = a["out_tok"].shape[0] - 1
        assert torch.equal(a["out_tok"][:R], b["out_tok"][:R]), seed
        assert torch.equal(a["out_lp"][:R], b["out_lp"][:R]), seed
        was_live = _state(seed)[0]["done"] == 0
        assert torch.equal(a["slot"][was_live], b["slot"][was_live]), seed
        assert live == b["done"].numel()
