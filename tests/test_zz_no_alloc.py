"""The allocation-free paged-decode entry point, called through its C symbol.

``meshy_paged_decode_noalloc`` (csrc/kernels/decode_noalloc.cu) is an
addition of this library with no counterpart in the reference framework. It
serves callers that cannot allocate device memory: a C/C++ host without
PyTorch's allocator, a server whose KV pool already holds nearly all HBM, or a
decode loop that must not pay cudaMalloc's implicit synchronisation. Its
split-KV partials live in a fixed device array inside the library.

The test loads the built extension as a plain shared library with ctypes and
checks the entry point against the regular one (``_C.paged_attention``) on two
calls in a row, with different inputs, so a stale partial from the first call
would show up in the second. This file sorts last so a run that stops at the
first failure has run every other test before it.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    import meshy_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.meshy_paged_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_void_p]
    lib.meshy_noalloc_last_error.restype = ctypes.c_char_p
    lib.meshy_paged_decode_noalloc_scratch_capacity.restype = ctypes.c_size_t
    lib.meshy_paged_decode_noalloc_scratch_need.restype = ctypes.c_size_t
    lib.meshy_paged_decode_noalloc_scratch_need.argtypes = [ctypes.c_int] * 4
    return C, lib, fn


def _case(seed, lens, Hq=12, Hkv=2, hd=128, page=64, n_pages=96, max_pages=24):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(n_pages, Hkv, page, hd, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(n_pages, Hkv, page, hd, device=DEV, generator=g).to(torch.bfloat16)
    B = len(lens)
    bt = torch.zeros(B, max_pages, dtype=torch.int32, device=DEV)
    perm = torch.randperm(n_pages, device=DEV, generator=g)
    used = 0
    for b, L in enumerate(lens):
        npg = (L + page - 1) // page
        bt[b, :npg] = perm[used:used + npg].int()
        used += npg
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = torch.randn(B, Hq, hd, device=DEV, generator=g).to(torch.bfloat16)
    return q, kc, vc, bt, seq


def _call(fn, q, kc, vc, bt, seq, out, scale, n_split=0):
    B, Hq, hd = q.shape
    Hkv, page = kc.shape[1], kc.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), seq.data_ptr(), out.data_ptr(), B, Hq, Hkv,
              hd, page, bt.shape[1], n_split, scale, stream)


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def test_noalloc_decode_matches_regular_entry_point_twice():
    C, lib, fn = _lib()
    cases = [_case(11, [1, 64, 65, 300, 1000, 1500]), _case(12, [700, 3, 129, 1536])]
    for q, kc, vc, bt, seq in cases:
        scale = 1.0 / math.sqrt(q.shape[-1])
        want = torch.empty_like(q)
        C.paged_attention(q, kc, vc, bt, seq, want, scale, None)
        got = torch.full_like(q, float("nan"))
        rc = _call(fn, q, kc, vc, bt, seq, got, scale)
        assert rc == 0, lib.meshy_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert _rel_err(got, want) < 1e-2
    assert C.device_error() == 0


def test_noalloc_decode_explicit_splits_and_rejects_oversize():
    C, lib, fn = _lib()
    q, kc, vc, bt, seq = _case(13, [900, 20, 1400])
    scale = 1.0 / math.sqrt(q.shape[-1])
    want = torch.empty_like(q)
    C.paged_attention(q, kc, vc, bt, seq, want, scale, None)
    for splits in (1, 3, 7):
        got = torch.zeros_like(q)
        assert _call(fn, q, kc, vc, bt, seq, got, scale, n_split=splits) == 0, lib.meshy_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert _rel_err(got, want) < 1e-2
    cap = lib.meshy_paged_decode_noalloc_scratch_capacity()
    B, Hq, hd = q.shape
    too_many = cap // (B * Hq * (hd + 2) * 4) + 1
    assert lib.meshy_paged_decode_noalloc_scratch_need(B, Hq, hd, too_many) > cap
    out = torch.zeros_like(q)
    rc = _call(fn, q, kc, vc, bt, seq, out, scale, n_split=too_many)
    assert rc != 0
    assert "scratch" in lib.meshy_noalloc_last_error().decode()
    torch.cuda.synchronize()
    assert int(out.float().abs().sum().item()) == 0  # nothing was launched


def test_noalloc_decode_rejects_unsupported_layout():
    """A page size other than 64 (or an unsupported head size) returns a non-zero code and a message, and
    launches nothing."""
    C, lib, fn = _lib()
    q, kc, vc, bt, seq = _case(14, [100, 40], page=32, n_pages=16, max_pages=8)
    out = torch.zeros_like(q)
    rc = _call(fn, q, kc, vc, bt, seq, out, 1.0 / math.sqrt(q.shape[-1]))
    assert rc != 0
    assert "page_size" in lib.meshy_noalloc_last_error().decode()
    torch.cuda.synchronize()
    assert int(out.float().abs().sum().item()) == 0
