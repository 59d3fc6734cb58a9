"""The allocation-free decode attention, b2_attn_decode_noalloc, against the allocating b2_attn_decode.

Callers that cannot allocate device memory (a host whose memory belongs to another allocator, an FFI caller holding
only its own buffers) use the variant whose split partials live in a fixed array inside the library. This file runs
last so that a failure here comes after every other test; it also passes alone in a fresh process. Two calls in a
row with different shapes check that the shared array's previous contents never reach a result.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _inputs(dev, B, H, Hkv, cap, lengths, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, 1, H, 128), generator=g).to(dev)
    k = torch.randn((B, cap, Hkv, 128), generator=g).to(dev)
    v = torch.randn((B, cap, Hkv, 128), generator=g).to(dev)
    return q, k, v, torch.tensor(lengths, dtype=torch.int32, device=dev)


def test_noalloc_matches_allocating_entry_point(pkg, dev):
    lib = pkg._lib.load()
    stream = P(torch.cuda.current_stream().cuda_stream)
    cases = [(1, 32, 8, 1024, [1024]), (3, 16, 4, 300, [299, 7, 150])]
    for seed, (B, H, Hkv, cap, lengths) in enumerate(cases):
        q, k, v, ln = _inputs(dev, B, H, Hkv, cap, lengths, seed)
        ref = pkg.ops.attn_decode(q, k, v, ln, 128 ** -0.5)
        out = torch.full_like(q, float("nan"))
        rc = lib.b2_attn_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ln.data_ptr()),
                                        P(out.data_ptr()), I(B), I(H), I(Hkv), I(cap), F(128 ** -0.5), stream)
        assert rc == 0, lib.b2_last_error()
        torch.cuda.synchronize()
        assert oatt.rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_noalloc_rejects_calls_beyond_its_scratch(pkg, dev):
    lib = pkg._lib.load()
    q, k, v, ln = _inputs(dev, 5, 32, 8, 16, [16] * 5, 9)
    out = torch.empty_like(q)
    rc = lib.b2_attn_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ln.data_ptr()),
                                    P(out.data_ptr()), I(5), I(32), I(8), I(16), F(1.0),
                                    P(torch.cuda.current_stream().cuda_stream))
    assert rc == 2
    assert b"exceeds" in lib.b2_last_error()
