"""The allocation-free decode attention, b2_attn_decode_noalloc, against the allocating b2_attn_decode.

Callers that cannot allocate device memory (a host whose memory belongs to another allocator, an FFI caller holding
only its own buffers) use the variant whose split partials live in a fixed array inside the library. This file runs
last so that a failure here comes after every other test; it also passes alone in a fresh process. Calls in a row
with different shapes check that the shared array's previous contents never reach a result; one of them fills the
array to its limit (batch x heads = 128 rows).
"""
import ctypes

import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec

pytestmark = pytest.mark.gpu

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _inputs(dev, B, H, Hkv, cap, lengths, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, 1, H, 128), generator=g).to(dev)
    k = torch.randn((B, cap, Hkv, 128), generator=g).to(dev)
    v = torch.randn((B, cap, Hkv, 128), generator=g).to(dev)
    return q, k, v, torch.tensor(lengths, dtype=torch.int32, device=dev)


def _noalloc(lib, q, k, v, ln, out, B, H, Hkv, cap, scale):
    return lib.b2_attn_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ln.data_ptr()),
                                      P(out.data_ptr()), I(B), I(H), I(Hkv), I(cap), F(scale),
                                      P(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_allocating_entry_point(pkg, dev):
    lib = pkg._lib.load()
    scale = 128 ** -0.5
    # The third case is batch x heads = 128, the array's limit: it reaches the last partial and statistics slot.
    cases = [(1, 32, 8, 1024, [1024]), (3, 16, 4, 300, [299, 7, 150]), (4, 32, 8, 200, [200, 1, 64, 133])]
    for seed, (B, H, Hkv, cap, lengths) in enumerate(cases):
        q, k, v, ln = _inputs(dev, B, H, Hkv, cap, lengths, seed)
        ref = pkg.ops.attn_decode(q, k, v, ln, scale)
        out = torch.full_like(q, float("nan"))
        assert _noalloc(lib, q, k, v, ln, out, B, H, Hkv, cap, scale) == 0, lib.b2_last_error()
        torch.cuda.synchronize()
        # Same kernels, same grid: only the scratch address differs, so the results are identical bit for bit.
        assert torch.equal(out, ref), f"case {seed}: noalloc differs from b2_attn_decode"
        if seed == 2:
            exact = odec.attn_decode(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), lengths, scale)
            assert oatt.rel_l2(out.cpu().numpy(), exact) < 1e-5


def test_noalloc_rejects_calls_beyond_its_scratch(pkg, dev):
    lib = pkg._lib.load()
    q, k, v, ln = _inputs(dev, 5, 32, 8, 16, [16] * 5, 9)
    out = torch.empty_like(q)
    assert _noalloc(lib, q, k, v, ln, out, 5, 32, 8, 16, 1.0) == 2
    assert b"exceeds" in lib.b2_last_error()
