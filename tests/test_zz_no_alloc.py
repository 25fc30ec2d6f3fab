"""The allocation-free attention entry point (si_attention_decode_noalloc_dev)
against the regular one (si_attention_decode).

It exists for callers that cannot allocate device memory when they call in
(for example while a stream is being captured, or under a runtime that
forbids cudaMalloc after start-up): its split-K scratch is a fixed array
inside the library. The test calls it twice in a row through the C ABI -- the
second call reuses the scratch the first left behind -- and checks both
outputs against the allocating entry point within the 1e-5 relative-L2
tolerance the other attention tests use. This file is collected last.
"""
import numpy as np
import pytest

import oracle as O
from helpers import rel_l2

pytestmark = pytest.mark.gpu


def _case(rng, qh, kvh, hd, cap, cached):
    q = (rng.normal(0, 1, qh * hd) / 4).astype(np.float32)
    kc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    vc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    nk = rng.normal(0, 1, kvh * hd).astype(np.float32)
    nv = rng.normal(0, 1, kvh * hd).astype(np.float32)
    return q, kc, vc, nk, nv


def test_noalloc_attention_matches_allocating_entry_point(mai, ctx):
    import torch
    rng = np.random.default_rng(2024)
    qh, kvh, hd, cap = 24, 4, 256, 1536
    dev = torch.device("cuda", 0)
    for cached in (700, 1300):  # two calls in a row, different chunk counts
        q, kc, vc, nk, nv = _case(rng, qh, kvh, hd, cap, cached)
        ref = ctx.attention_decode(mai.AttentionDecodeInput(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap))
        t = [torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(dev) for a in (q, kc, vc, nk, nv)]
        out = torch.empty(qh * hd, dtype=torch.float32, device=dev)
        mai.attention_decode_noalloc_dev(t[0], t[1], t[2], t[3], t[4], qh, kvh, hd, cached, cap,
                                         mai.CACHE_BF16, out, None)
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), ref) < 1e-5


def test_noalloc_attention_rejects_oversized_scratch(mai, ctx):
    import torch
    qh, kvh, hd, cap = 24, 4, 256, 65536
    dev = torch.device("cuda", 0)
    small = torch.zeros(qh * hd, device=dev)
    cache = torch.zeros(1, dtype=torch.int16, device=dev)
    with pytest.raises(mai.SiError, match="scratch floats"):
        mai.attention_decode_noalloc_dev(small, cache, cache, small, small, qh, kvh, hd, cap - 1, cap,
                                         mai.CACHE_BF16, small, None)


def test_noalloc_attention_f32_cache_generic_kernel(mai, ctx):
    """An f32 cache with head size 64 takes the general (CUDA-core) kernel."""
    import torch
    rng = np.random.default_rng(77)
    qh, kvh, hd, cap = 8, 2, 64, 900
    dev = torch.device("cuda", 0)
    for cached in (0, 333, 899):
        q = (rng.normal(0, 1, qh * hd) / 4).astype(np.float32)
        kc = rng.normal(0, 1, kvh * cap * hd).astype(np.float32)
        vc = rng.normal(0, 1, kvh * cap * hd).astype(np.float32)
        nk = rng.normal(0, 1, kvh * hd).astype(np.float32)
        nv = rng.normal(0, 1, kvh * hd).astype(np.float32)
        ref = ctx.attention_decode(mai.AttentionDecodeInput(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap))
        t = [torch.from_numpy(a).to(dev) for a in (q, kc, vc, nk, nv)]
        out = torch.empty(qh * hd, dtype=torch.float32, device=dev)
        mai.attention_decode_noalloc_dev(t[0], t[1], t[2], t[3], t[4], qh, kvh, hd, cached, cap,
                                         mai.CACHE_F32, out, None)
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), ref) < 1e-5


def test_noalloc_attention_replays_from_a_cuda_graph(mai, ctx):
    """Two calls captured into one CUDA graph (the second over a different
    cache length), replayed twice, give the allocating entry point's results."""
    import torch
    rng = np.random.default_rng(91)
    qh, kvh, hd, cap = 24, 4, 256, 1024
    dev = torch.device("cuda", 0)
    cases = [_case(rng, qh, kvh, hd, cap, 0) for _ in range(2)]
    cached = (500, 1000)
    refs = [ctx.attention_decode(mai.AttentionDecodeInput(*c, qh, kvh, hd, n, cap)) for c, n in zip(cases, cached)]
    dt = [[torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(dev) for a in c] for c in cases]
    outs = [torch.full((qh * hd,), float("nan"), device=dev) for _ in range(2)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):  # the set-up call comes before the capture
        mai.attention_decode_noalloc_dev(*dt[0], qh, kvh, hd, cached[0], cap, mai.CACHE_BF16, outs[0], s.cuda_stream)
    torch.cuda.synchronize()
    outs[0].fill_(float("nan"))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(2):
            mai.attention_decode_noalloc_dev(*dt[i], qh, kvh, hd, cached[i], cap, mai.CACHE_BF16, outs[i],
                                             s.cuda_stream)
    for _ in range(2):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, refs):
            assert rel_l2(o.cpu().numpy(), r) < 1e-5
