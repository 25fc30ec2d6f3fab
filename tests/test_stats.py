"""Command counters (CommandStats, metal.rs:1891-1947): the reference's
delta test restated against si_stats_delta (CPU), and the counting of
synchronous and asynchronous submissions on the GPU."""
import numpy as np
import pytest

from conftest import load_package


def test_delta_saturates_counters():  # metal.rs:7129-7150
    mai = load_package()
    before = {"submitted": 10, "async_submitted": 4, "waited": 8, "wait_nanos": 100}
    after = {"submitted": 13, "async_submitted": 5, "waited": 7, "wait_nanos": 90, "peak_kv_bytes": 7}
    d = mai.stats_delta(after, before)
    assert (d["submitted"], d["async_submitted"], d["waited"], d["wait_nanos"]) == (3, 1, 0, 0)
    assert d["peak_kv_bytes"] == 7  # byte fields are the later snapshot's


@pytest.mark.gpu
def test_sync_and_async_submissions_are_counted(mai, ctx):  # metal.rs:7112-7125
    """A host-memory call submits and waits once; a `_dev` call submits
    asynchronously and does not wait."""
    import torch
    from helpers import random_blocks
    rng = np.random.default_rng(4)
    w = random_blocks(rng, 12, 64 * 512 // 256)
    x = rng.normal(0, 1, 512).astype(np.float32)
    s0 = ctx.stats()
    ctx.gguf_quant_matvec_bytes(12, w, 64, 512, x)
    s1 = ctx.stats()
    d = mai.stats_delta(s1, s0)
    assert (d["submitted"], d["async_submitted"], d["waited"]) == (1, 0, 1) and d["wait_nanos"] > 0
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    yd = torch.empty(64, device="cuda")
    torch.cuda.synchronize()
    ctx.qmatvec_dev(12, wd, 64, 512, xd, yd, ctx.stream)
    torch.cuda.synchronize()
    d = mai.stats_delta(ctx.stats(), s1)
    assert (d["submitted"], d["async_submitted"], d["waited"]) == (1, 1, 0)
    with pytest.raises(mai.SiError):
        ctx.qmatvec_dev(1, wd, 64, 512, xd, yd, ctx.stream)  # not a K-quant type: refused, not counted
    d = mai.stats_delta(ctx.stats(), s1)
    assert d["async_submitted"] == 1
