"""The row-sharded matvec (si_sharded_qmatvec_dev) on one GPU.

With one rank it is the plain matvec into the peer buffer. A group of
buffers on this GPU standing in for two ranks (si_peer_buffer_create_local)
exercises the exchange on one device: the matvec's epilogue stores this
rank's rows into both ranks' copies of the vector, and, because the other
rank never runs, the launch's bounded wait for it runs out after about a
millisecond. The timeout is reported as SI_E_TIMEOUT by si_ctx_synchronize,
and the context then works normally. No wait here is unbounded and nothing
faults the GPU: the flag that is waited on is simply never set.
"""
import numpy as np
import pytest

import oracle as O
from helpers import d2h_f32, random_blocks, rel_l2

pytestmark = pytest.mark.gpu


def _read(ptr, n):
    import torch
    torch.cuda.synchronize()
    return d2h_f32(ptr, n)


def _matrix(rows, cols, seed=11):
    rng = np.random.default_rng(seed)
    w = random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    return w, x


def test_one_rank_sharded_matvec_is_the_matvec(mai, ctx):
    import torch
    rows, cols = 17408, 5120
    w, x = _matrix(rows, cols)
    wd = torch.from_numpy(np.concatenate([w, np.zeros(64, np.uint8)])).cuda()
    xd = torch.from_numpy(x).cuda()
    buf = ctx.peer_buffer(rows * 4 + 512)
    try:
        ctx.sharded_qmatvec_dev(buf, 12, wd, rows, cols, xd, 512)
        ctx.synchronize()
        got = _read(buf.local + 512, rows)
        y = torch.empty(rows, device="cuda")
        ctx.qmatvec_dev(12, wd, rows, cols, xd, y)
        torch.cuda.synchronize()
        assert np.array_equal(got, y.cpu().numpy())
        assert rel_l2(got, O.matvec(12, w, rows, cols, x)) < 1e-5
    finally:
        buf.close()


@pytest.mark.parametrize("rank", [0, 1])
def test_two_rank_exchange_times_out_without_the_peer(mai, ctx, rank):
    import torch
    rows, cols, world = 4352, 5120, 2
    w, x = _matrix(rows, cols, seed=21 + rank)
    rl = rows // world
    shard = np.concatenate([w.reshape(rows, -1)[rank * rl:(rank + 1) * rl].reshape(-1), np.zeros(64, np.uint8)])
    wd = torch.from_numpy(shard).cuda()
    xd = torch.from_numpy(x).cuda()
    ref = O.matvec(12, w, rows, cols, x)[rank * rl:(rank + 1) * rl]
    buf = ctx.peer_buffer_local(rows * 4, world, rank, wait_us=1000)
    try:
        ctx.sharded_qmatvec_dev(buf, 12, wd, rl, cols, xd, 0)
        with pytest.raises(mai.SiError) as ei:
            ctx.synchronize()
        assert ei.value.status == mai.SI_E_TIMEOUT
        # this rank's rows reached both ranks' copies before the wait ran out
        local = _read(buf.local, rows)[rank * rl:(rank + 1) * rl]
        assert rel_l2(local, ref) < 1e-5
    finally:
        buf.close()
    # the context is usable after the timeout
    got = ctx.q4_k_matvec(w, rows, cols, x)
    assert rel_l2(got, O.matvec(12, w, rows, cols, x)) < 1e-5
    ctx.synchronize()


@pytest.mark.parametrize("rows_per_rank", [2176, 4352, 8704])
def test_config1_shards_take_the_fused_exchange(mai, ctx, rows_per_rank):
    """The shards of config 1 at 8, 4 and 2 ranks (up to two CTAs per SM) run
    the matvec whose epilogue does the exchange, not the matvec plus the
    stand-alone all-gather: that kernel alone writes the exchange words that
    follow the buffer's 2,560-byte tail (the first launch, epoch 1, uses
    parity half 1, whose word 0 holds {y[0], 1}). Either path honours the
    buffer's wait bound."""
    import time
    import torch
    cols, world = 5120, 2
    w, x = _matrix(rows_per_rank, cols, seed=rows_per_rank)
    wd = torch.from_numpy(np.concatenate([w, np.zeros(64, np.uint8)])).cuda()
    xd = torch.from_numpy(x).cuda()
    nbytes = world * rows_per_rank * 4
    buf = ctx.peer_buffer_local(nbytes, world, 0, wait_us=1000)
    try:
        t0 = time.perf_counter()
        ctx.sharded_qmatvec_dev(buf, 12, wd, rows_per_rank, cols, xd, 0)
        with pytest.raises(mai.SiError) as ei:
            ctx.synchronize()
        assert ei.value.status == mai.SI_E_TIMEOUT
        assert time.perf_counter() - t0 < 1.0
        data_bytes = (nbytes + 255) // 256 * 256
        word = _read(buf.local + data_bytes + 2560 + 8 * (data_bytes // 4), 2).view(np.uint32)
        got = _read(buf.local, rows_per_rank)
        assert word[1] == 1 and word[0] == got[:1].view(np.uint32)[0]
        assert rel_l2(got, O.matvec(12, w, rows_per_rank, cols, x)) < 1e-5
    finally:
        buf.close()
    ctx.synchronize()


def test_q6k_shard_takes_the_fused_exchange(mai, ctx):
    """A Q6_K shard of the 27B ffn_down at two ranks (2560 x 17408) runs the
    Q6_K tensor-core matvec with the exchange in the kernel: its rows are in
    the exchange words (epoch 1, parity half 1) and unpacked into this
    rank's slice before the bounded wait for the absent rank runs out."""
    import torch
    rows, cols, world = 2560, 17408, 2
    rng = np.random.default_rng(2560)
    w = random_blocks(rng, 14, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    wd = torch.from_numpy(np.concatenate([w, np.zeros(64, np.uint8)])).cuda()
    xd = torch.from_numpy(x).cuda()
    nbytes = world * rows * 4
    buf = ctx.peer_buffer_local(nbytes, world, 0, wait_us=1000)
    try:
        ctx.sharded_qmatvec_dev(buf, 14, wd, rows, cols, xd, 0)
        with pytest.raises(mai.SiError) as ei:
            ctx.synchronize()
        assert ei.value.status == mai.SI_E_TIMEOUT
        data_bytes = (nbytes + 255) // 256 * 256
        word = _read(buf.local + data_bytes + 2560 + 8 * (data_bytes // 4), 2).view(np.uint32)
        got = _read(buf.local, rows)
        assert word[1] == 1 and word[0] == got[:1].view(np.uint32)[0]
        assert rel_l2(got, O.matvec(14, w, rows, cols, x)) < 1e-5
    finally:
        buf.close()
    ctx.synchronize()
