"""Row-sharded decode over NCCL against the same model on one GPU.

One process per GPU (2, 4 or 8, as many as are visible; skipped with fewer
than two). Every rank builds only its shard of a small Qwen3.6-shaped model,
decodes greedily with an all-gather of every sharded output vector, and must
produce the 1-GPU token IDs and logits exactly: sharding changes which GPU
computes a row, never a row's arithmetic. Both transports of the sharded
vectors are checked: stores into the peers' memory over NVLink (the default)
and NCCL all-gathers.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden=1024, intermediate=2048, layers=8, vocab=4096, attn_q_heads=8, attn_kv_heads=2,
           attn_head_dim=128, rotary_dim=32, gdn_key_heads=8, gdn_value_heads=16, kv_capacity=40)
PROMPT = [3, 141, 59, 2653, 17]
STEPS = 12


# hidden and intermediate of 4096 rows and more: one GPU runs these matrices
# on the tensor-core matvec, so the sharded model gathers the activation and
# the hidden vector inside that kernel (no stand-alone all-gather)
CFG_EXCHANGE = dict(CFG, hidden=4096, intermediate=8192, layers=4, attn_q_heads=16)


def _decode(mai, ctx, cfg=CFG):
    m = mai.Model(ctx, mai.qwen36_27b_config(**cfg), seed=77)
    try:
        m.reset()
        ids = m.generate(PROMPT, STEPS)
        m.reset()
        h = m.embed_token(PROMPT[0])
        h = m.decode_hidden(0, h)
        return ids, m.logits(h)
    finally:
        m.close()


def _worker(rank, world, uid, flags, out, cfg=CFG):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from conftest import load_package
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mai = load_package()
    ctx = mai.CudaContext(rank, flags=flags)
    ctx.comm_init(world, rank, uid)
    ids, logits = _decode(mai, ctx, cfg)
    ctx.close()
    out[rank] = (ids, logits.tobytes())


@pytest.mark.parametrize("transport", ["nvlink_peer", "nccl"])
def test_row_sharded_decode_matches_one_gpu(mai, transport):
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    uid = mai.CudaContext.comm_unique_id()
    ctx = mgr = None
    mgr = mp.Manager()
    out = mgr.dict()
    flags = mai.CTX_FLAG_NCCL_COLLECTIVES if transport == "nccl" else 0
    mp.spawn(_worker, args=(world, uid, flags, out), nprocs=world, join=True)
    ctx = mai.CudaContext(0)
    ref_ids, ref_logits = _decode(mai, ctx)
    ctx.close()
    for rank in range(world):
        ids, lb = out[rank]
        assert ids == ref_ids, rank
        assert np.array_equal(np.frombuffer(lb, np.float32), ref_logits), rank


def test_row_sharded_decode_with_in_kernel_gather(mai):
    """Sharded decode whose Q4_K gate/up pairs and residual matvecs gather
    their outputs inside the tensor-core matvec. Its shards add their blocks
    in another order than the whole matrix does on one GPU (the kernel
    splits a row's blocks over as many warps as its CTA has room for), so the
    logits agree within 1e-4 rather than bit for bit, and the greedy IDs
    agree exactly."""
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    uid = mai.CudaContext.comm_unique_id()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, uid, 0, out, CFG_EXCHANGE), nprocs=world, join=True)
    ctx = mai.CudaContext(0)
    ref_ids, ref_logits = _decode(mai, ctx, CFG_EXCHANGE)
    ctx.close()
    for rank in range(world):
        ids, lb = out[rank]
        got = np.frombuffer(lb, np.float32)
        assert ids == ref_ids, rank
        assert np.linalg.norm(got - ref_logits) / np.linalg.norm(ref_logits) < 1e-4, rank


def _sharded_worker(rank, world, uid, out):
    import sys
    import torch
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from conftest import load_package
    from helpers import d2h_f32, random_blocks
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mai = load_package()
    torch.cuda.set_device(rank)
    ctx = mai.CudaContext(rank)
    ctx.comm_init(world, rank, uid)
    res = {}
    for name, ty, rows, cols in (("q4k", 12, 17408, 5120), ("q6k", 14, 5120, 17408)):
        rng = np.random.default_rng(rows + ty)
        w = random_blocks(rng, ty, rows * cols // 256).reshape(rows, -1)
        x = rng.normal(0, 1, cols).astype(np.float32)
        rl = rows // world
        shard = torch.from_numpy(np.concatenate([w[rank * rl:(rank + 1) * rl].reshape(-1),
                                                 np.zeros(64, np.uint8)])).to(f"cuda:{rank}")
        xd = torch.from_numpy(x).to(f"cuda:{rank}")
        buf = ctx.peer_buffer(rows * 4 + 1024)
        ys = []
        for _ in range(2):  # two calls: the signal counters carry over correctly
            ctx.sharded_qmatvec_dev(buf, ty, shard, rl, cols, xd, 256)
            ctx.synchronize()
            ys.append(d2h_f32(buf.local + 256, rows).tobytes())
        buf.close()
        res[name] = ys
    ctx.close()
    out[rank] = res


def test_sharded_matvec_gathers_into_every_rank(mai):
    """si_sharded_qmatvec_dev on every GPU: Q4_K rows reach every rank from the
    tensor-core matvec's epilogue (NVLink stores + in-kernel completion
    signal), Q6_K through the matvec and the peer all-gather kernel. Every
    rank ends with the same full vector, equal to the oracle within 1e-5."""
    import torch
    import torch.multiprocessing as mp
    import oracle as O
    from helpers import random_blocks, rel_l2
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    uid = mai.CudaContext.comm_unique_id()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_sharded_worker, args=(world, uid, out), nprocs=world, join=True)
    for name, ty, rows, cols in (("q4k", 12, 17408, 5120), ("q6k", 14, 5120, 17408)):
        rng = np.random.default_rng(rows + ty)
        w = random_blocks(rng, ty, rows * cols // 256)
        x = rng.normal(0, 1, cols).astype(np.float32)
        ref = O.matvec(ty, w, rows, cols, x)
        first = out[0][name][0]
        for rank in range(world):
            for yb in out[rank][name]:
                assert yb == first, (name, rank)
        assert rel_l2(np.frombuffer(first, np.float32), ref) < 1e-5, name
