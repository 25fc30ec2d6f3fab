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


def _decode(mai, ctx):
    m = mai.Model(ctx, mai.qwen36_27b_config(**CFG), seed=77)
    try:
        m.reset()
        ids = m.generate(PROMPT, STEPS)
        m.reset()
        h = m.embed_token(PROMPT[0])
        h = m.decode_hidden(0, h)
        return ids, m.logits(h)
    finally:
        m.close()


def _worker(rank, world, uid, flags, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from conftest import load_package
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mai = load_package()
    ctx = mai.CudaContext(rank, flags=flags)
    ctx.comm_init(world, rank, uid)
    ids, logits = _decode(mai, ctx)
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
