"""Host-side logic of the row-sharded path, on CPU.

The shard ranges (si_model_shard_rows) and residency plans
(si_model_plan_dry) are pure host code; these tests check that the ranks'
shards partition every tensor of the 27B-shape model exactly (rows of a KV
head are replicated on the two ranks of its GQA group at 8 ranks), that plans
shrink with the rank count, and -- with two gloo ranks on this host -- the
rank-side plumbing bench.py uses: rendezvous, the broadcast of the NCCL id
bytes and the max-over-ranks timing reduction.
"""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO, load_package

# tensor ids (include/si_cuda.h)
T_FFN_GATE, T_FFN_DOWN, T_SSM_QKV, T_SSM_Z, T_SSM_OUT = 2, 4, 5, 6, 13
T_ATTN_Q, T_ATTN_K, T_ATTN_V, T_ATTN_O, T_OUTPUT, T_EMBD = 14, 15, 16, 17, 22, 20
SHARDED = [(0, T_FFN_GATE), (0, T_FFN_DOWN), (0, T_SSM_QKV), (0, T_SSM_Z), (0, T_SSM_OUT),
           (3, T_ATTN_Q), (3, T_ATTN_O), (64, T_OUTPUT), (64, T_EMBD)]


def _covered(ranges_per_rank):
    rows = {}
    for rk, ranges in enumerate(ranges_per_rank):
        for b, e in ranges:
            for r in range(b, e):
                rows.setdefault(r, []).append(rk)
    return rows


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_shards_partition_every_tensor(n):
    mai = load_package()
    c = mai.qwen36_27b_config()
    for layer, t in SHARDED:
        full = mai.shard_rows(c, 1, 0, layer, t)
        total = sum(e - b for b, e in full)
        cov = _covered([mai.shard_rows(c, n, r, layer, t) for r in range(n)])
        assert len(cov) == total, (layer, t)
        assert all(len(v) == 1 for v in cov.values()), (layer, t)
        # each rank holds the same number of rows
        sizes = [sum(e - b for b, e in mai.shard_rows(c, n, r, layer, t)) for r in range(n)]
        assert len(set(sizes)) == 1


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_kv_heads_follow_their_query_heads(n):
    mai = load_package()
    c = mai.qwen36_27b_config()
    group = c.attn_q_heads // c.attn_kv_heads
    hd = c.attn_head_dim
    for r in range(n):
        q = mai.shard_rows(c, n, r, 3, T_ATTN_Q)[0]      # query half of attn_q
        heads = range(q[0] // hd, q[1] // hd)
        kv_needed = {h // group for h in heads}
        for t in (T_ATTN_K, T_ATTN_V):
            (b, e), = mai.shard_rows(c, n, r, 3, t)
            assert set(range(b // hd, e // hd)) == kv_needed
    cov = _covered([mai.shard_rows(c, n, r, 3, T_ATTN_K) for r in range(n)])
    assert len(cov) == c.attn_kv_heads * hd
    assert {len(v) for v in cov.values()} == ({2} if n == 8 else {1})


def test_plans_shrink_with_ranks():
    mai = load_package()
    c = mai.qwen36_27b_config()
    budget = 4 << 30
    plans = {n: mai.plan_dry(c, n, 0, budget, 3) for n in (1, 2, 4, 8)}
    assert plans[1]["streamed_layers"] == 55 and plans[1]["head_resident"] == 1
    assert plans[2]["streamed_bytes_per_token"] < plans[1]["streamed_bytes_per_token"]
    assert plans[4]["streamed_bytes_per_token"] == 0 and plans[8]["streamed_bytes_per_token"] == 0
    for p in plans.values():
        fixed = p["resident_weight_bytes"] + p["ring_bytes"] + p["state_bytes"] + p["scratch_bytes"]
        assert fixed <= budget
    with pytest.raises(mai.SiError):
        mai.plan_dry(c, 1, 0, 1 << 30, 3)   # the head alone exceeds 1 GB


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import sys
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import bench
    from conftest import load_package as lp
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mai = lp()
        c = mai.qwen36_27b_config()
        mine = {(layer, t): mai.shard_rows(c, world, rank, layer, t) for layer, t in SHARDED}
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        uid = [bytes(range(128)) if rank == 0 else None]   # stands in for si_comm_unique_id
        dist.broadcast_object_list(uid, src=0)
        mx = bench.max_over_ranks(float(rank + 1) * 1.5, world)
        out[rank] = (allr, uid[0], mx)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_shards_and_timing():
    mai = load_package()
    c = mai.qwen36_27b_config()
    world = 2
    mgr = mp.get_context("spawn").Manager()  # no fork of this multi-threaded process
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for rank in range(world):
        allr, uid, mx = out[rank]
        assert uid == bytes(range(128))
        assert mx == pytest.approx(3.0)
        for key in allr[0]:
            layer, t = key
            cov = _covered([allr[r][key] for r in range(world)])
            full = mai.shard_rows(c, 1, 0, layer, t)
            assert len(cov) == sum(e - b for b, e in full)
            assert all(len(v) == 1 for v in cov.values())


def _failing_worker(rank, world, port, mode, out):
    """Rank 1 either never joins the group or leaves it between steps; rank 0
    must get an error from the rendezvous or its next collective, not hang."""
    import sys
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), SI_DIST_TIMEOUT_S="5")
    sys.path.insert(0, REPO)
    import bench

    class Args:
        impl = "reference"  # gloo

    if rank == 1:
        if mode == "never_joins":
            return
        bench.dist_init(Args())
        dist.barrier()  # one step together, then leave before the next
        dist.destroy_process_group()
        return
    t0 = time.time()
    try:
        bench.dist_init(Args())
        if mode == "leaves":
            dist.barrier()
            time.sleep(1.0)
        bench.max_over_ranks(1.0, world)
        out[rank] = ("no error", time.time() - t0)
    except Exception as e:  # the failure arrives on the host as an exception
        out[rank] = (type(e).__name__, time.time() - t0)


@pytest.mark.parametrize("mode", ["never_joins", "leaves"])
def test_a_missing_rank_is_reported_not_waited_for(mode):
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_failing_worker, args=(world, _free_port(), mode, out), nprocs=world, join=True)
    kind, seconds = out[0]
    assert kind != "no error"
    assert seconds < 60
    if mode == "never_joins":
        assert seconds >= 4  # the rendezvous waited for the configured 5 s, then failed
