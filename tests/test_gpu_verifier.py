"""Batched verifier on the GPU: the K<=8 matvec family against the oracle
(one matvec per candidate), and decode_tokens_many / logits_many /
verify_many of a small model against sequential decode by the oracle and by
the GPU itself (qwen35_runtime.rs:879-1289, 2048-2227; the reference's
si-qwen35-batch-probe compares the same pair)."""
import gc

import numpy as np
import pytest

import oracle as O
from helpers import random_blocks, rel_l2

pytestmark = pytest.mark.gpu

Q4, Q5, Q6 = 12, 13, 14


@pytest.mark.parametrize("ty", [Q4, Q5, Q6])
# shapes cover: one and several column panels (17408 columns: 2 at K=5, 3 at
# K=8), CTAs with more 16-row groups than warps (40000 rows), ragged row
# groups (1001, 17), a batch of one (the matvec path)
@pytest.mark.parametrize("rows,cols,batch", [(4096, 5120, 8), (1001, 512, 3), (17, 256, 1), (64, 17408, 5),
                                             (2048, 1024, 2), (5120, 17408, 8), (40000, 256, 7), (33, 768, 4)])
def test_matmul_many_matches_oracle(mai, ctx, ty, rows, cols, batch):
    rng = np.random.default_rng(rows + cols + batch + ty)
    w = random_blocks(rng, ty, rows * cols // 256)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    y = ctx.gguf_quant_matmul_many_bytes(ty, w, rows, cols, batch, x)
    ref = O.matmul_many(ty, w, rows, cols, batch, x)
    for k in range(batch):
        assert rel_l2(y[k], ref[k]) < 1e-5, k


@pytest.mark.parametrize("ty", [Q4, Q6])
def test_matmul_many_large_and_tiny_inputs(mai, ctx, ty):
    """Inputs far from unit scale: the tensor-core form keeps its per-block
    sums in units of the block's own power of two."""
    rng = np.random.default_rng(11 + ty)
    rows, cols, batch = 512, 2048, 6
    w = random_blocks(rng, ty, rows * cols // 256)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    x[:2] *= 3e6
    x[2:4] *= 1e-6
    x[4, :256] = 0.0  # an all-zero block
    y = ctx.gguf_quant_matmul_many_bytes(ty, w, rows, cols, batch, x)
    ref = O.matmul_many(ty, w, rows, cols, batch, x)
    for k in range(batch):
        assert rel_l2(y[k], ref[k]) < 1e-5, k


def test_matmul_many_retained_weight_and_device_form(mai, ctx):
    import torch
    rng = np.random.default_rng(5)
    rows, cols, batch = 3000, 2048, 8
    w = random_blocks(rng, Q6, rows * cols // 256)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    qw = ctx.upload_quant_weight_private(w, Q6)
    y = ctx.gguf_quant_matmul_many_weight(qw, rows, cols, batch, x)
    ref = O.matmul_many(Q6, w, rows, cols, batch, x)
    assert max(rel_l2(y[k], ref[k]) for k in range(batch)) < 1e-5
    wd = torch.from_numpy(w).cuda()
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(batch, rows, device="cuda")
    ctx.qmatmul_many_dev(Q6, wd, rows, cols, batch, xd, yd, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), y)
    ctx.free_weight(qw)


def test_matmul_many_validation_matches_reference(mai, ctx):
    rng = np.random.default_rng(2)
    w = random_blocks(rng, Q4, 4)
    x = np.zeros((9, 256), np.float32)
    with pytest.raises(mai.SiError, match="batched quantized matvec dimensions are invalid"):
        ctx.gguf_quant_matmul_many_bytes(Q4, w, 4, 256, 9, x)
    with pytest.raises(mai.SiError, match="batched quantized matvec dimensions are invalid"):
        ctx.gguf_quant_matmul_many_bytes(Q4, w, 4, 256, 0, x[:0])
    with pytest.raises(mai.SiError, match="byte length is invalid"):
        ctx.gguf_quant_matmul_many_bytes(Q4, w[:-1], 4, 256, 2, x[:2])
    with pytest.raises(mai.SiError, match="unsupported batched quantized weight type"):
        ctx.gguf_quant_matmul_many_bytes(1, w, 4, 256, 2, x[:2])


def small_config(mai, **kw):
    base = dict(hidden=512, intermediate=1024, layers=8, vocab=4096, attn_q_heads=4, attn_kv_heads=2,
                attn_head_dim=128, rotary_dim=32, gdn_key_heads=2, gdn_value_heads=4, kv_capacity=40)
    base.update(kw)
    return mai.qwen36_27b_config(**base)


def prefill(model, prompt):
    for pos, tok in enumerate(prompt):
        model.decode_token(tok, pos, want_logits=False)


def test_decode_tokens_many_matches_sequential_oracle(mai, ctx):
    m = mai.Model(ctx, small_config(mai), seed=77)
    orc = O.OracleModel(m.config, m.host_tensor)
    prompt = [9, 1000, 4000]
    prefill(m, prompt)
    for pos, tok in enumerate(prompt):
        orc.decode_hidden(pos, orc.embed(tok))
    window = [17, 17, 3021, 0, 4095, 8, 222]
    positions = list(range(len(prompt), len(prompt) + len(window)))
    hidden = m.decode_tokens_many(window, positions)
    logits, ids = m.logits_many(hidden)
    # every op is within 1e-5 of the oracle (the matmul tests above: ~3e-6);
    # over ten positions of an 8-layer random model the hidden states grow to
    # ~1e5 and the differences compound, as in the 27B-shape test (1e-4)
    for k, (tok, pos) in enumerate(zip(window, positions)):
        h = orc.decode_hidden(pos, orc.embed(tok))
        assert rel_l2(hidden[k], h) < 5e-5, k
        lo = orc.logits(h)
        assert rel_l2(logits[k], lo) < 5e-5, k
        assert ids[k] == int(O.argmax(lo)), k
    orc.close()
    m.close()


def test_verify_many_equals_gpu_sequential_decode(mai, ctx):
    """The verifier's greedy ids and logits equal sequential decode_token on
    the GPU from the same state, window sizes 1..8."""
    cfg = small_config(mai)
    a, b = mai.Model(ctx, cfg, seed=5), mai.Model(ctx, cfg, seed=5)
    prompt = [1, 2, 3]
    prefill(a, prompt)
    prefill(b, prompt)
    pos = len(prompt)
    rng = np.random.default_rng(3)
    for K in range(1, 9):
        window = rng.integers(0, cfg.vocab, K).tolist()
        ids, logits = a.verify_many(window, list(range(pos, pos + K)), want_logits=True)
        for k, tok in enumerate(window):
            nxt, lo = b.decode_token(tok, pos + k)
            assert ids[k] == nxt, (K, k)
            # both paths are within 1e-5 of the oracle (the batched one is
            # checked against it above; the sequential one in
            # test_gpu_model.py); they differ from each other by at most the sum
            assert rel_l2(logits[k], lo) < 2e-5, (K, k)
        # hidden states left on the device serve logits_many without a copy
        _, ids2 = a.logits_many(None, n=K, want_logits=False)
        assert ids2 == ids
        pos += K
    a.close()
    b.close()


def test_streamed_verifier_equals_resident(mai, ctx):
    cfg = small_config(mai)
    full = mai.plan_dry(cfg)
    total = full["resident_weight_bytes"] + full["state_bytes"] + full["scratch_bytes"]
    ctx_s = mai.CudaContext(0, hbm_budget_bytes=int(total * 0.75), stage_depth=3)
    ctx_r = mai.CudaContext(0)
    s, r = mai.Model(ctx_s, cfg, seed=9), mai.Model(ctx_r, cfg, seed=9)
    assert s.plan()["streamed_layers"] > 0
    window = [4, 40, 400, 4000]
    ids_s, lo_s = s.verify_many(window, [0, 1, 2, 3], want_logits=True)
    ids_r, lo_r = r.verify_many(window, [0, 1, 2, 3], want_logits=True)
    assert ids_s == ids_r and np.array_equal(lo_s, lo_r)
    s.close()
    r.close()
    ctx_s.close()
    ctx_r.close()


def test_window_overflowing_the_kv_cache_is_refused_without_state_change(mai, ctx):
    cfg = small_config(mai, kv_capacity=6)
    a, b = mai.Model(ctx, cfg, seed=1), mai.Model(ctx, cfg, seed=1)
    prefill(a, [1, 2, 3])
    prefill(b, [1, 2, 3])
    with pytest.raises(mai.SiError, match="capacity exhausted") as e:
        a.verify_many([5, 6, 7, 8], [3, 4, 5, 6])
    assert e.value.status == mai.SI_E_STATE
    ids, _ = a.verify_many([5, 6, 7], [3, 4, 5])
    ids_b, _ = b.verify_many([5, 6, 7], [3, 4, 5])
    assert ids == ids_b
    with pytest.raises(mai.SiError, match="1..8 tokens"):
        a.verify_many(list(range(9)), list(range(9)))
    a.close()
    b.close()


def test_snapshot_restore_rolls_a_speculative_window_back(mai, ctx):
    """The speculative probes' loop (si-qwen35-spec-probe.rs:155-169):
    snapshot the states, verify a window, restore. Decoding then continues
    like a model that never saw the window, and the snapshot restores again."""
    cfg = small_config(mai)
    a, b = mai.Model(ctx, cfg, seed=13), mai.Model(ctx, cfg, seed=13)
    prompt = [7, 70, 700]
    prefill(a, prompt)
    prefill(b, prompt)
    pos = len(prompt)
    gc.collect()  # no earlier test's objects are freed inside the measured span
    before = ctx.stats()["current_allocated_bytes"]
    snap = a.snapshot_states()
    assert ctx.stats()["current_allocated_bytes"] == before + a.plan()["state_bytes"]
    window = [11, 12, 13, 14, 15]
    positions = list(range(pos, pos + len(window)))
    a.verify_many(window, positions)
    a.restore_states(snap)
    # the window's keys and values stay in the cache past the restored token
    # count; attention never reads them, so ids are exact and logits agree
    for k, tok in enumerate([11, 12, 99, 5]):
        na, la = a.decode_token(tok, pos + k)
        nb, lb = b.decode_token(tok, pos + k)
        assert na == nb, k
        assert rel_l2(la, lb) < 1e-6, k
    a.restore_states(snap)
    b.reset()
    prefill(b, prompt)
    ids_a, lo_a = a.verify_many(window, positions, want_logits=True)
    ids_b, lo_b = b.verify_many(window, positions, want_logits=True)
    assert ids_a == ids_b
    assert max(rel_l2(lo_a[k], lo_b[k]) for k in range(len(window))) < 1e-6
    snap.close()
    assert ctx.stats()["current_allocated_bytes"] == before
    a.close()
    b.close()


def test_snapshot_of_another_layout_is_refused(mai, ctx):
    """restore_states refuses a snapshot of a different depth
    (qwen35_runtime.rs:1768-1772) and leaves the model usable."""
    a = mai.Model(ctx, small_config(mai), seed=2)
    b = mai.Model(ctx, small_config(mai, layers=4), seed=2)
    snap = b.snapshot_states()
    with pytest.raises(mai.SiError, match="snapshot depth does not match") as e:
        a.restore_states(snap)
    assert e.value.status == mai.SI_E_INVALID
    ref = mai.Model(ctx, small_config(mai), seed=2)
    assert a.decode_token(3, 0)[0] == ref.decode_token(3, 0)[0]
    snap.close()
    for m in (a, b, ref):
        m.close()
