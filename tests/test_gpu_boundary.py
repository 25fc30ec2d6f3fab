"""The rest of MetalContext's surface the runtime binds (metal.rs:2374-2378,
2585-2637, 3785-3811, 4780-4990, 5003-5015): staged layers promoted to device
memory or bound in host memory, grouped matvecs over bytes and F32 matrices,
file-backed row-range matvecs and embeddings, allocation sampling; each
against the oracle."""
import numpy as np
import pytest

import gguf_writer as W
import oracle as O
from helpers import random_blocks, rel_l2

pytestmark = pytest.mark.gpu

Q4, Q5, Q6 = 12, 13, 14


def test_staged_layer_private_and_shared(mai, ctx):
    rng = np.random.default_rng(1)
    a = random_blocks(rng, Q4, 512 * 1024 // 256)   # 512 x 1024 Q4_K
    b = random_blocks(rng, Q6, 256 * 512 // 256)    # 256 x 512 Q6_K
    c = random_blocks(rng, Q5, 64 * 256 // 256)     # 64 x 256 Q5_K
    # packed with unaligned offsets, as a staging thread may pack them
    packed = np.concatenate([np.zeros(3, np.uint8), a, np.zeros(5, np.uint8), b, c])
    o_a, o_b = 3, 3 + a.size + 5
    o_c = o_b + b.size
    ranges = {"blk.0.ffn_gate.weight": (o_a, o_a + a.size), "blk.0.ffn_down.weight": (o_b, o_b + b.size),
              "blk.0.attn_qkv.weight": (o_c, o_c + c.size)}
    x1024 = rng.normal(0, 1, 1024).astype(np.float32)
    x512 = rng.normal(0, 1, 512).astype(np.float32)
    x256 = rng.normal(0, 1, 256).astype(np.float32)
    for upload in (True, False):
        layer = ctx.upload_staged_layer_private(packed, ranges) if upload else ctx.bind_staged_layer_shared(packed, ranges)
        wa = layer.quant_weight("blk.0.ffn_gate.weight", Q4)
        wb = layer.quant_weight("blk.0.ffn_down.weight", Q6)
        wc = layer.quant_weight("blk.0.attn_qkv.weight", Q5)
        assert rel_l2(ctx.gguf_quant_matvec_weight(wa, 512, 1024, x1024), O.matvec(Q4, a, 512, 1024, x1024)) < 1e-5
        assert rel_l2(ctx.gguf_quant_matvec_weight(wb, 256, 512, x512), O.matvec(Q6, b, 256, 512, x512)) < 1e-5
        assert rel_l2(ctx.gguf_quant_matvec_weight(wc, 64, 256, x256), O.matvec(Q5, c, 64, 256, x256)) < 1e-5
        with pytest.raises(mai.SiError, match="unknown staged tensor"):
            layer.quant_weight("blk.0.nope", Q4)
        ctx.free_weight(wa)  # a view freed early is not freed again by the layer
        layer.close()
    with pytest.raises(mai.SiError, match="cannot promote an empty staged Qwen layer"):
        ctx.upload_staged_layer_private(np.zeros(0, np.uint8), {})
    with pytest.raises(mai.SiError, match="out of bounds"):
        ctx.upload_staged_layer_private(packed, {"x": (0, packed.size + 1)})


def test_grouped_matvecs_over_bytes_and_f32(mai, ctx):
    rng = np.random.default_rng(2)
    cols = 768
    ts = [(Q4, random_blocks(rng, Q4, 300 * cols // 256), 300), (Q6, random_blocks(rng, Q6, 40 * cols // 256), 40),
          (Q5, random_blocks(rng, Q5, 5 * cols // 256), 5)]
    x = rng.normal(0, 1, cols).astype(np.float32)
    outs = ctx.gguf_quant_matvec_many_bytes([(t, w, r, cols) for t, w, r in ts], x)
    for (t, w, r), y in zip(ts, outs):
        assert rel_l2(y, O.matvec(t, w, r, cols, x)) < 1e-5
    with pytest.raises(mai.SiError, match="at least one tensor"):
        ctx.gguf_quant_matvec_many_bytes([], x)
    for c2 in (5120, 130):
        ms = [rng.normal(0, 0.02, (48, c2)).astype(np.float32), rng.normal(0, 0.02, (7, c2)).astype(np.float32)]
        x2 = rng.normal(0, 1, c2).astype(np.float32)
        for m, y in zip(ms, ctx.f32_matvec_many(ms, x2)):
            assert rel_l2(y, m.astype(np.float64) @ x2.astype(np.float64)) < 1e-5


def test_file_backed_rows_and_embedding(mai, ctx, tmp_path):
    rng = np.random.default_rng(3)
    q5 = random_blocks(rng, Q5, 100 * 512 // 256)
    f32 = rng.normal(0, 0.1, (40, 96)).astype(np.float32)
    emb = random_blocks(rng, Q4, 50 * 256 // 256)
    path = tmp_path / "t.gguf"
    W.write(path, [("general.architecture", W.STRING, "qwen35")],
            [("w", [512, 100], Q5, q5.tobytes()), ("f", [96, 40], 0, f32.tobytes()),
             ("token_embd.weight", [256, 50], Q4, emb.tobytes())])
    x = rng.normal(0, 1, 512).astype(np.float32)
    x96 = rng.normal(0, 1, 96).astype(np.float32)
    with mai.GgufFile(path) as g:
        y = ctx.gguf_matvec_tensor_rows(g, "w", 30, 25, x)
        rb = 512 // 256 * 176
        assert rel_l2(y, O.matvec(Q5, q5[30 * rb:55 * rb], 25, 512, x)) < 1e-5
        yf = ctx.gguf_matvec_tensor_rows(g, "f", 3, 10, x96)
        assert rel_l2(yf, f32[3:13].astype(np.float64) @ x96.astype(np.float64)) < 1e-5
        with pytest.raises(mai.SiError, match="rows are out of range"):
            ctx.gguf_matvec_tensor_rows(g, "w", 90, 11, x)
        e = ctx.q4_k_embedding_tensor(g, "token_embd.weight", 17)
        assert np.array_equal(e.view(np.uint32), O.dequantize(Q4, emb[17 * 144:18 * 144], 256).view(np.uint32))
        with pytest.raises(mai.SiError, match="token id or dimension is invalid"):
            ctx.q4_k_embedding_tensor(g, "token_embd.weight", 50)
        with pytest.raises(mai.SiError, match="rank-2 Q4_K tensor"):
            ctx.q4_k_embedding_tensor(g, "w", 0)


def test_sample_allocated_folds_into_the_peak(mai, ctx):
    ctx.reset_peaks()
    before = ctx.stats()
    ctx.sample_allocated()
    after = ctx.stats()
    assert after["peak_allocated_bytes"] >= before["current_allocated_bytes"]


def test_grouped_matvec_over_file_tensors(mai, ctx, tmp_path):
    """gguf_quant_matvec_many_tensors (metal.rs:4532-4638): mixed K-quant
    tensors of one file against one input, and the reference's refusals."""
    rng = np.random.default_rng(12)
    cols = 512
    mats = {"q4": (Q4, 70), "q5": (Q5, 33), "q6": (Q6, 128)}
    blobs = {k: random_blocks(rng, ty, rows * cols // 256) for k, (ty, rows) in mats.items()}
    f32 = rng.normal(0, 1, (8, cols)).astype(np.float32)
    path = tmp_path / "g.gguf"
    W.write(path, [("general.architecture", W.STRING, "qwen35")],
            [(k, [cols, rows], ty, blobs[k].tobytes()) for k, (ty, rows) in mats.items()]
            + [("f", [cols, 8], 0, f32.tobytes()), ("narrow", [256, 4], Q4, random_blocks(rng, Q4, 4).tobytes())])
    x = rng.normal(0, 1, cols).astype(np.float32)
    with mai.GgufFile(path) as g:
        ys = ctx.gguf_quant_matvec_many_tensors(g, ["q4", "q5", "q6"], x)
        for (k, (ty, rows)), y in zip(mats.items(), ys):
            assert rel_l2(y, O.matvec(ty, blobs[k], rows, cols, x)) < 1e-5, k
        with pytest.raises(mai.SiError, match="requires at least one tensor"):
            ctx.gguf_quant_matvec_many_tensors(g, [], x)
        with pytest.raises(mai.SiError, match="input length is invalid"):
            ctx.gguf_quant_matvec_many_tensors(g, ["q4"], x[:256])
        with pytest.raises(mai.SiError, match="shapes or types differ"):
            ctx.gguf_quant_matvec_many_tensors(g, ["q4", "f"], x)
        with pytest.raises(mai.SiError, match="shapes or types differ"):
            ctx.gguf_quant_matvec_many_tensors(g, ["q4", "narrow"], x)


def test_file_staging_pipeline(mai, ctx, tmp_path):
    """stage_qwen35_layer_packed -> upload_staged_qwen_layer_private ->
    matvec, the reference's staging-worker path, from a GGUF file."""
    rng = np.random.default_rng(21)
    q4 = random_blocks(rng, Q4, 96 * 512 // 256)
    q6 = random_blocks(rng, Q6, 512 * 256 // 256)
    other = random_blocks(rng, Q4, 64 * 512 // 256)
    path = tmp_path / "s.gguf"
    W.write(path, [("general.architecture", W.STRING, "qwen35")],
            [("blk.2.ffn_up.weight", [512, 96], Q4, q4.tobytes()), ("blk.3.ffn_up.weight", [512, 64], Q4, other.tobytes()),
             ("blk.2.ffn_down.weight", [256, 512], Q6, q6.tobytes())], alignment=256)
    x512 = rng.normal(0, 1, 512).astype(np.float32)
    x256 = rng.normal(0, 1, 256).astype(np.float32)
    with mai.GgufFile(path) as g:
        packed, ranges = g.stage_layer_packed(2)
    assert sorted(ranges) == ["blk.2.ffn_down.weight", "blk.2.ffn_up.weight"]
    layer = ctx.upload_staged_layer_private(packed, ranges)
    up = layer.quant_weight("blk.2.ffn_up.weight", Q4)
    down = layer.quant_weight("blk.2.ffn_down.weight", Q6)
    assert rel_l2(ctx.gguf_quant_matvec_weight(up, 96, 512, x512), O.matvec(Q4, q4, 96, 512, x512)) < 1e-5
    assert rel_l2(ctx.gguf_quant_matvec_weight(down, 512, 256, x256), O.matvec(Q6, q6, 512, 256, x256)) < 1e-5
    layer.close()


def test_dequantize_file_tensor(mai, ctx, tmp_path):  # model.rs:792-850
    rng = np.random.default_rng(5)
    q5 = random_blocks(rng, Q5, 24)
    q6 = random_blocks(rng, Q6, 8)
    path = tmp_path / "d.gguf"
    W.write(path, [("general.architecture", W.STRING, "qwen35")],
            [("a", [512, 12], Q5, q5.tobytes()), ("b", [256, 8], Q6, q6.tobytes())])
    with mai.GgufFile(path) as g:
        a = ctx.dequantize_gguf_tensor(g, "a", Q5)
        assert np.array_equal(a.view(np.uint32), O.dequantize(Q5, q5, 512 * 12).view(np.uint32))
        b = ctx.dequantize_gguf_tensor(g, "b", Q6)
        assert np.array_equal(b.view(np.uint32), O.dequantize(Q6, q6, 256 * 8).view(np.uint32))
        with pytest.raises(mai.SiError, match="GGUF tensor a is not Q4_K \\(type 13\\)"):
            ctx.dequantize_gguf_tensor(g, "a", Q4)
        with pytest.raises(mai.SiError, match="GGUF tensor b has type 14; expected 13"):
            ctx.dequantize_gguf_tensor(g, "b", Q5)
