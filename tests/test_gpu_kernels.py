"""GPU parity of every hot-path kernel against the CPU oracle, through the
C ABI. Dequant is bit-exact; matvec / DeltaNet / attention within 1e-5
relative L2 (the tolerance BASELINE.json's north star states)."""
import math

import numpy as np
import pytest

import oracle as O
from helpers import random_blocks, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.mark.parametrize("ty", [12, 13, 14])
def test_dequant_bit_exact_random(ctx, ty):
    rng = np.random.default_rng(100 + ty)
    blocks = random_blocks(rng, ty, 3000)
    n = 3000 * 256
    got = ctx.dequantize(ty, blocks, n)
    ref = O.dequantize(ty, blocks, n)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("ty", [12, 13, 14])
def test_dequant_bit_exact_special_scales(ctx, ty):
    # subnormal, zero, negative and large fp16 d/dmin values
    rng = np.random.default_rng(7)
    blocks = random_blocks(rng, ty, 64).reshape(64, -1)
    specials = [0x0001, 0x03FF, 0x0000, 0x8000, 0x8001, 0x7BFF, 0xFBFF, 0x3C00]
    for i in range(64):
        v = specials[i % len(specials)]
        if ty == 14:
            blocks[i, 208], blocks[i, 209] = v & 0xFF, v >> 8
        else:
            blocks[i, 0], blocks[i, 1] = v & 0xFF, v >> 8
            w = specials[(i // 8) % len(specials)]
            blocks[i, 2], blocks[i, 3] = w & 0xFF, w >> 8
    blocks = blocks.reshape(-1)
    got = ctx.dequantize(ty, blocks, 64 * 256)
    ref = O.dequantize(ty, blocks, 64 * 256)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_kats(ctx):  # quant.rs:213-280 through the GPU
    b = np.zeros(144, np.uint8)
    b[0:2] = [0, 0x3C]
    b[4:16] = 1
    b[16:] = 0x10
    v = ctx.dequantize(12, b, 256).reshape(4, 64)
    assert np.all(v[:, :32] == 0) and np.all(v[:, 32:] == 1)
    b6 = np.zeros(210, np.uint8)
    b6[208:210] = [0, 0x3C]
    b6[:128] = 0x21
    b6[128:192] = 0xE4
    b6[192:208] = 1
    v6 = ctx.dequantize(14, b6, 256).reshape(2, 4, 32)
    assert np.all(v6[:, 0] == -31) and np.all(v6[:, 1] == -15) and np.all(v6[:, 2] == 2) and np.all(v6[:, 3] == 18)


def test_dequant_rejects_bad_shapes(ctx):  # quant.rs:233-238
    import mai_b200 as M
    with pytest.raises(M.SiError, match="multiple of 256"):
        ctx.dequantize(12, np.zeros(144, np.uint8), 255)
    with pytest.raises(M.SiError, match="expected 144"):
        ctx.dequantize(12, np.zeros(143, np.uint8), 256)


MV_SHAPES = [(1, 256), (2, 512), (17, 768), (333, 1280), (1000, 5120), (64, 17408)]


@pytest.mark.parametrize("ty", [12, 13, 14])
@pytest.mark.parametrize("rows,cols", MV_SHAPES)
def test_matvec_matches_oracle(ctx, ty, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols + ty)
    w = random_blocks(rng, ty, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    got = ctx.gguf_quant_matvec_bytes(ty, w, rows, cols, x)
    ref = O.matvec(ty, w, rows, cols, x)
    assert rel_l2(got, ref) < TOL
    # per-row check too: no row may be far off
    scale = np.abs(ref).max() + 1e-30
    assert np.max(np.abs(got - ref)) / scale < 1e-5


def test_q4k_matvec_full_config1(ctx):  # 17408 x 5120
    rng = np.random.default_rng(1)
    rows, cols = 17408, 5120
    w = random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    got = ctx.q4_k_matvec(w, rows, cols, x)
    ref = O.matvec(12, w, rows, cols, x)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("rows,cols", [
    (2368, 5120), (4096, 5120), (4736, 5120), (7104, 5120), (9472, 5120), (11840, 5120), (14208, 2560),
    (16576, 1024), (5000, 5120), (5120, 17408), (16, 256), (300, 256), (12288, 5120), (34816, 512),
])
def test_q4k_tensor_core_matvec_every_split(ctx, rows, cols):
    """Plain Q4_K matvecs of 4096 rows and more go to the tensor-core kernel;
    these shapes give a CTA 1..8 row groups (12..1 warps per group), ragged
    last groups, 2..68 column blocks, and smaller ones that stay on the
    CUDA-core kernel."""
    rng = np.random.default_rng(rows + cols)
    w = random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    assert rel_l2(ctx.q4_k_matvec(w, rows, cols, x), O.matvec(12, w, rows, cols, x)) < TOL


def test_q4k_matvec_reference_pattern(ctx):  # metal.rs:7443-7494
    rows, cols = 2, 512
    w = np.zeros(rows * 2 * 144, np.uint8)
    for r in range(rows):
        for b in range(2):
            s = (r * 2 + b) * 144
            w[s:s + 2] = [0, 0x3C]
            w[s + 4:s + 16] = [(i * 13 + 7) & 0xFF for i in range(12)]
            w[s + 16:s + 144] = [0x10 if (i + r + b) % 3 == 0 else 0x21 for i in range(128)]
    x = np.array([((i % 11) - 5.0) / 3.0 for i in range(cols)], np.float32)
    got = ctx.q4_k_matvec(w, rows, cols, x)
    ref = O.matvec(12, w, rows, cols, x)
    assert np.all(np.abs(got - ref) < 1e-4)


def test_q5_q6_reference_pattern(ctx):  # metal.rs:7563-7602
    x = np.array([((i % 13) - 6.0) / 5.0 for i in range(256)], np.float32)
    q5 = np.zeros(176, np.uint8)
    q5[0:2] = [0, 0x3C]
    q5[4:16] = 1
    q5[16:48] = 0xFF
    q5[48:] = 0x10
    assert abs(ctx.q5_k_matvec(q5, 1, 256, x)[0] - O.matvec(13, q5, 1, 256, x)[0]) < 1e-4
    q6 = np.zeros(210, np.uint8)
    q6[208:210] = [0, 0x3C]
    q6[:128] = 0x21
    q6[128:192] = 0xE4
    q6[192:208] = 1
    assert abs(ctx.q6_k_matvec(q6, 1, 256, x)[0] - O.matvec(14, q6, 1, 256, x)[0]) < 1e-4


def test_matvec_rejects_bad_shapes(ctx):  # metal.rs:3847-3858
    import mai_b200 as M
    with pytest.raises(M.SiError, match="Q4_K matvec dimensions are invalid"):
        ctx.q4_k_matvec(np.zeros(144, np.uint8), 1, 255, np.zeros(255, np.float32))
    with pytest.raises(M.SiError, match="Q4_K matvec byte length is invalid"):
        ctx.q4_k_matvec(np.zeros(143, np.uint8), 1, 256, np.zeros(256, np.float32))


def test_retained_and_grouped_weights(ctx):  # metal.rs:3923, 4652
    rng = np.random.default_rng(5)
    cols = 1024
    shapes = [300, 64, 1]
    ws = [random_blocks(rng, 12, r * cols // 256) for r in shapes]
    x = rng.normal(0, 1, cols).astype(np.float32)
    handles = [ctx.upload_quant_weight_private(w, 12) for w in ws]
    outs = ctx.gguf_quant_matvec_many_weights([(h, r, cols) for h, r in zip(handles, shapes)], x)
    for o, w, r in zip(outs, ws, shapes):
        assert rel_l2(o, O.matvec(12, w, r, cols, x)) < TOL
    single = ctx.gguf_quant_matvec_weight(handles[0], shapes[0], cols, x)
    assert np.array_equal(single, outs[0])
    mapped = ctx.bind_quant_weight_mapped(ws[1], 12)
    assert np.array_equal(ctx.gguf_quant_matvec_weight(mapped, shapes[1], cols, x), outs[1])
    for h in handles + [mapped]:
        ctx.free_weight(h)


def test_fused_gate_up_matches_oracle(ctx):
    rng = np.random.default_rng(9)
    rows, cols = 2176, 5120
    g = random_blocks(rng, 12, rows * cols // 256)
    u = random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    assert rel_l2(ctx.q4_k_fused_gate_up(g, u, rows, cols, x), O.fused_gate_up(g, u, rows, cols, x)) < TOL


@pytest.mark.parametrize("rows", [17408, 17400, 9000])
def test_fused_gate_up_tensor_core_two_ctas_per_sm(ctx, rows):
    """SwiGLU pairs of more row groups than four per SM (the 27B gate/up,
    17,408 x 5,120, and ragged variants) run on the tensor cores at two CTAs
    per SM, each staging at most four gate and four up groups."""
    rng = np.random.default_rng(rows)
    cols = 5120
    g = random_blocks(rng, 12, rows * cols // 256)
    u = random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    assert rel_l2(ctx.q4_k_fused_gate_up(g, u, rows, cols, x), O.fused_gate_up(g, u, rows, cols, x)) < TOL


def test_fused_gate_up_reference_pattern(ctx):  # metal.rs:7496-7540
    rows, cols = 2, 256
    gate = np.zeros(rows * 144, np.uint8)
    up = np.zeros(rows * 144, np.uint8)
    for r in range(rows):
        s = r * 144
        gate[s:s + 2] = [0, 0x3C]
        up[s:s + 2] = [0, 0x38]
        gate[s + 4:s + 16] = 7
        up[s + 4:s + 16] = 11
        gate[s + 16:s + 144] = 0x21
        up[s + 16:s + 144] = 0x12
    x = np.array([((i % 17) - 8.0) / 5.0 for i in range(cols)], np.float32)
    got = ctx.q4_k_fused_gate_up(gate, up, rows, cols, x)
    assert np.all(np.abs(got - O.fused_gate_up(gate, up, rows, cols, x)) < 1e-4)


def test_fused_mlp_config2_shape(ctx):
    rng = np.random.default_rng(2)
    H, I = 5120, 17408
    g = random_blocks(rng, 12, I * H // 256)
    u = random_blocks(rng, 12, I * H // 256)
    d = random_blocks(rng, 14, H * I // 256)
    x = rng.normal(0, 1, H).astype(np.float32)
    ws = [ctx.upload_quant_weight_private(a, t) for a, t in ((g, 12), (u, 12), (d, 14))]
    got = ctx.gguf_quant_fused_mlp_weights(ws[0], ws[1], ws[2], I, H, H, x)
    ref = O.fused_mlp(12, g, u, 14, d, I, H, x)
    assert rel_l2(got, ref) < TOL
    for w in ws:
        ctx.free_weight(w)


def test_embedding_row_kat(ctx):  # metal.rs:7542-7561
    row = np.zeros(144, np.uint8)
    row[0:2] = [0, 0x3C]
    row[4:16] = [7, 19, 31, 43, 55, 67, 79, 91, 103, 115, 127, 139]
    row[16:] = 0x21
    assert np.array_equal(ctx.q4_k_embedding_row(row, 256), O.dequantize(12, row, 256))


# ---- Gated DeltaNet primitives --------------------------------------------------
def test_gdn_step_kat(ctx):  # metal.rs:7362-7385 / qwen35.rs:273-288
    out, st = ctx.gated_delta_step([1, 0], [1, 0], [2], [0], [0.5], [0, 0], 1, 2, 1)
    assert abs(out[0] - 1.0) < 1e-5 and np.allclose(st, [1, 0], atol=1e-5)
    out, st = ctx.gated_delta_step([0, 1], [0, 1], [4], [math.log(0.5)], [1.0], st, 1, 2, 1)
    assert abs(out[0] - 4.0) < 1e-5 and np.allclose(st, [0.5, 4.0], atol=1e-5)


def test_gdn_step_random_matches_oracle(ctx):
    rng = np.random.default_rng(11)
    h, d = 48, 128
    q = rng.normal(0, 0.1, h * d).astype(np.float32)
    k = rng.normal(0, 0.1, h * d).astype(np.float32)
    v = rng.normal(0, 1, h * d).astype(np.float32)
    g = -np.log1p(np.exp(rng.normal(0, 1, h))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, h)))).astype(np.float32)
    s = rng.normal(0, 0.1, h * d * d).astype(np.float32)
    o1, s1 = ctx.gated_delta_step(q, k, v, g, beta, s, h, d, d)
    o2, s2 = O.gdn_step(q, k, v, g, beta, s, h, d, d)
    assert rel_l2(o1, o2) < TOL and rel_l2(s1, s2) < TOL
    # and against the reference's parallel formulation (metal.rs:688-740) on
    # the first heads
    n = 4
    o3, s3 = O.gdn_step_parallel(q[:n * d], k[:n * d], v[:n * d], g[:n], beta[:n], s[:n * d * d], n, d, d)
    assert rel_l2(o1[:n * d], o3) < TOL and rel_l2(s1[:n * d * d], s3) < TOL


def test_conv_kat_and_random(ctx):  # metal.rs:7387-7409
    out, st = ctx.causal_conv1d_step([5, 6], [1, 2, 3, 4, 5, 6], [1, 2, 3, 4, -1, 0.5, 1, 2], 2, 4)
    ro, rs = O.causal_conv1d_step([5, 6], [1, 2, 3, 4, 5, 6], [1, 2, 3, 4, -1, 0.5, 1, 2], 2, 4)
    assert np.allclose(out, ro, atol=1e-5) and st.tolist() == rs.tolist()
    rng = np.random.default_rng(3)
    C, K = 10240, 4
    x, s, w = rng.normal(0, 1, C), rng.normal(0, 1, C * 3), rng.normal(0, 0.5, C * K)
    o1, s1 = ctx.causal_conv1d_step(x, s, w, C, K)
    o2, s2 = O.causal_conv1d_step(x, s, w, C, K)
    assert rel_l2(o1, o2) < TOL and np.array_equal(s1, s2)


def test_norm_kats_and_random(ctx):  # metal.rs:7411-7441
    x = np.array([1, 2, -1, 3], np.float32)
    assert np.allclose(ctx.rms_norm_gated(x, [0, 1, -1, 0.5], [1, 0.5], 2, 2, 1e-6),
                       O.gated_rms_norm(x, [0, 1, -1, 0.5], [1, 0.5], 2, 2, 1e-6), atol=1e-5)
    assert np.allclose(ctx.rms_norm_heads(x, [0.25, -0.5], 2, 2, 1e-6),
                       O.rms_norm_heads(x, [0.25, -0.5], 2, 2, 1e-6), atol=1e-5)
    rng = np.random.default_rng(4)
    c, z, w = rng.normal(0, 3, 6144), rng.normal(0, 2, 6144), rng.normal(1, 0.1, 128)
    assert rel_l2(ctx.rms_norm_gated(c, z, w, 48, 128, 1e-6), O.gated_rms_norm(c, z, w, 48, 128, 1e-6)) < TOL
    h, wh = rng.normal(0, 5, 5120), rng.normal(0, 0.1, 5120)
    assert rel_l2(ctx.rms_norm_heads(h, wh, 1, 5120, 1e-6), O.rms_norm_heads(h, wh, 1, 5120, 1e-6)) < TOL


# ---- attention ---------------------------------------------------------------------
def test_rope_kat_and_large_position(ctx):  # metal.rs:8252-8276
    x = np.array([1, 2, 3, 4], np.float32)
    assert np.allclose(ctx.rope(x, 1, 4, 3, 1e6), O.rope(x, 1, 4, 3, 1e6), atol=1e-5)
    rng = np.random.default_rng(6)
    y = rng.normal(0, 1, 24 * 64).astype(np.float32)
    assert rel_l2(ctx.rope(y, 24, 64, 8192, 1e7), O.rope(y, 24, 64, 8192, 1e7)) < TOL


def test_attention_kat(ctx):  # metal.rs:8278-8364
    import mai_b200 as M
    q = np.array([1, 0, 0, 1, 1, 1, 1, -1], np.float32)
    keys = np.array([1, 0, 0, 1, 1, 1, 1, -1], np.float32)
    vals = np.array([10, 0, 0, 20, 30, 0, 0, 40], np.float32)
    nk, nv = np.array([1, -1, 1, 1], np.float32), np.array([50, 0, 0, 60], np.float32)
    got = ctx.attention_decode(M.AttentionDecodeInput(q, keys, vals, nk, nv, 4, 2, 2, 2, 2))
    assert np.allclose(got, O.attention_decode(q, keys, vals, nk, nv, 4, 2, 2, 2, 2), atol=1e-5)


def test_attention_capacity_strided(ctx):  # metal.rs:8366-8404
    import mai_b200 as M
    kc = np.zeros(8, np.float32)
    vc = np.zeros(8, np.float32)
    kc[0:4] = [1, 0, 0, 1]
    vc[0:4] = [10, 0, 20, 0]
    q = np.array([1, 1], np.float32)
    a = ctx.attention_decode(M.AttentionDecodeInput(q, kc, vc, [1, -1], [30, 0], 1, 1, 2, 2, 4))
    b = ctx.attention_decode(M.AttentionDecodeInput(q, kc[:4], vc[:4], [1, -1], [30, 0], 1, 1, 2, 2, 2))
    assert np.allclose(a, b, atol=1e-6)


@pytest.mark.parametrize("cached", [0, 1, 255, 256, 257, 8192])
def test_attention_bf16_cache_config4(ctx, cached):  # BASELINE config 4 shapes
    import mai_b200 as M
    rng = np.random.default_rng(cached + 1)
    qh, kvh, hd, cap = 24, 4, 256, 8192
    q = (rng.normal(0, 1, qh * hd) / 4).astype(np.float32)
    kc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    vc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    nk = rng.normal(0, 1, kvh * hd).astype(np.float32)
    nv = rng.normal(0, 1, kvh * hd).astype(np.float32)
    got = ctx.attention_decode(M.AttentionDecodeInput(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap))
    ref = O.attention_decode(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("qh,kvh,hd,cached,cap,kscale", [
    (8, 8, 128, 63, 64, 1.0),      # group 1, one partial tile
    (12, 4, 128, 64, 100, 1.0),    # group 3, exactly one tile
    (20, 4, 128, 65, 65, 3.0),     # group 5, tile + 1 row, full cache
    (16, 2, 128, 1000, 1024, 3.0),  # group 8, many splits
    (4, 2, 256, 700, 800, 3.0),    # group 2
    (28, 4, 256, 5000, 5001, 2.0),  # group 7, uneven splits
    (6, 1, 256, 3, 16, 1.0),       # fewer tokens than one tile
])
def test_attention_bf16_bulk_kernel_shapes(ctx, qh, kvh, hd, cached, cap, kscale):
    """Head dims 128/256 and every GQA group size through the bulk-copy split
    kernel; large key scales move the running max between tiles."""
    import mai_b200 as M
    rng = np.random.default_rng(qh * 1000 + cached)
    q = (rng.normal(0, 1, qh * hd) / 4).astype(np.float32)
    kc = O.f32_to_bf16((kscale * rng.normal(0, 1, kvh * cap * hd)).astype(np.float32))
    vc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    nk = rng.normal(0, 1, kvh * hd).astype(np.float32)
    nv = rng.normal(0, 1, kvh * hd).astype(np.float32)
    got = ctx.attention_decode(M.AttentionDecodeInput(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap))
    ref = O.attention_decode(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap)
    assert rel_l2(got, ref) < TOL


def test_argmax_semantics(ctx):  # runtime.rs:4301-4309
    assert ctx.argmax([1.0, 3.0, 3.0, 2.0]) == 2
    assert ctx.argmax([np.nan, np.inf, 0.5, -np.inf]) == 2
    assert ctx.argmax([0.0, -0.0]) == 0
    assert ctx.argmax([-0.0, 0.0, -0.0]) == 1
    rng = np.random.default_rng(8)
    v = rng.normal(0, 1, 248320).astype(np.float32)
    v[[5, 100000, 248319]] = v.max() + 1
    assert ctx.argmax(v) == O.argmax(v) == 248319
    import mai_b200 as M
    with pytest.raises(M.SiError, match="no finite"):
        ctx.argmax([np.nan, np.inf])


@pytest.mark.parametrize("rows,cols", [
    (256, 1024), (300, 3072), (1000, 5120), (4099, 1024), (5120, 17408), (2560, 17408), (640, 18432),
    (5121, 12288), (20000, 13312), (300, 12288), (3000, 256), (4096, 3072), (2048, 1024), (17408, 5120),
    (1024, 5120), (2049, 6144),
])
def test_q6k_tensor_core_matvec_shapes(ctx, rows, cols):
    """Q6_K matvecs whose rows hold a multiple of 4 super-blocks (at most 72)
    with 2,048 rows and more, or 64 blocks and more, run on the tensor cores
    (qmv_tc6_kernel): rows 8 mod 16 bytes long (4, 12, 20, 52, 68 blocks:
    even/odd row maps) and 16-byte multiples (8, 24, 72 blocks), 32-row groups
    shared by neighbouring CTAs, ragged last groups (5121, 2049 rows), one
    chunk per row (4 blocks). The other shapes stay on the CUDA-core kernel
    and must agree just the same."""
    rng = np.random.default_rng(rows * 3 + cols)
    w = random_blocks(rng, 14, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    ref = O.matvec(14, w, rows, cols, x)
    got = ctx.q6_k_matvec(w, rows, cols, x)
    assert rel_l2(got, ref) < TOL
    assert np.max(np.abs(got - ref)) / np.abs(ref).max() < 1e-5


def test_q6k_head_shape_rows_match_oracle(ctx):
    """The 27B output head's shape (248320 x 5120 Q6_K, 1.04 GB): rows sampled
    at the start, middle and end against the oracle."""
    import torch
    rng = np.random.default_rng(248320)
    rows, cols = 248320, 5120
    w = random_blocks(rng, 14, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    wd = torch.from_numpy(np.concatenate([w, np.zeros(64, np.uint8)])).cuda()
    y = torch.empty(rows, device="cuda")
    ctx.qmatvec_dev(14, wd, rows, cols, torch.from_numpy(x).cuda(), y)
    torch.cuda.synchronize()
    yc = y.cpu().numpy()
    rb = cols // 256 * 210
    for r0 in (0, rows // 2 + 8, rows - 200):
        ref = O.matvec(14, w[r0 * rb:(r0 + 200) * rb], 200, cols, x)
        assert rel_l2(yc[r0:r0 + 200], ref) < TOL, r0


def test_q6k_split_groups_on_concurrent_streams(ctx):
    """Tensor-core Q6_K matvecs queued on two streams at once: each stream
    finishes its straddling groups in its own scratch slot, so neither run
    disturbs the other's rows."""
    import torch
    rng = np.random.default_rng(77)
    rows, cols = 5120, 17408
    ws = [random_blocks(rng, 14, rows * cols // 256) for _ in range(2)]
    xs = [rng.normal(0, 1, cols).astype(np.float32) for _ in range(2)]
    wd = [torch.from_numpy(np.concatenate([w, np.zeros(64, np.uint8)])).cuda() for w in ws]
    xd = [torch.from_numpy(x).cuda() for x in xs]
    ys = [torch.empty(rows, device="cuda") for _ in range(2)]
    ref = [ctx.q6_k_matvec(w, rows, cols, x) for w, x in zip(ws, xs)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for _ in range(20):
        for k in range(2):
            ctx.qmatvec_dev(14, wd[k], rows, cols, xd[k], ys[k], streams[k].cuda_stream)
    torch.cuda.synchronize()
    for k in range(2):
        assert np.array_equal(ys[k].cpu().numpy(), ref[k])
