"""The oracle replays the reference's own known-answer tests (CPU only).

Each test cites the reference test it restates; passing them pins the C++
restatement in oracle/oracle.cpp to the reference's CPU code.
"""
import math

import numpy as np
import pytest

import oracle as O


def f16(v):
    return np.array([v], np.float16).view(np.uint16)[0]


def q4k_block():
    b = np.zeros(144, np.uint8)
    b[0:2] = [0x00, 0x3C]
    return b


def test_q4k_one_block_kat():  # quant.rs:213-231
    b = q4k_block()
    b[4:16] = 1
    b[16:] = 0x10
    v = O.dequantize(O.GGML_Q4_K, b, 256)
    for g in v.reshape(4, 64):
        assert np.all(g[:32] == 0.0) and np.all(g[32:] == 1.0)


def test_q4k_rejects_shape_and_byte_mismatch():  # quant.rs:233-238
    with pytest.raises(O.OracleError):
        O.dequantize(O.GGML_Q4_K, np.zeros(144, np.uint8), 255)
    with pytest.raises(O.OracleError):
        O.dequantize(O.GGML_Q4_K, np.zeros(143, np.uint8), 256)
    with pytest.raises(O.OracleError):
        O.dequantize(O.GGML_Q4_K, np.zeros(145, np.uint8), 256)
    with pytest.raises(O.OracleError):
        O.dequantize(O.GGML_Q4_K, np.zeros(0, np.uint8), 0)


def test_q5k_high_bits_kat():  # quant.rs:240-259
    b = np.zeros(176, np.uint8)
    b[0:2] = [0x00, 0x3C]
    b[4:16] = 1
    b[48:] = 0x10
    b[16:48] = 0xFF
    v = O.dequantize(O.GGML_Q5_K, b, 256)
    for g in v.reshape(4, 64):
        assert np.all(g[:32] == 16.0) and np.all(g[32:] == 17.0)


def test_q6k_high_bits_and_scales_kat():  # quant.rs:261-280
    b = np.zeros(210, np.uint8)
    b[208:210] = [0x00, 0x3C]
    b[:128] = 0x21
    b[128:192] = 0xE4
    b[192:208] = 1
    v = O.dequantize(O.GGML_Q6_K, b, 256)
    for c in v.reshape(2, 128):
        assert np.all(c[0:32] == -31.0)
        assert np.all(c[32:64] == -15.0)
        assert np.all(c[64:96] == 2.0)
        assert np.all(c[96:128] == 18.0)


def test_f16_subnormal_and_special_decode():  # quant.rs:187-207
    # d is a subnormal f16, dmin is +inf: exercises both non-normal branches.
    b = q4k_block()
    b[0:2] = [0x01, 0x00]          # smallest subnormal 2^-24
    b[2:4] = [0x00, 0x00]
    b[4:16] = 1
    b[16:] = 0x11
    v = O.dequantize(O.GGML_Q4_K, b, 256)
    assert v[0] == np.float32(2.0 ** -24)
    b[0:2] = [0x00, 0x7C]          # +inf
    v = O.dequantize(O.GGML_Q4_K, b, 256)
    assert np.isinf(v[0])


def silu(x):
    return x / (1.0 + math.exp(-x))


def test_gated_rms_norm_kat():  # qwen35.rs:232-244
    x = np.array([1.0, 2.0, -1.0, 3.0], np.float32)
    g = np.array([0.0, 1.0, -1.0, 0.5], np.float32)
    w = np.array([1.0, 0.5], np.float32)
    o = O.gated_rms_norm(x, g, w, 2, 2, 1e-6)
    inv0 = 1.0 / math.sqrt(2.5 + 1e-6)
    inv1 = 1.0 / math.sqrt(5.0 + 1e-6)
    assert abs(o[0]) < 1e-6
    assert abs(o[1] - 2.0 * inv0 * 0.5 * silu(1.0)) < 1e-6
    assert abs(o[2] - (-1.0) * inv1 * silu(-1.0)) < 1e-6


def test_head_rms_norm_kat():  # qwen35.rs:246-257
    x = np.array([1.0, 2.0, -1.0, 3.0], np.float32)
    w = np.array([0.25, -0.5], np.float32)
    o = O.rms_norm_heads(x, w, 2, 2, 1e-6)
    inv0 = 1.0 / math.sqrt(2.5 + 1e-6)
    inv1 = 1.0 / math.sqrt(5.0 + 1e-6)
    assert abs(o[0] - 1.0 * inv0 * 1.25) < 1e-6
    assert abs(o[1] - 2.0 * inv0 * 0.5) < 1e-6
    assert abs(o[2] - (-1.0) * inv1 * 1.25) < 1e-6


def test_causal_conv_kat():  # qwen35.rs:259-271
    state = np.array([1, 2, 3, 4, 5, 6], np.float32)
    x = np.array([5, 6], np.float32)
    w = np.array([1, 2, 3, 4, -1, 0.5, 1, 2], np.float32)
    o, st = O.causal_conv1d_step(x, state, w, 2, 4)
    first = 1 * 1 + 2 * 2 + 3 * 3 + 5 * 4
    second = -4 + 5 * 0.5 + 6 + 6 * 2
    assert abs(o[0] - silu(first)) < 1e-6
    assert abs(o[1] - silu(second)) < 1e-6
    assert st.tolist() == [2, 3, 5, 5, 6, 6]


def test_recurrent_step_two_token_kat():  # qwen35.rs:273-288
    st = np.zeros(2, np.float32)
    o, st = O.gdn_step([1, 0], [1, 0], [2], [0], [0.5], st, 1, 2, 1)
    assert o.tolist() == [1.0]
    assert st.tolist() == [1.0, 0.0]
    o, st = O.gdn_step([0, 1], [0, 1], [4], [math.log(0.5)], [1.0], st, 1, 2, 1)
    assert abs(o[0] - 4.0) < 1e-6
    assert abs(st[0] - 0.5) < 1e-6 and abs(st[1] - 4.0) < 1e-6


def test_rope_kat():  # metal.rs:8252-8276
    x = np.array([1, 2, 3, 4], np.float32)
    theta = np.float32(1e6)
    o = O.rope(x, 1, 4, 3, theta)
    a0 = np.float32(3.0)
    a1 = np.float32(3.0) * np.float32(theta ** -0.5)
    exp = [x[0] * math.cos(a0) - x[1] * math.sin(a0), x[0] * math.sin(a0) + x[1] * math.cos(a0),
           x[2] * math.cos(a1) - x[3] * math.sin(a1), x[2] * math.sin(a1) + x[3] * math.cos(a1)]
    assert np.allclose(o, exp, atol=1e-5)


def attention_expected(q, keys, values, nk, nv, qh, kvh, hd, cached):
    # metal.rs:8314-8357 CPU restatement (numpy float64 is enough at 1e-5).
    scale = 1.0 / math.sqrt(hd)
    out = []
    for h in range(qh):
        kv = h // (qh // kvh)
        qr = q[h * hd:(h + 1) * hd]
        sc = []
        for t in range(cached + 1):
            k = keys[(kv * cached + t) * hd:(kv * cached + t + 1) * hd] if t < cached else nk[kv * hd:(kv + 1) * hd]
            sc.append(float(np.dot(qr, k)) * scale)
        m = max(sc)
        w = [math.exp(s - m) for s in sc]
        z = sum(w)
        for d in range(hd):
            acc = 0.0
            for t in range(cached + 1):
                vr = values[(kv * cached + t) * hd:(kv * cached + t + 1) * hd] if t < cached else nv[kv * hd:(kv + 1) * hd]
                acc += w[t] / z * vr[d]
            out.append(acc)
    return np.array(out)


ATT_Q = np.array([1, 0, 0, 1, 1, 1, 1, -1], np.float32)
ATT_K = np.array([1, 0, 0, 1, 1, 1, 1, -1], np.float32)
ATT_V = np.array([10, 0, 0, 20, 30, 0, 0, 40], np.float32)
ATT_NK = np.array([1, -1, 1, 1], np.float32)
ATT_NV = np.array([50, 0, 0, 60], np.float32)


def test_attention_decode_kat():  # metal.rs:8278-8364
    o = O.attention_decode(ATT_Q, ATT_K, ATT_V, ATT_NK, ATT_NV, 4, 2, 2, 2, 2)
    e = attention_expected(ATT_Q, ATT_K, ATT_V, ATT_NK, ATT_NV, 4, 2, 2, 2)
    assert np.allclose(o, e, atol=1e-5)


def test_attention_capacity_strided_cache():  # metal.rs:8366-8404 + cache.rs:75-98
    cap, hd = 4, 2
    kc = np.zeros(cap * hd, np.float32)
    vc = np.zeros(cap * hd, np.float32)
    kc[0:2], vc[0:2] = [1, 0], [10, 0]
    kc[2:4], vc[2:4] = [0, 1], [20, 0]
    q = np.array([1, 1], np.float32)
    o = O.attention_decode(q, kc, vc, [1, -1], [30, 0], 1, 1, 2, 2, cap)
    compact = O.attention_decode(q, kc[:4], vc[:4], [1, -1], [30, 0], 1, 1, 2, 2, 2)
    assert np.allclose(o, compact, atol=1e-6)


def test_argmax_total_order_last_index():  # runtime.rs:4301-4309
    assert O.argmax([1.0, 3.0, 3.0, 2.0]) == 2
    assert O.argmax([np.nan, np.inf, 0.5, -np.inf]) == 2
    assert O.argmax([0.0, -0.0]) == 0          # +0 > -0 under total_cmp
    assert O.argmax([-0.0, 0.0, -0.0]) == 1
    assert O.argmax([np.nan, np.nan]) == -1


def test_q4k_matvec_pattern_against_dequant():  # metal.rs:7443-7494 expectation
    rows, cols = 2, 512
    w = np.zeros(rows * 2 * 144, np.uint8)
    for r in range(rows):
        for b in range(2):
            s = (r * 2 + b) * 144
            w[s:s + 2] = [0x00, 0x3C]
            w[s + 4:s + 16] = [(i * 13 + 7) & 0xFF for i in range(12)]
            w[s + 16:s + 144] = [0x10 if (i + r + b) % 3 == 0 else 0x21 for i in range(128)]
    x = np.array([((i % 11) - 5.0) / 3.0 for i in range(cols)], np.float32)
    deq = O.dequantize(O.GGML_Q4_K, w, rows * cols).reshape(rows, cols)
    y = O.matvec(O.GGML_Q4_K, w, rows, cols, x)
    ref = [np.float32(0)] * rows
    for r in range(rows):
        s = np.float32(0)
        for c in range(cols):
            s = np.float32(s + np.float32(deq[r, c] * x[c]))
        ref[r] = s
    assert np.array_equal(y, np.array(ref, np.float32))


def test_fused_gate_up_pattern():  # metal.rs:7496-7540 expectation
    rows, cols = 2, 256
    gate = np.zeros(rows * 144, np.uint8)
    up = np.zeros(rows * 144, np.uint8)
    for r in range(rows):
        s = r * 144
        gate[s:s + 2] = [0x00, 0x3C]
        up[s:s + 2] = [0x00, 0x38]
        gate[s + 4:s + 16] = 7
        up[s + 4:s + 16] = 11
        gate[s + 16:s + 144] = 0x21
        up[s + 16:s + 144] = 0x12
    x = np.array([((i % 17) - 8.0) / 5.0 for i in range(cols)], np.float32)
    g = O.matvec(O.GGML_Q4_K, gate, rows, cols, x)
    u = O.matvec(O.GGML_Q4_K, up, rows, cols, x)
    o = O.fused_gate_up(gate, up, rows, cols, x)
    assert np.allclose(o, g / (1 + np.exp(-g)) * u, rtol=1e-6)


# ---- KvCache (cache.rs:173-291) ----------------------------------------------
from oracle.kv_cache import CacheError, KvCache  # noqa: E402


def _addr(a):
    return a.__array_interface__["data"][0]


def test_kv_prefill_lands_in_head_major_capacity_layout():  # cache.rs:177-197
    c = KvCache(2, 2, 3)
    c.append_sequence([1, 2, 3, 4, 5, 6, 7, 8], [10, 20, 30, 40, 50, 60, 70, 80], 2)
    assert c.cached_tokens == 2 and c.remaining_tokens() == 1 and c.active_bytes() == 64
    assert c.keys.tolist() == [1, 2, 5, 6, 0, 0, 3, 4, 7, 8, 0, 0]
    assert c.values[0:4].tolist() == [10, 20, 50, 60] and c.values[6:10].tolist() == [30, 40, 70, 80]


def test_kv_rejects_bad_token_shape_and_capacity_overflow():  # cache.rs:199-207
    c = KvCache(1, 2, 1)
    with pytest.raises(CacheError):
        c.append_token([1.0], [2.0, 3.0])
    c.append_token([1.0, 2.0], [3.0, 4.0])
    with pytest.raises(CacheError, match="capacity exhausted"):
        c.append_token([5.0, 6.0], [7.0, 8.0])
    with pytest.raises(CacheError, match="non-zero"):
        KvCache(0, 2, 1)


def test_kv_clear_reuses_capacity():  # cache.rs:209-219
    c = KvCache(2, 4, 8)
    p = _addr(c.keys)
    c.append_token([0.0] * 8, [0.0] * 8)
    c.clear()
    assert c.cached_tokens == 0 and _addr(c.keys) == p


def test_kv_truncate_discards_suffix_in_place():  # cache.rs:221-237
    c = KvCache(1, 2, 4)
    c.append_sequence([1, 2, 3, 4], [5, 6, 7, 8], 2)
    pk, pv = _addr(c.keys), _addr(c.values)
    c.truncate_to(1)
    assert c.cached_tokens == 1 and (_addr(c.keys), _addr(c.values)) == (pk, pv)
    assert c.keys[:2].tolist() == [1, 2] and c.values[:2].tolist() == [5, 6]


def test_kv_truncate_rejects_future_position():  # cache.rs:239-246
    c = KvCache(1, 2, 2)
    c.append_token([1, 2], [3, 4])
    with pytest.raises(CacheError, match="future position"):
        c.truncate_to(2)


def test_kv_copy_prefix_reuses_destination():  # cache.rs:248-266
    src = KvCache(1, 2, 4)
    src.append_sequence([1, 2, 3, 4], [5, 6, 7, 8], 2)
    dst = KvCache(1, 2, 4)
    dst.append_sequence([9, 10, 11, 12], [13, 14, 15, 16], 2)
    p = _addr(dst.keys)
    dst.copy_prefix_from(src)
    assert _addr(dst.keys) == p and dst.cached_tokens == 2
    assert dst.keys[:4].tolist() == [1, 2, 3, 4] and dst.values[:4].tolist() == [5, 6, 7, 8]


def test_kv_copy_prefix_compact_source_into_larger_destination():  # cache.rs:268-290
    src = KvCache(2, 2, 3)
    src.append_sequence([1, 2, 3, 4, 5, 6, 7, 8], [11, 12, 13, 14, 15, 16, 17, 18], 2)
    dst = KvCache(2, 2, 8)
    dst.copy_prefix_from(src)
    assert dst.cached_tokens == 2
    assert dst.keys[:4].tolist() == [1, 2, 5, 6] and dst.keys[16:20].tolist() == [3, 4, 7, 8]
    assert dst.values[:4].tolist() == [11, 12, 15, 16] and dst.values[16:20].tolist() == [13, 14, 17, 18]
    with pytest.raises(CacheError, match="layouts do not match"):
        KvCache(2, 2, 1).copy_prefix_from(src)


def test_kv_cache_feeds_the_attention_oracle():  # cache.rs:1-4 layout read by metal.rs:1707
    """A cache built by appends is what the attention restatement reads:
    the same output as the hand-built capacity-strided cache above."""
    c = KvCache(1, 2, 4)
    c.append_sequence([1, 0, 0, 1], [10, 0, 20, 0], 2)
    q = np.array([1, 1], np.float32)
    o = O.attention_decode(q, c.keys, c.values, [1, -1], [30, 0], 1, 1, 2, c.cached_tokens, c.capacity_tokens)
    compact = O.attention_decode(q, c.keys[:4], c.values[:4], [1, -1], [30, 0], 1, 1, 2, 2, 2)
    assert np.allclose(o, compact, atol=1e-6)


def test_gdn_parallel_formulation_agrees_with_the_serial_one():  # metal.rs:630-740
    """The reference ships two formulations of the recurrence with different
    summation orders; both sit within the 1e-5 parity tolerance of each
    other, so the tolerance covers either as the reference's answer."""
    rng = np.random.default_rng(21)
    h, d = 4, 128
    q = rng.normal(0, 0.1, h * d).astype(np.float32)
    k = rng.normal(0, 0.1, h * d).astype(np.float32)
    v = rng.normal(0, 1, h * d).astype(np.float32)
    g = -np.log1p(np.exp(rng.normal(0, 1, h))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, h)))).astype(np.float32)
    s = rng.normal(0, 0.1, h * d * d).astype(np.float32)
    o1, s1 = O.gdn_step(q, k, v, g, beta, s, h, d, d)
    o2, s2 = O.gdn_step_parallel(q, k, v, g, beta, s, h, d, d)
    rel = lambda a, b: float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))
    assert rel(o1, o2) < 1e-5 and rel(s1, s2) < 1e-5
    # the two-token known answer (qwen35.rs:273-288) through the parallel form
    o, st = O.gdn_step_parallel([1, 0], [1, 0], [2], [0], [0.5], [0, 0], 1, 2, 1)
    assert o.tolist() == [1.0] and st.tolist() == [1.0, 0.0]
    o, st = O.gdn_step_parallel([0, 1], [0, 1], [4], [math.log(0.5)], [1.0], st, 1, 2, 1)
    assert o.tolist() == [4.0] and st.tolist() == [0.5, 4.0]
