"""Decode from a GGUF file (si_model_create_gguf): a small qwen35 model written
to a GGUF container with mixed K-quant types per tensor, loaded by the native
reader and checked against the oracle over the same bytes; a synthetic model
round-tripped through a file gives byte-identical host shards and identical
decode; malformed files are refused before any device allocation."""
import numpy as np
import pytest

import gguf_writer as W
import oracle as O
from helpers import rel_l2

pytestmark = pytest.mark.gpu

Q4, Q5, Q6, F32 = 12, 13, 14, 0


def small_config(mai, **kw):
    base = dict(hidden=512, intermediate=1024, layers=4, vocab=2048, attn_q_heads=4, attn_kv_heads=2,
                attn_head_dim=128, rotary_dim=32, gdn_key_heads=2, gdn_value_heads=4, kv_capacity=24,
                eos_token=0xFFFFFFFF)
    base.update(kw)
    return mai.qwen36_27b_config(**base)


def centered_blocks(rng, ty, nblocks):
    """Seeded K-quant super-blocks with roughly zero-mean rows: sub-block
    scales 0..8 and mins ~ offset * scale with dmin = d (Q4_K/Q5_K), int8
    scales in [-8, 8] (Q6_K)."""
    bb = {Q4: 144, Q5: 176, Q6: 210}[ty]
    b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    d = np.abs(rng.normal(0, 0.02, nblocks)).astype(np.float16).view(np.uint16)
    if ty == Q6:
        b[:, 192:208] = rng.integers(-8, 9, size=(nblocks, 16)).astype(np.int8).view(np.uint8)
        b[:, 208], b[:, 209] = d & 0xFF, d >> 8
        return b.reshape(-1)
    off, smax = (15.5, 4) if ty == Q5 else (7.5, 8)
    sc = rng.integers(0, smax + 1, size=(nblocks, 8))
    mn = np.minimum(np.rint(off * sc), 63).astype(np.int64)
    s = np.zeros((nblocks, 12), np.int64)
    s[:, 0:4] = (sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)
    s[:, 4:8] = (mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:] & 15) | ((mn[:, 4:] & 15) << 4)
    b[:, 4:16] = s.astype(np.uint8)
    b[:, 0], b[:, 1] = d & 0xFF, d >> 8
    b[:, 2], b[:, 3] = b[:, 0], b[:, 1]
    return b.reshape(-1)


def roles(c, layer):
    """(name, rows, cols, default type, f32 normal (mean, sd)) of one layer's
    tensors, in the shapes the reference reads (qwen35_runtime.rs:419-446,
    638-657); layer == c.layers: the globals."""
    H, I, d = c.hidden, c.intermediate, c.gdn_head_dim
    if layer == c.layers:
        return [("token_embd.weight", c.vocab, H, Q4, None), ("output_norm.weight", 1, H, F32, (0, 0.1)),
                ("output.weight", c.vocab, H, c.head_type, None)]
    pre = f"blk.{layer}."
    out = [(pre + "attn_norm.weight", 1, H, F32, (0, 0.1)), (pre + "post_attention_norm.weight", 1, H, F32, (0, 0.1)),
           (pre + "ffn_gate.weight", I, H, Q4, None), (pre + "ffn_up.weight", I, H, Q4, None),
           (pre + "ffn_down.weight", H, I, Q6, None)]
    if (layer + 1) % c.attn_interval:
        proj, vw = (2 * c.gdn_key_heads + c.gdn_value_heads) * d, c.gdn_value_heads * d
        out += [(pre + "attn_qkv.weight", proj, H, Q4, None), (pre + "attn_gate.weight", vw, H, Q4, None),
                (pre + "ssm_alpha.weight", c.gdn_value_heads, H, F32, (0, 0.02)),
                (pre + "ssm_beta.weight", c.gdn_value_heads, H, F32, (0, 0.02)),
                (pre + "ssm_conv1d.weight", proj, c.conv_kernel, F32, (0, 0.5)),
                (pre + "ssm_a", c.gdn_value_heads, 1, F32, (0, 0.5)),
                (pre + "ssm_dt.bias", c.gdn_value_heads, 1, F32, (0, 0.5)),
                (pre + "ssm_norm.weight", 1, d, F32, (1, 0.1)), (pre + "ssm_out.weight", H, vw, Q4, None)]
    else:
        qw, kvw = c.attn_q_heads * c.attn_head_dim, c.attn_kv_heads * c.attn_head_dim
        out += [(pre + "attn_q.weight", 2 * qw, H, Q4, None), (pre + "attn_k.weight", kvw, H, Q4, None),
                (pre + "attn_v.weight", kvw, H, Q4, None), (pre + "attn_output.weight", H, qw, Q4, None),
                (pre + "attn_q_norm.weight", 1, c.attn_head_dim, F32, (0, 0.1)),
                (pre + "attn_k_norm.weight", 1, c.attn_head_dim, F32, (0, 0.1))]
    return out


def f32_shape(rows, cols):
    return [rows] if cols == 1 else [cols] if rows == 1 else [cols, rows]


# GGUF name suffix -> backend tensor id
TENSOR_ID = {"attn_norm.weight": "ATTN_NORM", "post_attention_norm.weight": "POST_NORM",
             "ffn_gate.weight": "FFN_GATE", "ffn_up.weight": "FFN_UP", "ffn_down.weight": "FFN_DOWN",
             "attn_qkv.weight": "SSM_QKV", "attn_gate.weight": "SSM_Z", "ssm_alpha.weight": "SSM_ALPHA",
             "ssm_beta.weight": "SSM_BETA", "ssm_conv1d.weight": "SSM_CONV", "ssm_a": "SSM_A",
             "ssm_dt.bias": "SSM_DT", "ssm_norm.weight": "SSM_NORM", "ssm_out.weight": "SSM_OUT",
             "attn_q.weight": "ATTN_Q", "attn_k.weight": "ATTN_K", "attn_v.weight": "ATTN_V",
             "attn_output.weight": "ATTN_O", "attn_q_norm.weight": "ATTN_QNORM",
             "attn_k_norm.weight": "ATTN_KNORM", "token_embd.weight": "TOKEN_EMBD",
             "output_norm.weight": "OUTPUT_NORM", "output.weight": "OUTPUT"}


def model_tensors(c, seed, types=None, skip=(), override=None):
    """GGUF tensor list for config c: seeded payloads, per-name type overrides."""
    rng = np.random.default_rng(seed)
    types, override = types or {}, override or {}
    out = []
    for layer in range(c.layers + 1):
        for name, rows, cols, ty, f32 in roles(c, layer):
            if name in skip:
                continue
            ty = types.get(name, ty)
            if ty == F32:
                mean, sd = f32 or (0, 0.1)
                payload = (mean + sd * rng.normal(size=rows * cols)).astype(np.float32).tobytes()
                shape = f32_shape(rows, cols)
            else:
                payload = centered_blocks(rng, ty, rows * cols // 256).tobytes()
                shape = [cols, rows]
            out.append(override.get(name, (name, shape, ty, payload)))
    return out


MIXED = {"blk.0.attn_qkv.weight": Q5, "blk.0.attn_gate.weight": Q6, "blk.0.ssm_out.weight": Q6,
         "blk.0.ffn_up.weight": Q5, "blk.1.ffn_gate.weight": Q6, "blk.1.ffn_up.weight": Q6,
         "blk.1.ffn_down.weight": Q5, "blk.3.attn_q.weight": Q5, "blk.3.attn_k.weight": Q6,
         "blk.3.attn_v.weight": Q4, "blk.3.attn_output.weight": Q6, "blk.3.ffn_down.weight": Q4}


@pytest.fixture(scope="module")
def mixed_file(mai, tmp_path_factory):
    c = small_config(mai)
    path = tmp_path_factory.mktemp("gguf") / "mixed.gguf"
    W.write(path, W.qwen35_metadata(c, alignment=64), model_tensors(c, 5, MIXED), alignment=64)
    return path


def test_mixed_type_file_decodes_like_oracle(mai, ctx, mixed_file):
    m = mai.Model.from_gguf(ctx, mixed_file, kv_capacity=24)
    c = m.config
    assert m.host_tensor(0, mai.T["SSM_QKV"])[2] == Q5 and m.host_tensor(3, mai.T["ATTN_K"])[2] == Q6
    orc = O.OracleModel(c, m.host_tensor)
    for pos, tok in enumerate([7, 2047, 300]):
        e1, e2 = m.embed_token(tok), orc.embed(tok)
        assert np.array_equal(e1, e2)
        h1, h2 = m.decode_hidden(pos, e1), orc.decode_hidden(pos, e2)
        assert rel_l2(h1, h2) < 1e-5, pos
        assert rel_l2(m.logits(h1), orc.logits(h2)) < 1e-5
    m.reset()
    orc.close()
    orc = O.OracleModel(c, m.host_tensor)
    prompt = [5, 77, 1024]
    assert m.generate(prompt, 8) == orc.generate(prompt, 8)
    orc.close()
    m.close()


def test_file_payload_is_what_the_model_holds(mai, ctx, mixed_file):
    """Host shards are the file's bytes (read by row range with pread)."""
    m = mai.Model.from_gguf(ctx, mixed_file, kv_capacity=24)
    with mai.GgufFile(mixed_file) as g:
        for layer, tid, name in [(0, "SSM_QKV", "blk.0.attn_qkv.weight"), (3, "ATTN_O", "blk.3.attn_output.weight"),
                                 (1, "FFN_DOWN", "blk.1.ffn_down.weight"), (4, "OUTPUT", "output.weight"),
                                 (4, "TOKEN_EMBD", "token_embd.weight"), (0, "SSM_A", "blk.0.ssm_a")]:
            held = m.host_tensor_array(layer, mai.T[tid])
            assert np.array_equal(held, g.read(name)[:held.size]), name
    m.close()


def test_synthetic_model_round_trips_through_a_file(mai, ctx, tmp_path):
    c = small_config(mai, layers=4, kv_capacity=16)
    syn = mai.Model(ctx, c, seed=11)
    tensors = []
    for layer in range(c.layers + 1):
        for name, rows, cols, _, _ in roles(c, layer):
            tid = TENSOR_ID[name.split(".", 2)[2] if name.startswith("blk.") else name]
            _, _, ty = syn.host_tensor(layer, mai.T[tid])
            shape = f32_shape(rows, cols) if ty == F32 else [cols, rows]
            tensors.append((name, shape, ty, syn.host_tensor_array(layer, mai.T[tid]).tobytes()))
    path = tmp_path / "syn.gguf"
    W.write(path, W.qwen35_metadata(c), tensors)
    m = mai.Model.from_gguf(ctx, path, kv_capacity=16)
    for layer in range(c.layers + 1):
        for tid in range(mai.T_COUNT):
            a, b = syn.host_tensor(layer, tid), m.host_tensor(layer, tid)
            assert a[1:] == b[1:]
            if a[0]:
                assert np.array_equal(syn.host_tensor_array(layer, tid), m.host_tensor_array(layer, tid))
    prompt = [1, 2, 3]
    ids = m.generate(prompt, 6)
    assert ids == syn.generate(prompt, 6)
    n1, l1 = m.decode_token(ids[-1], len(prompt) + 6)
    n2, l2 = syn.decode_token(ids[-1], len(prompt) + 6)
    assert n1 == n2 and np.array_equal(l1, l2)
    m.close()
    syn.close()


@pytest.mark.parametrize("case", ["missing", "f32_type", "shape", "kind", "embd_type", "short"])
def test_malformed_files_are_refused_before_allocation(mai, ctx, tmp_path, case):
    c = small_config(mai)
    kw = {}
    msg = {"missing": "unknown GGUF tensor blk.2.ssm_norm.weight", "f32_type": "is not F32",
           "shape": "shape does not match", "kind": "does not have exactly one execution kind",
           "embd_type": "token embeddings must be Q4_K", "short": "payload is"}[case]
    if case == "missing":
        kw["skip"] = {"blk.2.ssm_norm.weight"}
    elif case == "f32_type":
        kw["override"] = {"blk.1.attn_norm.weight": ("blk.1.attn_norm.weight", [512], Q4, bytes(288))}
    elif case == "shape":
        kw["override"] = {"blk.0.ffn_up.weight": ("blk.0.ffn_up.weight", [1024, 512], Q4, bytes(144 * 2048))}
    elif case == "kind":
        kw["override"] = {"blk.3.attn_q_norm.weight": ("blk.3.ssm_a", [4], F32, bytes(16))}
    elif case == "embd_type":
        kw["types"] = {"token_embd.weight": Q6}
    tensors = model_tensors(c, 3, **kw)
    path = tmp_path / f"{case}.gguf"
    data = W.build(W.qwen35_metadata(c), tensors)
    if case == "short":
        data = data[:-1000]  # output.weight is last: its payload ends early
    path.write_bytes(data)
    before = ctx.stats()["current_allocated_bytes"]
    with pytest.raises(mai.SiError, match=msg):
        mai.Model.from_gguf(ctx, path, kv_capacity=16)
    assert ctx.stats()["current_allocated_bytes"] == before
