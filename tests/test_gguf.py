"""GGUF container reader (CPU only, no device): the native reader
(csrc/gguf.cu via si_gguf_*) against the reference's own GGUF tests
(src/model.rs:1913-2008) and against the Python restatement in oracle/gguf.py
on error cases and seeded mutations of valid files."""
import struct

import numpy as np
import pytest

import gguf_writer as W
from oracle import gguf as OG


def tiny_fixture() -> bytes:
    """tiny_gguf_fixture (model.rs:1982-2003), byte for byte."""
    b = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 1, 2))
    b += W.gguf_string("general.architecture") + struct.pack("<I", 8) + W.gguf_string("qwen35")
    b += W.gguf_string("general.alignment") + struct.pack("<II", 4, 32)
    b += W.gguf_string("blk.0.attn_q.weight") + struct.pack("<IQQIQ", 2, 4, 2, 0, 0)
    b += bytes(-len(b) % 32)
    b += bytes([1, 2, 3, 4, 5, 6, 7, 8])
    return bytes(b)


def open_bytes(mai, tmp_path, data: bytes, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return mai.GgufFile(str(p))


def native_error(mai, tmp_path, data: bytes):
    try:
        open_bytes(mai, tmp_path, data).close()
    except mai.SiError as e:
        return str(e)
    return None


def oracle_error(data: bytes):
    try:
        OG.parse(data)
    except OG.GgufError as e:
        return str(e)
    return None


def test_parses_tiny_fixture(mai, tmp_path):  # parses_gguf_metadata_and_tensor_index, model.rs:1913-1927
    data = tiny_fixture()
    with open_bytes(mai, tmp_path, data) as g:
        assert (g.version, g.tensor_count, g.metadata_count) == (3, 1, 2)
        assert g.meta_string("general.architecture") == "qwen35"
        assert g.meta_u64("general.alignment") == 32
        t = g.tensor_info(0)
        assert t["name"] == "blk.0.attn_q.weight" and t["shape"] == [4, 2] and t["ggml_type"] == 0
        assert t["data_start"] % 32 == 0 and t["data_end"] == len(data)
        assert g.read("blk.0.attn_q.weight").tolist() == [1, 2, 3, 4, 5, 6, 7, 8]
        assert g.read(0, 2, 3).tolist() == [3, 4, 5]
        assert g.find("blk.0.attn_q.weight") == 0
        with pytest.raises(mai.SiError, match="unknown GGUF tensor"):
            g.find("blk.0.attn_k.weight")
        with pytest.raises(mai.SiError, match="beyond tensor"):
            g.read(0, 4, 5)
    parsed = OG.parse(data)
    assert parsed["tensors"][0]["data_start"] == t["data_start"]


def test_rejects_magic_and_truncation(mai, tmp_path):  # model.rs:1974-1980
    assert "invalid magic" in native_error(mai, tmp_path, b"NOPE")
    assert "truncated" in native_error(mai, tmp_path, tiny_fixture()[:20])
    with pytest.raises(mai.SiError, match="open GGUF model"):
        mai.GgufFile(str(tmp_path / "missing.gguf"))


def kat_metadata(**changes):
    """derives_qwen35_execution_config_from_metadata (model.rs:1929-1971),
    plus the rotary width the runtime requires (qwen35_runtime.rs:811-813)."""
    m = {"general.architecture": (W.STRING, "qwen35"),
         "qwen35.embedding_length": (W.U32, 5120), "qwen35.feed_forward_length": (W.U32, 17408),
         "qwen35.block_count": (W.U32, 64), "qwen35.attention.head_count": (W.U32, 24),
         "qwen35.attention.head_count_kv": (W.U32, 4), "qwen35.attention.key_length": (W.U32, 256),
         "qwen35.attention.value_length": (W.U32, 256),
         "qwen35.attention.layer_norm_rms_epsilon": (W.F32, 1.0e-6), "qwen35.rope.freq_base": (W.F32, 1.0e7),
         "qwen35.context_length": (W.U32, 262144), "qwen35.full_attention_interval": (W.U32, 4),
         "qwen35.ssm.inner_size": (W.U32, 6144), "qwen35.ssm.state_size": (W.U32, 128),
         "qwen35.ssm.group_count": (W.U32, 16), "qwen35.ssm.conv_kernel": (W.U32, 4),
         "qwen35.ssm.time_step_rank": (W.U32, 48), "tokenizer.ggml.eos_token_id": (W.U32, 248046),
         "tokenizer.ggml.tokens": (W.ARRAY, (W.STRING, ["a"] * 248320)),
         "qwen35.rope.dimension_count": (W.U32, 64)}
    for k, v in changes.items():
        k = k.replace("__", ".")
        if v is None:
            m.pop(k)
        else:
            m[k] = v
    return [(k, t, v) for k, (t, v) in m.items()]


def test_derives_qwen35_config_kat(mai, tmp_path):  # model.rs:1929-1971
    with open_bytes(mai, tmp_path, W.build(kat_metadata(), [])) as g:
        c = g.qwen35_config(kv_capacity=1024)
        assert g.meta_array_len("tokenizer.ggml.tokens") == 248320
    ref = mai.qwen36_27b_config()
    for f in ("hidden", "intermediate", "layers", "vocab", "attn_interval", "attn_q_heads", "attn_kv_heads",
              "attn_head_dim", "rotary_dim", "gdn_key_heads", "gdn_value_heads", "gdn_head_dim", "conv_kernel"):
        assert getattr(c, f) == getattr(ref, f), f
    assert c.eos_token == 248046 and c.kv_capacity == 1024
    assert c.rms_eps == np.float32(1e-6) and c.rope_theta == np.float32(1e7)
    o = OG.qwen35_config(OG.parse(W.build(kat_metadata(), []))["metadata"])
    assert (o["hidden_size"], o["num_hidden_layers"], o["vocab_size"], o["ssm_inner_size"]) == (5120, 64, 248320, 6144)
    assert (o["ssm_key_heads"], o["ssm_value_heads"], o["rotary_dim"]) == (16, 48, 64)


CONFIG_ERRORS = [
    ({"general__architecture": (W.STRING, "llama")}, "unsupported GGUF architecture llama"),
    ({"qwen35__block_count": None}, "GGUF metadata is missing qwen35.block_count"),
    ({"qwen35__block_count": (W.I32, 64)}, "qwen35.block_count has unexpected value"),
    ({"qwen35__block_count": (W.U64, 1 << 33)}, "qwen35.block_count overflows u32"),
    ({"qwen35__block_count": (W.U8, 0)}, "invalid dimensions"),
    ({"qwen35__rope__freq_base": (W.U32, 10)}, "qwen35.rope.freq_base has unexpected value"),
    ({"qwen35__rope__freq_base": (W.F64, 1.0)}, "invalid dimensions"),
    ({"qwen35__attention__layer_norm_rms_epsilon": (W.F32, float("nan"))}, "invalid dimensions"),
    ({"qwen35__attention__head_count_kv": (W.U32, 5)}, "divisible by key/value heads"),
    ({"qwen35__ssm__inner_size": (W.U32, 6100)}, "divisible by state size"),
    ({"tokenizer__ggml__tokens": (W.U32, 3)}, "tokenizer.ggml.tokens has unexpected value"),
    ({"tokenizer__ggml__tokens": (W.ARRAY, (W.STRING, []))}, "invalid dimensions"),
    ({"qwen35__rope__dimension_count": None}, "missing qwen35.rope.dimension_count"),
]


@pytest.mark.parametrize("changes,message", CONFIG_ERRORS)
def test_config_errors_match_reference(mai, tmp_path, changes, message):
    data = W.build(kat_metadata(**changes), [])
    with pytest.raises(OG.GgufError, match=message.replace(".", r"\.")):
        OG.qwen35_config(OG.parse(data)["metadata"])
    with open_bytes(mai, tmp_path, data) as g:
        with pytest.raises(mai.SiError, match=message.replace(".", r"\.")):
            g.qwen35_config()


def test_unsupported_shapes_are_refused(mai, tmp_path):
    """One head width and one dt row per value head: other layouts are refused
    before any allocation, not decoded wrongly."""
    for changes in ({"qwen35__attention__value_length": (W.U32, 128)}, {"qwen35__ssm__time_step_rank": (W.U32, 16)}):
        with open_bytes(mai, tmp_path, W.build(kat_metadata(**changes), [])) as g:
            with pytest.raises(mai.SiError) as e:
                g.qwen35_config()
            assert e.value.status == mai.SI_E_UNSUPPORTED


def _meta(*extra):
    return [("general.architecture", W.STRING, "qwen35")] + list(extra)


HEADER_ERRORS = [
    (b"GGUF" + struct.pack("<IQQ", 1, 0, 0), "unsupported GGUF version 1"),
    (W.build(_meta(("k", W.U32, 1), ("k", W.U32, 2)), []), "duplicate keys"),
    (W.build(_meta(("general.alignment", W.U32, 0)), []), "non-zero power of two"),
    (W.build(_meta(("general.alignment", W.U64, 48)), []), "non-zero power of two"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string("k") + struct.pack("<I", 8) + W.gguf_string(b"qwen3\xff"),
     "not UTF-8"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string(b"\xed\xa0\x80") + struct.pack("<IB", 0, 1),
     "not UTF-8"),  # an encoded surrogate
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string("k") + struct.pack("<I", 13), "unsupported GGUF metadata type 13"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string("k") + struct.pack("<I", 8) + W.gguf_string(b"\xc3\x28"),
     "not UTF-8"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string("k") + struct.pack("<IIQ", 9, 4, 1 << 40), "truncated"),
]


@pytest.mark.parametrize("idx", range(len(HEADER_ERRORS)))
def test_header_errors_match_oracle(mai, tmp_path, idx):
    data, message = HEADER_ERRORS[idx]
    want = oracle_error(data)
    got = native_error(mai, tmp_path, data)
    if message is not None:
        assert want is not None and message in want
    assert (got is None) == (want is None) and (got is None or want in got), (got, want)


def test_empty_array_of_unknown_type_is_accepted(mai, tmp_path):
    """An empty array never reads an element, so its element type is not
    checked (read_value, model.rs:1218-1226)."""
    data = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W.gguf_string("k") + struct.pack("<IIQ", 9, 99, 0)
    assert oracle_error(data) is None
    with open_bytes(mai, tmp_path, data) as g:
        assert g.meta_array_len("k") == 0


def test_tensor_ranges_follow_sorted_offsets(mai, tmp_path):
    """A tensor's bytes run to the next offset in sorted order, or to EOF
    (model.rs:1095-1118); index order need not be offset order."""
    rng = np.random.default_rng(1)
    payloads = [rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in (40, 7, 100)]
    data = bytearray(W.build(_meta(("general.alignment", W.U32, 64)),
                             [(f"t{i}", [len(p)], 0, p) for i, p in enumerate(payloads)], alignment=64))
    # move t0 after t2 by swapping the index offsets of t0 and t2 and their payloads
    parsed = OG.parse(bytes(data))
    with open_bytes(mai, tmp_path, bytes(data)) as g:
        for i, t in enumerate(parsed["tensors"]):
            info = g.tensor_info(i)
            assert (info["data_start"], info["data_end"]) == (t["data_start"], t["data_end"])
            assert g.read(i)[:len(payloads[i])].tobytes() == payloads[i]
    # tensors listed out of offset order and sharing an offset
    m = _meta(("general.alignment", W.U32, 32))
    hdr = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 4, len(m)))
    for k, t, v in m:
        hdr += W.gguf_string(k) + struct.pack("<I", t) + W.encode_value(t, v)
    for name, off in (("c", 64), ("a", 0), ("b", 32), ("b2", 32)):
        hdr += W.gguf_string(name) + struct.pack("<IQIQ", 1, 8, 0, off)
    hdr += bytes(-len(hdr) % 32) + bytes(range(96)) + b"tail"
    data = bytes(hdr)
    parsed = OG.parse(data)
    with open_bytes(mai, tmp_path, data) as g:
        for i, t in enumerate(parsed["tensors"]):
            info = g.tensor_info(i)
            assert (info["data_start"], info["data_end"]) == (t["data_start"], t["data_end"]), t["name"]
    assert [t["data_end"] - t["data_start"] for t in parsed["tensors"]] == [36, 32, 0, 32]
    # an offset past the end of the file
    bad = bytearray(data)
    pos = bad.index(b"\x01\x00\x00\x00" + struct.pack("<Q", 8) + struct.pack("<IQ", 0, 64))
    bad[pos + 16:pos + 24] = struct.pack("<Q", 1 << 20)
    assert "exceeds file size" in oracle_error(bytes(bad))
    assert "exceeds file size" in native_error(mai, tmp_path, bytes(bad))


def test_seeded_mutations_agree_with_oracle(mai, tmp_path):
    """Random byte flips and truncations of a valid file: the native reader and
    the restatement accept or reject each variant alike, with the same message
    and the same tensor index (names compared up to a NUL: the C-ABI hands
    names out as C strings)."""
    base = W.build(_meta(("general.alignment", W.U32, 32), ("n", W.U64, 7), ("f", W.F32, 1.5),
                         ("arr", W.ARRAY, (W.U16, [1, 2, 3])), ("s", W.ARRAY, (W.STRING, ["x", "yz"]))),
                   [("w", [256, 2], 12, bytes(288)), ("v", [3], 0, bytes(12))])
    rng = np.random.default_rng(7)
    agree = accepted = 0
    for trial in range(300):
        d = bytearray(base)
        if trial % 3 == 0:
            d = d[:int(rng.integers(0, len(d)))]
        else:
            for _ in range(int(rng.integers(1, 4))):
                i = int(rng.integers(4, min(len(d), 400)))
                d[i] = int(rng.integers(0, 256))
        d = bytes(d)
        want, got = oracle_error(d), native_error(mai, tmp_path, d)
        assert (got is None) == (want is None) and (got is None or want in got), (trial, got, want)
        if want is None:
            accepted += 1
            parsed = OG.parse(d)
            with open_bytes(mai, tmp_path, d) as g:
                assert g.tensor_count == len(parsed["tensors"])
                for i, t in enumerate(parsed["tensors"]):
                    info = g.tensor_info(i)
                    assert (info["name"], info["ggml_type"], info["data_start"], info["data_end"]) == \
                        (t["name"].split("\0")[0], t["ggml_type"], t["data_start"], t["data_end"])
        agree += 1
    assert agree == 300 and accepted > 10


def test_detects_safetensors_directories_and_gguf_files(mai, tmp_path):  # model.rs:1881-1902
    root = tmp_path / "m"
    root.mkdir()
    (root / "manifest.json").write_text('{"model":"test","revision":"r","format":"safetensors","dtype":"bfloat16",'
                                        '"total_weight_bytes":0,"files":[]}')
    gguf = root / "tiny.gguf"
    gguf.write_bytes(b"GGUF")
    assert mai.detect_model_format(root) == "safetensors"
    assert mai.detect_model_format(gguf) == "gguf"
    # the manifest must say BF16 Safetensors; other containers are refused
    (root / "manifest.json").write_text('{"format":"safetensors","dtype":"float16","files":[{"a":[1,2.5e3,true,null]}]}')
    with pytest.raises(mai.SiError, match="not a BF16 Safetensors artifact"):
        mai.detect_model_format(root)
    (root / "manifest.json").write_text('{"format": "safetensors", "dtype": ')
    with pytest.raises(mai.SiError, match="invalid model manifest JSON"):
        mai.detect_model_format(root)
    (root / "manifest.json").write_text('{"format":"safe\\u0074ensors","dtype":"bfloat16"} ')
    assert mai.detect_model_format(root) == "safetensors"
    other = tmp_path / "x.bin"
    other.write_bytes(b"NOPE")
    with pytest.raises(mai.SiError, match="unsupported model container"):
        mai.detect_model_format(other)
    with pytest.raises(mai.SiError, match="stat model"):
        mai.detect_model_format(tmp_path / "missing")
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(mai.SiError, match="read model manifest"):
        mai.detect_model_format(empty)


def _kind_metadata(layers, interval):
    return kat_metadata(qwen35__block_count=(W.U32, layers), qwen35__full_attention_interval=(W.U32, interval))


def test_layer_kinds_follow_tensors_and_interval(mai, tmp_path):
    """qwen35_layer_kinds (model.rs:748-790), checked as the reference's real
    GGUF test checks a 64-layer file (model.rs:2199-2204), on an 8-layer one."""
    names = []
    for l in range(8):
        names.append(f"blk.{l}.attn_q.weight" if (l + 1) % 4 == 0 else f"blk.{l}.ssm_a")
    tensors = [(n, [4], 0, bytes(16)) for n in names]
    with open_bytes(mai, tmp_path, W.build(_kind_metadata(8, 4), tensors)) as g:
        kinds = g.layer_kinds()
        assert kinds[0] == "gated_delta_net" and kinds[3] == "full_attention" and kinds[7] == "full_attention"
        assert kinds.count("full_attention") == 2
        with pytest.raises(mai.SiError, match="exceeds 8 layers"):
            g.layer_kind(8)
    # a layer with both kinds, a layer with neither, and a kind against the interval
    bad = [("blk.0.ssm_a", [4], 0, bytes(16)), ("blk.0.attn_q.weight", [4], 0, bytes(16)),
           ("blk.2.ssm_a", [4], 0, bytes(16)), ("blk.3.ssm_a", [4], 0, bytes(16))]
    with open_bytes(mai, tmp_path, W.build(_kind_metadata(4, 4), bad), "bad.gguf") as g:
        with pytest.raises(mai.SiError, match="exactly one execution kind"):
            g.layer_kind(0)
        with pytest.raises(mai.SiError, match="exactly one execution kind"):
            g.layer_kind(1)
        with pytest.raises(mai.SiError, match="GatedDeltaNet disagrees with interval 4"):
            g.layer_kind(3)


def test_expected_payload_bytes(mai, tmp_path):  # GgufTensorInfo::expected_payload_bytes, model.rs:532-573
    tensors = [("f32", [3, 5], 0, bytes(60)), ("f16", [7], 1, bytes(14)), ("bf16", [2, 2], 30, bytes(8)),
               ("q4", [512, 3], 12, bytes(6 * 144)), ("q5", [256], 13, bytes(176)), ("q6", [256, 2], 14, bytes(420)),
               ("q8_0", [32], 8, bytes(34)), ("bad_q4", [100], 12, bytes(144))]
    with open_bytes(mai, tmp_path, W.build(_meta(), tensors)) as g:
        got = [g.tensor_payload(i) for i in range(7)]
        assert got == [(15, 60), (7, 14), (4, 8), (1536, 864), (256, 176), (512, 420), (32, None)]
        with pytest.raises(mai.SiError, match="GGUF Q4_K tensor bad_q4 has 100 elements; expected a multiple of 256"):
            g.tensor_payload(7)


def test_metadata_summaries(mai, tmp_path):
    data = W.build(kat_metadata(), [])
    with open_bytes(mai, tmp_path, data) as g:
        md = g.metadata()
    assert list(md) == sorted(md)
    assert md["qwen35.embedding_length"] == "U32(5120)"
    assert md["qwen35.attention.layer_norm_rms_epsilon"] == "F32(1e-6)"
    assert md["qwen35.rope.freq_base"] == "F32(10000000.0)"
    assert md["tokenizer.ggml.tokens"] == 'array(len=248320, first=[string("a"), string("a"), string("a")])'
