"""Minimal GGUF v2/v3 writer for tests: builds container bytes from typed
metadata and tensor payloads, laid out as the reference's parser expects
(src/model.rs:1034-1120: header, metadata, tensor index, data base aligned to
general.alignment, tensor offsets relative to that base)."""
from __future__ import annotations

import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def gguf_string(s) -> bytes:
    raw = s if isinstance(s, bytes) else s.encode()
    return struct.pack("<Q", len(raw)) + raw


def encode_value(t: int, v) -> bytes:
    if t in _FMT:
        return struct.pack(_FMT[t], v)
    if t == STRING:
        return gguf_string(v)
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(encode_value(et, x) for x in items)
    raise ValueError(t)


def build(metadata, tensors, alignment: int = 32, version: int = 3) -> bytes:
    """metadata: [(key, type, value)] (arrays: value = (elem_type, items));
    tensors: [(name, shape, ggml_type, payload bytes)] in index order. Payloads
    are placed in the same order, each at an `alignment`-aligned offset."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, t, v in metadata:
        out += gguf_string(key) + struct.pack("<I", t) + encode_value(t, v)
    offsets, off = [], 0
    for _, _, _, payload in tensors:
        offsets.append(off)
        off = (off + len(payload) + alignment - 1) // alignment * alignment
    for (name, shape, ty, _), o in zip(tensors, offsets):
        out += gguf_string(name) + struct.pack("<I", len(shape))
        out += b"".join(struct.pack("<Q", d) for d in shape) + struct.pack("<IQ", ty, o)
    out += bytes(-len(out) % alignment)
    base = len(out)
    for (_, _, _, payload), o in zip(tensors, offsets):
        out += bytes(base + o - len(out)) + bytes(payload)
    return bytes(out)


def write(path, metadata, tensors, alignment: int = 32, version: int = 3) -> None:
    with open(path, "wb") as f:
        f.write(build(metadata, tensors, alignment, version))


def qwen35_metadata(c, vocab_tokens=None, alignment=None, eos=None):
    """qwen35 metadata keys for a decode config (SiModelConfig fields)."""
    inner = c.gdn_value_heads * c.gdn_head_dim
    meta = [("general.architecture", STRING, "qwen35"),
            ("qwen35.embedding_length", U32, c.hidden),
            ("qwen35.feed_forward_length", U32, c.intermediate),
            ("qwen35.block_count", U32, c.layers),
            ("qwen35.attention.head_count", U32, c.attn_q_heads),
            ("qwen35.attention.head_count_kv", U32, c.attn_kv_heads),
            ("qwen35.attention.key_length", U32, c.attn_head_dim),
            ("qwen35.attention.value_length", U32, c.attn_head_dim),
            ("qwen35.attention.layer_norm_rms_epsilon", F32, c.rms_eps),
            ("qwen35.rope.freq_base", F32, c.rope_theta),
            ("qwen35.rope.dimension_count", U32, c.rotary_dim),
            ("qwen35.context_length", U32, 262144),
            ("qwen35.full_attention_interval", U32, c.attn_interval),
            ("qwen35.ssm.inner_size", U32, inner),
            ("qwen35.ssm.state_size", U32, c.gdn_head_dim),
            ("qwen35.ssm.group_count", U32, c.gdn_key_heads),
            ("qwen35.ssm.conv_kernel", U32, c.conv_kernel),
            ("qwen35.ssm.time_step_rank", U32, c.gdn_value_heads),
            ("tokenizer.ggml.eos_token_id", U32, c.eos_token if eos is None else eos),
            ("tokenizer.ggml.tokens", ARRAY, (STRING, vocab_tokens or [f"t{i}" for i in range(c.vocab)]))]
    if alignment is not None:
        meta.append(("general.alignment", U32, alignment))
    return meta
