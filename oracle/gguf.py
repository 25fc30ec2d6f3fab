"""Pure-Python restatement of the reference's GGUF container parser and qwen35
config derivation.

TEST INFRASTRUCTURE ONLY: the checker for the product's native GGUF reader
(memory-aware-inference_b200/csrc/gguf.cu). The product never imports it.

Follows src/model.rs:1034-1120 (parse_gguf), 1155-1236 (GgufReader),
350-417 (GgufQwen35Config::from_metadata), 444-496 (required_* helpers) and
src/qwen35_runtime.rs:811-813 (rotary width). Pinned by the reference's own
tests (src/model.rs:1913-2008: the tiny fixture, the 27B metadata KAT, the
magic and truncation rejections), restated in tests/test_gguf.py.
"""
from __future__ import annotations

import struct

import numpy as np


class GgufError(ValueError):
    pass


# metadata value types (GgufValue, model.rs:583-600)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FIXED = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
          U64: "<Q", I64: "<q", F64: "<d"}


class _Reader:
    """GgufReader (model.rs:1139-1236): bounds-checked little-endian reads."""

    def __init__(self, data: bytes):
        self.b, self.off = data, 0

    def bytes(self, n: int) -> bytes:
        if self.off + n > len(self.b):
            raise GgufError("GGUF header is truncated")
        v = self.b[self.off:self.off + n]
        self.off += n
        return v

    def pod(self, fmt: str):
        return struct.unpack(fmt, self.bytes(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.pod("<Q")
        raw = self.bytes(n)
        try:
            return raw.decode("utf-8")
        except UnicodeDecodeError:
            raise GgufError("GGUF string is not UTF-8") from None

    def value(self, t: int):
        """read_value (model.rs:1208-1235) -> (type, python value)."""
        if t in _FIXED:
            v = self.pod(_FIXED[t])
            return (t, v != 0) if t == BOOL else (t, v)
        if t == STRING:
            return t, self.string()
        if t == ARRAY:
            et = self.pod("<I")
            n = self.pod("<Q")
            return t, [self.value(et) for _ in range(n)]
        raise GgufError(f"unsupported GGUF metadata type {t}")


def parse(data: bytes) -> dict:
    """parse_gguf (model.rs:1034-1120): metadata {key: (type, value)} and the
    tensor index [{name, shape, ggml_type, offset, data_start, data_end}]."""
    r = _Reader(data)
    if r.bytes(4) != b"GGUF":
        raise GgufError("GGUF header has invalid magic")
    version = r.pod("<I")
    if version not in (2, 3):
        raise GgufError(f"unsupported GGUF version {version}")
    ntensors, nmeta = r.pod("<Q"), r.pod("<Q")
    meta = {}
    for _ in range(nmeta):
        key = r.string()
        t = r.pod("<I")
        v = r.value(t)
        if key in meta:
            raise GgufError("GGUF metadata contains duplicate keys")
        meta[key] = v
    tensors = []
    for _ in range(ntensors):
        name = r.string()
        nd = r.pod("<I")
        shape = [r.pod("<Q") for _ in range(nd)]
        ty = r.pod("<I")
        off = r.pod("<Q")
        tensors.append({"name": name, "shape": shape, "ggml_type": ty, "offset": off})
    al = meta.get("general.alignment")
    alignment = al[1] if al is not None and al[0] in (U32, U64) else 32
    if alignment == 0 or alignment & (alignment - 1):
        raise GgufError("GGUF alignment must be a non-zero power of two")
    base = (r.off + alignment - 1) // alignment * alignment
    order = sorted(range(len(tensors)), key=lambda i: tensors[i]["offset"])  # stable, like sort_by_key
    for pos, i in enumerate(order):
        start = base + tensors[i]["offset"]
        end = base + tensors[order[pos + 1]]["offset"] if pos + 1 < len(order) else len(data)
        if start > end or end > len(data):
            raise GgufError(f"GGUF tensor {tensors[i]['name']} exceeds file size")
        tensors[i]["data_start"], tensors[i]["data_end"] = start, end
    return {"version": version, "metadata": meta, "tensors": tensors}


def _required_u32(meta, key):
    """required_u32 (model.rs:454-469)."""
    if key not in meta:
        raise GgufError(f"GGUF metadata is missing {key}")
    t, v = meta[key]
    if t not in (U8, U16, U32, U64):
        raise GgufError(f"GGUF metadata {key} has unexpected value")
    if v > 0xFFFFFFFF:
        raise GgufError(f"GGUF metadata {key} overflows u32")
    return v


def _required_f32(meta, key):
    """required_f32 (model.rs:476-485): the value rounded to f32."""
    if key not in meta:
        raise GgufError(f"GGUF metadata is missing {key}")
    t, v = meta[key]
    if t not in (F32, F64):
        raise GgufError(f"GGUF metadata {key} has unexpected value")
    with np.errstate(over="ignore"):
        return float(np.float32(v))  # `as f32`: round to nearest, inf past the range


def _required(meta, key, t_want):
    if key not in meta:
        raise GgufError(f"GGUF metadata is missing {key}")
    t, v = meta[key]
    if t != t_want:
        raise GgufError(f"GGUF metadata {key} has unexpected value")
    return v


def qwen35_config(meta: dict) -> dict:
    """GgufQwen35Config::from_metadata (model.rs:350-417), fields in the
    reference's evaluation order, plus the rotary width the runtime reads."""
    arch = _required(meta, "general.architecture", STRING)
    if arch != "qwen35":
        raise GgufError(f"unsupported GGUF architecture {arch}; expected qwen35")
    c = {}
    for field, key, kind in [
            ("hidden_size", "qwen35.embedding_length", "u"),
            ("intermediate_size", "qwen35.feed_forward_length", "u"),
            ("num_hidden_layers", "qwen35.block_count", "u"),
            ("num_attention_heads", "qwen35.attention.head_count", "u"),
            ("num_key_value_heads", "qwen35.attention.head_count_kv", "u"),
            ("head_dim", "qwen35.attention.key_length", "u"),
            ("value_dim", "qwen35.attention.value_length", "u"),
            ("vocab_size", "tokenizer.ggml.tokens", "a"),
            ("context_length", "qwen35.context_length", "u"),
            ("rms_norm_eps", "qwen35.attention.layer_norm_rms_epsilon", "f"),
            ("rope_theta", "qwen35.rope.freq_base", "f"),
            ("eos_token_id", "tokenizer.ggml.eos_token_id", "u"),
            ("full_attention_interval", "qwen35.full_attention_interval", "u"),
            ("ssm_inner_size", "qwen35.ssm.inner_size", "u"),
            ("ssm_state_size", "qwen35.ssm.state_size", "u"),
            ("ssm_group_count", "qwen35.ssm.group_count", "u"),
            ("ssm_conv_kernel", "qwen35.ssm.conv_kernel", "u"),
            ("ssm_time_step_rank", "qwen35.ssm.time_step_rank", "u")]:
        c[field] = (_required_u32(meta, key) if kind == "u" else _required_f32(meta, key) if kind == "f"
                    else len(_required(meta, key, ARRAY)))
    ints = [k for k in c if k not in ("rms_norm_eps", "rope_theta", "eos_token_id")]
    eps, theta = c["rms_norm_eps"], c["rope_theta"]
    finite = lambda v: v == v and abs(v) != float("inf")  # noqa: E731
    if any(c[k] == 0 for k in ints) or not finite(eps) or eps <= 0 or not finite(theta) or theta <= 1:
        raise GgufError("Qwen3.6 GGUF config contains invalid dimensions")
    if c["num_attention_heads"] % c["num_key_value_heads"]:
        raise GgufError("Qwen3.6 attention heads must be divisible by key/value heads")
    if c["ssm_inner_size"] % c["ssm_state_size"]:
        raise GgufError("Qwen3.6 SSM inner size must be divisible by state size")
    rot = meta.get("qwen35.rope.dimension_count")
    if rot is None or rot[0] not in (U32, U64) or rot[1] > 0xFFFFFFFF:
        raise GgufError("GGUF model is missing qwen35.rope.dimension_count")
    c["rotary_dim"] = rot[1]
    c["ssm_value_heads"] = c["ssm_inner_size"] // c["ssm_state_size"]  # model.rs:424-426
    c["ssm_key_heads"] = c["ssm_group_count"]                           # model.rs:419-421
    return c


def layer_kind(tensor_names, layer: int, interval: int) -> str:
    """qwen35_layer_kind (model.rs:748-783): 'gdn' or 'attention'."""
    has_delta = f"blk.{layer}.ssm_a" in tensor_names
    has_attn = f"blk.{layer}.attn_q.weight" in tensor_names
    if has_delta == has_attn:
        raise GgufError(f"Qwen3.6 layer {layer} does not have exactly one execution kind")
    kind = "gdn" if has_delta else "attention"
    want = "attention" if (layer + 1) % interval == 0 else "gdn"
    if kind != want:
        raise GgufError(f"Qwen3.6 layer {layer} tensor kind disagrees with interval {interval}")
    return kind


def stage_layer_packed(data: bytes, parsed: dict, layer: int, excluded=()) -> tuple:
    """GgufModelStore::stage_qwen35_layer_packed (model.rs:920-985): the
    non-F32 tensors of blk.<layer>. that are not excluded, ordered by file
    offset, read as runs (a tensor starting within 4096 bytes of the current
    run's end extends it), packed back to back. Returns (bytes, {name:
    (start, end)}) with offsets into the packed bytes."""
    by_name = {}
    for t in parsed["tensors"]:  # a later duplicate name replaces the earlier one
        by_name[t["name"]] = t
    prefix = f"blk.{layer}."
    infos = [by_name[n] for n in sorted(by_name)
             if n.startswith(prefix) and n not in set(excluded) and by_name[n]["ggml_type"] != 0]
    infos.sort(key=lambda t: t["data_start"])  # stable
    runs = []
    for t in infos:
        if runs and t["data_start"] <= runs[-1][1] + 4096:
            runs[-1][1] = max(runs[-1][1], t["data_end"])
        else:
            runs.append([t["data_start"], t["data_end"]])
    out, ranges, off = bytearray(), {}, 0
    for a, b in runs:
        out += data[a:b]
        for t in infos:
            if t["data_start"] >= a and t["data_end"] <= b:
                s = off + (t["data_start"] - a)
                ranges[t["name"]] = (s, s + t["data_end"] - t["data_start"])
        off += b - a
    return bytes(out), ranges
