"""Host-side binding of the B200 decode backend (libsi_cuda.so, C ABI in
include/si_cuda.h).

`CudaContext` mirrors the reference's `MetalContext` surface for the batch-1
K-quant decode path (src/metal.rs of vrlda/memory-aware-inference): the same
method names, argument meaning and error behaviour (a failed call raises
`SiError` carrying the backend's message, the Python face of Rust's
`Err(String)`). `Model` mirrors `Qwen35Runtime` (src/qwen35_runtime.rs) for a
seeded synthetic Qwen3.6-shaped model.

There is no CPU fallback: importing this module loads the CUDA library, and a
missing library is an error.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsi_cuda.so")

GGML_TYPE_F32, GGML_TYPE_Q4_K, GGML_TYPE_Q5_K, GGML_TYPE_Q6_K = 0, 12, 13, 14
BLOCK_BYTES = {GGML_TYPE_Q4_K: 144, GGML_TYPE_Q5_K: 176, GGML_TYPE_Q6_K: 210}
CACHE_F32, CACHE_BF16 = 0, 1
# tensor ids of one decoder layer and of the globals (si_cuda.h SI_T_*)
(SI_T_ATTN_NORM, SI_T_POST_NORM, SI_T_FFN_GATE, SI_T_FFN_UP, SI_T_FFN_DOWN, SI_T_SSM_QKV, SI_T_SSM_Z,
 SI_T_SSM_ALPHA, SI_T_SSM_BETA, SI_T_SSM_CONV, SI_T_SSM_A, SI_T_SSM_DT, SI_T_SSM_NORM, SI_T_SSM_OUT,
 SI_T_ATTN_Q, SI_T_ATTN_K, SI_T_ATTN_V, SI_T_ATTN_O, SI_T_ATTN_QNORM, SI_T_ATTN_KNORM, SI_T_TOKEN_EMBD,
 SI_T_OUTPUT_NORM, SI_T_OUTPUT, SI_T_COUNT) = range(24)
SI_OK, SI_E_INVALID, SI_E_CUDA, SI_E_NOMEM, SI_E_BUDGET, SI_E_TIMEOUT, SI_E_COMM, SI_E_STATE, SI_E_UNSUPPORTED = \
    0, -1, -2, -3, -4, -5, -6, -7, -8
CTX_FLAG_NCCL_COLLECTIVES = 1  # sharded models exchange vectors with NCCL, not NVLink peer stores
TENSOR_IDS = ["ATTN_NORM", "POST_NORM", "FFN_GATE", "FFN_UP", "FFN_DOWN", "SSM_QKV", "SSM_Z", "SSM_ALPHA",
              "SSM_BETA", "SSM_CONV", "SSM_A", "SSM_DT", "SSM_NORM", "SSM_OUT", "ATTN_Q", "ATTN_K", "ATTN_V",
              "ATTN_O", "ATTN_QNORM", "ATTN_KNORM", "TOKEN_EMBD", "OUTPUT_NORM", "OUTPUT"]
T = {name: i for i, name in enumerate(TENSOR_IDS)}
T_COUNT = len(TENSOR_IDS)


class SiError(RuntimeError):
    """A backend call returned a non-zero status (reference: Err(String))."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class SiCtxConfig(C.Structure):
    _fields_ = [("hbm_budget_bytes", C.c_uint64), ("stage_depth", C.c_uint32), ("flags", C.c_uint32)]


class SiDeviceInfo(C.Structure):
    _fields_ = [("name", C.c_char * 256), ("total_bytes", C.c_uint64), ("sm_count", C.c_uint32),
                ("cc_major", C.c_uint32), ("cc_minor", C.c_uint32), ("device_count", C.c_uint32)]


def device_probe(device: int = 0) -> dict:
    """metal::probe (metal.rs:1770-1779) for a CUDA device."""
    info = SiDeviceInfo()
    rc = lib().si_device_probe(device, C.byref(info))
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())
    return {"name": info.name.decode(), "total_bytes": info.total_bytes, "sm_count": info.sm_count,
            "cc": (info.cc_major, info.cc_minor), "device_count": info.device_count}


ACT_PREFETCH, ACT_EXECUTE, ACT_RETAIN, ACT_EVICT, ACT_WAIT, ACT_RELEASE = range(6)
ACT_NAMES = ["prefetch", "execute", "retain", "evict", "wait", "release"]
TIER_MAPPED_SOURCE, TIER_PINNED_HOST, TIER_HBM, TIER_CPU, TIER_NVME = range(5)
MODE_RESIDENT, MODE_MMAP, MODE_LAYER_STREAM, MODE_SUBLAYER_STREAM, MODE_OVERLAP, MODE_HETEROGENEOUS = range(6)


class SiTraceAction(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("tier", C.c_uint32), ("operation_id", C.c_char_p),
                ("tensor_ids", C.c_char_p), ("bytes", C.c_uint64), ("started_ns", C.c_uint64),
                ("ended_ns", C.c_uint64), ("queue", C.c_char_p), ("reason", C.c_char_p)]


class SiTraceSummary(C.Structure):
    _fields_ = [("mode", C.c_uint32), ("observed", C.c_uint32), ("actions", C.c_uint64),
                ("planned_peak_hbm_bytes", C.c_uint64), ("observed_peak_hbm_bytes", C.c_uint64),
                ("observed_peak_rss_bytes", C.c_uint64), ("resident_hbm_tensors", C.c_uint64),
                ("resident_hbm_bytes", C.c_uint64)]


class SiStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("current_allocated_bytes", "peak_allocated_bytes",
                                          "peak_active_weight_bytes", "peak_kv_bytes", "peak_scratch_bytes",
                                          "submitted", "waited", "wait_nanos", "async_submitted")]


class SiAttentionDecodeInput(C.Structure):
    _fields_ = [("query", C.c_void_p), ("key_cache", C.c_void_p), ("value_cache", C.c_void_p),
                ("new_keys", C.c_void_p), ("new_values", C.c_void_p), ("query_heads", C.c_uint64),
                ("key_value_heads", C.c_uint64), ("head_dim", C.c_uint64), ("cached_tokens", C.c_uint64),
                ("cache_capacity_tokens", C.c_uint64), ("cache_type", C.c_int)]


class SiGdnLayerDesc(C.Structure):
    """si_gdn_layer_desc: one Gated DeltaNet token mixer (qwen35_runtime.rs:409-624)."""
    _fields_ = [("hidden", C.c_uint64), ("key_heads", C.c_uint32), ("value_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("conv_kernel", C.c_uint32), ("epsilon", C.c_float),
                ("qkv", C.c_void_p), ("qkv_type", C.c_uint32), ("z", C.c_void_p), ("z_type", C.c_uint32),
                ("out", C.c_void_p), ("out_type", C.c_uint32), ("conv", C.c_void_p), ("norm", C.c_void_p),
                ("alpha", C.c_void_p), ("beta", C.c_void_p), ("a_log", C.c_void_p), ("dt_bias", C.c_void_p)]


class SiAttentionLayerDesc(C.Structure):
    """si_attention_layer_desc: one full-attention token mixer (qwen35_runtime.rs:628-867)."""
    _fields_ = [("hidden", C.c_uint64), ("query_heads", C.c_uint32), ("kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("rotary_dim", C.c_uint32), ("rope_theta", C.c_float),
                ("epsilon", C.c_float), ("q", C.c_void_p), ("q_type", C.c_uint32), ("k", C.c_void_p),
                ("k_type", C.c_uint32), ("v", C.c_void_p), ("v_type", C.c_uint32), ("o", C.c_void_p),
                ("o_type", C.c_uint32), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)]


class SiModelConfig(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("layers", C.c_uint32),
                ("vocab", C.c_uint32), ("attn_interval", C.c_uint32), ("attn_q_heads", C.c_uint32),
                ("attn_kv_heads", C.c_uint32), ("attn_head_dim", C.c_uint32), ("rotary_dim", C.c_uint32),
                ("rope_theta", C.c_float), ("gdn_key_heads", C.c_uint32), ("gdn_value_heads", C.c_uint32),
                ("gdn_head_dim", C.c_uint32), ("conv_kernel", C.c_uint32), ("rms_eps", C.c_float),
                ("kv_capacity", C.c_uint32), ("eos_token", C.c_uint32), ("mlp_type", C.c_uint32),
                ("down_type", C.c_uint32), ("head_type", C.c_uint32), ("weight_init", C.c_uint32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class SiPlanInfo(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("budget_bytes", "resident_weight_bytes", "ring_bytes", "state_bytes",
                                          "scratch_bytes", "streamed_bytes_per_token")] + \
               [(n, C.c_uint32) for n in ("resident_layers", "streamed_layers", "stage_depth", "head_resident")]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class SiRetention(C.Structure):
    _fields_ = [("prefix_layers", C.c_uint32), ("stride", C.c_uint32), ("offset", C.c_uint32),
                ("layers", C.POINTER(C.c_uint32)), ("n_layers", C.c_uint32), ("flags", C.c_uint32),
                ("mlp_layers", C.c_uint32), ("mlp_stride", C.c_uint32), ("mlp_offset", C.c_uint32),
                ("q6_layers", C.c_uint32), ("down_stride", C.c_uint32), ("down_offset", C.c_uint32),
                ("attention_stride", C.c_uint32), ("attention_offset", C.c_uint32)]


RETAIN_EXACT = 1
RETAIN_TENSORS = 2


def retention(prefix_layers: int = 0, stride: int = 0, offset: int = 0, layers=(), exact: bool = False,
              mlp_layers: int = 0, mlp_stride: int = 0, mlp_offset: int = 0, q6_layers: int = 0,
              down_stride: int = 0, down_offset: int = 0, attention_stride: int = 0, attention_offset: int = 0):
    """A retention policy (si_retention). Whole layers: the first
    `prefix_layers` layers (retained_layers), every layer with
    layer % stride == offset % stride (retains_stride_layer), and the listed
    `layers` (SI_RETAIN_FULL_LAYERS) stay resident; `exact` streams all
    others (qwen35_runtime.rs:1552-1733, 2270-2280). Tensors (only while
    prefix_layers is 0, as in the reference, 1565-1682): gate/up of the first
    `mlp_layers` layers or of the mlp stride layers, every Q6_K tensor of the
    first `q6_layers` layers, ffn_down of the down stride layers and the
    q/k/v/output projections of the attention stride layers stay resident
    while the rest of their layer streams."""
    arr = (C.c_uint32 * max(len(layers), 1))(*layers)
    tensors = any((mlp_layers, mlp_stride, q6_layers, down_stride, attention_stride))
    flags = (RETAIN_EXACT if exact else 0) | (RETAIN_TENSORS if tensors else 0)
    r = SiRetention(prefix_layers, stride, offset, C.cast(arr, C.POINTER(C.c_uint32)), len(layers), flags,
                    mlp_layers, mlp_stride, mlp_offset, q6_layers, down_stride, down_offset,
                    attention_stride, attention_offset)
    r._keep = arr
    return r


def parse_layer_set(text: str) -> list:
    """parse_layer_set (qwen35_runtime.rs:2275-2280): comma-separated layer
    numbers; items that are not numbers are skipped; sorted, no repeats."""
    out = set()
    for item in text.split(","):
        item = item.strip()
        if re.fullmatch(r"\+?[0-9]+", item):  # what usize's FromStr accepts
            out.add(int(item))
    return sorted(out)


_lib = None


def lib():
    """Load libsi_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python memory-aware-inference_b200/build.py` "
                          "(or __graft_entry__.build()); there is no CPU fallback")
    L = C.CDLL(LIB_PATH)
    vp, u64, u32, i32, f32 = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int, C.c_float
    sig = {
        "si_ctx_create": ([i32, vp, vp], i32),
        "si_ctx_destroy": ([vp], None),
        "si_last_error": ([vp], C.c_char_p),
        "si_global_last_error": ([], C.c_char_p),
        "si_ctx_info": ([vp, vp, vp], i32),
        "si_device_probe": ([i32, vp], i32),
        "si_ctx_stream": ([vp], vp),
        "si_get_stats": ([vp, vp], i32),
        "si_reset_peaks": ([vp], i32),
        "si_weight_upload": ([vp, vp, u64, u32, vp], i32),
        "si_weight_bind_host": ([vp, vp, u64, u32, vp], i32),
        "si_weight_free": ([vp], None),
        "si_model_resident_part_bytes": ([vp, vp, u32], i32),
        "si_weight_bytes": ([vp], u64),
        "si_weight_type": ([vp], u32),
        "si_weight_device_ptr": ([vp], vp),
        "si_dequantize": ([vp, u32, vp, u64, u64, vp], i32),
        "si_dequantize_dev": ([vp, u32, vp, u64, vp, vp], i32),
        "si_q4_k_embedding_row": ([vp, vp, u64, u64, vp], i32),
        "si_gguf_quant_matvec_bytes": ([vp, u32, vp, u64, u64, u64, vp, vp], i32),
        "si_q4_k_matvec": ([vp, vp, u64, u64, u64, vp, vp], i32),
        "si_q5_k_matvec": ([vp, vp, u64, u64, u64, vp, vp], i32),
        "si_q6_k_matvec": ([vp, vp, u64, u64, u64, vp, vp], i32),
        "si_gguf_quant_matvec_weight": ([vp, vp, u64, u64, vp, vp], i32),
        "si_gguf_quant_matvec_many_weights": ([vp, u32, vp, vp, vp, vp, vp], i32),
        "si_qmatvec_dev": ([vp, u32, vp, u64, u64, vp, vp, vp], i32),
        "si_f32_matvec": ([vp, vp, u64, u64, vp, vp], i32),
        "si_f32_matvec_many": ([vp, u32, vp, vp, u64, vp, vp], i32),
        "si_gguf_quant_matvec_many_bytes": ([vp, u32, vp, vp, vp, vp, u64, vp, vp], i32),
        "si_staged_layer_upload": ([vp, vp, u64, u32, vp, vp, vp, vp], i32),
        "si_staged_layer_bind_host": ([vp, vp, u64, u32, vp, vp, vp, vp], i32),
        "si_staged_layer_weight": ([vp, C.c_char_p, u32, vp], i32),
        "si_staged_layer_free": ([vp], None),
        "si_gguf_matvec_tensor_rows": ([vp, vp, u64, u64, u64, vp, vp], i32),
        "si_gguf_quant_matvec_many_tensors": ([vp, vp, u32, vp, vp, u64, vp], i32),
        "si_gguf_stage_layer_packed": ([vp, u32, vp, u32, vp], i32),
        "si_gguf_packed_info": ([vp, vp, vp, vp], i32),
        "si_gguf_packed_range": ([vp, u32, vp, vp, vp], i32),
        "si_gguf_packed_free": ([vp], None),
        "si_gguf_advise_layer": ([vp, u32, vp], i32),
        "si_gguf_dequantize_tensor": ([vp, vp, u64, u32, vp, u64], i32),
        "si_gguf_q4_k_embedding": ([vp, vp, u64, u64, vp], i32),
        "si_sample_allocated": ([vp], i32),
        "si_gguf_quant_matmul_many_bytes": ([vp, u32, vp, u64, u64, u64, u64, vp, vp], i32),
        "si_gguf_quant_matmul_many_weight": ([vp, vp, u64, u64, u64, vp, vp], i32),
        "si_qmatmul_many_dev": ([vp, u32, vp, u64, u64, u64, vp, vp, vp], i32),
        "si_q4_k_fused_gate_up": ([vp, vp, vp, u64, u64, u64, vp, vp], i32),
        "si_q4_k_fused_gate_up_weights": ([vp, vp, vp, u64, u64, vp, vp], i32),
        "si_gguf_quant_fused_mlp_weights": ([vp, vp, vp, vp, u64, u64, u64, vp, vp], i32),
        "si_fused_gate_up_dev": ([vp, u32, vp, vp, u64, u64, vp, vp, vp], i32),
        "si_fused_mlp_dev": ([vp, u32, vp, vp, u32, vp, u64, u64, vp, vp, vp, vp], i32),
        "si_gated_delta_step": ([vp, vp, vp, vp, vp, vp, vp, u64, u64, u64, vp, vp], i32),
        "si_causal_conv1d_step": ([vp, vp, vp, vp, u64, u64, vp, vp], i32),
        "si_rms_norm_gated": ([vp, vp, vp, vp, u64, u64, f32, vp], i32),
        "si_rms_norm_heads": ([vp, vp, vp, u64, u64, f32, vp], i32),
        "si_rope": ([vp, vp, u64, u64, u64, f32, vp], i32),
        "si_attention_decode": ([vp, vp, vp], i32),
        "si_argmax": ([vp, vp, u64, vp], i32),
        "si_attention_decode_noalloc_dev": ([vp, vp, vp], i32),
        "si_gdn_layer_workspace_floats": ([vp], u64),
        "si_gdn_layer_dev": ([vp, vp, vp, vp, vp, vp, vp, vp, vp, vp], i32),
        "si_attention_layer_workspace_floats": ([vp, u64], u64),
        "si_attention_layer_dev": ([vp, vp, vp, u64, vp, vp, u64, u64, vp, vp, vp], i32),
        "si_peer_buffer_create": ([vp, u64, vp], i32),
        "si_peer_buffer_create_local": ([vp, u64, u32, u32, u64, vp], i32),
        "si_peer_buffer_destroy": ([vp], None),
        "si_peer_buffer_local": ([vp], vp),
        "si_sharded_qmatvec_dev": ([vp, vp, u32, vp, u64, u64, vp, u64, vp], i32),
        "si_ctx_synchronize": ([vp], i32),
        "si_model_config_qwen36_27b": ([vp], None),
        "si_model_create_synthetic": ([vp, vp, u64, vp], i32),
        "si_model_create_gguf": ([vp, C.c_char_p, u32, vp], i32),
        "si_model_destroy": ([vp], None),
        "si_model_plan": ([vp, vp], i32),
        "si_model_plan_dry": ([vp, i32, i32, u64, u32, vp], i32),
        "si_model_plan_dry_retained": ([vp, i32, i32, u64, u32, vp, vp, vp], i32),
        "si_model_resident_layers": ([vp, vp, u32], i32),
        "si_ctx_set_retention": ([vp, vp], i32),
        "si_fault_inject": ([u32, u32], i32),
        "si_stats_delta": ([vp, vp, vp], i32),
        "si_model_shard_rows": ([vp, i32, i32, u32, u32, vp, u32, vp], i32),
        "si_model_host_tensor": ([vp, u32, u32, vp, vp, vp], i32),
        "si_model_reset": ([vp], i32),
        "si_model_snapshot_states": ([vp, vp], i32),
        "si_model_restore_states": ([vp, vp], i32),
        "si_model_snapshot_free": ([vp], None),
        "si_model_embed": ([vp, u32, vp], i32),
        "si_model_decode_hidden": ([vp, u64, vp], i32),
        "si_model_logits": ([vp, vp, vp], i32),
        "si_model_decode_token": ([vp, u32, u64, vp, vp], i32),
        "si_model_generate": ([vp, vp, u64, u64, vp, vp], i32),
        "si_model_decode_tokens_many": ([vp, vp, vp, u32, vp], i32),
        "si_model_logits_many": ([vp, vp, u32, vp, vp], i32),
        "si_model_verify_many": ([vp, vp, vp, u32, vp, vp], i32),
        "si_gguf_open": ([C.c_char_p, vp], i32),
        "si_gguf_close": ([vp], None),
        "si_gguf_info": ([vp, vp, vp, vp], i32),
        "si_gguf_tensor_info": ([vp, u64, vp, vp, vp, vp, vp, vp], i32),
        "si_gguf_find_tensor": ([vp, C.c_char_p, vp], i32),
        "si_gguf_meta_u64": ([vp, C.c_char_p, vp], i32),
        "si_gguf_meta_f64": ([vp, C.c_char_p, vp], i32),
        "si_gguf_meta_string": ([vp, C.c_char_p, vp], i32),
        "si_gguf_meta_array_len": ([vp, C.c_char_p, vp], i32),
        "si_gguf_read": ([vp, u64, u64, vp, u64], i32),
        "si_gguf_qwen35_config": ([vp, u32, vp], i32),
        "si_gguf_qwen35_layer_kind": ([vp, u32, vp], i32),
        "si_gguf_meta_key_at": ([vp, u64, vp], i32),
        "si_gguf_meta_summary": ([vp, C.c_char_p, vp], i32),
        "si_gguf_tensor_payload": ([vp, u64, vp, vp, vp], i32),
        "si_detect_model_format": ([C.c_char_p, vp], i32),
        "si_trace_create": ([u32], vp),
        "si_trace_destroy": ([vp], None),
        "si_trace_record": ([vp, vp], i32),
        "si_trace_count": ([vp, vp], i32),
        "si_trace_action_at": ([vp, u64, vp], i32),
        "si_trace_summary": ([vp, vp], i32),
        "si_plan_sequential_layers": ([u32, vp, vp, vp, vp, u64, vp], i32),
        "si_model_trace_begin": ([vp], i32),
        "si_model_trace_end": ([vp, vp], i32),
        "si_comm_unique_id": ([vp], i32),
        "si_ctx_comm_init": ([vp, i32, i32, vp], i32),
        "si_ctx_comm_info": ([vp, vp, vp], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _p(a):
    """Address of a numpy array / torch tensor / int address / None. The
    result is a bare integer: the caller keeps `a` alive across the call."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if isinstance(a, bytes):  # the caller's own object, not a copy
        return C.cast(C.c_char_p(a), C.c_void_p).value
    if isinstance(a, bytearray):
        return C.addressof((C.c_char * len(a)).from_buffer(a)) if a else None
    raise TypeError(f"cannot take a pointer of {type(a)}")


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    if isinstance(a, (bytes, bytearray)):
        return np.frombuffer(bytes(a), dtype=np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8)


@dataclass
class QuantWeight:
    """Handle of a device-resident or host-bound quantized matrix (metal.rs:1840-1846)."""
    handle: int
    ggml_type: int
    byte_len: int
    _host_ref: object = None


class StagedLayer:
    """PrivateStagedQwenLayer (metal.rs:1852-1869): a packed layer promoted to
    device memory (or bound in host memory) with named tensor ranges."""

    def __init__(self, ctx, packed, ranges, upload=True):
        self.ctx = ctx
        self._bytes = _u8(packed)  # kept alive: a bound layer reads it on every use
        names = list(ranges)
        n = len(names)
        enc = (C.c_char_p * max(n, 1))(*[k.encode() for k in names])
        starts = (C.c_uint64 * max(n, 1))(*[ranges[k][0] for k in names])
        ends = (C.c_uint64 * max(n, 1))(*[ranges[k][1] for k in names])
        h = C.c_void_p()
        fn = lib().si_staged_layer_upload if upload else lib().si_staged_layer_bind_host
        ctx._ck(fn(ctx.h, _p(self._bytes), self._bytes.size, n, enc, starts, ends, C.byref(h)))
        self.h = h.value
        self._views = []

    def quant_weight(self, name: str, ggml_type: int) -> "QuantWeight":
        h = C.c_void_p()
        self.ctx._ck(lib().si_staged_layer_weight(self.h, name.encode(), ggml_type, C.byref(h)))
        w = QuantWeight(h.value, ggml_type, lib().si_weight_bytes(h.value), self)
        self._views.append(w)
        return w

    def close(self):
        if getattr(self, "h", None) and not getattr(self.ctx, "h", None):
            self.h = None  # freeing would touch the destroyed context; the copy stays until exit
            return
        if getattr(self, "h", None):
            for w in self._views:  # views the caller has not freed already
                if w.handle:
                    lib().si_weight_free(w.handle)
                    w.handle = 0
            self._views = []
            lib().si_staged_layer_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class AttentionDecodeInput:
    """metal.rs:27-38, plus the cache element type (f32 or bf16 bits as uint16)."""
    query: np.ndarray
    key_cache: np.ndarray
    value_cache: np.ndarray
    new_keys: np.ndarray
    new_values: np.ndarray
    query_heads: int
    key_value_heads: int
    head_dim: int
    cached_tokens: int
    cache_capacity_tokens: int


class CudaContext:
    """B200 replacement of MetalContext (src/metal.rs:1782-2445)."""

    def __init__(self, device: int = 0, hbm_budget_bytes: int = 0, stage_depth: int = 3, flags: int = 0):
        L = lib()
        cfg = SiCtxConfig(hbm_budget_bytes, stage_depth, flags)
        h = C.c_void_p()
        rc = L.si_ctx_create(device, C.byref(cfg), C.byref(h))
        if rc != 0:
            raise SiError(rc, L.si_global_last_error().decode())
        self.h = h.value
        self.device = device

    # -- plumbing -----------------------------------------------------------
    def _ck(self, rc):
        if rc != 0:
            raise SiError(rc, lib().si_last_error(self.h).decode())

    def close(self):
        if getattr(self, "h", None):
            lib().si_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().si_ctx_stream(self.h)

    def sm_count(self) -> int:
        d, s = C.c_int(), C.c_int()
        self._ck(lib().si_ctx_info(self.h, C.byref(d), C.byref(s)))
        return s.value

    def stats(self) -> dict:
        s = SiStats()
        self._ck(lib().si_get_stats(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in s._fields_}

    def reset_peaks(self):
        self._ck(lib().si_reset_peaks(self.h))

    def set_retention(self, retention: "SiRetention" = None):
        """The retention policy of models created on this context afterwards
        (si_ctx_set_retention); None restores the budget-filled prefix."""
        self._ck(lib().si_ctx_set_retention(self.h, C.byref(retention) if retention is not None else None))

    def comm_init(self, nranks: int, rank: int, uid: bytes):
        buf = C.create_string_buffer(bytes(uid), 128)
        self._ck(lib().si_ctx_comm_init(self.h, nranks, rank, buf))

    @staticmethod
    def comm_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        rc = lib().si_comm_unique_id(buf)
        if rc != 0:
            raise SiError(rc, lib().si_global_last_error().decode())
        return buf.raw

    # -- weights (metal.rs:2502, 2549) --------------------------------------
    def upload_quant_weight_private(self, weight_bytes, ggml_type: int) -> QuantWeight:
        b = _u8(weight_bytes)
        h = C.c_void_p()
        self._ck(lib().si_weight_upload(self.h, _p(b), b.size, ggml_type, C.byref(h)))
        return QuantWeight(h.value, ggml_type, b.size)

    def bind_quant_weight_mapped(self, weight_bytes, ggml_type: int) -> QuantWeight:
        b = _u8(weight_bytes)
        h = C.c_void_p()
        self._ck(lib().si_weight_bind_host(self.h, _p(b), b.size, ggml_type, C.byref(h)))
        return QuantWeight(h.value, ggml_type, b.size, _host_ref=b)

    def free_weight(self, w: QuantWeight):
        if w.handle:
            lib().si_weight_free(w.handle)
            w.handle = 0

    # -- dequant ---------------------------------------------------------------
    def dequantize(self, ggml_type: int, data, elements: int) -> np.ndarray:
        b = _u8(data)
        out = np.empty(max(elements, 1), np.float32)
        self._ck(lib().si_dequantize(self.h, ggml_type, _p(b), b.size, elements, _p(out)))
        return out[:elements]

    def q4_k_embedding_row(self, row_bytes, columns: int) -> np.ndarray:
        b = _u8(row_bytes)
        out = np.empty(max(columns, 1), np.float32)
        self._ck(lib().si_q4_k_embedding_row(self.h, _p(b), b.size, columns, _p(out)))
        return out[:columns]

    # -- matvec (metal.rs:3357, 3923, 4000, 4307, 4325, 4652) ----------------
    def gguf_quant_matvec_bytes(self, ggml_type, weight_bytes, rows, columns, x) -> np.ndarray:
        b, xv = _u8(weight_bytes), _f32(x)
        if xv.size != columns:
            raise SiError(-1, f"{_label(ggml_type)} matvec dimensions are invalid")
        y = np.empty(max(rows, 1), np.float32)
        self._ck(lib().si_gguf_quant_matvec_bytes(self.h, ggml_type, _p(b), b.size, rows, columns, _p(xv), _p(y)))
        return y[:rows]

    def q4_k_matvec(self, weight_bytes, rows, columns, x):
        return self.gguf_quant_matvec_bytes(GGML_TYPE_Q4_K, weight_bytes, rows, columns, x)

    def q5_k_matvec(self, weight_bytes, rows, columns, x):
        return self.gguf_quant_matvec_bytes(GGML_TYPE_Q5_K, weight_bytes, rows, columns, x)

    def q6_k_matvec(self, weight_bytes, rows, columns, x):
        return self.gguf_quant_matvec_bytes(GGML_TYPE_Q6_K, weight_bytes, rows, columns, x)

    def gguf_quant_matvec_weight(self, weight: QuantWeight, rows, columns, x) -> np.ndarray:
        return self.gguf_quant_matvec_many_weights([(weight, rows, columns)], x)[0]

    def gguf_quant_matvec_many_weights(self, items, x):
        xv = _f32(x)
        n = len(items)
        ws = (C.c_void_p * n)(*[w.handle for w, _, _ in items])
        rows = (C.c_uint64 * n)(*[r for _, r, _ in items])
        cols = (C.c_uint64 * n)(*[c for _, _, c in items])
        if any(c != xv.size for _, _, c in items):
            raise SiError(-1, "retained matvec dimensions are invalid")
        outs = [np.empty(max(r, 1), np.float32) for _, r, _ in items]
        ys = (C.c_void_p * n)(*[o.ctypes.data for o in outs])
        self._ck(lib().si_gguf_quant_matvec_many_weights(self.h, n, ws, rows, cols, _p(xv), ys))
        return [o[:r] for o, (_, r, _) in zip(outs, items)]

    def gguf_quant_matmul_many_bytes(self, ggml_type, weight_bytes, rows, columns, batch, inputs) -> np.ndarray:
        """MetalContext::gguf_quant_matmul_many_bytes: `batch` inputs (batch x
        columns) against one matrix; returns batch x rows."""
        w = _u8(weight_bytes)
        x = _f32(inputs)
        y = np.empty((batch, rows), np.float32)
        self._ck(lib().si_gguf_quant_matmul_many_bytes(self.h, ggml_type, _p(w), w.size, rows, columns, batch,
                                                       _p(x), _p(y)))
        return y

    def gguf_quant_matmul_many_weight(self, weight: QuantWeight, rows, columns, batch, inputs) -> np.ndarray:
        x = _f32(inputs)
        y = np.empty((batch, rows), np.float32)
        self._ck(lib().si_gguf_quant_matmul_many_weight(self.h, weight.handle, rows, columns, batch, _p(x), _p(y)))
        return y

    def qmatmul_many_dev(self, ggml_type, w, rows, cols, batch, x, y, stream=None):
        self._ck(lib().si_qmatmul_many_dev(self.h, ggml_type, _p(w), rows, cols, batch, _p(x), _p(y), stream))

    def sample_allocated(self):
        """MetalContext::sample_allocated: fold the current allocation into the peak."""
        self._ck(lib().si_sample_allocated(self.h))

    def gguf_quant_matvec_many_bytes(self, tensors, x):
        """MetalContext::gguf_quant_matvec_many_bytes: tensors = [(ggml_type,
        bytes, rows, columns)] sharing x; returns one output per tensor."""
        n = len(tensors)
        xs = _f32(x)
        arrs = [_u8(b) for _, b, _, _ in tensors]
        outs = [np.empty(r, np.float32) for _, _, r, _ in tensors]
        types = (C.c_uint32 * n)(*[t for t, _, _, _ in tensors])
        ptrs = (C.c_void_p * n)(*[a.ctypes.data for a in arrs])
        nbytes = (C.c_uint64 * n)(*[a.size for a in arrs])
        rows = (C.c_uint64 * n)(*[r for _, _, r, _ in tensors])
        ys = (C.c_void_p * n)(*[o.ctypes.data for o in outs])
        cols = tensors[0][3] if tensors else 0
        if any(t[3] != cols for t in tensors):
            raise SiError(SI_E_INVALID, "staged quantized matvec group input length is invalid")
        self._ck(lib().si_gguf_quant_matvec_many_bytes(self.h, n, types, ptrs, nbytes, rows, cols, _p(xs), ys))
        return outs

    def f32_matvec_many(self, matrices, x):
        """MetalContext::f32_matvec_many_gguf_tensors: F32 matrices (rows x cols) sharing x."""
        n = len(matrices)
        ms = [np.ascontiguousarray(m, np.float32) for m in matrices]
        outs = [np.empty(m.shape[0], np.float32) for m in ms]
        cols = ms[0].shape[1] if ms else 0
        ptrs = (C.c_void_p * n)(*[m.ctypes.data for m in ms])
        rows = (C.c_uint64 * n)(*[m.shape[0] for m in ms])
        ys = (C.c_void_p * n)(*[o.ctypes.data for o in outs])
        xs = _f32(x)  # held for the call: _p returns a bare address
        self._ck(lib().si_f32_matvec_many(self.h, n, ptrs, rows, cols, _p(xs), ys))
        return outs

    def upload_staged_layer_private(self, packed, ranges) -> "StagedLayer":
        """MetalContext::upload_staged_qwen_layer_private: ranges = {name: (start, end)}."""
        return StagedLayer(self, packed, ranges, upload=True)

    def bind_staged_layer_shared(self, packed, ranges) -> "StagedLayer":
        """MetalContext::bind_staged_qwen_layer_shared (the bytes stay in host memory)."""
        return StagedLayer(self, packed, ranges, upload=False)

    def gguf_matvec_tensor_rows(self, gguf: "GgufFile", name_or_index, row_start, row_count, x) -> np.ndarray:
        """MetalContext::gguf_matvec_tensor_rows over a tensor of an open GGUF file."""
        idx = gguf.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        y = np.empty(row_count, np.float32)
        xs = _f32(x)  # held for the call: _p returns a bare address
        self._ck(lib().si_gguf_matvec_tensor_rows(self.h, gguf.h, idx, row_start, row_count, _p(xs), _p(y)))
        return y

    def gguf_quant_matvec_many_tensors(self, gguf: "GgufFile", names_or_indices, x) -> list:
        """MetalContext::gguf_quant_matvec_many_tensors: several K-quant tensors
        of an open GGUF file against one input."""
        idx = [gguf.find(t) if isinstance(t, str) else int(t) for t in names_or_indices]
        xs = _f32(x)
        outs = [np.empty(gguf.tensor_info(i)["shape"][1] if len(gguf.tensor_info(i)["shape"]) > 1 else 0,
                         np.float32) for i in idx]
        ia = (C.c_uint64 * max(len(idx), 1))(*idx)
        ya = (C.c_void_p * max(len(idx), 1))(*[o.ctypes.data for o in outs])
        self._ck(lib().si_gguf_quant_matvec_many_tensors(self.h, gguf.h, len(idx), ia, _p(xs), xs.size, ya))
        return outs

    def dequantize_gguf_tensor(self, gguf: "GgufFile", name_or_index, ggml_type: int) -> np.ndarray:
        """GgufModelStore::dequantize_q4_k / _q5_k / _q6_k on the device."""
        idx = gguf.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        n = int(np.prod(gguf.tensor_info(idx)["shape"], dtype=np.uint64))
        out = np.empty(n, np.float32)
        self._ck(lib().si_gguf_dequantize_tensor(self.h, gguf.h, idx, ggml_type, _p(out), n))
        return out

    def q4_k_embedding_tensor(self, gguf: "GgufFile", name_or_index, token_id) -> np.ndarray:
        """MetalContext::q4_k_embedding_tensor over a tensor of an open GGUF file."""
        idx = gguf.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        cols = gguf.tensor_info(idx)["shape"][0]
        out = np.empty(cols, np.float32)
        self._ck(lib().si_gguf_q4_k_embedding(self.h, gguf.h, idx, token_id, _p(out)))
        return out

    def f32_matvec(self, weights, rows, columns, x):
        w, xv = _f32(weights), _f32(x)
        if w.size != rows * columns or xv.size != columns:
            raise SiError(-1, "F32 matvec dimensions are invalid")
        y = np.empty(rows, np.float32)
        self._ck(lib().si_f32_matvec(self.h, _p(w), rows, columns, _p(xv), _p(y)))
        return y

    # -- fused SwiGLU (metal.rs:3402, 3489, 3569) -----------------------------
    def q4_k_fused_gate_up(self, gate_weights, up_weights, rows, columns, x):
        g, u, xv = _u8(gate_weights), _u8(up_weights), _f32(x)
        if xv.size != columns or g.size != u.size:
            raise SiError(-1, "Q4_K fused gate/up dimensions are invalid")
        out = np.empty(max(rows, 1), np.float32)
        self._ck(lib().si_q4_k_fused_gate_up(self.h, _p(g), _p(u), g.size, rows, columns, _p(xv), _p(out)))
        return out[:rows]

    def q4_k_fused_gate_up_weights(self, gate: QuantWeight, up: QuantWeight, rows, columns, x):
        xv = _f32(x)
        out = np.empty(max(rows, 1), np.float32)
        self._ck(lib().si_q4_k_fused_gate_up_weights(self.h, gate.handle, up.handle, rows, columns, _p(xv), _p(out)))
        return out[:rows]

    def gguf_quant_fused_mlp_weights(self, gate, up, down, gate_rows, columns, down_rows, x):
        xv = _f32(x)
        y = np.empty(max(down_rows, 1), np.float32)
        self._ck(lib().si_gguf_quant_fused_mlp_weights(self.h, gate.handle, up.handle, down.handle, gate_rows,
                                                      columns, down_rows, _p(xv), _p(y)))
        return y[:down_rows]

    # -- Gated DeltaNet (metal.rs:2773, 2856, 3122, 3263) ---------------------
    def gated_delta_step(self, query, key, value, gate, beta, state, heads, key_dim, value_dim):
        q, k, v, g, b, s = map(_f32, (query, key, value, gate, beta, state))
        if (q.size != heads * key_dim or k.size != q.size or v.size != heads * value_dim or g.size != heads
                or b.size != heads or s.size != heads * key_dim * value_dim):
            raise SiError(-1, "Gated DeltaNet input or state dimensions are invalid")
        out = np.empty(heads * value_dim, np.float32)
        new_state = np.empty_like(s)
        self._ck(lib().si_gated_delta_step(self.h, _p(q), _p(k), _p(v), _p(g), _p(b), _p(s), heads, key_dim,
                                           value_dim, _p(out), _p(new_state)))
        return out, new_state

    def causal_conv1d_step(self, x, state, weights, channels, kernel_size):
        xv, s, w = _f32(x), _f32(state), _f32(weights)
        if xv.size != channels or kernel_size < 2 or s.size != channels * (kernel_size - 1) or \
                w.size != channels * kernel_size:
            raise SiError(-1, "causal convolution input, state, or weight lengths are invalid")
        out = np.empty(channels, np.float32)
        ns = np.empty_like(s)
        self._ck(lib().si_causal_conv1d_step(self.h, _p(xv), _p(s), _p(w), channels, kernel_size, _p(out), _p(ns)))
        return out, ns

    def rms_norm_gated(self, x, gate, weight, heads, head_dim, epsilon):
        xv, g, w = _f32(x), _f32(gate), _f32(weight)
        if xv.size != heads * head_dim or g.size != xv.size or w.size != head_dim:
            raise SiError(-1, "Gated RMSNorm dimensions are invalid")
        out = np.empty(heads * head_dim, np.float32)
        self._ck(lib().si_rms_norm_gated(self.h, _p(xv), _p(g), _p(w), heads, head_dim, epsilon, _p(out)))
        return out

    def rms_norm_heads(self, x, weight, heads, head_dim, epsilon):
        xv, w = _f32(x), _f32(weight)
        if xv.size != heads * head_dim or w.size != head_dim:
            raise SiError(-1, "head RMSNorm dimensions are invalid")
        out = np.empty(heads * head_dim, np.float32)
        self._ck(lib().si_rms_norm_heads(self.h, _p(xv), _p(w), heads, head_dim, epsilon, _p(out)))
        return out

    # -- attention (metal.rs:6860, 6915) ----------------------------------------
    def rope(self, x, heads, head_dim, position, theta):
        xv = _f32(x)
        if xv.size != heads * head_dim:
            raise SiError(-1, "RoPE dimensions are invalid")
        out = np.empty(max(xv.size, 1), np.float32)
        self._ck(lib().si_rope(self.h, _p(xv), heads, head_dim, position, theta, _p(out)))
        return out[:xv.size]

    def attention_decode(self, inp: AttentionDecodeInput) -> np.ndarray:
        q, nk, nv = _f32(inp.query), _f32(inp.new_keys), _f32(inp.new_values)
        kc, vc = np.ascontiguousarray(inp.key_cache), np.ascontiguousarray(inp.value_cache)
        ct = CACHE_BF16 if kc.dtype == np.uint16 else CACHE_F32
        if ct == CACHE_F32:
            kc, vc = _f32(kc), _f32(vc)
        qh, kvh, hd = inp.query_heads, inp.key_value_heads, inp.head_dim
        if q.size != qh * hd or nk.size != kvh * hd or nv.size != kvh * hd:
            raise SiError(-1, "attention query or new key/value lengths are invalid")
        if kc.size != kvh * inp.cache_capacity_tokens * hd or vc.size != kc.size:
            raise SiError(-1, "attention cache dimensions are invalid")
        s = SiAttentionDecodeInput(_p(q), _p(kc), _p(vc), _p(nk), _p(nv), qh, kvh, hd, inp.cached_tokens,
                                   inp.cache_capacity_tokens, ct)
        out = np.empty(qh * hd, np.float32)
        self._ck(lib().si_attention_decode(self.h, C.byref(s), _p(out)))
        return out

    def argmax(self, logits) -> int:
        v = _f32(logits)
        idx = C.c_uint32()
        self._ck(lib().si_argmax(self.h, _p(v), v.size, C.byref(idx)))
        return idx.value

    # -- device-pointer forms (torch tensors or raw addresses) ---------------
    def qmatvec_dev(self, ggml_type, w, rows, cols, x, y, stream=None):
        self._ck(lib().si_qmatvec_dev(self.h, ggml_type, _p(w), rows, cols, _p(x), _p(y), stream))

    def fused_gate_up_dev(self, ggml_type, gate, up, rows, cols, x, out, stream=None):
        self._ck(lib().si_fused_gate_up_dev(self.h, ggml_type, _p(gate), _p(up), rows, cols, _p(x), _p(out), stream))

    def fused_mlp_dev(self, gate_type, gate, up, down_type, down, inter, hidden, x, act, y, stream=None):
        self._ck(lib().si_fused_mlp_dev(self.h, gate_type, _p(gate), _p(up), down_type, _p(down), inter, hidden,
                                        _p(x), _p(act), _p(y), stream))

    def dequantize_dev(self, ggml_type, w, elements, out, stream=None):
        self._ck(lib().si_dequantize_dev(self.h, ggml_type, _p(w), elements, _p(out), stream))

    def synchronize(self):
        """si_ctx_synchronize: wait for the context's stream; device errors of earlier `_dev` calls."""
        self._ck(lib().si_ctx_synchronize(self.h))

    def peer_buffer(self, nbytes: int) -> "PeerBuffer":
        """si_peer_buffer_create (collective over the context's communicator)."""
        h = C.c_void_p()
        self._ck(lib().si_peer_buffer_create(self.h, nbytes, C.byref(h)))
        return PeerBuffer(self, h.value)

    def peer_buffer_local(self, nbytes: int, nranks: int, rank: int, wait_us: int = 0) -> "PeerBuffer":
        """si_peer_buffer_create_local: nranks buffers on this GPU, acting as `rank`."""
        h = C.c_void_p()
        self._ck(lib().si_peer_buffer_create_local(self.h, nbytes, nranks, rank, wait_us, C.byref(h)))
        return PeerBuffer(self, h.value, group=nranks)

    def sharded_qmatvec_dev(self, buf: "PeerBuffer", ggml_type, w_shard, rows_per_rank, cols, x, y_offset=0,
                            stream=None):
        """si_sharded_qmatvec_dev: row-sharded matvec, the whole y lands in every rank's buffer."""
        self._ck(lib().si_sharded_qmatvec_dev(self.h, buf.h, ggml_type, _p(w_shard), rows_per_rank, cols, _p(x),
                                              y_offset, stream))

    def gdn_layer_dev(self, desc: "SiGdnLayerDesc", x, conv_state_in, conv_state_out, state, gates, out, work,
                      stream=None):
        """si_gdn_layer_dev: one Gated DeltaNet token mixer on device buffers."""
        self._ck(lib().si_gdn_layer_dev(self.h, C.byref(desc), _p(x), _p(conv_state_in), _p(conv_state_out),
                                        _p(state), _p(gates), _p(out), _p(work), stream))

    def attention_layer_dev(self, desc: "SiAttentionLayerDesc", x, position, key_cache, value_cache, cached_tokens,
                            capacity_tokens, out, work, stream=None):
        """si_attention_layer_dev: one full-attention token mixer on device buffers (bf16 cache)."""
        self._ck(lib().si_attention_layer_dev(self.h, C.byref(desc), _p(x), position, _p(key_cache),
                                              _p(value_cache), cached_tokens, capacity_tokens, _p(out), _p(work),
                                              stream))


class PeerBuffer:
    """si_peer_buffer: a device buffer on every rank, mapped into every other rank."""

    def __init__(self, ctx, handle, group=None):
        self.ctx = ctx
        self.h = handle
        self.group = group

    @property
    def local(self) -> int:
        return lib().si_peer_buffer_local(self.h)

    def close(self):
        """Destroy the buffer. After its context was closed this only drops the
        handle: si_peer_buffer_destroy would touch the destroyed context."""
        if getattr(self, "h", None):
            if getattr(self.ctx, "h", None):
                lib().si_peer_buffer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def gdn_layer_workspace_floats(desc: "SiGdnLayerDesc") -> int:
    return int(lib().si_gdn_layer_workspace_floats(C.byref(desc)))


def attention_layer_workspace_floats(desc: "SiAttentionLayerDesc", cached_tokens: int) -> int:
    return int(lib().si_attention_layer_workspace_floats(C.byref(desc), cached_tokens))


def attention_decode_noalloc_dev(query, key_cache, value_cache, new_keys, new_values, query_heads,
                                 key_value_heads, head_dim, cached_tokens, cache_capacity_tokens,
                                 cache_type, out, stream=None):
    """si_attention_decode_noalloc_dev: device pointers (torch tensors or
    addresses) in and out; allocates nothing; does not synchronise."""
    s = SiAttentionDecodeInput(_p(query), _p(key_cache), _p(value_cache), _p(new_keys), _p(new_values),
                               query_heads, key_value_heads, head_dim, cached_tokens, cache_capacity_tokens,
                               cache_type)
    rc = lib().si_attention_decode_noalloc_dev(C.byref(s), _p(out), stream)
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())


def _label(t):
    return {GGML_TYPE_Q4_K: "Q4_K", GGML_TYPE_Q5_K: "Q5_K", GGML_TYPE_Q6_K: "Q6_K"}.get(t, "?")


def qwen36_27b_config(**overrides) -> SiModelConfig:
    """BASELINE config 5 shape (GgufQwen35Config of the 27B model, model.rs:1929-1971)."""
    c = SiModelConfig()
    lib().si_model_config_qwen36_27b(C.byref(c))
    for k, v in overrides.items():
        setattr(c, k, v)
    return c


def plan_dry(config: SiModelConfig, nranks: int = 1, rank: int = 0, budget: int = 0, stage_depth: int = 3,
             retention: SiRetention = None) -> dict:
    """Residency plan of a model without a device (si_model_plan_dry, or
    si_model_plan_dry_retained under a retention policy). The dict carries
    the per-layer residency as `resident` (a list of bools)."""
    p = SiPlanInfo()
    flags = (C.c_uint8 * max(config.layers, 1))()
    rc = lib().si_model_plan_dry_retained(C.byref(config), nranks, rank, budget, stage_depth,
                                          C.byref(retention) if retention is not None else None, C.byref(p), flags)
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())
    d = p.as_dict()
    d["resident"] = [bool(flags[i]) for i in range(config.layers)]
    return d


def shard_rows(config: SiModelConfig, nranks: int, rank: int, layer: int, tensor: int):
    """Full-tensor row ranges held by `rank` (si_model_shard_rows)."""
    buf = (C.c_uint64 * 16)()
    n = C.c_uint32()
    rc = lib().si_model_shard_rows(C.byref(config), nranks, rank, layer, tensor, buf, 8, C.byref(n))
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())
    return [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)]


def _gck(rc):
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())


def stats_delta(after: dict, before: dict) -> dict:
    """CommandStatsSnapshot::delta_since (si_stats_delta): the command
    counters of `after` minus `before`, saturating at 0."""
    a = SiStats(*[after.get(k, 0) for k, _ in SiStats._fields_])
    b = SiStats(*[before.get(k, 0) for k, _ in SiStats._fields_])
    out = SiStats()
    rc = lib().si_stats_delta(C.byref(a), C.byref(b), C.byref(out))
    if rc != 0:
        raise SiError(rc, "invalid stats")
    return {k: getattr(out, k) for k, _ in out._fields_}


FAULT_PINNED_ALLOC, FAULT_DEVICE_ALLOC, FAULT_FILE_READ = 1, 2, 3


def fault_inject(site: int, skip: int = 0):
    """Arm a host-side fault (si_fault_inject): the call at `site` after
    `skip` further calls fails once, as the real call would. site 0 disarms
    every site."""
    rc = lib().si_fault_inject(site, skip)
    if rc != 0:
        raise SiError(rc, lib().si_global_last_error().decode())


def detect_model_format(path) -> str:
    """detect_model_format (model.rs:42-78): "gguf" or "safetensors"."""
    f = C.c_uint32()
    _gck(lib().si_detect_model_format(os.fsencode(path), C.byref(f)))
    return "gguf" if f.value == 2 else "safetensors"


class GgufFile:
    """An open GGUF v2/v3 file: metadata and tensor index parsed on the host,
    payloads read on demand (GgufModelStore, model.rs:583-1030). No device."""

    def __init__(self, path):
        h = C.c_void_p()
        _gck(lib().si_gguf_open(os.fsencode(path), C.byref(h)))
        self.h = h.value
        ver, nt, nm = C.c_uint32(), C.c_uint64(), C.c_uint64()
        _gck(lib().si_gguf_info(self.h, C.byref(ver), C.byref(nt), C.byref(nm)))
        self.version, self.tensor_count, self.metadata_count = ver.value, nt.value, nm.value

    def close(self):
        if getattr(self, "h", None):
            lib().si_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def tensor_info(self, index: int) -> dict:
        name, nd, ty = C.c_char_p(), C.c_uint32(), C.c_uint32()
        dims, start, n = (C.c_uint64 * 4)(), C.c_uint64(), C.c_uint64()
        _gck(lib().si_gguf_tensor_info(self.h, index, C.byref(name), C.byref(nd), dims, C.byref(ty),
                                       C.byref(start), C.byref(n)))
        return {"name": name.value.decode(), "shape": [dims[i] for i in range(nd.value)], "ggml_type": ty.value,
                "data_start": start.value, "data_end": start.value + n.value}

    def tensors(self) -> list:
        return [self.tensor_info(i) for i in range(self.tensor_count)]

    def find(self, name: str) -> int:
        idx = C.c_uint64()
        _gck(lib().si_gguf_find_tensor(self.h, name.encode(), C.byref(idx)))
        return idx.value

    def meta_u64(self, key: str) -> int:
        v = C.c_uint64()
        _gck(lib().si_gguf_meta_u64(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_f64(self, key: str) -> float:
        v = C.c_double()
        _gck(lib().si_gguf_meta_f64(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_string(self, key: str) -> str:
        v = C.c_char_p()
        _gck(lib().si_gguf_meta_string(self.h, key.encode(), C.byref(v)))
        return v.value.decode()

    def meta_array_len(self, key: str) -> int:
        v = C.c_uint64()
        _gck(lib().si_gguf_meta_array_len(self.h, key.encode(), C.byref(v)))
        return v.value

    def read(self, name_or_index, offset: int = 0, nbytes: int = None) -> np.ndarray:
        idx = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        if nbytes is None:
            info = self.tensor_info(idx)
            nbytes = info["data_end"] - info["data_start"] - offset
        out = np.empty(nbytes, np.uint8)
        _gck(lib().si_gguf_read(self.h, idx, offset, _p(out), nbytes))
        return out

    def metadata(self) -> dict:
        """Every metadata key (in the store's byte order) with its value
        summarised as si-gguf-inspect prints it."""
        out = {}
        for i in range(self.metadata_count):
            k, v = C.c_char_p(), C.c_char_p()
            _gck(lib().si_gguf_meta_key_at(self.h, i, C.byref(k)))
            _gck(lib().si_gguf_meta_summary(self.h, k.value, C.byref(v)))
            out[k.value.decode()] = v.value.decode()
        return out

    def layer_kind(self, layer: int) -> str:
        """qwen35_layer_kind (model.rs:748-783): "gated_delta_net" or "full_attention"."""
        k = C.c_uint32()
        _gck(lib().si_gguf_qwen35_layer_kind(self.h, layer, C.byref(k)))
        return "full_attention" if k.value == 1 else "gated_delta_net"

    def layer_kinds(self) -> list:
        return [self.layer_kind(l) for l in range(self.meta_u64("qwen35.block_count"))]

    def tensor_payload(self, index: int):
        """(element_count, expected_payload_bytes or None) (model.rs:512-573)."""
        n, b, k = C.c_uint64(), C.c_uint64(), C.c_uint32()
        _gck(lib().si_gguf_tensor_payload(self.h, index, C.byref(n), C.byref(b), C.byref(k)))
        return n.value, (b.value if k.value else None)

    def advise_layer(self, layer: int) -> int:
        """GgufModelStore::advise_qwen35_layer: read-ahead hint for a layer;
        returns the page-aligned bytes advised."""
        n = C.c_uint64()
        _gck(lib().si_gguf_advise_layer(self.h, layer, C.byref(n)))
        return n.value

    def stage_layer_packed(self, layer: int, excluded=()):
        """GgufModelStore::stage_qwen35_layer_packed: (packed bytes, {name:
        (start, end)}) of a layer's quantized tensors, read from the file as
        merged runs; the pair feeds CudaContext.upload_staged_layer_private."""
        names = [n.encode() for n in excluded]
        arr = (C.c_char_p * max(len(names), 1))(*names)
        h = C.c_void_p()
        _gck(lib().si_gguf_stage_layer_packed(self.h, layer, arr, len(names), C.byref(h)))
        try:
            ptr, nb, nr = C.c_void_p(), C.c_uint64(), C.c_uint32()
            _gck(lib().si_gguf_packed_info(h, C.byref(ptr), C.byref(nb), C.byref(nr)))
            data = np.empty(nb.value, np.uint8)
            if nb.value:
                C.memmove(data.ctypes.data, ptr.value, nb.value)
            ranges = {}
            for i in range(nr.value):
                name, a, b = C.c_char_p(), C.c_uint64(), C.c_uint64()
                _gck(lib().si_gguf_packed_range(h, i, C.byref(name), C.byref(a), C.byref(b)))
                ranges[name.value.decode()] = (a.value, b.value)
            return data, ranges
        finally:
            lib().si_gguf_packed_free(h)

    def qwen35_config(self, kv_capacity: int = 0) -> SiModelConfig:
        c = SiModelConfig()
        _gck(lib().si_gguf_qwen35_config(self.h, kv_capacity, C.byref(c)))
        return c


class Trace:
    """A planner trace (PlannerTrace, planner.rs:62-170): actions validated as
    they are recorded against the residency they imply."""

    def __init__(self, mode: int = MODE_LAYER_STREAM, handle=None):
        self.h = handle if handle is not None else lib().si_trace_create(mode)

    def close(self):
        if getattr(self, "h", None):
            lib().si_trace_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def record(self, kind, operation_id, tensor_ids, nbytes, started_ns=0, ended_ns=0, tier=TIER_HBM, queue="",
               reason=""):
        a = SiTraceAction(kind, tier, operation_id.encode(), ",".join(tensor_ids).encode(), nbytes, started_ns,
                          ended_ns, queue.encode(), reason.encode())
        _gck(lib().si_trace_record(self.h, C.byref(a)))

    def actions(self) -> list:
        n = C.c_uint64()
        _gck(lib().si_trace_count(self.h, C.byref(n)))
        out = []
        for i in range(n.value):
            a = SiTraceAction()
            _gck(lib().si_trace_action_at(self.h, i, C.byref(a)))
            out.append({"kind": ACT_NAMES[a.kind], "tier": a.tier, "operation_id": a.operation_id.decode(),
                        "tensor_ids": a.tensor_ids.decode().split(",") if a.tensor_ids else [],
                        "bytes": a.bytes, "started_ns": a.started_ns, "ended_ns": a.ended_ns,
                        "queue": a.queue.decode(), "reason": a.reason.decode()})
        return out

    def summary(self) -> dict:
        s = SiTraceSummary()
        _gck(lib().si_trace_summary(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in s._fields_}


def plan_sequential_layers(layers, budget_bytes: int) -> Trace:
    """plan_sequential_layers (planner.rs:174-251): layers = [(operation_id,
    [(tensor_id, bytes), ...]), ...]."""
    n = len(layers)
    ops = (C.c_char_p * max(n, 1))(*[op.encode() for op, _ in layers])
    counts = (C.c_uint32 * max(n, 1))(*[len(t) for _, t in layers])
    flat = [t for _, ts in layers for t in ts]
    ids = (C.c_char_p * max(len(flat), 1))(*[tid.encode() for tid, _ in flat])
    nbytes = (C.c_uint64 * max(len(flat), 1))(*[b for _, b in flat])
    h = C.c_void_p()
    _gck(lib().si_plan_sequential_layers(n, ops, counts, ids, nbytes, budget_bytes, C.byref(h)))
    return Trace(handle=h.value)


class StateSnapshot:
    """A model's layer states at one point of decoding (si_model_snapshot).
    It holds a reference to its context. If that context was closed first,
    close() only drops the handle: the device copy stays allocated until the
    process exits, because freeing it would touch the destroyed context."""

    def __init__(self, ctx: "CudaContext", handle):
        self.ctx, self.h = ctx, handle

    def close(self):
        if getattr(self, "h", None):
            if getattr(self.ctx, "h", None):
                lib().si_model_snapshot_free(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """Synthetic Qwen3.6-shaped decoder (Qwen35Runtime, qwen35_runtime.rs:1519-2267)."""

    def __init__(self, ctx: CudaContext, config: SiModelConfig, seed: int):
        self.ctx = ctx
        self.config = config
        h = C.c_void_p()
        ctx._ck(lib().si_model_create_synthetic(ctx.h, C.byref(config), seed, C.byref(h)))
        self.h = h.value

    @classmethod
    def from_gguf(cls, ctx: CudaContext, path, kv_capacity: int = 0) -> "Model":
        """Load a qwen35 GGUF file (si_model_create_gguf): config from its
        metadata, this rank's row shards read from the file."""
        with GgufFile(path) as g:
            config = g.qwen35_config(kv_capacity)
        m = cls.__new__(cls)
        m.ctx, m.config = ctx, config
        h = C.c_void_p()
        ctx._ck(lib().si_model_create_gguf(ctx.h, os.fsencode(path), kv_capacity, C.byref(h)))
        m.h = h.value
        return m

    def close(self):
        """Destroy the model. After its context was closed this only drops the
        handle: si_model_destroy would touch the destroyed context."""
        if getattr(self, "h", None):
            if getattr(self.ctx, "h", None):
                lib().si_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def plan(self) -> dict:
        p = SiPlanInfo()
        self.ctx._ck(lib().si_model_plan(self.h, C.byref(p)))
        return p.as_dict()

    def resident_layers(self) -> list:
        """Per layer, whether it is resident in HBM (si_model_resident_layers)."""
        flags = (C.c_uint8 * max(self.config.layers, 1))()
        self.ctx._ck(lib().si_model_resident_layers(self.h, flags, self.config.layers))
        return [bool(flags[i]) for i in range(self.config.layers)]

    def resident_part_bytes(self) -> list:
        """Per layer, the bytes kept resident of a streamed layer by a
        tensor-level policy (si_model_resident_part_bytes)."""
        vals = (C.c_uint64 * max(self.config.layers, 1))()
        self.ctx._ck(lib().si_model_resident_part_bytes(self.h, vals, self.config.layers))
        return [int(vals[i]) for i in range(self.config.layers)]

    def host_tensor(self, layer: int, tensor: int):
        """(address, bytes, ggml_type) of this rank's pinned host copy of a tensor."""
        ptr, nb, ty = C.c_void_p(), C.c_uint64(), C.c_uint32()
        self.ctx._ck(lib().si_model_host_tensor(self.h, layer, tensor, C.byref(ptr), C.byref(nb), C.byref(ty)))
        return ptr.value, nb.value, ty.value

    def host_tensor_array(self, layer: int, tensor: int) -> np.ndarray:
        ptr, nb, ty = self.host_tensor(layer, tensor)
        if not ptr:
            return np.empty(0, np.uint8)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(nb,))

    def reset(self):
        self.ctx._ck(lib().si_model_reset(self.h))

    def snapshot_states(self) -> "StateSnapshot":
        """Qwen35Runtime::snapshot_states: a device copy of every layer's
        recurrent, conv and KV state (qwen35_runtime.rs:1764-1766)."""
        h = C.c_void_p()
        self.ctx._ck(lib().si_model_snapshot_states(self.h, C.byref(h)))
        return StateSnapshot(self.ctx, h.value)

    def restore_states(self, snapshot: "StateSnapshot"):
        """Qwen35Runtime::restore_states (qwen35_runtime.rs:1768-1775)."""
        self.ctx._ck(lib().si_model_restore_states(self.h, snapshot.h))

    def embed_token(self, token_id: int) -> np.ndarray:
        out = np.empty(self.config.hidden, np.float32)
        self.ctx._ck(lib().si_model_embed(self.h, token_id, _p(out)))
        return out

    def decode_hidden(self, position: int, hidden) -> np.ndarray:
        h = np.array(hidden, np.float32, copy=True)
        self.ctx._ck(lib().si_model_decode_hidden(self.h, position, _p(h)))
        return h

    def logits(self, hidden) -> np.ndarray:
        h = _f32(hidden)
        out = np.empty(self.config.vocab, np.float32)
        self.ctx._ck(lib().si_model_logits(self.h, _p(h), _p(out)))
        return out

    def decode_token(self, token_id: int, position: int, want_logits: bool = True):
        nxt = C.c_uint32()
        logits = np.empty(self.config.vocab, np.float32) if want_logits else None
        self.ctx._ck(lib().si_model_decode_token(self.h, token_id, position, C.byref(nxt), _p(logits)))
        return nxt.value, logits

    def trace_begin(self):
        """Start recording the ring's prefetch / execute / evict actions."""
        self.ctx._ck(lib().si_model_trace_begin(self.h))

    def trace_end(self) -> Trace:
        """The measured trace since trace_begin, validated (SI-003 invariants)."""
        h = C.c_void_p()
        self.ctx._ck(lib().si_model_trace_end(self.h, C.byref(h)))
        return Trace(handle=h.value)

    def decode_tokens_many(self, tokens, positions, want_hidden: bool = True):
        """Qwen35Runtime::decode_tokens_many: hidden states (n x hidden) of a
        1..8 token window, every layer's weights traversed once."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint64)
        out = np.empty((t.size, self.config.hidden), np.float32) if want_hidden else None
        self.ctx._ck(lib().si_model_decode_tokens_many(self.h, _p(t), _p(p), t.size, _p(out)))
        return out

    def logits_many(self, hidden=None, n: int = None, want_logits: bool = True):
        """Qwen35Runtime::logits_many: (logits n x vocab or None, greedy ids).
        hidden=None uses the device states of the last decode_tokens_many."""
        h = None if hidden is None else _f32(hidden).reshape(-1, self.config.hidden)
        n = h.shape[0] if h is not None else n
        logits = np.empty((n, self.config.vocab), np.float32) if want_logits else None
        ids = np.empty(n, np.uint32)
        self.ctx._ck(lib().si_model_logits_many(self.h, _p(h), n, _p(logits), _p(ids)))
        return logits, ids.tolist()

    def verify_many(self, tokens, positions, want_logits: bool = False):
        """decode_tokens_many + logits_many: (greedy ids, logits or None)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint64)
        logits = np.empty((t.size, self.config.vocab), np.float32) if want_logits else None
        ids = np.empty(t.size, np.uint32)
        self.ctx._ck(lib().si_model_verify_many(self.h, _p(t), _p(p), t.size, _p(ids), _p(logits)))
        return ids.tolist(), logits

    def generate(self, prompt, max_new_tokens: int):
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_new_tokens, 1), np.uint32)
        n = C.c_uint64()
        self.ctx._ck(lib().si_model_generate(self.h, _p(p), p.size, max_new_tokens, _p(out), C.byref(n)))
        return out[:n.value].tolist()
