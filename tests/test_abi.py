"""CPU-only checks of the C-ABI library: it loads and exports every symbol
that include/si_cuda.h declares (no compute calls without a GPU)."""
import ctypes
import os
import re

from conftest import REPO, load_package


def declared_symbols():
    h = open(os.path.join(REPO, "include", "si_cuda.h")).read()
    h = re.sub(r"/\*.*?\*/", "", h, flags=re.S)
    return sorted(set(re.findall(r"\b(si_[a-z0-9_]+)\s*\(", h)))


def test_library_exports_every_declared_symbol():
    mai = load_package()
    L = mai.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert len(declared_symbols()) >= 40


def test_binding_covers_every_declared_symbol():
    mai = load_package()
    src = open(os.path.join(REPO, "memory-aware-inference_b200", "__init__.py")).read()
    unbound = [s for s in declared_symbols() if f'"{s}"' not in src]
    assert not unbound, unbound


def test_context_creation_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        return
    mai = load_package()
    try:
        mai.CudaContext(0)
    except mai.SiError as e:
        assert str(e)
    else:
        raise AssertionError("context creation must fail without a device")


def test_config_helper():
    mai = load_package()
    c = mai.qwen36_27b_config()
    assert (c.hidden, c.intermediate, c.layers, c.vocab) == (5120, 17408, 64, 248320)
    assert (c.attn_q_heads, c.attn_kv_heads, c.attn_head_dim, c.rotary_dim) == (24, 4, 256, 64)
    assert (c.gdn_key_heads, c.gdn_value_heads, c.gdn_head_dim, c.conv_kernel) == (16, 48, 128, 4)
    assert abs(c.rope_theta - 1e7) < 1 and c.attn_interval == 4


# The C ABI's entry points. A change to the header's surface must be made
# here too, on purpose: bindings (Rust FFI, ctypes) are written against it.
ABI_ENTRY_POINTS = [
    'si_peer_buffer_create', 'si_peer_buffer_create_local', 'si_peer_buffer_destroy', 'si_peer_buffer_local',
    'si_sharded_qmatvec_dev', 'si_ctx_synchronize',
    'si_gdn_layer_workspace_floats', 'si_gdn_layer_dev', 'si_attention_layer_workspace_floats',
    'si_attention_layer_dev',
    'si_argmax', 'si_attention_decode', 'si_attention_decode_noalloc_dev', 'si_causal_conv1d_step',
    'si_comm_unique_id', 'si_ctx_comm_info', 'si_ctx_comm_init', 'si_ctx_create', 'si_ctx_destroy',
    'si_ctx_info', 'si_ctx_set_retention', 'si_ctx_stream', 'si_dequantize', 'si_dequantize_dev',
    'si_detect_model_format', 'si_device_probe', 'si_f32_matvec', 'si_f32_matvec_many', 'si_fault_inject',
    'si_fused_gate_up_dev', 'si_fused_mlp_dev', 'si_gated_delta_step', 'si_get_stats', 'si_gguf_advise_layer',
    'si_gguf_close', 'si_gguf_dequantize_tensor', 'si_gguf_find_tensor', 'si_gguf_info',
    'si_gguf_matvec_tensor_rows', 'si_gguf_meta_array_len', 'si_gguf_meta_f64', 'si_gguf_meta_key_at',
    'si_gguf_meta_string', 'si_gguf_meta_summary', 'si_gguf_meta_u64', 'si_gguf_open', 'si_gguf_packed_free',
    'si_gguf_packed_info', 'si_gguf_packed_range', 'si_gguf_q4_k_embedding', 'si_gguf_quant_fused_mlp_weights',
    'si_gguf_quant_matmul_many_bytes', 'si_gguf_quant_matmul_many_weight', 'si_gguf_quant_matvec_bytes',
    'si_gguf_quant_matvec_many_bytes', 'si_gguf_quant_matvec_many_tensors',
    'si_gguf_quant_matvec_many_weights', 'si_gguf_quant_matvec_weight', 'si_gguf_qwen35_config',
    'si_gguf_qwen35_layer_kind', 'si_gguf_read', 'si_gguf_stage_layer_packed', 'si_gguf_tensor_info',
    'si_gguf_tensor_payload', 'si_global_last_error', 'si_last_error', 'si_model_config_qwen36_27b',
    'si_model_create_gguf', 'si_model_create_synthetic', 'si_model_decode_hidden', 'si_model_decode_token',
    'si_model_decode_tokens_many', 'si_model_destroy', 'si_model_embed', 'si_model_generate',
    'si_model_host_tensor', 'si_model_logits', 'si_model_logits_many', 'si_model_plan', 'si_model_plan_dry',
    'si_model_plan_dry_retained', 'si_model_reset', 'si_model_resident_layers', 'si_model_resident_part_bytes', 'si_model_restore_states',
    'si_model_shard_rows', 'si_model_snapshot_free', 'si_model_snapshot_states', 'si_model_trace_begin',
    'si_model_trace_end', 'si_model_verify_many', 'si_plan_sequential_layers', 'si_q4_k_embedding_row',
    'si_q4_k_fused_gate_up', 'si_q4_k_fused_gate_up_weights', 'si_q4_k_matvec', 'si_q5_k_matvec',
    'si_q6_k_matvec', 'si_qmatmul_many_dev', 'si_qmatvec_dev', 'si_reset_peaks', 'si_rms_norm_gated',
    'si_rms_norm_heads', 'si_rope', 'si_sample_allocated', 'si_staged_layer_bind_host', 'si_staged_layer_free',
    'si_staged_layer_upload', 'si_staged_layer_weight', 'si_stats_delta', 'si_trace_action_at',
    'si_trace_count', 'si_trace_create', 'si_trace_destroy', 'si_trace_record', 'si_trace_summary',
    'si_weight_bind_host', 'si_weight_bytes', 'si_weight_device_ptr', 'si_weight_free', 'si_weight_type',
    'si_weight_upload',
]


def test_header_declares_exactly_the_abi_surface():
    import re
    header = open(os.path.join(REPO, "include", "si_cuda.h")).read()
    names = sorted(set(re.findall(r"\b(si_[a-z0-9_]+)\s*\(", header)))
    assert names == sorted(ABI_ENTRY_POINTS), (set(names) ^ set(ABI_ENTRY_POINTS))


def test_plain_c_program_uses_the_abi(tmp_path):
    """The header is C99 (-pedantic -Werror), and a C program linked against
    the library plans the 27B shape without a device, as a cgo / FFI caller
    would."""
    import subprocess
    load_package().lib()  # the library is built
    lib_dir = os.path.join(REPO, "memory-aware-inference_b200")
    src = tmp_path / "use_abi.c"
    src.write_text(r"""
#include <stdio.h>
#include "si_cuda.h"
int main(void) {
  si_model_config c;
  si_plan_info p;
  si_retention keep = {0};
  si_model_config_qwen36_27b(&c);
  if (si_model_plan_dry(&c, 1, 0, 4ull << 30, 3, &p) != SI_OK) return 1;
  keep.prefix_layers = 2;
  keep.flags = SI_RETAIN_EXACT;
  unsigned char resident[64];
  si_plan_info q;
  if (si_model_plan_dry_retained(&c, 1, 0, 0, 3, &keep, &q, resident) != SI_OK) return 2;
  if (si_model_plan_dry(&c, 1, 0, 1ull << 30, 3, &p) != SI_E_BUDGET) return 3;
  printf("%u %u %u %u\n", p.streamed_layers, q.resident_layers, resident[1], resident[2]);
  return 0;
}
""")
    exe = tmp_path / "use_abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(REPO, "include"),
                    str(src), "-L", lib_dir, "-lsi_cuda", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stderr)
    streamed_4gb, resident_exact, r1, r2 = map(int, r.stdout.split())
    assert (streamed_4gb, resident_exact, r1, r2) == (55, 2, 1, 0)
