"""si-bench command line (memory-aware-inference_b200/cli/si_bench.cpp): the
reference's argument parsing, reports and exit codes (src/main.rs:1-276,
src/lib.rs:45-264). CPU tests use the mock backend and the error paths; the
GPU test runs the CUDA backend on a synthetic model and checks its ids
against the Python API."""
import json
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import PKG_DIR, load_package

CLI = os.path.join(PKG_DIR, "si-bench")


def run(*args, env=None):
    load_package().lib()  # built alongside the library
    assert os.path.exists(CLI), "si-bench is built by build.py"
    r = subprocess.run([CLI, *args], capture_output=True, text=True, timeout=600,
                       env=None if env is None else {**os.environ, **env})
    return r.returncode, r.stdout, r.stderr


def test_help_and_no_arguments_print_usage():
    for args in ([], ["--help"], ["--model", "m", "-h"]):
        rc, out, _ = run(*args)
        assert rc == 0 and out.startswith("Usage: si-bench --model PATH --backend")


def test_validates_required_arguments():  # main.rs:182-188
    rc, _, err = run("--backend", "mock")
    assert rc == 1 and "error: --model is required" in err
    rc, _, err = run("--model", "m", "--prompt", "hi")
    assert rc == 1 and "--backend is required" in err
    rc, _, err = run("--model", "m", "--backend", "mock")
    assert rc == 1 and "--prompt is required" in err
    rc, _, err = run("--model", "m", "--backend", "rocm", "--prompt", "hi")
    assert rc == 1 and "unsupported backend: rocm" in err


@pytest.mark.parametrize("args,message", [
    (["--model"], "missing value for --model"),
    (["--max-tokens", "0"], "--max-tokens must be a positive integer"),
    (["--context", "x"], "--context must be a positive integer"),
    (["--repetitions", "-2"], "--repetitions must be a positive integer"),
    (["--warmup", "-1"], "--warmup must be a non-negative integer"),
    (["--output", "xml"], "--output must be text or json"),
    (["--frobnicate", "1"], "unknown option: --frobnicate"),
    (["--prompt-ids", "1,,2"], "--prompt-ids must be comma-separated token ids"),
])
def test_argument_errors_exit_1(args, message):
    rc, _, err = run("--model", "m", "--backend", "mock", "--prompt", "hi", *args)
    assert rc == 1 and message in err and "Usage:" in err


def test_mock_json_report():  # main.rs:191-212, lib.rs:210-230
    rc, out, _ = run("--model", "m", "--backend", "mock", "--prompt", "hello big world", "--output", "json",
                     "--max-tokens", "3", "--warmup", "0")
    assert rc == 0
    d = json.loads(out)
    assert list(d) == ["model_path", "backend", "prompt_tokens", "generated_tokens", "warmup_runs", "prefill_ms",
                       "decode_ms", "prefill_tok_s", "decode_tok_s", "total_tok_s", "peak_vram_mib", "peak_ram_mib",
                       "output_match", "generated_output"]
    assert (d["backend"], d["prompt_tokens"], d["generated_tokens"], d["warmup_runs"]) == ("mock", 3, 3, 0)
    assert d["generated_output"] == "mock-0 mock-1 mock-2"
    assert (d["peak_vram_mib"], d["peak_ram_mib"], d["output_match"]) == (64, 32, None)


def test_mock_text_report_and_escaping():
    path = 'model\\"x\nq'
    rc, out, _ = run("--model", path, "--backend", "mock", "--prompt", "a", "--max-tokens", "16")
    lines = out.splitlines()
    assert rc == 0 and lines[0] == "model=model\\\"x" and lines[1] == "q"
    keys = [l.split("=")[0] for l in lines[2:]]
    assert keys == ["backend", "prompt_tokens", "generated_tokens", "warmup_runs", "prefill_ms", "decode_ms",
                    "prefill_tok_s", "decode_tok_s", "total_tok_s", "peak_vram_mib", "peak_ram_mib", "output_match",
                    "generated_output"]
    assert "peak_vram_mib=66" in lines  # 64 + 16 / 8
    rc, out, _ = run("--model", path, "--backend", "mock", "--prompt", "a", "--output", "json")
    assert rc == 0 and '"model_path":"model\\\\\\"x\\nq"' in out and json.loads(out)["model_path"] == path


def test_mock_compares_expected_output():  # lib.rs:232-238; exit code 2 on a mismatch (main.rs:24-28)
    rc, out, _ = run("--model", "m", "--backend", "mock", "--prompt", "hi", "--max-tokens", "2",
                     "--expected-output", "mock-0 mock-1", "--output", "json")
    assert rc == 0 and json.loads(out)["output_match"] is True
    rc, out, _ = run("--model", "m", "--backend", "mock", "--prompt", "hi", "--max-tokens", "2",
                     "--expected-output", "mock-0 mock-2", "--output", "json")
    assert rc == 2 and json.loads(out)["output_match"] is False


@pytest.mark.parametrize("args,message", [
    (["--prompt", "hello"], "no tokenizer: pass the prompt as token ids with --prompt-ids"),
    (["--prompt-ids", "1,2", "--chunk-rows", "16"], "does not accept --chunk-rows"),
    (["--prompt-ids", "1,2", "--quality-fixture", "q.json"], "omit --quality-fixture"),
])
def test_cuda_backend_refusals_before_any_device_work(args, message):
    rc, _, err = run("--model", "synthetic:small", "--backend", "cuda-resident", *args)
    assert rc == 1 and message in err


def test_cuda_backend_model_checks(tmp_path):
    bogus = tmp_path / "x.bin"
    bogus.write_bytes(b"NOPE" + bytes(64))
    rc, _, err = run("--model", str(bogus), "--backend", "metal-resident", "--prompt-ids", "1")
    assert rc == 1 and "unsupported model container" in err
    rc, _, err = run("--model", str(tmp_path), "--backend", "cuda-streaming", "--prompt-ids", "1")
    assert rc == 1 and "Safetensors" in err
    rc, _, err = run("--model", "synthetic:70b", "--backend", "cuda-resident", "--prompt-ids", "1")
    assert rc == 1 and "unknown synthetic model" in err


def test_cuda_backend_without_a_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    rc, _, err = run("--model", "synthetic:small", "--backend", "cuda-resident", "--prompt-ids", "1,2")
    assert rc == 1 and "error: device probe" in err


@pytest.mark.gpu
def test_cuda_backend_ids_match_the_python_api(mai, ctx):
    rc, out, err = run("--model", "synthetic:small", "--backend", "cuda-resident", "--prompt-ids", "5,77,1024",
                       "--max-tokens", "6", "--context", "64", "--warmup", "0", "--repetitions", "2",
                       "--output", "json")
    assert rc == 0, err
    d = json.loads(out)
    cfg = mai.qwen36_27b_config(hidden=512, intermediate=1024, layers=8, vocab=4096, attn_q_heads=4,
                                attn_kv_heads=2, attn_head_dim=128, rotary_dim=32, gdn_key_heads=2,
                                gdn_value_heads=4, kv_capacity=64)
    m = mai.Model(ctx, cfg, seed=27)
    ids = m.generate([5, 77, 1024], 6)
    m.close()
    assert d["generated_token_ids"] == ids and d["repetition_outputs_match"] is True
    assert d["prompt_tokens"] == 3 and d["generated_tokens"] == len(ids) and d["device"]
    assert d["peak_vram_mib"] > 0 and d["decode_tok_s"] > 0
    expected = " ".join(str(i) for i in ids)
    rc, out, _ = run("--model", "synthetic:small", "--backend", "metal-streaming", "--retain-layers", "2",
                     "--prompt-ids", "5,77,1024", "--max-tokens", "6", "--context", "64", "--warmup", "0",
                     "--repetitions", "1", "--expected-output", expected)
    assert rc == 0 and "output_match=true" in out
    rc, _, _ = run("--model", "synthetic:small", "--backend", "cuda-resident", "--prompt-ids", "5,77,1024",
                   "--max-tokens", "6", "--context", "64", "--warmup", "0", "--repetitions", "1",
                   "--expected-output", expected + " 1")
    assert rc == 2


@pytest.mark.gpu
def test_profile_lines_per_layer_and_head():
    """SI_PROFILE_QWEN35 (qwen35_runtime.rs:1920-1926, 2185-2190): a line per
    layer per decode step and a line per output head, with device times. Three
    prompt ids and six new tokens are 9 steps of 8 layers, 7 of them with the
    head (the last prompt id and every generated id)."""
    rc, out, err = run("--model", "synthetic:small", "--backend", "metal-streaming", "--retain-layers", "2",
                       "--prompt-ids", "5,77,1024", "--max-tokens", "6", "--context", "64", "--warmup", "0",
                       "--repetitions", "1", env={"SI_PROFILE_QWEN35": "1"})
    assert rc == 0, err
    layers = re.findall(r"^si_qwen35_layer layer=(\d+) ms=(\d+\.\d{3})$", err, re.M)
    heads = re.findall(r"^si_qwen35_output_head ms=(\d+\.\d{3})$", err, re.M)
    assert len(layers) == 72 and len(heads) == 7
    assert sorted({int(l) for l, _ in layers}) == list(range(8))
    assert all(float(ms) > 0 for _, ms in layers) and all(float(ms) > 0 for ms in heads)
    rc, _, err = run("--model", "synthetic:small", "--backend", "cuda-resident", "--prompt-ids", "5,77,1024",
                     "--max-tokens", "2", "--context", "64", "--warmup", "0", "--repetitions", "1")
    assert rc == 0 and "si_qwen35_layer" not in err


INSPECT = os.path.join(PKG_DIR, "si-gguf-inspect")


def inspect(*args):
    load_package().lib()
    r = subprocess.run([INSPECT, *args], capture_output=True, text=True, timeout=120)
    return r.returncode, r.stdout, r.stderr


def test_gguf_inspect_report(tmp_path):
    """si-gguf-inspect (src/bin/si-gguf-inspect.rs): the same lines, sections
    and value summaries (Rust Debug formatting of the metadata variants)."""
    import gguf_writer as W
    meta = [("general.architecture", W.STRING, "qwen35"), ("eps", W.F32, 1e-6), ("theta", W.F32, 1e7),
            ("f64", W.F64, 0.1), ("big", W.F64, 1.5e20), ("e16", W.F64, 1e16), ("e15", W.F64, 1e15),
            ("tiny", W.F64, 1e-5), ("quarter", W.F64, 0.0001), ("neg", W.I32, -7), ("flag", W.BOOL, 1),
            ("long", W.STRING, "x" * 200 + "é"), ("arr", W.ARRAY, (W.STRING, ["a", 'b"q', "c", "d"])),
            ("nums", W.ARRAY, (W.U16, [1, 2])), ("ctl", W.STRING, "a\tb\x01"), ("none", W.ARRAY, (W.U8, []))]
    tensors = [(f"blk.{i:02d}.w", [256, 1], 12, bytes(144)) for i in range(14)]
    tensors += [("output.weight", [256, 2], 14, bytes(420)), ("output_norm.weight", [256], 0, bytes(1024))]
    path = tmp_path / "m.gguf"
    W.write(path, meta, tensors)
    rc, out, _ = inspect("--model", str(path))
    assert rc == 0
    lines = out.splitlines()
    assert lines[0] == f"model={path}" and lines[1] == "tensors=16"
    q4 = [l for l in lines if l.startswith("q4_k_tensor=")]
    assert len(q4) == 12 and q4[0] == "q4_k_tensor=blk.00.w shape=[256, 1] bytes=160 elements=256"
    assert "tensor_type_counts={0: 1, 12: 14, 14: 1}" in lines
    assert "special_tensor=output.weight type=14 shape=[256, 2] bytes=448" in lines
    assert "special_tensor=output_norm.weight type=0 shape=[256] bytes=1024" in lines
    assert [l for l in lines if l.startswith("non_q4_tensor=")] == [
        "non_q4_tensor=output.weight type=14 shape=[256, 2] bytes=448",
        "non_q4_tensor=output_norm.weight type=0 shape=[256] bytes=1024"]
    md = dict(l[len("metadata."):].split("=", 1) for l in lines if l.startswith("metadata."))
    assert list(md) == sorted(md)
    assert md["general.architecture"] == 'string("qwen35")'
    assert md["eps"] == "F32(1e-6)" and md["theta"] == "F32(10000000.0)"
    assert md["f64"] == "F64(0.1)" and md["big"] == "F64(1.5e20)" and md["e16"] == "F64(1e16)"
    assert md["e15"] == "F64(1000000000000000.0)" and md["tiny"] == "F64(1e-5)" and md["quarter"] == "F64(0.0001)"
    assert md["neg"] == "I32(-7)" and md["flag"] == "Bool(true)"
    assert md["long"] == 'string(len=202, prefix="' + "x" * 160 + '")'
    assert md["arr"] == 'array(len=4, first=[string("a"), string("b\\"q"), string("c")])'
    assert md["nums"] == "array(len=2, first=[U16(1), U16(2)])" and md["none"] == "array(len=0, first=[])"
    assert md["ctl"] == 'string("a\\tb\\u{1}")'


def test_gguf_inspect_usage_and_errors(tmp_path):
    for args in ([], ["--model"], ["--path", "x"], ["--model", "a", "--other", "b"]):
        rc, _, err = inspect(*args)
        assert rc == 2 and "Usage: si-gguf-inspect --model PATH" in err
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE")
    rc, _, err = inspect("--model", str(bad))
    assert rc == 1 and "error: GGUF header has invalid magic" in err
