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


def test_every_entry_point_is_documented_for_binders():
    """The integration guide names every function the header declares, so a binding
    author sees the whole surface."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    header = open(os.path.join(root, "include", "si_cuda.h")).read()
    doc = open(os.path.join(root, "INTEGRATION.md")).read()
    names = sorted(set(re.findall(r"\b(si_[a-z0-9_]+)\s*\(", header)))
    missing = [n for n in names if not re.search(r"\b%s\b" % n, doc)]
    assert not missing, missing


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
