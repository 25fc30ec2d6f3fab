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
    """INTEGRATION.md names every function the header declares, so a binding
    author sees the whole surface."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    header = open(os.path.join(root, "include", "si_cuda.h")).read()
    doc = open(os.path.join(root, "INTEGRATION.md")).read()
    names = sorted(set(re.findall(r"\b(si_[a-z0-9_]+)\s*\(", header)))
    missing = [n for n in names if not re.search(r"\b%s\b" % n, doc)]
    assert not missing, missing
