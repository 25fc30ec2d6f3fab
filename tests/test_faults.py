"""Host-side fault injection (si_fault_inject) on the paths that need no GPU:
GGUF header reads and payload reads fail as a short read would, the failure
comes back as a status with the reference's kind of message, and nothing is
left armed or half-open. Allocation faults are in test_gpu_failures.py."""
import numpy as np
import pytest

import gguf_writer as W

F32 = 0


@pytest.fixture
def gguf_path(tmp_path):
    payload = np.arange(64, dtype=np.float32).tobytes()
    meta = [("general.architecture", W.STRING, "qwen35"), ("general.name", W.STRING, "faults")]
    p = tmp_path / "f.gguf"
    W.write(p, meta, [("blk.0.attn_norm.weight", [64], F32, payload), ("output_norm.weight", [64], F32, payload)])
    return str(p)


@pytest.fixture(autouse=True)
def disarm(mai):
    yield
    mai.fault_inject(0)


def test_header_read_fault_fails_the_open_once(mai, gguf_path):
    mai.fault_inject(mai.FAULT_FILE_READ, 0)
    with pytest.raises(mai.SiError, match="GGUF read failed") as e:
        mai.GgufFile(gguf_path)
    assert e.value.status == mai.SI_E_INVALID
    with mai.GgufFile(gguf_path) as g:  # one-shot: the next open reads normally
        assert g.meta_string("general.name") == "faults"


def test_late_header_read_fault(mai, gguf_path):
    """A fault deep in the header (after the magic, version and counts)."""
    mai.fault_inject(mai.FAULT_FILE_READ, 5)
    with pytest.raises(mai.SiError, match="GGUF read failed"):
        mai.GgufFile(gguf_path)


def test_payload_read_fault_is_a_short_read(mai, gguf_path):
    with mai.GgufFile(gguf_path) as g:
        want = np.arange(64, dtype=np.float32).tobytes()
        mai.fault_inject(mai.FAULT_FILE_READ, 2)
        assert g.read(0).tobytes() == want
        assert g.read(1).tobytes() == want
        with pytest.raises(mai.SiError, match="unexpected end of file"):
            g.read(0)
        assert g.read(0).tobytes() == want


def test_disarm_and_unknown_site(mai, gguf_path):
    mai.fault_inject(mai.FAULT_FILE_READ, 0)
    mai.fault_inject(0)
    with mai.GgufFile(gguf_path) as g:
        assert g.read(1).size == 256
    with pytest.raises(mai.SiError, match="unknown fault site 9"):
        mai.fault_inject(9)


def test_allocation_sites_are_not_reached_without_a_device(mai, gguf_path):
    """Arming an allocation site changes nothing for host-only calls: the
    site stays armed until a device allocation asks for it, then disarms."""
    mai.fault_inject(mai.FAULT_DEVICE_ALLOC, 0)
    mai.fault_inject(mai.FAULT_PINNED_ALLOC, 0)
    with mai.GgufFile(gguf_path) as g:
        assert g.read(0).size == 256
    assert mai.plan_dry(mai.qwen36_27b_config())["streamed_layers"] == 0
