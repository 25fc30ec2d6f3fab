"""Failure paths of model, weight and snapshot creation on the GPU, driven by
host-side fault injection (si_fault_inject): an allocation or a file read
fails as the real call would, the call returns its status with nothing left
allocated, and the context goes on working. No GPU fault is involved."""
import numpy as np
import pytest

import gguf_writer as W
from test_gpu_gguf_model import model_tensors, small_config as gguf_config
from test_gpu_model import small_config

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def disarm(mai):
    mai.fault_inject(0)
    yield
    mai.fault_inject(0)


def allocated(ctx):
    return ctx.stats()["current_allocated_bytes"]


def test_pinned_allocation_failure_during_model_creation(mai, ctx):
    cfg = small_config(mai)
    ref = mai.Model(ctx, cfg, seed=41)
    want = ref.generate([1, 2, 3], 4)
    ref.close()
    before = allocated(ctx)
    # the first layer, a middle layer, and the mapped token embeddings (after
    # the layers and the globals)
    for skip in (0, 4, cfg.layers + 1):
        mai.fault_inject(mai.FAULT_PINNED_ALLOC, skip)
        with pytest.raises(mai.SiError, match="pinned|mapped host allocation") as e:
            mai.Model(ctx, cfg, seed=41)
        assert e.value.status == mai.SI_E_NOMEM
        assert allocated(ctx) == before
    m = mai.Model(ctx, cfg, seed=41)
    assert m.generate([1, 2, 3], 4) == want
    m.close()


def test_device_allocation_failure_at_every_site_of_a_streamed_model(mai, ctx):
    """Resident weights, each ring slot, state and scratch fail in turn."""
    cfg = small_config(mai)
    full = mai.plan_dry(cfg)
    budget = int((full["resident_weight_bytes"] + full["state_bytes"] + full["scratch_bytes"]) * 0.75)
    c2 = mai.CudaContext(0, hbm_budget_bytes=budget, stage_depth=3)
    failures = 0
    for skip in range(16):
        mai.fault_inject(mai.FAULT_DEVICE_ALLOC, skip)
        try:
            m = mai.Model(c2, cfg, seed=8)
        except mai.SiError as e:
            assert e.status == mai.SI_E_NOMEM, str(e)
            assert allocated(c2) == 0
            failures += 1
            continue
        break
    mai.fault_inject(0)
    assert failures >= 5  # resident block, three ring slots, state (and scratch)
    assert m.plan()["streamed_layers"] > 0
    r = mai.Model(ctx, cfg, seed=8)
    assert m.generate([9, 99], 5) == r.generate([9, 99], 5)
    m.close()
    r.close()
    c2.close()


def test_weight_upload_and_snapshot_failures(mai, ctx):
    rng = np.random.default_rng(1)
    w = rng.integers(0, 256, 144 * 8, dtype=np.uint8)
    before = allocated(ctx)
    mai.fault_inject(mai.FAULT_DEVICE_ALLOC, 0)
    with pytest.raises(mai.SiError, match="quantized weight upload") as e:
        ctx.upload_quant_weight_private(w, 12)
    assert e.value.status == mai.SI_E_NOMEM and allocated(ctx) == before
    qw = ctx.upload_quant_weight_private(w, 12)
    ctx.free_weight(qw)
    m = mai.Model(ctx, small_config(mai), seed=3)
    mid = allocated(ctx)
    mai.fault_inject(mai.FAULT_DEVICE_ALLOC, 0)
    with pytest.raises(mai.SiError, match="state snapshot allocation") as e:
        m.snapshot_states()
    assert e.value.status == mai.SI_E_NOMEM and allocated(ctx) == mid
    with m.snapshot_states():
        pass
    assert allocated(ctx) == mid
    m.close()


def test_file_read_failure_at_every_read_of_a_gguf_load(mai, ctx, tmp_path):
    """Every header read and payload read of Model.from_gguf fails in turn;
    each attempt is refused with nothing allocated, and once the fault lands
    past the last read the model loads and decodes like a clean load."""
    c = gguf_config(mai)
    path = tmp_path / "m.gguf"
    W.write(path, W.qwen35_metadata(c), model_tensors(c, 2))
    clean = mai.Model.from_gguf(ctx, path, kv_capacity=16)
    want = clean.generate([4, 5], 3)
    clean.close()
    before = allocated(ctx)
    kinds = set()
    for skip in range(100000):
        mai.fault_inject(mai.FAULT_FILE_READ, skip)
        try:
            m = mai.Model.from_gguf(ctx, path, kv_capacity=16)
        except mai.SiError as e:
            assert e.status == mai.SI_E_INVALID
            kind = "header" if "GGUF read failed" in str(e) else "payload"
            assert kind == "header" or "unexpected end of file" in str(e), str(e)
            kinds.add(kind)
            assert allocated(ctx) == before
            continue
        break
    mai.fault_inject(0)
    assert kinds == {"header", "payload"}
    assert m.generate([4, 5], 3) == want
    m.close()
