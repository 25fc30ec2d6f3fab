"""Planner traces: the reference's planner tests (src/planner.rs:253-325)
restated against the native trace core (csrc/planner.cu), the validator's
other rejections on CPU, and the model's measured ring trace on the GPU with
the SI-003 invariants (docs/SI-003-memory-planner-spec.md:61-68)."""
import pytest

from conftest import load_package


def test_sequential_plan_evicts_each_layer_within_budget():  # planner.rs:257-288
    mai = load_package()
    t = mai.plan_sequential_layers([("layer-0", [("q0", 30), ("mlp0", 40)]), ("layer-1", [("q1", 50)])], 70)
    s = t.summary()
    assert s["planned_peak_hbm_bytes"] == 70
    assert s["resident_hbm_tensors"] == 0
    acts = t.actions()
    assert sum(a["kind"] == "execute" for a in acts) == 2
    assert [a["kind"] for a in acts] == ["prefetch", "prefetch", "execute", "evict", "evict", "prefetch", "execute",
                                         "evict"]
    assert acts[2]["tensor_ids"] == ["q0", "mlp0"] and acts[2]["bytes"] == 70 and acts[2]["queue"] == "compute"


def test_rejects_layer_larger_than_budget():  # planner.rs:290-302
    mai = load_package()
    with pytest.raises(mai.SiError, match="budget"):
        mai.plan_sequential_layers([("layer-0", [("large", 101)])], 100)
    with pytest.raises(mai.SiError, match="at least one layer"):
        mai.plan_sequential_layers([], 100)
    with pytest.raises(mai.SiError, match="non-zero"):
        mai.plan_sequential_layers([("layer-0", [("a", 1)])], 0)
    with pytest.raises(mai.SiError, match="has no tensors"):
        mai.plan_sequential_layers([("layer-0", [])], 10)


def test_trace_rejects_execute_before_prefetch():  # planner.rs:304-324
    mai = load_package()
    t = mai.Trace(mai.MODE_LAYER_STREAM)
    with pytest.raises(mai.SiError, match="non-resident"):
        t.record(mai.ACT_EXECUTE, "layer-0", ["q0"], 4, queue="compute", reason="invalid test")


def test_trace_validator_rejections():
    mai = load_package()
    t = mai.Trace()
    with pytest.raises(mai.SiError, match="must name a tensor"):
        t.record(mai.ACT_PREFETCH, "layer-0", [], 4)
    with pytest.raises(mai.SiError, match="ends before it starts"):
        t.record(mai.ACT_PREFETCH, "layer-0", ["a"], 4, started_ns=10, ended_ns=5)
    with pytest.raises(mai.SiError, match="evicts non-resident tensor a"):
        t.record(mai.ACT_EVICT, "layer-0", ["a"], 4)
    # residency is per tier: a host-resident tensor does not make an HBM execution valid
    t.record(mai.ACT_PREFETCH, "layer-0", ["a"], 4, tier=mai.TIER_PINNED_HOST)
    with pytest.raises(mai.SiError, match="non-resident"):
        t.record(mai.ACT_EXECUTE, "layer-0", ["a"], 4)
    t.record(mai.ACT_RETAIN, "layer-0", ["a", "b"], 10)  # 5 bytes each
    t.record(mai.ACT_EXECUTE, "layer-0", ["a", "b"], 10)
    t.record(mai.ACT_WAIT, "layer-0", ["a"], 0)
    t.record(mai.ACT_RELEASE, "layer-0", ["a"], 5)
    s = t.summary()
    assert s["planned_peak_hbm_bytes"] == 10 and s["resident_hbm_tensors"] == 1 and s["resident_hbm_bytes"] == 5
    assert [a["kind"] for a in t.actions()] == ["prefetch", "retain", "execute", "wait", "release"]


def _check_ring_trace(mai, m, tokens):
    t = m.trace_end()
    acts = t.actions()
    layers = m.config.layers
    plan = m.plan()
    execs = [a for a in acts if a["kind"] == "execute"]
    # every layer once per token, plus the head
    assert len(execs) == tokens * (layers + 1)
    starts = [a["started_ns"] for a in acts]
    assert starts == sorted(starts)
    streamed = {a["operation_id"] for a in acts if a["kind"] == "prefetch"}
    assert len(streamed) == plan["streamed_layers"]
    assert all("@ring-" in a["tensor_ids"][0] for a in acts if a["kind"] in ("prefetch", "evict"))
    # measured order per staged copy (layer and slot): its prefetch lands
    # before its execution, and a slot is overwritten only after the copy in
    # it has executed
    last_prefetch_end, last_exec_end = {}, {}
    for a in acts:
        op = a["tensor_ids"][0]
        if a["kind"] == "prefetch":
            last_prefetch_end[op] = a["ended_ns"]
        elif a["kind"] == "execute":
            if op in last_prefetch_end:
                assert a["started_ns"] + 1000 >= last_prefetch_end[op], op
            last_exec_end[op] = a["ended_ns"]
        elif a["kind"] == "evict":
            assert a["started_ns"] + 1000 >= last_exec_end.get(op, 0), op
    s = t.summary()
    assert s["observed"] == 1 and s["observed_peak_hbm_bytes"] > 0 and s["observed_peak_rss_bytes"] > 0
    return t, s


@pytest.mark.gpu
def test_streamed_model_trace_meets_si003_invariants(mai, ctx):
    cfg = mai.qwen36_27b_config(hidden=512, intermediate=1024, layers=8, vocab=4096, attn_q_heads=4,
                                attn_kv_heads=2, attn_head_dim=128, rotary_dim=32, gdn_key_heads=2,
                                gdn_value_heads=4, kv_capacity=40)
    full = mai.plan_dry(cfg)
    total = full["resident_weight_bytes"] + full["state_bytes"] + full["scratch_bytes"]
    c2 = mai.CudaContext(0, hbm_budget_bytes=int(total * 0.75), stage_depth=3)
    m = mai.Model(c2, cfg, seed=3)
    plan = m.plan()
    assert plan["streamed_layers"] > 0
    m.decode_token(7, 0, want_logits=False)  # the ring is primed and running
    m.trace_begin()
    for pos, tok in enumerate([11, 12, 13], start=1):
        m.decode_token(tok, pos, want_logits=False)
    t, s = _check_ring_trace(mai, m, 3)
    # the planned peak is the resident set plus the ring's occupants
    assert s["planned_peak_hbm_bytes"] <= plan["resident_weight_bytes"] + plan["ring_bytes"]
    assert s["observed_peak_hbm_bytes"] <= int(total * 0.75)
    # the verifier's window runs through the same traced ring
    m.trace_begin()
    m.verify_many([1, 2, 3, 4], [4, 5, 6, 7])
    _check_ring_trace(mai, m, 1)
    m.close()
    c2.close()


@pytest.mark.gpu
def test_resident_model_trace_is_retains_and_executes(mai, ctx):
    cfg = mai.qwen36_27b_config(hidden=512, intermediate=1024, layers=4, vocab=2048, attn_q_heads=4,
                                attn_kv_heads=2, attn_head_dim=128, rotary_dim=32, gdn_key_heads=2,
                                gdn_value_heads=4, kv_capacity=16)
    m = mai.Model(ctx, cfg, seed=3)
    m.trace_begin()
    m.generate([1, 2], 2)
    t = m.trace_end()
    kinds = {a["kind"] for a in t.actions()}
    assert kinds == {"retain", "execute"}
    assert t.summary()["mode"] == mai.MODE_RESIDENT
    with pytest.raises(mai.SiError, match="no trace"):
        m.trace_end()
    m.close()
