"""Whole-layer retention policies of the residency plan (si_retention; the
layer-granular forms of new_with_retained_layers_and_head,
qwen35_runtime.rs:1552-1733, retains_stride_layer 2270-2272 and
parse_layer_set 2275-2280). The plan is host code, so these run on CPU
through the dry planner."""
import pytest

from conftest import load_package

GB = 1 << 30


@pytest.fixture(scope="module")
def mai():
    return load_package()


@pytest.fixture(scope="module")
def cfg(mai):
    return mai.qwen36_27b_config()


@pytest.fixture(scope="module")
def whole(mai, cfg):
    return mai.plan_dry(cfg)


def test_default_is_the_budget_filled_prefix(mai, cfg):
    p = mai.plan_dry(cfg, budget=4 * GB)
    q = mai.plan_dry(cfg, budget=4 * GB, retention=None)
    assert p == q
    n = p["resident_layers"]
    assert p["resident"] == [l < n for l in range(cfg.layers)] and p["streamed_layers"] == 55


def test_exact_prefix_streams_every_other_layer(mai, cfg, whole):
    """retained_layers = 3 and nothing else: the reference's
    new_with_retained_layers_and_head(.., 3, true)."""
    p = mai.plan_dry(cfg, retention=mai.retention(prefix_layers=3, exact=True))
    assert p["resident"] == [l < 3 for l in range(cfg.layers)]
    assert p["streamed_layers"] == 61 and p["stage_depth"] == 3 and p["ring_bytes"] > 0
    # every layer's bytes are either resident or streamed once per token
    assert p["resident_weight_bytes"] + p["streamed_bytes_per_token"] == whole["resident_weight_bytes"]


def test_stride_retains_every_fourth_layer(mai, cfg):
    """stride 4, offset 7 keeps layers with l % 4 == 3: the attention layers."""
    p = mai.plan_dry(cfg, retention=mai.retention(stride=4, offset=7, exact=True))
    assert p["resident"] == [l % 4 == 3 for l in range(cfg.layers)]
    assert p["resident_layers"] == 16


def test_explicit_layer_set(mai, cfg):
    layers = mai.parse_layer_set("0, 5,x,63,5,,+7, -1, 2.0")
    assert layers == [0, 5, 7, 63]
    p = mai.plan_dry(cfg, retention=mai.retention(layers=layers, exact=True))
    assert [l for l in range(cfg.layers) if p["resident"][l]] == [0, 5, 7, 63]


def test_union_of_prefix_stride_and_set(mai, cfg):
    r = mai.retention(prefix_layers=2, stride=16, offset=0, layers=[40], exact=True)
    p = mai.plan_dry(cfg, retention=r)
    assert [l for l in range(cfg.layers) if p["resident"][l]] == [0, 1, 16, 32, 40, 48]


def test_non_exact_policy_fills_the_budget_after_the_set(mai, cfg):
    base = mai.plan_dry(cfg, budget=4 * GB)
    p = mai.plan_dry(cfg, budget=4 * GB, retention=mai.retention(layers=[63]))
    assert p["resident"][63]
    lead = [l for l in range(63) if p["resident"][l]]
    assert lead == list(range(len(lead)))  # then a prefix, as far as it fits
    assert len(lead) <= base["resident_layers"]
    fixed = p["resident_weight_bytes"] + p["ring_bytes"] + p["state_bytes"] + p["scratch_bytes"]
    assert fixed <= 4 * GB


def test_non_exact_policy_keeps_a_model_that_fits_whole(mai, cfg, whole):
    p = mai.plan_dry(cfg, retention=mai.retention(prefix_layers=1))
    assert p["streamed_layers"] == 0 and p["ring_bytes"] == 0 and p == {**whole, "resident": p["resident"]}


def test_exact_policy_of_every_layer_needs_no_ring(mai, cfg):
    p = mai.plan_dry(cfg, retention=mai.retention(prefix_layers=cfg.layers, exact=True))
    assert p["streamed_layers"] == 0 and p["ring_bytes"] == 0 and p["stage_depth"] == 0
    with pytest.raises(mai.SiError, match="cannot hold the retained layers") as e:
        mai.plan_dry(cfg, budget=4 * GB, retention=mai.retention(prefix_layers=cfg.layers, exact=True))
    assert e.value.status == mai.SI_E_BUDGET


def test_retained_set_over_budget_is_refused(mai, cfg):
    with pytest.raises(mai.SiError, match="retained layers need") as e:
        mai.plan_dry(cfg, budget=4 * GB, retention=mai.retention(prefix_layers=20))
    assert e.value.status == mai.SI_E_BUDGET


def test_invalid_policies_are_refused(mai, cfg):
    with pytest.raises(mai.SiError, match="outside the model's 64 layers") as e:
        mai.plan_dry(cfg, retention=mai.retention(layers=[64]))
    assert e.value.status == mai.SI_E_INVALID
    r = mai.retention()
    r.flags = 6
    with pytest.raises(mai.SiError, match="unknown retention flags"):
        mai.plan_dry(cfg, retention=r)


def test_every_rank_retains_the_same_layers(mai, cfg):
    r = mai.retention(stride=8, offset=1, exact=True)
    flags = {mai.plan_dry(cfg, n, k, 0, 3, r)["resident"] == [l % 8 == 1 for l in range(cfg.layers)]
             for n in (1, 2, 4, 8) for k in range(n)}
    assert flags == {True}


def test_stage_depth_defaults_to_three_and_clamps_at_four(mai, cfg):  # qwen35_runtime.rs:2357-2364
    """stage_pipeline_depth: unset or 0 gives 3, 2 stays 2, 99 clamps to 4
    (the reference's unparsable-string case has no counterpart: the depth is
    an integer field here)."""
    stream_all = mai.retention(exact=True)
    depth = {d: mai.plan_dry(cfg, 1, 0, 0, d, stream_all)["stage_depth"] for d in (0, 2, 99)}
    assert depth == {0: 3, 2: 2, 99: 4}
    assert mai.plan_dry(cfg, retention=stream_all)["stage_depth"] == 3


def test_layer_set_parse_kat():  # qwen35_runtime.rs:2366-2372
    mai = load_package()
    assert mai.parse_layer_set("0, 8,invalid,8, 63") == [0, 8, 63]


def test_stride_residency_kat(mai):  # qwen35_runtime.rs:2340-2347
    """retains_stride_layer: stride 2 offset 0 keeps layer 0 not 1, offset 1
    keeps 1 not 0, stride 0 keeps nothing. (The neighbouring output-prefetch
    test has no counterpart: the output head is always resident here.)"""
    c = mai.qwen36_27b_config(layers=4)
    res = lambda **kw: mai.plan_dry(c, retention=mai.retention(exact=True, **kw))["resident"]
    assert res(stride=2, offset=0) == [True, False, True, False]
    assert res(stride=2, offset=1) == [False, True, False, True]
    assert res(stride=0, offset=1) == [False] * 4


def test_plan_invariants_hold_for_random_policies(mai):
    """Property test over random shapes, budgets, depths, ranks and policies:
    every layer's bytes are either resident or streamed once per token; a
    budgeted plan fits its budget; an exact policy keeps exactly its layers;
    a non-exact one keeps at least them; failures are statuses, not crashes."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=300, deadline=None, derandomize=True)
    @given(layers=st.sampled_from([4, 8, 12, 64]), hidden=st.sampled_from([512, 1024, 5120]),
           vocab=st.sampled_from([2048, 248320]), frac=st.one_of(st.just(0.0), st.floats(0.55, 1.3)),
           depth=st.integers(0, 6),
           nranks=st.sampled_from([1, 2, 4]), prefix=st.integers(0, 70), stride=st.integers(0, 9),
           offset=st.integers(0, 9), listed=st.lists(st.integers(0, 63), max_size=5), exact=st.booleans())
    def check(layers, hidden, vocab, frac, depth, nranks, prefix, stride, offset, listed, exact):
        c = mai.qwen36_27b_config(layers=layers, hidden=hidden, vocab=vocab, intermediate=2 * hidden,
                                  kv_capacity=64)
        listed = [l for l in listed if l < layers]
        rank = nranks - 1
        whole = mai.plan_dry(c, nranks, rank, 0, 3)
        budget = int((whole["resident_weight_bytes"] + whole["state_bytes"] + whole["scratch_bytes"]) * frac)
        r = mai.retention(prefix_layers=prefix, stride=stride, offset=offset, layers=listed, exact=exact)
        want = [l < prefix or (stride and l % stride == offset % stride) or l in listed for l in range(layers)]
        try:
            p = mai.plan_dry(c, nranks, rank, budget, depth, r)
        except mai.SiError as e:
            assert e.status == mai.SI_E_BUDGET and budget > 0, str(e)
            return
        assert p["resident_weight_bytes"] + p["streamed_bytes_per_token"] == whole["resident_weight_bytes"]
        assert p["resident_layers"] + p["streamed_layers"] == layers == len(p["resident"])
        assert p["resident_layers"] == sum(p["resident"])
        if budget:
            assert p["resident_weight_bytes"] + p["ring_bytes"] + p["state_bytes"] + p["scratch_bytes"] <= budget
        if exact:
            assert p["resident"] == want
        else:
            assert all(p["resident"][l] for l in range(layers) if want[l])
        assert (p["ring_bytes"] > 0) == (p["streamed_layers"] > 0)
        assert p["stage_depth"] == (0 if not p["streamed_layers"] else (min(depth, 4) if depth else 3))

    check()


# ---- tensor-level forms (SI_RETAIN_TENSORS; qwen35_runtime.rs:1646-1682) ----

def _span(nbytes):
    """Bytes one tensor occupies in a packed layer buffer: 256-aligned, with
    64 bytes of read-ahead padding."""
    return (nbytes + 64 + 255) // 256 * 256


def _q4k(rows, cols):
    return rows * cols // 256 * 144


def _q6k(rows, cols):
    return rows * cols // 256 * 210


@pytest.fixture(scope="module")
def stream_all(mai, cfg):
    """Every layer streams, only the output head is resident."""
    return mai.plan_dry(cfg, retention=mai.retention(exact=True))


def test_mlp_policy_keeps_gate_and_up_of_every_layer(mai, cfg, stream_all, whole):
    """SI_RETAIN_MLP_STRIDE = 1: gate and up of all 64 layers resident, the
    rest of every layer streamed once per token."""
    p = mai.plan_dry(cfg, retention=mai.retention(exact=True, mlp_stride=1))
    gate_up = 2 * _span(_q4k(cfg.intermediate, cfg.hidden))
    assert p["resident"] == [False] * cfg.layers and p["streamed_layers"] == cfg.layers
    assert p["resident_weight_bytes"] - stream_all["resident_weight_bytes"] == cfg.layers * gate_up
    assert stream_all["streamed_bytes_per_token"] - p["streamed_bytes_per_token"] == cfg.layers * gate_up
    assert p["resident_weight_bytes"] + p["streamed_bytes_per_token"] == whole["resident_weight_bytes"]


def test_mlp_prefix_and_stride(mai, cfg, stream_all):
    """SI_RETAIN_MLP_LAYERS = 3 with SI_RETAIN_MLP_STRIDE 10 / offset 5:
    layers 0, 1, 2 and 5, 15, ..., 55 (3 + 6 layers)."""
    p = mai.plan_dry(cfg, retention=mai.retention(exact=True, mlp_layers=3, mlp_stride=10, mlp_offset=5))
    gate_up = 2 * _span(_q4k(cfg.intermediate, cfg.hidden))
    assert p["resident_weight_bytes"] - stream_all["resident_weight_bytes"] == 9 * gate_up


def test_down_stride_keeps_ffn_down_only(mai, cfg, stream_all):
    p = mai.plan_dry(cfg, retention=mai.retention(exact=True, down_stride=4, down_offset=2))
    down = _span(_q6k(cfg.hidden, cfg.intermediate))
    assert p["resident_weight_bytes"] - stream_all["resident_weight_bytes"] == 16 * down


def test_attention_stride_skips_gdn_layers(mai, cfg, stream_all):
    """SI_RETAIN_ATTENTION_STRIDE = 1 selects the q/k/v/output projections
    wherever they exist: only the 16 full-attention layers have them."""
    p = mai.plan_dry(cfg, retention=mai.retention(exact=True, attention_stride=1))
    qw = cfg.attn_q_heads * cfg.attn_head_dim
    kvw = cfg.attn_kv_heads * cfg.attn_head_dim
    proj = _span(_q4k(2 * qw, cfg.hidden)) + 2 * _span(_q4k(kvw, cfg.hidden)) + _span(_q4k(cfg.hidden, qw))
    assert p["resident_weight_bytes"] - stream_all["resident_weight_bytes"] == 16 * proj
    # the GDN layers (l % 4 != 3) give nothing: stride 4 offset 0 selects none
    q = mai.plan_dry(cfg, retention=mai.retention(exact=True, attention_stride=4, attention_offset=0))
    assert q["resident_weight_bytes"] == stream_all["resident_weight_bytes"]


def test_q6_policy_keeps_the_q6k_tensors_of_the_first_layers(mai, cfg, stream_all):
    """SI_RETAIN_Q6_LAYERS = 4: every Q6_K tensor of layers 0..3 (here each
    layer's ffn_down)."""
    p = mai.plan_dry(cfg, retention=mai.retention(exact=True, q6_layers=4))
    assert p["resident_weight_bytes"] - stream_all["resident_weight_bytes"] == 4 * _span(
        _q6k(cfg.hidden, cfg.intermediate))


def test_tensor_forms_only_without_a_retained_prefix(mai, cfg):
    """The reference reads the tensor-level settings only when
    retained_layers is 0 (qwen35_runtime.rs:1565)."""
    a = mai.plan_dry(cfg, retention=mai.retention(exact=True, prefix_layers=2))
    b = mai.plan_dry(cfg, retention=mai.retention(exact=True, prefix_layers=2, mlp_stride=1, down_stride=1))
    assert a == b


def test_tensor_forms_count_against_the_budget(mai, cfg):
    with pytest.raises(mai.SiError, match="retained tensors of the others") as e:
        mai.plan_dry(cfg, budget=4 * GB, retention=mai.retention(exact=True, mlp_stride=1))
    assert e.value.status == mai.SI_E_BUDGET
    # without EXACT the rest of the budget goes to leading layers, each costing
    # its bytes less the part already set aside
    p = mai.plan_dry(cfg, budget=12 * GB, retention=mai.retention(mlp_stride=2))
    lead = [l for l in range(cfg.layers) if p["resident"][l]]
    assert lead == list(range(len(lead))) and 0 < len(lead) < cfg.layers
    fixed = p["resident_weight_bytes"] + p["ring_bytes"] + p["state_bytes"] + p["scratch_bytes"]
    assert fixed <= 12 * GB


def test_sharded_ranks_keep_their_shard_of_the_same_tensors(mai, cfg, stream_all):
    """Row-sharded over 4 ranks each rank keeps its quarter of gate and up."""
    r = mai.retention(exact=True, mlp_stride=1)
    for k in range(4):
        base = mai.plan_dry(cfg, 4, k, 0, 3, mai.retention(exact=True))
        p = mai.plan_dry(cfg, 4, k, 0, 3, r)
        assert p["resident_weight_bytes"] - base["resident_weight_bytes"] == \
            cfg.layers * 2 * _span(_q4k(cfg.intermediate // 4, cfg.hidden))
