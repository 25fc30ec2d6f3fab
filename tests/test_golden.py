"""The committed golden record (tests/golden/golden.npz, made by
tests/golden/make_golden.py from the oracle) against the oracle (CPU) and
against the CUDA path (GPU): dequant and argmax exact, the rest within the
1e-5 relative L2 the other parity tests use."""
import os
import sys

import numpy as np
import pytest

import oracle as O
from helpers import rel_l2

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "golden.npz"))
TOL = 1e-5


def test_golden_inputs_are_reproducible_and_oracle_matches_record():
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_golden
    fresh = make_golden.cases()
    assert sorted(fresh) == sorted(G.files)
    for k in G.files:
        assert np.array_equal(fresh[k], G[k]), k


@pytest.mark.gpu
def test_cuda_path_matches_golden_record(ctx):
    import mai_b200 as M
    for ty in (12, 13, 14):
        assert np.array_equal(ctx.dequantize(ty, G[f"dequant_{ty}_in"], 768), G[f"dequant_{ty}_out"])
        y = ctx.gguf_quant_matvec_bytes(ty, G[f"matvec_{ty}_w"], 7, 512, G[f"matvec_{ty}_x"])
        assert rel_l2(y, G[f"matvec_{ty}_out"]) < TOL
    assert rel_l2(ctx.q4_k_fused_gate_up(G["gateup_g"], G["gateup_u"], 5, 512, G["gateup_x"]), G["gateup_out"]) < TOL
    co, cso = ctx.causal_conv1d_step(G["conv_x"], G["conv_state"], G["conv_w"], 24, 4)
    assert rel_l2(co, G["conv_out"]) < TOL and np.array_equal(cso, G["conv_state_out"])
    go, gso = ctx.gated_delta_step(G["gdn_q"], G["gdn_k"], G["gdn_v"], G["gdn_gate"], G["gdn_beta"],
                                   G["gdn_state"], 3, 8, 8)
    assert rel_l2(go, G["gdn_out"]) < TOL and rel_l2(gso, G["gdn_state_out"]) < TOL
    assert rel_l2(ctx.rms_norm_gated(G["gnorm_x"], G["gnorm_z"], G["gnorm_w"], 4, 16, 1e-6), G["gnorm_out"]) < TOL
    assert rel_l2(ctx.rms_norm_heads(G["gnorm_x"], G["hnorm_w"], 4, 16, 1e-6), G["hnorm_out"]) < TOL
    assert rel_l2(ctx.rope(G["rope_x"], 2, 16, 1234, 1e7), G["rope_out"]) < TOL
    att = ctx.attention_decode(M.AttentionDecodeInput(G["att_q"], G["att_kc"], G["att_vc"], G["att_nk"], G["att_nv"],
                                                      4, 2, 32, 37, 40))
    assert rel_l2(att, G["att_out"]) < TOL
    assert ctx.argmax(G["argmax_in"]) == int(G["argmax_out"][0]) == 999
