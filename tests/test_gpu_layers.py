"""Whole token mixers at the BASELINE shapes against the oracle.

Config 3: one Gated DeltaNet layer (16 key / 48 value heads, head_dim 128,
conv kernel 4, hidden 5120, Q4_K qkv / z / ssm_out), recurrent state
~N(0, 0.1), gates supplied directly (g = -softplus(N(0,1)),
beta = sigmoid(N(0,1))), 64 consecutive tokens carrying the conv and recurrent
state (gdn_token_mixer, qwen35_runtime.rs:409-624).

Config 4: one full-attention layer (24 q / 4 kv heads, head_dim 256, partial
RoPE on 64 dims, theta 1e7, Q4_K q/k/v/o) over a bf16 cache holding 8192
positions ~N(0,1), queried at position 8192 and then 8193
(attention_token_mixer, qwen35_runtime.rs:628-867).

Both run through si_gdn_layer_dev / si_attention_layer_dev; each token's
mixer output and the carried state agree with the oracle within the 1e-5
relative-L2 tolerance of the other float tests.
"""
import numpy as np
import pytest

import oracle as O
from helpers import random_blocks, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5


def bf16_to_f32(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_gdn_layer_config3_64_tokens_match_oracle(mai, ctx):
    import torch
    cfg = mai.qwen36_27b_config()
    H, kh, vh, d, K = cfg.hidden, cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.gdn_head_dim, cfg.conv_kernel
    vw, proj = vh * d, (2 * kh + vh) * d
    rng = np.random.default_rng(3003)
    qkv = random_blocks(rng, 12, proj * H // 256)
    z = random_blocks(rng, 12, vw * H // 256)
    out_w = random_blocks(rng, 12, H * vw // 256)
    conv = rng.normal(0, 0.3, proj * K).astype(np.float32)
    norm = (1.0 + rng.normal(0, 0.1, d)).astype(np.float32)
    state0 = rng.normal(0, 0.1, vh * d * d).astype(np.float32)
    tensors = {mai.SI_T_SSM_QKV: (qkv, 12), mai.SI_T_SSM_Z: (z, 12), mai.SI_T_SSM_OUT: (out_w, 12),
               mai.SI_T_SSM_CONV: (conv, 0), mai.SI_T_SSM_NORM: (norm, 0)}
    desc = mai.SiGdnLayerDesc()
    desc.hidden, desc.key_heads, desc.value_heads, desc.head_dim, desc.conv_kernel = H, kh, vh, d, K
    desc.epsilon = cfg.rms_eps
    dq, dz, do, dc, dn = (_dev(torch, a) for a in (qkv, z, out_w, conv, norm))
    desc.qkv, desc.qkv_type = dq.data_ptr(), 12
    desc.z, desc.z_type = dz.data_ptr(), 12
    desc.out, desc.out_type = do.data_ptr(), 12
    desc.conv, desc.norm = dc.data_ptr(), dn.data_ptr()
    work = torch.empty(mai.gdn_layer_workspace_floats(desc), device="cuda")
    conv_dev = [torch.zeros(proj * (K - 1), device="cuda") for _ in range(2)]
    state_dev = _dev(torch, state0)
    out_dev = torch.empty(H, device="cuda")
    conv_cpu = np.zeros(proj * (K - 1), np.float32)
    state_cpu = state0.copy()
    worst = 0.0
    for t in range(64):
        x = rng.normal(0, 1, H).astype(np.float32)
        a = rng.normal(0, 1, vh)
        gates = np.concatenate([-np.log1p(np.exp(a)), 1.0 / (1.0 + np.exp(-rng.normal(0, 1, vh)))]).astype(np.float32)
        ctx.gdn_layer_dev(desc, _dev(torch, x), conv_dev[t % 2], conv_dev[(t + 1) % 2], state_dev,
                          _dev(torch, gates), out_dev, work)
        ref = O.gdn_layer(cfg, tensors, x, conv_cpu, state_cpu, gates)
        got = out_dev.cpu().numpy()
        e = rel_l2(got, ref)
        worst = max(worst, e)
        assert e < TOL, (t, e)
    assert rel_l2(state_dev.cpu().numpy(), state_cpu) < TOL
    assert rel_l2(conv_dev[0].cpu().numpy(), conv_cpu) < TOL  # 64 tokens: the last write went to buffer 0
    assert worst > 0.0  # the comparison is not vacuous


def test_gdn_layer_computed_gates_match_oracle(mai, ctx):
    """Without supplied gates, g and beta come from the F32 alpha/beta
    projections, A_log and dt_bias (qwen35_runtime.rs:577-601)."""
    import torch
    cfg = mai.qwen36_27b_config(hidden=1024, gdn_key_heads=4, gdn_value_heads=8)
    H, kh, vh, d, K = cfg.hidden, cfg.gdn_key_heads, cfg.gdn_value_heads, 128, cfg.conv_kernel
    vw, proj = vh * d, (2 * kh + vh) * d
    rng = np.random.default_rng(3004)
    qkv, z, out_w = (random_blocks(rng, ty, r * c // 256) for ty, r, c in ((13, proj, H), (14, vw, H), (12, H, vw)))
    conv = rng.normal(0, 0.3, proj * K).astype(np.float32)
    norm = (1.0 + rng.normal(0, 0.1, d)).astype(np.float32)
    alpha = rng.normal(0, 0.02, vh * H).astype(np.float32)
    beta = rng.normal(0, 0.02, vh * H).astype(np.float32)
    a_log = rng.normal(0, 0.5, vh).astype(np.float32)
    dt = rng.normal(0, 0.5, vh).astype(np.float32)
    tensors = {mai.SI_T_SSM_QKV: (qkv, 13), mai.SI_T_SSM_Z: (z, 14), mai.SI_T_SSM_OUT: (out_w, 12),
               mai.SI_T_SSM_CONV: (conv, 0), mai.SI_T_SSM_NORM: (norm, 0), mai.SI_T_SSM_ALPHA: (alpha, 0),
               mai.SI_T_SSM_BETA: (beta, 0), mai.SI_T_SSM_A: (a_log, 0), mai.SI_T_SSM_DT: (dt, 0)}
    dev = {k: _dev(torch, v[0]) for k, v in tensors.items()}
    desc = mai.SiGdnLayerDesc()
    desc.hidden, desc.key_heads, desc.value_heads, desc.head_dim, desc.conv_kernel = H, kh, vh, d, K
    desc.epsilon = cfg.rms_eps
    desc.qkv, desc.qkv_type = dev[mai.SI_T_SSM_QKV].data_ptr(), 13
    desc.z, desc.z_type = dev[mai.SI_T_SSM_Z].data_ptr(), 14
    desc.out, desc.out_type = dev[mai.SI_T_SSM_OUT].data_ptr(), 12
    desc.conv, desc.norm = dev[mai.SI_T_SSM_CONV].data_ptr(), dev[mai.SI_T_SSM_NORM].data_ptr()
    desc.alpha, desc.beta = dev[mai.SI_T_SSM_ALPHA].data_ptr(), dev[mai.SI_T_SSM_BETA].data_ptr()
    desc.a_log, desc.dt_bias = dev[mai.SI_T_SSM_A].data_ptr(), dev[mai.SI_T_SSM_DT].data_ptr()
    work = torch.empty(mai.gdn_layer_workspace_floats(desc), device="cuda")
    conv_dev = [torch.zeros(proj * (K - 1), device="cuda") for _ in range(2)]
    state_dev = torch.zeros(vh * d * d, device="cuda")
    out_dev = torch.empty(H, device="cuda")
    conv_cpu = np.zeros(proj * (K - 1), np.float32)
    state_cpu = np.zeros(vh * d * d, np.float32)
    for t in range(8):
        x = rng.normal(0, 1, H).astype(np.float32)
        ctx.gdn_layer_dev(desc, _dev(torch, x), conv_dev[t % 2], conv_dev[(t + 1) % 2], state_dev, None, out_dev,
                          work)
        ref = O.gdn_layer(cfg, tensors, x, conv_cpu, state_cpu)
        assert rel_l2(out_dev.cpu().numpy(), ref) < TOL, t
    assert rel_l2(state_dev.cpu().numpy(), state_cpu) < TOL


def test_gdn_layer_rejects_aliased_conv_state(mai, ctx):
    import torch
    desc = mai.SiGdnLayerDesc()
    desc.hidden, desc.key_heads, desc.value_heads, desc.head_dim, desc.conv_kernel = 256, 1, 2, 128, 4
    buf = torch.zeros(1 << 16, device="cuda")
    desc.qkv = desc.z = desc.out = desc.conv = desc.norm = buf.data_ptr()
    desc.qkv_type = desc.z_type = desc.out_type = 12
    with pytest.raises(mai.SiError, match="different buffers"):
        ctx.gdn_layer_dev(desc, buf, buf, buf, buf, buf, buf, buf)


def test_attention_layer_config4_at_position_8192_matches_oracle(mai, ctx):
    import torch
    cfg = mai.qwen36_27b_config(kv_capacity=8194)
    H, qh, kvh, hd = cfg.hidden, cfg.attn_q_heads, cfg.attn_kv_heads, cfg.attn_head_dim
    qw, kvw, cap = qh * hd, kvh * hd, cfg.kv_capacity
    rng = np.random.default_rng(4004)
    wq = random_blocks(rng, 12, 2 * qw * H // 256)
    wk = random_blocks(rng, 12, kvw * H // 256)
    wv = random_blocks(rng, 12, kvw * H // 256)
    wo = random_blocks(rng, 12, H * qw // 256)
    qn = rng.normal(0, 0.1, hd).astype(np.float32)
    kn = rng.normal(0, 0.1, hd).astype(np.float32)
    cached = 8192
    kc = np.zeros((kvh, cap, hd), np.uint16)
    vc = np.zeros((kvh, cap, hd), np.uint16)
    kc[:, :cached] = O.f32_to_bf16(rng.normal(0, 1, (kvh, cached, hd)).astype(np.float32)).reshape(kvh, cached, hd)
    vc[:, :cached] = O.f32_to_bf16(rng.normal(0, 1, (kvh, cached, hd)).astype(np.float32)).reshape(kvh, cached, hd)
    tensors = {mai.SI_T_ATTN_Q: (wq, 12), mai.SI_T_ATTN_K: (wk, 12), mai.SI_T_ATTN_V: (wv, 12),
               mai.SI_T_ATTN_O: (wo, 12), mai.SI_T_ATTN_QNORM: (qn, 0), mai.SI_T_ATTN_KNORM: (kn, 0)}
    dev = {k: _dev(torch, v[0]) for k, v in tensors.items()}
    desc = mai.SiAttentionLayerDesc()
    desc.hidden, desc.query_heads, desc.kv_heads, desc.head_dim = H, qh, kvh, hd
    desc.rotary_dim, desc.rope_theta, desc.epsilon = cfg.rotary_dim, cfg.rope_theta, cfg.rms_eps
    desc.q, desc.q_type = dev[mai.SI_T_ATTN_Q].data_ptr(), 12
    desc.k, desc.k_type = dev[mai.SI_T_ATTN_K].data_ptr(), 12
    desc.v, desc.v_type = dev[mai.SI_T_ATTN_V].data_ptr(), 12
    desc.o, desc.o_type = dev[mai.SI_T_ATTN_O].data_ptr(), 12
    desc.q_norm, desc.k_norm = dev[mai.SI_T_ATTN_QNORM].data_ptr(), dev[mai.SI_T_ATTN_KNORM].data_ptr()
    kc_dev = _dev(torch, kc.view(np.int16))
    vc_dev = _dev(torch, vc.view(np.int16))
    out_dev = torch.empty(H, device="cuda")
    for pos in (8192, 8193):
        x = rng.normal(0, 1, H).astype(np.float32)
        work = torch.empty(mai.attention_layer_workspace_floats(desc, cached), device="cuda")
        ctx.attention_layer_dev(desc, _dev(torch, x), pos, kc_dev, vc_dev, cached, cap, out_dev, work)
        ref, n = O.attention_layer(cfg, tensors, x, pos, kc, vc, cached)
        assert rel_l2(out_dev.cpu().numpy(), ref) < TOL, pos
        # the appended key/value slot: bf16 roundings of values that agree to
        # ~1e-6 relative, so a few elements may round the other way
        got_k = kc_dev.cpu().numpy().view(np.uint16).reshape(kvh, cap, hd)[:, cached]
        got_v = vc_dev.cpu().numpy().view(np.uint16).reshape(kvh, cap, hd)[:, cached]
        for g, r in ((got_k, kc[:, cached]), (got_v, vc[:, cached])):
            assert np.mean(g == r) > 0.99
            assert rel_l2(bf16_to_f32(g), bf16_to_f32(r)) < 2 ** -8
        cached = n
    with pytest.raises(mai.SiError, match="capacity exhausted"):
        ctx.attention_layer_dev(desc, out_dev, 8194, kc_dev, vc_dev, cap, cap, out_dev, work)
