"""Generate tests/golden/golden.npz: seeded small inputs for every hot-path op
with the oracle's outputs (the C++ restatement of the reference's CPU code,
pinned by tests/test_oracle_kats.py to the reference's own known-answer
tests). The CPU suite checks that the oracle still reproduces every entry
bit for bit; the GPU suite checks the CUDA path against the same entries
(dequant bit-exact, the rest within 1e-5 relative L2), so a change to either
side is caught against a fixed record.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

import oracle as O  # noqa: E402
from helpers import random_blocks  # noqa: E402


def cases():
    rng = np.random.default_rng(20261201)
    out = {}
    for ty in (12, 13, 14):
        w = random_blocks(rng, ty, 3)
        out[f"dequant_{ty}_in"] = w
        out[f"dequant_{ty}_out"] = O.dequantize(ty, w, 768)
        rows, cols = 7, 512
        wm = random_blocks(rng, ty, rows * cols // 256)
        x = rng.normal(0, 1, cols).astype(np.float32)
        out[f"matvec_{ty}_w"], out[f"matvec_{ty}_x"] = wm, x
        out[f"matvec_{ty}_out"] = O.matvec(ty, wm, rows, cols, x, 1)
    rows, cols = 5, 512
    g, u = random_blocks(rng, 12, rows * cols // 256), random_blocks(rng, 12, rows * cols // 256)
    x = rng.normal(0, 1, cols).astype(np.float32)
    out.update(gateup_g=g, gateup_u=u, gateup_x=x, gateup_out=O.fused_gate_up(g, u, rows, cols, x, 1))
    ch, k = 24, 4
    cx = rng.normal(0, 1, ch).astype(np.float32)
    cs = rng.normal(0, 1, ch * (k - 1)).astype(np.float32)
    cw = rng.normal(0, 0.5, ch * k).astype(np.float32)
    co, cso = O.causal_conv1d_step(cx, cs, cw, ch, k)
    out.update(conv_x=cx, conv_state=cs, conv_w=cw, conv_out=co, conv_state_out=cso)
    heads, kd, vd = 3, 8, 8
    q, kk, v = (rng.normal(0, 1, heads * kd).astype(np.float32), rng.normal(0, 1, heads * kd).astype(np.float32),
                rng.normal(0, 1, heads * vd).astype(np.float32))
    gate = (-np.abs(rng.normal(0, 1, heads))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, heads)))).astype(np.float32)
    st = rng.normal(0, 0.1, heads * kd * vd).astype(np.float32)
    go, gso = O.gdn_step(q, kk, v, gate, beta, st, heads, kd, vd)
    out.update(gdn_q=q, gdn_k=kk, gdn_v=v, gdn_gate=gate, gdn_beta=beta, gdn_state=st, gdn_out=go,
               gdn_state_out=gso)
    nx, nz, nw = (rng.normal(0, 1, 4 * 16).astype(np.float32), rng.normal(0, 1, 4 * 16).astype(np.float32),
                  rng.normal(0, 1, 16).astype(np.float32))
    out.update(gnorm_x=nx, gnorm_z=nz, gnorm_w=nw, gnorm_out=O.gated_rms_norm(nx, nz, nw, 4, 16, 1e-6))
    hw = rng.normal(0, 0.5, 16).astype(np.float32)
    out.update(hnorm_w=hw, hnorm_out=O.rms_norm_heads(nx, hw, 4, 16, 1e-6))
    rx = rng.normal(0, 1, 2 * 16).astype(np.float32)
    out.update(rope_x=rx, rope_out=O.rope(rx, 2, 16, 1234, 1e7))
    qh, kvh, hd, cap, cached = 4, 2, 32, 40, 37
    aq = (rng.normal(0, 1, qh * hd) / 4).astype(np.float32)
    kc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    vc = O.f32_to_bf16(rng.normal(0, 1, kvh * cap * hd).astype(np.float32))
    nk = rng.normal(0, 1, kvh * hd).astype(np.float32)
    nv = rng.normal(0, 1, kvh * hd).astype(np.float32)
    out.update(att_q=aq, att_kc=kc, att_vc=vc, att_nk=nk, att_nv=nv,
               att_out=O.attention_decode(aq, kc, vc, nk, nv, qh, kvh, hd, cached, cap))
    lg = rng.normal(0, 1, 1000).astype(np.float32)
    lg[[17, 401, 999]] = 5.0  # ties: the last index wins
    out.update(argmax_in=lg, argmax_out=np.array([O.argmax(lg)], np.int64))
    return out


if __name__ == "__main__":
    O.build()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **cases())
    print("wrote", os.path.join(HERE, "golden.npz"))
