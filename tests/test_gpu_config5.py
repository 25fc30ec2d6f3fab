"""BASELINE config 5 end to end: the 64-layer Qwen3.6-27B-shaped Q4_K_M
synthetic decoder (Q6_K ffn_down and output head), 4 GB HBM budget with the
depth-3 staging ring, a 16-token random prompt and 128 greedy tokens. Every
generated id must equal the oracle's run over the same pinned host tensors
(runtime.rs:3560-3614 generation loop, runtime.rs:4301-4309 argmax). This is
the bench's decode workload (model seed 27, prompt from seed 16)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def test_config5_128_greedy_ids_identical_to_oracle(mai):
    ctx = mai.CudaContext(0, hbm_budget_bytes=4 << 30, stage_depth=3)
    cfg = mai.qwen36_27b_config()
    m = mai.Model(ctx, cfg, seed=27)
    try:
        plan = m.plan()
        assert plan["streamed_layers"] > 0 and plan["stage_depth"] == 3
        prompt = np.random.default_rng(16).integers(0, cfg.vocab, 16).tolist()
        ids_gpu = m.generate(prompt, 128)
        orc = O.OracleModel(m.config, m.host_tensor)
        try:
            ids_cpu = orc.generate(prompt, 128)
        finally:
            orc.close()
        assert len(ids_gpu) == len(ids_cpu) == 128
        first = next((i for i, (a, b) in enumerate(zip(ids_gpu, ids_cpu)) if a != b), None)
        assert first is None, f"first differing id at step {first}: {ids_gpu[first]} vs {ids_cpu[first]}"
        assert len(set(ids_gpu)) > 8  # the synthetic decode does not collapse onto one token
    finally:
        m.close()
        ctx.close()
