"""Packed layer staging from a GGUF file (GgufModelStore::
stage_qwen35_layer_packed, model.rs:920-985) against its restatement in
oracle/gguf.py: the same packed bytes and name -> range map, runs merged
across gaps up to 4096 bytes, excluded and F32 tensors left out."""
import numpy as np
import pytest

import gguf_writer as W
from oracle import gguf as OG

Q4, Q6, F32 = 12, 14, 0


def blob(rng, n):
    return rng.integers(0, 256, n, dtype=np.uint8).tobytes()


@pytest.fixture
def layered(tmp_path):
    """blk.0 tensors interleaved with a large blk.1 tensor and an F32 norm;
    one small and one large blk.0 tensor to exclude."""
    rng = np.random.default_rng(7)
    tensors = [("blk.0.attn_qkv.weight", [512, 8], Q4, blob(rng, 144 * 16)),
               ("blk.0.attn_norm.weight", [512], F32, blob(rng, 2048)),
               ("blk.0.small.weight", [256, 2], Q4, blob(rng, 288)),
               ("blk.0.ffn_up.weight", [512, 4], Q4, blob(rng, 144 * 8)),
               ("blk.1.ffn_down.weight", [1024, 40], Q6, blob(rng, 210 * 160)),
               ("blk.0.ffn_down.weight", [512, 32], Q6, blob(rng, 210 * 64)),
               ("blk.0.big.weight", [1024, 40], Q4, blob(rng, 144 * 160)),
               ("blk.0.ssm_out.weight", [256, 4], Q4, blob(rng, 144 * 4)),
               ("blk.10.ffn_up.weight", [256, 1], Q4, blob(rng, 144))]
    p = tmp_path / "layered.gguf"
    W.write(p, [("general.architecture", W.STRING, "qwen35")], tensors, alignment=64)
    data = p.read_bytes()
    return p, data, OG.parse(data)


@pytest.mark.parametrize("layer,excluded", [(0, ()), (0, ("blk.0.small.weight",)), (0, ("blk.0.big.weight",)),
                                            (0, ("blk.0.small.weight", "blk.0.big.weight", "nope")), (1, ()),
                                            (10, ()), (7, ())])
def test_packed_layer_matches_restatement(mai, layered, layer, excluded):
    path, data, parsed = layered
    want_bytes, want_ranges = OG.stage_layer_packed(data, parsed, layer, excluded)
    with mai.GgufFile(path) as g:
        got, ranges = g.stage_layer_packed(layer, excluded)
    assert got.tobytes() == want_bytes and ranges == want_ranges
    for name, (a, b) in ranges.items():  # each range is that tensor's payload
        t = next(t for t in parsed["tensors"] if t["name"] == name)
        assert got[a:b].tobytes() == data[t["data_start"]:t["data_end"]]


def test_runs_merge_small_gaps_and_split_large_ones(mai, layered):
    path, data, parsed = layered
    size = lambda n: next(t["data_end"] - t["data_start"] for t in parsed["tensors"] if t["name"] == n)
    with mai.GgufFile(path) as g:
        all_, r_all = g.stage_layer_packed(0)
        no_small, r1 = g.stage_layer_packed(0, ["blk.0.small.weight"])
        no_big, r2 = g.stage_layer_packed(0, ["blk.0.big.weight"])
    assert "blk.0.attn_norm.weight" not in r_all and "blk.1.ffn_down.weight" not in r_all
    # a small excluded tensor sits inside a run: its bytes are still read
    assert "blk.0.small.weight" not in r1 and no_small.size == all_.size
    # a large excluded tensor splits the run and is not read
    assert no_big.size == all_.size - size("blk.0.big.weight")


def test_packed_staging_read_failure(mai, layered):
    path, _, _ = layered
    with mai.GgufFile(path) as g:
        mai.fault_inject(mai.FAULT_FILE_READ, 0)
        try:
            with pytest.raises(mai.SiError, match="read packed staged layer: .*unexpected end of file"):
                g.stage_layer_packed(0)
        finally:
            mai.fault_inject(0)
        assert g.stage_layer_packed(0)[0].size > 0


def test_advise_layer_counts_page_aligned_payloads(mai, layered):  # model.rs:986-1024
    import os
    path, data, parsed = layered
    page = os.sysconf("SC_PAGE_SIZE")
    want = {}
    for layer in (0, 1, 10, 7):
        by_name = {t["name"]: t for t in parsed["tensors"]}
        total = 0
        for name, t in by_name.items():
            if name.startswith(f"blk.{layer}."):
                a = t["data_start"] // page * page
                b = -(-t["data_end"] // page) * page
                total += max(b - a, 0)
        want[layer] = total
    with mai.GgufFile(path) as g:
        assert {layer: g.advise_layer(layer) for layer in want} == want
    assert want[0] > 0 and want[7] == 0


def test_packed_staging_matches_restatement_on_random_files(mai, tmp_path):
    """Random files: tensor order, sizes (some over the 4096-byte merge
    gap), types (F32 among them), alignment, layer and exclusions."""
    from hypothesis import given, settings, strategies as st

    tensor = st.tuples(st.integers(0, 3), st.sampled_from(["a", "b", "c", "d", "e"]),
                       st.sampled_from([Q4, Q6, F32]), st.integers(1, 40))

    @settings(max_examples=150, deadline=None, derandomize=True)
    @given(ts=st.lists(tensor, min_size=1, max_size=12), alignment=st.sampled_from([32, 64, 4096, 8192]),
           layer=st.integers(0, 3), nexcl=st.integers(0, 3), seed=st.integers(0, 1 << 16))
    def check(ts, alignment, layer, nexcl, seed):
        rng = np.random.default_rng(seed)
        tensors, names = [], set()
        for lay, suffix, ty, n in ts:
            name = f"blk.{lay}.{suffix}.weight"
            if name in names:
                continue
            names.add(name)
            size = {Q4: 144, Q6: 210, F32: 1024}[ty] * n
            shape = [256, n] if ty != F32 else [256 * n]
            tensors.append((name, shape, ty, blob(rng, size)))
        path = tmp_path / f"r{seed}.gguf"
        W.write(path, [("general.architecture", W.STRING, "qwen35")], tensors, alignment=alignment)
        data = path.read_bytes()
        parsed = OG.parse(data)
        excl = sorted(names)[:nexcl]
        want_bytes, want_ranges = OG.stage_layer_packed(data, parsed, layer, excl)
        with mai.GgufFile(path) as g:
            got, ranges = g.stage_layer_packed(layer, excl)
        assert got.tobytes() == want_bytes and ranges == want_ranges

    check()
