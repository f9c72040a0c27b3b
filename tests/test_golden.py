"""Pins the CPU oracle to the reference: golden fixtures recorded from the
reference's own CUDA kernels on a B200 (tests/golden/make_golden.py).

RoPE, the KV append, the greedy index and the sampling candidates must match
bit for bit; attention must match within 4e-3 (the oracle follows
attention.cu's warp structure and summation order; only the last bits of expf
differ between glibc and CUDA). No GPU needed."""
from pathlib import Path

import numpy as np
import pytest

import oracle.oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = ["rope_hd64", "rope_hd128", "update_kv_cache", "attention_hd64", "attention_hd128",
            "attention_hd128_gqa8", "sampling"]


def load(name):
    path = GOLDEN / f"{name}.npz"
    assert path.exists(), f"missing golden fixture {path}; run tests/golden/make_golden.py on a GPU"
    return dict(np.load(path))


@pytest.mark.parametrize("name", ["rope_hd64", "rope_hd128"])
def test_rope_oracle_matches_reference_kernel(name):
    f = load(name)
    hd, hq, hkv = int(f["hd"]), int(f["hq"]), int(f["hkv"])
    cos, sin = O.rope_table(int(f["positions"].max()) + 1, hd, 1e6)
    assert np.array_equal(cos[f["positions"]].view(np.uint32), f["cos_rows"].view(np.uint32))
    assert np.array_equal(sin[f["positions"]].view(np.uint32), f["sin_rows"].view(np.uint32))
    for i, pos in enumerate(f["positions"]):
        q, k = f["q"][i].copy(), f["k"][i].copy()
        O.rope(q, f["q_bias"], k, f["k_bias"], cos, sin, int(pos), hd, hq, hkv)
        assert np.array_equal(q, f["q_out"][i]), f"q mismatch at pos {pos}"
        assert np.array_equal(k, f["k_out"][i]), f"k mismatch at pos {pos}"


@pytest.mark.skipif(not O.REF_LIB.exists(), reason="oracle/_ref not built")
@pytest.mark.parametrize("hd", [64, 128])
def test_reference_arm_rope_tables_match(hd):
    """The tables bench.py's reference arm builds with the reference library's
    host code equal the oracle's (and so the product's) bit for bit, and the
    golden rows recorded from the reference."""
    a_cos, a_sin = O.ref_rope_table(32768, hd, 1e6)
    b_cos, b_sin = O.rope_table(32768, hd, 1e6)
    assert np.array_equal(a_cos.view(np.uint32), b_cos.view(np.uint32))
    assert np.array_equal(a_sin.view(np.uint32), b_sin.view(np.uint32))
    f = load(f"rope_hd{hd}")
    assert np.array_equal(a_cos[f["positions"]].view(np.uint32), f["cos_rows"].view(np.uint32))


def test_update_oracle_matches_reference_kernel():
    f = load("update_kv_cache")
    kp, vp = f["k_pool"].copy(), f["v_pool"].copy()
    for i, pos in enumerate(f["positions"]):
        O.update_kv_cache(kp, vp, f["k"][i], f["v"][i], f["v_bias"], f["table"], int(f["layer"]),
                          int(pos), int(f["num_layers"]), int(f["hkv"]), int(f["hd"]))
    assert np.array_equal(kp, f["k_pool_out"])
    assert np.array_equal(vp, f["v_pool_out"])


@pytest.mark.parametrize("name", ["attention_hd64", "attention_hd128", "attention_hd128_gqa8"])
def test_attention_oracle_matches_reference_kernel(name):
    f = load(name)
    out = O.flash_decoding(f["q"], f["k_pool"], f["v_pool"], f["table"], int(f["layer"]),
                           int(f["hq"]), int(f["hkv"]), int(f["hd"]), int(f["pos"]),
                           int(f["num_layers"]))
    err = np.abs(O.bf16_to_f32(out) - O.bf16_to_f32(f["out"])).max()
    assert err <= 4e-3
    # most elements are bit-identical
    assert (out == f["out"]).mean() > 0.9


def test_sampling_oracle_matches_reference_kernels():
    """argmax_kernel, top_k_filter and fused_top_p_sample (run on a GPU by
    tests/golden/make_golden.py) against the CPU oracle: the greedy index and the
    candidate keys and values exactly, ties included (the logits are quantised);
    the draws wherever they are not within rounding of a boundary."""
    g = np.load(GOLDEN / "sampling.npz")
    logits, draws = g["logits"], g["draws"]
    assert list(O.argmax(logits)) == list(g["argmax"])
    checked = 0
    for top_k in (64, 256):
        for r in range(logits.shape[0]):
            keys, vals = O.top_k_filter(logits[r], top_k)
            assert np.array_equal(keys, g[f"keys_{top_k}"][r])
            assert np.array_equal(vals, g[f"values_{top_k}"][r])
            for j, (top_p, rand) in enumerate(draws):
                want, margin = O.top_p_sample(keys, vals, top_p, rand)
                if margin < 1e-5:
                    continue
                assert want == g[f"picks_{top_k}"][r, j]
                checked += 1
    assert checked >= 24
