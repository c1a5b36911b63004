"""Pin the CPU oracle against the golden fixtures built from the reference's own tests.

The fixtures hold the exact inputs the reference's tests feed (extracted from its
builders) and float64 expected outputs (tests/golden/gen_golden.py).  These tests
run on CPU only and must pass before any GPU parity claim is trusted.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_case, load_golden
from oracle import oracle

with open(os.path.join(GOLDEN, "manifest.json")) as _f:
    MANIFEST = json.load(_f)

MNB = load_golden("matmulnbits.npz")
GQA = load_golden("gqa.npz")
NORMS = load_golden("norms.npz")
GBQ = load_golden("gather_block_quantized.npz")
PAGED = load_golden("paged_attention.npz")

MNB_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "matmulnbits")
GQA_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "gqa")
PAGED_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "paged")
SLIDING_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "gqa_sliding")


@pytest.mark.parametrize("name", MNB_CASES)
def test_oracle_matmulnbits_dequant_bit_exact(name):
    meta, c = MANIFEST[name], golden_case(MNB, name)
    w = oracle.matmulnbits_dequant(c["b"], c["scales"], c.get("zero_points"), N=meta["N"], K=meta["K"],
                                   bits=meta["bits"], block_size=meta["block_size"])
    np.testing.assert_array_equal(w, c["w"])


@pytest.mark.parametrize("name", MNB_CASES)
def test_oracle_matmulnbits(name):
    meta, c = MANIFEST[name], golden_case(MNB, name)
    y = oracle.matmulnbits(c["a"], c["b"], c["scales"], c.get("zero_points"), N=meta["N"], K=meta["K"],
                           bits=meta["bits"], block_size=meta["block_size"])
    assert y.shape == c["y"].shape and y.dtype == c["y"].dtype
    if meta["dtype"] == "f32":
        np.testing.assert_allclose(y, c["y"], rtol=1e-6, atol=1e-6)
    else:  # both sides round the same double-precision value to fp16
        np.testing.assert_array_equal(y, c["y"])


@pytest.mark.parametrize("name", GQA_CASES)
def test_oracle_gqa(name):
    meta, c = MANIFEST[name], golden_case(GQA, name)
    a = meta["attrs"]
    shared = meta["shared"]
    pk, pv = c["past_key"].copy(), c["past_value"].copy()
    packed = "key" not in c
    out, present_k, present_v = oracle.gqa(
        c["query"], None if packed else c["key"], None if packed else c["value"], pk, pv,
        c["seqlens_k"], c.get("cos_cache"), c.get("sin_cache"), num_heads=a["num_heads"],
        kv_heads=a["kv_num_heads"], scale=a.get("scale", 0.0),
        do_rotary=a.get("do_rotary", 1) if "cos_cache" in c else 0,
        interleaved=a.get("rotary_interleaved", 0), shared_buffer=shared,
        q_norm=c.get("q_norm"), k_norm=c.get("k_norm"), qk_norm_eps=a.get("qk_norm_epsilon", 1e-6),
        attention_bias=c.get("attention_bias"))
    np.testing.assert_allclose(out, c["out"], rtol=2e-5, atol=2e-5)
    valid = int(c["total_sequence_length"][0])
    np.testing.assert_allclose(present_k[:, :, :valid], c["present_key"][:, :, :valid], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(present_v[:, :, :valid], c["present_value"][:, :, :valid], rtol=0, atol=0)
    if shared:
        assert present_k.shape[2] == c["past_key"].shape[2]


@pytest.mark.parametrize("name", SLIDING_CASES)
def test_oracle_gqa_sliding_window_cache(name):
    """The sliding-window KV cache (attention.rs:725-880) on the reference test's three geometries
    (a decode step that reclaims rows, a 3-row chunk that needs the staging form, a batched step
    with rotary): attention output and the resident rows of present (the reference compares rows
    [0, end) at 3e-3; tests/ops/test_mlx_ops.py:301-323)."""
    assert len(SLIDING_CASES) == 3
    meta, c = MANIFEST[name], golden_case(GQA, name)
    a = meta["attrs"]
    out, pk, pv = oracle.gqa_sliding(
        c["query"], c["key"], c["value"], c["past_key"], c["past_value"], c["seqlens_k"], c.get("cos_cache"),
        c.get("sin_cache"), num_heads=a["num_heads"], kv_heads=a["kv_num_heads"], local_window=a["local_window_size"],
        scale=a.get("scale", 0.0), do_rotary=a.get("do_rotary", 1), interleaved=a.get("rotary_interleaved", 0))
    np.testing.assert_allclose(out, c["out"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(pk, c["present_key"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(pv, c["present_value"])


@pytest.mark.parametrize("name,eps,dt", [("rms", 1e-6, None), ("sln", 1e-5, None), ("rms16", 1e-6, None)])
def test_oracle_rms_norm(name, eps, dt):
    c = golden_case(NORMS, name)
    y = oracle.rms_norm(c["x"], c["scale"], eps)
    if y.dtype == np.float16:
        np.testing.assert_allclose(y.astype(np.float32), c["y"].astype(np.float32), rtol=1e-3, atol=1e-3)
    else:
        np.testing.assert_allclose(y, c["y"], rtol=1e-6, atol=1e-6)


def test_oracle_rms_norm_bf16_matches_reference_expected():
    # the reference compares its bf16 interior to an fp32 numpy value at 2e-2 (test_mlx_ops.py:37)
    c = golden_case(NORMS, "rmsbf16")
    xb = oracle.f32_to_bf16_bits(c["x"])
    gb = oracle.f32_to_bf16_bits(c["scale"])
    y = oracle.bf16_bits_to_f32(oracle.rms_norm(xb, gb, 1e-6, dtype="bf16"))
    np.testing.assert_allclose(y, c["y"], rtol=2e-2, atol=2e-2)


def test_oracle_skip_rms_norm():
    c = golden_case(NORMS, "skiprms")
    y, r = oracle.skip_rms_norm(c["x"], c["skip"], c["gamma"], 1e-6)
    np.testing.assert_allclose(y, c["y"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(r, c["residual"])


@pytest.mark.parametrize("name", PAGED_CASES)
def test_oracle_paged_attention(name):
    """The reference's PagedAttention cases (test_paged_attention.py): the scattered caches match
    bit for bit (the same fp32 RoPE rounded once to fp16); the output matches the reference's
    fp32 numpy port within 2e-3 — the oracle, like the reference op, attends with q / k rounded to
    fp16 after RoPE, the numpy port with unrounded fp32 values (its own test allows 2e-2)."""
    a, c = MANIFEST[name]["attrs"], golden_case(PAGED, name)
    out, kc, vc = oracle.paged_attention(
        c["query"], c["key"], c["value"], c["key_cache"], c["value_cache"], c["cumulative_sequence_length"],
        c["past_seqlens"], c["block_table"], c.get("cos_cache"), c.get("sin_cache"), num_heads=a["num_heads"],
        kv_heads=a["kv_num_heads"], interleaved=a["rotary_interleaved"])
    np.testing.assert_array_equal(kc, c["expected_key_cache"])
    np.testing.assert_array_equal(vc, c["expected_value_cache"])
    np.testing.assert_allclose(out.astype(np.float32), c["expected"], rtol=2e-3, atol=2e-3)


def test_oracle_paged_attention_rejects_slots_outside_the_caches():
    c = golden_case(PAGED, PAGED_CASES[0])
    a = MANIFEST[PAGED_CASES[0]]["attrs"]
    bt = c["block_table"].copy()
    bt[0, 0] = c["key_cache"].shape[0]  # one past the last physical block
    past = c["past_seqlens"].copy()
    past[0] = max(int(past[0]), 1)
    with pytest.raises(oracle.OracleError):
        oracle.paged_attention(c["query"], c["key"], c["value"], c["key_cache"], c["value_cache"],
                               c["cumulative_sequence_length"], past, bt, num_heads=a["num_heads"],
                               kv_heads=a["kv_num_heads"])


def test_oracle_gather_block_quantized():
    c = golden_case(GBQ, "gbq")
    y = oracle.gather_block_quantized(c["data"], c["scales"], c["indices"], block_size=16)
    np.testing.assert_array_equal(y, c["y"])


def test_oracle_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 1e-5,
                        rng.standard_normal(20000).astype(np.float32) * 100,
                        np.array([65504, 65519.9, 65520, -70000, 6e-8, 3e-8, 0.0, -0.0], np.float32)])
    L = oracle.lib()
    got = np.array([L.oracle_float_to_half(float(v)) for v in x], dtype=np.uint16)
    np.testing.assert_array_equal(got, x.astype(np.float16).view(np.uint16))
    back = np.array([L.oracle_half_to_float(int(h)) for h in got], dtype=np.float32)
    np.testing.assert_array_equal(back, got.view(np.float16).astype(np.float32))


def test_oracle_bf16_conversion_round_trip():
    L = oracle.lib()
    rng = np.random.default_rng(1)
    x = rng.standard_normal(5000).astype(np.float32) * 37
    got = np.array([L.oracle_float_to_bf16(float(v)) for v in x], dtype=np.uint16)
    np.testing.assert_array_equal(got, oracle.f32_to_bf16_bits(x))
