"""GPU parity of the kernel-level C ABI (include/b200ep.h) against the CPU oracle and the golden
fixtures built from the reference's tests.

Tolerances: fp32 paths rtol = atol = 6e-5; fp16 / bf16 paths
max-abs 1e-3 + rel 1e-2; dequantised weights bit-exact.  Reference test geometries come from
tests/golden (tests/ops/test_matmulnbits_asym.py, test_mlx_ops.py, test_gqa11.py).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_case, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

with open(os.path.join(GOLDEN, "manifest.json")) as _f:
    MANIFEST = json.load(_f)

TOL = {"f32": dict(rtol=6e-5, atol=6e-5), "f16": dict(rtol=1e-2, atol=1e-3), "bf16": dict(rtol=1e-2, atol=1e-3)}


@pytest.fixture(scope="module")
def ops():
    from onnxruntime_ep_b200 import ops as _ops

    return _ops


@pytest.fixture(autouse=True)
def _device_error_clean(ops):
    ops.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    code, detail = ops.device_error(clear=True)
    assert code == 0, f"kernel reported device error {code} (detail {detail})"


def cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def to_np(t):
    return t.detach().cpu().numpy()


# ---- MatMulNBits ---------------------------------------------------------------------------
MNB = load_golden("matmulnbits.npz")
MNB_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "matmulnbits")


@pytest.mark.parametrize("name", MNB_CASES)
def test_matmulnbits_golden(ops, name):
    meta, c = MANIFEST[name], golden_case(MNB, name)
    zp = cuda(c["zero_points"]) if "zero_points" in c else None
    y = ops.matmulnbits(cuda(c["a"]), cuda(c["b"]), cuda(c["scales"]), zp, K=meta["K"], N=meta["N"],
                       bits=meta["bits"], block_size=meta["block_size"])
    got = to_np(y).astype(np.float32)
    want = c["y"].astype(np.float32)
    np.testing.assert_allclose(got, want, **TOL[meta["dtype"]])


@pytest.mark.parametrize("name", MNB_CASES)
def test_matmulnbits_dequant_bit_exact(ops, name):
    meta, c = MANIFEST[name], golden_case(MNB, name)
    zp = cuda(c["zero_points"]) if "zero_points" in c else None
    w = ops.matmulnbits_dequant(cuda(c["b"]), cuda(c["scales"]), zp, K=meta["K"], N=meta["N"],
                                bits=meta["bits"], block_size=meta["block_size"])
    np.testing.assert_array_equal(to_np(w), c["w"])


def make_mnb(rng, M, K, N, block=32, bits=4, dtype=np.float32, asym=True):
    """Single-MatMulNBits workload distributions: A ~ N(0,1), scales ~ U(0.005, 0.02), zp ~ U{0..15}."""
    nblocks = (K + block - 1) // block
    a = rng.standard_normal((M, K)).astype(dtype)
    q = rng.integers(0, 1 << bits, size=(N, nblocks, block), dtype=np.uint8)
    b = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8) if bits == 4 else q
    scales = rng.uniform(0.005, 0.02, size=N * nblocks).astype(dtype)
    zp = None
    if asym:
        z = rng.integers(0, 1 << bits, size=(N, nblocks), dtype=np.uint8)
        if bits == 4:
            if nblocks % 2:
                z = np.concatenate([z, np.zeros((N, 1), np.uint8)], axis=1)
            zp = (z[:, 0::2] | (z[:, 1::2] << 4)).reshape(-1).astype(np.uint8)
        else:
            zp = z.reshape(-1)
    return a, b, scales, zp


@pytest.mark.parametrize("M", [1, 16, 512])
def test_matmulnbits_config1_fp32(ops, M):
    """Single-MatMulNBits workload: fp32 A [M, 4096], B [4096, 4096] int4 block 32, fp32 scales, uint8 zp."""
    rng = np.random.default_rng(0)
    a, b, s, zp = make_mnb(rng, M, 4096, 4096)
    want = oracle.matmulnbits(a, b, s, zp, N=4096, K=4096)
    got = to_np(ops.matmulnbits(cuda(a), cuda(b), cuda(s), cuda(zp), K=4096, N=4096))
    np.testing.assert_allclose(got, want, **TOL["f32"])


@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (1, 14336, 4096), (1, 4096, 28672), (2, 4096, 4096),
                                   (4, 4096, 1024), (16, 4096, 4096)])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_matmulnbits_llama_shapes(ops, M, K, N, dt):
    rng = np.random.default_rng(M * 7 + K + N)
    a, b, s, zp = make_mnb(rng, M, K, N, dtype=np.float32)
    if dt == "f16":
        a16, s16 = a.astype(np.float16), s.astype(np.float16)
        want = oracle.matmulnbits(a16, b, s16, zp, N=N, K=K).astype(np.float32)
        got = ops.matmulnbits(cuda(a16), cuda(b), cuda(s16), cuda(zp), K=K, N=N)
    else:
        ab, sb = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(s)
        want = oracle.bf16_bits_to_f32(oracle.matmulnbits(ab, b, sb, zp, N=N, K=K, dtype="bf16"))
        got = ops.matmulnbits(cuda(ab).view(torch.bfloat16), cuda(b), cuda(sb).view(torch.bfloat16), cuda(zp),
                              K=K, N=N)
    np.testing.assert_allclose(to_np(got.float()), want, **TOL[dt])


def test_matmulnbits_symmetric_int8_and_odd_k(ops):
    rng = np.random.default_rng(5)
    for bits, K, block in [(8, 4096, 32), (4, 1176, 32), (4, 48, 16), (4, 4100, 128)]:
        a, b, s, zp = make_mnb(rng, 3, K, 256, block=block, bits=bits, asym=False)
        want = oracle.matmulnbits(a, b, s, None, N=256, K=K, bits=bits, block_size=block)
        got = to_np(ops.matmulnbits(cuda(a), cuda(b), cuda(s), None, K=K, N=256, bits=bits, block_size=block))
        np.testing.assert_allclose(got, want, **TOL["f32"])


def test_matmulnbits_empty_m(ops):
    rng = np.random.default_rng(1)
    a, b, s, zp = make_mnb(rng, 1, 64, 32)
    y = ops.matmulnbits(cuda(a[:0]), cuda(b), cuda(s), cuda(zp), K=64, N=32)
    assert y.shape == (0, 32)


def test_matmulnbits_rejects_bad_block(ops):
    from onnxruntime_ep_b200 import B200EPError

    rng = np.random.default_rng(1)
    a, b, s, zp = make_mnb(rng, 1, 64, 32)
    with pytest.raises(B200EPError, match="block_size"):
        ops.matmulnbits(cuda(a), cuda(b), cuda(s), cuda(zp), K=64, N=32, block_size=24)


# ---- RMS norms -----------------------------------------------------------------------------
NORMS = load_golden("norms.npz")


@pytest.mark.parametrize("name,eps", [("rms", 1e-6), ("sln", 1e-5), ("rms16", 1e-6)])
def test_rms_norm_golden(ops, name, eps):
    c = golden_case(NORMS, name)
    y = to_np(ops.rms_norm(cuda(c["x"]), cuda(c["scale"]), eps))
    dt = "f16" if c["x"].dtype == np.float16 else "f32"
    np.testing.assert_allclose(y.astype(np.float32), c["y"].astype(np.float32),
                               **(TOL[dt] if dt == "f16" else dict(rtol=1e-5, atol=1e-5)))


def test_skip_rms_norm_golden(ops):
    c = golden_case(NORMS, "skiprms")
    y, r = ops.skip_rms_norm(cuda(c["x"]), cuda(c["skip"]), cuda(c["gamma"]), 1e-6)
    np.testing.assert_allclose(to_np(y), c["y"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(to_np(r), c["residual"])


@pytest.mark.parametrize("rows,hidden", [(1, 4096), (16, 4096), (512, 4096), (3, 8192), (5, 100)])
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_rms_norms_vs_oracle(ops, rows, hidden, dt):
    rng = np.random.default_rng(rows + hidden)
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    sk = rng.standard_normal((rows, hidden)).astype(np.float32)
    g = rng.standard_normal(hidden).astype(np.float32)
    if dt == "f32":
        conv, back, tdt, odt = (lambda v: v), (lambda v: v), torch.float32, None
    elif dt == "f16":
        conv, back, tdt, odt = (lambda v: v.astype(np.float16)), (lambda v: v.astype(np.float32)), torch.float16, None
    else:
        conv, back, tdt, odt = oracle.f32_to_bf16_bits, oracle.bf16_bits_to_f32, torch.bfloat16, "bf16"
    xc, sc, gc = conv(x), conv(sk), conv(g)
    tx = cuda(xc).view(tdt) if dt == "bf16" else cuda(xc)
    ts = cuda(sc).view(tdt) if dt == "bf16" else cuda(sc)
    tg = cuda(gc).view(tdt) if dt == "bf16" else cuda(gc)
    tol = TOL[dt] if dt != "f32" else dict(rtol=1e-5, atol=1e-5)
    want = back(oracle.rms_norm(xc, gc, 1e-5, dtype=odt))
    got = ops.rms_norm(tx, tg, 1e-5)
    np.testing.assert_allclose(to_np(got.float()), want, **tol)
    wy, wr = oracle.skip_rms_norm(xc, sc, gc, 1e-5, dtype=odt)
    y, r = ops.skip_rms_norm(tx, ts, tg, 1e-5)
    np.testing.assert_allclose(to_np(y.float()), back(wy), **tol)
    np.testing.assert_array_equal(to_np(r.float()), back(wr))


# ---- GroupQueryAttention -------------------------------------------------------------------
GQA = load_golden("gqa.npz")
GQA_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "gqa")


def run_gqa_case(ops, c, a, shared):
    """Drive the shared-buffer kernel; the growing contract copies past into a present buffer."""
    S = c["query"].shape[1]
    total = int(c["total_sequence_length"][0])
    past_cap = c["past_key"].shape[2]
    if shared:
        kk, vv = cuda(c["past_key"]), cuda(c["past_value"])
    else:
        B, HK, _, D = c["past_key"].shape
        kk = torch.zeros(B, HK, total, D, dtype=torch.float32, device="cuda")
        vv = torch.zeros_like(kk)
        kk[:, :, :past_cap] = cuda(c["past_key"])
        vv[:, :, :past_cap] = cuda(c["past_value"])
    packed = "key" not in c
    rope = "cos_cache" in c and a.get("do_rotary", 1)
    out = ops.group_query_attention(
        cuda(c["query"]), None if packed else cuda(c["key"]), None if packed else cuda(c["value"]), kk, vv,
        cuda(c["seqlens_k"]), cuda(c["cos_cache"]) if rope else None, cuda(c["sin_cache"]) if rope else None,
        num_heads=a["num_heads"], kv_heads=a["kv_num_heads"], scale=a.get("scale", 0.0),
        do_rotary=rope, interleaved=a.get("rotary_interleaved", 0),
        q_norm=cuda(c["q_norm"]) if "q_norm" in c else None, k_norm=cuda(c["k_norm"]) if "k_norm" in c else None,
        qk_norm_eps=a.get("qk_norm_epsilon", 1e-6),
        attention_bias=cuda(c["attention_bias"]) if "attention_bias" in c else None)
    return to_np(out), to_np(kk), to_np(vv), total, S


@pytest.mark.parametrize("name", GQA_CASES)
def test_gqa_golden(ops, name):
    meta, c = MANIFEST[name], golden_case(GQA, name)
    out, pk, pv, total, S = run_gqa_case(ops, c, meta["attrs"], meta["shared"])
    np.testing.assert_allclose(out, c["out"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(pk[:, :, :total], c["present_key"][:, :, :total], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(pv[:, :, :total], c["present_value"][:, :, :total])
    if meta["shared"]:  # rows beyond the valid prefix are untouched
        np.testing.assert_array_equal(pk[:, :, total:], c["past_key"][:, :, total:])


def make_gqa_inputs(rng, B, S, H, HK, D, past, cap, dtype=np.float16, max_seq=None):
    q = rng.standard_normal((B, S, H * D)).astype(dtype)
    k = rng.standard_normal((B, S, HK * D)).astype(dtype)
    v = rng.standard_normal((B, S, HK * D)).astype(dtype)
    kc = np.zeros((B, HK, cap, D), dtype=dtype)
    vc = np.zeros((B, HK, cap, D), dtype=dtype)
    kc[:, :, :past] = rng.standard_normal((B, HK, past, D)).astype(dtype)
    vc[:, :, :past] = rng.standard_normal((B, HK, past, D)).astype(dtype)
    max_seq = max_seq or cap + 4
    half = D // 2
    inv = 1.0 / (10000.0 ** (np.arange(half, dtype=np.float64) / half))
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)
    seqlens = np.full((B,), past + S - 1, dtype=np.int32)
    return q, k, v, kc, vc, cos, sin, seqlens


@pytest.mark.parametrize("B,past", [(1, 128), (1, 1024), (1, 8191), (8, 512), (8, 4096)])
def test_gqa_config2_decode_fp16(ops, B, past):
    """Single-GQA-decode workload: 32 q heads, 8 kv heads, D 128, fp16, rotary base 10000 non-interleaved."""
    rng = np.random.default_rng(B * 100003 + past)
    H, HK, D, S = 32, 8, 128, 1
    cap = past + S + 7
    q, k, v, kc, vc, cos, sin, seqlens = make_gqa_inputs(rng, B, S, H, HK, D, past, cap)
    want, wk, wv = oracle.gqa(q, k, v, kc.copy(), vc.copy(), seqlens, cos, sin, num_heads=H, kv_heads=HK,
                              shared_buffer=True)
    tk, tv = cuda(kc), cuda(vc)
    out = ops.group_query_attention(cuda(q), cuda(k), cuda(v), tk, tv, cuda(seqlens), cuda(cos), cuda(sin),
                                    num_heads=H, kv_heads=HK)
    np.testing.assert_allclose(to_np(out).astype(np.float32), want.astype(np.float32), **TOL["f16"])
    np.testing.assert_array_equal(to_np(tk), wk)  # append is bit-exact (same fp32 RoPE, one rounding)
    np.testing.assert_array_equal(to_np(tv), wv)


@pytest.mark.parametrize("S,H,HK,D,interleaved,window", [(1, 32, 8, 128, 1, -1), (2, 32, 8, 128, 0, -1),
                                                        (3, 8, 1, 64, 0, 5), (1, 14, 2, 64, 0, -1),
                                                        (1, 16, 16, 128, 0, -1), (4, 8, 2, 256, 0, -1)])
def test_gqa_variants_fp16(ops, S, H, HK, D, interleaved, window):
    rng = np.random.default_rng(S * 31 + H + D)
    B, past = 2, 300
    cap = past + S + 3
    q, k, v, kc, vc, cos, sin, _ = make_gqa_inputs(rng, B, S, H, HK, D, past, cap)
    seqlens = np.array([past + S - 1, past - 40 + S - 1], dtype=np.int32)  # ragged batch
    want, wk, wv = oracle.gqa(q, k, v, kc.copy(), vc.copy(), seqlens, cos, sin, num_heads=H, kv_heads=HK,
                              interleaved=interleaved, shared_buffer=True, local_window=window)
    tk, tv = cuda(kc), cuda(vc)
    out = ops.group_query_attention(cuda(q), cuda(k), cuda(v), tk, tv, cuda(seqlens), cuda(cos), cuda(sin),
                                    num_heads=H, kv_heads=HK, interleaved=interleaved, local_window=window)
    np.testing.assert_allclose(to_np(out).astype(np.float32), want.astype(np.float32), **TOL["f16"])
    np.testing.assert_array_equal(to_np(tk), wk)
    np.testing.assert_array_equal(to_np(tv), wv)


@pytest.mark.parametrize("B,S,H,HK,D,past,window,interleaved", [
    (1, 64, 32, 8, 128, 0, -1, 0), (2, 130, 8, 2, 64, 57, -1, 1), (2, 200, 16, 4, 128, 300, 64, 0),
    (1, 512, 32, 8, 128, 0, -1, 0), (2, 97, 32, 8, 128, 1000, -1, 0), (2, 1200, 32, 8, 128, 40, -1, 0)])
def test_gqa_prefill_fp16(ops, B, S, H, HK, D, past, window, interleaved):
    """Prompt rows (S > 1) on the tensor-core prefill kernel: causal bottom-right alignment, GQA
    head map, local window, ragged batch (the second sequence 40 keys shorter)."""
    rng = np.random.default_rng(S * 7 + H + D + past)
    cap = past + S + 3
    q, k, v, kc, vc, cos, sin, seqlens = make_gqa_inputs(rng, B, S, H, HK, D, past, cap)
    if B > 1:
        seqlens[1] -= 40
    want, wk, wv = oracle.gqa(q, k, v, kc.copy(), vc.copy(), seqlens, cos, sin, num_heads=H, kv_heads=HK,
                              interleaved=interleaved, shared_buffer=True, local_window=window)
    tk, tv = cuda(kc), cuda(vc)
    out = ops.group_query_attention(cuda(q), cuda(k), cuda(v), tk, tv, cuda(seqlens), cuda(cos), cuda(sin),
                                    num_heads=H, kv_heads=HK, interleaved=interleaved, local_window=window)
    np.testing.assert_allclose(to_np(out).astype(np.float32), want.astype(np.float32), **TOL["f16"])
    np.testing.assert_array_equal(to_np(tk), wk)
    np.testing.assert_array_equal(to_np(tv), wv)


def test_gqa_prefill_bf16(ops):
    rng = np.random.default_rng(12)
    B, S, H, HK, D, past = 1, 300, 32, 8, 128, 100
    cap = past + S + 8
    q, k, v, kc, vc, cos, sin, seqlens = make_gqa_inputs(rng, B, S, H, HK, D, past, cap, dtype=np.float32)
    bf = oracle.f32_to_bf16_bits
    args = [bf(x) for x in (q, k, v, kc, vc, cos, sin)]
    kco, vco = args[3].copy(), args[4].copy()
    want, wk, _ = oracle.gqa(args[0], args[1], args[2], kco, vco, seqlens, args[5], args[6], num_heads=H,
                             kv_heads=HK, shared_buffer=True, dtype="bf16")
    t = [cuda(x).view(torch.bfloat16) for x in args]
    out = ops.group_query_attention(t[0], t[1], t[2], t[3], t[4], cuda(seqlens), t[5], t[6], num_heads=H,
                                    kv_heads=HK)
    np.testing.assert_allclose(to_np(out.float()), oracle.bf16_bits_to_f32(want), **TOL["bf16"])
    np.testing.assert_array_equal(to_np(t[3].view(torch.int16)).view(np.uint16), wk)


def test_gqa_bf16_decode(ops):
    rng = np.random.default_rng(11)
    B, S, H, HK, D, past = 1, 1, 32, 8, 128, 2000
    cap = past + 64
    q, k, v, kc, vc, cos, sin, seqlens = make_gqa_inputs(rng, B, S, H, HK, D, past, cap, dtype=np.float32)
    bf = oracle.f32_to_bf16_bits
    args = [bf(x) for x in (q, k, v, kc, vc, cos, sin)]
    kco, vco = args[3].copy(), args[4].copy()
    want, wk, _ = oracle.gqa(args[0], args[1], args[2], kco, vco, seqlens, args[5], args[6], num_heads=H,
                             kv_heads=HK, shared_buffer=True, dtype="bf16")
    t = [cuda(x).view(torch.bfloat16) for x in args]
    out = ops.group_query_attention(t[0], t[1], t[2], t[3], t[4], cuda(seqlens), t[5], t[6], num_heads=H,
                                    kv_heads=HK)
    np.testing.assert_allclose(to_np(out.float()), oracle.bf16_bits_to_f32(want), **TOL["bf16"])
    np.testing.assert_array_equal(to_np(t[3].view(torch.int16)).view(np.uint16), wk)


def test_gqa_repeated_decode_steps_match_oracle(ops):
    """Sixteen consecutive decode steps on one shared buffer: the arrival counters reset and the
    append offset advances from device-side seqlens_k."""
    rng = np.random.default_rng(3)
    B, H, HK, D, past0, steps = 2, 32, 8, 128, 700, 16
    cap = past0 + steps + 1
    q, k, v, kc, vc, cos, sin, _ = make_gqa_inputs(rng, B, 1, H, HK, D, past0, cap)
    tk, tv = cuda(kc), cuda(vc)
    ok, ov = kc.copy(), vc.copy()
    for t in range(steps):
        qs = rng.standard_normal(q.shape).astype(np.float16)
        ks = rng.standard_normal(k.shape).astype(np.float16)
        vs = rng.standard_normal(v.shape).astype(np.float16)
        seqlens = np.full((B,), past0 + t, dtype=np.int32)
        want, ok, ov = oracle.gqa(qs, ks, vs, ok, ov, seqlens, cos, sin, num_heads=H, kv_heads=HK,
                                  shared_buffer=True)
        out = ops.group_query_attention(cuda(qs), cuda(ks), cuda(vs), tk, tv, cuda(seqlens), cuda(cos),
                                        cuda(sin), num_heads=H, kv_heads=HK)
        np.testing.assert_allclose(to_np(out).astype(np.float32), want.astype(np.float32), **TOL["f16"])
    np.testing.assert_array_equal(to_np(tk), ok)


SLIDING_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "gqa_sliding")


@pytest.mark.parametrize("name", SLIDING_CASES)
def test_gqa_sliding_window_cache_golden(ops, name):
    """The reference test's sliding-window cache geometries (tests/ops/test_mlx_ops.py:251-323: a
    decode step that reclaims rows, a 3-row chunk in the staging form, a batched step with rotary),
    fp32, through b200ep_group_query_attention_sliding; present compared over the resident rows and
    zero after them."""
    meta, c = MANIFEST[name], golden_case(GQA, name)
    a = meta["attrs"]
    tk, tv = cuda(c["past_key"]), cuda(c["past_value"])
    out, pk, pv = ops.group_query_attention_sliding(
        cuda(c["query"]), cuda(c["key"]), cuda(c["value"]), tk, tv, cuda(c["seqlens_k"]),
        cuda(c["cos_cache"]) if "cos_cache" in c else None, cuda(c["sin_cache"]) if "sin_cache" in c else None,
        num_heads=a["num_heads"], kv_heads=a["kv_num_heads"], local_window=a["local_window_size"],
        scale=a.get("scale", 0.0), do_rotary=a.get("do_rotary", 1) if "cos_cache" in c else 0)
    np.testing.assert_allclose(to_np(out), c["out"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(to_np(pk), c["present_key"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(to_np(pv), c["present_value"])


@pytest.mark.parametrize("dt", [np.float16, "bf16"])
def test_gqa_sliding_window_cache_decode_run(ops, dt):
    """A 40-row prompt then 40 decode steps on a 48-row cache with a 32-key window (rows reclaimed 17
    at a time, three times), two sequences of different lengths, 32 / 8 heads of 128 with rotary: every
    step's output and the resident cache rows against the oracle run on the same state."""
    rng = np.random.default_rng(21)
    B, H, HK, D, cap, W = 2, 32, 8, 128, 48, 32
    npdt = np.float16 if dt == np.float16 else np.float32
    def cast(x):
        x = np.asarray(x, np.float32)
        return x.astype(np.float16) if dt == np.float16 else oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(x))
    def dev(x):
        t = cuda(np.ascontiguousarray(x, np.float32))
        return t.half() if dt == np.float16 else t.bfloat16()
    def host(t):
        return t.float().cpu().numpy()
    half = D // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) / half))
    ang = np.arange(128)[:, None] * inv[None, :]
    cos, sin = cast(np.cos(ang)), cast(np.sin(ang))
    okc = np.zeros((B, HK, cap, D), np.float32)
    ovc = np.zeros_like(okc)
    tk, tv = dev(okc), dev(ovc)
    lens = np.array([0, 5])  # sequence 1 starts 5 tokens ahead (its first 5 rows were filled before)
    okc[1, :, :5] = cast(rng.standard_normal((HK, 5, D)))
    ovc[1, :, :5] = cast(rng.standard_normal((HK, 5, D)))
    tk.copy_(dev(okc)), tv.copy_(dev(ovc))
    code = None if dt == np.float16 else "bf16"
    def oracle_run(q, k, v, seq):
        if code is None:
            return oracle.gqa_sliding(q.astype(np.float16), k.astype(np.float16), v.astype(np.float16),
                                      okc.astype(np.float16), ovc.astype(np.float16), seq, cos, sin,
                                      num_heads=H, kv_heads=HK, local_window=W)
        bf = oracle.f32_to_bf16_bits
        o, pk, pv = oracle.gqa_sliding(bf(q), bf(k), bf(v), bf(okc), bf(ovc), seq, bf(cos), bf(sin), num_heads=H,
                                       kv_heads=HK, local_window=W, dtype="bf16")
        return tuple(oracle.bf16_bits_to_f32(x) for x in (o, pk, pv))
    for step, S in enumerate([40] + [1] * 40):
        q = cast(rng.standard_normal((B, S, H * D)))
        k = cast(rng.standard_normal((B, S, HK * D)))
        v = cast(rng.standard_normal((B, S, HK * D)))
        seq = (lens + S - 1).astype(np.int32)
        want, wk, wv = oracle_run(q, k, v, seq)
        out, _, _ = ops.group_query_attention_sliding(dev(q), dev(k), dev(v), tk, tv, cuda(seq), dev(cos), dev(sin),
                                                      num_heads=H, kv_heads=HK, local_window=W)
        tol = dict(rtol=1e-2, atol=1e-3) if dt == np.float16 else dict(rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(host(out), np.asarray(want, np.float32), err_msg=f"step {step}", **tol)
        np.testing.assert_allclose(host(tk), np.asarray(wk, np.float32), err_msg=f"step {step} keys", **tol)
        np.testing.assert_array_equal(host(tv), np.asarray(wv, np.float32), err_msg=f"step {step} values")
        okc, ovc = np.asarray(wk, np.float32), np.asarray(wv, np.float32)
        lens = lens + S


def test_gqa_out_of_range_is_reported_not_faulted(ops):
    rng = np.random.default_rng(4)
    B, S, H, HK, D, past = 1, 1, 8, 2, 64, 10
    cap = 12
    q, k, v, kc, vc, cos, sin, _ = make_gqa_inputs(rng, B, S, H, HK, D, past, cap)
    seqlens = np.array([cap + 5], dtype=np.int32)  # beyond the buffer: the kernel must refuse it
    ops.group_query_attention(cuda(q), cuda(k), cuda(v), cuda(kc), cuda(vc), cuda(seqlens), cuda(cos),
                              cuda(sin), num_heads=H, kv_heads=HK)
    torch.cuda.synchronize()
    code, _ = ops.device_error(clear=True)
    assert code == 101


# ---- prepacked tensor-core MatMulNBits -------------------------------------------------------
@pytest.mark.parametrize("block", [16, 32, 64, 128])
@pytest.mark.parametrize("M", [1, 3, 8, 16, 37])
@pytest.mark.parametrize("asym", [True, False], ids=["asym", "sym"])
def test_matmulnbits_prepacked_vs_oracle(ops, block, M, asym):
    rng = np.random.default_rng(block * 131 + M)
    K, N = 512, 200  # N not a multiple of 16, K a multiple of 16 but not of 64 when block 16
    a, b, s, zp = make_mnb(rng, M, K, N, block=block, dtype=np.float16, asym=asym)
    packed = ops.matmulnbits_prepack(cuda(b), cuda(s), cuda(zp) if asym else None, K=K, N=N, block_size=block)
    got = ops.matmulnbits_prepacked(cuda(a), packed, K=K, N=N, block_size=block).float().cpu().numpy()
    want = oracle.matmulnbits(a, b, s, zp if asym else None, N=N, K=K, block_size=block).astype(np.float32)
    np.testing.assert_allclose(got, want, **TOL["f16"])


@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (1, 14336, 4096), (1, 4096, 28672), (16, 4096, 4096),
                                   (512, 4096, 1024), (1, 1168, 96), (200, 1024, 18944), (300, 4096, 20480),
                                   (1000, 256, 28672), (16, 14336, 4096), (5, 14336, 200),
                                   # Llama-3-70B shapes at 16 rows, whole and per rank of 2
                                   (16, 8192, 10240), (16, 8192, 5120), (16, 4096, 8192), (16, 8192, 28672),
                                   (16, 14336, 8192), (2, 8192, 28672)])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_matmulnbits_prepacked_llama_shapes(ops, M, K, N, dt):
    rng = np.random.default_rng(M + K * 3 + N)
    a, b, s, zp = make_mnb(rng, M, K, N)
    if dt == "f16":
        a16, s16 = a.astype(np.float16), s.astype(np.float16)
        want = oracle.matmulnbits(a16, b, s16, zp, N=N, K=K).astype(np.float32)
        packed = ops.matmulnbits_prepack(cuda(b), cuda(s16), cuda(zp), K=K, N=N)
        got = ops.matmulnbits_prepacked(cuda(a16), packed, K=K, N=N)
    else:
        ab, sb = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(s)
        want = oracle.bf16_bits_to_f32(oracle.matmulnbits(ab, b, sb, zp, N=N, K=K, dtype="bf16"))
        packed = ops.matmulnbits_prepack(cuda(b), cuda(sb).view(torch.bfloat16), cuda(zp), K=K, N=N)
        got = ops.matmulnbits_prepacked(cuda(ab).view(torch.bfloat16), packed, K=K, N=N)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, **TOL[dt])


@pytest.mark.parametrize("block", [32, 64, 128])
@pytest.mark.parametrize("M", [3, 12])
def test_matmulnbits_prepacked_long_rows_stream_activation_chunks(ops, block, M):
    """Rows too long to stage whole (M x K = 12 x 14336): each weight stage brings its k-range of
    the activation rows by bulk copy; rows beyond M read zeros."""
    rng = np.random.default_rng(block * 7 + M)
    K, N = 14336, 72
    a, b, s, zp = make_mnb(rng, M, K, N, block=block, dtype=np.float16)
    packed = ops.matmulnbits_prepack(cuda(b), cuda(s), cuda(zp), K=K, N=N, block_size=block)
    got = ops.matmulnbits_prepacked(cuda(a), packed, K=K, N=N, block_size=block).float().cpu().numpy()
    want = oracle.matmulnbits(a, b, s, zp, N=N, K=K, block_size=block).astype(np.float32)
    np.testing.assert_allclose(got, want, **TOL["f16"])


def test_matmulnbits_prepacked_matches_ort_layout_kernel(ops):
    """The tensor-core path and the ORT-layout GEMV agree on the same weights (fp16 activations)."""
    rng = np.random.default_rng(9)
    a, b, s, zp = make_mnb(rng, 2, 2048, 512, dtype=np.float16)
    ref = ops.matmulnbits(cuda(a), cuda(b), cuda(s), cuda(zp), K=2048, N=512).float()
    packed = ops.matmulnbits_prepack(cuda(b), cuda(s), cuda(zp), K=2048, N=512)
    got = ops.matmulnbits_prepacked(cuda(a), packed, K=2048, N=512).float()
    torch.testing.assert_close(got, ref, rtol=1e-2, atol=1e-3)


# ---- PagedAttention ------------------------------------------------------------------------
PAGED = load_golden("paged_attention.npz")
PAGED_CASES = sorted(k for k, v in MANIFEST.items() if v["family"] == "paged")


def _paged_run(ops, c, a, dt=None):
    kc, vc = cuda(c["key_cache"]), cuda(c["value_cache"])
    conv = (lambda x: cuda(oracle.f32_to_bf16_bits(x.astype(np.float32))).view(torch.bfloat16)) if dt == "bf16" \
        else cuda
    if dt == "bf16":
        kc, vc = conv(c["key_cache"]), conv(c["value_cache"])
    out = ops.paged_attention(
        conv(c["query"]), conv(c["key"]), conv(c["value"]), kc, vc, cuda(c["cumulative_sequence_length"]),
        cuda(c["past_seqlens"]), cuda(c["block_table"]),
        None if c.get("cos_cache") is None else conv(c["cos_cache"]),
        None if c.get("sin_cache") is None else conv(c["sin_cache"]),
        num_heads=a["num_heads"], kv_heads=a["kv_num_heads"], interleaved=a.get("rotary_interleaved", 0))
    torch.cuda.synchronize()
    return out, kc, vc


@pytest.mark.parametrize("name", PAGED_CASES)
def test_paged_attention_golden(ops, name):
    """The reference's own PagedAttention cases (test_paged_attention.py): the scattered caches are
    bit-exact, the output matches the oracle at the fp16 tolerance and the reference's fp32 port at
    its own test's 2e-2.  head_size 16 (outside the kernels' 32 / 64 / 128) is refused up front."""
    from onnxruntime_ep_b200 import B200EPError

    a, c = MANIFEST[name]["attrs"], golden_case(PAGED, name)
    D = c["query"].shape[1] // a["num_heads"]
    if D not in (32, 64, 128):
        with pytest.raises(B200EPError, match="head_size"):
            _paged_run(ops, c, a)
        return
    out, kc, vc = _paged_run(ops, c, a)
    np.testing.assert_array_equal(to_np(kc), c["expected_key_cache"])
    np.testing.assert_array_equal(to_np(vc), c["expected_value_cache"])
    want, _, _ = oracle.paged_attention(c["query"], c["key"], c["value"], c["key_cache"], c["value_cache"],
                                        c["cumulative_sequence_length"], c["past_seqlens"], c["block_table"],
                                        c.get("cos_cache"), c.get("sin_cache"), num_heads=a["num_heads"],
                                        kv_heads=a["kv_num_heads"], interleaved=a["rotary_interleaved"])
    got = to_np(out).astype(np.float32)
    np.testing.assert_allclose(got, want.astype(np.float32), **TOL["f16"])
    np.testing.assert_allclose(got, c["expected"], rtol=2e-2, atol=2e-2)


def _paged_case(rng, *, H, KV, D, bs, new_lens, pasts, nb_extra=3, rotary=True, interleaved=0):
    batch = len(new_lens)
    cum = np.concatenate([[0], np.cumsum(new_lens)]).astype(np.int32)
    past = np.asarray(pasts, dtype=np.int32)
    need = [(p + n + bs - 1) // bs for p, n in zip(pasts, new_lens)]
    maxb = max(need) + 1
    nb = sum(need) + nb_extra
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((batch, maxb), -1, dtype=np.int32)  # unused tail entries stay invalid (never read)
    o = 0
    for b, nblk in enumerate(need):
        bt[b, :nblk] = perm[o:o + nblk]
        o += nblk
    T = int(cum[-1])
    c = {"query": (rng.standard_normal((T, H * D)) * 0.5).astype(np.float16),
         "key": (rng.standard_normal((T, KV * D)) * 0.5).astype(np.float16),
         "value": rng.standard_normal((T, KV * D)).astype(np.float16),
         "key_cache": (rng.standard_normal((nb, bs, KV, D)) * 0.5).astype(np.float16),
         "value_cache": rng.standard_normal((nb, bs, KV, D)).astype(np.float16),
         "cumulative_sequence_length": cum, "past_seqlens": past, "block_table": bt}
    if rotary:
        half = D // 2
        ms = int(max(p + n for p, n in zip(pasts, new_lens))) + 5
        ang = np.arange(ms)[:, None] * (1.0 / (10000.0 ** (np.arange(half) / half)))[None, :]
        c["cos_cache"], c["sin_cache"] = np.cos(ang).astype(np.float16), np.sin(ang).astype(np.float16)
    return c, {"num_heads": H, "kv_num_heads": KV, "rotary_interleaved": interleaved}


@pytest.mark.parametrize("H,KV,D,bs,new_lens,pasts,inter", [
    (32, 8, 128, 16, [1, 1, 1, 1], [1023, 77, 0, 500], 0),       # Llama-3-8B decode batch
    (32, 8, 128, 16, [37, 1, 5], [0, 1200, 33], 0),               # prompt + decode + chunk mixed
    (64, 8, 128, 32, [1, 3], [2047, 64], 0),                      # 70B-style group of 8
    (32, 2, 64, 16, [4, 1], [9, 300], 1),                         # group of 16 (two CTAs per kv head)
    (8, 8, 32, 4, [2, 1, 6], [5, 0, 11], 1),                      # MHA, tiny blocks
    (32, 8, 128, 16, [200], [0], 0),                              # prompt (64-row tiles)
    (32, 8, 128, 16, [70, 45], [300, 0], 0),                      # two prompt chunks, one after a past
    (16, 4, 64, 32, [40], [77], 1),                               # prompt chunk, head 64, interleaved
])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_paged_attention_vs_oracle(ops, H, KV, D, bs, new_lens, pasts, inter, dt):
    rng = np.random.default_rng(H * 7 + D + sum(pasts))
    c, a = _paged_case(rng, H=H, KV=KV, D=D, bs=bs, new_lens=new_lens, pasts=pasts, interleaved=inter)
    if dt == "bf16":
        cb = {k: (oracle.f32_to_bf16_bits(v.astype(np.float32)) if v.dtype == np.float16 else v) for k, v in c.items()}
        want, wk, wv = oracle.paged_attention(cb["query"], cb["key"], cb["value"], cb["key_cache"], cb["value_cache"],
                                              cb["cumulative_sequence_length"], cb["past_seqlens"], cb["block_table"],
                                              cb.get("cos_cache"), cb.get("sin_cache"), num_heads=H, kv_heads=KV,
                                              interleaved=inter, dtype="bf16")
        out, kc, vc = _paged_run(ops, c, a, dt="bf16")
        got = oracle.bf16_bits_to_f32(to_np(out.view(torch.int16)).view(np.uint16))
        np.testing.assert_allclose(got, oracle.bf16_bits_to_f32(want), **TOL["bf16"])
        np.testing.assert_array_equal(to_np(kc.view(torch.int16)).view(np.uint16), wk)
        np.testing.assert_array_equal(to_np(vc.view(torch.int16)).view(np.uint16), wv)
    else:
        want, wk, wv = oracle.paged_attention(c["query"], c["key"], c["value"], c["key_cache"], c["value_cache"],
                                              c["cumulative_sequence_length"], c["past_seqlens"], c["block_table"],
                                              c.get("cos_cache"), c.get("sin_cache"), num_heads=H, kv_heads=KV,
                                              interleaved=inter)
        out, kc, vc = _paged_run(ops, c, a)
        np.testing.assert_allclose(to_np(out).astype(np.float32), want.astype(np.float32), **TOL["f16"])
        np.testing.assert_array_equal(to_np(kc), wk)
        np.testing.assert_array_equal(to_np(vc), wv)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_paged_attention_simt_path_vs_oracle(ops, dt, monkeypatch):
    """The SIMT attention kernel on shapes the tensor-core kernel also takes (forced by the
    ONNXRUNTIME_EP_B200_PAGED_SIMT switch), so both paths stay checked against the oracle."""
    monkeypatch.setenv("ONNXRUNTIME_EP_B200_PAGED_SIMT", "1")
    test_paged_attention_vs_oracle(ops, 32, 8, 128, 16, [37, 1, 5], [0, 1200, 33], 0, dt)


def test_paged_attention_block_outside_cache_reports_error(ops):
    """A block-table entry past the caches is never dereferenced: the append skips that row, the
    attention masks the key, and the device error word records it (then the test clears it)."""
    rng = np.random.default_rng(5)
    c, a = _paged_case(rng, H=4, KV=2, D=64, bs=8, new_lens=[1, 2], pasts=[20, 3], rotary=False)
    bt = c["block_table"].copy()
    bt[0, 1] = c["key_cache"].shape[0] + 100
    c["block_table"] = bt
    out, kc, _ = _paged_run(ops, c, a)
    code, _ = ops.device_error(clear=True)
    assert code != 0
    assert torch.isfinite(out.float()).all()
    # the untouched sequence still matches the oracle
    want, _, _ = oracle.paged_attention(c["query"][1:], c["key"][1:], c["value"][1:], c["key_cache"],
                                        c["value_cache"], np.array([0, 2], np.int32), c["past_seqlens"][1:],
                                        c["block_table"][1:], num_heads=4, kv_heads=2)
    np.testing.assert_allclose(to_np(out)[1:].astype(np.float32), want.astype(np.float32), **TOL["f16"])
