"""Generate the golden fixtures that pin the CPU oracle to the reference's own tests.

The reference (justinchuby/onnxruntime-mlx) stores no golden vectors for this path: its
tests build ONNX models with ``onnx_ir`` and compare against ORT's CPU EP at run time
(tests/ops/test_matmulnbits_asym.py:105-115, tests/ops/test_mlx_ops.py:126-249,
tests/ops/test_gqa11.py:245-264, tests/ops/test_norm_ext.py:96-146).  Neither
onnxruntime nor onnx_ir is installable here, so this script:

1. extracts, with ``ast``, the reference's own input builders and numpy references
   from its test files (``_models.py``: ``np_rms_norm``, ``np_softmax``,
   ``rotary_caches``, ``gqa_model``, ``gqa_shared_buffer_model``,
   ``matmulnbits_model``, ``rmsnorm_model``, ``skip_rmsnorm_model``,
   ``gather_block_quantized_model``; ``test_matmulnbits_asym.py``:
   ``_pack_int4_last``, ``_matmulnbits_model``; ``test_gqa11.py``:
   ``_attention_bias``, ``_gqa11_model`` and the qk-norm test's inline numpy
   reference; ``test_mlx_ops.py``: the module-level RMS inputs; ``test_paged_attention.py``:
   ``_inputs`` and ``_paged_ref``, its numpy port of ORT's PagedAttention reference) and runs them with
   stand-ins for the ONNX-building calls, so the fixtures carry exactly the inputs
   the reference's tests feed;
2. computes the expected outputs in float64 numpy — with the reference's numpy
   references where the test has one (RMS norm, the qk-norm GQA case) and with a
   numpy restatement of the reference's composed path otherwise (MatMulNBits:
   quant.rs:1078-1118; GQA: test_gqa11.py:82-98 extended with the rotary of
   attention.rs:417-461 and the shared-buffer write of attention.rs:893-902);
3. writes ``*.npz`` fixtures and ``manifest.json`` next to this file.

Run it in a container that has the reference checkout, with $REFERENCE_ROOT set to its path
(required).  It re-executes itself with PYTHONHASHSEED=0 because
several reference builders seed their RNG from ``hash((name, ...))``.
"""

from __future__ import annotations

import ast
import enum
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REFERENCE_ROOT", "")  # checkout of the reference repository (required)


# ---- stand-ins for the ONNX-building calls the reference builders make ----------------------
class DataType(enum.IntEnum):  # TensorProto element-type numbers, as onnx_ir.DataType
    FLOAT = 1
    UINT8 = 2
    INT8 = 3
    INT32 = 6
    INT64 = 7
    FLOAT16 = 10
    BFLOAT16 = 16


class _Value:
    def __init__(self, name="", type=None, shape=None, **_):
        self.name = name
        self.shape = shape


class _Spec:
    def __init__(self, name, dtype, shape):
        self.name, self.dtype, self.shape = name, dtype, list(shape)


_captured: dict = {}


def _tensor(name, dtype, shape):
    return _Spec(name, dtype, shape)


def _make_model(op_type, inputs, outputs, *, domain="", attributes=None, opset=24):
    _captured["last_model"] = dict(op_type=op_type, domain=domain, attributes=attributes or {},
                                   inputs=[getattr(i, "name", "") for i in inputs])
    return b""


def _ir_stub():
    ir = types.SimpleNamespace()
    ir.Value = _Value
    ir.DataType = DataType
    return ir


def _load_functions(path: str, names: list[str], namespace: dict, assigns: list[str] = ()):
    """Exec the named top-level defs (and simple module-level assigns) of a reference file."""
    with open(path) as f:
        tree = ast.parse(f.read(), filename=path)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id in assigns for t in node.targets):
            keep.append(node)
    found = {n.name for n in keep if isinstance(n, ast.FunctionDef)}
    missing = set(names) - found
    if missing:
        raise SystemExit(f"{path}: missing {sorted(missing)}")
    mod = ast.Module(body=keep, type_ignores=[])
    exec(compile(mod, path, "exec"), namespace)
    return namespace


def reference_namespace():
    models_path = os.path.join(REF, "tests/ops/_models.py")
    m = {"np": np, "ir": _ir_stub(), "DataType": DataType}
    m["tensor"], m["make_model"] = _tensor, _make_model
    _load_functions(models_path, [
        "np_softmax", "np_rms_norm", "rotary_caches", "gqa_shared_buffer_model", "gqa_model",
        "matmulnbits_model", "rmsnorm_model", "skip_rmsnorm_model", "gather_block_quantized_model",
    ], m)
    m_mod = types.SimpleNamespace(**{k: v for k, v in m.items() if not k.startswith("__")})

    nb = {"np": np, "m": m_mod, "DT": DataType}
    _load_functions(os.path.join(REF, "tests/ops/test_matmulnbits_asym.py"),
                    ["_pack_int4_last", "_matmulnbits_model"], nb)

    ops = {"np": np, "m": m_mod, "DT": DataType}
    _load_functions(os.path.join(REF, "tests/ops/test_mlx_ops.py"), [], ops,
                    assigns=["F16", "_rng", "RA", "RB", "RX", "RMS_X", "RMS_G"])

    # test_gqa11: the qk-norm test builds its own numpy reference and hands it to
    # m.assert_matches_ref; capture it through stand-ins.
    captured = {}

    def assert_matches_ref(model, feeds, expected, *, rtol, atol):
        captured["feeds"], captured["expected"] = feeds, expected
        captured["tol"] = (rtol, atol)

    m11 = types.SimpleNamespace(**vars(m_mod))
    m11.assert_mlx_claims = lambda model, feeds: None
    m11.assert_matches_ref = assert_matches_ref
    g11 = {"np": np, "m": m11, "DT": DataType, "ir": _ir_stub(), "NEG": np.float32(-1e4)}
    _load_functions(os.path.join(REF, "tests/ops/test_gqa11.py"),
                    ["_build_11", "_attention_bias", "_gqa11_model",
                     "test_group_query_attention_qk_norm_inputs_ort129"], g11)
    g11["_build_11"] = lambda inputs, outputs, attrs: (_captured.__setitem__("attrs11", attrs), b"")[1]
    return m_mod, nb, ops, g11, captured


# ---- numpy restatements used for expected outputs ------------------------------------------
def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Low nibble first (quant.rs:178-205)."""
    lo = packed & 0x0F
    hi = packed >> 4
    return np.stack([lo, hi], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def np_matmulnbits_dequant(b, scales, zp, *, N, K, bits, block):
    """W[N,K] fp32 = (q - zp) * scale (quant.rs:1078-1118, one fp32 multiply)."""
    nblocks = (K + block - 1) // block
    q = unpack_int4(b.reshape(N, nblocks, -1)) if bits == 4 else b.reshape(N, nblocks, block)
    q = q.reshape(N, nblocks * block).astype(np.int32)
    if zp is None:
        z = np.full((N, nblocks), 1 << (bits - 1), dtype=np.int32)
    elif bits == 4:
        z = unpack_int4(zp.reshape(N, (nblocks + 1) // 2))[:, :nblocks].astype(np.int32)
    else:
        z = zp.reshape(N, nblocks).astype(np.int32)
    d = (q - np.repeat(z, block, axis=1)).astype(np.float32)
    s = np.repeat(scales.reshape(N, nblocks).astype(np.float32), block, axis=1)
    return (d * s)[:, :K]


def np_rope(x, cos, sin, pos, interleaved):
    """x [..., S, D] float64; cos/sin rows at ``pos`` (attention.rs:417-461)."""
    half = cos.shape[1]
    c = cos[pos].astype(np.float64)
    s = sin[pos].astype(np.float64)
    out = x.copy()
    if not interleaved:
        x1, x2 = x[..., :half], x[..., half:2 * half]
        out[..., :half] = x1 * c - x2 * s
        out[..., half:2 * half] = x2 * c + x1 * s
    else:
        xe, xo = x[..., 0:2 * half:2], x[..., 1:2 * half:2]
        out[..., 0:2 * half:2] = xe * c - xo * s
        out[..., 1:2 * half:2] = xo * c + xe * s
    return out


def np_gqa(feeds, attrs, *, cap_shared):
    """GQA in float64 following test_gqa11.py:82-98 plus rotary and the shared buffer."""
    q = feeds["query"].astype(np.float64)
    H, HK = attrs["num_heads"], attrs["kv_num_heads"]
    packed = "key" not in feeds
    B, S, W = q.shape
    D = W // (H + 2 * HK) if packed else W // H
    if packed:
        k = q[..., H * D:(H + HK) * D]
        v = q[..., (H + HK) * D:]
        q = q[..., :H * D]
    else:
        k = feeds["key"].astype(np.float64)
        v = feeds["value"].astype(np.float64)
    pk = feeds["past_key"].astype(np.float64)
    pv = feeds["past_value"].astype(np.float64)
    total = int(feeds["total_sequence_length"][0])
    past = total - S  # the reference's valid_past (attention.rs:630-642)
    qh = q.reshape(B, S, H, D).transpose(0, 2, 1, 3)
    kh = k.reshape(B, S, HK, D).transpose(0, 2, 1, 3)
    vh = v.reshape(B, S, HK, D).transpose(0, 2, 1, 3)
    if attrs.get("do_rotary", 1) and "cos_cache" in feeds:
        pos = np.arange(past, past + S)
        qh = np_rope(qh, feeds["cos_cache"], feeds["sin_cache"], pos, attrs.get("rotary_interleaved", 0))
        kh = np_rope(kh, feeds["cos_cache"], feeds["sin_cache"], pos, attrs.get("rotary_interleaved", 0))
        # ORT stores the rotated rows in the I/O dtype (fp32 here)
        qh = qh.astype(np.float32).astype(np.float64)
        kh = kh.astype(np.float32).astype(np.float64)
    if cap_shared:
        present_k = pk.copy()
        present_v = pv.copy()
        present_k[:, :, past:past + S] = kh
        present_v[:, :, past:past + S] = vh
    else:
        present_k = np.concatenate([pk[:, :, :past], kh], axis=2)
        present_v = np.concatenate([pv[:, :, :past], vh], axis=2)
    keys = np.repeat(present_k[:, :, :total], H // HK, axis=1)
    vals = np.repeat(present_v[:, :, :total], H // HK, axis=1)
    scale = attrs.get("scale") or 1.0 / np.sqrt(D)
    scores = np.matmul(qh, keys.transpose(0, 1, 3, 2)) * scale
    if "attention_bias" in feeds:
        scores = scores + feeds["attention_bias"][..., :total].astype(np.float64)
    causal = np.arange(total)[None, :] <= (past + np.arange(S))[:, None]
    scores = np.where(causal[None, None], scores, -np.inf)
    probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    out = np.matmul(probs, vals).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    return out, present_k, present_v


def np_gqa_sliding(feeds, attrs):
    """GroupQueryAttention with sliding_window_cache = 1 in float64, following attention.rs:725-880:
    per batch the resident rows end at end(L) = L - gap * ceil((L - cap) / gap) once L exceeds the
    capacity (gap = cap - window + 1); the attention runs over the seed rows (from row 0 when any
    batch's kept rows cannot cover the window: the staging form) followed by the new rows, with the
    causal window mask; q / k are rotated at their absolute positions; present holds the rows kept
    after this step from row 0, zeros after them."""
    H, HK = attrs["num_heads"], attrs["kv_num_heads"]
    W = attrs["local_window_size"]
    q = feeds["query"].astype(np.float64)
    B, S, width = q.shape
    D = width // H
    k = feeds["key"].astype(np.float64).reshape(B, S, HK, D).transpose(0, 2, 1, 3)
    v = feeds["value"].astype(np.float64).reshape(B, S, HK, D).transpose(0, 2, 1, 3)
    q = q.reshape(B, S, H, D).transpose(0, 2, 1, 3)
    pk, pv = feeds["past_key"].astype(np.float64), feeds["past_value"].astype(np.float64)
    cap = pk.shape[2]
    gap = cap - W + 1

    def end(length):
        return length if length <= cap else length - gap * ((length - cap + gap - 1) // gap)

    geo, staging = [], False
    for b in range(B):
        p = max(int(feeds["seqlens_k"][b]) + 1 - S, 0)
        before, after = end(p), end(p + S)
        kept = after - S
        staging |= kept < min(p, W - 1)
        geo.append((p, before, after, before - kept))
    scale = attrs.get("scale") or 1.0 / np.sqrt(D)
    out = np.zeros((B, H, S, D))
    present_k, present_v = np.zeros_like(pk), np.zeros_like(pv)
    for b, (p, before, after, off) in enumerate(geo):
        qb, kb = q[b], k[b]
        if attrs.get("do_rotary", 1) and "cos_cache" in feeds:
            pos = np.arange(p, p + S)
            il = attrs.get("rotary_interleaved", 0)
            qb = np_rope(qb, feeds["cos_cache"], feeds["sin_cache"], pos, il).astype(np.float32).astype(np.float64)
            kb = np_rope(kb, feeds["cos_cache"], feeds["sin_cache"], pos, il).astype(np.float32).astype(np.float64)
        start = 0 if staging else off
        wk = np.concatenate([pk[b, :, start:before], kb], axis=1)
        wv = np.concatenate([pv[b, :, start:before], v[b]], axis=1)
        seed, klen = before - start, before - start + S
        qpos = seed + np.arange(S)[:, None]
        kpos = np.arange(klen)[None, :]
        allow = (kpos <= qpos) & (kpos >= qpos - W + 1)
        keys = np.repeat(wk, H // HK, axis=0)
        vals = np.repeat(wv, H // HK, axis=0)
        sc = np.matmul(qb, keys.transpose(0, 2, 1)) * scale
        sc = np.where(allow[None], sc, -np.inf)
        pr = np.exp(sc - sc.max(-1, keepdims=True))
        pr /= pr.sum(-1, keepdims=True)
        out[b] = np.matmul(pr, vals)
        ws = off if staging else 0
        present_k[b, :, :after] = wk[:, ws:ws + after]
        present_v[b, :, :after] = wv[:, ws:ws + after]
    return out.transpose(0, 2, 1, 3).reshape(B, S, H * D), present_k, present_v


# ---- fixture families ----------------------------------------------------------------------
def gen_matmulnbits(nb, m, out, manifest):
    cases = []
    for block in (16, 32, 64, 128):
        for M in (1, 8):
            cases.append(("sym", dict(M=M, K=block * 2, N=32, block=block, asymmetric=False)))
            cases.append(("asym", dict(M=M, K=block * 3, N=16, block=block, asymmetric=True)))
            for asym in (False, True):
                cases.append(("fp16", dict(M=M, K=block * 3, N=16, block=block, asymmetric=asym,
                                           dtype=DataType.FLOAT16)))
    for M in (1, 8):
        for asym in (False, True):
            cases.append(("int8", dict(M=M, K=96, N=32, block=32, asymmetric=asym, bits=8)))
    cases.append(("fp16-partial", dict(M=4, K=1176, N=16, block=32, asymmetric=True,
                                       dtype=DataType.FLOAT16)))
    for idx, (tag, kw) in enumerate(cases):
        _model, feeds = nb["_matmulnbits_model"](**kw)
        bits = kw.get("bits", 4)
        dt = kw.get("dtype", DataType.FLOAT)
        a = feeds["a"]
        zp = feeds.get("zero_points")
        W = np_matmulnbits_dequant(feeds["b"], feeds["scales"], zp, N=kw["N"], K=kw["K"], bits=bits,
                                   block=kw["block"])
        K = kw["K"]
        y = a.reshape(-1, K).astype(np.float64) @ W.astype(np.float64).T
        y = y.reshape(a.shape[:-1] + (kw["N"],)).astype(a.dtype)
        name = f"mnb{idx:02d}"
        out[f"{name}/a"], out[f"{name}/b"], out[f"{name}/scales"] = a, feeds["b"], feeds["scales"]
        if zp is not None:
            out[f"{name}/zero_points"] = zp
        out[f"{name}/w"], out[f"{name}/y"] = W, y
        manifest[name] = dict(family="matmulnbits", tag=tag, M=kw["M"], K=K, N=kw["N"], bits=bits,
                              block_size=kw["block"], asymmetric=kw["asymmetric"],
                              dtype="f16" if dt == DataType.FLOAT16 else "f32",
                              source="tests/ops/test_matmulnbits_asym.py:_matmulnbits_model")
    for M in (1, 8):  # test_mlx_ops.py:test_matmulnbits (3-input, random packed bytes)
        _model, feeds = m.matmulnbits_model(M=M, K=64, N=32)
        W = np_matmulnbits_dequant(feeds["b"], feeds["scales"], None, N=32, K=64, bits=4, block=32)
        y = (feeds["a"].reshape(-1, 64).astype(np.float64) @ W.astype(np.float64).T)
        name = f"mnbops{M}"
        out[f"{name}/a"], out[f"{name}/b"], out[f"{name}/scales"] = feeds["a"], feeds["b"], feeds["scales"]
        out[f"{name}/w"] = W
        out[f"{name}/y"] = y.reshape(1, M, 32).astype(np.float32)
        manifest[name] = dict(family="matmulnbits", tag="ops", M=M, K=64, N=32, bits=4, block_size=32,
                              asymmetric=False, dtype="f32",
                              source="tests/ops/_models.py:matmulnbits_model")


GQA_CASES = [  # tests/ops/test_mlx_ops.py:143-215
    ("decode-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=1, past=40, do_rotary=1)),
    ("prefill-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=26, past=0, do_rotary=1)),
    ("chunked-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=3, past=8, do_rotary=1)),
    ("decode", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=1, past=5, do_rotary=1)),
    ("prefill", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=6, past=0, do_rotary=1)),
    ("decode-packed", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=1, past=40, do_rotary=1,
                           packed_qkv=True)),
    ("prefill-packed", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=8, past=0, do_rotary=1,
                            packed_qkv=True)),
    ("decode-norope", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=1, past=5, do_rotary=0)),
    ("decode-extrope-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=1, past=40,
                                do_rotary=0, rope_cache=False)),
    ("prefill-extrope-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=8, past=0,
                                 do_rotary=0, rope_cache=False)),
]
SHARED_GQA_CASES = [  # tests/ops/test_mlx_ops.py:218-224
    ("shared-decode-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=1, past=40, cap=128,
                               do_rotary=1)),
    ("shared-chunked-h64", dict(batch=1, num_heads=14, kv_heads=2, head=64, seq=3, past=8, cap=64,
                                do_rotary=1)),
    ("shared-decode", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=1, past=5, cap=32, do_rotary=1)),
    ("shared-decode-norope", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=1, past=5, cap=32,
                                  do_rotary=0)),
]
SLIDING_GQA_CASES = [  # tests/ops/test_mlx_ops.py:251-297 (sliding_window_cache = 1)
    ("sliding-decode", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=1, past=8, cap=5, do_rotary=0,
                            sliding_window=1, local_window=3)),
    ("sliding-chunk-staging", dict(batch=1, num_heads=4, kv_heads=2, head=16, seq=3, past=5, cap=5,
                                   do_rotary=0, sliding_window=1, local_window=4)),
    ("sliding-batched-rope", dict(batch=2, num_heads=4, kv_heads=2, head=16, seq=1, past=7, cap=6,
                                  do_rotary=1, sliding_window=1, local_window=4)),
]
GQA11_CASES = [  # tests/ops/test_gqa11.py:215-221
    ("prefill", dict(batch=1, seq=6, past=0, cap=6, num_heads=4, kv_heads=2, head=16, window=4)),
    ("chunked", dict(batch=1, seq=3, past=4, cap=7, num_heads=4, kv_heads=2, head=16, window=3)),
    ("decode", dict(batch=1, seq=1, past=5, cap=6, num_heads=4, kv_heads=2, head=16, window=3)),
    ("shared-decode", dict(batch=1, seq=1, past=5, cap=32, num_heads=4, kv_heads=2, head=16, window=3)),
    ("shared-chunked", dict(batch=1, seq=3, past=8, cap=64, num_heads=8, kv_heads=1, head=32, window=4)),
]


def _store_gqa(out, manifest, name, feeds, attrs, expected, *, shared, source):
    for key, val in feeds.items():
        out[f"{name}/{key}"] = val
    o, pk, pv = expected
    dt = feeds["query"].dtype
    out[f"{name}/out"] = o.astype(dt)
    out[f"{name}/present_key"] = pk.astype(dt)
    out[f"{name}/present_value"] = pv.astype(dt)
    manifest[name] = dict(family="gqa", shared=shared, source=source,
                          attrs={k: (float(v) if isinstance(v, (float, np.floating)) else int(v))
                                 for k, v in attrs.items()})


def gen_gqa(m, g11, captured, out, manifest):
    for name, geom in GQA_CASES:
        _model, feeds = m.gqa_model(name, **geom)
        attrs = dict(_captured["last_model"]["attributes"])
        _store_gqa(out, manifest, f"gqa/{name}", feeds, attrs, np_gqa(feeds, attrs, cap_shared=False),
                   shared=False, source="tests/ops/_models.py:gqa_model")
    for name, geom in SHARED_GQA_CASES:
        _model, feeds = m.gqa_shared_buffer_model(name, **geom)
        attrs = dict(_captured["last_model"]["attributes"])
        _store_gqa(out, manifest, f"gqa/{name}", feeds, attrs, np_gqa(feeds, attrs, cap_shared=True),
                   shared=True, source="tests/ops/_models.py:gqa_shared_buffer_model")
    for name, geom in SLIDING_GQA_CASES:
        _model, feeds = m.gqa_shared_buffer_model(name, **geom)
        attrs = dict(_captured["last_model"]["attributes"])
        _store_gqa(out, manifest, f"gqasliding/{name}", feeds, attrs, np_gqa_sliding(feeds, attrs), shared=True,
                   source="tests/ops/_models.py:gqa_shared_buffer_model (sliding_window=1)")
        manifest[f"gqasliding/{name}"]["family"] = "gqa_sliding"
    for name, geom in GQA11_CASES:
        _model, feeds = g11["_gqa11_model"](with_position_ids=False, **geom)
        attrs = dict(_captured["attrs11"])
        shared = geom["cap"] > geom["past"] + geom["seq"]
        _store_gqa(out, manifest, f"gqa11/{name}", feeds, attrs,
                   np_gqa(feeds, attrs, cap_shared=shared), shared=shared,
                   source="tests/ops/test_gqa11.py:_gqa11_model")
    # qk-norm case: the reference's own numpy expected output (test_gqa11.py:52-131)
    g11["test_group_query_attention_qk_norm_inputs_ort129"]()
    feeds = {"query": captured["feeds"]["q"], "key": captured["feeds"]["k"],
             "value": captured["feeds"]["v"], "past_key": captured["feeds"]["pk"],
             "past_value": captured["feeds"]["pv"], "seqlens_k": captured["feeds"]["seqlens"],
             "total_sequence_length": captured["feeds"]["total"],
             "q_norm": captured["feeds"]["qw"], "k_norm": captured["feeds"]["kw"]}
    attrs = dict(_captured["attrs11"])
    _store_gqa(out, manifest, "gqa11/qk-norm", feeds, attrs, captured["expected"], shared=False,
               source="tests/ops/test_gqa11.py:test_group_query_attention_qk_norm_inputs_ort129 (numpy)")


def gen_norms(m, ops, out, manifest):
    _model, f = m.rmsnorm_model(rows=4, hidden=64)  # test_mlx_ops.py:test_rmsnorm
    out["rms/x"], out["rms/scale"] = f["x"], f["scale"]
    out["rms/y"] = m.np_rms_norm(f["x"].astype(np.float64), f["scale"].astype(np.float64), 1e-6).astype(np.float32)
    manifest["rms"] = dict(family="rms", eps=1e-6, dtype="f32", source="tests/ops/_models.py:rmsnorm_model")
    _model, f = m.skip_rmsnorm_model(rows=4, hidden=64)  # test_mlx_ops.py:test_skip_simplified_layernorm
    out["skiprms/x"], out["skiprms/skip"], out["skiprms/gamma"] = f["x"], f["skip"], f["gamma"]
    r = f["x"].astype(np.float64) + f["skip"].astype(np.float64)
    out["skiprms/y"] = m.np_rms_norm(r, f["gamma"].astype(np.float64), 1e-6).astype(np.float32)
    out["skiprms/residual"] = r.astype(np.float32)
    manifest["skiprms"] = dict(family="skiprms", eps=1e-6, dtype="f32",
                               source="tests/ops/_models.py:skip_rmsnorm_model")
    # RMSNormalization dtype-generic inputs (test_mlx_ops.py:25-31, 382-474)
    x, g = ops["RMS_X"], ops["RMS_G"]
    out["rms16/x"], out["rms16/scale"] = x.astype(np.float16), g.astype(np.float16)
    out["rms16/y"] = m.np_rms_norm(x.astype(np.float16).astype(np.float64),
                                   g.astype(np.float16).astype(np.float64)).astype(np.float16)
    manifest["rms16"] = dict(family="rms", eps=1e-6, dtype="f16", source="tests/ops/test_mlx_ops.py:_fp16_rmsnorm")
    out["rmsbf16/x"], out["rmsbf16/scale"] = x, g
    out["rmsbf16/y"] = m.np_rms_norm(x, g)  # the reference's bf16 expected value (fp32 numpy)
    manifest["rmsbf16"] = dict(family="rms", eps=1e-6, dtype="bf16",
                               source="tests/ops/test_mlx_ops.py:_bf16_cases RMSNormalization")
    rng = np.random.default_rng(3)  # test_norm_ext.py:test_simplified_layer_norm
    x = rng.standard_normal((2, 4, 8)).astype(np.float32)
    s = rng.standard_normal((8,)).astype(np.float32)
    out["sln/x"], out["sln/scale"] = x, s
    out["sln/y"] = m.np_rms_norm(x.astype(np.float64), s.astype(np.float64), 1e-5).astype(np.float32)
    manifest["sln"] = dict(family="rms", eps=1e-5, dtype="f32",
                           source="tests/ops/test_norm_ext.py:test_simplified_layer_norm")


def gen_gbq(m, out, manifest):
    _model, f = m.gather_block_quantized_model()
    attrs = _captured["last_model"]["attributes"]
    data, idx, scales = f["data"], f["indices"], f["scales"]
    vocab, dim, block = data.shape[0], data.shape[1] * 2, attrs["block_size"]
    rows = np.where(idx < 0, idx + vocab, idx)
    q = unpack_int4(data[rows]).astype(np.float32)
    s = np.repeat(scales[rows], block, axis=1)
    out["gbq/data"], out["gbq/indices"], out["gbq/scales"] = data, idx, scales
    out["gbq/y"] = (q - 8.0) * s
    manifest["gbq"] = dict(family="gbq", block_size=block, source="tests/ops/_models.py:gather_block_quantized_model")


def gen_paged(out, manifest):
    """PagedAttention: the inputs and expected outputs of the reference's own test parameter sets
    (test_paged_attention.py ``_inputs`` and its numpy port of ORT's reference ``_paged_ref``),
    plus the caches after the scatter of the new rows."""
    import math

    path = os.path.join(REF, "tests/ops/test_paged_attention.py")
    ns = _load_functions(path, ["_rotate_half", "_apply_rope", "_paged_ref", "_inputs"], {"np": np, "math": math})
    src = "tests/ops/test_paged_attention.py"
    cases = []
    for H, KV in ((4, 2), (4, 4), (8, 2), (2, 1)):  # test_paged_attention_core
        for batch in (1, 3):
            cases.append((f"core-h{H}kv{KV}-b{batch}", H, KV, 16, 8 * batch, 4, batch, 0, 0, H * 10 + KV + batch))
    for blk in (2, 8):  # test_paged_attention_multiblock
        cases.append((f"multiblock-blk{blk}", 8, 2, 32, 16, blk, 2, 0, 0, blk + 7))
    for inter in (0, 1):  # test_paged_attention_rotary
        for H, KV, d in ((4, 2, 16), (2, 1, 64)):
            cases.append((f"rotary-{'gptj' if inter else 'neox'}-h{H}d{d}", H, KV, d, 16, 4, 2, 1, inter,
                           H + d + inter))
    for name, H, KV, d, nb, blk, batch, rot, inter, seed in cases:
        feeds, ref = ns["_inputs"](H, KV, d, nb, blk, batch, rot, inter, seed)
        cos, sin = feeds.get("cos_cache"), feeds.get("sin_cache")
        _, kc, vc = ns["_paged_ref"](feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"],
                                     feeds["value_cache"], feeds["cumulative_sequence_length"],
                                     feeds["past_seqlens"], feeds["block_table"], H, KV, d,
                                     cos=None if cos is None else cos.astype(np.float32),
                                     sin=None if sin is None else sin.astype(np.float32), interleaved=inter,
                                     return_cache=True)
        key = f"paged/{name}"
        for fname, val in feeds.items():
            out[f"{key}/{fname}"] = val
        out[f"{key}/expected"] = ref.astype(np.float32)
        out[f"{key}/expected_key_cache"] = kc
        out[f"{key}/expected_value_cache"] = vc
        manifest[key] = {"family": "paged", "source": f"{src}:_inputs/_paged_ref",
                         "attrs": {"num_heads": H, "kv_num_heads": KV, "do_rotary": rot, "rotary_interleaved": inter},
                         "tolerance": {"rtol": 2e-2, "atol": 2e-2}}


def main() -> None:
    if os.environ.get("PYTHONHASHSEED") != "0":
        os.environ["PYTHONHASHSEED"] = "0"
        os.execv(sys.executable, [sys.executable] + sys.argv)
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set REFERENCE_ROOT to a checkout of the reference repository "
                         f"(got {REF!r})")
    m, nb, ops, g11, captured = reference_namespace()
    manifest: dict = {}
    mnb, gq, nm, gb = {}, {}, {}, {}
    gen_matmulnbits(nb, m, mnb, manifest)
    gen_gqa(m, g11, captured, gq, manifest)
    gen_norms(m, ops, nm, manifest)
    gen_gbq(m, gb, manifest)
    pa: dict = {}
    gen_paged(pa, manifest)
    np.savez_compressed(os.path.join(HERE, "matmulnbits.npz"), **mnb)
    np.savez_compressed(os.path.join(HERE, "gqa.npz"), **gq)
    np.savez_compressed(os.path.join(HERE, "norms.npz"), **nm)
    np.savez_compressed(os.path.join(HERE, "gather_block_quantized.npz"), **gb)
    np.savez_compressed(os.path.join(HERE, "paged_attention.npz"), **pa)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"wrote {len(manifest)} golden cases")


if __name__ == "__main__":
    main()
