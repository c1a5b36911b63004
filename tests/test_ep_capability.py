"""Host-side EP logic on CPU: claim predicates, convex clustering, layer partitions.

Restates the reference's claim rules (rust/src/ops/quant.rs:1655-1711,
attention.rs:1520-1738, norm.rs:460-610) and its Rust unit tests for partitioning
(rust/src/ep.rs:518-572).  No GPU is touched: GetCapability is pure host code.
"""

from __future__ import annotations

import numpy as np
import pytest

from onnxruntime_ep_b200.ep import FLOAT, FLOAT16, INT32, INT64, UINT8, ExecutionProvider, GraphBuilder


def mnb_graph(*, bits=4, block=32, K=64, N=32, a_dtype=FLOAT, s_dtype=FLOAT, out_dtype=FLOAT, zp=True,
              extra_inputs=0, weights_as_inputs=False):
    g = GraphBuilder()
    nb = (K + block - 1) // block
    g.input("a", a_dtype, [1, 2, K])
    np_s = np.float16 if s_dtype == FLOAT16 else np.float32
    if weights_as_inputs:
        g.input("b", UINT8, [N, nb, block * bits // 8])
    else:
        g.initializer("b", np.zeros((N, nb, block * bits // 8), np.uint8))
    g.initializer("s", np.ones(N * nb, np_s), s_dtype)
    ins = ["a", "b", "s"]
    if zp:
        g.initializer("z", np.zeros(N * ((nb + 1) // 2) if bits == 4 else N * nb, np.uint8))
        ins.append("z")
    for i in range(extra_inputs):
        if len(ins) == 3:
            ins.append("")
        g.input(f"x{i}", INT32, [K])
        ins.append(f"x{i}")
    g.output("y", out_dtype, [1, 2, N])
    g.node("MatMulNBits", ins, ["y"], domain="com.microsoft", K=K, N=N, bits=bits, block_size=block)
    return g


def claimed(g, **opts):
    ep = ExecutionProvider(**opts)
    groups, num = ep.get_capability(g)
    return ep, groups, num


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("block", [16, 32, 64, 128])
def test_matmulnbits_claims_supported_forms(bits, block):
    _, groups, num = claimed(mnb_graph(bits=bits, block=block, K=block * 3))
    assert groups == [0] and num == 1


@pytest.mark.parametrize("kw,reason", [
    (dict(block=24), "block_size"),
    (dict(bits=2), "4-bit and 8-bit"),
    (dict(s_dtype=FLOAT16), "share one float dtype"),
    (dict(out_dtype=FLOAT16), "share one float dtype"),
    (dict(extra_inputs=1), "g_idx and bias"),
    (dict(weights_as_inputs=True), "initializers"),
])
def test_matmulnbits_declines_with_reason(kw, reason):
    ep, groups, num = claimed(mnb_graph(**kw))
    assert groups == [-1] and num == 0
    assert reason in ep.claim_reason(0)


def gqa_graph(*, packed=False, do_rotary=1, nin=9, softcap=0.0, qk_output=0, smooth=0, pos_ids=False,
              dtype=FLOAT16, cos_dtype=None, kquant=None, qk_norm=False, present=True, sliding_window=None,
              bias=False):
    g = GraphBuilder()
    B, S, H, HK, D, cap = 1, 1, 4, 2, 16, 32
    qw = (H + 2 * HK) * D if packed else H * D
    g.input("q", dtype, [B, S, qw])
    if not packed:
        g.input("k", dtype, [B, S, HK * D])
        g.input("v", dtype, [B, S, HK * D])
    g.input("pk", dtype, [B, HK, cap, D])
    g.input("pv", dtype, [B, HK, cap, D])
    g.input("seqlens", INT32, [B])
    g.input("total", INT32, [1])
    ins = ["q", "" if packed else "k", "" if packed else "v", "pk", "pv", "seqlens", "total"]
    if nin >= 9:
        cd = cos_dtype or dtype
        npd = np.float16 if cd == FLOAT16 else np.float32
        g.initializer("cos", np.ones((64, D // 2), npd), cd)
        g.initializer("sin", np.zeros((64, D // 2), npd), cd)
        ins += ["cos", "sin"]
    if pos_ids:
        g.input("pos", INT64, [B, S])
        ins += ["pos"]
    if bias:
        while len(ins) < 10:
            ins.append("")
        g.input("bias", dtype, [B, 1, S, cap])
        ins.append("bias")
    if qk_norm:
        while len(ins) < 14:
            ins.append("")
        npd = np.float16 if dtype == FLOAT16 else np.float32
        g.initializer("qn", np.ones(D, npd), dtype)
        g.initializer("kn", np.ones(D, npd), dtype)
        ins += ["qn", "kn"]
    g.output("out", dtype, [B, S, H * D])
    outs = ["out"]
    if present:
        g.output("prk", dtype, [B, HK, cap, D])
        g.output("prv", dtype, [B, HK, cap, D])
        outs += ["prk", "prv"]
    attrs = dict(num_heads=H, kv_num_heads=HK, do_rotary=do_rotary)
    if softcap:
        attrs["softcap"] = softcap
    if qk_output:
        attrs["qk_output"] = qk_output
    if smooth:
        attrs["smooth_softmax"] = smooth
    if kquant:
        attrs["k_quant_type"] = kquant
    if sliding_window is not None:
        attrs["sliding_window_cache"] = 1
        attrs["local_window_size"] = sliding_window
    g.node("GroupQueryAttention", ins, outs, domain="com.microsoft", **attrs)
    return g


@pytest.mark.parametrize("kw", [dict(), dict(packed=True), dict(nin=7, do_rotary=0), dict(dtype=FLOAT),
                                dict(qk_norm=True), dict(sliding_window=16), dict(sliding_window=32, packed=True)])
def test_gqa_claims(kw):
    _, groups, _ = claimed(gqa_graph(**kw))
    assert groups == [0]


@pytest.mark.parametrize("kw,reason", [
    (dict(nin=7, do_rotary=1), "do_rotary=0"),
    (dict(softcap=30.0), "softcap"),
    (dict(qk_output=1), "qk_output"),
    (dict(smooth=1), "smooth_softmax"),
    (dict(kquant="PER_TENSOR"), "quantized KV"),
    (dict(cos_dtype=FLOAT), "must have output dtype"),
    # sliding-window cache conditions (attention.rs:1552-1575)
    (dict(sliding_window=0), "local_window_size > 0"),
    (dict(sliding_window=8, bias=True), "incompatible with attention_bias"),
    (dict(sliding_window=8, present=False), "present key/value"),
    (dict(sliding_window=64), "capacity must be at least local_window_size"),
])
def test_gqa_declines_with_reason(kw, reason):
    ep, groups, _ = claimed(gqa_graph(**kw))
    assert groups == [-1]
    assert reason in ep.claim_reason(0)


def norm_graph(op, domain, *, axis=None, dtype=FLOAT, opset=24, nin=2):
    g = GraphBuilder(opset=opset)
    g.input("x", dtype, [2, 4, 8])
    npd = np.float16 if dtype == FLOAT16 else np.float32
    g.initializer("s", np.ones(8, npd), dtype)
    ins = ["x", "s"]
    if nin == 3:
        g.input("skip", dtype, [2, 4, 8])
        ins = ["x", "skip", "s"]
    g.output("y", dtype, [2, 4, 8])
    attrs = {} if axis is None else {"axis": axis}
    g.node(op, ins, ["y"], domain=domain, **attrs)
    return g


def test_norm_claims():
    assert claimed(norm_graph("SimplifiedLayerNormalization", "com.microsoft"))[1] == [0]
    # mis-stamped default-domain SimplifiedLayerNormalization is claimed (norm.rs:938-952)
    assert claimed(norm_graph("SimplifiedLayerNormalization", ""))[1] == [0]
    assert claimed(norm_graph("RMSNormalization", "", opset=23))[1] == [0]
    assert claimed(norm_graph("SkipSimplifiedLayerNormalization", "com.microsoft", nin=3))[1] == [0]


def test_norm_declines():
    ep, groups, _ = claimed(norm_graph("RMSNormalization", "", opset=22))
    assert groups == [-1] and "opset 22" in ep.claim_reason(0)
    ep, groups, _ = claimed(norm_graph("SimplifiedLayerNormalization", "com.microsoft", axis=1))
    assert groups == [-1] and "last axis" in ep.claim_reason(0)
    ep, groups, _ = claimed(norm_graph("LayerNormalization", ""))
    assert groups == [-1] and "no B200 handler" in ep.claim_reason(0)


def test_convex_clusters_split_around_unclaimed_node():
    """a -> relu(unclaimed) -> c with a -> c directly: {a, c} is not convex, so two partitions."""
    g = GraphBuilder()
    g.input("x", FLOAT, [4])
    for n in ("a", "r", "c"):
        g.tensor(n, FLOAT, [4])
    g.output("c", FLOAT, [4])
    g.node("Sigmoid", ["x"], ["a"], name="a")
    g.node("Relu", ["a"], ["r"], name="relu")
    g.node("Add", ["a", "r"], ["c"], name="c")
    ep, groups, num = claimed(g)
    assert groups[1] == -1 and "no B200 handler" in ep.claim_reason(1)
    assert groups[0] >= 0 and groups[2] >= 0 and groups[0] != groups[2] and num == 2


def test_session_summary_counts_claims_and_reasons():
    """The session summary (reference: MlxTracer::log_summary, rust/src/trace.rs:640-735) counts
    claimed nodes, partitions and, per op type, why nodes stayed on CPU; no GPU work recorded."""
    g = GraphBuilder()
    g.input("x", FLOAT, [4])
    for n in ("a", "r", "c"):
        g.tensor(n, FLOAT, [4])
    g.output("c", FLOAT, [4])
    g.node("Sigmoid", ["x"], ["a"], name="a")
    g.node("Relu", ["a"], ["r"], name="relu")
    g.node("Add", ["a", "r"], ["c"], name="c")
    ep, _, num = claimed(g)
    ep.get_capability(g)
    s = ep.summary()
    assert s["getcap_calls"] == 2 and s["total_nodes"] == 6 and s["claimed_nodes"] == 4
    assert s["partitions"] == 2 * num
    assert s["rejected"]["Relu"]["nodes"] == 2 and "no B200 handler" in s["rejected"]["Relu"]["reason"]
    assert s["compiles"] == 0 and s["path_decode"] == s["path_prefill"] == s["eager_runs"] == 0


def test_convex_cluster_merges_chain():
    g = GraphBuilder()
    g.input("x", FLOAT, [4])
    prev = "x"
    for i in range(5):
        g.tensor(f"t{i}", FLOAT, [4])
        g.node("Sigmoid" if i % 2 else "Mul", [prev] if i % 2 else [prev, prev], [f"t{i}"])
        prev = f"t{i}"
    g.output(prev, FLOAT, [4])
    _, groups, num = claimed(g)
    assert groups == [0] * 5 and num == 1


def layered_graph(layers):
    """GQA -> Add (residual) -> Sigmoid -> Add per layer, the structure the reference's boundary
    inference test uses (ep.rs:543-571): each layer's last residual Add closes it."""
    g = GraphBuilder()
    B, S, H, HK, D, cap = 1, 1, 2, 1, 16, 8
    g.input("x", FLOAT16, [B, S, H * D])
    g.input("seqlens", INT32, [B])
    g.input("total", INT32, [1])
    prev = "x"
    for i in range(layers):
        g.input(f"pk{i}", FLOAT16, [B, HK, cap, D])
        g.input(f"pv{i}", FLOAT16, [B, HK, cap, D])
        g.output(f"prk{i}", FLOAT16, [B, HK, cap, D])
        g.output(f"prv{i}", FLOAT16, [B, HK, cap, D])
        for t in ("k", "v"):
            g.initializer(f"{t}{i}", np.zeros((B, S, HK * D), np.float16), FLOAT16)
        for t in ("attn", "r1", "s", "r2"):
            g.tensor(f"{t}{i}", FLOAT16, [B, S, H * D])
        g.node("GroupQueryAttention", [prev, f"k{i}", f"v{i}", f"pk{i}", f"pv{i}", "seqlens", "total"],
               [f"attn{i}", f"prk{i}", f"prv{i}"], domain="com.microsoft", num_heads=H, kv_num_heads=HK,
               do_rotary=0, name=f"gqa{i}")
        g.node("Add", [prev, f"attn{i}"], [f"r1{i}"], name=f"add_attn{i}")
        g.node("Sigmoid", [f"r1{i}"], [f"s{i}"], name=f"mlp{i}")
        g.node("Add", [f"r1{i}", f"s{i}"], [f"r2{i}"], name=f"add_mlp{i}")
        prev = f"r2{i}"
    g.output(prev, FLOAT16, [B, S, H * D])
    return g


@pytest.mark.parametrize("setting,layers,expected", [
    ("off", 24, 1), ("0", 24, 1), ("auto", 16, 1), ("auto", 24, 6), ("5", 24, 5), ("auto", 52, 7),
    ("invalid", 24, 1),
])
def test_layer_partition_span(setting, layers, expected):
    """select_layer_partition_span (ep.rs:359-370 and its tests ep.rs:522-540): auto splits decoders of
    >= 23 layers into spans of ceil(L/7) clamped to [4, 8]; explicit spans and off-switches."""
    _, groups, num = claimed(layered_graph(layers), layer_partitions=setting)
    assert num == expected
    assert all(gi >= 0 for gi in groups)


def test_layer_boundaries_follow_metadata():
    g = layered_graph(4)
    g.metadata("onnxruntime_ep_mlx.layer_boundary_outputs", "r10,r22")
    _, groups, num = claimed(g, layer_partitions="1")
    # boundaries after layer 1's attention residual and layer 2's mlp residual -> 3 partitions
    assert num == 3


def test_unset_layer_partitions_keep_one_partition():
    _, _, num = claimed(layered_graph(24))
    assert num == 1


def paged_graph(*, H=4, KV=2, D=64, dtype=FLOAT16, do_rotary=1, layout=None, extra=(), rotary_offset=0,
                local_window=None, cos_dtype=None):
    g = GraphBuilder()
    nb, blk, batch, maxb = 16, 8, 2, 8
    g.input("q", dtype, [-1, H * D])
    g.input("k", dtype, [-1, KV * D])
    g.input("v", dtype, [-1, KV * D])
    g.input("kc", dtype, [nb, blk, KV, D])
    g.input("vc", dtype, [nb, blk, KV, D])
    g.input("cum", INT32, [batch + 1])
    g.input("past", INT32, [batch])
    g.input("bt", INT32, [batch, maxb])
    ins = ["q", "k", "v", "kc", "vc", "cum", "past", "bt"]
    if do_rotary:
        cd = cos_dtype or dtype
        npd = np.float16 if cd == FLOAT16 else np.float32
        g.initializer("cos", np.ones((64, D // 2), npd), cd)
        g.initializer("sin", np.zeros((64, D // 2), npd), cd)
        ins += ["cos", "sin"]
    for name in extra:  # optional inputs 10.. (slot_mapping, head_sink, ...)
        while len(ins) < 10:
            ins.append("")
        g.input(name, INT32, [-1])
        ins.append(name)
    g.output("out", dtype, [-1, H * D])
    attrs = dict(num_heads=H, kv_num_heads=KV, do_rotary=do_rotary)
    if layout:
        attrs["kv_cache_layout"] = layout
    if rotary_offset:
        attrs["rotary_offset"] = rotary_offset
    if local_window is not None:
        attrs["local_window_size"] = local_window
    g.node("PagedAttention", ins, ["out"], domain="com.microsoft", **attrs)
    return g


@pytest.mark.parametrize("kw", [dict(), dict(do_rotary=0), dict(H=8, KV=8, D=32), dict(H=32, KV=8, D=128)])
def test_paged_attention_claims(kw):
    _, groups, _ = claimed(paged_graph(**kw))
    assert groups == [0]


@pytest.mark.parametrize("kw,reason", [
    (dict(dtype=FLOAT), "fp16/bf16"),
    (dict(D=16), "head_size 16"),
    (dict(layout="LATENT"), "SEPARATE"),
    (dict(extra=("slot_mapping",)), "slot_mapping"),
    (dict(rotary_offset=8), "rotary_offset"),
    (dict(local_window=16), "local_window_size"),
    (dict(cos_dtype=FLOAT), "cos_cache/sin_cache"),
])
def test_paged_attention_declines_with_reason(kw, reason):
    ep, groups, _ = claimed(paged_graph(**kw))
    assert groups == [-1]
    assert reason in ep.claim_reason(0)


def test_mask_glue_decoder_claimed_whole():
    """A GenAI-style decoder (attention_mask in, seqlens_k / total_sequence_length derived in the
    graph by ReduceSum / Sub / Cast and Shape / Gather / Cast) is claimed as one partition."""
    from onnxruntime_ep_b200.decoder import DecoderConfig, build_decoder

    cfg = DecoderConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000, max_seq=256)
    g = build_decoder(cfg, batch=2, seq=1, cap=64, mask_glue=True)
    _, groups, num = claimed(g)
    assert num == 1 and set(groups) == {0}
    assert {"mask_sum", "mask_past", "seqlens_k", "mask_shape", "mask_width", "total_sequence_length"} <= set(g.node_names)


def _glue_graph(op, data_dtype, data_shape, out_dtype, out_shape, extra=None, **attrs):
    g = GraphBuilder()
    g.input("x", data_dtype, data_shape)
    ins = ["x"]
    for name, arr in (extra or []):
        g.initializer(name, arr)
        ins.append(name)
    g.output("y", out_dtype, out_shape)
    g.node(op, ins, ["y"], **attrs)
    return g


@pytest.mark.parametrize("op,args,attrs", [
    ("Shape", (INT64, [2, -1], INT64, [2], None), {}),
    ("Shape", (FLOAT16, [2, 3, 4], INT64, [1], None), dict(start=-1)),
    ("Gather", (INT64, [4], INT64, [], [("i", np.array(1, np.int64))]), dict(axis=0)),
    ("Gather", (INT64, [4], INT64, [2], [("i", np.array([0, -1], np.int64))]), {}),
    ("ReduceSum", (INT64, [2, -1], INT64, [2], [("a", np.array([1], np.int64))]), dict(keepdims=0)),
    ("ReduceSum", (INT32, [2, 5], INT32, [2, 1], [("a", np.array([-1], np.int64))]), {}),
    ("Unsqueeze", (INT64, [2], INT64, [1, 2], [("a", np.array([0], np.int64))]), {}),
    ("Squeeze", (INT64, [1, 2], INT64, [2], [("a", np.array([0], np.int64))]), {}),
    ("Reshape", (INT32, [2, 3], INT32, [6], [("s", np.array([-1], np.int64))]), {}),
    ("Cast", (INT64, [2], INT32, [2], None), dict(to=INT32)),
    ("Sub", (INT64, [2], INT64, [2], [("b", np.array(1, np.int64))]), {}),
])
def test_integer_glue_claims(op, args, attrs):
    g = _glue_graph(op, *args, **attrs)
    ep, groups, num = claimed(g)
    assert groups == [0] and num == 1, ep.claim_reason(0)


@pytest.mark.parametrize("op,args,attrs,reason", [
    ("Gather", (FLOAT, [4, 8], FLOAT, [8], [("i", np.array(1, np.int64))]), dict(axis=0), "1-D int32 / int64"),
    ("ReduceSum", (INT64, [2, 5], INT64, [5], [("a", np.array([0], np.int64))]), dict(keepdims=0), "last axis"),
    ("ReduceSum", (FLOAT, [2, 5], FLOAT, [2], [("a", np.array([1], np.int64))]), dict(keepdims=0), "int32 / int64"),
    ("Cast", (INT64, [2], FLOAT, [2], None), dict(to=FLOAT), "casts are claimed"),
    ("Reshape", (INT32, [2, 3], INT32, [6], [("s", np.array([-1, -1], np.int64))]), {}, "at most one -1"),
    ("Unsqueeze", (FLOAT, [2], FLOAT, [1, 2], [("a", np.array([0], np.int64))]), {}, "int32 / int64"),
])
def test_integer_glue_declines_with_reason(op, args, attrs, reason):
    g = _glue_graph(op, *args, **attrs)
    ep, groups, num = claimed(g)
    assert groups == [-1] and num == 0
    assert reason in ep.claim_reason(0)


def test_gather_with_runtime_indices_declined():
    g = GraphBuilder()
    g.input("x", INT64, [4])
    g.input("i", INT64, [])
    g.output("y", INT64, [])
    g.node("Gather", ["x", "i"], ["y"], axis=0)
    ep, groups, _ = claimed(g)
    assert groups == [-1] and "constant" in ep.claim_reason(0)
