"""Llama-shaped int4 decoder graphs, in the node layout ONNX Runtime GenAI exporters emit for
q4 decoders: GatherBlockQuantized embedding; per layer SimplifiedLayerNormalization /
SkipSimplifiedLayerNormalization, three MatMulNBits projections, GroupQueryAttention with
in-op rotary over shared past/present KV buffers, o projection, a SwiGLU FFN written as
Sigmoid/Mul/Mul around gate/up MatMulNBits, and a MatMulNBits lm_head.  Weights are random
(seeded), int4 block-quantised with fp16/fp32 scales and uint8 zero points.

Used by the benchmark and the tests to drive the EP the way an exported decoder does.
"""

from __future__ import annotations

import dataclasses

import numpy as np

from .ep import FLOAT, FLOAT16, INT32, INT64, GraphBuilder


@dataclasses.dataclass
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    block: int = 32
    eps: float = 1e-5
    rope_base: float = 10000.0
    max_seq: int = 4096
    dtype: str = "float16"
    seed: int = 0

    @property
    def np_dtype(self):
        return np.float16 if self.dtype == "float16" else np.float32

    @property
    def code(self):
        return FLOAT16 if self.dtype == "float16" else FLOAT


LLAMA3_8B = DecoderConfig()
LLAMA3_70B = DecoderConfig(layers=80, hidden=8192, heads=64, kv_heads=8, ffn=28672)


def quantize_params(rng, n, k, block, np_dtype, zp=True):
    """Random int4 MatMulNBits initializers: packed B [n, nblocks, block/2], scales, zero points.
    Scales ~ U(0.5, 1.5) / (8 sqrt(k)) keep activations O(1) through deep stacks."""
    nblocks = (k + block - 1) // block
    b = np.frombuffer(rng.bytes(n * nblocks * block // 2), dtype=np.uint8).reshape(n, nblocks, block // 2)
    scales = (rng.uniform(0.5, 1.5, size=n * nblocks) / (8.0 * np.sqrt(k))).astype(np_dtype)
    zps = np.frombuffer(rng.bytes(n * ((nblocks + 1) // 2)), dtype=np.uint8).copy() if zp else None
    return b, scales, zps


def rotary_caches(max_seq, rotary_dim, base, np_dtype):
    half = rotary_dim // 2
    inv = 1.0 / (base ** (np.arange(0, half, dtype=np.float64) / half))
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np_dtype), np.sin(ang).astype(np_dtype)


def build_decoder(cfg: DecoderConfig, *, batch: int, seq: int, cap: int, with_lm_head: bool = True,
                  weights_out: dict | None = None, mask_glue: bool = False) -> GraphBuilder:
    """One graph for a [batch, seq] step over KV buffers of capacity `cap`.

    Inputs: input_ids int64 [B, S], seqlens_k int32 [B], total_sequence_length int32 [1],
    past_key_values.{i}.key / .value [B, kv_heads, cap, head_dim].
    Outputs: logits [B, S, vocab] (or the final hidden state), present.{i}.key / .value.
    ``weights_out`` (optional) receives every initializer, for oracle cross-checks.
    ``mask_glue``: take attention_mask int64 [B, past + S] instead of seqlens_k /
    total_sequence_length and derive both in the graph the way GenAI-exported decoders do:
    seqlens_k = Cast(Sub(ReduceSum(mask, axes=[1]), 1)), total = Cast(Gather(Shape(mask), 1)).
    The weights are drawn identically, so both forms compute the same logits.
    """
    rng = np.random.default_rng(cfg.seed)
    dt, code = cfg.np_dtype, cfg.code
    H, HK, D, hid = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden
    g = GraphBuilder()

    def init(name, arr, dtype=None):
        if weights_out is not None:
            weights_out[name] = arr
        return g.initializer(name, arr, dtype)

    def mnb(x, out, n, k, prefix, out_shape):
        b, s, z = quantize_params(rng, n, k, cfg.block, dt)
        init(prefix + ".B", b)
        init(prefix + ".scales", s)
        init(prefix + ".zp", z)
        g.tensor(out, code, out_shape)
        g.node("MatMulNBits", [x, prefix + ".B", prefix + ".scales", prefix + ".zp"], [out],
               domain="com.microsoft", name=prefix, K=k, N=n, bits=4, block_size=cfg.block)
        return out

    g.input("input_ids", INT64, [batch, seq])
    if mask_glue:
        g.input("attention_mask", INT64, [batch, -1])
        g.initializer("mask_axes", np.array([1], np.int64))
        g.initializer("one_i64", np.array(1, np.int64))
        g.initializer("mask_len_axis", np.array(1, np.int64))
        g.tensor("mask_sum", INT64, [batch])
        g.node("ReduceSum", ["attention_mask", "mask_axes"], ["mask_sum"], name="mask_sum", keepdims=0)
        g.tensor("mask_past", INT64, [batch])
        g.node("Sub", ["mask_sum", "one_i64"], ["mask_past"], name="mask_past")
        g.tensor("seqlens_k", INT32, [batch])
        g.node("Cast", ["mask_past"], ["seqlens_k"], name="seqlens_k", to=INT32)
        g.tensor("mask_shape", INT64, [2])
        g.node("Shape", ["attention_mask"], ["mask_shape"], name="mask_shape")
        g.tensor("mask_width", INT64, [])
        g.node("Gather", ["mask_shape", "mask_len_axis"], ["mask_width"], name="mask_width", axis=0)
        g.tensor("total_sequence_length", INT32, [])
        g.node("Cast", ["mask_width"], ["total_sequence_length"], name="total_sequence_length", to=INT32)
    else:
        g.input("seqlens_k", INT32, [batch])
        g.input("total_sequence_length", INT32, [1])
    cos, sin = rotary_caches(cfg.max_seq, D, cfg.rope_base, dt)
    init("cos_cache", cos)
    init("sin_cache", sin)

    # embedding: int4 GatherBlockQuantized (symmetric, block 32)
    nb = hid // cfg.block
    emb = np.frombuffer(rng.bytes(cfg.vocab * hid // 2), dtype=np.uint8).reshape(cfg.vocab, hid // 2)
    emb_s = rng.uniform(0.02, 0.06, size=(cfg.vocab, nb)).astype(dt)
    init("embed.q", emb)
    init("embed.scales", emb_s)
    g.tensor("x0", code, [batch, seq, hid])
    g.node("GatherBlockQuantized", ["embed.q", "input_ids", "embed.scales"], ["x0"], domain="com.microsoft",
           name="embed", bits=4, block_size=cfg.block, gather_axis=0, quantize_axis=1)

    act = [batch, seq]
    residual_in, x_in = None, "x0"
    for i in range(cfg.layers):
        p = f"l{i}"
        ln1 = init(f"{p}.ln1", rng.uniform(0.8, 1.2, hid).astype(dt))
        n1 = g.tensor(f"{p}.n1", code, act + [hid])
        if residual_in is None:
            g.node("SimplifiedLayerNormalization", [x_in, ln1], [n1], domain="", name=f"{p}.norm1", epsilon=cfg.eps,
                   axis=-1)
            res1 = x_in
        else:
            res1 = g.tensor(f"{p}.res1", code, act + [hid])
            g.node("SkipSimplifiedLayerNormalization", [x_in, residual_in, ln1], [n1, "", "", res1],
                   domain="com.microsoft", name=f"{p}.norm1", epsilon=cfg.eps)
        q = mnb(n1, f"{p}.q", H * D, hid, f"{p}.q_proj", act + [H * D])
        k = mnb(n1, f"{p}.k", HK * D, hid, f"{p}.k_proj", act + [HK * D])
        v = mnb(n1, f"{p}.v", HK * D, hid, f"{p}.v_proj", act + [HK * D])
        pk = g.input(f"past_key_values.{i}.key", code, [batch, HK, cap, D])
        pv = g.input(f"past_key_values.{i}.value", code, [batch, HK, cap, D])
        ok = g.output(f"present.{i}.key", code, [batch, HK, cap, D])
        ov = g.output(f"present.{i}.value", code, [batch, HK, cap, D])
        attn = g.tensor(f"{p}.attn", code, act + [H * D])
        g.node("GroupQueryAttention", [q, k, v, pk, pv, "seqlens_k", "total_sequence_length", "cos_cache", "sin_cache"],
               [attn, ok, ov], domain="com.microsoft", name=f"{p}.attn", num_heads=H, kv_num_heads=HK,
               do_rotary=1, rotary_interleaved=0, scale=float(1.0 / np.sqrt(D)))
        o = mnb(attn, f"{p}.o", hid, H * D, f"{p}.o_proj", act + [hid])
        ln2 = init(f"{p}.ln2", rng.uniform(0.8, 1.2, hid).astype(dt))
        n2 = g.tensor(f"{p}.n2", code, act + [hid])
        res2 = g.tensor(f"{p}.res2", code, act + [hid])
        g.node("SkipSimplifiedLayerNormalization", [o, res1, ln2], [n2, "", "", res2], domain="com.microsoft",
               name=f"{p}.norm2", epsilon=cfg.eps)
        gate = mnb(n2, f"{p}.gate", cfg.ffn, hid, f"{p}.gate_proj", act + [cfg.ffn])
        up = mnb(n2, f"{p}.up", cfg.ffn, hid, f"{p}.up_proj", act + [cfg.ffn])
        sg = g.tensor(f"{p}.sig", code, act + [cfg.ffn])
        g.node("Sigmoid", [gate], [sg], name=f"{p}.sigmoid")
        silu = g.tensor(f"{p}.silu", code, act + [cfg.ffn])
        g.node("Mul", [gate, sg], [silu], name=f"{p}.silu")
        h = g.tensor(f"{p}.h", code, act + [cfg.ffn])
        g.node("Mul", [silu, up], [h], name=f"{p}.swiglu")
        down = mnb(h, f"{p}.down", hid, cfg.ffn, f"{p}.down_proj", act + [hid])
        residual_in, x_in = res2, down

    lnf = init("final_norm", rng.uniform(0.8, 1.2, hid).astype(dt))
    nf = g.tensor("final_hidden", code, act + [hid])
    resf = g.tensor("final_residual", code, act + [hid])
    g.node("SkipSimplifiedLayerNormalization", [x_in, residual_in, lnf], [nf, "", "", resf],
           domain="com.microsoft", name="final_norm", epsilon=cfg.eps)
    if with_lm_head:
        mnb(nf, "logits", cfg.vocab, hid, "lm_head", act + [cfg.vocab])
        g.output("logits", code, act + [cfg.vocab])
    else:
        g.output("final_hidden", code, act + [hid])
    return g
