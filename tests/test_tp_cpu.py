"""Tensor-parallel sharding on the host (no GPU): the plan of every rank, previewed through
b200ep_tp_shard_preview, must slice each MatMulNBits exactly as the sharding scheme says —
q/k/v and gate/up by output rows (attention by KV head), o_proj and down_proj by K blocks followed
by an all-reduce, the vocabulary projection by rows followed by an all-gather — and every rank
must issue the same collectives in the same order (checked across gloo ranks)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from onnxruntime_ep_b200 import ep as E
from onnxruntime_ep_b200.decoder import DecoderConfig, build_decoder

CFG = dict(layers=2, hidden=256, heads=8, kv_heads=4, head_dim=32, ffn=512, vocab=1000, max_seq=64)


def fnv(b: bytes) -> str:
    h = 1469598103934665603
    for c in b:
        h = ((h ^ c) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return format(h, "x")


def rows(a, n):
    return np.asarray(a).reshape(n, -1)


def take_rows(W, prefix, n, ranges):
    out = {}
    for key in ("B", "scales", "zp"):
        full = rows(W[f"{prefix}.{key}"], n)
        out[key] = np.concatenate([full[a:b] for a, b in ranges], axis=0)
    return out


def cat_rows(parts):
    return {k: np.concatenate([p[k] for p in parts], axis=0) for k in parts[0]}


def take_blocks(W, prefix, n, nblocks, b0, b1):
    B = np.asarray(W[f"{prefix}.B"]).reshape(n, nblocks, -1)[:, b0:b1]
    S = rows(W[f"{prefix}.scales"], n)[:, b0:b1]
    zp = rows(W[f"{prefix}.zp"], n)
    nib = np.empty((n, zp.shape[1] * 2), np.uint8)
    nib[:, 0::2], nib[:, 1::2] = zp & 0x0F, zp >> 4
    sel = nib[:, b0:b1]
    if sel.shape[1] % 2:
        sel = np.concatenate([sel, np.zeros((n, 1), np.uint8)], axis=1)
    Z = (sel[:, 0::2] | (sel[:, 1::2] << 4)).astype(np.uint8)
    return {"B": B, "scales": S, "zp": Z}


def expected_mnb(cfg, W, rank, world):
    """Expected per-rank weights of every MatMulNBits step, in plan order per layer."""
    H, HK, D, hid, F, V, blk = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.ffn, cfg.vocab, cfg.block
    hq, hk, f = H // world, HK // world, F // world
    exp = []
    for i in range(cfg.layers):
        p = f"l{i}"
        qkv = cat_rows([take_rows(W, f"{p}.q_proj", H * D, [(rank * hq * D, (rank + 1) * hq * D)]),
                        take_rows(W, f"{p}.k_proj", HK * D, [(rank * hk * D, (rank + 1) * hk * D)]),
                        take_rows(W, f"{p}.v_proj", HK * D, [(rank * hk * D, (rank + 1) * hk * D)])])
        exp.append(((hq + 2 * hk) * D, hid, qkv))
        nbo = H * D // blk
        exp.append((hid, hq * D, take_blocks(W, f"{p}.o_proj", hid, nbo, rank * hq * D // blk,
                                             (rank + 1) * hq * D // blk)))
        gu = cat_rows([take_rows(W, f"{p}.gate_proj", F, [(rank * f, (rank + 1) * f)]),
                       take_rows(W, f"{p}.up_proj", F, [(rank * f, (rank + 1) * f)])])
        exp.append((2 * f, hid, gu))
        exp.append((hid, f, take_blocks(W, f"{p}.down_proj", hid, F // blk, rank * f // blk, (rank + 1) * f // blk)))
    v = V // world
    exp.append((v, hid, take_rows(W, "lm_head", V, [(rank * v, (rank + 1) * v)])))
    return exp


@pytest.mark.parametrize("world", [2, 4])
def test_tp_preview_slices_match_numpy(world):
    cfg = DecoderConfig(**CFG)
    W = {}
    g = build_decoder(cfg, batch=1, seq=1, cap=16, weights_out=W)
    for rank in range(world):
        steps = E.tp_shard_preview(g, rank, world)
        mnb = [s for s in steps if s["op"] == "MatMulNBits"]
        exp = expected_mnb(cfg, W, rank, world)
        assert len(mnb) == len(exp)
        for s, (n, k, arrs) in zip(mnb, exp):
            assert (s["N"], s["K"]) == (n, k), s["name"]
            for key in ("B", "scales", "zp"):
                assert s[key] == fnv(np.ascontiguousarray(arrs[key]).tobytes()), (s["name"], key)
        heads = {(s["heads"], s["kv_heads"]) for s in steps if s["op"] == "GroupQueryAttention"}
        assert heads == {(cfg.heads // world, cfg.kv_heads // world)}
        ops = [s["op"] for s in steps]
        # one all-reduce after each row-parallel projection, one all-gather of the logits
        assert ops.count("AllReduce") == 2 * cfg.layers and ops.count("AllGather") == 1
        for i, op in enumerate(ops):
            if op == "AllReduce":
                assert ops[i - 1] == "MatMulNBits"
        assert ops[-1] == "AllGather" and ops[-2] == "MatMulNBits"


def test_tp_preview_world1_is_unsharded():
    cfg = DecoderConfig(**CFG)
    g = build_decoder(cfg, batch=1, seq=1, cap=16)
    ops = [s["op"] for s in E.tp_shard_preview(g, 0, 1)]
    assert "AllReduce" not in ops and "AllGather" not in ops


def test_tp_rejects_heads_that_do_not_divide():
    cfg = DecoderConfig(**dict(CFG, heads=6, kv_heads=3, head_dim=32))
    g = build_decoder(cfg, batch=1, seq=1, cap=16)
    with pytest.raises(Exception, match="do not divide"):
        E.tp_shard_preview(g, 0, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = DecoderConfig(**CFG)
        g = build_decoder(cfg, batch=1, seq=1, cap=16)
        steps = E.tp_shard_preview(g, rank, world)
        coll = [(s["op"], s["name"]) for s in steps if s["op"] in ("AllReduce", "AllGather")]
        cols = [(s["name"], s["N"]) for s in steps if s["op"] == "MatMulNBits"]
        gathered = [None] * world
        dist.all_gather_object(gathered, {"coll": coll, "cols": cols})
        ok = all(x["coll"] == gathered[0]["coll"] for x in gathered)
        # the per-rank output widths of the vocabulary projection add up to the vocabulary
        vocab = sum(dict(x["cols"])["lm_head"] for x in gathered)
        q.put((rank, ok, vocab))
    finally:
        dist.destroy_process_group()


def test_tp_gloo_ranks_issue_identical_collectives():
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res)
    assert all(v == CFG["vocab"] for _, _, v in res)
