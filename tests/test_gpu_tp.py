"""Tensor-parallel decoder on 2 GPUs (one process per GPU): prefill then decode steps of a small
decoder sharded by KV head / FFN column / vocabulary, checked against the CPU oracle run of the
unsharded graph.  The prefill's 32-row partial sums go through NCCL all-reduces; the decode steps'
through the peer-memory mailboxes fused into the GEMVs.  Skipped with fewer than 2 GPUs."""

from __future__ import annotations

import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFGS = {
    # prefill: 32 rows (NCCL all-reduce); decode: 2 rows (peer mailboxes)
    "small": (dict(layers=2, hidden=256, heads=8, kv_heads=4, head_dim=32, ffn=512, vocab=1000, max_seq=64), 2),
    # two Llama-3-70B-shaped layers (hidden 8192, 64 / 8 heads, FFN 28672) at batch 1: 8192-wide norm
    # prologues over the mailbox sums, 8 query heads per local kv head
    "70b-layers": (dict(layers=2, hidden=8192, heads=64, kv_heads=8, head_dim=128, ffn=28672, vocab=512,
                        max_seq=64), 1),
}
P, CAP, STEPS = 16, 32, 3


def _gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:  # noqa: BLE001
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, shape, tp_attention):
    import datetime

    import torch
    import torch.distributed as dist

    from onnxruntime_ep_b200 import ep as E
    from onnxruntime_ep_b200.decoder import DecoderConfig, build_decoder

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    sess_p = sess_d = None
    CFG, B = CFGS[shape]
    try:
        obj = [E.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        cfg = DecoderConfig(**CFG)
        ep_p = E.ExecutionProvider(device_id=rank, tp_attention=tp_attention)
        ep_p.set_tensor_parallel(rank, world, obj[0])
        sess_p = E.Session(build_decoder(cfg, batch=B, seq=P, cap=CAP), ep_p)
        ep_d = E.ExecutionProvider(device_id=rank, tp_attention=tp_attention)
        obj2 = [E.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj2, src=0)
        ep_d.set_tensor_parallel(rank, world, obj2[0])
        sess_d = E.Session(build_decoder(cfg, batch=B, seq=1, cap=CAP), ep_d)
        import json

        desc = json.loads(sess_d.parts[0].describe())
        hk = cfg.kv_heads // world if tp_attention == "sharded" else cfg.kv_heads
        kv = [[torch.zeros(B, hk, CAP, cfg.head_dim, dtype=torch.float16, device="cuda") for _ in range(2)]
              for _ in range(cfg.layers)]
        rng = np.random.default_rng(7)
        logits = []

        def feeds(ids, past):
            f = {"input_ids": torch.from_numpy(ids).cuda(),
                 "seqlens_k": torch.full((B,), past + ids.shape[1] - 1, dtype=torch.int32, device="cuda"),
                 "total_sequence_length": torch.tensor([past + ids.shape[1]], dtype=torch.int32, device="cuda")}
            o = {}
            for i in range(cfg.layers):
                f[f"past_key_values.{i}.key"], f[f"past_key_values.{i}.value"] = kv[i]
                o[f"present.{i}.key"], o[f"present.{i}.value"] = kv[i]
            return f, o

        ids_all = [rng.integers(0, cfg.vocab, size=(B, P), dtype=np.int64)]
        ids_all += [rng.integers(0, cfg.vocab, size=(B, 1), dtype=np.int64) for _ in range(STEPS)]
        f, o = feeds(ids_all[0], 0)
        logits.append(sess_p.run(f, o)["logits"].float().cpu().numpy())
        for t in range(STEPS):
            f, o = feeds(ids_all[t + 1], P + t)
            logits.append(sess_d.run(f, o)["logits"].float().cpu().numpy())
        torch.cuda.synchronize()
        sites = (2 if tp_attention == "sharded" else 1) * cfg.layers
        q.put((rank, logits, ids_all, None if desc["peer_allreduce"] == sites
               else f"peer_allreduce sites {desc['peer_allreduce']}"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, None, None, repr(e)))
    finally:
        del sess_p, sess_d  # release the CUDA graphs holding NCCL calls before the teardown
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shape,tp_attention", [("small", "sharded"), ("70b-layers", "sharded"),
                                                ("small", "replicated"), ("70b-layers", "replicated")])
def test_tp2_decoder_matches_oracle(shape, tp_attention):
    """Two ranks against the oracle of the unsharded graph.  tp_attention = "replicated" runs attention
    in full on every rank (one all-reduce per layer, after the FFN)."""
    import torch.multiprocessing as mp

    from oracle import oracle  # noqa: F401  (builds the C oracle)
    from onnxruntime_ep_b200.decoder import DecoderConfig, build_decoder
    from test_gpu_ep import _compare_logits, oracle_decoder_step

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, shape, tp_attention)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
    for r, _, _, err in res:
        assert err is None, f"rank {r}: {err}"
    # every rank holds the full (all-gathered) logits
    for step in range(STEPS + 1):
        np.testing.assert_array_equal(res[0][1][step], res[1][1][step])
    CFG, B = CFGS[shape]
    cfg = DecoderConfig(**CFG)
    ids_all = res[0][2]
    Wp, Wd = {}, {}
    build_decoder(cfg, batch=B, seq=P, cap=CAP, weights_out=Wp)
    build_decoder(cfg, batch=B, seq=1, cap=CAP, weights_out=Wd)
    kv_ref = [[np.zeros((B, cfg.kv_heads, CAP, cfg.head_dim), np.float16) for _ in range(2)]
              for _ in range(cfg.layers)]
    want = oracle_decoder_step(cfg, Wp, ids_all[0], kv_ref, np.full(B, P - 1, np.int32)).astype(np.float32)
    _compare_logits(res[0][1][0], want, "prefill")
    for t in range(STEPS):
        want = oracle_decoder_step(cfg, Wd, ids_all[t + 1], kv_ref, np.full(B, P + t, np.int32)).astype(np.float32)
        _compare_logits(res[0][1][t + 1], want, f"decode step {t}")
