"""Benchmark: Llama-3-8B-shaped int4 decode tokens/s through the B200 EP.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload (single GPU): 32 layers, hidden 4096, 32/8 heads, head 128, FFN 14336,
vocab 128256, every projection MatMulNBits int4 block 32 with fp16 scales and uint8 zero points,
random-init weights (seed 0), int4 GatherBlockQuantized embedding, prompt of 1024 random token
ids prefilled through the same EP graph (untimed), then decode steps.  One step = one decode
token for every sequence of the batch: the whole graph runs as one compiled partition (a CUDA
graph replay) whose positions advance from device-side seqlens_k.

Reported: `value` = decode tokens/s with inputs resident in HBM (CUDA events, max over ranks);
`e2e` = the same through the compiled partition's C ABI with host buffers (token ids and
sequence lengths staged host->device, logits read back every step); `roofline` = the dominant
kernel (the fused gate/up MatMulNBits GEMV) timed live with CUDA events on a weight set larger
than L2; `cpu_baseline` = the C oracle timed on the host cores for one decoder layer + lm_head
and extrapolated to 32 layers.  --impl reference times that CPU oracle path alone (the
reference implementation — Rust over MLX/Metal — cannot run on Linux; ORT's CPU EP is not
installable here).

Multi-GPU: one process per GPU under torchrun, one model sharded over the ranks (tensor
parallel, strong scaling): q/k/v, gate/up and the vocabulary projection split by output rows
(attention by KV head), o_proj / down_proj split by K blocks and followed by an NCCL all-reduce,
the logits all-gathered; every rank decodes the same tokens; value = tokens / max rank time.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "onnxruntime-mlx_b200"))
sys.path.insert(0, ROOT)

PROMPT = 1024
GEN = 256
HBM_FALLBACK = 6553.0
TENSOR_FALLBACK = 1590.0


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": HBM_FALLBACK, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed region runs: NVML every
    10 ms (read-only queries), else nvidia-smi every 200 ms."""

    NAMES = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []  # (sm_mhz, max_mhz, reason_names)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None

    def _handle(self):
        import pynvml  # nvidia_ml_py

        pynvml.nvmlInit()
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:  # noqa: BLE001
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _run(self):
        try:
            nv, h = self._handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self._stop.is_set():
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = get_reasons(h)
                self.samples.append((float(sm), float(mx), [n for b, n in self.NAMES.items() if bits & b]))
                self._stop.wait(0.01)
            return
        except Exception:  # noqa: BLE001
            pass
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={fields}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                p = [x.strip() for x in out.stdout.strip().split(",")]
                if len(p) >= 6:
                    self.samples.append((float(p[0]), float(p[1]),
                                         [names[i] for i in range(4) if "Active" in p[2 + i] and "Not" not in p[2 + i]]))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": sorted({n for s in self.samples for n in s[2]}), "samples": len(self.samples)}


def dist_setup(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- the CPU baseline (oracle port) --------------------------------------------------------
def cpu_layer_sample(cfg, batch, ctx, threads=0):
    """One decoder layer + lm_head of a decode step on the C oracle; returns (seconds, desc)."""
    import numpy as np

    from oracle import oracle
    from onnxruntime_ep_b200.decoder import quantize_params, rotary_caches

    rng = np.random.default_rng(1)
    dt = np.float16
    hid, H, HK, D = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
    W = {}
    for name, n, k in (("q", H * D, hid), ("k", HK * D, hid), ("v", HK * D, hid), ("o", hid, H * D),
                       ("gate", cfg.ffn, hid), ("up", cfg.ffn, hid), ("down", hid, cfg.ffn),
                       ("lm", cfg.vocab, hid)):
        W[name] = (quantize_params(rng, n, k, cfg.block, dt), n, k)
    x = rng.standard_normal((batch, 1, hid)).astype(dt)
    g = rng.uniform(0.8, 1.2, hid).astype(dt)
    cap = ctx + 8
    kc = rng.standard_normal((batch, HK, cap, D)).astype(dt)
    vc = rng.standard_normal((batch, HK, cap, D)).astype(dt)
    cos, sin = rotary_caches(cap + 8, D, 10000.0, dt)
    seq = np.full(batch, ctx, np.int32)

    def mnb(a, key):
        (b, s, z), n, k = W[key]
        return oracle.matmulnbits(a, b, s, z, N=n, K=k, threads=threads)

    t0 = time.perf_counter()
    n1 = oracle.rms_norm(x, g, 1e-5, threads=threads)
    q, k, v = mnb(n1, "q"), mnb(n1, "k"), mnb(n1, "v")
    attn, _, _ = oracle.gqa(q, k, v, kc, vc, seq, cos, sin, num_heads=H, kv_heads=HK, shared_buffer=True,
                            threads=threads)
    o = mnb(attn, "o")
    n2, r2 = oracle.skip_rms_norm(o, x, g, 1e-5, threads=threads)
    ga, up = mnb(n2, "gate").astype(np.float32), mnb(n2, "up").astype(np.float32)
    h = (ga / (1 + np.exp(-ga)) * up).astype(dt)
    mnb(h, "down")
    t_layer = time.perf_counter() - t0
    t0 = time.perf_counter()
    mnb(n2, "lm")
    t_lm = time.perf_counter() - t0
    return t_layer, t_lm


def cpu_baseline(cfg, batch, samples=2):
    from oracle import oracle

    oracle.build()
    cores = oracle.max_threads()
    cpu_layer_sample(cfg, batch, PROMPT)  # warm (page in, thread pool)
    best = None
    for _ in range(samples):
        tl, tlm = cpu_layer_sample(cfg, batch, PROMPT)
        step = cfg.layers * tl + tlm
        best = step if best is None else min(best, step)
    return {"value": batch / best, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"C oracle, 1 decoder layer + lm_head of a B={batch} decode step at context {PROMPT}, "
                      f"extrapolated to {cfg.layers} layers (best of {samples}); ORT CPU EP unavailable here"}


# ---- the GPU arm ---------------------------------------------------------------------------
def dominant_kernel_roofline(batch, peaks, peak_kind, reps=10):
    """Live CUDA-event timing of the dominant decode kernel — the fused gate/up int4 GEMV (N = 2 x
    14336, K = 4096, block 32, fp16 scales + uint8 zero points) on the tensor-core path the plan
    uses (weights prepacked into group records) — over rotating weight copies larger than L2,
    replayed from a CUDA graph on the stream the kernels run on."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    K, N, block = 4096, 2 * 14336, 32
    nb = K // block
    per = N * nb * block // 2 + N * nb * 2 + N * nb // 2  # ORT-layout bytes of one weight set
    copies = max(3, int(np.ceil(3 * 126e6 / per)))
    g = torch.Generator(device="cuda").manual_seed(0)
    packs = []
    for _ in range(copies):
        Bq = torch.randint(0, 256, (N, nb, block // 2), dtype=torch.uint8, device="cuda", generator=g)
        S = (torch.rand(N * nb, device="cuda", generator=g) * 0.01 + 0.001).half()
        Z = torch.randint(0, 256, (N * nb // 2,), dtype=torch.uint8, device="cuda", generator=g)
        packs.append(ops.matmulnbits_prepack(Bq, S, Z, K=K, N=N, block_size=block))
        del Bq, S, Z
    a = torch.randn(batch, K, device="cuda").half()
    y = torch.empty(batch, N, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(copies):
            ops.matmulnbits_prepacked(a, packs[i], K=K, N=N, out=y)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                ops.matmulnbits_prepacked(a, packs[i], K=K, N=N, out=y)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    alg = per + a.numel() * 2 + y.numel() * 2
    achieved = alg / launch_s / 1e9
    peak = float(peaks.get("hbm_gbs", HBM_FALLBACK))
    traffic = None
    summ = os.path.join(ROOT, "profiles", "mnb_tma_kernel_gate_up_m1.md")
    if os.path.exists(summ):
        for line in open(summ):
            if line.startswith("dram_bytes_per_launch:"):
                traffic = int(float(line.split(":")[1]))
    return {"kernel": "mnb_tma_kernel (fused gate/up: N=28672, K=4096, int4 b32, fp16, prepacked records)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs (of {peak_kind})",
            "algorithmic_bytes_per_launch": alg, "launch_us": round(launch_s * 1e6, 2), "traffic": traffic}


def gqa_kernel_timing(batch, ctx, peaks, peak_kind, reps=5):
    """GroupQueryAttention decode alone (32 q / 8 kv heads, head 128, fp16, shared KV buffer of
    capacity ctx + 16 holding ctx valid rows): CUDA-event timing over rotating KV buffers larger than
    L2, replayed from a CUDA graph.  Algorithmic bytes: the K and V rows read plus q / k / v / out."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    H, HK, D = 32, 8, 128
    cap = ctx + 16
    per = 2 * batch * HK * cap * D * 2
    copies = max(2, int(np.ceil(3 * 126e6 / per)))
    g = torch.Generator(device="cuda").manual_seed(0)
    kvs = [(torch.randn(batch, HK, cap, D, device="cuda", generator=g).half(),
            torch.randn(batch, HK, cap, D, device="cuda", generator=g).half()) for _ in range(copies)]
    q = torch.randn(batch, 1, H * D, device="cuda", generator=g).half()
    k = torch.randn(batch, 1, HK * D, device="cuda", generator=g).half()
    v = torch.randn(batch, 1, HK * D, device="cuda", generator=g).half()
    seq = torch.full((batch,), ctx - 1, dtype=torch.int32, device="cuda")
    ang = torch.arange(cap + 8, device="cuda", dtype=torch.float64)[:, None] / (
        10000.0 ** (torch.arange(D // 2, device="cuda", dtype=torch.float64) / (D // 2)))[None, :]
    cos, sin = ang.cos().half(), ang.sin().half()
    out = torch.empty(batch, 1, H * D, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(copies):
            ops.group_query_attention(q, k, v, kvs[i][0], kvs[i][1], seq, cos, sin, num_heads=H, kv_heads=HK, out=out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                ops.group_query_attention(q, k, v, kvs[i][0], kvs[i][1], seq, cos, sin, num_heads=H, kv_heads=HK,
                                          out=out)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    alg = 2 * batch * HK * ctx * D * 2 + (q.numel() + k.numel() + v.numel() + out.numel()) * 2
    peak = float(peaks.get("hbm_gbs", HBM_FALLBACK))
    return {"kernel": "gqa_mma_decode_kernel", "batch": batch, "context": ctx, "launch_us": round(launch_s * 1e6, 2),
            "algorithmic_bytes_per_launch": alg, "achieved": round(alg / launch_s / 1e9, 1), "unit": "GB/s",
            "frac": round(alg / launch_s / 1e9 / peak, 4), "peak": peak, "peak_source": f"{peak_kind} hbm_gbs"}


def paged_kernel_timing(batch, ctx, peaks, peak_kind, reps=5, block=16):
    """PagedAttention decode alone (32 q / 8 kv heads, head 128, fp16, 16-row blocks scattered by a
    random block table): each sequence appends one token after ctx - 1 cached ones.  CUDA-event
    timing of the append + attention launches over rotating cache pairs larger than L2, replayed
    from a CUDA graph.  Algorithmic bytes: the K and V rows read plus q / k / v / out."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    H, HK, D = 32, 8, 128
    nblk = (ctx + block - 1) // block
    nb = batch * nblk
    per = 2 * nb * block * HK * D * 2
    copies = max(2, int(np.ceil(3 * 126e6 / per)))
    g = torch.Generator(device="cuda").manual_seed(0)
    caches = [(torch.randn(nb, block, HK, D, device="cuda", generator=g).half(),
               torch.randn(nb, block, HK, D, device="cuda", generator=g).half()) for _ in range(copies)]
    bt = torch.randperm(nb, device="cuda", generator=g).to(torch.int32).reshape(batch, nblk)
    q = torch.randn(batch, H * D, device="cuda", generator=g).half()
    k = torch.randn(batch, HK * D, device="cuda", generator=g).half()
    v = torch.randn(batch, HK * D, device="cuda", generator=g).half()
    cum = torch.arange(batch + 1, dtype=torch.int32, device="cuda")
    past = torch.full((batch,), ctx - 1, dtype=torch.int32, device="cuda")
    ang = torch.arange(ctx + 8, device="cuda", dtype=torch.float64)[:, None] / (
        10000.0 ** (torch.arange(D // 2, device="cuda", dtype=torch.float64) / (D // 2)))[None, :]
    cos, sin = ang.cos().half(), ang.sin().half()
    out = torch.empty(batch, H * D, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()

    def step(i):
        ops.paged_attention(q, k, v, caches[i][0], caches[i][1], cum, past, bt, cos, sin, num_heads=H,
                            kv_heads=HK, out=out)

    with torch.cuda.stream(stream):
        for i in range(copies):
            step(i)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                step(i)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    alg = 2 * batch * HK * ctx * D * 2 + (q.numel() + k.numel() + v.numel() + out.numel()) * 2
    peak = float(peaks.get("hbm_gbs", HBM_FALLBACK))
    kern = "paged_append_kernel + " + ("paged_attn_kernel" if os.environ.get("ONNXRUNTIME_EP_B200_PAGED_SIMT")
                                       else "gqa_mma_decode_kernel<PAGED>")
    return {"kernel": kern, "batch": batch, "context": ctx, "block": block,
            "launch_us": round(launch_s * 1e6, 2), "algorithmic_bytes_per_launch": alg,
            "achieved": round(alg / launch_s / 1e9, 1), "unit": "GB/s", "frac": round(alg / launch_s / 1e9 / peak, 4),
            "peak": peak, "peak_source": f"{peak_kind} hbm_gbs"}


def paged_prompt_timing(S, past, peaks, peak_kind, reps=10, block=16):
    """PagedAttention over one S-row prompt chunk after `past` cached tokens (32 q / 8 kv heads,
    head 128, fp16, 16-row blocks, random block table): CUDA-event timing of append + attention,
    replayed from a CUDA graph.  Useful flops: 4 * H * D per visible (query, key) pair."""
    import torch

    from onnxruntime_ep_b200 import ops

    H, HK, D = 32, 8, 128
    nblk = (past + S + block - 1) // block
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = torch.randn(nblk, block, HK, D, device="cuda", generator=g).half()
    vc = torch.randn(nblk, block, HK, D, device="cuda", generator=g).half()
    bt = torch.randperm(nblk, device="cuda", generator=g).to(torch.int32).reshape(1, nblk)
    q = torch.randn(S, H * D, device="cuda", generator=g).half()
    k = torch.randn(S, HK * D, device="cuda", generator=g).half()
    v = torch.randn(S, HK * D, device="cuda", generator=g).half()
    cum = torch.tensor([0, S], dtype=torch.int32, device="cuda")
    pst = torch.tensor([past], dtype=torch.int32, device="cuda")
    ang = torch.arange(past + S + 8, device="cuda", dtype=torch.float64)[:, None] / (
        10000.0 ** (torch.arange(D // 2, device="cuda", dtype=torch.float64) / (D // 2)))[None, :]
    cos, sin = ang.cos().half(), ang.sin().half()
    out = torch.empty(S, H * D, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ops.paged_attention(q, k, v, kc, vc, cum, pst, bt, cos, sin, num_heads=H, kv_heads=HK, out=out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            ops.paged_attention(q, k, v, kc, vc, cum, pst, bt, cos, sin, num_heads=H, kv_heads=HK, out=out)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / reps
    flops = 4 * H * D * sum(past + i + 1 for i in range(S))
    peak = float(peaks.get("bf16_tflops", TENSOR_FALLBACK))
    tf = flops / launch_s / 1e12
    return {"kernel": "paged_append_kernel + gqa_mma_prefill_kernel<PAGED>", "S": S, "past": past,
            "launch_us": round(launch_s * 1e6, 2), "achieved": round(tf, 1), "unit": "TFLOP/s",
            "frac": round(tf / peak, 4), "peak": peak, "peak_source": f"{peak_kind} bf16_tflops"}


def gqa_prefill_timing(S, peaks, peak_kind, reps=10):
    """GroupQueryAttention over a whole prompt (32 q / 8 kv heads, head 128, fp16, past 0): the
    rotate-and-append kernel plus the tensor-core prefill kernel, CUDA-event timed over graph
    replays.  Algorithmic work: causal q.k and p.v, 4 * H * D * S * (S + 1) / 2 flops."""
    import torch

    from onnxruntime_ep_b200 import ops

    H, HK, D = 32, 8, 128
    cap = S + 16
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = torch.zeros(1, HK, cap, D, device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    q = torch.randn(1, S, H * D, device="cuda", generator=g).half()
    k = torch.randn(1, S, HK * D, device="cuda", generator=g).half()
    v = torch.randn(1, S, HK * D, device="cuda", generator=g).half()
    seq = torch.full((1,), S - 1, dtype=torch.int32, device="cuda")
    ang = torch.arange(cap + 8, device="cuda", dtype=torch.float64)[:, None] / (
        10000.0 ** (torch.arange(D // 2, device="cuda", dtype=torch.float64) / (D // 2)))[None, :]
    cos, sin = ang.cos().half(), ang.sin().half()
    out = torch.empty(1, S, H * D, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ops.group_query_attention(q, k, v, kc, vc, seq, cos, sin, num_heads=H, kv_heads=HK, out=out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            ops.group_query_attention(q, k, v, kc, vc, seq, cos, sin, num_heads=H, kv_heads=HK, out=out)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / reps
    flops = 4 * H * D * S * (S + 1) / 2
    peak = float(peaks.get("bf16_tflops", TENSOR_FALLBACK))
    tf = flops / launch_s / 1e12
    return {"kernel": "gqa_append_kernel + gqa_mma_prefill_kernel", "S": S, "launch_us": round(launch_s * 1e6, 2),
            "achieved": round(tf, 1), "unit": "TFLOP/s", "peak": peak, "frac": round(tf / peak, 4),
            "peak_source": f"{peak_kind} bf16_tflops (burst)"}


GEMM_SHAPES = (("gate/up", 512, 4096, 28672), ("q/k/v", 512, 4096, 6144), ("o_proj", 512, 4096, 4096),
               ("down", 512, 14336, 4096), ("gate/up", 2048, 4096, 28672))


def gemm_kernel_timing(name, M, K, N, peaks, peak_kind, reps=5):
    """Prefill MatMulNBits alone (the tcgen05 GEMM: int4 block 32, fp16 scales + uint8 zero points,
    fp16 activations) at a Llama-3-8B prefill shape: CUDA-event timing over rotating weight copies
    larger than L2, replayed from a CUDA graph.  Algorithmic work: 2 M N K flops (the hi / lo weight
    split that keeps the dequantised weights exact doubles the tensor-core work actually issued)."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    block = 32
    nb = K // block
    per = N * nb * block // 2 + N * nb * 2 + N * nb // 2
    copies = max(2, int(np.ceil(3 * 126e6 / per)))
    g = torch.Generator(device="cuda").manual_seed(0)
    packs = []
    for _ in range(copies):
        Bq = torch.randint(0, 256, (N, nb, block // 2), dtype=torch.uint8, device="cuda", generator=g)
        S = (torch.rand(N * nb, device="cuda", generator=g) * 0.01 + 0.001).half()
        Z = torch.randint(0, 256, (N * nb // 2,), dtype=torch.uint8, device="cuda", generator=g)
        packs.append(ops.matmulnbits_prepack(Bq, S, Z, K=K, N=N, block_size=block))
        del Bq, S, Z
    a = torch.randn(M, K, device="cuda", generator=g).half()
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(copies):
            ops.matmulnbits_prepacked(a, packs[i], K=K, N=N, out=y)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                ops.matmulnbits_prepacked(a, packs[i], K=K, N=N, out=y)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    flops = 2 * M * N * K
    peak = float(peaks.get("bf16_tflops", TENSOR_FALLBACK))
    tf = flops / launch_s / 1e12
    return {"kernel": "mnb_gemm_kernel", "proj": name, "M": M, "K": K, "N": N, "launch_us": round(launch_s * 1e6, 2),
            "bound": "tensor", "achieved": round(tf, 1), "unit": "TFLOP/s", "peak": peak,
            "frac": round(tf / peak, 4), "issued_frac": round(2 * tf / peak, 4),
            "peak_source": f"{peak_kind} bf16_tflops (burst)"}


def run_ours(args, rank, world, local, tp=False, with_cpu=True, steps=None):
    """One decode measurement.  tp=False: every rank holds a full model and decodes its own
    sequences (data-parallel replicas, no collective on the data path; weak scaling).  tp=True: one
    model sharded over the ranks (tensor parallel), the same tokens on every rank (strong scaling)."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ep as E
    from onnxruntime_ep_b200.decoder import LLAMA3_8B, build_decoder

    cfg = LLAMA3_8B
    B = args.batch
    cap = PROMPT + GEN + 64
    n_steps = steps or args.steps
    tp = tp and world > 1
    t_build = time.time()
    ep = E.ExecutionProvider(device_id=local)
    if tp:
        import torch.distributed as dist

        uid = [E.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep.set_tensor_parallel(rank, world, uid[0])
    g = build_decoder(cfg, batch=-1, seq=-1, cap=-1)
    sess = E.Session(g, ep)
    part = sess.parts[0]
    t_build = time.time() - t_build

    hk = cfg.kv_heads // world if tp else cfg.kv_heads
    kv = []
    for i in range(cfg.layers):
        kv.append([torch.zeros(B, hk, cap, cfg.head_dim, dtype=torch.float16, device="cuda")
                   for _ in range(2)])
    names_in = part.input_names
    names_out = part.output_names

    def bind(ids, seqlens, total, logits):
        feeds = {"input_ids": ids, "seqlens_k": seqlens, "total_sequence_length": total}
        outs = {"logits": logits}
        for i in range(cfg.layers):
            feeds[f"past_key_values.{i}.key"], feeds[f"past_key_values.{i}.value"] = kv[i]
            outs[f"present.{i}.key"], outs[f"present.{i}.value"] = kv[i]
        ins = (E.Tensor * len(names_in))(*[E.make_tensor(feeds[n]) for n in names_in])
        out = (E.Tensor * len(names_out))(*[E.make_tensor(outs[n]) for n in names_out])
        return ins, out

    L = E._lib()
    stream = torch.cuda.current_stream()

    def step(ins, outs):
        E.check(L.b200ep_compiled_run(part._c, ins, len(names_in), outs, len(names_out),
                                      ctypes.c_void_p(stream.cuda_stream)))

    # prefill the prompt through the same graph (untimed)
    rng = np.random.default_rng(0 if tp else rank)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, size=(B, PROMPT), dtype=np.int64)).cuda()
    pre_logits = torch.empty(B, PROMPT, cfg.vocab, dtype=torch.float16, device="cuda")
    t_pre = time.time()
    ins, outs = bind(prompt, torch.full((B,), PROMPT - 1, dtype=torch.int32, device="cuda"),
                     torch.tensor([PROMPT], dtype=torch.int32, device="cuda"), pre_logits)
    step(ins, outs)
    torch.cuda.synchronize()
    t_pre = time.time() - t_pre
    del pre_logits

    # decode: persistent device buffers, advanced in place every step
    ids = torch.zeros(B, 1, dtype=torch.int64, device="cuda")
    seqlens = torch.full((B,), PROMPT - 1, dtype=torch.int32, device="cuda")
    total = torch.tensor([PROMPT], dtype=torch.int32, device="cuda")
    logits = torch.empty(B, 1, cfg.vocab, dtype=torch.float16, device="cuda")
    pool = torch.from_numpy(rng.integers(0, cfg.vocab, size=(max(GEN, n_steps + args.warmup) + 8, B, 1),
                                         dtype=np.int64)).cuda()
    ins, outs = bind(ids, seqlens, total, logits)
    n_step = [0]

    def decode_step():
        ids.copy_(pool[n_step[0] % pool.shape[0]])
        seqlens.add_(1)
        total.add_(1)
        step(ins, outs)
        n_step[0] += 1

    def reset_positions():
        seqlens.fill_(PROMPT - 1)
        total.fill_(PROMPT)

    for _ in range(args.warmup):
        decode_step()
    torch.cuda.synchronize()
    reset_positions()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(n_steps):
            decode_step()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    dev_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
    seqs = B if tp else world * B  # sequences the whole job decodes per step
    value = seqs * n_steps / dev_s

    # e2e through the C ABI with host buffers: ids / lengths staged H2D, logits read back per step
    h_ids = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    h_seq = torch.full((B,), PROMPT - 1, dtype=torch.int32).pin_memory()
    h_tot = torch.tensor([PROMPT], dtype=torch.int32).pin_memory()
    h_logits = torch.empty(B, 1, cfg.vocab, dtype=torch.float16).pin_memory()
    ins_h, outs_h = bind(h_ids, h_seq, h_tot, h_logits)
    pool_h = pool.cpu().numpy()
    # numpy views of the pinned buffers: the per-step host updates cost ~1 us instead of a torch
    # CPU op each
    n_ids, n_seq, n_tot = h_ids.numpy(), h_seq.numpy(), h_tot.numpy()

    def e2e_step(t):
        n_ids[...] = pool_h[t % pool_h.shape[0]]
        n_seq[...] += 1
        n_tot[...] += 1
        step(ins_h, outs_h)  # synchronises: the logits are host-resident

    for t in range(max(2, args.warmup)):
        e2e_step(t)
    h_seq.fill_(PROMPT - 1)
    h_tot.fill_(PROMPT)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record()
    for t in range(n_steps):
        e2e_step(t)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    e2e_s = max_over_ranks(max(e0.elapsed_time(e1) / 1e3, wall), world)
    e2e = {"value": round(seqs * n_steps / e2e_s, 2), "unit": "tokens/s",
           "h2d_bytes_per_step": B * 8 + B * 4 + 4, "d2h_bytes_per_step": B * cfg.vocab * 2,
           "path": "b200ep_compiled_run with pinned host tensors"}

    peaks, peak_kind = measured_peaks()
    roof = dominant_kernel_roofline(B, peaks, peak_kind) if with_cpu else None
    desc = json.loads(part.describe())
    result = {
        "metric": f"int4 decode tokens/s (Llama-3-8B shape, batch {B})",
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": n_steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_s / n_steps * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None,
        "dtype": "int4 weights, fp16 activations, fp32 accumulate",
        "data": "synthetic: random-init int4 weights (seed 0), random token ids",
        "config": {"workload": "Llama-3-8B-shaped int4 decoder decode step (BASELINE config 4)",
                   "layers": cfg.layers, "hidden": cfg.hidden, "heads": f"{cfg.heads}/{cfg.kv_heads}",
                   "ffn": cfg.ffn, "vocab": cfg.vocab, "batch_per_gpu": B, "global_batch": seqs,
                   "prompt": PROMPT, "context_during_timing": f"{PROMPT}..{PROMPT + n_steps}",
                   "kv_capacity": cap,
                   "parallelism": (f"tp{world}: q/k/v, gate/up and lm_head split by output rows (attention by "
                                   f"KV head), o/down by K blocks + peer-memory / NCCL all-reduce, logits "
                                   f"all-gathered")
                   if tp else (f"dp{world}: data-parallel replicas, a full int4 model and its own sequences "
                               f"per GPU, no collective on the data path" if world > 1 else "single GPU"),
                   "l2": "weights 4.4 GB/step streamed from HBM (>> 126 MB L2)",
                   "cuda_graph_replays": desc["graph_replays"], "fused_qkv": desc["fused_qkv"],
                   "fused_swiglu": desc["fused_swiglu"], "prefill_s": round(t_pre, 2),
                   "build_compile_s": round(t_build, 1)},
        "e2e": e2e,
        "roofline": roof,
        "clocks": clocks.summary(),
        "gpu_launches": part.launches_per_run() * n_steps,
    }
    # release the compiled partition (its CUDA graphs hold NCCL calls) before the process group goes
    del part, sess, ep, ins, outs, ins_h, outs_h
    import gc

    gc.collect()
    torch.cuda.synchronize()
    if rank == 0 and with_cpu and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(cfg, B)
    return result


def run_reference(args, rank, world):
    """The reference path's CPU timing (oracle port; see module docstring)."""
    from onnxruntime_ep_b200.decoder import LLAMA3_8B

    if rank != 0:
        return None
    from oracle import oracle

    oracle.build()
    cfg = LLAMA3_8B
    B = args.batch
    cores = oracle.max_threads()
    for _ in range(max(1, min(args.warmup, 1))):
        cpu_layer_sample(cfg, B, PROMPT)
    t_total = 0.0
    for _ in range(args.steps):
        tl, tlm = cpu_layer_sample(cfg, B, PROMPT)
        t_total += cfg.layers * tl + tlm
    value = B * args.steps / t_total
    sample = (f"C oracle (restatement of ORT CPU semantics), one decoder layer + lm_head per step at context "
              f"{PROMPT}, extrapolated to {cfg.layers} layers; reference (Rust/MLX/Metal) and ORT CPU EP "
              f"cannot run here")
    return {
        "impl": "reference",
        "metric": f"int4 decode tokens/s (Llama-3-8B shape, batch {B})",
        "value": round(value, 4),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_total / args.steps * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4 weights, fp16 activations, double accumulate",
        "data": "synthetic",
        "config": {"workload": "Llama-3-8B-shaped int4 decoder decode step (BASELINE config 4)", "batch": B},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--context", type=int, default=0,
                    help="--kernel-only paged: time this one (batch, context) case instead of the default set")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--parallel", default="dp", choices=["dp", "tp"],
                    help="N > 1: data-parallel replicas (default, weak scaling) or one tensor-parallel model")
    ap.add_argument("--no-tp-leg", action="store_true",
                    help="N > 1 with --parallel dp: skip the tensor-parallel measurement reported beside it")
    ap.add_argument("--kernel-only", nargs="?", const="gemv", choices=["gemv", "gqa", "gemm", "paged"],
                    help="time one kernel alone (gemv: the roofline leg; gqa: decode attention, B=1 and 8 at "
                         "context 1024 and 8192; gemm: the prefill GEMM at Llama-3-8B projection shapes; "
                         "paged: PagedAttention decode); "
                         "used for ncu captures")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if args.kernel_only:
        import torch

        from onnxruntime_ep_b200 import load_library

        load_library()
        torch.cuda.set_device(0)
        peaks, peak_kind = measured_peaks()
        if args.kernel_only == "gqa":
            for b, ctx in ((1, 1024), (1, 8192), (8, 8192)):
                print(json.dumps(gqa_kernel_timing(b, ctx, peaks, peak_kind)), flush=True)
            for S in (512, 1024, 4096):
                print(json.dumps(gqa_prefill_timing(S, peaks, peak_kind)), flush=True)
        elif args.kernel_only == "paged":
            cases = ((args.batch, args.context),) if args.context else ((1, 1024), (8, 1024), (8, 8192), (32, 2048))
            for b, ctx in cases:
                print(json.dumps(paged_kernel_timing(b, ctx, peaks, peak_kind)), flush=True)
            if not args.context:
                for S, past in ((512, 0), (2048, 0), (128, 1024)):
                    print(json.dumps(paged_prompt_timing(S, past, peaks, peak_kind)), flush=True)
        elif args.kernel_only == "gemm":
            for name, m, k, n in GEMM_SHAPES:
                print(json.dumps(gemm_kernel_timing(name, m, k, n, peaks, peak_kind)), flush=True)
        else:
            print(json.dumps(dominant_kernel_roofline(args.batch, peaks, peak_kind, reps=2)), flush=True)
        return

    # N > 1: libraries that write to file descriptor 1 directly (NCCL's version banner when the
    # environment sets NCCL_DEBUG) write to stderr instead; rank 0 prints the result line on the
    # original stdout, which then carries that line only
    out_fd = None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        sys.stdout.flush()
        out_fd = os.dup(1)
        os.dup2(2, 1)
    rank, world, local = dist_setup(args.gpus)
    res = run_ours(args, rank, world, local, tp=args.parallel == "tp")
    if world > 1 and args.parallel == "dp" and not args.no_tp_leg:
        # the tensor-parallel form of the same decoder, measured beside the replicas
        t = run_ours(args, rank, world, local, tp=True, with_cpu=False, steps=min(args.steps, 32))
        res["tp"] = {k: t[k] for k in ("value", "unit", "ms_per_step", "steps", "scaling")}
        res["tp"]["parallelism"] = t["config"]["parallelism"]
        res["tp"]["e2e"] = t["e2e"]["value"]
    if rank == 0:
        if out_fd is not None:
            os.write(out_fd, (json.dumps(res) + "\n").encode())
        else:
            print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
