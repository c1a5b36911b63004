"""Benchmark: Llama-3-8B-shaped int4 decode tokens/s through the B200 EP.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload (the Llama-3-8B-shaped int4 decoder, single GPU): 32 layers, hidden 4096, 32/8 heads,
head 128, FFN 14336, vocab 128256, every projection MatMulNBits int4 block 32 with fp16 scales and
uint8 zero points, random-init weights (seed 0), int4 GatherBlockQuantized embedding, prompt of 1024
random token ids prefilled through the same EP graph (untimed), then decode steps.  One step = one
decode token for every sequence of the batch: the whole graph runs as one compiled partition (a
CUDA graph replay) whose positions advance from device-side seqlens_k.

Reported: `value` = decode tokens/s with inputs resident in HBM (CUDA events, max over ranks);
`e2e` = the same through the compiled partition's C ABI with host buffers (token ids and
sequence lengths staged host->device, logits read back every step); `roofline` = the dominant
kernel (the fused gate/up MatMulNBits GEMV) timed live with CUDA events on a weight set larger
than L2; `cpu_baseline` = the C oracle (a restatement of ORT CPU semantics) timed on every host core
for whole decode steps (all 32 layers + lm_head).  --impl reference times that CPU path alone, one
full decode step per timed step (the reference implementation — Rust over MLX/Metal — cannot run
on Linux, and ORT's CPU EP is not installed on this image).

Multi-GPU (N > 1, one process per GPU under torchrun): by default one model sharded over the ranks
(tensor parallel, strong scaling): gate/up and the vocabulary projection split by output rows,
down_proj split by K blocks and followed by one all-reduce per layer (peer memory for decode rows,
NCCL for prompts), attention (q/k/v, GroupQueryAttention, o_proj) run in full on every rank
(`--tp-attention sharded` splits it by KV head instead, with a second all-reduce after o_proj), the
logits all-gathered; every rank decodes the same tokens; value = tokens / max rank time.  The line also carries `tp_parity` (the sharded decoder's
logits against a one-GPU plan of the same graph, prompt + decode steps, compared on rank 0) and
`replicas` (the same N GPUs as independent data-parallel replicas, weak scaling).  Every rank reads
the library's device error word after the warm-up and after the timed region; a non-zero code fails
the run.
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
MODEL = "8b"  # --model: "8b" (the headline workload) or "70b"
MODEL_NAMES = {"8b": "Llama-3-8B", "70b": "Llama-3-70B"}


LAYERS = 0  # --layers: decoder depth override (0 = the model's own)


def model_cfg():
    import dataclasses

    from onnxruntime_ep_b200.decoder import LLAMA3_8B, LLAMA3_70B

    cfg = {"8b": LLAMA3_8B, "70b": LLAMA3_70B}[MODEL]
    return dataclasses.replace(cfg, layers=LAYERS) if LAYERS else cfg
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
def host_cores():
    """Host cores this process may run on (the affinity mask, not an inherited OMP_NUM_THREADS)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


class CpuDecoder:
    """Whole decode steps of the decoder on the C oracle (ORT CPU semantics, every host core): per
    layer RMS norm, q / k / v, GroupQueryAttention over a shared KV buffer holding `ctx` rows, o,
    skip RMS norm, gate / up, SiLU * up, down, skip RMS norm; then the final norm and lm_head.  Layer
    weights are `nsets` distinct random sets used round-robin over the layers (4 x 126 MB of int4
    records exceed any host cache, so every layer streams its weights from DRAM as a real model
    does); each layer has its own KV cache."""

    def __init__(self, cfg, batch, ctx, threads, nsets=4):
        import numpy as np

        from onnxruntime_ep_b200.decoder import quantize_params, rotary_caches

        self.cfg, self.batch, self.ctx, self.threads = cfg, batch, ctx, threads
        rng = np.random.default_rng(1)
        dt = np.float16
        hid, H, HK, D = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        self.sets = []
        for _ in range(nsets):
            W = {}
            for name, n, k in (("q", H * D, hid), ("k", HK * D, hid), ("v", HK * D, hid), ("o", hid, H * D),
                               ("gate", cfg.ffn, hid), ("up", cfg.ffn, hid), ("down", hid, cfg.ffn)):
                W[name] = (quantize_params(rng, n, k, cfg.block, dt), n, k)
            self.sets.append(W)
        self.lm = (quantize_params(rng, cfg.vocab, hid, cfg.block, dt), cfg.vocab, hid)
        self.x = rng.standard_normal((batch, 1, hid)).astype(dt)
        self.g = rng.uniform(0.8, 1.2, hid).astype(dt)
        cap = ctx + 8
        self.kv = [(rng.standard_normal((batch, HK, cap, D)).astype(dt),
                    rng.standard_normal((batch, HK, cap, D)).astype(dt)) for _ in range(cfg.layers)]
        self.cos, self.sin = rotary_caches(cap + 8, D, 10000.0, dt)
        self.seq = np.full(batch, ctx, np.int32)

    def _mnb(self, a, w):
        from oracle import oracle

        (b, s, z), n, k = w
        return oracle.matmulnbits(a, b, s, z, N=n, K=k, threads=self.threads)

    def step(self, layers=None):
        """One decode step (one token per sequence) through `layers` layers (default: all) and the
        vocabulary projection; returns its wall time in seconds."""
        import numpy as np

        from oracle import oracle

        cfg, th, dt = self.cfg, self.threads, np.float16
        t0 = time.perf_counter()
        x, res = self.x, None
        for li in range(layers or cfg.layers):
            W = self.sets[li % len(self.sets)]
            if res is None:
                n1, res1 = oracle.rms_norm(x, self.g, 1e-5, threads=th), x
            else:
                n1, res1 = oracle.skip_rms_norm(x, res, self.g, 1e-5, threads=th)
            q, k, v = self._mnb(n1, W["q"]), self._mnb(n1, W["k"]), self._mnb(n1, W["v"])
            kc, vc = self.kv[li]
            attn, _, _ = oracle.gqa(q, k, v, kc, vc, self.seq, self.cos, self.sin, num_heads=cfg.heads,
                                    kv_heads=cfg.kv_heads, shared_buffer=True, threads=th)
            o = self._mnb(attn, W["o"])
            n2, res = oracle.skip_rms_norm(o, res1, self.g, 1e-5, threads=th)
            ga, up = self._mnb(n2, W["gate"]).astype(np.float32), self._mnb(n2, W["up"]).astype(np.float32)
            x = self._mnb((ga / (1 + np.exp(-ga)) * up).astype(dt), W["down"])
        nf, _ = oracle.skip_rms_norm(x, res, self.g, 1e-5, threads=th)
        self._mnb(nf, self.lm)
        return time.perf_counter() - t0


def cpu_baseline(cfg, batch, samples=2):
    """The oracle on every host core for `samples` whole decode steps after one warm step (~10-30 s)."""
    from oracle import oracle

    oracle.build()
    cores = host_cores()
    dec = CpuDecoder(cfg, batch, PROMPT, cores)
    if cfg.layers <= 32:
        dec.step()  # warm (page in, thread pool)
        best = min(dec.step() for _ in range(samples))
        what = f"{samples} whole B={batch} decode steps ({cfg.layers} layers + lm_head)"
    else:
        # deep models: 8 layers + lm_head per sample (the layer time scaled to every layer)
        dec.step(8)
        t8 = min(dec.step(8) for _ in range(samples))
        t0 = min(dec.step(1) for _ in range(samples))  # 1 layer + lm_head: separates the lm_head
        per_layer = (t8 - t0) / 7
        best = t0 + (cfg.layers - 1) * per_layer
        what = (f"8 and 1 layers + lm_head of a B={batch} decode step (best of {samples}), the measured per-layer "
                f"time {per_layer * 1e3:.0f} ms scaled to {cfg.layers} layers")
    return {"value": batch / best, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"C oracle (ORT CPU semantics), {what} at context {PROMPT} on {cores} threads; ORT's CPU EP "
                      f"is not installed on this image"}


def workload_config(cfg, B, world, mode, n_steps, cap):
    """The `config` object both arms report (the same keys for the same workload)."""
    seqs = B if mode in ("tp", "single") else world * B
    par = {"single": "single GPU",
           "tp": (f"tp{world}: q/k/v, gate/up and lm_head split by output rows (attention by KV head), o/down "
                  f"by K blocks + peer-memory (decode) / NCCL (prompt) all-reduce, logits all-gathered"
                  if TP_ATTENTION == "sharded" else
                  f"tp{world}: attention (q/k/v, GQA, o_proj) in full on every rank, gate/up and lm_head split "
                  f"by output rows, down by K blocks + one peer-memory (decode) / NCCL (prompt) all-reduce per "
                  f"layer, logits all-gathered"),
           "dp": (f"dp{world}: data-parallel replicas, a full int4 model and its own sequences per GPU, no "
                  f"collective on the data path")}[mode]
    return {"workload": f"{MODEL_NAMES[MODEL]}-shaped int4 decoder, decode step", "layers": cfg.layers,
            "hidden": cfg.hidden,
            "heads": f"{cfg.heads}/{cfg.kv_heads}", "ffn": cfg.ffn, "vocab": cfg.vocab, "batch_per_gpu": B,
            "global_batch": seqs, "prompt": PROMPT, "context_during_timing": f"{PROMPT}..{PROMPT + n_steps}",
            "kv_capacity": cap, "parallelism": par,
            "l2": f"weights {weight_gb(cfg):.1f} GB/step streamed from HBM (>> 126 MB L2)"}


def weight_gb(cfg):
    """int4 weights + fp16 scales + packed zero points read per decode token (all projections and
    the vocabulary projection)."""
    per_layer = (cfg.heads * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim) * cfg.hidden + \
        cfg.hidden * cfg.heads * cfg.head_dim + 3 * cfg.ffn * cfg.hidden
    params = cfg.layers * per_layer + cfg.vocab * cfg.hidden
    return params * (0.5 + 2 / cfg.block + 0.5 / cfg.block) / 1e9


# ---- the GPU arm ---------------------------------------------------------------------------
GEMV_SHAPES = (("q/k/v", 6144, 4096), ("o_proj", 4096, 4096), ("gate/up", 28672, 4096), ("down", 4096, 14336),
               ("lm_head", 128256, 4096))


def gemv_shape_timing(name, N, K, batch, peaks, peak_kind, reps=10):
    """One decode GEMV shape alone (prepacked int4 block 32, fp16 scales + uint8 zero points, fp16
    activations, no fused prologue): CUDA-event timing over rotating weight copies larger than L2,
    replayed from a CUDA graph."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    block = 32
    nb = K // block
    per = N * nb * block // 2 + N * nb * 2 + N * nb // 2
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
    peak = float(peaks.get("hbm_gbs", HBM_FALLBACK))
    return {"kernel": "mnb_tma_kernel", "proj": name, "M": batch, "N": N, "K": K, "launch_us": round(launch_s * 1e6, 2),
            "algorithmic_bytes_per_launch": alg, "achieved": round(alg / launch_s / 1e9, 1), "unit": "GB/s",
            "frac": round(alg / launch_s / 1e9 / peak, 4), "peak": peak, "peak_source": f"{peak_kind} hbm_gbs"}


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
    rotate-and-append kernel, the value transpose and the tcgen05 prompt kernel
    (ONNXRUNTIME_EP_B200_NO_UMMA_ATTN=1: the mma.sync prompt kernel), CUDA-event timed over graph
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
    kern = ("gqa_append_kernel + gqa_mma_prefill_kernel" if os.environ.get("ONNXRUNTIME_EP_B200_NO_UMMA_ATTN")
            else "gqa_append_kernel + gqa_vt_kernel + gqa_umma_prefill_kernel")
    return {"kernel": kern, "S": S, "launch_us": round(launch_s * 1e6, 2),
            "achieved": round(tf, 1), "unit": "TFLOP/s", "peak": peak, "frac": round(tf / peak, 4),
            "peak_source": f"{peak_kind} bf16_tflops (burst)"}


def c1_kernel_timing(M, peaks, peak_kind, reps=10):
    """The single-MatMulNBits workload exactly as specified: fp32 A [M, 4096] ~ N(0, 1), B [4096,
    4096] int4 block 32, fp32 scales ~ U(0.005, 0.02), uint8 zero points ~ U{0..15}, fp32 output,
    through the ORT-layout entry point (b200ep_matmulnbits: the fp32 SIMT GEMV / tiled kernel, which
    keep the fp32 contract's 6e-5 tolerance).  CUDA-event timing over rotating weight copies larger
    than L2, replayed from a CUDA graph.  Algorithmic bytes: weights + scales + zero points + A + Y."""
    import numpy as np
    import torch

    from onnxruntime_ep_b200 import ops

    K = N = 4096
    block = 32
    nb = K // block
    per = N * nb * block // 2 + N * nb * 4 + N * nb // 2
    copies = max(3, int(np.ceil(3 * 126e6 / per)))
    g = torch.Generator(device="cuda").manual_seed(0)
    ws = []
    for _ in range(copies):
        q = torch.randint(0, 16, (N, nb, block), dtype=torch.uint8, device="cuda", generator=g)
        b = (q[..., 0::2] | (q[..., 1::2] << 4)).contiguous()
        s = torch.rand(N * nb, device="cuda", generator=g) * 0.015 + 0.005
        z = torch.randint(0, 16, (N * nb,), dtype=torch.uint8, device="cuda", generator=g)
        z = (z[0::2] | (z[1::2] << 4)).contiguous()
        ws.append((b, s, z))
    a = torch.randn(M, K, device="cuda", generator=g)
    y = torch.empty(M, N, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for w in ws:
            ops.matmulnbits(a, *w, K=K, N=N, out=y)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for w in ws:
                ops.matmulnbits(a, *w, K=K, N=N, out=y)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    launch_s = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    alg = per + M * K * 4 + M * N * 4
    peak = float(peaks.get("hbm_gbs", HBM_FALLBACK))
    gbs = alg / launch_s / 1e9
    return {"kernel": "b200ep_matmulnbits fp32 (SIMT GEMV / tiled kernel)", "M": M, "K": K, "N": N,
            "launch_us": round(launch_s * 1e6, 2), "algorithmic_bytes_per_launch": alg, "achieved": round(gbs, 1),
            "unit": "GB/s", "frac": round(gbs / peak, 4), "peak": peak, "peak_source": f"{peak_kind} hbm_gbs",
            "tflops": round(2 * M * N * K / launch_s / 1e12, 2)}


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


def device_error_check(where):
    """Read and clear the library's device error word (bounded waits that expired, bad positions);
    a non-zero code fails the run instead of reporting a number taken over stalled or wrong steps."""
    from onnxruntime_ep_b200 import ops

    code, detail = ops.device_error(clear=True)
    if code:
        raise RuntimeError(f"device error {code} (detail {detail}) reported by a kernel {where}")


def kv_buffers(cfg, B, hk, cap):
    import torch

    return [[torch.zeros(B, hk, cap, cfg.head_dim, dtype=torch.float16, device="cuda") for _ in range(2)]
            for _ in range(cfg.layers)]


def bind_decoder(part, cfg, kv, ids, seqlens, total, logits):
    """C-ABI tensor arrays for one run of the decoder partition (KV caches shared past / present)."""
    from onnxruntime_ep_b200 import ep as E

    feeds = {"input_ids": ids, "seqlens_k": seqlens, "total_sequence_length": total}
    outs = {"logits": logits}
    for i in range(cfg.layers):
        feeds[f"past_key_values.{i}.key"], feeds[f"past_key_values.{i}.value"] = kv[i]
        outs[f"present.{i}.key"], outs[f"present.{i}.value"] = kv[i]
    ins = (E.Tensor * len(part.input_names))(*[E.make_tensor(feeds[n]) for n in part.input_names])
    out = (E.Tensor * len(part.output_names))(*[E.make_tensor(outs[n]) for n in part.output_names])
    return ins, out


def run_part(part, ins, outs, stream):
    from onnxruntime_ep_b200 import ep as E

    E.check(E._lib().b200ep_compiled_run(part._c, ins, len(part.input_names), outs, len(part.output_names),
                                         ctypes.c_void_p(stream.cuda_stream)))


PARITY_PROMPT, PARITY_STEPS = 16, 4


def parity_logits(part, cfg, hk, B):
    """Logits of a fixed short sequence (a PARITY_PROMPT-token prompt then PARITY_STEPS decode steps,
    token ids from a fixed seed) through `part`, as one float32 array [rows, vocab] on the host."""
    import numpy as np
    import torch

    cap = PARITY_PROMPT + PARITY_STEPS + 8
    kv = kv_buffers(cfg, B, hk, cap)
    rng = np.random.default_rng(12345)
    ids = rng.integers(0, cfg.vocab, size=(B, PARITY_PROMPT + PARITY_STEPS), dtype=np.int64)
    stream = torch.cuda.current_stream()
    rows = []
    lg = torch.empty(B, PARITY_PROMPT, cfg.vocab, dtype=torch.float16, device="cuda")
    ins, outs = bind_decoder(part, cfg, kv, torch.from_numpy(ids[:, :PARITY_PROMPT].copy()).cuda(),
                             torch.full((B,), PARITY_PROMPT - 1, dtype=torch.int32, device="cuda"),
                             torch.tensor([PARITY_PROMPT], dtype=torch.int32, device="cuda"), lg)
    run_part(part, ins, outs, stream)
    rows.append(lg.float().cpu().numpy().reshape(-1, cfg.vocab))
    for t in range(PARITY_STEPS):
        p = PARITY_PROMPT + t
        lg1 = torch.empty(B, 1, cfg.vocab, dtype=torch.float16, device="cuda")
        ins, outs = bind_decoder(part, cfg, kv, torch.from_numpy(ids[:, p:p + 1].copy()).cuda(),
                                 torch.full((B,), p, dtype=torch.int32, device="cuda"),
                                 torch.tensor([p + 1], dtype=torch.int32, device="cuda"), lg1)
        run_part(part, ins, outs, stream)
        rows.append(lg1.float().cpu().numpy().reshape(-1, cfg.vocab))
    torch.cuda.synchronize()
    del kv
    return np.concatenate(rows, 0)


def compare_logits(got, ref):
    """Composite-decoder comparison: max |diff| against 2e-2 of the reference logit range, and the
    share of rows whose argmax agrees (ties within the tolerance count as agreement)."""
    import numpy as np

    rng_ = float(ref.max() - ref.min())
    d = np.abs(got - ref)
    tol = 2e-2 * rng_
    am_g, am_r = got.argmax(-1), ref.argmax(-1)
    agree = np.mean([(a == b) or (ref[i, a] >= ref[i, b] - tol) for i, (a, b) in enumerate(zip(am_g, am_r))])
    return {"rows": int(ref.shape[0]), "max_abs": round(float(d.max()), 5), "mean_abs": round(float(d.mean()), 6),
            "logit_range": round(rng_, 4), "tol": round(tol, 5), "argmax_agree": round(float(agree), 4),
            "ok": bool(d.max() <= tol and agree >= 0.95)}


TP_ATTENTION = "sharded"  # --tp-attention


def build_part(cfg, local, rank, world, tp):
    from onnxruntime_ep_b200 import ep as E
    from onnxruntime_ep_b200.decoder import build_decoder

    ep = E.ExecutionProvider(device_id=local, tp_attention=TP_ATTENTION) if tp else E.ExecutionProvider(device_id=local)
    if tp:
        import torch.distributed as dist

        uid = [E.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep.set_tensor_parallel(rank, world, uid[0])
    sess = E.Session(build_decoder(cfg, batch=-1, seq=-1, cap=-1), ep)
    return ep, sess, sess.parts[0]


def run_ours(args, rank, world, local, tp=False, with_cpu=True, steps=None, parity=False):
    """One decode measurement.  tp=False: every rank holds a full model and decodes its own
    sequences (data-parallel replicas, no collective on the data path; weak scaling).  tp=True: one
    model sharded over the ranks (tensor parallel), the same tokens on every rank (strong scaling);
    parity=True then also compares the sharded logits with a one-GPU plan on rank 0."""
    import numpy as np
    import torch

    cfg = model_cfg()
    B = args.batch
    cap = PROMPT + GEN + 64
    n_steps = steps or args.steps
    tp = tp and world > 1
    t_build = time.time()
    ep, sess, part = build_part(cfg, local, rank, world, tp)
    t_build = time.time() - t_build
    hk = cfg.kv_heads // world if tp and TP_ATTENTION == "sharded" else cfg.kv_heads
    kv = kv_buffers(cfg, B, hk, cap)
    stream = torch.cuda.current_stream()
    device_error_check("before the run")

    # prefill the prompt through the same graph (untimed)
    rng = np.random.default_rng(0 if tp else rank)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, size=(B, PROMPT), dtype=np.int64)).cuda()
    pre_logits = torch.empty(B, PROMPT, cfg.vocab, dtype=torch.float16, device="cuda")
    t_pre = time.time()
    ins, outs = bind_decoder(part, cfg, kv, prompt, torch.full((B,), PROMPT - 1, dtype=torch.int32, device="cuda"),
                             torch.tensor([PROMPT], dtype=torch.int32, device="cuda"), pre_logits)
    run_part(part, ins, outs, stream)
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
    ins, outs = bind_decoder(part, cfg, kv, ids, seqlens, total, logits)
    n_step = [0]

    def decode_step():
        ids.copy_(pool[n_step[0] % pool.shape[0]])
        seqlens.add_(1)
        total.add_(1)
        run_part(part, ins, outs, stream)
        n_step[0] += 1

    for _ in range(args.warmup):
        decode_step()
    torch.cuda.synchronize()
    device_error_check("during the warm-up")
    seqlens.fill_(PROMPT - 1)
    total.fill_(PROMPT)
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
    device_error_check("in the timed region")
    dev_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
    seqs = B if tp else world * B  # sequences the whole job decodes per step
    value = seqs * n_steps / dev_s

    # e2e through the C ABI with host buffers: ids / lengths staged H2D, logits read back per step
    h_ids = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    h_seq = torch.full((B,), PROMPT - 1, dtype=torch.int32).pin_memory()
    h_tot = torch.tensor([PROMPT], dtype=torch.int32).pin_memory()
    h_logits = torch.empty(B, 1, cfg.vocab, dtype=torch.float16).pin_memory()
    ins_h, outs_h = bind_decoder(part, cfg, kv, h_ids, h_seq, h_tot, h_logits)
    pool_h = pool.cpu().numpy()
    # numpy views of the pinned buffers: the per-step host updates cost ~1 us instead of a torch
    # CPU op each
    n_ids, n_seq, n_tot = h_ids.numpy(), h_seq.numpy(), h_tot.numpy()

    def e2e_step(t):
        n_ids[...] = pool_h[t % pool_h.shape[0]]
        n_seq[...] += 1
        n_tot[...] += 1
        run_part(part, ins_h, outs_h, stream)  # synchronises: the logits are host-resident

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
    device_error_check("in the end-to-end region")
    e2e_s = max_over_ranks(max(e0.elapsed_time(e1) / 1e3, wall), world)
    e2e = {"value": round(seqs * n_steps / e2e_s, 2), "unit": "tokens/s",
           "h2d_bytes_per_step": B * 8 + B * 4 + 4, "d2h_bytes_per_step": B * cfg.vocab * 2,
           "path": "b200ep_compiled_run with pinned host tensors"}

    tp_parity = None
    if tp and parity:
        # the sharded decoder's logits on a fixed prompt + decode steps (every rank takes the same
        # collective steps), then a one-GPU plan of the same graph on rank 0
        got = parity_logits(part, cfg, hk, B)
        device_error_check("in the parity run")
        if rank == 0:
            ep1, sess1, part1 = build_part(cfg, local, 0, 1, False)
            ref = parity_logits(part1, cfg, cfg.kv_heads, B)
            del part1, sess1, ep1
            tp_parity = compare_logits(got, ref)
            tp_parity["against"] = "one-GPU plan of the same graph (rank 0)"
        barrier(world)

    peaks, peak_kind = measured_peaks()
    roof = dominant_kernel_roofline(B, peaks, peak_kind) if with_cpu else None
    desc = json.loads(part.describe())
    mode = "tp" if tp else ("dp" if world > 1 else "single")
    config = workload_config(cfg, B, world, mode, n_steps, cap)
    config.update({"cuda_graph_replays": desc["graph_replays"], "fused_qkv": desc["fused_qkv"],
                   "fused_swiglu": desc["fused_swiglu"], "peer_allreduce": desc.get("peer_allreduce", 0),
                   "prefill_s": round(t_pre, 2), "build_compile_s": round(t_build, 1)})
    result = {
        "metric": f"int4 decode tokens/s ({MODEL_NAMES[MODEL]} shape, batch {B})",
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
        "config": config,
        "e2e": e2e,
        "roofline": roof,
        "clocks": clocks.summary(),
        "gpu_launches": part.launches_per_run() * n_steps,
    }
    if tp_parity is not None:
        result["tp_parity"] = tp_parity
    # release the compiled partition (its CUDA graphs hold NCCL calls) before the process group goes
    del part, sess, ep, ins, outs, ins_h, outs_h, kv
    import gc

    gc.collect()
    torch.cuda.synchronize()
    if rank == 0 and with_cpu and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(cfg, B)
    return result


def run_reference(args, rank, world):
    """The reference arm: the CPU oracle (the ORT CPU semantics the reference is checked against)
    on every host core, one whole decode step (32 layers + lm_head) per timed step, rank 0 only."""
    if rank != 0:
        return None
    from oracle import oracle

    oracle.build()
    cfg = model_cfg()
    B = args.batch
    cores = host_cores()
    dec = CpuDecoder(cfg, B, PROMPT, cores)
    for _ in range(args.warmup):
        dec.step()
    t_total = sum(dec.step() for _ in range(args.steps))
    value = B * args.steps / t_total
    sample = (f"C oracle (restatement of ORT CPU semantics) on {cores} threads, every step a whole decode step "
              f"({cfg.layers} layers + lm_head) at context {PROMPT}; the reference (Rust over MLX/Metal) cannot "
              f"run on Linux and ORT's CPU EP is not installed on this image")
    return {
        "impl": "reference",
        "metric": f"int4 decode tokens/s ({MODEL_NAMES[MODEL]} shape, batch {B})",
        "value": round(value, 4),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_total / args.steps * 1e3, 2),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "int4 weights, fp16 activations, double accumulate",
        "data": "synthetic: random-init int4 weights, random activations",
        "config": workload_config(cfg, B, world, "tp" if world > 1 else "single", args.steps, PROMPT + GEN + 64),
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
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="decoder shape: Llama-3-8B (the headline workload, prompt 1024) or Llama-3-70B "
                         "(prompt 2048)")
    ap.add_argument("--prompt", type=int, default=0, help="prompt length prefilled before the timed decode steps")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder depth override for diagnosis (a shallower model is not the named workload)")
    ap.add_argument("--context", type=int, default=0,
                    help="--kernel-only paged: time this one (batch, context) case instead of the default set")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--parallel", default="tp", choices=["dp", "tp"],
                    help="N > 1: one tensor-parallel model (default, strong scaling) or data-parallel replicas")
    ap.add_argument("--no-side-leg", action="store_true",
                    help="N > 1: skip the other parallel form's measurement reported beside the headline")
    ap.add_argument("--no-parity", action="store_true", help="N > 1 tensor parallel: skip the tp_parity check")
    ap.add_argument("--tp-attention", default="auto", choices=["auto", "sharded", "replicated"],
                    help="tensor parallel: attention sharded by KV head (two all-reduces per layer) or run in "
                         "full on every rank (one all-reduce per layer, after the FFN); auto = the faster form "
                         "measured at 2 GPUs (replicated for both the 8B and the 70B shape)")
    ap.add_argument("--kernel-only", nargs="?", const="gemv",
                    choices=["gemv", "gemv-shapes", "gqa", "gemm", "paged", "c1"],
                    help="time one kernel alone (gemv: the roofline leg; gemv-shapes: every decode projection of "
                         "the Llama-3-8B layer; gqa: decode attention, B=1 and 8 at "
                         "context 1024 and 8192; gemm: the prefill GEMM at Llama-3-8B projection shapes; "
                         "paged: PagedAttention decode; c1: the fp32 single-MatMulNBits workload at M 1/16/512); "
                         "used for ncu captures")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    global MODEL, PROMPT, LAYERS, TP_ATTENTION
    MODEL = args.model
    TP_ATTENTION = args.tp_attention if args.tp_attention != "auto" else "replicated"
    LAYERS = args.layers
    PROMPT = args.prompt or (2048 if MODEL == "70b" else 1024)

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
            for S in (512, 1024, 4096, 8192):
                print(json.dumps(gqa_prefill_timing(S, peaks, peak_kind)), flush=True)
        elif args.kernel_only == "paged":
            cases = ((args.batch, args.context),) if args.context else ((1, 1024), (8, 1024), (8, 8192), (32, 2048))
            for b, ctx in cases:
                print(json.dumps(paged_kernel_timing(b, ctx, peaks, peak_kind)), flush=True)
            if not args.context:
                for S, past in ((512, 0), (2048, 0), (128, 1024)):
                    print(json.dumps(paged_prompt_timing(S, past, peaks, peak_kind)), flush=True)
        elif args.kernel_only == "gemv-shapes":
            for name, n, k in GEMV_SHAPES:
                print(json.dumps(gemv_shape_timing(name, n, k, args.batch, peaks, peak_kind)), flush=True)
        elif args.kernel_only == "c1":
            for m in (1, 16, 512):
                print(json.dumps(c1_kernel_timing(m, peaks, peak_kind)), flush=True)
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
    tp = args.parallel == "tp"
    res = run_ours(args, rank, world, local, tp=tp, parity=tp and not args.no_parity)
    if world > 1 and not args.no_side_leg:
        # the other multi-GPU form of the same decoder, measured beside the headline
        t = run_ours(args, rank, world, local, tp=not tp, with_cpu=False, steps=min(args.steps, 32))
        side = {k: t[k] for k in ("value", "unit", "ms_per_step", "steps", "scaling")}
        side["parallelism"] = t["config"]["parallelism"]
        side["e2e"] = t["e2e"]["value"]
        res["replicas" if tp else "tp"] = side
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
