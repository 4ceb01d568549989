#!/usr/bin/env python
"""Headline benchmark of the zwhisper attention engine on B200.

Headline workload: Whisper small.en encoder self-attention,
64 consecutive 30 s windows x 12 layers x 12 heads of d=64 over n_ctx=1500, bf16
tensor-core compute with f32 softmax and accumulation. One step = all 12 layers' attention
over the job's 64 windows (distinct Q/K/V per layer, inputs far larger than L2). Windows
are sharded in contiguous blocks over the ranks (64 / N each, no collective on the data
path): total work is fixed, so scaling is "strong".

Reported (one JSON line from rank 0):
  value      windows/s with inputs resident in HBM (CUDA events, max over ranks);
  e2e        windows/s through the C-ABI drop-in (zwg_attention_batch_host, math mode
             bf16) from pinned host f32 buffers, host<->device copies timed;
  roofline   the tcgen05 encoder kernel: algorithmic FLOPs per launch / average launch
             time, against the measured bf16 peak;
  cpu_baseline  the C restatement of the reference attention (oracle/attn_ref.c) on the
             host cores, rank 0 at N=1;
  secondary  decode-attention workloads (configs 1, 3, 4) at N=1: tok/s and HBM roofline,
             each decode step (all layers) replayed from a CUDA graph; prefill attention;
             the whole small.en encoder on the device; the Q8 projections;
             and the whole Qwen2.5-1.5B greedy decode step on the device (B = 1 and 64).

`--impl reference` times the reference's CPU attention (the C restatement; the Zig source
cannot be built here) on the same workload and prints the same line with "impl".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_CTX, N_STATE, N_HEAD, N_LAYER, WINDOWS = 1500, 768, 12, 12, 64
METRIC = "whisper_small_en_encoder_attention_windows_per_s"
UNIT = "windows/s"
FLOP_PER_WINDOW_LAYER = 4 * N_CTX * N_CTX * N_STATE          # QK^T and PV, 2 flops per MAC
SIGMA = (N_STATE ** 0.5) * 0.02                               # LN output x N(0, 0.02^2) weights


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def profiled_traffic(name: str, units: float):
    """DRAM bytes (read + write) of one launch over `units` windows or sequences, from the
    committed ncu summary of a smaller case of the same kernel, scaled by the units
    processed (the traffic of these kernels grows in proportion); None without a summary."""
    path = os.path.join(ROOT, "profiles", name)
    bytes_, per = None, None
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    bytes_ = float(line.split(":", 1)[1].split()[0])
                elif line.startswith("units_per_launch:"):
                    per = float(line.split(":", 1)[1].split()[0])
    except OSError:
        return None
    if bytes_ is None or not per:
        return None
    return bytes_ * units / per


# ---------------------------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="zwg_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxes.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


# ---------------------------------------------------------------------------------------------
# distributed plumbing (one process per GPU; no collective on the data path)

def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        # keep stdout to the one JSON line: no NCCL banner
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(n: int, rank: int, world: int):
    return n * rank // world, n * (rank + 1) // world


# ---------------------------------------------------------------------------------------------
# CPU baseline: the C restatement of the reference attention

class CpuSample:
    """One window through all 12 layers' attention (12 calls of the small.en shape) in the
    C restatement of the reference attention, on `threads` host cores."""

    def __init__(self, threads: int = 0):
        import numpy as np

        from oracle import attention as OA
        from oracle import cref
        self.threads = threads or os.cpu_count() or 1
        self.isa = cref.isa()
        rng = np.random.default_rng(0)
        self.run = cref.Runner(OA.mha_shape(N_CTX, N_CTX, N_STATE, N_HEAD, False), self.threads)
        self.q, self.k, self.v = ((rng.standard_normal(N_CTX * N_STATE, dtype=np.float32) * SIGMA) for _ in range(3))
        self.out = np.zeros(N_CTX * N_STATE, np.float32)

    def window(self):
        for _ in range(N_LAYER):
            self.run(self.q, self.k, self.v, self.out)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_windows_per_s(min_seconds: float = 10.0, max_reps: int = 40, threads: int = 0):
    """Windows/s of the CPU restatement, repeated until min_seconds of work."""
    s = CpuSample(threads)
    s.run(s.q, s.k, s.v, s.out)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        s.window()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            break
    return {"value": reps / el, "unit": UNIT, "cores": s.threads, "kind": "port",
            "sample": f"{reps} window(s) x {N_LAYER} layers of {N_HEAD}-head 1500x1500 d64 f32 attention, "
                      f"oracle/attn_ref.c ({s.isa}), {el:.1f} s", "isa": s.isa}


def reference_binary_baseline(threads: int):
    """The reference's shipped binary (copied into oracle/_ref by the build) timed by its own
    `bench <threads>` command on the base.en attention shape (src/bench.zig:50-77), next to
    the C restatement on the same shape and threads. None when the binary is absent or does
    not run on this host."""
    import numpy as np

    from oracle import attention as OA
    from oracle import cref, ref_binary
    rb = ref_binary.bench_attention(threads)
    if rb is None:
        return None
    n_ctx, ns, H = 1500, 512, 8
    run = cref.Runner(OA.mha_shape(n_ctx, n_ctx, ns, H, False), threads)
    rng = np.random.default_rng(0)
    q, k, v = ((rng.standard_normal(n_ctx * ns, dtype=np.float32) * SIGMA) for _ in range(3))
    out = np.zeros(n_ctx * ns, np.float32)
    run(q, k, v, out)
    reps, t0 = 0, time.perf_counter()
    while reps < 20 or time.perf_counter() - t0 < 1.0:
        run(q, k, v, out)
        reps += 1
    ms = (time.perf_counter() - t0) / reps * 1e3
    return {"shape": "base.en encoder attention, 8 heads x 1500 x 1500, d 64 (the binary's bench line)",
            "threads": threads,
            "binary": {"ms": rb["ms"], "gflops": rb["gflops"], "line": rb["line"]},
            "port": {"ms": ms, "gflops": ref_binary.ATTN_FLOP / ms / 1e6},
            "binary_windows_per_s_equiv": rb["gflops"] * 1e9 / (FLOP_PER_WINDOW_LAYER * N_LAYER),
            "note": "windows/s the binary's attention rate gives on the small.en window's 82.9 GFLOP"}


def run_reference(args, rank, world):
    """The reference's CPU attention on the host cores, on the same job as our arm: each step
    is all 64 windows through all 12 layers (the C restatement of attentionEx with all host
    threads; every window reuses one set of Q/K/V, the work being compute-bound)."""
    if rank != 0:
        return
    s = CpuSample()
    s.window()  # warm-up
    warm = min(args.warmup, 1)
    for _ in range(warm):
        for _ in range(WINDOWS):
            s.window()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(WINDOWS):
            s.window()
    el = time.perf_counter() - t0
    value = WINDOWS * args.steps / el
    rb = reference_binary_baseline(s.threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "whisper small.en encoder self-attention (configs[2]): 64 "
                                                     "windows x 12 layers x 12 heads, n_ctx 1500, d 64",
                                        "windows": WINDOWS, "n_ctx": N_CTX, "n_state": N_STATE, "n_head": N_HEAD,
                                        "n_layer": N_LAYER},
        "same_config": True,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": s.threads, "kind": "port",
                         "sample": f"{WINDOWS} windows x {N_LAYER} layers per step (the whole job), oracle/attn_ref.c "
                                   f"({s.isa}), f32; the reference's Zig source cannot be built here (no Zig "
                                   "toolchain)", "cpu": cpu_model()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if rb is not None:
        line["cpu_baseline"]["reference_binary"] = rb
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm

def time_graph(fn, steps, warmup=3):
    """Capture one call of fn (a whole decode step: every layer's attention) in a CUDA
    graph and time `steps` replays with CUDA events. Decode steps are launch-bound at these
    sizes; a serving loop replays a captured step the same way."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    t = time_cuda(graph.replay, steps)
    del graph
    return t


def time_cuda(fn, steps, stream=None):
    import torch
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e-3


def secondary_decode(dev, hbm_peak, rank, world, steps=20, warmup=3):
    """Decode-attention workloads (configs 1, 3, 4): one step = one new token for every item
    through all layers' attention (f32 K/V, the reference's precision), captured once in a
    CUDA graph and replayed. Items (windows, sequences) are sharded over the ranks; the
    figures are the whole job's (items of all ranks over the slowest rank's time) and the
    per-GPU HBM fraction."""
    import torch

    from zwhisper_b200 import ops
    res = []
    g = torch.Generator(device=dev)
    g.manual_seed(1 + rank)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32)

    # config 1: whisper base.en decoder step, 32 windows, 6 layers, each with its own self
    # cache (224 of 448 positions) and cross K/V (1500 frames)
    B_all, H, d, ns, L = 32, 8, 64, 512, 6
    b0, b1 = shard(B_all, rank, world)
    B = b1 - b0
    layers = [(randn(B, 448, ns), randn(B, 448, ns), randn(B, 1500, ns), randn(B, 1500, ns)) for _ in range(L)]
    q, o = randn(B, 1, ns), torch.empty(B, 1, ns, device=dev)
    sh_s = ops.mha_shape(1, 224, ns, H, True)
    sh_c = ops.mha_shape(1, 1500, ns, H, False)
    ws_s = torch.empty(max(1, ops.attention_workspace_bytes(sh_s, B)), dtype=torch.uint8, device=dev)
    ws_c = torch.empty(max(1, ops.attention_workspace_bytes(sh_c, B)), dtype=torch.uint8, device=dev)

    def step1():
        for ck, cv, xk, xv in layers:
            ops.attention_dev(q, ck, cv, sh_s, o, n_batch=B, batch_strides=(ns, 448 * ns, 448 * ns, ns), workspace=ws_s)
            ops.attention_dev(q, xk, xv, sh_c, o, n_batch=B, batch_strides=(ns, 1500 * ns, 1500 * ns, ns),
                              workspace=ws_c)
    t = max_over_ranks(time_graph(step1, steps, warmup) / steps, world)
    byts = L * B_all * (224 + 1500) * ns * 4 * 2
    res.append({"workload": f"whisper base.en decoder self+cross attention step (configs[1]): {B_all} windows "
                            f"({B} per GPU), {L} layers with distinct caches",
                "metric": "whisper_base_en_decoder_attention_tok_per_s", "value": B_all / t, "unit": "tok/s",
                "ms_per_step": t * 1e3, "math": "f32",
                "roofline": {"bound": "hbm", "achieved": byts / world / t / 1e9, "peak": hbm_peak, "unit": "GB/s",
                             "frac": byts / world / t / 1e9 / hbm_peak, "traffic": None, "per": "GPU"}})
    del layers
    # configs 3 and 4: Qwen2 decode over the transposed key cache at the mean cache length,
    # through the state's decode entry point (zwg_llm_attn_decode, src/llm.zig:191-202) over
    # the state's own per-layer caches
    for cfg, B_all, L, H, Hkv, d, n_kv in (("configs[3] Qwen2.5-0.5B", 16, 24, 14, 2, 64, 2128),
                                           ("configs[4] Qwen2.5-1.5B", 64, 28, 12, 2, 128, 2256)):
        n_ctx = 2560
        b0, b1 = shard(B_all, rank, world)
        B = b1 - b0
        st = ops.LlmState(L, B, H, Hkv, d, n_ctx, device=dev.index or 0)
        for layer in range(L):
            for t_ in st.cache_views(layer):
                t_.normal_(generator=g)
        q, o = randn(B, 1, H * d), torch.empty(B, 1, H * d, device=dev)
        byts = B_all * n_kv * Hkv * d * 4 * 2 * L

        def step(st=st, q=q, o=o, L=L, n_kv=n_kv):
            for layer in range(L):
                st.attn(layer, q, n_kv - 1, out=o)
        # math "f32": the SIMT split-K kernel (the reference's arithmetic); "tf32": the
        # tcgen05 kernel (tf32 operands, f32 accumulation; parity within max-abs 2e-3)
        for math, kernel in (("f32", "decode_tma_kernel"), ("tf32", "decode_tc_kernel")):
            ops.set_math(math, dev.index or 0)
            try:
                t = max_over_ranks(time_graph(step, steps, warmup) / steps, world)
            finally:
                ops.set_math("f32", dev.index or 0)
            achieved = byts / world / t / 1e9
            traffic = profiled_traffic("decode_tma_qwen15_b16.txt", B) if (d == 128 and math == "f32") else None
            res.append({"workload": f"{cfg} decode attention, {B_all} sequences ({B} per GPU) x {L} layers, "
                                    f"n_kv={n_kv} (mean of the decode), K^T cache n_ctx={n_ctx}, math {math} ({kernel})",
                        "metric": "qwen_decode_attention_tok_per_s", "value": B_all / t, "unit": "tok/s",
                        "ms_per_step": t * 1e3, "math": math,
                        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                                     "frac": achieved / hbm_peak, "traffic": traffic, "per": "GPU",
                                     "bytes_per_step": byts}})
        st.close()
    torch.cuda.empty_cache()
    return res


def secondary_prefill(dev, tc_peak, peak_kind, rank, world, steps=2, warmup=1):
    """Qwen2 prefill attention (configs 3 and 4) at one GPU: one step = the whole 2000-token
    prompt in 256-token causal chunks (src/llm.zig:257-266) through every layer, for every
    sequence, on the tf32 tensor-core kernel over f32 K^T/V caches (distinct per layer)."""
    import torch

    from zwhisper_b200 import ops
    res = []
    g = torch.Generator(device=dev)
    g.manual_seed(2 + rank)
    ops.set_math("tf32", dev.index or 0)
    try:
        for cfg, B_all, layers, H, Hkv, d in (("configs[3] Qwen2.5-0.5B", 16, 24, 14, 2, 64),
                                              ("configs[4] Qwen2.5-1.5B", 64, 28, 12, 2, 128)):
            b0, b1 = shard(B_all, rank, world)
            B = b1 - b0
            n_prompt, chunk, n_ctx = 2000, 256, 2048
            kvw = Hkv * d
            kts = [torch.randn(B, Hkv, d, n_ctx, generator=g, device=dev) for _ in range(layers)]
            vs = [torch.randn(B, n_ctx, kvw, generator=g, device=dev) for _ in range(layers)]
            chunks = []
            for p0 in range(0, n_prompt, chunk):
                n_q = min(chunk, n_prompt - p0)
                q = torch.randn(B, n_q, H * d, generator=g, device=dev)
                sh = ops.AttnShape(n_q, p0 + n_q, H, Hkv, d, H * d, kvw, H * d, True, n_ctx)
                chunks.append((sh, q, torch.empty_like(q), (n_q * H * d, Hkv * d * n_ctx, n_ctx * kvw, n_q * H * d)))

            def step(kts=kts, vs=vs, chunks=chunks, B=B):
                for layer in range(len(kts)):
                    for sh, q, o, bs in chunks:
                        ops.attention_dev(q, kts[layer], vs[layer], sh, o, n_batch=B, batch_strides=bs)
            for _ in range(warmup):
                step()
            torch.cuda.synchronize()
            t = max_over_ranks(time_cuda(step, steps) / steps, world)
            ops.sync()
            pairs = n_prompt * (n_prompt + 1) // 2
            flops = 4 * d * H * layers * pairs * B_all
            peak = tc_peak / 2
            res.append({"workload": f"{cfg} prefill attention: {n_prompt}-token prompt in {chunk}-token causal "
                                    f"chunks, {B_all} sequences ({B} per GPU) x {layers} layers, tf32 tensor cores "
                                    "over f32 caches",
                        "metric": "qwen_prefill_attention_tok_per_s", "value": B_all * n_prompt / t, "unit": "tok/s",
                        "ms_per_step": t * 1e3, "math": "tf32",
                        "roofline": {"bound": "tensor", "achieved": flops / world / t / 1e12, "peak": peak,
                                     "unit": "TFLOP/s", "frac": flops / world / t / 1e12 / peak, "per": "GPU",
                                     "peak_source": f"{peak_kind} bf16 (burst) / 2: dense tf32 runs at half the "
                                                    "bf16 rate", "traffic": None,
                                     "flops_per_step": flops}})
            del kts, vs, chunks
            torch.cuda.empty_cache()
    finally:
        ops.set_math("f32", dev.index or 0)
    return res


def secondary_encoder(dev, tc_peak, peak_kind, rank, world, steps=3, warmup=2):
    """The whole Whisper small.en encoder on the device for 64 consecutive
    windows: mel rows, both convolutions, 12 pre-norm blocks (f16 tcgen05 GEMMs with fused
    bias / GELU / residual epilogues, the bf16 attention kernel) and ln_post
    (zwg_enc_forward_f16), random-init f16 weights N(0, 0.02^2), a synthetic mel."""
    import torch

    from oracle import whisper as W
    from zwhisper_b200 import ops
    hp = W.SMALL_EN
    B_all, n_ctx, ns, L = 64, hp.n_audio_ctx, hp.n_audio_state, hp.n_audio_layer
    b0, b1 = shard(B_all, rank, world)
    B = b1 - b0
    Wg = ops.EncoderWeightsF16(W.weights_dict(W.synth_model(hp, seed=0, encoder_only=True)), L, hp.n_audio_head,
                               device=dev.index or 0)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    mel = torch.randn(hp.n_mels, B * 2 * n_ctx, generator=g, device=dev) * 0.5
    out = torch.empty(B, n_ctx, ns, device=dev)
    scratch = torch.empty(Wg.scratch_bytes(B), dtype=torch.uint8, device=dev)
    t = max_over_ranks(time_graph(lambda: ops.encoder_forward(Wg, mel, B, out=out, scratch=scratch), steps,
                                  warmup) / steps, world)
    T = 2 * n_ctx
    flops = B_all * (2 * T * ns * 3 * hp.n_mels + 2 * n_ctx * ns * 3 * ns
                     + L * (2 * n_ctx * ns * 12 * ns + 4 * n_ctx * n_ctx * ns))
    del Wg, mel, out, scratch
    torch.cuda.empty_cache()
    return [{"workload": f"configs[2] Whisper small.en whole encoder (convolutions, {L} blocks, ln_post), {B_all} "
                         f"windows ({B} per GPU): f16 tcgen05 GEMMs + bf16 attention",
             "metric": "whisper_small_en_encoder_windows_per_s", "value": B_all / t, "unit": "windows/s",
             "ms_per_step": t * 1e3,
             "math": "f16 GEMM operands (activations rounded to f16), bf16 attention operands, f32 accumulation",
             "roofline": {"bound": "tensor", "achieved": flops / world / t / 1e12, "peak": tc_peak, "unit": "TFLOP/s",
                          "frac": flops / world / t / 1e12 / tc_peak, "peak_source": f"{peak_kind} bf16 (burst); f16 "
                          "runs at the bf16 rate", "traffic": None, "flops_per_step": flops, "per": "GPU"}}]


def secondary_q8(dev, hbm_peak, steps=20, warmup=3):
    """Q8 projections of one decode step at one GPU (the "next" row around the attention):
    every Qwen2.5-1.5B linear of all 28 layers for one sequence (q, k, v, o, gate, up, down:
    the reference's batch of one, src/llm.zig:179-216), and the Whisper base.en logits
    product (51864 x 512, src/decoder.zig:412-413). Weights are int8 blocks of 32 with f32
    scales (1.125 B per weight), distinct per layer; the bytes are the weight bytes read."""
    import torch

    from zwhisper_b200 import ops
    res = []
    g = torch.Generator(device=dev)
    g.manual_seed(4)

    def q8w(n, k):
        w = torch.randn(n, k, generator=g, device=dev) * 0.02
        return ops.quantize_q8(w)

    hidden, inter, kvw, layers = 1536, 8960, 256, 28
    shapes = [(hidden, hidden), (kvw, hidden), (kvw, hidden), (hidden, hidden), (inter, hidden), (inter, hidden),
              (hidden, inter)]
    ws = [[q8w(n, k) for (n, k) in shapes] for _ in range(layers)]
    xs = {k: torch.randn(1, k, generator=g, device=dev) for k in (hidden, inter)}
    outs = {n: torch.empty(1, n, device=dev) for n in (hidden, kvw, inter)}

    def step():
        for lw in ws:
            for (n, k), (q, sc) in zip(shapes, lw):
                ops.linear_q8(xs[k], q, sc, out=outs[n])
    t = time_graph(step, steps, warmup) / steps
    byts = layers * sum(n * k * 1.125 for n, k in shapes)
    res.append({"workload": "Qwen2.5-1.5B decode-step projections, 1 sequence x 28 layers x 7 Q8 linears "
                            "(q/k/v/o/gate/up/down), int8 blocks of 32 + f32 scales",
                "metric": "q8_projection_weight_GBps", "value": byts / t / 1e9, "unit": "GB/s", "math": "f32",
                "ms_per_step": t * 1e3,
                "roofline": {"bound": "hbm", "achieved": byts / t / 1e9, "peak": hbm_peak, "unit": "GB/s",
                             "frac": byts / t / 1e9 / hbm_peak, "traffic": None, "bytes_per_step": byts}})
    del ws
    q, sc = q8w(51864, 512)
    x1 = torch.randn(1, 512, generator=g, device=dev)
    o1 = torch.empty(1, 51864, device=dev)
    t = time_graph(lambda: ops.linear_q8(x1, q, sc, out=o1), steps, warmup) / steps
    byts = 51864 * 512 * 1.125
    res.append({"workload": "Whisper base.en logits, 51864 x 512 Q8 weights, 1 token",
                "metric": "q8_logits_weight_GBps", "value": byts / t / 1e9, "unit": "GB/s", "ms_per_step": t * 1e3,
                "math": "f32",
                "roofline": {"bound": "hbm", "achieved": byts / t / 1e9, "peak": hbm_peak, "unit": "GB/s",
                             "frac": byts / t / 1e9 / hbm_peak, "traffic": None, "bytes_per_step": byts}})
    torch.cuda.empty_cache()
    return res


QWEN15 = dict(n_layer=28, n_head=12, n_head_kv=2, d=128, n_ff=8960, n_vocab=151936, eps=1e-6)


def qwen15_weights(dev, seed=5, n_layer=None):
    """Random Qwen2.5-1.5B weights in Q8 on the device (configs[4]: N(0, 0.02^2), tied
    embedding/output), distinct per layer so a step's weight stream (1.74 GB) is far above L2."""
    import torch

    from zwhisper_b200 import ops
    c = QWEN15
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    ne, kvw = c["n_head"] * c["d"], c["n_head_kv"] * c["d"]

    def q8w(n, k):
        return ops.quantize_q8(torch.randn(n, k, generator=g, device=dev) * 0.02)

    def vec(n, mean, sd):
        return mean + torch.randn(n, generator=g, device=dev) * sd

    layers = [{"attn_norm": vec(ne, 1.0, 0.1), "wq": q8w(ne, ne), "wk": q8w(kvw, ne), "wv": q8w(kvw, ne),
               "bq": vec(ne, 0.0, 0.1), "bk": vec(kvw, 0.0, 0.1), "bv": vec(kvw, 0.0, 0.1), "wo": q8w(ne, ne),
               "ffn_norm": vec(ne, 1.0, 0.1), "w_gate": q8w(c["n_ff"], ne), "w_up": q8w(c["n_ff"], ne),
               "w_down": q8w(ne, c["n_ff"])} for _ in range(n_layer or c["n_layer"])]
    embd = q8w(c["n_vocab"] if n_layer is None else 64, ne)
    return ops.LlmWeightsQ8(layers, embd, None, vec(ne, 1.0, 0.1), c["eps"], device=dev.index or 0)


def qwen15_step_fn(W, B, n_ctx, n_past, dev, seed=6):
    """One greedy decode step of B sequences through the C ABI (zwg_llm_forward_q8 then
    zwg_llm_greedy), the chosen token written back as the next step's input."""
    import torch

    from zwhisper_b200 import ops
    c = QWEN15
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    st = ops.LlmState(c["n_layer"], B, c["n_head"], c["n_head_kv"], c["d"], n_ctx, rope_base=1e6,
                      device=dev.index or 0)
    tok = torch.randint(0, c["n_vocab"], (B, 1), generator=g, device=dev, dtype=torch.int32)
    recent = torch.randint(0, c["n_vocab"], (B, 64), generator=g, device=dev, dtype=torch.int32)
    x = torch.empty(B, 1, W.n_embd, device=dev)
    logits = torch.empty(B, W.n_vocab, device=dev)
    scratch = st.scratch(1, W.n_ff)

    def step():
        st.forward_q8(W, tok, n_past, x=x, logits=logits, scratch=scratch)
        ops.llm_greedy(logits, recent, n_recent=64, window=64, penalty=1.1, out=tok.view(-1))
    return st, step


def whisper_base_decoder(dev, seed=7):
    """Random Whisper base.en decoder weights on the device (configs[1]: n_state 512, 8 heads,
    6 layers, vocab 51864; N(0, 0.02^2) matrices quantized to Q8, LayerNorm gains 1)."""
    import torch

    from zwhisper_b200 import ops
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    ns, nv, nl, nctx = 512, 51864, 6, 448

    def r(*shape):
        return torch.randn(*shape, generator=g, device=dev) * 0.02

    t = {"decoder.token_embedding.weight": r(nv, ns), "decoder.positional_embedding": r(nctx, ns),
         "decoder.ln.weight": torch.ones(ns, device=dev), "decoder.ln.bias": torch.zeros(ns, device=dev)}
    for i in range(nl):
        p = f"decoder.blocks.{i}."
        for ln in ("attn_ln", "cross_attn_ln", "mlp_ln"):
            t[p + ln + ".weight"] = torch.ones(ns, device=dev)
            t[p + ln + ".bias"] = torch.zeros(ns, device=dev)
        for a in ("attn", "cross_attn"):
            for m in ("query", "key", "value", "out"):
                t[p + f"{a}.{m}.weight"] = r(ns, ns)
                t[p + f"{a}.{m}.bias"] = r(ns)
        t[p + "mlp.0.weight"], t[p + "mlp.0.bias"] = r(4 * ns, ns), r(4 * ns)
        t[p + "mlp.2.weight"], t[p + "mlp.2.bias"] = r(ns, 4 * ns), r(ns)
    W = ops.DecoderWeightsQ8(t, nl, device=dev.index or 0)
    del t
    return W


def secondary_step(dev, hbm_peak, rank, world, steps=10, warmup=3):
    """The whole Qwen2.5-1.5B greedy decode step on the device (the "next" rows around the
    attention, src/llm.zig:169-216, 313-321): embedding, 28 layers of RMSNorm, Q8 q/k/v with
    bias + RoPE + K^T/V append in one launch, decode attention over n_kv = 2256, wo +
    residual, RMSNorm, gate/up + SiLU*up in one launch, w_down + residual; final norm,
    151936-row logits and the penalized argmax, the token fed back on the device. B = 1 (the
    reference's own generate loop) and B = 64 (configs[4]'s batch). Algorithmic bytes: the
    Q8 weights once (1.74 GB with the tied output matrix) plus each sequence's K/V reads."""
    import torch
    c = QWEN15
    W = qwen15_weights(dev)
    n_ctx, n_kv = 2560, 2256
    wbytes = (c["n_layer"] * (2 * 1536 * 1536 + 2 * 256 * 1536 + 3 * c["n_ff"] * 1536) + c["n_vocab"] * 1536) * 1.125
    res = []
    from zwhisper_b200 import ops
    # one sequence (the reference's own generate loop) on one GPU; configs[4]'s 64 sequences
    # sharded over the ranks, each GPU holding all the weights
    for B_all in ((1, 64) if world == 1 else (64,)):
        b0, b1 = shard(B_all, rank, world)
        B = b1 - b0
        st, step = qwen15_step_fn(W, B, n_ctx, n_kv - 1, dev, seed=6 + rank)
        kv = B * c["n_layer"] * n_kv * c["n_head_kv"] * c["d"] * 2 * 4
        byts = wbytes + kv   # per GPU
        # math "tf32" changes only the attention (the tcgen05 decode kernel)
        for math in ("f32", "tf32"):
            ops.set_math(math, dev.index or 0)
            try:
                t = max_over_ranks(time_graph(step, steps, warmup) / steps, world)
            finally:
                ops.set_math("f32", dev.index or 0)
            res.append({"workload": f"Qwen2.5-1.5B greedy decode step on the device, {B_all} sequence(s) ({B} per "
                                    f"GPU) x 28 layers + logits (vocab 151936) + penalized argmax, Q8 weights, "
                                    f"n_kv={n_kv}, attention math {math}",
                        "metric": "qwen_decode_step_tok_per_s", "value": B_all / t, "unit": "tok/s",
                        "ms_per_step": t * 1e3, "math": f"f32 projections, {math} attention",
                        "roofline": {"bound": "hbm", "achieved": byts / t / 1e9, "peak": hbm_peak, "unit": "GB/s",
                                     "frac": byts / t / 1e9 / hbm_peak, "traffic": None, "bytes_per_step": byts,
                                     "per": "GPU"}})
        st.close()
        torch.cuda.empty_cache()
    del W
    torch.cuda.empty_cache()
    # the Whisper base.en decoder step: 32 windows, 6 layers, 224 of 448 cache
    # positions filled, cross-attention over 1500 frames, Q8 weights, logits and argmax
    B_all, n_past, na, ns = 32, 224, 1500, 512
    b0, b1 = shard(B_all, rank, world)
    B = b1 - b0
    Wd = whisper_base_decoder(dev)
    from zwhisper_b200 import ops
    st = ops.DecoderState(6, B, ns, 8, 448, na, device=dev.index or 0)
    g = torch.Generator(device=dev)
    g.manual_seed(8 + rank)
    for w in range(B):
        st.set_audio_q8(Wd, w, torch.randn(na, ns, generator=g, device=dev))
    tok = torch.randint(0, 51864, (B, 1), generator=g, device=dev, dtype=torch.int32)
    x = torch.empty(B, 1, ns, device=dev)
    logits = torch.empty(B, 51864, device=dev)
    scratch = st.scratch(1)

    def wstep():
        st.forward_q8(Wd, tok, n_past, x=x, logits=logits, scratch=scratch)
        ops.llm_greedy(logits, penalty=1.0, out=tok.view(-1))
    t = max_over_ranks(time_graph(wstep, steps, warmup) / steps, world)
    # per layer q, k, v, o, cq, co (n_state^2 each) and the two mlp matrices (4 n_state^2
    # each); ck and cv are read only by set_audio
    wbytes = (6 * (6 * ns * ns + 8 * ns * ns) + 51864 * ns) * 1.125
    kv = B * 6 * (n_past + 1 + na) * ns * 4 * 2
    byts = wbytes + kv   # per GPU
    res.append({"workload": f"Whisper base.en decoder step on the device (configs[1]): {B_all} windows ({B} per GPU) "
                            f"x 6 layers (self over {n_past + 1} of 448, cross over {na}) + logits (vocab 51864) + "
                            f"argmax, Q8 weights",
                "metric": "whisper_decoder_step_tok_per_s", "value": B_all / t, "unit": "tok/s",
                "ms_per_step": t * 1e3, "math": "f32",
                "roofline": {"bound": "hbm", "achieved": byts / t / 1e9, "peak": hbm_peak, "unit": "GB/s",
                             "frac": byts / t / 1e9 / hbm_peak, "traffic": None, "bytes_per_step": byts,
                             "per": "GPU"}})
    st.close()
    del Wd
    torch.cuda.empty_cache()
    return res


def run_ours(args, rank, world, local):
    import numpy as np
    import torch

    from zwhisper_b200 import _lib, ops
    hbm_peak, tc_peak, peak_kind = load_peaks()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w0, w1 = shard(WINDOWS, rank, world)
    nw = w1 - w0
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)

    def rand_bf16():
        return (torch.randn(nw, N_CTX, N_STATE, generator=g, device=dev, dtype=torch.float32) * SIGMA).to(torch.bfloat16)

    layers = [(rand_bf16(), rand_bf16(), rand_bf16()) for _ in range(N_LAYER)]
    out = torch.empty(nw, N_CTX, N_STATE, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def step():
        for q, k, v in layers:
            ops.enc_attn_bf16(q, k, v, N_HEAD, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.check(_lib.load().zwg_sync())
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    t = time_cuda(step, args.steps, stream)
    clk = clocks.stop()
    _lib.check(_lib.load().zwg_sync())
    barrier(world)
    t_max = max_over_ranks(t, world)
    value = WINDOWS * args.steps / t_max
    launches = args.steps * N_LAYER
    per_launch = t / launches
    flops_launch = FLOP_PER_WINDOW_LAYER * nw
    achieved = flops_launch / per_launch / 1e12

    # ---- end to end through the C-ABI drop-in with pinned host buffers
    e2e_steps = max(1, args.e2e_steps)
    nel = nw * N_CTX * N_STATE
    hq = torch.empty(nel, dtype=torch.float32, pin_memory=True)
    hk = torch.empty(nel, dtype=torch.float32, pin_memory=True)
    hv = torch.empty(nel, dtype=torch.float32, pin_memory=True)
    ho = torch.empty(nel, dtype=torch.float32, pin_memory=True)
    hq.copy_(layers[0][0].float().reshape(-1).cpu())
    hk.copy_(layers[0][1].float().reshape(-1).cpu())
    hv.copy_(layers[0][2].float().reshape(-1).cpu())
    del layers
    torch.cuda.empty_cache()
    _lib.ensure_init(local)
    ops.set_math("bf16", local)
    sh = ops.mha_shape(N_CTX, N_CTX, N_STATE, N_HEAD, False)
    c_sh = sh.to_c()
    c_b = _lib.BatchC(nw, N_CTX * N_STATE, N_CTX * N_STATE, N_CTX * N_STATE, N_CTX * N_STATE)
    import ctypes
    lib = _lib.load()

    def e2e_step():
        for _ in range(N_LAYER):
            _lib.check(lib.zwg_attention_batch_host(ctypes.byref(c_sh), ctypes.byref(c_b), hq.data_ptr(),
                                                    hk.data_ptr(), hv.data_ptr(), ho.data_ptr()))
    e2e_step()  # warm-up (allocates the context's staging)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    t_e2e = time.perf_counter() - t0
    barrier(world)
    t_e2e = max_over_ranks(t_e2e, world)
    ops.set_math("f32", local)
    e2e_value = WINDOWS * e2e_steps / t_e2e
    h2d = N_LAYER * 3 * WINDOWS * N_CTX * N_STATE * 4
    d2h = N_LAYER * WINDOWS * N_CTX * N_STATE * 4
    # the bound the host-pointer contract sets: this step's bytes over the measured copy rates
    # (pinned memory, one direction at a time, one Q tensor of this rank's windows, CUDA events)
    dbuf = torch.empty(nel, dtype=torch.float32, device=dev)
    h2d_gbs = nel * 4 / time_cuda(lambda: dbuf.copy_(hq, non_blocking=True), 3) * 3 / 1e9
    d2h_gbs = nel * 4 / time_cuda(lambda: ho.copy_(dbuf, non_blocking=True), 3) * 3 / 1e9
    t_bound = max(h2d / world / (h2d_gbs * 1e9), d2h / world / (d2h_gbs * 1e9))
    # the same copies in both directions at once (two streams): the rates the overlapped
    # pipeline actually gets; the bound then runs the copies out beside the copies in and
    # the rest of the copies in alone
    dbuf2 = torch.empty_like(dbuf)
    sa, sb = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    with torch.cuda.stream(sa):
        ev[0].record(sa)
        for _ in range(3):
            dbuf.copy_(hq, non_blocking=True)
        ev[1].record(sa)
    with torch.cuda.stream(sb):
        ev[2].record(sb)
        for _ in range(3):
            ho.copy_(dbuf2, non_blocking=True)
        ev[3].record(sb)
    torch.cuda.synchronize()
    h2d_c = 3 * nel * 4 / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9
    d2h_c = 3 * nel * 4 / (ev[2].elapsed_time(ev[3]) * 1e-3) / 1e9
    del dbuf, dbuf2
    b_in, b_out = h2d / world, d2h / world
    t_in_c, t_out_c = b_in / (h2d_c * 1e9), b_out / (d2h_c * 1e9)
    if t_out_c <= t_in_c:
        t_bound_c = t_out_c + (b_in - h2d_c * 1e9 * t_out_c) / (h2d_gbs * 1e9)
    else:
        t_bound_c = t_in_c + (b_out - d2h_c * 1e9 * t_in_c) / (d2h_gbs * 1e9)
    del hq, hk, hv, ho

    secondary = None
    cpu = None
    if not args.no_secondary:
        # every rank runs the same workloads (its shard of each) and the same max-over-ranks
        # reductions; the one-sequence Q8 projections run on one GPU only
        secondary = (secondary_decode(dev, hbm_peak, rank, world) +
                     secondary_prefill(dev, tc_peak, peak_kind, rank, world) +
                     secondary_encoder(dev, tc_peak, peak_kind, rank, world) +
                     (secondary_q8(dev, hbm_peak) if world == 1 else []) +
                     secondary_step(dev, hbm_peak, rank, world))
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_windows_per_s(min_seconds=args.cpu_seconds)
        cpu["cpu"] = cpu_model()
        cpu["reference_binary"] = reference_binary_baseline(cpu["cores"])

    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "whisper small.en encoder self-attention (configs[2]): 64 windows x 12 layers x "
                               "12 heads, n_ctx 1500, d 64, bf16 operands, f32 softmax/accumulation, f32 out",
                   "windows": WINDOWS, "n_ctx": N_CTX, "n_state": N_STATE, "n_head": N_HEAD, "n_layer": N_LAYER,
                   "parallelism": f"windows sharded {WINDOWS // world if WINDOWS % world == 0 else 'uneven'} "
                                  f"per GPU over {world}, no collective",
                   "l2": "inputs larger than L2: distinct Q/K/V per layer, 5.3 GB per step"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "copy_bound": {"h2d_gbs": h2d_gbs, "d2h_gbs": d2h_gbs, "windows_per_s": WINDOWS / t_bound,
                               "note": "the step's copies at the pinned copy rates measured one direction at a "
                                       "time, directions overlapped",
                               "concurrent_h2d_gbs": h2d_c, "concurrent_d2h_gbs": d2h_c,
                               "windows_per_s_concurrent": WINDOWS / t_bound_c,
                               "concurrent_note": "the rates of both directions copying at once; the copies out "
                                                  "beside the copies in, the rest of the copies in alone"},
                "path": "zwg_attention_batch_host (ops.attentionEx drop-in), math mode bf16, pinned f32 host "
                        "buffers, copies in / conversion + tcgen05 kernel / copies out on three streams",
                "steps": e2e_steps},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": achieved / tc_peak, "peak_source": f"{peak_kind} bf16 (burst)",
                     "kernel": "enc_attn_tc_kernel", "flops_per_launch": flops_launch,
                     "avg_launch_ms": per_launch * 1e3,
                     "traffic": profiled_traffic("enc_attn_tc_small_en.txt", nw),
                     "traffic_note": "ncu DRAM read+write of a 16-window launch scaled to this launch's windows"},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu")}
        if cpu.get("reference_binary"):
            line["cpu_baseline"]["reference_binary"] = cpu["reference_binary"]
    if secondary is not None:
        line["secondary"] = secondary
        # the same figures in short, last in the line
        line["secondary_summary"] = [
            {"metric": r["metric"], "math": r.get("math"), "value": round(r["value"], 1), "unit": r["unit"],
             "frac": round(r["roofline"]["frac"], 3), "of": r["roofline"]["unit"]} for r in secondary]
    print(json.dumps(line), flush=True)


def run_kernel_case(args):
    """One kernel on a small case, for ncu captures: `enc_tc` = the tcgen05 encoder kernel
    on 16 small.en windows (one layer, 184 MB of inputs and output, above L2); `decode_qwen`
    = the split-K decode kernel on 16 Qwen2.5-1.5B sequences (n_kv 2256, K^T cache 2560);
    `decode_qwen05` = the same on 16 Qwen2.5-0.5B sequences (d 64, n_kv 2128);
    `decode_qwen_b1` = the same on one Qwen2.5-1.5B sequence (the reference's own batch);
    `decode_tc_qwen64` / `decode_tc_qwen_b1` = the tf32 tcgen05 decode kernel on 64 / one
    Qwen2.5-1.5B sequences (296 MB / 4.6 MB of K/V per launch);
    `decode_whisper` = the split-K kernel on 32 base.en windows of cross-attention;
    `prefill_qwen` = the tf32 prefill kernel on the last 208-query chunk of a 2000-token
    prompt for 64 Qwen2.5-1.5B sequences (one layer, 268 MB of K^T/V, above L2);
    `prefill_qwen05` = the same chunk for 16 Qwen2.5-0.5B sequences (d 64, config 3's shape;
    33.5 MB of K^T/V);
    `q8_logits` = the Q8 linear kernel on the Whisper base.en logits product (51864 x 512);
    `step_qwen15` = one whole Qwen2.5-1.5B greedy decode step for one sequence (n_kv 2256),
    every kernel of the step in launch order (about 200 launches); `step_whisper_base` = one
    Whisper base.en decoder step for 32 windows (config 1: 224 cached positions, 1500 audio
    frames); `pair_qwen15` = the two
    paired-row Q8 kernels of one Qwen2.5-1.5B layer for one sequence: q/k/v + RoPE + cache
    append (3.5 MB of weights) then gate/up + SiLU*up (31 MB)."""
    import torch

    from zwhisper_b200 import ops
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    if args.kernel_case == "enc_tc":
        B = 16
        q, k, v = ((torch.randn(B, N_CTX, N_STATE, generator=g, device=dev) * SIGMA).to(torch.bfloat16) for _ in range(3))
        out = torch.empty(B, N_CTX, N_STATE, device=dev)

        def fn():
            ops.enc_attn_bf16(q, k, v, N_HEAD, out)
        work = f"{FLOP_PER_WINDOW_LAYER * B / 1e9:.1f} GFLOP per launch"
    elif args.kernel_case in ("decode_qwen", "decode_qwen05", "decode_qwen_b1", "decode_tc_qwen64", "decode_tc_qwen_b1",
                              "decode_tc_qwen05"):
        B, H, Hkv, d, n_ctx, n_kv = {"decode_qwen": (16, 12, 2, 128, 2560, 2256),
                                     "decode_qwen05": (16, 14, 2, 64, 2560, 2128),
                                     "decode_qwen_b1": (1, 12, 2, 128, 2560, 2256),
                                     "decode_tc_qwen64": (64, 12, 2, 128, 2560, 2256),
                                     "decode_tc_qwen_b1": (1, 12, 2, 128, 2560, 2256),
                                     "decode_tc_qwen05": (16, 14, 2, 64, 2560, 2128)}[args.kernel_case]
        if args.kernel_case.startswith("decode_tc"):
            ops.set_math("tf32")
        q = torch.randn(B, H * d, generator=g, device=dev)
        kt = torch.randn(B, Hkv, d, n_ctx, generator=g, device=dev)
        v = torch.randn(B, n_ctx, Hkv * d, generator=g, device=dev)
        out = torch.empty_like(q)
        sh = ops.AttnShape(1, n_kv, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
        ws = torch.empty(max(1, ops.attention_workspace_bytes(sh, B)), dtype=torch.uint8, device=dev)

        def fn():
            ops.attention_dev(q, kt, v, sh, out, n_batch=B, workspace=ws)
        work = f"{B * n_kv * Hkv * d * 8 / 1e6:.1f} MB of K/V per launch"
    elif args.kernel_case == "q8_logits":
        n, k = 51864, 512
        w = torch.randn(n, k, generator=g, device=dev) * 0.02
        q, sc = ops.quantize_q8(w)
        del w
        x = torch.randn(1, k, generator=g, device=dev)
        out = torch.empty(1, n, device=dev)

        def fn():
            ops.linear_q8(x, q, sc, out=out)
        work = f"{n * k * 1.125 / 1e6:.1f} MB of Q8 weights per launch"
    elif args.kernel_case == "step_qwen15":
        W = qwen15_weights(dev)
        st, fn = qwen15_step_fn(W, 1, 2560, 2255, dev)
        work = "one decode step: 1.74 GB of Q8 weights + 129 MB of K/V"
    elif args.kernel_case == "step_whisper_base":
        B, n_past, na, ns = 32, 224, 1500, 512
        Wd = whisper_base_decoder(dev)
        st = ops.DecoderState(6, B, ns, 8, 448, na, device=0)
        for w in range(B):
            st.set_audio_q8(Wd, w, torch.randn(na, ns, generator=g, device=dev))
        tok = torch.randint(0, 51864, (B, 1), generator=g, device=dev, dtype=torch.int32)
        x = torch.empty(B, 1, ns, device=dev)
        logits = torch.empty(B, 51864, device=dev)
        scratch = st.scratch(1)

        def fn():
            st.forward_q8(Wd, tok, n_past, x=x, logits=logits, scratch=scratch)
            ops.llm_greedy(logits, penalty=1.0, out=tok.view(-1))
        work = "one decoder step for 32 windows: 27 MB of Q8 weights + 259 MB of K/V"
    elif args.kernel_case == "pair_qwen15":
        W = qwen15_weights(dev, n_layer=1)
        st = ops.LlmState(1, 1, QWEN15["n_head"], QWEN15["n_head_kv"], QWEN15["d"], 2560, device=0)
        h = torch.randn(1, 1, W.n_embd, generator=g, device=dev)
        qo = torch.empty_like(h)
        L = W.layers[0]
        gate = torch.empty(1, W.n_ff, device=dev)

        def fn():
            st.qkv_q8(0, h, W, 2255, q_out=qo)
            ops.linear_q8_silu_mul(h.view(1, -1), L["w_gate"], L["w_up"], out=gate)
        work = f"{(1536 + 512) * 1536 * 1.125 / 1e6:.1f} + {2 * 8960 * 1536 * 1.125 / 1e6:.1f} MB of Q8 weights"
    elif args.kernel_case == "q8_gateup64":
        # the gate/up SiLU pair of a Qwen2.5-1.5B layer for 64 sequences (the tiled Q8 product)
        m, n_ff, k = 64, 8960, 1536
        xg = torch.randn(m, k, generator=g, device=dev)
        qg = torch.randint(-127, 128, (n_ff, k), generator=g, device=dev, dtype=torch.int8)
        qu = torch.randint(-127, 128, (n_ff, k), generator=g, device=dev, dtype=torch.int8)
        sc = torch.rand(n_ff, k // 32, generator=g, device=dev) * 1e-3
        og = torch.empty(m, n_ff, device=dev)

        def fn():
            ops.linear_q8_silu_mul(xg, (qg, sc), (qu, sc), out=og)
        work = f"{2 * 2 * m * n_ff * k / 1e9:.2f} GFLOP, {2 * n_ff * k * 1.125 / 1e6:.1f} MB of Q8 weights per launch"
    elif args.kernel_case == "gemm_mlp2":
        # the MLP down-projection of 16 small.en windows into the f32 residual stream
        B, M, N, K = 16, 1500, 768, 3072
        a = torch.randn(B, M, K, generator=g, device=dev).half()
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
        bias = torch.zeros(N, device=dev)
        out = torch.zeros(B, M, N, device=dev)

        def fn():
            ops.gemm_f16(a, w, bias=bias, accumulate=True, out=out)
        work = f"{2 * B * M * N * K / 1e9:.1f} GFLOP per launch"
    elif args.kernel_case == "encoder_small_en":
        from oracle import whisper as Wh
        hp = Wh.SMALL_EN
        B = 4
        Wg = ops.EncoderWeightsF16(Wh.weights_dict(Wh.synth_model(hp, seed=0, encoder_only=True)), hp.n_audio_layer,
                                   hp.n_audio_head)
        mel = torch.randn(hp.n_mels, B * 3000, generator=g, device=dev) * 0.5
        out = torch.empty(B, hp.n_audio_ctx, hp.n_audio_state, device=dev)
        scratch = torch.empty(Wg.scratch_bytes(B), dtype=torch.uint8, device=dev)

        def fn():
            ops.encoder_forward(Wg, mel, B, out=out, scratch=scratch)
        work = f"the whole small.en encoder for {B} windows"
    elif args.kernel_case in ("prefill_qwen", "prefill_qwen05"):
        B, H, Hkv, d, n_ctx, n_past, n_q = ((64, 12, 2, 128, 2048, 1792, 208) if args.kernel_case == "prefill_qwen"
                                            else (16, 14, 2, 64, 2048, 1792, 208))
        q = torch.randn(B, n_q, H * d, generator=g, device=dev)
        kt = torch.randn(B, Hkv, d, n_ctx, generator=g, device=dev)
        v = torch.randn(B, n_ctx, Hkv * d, generator=g, device=dev)
        out = torch.empty_like(q)
        sh = ops.AttnShape(n_q, n_past + n_q, H, Hkv, d, H * d, Hkv * d, H * d, True, n_ctx)
        ops.set_math("tf32")

        def fn():
            ops.attention_dev(q, kt, v, sh, out, n_batch=B)
        pairs = sum(n_past + i + 1 for i in range(n_q))
        work = f"{4 * d * H * pairs * B / 1e9:.1f} GFLOP per launch"
    else:
        B, ns = 32, 512
        q = torch.randn(B, 1, ns, generator=g, device=dev)
        k = torch.randn(B, 1500, ns, generator=g, device=dev)
        v = torch.randn(B, 1500, ns, generator=g, device=dev)
        out = torch.empty_like(q)
        sh = ops.mha_shape(1, 1500, ns, 8, False)
        ws = torch.empty(max(1, ops.attention_workspace_bytes(sh, B)), dtype=torch.uint8, device=dev)

        def fn():
            ops.attention_dev(q, k, v, sh, out, n_batch=B, workspace=ws)
        work = f"{B * 1500 * ns * 8 / 1e6:.1f} MB of K/V per launch"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    t = time_cuda(fn, args.steps)
    ops.sync()
    print(json.dumps({"kernel_case": args.kernel_case, "ms_per_launch": t / args.steps * 1e3, "work": work}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--kernel-case", choices=["enc_tc", "decode_qwen", "decode_qwen05", "decode_qwen_b1", "decode_tc_qwen64",
                                             "decode_tc_qwen_b1", "decode_whisper", "prefill_qwen", "prefill_qwen05",
                                             "q8_logits", "step_qwen15", "step_whisper_base", "pair_qwen15",
                                             "gemm_mlp2", "encoder_small_en", "q8_gateup64", "decode_tc_qwen05"],
                    default=None)
    args = ap.parse_args()
    if args.kernel_case:
        run_kernel_case(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup()
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
