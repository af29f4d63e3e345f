#!/usr/bin/env python
"""Decode throughput of the continuous-batching forward step on B200.

Workload (Llama-3-8B shape, random-init bf16 weights, seed 2): hidden 4096,
32 layers, 32 query / 8 KV heads, head_dim 128, SwiGLU 14336, vocab 128256,
RoPE theta 5e5, untied LM head.  256 concurrent requests per GPU, prompt
lengths lognormal(median 512, sigma 0.8) clipped to [32, 4096], token ids
uniform, 256 greedy output tokens each, a new request arriving as soon as
one finishes.  The engine starts in steady state: each initial request has a
random share (0..255) of its 256 tokens already generated, so finishes and
arrivals are spread over the steps.

A "step" is one scheduler step of the engine: all running requests decode
one token and newly arrived requests are prefilled in the same flat batch.
The metric counts generated tokens (one per scheduled sequence per step).

  value     device throughput: the timed steps, recorded once, replayed with
            their packed arrays already in HBM (no host work between steps)
  e2e       the same steps through the public StepEngine.step() API: host
            scheduling, packing, host->device copy of each step's arrays and
            device->host read of the sampled ids inside the timed region
  roofline  the dominant kernel, muk_gemm_bf16 (tensor-bound): every GEMM
            launch of the recorded eager steps timed with CUDA events;
            beside it paged decode attention of the running batch and of
            the isolated 128-sequence case (HBM-bound)

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                        [--workload c3|c2|c5] [--parallel replicas|tp|ep]
Under torchrun the ranks run one engine tensor-parallel by default for c3
(heads and MLP columns split over the GPUs; strong scaling of the same
256-request stream), and for the DeepForCausalLM workloads also distribute
the experts whole (--parallel ep; expert e on GPU e // (E/P)).
--parallel replicas lets every rank serve its own copy of the request stream
instead (no collective on the data path; value is the sum over ranks / max
time; weak scaling).
The c2 / c5 workloads are the DeepForCausalLM configurations (token-routed
MLP, INL dynamics, mu-guided attention, mu_clamp); c3 is the headline.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "complexity-inference_b200"))

METRIC = "decode tokens/s @256 ragged reqs; paged-attn HBM GB/s vs 8 TB/s roofline"
# The default workload is "c3"; "c2" and "c5" are the two DeepForCausalLM
# (token-routed MLP, INL dynamics, mu-guided attention, mu_clamp) workloads.
WORKLOADS = {
    "c3": dict(desc="Llama-3-8B-shape (H4096 L32 32/8 heads D128 I14336 V128256 theta5e5), "
                    "256 concurrent ragged requests, steady-state continuous batching, greedy",
               arch="llama", hidden=4096, layers=32, heads=32, kv=8, head_dim=128, inter=14336,
               experts=0, vocab=128256, theta=500000.0, eps=1e-5, seed=2, mu=False,
               concurrency=256, prompt=("lognormal", 512, 0.8, 32, 4096), out=256,
               sampling=(0.0, 0, 1.0), blocks=45000),
    "c2": dict(desc="DeepForCausalLM (H2048 L24 16/8 heads D128, 4 experts x 2816, V32000, "
                    "mu_clamp on), 64 concurrent requests, prompts U[64,512], 128 tokens at "
                    "T0.7 / top-k 50 / top-p 0.9",
               arch="deep", hidden=2048, layers=24, heads=16, kv=8, head_dim=128, inter=11264,
               experts=4, vocab=32000, theta=10000.0, eps=1e-6, seed=1, mu=True,
               concurrency=64, prompt=("uniform", 64, 512), out=128, sampling=(0.7, 50, 0.9),
               blocks=4000),
    "c5": dict(desc="scaled DeepForCausalLM (H4096 L32 32/8 heads D128, 8 experts x 3584, "
                    "V32000, mu_clamp on), 512 concurrent requests, prompts U[128,2048], "
                    "128 greedy tokens",
               arch="deep", hidden=4096, layers=32, heads=32, kv=8, head_dim=128, inter=28672,
               experts=8, vocab=32000, theta=10000.0, eps=1e-6, seed=4, mu=True,
               concurrency=512, prompt=("uniform", 128, 2048), out=128, sampling=(0.0, 0, 1.0),
               blocks=48000),
}
C3 = WORKLOADS["c3"]
# One ncu capture (dram__bytes_read.sum + dram__bytes_write.sum, clocks not
# locked) of the gate|up GEMM launch at the mean C3 step shape, beside that
# launch's algorithmic bytes (A + B + C).
GEMM_NCU_TRAFFIC = {"shape": "M857 N28672 K4096 (gate|up at the C3 mean step)",
                    "dram_bytes": 243.678e6 + 36.179e6, "algorithmic_bytes": 290.9e6}
WORKLOAD = C3["desc"]


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = float(d["bf16_tflops"])
        return float(d["hbm_gbs"]), burst, float(d.get("bf16_tflops_sustained", burst)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            # nvidia-smi's start-up (NVML init on every GPU) must not fall in
            # the timed region: wait for its first sample
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 10.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def mark(self) -> int:
        """Index of the next sample (bracket a timed region with two marks)."""
        return len(self.lines)

    def summary(self, lo: int = 0, hi: int | None = None):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[lo:hi]:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def model_config(wl=C3):
    from mu_b200.core.config import ModelConfig

    return ModelConfig(vocab_size=wl["vocab"], hidden_size=wl["hidden"],
                       intermediate_size=wl["inter"], num_hidden_layers=wl["layers"],
                       num_attention_heads=wl["heads"], num_key_value_heads=wl["kv"],
                       head_dim=wl["head_dim"], max_position_embeddings=8192,
                       rope_theta=wl["theta"], rms_norm_eps=wl["eps"],
                       num_experts=max(wl["experts"], 1), tie_word_embeddings=False)


class Arrivals:
    def __init__(self, seed: int, wl=C3):
        self.rng = np.random.default_rng(seed)
        self.wl = wl
        self.n = 0

    def prompt(self):
        kind, *a = self.wl["prompt"]
        if kind == "lognormal":
            med, sig, lo, hi = a
            L = int(np.clip(np.round(self.rng.lognormal(math.log(med), sig)), lo, hi))
        else:
            L = int(self.rng.integers(a[0], a[1] + 1))
        return self.rng.integers(0, self.wl["vocab"], L).tolist()

    def new_request(self, engine, params_cls, already=0):
        prompt = self.prompt()
        if already:
            prompt = prompt + self.rng.integers(0, self.wl["vocab"], already).tolist()
        self.n += 1
        t, k, p = self.wl["sampling"]
        sp = params_cls(temperature=t, top_k=k, top_p=p, repetition_penalty=1.0,
                        max_tokens=self.wl["out"] - already)
        return engine.add_request(prompt, sp, f"q{self.n}")


def build(rank: int, tp: int = 1, wl=C3, ep: bool = False, align: int = 0):
    from mu_b200.core.config import CacheConfig, EngineConfig, MuConfig, SchedulerConfig
    from mu_b200.models.weights import random_state_dict
    from mu_b200.serving.engine import StepEngine
    from mu_b200.serving.worker import MuWorker

    cfg = model_config(wl)
    max_len = wl["prompt"][-1] + wl["out"] + 16
    # headroom over the expected KV (C3: 256 x ~830 tokens, 3x) for bursts of long prompts
    ec = EngineConfig(model=cfg, dtype="bfloat16", tensor_parallel_size=tp, expert_parallel=ep,
                      mu=MuConfig(enabled=wl["mu"]),
                      cache=CacheConfig(max_seq_len=max_len, block_size=16,
                                        max_num_blocks=wl["blocks"],
                                        max_num_seqs=wl["concurrency"]),
                      scheduler=SchedulerConfig(max_batch_size=wl["concurrency"],
                                                max_num_batched_tokens=8192,
                                                max_prefill_tokens=8192,
                                                step_token_alignment=align))
    sd = random_state_dict(cfg, wl["arch"], wl["seed"], device="cuda", dtype=torch.bfloat16,
                           include_unused=False)
    worker = MuWorker(ec, "cuda")
    worker.load_state_dict(wl["arch"], cfg, sd)
    del sd
    torch.cuda.empty_cache()
    engine = StepEngine(worker, ec)
    return engine, worker, ec


class Recorder:
    """Wraps worker.run_staged and the engine's sampler launch to keep, per
    step, the step's device arrays (decode inputs already filled in from the
    previous samples) and the sampler's device parameter blob, so the replay
    issues exactly the engine's launches from HBM-resident inputs."""

    def __init__(self, engine, worker):
        self.worker = worker
        self.sampler = engine.sampler
        self.orig = worker.run_staged
        self.orig_launch = engine.sampler.launch
        self.steps = []
        self.blobs = []
        self.on = False
        worker.run_staged = self.run_staged
        engine.sampler.launch = self.launch

    def run_staged(self, st, sampled=None):
        out = self.orig(st, sampled)
        if self.on:
            buf = self.worker.packer.dev[:st.end].clone()
            self.steps.append((dataclasses.replace(st, patch=0), buf))
        return out

    def launch(self, logits, request_ids, params, steps, token_rows=None, input_ids=None,
               num_tokens=0):
        h = self.orig_launch(logits, request_ids, params, steps, token_rows, input_ids,
                             num_tokens)
        if self.on:  # stream-ordered after the blob's host-to-device copy
            self.blobs.append((len(request_ids), num_tokens, self.sampler._blob_d.clone(),
                               all(p.temperature <= 0 for p in params)))
        return h


def steady_state_step(engine, arrivals, params_cls, outs=None):
    outs = engine.step() if outs is None else outs
    produced = sum(1 for o in outs if o.token_id >= 0)
    for o in outs:
        if o.finished:
            arrivals.new_request(engine, params_cls)
    return produced


def time_attention(worker, reps=10):
    """Decode attention of the current running batch, layer 0, timed alone."""
    from mu_b200 import kernels as K

    cache = worker.cache
    rids = [r for r in worker.active_requests]
    lens = np.array([cache.get_seq_len(r) for r in rids], dtype=np.int32)
    maxb = max(len(cache.block_table(r)) for r in rids)
    bt = np.zeros((len(rids), maxb), np.int32)
    for i, r in enumerate(rids):
        b = cache.block_table(r)
        bt[i, :len(b)] = b
    cfg = worker.model.config
    Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    B = len(rids)
    q = torch.randn(B, Hq * D, device="cuda").bfloat16()
    out = torch.empty_like(q)
    btd = torch.from_numpy(bt).cuda()
    sl = torch.from_numpy(lens).cuda()
    mx = int(lens.max())
    ws = torch.empty(K.decode_attn_workspace_size(B, Hq, D, mx) // 4 + 4, device="cuda")
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for layer in range(3):
        K.decode_attn(q, out, cache.k_cache(layer), cache.v_cache(layer), btd, sl, Hq, Hkv, D, mx,
                      workspace=ws)
    torch.cuda.synchronize()
    s.record()
    for i in range(reps):  # rotate layers so each launch streams fresh KV (>> L2)
        layer = i % cfg.num_hidden_layers
        K.decode_attn(q, out, cache.k_cache(layer), cache.v_cache(layer), btd, sl, Hq, Hkv, D, mx,
                      workspace=ws)
    e.record()
    torch.cuda.synchronize()
    t = s.elapsed_time(e) / reps * 1e-3
    byts = float(lens.sum()) * Hkv * D * 2 * 2
    return byts, t, B, int(lens.sum())


def time_attention_c4(reps=10, seed=3):
    """The isolated paged-attention decode case: 128 sequences, context
    U[1024, 32768], 32/8 heads, D 128, bf16 Q/K/V ~ N(0, 1), block size 16,
    every block table a slice of a random permutation of a pool of
    1.2 x the total tokens.  Returns (algorithmic bytes, seconds per launch,
    sequences, total context)."""
    from mu_b200 import kernels as K

    Hq, Hkv, D, bs, B = 32, 8, 128, 16, 128
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1024, 32768 + 1, B)
    nblk = (ctx + bs - 1) // bs
    pool = int(math.ceil(1.2 * ctx.sum() / bs))
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=g, dtype=torch.bfloat16)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=g, dtype=torch.bfloat16)
    perm = rng.permutation(pool)
    bt = np.zeros((B, int(nblk.max())), np.int32)
    i = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[i:i + n]
        i += n
    btd = torch.from_numpy(bt).cuda()
    sl = torch.from_numpy(ctx.astype(np.int32)).cuda()
    q = torch.randn(B, Hq * D, device="cuda", generator=g, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    mx = int(ctx.max())
    ws = torch.empty(K.decode_attn_workspace_size(B, Hq, D, mx) // 4 + 4, device="cuda")

    def fn():
        K.decode_attn(q, out, kc, vc, btd, sl, Hq, Hkv, D, mx, workspace=ws)

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):  # the 10.5 GB pool is far larger than L2
        fn()
    e.record()
    torch.cuda.synchronize()
    t = s.elapsed_time(e) / reps * 1e-3
    byts = float(ctx.sum()) * Hkv * D * 2 * 2
    del kc, vc
    torch.cuda.empty_cache()
    return byts, t, B, int(ctx.sum())


class GemmProbe:
    """Times every muk_gemm_bf16 launch with CUDA events on the launching stream."""

    def __init__(self):
        self.recs = []

    def __call__(self, flops):
        import contextlib

        @contextlib.contextmanager
        def cm():
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            yield
            e.record()
            self.recs.append((flops, s, e))

        return cm()

    def result(self):
        torch.cuda.synchronize()
        flops = sum(f for f, _, _ in self.recs)
        t = sum(s.elapsed_time(e) for _, s, e in self.recs) * 1e-3
        return flops, t, len(self.recs)


def time_gemms(worker, M=256, reps=10):
    """The decode-shape GEMMs of one layer (QKV, O, gate|up, down), back to back."""
    from mu_b200 import kernels as K
    from mu_b200.models.base import choose_split

    m = worker.model
    ws = m.ws
    H = m.config.hidden_size
    x = torch.randn(M, 2 * H, device="cuda").bfloat16()[:, :H]
    flops = 0
    Ls = [m.layers[i % len(m.layers)] for i in range(reps)]

    def run(L):
        K.gemm(x, L["wqkv"], ws.qkv, K.MUK_EPI_BF16, M=M)
        s = choose_split(M, H, ws.attn.shape[1], ws.part_rows)
        K.gemm(ws.attn, L["wo"], ws.part_view(s, M, H), K.MUK_EPI_F32, split_k=s, M=M)
        K.gemm(x, L["wgu"], ws.act, K.MUK_EPI_SWIGLU, M=M)
        s = choose_split(M, H, m.i_pad, ws.part_rows)
        K.gemm(ws.act, L["wd"], ws.part_view(s, M, H), K.MUK_EPI_F32, split_k=s, M=M)

    L0 = m.layers[0]
    for w in (L0["wqkv"], L0["wo"], L0["wgu"], L0["wd"]):
        flops += 2 * M * w.shape[0] * w.shape[1]
    run(L0)
    torch.cuda.synchronize()
    # pure-decode steps replay CUDA graphs in the engine, so the layers'
    # launches are captured and replayed here too (no host issue gaps)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(graph, stream=st):
            for L in Ls:
                run(L)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    del graph
    t = s.elapsed_time(e) / reps * 1e-3
    wbytes = sum(L0[k].numel() * 2 for k in ("wqkv", "wo", "wgu", "wd"))
    return flops, t, wbytes


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (numpy restatement of the reference path)
# ---------------------------------------------------------------------------
class CpuBaseline:
    """The reference algorithm on the host cores, via the oracle (numpy port).

    The reference decodes one request at a time (batch-1 forwards with a
    dense per-request KV cache).  Sample: one Llama-3-8B-shape layer (random
    f32 weights) decoding one token at context ``ctx`` per step, plus one
    LM-head matvec; the per-token time is scaled to 32 layers."""

    def __init__(self, ctx=830, seed=0):
        sys.path.insert(0, str(ROOT))
        import oracle as O

        H, Hq, Hkv, D, I, V = (C3["hidden"], C3["heads"], C3["kv"], C3["head_dim"], C3["inter"],
                               C3["vocab"])
        rng = np.random.default_rng(seed)

        def w(*s):
            return rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)

        p = {"embed_tokens.weight": w(64, H), "norm.weight": np.ones(H, np.float32),
             "layers.0.input_layernorm.weight": np.ones(H, np.float32),
             "layers.0.post_attention_layernorm.weight": np.ones(H, np.float32),
             "layers.0.self_attn.q_proj.weight": w(Hq * D, H),
             "layers.0.self_attn.k_proj.weight": w(Hkv * D, H),
             "layers.0.self_attn.v_proj.weight": w(Hkv * D, H),
             "layers.0.self_attn.o_proj.weight": w(H, Hq * D),
             "layers.0.mlp.gate_proj.weight": w(I, H), "layers.0.mlp.up_proj.weight": w(I, H),
             "layers.0.mlp.down_proj.weight": w(H, I)}
        shape = O.ModelShape("llama", H, 1, Hq, Hkv, D, 64, 1e-5, C3["theta"], tie=True,
                             max_pos=ctx + 4096)
        self.model = O.OracleModel(shape, p, O.MuCfg(False))
        self.past = [(rng.standard_normal((Hkv, ctx, D), dtype=np.float32),
                      rng.standard_normal((Hkv, ctx, D), dtype=np.float32))]
        self.lm = w(V, H)
        self.x = rng.standard_normal(H, dtype=np.float32)
        self.ctx = ctx
        self.sample = (f"1 of 32 layers x 1 decode token at ctx {ctx} + 1 LM-head matvec "
                       f"(numpy f32) per step, scaled to 32 layers")
        self.step()  # warm

    def step(self) -> float:
        """Seconds per generated token (one layer timed, scaled to the model)."""
        t0 = time.perf_counter()
        self.model.forward([3], self.past)  # cache not grown: every step at the same context
        layer_t = time.perf_counter() - t0
        t0 = time.perf_counter()
        _ = self.lm @ self.x
        lm_t = time.perf_counter() - t0
        return layer_t * C3["layers"] + lm_t


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    cb = CpuBaseline()
    per_tok = []
    for i in range(args.warmup + args.steps):
        t = cb.step()
        if i >= args.warmup:
            per_tok.append(t)
    sample = cb.sample
    tps = 1.0 / float(np.mean(per_tok))
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": float(np.mean(per_tok)) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "cpu_path": "oracle port of the reference "
                       "(per-request batch-1 decode, dense KV), numpy f32"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cpu_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def release(worker):
    """Drop captured CUDA graphs (they may hold NCCL calls) and peer mappings
    before the process group goes."""
    import gc

    worker.close()
    gc.collect()
    torch.cuda.synchronize()


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist
    from mu_b200 import _lib
    from mu_b200 import kernels as K
    from mu_b200.core.config import SamplingParams

    torch.cuda.set_device(local_rank)
    wl = WORKLOADS[args.workload]
    tp = world if args.parallel in ("tp", "ep") else 1
    engine, worker, ec = build(rank, tp, wl, ep=args.parallel == "ep", align=args.step_align)
    conc, out_tokens = wl["concurrency"], wl["out"]
    # tensor-parallel ranks serve the same requests; replicas serve their own
    # Every engine serves the same seeded request stream (replicas each serve
    # their own copy of it): the step-to-step mix of prompt lengths is then
    # the same on every GPU, so the max-over-ranks time measures the scaling
    # of the hardware, not the spread of eight independent random draws.
    seed_rank = 0
    arrivals = Arrivals(1000 + seed_rank, wl)
    rng = np.random.default_rng(7 + seed_rank)
    for _ in range(conc):
        arrivals.new_request(engine, SamplingParams, already=int(rng.integers(0, out_tokens)))
    # initial fill: prefill every starting request (untimed)
    fill_steps = 0
    while engine.scheduler.waiting:
        steady_state_step(engine, arrivals, SamplingParams)
        fill_steps += 1
    # The clock sampler starts before the warm-up steps (its start-up would
    # otherwise leave the GPU idle, and cooler, right before the timed
    # region); only the samples taken inside the timed region are reported.
    clocks = ClockSampler(local_rank).__enter__()
    for _ in range(args.warmup):
        steady_state_step(engine, arrivals, SamplingParams)
    # the engine overlaps host work with the step before: start the timed
    # region with nothing in flight and end it with the last step read back
    steady_state_step(engine, arrivals, SamplingParams, engine.flush())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- e2e: the public step API, host work and copies included ----------
    rec = Recorder(engine, worker)
    rec.on = True
    n_tok = 0
    launches0 = _lib.launch_count
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clk0 = clocks.mark()
        torch.cuda.nvtx.range_push("timed")
        start.record()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            n_tok += steady_state_step(engine, arrivals, SamplingParams)
        n_tok += steady_state_step(engine, arrivals, SamplingParams, engine.flush())
        end.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        clk1 = clocks.mark()
    finally:
        clocks.__exit__(None, None, None)
    launches = _lib.launch_count - launches0
    rec.on = False
    e2e_t = start.elapsed_time(end) * 1e-3
    # packed step arrays + the sampler's parameter blob (9 words per sequence)
    h2d = sum(st.end * 4 + 36 * st.B for st, _ in rec.steps) / max(1, len(rec.steps))
    steps_meta = [(st.B, st.T, st.num_decode) for st, _ in rec.steps]

    # ---- value: same steps, arrays resident in HBM, no host work in between ----
    # Each recorded step is re-issued exactly as the engine issued it: its
    # packed arrays and the sampler's parameter blob are restored from HBM
    # (device-to-device), then the model step and the engine's sampler
    # launches (bitmap marking of the step's inputs, one sampling launch)
    # run.  Only the host work and the host<->device copies of the engine
    # path are absent.
    smp = engine.sampler
    assert len(rec.blobs) == len(rec.steps)
    assert all(b.numel() == smp._blob_d.numel() for _, _, b, _ in rec.blobs)

    @torch.inference_mode()  # the engine's buffers are inference tensors
    def replay():
        for (st, buf), (B, T, blob, greedy) in zip(rec.steps, rec.blobs):
            worker.packer.dev[:st.end].copy_(buf, non_blocking=True)
            logits, batch = worker.run_staged(st)
            smp._blob_d[:blob.numel()].copy_(blob, non_blocking=True)
            if T > 0:
                smp.mark_inputs(batch.token_rows, batch.input_ids, T)
            smp.device_sample(logits, B, greedy)

    replay()  # graphs for every bucket exist already; this warms the replay path
    torch.cuda.synchronize()
    # Three timed passes over the same K steps; value uses the median pass.
    # On this power-capped part one sub-second pass varies by a few percent
    # with the clock, in either direction.
    passes = []
    for _ in range(3):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        replay()
        e2.record()
        torch.cuda.synchronize()
        passes.append(s2.elapsed_time(e2) * 1e-3)
    dev_t = statistics.median(passes)

    # ---- roofline pieces ------------------------------------------------------
    hbm, tflops, tflops_sus, peak_kind = peaks()
    # the dominant kernel (GEMM, ~60 % of the step): every launch of the same
    # steps timed with CUDA events (steps replayed from graphs are not seen)
    probe = GemmProbe()
    K.gemm_probe = probe
    # the per-kernel Python step issues the same GEMM launches as the native
    # executor, one at a time, so each can be bracketed by events
    native = getattr(worker.model, "native", False)
    worker.model.native = False
    replay()
    worker.model.native = native
    K.gemm_probe = None
    gp_flops, gp_t, gp_n = probe.result()
    att_bytes, att_t, att_b, att_tok = time_attention(worker)
    g_flops, g_t, g_wbytes = time_gemms(worker) if wl["arch"] == "llama" else (0.0, 0.0, 0.0)
    c4 = time_attention_c4() if args.workload == "c3" and (rank == 0 or tp == 1) else None

    # ---- reduce over ranks ------------------------------------------------------
    vals = torch.tensor([n_tok, dev_t, e2e_t, wall], device="cuda", dtype=torch.float64)
    if world > 1:
        tot = vals.clone()
        if tp == 1:  # replicas: tokens add up; tensor-parallel ranks produce the same tokens
            dist.all_reduce(tot[:1], op=dist.ReduceOp.SUM)
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        n_all, dev_max, e2e_max, wall_max = float(tot[0]), float(mx[1]), float(mx[2]), float(mx[3])
    else:
        n_all, dev_max, e2e_max, wall_max = n_tok, dev_t, e2e_t, wall
    release(worker)
    if rank != 0:
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.workload == "c3":
        cb = CpuBaseline()
        per_tok = float(np.mean([cb.step() for _ in range(5)]))
        sample = cb.sample + ", mean of 5 steps"
        cpu = {"value": 1.0 / per_tok, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": sample}
    clk = clocks.summary(clk0, clk1)
    c3 = args.workload == "c3"
    par = {"tp": f"tp{tp}", "ep": f"tp{tp}+ep{tp}", "replicas": f"replicas{world}"}[args.parallel]
    line = {
        "metric": METRIC if c3 else f"decode tokens/s ({args.workload})",
        "value": n_all / dev_max,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_max / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if tp > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": f"synthetic: random-init bf16 weights (seed {wl['seed']}), {wl['prompt'][0]} "
                "prompt lengths, uniform ids",
        "config": {
            "workload": wl["desc"],
            "model": {"c3": "llama-3-8b-shape", "c2": "deep-c2", "c5": "deep-c5"}[args.workload],
            "global_batch": conc * (world // tp),
            "seq_len": f"prompt {wl['prompt']} + {out_tokens} generated",
            "parallelism": par if world > 1 else "single",
            "request_stream": ("one seeded stream; every replica serves its own copy"
                               if world > 1 and tp == 1 else "one seeded stream"),
            "l2": "no flush needed: each step streams the weights (GBs) and the KV of every "
                  "running request (GBs) through HBM (L2 126 MB)",
            "tokens_timed": int(n_all),
            "steps_pure_decode": sum(1 for b, t, d in steps_meta if d == b),
            "mean_tokens_per_step": float(np.mean([t for _, t, _ in steps_meta])),
            "initial_fill_steps": fill_steps,
            "step_token_alignment": args.step_align,
            "value_passes_ms": [round(t * 1e3, 3) for t in passes],
        },
        "e2e": {"value": n_all / e2e_max, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(4 * conc), "wall_s": wall_max,
                "api": "mu_b200.serving.engine.StepEngine.step"},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "muk_gemm_bf16 (every launch of the eager steps of the timed "
                               "workload, CUDA events per launch)",
                     "bound": "tensor", "achieved": gp_flops / gp_t / 1e12, "peak": tflops_sus,
                     "unit": "TFLOP/s", "frac": gp_flops / gp_t / 1e12 / tflops_sus,
                     "traffic": GEMM_NCU_TRAFFIC["dram_bytes"],
                     "traffic_launch": GEMM_NCU_TRAFFIC,
                     "peak_source": f"{peak_kind} sustained bf16 (MEASURED_PEAKS.json "
                                    "bf16_tflops_sustained; kernel runs inside a long step)",
                     "launches": gp_n, "flops_per_launch": gp_flops / max(gp_n, 1),
                     "us_per_launch": gp_t / max(gp_n, 1) * 1e6},
        "roofline_attention": {"kernel": "muk_paged_decode_attn (layer, running batch)",
                               "bound": "hbm", "achieved": att_bytes / att_t / 1e9, "peak": hbm,
                               "unit": "GB/s", "frac": att_bytes / att_t / 1e9 / hbm,
                               "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                               "algorithmic_bytes": att_bytes, "seqs": att_b,
                               "context_tokens": att_tok},
        "roofline_attention_c4": None if c4 is None else {
            "kernel": "muk_paged_decode_attn, 128 seqs ctx U[1024,32768], 32/8 heads D128, "
                      "random-permutation block tables, pool 1.2x tokens",
            "bound": "hbm", "achieved": c4[0] / c4[1] / 1e9, "peak": hbm, "unit": "GB/s",
            "frac": c4[0] / c4[1] / 1e9 / hbm, "vs_8TBps": c4[0] / c4[1] / 8e12,
            "algorithmic_bytes": c4[0], "us_per_launch": c4[1] * 1e6, "context_tokens": c4[3]},
        "roofline_gemm_decode": None if not g_t else {
                                 "kernel": "muk_gemm_bf16 decode layer (QKV+O+gate|up+down, "
                                           "M=256; 10 layers replayed from a CUDA graph, as "
                                           "the engine replays pure-decode steps)",
                                 "bound": "tensor", "achieved": g_flops / g_t / 1e12,
                                 "peak": tflops, "unit": "TFLOP/s",
                                 "frac": g_flops / g_t / 1e12 / tflops,
                                 "weight_GBps": g_wbytes / g_t / 1e9,
                                 "peak_source": f"{peak_kind} burst bf16"},
        "cpu_baseline": cpu,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_micro(args):
    """Single-kernel cases sized for ncu captures (a few GB on the device)."""
    from mu_b200 import kernels as K

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(3)
    res = {"micro": args.micro}
    if args.streamk is not None:
        K.gemm_set_stream_k(args.streamk)
        res["stream_k_mode"] = args.streamk
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.micro == "decode_attn":
        Hq, Hkv, D = 32, 8, 128
        rng = np.random.default_rng(3)
        ctx = rng.integers(args.ctx_min, args.ctx_max + 1, args.seqs)
        nblk = (ctx + 15) // 16
        NB = int(nblk.sum()) + 8
        kc = torch.randn(NB, Hkv, 16, D, device="cuda", generator=g).bfloat16()
        vc = torch.randn(NB, Hkv, 16, D, device="cuda", generator=g).bfloat16()
        perm = rng.permutation(NB)
        bt = np.zeros((args.seqs, int(nblk.max())), np.int32)
        i = 0
        for b, n in enumerate(nblk):
            bt[b, :n] = perm[i:i + n]
            i += n
        btd = torch.from_numpy(bt).cuda()
        sl = torch.from_numpy(ctx.astype(np.int32)).cuda()
        q = torch.randn(args.seqs, Hq * D, device="cuda", generator=g).bfloat16()
        out = torch.empty_like(q)
        mx = int(ctx.max())
        ws = torch.empty(K.decode_attn_workspace_size(args.seqs, Hq, D, mx) // 4 + 4, device="cuda")

        def fn():
            K.decode_attn(q, out, kc, vc, btd, sl, Hq, Hkv, D, mx, workspace=ws)
        byts = float(ctx.sum()) * Hkv * D * 4
        res.update(seqs=args.seqs, ctx_sum=int(ctx.sum()), algorithmic_bytes=byts)
    elif args.micro == "prefill_attn":
        # causal prefill of fresh prompts (no cached prefix), Llama-3-8B heads
        Hq, Hkv, D = 32, 8, 128
        lens = [int(x) for x in args.prompts.split(",")]
        nblk = [(n + 15) // 16 for n in lens]
        NB = sum(nblk) + 8
        kc = torch.randn(NB, Hkv, 16, D, device="cuda", generator=g).bfloat16()
        vc = torch.randn(NB, Hkv, 16, D, device="cuda", generator=g).bfloat16()
        bt = np.zeros((len(lens), max(nblk)), np.int32)
        i = 0
        for b, n in enumerate(nblk):
            bt[b, :n] = np.arange(i, i + n)
            i += n
        btd = torch.from_numpy(bt).cuda()
        sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device="cuda")
        q = torch.randn(sum(lens), Hq * D, device="cuda", generator=g).bfloat16()
        out = torch.empty_like(q)

        def fn():
            K.prefill_attn(q, out, kc, vc, btd, sl, cu, max(lens), Hq, Hkv, D)
        byts = float(sum(4.0 * n * (n + 1) / 2 * Hq * D for n in lens))
        res.update(prompts=lens, flops=byts)
    elif args.micro == "qkv_rope":
        # q|k|v projection with RoPE and the paged-KV append in its epilogue,
        # Llama-3-8B shape (H 4096, 32/8 heads, D 128), M tokens
        M, Kd, Hq, Hkv, D = args.m, 4096, 32, 8, 128
        N = (Hq + 2 * Hkv) * D
        A = torch.randn(M, Kd, device="cuda", generator=g).bfloat16()
        B = (torch.randn(N, Kd, device="cuda", generator=g) * 0.02).bfloat16()
        qo = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        NB = (M + 15) // 16 + 8
        kc = torch.zeros(NB, Hkv, 16, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        pos = torch.arange(M, device="cuda", dtype=torch.int32)
        slots = torch.randperm(NB * 16, device="cuda", generator=g)[:M].to(torch.int32)
        inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
        ang = torch.arange(M + 1, device="cuda").float()[:, None] * inv[None]
        cos, sin = ang.cos().contiguous(), ang.sin().contiguous()

        def fn():
            K.gemm_qkv_rope(A, B, qo, pos, slots, cos, sin, Hq, Hkv, D, kc, vc)
        byts = 2.0 * M * N * Kd
        res.update(M=M, N=N, K=Kd, flops=byts, plan=K.gemm_plan_info(M, N, Kd, K.MUK_EPI_ROPE_KV))
    elif args.micro == "norm":
        # residual + RMSNorm (+ bf16 out) over a step's rows, H = args.k
        T, H = args.m, args.k
        resid = torch.randn(T, H, device="cuda", generator=g)
        part = torch.randn(1, T, H, device="cuda", generator=g)
        w = torch.ones(H, device="cuda")
        out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)

        def fn():
            K.residual_rmsnorm(resid, part, w, 1e-5, out)
        byts = float(T * H * (4 + 4 + 4 + 2))  # partial + resid read, resid + out written
        res.update(T=T, H=H, algorithmic_bytes=byts)
    elif args.micro == "inl":
        # INL dynamics row kernel of a Deep step (post-norm and routing fused), H = args.k
        T, H, E, V = args.m, args.k, 8, 32000
        h = torch.randn(T, H, device="cuda", generator=g)
        ctrl = torch.randn(T, 3 * H, device="cuda", generator=g)
        cb = torch.randn(3 * H, device="cuda", generator=g)
        mp = torch.randn(T, H, device="cuda", generator=g) * 0.1
        mu_param = torch.zeros(H, device="cuda")
        v = torch.randn(T, H, device="cuda", generator=g)
        resid = torch.randn(T, H, device="cuda", generator=g)
        router = (torch.randn(E, H, device="cuda", generator=g) * 0.02).bfloat16()
        ids = torch.randint(0, V, (T,), device="cuda", generator=g, dtype=torch.int32)
        w = torch.ones(H, device="cuda")
        v_bf = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
        mu_out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
        nout = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
        eids = torch.empty(T, device="cuda", dtype=torch.int32)
        cl = K.Clamp(True)

        def fn():
            K.inl_dynamics(h, ctrl, cb, mp, mu_param, 0.1, v, v_bf, resid, mu_out, w, 1e-6, nout,
                           ids, router, E, V, eids, cl)
        # f32 in: h, ctrl (3H), muproj, v, resid; out: v, resid f32 + v, mu, norm bf16
        byts = float(T * H * (4 * 7 + 4 * 2 + 2 * 3))
        res.update(T=T, H=H, algorithmic_bytes=byts)
    elif args.micro == "route":
        # stable expert sort of a step's tokens, then the row gather (H = args.k)
        T, H, E = args.m, args.k, 8
        eids = torch.randint(0, E, (T,), device="cuda", generator=g, dtype=torch.int32)
        offs = torch.zeros(E + 1, device="cuda", dtype=torch.int32)
        perm = torch.empty(T, device="cuda", dtype=torch.int32)
        inv = torch.empty(T, device="cuda", dtype=torch.int32)
        x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        xs = torch.empty_like(x)

        def fn():
            K.route_permute(eids, E, offs, perm, inv)
            K.gather_rows(x, perm, xs)
        byts = float(T * H * 2 * 2)
        res.update(T=T, H=H, algorithmic_bytes=byts)
    elif args.micro == "grouped_gemm":
        # a Deep step's expert gate|up GEMM (SwiGLU epilogue): T rows spread evenly over
        # E experts, per-expert width args.n (gate + up), K = args.k
        T, E, N2, Kd = args.m, args.experts, args.n, args.k
        counts = [T // E + (1 if e < T % E else 0) for e in range(E)]
        offs = torch.tensor(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32),
                            device="cuda")
        A = torch.randn(T, Kd, device="cuda", generator=g).bfloat16()
        W = (torch.randn(E * N2, Kd, device="cuda", generator=g) * 0.02).bfloat16()
        C = torch.empty(T, N2 // 2, device="cuda", dtype=torch.bfloat16)

        def fn():
            K.grouped_gemm(A, W, C, offs, E, N2, K.MUK_EPI_SWIGLU)
        byts = 2.0 * T * N2 * Kd
        res.update(T=T, E=E, N=N2, K=Kd, flops=byts)
    elif args.micro == "sampler":
        # one sampling launch over [B, V] f32 logits: greedy (--k 0) or top-p 0.9 at T 0.7
        B, V = args.m, args.n
        logits = torch.randn(B, V, device="cuda", generator=g) * 2.5
        greedy = args.k == 0
        temp = torch.full((B,), 0.0 if greedy else 0.7, device="cuda")
        tk = torch.zeros(B, device="cuda", dtype=torch.int32)
        tp = torch.full((B,), 1.0 if greedy else 0.9, device="cuda")
        rp = torch.ones(B, device="cuda")
        seeds = torch.arange(B, device="cuda", dtype=torch.int64)
        out = torch.empty(B, device="cuda", dtype=torch.int32)

        def fn():
            K.sample(logits, temp, tk, tp, rp, None, seeds, seeds, out)
        byts = float(B * V * 4)
        res.update(B=B, V=V, mode="greedy" if greedy else "top_p 0.9, T 0.7",
                   algorithmic_bytes=byts)
    else:
        M, N, Kd = args.m, args.n, args.k
        A = torch.randn(M, Kd, device="cuda", generator=g).bfloat16()
        B = (torch.randn(N, Kd, device="cuda", generator=g) * 0.02).bfloat16()
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

        def fn():
            K.gemm(A, B, C, K.MUK_EPI_BF16)
        byts = 2.0 * M * N * Kd
        res.update(M=M, N=N, K=Kd, flops=byts, plan=K.gemm_plan_info(M, N, Kd, K.MUK_EPI_BF16))
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    # a device-side wait keeps the GPU busy while the timed launches queue up,
    # so the events see kernel time, not the host's launch rate
    torch.cuda._sleep(20_000_000)
    s.record()
    for _ in range(args.reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = s.elapsed_time(e) / args.reps * 1e-3
    res["us_per_launch"] = t * 1e6
    if "algorithmic_bytes" in res:
        res["GBps"] = byts / t / 1e9
    else:
        res["TFLOPs"] = byts / t / 1e12
    print(json.dumps(res), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--step-align", type=int, default=0,
                    help="trim each step's last prefill chunk to a multiple of this many tokens")
    ap.add_argument("--parallel", choices=["replicas", "tp", "ep"], default=None,
                    help="N>1: one tensor-parallel engine (default for c3), tensor-parallel "
                         "attention with expert-parallel experts (default for the Deep "
                         "workloads c2/c5), or independent replicas")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c3",
                    help="c3 (default, the headline), c2 / c5 (DeepForCausalLM)")
    ap.add_argument("--micro", choices=["decode_attn", "gemm", "prefill_attn", "qkv_rope", "norm",
                                        "inl", "route", "grouped_gemm", "sampler"],
                    default=None,
                    help="time one kernel on a small case (for ncu captures)")
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--ctx-min", type=int, default=256)
    ap.add_argument("--ctx-max", type=int, default=4096)
    ap.add_argument("--m", type=int, default=256)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--experts", type=int, default=8, help="grouped_gemm micro: experts")
    ap.add_argument("--prompts", default="600", help="prefill_attn micro: comma-separated prompt lengths")
    ap.add_argument("--streamk", type=int, choices=[0, 1, 2], default=None,
                    help="GEMM micro cases: stream-K planning mode (0 off, 1 on, 2 auto)")
    args = ap.parse_args()
    if args.parallel is None:
        args.parallel = "tp" if WORKLOADS[args.workload]["arch"] == "llama" else "ep"
    if args.micro:
        return run_micro(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
