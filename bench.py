#!/usr/bin/env python
"""Decode throughput of the B200 minq path (one JSON line on rank 0).

Workload (default `qwen3-4b-q4_0`): the Qwen3-4B-shaped model (36 layers,
hidden 2560, 32/8 heads, head_dim 128, q/k RMSNorm, intermediate 9728,
vocab 151936, tied f32 lm_head) with seeded N(0, 0.02) random-init weights
quantized to Q4_0, batch 1: a 2048-token random prompt is prefilled, then
every step is ONE greedy decode token (the full forward: 36 layers of fused
Q4_0 matvecs, RoPE / q-k norm / KV append, split-KV decode attention over
the f32 cache, f32 lm_head + argmax), each step's token fed from the
previous step's argmax on the device. Weights (3.8 GB) are far larger than
L2 (126 MB), so every step streams them from HBM.

  metric   decode tok/s (whole job: sum over ranks)
  value    device-resident loop, CUDA events on the model stream
  e2e      same metric through the public C-ABI call minq_forward with host
           buffers: the token id from pinned host memory in, logits
           (vocab floats) and the argmax out to host memory, every step
  roofline dominant kernel (largest device-time share), per-launch CUDA
           events over a second pass of the same timed loop
  cpu_baseline  the C++ oracle (reference algorithm, AVX2, OpenMP on all
           host cores) decoding the same model from the same cache state

`--impl reference` times the reference's CPU algorithm (oracle) alone.
With torchrun (N>1) every rank decodes its own replica (the batch-1 decode
does not shard; replicas only) and value = N * steps / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic
# byte, from ncu --set full captures (summaries and commands under profiles/):
# three decode-shaped Q4_0 qmatvec launches (q/k/v, o_proj, gate/up), 47.72 MB
# / 47.62 MB; one decode megakernel launch of a 12-layer cut of the Q4_0
# model, 2.37069 GB / 2.36344 GB.
NCU_TRAFFIC_RATIO = {"qmatvec": 1.002, "decode_mk": 1.003}
sys.path.insert(0, ROOT)

# Greedy tokens the GPU decodes from the bench's cache state for the parity
# record (the oracle decodes from a copy of the same state).
PARITY_TOKENS = 64

WORKLOADS = {
    # name: (arch, prompt tokens)
    "qwen3-4b-q4_0": ("qwen3-4b", 2048),
    "qwen2-0.5b-q8_0": ("qwen2-0.5b", 128),
}
# Long-context tensor-parallel decode: the Qwen3-4B shape in Q8_0 with the KV
# cache pre-filled (N(0, 1)) at 32768 positions, greedy decode split over the
# ranks (heads and intermediate rows; the o_proj / down_proj partial sums
# exchanged through peer memory inside the decode megakernel).
TP_WORKLOAD = "qwen3-4b-q8_0-tp32k"
# Batched decode: 64 independent greedy sequences of the LLaMA-3-8B shape in
# Q4_0 (512-token prompts), data-sharded over the ranks with no collective.
BATCH_WORKLOAD = "llama3-8b-q4_0-b64"
# Greedy steps of the whole batch whose sequence-0 tokens are checked against
# the oracle (one GPU, CPU baseline on).
BATCH_PARITY_TOKENS = 16
# Isolated GQA decode attention (32 query / 8 kv heads, head_dim 128): RoPE +
# append + attend over L+1 positions for B sequences, swept over
# L in {512, 2048, 8192, 32768} x B in {1, 8, 64}.
ATTN_WORKLOAD = "attn-gqa32-8-hd128"
# Perplexity evaluation: the Qwen3-4B shape in Q4_0 over seeded synthetic
# token ids in non-overlapping windows of 512 (the reference's protocol is
# 10,000 tokens at context 512, i.e. 20 windows); one step = one window.
PPL_WORKLOAD = "qwen3-4b-q4_0-ppl"
PPL_CONTEXT = 512
# Device sampling: Sampler::sample on seeded logits over the Qwen vocabulary
# (151,936), one draw per step, for four sampler settings.
SAMPLER_WORKLOAD = "sampler-v151936"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["minq", "reference"], default="minq")
    ap.add_argument("--workload",
                    choices=sorted(WORKLOADS) + [TP_WORKLOAD, ATTN_WORKLOAD, BATCH_WORKLOAD,
                                                 PPL_WORKLOAD, SAMPLER_WORKLOAD],
                    default="qwen3-4b-q4_0")
    ap.add_argument("--prompt", type=int, default=None, help="prefill length override")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="default workload only: skip the batched (data-sharded) and "
                         "tensor-parallel sub-records")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--layers", type=int, default=None,
                    help="keep only the first N layers: a smaller case of the same kernels "
                         "for profiler captures (its number is not the workload's)")
    ap.add_argument("--attn-points", default=None,
                    help="attention sweep: only these BxL points (e.g. 64x512,8x8192), for "
                         "profiler captures of one point (the line's value needs 8x8192)")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ helpers

def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v: float) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def physical_gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].strip().isdigit():
            return int(ids[local])
    return local


def build_model(mq, synth, cfg, qk_norm, tied, seed):
    import torch
    recs = synth.synth_records(cfg, seed, qk_norm, tied, device="cuda")
    model = mq.Model.from_tensors(cfg, recs)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return model


def cpu_model(orc, synth, cfg, qk_norm, tied, seed):
    """The same seeded model for the oracle: drawn on the GPU (plumbing; on
    the CPU where there is none), then quantized on the host by the oracle's
    own quantizer (reference algorithm)."""
    import torch
    from minq_b200.minq_format import quantize_tensor_rule, DTYPE_TAGS
    qtag = DTYPE_TAGS[cfg.dtype]
    tensors = {}
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    for name, tag, shape, data in synth.synth_records(cfg, seed, qk_norm, tied, device=dev,
                                                      quantize=lambda t, x: x):
        host = data.detach().cpu().numpy()
        if qtag and quantize_tensor_rule(name, shape):
            tensors[name] = (qtag, shape, orc.quantize(qtag, host))
        else:
            tensors[name] = (0, shape, host)
        del data
    cfgd = {k: getattr(cfg, k) for k in cfg.__dataclass_fields__}
    return orc.Model.from_tensors(cfgd, tensors)


def time_cpu_decode(orc, om, oc, first_tok, min_tokens, seconds):
    """Greedy decode on the oracle for about `seconds` (at least `min_tokens`)."""
    tok = first_tok
    n = 0
    t0 = time.perf_counter()
    while True:
        logits = om.forward([tok], oc)
        tok = orc.argmax(logits)
        n += 1
        el = time.perf_counter() - t0
        if n >= min_tokens and el >= seconds:
            return n, el


# ------------------------------------------------------------------ arms

def run_reference(args, world, rank):
    """The reference's CPU algorithm (oracle, AVX2 + OpenMP on all host cores)."""
    if rank != 0:
        return
    from oracle import oracle as orc
    from minq_b200 import synth
    from dataclasses import replace
    # torchrun sets OMP_NUM_THREADS=1: the arm uses every host core
    orc.set_threads(os.cpu_count() or 1)
    arch, prompt_len = WORKLOADS[args.workload]
    prompt_len = args.prompt or prompt_len
    cfg0, qk_norm, tied = synth.ARCH[arch]
    max_seq = prompt_len + args.warmup + args.steps + 8
    cfg = replace(cfg0, max_seq_len=max_seq)
    om = cpu_model(orc, synth, cfg, qk_norm, tied, args.seed)
    oc = om.new_cache()
    # KV history of `prompt_len` positions (seeded N(0,1)); decode cost per
    # token depends only on the history length.
    kvd = cfg.n_kv_heads * cfg.head_dim
    rng = np.random.default_rng(args.seed)
    k = rng.standard_normal((cfg.n_layers, prompt_len, kvd), dtype=np.float32)
    v = rng.standard_normal((cfg.n_layers, prompt_len, kvd), dtype=np.float32)
    oc.fill(k, v)
    del k, v
    tok = 1
    for _ in range(args.warmup):
        tok = orc.argmax(om.forward([tok], oc))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = orc.argmax(om.forward([tok], oc))
    el = time.perf_counter() - t0
    value = args.steps / el
    cores = orc.max_threads()
    line = {
        "impl": "reference", "metric": "decode tok/s", "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * el / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload} decode bs=1 after a {prompt_len}-token prefill",
                   "kv_length": f"{prompt_len}..{prompt_len + args.warmup + args.steps}",
                   "host": "whole host CPU: OpenMP threads = os.cpu_count()",
                   "cache_flush": "weights 3.8 GB > L2"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} decode tokens after {args.warmup} warm-up, "
                                   f"KV history {prompt_len}"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _reference_line(args, metric, value, unit, steps, warmup, ms, scaling, dtype, config,
                    cores, sample, higher=True):
    return {"impl": "reference", "metric": metric, "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "ms_per_step": ms,
            "higher_is_better": higher, "scaling": scaling, "vs_baseline": None, "dtype": dtype,
            "data": "synthetic", "config": config,
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_reference_workload(args, rank):
    """The reference arm of the long-context, batched, attention and sampler
    workloads: the reference's CPU algorithm (the oracle, AVX2 + OpenMP on all
    host cores; its sampler on one core, as sampler.rs runs) on a bounded
    sample of the same workload, rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as orc
    from minq_b200 import synth
    from dataclasses import replace
    K, W = max(1, min(args.steps, 3)), max(0, min(args.warmup, 1))
    # torchrun sets OMP_NUM_THREADS=1: the arm uses every host core
    orc.set_threads(os.cpu_count() or 1)
    cores = orc.max_threads()
    if args.workload in (TP_WORKLOAD, BATCH_WORKLOAD):
        tp = args.workload == TP_WORKLOAD
        arch = "qwen3-4b" if tp else "llama3-8b"
        hist = args.prompt or (32768 if tp else 512)
        cfg0, qk_norm, tied = synth.ARCH[arch]
        if args.layers:
            cfg0 = replace(cfg0, n_layers=args.layers)
        cfg = replace(cfg0, max_seq_len=hist + W + K + 8, **({"dtype": "q8_0"} if tp else {}))
        om = cpu_model(orc, synth, cfg, qk_norm, tied, args.seed)
        oc = om.new_cache()
        kvd = cfg.n_kv_heads * cfg.head_dim
        rng = np.random.default_rng(args.seed)
        k = rng.standard_normal((cfg.n_layers, hist, kvd), dtype=np.float32)
        v = rng.standard_normal((cfg.n_layers, hist, kvd), dtype=np.float32)
        oc.fill(k, v)
        del k, v
        tok = 1
        for _ in range(W):
            tok = orc.argmax(om.forward([tok], oc))
        t0 = time.perf_counter()
        for _ in range(K):
            tok = orc.argmax(om.forward([tok], oc))
        el = time.perf_counter() - t0
        value = K / el  # one sequence-token per forward, for either workload
        if tp:
            metric, scaling = "decode tok/s", "strong"
            config = {"workload": f"{TP_WORKLOAD}: Qwen3-4B shape, Q8_0, KV pre-filled at "
                                  f"{hist} positions", "layers": cfg.n_layers}
        else:
            metric, scaling = "decode tok/s (batched)", "strong"
            config = {"workload": f"{BATCH_WORKLOAD}: LLaMA-3-8B shape, Q4_0, 64 sequences, "
                                  f"history {hist}; the reference decodes the sequences one "
                                  f"forward at a time", "layers": cfg.n_layers}
        line = _reference_line(args, metric, value, "tok/s", K, W, 1000 * el / K, scaling, "f32",
                               config, cores, f"{K} decode tokens at KV history {hist} after "
                               f"{W} warm-up, {el:.1f} s")
    elif args.workload == ATTN_WORKLOAD:
        B, L, nh, nkv, hd = 8, 8192, 32, 8, 128
        rng = np.random.default_rng(args.seed)
        ks = [rng.standard_normal((L + 1, nkv * hd), dtype=np.float32) for _ in range(B)]
        vs = [rng.standard_normal((L + 1, nkv * hd), dtype=np.float32) for _ in range(B)]
        qs = [rng.standard_normal(nh * hd, dtype=np.float32) for _ in range(B)]
        for b in range(B if W else 0):
            orc.attend(qs[b], ks[b], vs[b], L + 1, nh, nkv, hd)
        t0 = time.perf_counter()
        for _ in range(K):
            for b in range(B):
                orc.attend(qs[b], ks[b], vs[b], L + 1, nh, nkv, hd)
        el = time.perf_counter() - t0
        byts = 2.0 * 4 * B * nkv * hd * (L + 1)
        value = byts * K / el / 1e9
        line = _reference_line(args, "decode attention GB/s", value, "GB/s", K, W,
                               1000 * el / K, "weak", "f32",
                               {"workload": f"{ATTN_WORKLOAD}: RoPE + append + attend, B = 8, "
                                            f"L = 8192"}, 1,
                               f"{K} x attend (model.rs:223-248, single-threaded loops as in "
                               f"the reference) over {B} sequences of {L + 1} positions, "
                               f"{el:.1f} s")
    elif args.workload == SAMPLER_WORKLOAD:
        n = 151936
        x = (np.random.default_rng(args.seed).standard_normal(n) * 3.0).astype(np.float32)
        o = orc.Sampler(0.8, 40, 0.9, args.seed)
        for _ in range(W):
            o.sample(x)
        t0 = time.perf_counter()
        nd = 0
        while nd < 3 or time.perf_counter() - t0 < 5.0:
            o.sample(x)
            nd += 1
        el = time.perf_counter() - t0
        line = _reference_line(args, "device sampling draws/s", nd / el, "draws/s", nd, W,
                               1000 * el / nd, "weak", "f32 probabilities, f64 sums",
                               {"workload": f"{SAMPLER_WORKLOAD}: Sampler::sample over 151936 "
                                            f"logits"}, 1,
                               f"{nd} draws of the temperature 0.8 / top_k 40 / top_p 0.9 "
                               f"setting, {el:.1f} s")
    else:
        raise SystemExit(f"no reference arm for {args.workload}")
    print(json.dumps(line), flush=True)


def run_minq(args, world, rank, local):
    import torch
    import minq_b200 as mq
    from minq_b200 import _lib, synth
    from dataclasses import replace
    torch.cuda.set_device(local)
    L = _lib.lib()
    arch, prompt_len = WORKLOADS[args.workload]
    prompt_len = args.prompt or prompt_len
    cfg0, qk_norm, tied = synth.ARCH[arch]
    if args.layers:
        cfg0 = replace(cfg0, n_layers=args.layers)
    K, W = args.steps, args.warmup
    max_seq = prompt_len + W + 2 * K + 3 * min(K, 16) + PARITY_TOKENS + 40
    cfg = replace(cfg0, max_seq_len=max_seq)
    model = build_model(mq, synth, cfg, qk_norm, tied, args.seed + rank)
    cache = model.new_cache()
    stream = torch.cuda.ExternalStream(model.stream)
    V = cfg.vocab_size

    # ---- prefill (chunks of 64 prompt tokens, the last token as a decode step) ----
    prompt = np.random.default_rng(args.seed).integers(0, V, prompt_len).astype(np.uint32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = model.forward_argmax(prompt, cache)
    prefill_s = time.perf_counter() - t0

    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")

    def step():
        # one greedy decode token, fed on the device by the previous argmax
        model.decode_steps(cache, 1)

    for _ in range(W):
        step()
    torch.cuda.synchronize()

    # ---- timed device-resident loop ----
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    len_timed0 = cache.len  # history length at the first timed step
    ev0.record(stream)
    # NVTX range: lets `ncu --nvtx --nvtx-include timed_decode/` list exactly
    # the launches of the timed region
    torch.cuda.nvtx.range_push("timed_decode")
    th0 = time.perf_counter()
    for _ in range(K):
        step()
    host_enqueue_ms = 1000.0 * (time.perf_counter() - th0)
    torch.cuda.nvtx.range_pop()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(world, ms)
    value = world * K / (ms_max / 1000.0)

    # ---- e2e through the public C-ABI call with host buffers ----
    h_tok = torch.empty(1, dtype=torch.int32, pin_memory=True)
    h_logits = torch.empty(V, dtype=torch.float32, pin_memory=True)
    h_arg = torch.empty(1, dtype=torch.int32, pin_memory=True)
    model.decode_steps(cache, 1, d_out.data_ptr())
    h_tok[0] = int(d_out.item())
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(K):
        _lib.check(L.minq_forward(model._h, cache._h, C.c_void_p(h_tok.data_ptr()), 1,
                                  C.c_void_p(h_logits.data_ptr()), C.c_void_p(h_arg.data_ptr())))
        h_tok[0] = h_arg[0]
    e1.record(stream)
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - t0
    ms_e2e = max(e0.elapsed_time(e1), 1000.0 * wall_e2e)
    ms_e2e_max = max_over_ranks(world, ms_e2e)
    e2e_value = world * K / (ms_e2e_max / 1000.0)

    # ---- parity state (rank 0, N=1): the cache after the timed and e2e
    # steps, then PARITY_TOKENS greedy tokens decoded from it on the GPU
    # (decode megakernel through minq_forward); the oracle later decodes from
    # a copy of the same state and the two token streams are compared ----
    par_state = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_pos = cache.len
        kvd = cfg.n_kv_heads * cfg.head_dim
        kall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
        vall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
        for li in range(cfg.n_layers):
            kall[li], vall[li] = cache.read(li, 0, n_pos)
        start = int(h_tok[0])
        gpu_toks = []
        tok = start
        for _ in range(PARITY_TOKENS):
            tok = model.forward_argmax([tok], cache)
            gpu_toks.append(int(tok))
        par_state = (n_pos, kall, vall, start, gpu_toks)

    # ---- per-kernel timing pass (same loop launched eagerly, events around
    # each launch of one kernel family) ----
    model.set_graphs(False)
    n0 = L.minq_kernel_launches()
    step()
    torch.cuda.synchronize()
    launches_per_step = L.minq_kernel_launches() - n0
    launches = launches_per_step * K
    fams = {}
    for fam in ("qmatvec", "f32_matvec", "attention"):
        _lib.check(L.minq_kernel_timer_start(fam.encode()))
        for _ in range(min(K, 16)):
            step()
        n = C.c_uint64()
        tms = C.c_double()
        byt = C.c_double()
        _lib.check(L.minq_kernel_timer_stop(C.byref(n), C.byref(tms), C.byref(byt)))
        if n.value:
            fams[fam] = {"launches": n.value, "ms": tms.value, "bytes": byt.value,
                         "avg_us": 1000 * tms.value / n.value,
                         "gbs": byt.value / (tms.value / 1000.0) / 1e9}
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    peak_src = "measured" if peaks.get("hbm_gbs") else "fallback"
    dom = max(fams, key=lambda k: fams[k]["ms"]) if fams else None
    roof = None
    if launches_per_step == 1:
        # The whole token is one launch of the decode megakernel, so the
        # dominant kernel is that launch and its duration is the timed step
        # (CUDA events on the model's stream around K back-to-back launches).
        # Algorithmic bytes per launch: every weight byte (quantized
        # projections + the f32 lm_head) plus the K/V history read at the
        # average position of the timed steps.
        kv_pos = len_timed0 + (K - 1) / 2.0
        kv_bytes = 2 * 4 * cfg.n_kv_heads * cfg.head_dim * kv_pos * cfg.n_layers
        per_launch = float(model.weight_bytes) + kv_bytes
        avg_us = 1000.0 * ms_max / K
        gbs = per_launch / (avg_us * 1e-6) / 1e9
        fams = {"decode_mk": {"launches": K, "ms": ms_max, "bytes": per_launch * K,
                              "avg_us": avg_us, "gbs": gbs}}
        roof = {"bound": "hbm", "kernel": "decode_mk", "achieved": gbs, "peak": peak,
                "unit": "GB/s", "frac": gbs / peak, "peak_source": peak_src,
                "traffic": (per_launch * NCU_TRAFFIC_RATIO["decode_mk"]
                            if "decode_mk" in NCU_TRAFFIC_RATIO else None),
                "per_launch_bytes": per_launch, "avg_launch_us": avg_us}
    elif dom:
        d = fams[dom]
        roof = {"bound": "hbm", "kernel": dom, "achieved": d["gbs"], "peak": peak,
                "unit": "GB/s", "frac": d["gbs"] / peak, "peak_source": peak_src,
                "traffic": (d["bytes"] / d["launches"] * NCU_TRAFFIC_RATIO[dom]
                            if dom in NCU_TRAFFIC_RATIO else None),
                "per_launch_bytes": d["bytes"] / d["launches"], "avg_launch_us": d["avg_us"]}

    # ---- CPU baseline (rank 0, N=1): the oracle continues the same sequence
    # from the same cache state; its tokens are the parity record ----
    cpu = None
    parity = None
    if par_state is not None:
        try:
            from oracle import oracle as orc
            orc.set_threads(os.cpu_count() or 1)
            n_pos, kall, vall, start, gpu_toks = par_state
            om = cpu_model(orc, synth, replace(cfg, max_seq_len=n_pos + 256), qk_norm, tied,
                           args.seed + rank)
            oc = om.new_cache()
            oc.fill(kall, vall)
            del kall, vall
            par_state = None
            ref_toks = []
            tok = start
            t0 = time.perf_counter()
            while True:
                tok = orc.argmax(om.forward([tok], oc))
                ref_toks.append(int(tok))
                el = time.perf_counter() - t0
                if len(ref_toks) >= PARITY_TOKENS or (len(ref_toks) >= 32 and el >= args.cpu_seconds):
                    break
            n = len(ref_toks)
            cpu = {"value": n / el, "unit": "tok/s", "cores": orc.max_threads(), "kind": "port",
                   "sample": f"{n} greedy decode tokens of the same model from the same "
                             f"{n_pos}-position cache state, {el:.1f} s"}
            first = next((i for i, (a, b) in enumerate(zip(gpu_toks, ref_toks)) if a != b), None)
            parity = {"tokens": n, "match": first is None, "first_mismatch": first,
                      "from": f"the GPU's cache after prefill + timed steps ({n_pos} positions)",
                      "gpu": "decode megakernel (minq_forward)", "oracle": "forward_token + argmax"}
            del om, oc
        except Exception as e:  # the baseline must not sink the GPU number
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {type(e).__name__}: {e}"}
            parity = {"tokens": 0, "match": None, "first_mismatch": None,
                      "error": f"{type(e).__name__}: {e}"}

    if rank == 0:
        line = {
            "metric": "decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.workload} decode bs=1 after a {prompt_len}-token prefill",
                       "kv_length": f"{prompt_len}..{prompt_len + W + K}",
                       "model": arch, "layers": cfg.n_layers, "quant": cfg.dtype, "global_batch": world,
                       "parallelism": f"replicas x{world}",
                       "cache_flush": "inputs > L2: 3.8 GB of weights streamed per step"
                       if arch == "qwen3-4b" else "inputs > L2",
                       "weight_bytes": model.weight_bytes},
            "prefill": {"tokens": prompt_len, "tok_s": prompt_len / prefill_s,
                        "mode": "chunks of 64 tokens (batched projections and causal flash attention on the tensor cores: tcgen05 kind::f16 / kind::tf32), then the last token as a decode step" if os.environ.get("MINQ_FLASH_PREFILL", "1") != "0" else "chunks of 64 tokens (batched projections on the tensor cores, split-KV attention per token), then the last token as a decode step"},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * V + 4},
            "gpu_launches": int(launches),
            "host_enqueue_ms_per_step": host_enqueue_ms / K,
            "roofline": roof,
            "kernels": fams,
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clk,
        }
    del cache, model
    torch.cuda.empty_cache()
    # ---- sub-records of the partitioned workloads at the same N: the
    # LLaMA-3-8B batch of 64 sequences data-sharded over the ranks, and the
    # long-context Qwen3-4B Q8_0 decode tensor-parallel over them (1 GPU: the
    # decode megakernel), each with its own clock and roofline ----
    if not args.no_sub_records and args.workload == "qwen3-4b-q4_0" and not args.layers:
        # a sub-record that fails reports its error instead of sinking the
        # headline line (every rank runs the same steps, so a failing shape
        # fails on all of them alike)
        def sub(fn, *a, **kw):
            try:
                return fn(*a, **kw)
            except Exception as e:
                torch.cuda.synchronize()
                return {"error": repr(e)[:400]}
        bline = sub(run_batch, args, world, rank, local, steps=16, warmup=4, emit=False)
        tline = sub(run_tp, args, world, rank, local, steps=16, warmup=4, emit=False)
        tpar = sub(tp_parity, world, rank, local) if world > 1 else None
        if rank == 0:
            line["batched"] = bline
            if isinstance(tline, dict) and "error" not in tline:
                tline["parity"] = tpar
            line["tp"] = tline
            if world == 1:
                line["load"] = load_record(args, cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)


def load_record(args, cfg):
    """minq_model_load (format.rs:149-277 + model.rs:711-715) of the bench's
    own model written to a .minq file: the file mapped and indexed in place,
    each tensor uploaded through pinned double buffers on a copy stream. Timed
    wall clock around the call, once after evicting the file's pages from the
    page cache (posix_fadvise DONTNEED: read from the file system) and once
    with them cached. Returns the record, or its error."""
    import tempfile
    import torch
    import minq_b200 as mq
    from minq_b200 import synth
    from minq_b200.minq_format import write_minq_header, write_minq_record
    arch, _ = WORKLOADS[args.workload]
    _, qk_norm, tied = synth.ARCH[arch]
    path = os.path.join(tempfile.gettempdir(), f"minq_bench_{os.getpid()}.minq")
    try:
        with open(path, "wb") as f:
            write_minq_header(f, cfg)
            for name, tag, shape, data in synth.synth_records(cfg, args.seed, qk_norm, tied):
                write_minq_record(f, name, tag, shape, data.detach().cpu().numpy())
                del data
            f.flush()
            os.fsync(f.fileno())
        size = os.path.getsize(path)
        out = {"file_bytes": size, "model": f"{arch} {cfg.dtype}, {cfg.n_layers} layers"}
        for kind in ("uncached", "page_cached"):
            if kind == "uncached":
                fd = os.open(path, os.O_RDONLY)
                try:
                    os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                finally:
                    os.close(fd)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            m = mq.Model.load_minq(path)
            torch.cuda.synchronize()
            el = time.perf_counter() - t0
            out[kind] = {"s": el, "gb_s": size / el / 1e9}
            del m
            torch.cuda.empty_cache()
        out["how"] = ("mmap + index in place, per tensor one cudaMalloc, host threads copy "
                      "64 MiB chunks into two pinned buffers, one cudaMemcpyAsync per chunk on "
                      "a copy stream; the tied lm_head aliases the f32 embedding (uploaded once)")
        return out
    except Exception as e:  # the load record must not sink the decode number
        return {"error": f"{type(e).__name__}: {e}"}
    finally:
        try:
            os.unlink(path)
        except OSError:
            pass


def run_tp(args, world, rank, local, steps=None, warmup=None, emit=True):
    """One greedy sequence of the long-context workload, tensor-parallel over
    the `world` ranks (single GPU: the decode megakernel). Returns rank 0's
    JSON line (printed when `emit`)."""
    import torch
    import minq_b200 as mq
    from minq_b200 import synth
    from dataclasses import replace
    torch.cuda.set_device(local)
    ctx = 32768
    K = steps if steps is not None else args.steps
    W = warmup if warmup is not None else args.warmup
    cfg0, qk_norm, tied = synth.ARCH["qwen3-4b"]
    cfg = replace(cfg0, dtype="q8_0", max_seq_len=ctx + W + 2 * K + 16)
    model = build_model(mq, synth, cfg, qk_norm, tied, args.seed)  # every rank: the same weights
    if world > 1:
        import torch.distributed as dist
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(mq.tp_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        model.tp_init(rank, world, bytes(uid.cpu().numpy().tobytes()))
    cache = model.new_cache()
    nkv_l = cfg.n_kv_heads // world
    g = torch.Generator(device="cuda").manual_seed(args.seed + 7)
    for li in range(cfg.n_layers):  # the KV history (model.rs:103-114 public fields)
        k = torch.randn(ctx, nkv_l * cfg.head_dim, device="cuda", generator=g)
        v = torch.randn(ctx, nkv_l * cfg.head_dim, device="cuda", generator=g)
        cache.write_device(li, 0, k.data_ptr(), v.data_ptr(), ctx)
        del k, v
    cache.set_len(ctx)
    stream = torch.cuda.ExternalStream(model.stream)
    model.forward_argmax([1], cache)
    model.decode_steps(cache, W)
    torch.cuda.synchronize()
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    model.decode_steps(cache, K)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_max = max_over_ranks(world, ev0.elapsed_time(ev1))
    # e2e: the public call with host buffers (token in, logits + argmax out)
    V = cfg.vocab_size
    h_tok = np.zeros(1, dtype=np.uint32)
    h_tok[0] = model.forward_argmax([1], cache)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        tok, _ = model.forward_argmax([int(h_tok[0])], cache, logits=True)
        h_tok[0] = tok
    e2e_ms = max_over_ranks(world, 1000.0 * (time.perf_counter() - t0))
    # this library's kernel launches of one step (eager; the timed steps run
    # the same kernels)
    from minq_b200 import _lib
    n0 = _lib.lib().minq_kernel_launches()
    model.forward_argmax([int(h_tok[0])], cache)
    torch.cuda.synchronize()
    launches_per_step = _lib.lib().minq_kernel_launches() - n0
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    # per-GPU algorithmic bytes of a step: this rank's share of the quantized
    # weights and of the K/V history, the replicated f32 lm_head
    lm = 4.0 * V * cfg.hidden_size
    per_gpu = (model.weight_bytes - lm) / world + lm + \
        2 * 4 * cfg.n_kv_heads * cfg.head_dim * (ctx + W + K / 2) * cfg.n_layers / world
    gbs = per_gpu / (ms_max / K * 1e-3) / 1e9
    del cache, model
    torch.cuda.empty_cache()
    ar = allreduce_cost(world, cfg) if world > 1 else None
    if launches_per_step == 1:
        path = ("decode megakernel, one launch per token" if world == 1 else
                "decode megakernel, one launch per token per rank; o_proj and down_proj rows "
                "exchanged inside the launch as (value, epoch) pairs stored into every rank's "
                "peer-mapped slots")
    else:
        path = (f"per-op kernels replayed as a CUDA graph, {launches_per_step} launches per "
                f"token" + ("" if world == 1 else
                            ", all-reduces by the one-shot peer-memory kernel (NCCL when "
                            "MINQ_TP_NCCL=1 or peers cannot be mapped)"))
    if ar is not None and launches_per_step == 1:
        ar["note"] = ("the timed step does not call NCCL: its exchange runs inside the "
                      "megakernel; this is what the same 2 x n_layers all-reduces would cost "
                      "as separate NCCL calls")
    line = None
    if rank == 0:
        line = {
            "metric": "decode tok/s", "value": K / (ms_max / 1000.0), "unit": "tok/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_max / K,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"{TP_WORKLOAD}: Qwen3-4B shape, Q8_0, KV pre-filled at "
                                   f"{ctx} positions, 1 sequence",
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "cache_flush": "inputs > L2"},
            "e2e": {"value": K / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * V + 4},
            "gpu_launches": int(launches_per_step * K),
            "roofline": {"bound": "hbm", "kernel": "decode step (per GPU)", "achieved": gbs,
                         "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "traffic": None, "per_launch_bytes": per_gpu},
            "path": path,
            "allreduce": ar,
            "cpu_baseline": None,
            "clocks": clk,
        }
        if emit:
            print(json.dumps(line), flush=True)
    return line


def allreduce_cost(world, cfg):
    """Device time of the step's collective, measured beside it: 2 all-reduces
    of hidden_size f32 per layer (after o_proj and down_proj) as NCCL
    all-reduces of the same size over the same GPUs (torch's communicator),
    1000 back to back between CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    x = torch.ones(cfg.hidden_size, dtype=torch.float32, device="cuda")
    for _ in range(50):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 1000
    e0.record()
    for _ in range(n):
        dist.all_reduce(x)
    e1.record()
    torch.cuda.synchronize()
    us = max_over_ranks(world, 1000.0 * e0.elapsed_time(e1) / n)
    per_tok = 2 * cfg.n_layers
    return {"per_allreduce_us": us, "per_token": per_tok, "us_per_token": us * per_tok,
            "bytes": 4 * cfg.hidden_size,
            "how": "NCCL all-reduce of hidden_size f32 on the same GPUs, 1000 back to back"}


# A model small enough for the oracle whose heads and intermediate rows split
# over 2, 4 or 8 ranks (tensor-parallel parity inside the scaling run).
TP_PARITY_CFG = dict(hidden_size=512, intermediate_size=1024, n_layers=2, n_heads=16,
                     n_kv_heads=8, head_dim=64, vocab_size=300, max_seq_len=64, rope_theta=1e6,
                     rms_norm_eps=1e-6, has_qkv_bias=True, dtype="q8_0")
TP_PARITY_PROMPT = [5, 17, 230, 41, 99, 7]


def tp_parity(world, rank, local):
    """Tensor-parallel decode over the ranks of a 2-layer Q8_0 model with
    q|k|v bias against the oracle (rank 0): last-prompt logits max-abs < 1e-3
    and 9 greedy tokens identical (model.rs:932-940 tolerance)."""
    import torch
    import torch.distributed as dist
    import minq_b200 as mq
    from minq_b200 import synth
    from minq_b200.minq_format import ModelConfig, quantize_tensor_rule
    from oracle import oracle as orc
    cfg = ModelConfig(**TP_PARITY_CFG)
    recs = []
    for n, t, sh, d in synth.random_model_records(cfg, 31, qk_norm=True, with_bias=True):
        if n == "lm_head.weight":
            continue
        recs.append((n, 1, sh, orc.quantize(1, d)) if quantize_tensor_rule(n, sh) else (n, t, sh, d))
    model = mq.Model.from_tensors(cfg, recs)
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(mq.tp_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    model.tp_init(rank, world, bytes(uid.cpu().numpy().tobytes()))
    cache = model.new_cache()
    tok, logits = model.forward_argmax(TP_PARITY_PROMPT, cache, logits=True)
    toks = [tok]
    for _ in range(8):
        toks.append(model.forward_argmax([toks[-1]], cache))
    torch.cuda.synchronize()
    del cache, model
    res = None
    if rank == 0:
        om = orc.Model.from_tensors(TP_PARITY_CFG, {n: (t, sh, d) for n, t, sh, d in recs})
        ref = om.forward(TP_PARITY_PROMPT, om.new_cache())
        ref_toks, _ = orc.greedy_generate(om, TP_PARITY_PROMPT, 9)
        err = float(np.abs(np.asarray(logits) - ref).max())
        first = next((i for i, (a, b) in enumerate(zip(toks, ref_toks)) if a != b), None)
        res = {"ranks": world, "logits_max_abs": err, "tokens": len(toks),
               "tokens_match": toks == list(ref_toks), "first_mismatch": first,
               "ok": bool(err < 1e-3 and toks == list(ref_toks)),
               "model": "2 layers, hidden 512, 16/8 heads, hd 64, Q8_0 + q|k|v bias"}
    dist.barrier()
    return res


def run_batch(args, world, rank, local, steps=None, warmup=None, emit=True):
    """64 independent greedy sequences of the LLaMA-3-8B shape in Q4_0, 64 /
    world per rank (no collective): the prompts go through minq_prefill_batch
    (chunks of one sequence's tokens), then batched decode steps with
    each step's argmax fed back on the device. On one GPU (with the CPU
    baseline on) the line carries a parity record: sequence 0's greedy
    continuation inside the batch against the oracle decoding from a copy of
    sequence 0's cache. Returns rank 0's JSON line (printed when `emit`)."""
    import torch
    import minq_b200 as mq
    from minq_b200 import synth
    from dataclasses import replace
    torch.cuda.set_device(local)
    total = 64
    K = steps if steps is not None else args.steps
    W = warmup if warmup is not None else args.warmup
    prompt = args.prompt or 512
    if total % world:
        raise SystemExit(f"{BATCH_WORKLOAD}: 64 sequences do not split over {world} ranks")
    B = total // world
    cfg0, qk_norm, tied = synth.ARCH["llama3-8b"]
    if args.layers:
        cfg0 = replace(cfg0, n_layers=args.layers)
    cfg = replace(cfg0, max_seq_len=prompt + W + 2 * K + 16 + BATCH_PARITY_TOKENS)
    parity = world == 1 and not args.no_cpu_baseline
    model = build_model(mq, synth, cfg, qk_norm, tied, args.seed)
    weight_bytes = model.weight_bytes
    cache = model.new_cache(batch=B)
    rng = np.random.default_rng(args.seed + 100 + rank)
    prompts = rng.integers(0, cfg.vocab_size, (B, prompt))
    torch.cuda.synchronize()
    tp0 = time.perf_counter()
    # minq_prefill_batch: each sequence's prompt in chunks of 64 tokens on the
    # tensor cores, the last tokens as one batched step
    model.prefill_batch(prompts, cache, logits=False)
    torch.cuda.synchronize()
    prefill_s = max_over_ranks(world, time.perf_counter() - tp0)
    stream = torch.cuda.ExternalStream(model.stream)
    model.forward_batch_steps(cache, W)
    torch.cuda.synchronize()
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed_decode")
    ev0.record(stream)
    model.forward_batch_steps(cache, K)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_max = max_over_ranks(world, ev0.elapsed_time(ev1))
    # e2e: the public batched call with host tokens in and host argmax out
    toks = rng.integers(0, cfg.vocab_size, B).tolist()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        am, _ = model.forward_batch(toks, cache, logits=False)
        toks = [int(t) for t in am]
    e2e_ms = max_over_ranks(world, 1000.0 * (time.perf_counter() - t0))
    # this library's kernel launches of one step (an eager step; the timed
    # device continuation replays the same kernels)
    from minq_b200 import _lib
    n0 = _lib.lib().minq_kernel_launches()
    am, _ = model.forward_batch(toks, cache, logits=False)
    torch.cuda.synchronize()
    launches_per_step = _lib.lib().minq_kernel_launches() - n0
    toks = [int(t) for t in am]
    # parity state: sequence 0's cache (minq_cache_read reads sequence 0 of a
    # batch), then BATCH_PARITY_TOKENS greedy steps of the whole batch, of
    # which sequence 0's tokens are kept
    par_state = None
    if parity:
        n_pos = cache.len
        kvd = cfg.n_kv_heads * cfg.head_dim
        kall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
        vall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
        for li in range(cfg.n_layers):
            kall[li], vall[li] = cache.read(li, 0, n_pos)
        start = toks[0]
        gpu_toks = []
        for _ in range(BATCH_PARITY_TOKENS):
            am, _ = model.forward_batch(toks, cache, logits=False)
            toks = [int(t) for t in am]
            gpu_toks.append(toks[0])
        par_state = (n_pos, kall, vall, start, gpu_toks)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    # the step's algorithmic work per GPU: 2 flops per weight per sequence
    # (every projection and the lm_head), on the tensor cores from 16 sequences
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qd, kvd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    params = cfg.n_layers * (H * (qd + 2 * kvd) + qd * H + 3 * I * H) + cfg.vocab_size * H
    flops = 2.0 * params * B
    tfs = flops / (ms_max / K * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops") or 1590.0
    hbm_peak = peaks.get("hbm_gbs") or 6650.0
    kv_len = prompt + W + (K - 1) / 2.0
    step_bytes = float(weight_bytes) + B * 2 * 4 * cfg.n_kv_heads * hd * kv_len * cfg.n_layers
    gbs = step_bytes / (ms_max / K * 1e-3) / 1e9
    roof = {"bound": "hbm", "kernel": "batched step (per GPU)", "achieved": gbs,
            "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "traffic": None,
            "per_step_bytes": step_bytes,
            "note": "weights once per step + every sequence's K/V history; the tensor-core "
                    "view of the same step is roofline_tensor"}
    del cache, model
    torch.cuda.empty_cache()
    par = None
    if par_state is not None:
        try:
            from oracle import oracle as orc
            orc.set_threads(os.cpu_count() or 1)
            n_pos, kall, vall, start, gpu_toks = par_state
            par_state = None
            om = cpu_model(orc, synth, replace(cfg, max_seq_len=n_pos + BATCH_PARITY_TOKENS + 8),
                           qk_norm, tied, args.seed)
            oc = om.new_cache()
            oc.fill(kall, vall)
            del kall, vall
            ref_toks = []
            tok = start
            for _ in range(len(gpu_toks)):
                tok = int(orc.argmax(om.forward([tok], oc)))
                ref_toks.append(tok)
            first = next((i for i, (a, b) in enumerate(zip(gpu_toks, ref_toks)) if a != b), None)
            par = {"tokens": len(ref_toks), "match": first is None, "first_mismatch": first,
                   "from": f"sequence 0 of the batch of {B}: its cache after prefill + timed "
                           f"steps ({n_pos} positions)",
                   "gpu": "batched step (minq_forward_batch, tcgen05 projections)",
                   "oracle": "forward_token + argmax, one sequence"}
            del om, oc
        except Exception as e:  # the check must not sink the GPU number
            par = {"tokens": 0, "match": None, "first_mismatch": None,
                   "error": f"{type(e).__name__}: {e}"}
    line = None
    if rank == 0:
        line = {
            "metric": "decode tok/s (batched)", "value": total * K / (ms_max / 1000.0),
            "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 x 2 (hi/lo split inputs), f32 accumulate",
            "data": "synthetic",
            "config": {"workload": f"{BATCH_WORKLOAD}: LLaMA-3-8B shape, Q4_0, 64 sequences, "
                                   f"{prompt}-token prompts, {B} per GPU",
                       "layers": cfg.n_layers,
                       "parallelism": f"data{world}" if world > 1 else "single GPU",
                       "cache_flush": "inputs > L2"},
            "e2e": {"value": total * K / (e2e_ms / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
            "prefill": {"tokens": total * prompt, "tok_s": total * prompt / prefill_s,
                        "mode": "minq_prefill_batch: each sequence's prompt in chunks of 64 tokens "
                                "(projections and causal attention on the tensor cores), the last "
                                "tokens as one batched step"},
            "gpu_launches": int(launches_per_step * K),
            "roofline": roof,
            "roofline_tensor": {"achieved": tfs, "peak": peak, "unit": "TFLOP/s",
                                "frac": tfs / peak, "per_step_flops": flops},
            "cpu_baseline": None,
            "parity": par,
            "clocks": clk,
        }
        if emit:
            print(json.dumps(line), flush=True)
    return line


def _ppl_flops(cfg, n_pos, n_scored, context):
    """Algorithmic flops of scoring: 2 per weight per swept position (every
    projection), 2 per lm_head weight per scored position, and the causal
    q.k and p.v products (2 * 2 * hd per head per attended position)."""
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qd, kvd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    proj = cfg.n_layers * (H * (qd + 2 * kvd) + qd * H + 3 * I * H)
    attn = 0
    left = n_pos
    while left > 0:  # windows of `context` - 1 swept positions
        t = min(context - 1, left)
        attn += cfg.n_layers * cfg.n_heads * 4 * hd * t * (t + 1) // 2
        left -= t
    return 2.0 * proj * n_pos + 2.0 * cfg.vocab_size * H * n_scored + attn


def run_ppl(args, world, rank, local):
    """Perplexity evaluation (eval_ppl, ppl.rs:44-103) of the Qwen3-4B shape in
    Q4_0: K windows of 512 synthetic token ids, the windows split over the
    ranks (independent, no collective). The public call takes host token ids
    and returns the mean nll; it synchronises per 64-position chunk to read
    the chunk's f64 nll, so the device-timed value and e2e cover the same
    work."""
    from minq_b200 import synth
    from dataclasses import replace
    K, W, ctx = args.steps, args.warmup, PPL_CONTEXT
    cfg0, qk_norm, tied = synth.ARCH["qwen3-4b"]
    if args.layers:
        cfg0 = replace(cfg0, n_layers=args.layers)
    cfg = replace(cfg0, max_seq_len=ctx)
    rng = np.random.default_rng(args.seed + 7)
    tokens = rng.integers(0, cfg.vocab_size, K * ctx).astype(np.uint32)
    scored_per_window = ctx - 2
    # the reference arm: the oracle's eval_ppl on all host cores, one sample
    # window of `cpu_ctx` tokens per step (about 10 s; scored positions / s)
    cpu_ctx = 256

    def cpu_line(om, orc, steps, warm):
        for _ in range(warm):
            om.eval_ppl(tokens[:cpu_ctx], cpu_ctx)
        t0 = time.perf_counter()
        for i in range(steps):
            r = om.eval_ppl(tokens[i * cpu_ctx:(i + 1) * cpu_ctx], cpu_ctx)
        el = time.perf_counter() - t0
        return steps * (cpu_ctx - 2) / el, el, r

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import oracle as orc
        om = cpu_model(orc, synth, cfg, qk_norm, tied, args.seed)
        steps = max(1, min(K, 2))
        value, el, _ = cpu_line(om, orc, steps, 0)
        line = {
            "impl": "reference", "metric": "perplexity scored tok/s", "value": value,
            "unit": "tok/s", "n_gpus": args.gpus, "steps": steps, "warmup": 0,
            "ms_per_step": 1000 * el / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (f64 log-sum-exp)", "data": "synthetic",
            "config": {"workload": f"{PPL_WORKLOAD}: Qwen3-4B shape, Q4_0, windows of {ctx}",
                       "cache_flush": "weights 3.8 GB > L2"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": orc.max_threads(),
                             "kind": "port",
                             "sample": f"{steps} windows of {cpu_ctx} tokens "
                                       f"({cpu_ctx - 2} scored each), {el:.1f} s"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    import torch
    import minq_b200 as mq
    from minq_b200 import _lib
    torch.cuda.set_device(local)
    if K % world:
        raise SystemExit(f"{PPL_WORKLOAD}: {K} windows do not split over {world} ranks")
    kw = K // world
    mine = tokens[rank * kw * ctx:(rank + 1) * kw * ctx]
    model = build_model(mq, synth, cfg, qk_norm, tied, args.seed)
    stream = torch.cuda.ExternalStream(model.stream)
    warm = rng.integers(0, cfg.vocab_size, max(1, W) * ctx).astype(np.uint32)
    mq.eval_ppl(model, warm, ctx)
    torch.cuda.synchronize()
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    n0 = _lib.lib().minq_kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed_ppl")
    t0 = time.perf_counter()
    ev0.record(stream)
    res = mq.eval_ppl(model, mine, ctx)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall_ms = 1000.0 * (time.perf_counter() - t0)
    torch.cuda.nvtx.range_pop()
    launches = _lib.lib().minq_kernel_launches() - n0
    barrier(world)
    clk = clocks.stop()
    ms_max = max_over_ranks(world, ev0.elapsed_time(ev1))
    e2e_ms = max_over_ranks(world, wall_ms)
    scored = K * scored_per_window
    assert res.scored_positions == kw * scored_per_window
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    flops = _ppl_flops(cfg, kw * (ctx - 1), kw * scored_per_window, ctx)
    tfs = flops / (ms_max * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops") or 1590.0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import oracle as orc
            om = cpu_model(orc, synth, cfg, qk_norm, tied, args.seed)
            v, el, _ = cpu_line(om, orc, 1, 0)
            cpu = {"value": v, "unit": "tok/s", "cores": orc.max_threads(), "kind": "port",
                   "sample": f"one window of {cpu_ctx} tokens ({cpu_ctx - 2} scored) of the "
                             f"same model, {el:.1f} s"}
            del om
        except Exception as e:  # the baseline must not sink the GPU number
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {type(e).__name__}: {e}"}
    if rank == 0:
        print(json.dumps({
            "metric": "perplexity scored tok/s", "value": scored / (ms_max / 1000.0),
            "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": max(1, W),
            "ms_per_step": ms_max / kw, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "projections bf16 x 2 (hi/lo split inputs) on the tensor cores, f32 "
                     "accumulate; f32 lm_head; f64 log-sum-exp",
            "data": "synthetic",
            "config": {"workload": f"{PPL_WORKLOAD}: Qwen3-4B shape, Q4_0, {K} windows of "
                                   f"{ctx} seeded token ids ({kw} per GPU)",
                       "layers": cfg.n_layers, "context": ctx,
                       "parallelism": f"data{world}" if world > 1 else "single GPU",
                       "cache_flush": "inputs > L2: 3.8 GB of weights per 64-position chunk",
                       "mean_nll_rank0": res.mean_nll},
            "e2e": {"value": scored / (e2e_ms / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * ctx, "d2h_bytes_per_step": 8 * scored_per_window},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "window (sweep + lm_head + nll)",
                         "achieved": tfs, "peak": peak, "unit": "TFLOP/s", "frac": tfs / peak,
                         "traffic": None, "per_launch_flops": flops / kw},
            "cpu_baseline": cpu,
            "clocks": clk,
        }), flush=True)
    del model


def run_sampler(args):
    """Device draws (minq_sampler_sample_device) on seeded N(0, 3^2) logits of
    151,936 entries, timed with CUDA events over K draws per setting; the
    line's value is the temperature 0.8 / top_k 40 / top_p 0.9 setting. The
    CPU baseline is the oracle's Sampler::sample on the same logits."""
    import torch
    import minq_b200 as mq
    n, K, W = 151936, args.steps, args.warmup
    x = (np.random.default_rng(args.seed).standard_normal(n) * 3.0).astype(np.float32)
    d = torch.from_numpy(x).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    settings = {"t0.8_k40_p0.9": (0.8, 40, 0.9), "t1_nofilter": (1.0, 0, 1.0),
                "t1_k0_p0.9": (1.0, 0, 0.9), "greedy": (0.0, 0, 1.0)}
    res = {}
    stream = torch.cuda.current_stream()
    for name, (t, k, p) in settings.items():
        smp = mq.Sampler(t, k, p, args.seed)
        for _ in range(max(3, W)):
            smp.sample_device(d, out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K):
            smp.sample_device(d, out)
        e1.record(stream)
        torch.cuda.synchronize()
        res[name] = {"us_per_draw": 1000.0 * e0.elapsed_time(e1) / K}
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as orc
        o = orc.Sampler(0.8, 40, 0.9, args.seed)
        t0 = time.perf_counter()
        nd = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0) or nd < 3:
            o.sample(x)
            nd += 1
        el = time.perf_counter() - t0
        cpu = {"value": nd / el, "unit": "draws/s", "cores": 1, "kind": "port",
               "sample": f"{nd} draws of the t0.8_k40_p0.9 setting, {el:.1f} s"}
    us = res["t0.8_k40_p0.9"]["us_per_draw"]
    print(json.dumps({
        "metric": "device sampling draws/s", "value": 1e6 / us, "unit": "draws/s",
        "n_gpus": 1, "steps": K, "warmup": max(3, W), "ms_per_step": us / 1000.0,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 probabilities, f64 sums", "data": "synthetic",
        "config": {"workload": f"{SAMPLER_WORKLOAD}: Sampler::sample over 151936 logits",
                   "settings": res, "cache_flush": "none: 0.6 MB of logits stay in L2, as "
                   "after a decode step's lm_head"},
        "cpu_baseline": cpu,
    }), flush=True)


def run_attn(args, world, rank, local):
    """The decode-attention op (minq_attn_decode) over the sweep; the line's
    value is the B = 8, L = 8192 point, `sweep` holds every point. Each
    point's K/V history (N(0, 1), 2*4*B*8*128*(L+1) bytes) exceeds L2 from
    L = 8192 at B = 8; smaller points are timed with an L2 flush between
    calls."""
    import torch
    from minq_b200 import _lib
    torch.cuda.set_device(local)
    L_ = _lib.lib()
    nh, nkv, hd, eps = 32, 8, 128, 1e-6
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    sweep = []
    points = [(B, L) for B in (1, 8, 64) for L in (512, 2048, 8192, 32768)]
    if args.attn_points:
        points = [tuple(int(v) for v in pt.split("x")) for pt in args.attn_points.split(",")]
    for B, L in points:
        ms_ = L + 1
        g = torch.Generator(device="cuda").manual_seed(B * 100003 + L)
        kc = torch.randn((B, nkv, ms_, hd), device="cuda", generator=g)
        vc = torch.randn((B, nkv, ms_, hd), device="cuda", generator=g)
        q = torch.randn((B, nh, hd), device="cuda", generator=g)
        kn = torch.randn((B, nkv, hd), device="cuda", generator=g)
        vn = torch.randn((B, nkv, hd), device="cuda", generator=g)
        pos = torch.arange(ms_, dtype=torch.float32, device="cuda")[:, None]
        inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device="cuda", dtype=torch.float32) / hd))
        cs, sn = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
        out = torch.empty((B, nh, hd), device="cuda")
        wsb = L_.minq_attn_workspace_bytes(B, nh, L + 1)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
        big = 8.0 * B * nkv * hd * (L + 1) > 4 * (126 << 20)

        def call():
            _lib.check(L_.minq_attn_decode(
                P(q), P(kn), P(vn), None, None, eps, P(cs), P(sn), B, nh, nkv, hd, L, P(kc),
                P(vc), nkv * ms_ * hd, ms_ * hd, hd, P(out), P(ws), wsb,
                C.c_void_p(s.cuda_stream)))
        for _ in range(max(3, args.warmup)):
            call()
        torch.cuda.synchronize()
        tot, n = 0.0, max(8, args.steps // 4)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(n):
            if not big:
                flush.zero_()
            e0.record(s)
            call()
            e1.record(s)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        us = 1000.0 * tot / n
        byts = 8.0 * B * nkv * hd * (L + 1) + 4.0 * B * (2 * nh + 4 * nkv) * hd
        sweep.append({"B": B, "L": L, "us": round(us, 2), "GB_s": round(byts / us / 1e3, 1),
                      "frac": round(byts / us / 1e3 / peak, 3)})
        del kc, vc, q, kn, vn, out, ws
        torch.cuda.empty_cache()
    head = next((x for x in sweep if x["B"] == 8 and x["L"] == 8192), sweep[0])
    if rank == 0:
        print(json.dumps({
            "metric": "decode attention GB/s", "value": head["GB_s"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["us"] / 1000.0, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{ATTN_WORKLOAD}: RoPE + append + attend, B = 8, L = 8192",
                       "cache_flush": "256 MB buffer written between calls below 4 x L2"},
            "roofline": {"bound": "hbm", "kernel": "attn_tma_kernel + attn_combine_kernel",
                         "achieved": head["GB_s"], "peak": peak, "unit": "GB/s",
                         "frac": head["frac"], "traffic": None},
            "sweep": sweep, "cpu_baseline": None,
        }), flush=True)


def main():
    args = parse()
    world, rank, local = dist_init()
    try:
        if args.impl == "reference" and args.workload in (TP_WORKLOAD, BATCH_WORKLOAD,
                                                          ATTN_WORKLOAD, SAMPLER_WORKLOAD):
            run_reference_workload(args, rank)
        elif args.workload == ATTN_WORKLOAD:
            if rank == 0:
                run_attn(args, world, rank, local)
        elif args.workload == TP_WORKLOAD:
            run_tp(args, world, rank, local)
        elif args.workload == BATCH_WORKLOAD:
            run_batch(args, world, rank, local)
        elif args.workload == PPL_WORKLOAD:
            run_ppl(args, world, rank, local)
        elif args.workload == SAMPLER_WORKLOAD:
            if rank == 0:
                run_sampler(args)
        elif args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_minq(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
