#!/usr/bin/env python
"""Benchmark of the B200 token loop (HanzCEO/TinyMiniGo's decode path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5|attn]

Workload c2 (default): the 1B-class Llama decoder
(hidden 2048, 16 layers, 32/8 heads, head_dim 64, intermediate 8192, vocab
128256, tied embeddings) on seeded random BF16 weights, a 64-token random
prompt, greedy decode of 256 tokens.  One step = the 256-token greedy decode
from the prefilled 64-token context (the cache is rewound to 64 between
steps).  value = decode tok/s over the K timed steps on the device (CUDA
events on the library's stream, inputs resident; weights 2.47 GB > L2, so no
flush is needed); e2e = the same metric through the public API
(tmg_generate with host prompt buffers, tokens read back every 8 steps),
decode tok/s as the reference's main.rs defines it.

The decode runs as ONE persistent kernel per step (decode_fused_kernel: all
256 tokens, every layer, the LM head and the argmax), so the roofline entry
describes that kernel: achieved = algorithmic bytes per launch (BF16
weights of every layer and the LM head plus the KV rows read, per token,
times 256 tokens) / the launch's device time.  traffic = DRAM bytes of an
ncu capture of the same kernel on a smaller case, scaled per algorithmic
byte (profiles/decode_fused_c2.json).

With --gpus N > 1 every rank runs an independent replica of c2 (the 1B
config fits one GPU; "replicas only", weak scaling): `value` is c2's
whole-job throughput at every N.  The same line carries a `c4_tp` block: the
8B-class config decoded as ONE sequence by all N
ranks of the same process group, 128-token prompt, greedy 512 per step:
decode tok/s of the one sequence (strong scaling), per-GPU algorithmic GB/s
and its fraction of the HBM peak.  By default (TMG_C4_MULTI=fused) one
fused decode kernel is spread over every rank's SMs: each GPU holds the full
weights, reads only the rows its CTAs own, and stores every exchanged value
and KV row into every GPU's memory over NVLink (tmg_fused_group_init).
TMG_C4_MULTI=nccl shards the weights tensor-parallel instead (q/k/v and
gate/up split by heads and rows, o/down by input columns with one NCCL
allreduce per sublayer, the LM head by vocabulary rows) and adds the
allreduce time per token from a profiling pass.  At N = 1 the block is c4
on one GPU.  NCCL logs its communicator set-up (NCCL_DEBUG=INFO, subsystem
INIT) on stderr.

--impl reference times the reference's CPU algorithm (the C++ restatement in
oracle/, with the reference's thread policy) on the host cores, rank 0 only,
for the same workload (c2); each step is a bounded sample of its decode loop
(stated in cpu_baseline.sample).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 64
GEN = 256
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print("[bench]", *a, file=sys.stderr, flush=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init(world: int, local_rank: int, backend: str = "nccl"):
    """The process group of a multi-GPU run (one process per GPU, replicas):
    used only for the barriers around the timed region and the max over
    ranks.  A short timeout so that ranks waiting on a dead peer fail."""
    if world <= 1:
        return None
    import datetime

    import torch
    import torch.distributed as dist

    # rank 0 prints exactly one JSON line on stdout: NCCL's log (the
    # communicators it sets up, with their rank counts) goes to stderr
    os.environ["NCCL_DEBUG"] = os.environ.get("TMG_BENCH_NCCL_DEBUG", "INFO")
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    kw = {"device_id": torch.device("cuda", local_rank)} if backend == "nccl" else {}
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    return dist


def replica_tok_s(world: int, tokens_per_rank: int, max_elapsed_ms: float) -> float:
    """Whole-job decode throughput of `world` independent replicas: all the
    tokens every rank produced over the slowest rank's time."""
    return world * tokens_per_rank / (max_elapsed_ms / 1e3)


def max_over_ranks(dist, v: float) -> float:
    """The slowest rank's time: every rank gets the max of v over ranks."""
    if dist is None:
        return v
    import torch

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (C++ restatement of the reference's AVX2 path)
# ---------------------------------------------------------------------------
def cpu_decode_sample(cfg, tensors, prompt, n_tokens):
    from oracle import oracle

    t0 = time.time()
    om = oracle.OracleModel(cfg, tensors)
    log(f"oracle model ready in {time.time() - t0:.1f}s, threads={oracle.num_threads()}")
    t0 = time.perf_counter()
    logits = om.forward_seq(prompt)
    t_pre = time.perf_counter() - t0
    first = logits.copy()
    tok = oracle.argmax(logits)
    ids = [tok]
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        logits = om.forward_token(tok)
        tok = oracle.argmax(logits)
        ids.append(tok)
    t_dec = time.perf_counter() - t0
    return {"decode_tok_s": n_tokens / t_dec, "prefill_tok_s": len(prompt) / t_pre,
            "cores": oracle.num_threads(), "decode_s": t_dec, "prefill_s": t_pre,
            "ids": ids, "first_logits": first}


C2_WORKLOAD = "c2: 1B-class Llama, tied, 64-token prompt, greedy 256 decode"


def c2_config(world: int) -> dict:
    """The `config` of a c2 line (both arms print the same one)."""
    return {"workload": C2_WORKLOAD, "global_batch": world, "seq_len": PROMPT + GEN,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (2.47 GB of weights per token)"}


def make_c2(device: str, layers: int = 0):
    from tinyminigo_b200 import synth

    cfg = synth.CONFIGS["c2"]
    if layers:
        cfg = synth.with_layers(cfg, layers)
    t0 = time.time()
    w = synth.make_weights(cfg, 2024, device=device)
    log(f"c2 weights generated on {device} in {time.time() - t0:.1f}s")
    return cfg, w


def run_reference(args, rank):
    if rank != 0:
        return
    import torch

    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cfg, w = make_c2(dev)
    from oracle import oracle
    from tinyminigo_b200 import synth

    prompt = synth.random_prompt(cfg["vocab_size"], PROMPT, 7)
    om = oracle.OracleModel(cfg, w)
    logits = om.forward_seq(prompt)
    tok = int(np.argmax(logits))
    per_step = 4  # decode tokens per step: a bounded sample of the 256-token loop
    for _ in range(args.warmup):
        for _ in range(per_step):
            tok = oracle.argmax(om.forward_token(tok))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(per_step):
            tok = oracle.argmax(om.forward_token(tok))
    dt = time.perf_counter() - t0
    v = args.steps * per_step / dt
    sample = (f"each step: {per_step} greedy decode tokens of the 256-token loop, after a "
              f"{PROMPT}-token prefill; reference thread policy (gemv nproc/4, gemm nproc)")
    out = {
        "impl": "reference", "metric": "decode_tok_s", "value": round(v, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 weights)",
        "data": "synthetic (seeded N(0,0.02^2) bf16 weights, random prompt)",
        "config": c2_config(args.gpus),
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": oracle.num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def c2_bytes(cfg):
    h, L, I, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["intermediate_size"], cfg["vocab_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kd = cfg["num_key_value_heads"] * cfg["head_dim"]
    per_layer = {"qkv_gemv": 2 * (qd + 2 * kd) * h, "o_gemv": 2 * h * qd,
                 "gateup_gemv": 2 * 2 * I * h, "down_gemv": 2 * h * I}
    return per_layer, 2 * V * h


def run_ours(args, rank, world, local_rank):
    import torch

    torch.cuda.set_device(local_rank)
    dist = dist_init(world, local_rank)
    from tinyminigo_b200 import synth
    from tinyminigo_b200.model import GenParams, Model, ModelConfig, generate

    cfg, w = make_c2("cuda", args.ncu_layers if args.ncu_steps else 0)
    mc = ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                     cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                     cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)
    t0 = time.time()
    model = Model.from_tensors(mc, w, device=local_rank)
    log(f"weights uploaded in {time.time() - t0:.1f}s ({model.weight_bytes() / 1e9:.3f} GB)")
    prompt = synth.random_prompt(cfg["vocab_size"], PROMPT, 7 + rank)
    stream = torch.cuda.ExternalStream(model.stream_handle(), device=local_rank)

    # --- device-resident decode loop (value) ---
    cache = model.new_cache(PROMPT + GEN + 8)
    if args.ncu_steps:
        # profiling mode: one prefill and a short greedy decode, nothing else
        logits = model.forward_seq(prompt, cache)
        model.decode([int(np.argmax(logits))], cache, args.ncu_steps)
        cache.close()
        model.close()
        return
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one untimed prefill first (first-use allocations of the prefill scratch)
    warm = model.new_cache(PROMPT + 8)
    model.forward_seq(prompt, warm)
    model.sync()
    warm.close()
    with torch.cuda.stream(stream):
        pe0.record(stream)
        logits = model.forward_seq(prompt, cache)
        pe1.record(stream)
    model.sync()
    prefill_ms = pe0.elapsed_time(pe1)
    t0_tok = int(np.argmax(logits))

    def step():
        cache_trunc(cache, PROMPT)
        model.decode([t0_tok], cache, GEN, wait=False)

    for _ in range(args.warmup):
        step()
    model.sync()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        model.sync()
        torch.cuda.synchronize()
    elapsed_ms = ev0.elapsed_time(ev1)
    if dist is not None:
        dist.barrier()
    elapsed_ms = max_over_ranks(dist, elapsed_ms)
    value = replica_tok_s(world, GEN * args.steps, elapsed_ms)
    per_tok_ms = elapsed_ms / (args.steps * GEN)
    layer_bytes, head_bytes = c2_bytes(cfg)
    L = cfg["num_hidden_layers"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    mean_ctx = PROMPT + GEN / 2
    kv_bytes_tok = L * (2 * kvd * 4 * mean_ctx + 2 * kvd * 4)
    weight_bytes_tok = L * sum(layer_bytes.values()) + head_bytes
    step_gbs = (weight_bytes_tok + kv_bytes_tok) / (per_tok_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    # greedy tokens of the decode loop (for the record and a sanity check)
    cache_trunc(cache, PROMPT)
    dec_toks = model.decode([t0_tok], cache, GEN)[0]

    if args.trace:
        # device timeline of one captured step (globaltimer stamps), in us
        # from the step's first kernel start
        cache_trunc(cache, PROMPT)
        tl = model.trace_decode([t0_tok], cache)
        base = min(r[1] for r in tl)
        with open(args.trace, "w") as f:
            f.write("kernel            start   wait0   wait1     end     dur  gap_from_prev_end\n")
            prev_end = base
            for r in tl:
                s, w0, w1, e = [(v - base) / 1e3 for v in r[1:]]
                f.write(f"{r[0]:14s} {s:7.2f} {w0:7.2f} {w1:7.2f} {e:7.2f} {e - w0:7.2f} "
                        f"{w0 - (prev_end - base) / 1e3:7.2f}\n")
                prev_end = r[4]
            f.write(f"step total {(max(r[4] for r in tl) - base) / 1e3:.2f} us\n")

    # --- roofline of the dominant kernel: the fused decode kernel is the
    # whole timed step (one launch per step) ---
    launch_ms = elapsed_ms / args.steps
    alg_bytes_launch = (weight_bytes_tok + kv_bytes_tok) * GEN
    achieved = alg_bytes_launch / (launch_ms / 1e3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "decode_fused_c2.json"
    if tf.exists():
        ratio = json.loads(tf.read_text()).get("dram_bytes_per_algorithmic_byte")
        if ratio:
            traffic = int(ratio * alg_bytes_launch)

    # --- end to end through the public API (host buffers) ---
    e2e_vals, h2d, d2h = [], 0, 0
    gp = GenParams(max_tokens=GEN)
    for i in range(args.warmup + args.steps):
        t_a = time.perf_counter()
        out = generate(model, prompt, gp)
        wall = time.perf_counter() - t_a
        if i >= args.warmup:
            e2e_vals.append((len(out.tokens) - 1) / max(wall - out.prefill_secs, 1e-9))
    # bytes the generate call copies: the prompt in; the first-step logits,
    # then per 8-step chunk the state block (256 B) and the token buffer, and
    # a final state + tokens + error word out
    h2d = PROMPT * 4
    d2h = cfg["vocab_size"] * 4 + (GEN // 8 + 1) * (256 + GEN * 4) + 4
    e2e = statistics.median(e2e_vals) * world
    ok = out.tokens[1:] == [int(t) for t in dec_toks[:GEN - 1]] and out.tokens[0] == t0_tok

    # --- CPU baseline and oracle parity (rank 0, N = 1) ---
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_decode_sample(cfg, w, prompt, args.cpu_tokens)
        except Exception as e:  # pragma: no cover
            log("cpu baseline failed:", e)
    parity = None
    if cpu:
        gpu_ids = [t0_tok] + [int(t) for t in dec_toks[:args.cpu_tokens]]
        diff = np.abs(logits - cpu["first_logits"])
        parity = {"checker": "oracle (C++ restatement of the reference's CPU path)",
                  "first_step_max_abs_logit_diff": round(float(diff.max()), 6),
                  "first_step_logits_within_1e-3_rel_1e-2_abs":
                      bool(np.all(diff <= 1e-2 + 1e-3 * np.abs(cpu["first_logits"]))),
                  "greedy_ids_compared": len(gpu_ids),
                  "greedy_ids_equal": gpu_ids == cpu["ids"]}
    cache.close()
    model.close()

    # --- the tensor-parallel 8B block over the same ranks ---
    c4 = None
    if not args.no_c4:
        c4_head = {"workload": "c4: 8B-class Llama, untied, 128-token prompt, greedy 512 decode",
                   "parallelism": c4_parallelism(world), "n_gpus": world,
                   "scaling": "strong", "steps": min(args.steps, 3), "warmup": 3}
        try:
            v4, ms4, gbs4, per_gpu4, extra4 = measure_c4(
                args, rank, world, local_rank, dist, steps=min(args.steps, 3), warmup=3,
                host_leg=world == 1 and not args.no_cpu_baseline)
        except Exception as e:  # the c2 line still prints; the block says what failed
            log(f"c4 block failed: {e!r}")
            c4 = {**c4_head, "error": repr(e)[:300]}
        else:
            peak4, _ = peaks()
            c4 = {**c4_head,
                  "decode_tok_s": round(v4, 2), "ms_per_step": round(ms4, 3),
                  "per_gpu_algorithmic_gbs": round(gbs4, 1), "peak": peak4,
                  "frac": round(gbs4 / peak4, 4),
                  "algorithmic_bytes_per_token_per_gpu": int(per_gpu4), **extra4}

    if rank == 0:
        clocks = clk.summary()
        res = {
            "metric": "decode_tok_s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 weights)",
            "data": "synthetic (seeded N(0,0.02^2) bf16 weights, random prompt)",
            "config": c2_config(world),
            "decode_hbm_gbs": round(step_gbs, 1),
            "decode_hbm_frac": round(step_gbs / peak, 4),
            "prefill_tok_s": round(PROMPT / (prefill_ms / 1e3), 1),
            "roofline": {"bound": "hbm", "kernel": "decode_fused_kernel",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": int(alg_bytes_launch),
                         "launch_ms": round(launch_ms, 3), "peak_kind": peak_kind},
            "clocks": clocks,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps,  # one decode_fused_kernel launch per step
            "greedy_consistent": bool(ok),
        }
        if parity:
            res["parity"] = parity
        if c4:
            res["c4_tp"] = c4
        if cpu:
            res["cpu_baseline"] = {
                "value": round(cpu["decode_tok_s"], 4), "unit": "tok/s", "cores": cpu["cores"],
                "kind": "port",
                "sample": f"c2 prefill {PROMPT} tokens ({cpu['prefill_tok_s']:.1f} tok/s) + "
                          f"{args.cpu_tokens} greedy decode tokens, reference thread policy"}
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def model_config(cfg):
    from tinyminigo_b200.model import ModelConfig

    return ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                       cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                       cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)


def base_line(args, world, metric, value, unit, ms_per_step, workload, scaling, clocks, **extra):
    d = {"metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world,
         "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
         "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
         "dtype": "f32 (bf16 weights)", "data": "synthetic (seeded N(0,0.02^2) bf16 weights, "
         "random prompt)", "config": workload, "clocks": clocks}
    d.update(extra)
    return d


def run_c3(args, rank, world, local_rank):
    """C3: a 2048-token random prompt through the prefill path of the c2
    shape (tcgen05 GEMMs, prefill attention); one step = one prefill from an
    empty cache.  value = prompt tokens / s on the device; e2e = the same
    through forward_seq with the prompt and the logits in host memory."""
    import torch

    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    from tinyminigo_b200 import synth
    from tinyminigo_b200.model import Model

    T = 2048
    cfg, w = make_c2("cuda")
    model = Model.from_tensors(model_config(cfg), w, device=local_rank)
    prompt = synth.random_prompt(cfg["vocab_size"], T, 13)
    cache = model.new_cache(T + 8)
    stream = torch.cuda.ExternalStream(model.stream_handle(), device=local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def step():
        cache.truncate(0)
        model.forward_seq(prompt, cache, want_logits=False)

    for _ in range(args.warmup):
        step()
    model.sync()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        model.sync()
    ms = ev0.elapsed_time(ev1) / args.steps
    # e2e: host prompt in, host logits out, every step
    t_e = []
    for _ in range(args.steps):
        cache.truncate(0)
        t0 = time.perf_counter()
        model.forward_seq(prompt, cache)
        t_e.append(time.perf_counter() - t0)
    h, L = cfg["hidden_size"], cfg["num_hidden_layers"]
    layer_params = sum(v // 2 for v in c2_bytes(cfg)[0].values())
    nq, d = cfg["num_attention_heads"], cfg["head_dim"]
    flops = (2 * T * layer_params * L + L * 4 * d * nq * T * (T + 1) // 2
             + 2 * cfg["vocab_size"] * h)
    tflops = flops / (ms / 1e3) / 1e12
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(pk.get("bf16_tflops", 1590.0))
    extra = {}
    if not args.no_cpu_baseline:
        extra = c3_cpu_leg(model, cfg, w, prompt)
    res = base_line(args, world, "prefill_tok_s", T / (ms / 1e3), "tok/s", ms,
                    {"workload": "c3: c2 shape, 2048-token random prompt, prefill", "global_batch": 1,
                     "seq_len": T, "parallelism": "single GPU"}, "weak", clk.summary(),
                    roofline={"bound": "tensor", "kernel": "gemm_tc_kernel (whole prefill)",
                              "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                              "frac": round(tflops / peak, 4), "traffic": None,
                              "algorithmic_flops_per_step": int(flops),
                              "note": "f32 activations as bf16 hi+lo: the tensor cores run 2x these "
                                      "flops for the linear layers"},
                    e2e={"value": round(T / statistics.median(t_e), 2), "unit": "tok/s",
                         "h2d_bytes_per_step": T * 4, "d2h_bytes_per_step": cfg["vocab_size"] * 4},
                    **extra)
    print(json.dumps(res), flush=True)
    cache.close()
    model.close()


def c4_mode(world):
    """How c4 runs over `world` ranks: "single" on one GPU; "fused" (the
    default at world > 1, TMG_C4_MULTI=fused) spreads the fused decode
    kernel over every rank's SMs with the full weights on each GPU;
    TMG_C4_MULTI=nccl shards the weights tensor-parallel with NCCL
    allreduces between per-kernel launches."""
    if world == 1:
        return "single"
    mode = os.environ.get("TMG_C4_MULTI", "fused")
    if mode not in ("fused", "nccl"):
        raise SystemExit(f"TMG_C4_MULTI={mode!r}: expected fused or nccl")
    return mode


def c4_parallelism(world):
    mode = c4_mode(world)
    return {"single": "single GPU", "fused": f"fused kernel over {world} GPUs",
            "nccl": f"tp{world}"}[mode]


def measure_c4(args, rank, world, local_rank, dist, steps, warmup, host_leg):
    """C4: the 8B-class config sharded tensor-parallel over the ranks of
    `dist` (one process per GPU, NCCL allreduce per sublayer; world 1: one
    GPU); 128-token prompt, then a 512-token greedy decode per step from the
    rewound cache.  Returns (tok/s of the one sequence, max over ranks;
    ms per step; per-GPU algorithmic GB/s; allreduce ms per token; extra
    fields) on every rank.  Every rank takes the same collective steps."""
    import ctypes

    import torch

    from tinyminigo_b200 import synth
    from tinyminigo_b200._lib import check, lib
    from tinyminigo_b200.model import Model

    P4, G4 = 128, 512
    cfg = synth.CONFIGS["c4"]
    mode = c4_mode(world)
    tp = uid_b = None
    if world > 1:
        uid = (ctypes.c_uint8 * 128)()
        if rank == 0:
            check(lib().tmg_tp_unique_id(uid))
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device="cuda")
        dist.broadcast(t, 0)
        uid_b = bytes(t.cpu().tolist())
        if mode == "nccl":
            tp = (uid_b, rank, world)
    t0 = time.time()
    if host_leg:  # the oracle needs every tensor in host memory
        w = synth.make_weights(cfg, 2025, device="cuda")
        model = Model.from_tensors(model_config(cfg), w, device=local_rank, tp=tp)
    else:  # one tensor in host memory at a time
        w = None
        model = Model.from_tensors(model_config(cfg), synth.iter_weights(cfg, 2025, device="cuda"),
                                   device=local_rank, tp=tp)
    log(f"c4 weights generated and uploaded in {time.time() - t0:.1f}s "
        f"({model.weight_bytes() / 1e9:.2f} GB on this rank)")
    prompt = synth.random_prompt(cfg["vocab_size"], P4, 17)
    cache = model.new_cache(P4 + G4 + 8)
    logits = model.forward_seq(prompt, cache)
    tok = int(np.argmax(logits))
    if mode == "fused":
        model.fused_group(cache, uid_b, rank, world)
    stream = torch.cuda.ExternalStream(model.stream_handle(), device=local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def step():
        cache.truncate(P4)
        model.decode([tok], cache, G4, wait=False)

    for _ in range(warmup):
        step()
    model.sync()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    model.sync()
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, ev0.elapsed_time(ev1)) / steps
    value = G4 / (ms / 1e3)
    extra = {"multi_gpu_path": {"single": "fused kernel on one GPU",
                                "fused": "one fused kernel spread over all ranks' SMs "
                                         "(peer stores over NVLink, full weights per rank)",
                                "nccl": "tensor-parallel shards, NCCL allreduce per sublayer"}[mode]}
    if mode != "fused":
        # the collectives' share: one profiling pass (kernels launched one
        # at a time with CUDA events around each, so slower than the graph)
        cache.truncate(P4)
        n_prof = 8
        prof = model.profile_decode([tok], cache, n_prof)
        ar_ms_tok = max_over_ranks(dist, prof["allreduce"][0] / n_prof)
        ag_ms_tok = max_over_ranks(dist, prof["allgather_step_end"][0] / n_prof)
        prof_ms_tok = max_over_ranks(dist, sum(v[0] for v in prof.values()) / n_prof)
        extra.update({
            "profile_pass_ms_per_token": round(prof_ms_tok, 4),
            "profile_pass_ms_per_token_by_kernel": {k: round(v[0] / n_prof, 4)
                                                    for k, v in prof.items() if v[1]},
            "allreduce_ms_per_token": round(ar_ms_tok, 4),
            "allreduces_per_token": int(prof["allreduce"][1] // n_prof),
            "allgather_step_end_ms_per_token": round(ag_ms_tok, 4)})
    h, L, I, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["intermediate_size"], cfg["vocab_size"]
    qd, kd = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]
    wbytes = 2 * (L * ((qd + 2 * kd) * h + h * qd + 3 * I * h) + V * h)
    kvb = L * 2 * kd * 4 * (P4 + G4 / 2)
    per_gpu = (wbytes + kvb) / world
    gbs = per_gpu / (ms / 1e3 / G4) / 1e9
    if host_leg:
        cache.truncate(P4)
        gpu_ids = model.decode([tok], cache, 16)[0].tolist()
        extra.update(c4_cpu_leg(cfg, w, prompt, logits, [tok] + gpu_ids[:15]))
    if dist is not None:
        dist.barrier()
    cache.close()
    model.close()
    return value, ms, gbs, per_gpu, extra


def run_c4(args, rank, world, local_rank):
    """C4 as its own line (see measure_c4)."""
    import torch

    torch.cuda.set_device(local_rank)
    dist = dist_init(world, local_rank)
    with ClockSampler(local_rank) as clk:
        value, ms, gbs, per_gpu, extra = measure_c4(
            args, rank, world, local_rank, dist, args.steps, args.warmup,
            world == 1 and not args.no_cpu_baseline)
    peak, peak_kind = peaks()
    if rank == 0:
        res = base_line(args, world, "decode_tok_s", value, "tok/s", ms,
                        {"workload": "c4: 8B-class, untied, 128-token prompt, greedy 512",
                         "global_batch": 1, "seq_len": 128 + 512,
                         "parallelism": c4_parallelism(world)},
                        "strong", clk.summary(),
                        roofline={"bound": "hbm", "kernel": "decode step (per-GPU bytes)",
                                  "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(gbs / peak, 4), "traffic": None,
                                  "algorithmic_bytes_per_token_per_gpu": int(per_gpu),
                                  "peak_kind": peak_kind},
                        gpu_launches=None, **extra)
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_c5(args, rank, world, local_rank):
    """C5: 16 streams, each with its own random 32768-token prompt prefilled,
    then 256 sampled steps (T 0.8, top-k 40, top-p 0.95, penalty 1.1, seed
    base + i) through generate_batch.  value = aggregate decode tok/s: the
    generate_batch time minus the time of the same 16 prefills measured
    alone (the API prefills inside generate).  The subtraction is paired:
    the same generate_batch with max_tokens = 1 (its 16 prefills and the
    first token) is timed right after, so the value is the 16 x (steps - 1)
    tokens after the first over the time difference.  Both calls are timed
    with CUDA events recorded on the library's stream around them."""
    import torch

    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    from tinyminigo_b200 import synth
    from tinyminigo_b200.model import GenParams, Model, generate_batch

    M, T5, G5 = 16, args.c5_ctx, args.c5_steps
    cfg, w = make_c2("cuda")
    model = Model.from_tensors(model_config(cfg), w, device=local_rank)
    prompts = np.stack([synth.random_prompt(cfg["vocab_size"], T5, 100 + i) for i in range(M)])
    cache = model.new_cache(T5 + G5 + 8, n_streams=M)
    params = [GenParams(max_tokens=G5, temperature=0.8, top_k=40, top_p=0.95,
                        repetition_penalty=1.1, seed=1000 + i) for i in range(M)]
    params1 = [GenParams(max_tokens=1, temperature=0.8, top_k=40, top_p=0.95,
                         repetition_penalty=1.1, seed=1000 + i) for i in range(M)]
    stream = torch.cuda.ExternalStream(model.stream_handle(), device=local_rank)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with ClockSampler(local_rank) as clk:  # the long call first: it sizes the token buffers
        ev[0].record(stream)
        outs = generate_batch(model, prompts, params, cache=cache)
        ev[1].record(stream)
        ev[2].record(stream)
        generate_batch(model, prompts, params1, cache=cache)
        ev[3].record(stream)
        ev[3].synchronize()
    t_all = ev[0].elapsed_time(ev[1]) / 1e3
    t_pre = ev[2].elapsed_time(ev[3]) / 1e3
    dec = max(t_all - t_pre, 1e-9)
    n_tok = sum(len(o) - 1 for o in outs)
    extra = {}
    if not args.no_cpu_baseline:
        extra = c5_cpu_leg(model, cache, cfg, w, T5, [int(o[0]) for o in outs])
    kv_step = M * cfg["num_hidden_layers"] * 2 * cfg["num_key_value_heads"] * cfg["head_dim"] * 4 * (T5 + G5 / 2)
    wbytes = sum(c2_bytes(cfg)[0].values()) * cfg["num_hidden_layers"] + c2_bytes(cfg)[1]
    gbs = (wbytes + kv_step) * (G5 - 1) / dec / 1e9
    peak, peak_kind = peaks()
    res = base_line(args, world, "decode_tok_s", n_tok / dec, "tok/s", dec * 1e3,
                    {"workload": f"c5: c2 shape, 16 streams x {T5}-token prompts, {G5} sampled "
                                 "steps (T 0.8, k 40, p 0.95, penalty 1.1)", "global_batch": M,
                     "seq_len": T5 + G5, "parallelism": "single GPU"}, "weak", clk.summary(),
                    roofline={"bound": "hbm", "kernel": "decode steps (weights once + 16 KV)",
                              "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(gbs / peak, 4), "traffic": None,
                              "peak_kind": peak_kind},
                    prefill_and_first_token_s=round(t_pre, 2), generate_batch_s=round(t_all, 2),
                    timing="CUDA events on the library's stream: generate_batch minus the same "
                           "call with max_tokens 1 (16 prefills + the first token)",
                    **extra)
    print(json.dumps(res), flush=True)
    cache.close()
    model.close()


def run_c2i8(args, rank, world, local_rank):
    """C2 with int8 layer weights (the reference's TMG_I8=1: per-row
    quantized q/k/v/o/gate/up/down, BF16 LM head): 64-token prompt, 256
    greedy tokens per step through the per-step graph of int8 GEMVs.  value
    = decode tok/s on the device; roofline = algorithmic bytes per token
    (int8 layer weights + row scales + BF16 LM head + KV) over the step
    time.  Parity rides along: the first 8 greedy ids and the first-step
    logits against the oracle's int8 model."""
    import torch

    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    from tinyminigo_b200 import synth
    from tinyminigo_b200.model import Model

    cfg, w = make_c2("cuda")
    os.environ["TMG_I8"] = "1"
    try:
        model = Model.from_tensors(model_config(cfg), w, device=local_rank)
    finally:
        del os.environ["TMG_I8"]
    prompt = synth.random_prompt(cfg["vocab_size"], PROMPT, 7)
    cache = model.new_cache(PROMPT + GEN + 8)
    logits = model.forward_seq(prompt, cache)
    t0_tok = int(np.argmax(logits))
    stream = torch.cuda.ExternalStream(model.stream_handle(), device=local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def step():
        cache.truncate(PROMPT)
        model.decode([t0_tok], cache, GEN, wait=False)

    for _ in range(args.warmup):
        step()
    model.sync()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        model.sync()
    ms = ev0.elapsed_time(ev1) / args.steps
    cache.truncate(PROMPT)
    gpu_ids = [t0_tok] + [int(t) for t in model.decode([t0_tok], cache, 8)[0]]
    h, L, I, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["intermediate_size"], cfg["vocab_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kd = cfg["num_key_value_heads"] * cfg["head_dim"]
    layer_b = (qd + 2 * kd) * h + h * qd + 3 * I * h + 4 * (qd + 2 * kd + 2 * h + 2 * I)
    kvb = L * (2 * kd * 4 * (PROMPT + GEN / 2) + 2 * kd * 4)
    tok_b = L * layer_b + 2 * V * h + kvb
    gbs = tok_b / (ms / 1e3 / GEN) / 1e9
    peak, peak_kind = peaks()
    extra = {}
    if not args.no_cpu_baseline:
        from oracle import oracle

        om = oracle.OracleModel(cfg, w, i8=True)
        ref = om.forward_seq(prompt)
        ids = [oracle.argmax(ref)]
        for _ in range(8):
            ids.append(oracle.argmax(om.forward_token(ids[-1])))
        diff = np.abs(logits - ref)
        extra["parity"] = {"checker": "oracle int8 model (TMG_I8=1 arms)",
                           "first_step_max_abs_logit_diff": round(float(diff.max()), 6),
                           "first_step_logits_within_1e-3_rel_1e-2_abs":
                               bool(np.all(diff <= 1e-2 + 1e-3 * np.abs(ref))),
                           "greedy_ids_compared": len(ids), "greedy_ids_equal": gpu_ids == ids}
    res = base_line(args, world, "decode_tok_s", GEN / (ms / 1e3), "tok/s", ms,
                    {"workload": "c2 with int8 layer weights (TMG_I8=1): 1B-class, tied, "
                                 "64-token prompt, greedy 256 decode", "global_batch": 1,
                     "seq_len": PROMPT + GEN, "parallelism": "single GPU"}, "weak", clk.summary(),
                    roofline={"bound": "hbm", "kernel": "decode step (int8 GEMVs + BF16 LM head)",
                              "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(gbs / peak, 4), "traffic": None,
                              "algorithmic_bytes_per_token": int(tok_b), "peak_kind": peak_kind},
                    **extra)
    res["dtype"] = "int8 weights, f32 activations, i32 dots"
    print(json.dumps(res), flush=True)
    cache.close()
    model.close()


def run_attn(args, rank, world, local_rank):
    """Attention kernels alone, through the op-level C ABI (rank 0): decode
    attention of one stream over --attn-ctx cached positions (default 131072;
    32 query / 8 kv heads, head dim 64: 537 MB of f32 K/V, larger than L2,
    flushed between runs) and causal prefill attention of 2048 rows (the c3
    shape).  value = the decode kernel's algorithmic GB/s (K and V read
    once); the prefill's TFLOP/s rides along.  The decode kernel is the
    TMA-staged one; TMG_ATTN_KERNEL=reg or tiled selects the register-
    streaming or the cp.async tiled kernel instead, for comparison."""
    import ctypes

    import torch

    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    from tinyminigo_b200._lib import check, lib

    h = ctypes.c_void_p()
    check(lib().tmg_create(local_rank, None, ctypes.byref(h)))
    stream = torch.cuda.ExternalStream(lib().tmg_stream(h), device=local_rank)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(1)
    nq, nkv, d = 32, 8, 64

    def timed(call):
        for _ in range(args.warmup):
            call()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    n_ctx = args.attn_ctx
    q = torch.randn(nq * d, device="cuda", generator=g)
    k = torch.randn(n_ctx, nkv * d, device="cuda", generator=g)
    v = torch.randn(n_ctx, nkv * d, device="cuda", generator=g)
    o = torch.zeros(nq * d, device="cuda")
    with ClockSampler(local_rank) as clk:
        ms_dec = timed(lambda: check(lib().tmg_op_attn_decode(h, P(q), P(k), P(v), n_ctx, nq, nkv,
                                                              d, P(o)), h))
        T = 2048
        qp = torch.randn(T, nq * d, device="cuda", generator=g)
        kp = torch.randn(T, nkv * d, device="cuda", generator=g)
        vp = torch.randn(T, nkv * d, device="cuda", generator=g)
        op = torch.zeros(T, nq * d, device="cuda")
        ms_pf = timed(lambda: check(lib().tmg_op_attn_prefill(h, P(qp), P(kp), P(vp), T, 0, nq,
                                                              nkv, d, P(op)), h))
    lib().tmg_destroy(h)
    dec_bytes = 2 * n_ctx * nkv * d * 4
    gbs = dec_bytes / (ms_dec / 1e3) / 1e9
    pf_flop = 4 * d * nq * T * (T + 1) // 2
    peak, peak_kind = peaks()
    kern = {"reg": "attn_decode_reg_kernel", "tiled": "attn_decode_kernel"}.get(
        os.environ.get("TMG_ATTN_KERNEL", "tma"), "attn_decode_tma_kernel<64>")
    if os.environ.get("TMG_ATTN_TILED", "0") == "1":
        kern = "attn_decode_kernel"
    res = base_line(args, world, "decode_attention_gbs", gbs, "GB/s", ms_dec,
                    {"workload": f"attention kernels: decode over {n_ctx} positions (32/8 heads, "
                                 "d 64, one stream); causal prefill of 2048 rows",
                     "global_batch": 1, "seq_len": n_ctx, "parallelism": "single GPU",
                     "l2": "flushed between runs (256 MB write)"}, "weak", clk.summary(),
                    roofline={"bound": "hbm", "kernel": kern, "achieved": round(gbs, 1),
                              "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                              "traffic": None, "peak_kind": peak_kind},
                    prefill_attention={"ms": round(ms_pf, 3),
                                       "tflops": round(pf_flop / (ms_pf / 1e3) / 1e12, 1),
                                       "kernel": ("attn_prefill_tiled_kernel<64>"
                                                  if os.environ.get("TMG_PREFILL_ATTN") == "simt"
                                                  else "attn_pf_split_q/kv_kernel + "
                                                       "attn_prefill_tc_kernel"),
                                       "flops": "algorithmic: 4 d per (q head, row, visible key)"},
                    timing="CUDA events around the op call (includes its ticket memset and "
                           "position upload for decode)")
    res["dtype"] = "f32"
    res["data"] = "synthetic (random normal q, K, V)"
    print(json.dumps(res), flush=True)


def c3_cpu_leg(model, cfg, w, prompt, n=256):
    """The C3 host leg: the oracle prefills the first n prompt tokens (timed,
    reference thread policy: GEMM on every core, attention single-threaded);
    the GPU prefills the same n tokens into a fresh cache; the last rows'
    logits are compared (1e-3 relative / 1e-2 absolute)."""
    from oracle import oracle

    part = np.asarray(prompt[:n])
    om = oracle.OracleModel(cfg, w)
    t0 = time.perf_counter()
    ref = om.forward_seq(part)
    t_cpu = time.perf_counter() - t0
    c = model.new_cache(n + 8)
    g = model.forward_seq(part, c)
    c.close()
    diff = np.abs(g - ref)
    return {
        "cpu_baseline": {"value": round(n / t_cpu, 4), "unit": "tok/s", "cores": oracle.num_threads(),
                         "kind": "port", "sample": f"prefill of the first {n} prompt tokens "
                                                   "(reference thread policy)"},
        "parity": {"tokens": n, "max_abs_logit_diff": round(float(diff.max()), 6),
                   "logits_within_1e-3_rel_1e-2_abs": bool(np.all(diff <= 1e-2 + 1e-3 * np.abs(ref))),
                   "argmax_equal": int(np.argmax(g)) == oracle.argmax(ref)},
    }


def c4_cpu_leg(cfg, w, prompt, gpu_logits, gpu_ids, n_steps=16):
    """The C4 host leg (one GPU): the oracle prefills the 128-token prompt and
    decodes n_steps greedy tokens (timed separately, reference thread
    policy); parity: the prefill's logits against the GPU's, and the greedy
    ids against the GPU's up to the first step whose top-2 margin is below
    1e-3 (reported)."""
    from oracle import oracle

    om = oracle.OracleModel(cfg, w)
    t0 = time.perf_counter()
    logits = om.forward_seq(np.asarray(prompt))
    t_pre = time.perf_counter() - t0
    diff = np.abs(gpu_logits - logits)
    ids, first_diff, tie = [], None, None
    t0 = time.perf_counter()
    for i in range(n_steps):
        top = np.argsort(-logits)[:2]
        tok = oracle.argmax(logits)
        ids.append(tok)
        if first_diff is None and i < len(gpu_ids) and gpu_ids[i] != tok:
            first_diff = i
            tie = float(logits[top[0]] - logits[top[1]])
        logits = om.forward_token(tok)
    t_dec = time.perf_counter() - t0
    return {
        "cpu_baseline": {"value": round(n_steps / t_dec, 4), "unit": "tok/s",
                         "cores": oracle.num_threads(), "kind": "port",
                         "sample": f"{len(prompt)}-token prefill ({len(prompt) / t_pre:.2f} tok/s) "
                                   f"+ {n_steps} greedy decode tokens, reference thread policy"},
        "parity": {"prefill_max_abs_logit_diff": round(float(diff.max()), 6),
                   "prefill_logits_within_1e-3_rel_1e-2_abs":
                       bool(np.all(diff <= 1e-2 + 1e-3 * np.abs(gpu_logits))),
                   "greedy_steps": n_steps, "greedy_ids_equal": first_diff is None,
                   "first_divergence": first_diff, "margin_there": tie},
    }


def c5_cpu_leg(model, cache, cfg, w, T5, first, n_steps=8):
    """The C5 host leg: a CPU prefill of 16 x 32K tokens is out of reach, so
    the oracle (the reference's CPU algorithm) decodes stream 0 from the
    GPU-prefilled f32 KV cache of its prompt: n_steps greedy steps, timed
    (cpu_baseline), while the GPU decodes the same tokens from the same
    cache; the logits of every step are compared (1e-3 relative / 1e-2
    absolute) and so are the greedy ids."""
    from oracle import oracle

    M, L = cache.n_streams, cfg["num_hidden_layers"]
    for i in range(M):
        cache.truncate(T5, stream=i)
    om = oracle.OracleModel(cfg, w)
    for layer in range(L):
        om.kv_load(layer, cache.keys_flat(layer, 0), cache.values_flat(layer, 0))
    toks = np.asarray(first, np.uint32)
    t_cpu, max_diff, within, ids_equal = 0.0, 0.0, True, True
    for _ in range(n_steps):
        g = model.forward_token(toks, cache)[0]
        t0 = time.perf_counter()
        ref = om.forward_token(int(toks[0]))
        t_cpu += time.perf_counter() - t0
        diff = np.abs(g - ref)
        max_diff = max(max_diff, float(diff.max()))
        within = within and bool(np.all(diff <= 1e-2 + 1e-3 * np.abs(ref)))
        nxt = oracle.argmax(ref)
        ids_equal = ids_equal and int(np.argmax(g)) == nxt
        toks = np.full(M, nxt, np.uint32)
    return {
        "cpu_baseline": {"value": round(n_steps / t_cpu, 4), "unit": "tok/s",
                         "cores": oracle.num_threads(), "kind": "port",
                         "sample": f"stream 0 only: {n_steps} greedy decode steps at {T5} "
                                   "context from the GPU-prefilled f32 KV cache (reference "
                                   "thread policy; attention single-threaded)"},
        "parity": {"stream": 0, "steps": n_steps, "context": T5,
                   "max_abs_logit_diff": round(max_diff, 6),
                   "logits_within_1e-3_rel_1e-2_abs": within, "greedy_ids_equal": ids_equal},
    }


def cache_trunc(cache, n):
    cache.truncate(n)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "attn", "c2i8"], default="c2",
                    help="c2 (default): the headline decode; c3: 2048-token prefill; "
                         "c4: 8B tensor-parallel decode over the ranks; c5: 16 streams at 32K "
                         "context, sampled; attn: the attention kernels alone; c2i8: c2 with "
                         "int8 layer weights (TMG_I8=1)")
    ap.add_argument("--cpu-tokens", type=int, default=8)
    ap.add_argument("--c5-ctx", type=int, default=32768, help="c5: prompt length per stream")
    ap.add_argument("--c5-steps", type=int, default=256, help="c5: sampled steps")
    ap.add_argument("--attn-ctx", type=int, default=131072,
                    help="attn: cached positions of the decode attention")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c4", action="store_true",
                    help="c2: leave out the tensor-parallel 8B block")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="profiling mode: prefill + this many decode steps, no timing, no output")
    ap.add_argument("--trace", default="",
                    help="write the device timeline of one decode step to this file")
    ap.add_argument("--ncu-layers", type=int, default=0,
                    help="profiling mode only: build the c2 shape with this many layers")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "c3":
        run_c3(args, rank, world, local_rank)
    elif args.workload == "c4":
        run_c4(args, rank, world, local_rank)
    elif args.workload == "c5":
        run_c5(args, rank, world, local_rank)
    elif args.workload == "attn":
        run_attn(args, rank, world, local_rank)
    elif args.workload == "c2i8":
        run_c2i8(args, rank, world, local_rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
