"""Benchmark: greedy batch-1 decode of the Qwen2.5-0.5B-architecture int4 model (config 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl enx|reference]

A step is one decode token: the whole decoder (24 layers of int4 projections, f16-KV GQA
attention), the tied int8 head and the sampler, for one sequence, at positions 32..95 (a
32-id prompt decoded out to 64 tokens, as config 0 specifies; longer runs restart the
sequence every 64 tokens, the re-prefill being outside the timed events).  Weights are seeded
random-init (normal(0, 0.02), norm gains 1), quantised with the reference's scheme; the prompt
is uniform random ids.  Each step streams all 351 MB of weights, more than the 126 MB L2, so
consecutive steps cannot reuse cached weights.

value: device-fed loop (enx_decode_loop: the sampled id feeds the next step on the GPU), CUDA
events on the context stream, max over ranks.  e2e: the public per-token API
(Session.decode_step -> enx_decode_step), which copies each step's inputs host->device from
pinned memory and reads the id back, timed with events around the same steps.

N > 1: one independent replica per GPU (independent sequences are data-parallel; the path has no
exchange step), weak scaling.  --impl reference times the CPU restatement of the reference's
path (oracle/, the reference itself is TypeScript/WebGPU and cannot run here) on rank 0.
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

from enargeia_b200.checkpoint import QWEN2_0_5B, build_model_file  # noqa: E402

PROMPT = 32
GEN = 64            # config 0 decodes 64 tokens per sequence
SEED = 20251201     # model seed
METRIC = "decode tok/s (greedy, batch 1, Qwen2.5-0.5B int4 + int8 head, ctx 32..96)"
MODEL_DIR = Path(os.environ.get("ENX_MODEL_DIR", "/tmp/enx_models"))


def model_path() -> Path:
    return MODEL_DIR / f"qwen2.5-0.5b-random-s{SEED}-q4q8.enargeia"


def algorithmic_bytes():
    """Bytes one decode step must move at the reference layout: every weight range once
    (packed + scales + zeros + norms + biases), plus the per-step KV reads."""
    from enargeia_b200.format import read_enargeia

    f = read_enargeia(model_path())
    weights = sum(t.nbytes for t in f.tensors.values())
    head = f.quant("model.embed_tokens.weight")
    return f, weights, head.nbytes


# ---------------------------------------------------------------------------------------------
# clocks


class ClockSampler:
    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.t = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        time.sleep(0.25)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        loaded = [r[0] for r in rows if r[0] > 0.5 * r[1]] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# GPU arm


def run_enx(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from enargeia_b200 import build, kernels as K
    from enargeia_b200.session import GREEDY, Model, Session

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if local_rank == 0:
        build_model_file(QWEN2_0_5B, SEED, model_path())
    if world > 1:
        dist.barrier()
    else:
        build_model_file(QWEN2_0_5B, SEED, model_path())
    f, weight_bytes, head_bytes = algorithmic_bytes()
    cfg = QWEN2_0_5B

    ctx = PROMPT + GEN + 1
    m = Model(cfg, local_rank).load(model_path()).kv_alloc(ctx, 1)
    stream = torch.cuda.ExternalStream(m.stream_handle(), device=dev)
    prompt = [int(v) for v in np.random.default_rng(1000 + rank).integers(0, cfg.vocab, PROMPT)]
    greedy = [GREEDY]

    def restart():
        m.reset(0)
        m.prefill(0, prompt)
        return m.sample_prefill(0, GREEDY, 0.5)

    def segments(total):
        while total > 0:
            n = min(GEN - 1, total)
            yield n
            total -= n

    # warm-up: W device-fed steps and W public-API steps (graphs captured, clocks up)
    first = restart()
    m.decode_loop([first], greedy, np.full(max(args.warmup, 1), 0.5, np.float32), max(args.warmup, 1))
    first = restart()
    s = Session(m, GREEDY)
    tok = first
    for _ in range(max(args.warmup, 1)):
        tok = s.decode_step(tok)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # --- value: device-fed loop -----------------------------------------------------------
    loop_ids = []
    ms_total = 0.0
    with ClockSampler(local_rank) as clocks:
        barrier()
        for n in segments(args.steps):
            first = restart()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            m.decode_loop([first], greedy, np.full(n, 0.5, np.float32), n, sync=False)
            e1.record(stream)
            m.synchronize()
            ms_total += e0.elapsed_time(e1)
            loop_ids.append([first] + list(m.loop_ids(n)[:, 0]))
        barrier()
    launches_per_step = m.step_launches()
    ms_total = max_over_ranks(ms_total)
    value = world * args.steps / (ms_total / 1e3)

    # --- e2e: public per-token API ---------------------------------------------------------
    e2e_ms = 0.0
    api_ids = []
    barrier()
    for n in segments(args.steps):
        first = restart()
        sess = Session(m, GREEDY)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ids = [first]
        e0.record(stream)
        tok = first
        for _ in range(n):
            tok = sess.decode_step(tok)
            ids.append(tok)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms += e0.elapsed_time(e1)
        api_ids.append(ids)
    barrier()
    e2e_ms = max_over_ranks(e2e_ms)
    e2e_value = world * args.steps / (e2e_ms / 1e3)
    consistent = api_ids == loop_ids

    # --- TTFT: a 32-id prompt in, the first sampled id out, through the public Session API ------
    # (host ids -> enx_prefill -> enx_sample_prefill -> 4-byte id back), wall clock, median of 10
    ttfts = []
    for _ in range(12):
        m.reset(0)
        sess = Session(m, GREEDY)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        sess.prime(prompt)
        sess.sample_from_prefill()
        ttfts.append(time.perf_counter() - t0)
    ttft_ms = statistics.median(ttfts[2:]) * 1e3
    ttft_ms = max_over_ranks(ttft_ms)

    # --- roofline: the step's weight-streaming kernels (persistent layers + tensor-core head) ----
    # One decode step at position PROMPT + 1, then those two kernels alone, `reps` times back to
    # back on the context stream (enx_launch_step_kernel: no sampler, no host copies), timed with
    # events on that stream.  Each pass streams every weight once (351 MB > 126 MB L2).
    restart_tok = restart()
    Session(m, GREEDY).decode_step(restart_tok)
    torch.cuda.synchronize()
    from enargeia_b200._lib import call

    reps = 50
    call("enx_launch_step_kernel", m.handle, 1, 3)  # warm
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    call("enx_launch_step_kernel", m.handle, 1, reps)
    e1.record(stream)
    torch.cuda.synchronize()
    kern_us = e0.elapsed_time(e1) / reps * 1e3
    shares = kernel_shares(m, stream, ms_total / args.steps * 1e3)
    kv_positions = PROMPT + 2  # positions attended by the step at position PROMPT + 1
    kern_bytes = weight_bytes + cfg.layers * 2 * kv_positions * cfg.kv_dim * 2
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    achieved = kern_bytes / (kern_us / 1e6) / 1e9
    step_bytes = weight_bytes  # plus KV reads, added below at the mean position
    mean_pos = PROMPT + GEN / 2
    kv_bytes = cfg.layers * 2 * int(mean_pos) * cfg.kv_dim * 2
    step_achieved = (step_bytes + kv_bytes) / (ms_total / args.steps / 1e3) / 1e9

    traffic = None
    tf = ROOT / "profiles" / "k_mega_decode_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")

    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_total / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4/int8 weights x f32 activations, f32 accumulate, f16 KV",
        "data": "synthetic: seeded random-init weights normal(0,0.02) quantised int4 + int8 head; uniform random prompt ids",
        "config": {"workload": "config 0: greedy batch-1 decode, 24 layers, hidden 896, 14q/2kv x 64, FFN 4864, "
                               "vocab 151936, prompt 32 -> 64 new tokens, f16 KV",
                   "batch_per_gpu": 1, "parallelism": f"replicas x{world} (independent sequences)",
                   "l2": "inputs larger than L2: 351 MB of weights streamed per step vs 126 MB L2",
                   "step_bytes": step_bytes + kv_bytes},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 116, "d2h_bytes_per_step": 4,
                "api": "Session.decode_step -> enx_decode_step (pinned step block in, 4-byte id out)"},
        "roofline": {"kernel": "k_mega<1,8> (persistent decode: 24 layers) + k_head_tc<2> (tied int8 head, tcgen05), batch 1",
                     "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": kern_bytes, "launch_us": round(kern_us, 2),
                     "peak_source": f"{peak_src} MEASURED_PEAKS.json hbm_gbs (burst copy)"},
        "step_roofline": {"bound": "hbm", "bytes_per_step": step_bytes + kv_bytes,
                          "achieved": round(step_achieved, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(step_achieved / hbm, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "launches_per_step": launches_per_step,
        "ttft": {"value": round(ttft_ms, 3), "unit": "ms", "prompt_ids": PROMPT,
                 "api": "Session.prime + Session.sample_from_prefill (host ids in, first id out), median of 10"},
        "kernel_shares": shares,
        "ids_consistent_loop_vs_api": consistent,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(f, prompt, budget_s=args.cpu_budget)
    m.close()
    if not args.no_blocks:
        # the work that shards, measured at this N beside the replicated headline: config 4 (DP
        # sequences, 256/N per GPU, a bounded number of steps) and config 2 (vocab-sharded head)
        out["dp_batched"] = scaling_block(run_batched(block_args(args, steps=BLOCK_STEPS + args.warmup + 8, batch=256),
                                                      rank, world, local_rank, emit=False))
        out["vocab_sharded"] = scaling_block(run_head(block_args(args, steps=50, batch=64), rank, world, local_rank,
                                                      emit=False))
    if rank == 0:
        print(json.dumps(out), flush=True)


BLOCK_STEPS = 64  # timed config-4 steps in the default line's dp_batched block


def block_args(args, **kw):
    b = argparse.Namespace(**vars(args))
    b.no_cpu_baseline = True
    for k, v in kw.items():
        setattr(b, k, v)
    return b


def scaling_block(line):
    """The fields of a workload's own line that the scaling run compares across N."""
    if line is None:
        return None
    keep = ["metric", "value", "unit", "n_gpus", "steps", "ms_per_step", "scaling"]
    blk = {k: line[k] for k in keep if k in line}
    blk["frac"] = line.get("roofline", {}).get("frac")
    blk["roofline_kernel"] = line.get("roofline", {}).get("kernel")
    blk["workload"] = line.get("config", {}).get("workload")
    if "positions_timed" in line.get("config", {}):
        blk["positions_timed"] = line["config"]["positions_timed"]
    return blk


# ---------------------------------------------------------------------------------------------
# launch counting


def count_library_launches(fn) -> int:
    """Kernels of libenx (all named enx::k_*) launched by fn(), counted from the CUDA activity
    torch's profiler records; used for workloads whose API launches kernels eagerly."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        name = ev.name or ""
        if ev.device_type == torch.autograd.DeviceType.CUDA and ("enx::k_" in name or name.startswith("k_")):
            n += 1
    return n


# ---------------------------------------------------------------------------------------------
# config 3: chunked prefill (bench.py --workload config3)

PREFILL_LEN, PREFILL_CHUNK = 2048, 256
PREFILL_METRIC = "prefill tok/s (2048-token prompt in 256-query chunks, Qwen2.5-0.5B int4 + int8 head)"


def run_prefill(args, rank, world, local_rank):
    """One step = enx_prefill of a fresh 2048-token uniform-random prompt in 256-query chunks: per
    chunk and layer the q|k|v, o, gate|up and down projections on the tcgen05 limb GEMM, RoPE and
    the f16 cache writes, causal GQA attention over the cache so far; the tied head for the last
    row.  N > 1: independent replicas (independent prompts are data-parallel)."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from enargeia_b200 import build
    from enargeia_b200._lib import MatmulQ4Dims, call
    from enargeia_b200.session import Model

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if local_rank == 0:
        build_model_file(QWEN2_0_5B, SEED, model_path())
    if world > 1:
        dist.barrier()
    cfg = QWEN2_0_5B
    m = Model(cfg, local_rank).load(model_path()).kv_alloc(PREFILL_LEN + 1, 1)
    stream = torch.cuda.ExternalStream(m.stream_handle(), device=dev)
    prompt = [int(v) for v in np.random.default_rng(3000 + rank).integers(0, cfg.vocab, PREFILL_LEN)]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    steps = min(args.steps, 20)
    for _ in range(args.warmup):
        m.reset(0)
        m.prefill(0, prompt, PREFILL_CHUNK)
    def one_prefill():
        m.reset(0)
        m.prefill(0, prompt, PREFILL_CHUNK)

    launches_per_step = count_library_launches(one_prefill)  # an extra, untimed prefill
    with ClockSampler(local_rank) as clocks:
        barrier()
        dev_ms, wall = 0.0, 0.0
        for _ in range(steps):
            m.reset(0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record(stream)
            m.prefill(0, prompt, PREFILL_CHUNK)  # host ids in; returns when the chunks are done
            e1.record(stream)
            torch.cuda.synchronize()
            wall += time.perf_counter() - t0
            dev_ms += e0.elapsed_time(e1)
        barrier()
    dev_ms = max_over_ranks(dev_ms)
    wall_ms = max_over_ranks(wall * 1e3)
    value = world * steps * PREFILL_LEN / (dev_ms / 1e3)
    # roofline: layer 0's gate projection at the chunk size, alone, 20 launches on the model stream
    g = m.tensor_view("model.layers.0.mlp.gate_proj.weight")
    x = torch.randn(PREFILL_CHUNK, g["cols"], device=dev)
    out = torch.empty(PREFILL_CHUNK * g["rows"], device=dev)
    d = MatmulQ4Dims(PREFILL_CHUNK, g["rows"], g["cols"], 0, 64, g["cols"] // 64, g["rows"], 0,
                     min(g["rows"], 65535), 0, 0, 0)
    sh = C.c_void_p(m.stream_handle())

    def launch():
        call("enx_matmul_q4", C.c_void_p(x.data_ptr()), C.c_void_p(g["packed"]), C.c_void_p(g["scales"]),
             C.c_void_p(g["zeros"]), None, C.c_void_p(out.data_ptr()), C.byref(d), sh)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    gemm_us = e0.elapsed_time(e1) / reps * 1e3
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    i8_peak = 2 * bf16
    groups = -(-PREFILL_CHUNK // 32)
    mma_ops = 2 * (-(-g["rows"] // 128) * 128) * groups * 192 * g["cols"]  # 6 limb columns x 32 tokens
    useful = 2 * PREFILL_CHUNK * g["rows"] * g["cols"]
    proj_macs = cfg.layers * (cfg.hidden * (cfg.hidden + 2 * cfg.kv_dim) + cfg.hidden * cfg.hidden
                              + 3 * cfg.hidden * cfg.intermediate)
    attn_macs = cfg.layers * cfg.heads * cfg.head_dim * 2 * (PREFILL_LEN * (PREFILL_LEN + 1) // 2)
    step_flops = 2 * (proj_macs * PREFILL_LEN + attn_macs + cfg.vocab * cfg.hidden)
    out_line = {
        "metric": PREFILL_METRIC,
        "value": round(value, 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4/int8 weights x f32 activations (exact int8-limb tensor-core block sums, f64 accumulate), f16 KV",
        "data": "synthetic: seeded random-init weights normal(0,0.02); 2048 uniform random prompt ids",
        "config": {"workload": "config 3: chunked prefill of a 2048-token prompt in 256-query chunks through the "
                               "config-0 model", "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: 351 MB of weights per chunk",
                   "step_flops": step_flops},
        "e2e": {"value": round(world * steps * PREFILL_LEN / (wall_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": PREFILL_LEN * 4, "d2h_bytes_per_step": 0,
                "api": "Model.prefill -> enx_prefill (host ids in, synchronous), wall clock"},
        "roofline": {"kernel": f"enx_matmul_q4 M={PREFILL_CHUNK} gate ({g['rows']}x{g['cols']}, tcgen05 limb GEMM)",
                     "bound": "tensor", "achieved": round(mma_ops / (gemm_us / 1e6) / 1e12, 2),
                     "peak": i8_peak, "unit": "TOP/s (int8 MMA)",
                     "frac": round(mma_ops / (gemm_us / 1e6) / 1e12 / i8_peak, 4), "traffic": None,
                     "useful_tflops": round(useful / (gemm_us / 1e6) / 1e12, 2), "launch_us": round(gemm_us, 2),
                     "peak_source": "2 x measured MEASURED_PEAKS.json bf16_tflops (dense int8 = 2x dense bf16)"},
        "step_tflops": round(step_flops / (dev_ms / steps / 1e3) / 1e12, 2),
        "gpu_launches": launches_per_step * steps,
        "launches_per_step": launches_per_step,
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(out_line), flush=True)
    m.close()


# ---------------------------------------------------------------------------------------------
# config 4: batched sampled decode (bench.py --workload config4)

BATCH_PROMPT, BATCH_CTX = 512, 2048
BATCH_METRIC = "batched sampled decode tok/s (256 sequences, prompt 512 -> context 2048, T 0.7 / top-p 0.9 / rp 1.1)"


def run_batched(args, rank, world, local_rank, emit=True):
    """Independent sequences, data-parallel: each rank decodes its share of the 256 with its own
    weight replica and caches (strong scaling: total work fixed).  Projections and the tied head run
    on the tensor-core GEMM (exact integer block sums), attention reads each sequence's f16 cache."""
    import torch
    import torch.distributed as dist

    from enargeia_b200 import build
    from enargeia_b200.session import Model, SamplingParams, mulberry32

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if local_rank == 0:
        build_model_file(QWEN2_0_5B, SEED, model_path())
    if world > 1:
        dist.barrier()
    total = args.batch
    B = total // world
    if B * world != total or B < 1:
        raise SystemExit("--batch must be a multiple of the GPU count")
    cfg = QWEN2_0_5B
    params = SamplingParams(0.7, 0.9, 1.1)
    m = Model(cfg, local_rank).load(model_path()).kv_alloc(BATCH_CTX, B)
    stream = torch.cuda.ExternalStream(m.stream_handle(), device=dev)
    rng = np.random.default_rng(4000 + rank)
    draws = [mulberry32(0x5EED + rank * B + b) for b in range(B)]
    t0 = time.perf_counter()
    first = []
    for b in range(B):
        m.prefill(b, [int(v) for v in rng.integers(0, cfg.vocab, BATCH_PROMPT)])
        first.append(m.sample_prefill(b, params, float(np.float32(draws[b]()))))
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    steps = min(args.steps, BATCH_CTX - BATCH_PROMPT)
    e2e_steps = min(16, max(steps // 8, 1))
    loop_steps = steps - e2e_steps - args.warmup
    if loop_steps < 1:
        raise SystemExit("--steps too small for config 4")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    plist = [params] * B
    # warm-up: W steps through the public API (graph capture, clocks up)
    toks = first
    for _ in range(args.warmup):
        toks = m.decode_step(toks, plist, [float(np.float32(d())) for d in draws])
    # e2e: the public per-step API, host ids in and out every step
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        toks = m.decode_step(toks, plist, [float(np.float32(d())) for d in draws])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    # value: the device-fed loop over the rest of the context
    randoms = np.array([[np.float32(d()) for d in draws] for _ in range(loop_steps)], np.float32)
    with ClockSampler(local_rank) as clocks:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.decode_loop(toks, plist, randoms, loop_steps, sync=False)
        e1.record(stream)
        m.synchronize()
        barrier()
    loop_ms = max_over_ranks(e0.elapsed_time(e1))
    launches = m.step_launches()
    value = total * loop_steps / (loop_ms / 1e3)
    _, weight_bytes, _ = algorithmic_bytes()
    start = BATCH_PROMPT + args.warmup + e2e_steps
    mean_ctx = start + loop_steps / 2
    kv_bytes = B * cfg.layers * 2 * mean_ctx * cfg.kv_dim * 2
    step_bytes = weight_bytes + kv_bytes
    step_ms = loop_ms / loop_steps
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    achieved = step_bytes / (step_ms / 1e3) / 1e9
    macs = B * (cfg.layers * (cfg.hidden * (cfg.hidden * 2 + 2 * cfg.kv_dim) + 3 * cfg.hidden * cfg.intermediate)
                + cfg.vocab * cfg.hidden)
    out = {
        "metric": BATCH_METRIC,
        "value": round(value, 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": loop_steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int4/int8 weights x f32 activations (exact int8-limb tensor-core block sums, f64 accumulate), f16 KV",
        "data": "synthetic: seeded random-init weights normal(0,0.02); 512 uniform random prompt ids per sequence",
        "config": {"workload": "config 4: batched sampled decode, 256 sequences, prompt 512 -> context 2048, "
                               "T 0.7, top-p 0.9, rp 1.1, per-sequence seeds", "sequences": total,
                   "sequences_per_gpu": B, "parallelism": f"sequences data-parallel x{world}",
                   "positions_timed": [start, start + loop_steps],
                   "l2": "inputs larger than L2: 351 MB of weights and the KV caches per step"},
        "e2e": {"value": round(total * e2e_steps / (e2e_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": B * 28, "d2h_bytes_per_step": B * 4,
                "api": "enx_decode_step with B sequences (ids, positions, sampling rows in; B ids out)"},
        "roofline": {"kernel": "whole batched step (tensor-core projections + f16-KV attention)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": None, "algorithmic_bytes_per_launch": int(step_bytes),
                     "tensor_macs_per_step": macs,
                     "peak_source": "measured MEASURED_PEAKS.json hbm_gbs (burst copy)"},
        "prefill_tok_per_s": round(B * BATCH_PROMPT / prefill_s, 1),
        "gpu_launches": launches * loop_steps,
        "launches_per_step": launches,
        "clocks": clocks.summary(),
    }
    if rank == 0 and emit:
        print(json.dumps(out), flush=True)
    m.close()
    return out


# ---------------------------------------------------------------------------------------------
# config 1: isolated int4 matvec / GEMM sweep (bench.py --workload config1)

SWEEP_SHAPES = [("q/o", 896, 896), ("k/v", 128, 896), ("gate/up", 4864, 896), ("down", 896, 4864)]  # (n, k)
SWEEP_M = [1, 8, 64, 256]
SWEEP_METRIC = "int4 matvec HBM GB/s at M=1 over the projection shapes (q/o, k/v, gate/up, down)"
L2_BYTES = 126 * 2 ** 20


def run_sweep(args, rank, world, local_rank):
    """One launch = enx_matmul_q4 over one projection shape at M tokens: CUDA-core matvec for
    M < 16, the tcgen05 exact-limb GEMM from 16.  Each case cycles through enough copies of its
    weights to exceed twice the L2, so every launch reads its weights from HBM.  N > 1 runs the
    same sweep on every GPU (independent replicas)."""
    import torch
    import torch.distributed as dist

    from enargeia_b200 import build, kernels as K
    from enargeia_b200.format import quantize_tensor
    from enargeia_b200._lib import MatmulQ4Dims, call
    import ctypes as C

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    i8_peak = 2 * bf16  # dense int8 tensor ops/s: twice the measured dense bf16 rate (the nominal ratio)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    shapes = SWEEP_SHAPES
    ms_list = SWEEP_M
    if args.case:
        n_, k_, m_ = (int(v) for v in args.case.split(","))
        shapes, ms_list = [("case", n_, k_)], [m_]
    rng = np.random.default_rng(SEED + 1)
    cases = []
    for name, n, k in shapes:
        t = quantize_tensor(name, rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02), 4)
        wbytes = t.nbytes
        copies = 1 if args.case else max(2, int(np.ceil(2 * L2_BYTES / wbytes)))
        packed = K.to_device_u32(t.packed)
        scales = torch.from_numpy(t.scales).to(dev)
        zeros = K.to_device_u32(t.zeros)
        ws = [(packed.clone(), scales.clone(), zeros.clone()) for _ in range(copies)]
        for m in ms_list:
            x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
            out = torch.empty(m * n, dtype=torch.float32, device=dev)
            d = MatmulQ4Dims(m, n, k, 0, 64, k // 64, n, 0, min(n, 65535), 0, 0, 0)
            s = C.c_void_p(stream.cuda_stream)

            def launch(i, x=x, out=out, d=d, s=s, ws=ws):
                p_, sc_, z_ = ws[i % len(ws)]
                call("enx_matmul_q4", C.c_void_p(x.data_ptr()), C.c_void_p(p_.data_ptr()),
                     C.c_void_p(sc_.data_ptr()), C.c_void_p(z_.data_ptr()), None, C.c_void_p(out.data_ptr()),
                     C.byref(d), s)

            reps = 3 if args.case else max(args.steps, len(ws))
            for i in range(args.warmup):
                launch(i)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if args.case:  # a few eager launches (profiling)
                e0.record(stream)
                for i in range(reps):
                    launch(i)
                e1.record(stream)
            else:  # the launches captured in one CUDA graph: device time, not Python launch time
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    cs = torch.cuda.current_stream()
                    sc = C.c_void_p(cs.cuda_stream)
                    for i in range(reps):
                        launch(i, s=sc)
                g.replay()
                torch.cuda.synchronize()
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = max_over_ranks(e0.elapsed_time(e1)) / reps * 1e3
            if not args.case:
                del g
            # e2e through the C ABI with host buffers: x in from pinned memory, y back, per launch
            xh = x.cpu().pin_memory()
            yh = torch.empty(m * n, dtype=torch.float32).pin_memory()
            e2e_reps = 3 if args.case else min(reps, 50)
            e0.record(stream)
            for i in range(e2e_reps):
                x.copy_(xh, non_blocking=True)
                launch(i)
                yh.copy_(out, non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize()
            e2e_us = max_over_ranks(e0.elapsed_time(e1)) / e2e_reps * 1e3
            io = m * k * 4 + m * n * 4
            gbs = (wbytes + io) / (us / 1e6) / 1e9
            tc = m >= 16
            per_call = count_library_launches(lambda: launch(0))  # one enx_matmul_q4 call, counted
            c = {"shape": name, "n": n, "k": k, "m": m, "path": "tcgen05 limb GEMM" if tc else "CUDA-core matvec",
                 "us": round(us, 3), "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                 "weight_bytes": wbytes, "e2e_us": round(e2e_us, 3), "launches": per_call,
                 "timed_launches": reps * per_call}
            if tc:
                groups = -(-m // 32)
                mma_ops = 2 * (-(-n // 128) * 128) * groups * 192 * k  # issued int8 MMA ops (6 limbs x 32 tokens)
                c["useful_tflops"] = round(2 * m * n * k / (us / 1e6) / 1e12, 2)
                c["int8_mma_tops"] = round(mma_ops / (us / 1e6) / 1e12, 1)
                c["tensor_frac_of_int8_peak"] = round(mma_ops / (us / 1e6) / 1e12 / i8_peak, 4)
            cases.append(c)
            del out, x
        del ws
    m1 = [c for c in cases if c["m"] == 1]
    base = m1 if m1 else cases
    tot_bytes = sum(c["weight_bytes"] + c["m"] * (c["k"] + c["n"]) * 4 for c in base)
    tot_us = sum(c["us"] for c in base)
    tot_e2e = sum(c["e2e_us"] for c in base)
    value = tot_bytes / (tot_us / 1e6) / 1e9
    top = max(base, key=lambda c: c["weight_bytes"])
    out = {
        "metric": SWEEP_METRIC,
        "value": round(value * world, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(tot_us / 1e3, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4 weights x f32 activations (f64 accumulate)",
        "data": "synthetic: seeded int4-quantised normal(0,0.02) weights, activations N(0,1)",
        "config": {"workload": "config 1: int4 matvec/GEMM sweep over the projection shapes, M in {1, 8, 64, 256}",
                   "parallelism": f"replicas x{world}",
                   "l2": "weights cycled over copies totalling > 2x the 126 MB L2 (every launch reads HBM)",
                   "step": "one launch of each projection shape at M=1"},
        "e2e": {"value": round(tot_bytes / (tot_e2e / 1e6) / 1e9 * world, 1), "unit": "GB/s",
                "h2d_bytes_per_step": sum(c["m"] * c["k"] * 4 for c in base),
                "d2h_bytes_per_step": sum(c["m"] * c["n"] * 4 for c in base),
                "api": "enx_matmul_q4 with x copied in from pinned host memory and y copied back per launch"},
        "roofline": {"kernel": f"enx_matmul_q4 M=1 {top['shape']} ({top['n']}x{top['k']})", "bound": "hbm",
                     "achieved": top["hbm_gbs"], "peak": hbm, "unit": "GB/s", "frac": top["hbm_frac"],
                     "traffic": None, "algorithmic_bytes_per_launch": top["weight_bytes"]
                     + top["m"] * (top["k"] + top["n"]) * 4, "launch_us": top["us"],
                     "peak_source": f"{peak_src} MEASURED_PEAKS.json hbm_gbs (burst copy)"},
        "int8_peak_tops": i8_peak,
        "cases": cases,
        "gpu_launches": sum(c["timed_launches"] for c in cases),
    }
    if rank == 0:
        print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------------------------
# config 2: tied int8 LM head + sampling, vocab-sharded across GPUs (bench.py --workload config2)

HEAD_VOCAB, HEAD_HIDDEN, HEAD_HIST = 151936, 896, 2048
HEAD_METRIC = ("LM head + sampling rows/s (int8 151936x896 tied head, T 0.7 / top-p 0.9 / rp 1.1, "
               "2048-id history)")


def head_table():
    from enargeia_b200.format import quantize_tensor

    rng = np.random.default_rng(SEED + 2)
    w = rng.standard_normal((HEAD_VOCAB, HEAD_HIDDEN), dtype=np.float32) * np.float32(0.02)
    return quantize_tensor("model.embed_tokens.weight", w, 8)


def run_head(args, rank, world, local_rank, emit=True):
    """Each rank holds the contiguous row range of the table its shard owns; one step computes the
    logits of B hidden states on every shard and samples B ids.  N = 1: the fused single-GPU
    sampler (one cluster per row); N > 1: the sharded sampler's phases with an NCCL allgather of
    the per-shard candidates / sums / top-p bucket masses / kept masses / picks between them.
    Total work is fixed as N grows (strong scaling)."""
    import torch
    import torch.distributed as dist

    from enargeia_b200 import build, kernels as K
    from enargeia_b200.vocab_shard import PeerGather, ShardedHead, ShardedSampler, ShardInputs, run_distributed, \
        sampling_rows_tensor

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    table = head_table()
    head = ShardedHead(table, HEAD_VOCAB, rank, world, dev)
    shard_bytes = head.packed.numel() * 4 + head.scales.numel() * 4 + head.zeros.numel() * 4
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    def one_batch(B, steps, warmup, clocks=None):
        rng = np.random.default_rng(7000 + B)  # same inputs on every rank
        total = steps + warmup
        xs_host = torch.from_numpy(rng.standard_normal((total, B, HEAD_HIDDEN)).astype(np.float32)).pin_memory()
        xs = xs_host.to(dev)
        history = torch.from_numpy(rng.integers(0, HEAD_VOCAB, (B, HEAD_HIST)).astype(np.int32)).to(dev)
        hlen = torch.full((B,), HEAD_HIST, dtype=torch.int32, device=dev)
        params = [[(0.7, 0.9, 1.1, float(np.float32(v))) for v in rng.random(B)] for _ in range(total)]
        params_dev = [sampling_rows_tensor(p, dev) for p in params]
        logits = torch.empty((B, head.n), dtype=torch.float32, device=dev)
        out = torch.empty(B, dtype=torch.int32, device=dev)
        sampler = ShardedSampler(HEAD_VOCAB, rank, world, B, dev) if world > 1 else None
        # the phase exchange: peer-memory stores over NVLink or NCCL all-gathers.  "auto" takes the
        # measured faster one: peer stores at a few rows (1 row on 2 GPUs: 0.22 vs 0.34 ms per
        # step), NCCL at 64 rows (0.74 vs 0.77 ms, where the phase kernels dominate)
        gather = None
        mode = os.environ.get("ENX_SHARD_EXCHANGE", "auto")
        if sampler is not None and (mode == "peer" or (mode == "auto" and B <= 16)):
            gather = PeerGather(sampler.max_record_bytes())
        graph = None
        if sampler is None:
            # one GPU: the head and the fused sampler replayed as one CUDA graph over static input
            # buffers (the sharded step's NCCL exchanges stay eager)
            gx = torch.zeros((B, HEAD_HIDDEN), dtype=torch.float32, device=dev)
            gp = params_dev[0].clone()
            head.logits(gx, logits)
            K.sample_batched(logits, history, hlen, gp, out)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                head.logits(gx, logits)
                K.sample_batched(logits, history, hlen, gp, out)

        def step(i, x, prow_dev):
            if graph is not None:
                gx.copy_(x, non_blocking=True)
                gp.copy_(prow_dev, non_blocking=True)
                graph.replay()
                return out
            head.logits(x, logits)
            return run_distributed(sampler, ShardInputs(logits, history, hlen, params[i]), gather, params_dev=prow_dev)

        for i in range(warmup):
            step(i, xs[i], params_dev[i])
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(warmup, total):
            step(i, xs[i], params_dev[i])
        e1.record(stream)
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / steps
        # e2e: hidden states and sampling rows copied in from pinned host memory, ids read back,
        # every step
        prow_host = [torch.frombuffer(bytearray(p.cpu().numpy().tobytes()), dtype=torch.uint8).pin_memory()
                     for p in params_dev]
        xbuf = torch.empty((B, HEAD_HIDDEN), dtype=torch.float32, device=dev)
        pbuf = torch.empty_like(params_dev[0])
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(warmup, total):
            xbuf.copy_(xs_host[i], non_blocking=True)
            pbuf.copy_(prow_host[i], non_blocking=True)
            ids = step(i, xbuf, pbuf).cpu()
        e1.record(stream)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / steps
        # the head GEMM/matvec alone: R launches back to back on this rank's shard
        reps = 20
        head.logits(xs[0], logits)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            head.logits(xs[0], logits)
        e1.record(stream)
        torch.cuda.synchronize()
        head_us = e0.elapsed_time(e1) / reps * 1e3
        if gather is not None:
            gather.check()
            barrier()
            gather.close()
        head_bytes = shard_bytes + B * HEAD_HIDDEN * 4 + B * head.n * 4
        achieved = head_bytes / (head_us / 1e6) / 1e9
        head_launches = 2 if B >= 16 else 1
        launches = head_launches + (1 if sampler is None else 9)
        del ids
        return {"rows": B, "value": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
                "e2e": {"value": round(B / (e2e_ms / 1e3), 1), "unit": "rows/s",
                        "h2d_bytes_per_step": B * HEAD_HIDDEN * 4 + B * 16, "d2h_bytes_per_step": B * 4,
                        "api": "enx_lm_head_q8 + enx_sample_batched (one CUDA graph) / enx_shard_* phases + NCCL"},
                "head_roofline": {"kernel": "enx_lm_head_q8 over this rank's rows"
                                            + (" (tcgen05 limb GEMM)" if B >= 16 else " (CUDA-core matvec)"),
                                  "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                                  "frac": round(achieved / hbm, 4), "traffic": None,
                                  "algorithmic_bytes_per_launch": int(head_bytes), "launch_us": round(head_us, 2),
                                  "peak_source": f"{peak_src} MEASURED_PEAKS.json hbm_gbs (burst copy)"},
                "sampler_ms_per_step": round(ms - head_us / 1e3, 4),
                "exchange": None if sampler is None else ("peer stores over NVLink (enx_peer_allgather)"
                                                          if gather is not None else "NCCL all_gather_into_tensor"),
                "gpu_launches": launches * steps, "launches_per_step": launches}

    steps = min(args.steps, 200)
    small = one_batch(1, steps, args.warmup)
    with ClockSampler(local_rank) as clocks:
        big = one_batch(args.batch if args.batch != 256 else 64, steps, args.warmup)
    out = {
        "metric": HEAD_METRIC,
        "value": big["value"],
        "unit": "rows/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": big["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 table x f32 hidden (exact block sums, f64 accumulate), f64 sampling",
        "data": "synthetic: seeded int8-quantised normal(0,0.02) table, hidden N(0,1), 2048 uniform random history ids",
        "config": {"workload": f"config 2: tied int8 LM head + sampling, batch {big['rows']} (batch 1 below), "
                               f"vocab {HEAD_VOCAB} x hidden {HEAD_HIDDEN}", "rows": big["rows"],
                   "parallelism": f"vocab-sharded x{world}" if world > 1 else "one GPU",
                   "rows_per_gpu": head.n, "l2": "inputs larger than L2: 137 MB table per step at N=1"},
        "e2e": big["e2e"],
        "roofline": big["head_roofline"],
        "sampler_ms_per_step": big["sampler_ms_per_step"],
        "gpu_launches": big["gpu_launches"],
        "launches_per_step": big["launches_per_step"],
        "batch_1": small,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = head_cpu_baseline(table, budget_s=args.cpu_budget)
    if rank == 0 and emit:
        print(json.dumps(out), flush=True)
    return out


def head_cpu_baseline(table, budget_s=15.0):
    from oracle import oracle as O

    O.build()
    cores = O.max_threads()
    rng = np.random.default_rng(99)
    hist = rng.integers(0, HEAD_VOCAB, HEAD_HIST).astype(np.uint32)
    n = 0
    t0 = time.perf_counter()
    while n < 2 or time.perf_counter() - t0 < budget_s:
        x = rng.standard_normal(HEAD_HIDDEN).astype(np.float32)
        logits = O.linear_q(table, x)
        O.sample(logits, hist, 0.7, 0.9, 1.1, float(np.float32(rng.random())))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"{n} rows: oracle int8 head (f64 accumulate, OpenMP over vocab rows) + oracle sampler, "
                      f"{dt:.1f} s"}


# ---------------------------------------------------------------------------------------------
# CPU legs (the oracle: a restatement of the reference's CPU path; the reference itself is
# TypeScript and cannot run on this box)


def kernel_shares(m, stream, step_us):
    """The reference's telemetry share table (src/runtime/telemetry.ts:12-20) for one decode step:
    the traced stages of the layer kernel, plus CUDA-event times of the head kernel and the
    sampler run alone on the model's own tensors (20 launches each)."""
    import torch
    from enargeia_b200 import kernels as K
    from enargeia_b200._lib import EmbeddingDims, call
    from enargeia_b200.session import GREEDY
    from enargeia_b200.telemetry import step_shares

    m.set_tracing(True)
    tok = m.decode_step([7], [GREEDY], [0.5])[0]
    stage = m.stage_times()
    m.set_tracing(False)
    cfg = m.config
    hv = m.tensor_view("model.embed_tokens.weight")
    x = torch.from_numpy(m.hidden(0)).cuda()
    logits = torch.zeros(cfg.vocab, dtype=torch.float32, device="cuda")
    d = EmbeddingDims(1, cfg.hidden, 0, cfg.vocab, 64, cfg.hidden // 64, cfg.vocab, 0, min(cfg.vocab, 65535), 0, 0, 0)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    hist = torch.zeros(64, dtype=torch.int32, device="cuda")

    def timed(fn, reps=20):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps * 1e3

    import ctypes as C
    head_us = timed(lambda: call("enx_lm_head_q8", x.data_ptr(), hv["packed"], hv["scales"], hv["zeros"],
                                 logits.data_ptr(), C.byref(d), None))
    sample_us = timed(lambda: K.sample(logits, hist, out, 0.0, 1.0, 1.0, 0.5))
    return step_shares(stage, head_us, sample_us, step_us)


def cpu_baseline(f, prompt, budget_s=15.0, threads=None):
    from oracle import oracle as O

    O.build()
    if threads:
        O.set_threads(threads)
    cores = O.max_threads()
    om = O.OracleModel(f, QWEN2_0_5B, PROMPT + GEN + 1)
    logits = om.prefill(prompt)
    tok = O.argmax(logits)
    n = 0
    t0 = time.perf_counter()
    while n < GEN - 1 and (n < 2 or time.perf_counter() - t0 < budget_s):
        logits = om.decode(tok)
        tok = O.argmax(logits)
        n += 1
    dt = time.perf_counter() - t0
    # the same decode continued on one host thread (the reference's JS path is single-threaded)
    O.set_threads(1)
    n1 = 0
    t1 = time.perf_counter()
    while n1 < 2 or (n1 < GEN - 1 - n and time.perf_counter() - t1 < budget_s / 2):
        logits = om.decode(tok)
        tok = O.argmax(logits)
        n1 += 1
    dt1 = time.perf_counter() - t1
    O.set_threads(cores)
    return {"value": round(n / dt, 4), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy decode steps of config 0 after a 32-id prefill (oracle/enx_oracle.cpp, "
                      f"f64 accumulate, OpenMP over output rows), {dt:.1f} s",
            "single_thread": {"value": round(n1 / dt1, 4), "unit": "tok/s", "cores": 1,
                              "sample": f"{n1} further decode steps on one host thread, {dt1:.1f} s"}}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O

    O.build()
    build_model_file(QWEN2_0_5B, SEED, model_path())
    from enargeia_b200.format import read_enargeia

    f = read_enargeia(model_path())
    cores = O.max_threads()
    prompt = [int(v) for v in np.random.default_rng(1000).integers(0, QWEN2_0_5B.vocab, PROMPT)]
    om = O.OracleModel(f, QWEN2_0_5B, PROMPT + GEN + 1)

    def restart():
        om.reset()
        return O.argmax(om.prefill(prompt))

    tok = restart()
    for _ in range(args.warmup):
        tok = O.argmax(om.decode(tok))
    total = 0.0
    done = 0
    while done < args.steps:
        n = min(GEN - 1, args.steps - done)
        tok = restart()
        t0 = time.perf_counter()
        for _ in range(n):
            tok = O.argmax(om.decode(tok))
        total += time.perf_counter() - t0
        done += n
    value = args.steps / total
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 accumulate / f32 store",
        "data": "synthetic: same seeded random-init model and prompt as the enx arm",
        "config": {"workload": "config 0: greedy batch-1 decode (CPU restatement of the reference path)"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} decode steps, host threads {cores}; the reference's own path is "
                                   "TypeScript/WebGPU (no node, browser or graphics stack on this box)"},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2016)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["enx", "reference"], default="enx")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-blocks", action="store_true",
                    help="config0: skip the dp_batched (config 4) and vocab_sharded (config 2) blocks")
    ap.add_argument("--workload", choices=["config0", "config1", "config2", "config3", "config4"], default="config0",
                    help="config0: greedy batch-1 decode (the headline); config1: int4 matvec/GEMM sweep; "
                         "config2: vocab-sharded LM head + sampling; config3: chunked prefill; "
                         "config4: batched sampled decode")
    ap.add_argument("--case", default="", help="config1: one case n,k,m with 3 timed launches (profiling)")
    ap.add_argument("--batch", type=int, default=256,
                    help="config4: total sequences over all GPUs; config2: rows per step (default 64)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.steps > 256:
            args.steps = 64  # the CPU leg times a bounded sample (about 0.3-1 s per step)
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        # the communicator's start-up banner goes to stderr: stdout carries the one JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    try:
        if args.workload == "config1":
            if args.steps == 2016:
                args.steps = 200
            run_sweep(args, rank, world, local_rank)
        elif args.workload == "config3":
            run_prefill(args, rank, world, local_rank)
        elif args.workload == "config2":
            run_head(args, rank, world, local_rank)
        elif args.workload == "config4":
            if args.steps == 2016:
                args.steps = BATCH_CTX - BATCH_PROMPT
            run_batched(args, rank, world, local_rank)
        else:
            run_enx(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
