"""Gemma-2B Q8_0 token-loop benchmark on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: random-init Gemma-2B, Q8_0 weights,
batch-1 greedy decode after a 16-token seeded prompt. A step is one decode
token: embed -> 18 layers -> logits -> on-device argmax feeding the next step.
Every rank decodes its own sequence on its own GPU (independent replicas, no
collective on the data path; weak scaling), and `value` is the whole-job
tok/s: the tokens all ranks decoded over the max-over-ranks device time.

The `prefill` object is configs[4]: eight 2048-token seeded prompts (seed 4)
prefilled one after another, device-timed, against the tensor-core roofline.
The `long_context` object is configs[2]: an 8,064-token seeded prompt, then
the 128 decode steps to an 8,192-position window, device-timed. The metric's
second half, b=64/GPU, is the `batched` object of the same line: each rank decodes 64 independent sequences (512-token seeded
prompts, seed 3) with batched greedy steps on the tensor cores; its value is
the whole-job tok/s over the max-over-ranks device time of `--batched-steps`
steps (256 by default, the config's length).

`value` is device-timed (CUDA events on the engine's stream around K decode
steps, weights resident in HBM). `e2e` is the same metric through the public
generate call (HF::Gemma::generate's C-ABI, hf_cuda_generate_greedy) with the
prompt in pinned host memory and every generated token read back to the host.
`roofline` reports the dominant kernel of the step against the measured HBM
copy bandwidth; `cpu_baseline` the fp32 oracle port on this host's cores.
With --impl reference the same metric is timed on the reference's arithmetic
restated for the CPU (the reference has no runnable GPU path here: its eacp
kernels target Metal/D3D12 only).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import numpy as np  # noqa: E402

METRIC = "Gemma-2B Q8_0 decode tok/s (b=1, b=64/GPU) and achieved HBM GB/s vs peak"
WORKLOAD = "config0: Gemma-2B Q8_0 batch-1 greedy decode, BOS + 15 seeded prompt ids (seed 0)"
PUBLISHED_TOK_S = 161.6  # the reference's published int8-blocks decode, 16 tokens (Apple M4 Max, Metal; plan.md:1083)
PROMPT_LENGTH = 16
SEED = 0
BATCH_SEQUENCES = 64      # configs[3]: sequences per GPU
BATCH_PROMPT = 512        # configs[3]: prompt tokens per sequence
BATCH_SEED = 3
BATCH_WORKLOAD = "config3: 64 independent sequences per GPU, 512-token seeded prompts (seed 3), greedy steps"
LONG_PROMPT = 8064        # configs[2]: prompt tokens, then decode to an 8,192-position window
LONG_SEED = 2
LONG_WORKLOAD = "config2: Gemma-2B batch-1 prefill of 8064 seeded ids (seed 2), greedy decode to 8192 positions"
PREFILL_STEP_ROWS = 2048  # prefill rows per step (long prompts: 354 ms at 2048 against 368.5 at 512)
PREFILL_SEQUENCES = 8     # configs[4]: 8 x 2048-token prompts
PREFILL_PROMPT = 2048
PREFILL_SEED = 4
PREFILL_WORKLOAD = ("config4: Gemma-2B prefill of 8 independent 2048-token seeded prompts (seed 4), one after another "
                    "through one context on the tcgen05 products")


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def prefill_flops(shape, prompt: int) -> float:
    """Algorithmic FLOPs of one prompt's prefill: 2 per multiply-add of every
    linear weight for every row, causal attention (q.k and p.v over the
    prefix), and the last row's logits (only the last row is sampled)."""
    q, kv = shape.heads * shape.head_width, shape.kv_heads * shape.head_width
    linear = shape.width * (q + 2 * kv) + q * shape.width + 3 * shape.width * shape.intermediate
    attention = 2 * 2 * shape.heads * shape.head_width * prompt * (prompt + 1) / 2
    return shape.layers * (2.0 * prompt * linear + attention) + 2.0 * shape.width * shape.vocab


def measured_tensor_peak():
    """The bf16 tensor peak for a region of hundreds of milliseconds: the
    measured sustained figure (a long cuBLAS loop under the power cap)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        if "bf16_tflops_sustained" in peaks:
            return float(peaks["bf16_tflops_sustained"]), "measured (cuBLAS bf16, sustained)"
        return float(peaks["bf16_tflops"]), "measured (cuBLAS bf16, burst)"
    return 1400.0, "fallback (sustained)"


def prefill_roofline(flops_per_gpu: float, ms: float, peak: float, peak_kind: str) -> dict:
    """Tensor roofline of one GPU's prefill: its own algorithmic FLOPs over the
    max-over-ranks time, against one GPU's peak (every rank does the same work)."""
    achieved = flops_per_gpu / (ms * 1e9)
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_kind": peak_kind, "algorithmic_flops_per_gpu": flops_per_gpu}


def committed_traffic():
    """DRAM bytes per algorithmic byte of the dominant kernel, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.lines = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, sm_max, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = max(sm_max, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": sm_max or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_index(local_rank: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        entries = [v.strip() for v in visible.split(",") if v.strip()]
        if local_rank < len(entries) and entries[local_rank].isdigit():
            return int(entries[local_rank])
    return local_rank


def build_model(native, shape, keep: bool, sequences: int = 1, pages: int | None = None):
    ctx = native.Context(shape, device=int(os.environ.get("LOCAL_RANK", "0")), sequences=sequences, pages=pages)
    tensors = ctx.load_synthetic(seed=SEED, keep=keep)
    return ctx, tensors


def cpu_decode_rate(shape, tensors, prompt, steps: int, warmup: int = 1):
    """fp32 oracle (the reference's arithmetic, 16-lane fp32 sums) on every host core."""
    import oracle_bindings as ob

    model = ob.OracleModel(shape.replace(max_positions=PROMPT_LENGTH + warmup + steps + 2), tensors, "float")
    _, logits = model.step(prompt, last_row_only=True, want_hidden=False)
    token = ob.argmax(logits[-1])
    for _ in range(warmup):
        _, logits = model.step([token], want_hidden=False)
        token = ob.argmax(logits[-1])
    start = time.perf_counter()
    for _ in range(steps):
        _, logits = model.step([token], want_hidden=False)
        token = ob.argmax(logits[-1])
    elapsed = time.perf_counter() - start
    threads = model.threads
    model.close()
    return steps / elapsed, threads, elapsed


def max_over_ranks(dist, values, device="cuda"):
    """The element-wise maximum of `values` over all ranks (every rank gets it):
    a multi-GPU time is the slowest rank's. Every rank must call it at the same
    point; `dist` None (one process) returns the values unchanged."""
    if not dist:
        return [float(v) for v in values]
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


CONFIG1_SHAPES = [(2048, 2048), (2048, 256), (2048, 16384), (16384, 2048), (2048, 256000)]  # configs[1] (K -> N)
CONFIG1_ROWS = (1, 8, 64)


def run_config1(native, peak, peak_kind, reps=10):
    """the Q8_0 op sweep (W[N,K] ~ N(0, 0.02) quantized, x[M,K] ~
    N(0, 1), seed 1) through prepared weights (hf_cuda_linear_*), so each row
    count runs the kernel the decoder runs for it. Every launch is timed alone
    with CUDA events on its stream after a write of 256 MiB (twice the L2),
    so the weight comes from HBM. Algorithmic bytes = 17/16 N K + 4 M K + 4 M N."""
    import torch

    stream = torch.cuda.current_stream()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    x = torch.from_numpy(native.synthetic_normal(1, 200, 64, 64 * 16384, 1.0)).cuda()
    cases = []
    for K, N in CONFIG1_SHAPES:
        q = native.quantize(native.synthetic_normal(1, 100 + N % 97, K, N * K, 0.02))
        out = torch.empty(64 * N, dtype=torch.float32, device="cuda")
        with native.Linear(q, K, N, max(CONFIG1_ROWS)) as lin:
            for M in CONFIG1_ROWS:
                times = []
                for rep in range(reps + 2):
                    flush.zero_()
                    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    start.record(stream)
                    lin.run(x.data_ptr(), out.data_ptr(), M, stream=stream.cuda_stream)
                    stop.record(stream)
                    stop.synchronize()
                    if rep >= 2:
                        times.append(start.elapsed_time(stop) * 1000.0)
                us = statistics.mean(times)
                nbytes = 17 * N * K // 16 + 4 * M * K + 4 * M * N
                gbs = nbytes / us / 1e3
                cases.append({"K": K, "N": N, "M": M, "kernel": native.LINEAR_PATH_NAMES[lin.path(M)],
                              "us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3),
                              "tflops": round(2.0 * M * N * K / us / 1e6, 2)})
        del out
    return {"workload": "config1: Q8_0 op sweep, seed 1, through prepared weights (hf_cuda_linear_run)",
            "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "bound": "hbm",
            "l2": "256 MiB written before every timed launch", "reps": reps, "cases": cases}


def run_reference(args):
    """--impl reference: the reference's arithmetic on the host cores, same metric and workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle_bindings as ob
    from huggingfaceeacp_b200.native import GEMMA_2B  # a shape description; loads no library

    # The model and prompt come from oracle.c's restatement of the seeded
    # generator and quantizer (pinned bit for bit to the product's host
    # library by tests/test_oracle_generator.py): this arm loads none of the
    # product's libraries.
    shape = GEMMA_2B
    tensors = ob.synthetic_model(shape, SEED)
    prompt = ob.synthetic_tokens(SEED, PROMPT_LENGTH, shape.vocab)
    rate, threads, elapsed = cpu_decode_rate(shape, tensors, prompt, args.steps, args.warmup)
    sample = f"{args.steps} fp32 decode steps after a {PROMPT_LENGTH}-token prefill and {args.warmup} warm-up steps"
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": rate / PUBLISHED_TOK_S, "dtype": "f32",
        "data": "synthetic: random-init Gemma-2B, N(0,0.02) weights quantized to Q8_0, seeded prompt",
        "config": {"workload": WORKLOAD, "batch_per_gpu": 1, "parallelism": "host cores",
                   "implementation": "oracle/oracle.c fp32 restatement of the reference's kernels"},
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    from huggingfaceeacp_b200 import native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL writes its log (its version banner included, at NCCL_DEBUG=WARN or
        # VERSION) to stdout unless told otherwise; stdout carries the one JSON line.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist:
            dist.barrier()

    # One context of 64 sequences: sequence 0 runs the batch-1 decode, all 64
    # the batched steps (the weights are uploaded once).
    window = max(LONG_PROMPT + 128, BATCH_PROMPT + args.batched_steps + args.warmup,
                 PROMPT_LENGTH + 2 * (args.warmup + args.steps) + 8)
    shape = native.GEMMA_2B.replace(max_step_rows=PREFILL_STEP_ROWS, max_positions=window)
    keep = rank == 0 and world == 1 and not args.no_cpu_baseline
    # The batched sequences' K/V live in pages: enough for each sequence's
    # prompt and every step it takes here (not its whole window).
    batch_positions = BATCH_PROMPT + args.warmup + args.batched_steps + 1
    pages = BATCH_SEQUENCES * -(-batch_positions // native.PAGE_ROWS)
    ctx, tensors = build_model(native, shape, keep, BATCH_SEQUENCES, pages)
    # Every rank decodes its own sequences: rank r's batch-1 prompt has seed
    # SEED + r (rank 0 is config 0's), its batched sequence q is global sequence
    # r * 64 + q (seed BATCH_SEED + r * 64 + q), its long prompt seed LONG_SEED + r,
    # its prefill prompt q seed PREFILL_SEED + r * 8 + q.
    prompt = native.synthetic_tokens(SEED + rank, PROMPT_LENGTH, shape.vocab)

    # ---- device-timed decode: K steps with the weights resident
    ctx.prefill_async(prompt)
    ctx.decode_async(args.warmup)
    ctx.sync()
    stream = torch.cuda.ExternalStream(ctx.stream)
    launches = ctx.decode_launches(args.steps)
    path = ctx.decode_path
    first_pos = ctx.position
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(physical_index(local_rank)) as clocks:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        ctx.decode_async(args.steps)
        stop.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    barrier()
    (elapsed_ms,) = max_over_ranks(dist, [elapsed_ms])
    tokens = ctx.read_slots(first_pos + 1, args.steps)
    ms_per_step = elapsed_ms / args.steps
    value = world * args.steps / (elapsed_ms / 1000.0)
    keys = first_pos + args.steps // 2
    step_bytes = native.decode_bytes(shape, keys)
    peak, peak_kind = measured_peaks()

    # ---- e2e: the public generate call, host prompt in, host tokens out
    pinned_prompt = torch.from_numpy(prompt).pin_memory().numpy()
    barrier()
    e2e_start = time.perf_counter()
    generated = ctx.generate(pinned_prompt, args.steps)
    e2e_s = time.perf_counter() - e2e_start
    (e2e_s,) = max_over_ranks(dist, [e2e_s])
    e2e = {"value": world * len(generated) / e2e_s, "unit": "tok/s",
           "h2d_bytes_per_step": 4.0 * PROMPT_LENGTH / max(1, len(generated)), "d2h_bytes_per_step": 4,
           "call": "hf_cuda_generate_greedy (prefill + decode, wall clock)"}

    # ---- batched decode: 64 sequences, device-timed batched steps
    prompts = np.stack([native.synthetic_tokens(BATCH_SEED + rank * BATCH_SEQUENCES + q, BATCH_PROMPT, shape.vocab)
                        for q in range(BATCH_SEQUENCES)])
    barrier()
    torch.cuda.synchronize()
    p_start, p_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record(stream)
    ctx.prefill_batch_async(prompts)
    p_stop.record(stream)
    ctx.decode_batch_async(args.warmup)
    ctx.sync()
    batch_first = ctx.sequence_position(0)  # every batched sequence is at the same position here
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(physical_index(local_rank)) as batch_clocks:
        b_start, b_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b_start.record(stream)
        ctx.decode_batch_async(args.batched_steps)
        b_stop.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
    batch_ms = b_start.elapsed_time(b_stop)
    prefill_ms = p_start.elapsed_time(p_stop)
    barrier()
    batch_ms, prefill_ms = max_over_ranks(dist, [batch_ms, prefill_ms])
    batch_tokens = ctx.read_batch_slots(batch_first + 1, min(4, args.batched_steps))
    batch_step_ms = batch_ms / args.batched_steps
    batch_keys = batch_first + args.batched_steps // 2
    batch_step_bytes = native.batched_decode_bytes(shape, BATCH_SEQUENCES, batch_keys)
    batch_gbs = batch_step_bytes / (batch_step_ms * 1e6)
    batched = {
        "workload": BATCH_WORKLOAD, "value": world * BATCH_SEQUENCES * args.batched_steps / (batch_ms / 1000.0),
        "unit": "tok/s", "n_gpus": world, "sequences_per_gpu": BATCH_SEQUENCES, "steps": args.batched_steps,
        "warmup": args.warmup, "ms_per_step": batch_step_ms, "scaling": "weak",
        "prefill_tok_s": world * BATCH_SEQUENCES * BATCH_PROMPT / (prefill_ms / 1000.0),
        "roofline": {"bound": "hbm", "achieved": batch_gbs, "peak": peak, "unit": "GB/s", "frac": batch_gbs / peak,
                     "peak_kind": peak_kind, "algorithmic_bytes_per_step": batch_step_bytes,
                     "note": "weights once per step + every sequence's K/V rows and logits"},
        "clocks": batch_clocks.summary(),
        "tokens_head": [[int(t) for t in row] for row in batch_tokens[:2]],
        "kv_cache": f"paged: {pages} pages of {native.PAGE_ROWS} positions shared by the {BATCH_SEQUENCES} sequences",
    }

    # ---- long context: prefill 8064 tokens, decode 128 steps to 8192
    long_prompt = native.synthetic_tokens(LONG_SEED + rank, LONG_PROMPT, shape.vocab)
    ctx.begin_sequence()
    barrier()
    torch.cuda.synchronize()
    l_start, l_mid, l_stop = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    l_start.record(stream)
    ctx.prefill_async(long_prompt)
    l_mid.record(stream)
    ctx.decode_async(127)
    l_stop.record(stream)
    ctx.sync()
    long_prefill_ms, long_decode_ms = l_start.elapsed_time(l_mid), l_mid.elapsed_time(l_stop)
    barrier()
    long_prefill_ms, long_decode_ms = max_over_ranks(dist, [long_prefill_ms, long_decode_ms])
    long_bytes = sum(native.decode_bytes(shape, LONG_PROMPT + i + 1) for i in range(1, 128))
    long_gbs = long_bytes / (long_decode_ms * 1e6)
    long_context = {
        "workload": LONG_WORKLOAD, "value": world * 127 / (long_decode_ms / 1000.0), "unit": "tok/s",
        "n_gpus": world, "steps": 127, "ms_per_step": long_decode_ms / 127,
        "prefill_tok_s": world * LONG_PROMPT / (long_prefill_ms / 1000.0),
        "roofline": {"bound": "hbm", "achieved": long_gbs, "peak": peak, "unit": "GB/s", "frac": long_gbs / peak,
                     "peak_kind": peak_kind, "note": "weights + the step's K/V reads at 8065..8191 keys"},
    }

    # ---- prefill throughput: 8 x 2048-token prompts, device-timed
    prefill_prompts = [native.synthetic_tokens(PREFILL_SEED + rank * PREFILL_SEQUENCES + q, PREFILL_PROMPT, shape.vocab)
                       for q in range(PREFILL_SEQUENCES)]
    barrier()
    torch.cuda.synchronize()
    f_start, f_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f_start.record(stream)
    for prompt_q in prefill_prompts:
        ctx.begin_sequence()
        ctx.prefill_async(prompt_q)
    f_stop.record(stream)
    ctx.sync()
    prefill_run_ms = f_start.elapsed_time(f_stop)
    barrier()
    (prefill_run_ms,) = max_over_ranks(dist, [prefill_run_ms])
    tensor_peak, tensor_peak_kind = measured_tensor_peak()
    flops = PREFILL_SEQUENCES * prefill_flops(shape, PREFILL_PROMPT)
    prefill_rl = prefill_roofline(flops, prefill_run_ms, tensor_peak, tensor_peak_kind)
    prefill_rl["note"] = ("per GPU: 2 FLOPs per weight multiply-add of every row, causal attention, last-row logits; "
                          "each Q8_0 product runs as three exact f16 tensor-core products")
    prefill = {
        "workload": PREFILL_WORKLOAD, "value": world * PREFILL_SEQUENCES * PREFILL_PROMPT / (prefill_run_ms / 1000.0),
        "unit": "tok/s", "n_gpus": world, "ms": prefill_run_ms, "scaling": "weak", "roofline": prefill_rl,
    }

    # ---- config 1: the op sweep (rank 0 only; a per-GPU kernel measurement)
    config1 = run_config1(native, peak, peak_kind) if rank == 0 and not args.no_config1 else None

    # ---- roofline of every decode kernel, live (cycling layers: HBM, not L2)
    ctx.begin_sequence()
    ctx.prefill_async(prompt)
    ctx.decode_async(keys - PROMPT_LENGTH)
    ctx.sync()
    kernels = {}
    for kernel, name in enumerate(native.KERNEL_NAMES):
        us, nbytes = ctx.time_kernel(kernel, 36 if kernel != native.KERNEL_LOGITS else 8)
        kernels[name] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3}
    graph_kernels = {n: {"us": round(k["us"], 2), "gbs": round(k["gbs"], 1)} for n, k in kernels.items()}
    if path == native.DECODE_PERSISTENT:
        # One cooperative launch runs all K steps: the dominant (only) kernel.
        dominant = "decode_persistent"
        launch_bytes = step_bytes * args.steps
        launch_us = elapsed_ms * 1000.0
        achieved = launch_bytes / launch_us / 1e3
    else:
        per_step_us = {
            name: k["us"] * (1 if name == "logits_argmax" else shape.layers) for name, k in kernels.items()}
        dominant = max(per_step_us, key=per_step_us.get)
        launch_bytes, launch_us = kernels[dominant]["bytes"], kernels[dominant]["us"]
        achieved = kernels[dominant]["gbs"]
    # DRAM bytes per launch: the ncu capture's traffic per algorithmic byte
    # (profiles/traffic.json) times this launch's algorithmic bytes.
    ratio = committed_traffic().get(dominant, {}).get("dram_bytes_per_algorithmic_byte")
    traffic = ratio * launch_bytes if ratio else None
    roofline = {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": launch_bytes, "mean_launch_us": launch_us,
                "graph_path_kernels": graph_kernels}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "f32",
        "data": "synthetic: random-init Gemma-2B, N(0,0.02) weights quantized to Q8_0, seeded prompt",
        "config": {"workload": WORKLOAD, "batch_per_gpu": 1, "seq_len": first_pos + args.steps,
                   "parallelism": f"replicas{world}", "l2": "inputs larger than L2 (2.66 GB of weights per step)",
                   "step_bytes": step_bytes,
                   "sequences": "rank r: batch-1 prompt seed 0 + r; batched sequence q is global r*64 + q (seed 3 + "
                                "r*64 + q); long prompt seed 2 + r; prefill prompt q seed 4 + r*8 + q"},
        "step_roofline": {"achieved": step_bytes / (ms_per_step * 1e6), "peak": peak, "unit": "GB/s",
                          "frac": step_bytes / (ms_per_step * 1e6) / peak},
        "roofline": roofline,
        "e2e": e2e,
        "batched": batched,
        "long_context": long_context,
        "prefill": prefill,
        "config1": config1,
        "gpu_launches": launches,
        "decode_path": {0: "generic", 1: "graph", 2: "persistent"}[path],
        "clocks": clocks.summary(),
        "tokens_head": [int(t) for t in tokens[:4]],
    }

    if rank == 0 and keep:
        rate, threads, elapsed = cpu_decode_rate(shape, tensors, prompt, args.cpu_steps)
        line["cpu_baseline"] = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{args.cpu_steps} fp32 decode steps of the same model and prompt"
                                          f" ({elapsed:.1f} s)"}
    elif rank == 0:
        line["cpu_baseline"] = None
    ctx.close()
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_tp_prefill(args):
    """Tensor-parallel prefill (configs[4]'s tensor-parallel variant) of
    configs[2]'s single 8,064-token prompt: `--gpus N` ranks, one context per
    GPU holding the whole model, the feed-forward split over the ranks with one
    NCCL allreduce per layer (hf_cuda_set_tensor_parallel); N = 1 is the
    one-GPU prefill. Device-timed over `--steps` prefills after `--warmup`,
    max over ranks. Not the bench line: one JSON object {"tp_prefill": ...}."""
    import datetime

    import torch

    from huggingfaceeacp_b200 import native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    shape = native.GEMMA_2B.replace(max_step_rows=args.tp_rows, max_positions=LONG_PROMPT + 128)
    with native.Context(shape, device=local_rank) as ctx:
        ctx.load_synthetic(seed=SEED)
        if dist:
            nccl_id = native.broadcast_bytes(dist, native.nccl_unique_id() if rank == 0 else None,
                                             native.NCCL_ID_BYTES, device="cuda")
            ctx.set_tensor_parallel(rank, world, nccl_id)
        prompt = native.synthetic_tokens(LONG_SEED, LONG_PROMPT, shape.vocab)
        stream = torch.cuda.ExternalStream(ctx.stream)
        for _ in range(args.warmup):
            ctx.prefill_async(prompt)
        ctx.sync()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            ctx.prefill_async(prompt)
        stop.record(stream)
        ctx.sync()
        ms = start.elapsed_time(stop) / args.steps
        first = int(ctx.read_slots(LONG_PROMPT, 1)[0])
        (ms,) = max_over_ranks(dist, [ms])
        firsts = [first]
        if dist:
            gathered = [None] * world
            dist.all_gather_object(gathered, first)
            firsts = gathered
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"tp_prefill": {
            "workload": "config2's prompt: one 8064-token seeded prompt (seed 2), Gemma-2B, prefill only",
            "n_gpus": world, "step_rows": args.tp_rows, "ms": ms, "tok_s": LONG_PROMPT / (ms / 1000.0),
            "first_token_per_rank": firsts, "steps": args.steps, "warmup": args.warmup,
            "parallelism": f"tensor-parallel feed-forward x{world}, q/k/v, attention and o_proj on every rank"
                           if world > 1 else "one GPU"}}), flush=True)
    return 0


def run_profile_case(args):
    """A small case of the bench's decode kernel for ncu captures (not a bench
    line): Gemma-2B's layer and head shapes with 4 layers and a 32,000-token
    vocabulary (0.54 GB of weights per decode step, above L2), two launches of
    `--steps` decode steps after the seeded prompt; capture the second launch
    (`-k regex:decode_persistent -s 1 -c 1`). Prints the case's algorithmic
    bytes per launch so DRAM traffic can be compared and scaled."""
    from huggingfaceeacp_b200 import native

    shape = native.GEMMA_2B.replace(layers=4, vocab=32000, max_positions=256, max_step_rows=16)
    with native.Context(shape) as ctx:
        ctx.load_synthetic(seed=SEED)
        prompt = native.synthetic_tokens(SEED, PROMPT_LENGTH, shape.vocab)
        ctx.prefill_async(prompt)
        ctx.decode_async(args.steps)
        ctx.sync()
        first = ctx.position
        ctx.decode_async(args.steps)
        ctx.sync()
        launch_bytes = sum(native.decode_bytes(shape, first + i + 1) for i in range(args.steps))
    print(json.dumps({"profile_case": "Gemma-2B shapes, 4 layers, vocab 32000", "steps_per_launch": args.steps,
                      "algorithmic_bytes_per_launch": launch_bytes}), flush=True)
    return 0


def run_profile_long(args):
    """A small case of the decode kernel at config 2's context (not a bench
    line): Gemma-2B's layer and head shapes with 4 layers and a 32,000-token
    vocabulary, config 2's 8064-token seeded prompt, then two launches of
    `--steps` decode steps (keys 8065 on); capture the second launch
    (`-k regex:decode_persistent -s 1 -c 1`). Prints the case's algorithmic
    bytes per launch (weights + every step's K/V reads)."""
    from huggingfaceeacp_b200 import native

    shape = native.GEMMA_2B.replace(layers=4, vocab=32000, max_positions=LONG_PROMPT + 128, max_step_rows=2048)
    with native.Context(shape) as ctx:
        ctx.load_synthetic(seed=SEED)
        prompt = native.synthetic_tokens(LONG_SEED, LONG_PROMPT, shape.vocab)
        ctx.prefill_async(prompt)
        ctx.decode_async(args.steps)
        ctx.sync()
        first = ctx.position
        ctx.decode_async(args.steps)
        ctx.sync()
        launch_bytes = sum(native.decode_bytes(shape, first + i + 1) for i in range(args.steps))
    print(json.dumps({"profile_case": f"Gemma-2B shapes, 4 layers, vocab 32000, {LONG_PROMPT}-token prompt",
                      "steps_per_launch": args.steps, "first_keys": first + 1,
                      "algorithmic_bytes_per_launch": launch_bytes}), flush=True)
    return 0


def run_profile_batched(args):
    """A small case of the batched decode step for ncu captures (not a bench
    line): Gemma-2B's layer and head shapes with 2 layers and a 64,000-token
    vocabulary, 64 sequences (one 64-row x tile) of 8-token prompts, then
    `--steps` batched steps. The prompts' prefill runs the int8 MMA (8 rows), so
    the first q8_tc_gemm_ts launch is step 1's q/k/v; per step the launches are
    q/k/v, o, gate/up, down per layer, then the logits (139 MB of weights, above
    L2): `-k regex:q8_tc_gemm_ts -s 8 -c 1` captures step 1's logits product."""
    from huggingfaceeacp_b200 import native

    shape = native.GEMMA_2B.replace(layers=2, vocab=64000, max_positions=64, max_step_rows=64)
    sequences = 64
    with native.Context(shape, sequences=sequences) as ctx:
        ctx.load_synthetic(seed=SEED)
        prompts = np.stack([native.synthetic_tokens(BATCH_SEED + q, 8, shape.vocab) for q in range(sequences)])
        ctx.prefill_batch_async(prompts)
        ctx.decode_batch_async(args.steps)
        ctx.sync()
    logits_bytes = 64000 * 2048 * 17 // 16
    print(json.dumps({"profile_case": "Gemma-2B shapes, 2 layers, vocab 64000, 64 sequences, batched steps",
                      "steps": args.steps, "logits_weight_bytes": logits_bytes}), flush=True)
    return 0


def run_profile_full(args):
    """Full-size cases for launch lists and single-kernel ncu captures (not a
    bench line), each with a profiler range (cudaProfilerStart/Stop) around
    the launches to capture, so `ncu --profile-from-start off` sees only them:
      batched-full  Gemma-2B, 64 sequences of 512-token seeded prompts (config
                    3's), 3 warm-up batched steps, then `--steps` batched steps
                    in the range (~3.5 GB on the device);
      prefill-full  Gemma-2B, config 4's first 2048-token seeded prompt as one
                    2048-row step, once to warm up, then once in the range.
    Prints the case and the range's device time."""
    import torch

    from huggingfaceeacp_b200 import native

    shape = native.GEMMA_2B.replace(max_step_rows=PREFILL_STEP_ROWS, max_positions=PREFILL_STEP_ROWS + 8)
    batched = args.profile_case == "batched-full"
    sequences = BATCH_SEQUENCES if batched else 1
    pages = sequences * -(-(BATCH_PROMPT + 3 + args.steps + 1) // native.PAGE_ROWS) if batched else None
    with native.Context(shape, sequences=sequences, pages=pages) as ctx:
        ctx.load_synthetic(seed=SEED)
        stream = torch.cuda.ExternalStream(ctx.stream)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if batched:
            prompts = np.stack([native.synthetic_tokens(BATCH_SEED + q, BATCH_PROMPT, shape.vocab)
                                for q in range(sequences)])
            ctx.prefill_batch_async(prompts)
            ctx.decode_batch_async(3)
            ctx.sync()
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            start.record(stream)
            ctx.decode_batch_async(args.steps)
            stop.record(stream)
            ctx.sync()
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            case = f"Gemma-2B, {sequences} sequences of {BATCH_PROMPT}-token prompts, {args.steps} batched steps"
        else:
            prompt = native.synthetic_tokens(PREFILL_SEED, PREFILL_PROMPT, shape.vocab)
            ctx.prefill_async(prompt)
            ctx.begin_sequence()
            ctx.sync()
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            start.record(stream)
            ctx.prefill_async(prompt)
            stop.record(stream)
            ctx.sync()
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            case = f"Gemma-2B, one {PREFILL_PROMPT}-token prompt as one {PREFILL_STEP_ROWS}-row step"
    print(json.dumps({"profile_case": case, "range_ms": start.elapsed_time(stop)}), flush=True)
    return 0


def run_profile_prefill(args):
    """A small case of prefill for ncu captures (not a bench line): Gemma-2B's
    layer and head shapes with 2 layers and a 64,000-token vocabulary, a
    2048-token seeded prompt (seed 4, config 4's) prefilled twice in 512-row
    blocks. Per prefill and block the attention launches are one per layer
    (mqa_rows): `-k regex:mqa_rows -s 2 -c 1` captures block 1 of layer 0
    (rows 512..1023 over keys up to 1024). Prints the algorithmic FLOPs of that
    launch (2 per multiply-add of scores and values, causal)."""
    from huggingfaceeacp_b200 import native

    shape = native.GEMMA_2B.replace(layers=2, vocab=64000, max_step_rows=512, max_positions=2056)
    prompt = native.synthetic_tokens(4, 2048, shape.vocab)
    with native.Context(shape) as ctx:
        ctx.load_synthetic(seed=4)
        for _ in range(2):
            ctx.prefill_async(prompt)
            ctx.sync()
    pairs = sum(512 + r + 1 for r in range(512))  # (row, key) pairs of block 1
    flops = pairs * shape.heads * shape.head_width * 2 * 2
    print(json.dumps({"profile_case": "Gemma-2B shapes, 2 layers, vocab 64000, one 2048-token prompt, 512-row blocks",
                      "captured_attention_flops": flops}), flush=True)
    return 0


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=4)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--cpu-steps", type=int, default=16)
    parser.add_argument("--batched-steps", type=int, default=256,
                        help="batched decode steps timed for the b=64/GPU half of the metric")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-config1", action="store_true", help="skip the configs[1] op sweep")
    parser.add_argument("--tp-prefill", action="store_true",
                        help="time tensor-parallel prefill of config 2's prompt over --gpus ranks (not the bench line)")
    parser.add_argument("--tp-rows", type=int, default=PREFILL_STEP_ROWS, help="prefill rows per step for --tp-prefill")
    parser.add_argument("--profile-case", nargs="?", const="decode",
                        choices=["decode", "decode-long", "batched", "prefill", "batched-full", "prefill-full"],
                        help="run an ncu capture case instead of the bench: the decode kernel (default), a batched "
                             "step's tensor-core products, a prompt's prefill (small cases), or a full-size batched "
                             "step or 2048-row prefill step inside a profiler range")
    args = parser.parse_args()
    args.warmup = max(3, args.warmup)
    if args.profile_case == "batched":
        return run_profile_batched(args)
    if args.profile_case == "prefill":
        return run_profile_prefill(args)
    if args.profile_case in ("batched-full", "prefill-full"):
        return run_profile_full(args)
    if args.profile_case == "decode-long":
        return run_profile_long(args)
    if args.profile_case:
        return run_profile_case(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.tp_prefill:
        return run_tp_prefill(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
