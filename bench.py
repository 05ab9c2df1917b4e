#!/usr/bin/env python
"""Benchmark of the Cheetah decoder hot path on B200 (driver contract).

Default workload: Qwen2-0.5B-architecture decoder,
seeded random-init bf16 weights in the prepared (`cheetah init`) layout,
batch 1, a 512-token uniform-random prompt, then greedy decode. A timed
"step" is one decode token through the whole model (embedding, 24 layers,
final norm, lm_head, greedy argmax).

  value  device-resident decode tok/s: K greedy steps chained on the device
         (cheetah_cuda_generate_greedy), CUDA events on the sequence stream.
  e2e    the same tokens through the public ModelForward call
         (cheetah_cuda_forward_ex): host token in, host logits (vocab f32) +
         greedy id out, every step, host wall clock.
  roofline  the dominant kernel (bf16 weight-streaming GEMV) timed live with
         CUDA events against MEASURED_PEAKS.json's copy bandwidth.
  cpu_baseline  the C++ restatement of the reference AVX2 path (oracle/),
         all host threads, on a bounded sample of the same workload.

`--impl reference` times that CPU restatement alone (the reference is Rust
and cannot be built in this image). Under torchrun (N>1) each rank decodes
its own sequence on its own GPU (sequence-sharded replicas, no collective on
the data path); value = all ranks' tokens / max-over-ranks time.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT_LEN = 512
METRIC = "decode tok/s (B=1 & batched) + GQA attn HBM GB/s vs peak; prefill tok/s"


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), float(data.get("bf16_tflops", 1634.5)), "measured"
    return 6650.0, 1590.0, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def synthetic_model(name):
    """The seeded synthetic model, written once per box: local rank 0 writes
    it, the other ranks wait for its completion marker (no collective, so a
    slow write cannot time out a process group)."""
    from cheetah_b200.prepared import cached_synthetic, cached_synthetic_path
    _, _, local = dist_env()
    if local == 0:
        return cached_synthetic(name)
    target = cached_synthetic_path(name)
    deadline = time.time() + 1800
    while not (target / ".complete").exists():
        if time.time() > deadline:
            raise RuntimeError(f"timed out waiting for {target}")
        time.sleep(1.0)
    return target


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region.
    The constructor returns once the sampler has produced its first line (so
    sampling is running when the timed region starts); stop() waits for one
    sample past the end and keeps the samples taken from construction to one
    interval after stop()."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, interval_ms: int = 25):
        import threading
        self.device_index = device_index
        self.interval = interval_ms / 1e3
        self.lines = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device_index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", str(interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        if self.proc is not None:
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            deadline = time.monotonic() + 5.0
            while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.005)
        self.t0 = time.monotonic()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t1 = time.monotonic()
        deadline = t1 + 1.0
        while (not self.lines or self.lines[-1][0] < t1) and time.monotonic() < deadline:
            time.sleep(0.005)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, line in list(self.lines):
            if ts < self.t0 or ts > t1 + self.interval:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def cpu_baseline(model_dir, cfg, decode_steps: int):
    """Oracle (C++ restatement of the reference AVX2 path) decode tok/s on a
    bounded sample: 512-token prompt (untimed prefill) + decode steps."""
    import oracle as O
    from cheetah_b200.prepared import PreparedModel

    O.set_threads(os.cpu_count() or 1)
    pm = PreparedModel(model_dir)
    ref = O.OracleModel(pm, cfg, "bf16")
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)
    logits = ref.forward(prompt, 0)
    tok = int(np.argmax(logits))
    t0 = time.perf_counter()
    for i in range(decode_steps):
        logits = ref.forward([tok], PROMPT_LEN + i)
        tok = int(np.argmax(logits))
    dt = time.perf_counter() - t0
    return {"value": decode_steps / dt, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": f"Qwen2-0.5B B=1: {decode_steps} greedy decode steps after a {PROMPT_LEN}-token "
                      f"prompt (C++ restatement of the reference AVX2 path, -O3)",
            "ms_per_token": 1e3 * dt / decode_steps}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config
    model_dir = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(model_dir))
    per_step = []
    import oracle as O
    O.set_threads(os.cpu_count() or 1)
    ref = O.OracleModel(PreparedModel(model_dir), cfg, "bf16")
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)
    tok = int(np.argmax(ref.forward(prompt, 0)))
    pos = PROMPT_LEN
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        tok = int(np.argmax(ref.forward([tok], pos)))
        pos += 1
        if i >= args.warmup:
            per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    value = len(per_step) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(per_step),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init bf16 weights, uniform-random prompt ids)",
        "config": {"workload": "qwen2-0.5b decode B=1 (512-token prompt, greedy)", "batch": 1,
                   "prompt": PROMPT_LEN, "parallelism": "single process (CPU)"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": O.threads(), "kind": "port",
                         "sample": f"{args.steps} decode steps after a {PROMPT_LEN}-token prompt; the "
                                   "reference is Rust (no toolchain here), so its AVX2 path runs as the "
                                   "C++ restatement in oracle/"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# DRAM bytes (read + write) of one decode step of the persistent kernel,
# Qwen2-0.5B, context ~600: ncu dram__bytes_read.sum + dram__bytes_write.sum
# of a one-step launch (summary and command in profiles/).
DECODE_STEP_DRAM_BYTES = 998049536


def gemv_roofline(torch, R, hbm_peak, reps=20):
    """Time the lm_head-shaped bf16 GEMV (151936 x 896, 272 MB > L2) with CUDA
    events on its launching stream."""
    rows, cols = 151936, 896
    w = (torch.randn(rows, cols, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)
    x = torch.randn(1, cols, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(3):
        R.gemv_bf16(w, x, stream=stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        R.gemv_bf16(w, x, stream=stream)
    end.record(stream)
    end.synchronize()
    sec = start.elapsed_time(end) / 1e3 / reps
    bytes_ = rows * cols * 2 + cols * 4 + rows * 4
    achieved = bytes_ / sec / 1e9
    return {"bound": "hbm", "kernel": "gemv_bf16_kernel (lm_head 151936x896)", "achieved": achieved,
            "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": None,
            "bytes_per_launch": bytes_, "us_per_launch": sec * 1e6}


def attention_microbench(torch, R, hbm_peak, quick: bool):
    """Config 2: paged GQA decode attention, bf16 K/V ~N(0,1), shuffled pages."""
    rows = []
    shapes = [(14, 2, 64), (28, 4, 128)]
    batches = [1, 8, 32, 64]
    lengths = [1024, 4096, 16384, 32768]
    if quick:
        batches, lengths = [1, 64], [1024, 32768]
    page = 64
    for qh, kvh, D in shapes:
        for B in batches:
            for L in lengths:
                pages_per = L // page
                total = B * pages_per
                gen = torch.Generator(device="cuda").manual_seed(B * 100003 + L + D)
                k = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
                v = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
                perm = torch.randperm(total, device="cuda", generator=gen).to(torch.int32)
                table = perm.view(B, pages_per).contiguous()
                q = torch.randn(B, qh, D, device="cuda", generator=gen)
                lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
                out = torch.empty_like(q)
                stream = torch.cuda.current_stream()
                for _ in range(3):
                    R.decode_attention(q, k, v, table, lens, L, out=out, stream=stream)
                reps = 10
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                s.record(stream)
                for _ in range(reps):
                    R.decode_attention(q, k, v, table, lens, L, out=out, stream=stream)
                e.record(stream)
                e.synchronize()
                sec = s.elapsed_time(e) / 1e3 / reps
                bytes_ = B * kvh * L * D * 2 * 2 + B * qh * D * 4 * 2
                gbs = bytes_ / sec / 1e9
                rows.append({"shape": f"{qh}/{kvh}/{D}", "B": B, "L": L, "us": round(sec * 1e6, 2),
                             "GBps": round(gbs, 1), "frac_measured": round(gbs / hbm_peak, 4),
                             "frac_8TBps": round(gbs / 8000.0, 4)})
                del k, v, q, out, table, perm
                torch.cuda.empty_cache()
    return rows


def prefill_bench(torch, R, model_dir, cfg, reps: int = 3):
    """Config 3: 2048-token cached prefix, then a 4096-token prompt in chunks
    of 512 (CHEETAH_PREFILL_CHUNK=512); the prefix is restored from a device
    snapshot before every repetition. CUDA events on the sequence stream."""
    prefix, prompt = 2048, 4096
    os.environ["CHEETAH_PREFILL_CHUNK"] = "512"
    model = R.CudaModel(model_dir, max_positions=prefix + prompt + 64)
    toks = np.random.default_rng(3).integers(0, cfg["vocab_size"], prefix + prompt).astype(np.uint32)
    seq = model.new_sequence()
    seq.forward(toks[:prefix], 0)
    snap = seq.kv_snapshot()
    stream = torch.cuda.ExternalStream(seq.stream_handle())
    times = []
    for r in range(reps + 1):
        seq.restore_kv_prefix(snap, prefix)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        seq.forward(toks[prefix:], prefix)
        e.record(stream)
        e.synchronize()
        if r > 0:
            times.append(s.elapsed_time(e) / 1e3)
    sec = min(times)
    L, H, I, QD, KD = cfg["num_layers"], cfg["hidden_size"], cfg["intermediate_size"], \
        cfg["q_heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    linear_params = L * (H * (QD + 2 * KD) + QD * H + 2 * I * H + I * H)
    lin_flops = 2.0 * linear_params * prompt
    attn_flops = 4.0 * cfg["head_dim"] * cfg["q_heads"] * L * sum(p + 1 for p in range(prefix, prefix + prompt))
    lm_flops = 2.0 * cfg["vocab_size"] * H * (prompt // 512)
    total = lin_flops + attn_flops + lm_flops
    del seq, snap
    model.close()
    os.environ.pop("CHEETAH_PREFILL_CHUNK", None)
    return {"workload": "config 3: 0.5B, 2048-token cached prefix + 4096-token prompt, chunks of 512",
            "tok_per_s": prompt / sec, "ms": sec * 1e3, "tflops": total / sec / 1e12,
            "flops": {"linear": lin_flops, "attention": attn_flops, "lm_head": lm_flops},
            "timing": f"min of {reps} repetitions, CUDA events on the sequence stream"}


def decode_7b(args):
    """Config 4: Qwen2-7B-architecture decode (B=1) with q8 / q4 / bf16 linears:
    1024-token prompt, then device-chained greedy steps."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config
    quant = args.workload.split("-")[-1]
    model_dir = synthetic_model("qwen2-7b")
    cfg = resolve_config(PreparedModel(model_dir))
    hbm_peak, _, peak_kind = peaks()
    model = R.CudaModel(model_dir, quant=quant, max_positions=4096)
    seq = model.new_sequence()
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], 1024).astype(np.uint32)
    first = int(np.argmax(seq.forward(prompt, 0)))
    warm = seq.generate_greedy(first, 1024, args.warmup)
    stream = torch.cuda.ExternalStream(seq.stream_handle())
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    seq.generate_greedy(int(warm[-1]), 1024 + args.warmup, args.steps, wait=False)
    e.record(stream)
    e.synchronize()
    clock_info = clocks.stop()
    sec = s.elapsed_time(e) / 1e3
    info = model.info()
    ctx = 1024 + args.warmup + args.steps / 2
    kv = cfg["num_layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * 2 * ctx
    # An untied embedding table is not streamed per token: one bf16 row is.
    embed = 0 if cfg["tie_word_embeddings"] else (cfg["vocab_size"] - 1) * cfg["hidden_size"] * 2
    step_bytes = info["weight_bytes"] - embed + kv
    gbs = step_bytes / (sec / args.steps) / 1e9
    line = {"metric": METRIC, "value": args.steps / sec, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * sec / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": quant,
            "data": "synthetic (seeded random-init bf16 weights quantised per row at load)",
            "config": {"workload": f"qwen2-7b decode B=1 {quant} (config 4: 1024-token prompt)",
                       "model": "Qwen2-7B architecture", "global_batch": 1, "seq_len": 1024},
            "clocks": clock_info,
            "step_roofline": {"bytes_per_token": step_bytes, "achieved_GBps": gbs, "peak": hbm_peak,
                              "peak_kind": peak_kind, "frac_measured": gbs / hbm_peak, "frac_8TBps": gbs / 8000.0}}
    print(json.dumps(line), flush=True)
    return 0


def serve_bench(args):
    """Config 5: 64 concurrent sequences, prompts ~U[128, 8192], outputs
    ~U[32, 512] (seed 2); half share a 1024-token prefix (prefilled once per
    rank, restored from a device snapshot like the engine's prefix cache). The
    64 sequences are sharded across the ranks by the KV-token planner
    (cheetah_b200.dispatch.plan_shards; strong scaling); each rank
    prefills its share, then decodes it with batched greedy steps chained on
    the device (cheetah_cuda_forward_batch_greedy, one call per change of the
    batch) until every sequence has its output length.
    value = generated tokens of all ranks / max-over-ranks decode time."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.dispatch import SeqRequest, plan_shards
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
    name = "qwen2-0.5b" if args.workload == "serve-0.5b" else "qwen2-7b"
    model_dir = synthetic_model(name)
    cfg = resolve_config(PreparedModel(model_dir))
    rng = np.random.default_rng(2)
    n_seq = 64
    prompt_len = rng.integers(128, 8193, n_seq)
    out_len = rng.integers(32, 513, n_seq)
    shared = rng.permutation(n_seq)[: n_seq // 2]
    prefix = rng.integers(0, cfg["vocab_size"], 1024).astype(np.uint32)
    reqs = [SeqRequest(i, int(prompt_len[i]), int(out_len[i]),
                       0 if (i in shared and prompt_len[i] > 1024) else None) for i in range(n_seq)]
    mine = plan_shards(reqs, world)[rank]
    pool = int(sum(prompt_len[i] + out_len[i] + 64 for i in mine)) + 4096
    model = R.CudaModel(model_dir, max_positions=8192 + 512 + 128, kv_pool_tokens=pool, device=local)
    prompts = {}
    for i in range(n_seq):
        body = rng.integers(0, cfg["vocab_size"], int(prompt_len[i])).astype(np.uint32)
        if i in shared and prompt_len[i] > 1024:
            body[:1024] = prefix
        prompts[i] = body
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    snap = None
    if any(i in shared and prompt_len[i] > 1024 for i in mine):
        pre = model.new_sequence()
        pre.forward(prefix, 0)
        snap = pre.kv_snapshot()
    seqs, toks, offs, left = [], [], [], []
    for i in mine:
        seq = model.new_sequence()
        start = 0
        if snap is not None and i in shared and prompt_len[i] > 1024:
            seq.restore_kv_prefix(snap, 1024)
            start = 1024
        logits = seq.forward(prompts[i][start:], start)
        seqs.append(seq)
        toks.append(int(np.argmax(logits)))
        offs.append(int(prompt_len[i]))
        left.append(int(out_len[i]) - 1)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_tokens = int(sum(prompt_len[i] for i in mine))
    if world > 1:
        torch.distributed.barrier()
    generated, steps, batch_sizes = len(mine), 0, []
    t1 = time.perf_counter()
    active = [j for j in range(len(seqs)) if left[j] > 0]
    while active:
        # Greedy ids stay on the device until the next sequence finishes.
        n = min(left[j] for j in active)
        out = model.forward_batch_greedy([seqs[j] for j in active], [toks[j] for j in active],
                                         [offs[j] for j in active], n)
        batch_sizes.extend([len(active)] * n)
        for k, j in enumerate(active):
            toks[j] = int(out[k, -1])
            offs[j] += n
            left[j] -= n
            generated += n
        active = [j for j in active if left[j] > 0]
        steps += n
    decode_s = time.perf_counter() - t1
    totals = torch.tensor([decode_s, prefill_s], device="cuda", dtype=torch.float64)
    counts = torch.tensor([generated, prefill_tokens], device="cuda", dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(totals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(counts, op=torch.distributed.ReduceOp.SUM)
    decode_s, prefill_s = float(totals[0]), float(totals[1])
    generated, prefill_tokens = int(counts[0]), int(counts[1])
    if rank == 0:
        line = {"metric": METRIC, "value": generated / decode_s, "unit": "tok/s", "n_gpus": world,
                "steps": steps, "warmup": 0, "ms_per_step": 1e3 * decode_s / max(steps, 1),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random-init bf16 weights; seeded prompt/output lengths and ids)",
                "config": {"workload": f"config 5: {name} batched serving, 64 sequences sharded over {world} GPU(s)",
                           "model": name, "global_batch": n_seq, "parallelism": f"sequence-sharded x{world}"},
                "decode": {"tokens": generated, "seconds": decode_s,
                           "timing": "host wall clock around the batched decode loop (cheetah_cuda_forward_batch_greedy: "
                                     "ids stay on the device between changes of the batch)",
                           "mean_batch": float(np.mean(batch_sizes)) if batch_sizes else 0.0},
                "prefill": {"tokens": prefill_tokens, "seconds": prefill_s, "tok_per_s": prefill_tokens / prefill_s}}
        print(json.dumps(line), flush=True)
    del seqs
    model.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def op_bench(args):
    """Config 3 (chunked prefill) or config 2 (decode attention) alone, one GPU."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config
    torch.cuda.set_device(dist_env()[2])
    hbm_peak, _, peak_kind = peaks()
    if args.workload == "attention":
        rows = attention_microbench(torch, R, hbm_peak, quick=args.quick_attention)
        best = max((r for r in rows if r["L"] == 32768), key=lambda r: r["GBps"])
        line = {"metric": METRIC, "value": best["GBps"], "unit": "GB/s", "n_gpus": 1, "steps": 1,
                "warmup": 3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) Q/K/V, shuffled pages)",
                "config": {"workload": "config 2: paged GQA decode attention microbench"},
                "attention": rows, "peak_kind": peak_kind}
    else:
        model_dir = synthetic_model("qwen2-0.5b")
        cfg = resolve_config(PreparedModel(model_dir))
        pre = prefill_bench(torch, R, model_dir, cfg)
        line = {"metric": METRIC, "value": pre["tok_per_s"], "unit": "tok/s", "n_gpus": 1, "steps": 1,
                "warmup": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random-init bf16 weights, uniform-random prompt ids)",
                "config": {"workload": pre["workload"]}, "prefill": pre}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config

    world, rank, local = dist_env()
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    else:
        torch.cuda.set_device(local)
    hbm_peak, _, peak_kind = peaks()

    model_dir = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(model_dir))
    total_positions = PROMPT_LEN + args.warmup + args.steps + 8
    model = R.CudaModel(model_dir, device=local, max_positions=max(4096, total_positions + 64))
    prompt = np.random.default_rng(1 + rank).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)

    # ---- value: device-resident greedy chain ----
    seq = model.new_sequence()
    first = int(np.argmax(seq.forward(prompt, 0)))
    warm = seq.generate_greedy(first, PROMPT_LEN, max(args.warmup, 3))
    next_tok = int(warm[-1])
    pos = PROMPT_LEN + max(args.warmup, 3)
    stream = torch.cuda.ExternalStream(seq.stream_handle())
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    seq.generate_greedy(next_tok, pos, args.steps, wait=False)
    end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    elapsed = start.elapsed_time(end) / 1e3
    if world > 1:
        t = torch.tensor([elapsed], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed = float(t.item())
    value = world * args.steps / elapsed
    ms_per_step = 1e3 * elapsed / args.steps

    # ---- e2e: public ModelForward call, host buffers, every step ----
    seq2 = model.new_sequence()
    # Host logits in page-locked memory (the device writes them directly).
    logits = torch.empty(cfg["vocab_size"], dtype=torch.float32, pin_memory=True).numpy()
    tok = int(np.argmax(seq2.forward(prompt, 0, out=logits)))
    pos2 = PROMPT_LEN
    for _ in range(max(args.warmup, 3)):
        tok = seq2.forward_greedy([tok], pos2, logits_out=logits)
        pos2 += 1
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = seq2.forward_greedy([tok], pos2, logits_out=logits)
        pos2 += 1
    e2e_elapsed = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_elapsed], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_elapsed = float(t.item())
    e2e = {"value": world * args.steps / e2e_elapsed, "unit": "tok/s",
           "h2d_bytes_per_step": 4, "d2h_bytes_per_step": cfg["vocab_size"] * 4 + 4,
           "ms_per_step": 1e3 * e2e_elapsed / args.steps,
           "api": "cheetah_cuda_forward_ex (host token in, host logits in pinned memory + greedy id out)"}
    del seq2

    # Algorithmic bytes per decode token at the mean context of the timed run:
    # every weight byte once + the bf16 K/V rows of the context.
    info = model.info()
    mean_ctx = pos + args.steps / 2
    kv_bytes_per_pos = cfg["num_layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * 2
    weight_bytes = info["weight_bytes"]
    step_bytes = weight_bytes + kv_bytes_per_pos * mean_ctx
    step_gbs = step_bytes / (elapsed / args.steps) / 1e9
    persistent = bool(info.get("persistent_decode", 0))

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init bf16 N(0,0.02) weights in the cheetah-init layout; "
                "uniform-random prompt ids)",
        "config": {"workload": "qwen2-0.5b decode B=1 (config 1: 512-token prompt, greedy decode)",
                   "model": "Qwen2-0.5B architecture", "global_batch": world, "seq_len": PROMPT_LEN,
                   "parallelism": f"sequence-sharded replicas x{world}" if world > 1 else "single GPU",
                   "kv_cache": "paged bf16, 64-token pages", "l2": "inputs larger than L2 "
                   f"(weights {weight_bytes / 1e6:.0f} MB per step > 126 MB L2)"},
        "e2e": e2e,
        # The timed greedy run is one cooperative launch of the persistent
        # decode kernel (all steps); the multi-kernel path launches an
        # embedding, 5 kernels per layer and the lm_head per step.
        "gpu_launches": 1 if persistent else args.steps * (2 + 5 * cfg["num_layers"]),
        "clocks": clock_info,
        # Dominant kernel: the persistent decode kernel, per decode step.
        # traffic: DRAM bytes of one step from an ncu capture of a one-step
        # launch at context ~600 (DECODE_STEP_DRAM_BYTES).
        "roofline": {"bound": "hbm", "kernel": "decode_megakernel" if persistent else "decode step (multi-kernel)",
                     "achieved": step_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": step_gbs / hbm_peak,
                     "traffic": DECODE_STEP_DRAM_BYTES if persistent else None,
                     "algorithmic_bytes_per_step": step_bytes, "us_per_step": 1e6 * elapsed / args.steps,
                     "frac_8TBps": step_gbs / 8000.0, "peak_kind": peak_kind},
    }

    if rank == 0:
        line["lm_head_gemv"] = gemv_roofline(torch, R, hbm_peak)
        # The op microbench and prefill figures are single-GPU measurements;
        # a multi-rank run reports the scaled decode line only.
        if not args.no_attention and world == 1:
            line["attention"] = attention_microbench(torch, R, hbm_peak, quick=args.quick_attention)
        if not args.no_prefill and world == 1:
            line["prefill"] = prefill_bench(torch, R, model_dir, cfg)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(model_dir, cfg, args.cpu_steps)
        print(json.dumps(line), flush=True)
    del seq
    model.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-attention", action="store_true")
    ap.add_argument("--quick-attention", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--workload", default="decode-0.5b",
                    choices=["decode-0.5b", "decode-7b-q8", "decode-7b-q4", "decode-7b-bf16",
                             "serve-0.5b", "serve-7b", "prefill-0.5b", "attention"])
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload.startswith("decode-7b"):
        return decode_7b(args)
    if args.workload.startswith("serve"):
        return serve_bench(args)
    if args.workload in ("prefill-0.5b", "attention"):
        return op_bench(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
