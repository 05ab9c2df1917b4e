#!/usr/bin/env python
"""Benchmark of the Cheetah decoder hot path on B200 (driver contract).

One GPU (`--gpus 1`, the default). `value` is Qwen2-0.5B-architecture B=1
greedy decode (config 1): seeded random-init bf16 weights in the prepared
(`cheetah init`) layout, a 512-token uniform-random prompt, then greedy
decode; a timed step is one token through the whole model (embedding, 24
layers, final norm, lm_head, greedy argmax).

  value      device-resident decode tok/s: K greedy steps chained on the
             device (cheetah_cuda_generate_greedy), CUDA events on the
             sequence stream.
  e2e        the same tokens through the public ModelForward call
             (cheetah_cuda_forward_ex): host token in, host logits (vocab
             f32) + greedy id out, every step, host wall clock.
  roofline   the persistent decode kernel per step against the measured copy
             bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the C++ restatement of the reference AVX2 path (oracle/),
             all host threads, on a bounded sample of the same workload.

The other configurations of the path are sub-objects of the same line, each
with its own roofline and CPU baseline:

  attention  config 2: paged GQA decode attention, 14/2/64 and 28/4/128,
             B in {1, 8, 32, 64}, L in {1k, 4k, 16k, 32k}.
  prefill    config 3: 2048-token cached prefix + 4096-token prompt in
             chunks of 512 (tensor-pipe roofline against the sustained bf16
             figure).
  serve      config 5 on one GPU: 64 sequences, prompts U[128, 8192],
             outputs U[32, 512], half sharing a 1024-token prefix.
  ant        the Ant VRAM tier: the 0.5B model planned into a VRAM pool of
             half its bytes, later layers streamed from pinned host memory.
  decode_7b  config 4: Qwen2-7B architecture, q8 / q4 / bf16 linears,
             1024-token prompt, device-chained greedy steps.

N GPUs (torchrun, N > 1): `value` is config 5, the 64 sequences sharded over
the ranks by the KV-token planner (cheetah_b200.dispatch.plan_shards); each
rank decodes its share with batched greedy steps, and value = generated
tokens of all ranks / max-over-ranks device time (strong scaling of a fixed
sequence set; no collective on the data path).

`--impl reference` times the reference's CPU path for the same config (the
reference is Rust and cannot be built in this image: its AVX2 path runs as
the C++ restatement in oracle/).
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
SERVE_SEQS = 64
SERVE_PREFIX = 1024
# Kernels one chained batched step launches: embedding, 7 per layer (norm,
# QKV GEMM, attention, o_proj GEMM, norm, gate/up GEMM, down GEMM), final
# norm, lm_head GEMM + argmax, and the row-advance kernel.
BATCH_STEP_FIXED_LAUNCHES = 4
BATCH_STEP_LAUNCHES_PER_LAYER = 7


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return (float(data["hbm_gbs"]), float(data.get("bf16_tflops", 1590.0)),
                float(data.get("bf16_tflops_sustained", data.get("bf16_tflops", 1400.0))), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


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


def workload_config(world: int) -> dict:
    """The `config` of the line: identical in both arms (ours and the
    reference's) for the same number of GPUs."""
    if world == 1:
        return {"workload": "qwen2-0.5b decode B=1 (config 1: 512-token prompt, greedy decode)",
                "model": "Qwen2-0.5B architecture", "global_batch": 1, "seq_len": PROMPT_LEN,
                "parallelism": "single GPU", "kv_cache": "paged bf16, 64-token pages",
                "l2": "inputs larger than L2 (988 MB of weights streamed per step > 126 MB L2)"}
    return serve_config(world)


def serve_config(world: int) -> dict:
    return {"workload": f"config 5: qwen2-0.5b batched serving, {SERVE_SEQS} sequences sharded over {world} GPU(s)",
            "model": "Qwen2-0.5B architecture", "global_batch": SERVE_SEQS,
            "seq_len": "prompts U[128, 8192], outputs U[32, 512], half share a 1024-token prefix",
            "parallelism": f"sequence-sharded x{world} (KV-token planner; no collective on the data path)",
            "kv_cache": "paged bf16, 64-token pages",
            "l2": "inputs larger than L2 (988 MB of weights + the batch's K/V per step)"}


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


# ---------------------------------------------------------------------------
# CPU baselines: the C++ restatement of the reference AVX2 path (oracle/),
# all host threads, bounded samples. The oracle is the timed baseline here,
# never the thing measured as ours.

def _oracle(threads: int = 0):
    import oracle as O
    O.set_threads(threads or os.cpu_count() or 1)
    return O


def _oracle_model(model_dir, cfg, quant="bf16"):
    from cheetah_b200.prepared import PreparedModel
    O = _oracle()
    return O, O.OracleModel(PreparedModel(model_dir), cfg, quant)


def _random_kv(ref, cfg, positions: int, seed: int) -> None:
    """Fill the oracle's KV cache with `positions` seeded N(0, 1) rows (the
    cost of a decode step does not depend on the cached values)."""
    rng = np.random.default_rng(seed)
    n = positions * cfg["kv_heads"] * cfg["head_dim"]
    layers = [(rng.standard_normal(n, dtype=np.float32), rng.standard_normal(n, dtype=np.float32))
              for _ in range(cfg["num_layers"])]
    ref.clear_cache()
    ref.restore_kv_prefix((positions, layers), positions)


def cpu_decode_05b(model_dir, cfg, decode_steps: int):
    """Config 1 on the CPU: 512-token prompt (untimed prefill), then timed
    greedy decode steps."""
    O, ref = _oracle_model(model_dir, cfg)
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)
    tok = int(np.argmax(ref.forward(prompt, 0)))
    t0 = time.perf_counter()
    for i in range(decode_steps):
        tok = int(np.argmax(ref.forward([tok], PROMPT_LEN + i)))
    dt = time.perf_counter() - t0
    return {"value": decode_steps / dt, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": f"Qwen2-0.5B B=1: {decode_steps} greedy decode steps after a {PROMPT_LEN}-token "
                      f"prompt (C++ restatement of the reference AVX2 path, -O3)",
            "ms_per_token": 1e3 * dt / decode_steps}


def cpu_attention(rows_gpu):
    """Config 2 on the CPU: the restated `attention` (`ops.rs:1357-1467`,
    parallel over heads) for one sequence at each shape and L, timed per call;
    reported in the GPU rows' unit (algorithmic bytes of a B=1 call / time)."""
    O = _oracle()
    out = []
    for qh, kvh, D in [(14, 2, 64), (28, 4, 128)]:
        for L in (1024, 32768):
            rng = np.random.default_rng(L + D)
            k = rng.standard_normal(L * kvh * D, dtype=np.float32)
            v = rng.standard_normal(L * kvh * D, dtype=np.float32)
            q = rng.standard_normal(qh * D, dtype=np.float32)
            O.attention(k, v, q, qh, kvh, D)
            reps = 20 if L <= 4096 else 5
            t0 = time.perf_counter()
            for _ in range(reps):
                O.attention(k, v, q, qh, kvh, D)
            sec = (time.perf_counter() - t0) / reps
            bytes_ = kvh * L * D * 2 * 2 + qh * D * 4 * 2
            out.append({"shape": f"{qh}/{kvh}/{D}", "B": 1, "L": L, "us": round(sec * 1e6, 1),
                        "GBps": round(bytes_ / sec / 1e9, 2)})
    best = max(out, key=lambda r: r["GBps"])
    return {"value": best["GBps"], "unit": "GB/s", "cores": O.threads(), "kind": "port",
            "sample": "one sequence (B=1) per call at L=1k and 32k for both shapes, f32 cache; GB/s counts "
                      "the GPU rows' algorithmic bytes (bf16 K/V) for the same work; value = best row",
            "rows": out}


def cpu_prefill(model_dir, cfg):
    """Config 3 on the CPU: the restated chunked prefill (`forward_chunked`
    with 512-row chunks) of the first and the last 512-token chunk of the
    4096-token prompt (positions 2048-2559 and 5632-6143) over a 2048-token
    cached prefix and the chunks before them (seeded KV); the 8 chunks are
    interpolated linearly between the two (attention grows linearly with the
    position, the GEMMs do not change)."""
    O, ref = _oracle_model(model_dir, cfg)
    toks = np.random.default_rng(3).integers(0, cfg["vocab_size"], 512).astype(np.uint32)
    times = []
    for start in (2048, 5632):
        _random_kv(ref, cfg, start, seed=start)
        t0 = time.perf_counter()
        ref.forward(toks, start, chunk_rows=512)
        times.append(time.perf_counter() - t0)
    est = sum(times[0] + (times[1] - times[0]) * k / 7 for k in range(8))
    return {"value": 4096 / est, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": "first and last 512-token chunk of the 4096-token prompt timed (seeded KV stands in for "
                      "the cached positions), the 8 chunks interpolated linearly between them",
            "chunk_s": [round(t, 3) for t in times]}


def cpu_serve(model_dir, cfg, reqs):
    """Config 5 on the CPU: the reference serves one sequence at a time on all
    host cores (max-concurrent 1). A decode step is timed at a short and a
    long context (seeded KV) and the per-token time, linear in the context,
    is summed over every generated token of the 64 sequences (a tokens-only
    projection of the whole run)."""
    O, ref = _oracle_model(model_dir, cfg)
    pts = []
    for ctx in (256, 8192):
        _random_kv(ref, cfg, ctx, seed=ctx)
        tok = 17
        ref.forward([tok], ctx)
        t0 = time.perf_counter()
        for i in range(4):
            ref.forward([tok], ctx + 1 + i)
        pts.append((ctx, (time.perf_counter() - t0) / 4))
    (c0, t0_), (c1, t1_) = pts
    slope = (t1_ - t0_) / (c1 - c0)
    total_s = 0.0
    tokens = 0
    for r in reqs:
        n = r.output_len - 1  # the first token comes from the prefill
        mean_ctx = r.prompt_len + (n + 1) / 2
        total_s += n * (t0_ + slope * (mean_ctx - c0))
        tokens += n
    return {"value": tokens / total_s, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": f"decode steps timed at contexts {c0} and {c1} (seeded KV); per-token time linear in the "
                      f"context, summed over the {tokens} decode tokens of the {len(reqs)} sequences served one "
                      "at a time (projection)",
            "ms_per_token_at": {str(c0): round(1e3 * t0_, 3), str(c1): round(1e3 * t1_, 3)}}


def cpu_decode_7b(model_dir, cfg, quant: str, steps: int = 3):
    """Config 4 on the CPU: the restated 7B decoder with the reference's
    per-row q8/q4 quantisation (or bf16) at load, decode steps at context
    1024 (seeded KV stands in for the 1024-token prompt)."""
    O, ref = _oracle_model(model_dir, cfg, quant)
    _random_kv(ref, cfg, 1024, seed=7)
    ref.forward([11], 1024)
    t0 = time.perf_counter()
    for i in range(steps):
        ref.forward([11], 1025 + i)
    dt = (time.perf_counter() - t0) / steps
    return {"value": 1.0 / dt, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": f"Qwen2-7B {quant}: {steps} decode steps at context 1024 (seeded KV stands in for the "
                      "1024-token prompt)", "ms_per_token": 1e3 * dt}


# ---------------------------------------------------------------------------
# GPU measurements

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
    """Config 2: paged GQA decode attention, bf16 K/V ~N(0,1), shuffled pages.

    Device time of the kernel alone: `reps` back-to-back launches are
    captured into one CUDA graph on a private stream and the graph replay is
    timed with CUDA events (no host or ctypes time between launches). Inputs
    smaller than L2 are replicated (disjoint pages, own q/out) so that the
    launches of one replay cycle through more than 256 MB of K/V: no launch
    finds its K/V in the 126 MB L2."""
    rows = []
    shapes = [(14, 2, 64), (28, 4, 128)]
    batches = [1, 8, 32, 64]
    lengths = [1024, 4096, 16384, 32768]
    if quick:
        batches, lengths = [1, 64], [1024, 32768]
    page = 64
    stream = torch.cuda.Stream()
    for qh, kvh, D in shapes:
        for B in batches:
            for L in lengths:
                pages_per = L // page
                bytes_ = B * kvh * L * D * 2 * 2 + B * qh * D * 4 * 2
                reps_l2 = -(-(256 << 20) // bytes_)
                copies = 1 if reps_l2 <= 1 else min(reps_l2, 512)
                reps = max(copies, 10)
                total = copies * B * pages_per
                gen = torch.Generator(device="cuda").manual_seed(B * 100003 + L + D)
                k = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
                v = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
                perm = torch.randperm(total, device="cuda", generator=gen).to(torch.int32)
                tables = perm.view(copies, B, pages_per).contiguous()
                q = torch.randn(copies, B, qh, D, device="cuda", generator=gen)
                lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
                out = torch.empty_like(q)
                torch.cuda.synchronize()
                for r in range(min(copies, 3)):
                    R.decode_attention(q[r], k, v, tables[r], lens, L, out=out[r], stream=stream)
                stream.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(reps):
                        r = i % copies
                        R.decode_attention(q[r], k, v, tables[r], lens, L, out=out[r], stream=stream)
                best = float("inf")
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):  # replay() launches on the current stream
                    graph.replay()
                    stream.synchronize()
                    for _ in range(3):
                        s.record(stream)
                        graph.replay()
                        e.record(stream)
                        e.synchronize()
                        best = min(best, s.elapsed_time(e) / 1e3 / reps)
                gbs = bytes_ / best / 1e9
                rows.append({"shape": f"{qh}/{kvh}/{D}", "B": B, "L": L, "us": round(best * 1e6, 2),
                             "GBps": round(gbs, 1), "frac_measured": round(gbs / hbm_peak, 4),
                             "frac_8TBps": round(gbs / 8000.0, 4), "launches_per_replay": reps,
                             "input_copies": copies})
                del graph, k, v, q, out, tables, perm
                torch.cuda.empty_cache()
    return rows


def ant_bench(torch, R, model_dir, cfg, steps: int = 16):
    """Ant VRAM tier (`ant.rs:655-710`): the 0.5B model opened with the
    reference planner's plan for a VRAM pool of half its unit bytes, so the
    later layers' linears stream from pinned host memory every token. Greedy
    decode tok/s after a 512-token prompt, against the host-to-device copy
    bandwidth measured here with one large pinned copy (the bound of a
    streamed layer)."""
    from cheetah_b200.ant import layer_residency_summary, plan_residency, units_of
    from cheetah_b200.prepared import PreparedModel
    units = units_of(PreparedModel(model_dir))
    pool = sum(u.bytes for u in units) // 2
    plan = plan_residency(units, vram_pool_bytes=pool, ram_budget_bytes=1 << 40)
    states = [e.state() for e in layer_residency_summary(units, plan)]
    host = torch.empty(512 << 20, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty_like(host, device="cuda")
    link = 0.0
    for _ in range(3):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        dev.copy_(host, non_blocking=True)
        e.record()
        e.synchronize()
        link = max(link, host.numel() / (s.elapsed_time(e) / 1e3) / 1e9)
    del host, dev
    model = R.CudaModel(model_dir, max_positions=1024, residency=plan)
    res = model.residency()
    seq = model.new_sequence()
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)
    tok = int(np.argmax(seq.forward(prompt, 0)))
    seq.generate_greedy(tok, PROMPT_LEN, 2)
    t0 = time.perf_counter()
    seq.generate_greedy(tok, PROMPT_LEN + 2, steps)
    sec = (time.perf_counter() - t0) / steps
    gbs = res["streamed_linear_bytes"] / sec / 1e9
    seq.close()
    model.close()
    return {"value": 1.0 / sec, "unit": "tok/s", "steps": steps, "ms_per_step": 1e3 * sec,
            "vram_pool_bytes": pool, "resident_linear_bytes": res["resident_linear_bytes"],
            "streamed_linear_bytes_per_token": res["streamed_linear_bytes"],
            "staging_bytes": res["staging_bytes"],
            "layers": {k: states.count(k) for k in sorted(set(states))},
            "timing": "host wall clock around a device-chained greedy run (cheetah_cuda_generate_greedy, "
                      "eager launches: planned models run without graphs)",
            "roofline": {"bound": "host link", "kernel": "staging copies of the streamed linears",
                         "achieved": gbs, "peak": link, "unit": "GB/s", "frac": gbs / link,
                         "peak_kind": "pinned host-to-device copy of 512 MiB measured here", "traffic": None}}


def prefill_bench(torch, R, model_dir, cfg, tensor_peak, reps: int = 3):
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
    tflops = total / sec / 1e12
    return {"workload": "config 3: 0.5B, 2048-token cached prefix + 4096-token prompt, chunks of 512",
            "value": prompt / sec, "unit": "tok/s", "tok_per_s": prompt / sec, "ms": sec * 1e3,
            "tflops": tflops,
            "flops": {"linear": lin_flops, "attention": attn_flops, "lm_head": lm_flops},
            "roofline": {"bound": "tensor", "kernel": "whole prefill (tcgen05 GEMMs + tcgen05 attention)",
                         "achieved": tflops, "peak": tensor_peak, "unit": "TFLOP/s", "frac": tflops / tensor_peak,
                         "peak_kind": "bf16_tflops_sustained (measured)", "traffic": None},
            "timing": f"min of {reps} repetitions, CUDA events on the sequence stream"}


def decode_7b_run(torch, R, model_dir, cfg, quant, steps, warmup, hbm_peak, prompt_len=1024):
    """Config 4 on one GPU: 1024-token prompt, then device-chained greedy
    steps; CUDA events on the sequence stream."""
    model = R.CudaModel(model_dir, quant=quant, max_positions=4096)
    seq = model.new_sequence()
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], prompt_len).astype(np.uint32)
    first = int(np.argmax(seq.forward(prompt, 0)))
    warm = seq.generate_greedy(first, prompt_len, warmup)
    stream = torch.cuda.ExternalStream(seq.stream_handle())
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    seq.generate_greedy(int(warm[-1]), prompt_len + warmup, steps, wait=False)
    e.record(stream)
    e.synchronize()
    clock_info = clocks.stop()
    sec = s.elapsed_time(e) / 1e3
    info = model.info()
    ctx = prompt_len + warmup + steps / 2
    kv = cfg["num_layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * 2 * ctx
    # An untied embedding table is not streamed per token: one bf16 row is.
    embed = 0 if cfg["tie_word_embeddings"] else (cfg["vocab_size"] - 1) * cfg["hidden_size"] * 2
    step_bytes = info["weight_bytes"] - embed + kv
    gbs = step_bytes / (sec / steps) / 1e9
    del seq
    model.close()
    return {"value": steps / sec, "unit": "tok/s", "steps": steps, "warmup": warmup,
            "ms_per_step": 1e3 * sec / steps, "dtype": quant, "clocks": clock_info,
            "roofline": {"bound": "hbm", "kernel": "7B decode step (multi-kernel graph)", "achieved": gbs,
                         "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "frac_8TBps": gbs / 8000.0,
                         "algorithmic_bytes_per_step": step_bytes, "traffic": None}}


def serve_requests(cfg):
    """Config 5's 64 sequences (seed 2): prompt and output lengths, which ones
    share the 1024-token prefix, and every prompt's ids."""
    from cheetah_b200.dispatch import SeqRequest
    rng = np.random.default_rng(2)
    prompt_len = rng.integers(128, 8193, SERVE_SEQS)
    out_len = rng.integers(32, 513, SERVE_SEQS)
    shared = set(rng.permutation(SERVE_SEQS)[: SERVE_SEQS // 2].tolist())
    prefix = rng.integers(0, cfg["vocab_size"], SERVE_PREFIX).astype(np.uint32)
    uses_prefix = [i in shared and prompt_len[i] > SERVE_PREFIX for i in range(SERVE_SEQS)]
    reqs = [SeqRequest(i, int(prompt_len[i]), int(out_len[i]), 0 if uses_prefix[i] else None)
            for i in range(SERVE_SEQS)]
    prompts = {}
    for i in range(SERVE_SEQS):
        body = rng.integers(0, cfg["vocab_size"], int(prompt_len[i])).astype(np.uint32)
        if uses_prefix[i]:
            body[:SERVE_PREFIX] = prefix
        prompts[i] = body
    return reqs, prompts, prefix, uses_prefix


def serve_run(torch, R, model_dir, cfg, world, rank, local, hbm_peak, reqs, prompts, prefix, uses_prefix):
    """Config 5 on this rank: prefill its share of the sequences (the shared
    prefix once, restored from a device snapshot like the engine's prefix
    cache), then decode them twice from the same state:

    value  batched greedy steps chained on the device
           (cheetah_cuda_forward_batch_greedy, one call per change of the
           batch); CUDA events on the model's batch stream.
    e2e    one public batched call per step (cheetah_cuda_forward_batch):
           host token ids in, greedy ids out, host wall clock.
    Returns this rank's numbers (not yet reduced over ranks)."""
    from cheetah_b200.dispatch import plan_shards, rank_load
    plan = plan_shards(reqs, world)
    mine = plan[rank]
    kv_tokens = int(sum(reqs[i].kv_tokens for i in mine))
    # Room for the sequences, their per-sequence snapshots and the prefix.
    pool = 2 * int(sum(reqs[i].kv_tokens + 64 for i in mine)) + 2 * SERVE_PREFIX + 4096
    model = R.CudaModel(model_dir, max_positions=8192 + 512 + 128, kv_pool_tokens=pool, device=local)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    snap = None
    if any(uses_prefix[i] for i in mine):
        pre = model.new_sequence()
        pre.forward(prefix, 0)
        snap = pre.kv_snapshot()
    seqs, first, offs, left, snaps = [], [], [], [], []
    for i in mine:
        seq = model.new_sequence()
        start = 0
        if snap is not None and uses_prefix[i]:
            seq.restore_kv_prefix(snap, SERVE_PREFIX)
            start = SERVE_PREFIX
        logits = seq.forward(prompts[i][start:], start)
        seqs.append(seq)
        first.append(int(np.argmax(logits)))
        offs.append(reqs[i].prompt_len)
        left.append(reqs[i].output_len - 1)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_tokens = int(sum(reqs[i].prompt_len for i in mine))
    snaps = [s.kv_snapshot() for s in seqs]
    kv_per_pos = cfg["num_layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * 2
    weight_bytes = model.info()["weight_bytes"]

    def decode(chained: bool):
        toks, o, lf = list(first), list(offs), list(left)
        generated, steps, batch_sizes, algo_bytes = 0, 0, [], 0.0
        active = [j for j in range(len(seqs)) if lf[j] > 0]
        while active:
            n = min(lf[j] for j in active) if chained else 1
            for i in range(n):
                algo_bytes += weight_bytes + kv_per_pos * sum(o[j] + i + 1 for j in active)
            if chained:
                out = model.forward_batch_greedy([seqs[j] for j in active], [toks[j] for j in active],
                                                 [o[j] for j in active], n)
                last = out[:, -1]
            else:
                last = model.forward_batch([seqs[j] for j in active], [toks[j] for j in active],
                                           [o[j] for j in active])
            batch_sizes.extend([len(active)] * n)
            for k, j in enumerate(active):
                toks[j] = int(last[k])
                o[j] += n
                lf[j] -= n
                generated += n
            active = [j for j in active if lf[j] > 0]
            steps += n
        return generated, steps, batch_sizes, algo_bytes

    def rewind():
        for s, sn, j in zip(seqs, snaps, range(len(seqs))):
            s.restore_kv_prefix(sn, offs[j])
        torch.cuda.synchronize()

    # Warm-up: one untimed pass of the whole decode (both forms) captures the
    # step graph of every (batch rows, page-table width) the run meets, so
    # the timed passes replay graphs only; the K/V is rewound after each.
    if seqs:
        decode(True)
        rewind()
        decode(False)
        rewind()
    stream = torch.cuda.ExternalStream(model.batch_stream_handle()) if seqs else torch.cuda.current_stream()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    generated, steps, batch_sizes, algo_bytes = decode(True)
    e.record(stream)
    e.synchronize()
    clock_info = clocks.stop()
    decode_s = s.elapsed_time(e) / 1e3
    rewind()
    if world > 1:
        torch.distributed.barrier()
    t1 = time.perf_counter()
    g2, steps2, _, _ = decode(False)
    e2e_s = time.perf_counter() - t1
    assert g2 == generated
    del snaps, seqs, snap
    model.close()
    return {"generated": generated, "steps": steps, "decode_s": decode_s, "e2e_s": e2e_s, "e2e_steps": steps2,
            "mean_batch": float(np.mean(batch_sizes)) if batch_sizes else 0.0, "algo_bytes": algo_bytes,
            "kv_tokens": kv_tokens, "kv_share": kv_tokens / max(1, sum(rank_load(plan, reqs))),
            "prefill_tokens": prefill_tokens, "prefill_s": prefill_s, "sequences": len(mine),
            "clocks": clock_info}


def serve_summary(per_rank, world, hbm_peak, cpu=None):
    """Whole-job numbers from every rank's serve_run (max-over-ranks times)."""
    decode_s = max(r["decode_s"] for r in per_rank)
    e2e_s = max(r["e2e_s"] for r in per_rank)
    generated = sum(r["generated"] for r in per_rank)
    steps = max(r["steps"] for r in per_rank)
    busiest = max(per_rank, key=lambda r: r["decode_s"])
    gbs = busiest["algo_bytes"] / busiest["decode_s"] / 1e9 if busiest["decode_s"] else 0.0
    out = {
        "value": generated / decode_s, "unit": "tok/s", "n_gpus": world, "steps": steps,
        "ms_per_step": 1e3 * decode_s / max(steps, 1), "scaling": "strong",
        "decode": {"tokens": generated, "seconds": decode_s,
                   "timing": "CUDA events on each rank's batch stream around the chained batched decode "
                             "(cheetah_cuda_forward_batch_greedy, one call per change of the batch); max over ranks"},
        "e2e": {"value": generated / e2e_s, "unit": "tok/s", "ms_per_step": 1e3 * e2e_s / max(steps, 1),
                "h2d_bytes_per_step": int(round(np.mean([12 * r["mean_batch"] for r in per_rank]))),
                "d2h_bytes_per_step": int(round(np.mean([4 * r["mean_batch"] for r in per_rank]))),
                "api": "cheetah_cuda_forward_batch once per step (host token ids + offsets in, greedy ids out), "
                       "host wall clock, max over ranks"},
        "per_rank": [{"rank": k, "sequences": r["sequences"], "mean_batch": round(r["mean_batch"], 2),
                      "kv_share": round(r["kv_share"], 4), "decode_s": round(r["decode_s"], 4),
                      "steps": r["steps"], "tokens": r["generated"]} for k, r in enumerate(per_rank)],
        "busiest_rank_kv_share": max(r["kv_share"] for r in per_rank),
        "roofline": {"bound": "hbm", "kernel": "batched decode step (slowest rank)", "achieved": gbs,
                     "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "traffic": None,
                     "algorithmic_bytes": "per step: every weight byte once + the K/V rows of every active "
                                          "sequence's context"},
        "prefill": {"tokens": sum(r["prefill_tokens"] for r in per_rank),
                    "seconds": max(r["prefill_s"] for r in per_rank)},
        "clocks": busiest["clocks"],
    }
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


def _gather_dicts(torch, obj, world):
    """Every rank's JSON-serialisable dict, on every rank (NCCL all_gather of
    a fixed-size byte tensor; every rank takes this step)."""
    if world == 1:
        return [obj]
    data = json.dumps(obj).encode()
    buf = torch.zeros(8192, dtype=torch.uint8, device="cuda")
    assert len(data) <= buf.numel()
    buf[: len(data)] = torch.tensor(list(data), dtype=torch.uint8, device="cuda")
    outs = [torch.zeros_like(buf) for _ in range(world)]
    torch.distributed.all_gather(outs, buf)
    return [json.loads(bytes(o.cpu().numpy().tolist()).rstrip(b"\0").decode()) for o in outs]


def clones_bench(torch, R, model_dir, cfg, single_e2e, clones=16, steps=32, warmup=4, prompt_len=128):
    """`ModelForward` clones driven concurrently: one host thread per clone
    calls the plain per-sequence forward (`cheetah_cuda_forward_ex`, host
    token in, pinned host logits and greedy id out) every step, the way the
    reference's serve loop drives one clone per generation. The backend's
    batcher folds calls that meet into batched steps. Aggregate tok/s over
    the timed steps, wall clock (host-visible end to end)."""
    import threading
    model = R.CudaModel(model_dir, max_positions=1024, kv_pool_tokens=clones * 512 + 4096)
    rng = np.random.default_rng(5)
    seqs = [model.new_sequence() for _ in range(clones)]
    toks = [int(np.argmax(s.forward(rng.integers(0, cfg["vocab_size"], prompt_len).astype(np.uint32), 0)))
            for s in seqs]
    pos = [prompt_len] * clones
    bufs = [torch.empty(cfg["vocab_size"], dtype=torch.float32, pin_memory=True).numpy() for _ in range(clones)]

    def drive(n):
        barrier = threading.Barrier(clones + 1)
        errors = []

        def worker(i):
            try:
                barrier.wait()
                for _ in range(n):
                    toks[i] = seqs[i].forward_greedy([toks[i]], pos[i], logits_out=bufs[i])
                    pos[i] += 1
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append(e)

        threads = [threading.Thread(target=worker, args=(i,)) for i in range(clones)]
        for t in threads:
            t.start()
        barrier.wait()
        t0 = time.perf_counter()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return time.perf_counter() - t0

    drive(warmup)
    before = model.coalesce_stats()
    elapsed = drive(steps)
    after = model.coalesce_stats()
    calls = after["calls"] - before["calls"]
    batched = after["batched_calls"] - before["batched_calls"]
    batches = after["batches"] - before["batches"]
    del seqs
    model.close()
    value = clones * steps / elapsed
    return {"value": value, "unit": "tok/s", "clones": clones, "steps_per_clone": steps,
            "prompt_len": prompt_len, "ms_per_round": 1e3 * elapsed / steps,
            "batched_share": batched / max(1, calls), "mean_batch": batched / max(1, batches),
            "api": "cheetah_cuda_forward_ex, one host thread per clone (host token in, pinned host logits "
                   "+ greedy id out)",
            "vs_single_sequence_e2e": value / single_e2e,
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 4 * clones,
                    "d2h_bytes_per_step": (cfg["vocab_size"] * 4 + 4) * clones}}


def run_serve(args):
    """`--gpus N` with N > 1 (or `--workload serve-0.5b`): config 5 is the value."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config
    from datetime import timedelta

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300))
    hbm_peak, _, _, peak_kind = peaks()
    model_dir = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(model_dir))
    reqs, prompts, prefix, uses_prefix = serve_requests(cfg)
    mine = serve_run(torch, R, model_dir, cfg, world, rank, local, hbm_peak, reqs, prompts, prefix, uses_prefix)
    per_rank = _gather_dicts(torch, mine, world)
    if rank == 0:
        summ = serve_summary(per_rank, world, hbm_peak)
        launches = sum(r["steps"] for r in per_rank) * (BATCH_STEP_FIXED_LAUNCHES +
                                                         BATCH_STEP_LAUNCHES_PER_LAYER * cfg["num_layers"])
        line = {"metric": METRIC, "value": summ["value"], "unit": "tok/s", "n_gpus": world,
                "steps": summ["steps"], "warmup": args.warmup, "ms_per_step": summ["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random-init bf16 weights; seeded prompt/output lengths and ids)",
                "config": workload_config(world) if world > 1 else serve_config(1),
                "e2e": summ["e2e"], "gpu_launches": launches, "clocks": summ["clocks"],
                "roofline": summ["roofline"] | {"peak_kind": peak_kind},
                "serve": {k: v for k, v in summ.items() if k not in ("e2e", "roofline", "clocks")},
                "warmup_note": "one untimed pass of the whole decode per rank (chained and per-step forms) "
                               "captures every step graph before the timed region"}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def run_ours(args):
    """`--gpus 1`: config 1 is the value; configs 2-5 are sub-objects."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    hbm_peak, _, tensor_sustained, peak_kind = peaks()

    model_dir = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(model_dir))
    total_positions = PROMPT_LEN + args.warmup + args.steps + 8
    model = R.CudaModel(model_dir, device=local, max_positions=max(4096, total_positions + 64))
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)

    # ---- value: device-resident greedy chain ----
    seq = model.new_sequence()
    first = int(np.argmax(seq.forward(prompt, 0)))
    warm = seq.generate_greedy(first, PROMPT_LEN, args.warmup)
    next_tok = int(warm[-1])
    pos = PROMPT_LEN + args.warmup
    stream = torch.cuda.ExternalStream(seq.stream_handle())
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
    value = args.steps / elapsed
    ms_per_step = 1e3 * elapsed / args.steps

    # ---- e2e: public ModelForward call, host buffers, every step ----
    seq2 = model.new_sequence()
    # Host logits in page-locked memory (the device writes them directly).
    logits = torch.empty(cfg["vocab_size"], dtype=torch.float32, pin_memory=True).numpy()
    tok = int(np.argmax(seq2.forward(prompt, 0, out=logits)))
    pos2 = PROMPT_LEN
    for _ in range(args.warmup):
        tok = seq2.forward_greedy([tok], pos2, logits_out=logits)
        pos2 += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = seq2.forward_greedy([tok], pos2, logits_out=logits)
        pos2 += 1
    e2e_elapsed = time.perf_counter() - t0
    e2e = {"value": args.steps / e2e_elapsed, "unit": "tok/s",
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
    del seq
    model.close()

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init bf16 N(0,0.02) weights in the cheetah-init layout; "
                "uniform-random prompt ids)",
        "config": workload_config(1),
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

    line["lm_head_gemv"] = gemv_roofline(torch, R, hbm_peak)
    if not args.no_attention:
        rows = attention_microbench(torch, R, hbm_peak, quick=args.quick_attention)
        best = max((r for r in rows if r["L"] == 32768), key=lambda r: r["GBps"])
        line["attention"] = {"value": best["GBps"], "unit": "GB/s", "rows": rows,
                             "roofline": {"bound": "hbm", "kernel": "decode_attention_mma_kernel (best row at 32k)",
                                          "achieved": best["GBps"], "peak": hbm_peak, "unit": "GB/s",
                                          "frac": best["GBps"] / hbm_peak, "traffic": None}}
    if not args.no_prefill:
        line["prefill"] = prefill_bench(torch, R, model_dir, cfg, tensor_sustained)
    if not args.no_ant:
        line["ant"] = ant_bench(torch, R, model_dir, cfg)
    if not args.no_serve:
        reqs, prompts, prefix, uses_prefix = serve_requests(cfg)
        mine = serve_run(torch, R, model_dir, cfg, 1, 0, local, hbm_peak, reqs, prompts, prefix, uses_prefix)
        line["serve"] = serve_summary([mine], 1, hbm_peak)
        line["serve"]["gpu_launches"] = mine["steps"] * (BATCH_STEP_FIXED_LAUNCHES +
                                                          BATCH_STEP_LAUNCHES_PER_LAYER * cfg["num_layers"])
    if not args.no_serve:
        line["clones"] = clones_bench(torch, R, model_dir, cfg, e2e["value"])
    if not args.no_7b:
        dir7 = synthetic_model("qwen2-7b")
        cfg7 = resolve_config(PreparedModel(dir7))
        line["decode_7b"] = {}
        for quant in args.quant_7b.split(","):
            line["decode_7b"][quant] = decode_7b_run(torch, R, dir7, cfg7, quant, args.steps_7b, args.warmup,
                                                     hbm_peak)
    # CPU baselines last: the GPU work is done.
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_05b(model_dir, cfg, args.cpu_steps)
        if "attention" in line:
            line["attention"]["cpu_baseline"] = cpu_attention(line["attention"]["rows"])
        if "prefill" in line:
            line["prefill"]["cpu_baseline"] = cpu_prefill(model_dir, cfg)
        if "serve" in line:
            line["serve"]["cpu_baseline"] = cpu_serve(model_dir, cfg, serve_requests(cfg)[0])
        if "decode_7b" in line:
            for quant, row in line["decode_7b"].items():
                row["cpu_baseline"] = cpu_decode_7b(dir7, cfg7, quant)
    print(json.dumps(line), flush=True)
    return 0


# DRAM bytes (read + write) of one decode step of the persistent kernel,
# Qwen2-0.5B, context ~600: ncu dram__bytes_read.sum + dram__bytes_write.sum
# of a one-step launch (summary and command in profiles/).
DECODE_STEP_DRAM_BYTES = 998049536


def run_reference(args):
    """The reference arm: the reference's CPU path (C++ restatement of the
    AVX2 backend, oracle/) on all host threads, on the same config as ours
    for this number of GPUs. Under torchrun only rank 0 runs and prints."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from cheetah_b200.prepared import PreparedModel, resolve_config
    model_dir = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(model_dir))
    O = _oracle()
    if world == 1:
        ref = O.OracleModel(PreparedModel(model_dir), cfg, "bf16")
        prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.uint32)
        tok = int(np.argmax(ref.forward(prompt, 0)))
        pos = PROMPT_LEN
        per_step = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            tok = int(np.argmax(ref.forward([tok], pos)))
            pos += 1
            if i >= args.warmup:
                per_step.append(time.perf_counter() - t0)
        total = sum(per_step)
        value = len(per_step) / total
        sample = (f"{args.steps} greedy decode steps after a {PROMPT_LEN}-token prompt; the reference is Rust (no "
                  "toolchain here), so its AVX2 path runs as the C++ restatement in oracle/")
        ms = 1e3 * total / len(per_step)
        scaling = "weak"
    else:
        cpu = cpu_serve(model_dir, cfg, serve_requests(cfg)[0])
        value = cpu["value"]
        sample = cpu["sample"] + "; the reference serves on one host, whatever the GPU count"
        ms = 1e3 / value
        scaling = "strong"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init bf16 weights, uniform-random prompt ids)",
        "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": O.threads(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Single-kernel cases for ncu captures (small, seeded, end by themselves).

def case_gemv(fmt: str, rows: int, cols: int) -> int:
    """Device quantisation of a [rows, cols] bf16 matrix, then three quantised
    GEMVs through the C-ABI op entry."""
    import torch
    from cheetah_b200 import runtime as R
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    buf = R.quantize(w, fmt)
    x = torch.randn(cols, device="cuda", generator=g)
    for _ in range(3):
        y = R.gemv_quant(buf, fmt, rows, cols, x)
    torch.cuda.synchronize()
    print(f"{fmt} gemv {rows}x{cols}: sum|y| = {float(y.abs().sum()):.6f}")
    return 0


def case_batch_decode(batch: int, context: int, steps: int) -> int:
    """Qwen2-0.5B: `batch` sequences prefilled with `context` tokens each (one
    chunk per prompt), then `steps` host-synchronous batched decode steps."""
    os.environ.setdefault("CHEETAH_PREFILL_CHUNK", str(context))
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config
    root = synthetic_model("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(root))
    model = R.CudaModel(root, max_positions=context + steps + 8,
                        kv_pool_tokens=batch * (context + steps + 128))
    rng = np.random.default_rng(3)
    seqs, toks = [], []
    for _ in range(batch):
        seq = model.new_sequence()
        prompt = rng.integers(0, cfg["vocab_size"], context).astype(np.uint32)
        toks.append(int(np.argmax(seq.forward(prompt, 0))))
        seqs.append(seq)
    import torch
    pos = context
    for i in range(steps + 2):
        if i == 2:
            torch.cuda.profiler.start()  # `ncu --profile-from-start off` captures the timed steps only
            t0 = time.perf_counter()
        toks = model.forward_batch(seqs, toks, [pos] * batch).tolist()
        pos += 1
    ms = (time.perf_counter() - t0) * 1e3 / steps
    torch.cuda.profiler.stop()
    print(f"batch-decode B={batch} L={context}: {ms:.4f} ms/step (host-synchronous calls)")
    return 0


def case_attention(shape: str, batch: int, context: int, launches: int = 3) -> int:
    """One config-2 case, `launches` plain back-to-back launches of the
    decode attention op (no graph): the profiling target for one kernel."""
    import torch
    from cheetah_b200 import runtime as R
    qh, kvh, D = (int(v) for v in shape.split("/"))
    page = 64
    pages_per = context // page
    total = batch * pages_per
    gen = torch.Generator(device="cuda").manual_seed(batch * 100003 + context + D)
    k = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
    v = torch.randn(total, kvh, page, D, device="cuda", dtype=torch.bfloat16, generator=gen)
    table = torch.randperm(total, device="cuda", generator=gen).to(torch.int32).view(batch, pages_per).contiguous()
    q = torch.randn(batch, qh, D, device="cuda", generator=gen)
    lens = torch.full((batch,), context, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    R.decode_attention(q, k, v, table, lens, context, out=out)  # scratch allocation, function attributes
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(launches):
        R.decode_attention(q, k, v, table, lens, context, out=out)
    torch.cuda.synchronize()
    us = (time.perf_counter() - t0) / launches * 1e6
    print(f"attention {shape} B={batch} L={context}: 1 + {launches} launches, {us:.1f} us each after the "
          "first (host clock)")
    return 0


def run_decode_7b(args):
    """`--workload decode-7b-<quant>`: config 4 alone, one line."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config
    torch.cuda.set_device(dist_env()[2])
    hbm_peak, _, _, peak_kind = peaks()
    quant = args.workload.split("-")[-1]
    dir7 = synthetic_model("qwen2-7b")
    cfg7 = resolve_config(PreparedModel(dir7))
    row = decode_7b_run(torch, R, dir7, cfg7, quant, args.steps, args.warmup, hbm_peak, args.prompt_7b)
    line = {"metric": METRIC, "value": row["value"], "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": row["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": quant,
            "data": "synthetic (seeded random-init bf16 weights quantised per row at load)",
            "config": {"workload": f"qwen2-7b decode B=1 {quant} (config 4: {args.prompt_7b}-token prompt)",
                       "model": "Qwen2-7B architecture", "global_batch": 1, "seq_len": args.prompt_7b},
            "clocks": row["clocks"], "roofline": row["roofline"] | {"peak_kind": peak_kind}}
    print(json.dumps(line), flush=True)
    return 0


def attention_trace(R, cfg, sms: int):
    """Per-key-tile timeline of the two-tile prefill attention kernel from a
    profiling build (`python -m cheetah_b200.build --define CHEETAH_ATTN_TRACE
    --out cheetah_b200/libcheetah_cuda_attn_trace.so`, selected with
    CHEETAH_CUDA_LIB): query block 0, head 0, split 0 of the last layer-0
    launch of config 3 (the last chunk), in SM cycles since the CTA started."""
    import ctypes
    import statistics
    lib = R.lib()
    if not hasattr(lib, "cheetah_cuda_debug_attn_trace"):
        raise SystemExit("prefill-attention-trace needs a library built with -DCHEETAH_ATTN_TRACE "
                         "(python -m cheetah_b200.build --define CHEETAH_ATTN_TRACE --out <lib>; "
                         "CHEETAH_CUDA_LIB=<lib>)")
    buf = (ctypes.c_longlong * 256)()
    if lib.cheetah_cuda_debug_attn_trace(buf) != 0:
        raise SystemExit(lib.cheetah_cuda_last_error().decode())
    ev = [list(buf[16 * j:16 * j + 16]) for j in range(16)]
    # Split 0 of query block 0 in the last chunk (the launcher's split rule).
    prefix, prompt, chunk = 2048, 4096, 512  # prefill_bench's config 3
    offset = prefix + prompt - chunk
    blocks = ((chunk + 255) // 256) * cfg["q_heads"]
    key_tiles = (offset + chunk + 127) // 128
    splits = max(1, min(8, sms // blocks, key_tiles // 2))
    all_hi = (offset + 255) // 128 + 1
    n = min(16, -(-all_hi // splits))
    med = lambda xs: statistics.median(xs) if xs else None
    rows = ev[:n]
    return {
        "launch": f"last chunk (positions {offset}..{offset + chunk - 1}), layer 0, query block 0, head 0, split 0 of {splits}",
        "key_tiles": n,
        "events": rows,
        "event_names": ["A S landed", "A row max", "A O rescaled", "A P released", "B S landed", "B row max",
                        "B O rescaled", "B P released", "MMA saw P_A", "MMA issued PV_A", "MMA issued S_B(j+1)",
                        "MMA saw P_B", "MMA issued PV_B", "MMA issued S_A(j+2)", "producer issued tile", "-"],
        "median_cycles": {
            "tile_pair": med([rows[j + 1][0] - rows[j][0] for j in range(1, n - 1)]),
            "A_max_pass": med([r[1] - r[0] for r in rows[1:]]),
            "A_rescale": med([r[2] - r[1] for r in rows[1:]]),
            "A_exp_pass": med([r[3] - r[2] for r in rows[1:]]),
            "mma_issue_pv_a": med([r[9] - r[8] for r in rows[1:]]),
            "mma_issue_s_b": med([r[10] - r[9] for r in rows[1:n - 1]]),
            "mma_issue_pv_b": med([r[12] - r[11] for r in rows[1:]]),
        },
    }


def run_op(args):
    """`--workload prefill-0.5b | prefill-attention-trace | attention`: config 3
    or config 2 alone."""
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, resolve_config
    torch.cuda.set_device(dist_env()[2])
    hbm_peak, _, tensor_sustained, peak_kind = peaks()
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
        pre = prefill_bench(torch, R, model_dir, cfg, tensor_sustained)
        line = {"metric": METRIC, "value": pre["tok_per_s"], "unit": "tok/s", "n_gpus": 1, "steps": 1,
                "warmup": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random-init bf16 weights, uniform-random prompt ids)",
                "config": {"workload": pre["workload"]}, "prefill": pre}
        if args.workload == "prefill-attention-trace":
            props = torch.cuda.get_device_properties(torch.cuda.current_device())
            line["attention_trace"] = attention_trace(R, cfg, props.multi_processor_count)
    print(json.dumps(line), flush=True)
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
    ap.add_argument("--no-serve", action="store_true")
    ap.add_argument("--no-ant", action="store_true")
    ap.add_argument("--no-7b", action="store_true")
    ap.add_argument("--quant-7b", default="q8,q4,bf16")
    ap.add_argument("--steps-7b", type=int, default=64)
    ap.add_argument("--prompt-7b", type=int, default=1024, help="decode-7b-* workloads: prompt tokens")
    ap.add_argument("--workload", default="default",
                    choices=["default", "decode-7b-q8", "decode-7b-q4", "decode-7b-bf16", "serve-0.5b",
                             "prefill-0.5b", "prefill-attention-trace", "attention", "attention-case",
                             "gemv-q8", "gemv-q4",
                             "batch-decode"])
    ap.add_argument("--rows", type=int, default=18944, help="gemv-q8/q4 case")
    ap.add_argument("--cols", type=int, default=3584, help="gemv-q8/q4 case")
    ap.add_argument("--batch", type=int, default=32, help="batch-decode case")
    ap.add_argument("--context", type=int, default=4096, help="batch-decode / attention-case")
    ap.add_argument("--shape", default="14/2/64", help="attention-case: q_heads/kv_heads/head_dim")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, _, _ = dist_env()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload.startswith("decode-7b"):
        return run_decode_7b(args)
    if args.workload in ("prefill-0.5b", "prefill-attention-trace", "attention"):
        return run_op(args)
    if args.workload in ("gemv-q8", "gemv-q4"):
        return case_gemv(args.workload.split("-")[1], args.rows, args.cols)
    if args.workload == "batch-decode":
        return case_batch_decode(args.batch, args.context, args.steps)
    if args.workload == "attention-case":
        return case_attention(args.shape, args.batch, args.context)
    if world > 1 or args.workload == "serve-0.5b":
        return run_serve(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
