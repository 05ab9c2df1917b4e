"""Small, self-contained GPU cases for profiling single kernels under ncu.

Each case runs a few launches of one hot-path kernel family on a fixed,
seeded input and exits, so an `ncu -k ... -s N -c 1` capture ends by itself:

  gemv-q8 / gemv-q4   device quantisation of a [rows, cols] bf16 matrix, then
                      three quantised GEMVs (the integer tensor-core kernel
                      for q8, the register-streaming kernel for reference-
                      layout q4) through the C-ABI op entry.
  decode-7b           Qwen2-7B architecture (synthetic weights), q8/q4/bf16:
                      a 16-token prompt, then greedy decode steps through
                      the captured decode graph; prints ms per step.
  batch-decode        Qwen2-0.5B architecture: --batch sequences prefilled
                      with --context tokens each, then --steps batched decode
                      steps (cheetah_cuda_forward_batch); prints ms per step.

Usage: python -m cheetah_b200.profile_cases gemv-q8 [--rows R --cols C]
       python -m cheetah_b200.profile_cases decode-7b [--quant q8] [--steps N]
       python -m cheetah_b200.profile_cases batch-decode [--batch B --context L]
"""

from __future__ import annotations

import argparse
import sys

import numpy as np


def gemv_case(fmt: str, rows: int, cols: int) -> None:
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


def decode_7b_case(quant: str, steps: int) -> None:
    import torch
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config
    root = cached_synthetic("qwen2-7b")
    cfg = resolve_config(PreparedModel(root))
    model = R.CudaModel(root, quant=quant, max_positions=2048)
    seq = model.new_sequence()
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], 16).astype(np.uint32)
    first = int(np.argmax(seq.forward(prompt, 0)))
    toks = seq.generate_greedy(first, 16, 3)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(seq.stream_handle())
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    seq.generate_greedy(int(toks[-1]), 19, steps, wait=False)
    b.record(stream)
    b.synchronize()
    print(f"decode-7b {quant}: {a.elapsed_time(b) / steps:.4f} ms/step")


def batch_decode_case(batch: int, context: int, steps: int) -> None:
    import os
    import time
    # Each prompt is prefilled as one chunk (about 200 launches per sequence),
    # so the batched steps start after a predictable number of launches.
    os.environ.setdefault("CHEETAH_PREFILL_CHUNK", str(context))
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config
    root = cached_synthetic("qwen2-0.5b")
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
    pos = context
    for i in range(steps + 2):
        if i == 2:
            t0 = time.perf_counter()
        toks = model.forward_batch(seqs, toks, [pos] * batch).tolist()
        pos += 1
    ms = (time.perf_counter() - t0) * 1e3 / steps
    print(f"batch-decode B={batch} L={context}: {ms:.4f} ms/step (host-synchronous calls)")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=["gemv-q8", "gemv-q4", "decode-7b", "batch-decode"])
    ap.add_argument("--rows", type=int, default=18944)
    ap.add_argument("--cols", type=int, default=3584)
    ap.add_argument("--quant", default="q8", choices=["q8", "q4", "bf16"])
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--context", type=int, default=4096)
    args = ap.parse_args(argv)
    if args.case.startswith("gemv"):
        gemv_case(args.case.split("-")[1], args.rows, args.cols)
    elif args.case == "batch-decode":
        batch_decode_case(args.batch, args.context, args.steps)
    else:
        decode_7b_case(args.quant, args.steps)
    return 0


if __name__ == "__main__":
    sys.exit(main())
