"""Parity on the benchmark configurations' real shapes, against the CPU
oracle (the restatement of the reference native path), not against the CUDA
backend itself:

  config 3  Qwen2-0.5B shape, a 2048-token cached prefix, then 1024 prompt
            tokens in 512-row chunks (`qwen2.rs:193-426`; chunked equals
            per-position, `decoder.rs:1824`).
  config 4  Qwen2-7B shape, all 28 layers, with the reference's per-row q8
            and q4 quantisation (`q8.rs:91-125`, `q4.rs:126-161`): a short
            prompt, then greedy steps (tokens identical, logits 2e-2).
  config 2  decode attention 28/4/128 at L = 32k, B = 32 (`ops.rs:1357-1467`).
  config 5  one batched decode step over 16 sequences at mixed contexts up to
            8k on the 0.5B shape, against per-sequence oracle steps over the
            same cached K/V.

The synthetic models are written once per machine (seeded, cached under
$CHEETAH_MODEL_CACHE); the oracle runs on all host cores.
"""

import os

import numpy as np
import pytest

import oracle as O
from tests.greedy import check_greedy, reference_choice
from cheetah_b200.prepared import PreparedModel, cached_synthetic, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

# Contract tolerance for bf16 paths against the f32 oracle (logits max-abs).
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    O.set_threads(os.cpu_count() or 1)


def _toks(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


def test_config3_chunked_prefill_matches_oracle(monkeypatch):
    from cheetah_b200 import runtime as R
    root = cached_synthetic("qwen2-0.5b")
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", "512")
    model = R.CudaModel(root, max_positions=4096)
    ref = O.OracleModel(pm, cfg)
    toks = _toks(2048 + 1024, cfg["vocab_size"], 11)
    seq = model.new_sequence()
    seq.forward(toks[:2048], 0)
    ref.forward(toks[:2048], 0, chunk_rows=512)
    got = seq.forward(toks[2048:], 2048)
    want = ref.forward(toks[2048:], 2048, chunk_rows=512)
    assert np.abs(got - want).max() < LOGIT_TOL
    check_greedy(int(np.argmax(got)), want, LOGIT_TOL, "last prompt row")
    # One layer's K/V (bf16 cache) against the oracle's f32 cache.
    for layer in (0, cfg["num_layers"] - 1):
        gk, gv = seq.kv_layer(layer)
        rk, rv = ref.kv_layer(layer)
        assert np.abs(gk - rk).max() < 2e-2 * max(1.0, np.abs(rk).max())
        assert np.abs(gv - rv).max() < 2e-2 * max(1.0, np.abs(rv).max())
    model.close()


@pytest.mark.parametrize("quant", ["q8", "q4"])
def test_config4_7b_quantised_greedy_matches_oracle(quant):
    """All 28 layers of the 7B shape: a 32-token prompt, then 16 greedy
    steps. The device quantises with the reference's rule (byte-identical,
    tested elsewhere), so both sides compute from the same codes."""
    from cheetah_b200 import runtime as R
    root = cached_synthetic("qwen2-7b")
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    model = R.CudaModel(root, quant=quant, max_positions=512)
    ref = O.OracleModel(pm, cfg, quant)
    prompt = _toks(32, cfg["vocab_size"], 5)
    seq = model.new_sequence()
    got = seq.forward(prompt, 0)
    want = ref.forward(prompt, 0)
    assert np.abs(got - want).max() < LOGIT_TOL
    check_greedy(int(np.argmax(got)), want, LOGIT_TOL, "prompt")
    tok = reference_choice(want)
    exact = 0
    for i in range(16):
        want = ref.forward([tok], 32 + i)
        got = np.empty_like(want)
        am = seq.forward_greedy([tok], 32 + i, logits_out=got)
        assert np.abs(got - want).max() < LOGIT_TOL, f"step {i}"
        exact += check_greedy(am, want, LOGIT_TOL, f"step {i}")
        tok = reference_choice(want)
    assert exact >= 15, f"only {exact} of 16 greedy tokens identical"
    del ref
    model.close()


def test_config2_attention_28_4_128_long_context_batch32():
    """B = 32 sequences at L = 32768, 28/4/128, bf16 cache, shuffled pages:
    every sequence's output against the oracle."""
    from cheetah_b200 import runtime as R
    from tests.test_gpu_kernels import make_paged_kv
    B, L, qh, kvh, D = 32, 32768, 28, 4, 128
    kt, vt, table, dense = make_paged_kv(B, [L] * B, kvh, D, 64, "bf16", seed=29, extra_pages=0)
    q = np.random.default_rng(30).standard_normal((B, qh, D), dtype=np.float32)
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = R.decode_attention(torch.from_numpy(q).cuda(), kt, vt, table, lens, L).cpu().numpy()
    for b in range(B):
        ref = O.attention(dense[b][0], dense[b][1], q[b].reshape(-1), qh, kvh, D)
        err = np.abs(out[b].reshape(-1) - ref).max()
        assert err < 1e-2, f"b={b} max err {err}"


@pytest.mark.parametrize("lengths", [
    [8192, 1, 4097, 63, 64, 65, 7000, 129, 2048, 3001, 511, 6144, 17, 1000, 5555, 300],  # tensor-core GEMM step
    [6000, 1, 700, 64, 8192, 129],                                                      # weight-streaming GEMV step
])
def test_config5_batched_step_mixed_long_contexts_matches_oracle(lengths):
    """Sequences of the 0.5B shape at contexts from 1 to 8192 tokens:
    prefilled on the GPU, their cached K/V copied into per-sequence oracle
    models, then three batched greedy steps compared step by step with the
    oracle's single-sequence steps (logits 2e-2, greedy ids identical). 16
    rows take the tensor-core GEMM step, 6 rows (padded to 8) the GEMV step."""
    from cheetah_b200 import runtime as R
    root = cached_synthetic("qwen2-0.5b")
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    pool = sum(lengths) + 64 * (len(lengths) + 4) + 4096
    model = R.CudaModel(root, max_positions=8192 + 64, kv_pool_tokens=pool)
    rng = np.random.default_rng(31)
    seqs, toks = [], []
    for n in lengths:
        seq = model.new_sequence()
        toks.append(int(np.argmax(seq.forward(rng.integers(0, cfg["vocab_size"], n).astype(np.uint32), 0))))
        seqs.append(seq)
    ref = O.OracleModel(pm, cfg)
    snaps = []
    for seq in seqs:
        layers = [seq.kv_layer(layer) for layer in range(cfg["num_layers"])]
        snaps.append((seq.positions(), layers))
    offsets = list(lengths)
    for step in range(3):
        am, logits = model.forward_batch(seqs, toks, offsets, want_logits=True)
        for b in range(len(seqs)):
            ref.clear_cache()
            ref.restore_kv_prefix(snaps[b], snaps[b][0])
            want = ref.forward([toks[b]], offsets[b])
            err = np.abs(logits[b] - want).max()
            assert err < LOGIT_TOL, f"step {step} sequence {b} (context {offsets[b]}): {err}"
            check_greedy(int(am[b]), want, LOGIT_TOL, f"step {step} sequence {b}")
            # The GPU's cache (the new row included) feeds the next step.
            snaps[b] = (offsets[b] + 1, [seqs[b].kv_layer(layer) for layer in range(cfg["num_layers"])])
        toks = [int(a) for a in am]
        offsets = [o + 1 for o in offsets]
    model.close()
