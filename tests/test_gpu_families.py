"""The other dense families on the CUDA backend, against the oracle:

  llama    no attention biases, multi-head (4 q / 4 kv heads), rope theta 1e4,
           eps 1e-5, untied head (`llama.rs:431-560`);
  mistral  4:1 GQA with a 48-token decode-time window (`mistral.rs`,
           `ops.rs:1366-1372`), so prompts and decode run past the window;
  qwen3    per-head q/k RMSNorm between the bias and RoPE (`qwen3.rs:441-585`,
           `ops.rs:1130-1152`): fused into the tensor-core QKV epilogue, and a
           follow-up kernel after the GEMV QKV (the persistent decode kernel is
           off for this family).

Every path a sequence takes is covered: chunked tensor-core prefill (bf16
cache) or per-position prefill (f32 cache), single-token steps, the
device-resident greedy chain, and both batched-step kinds.
"""

import numpy as np
import pytest

import oracle as O
from tests.greedy import check_greedy, reference_choice
from cheetah_b200.prepared import PreparedModel, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _tokens(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_family_prefill_decode_and_chain_match_oracle(family_prepared, kv_dtype, monkeypatch):
    from cheetah_b200 import runtime as R
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", "32")  # three chunks for the 70-token prompt
    pm = PreparedModel(family_prepared)
    cfg = resolve_config(pm)
    ref = O.OracleModel(pm, cfg)
    model = R.CudaModel(family_prepared, kv_dtype=kv_dtype, max_positions=1024)
    tol = 1e-4 if kv_dtype == "f32" else 2e-3
    seq = model.new_sequence()
    prompt = _tokens(70, cfg["vocab_size"], 4)
    got = seq.forward(prompt, 0)
    want = ref.forward(prompt, 0, chunk_rows=32)
    assert np.abs(got - want).max() < tol
    check_greedy(int(np.argmax(got)), want, tol, "prompt")
    tok, pos = reference_choice(want), len(prompt)
    for step in range(16):
        want = ref.forward([tok], pos)
        got = np.empty_like(want)
        am = seq.forward_greedy([tok], pos, logits_out=got)
        assert np.abs(got - want).max() < tol, f"step {step}"
        check_greedy(am, want, tol, f"step {step}")
        tok, pos = reference_choice(want), pos + 1
    # The device-resident chain: the oracle follows the GPU's own tokens.
    chain = seq.generate_greedy(tok, pos, 12).tolist()
    prev = tok
    for i, t in enumerate(chain):
        want = ref.forward([prev], pos + i)
        check_greedy(int(t), want, tol, f"chain step {i}")
        prev = int(t)
    model.close()


@pytest.mark.parametrize("step", ["gemv", "gemm"])
def test_family_batched_steps_match_per_sequence_oracle(family_prepared, step, monkeypatch):
    """Sequences at contexts on both sides of mistral's window: the small-batch
    GEMV step and the tensor-core GEMM step, four steps each."""
    from cheetah_b200 import runtime as R
    monkeypatch.setenv("CHEETAH_CUDA_BATCH_GEMV", "1" if step == "gemv" else "0")
    pm = PreparedModel(family_prepared)
    cfg = resolve_config(pm)
    model = R.CudaModel(family_prepared, max_positions=1024)
    lengths = [5, 47, 48, 49, 130, 1]
    rng = np.random.default_rng(23)
    seqs, refs, toks = [], [], []
    for n in lengths:
        prompt = rng.integers(0, cfg["vocab_size"], n).astype(np.uint32)
        seq, ref = model.new_sequence(), O.OracleModel(pm, cfg)
        want = ref.forward(prompt, 0)
        assert np.abs(seq.forward(prompt, 0) - want).max() < 2e-3
        seqs.append(seq)
        refs.append(ref)
        toks.append(reference_choice(want))
    offsets = list(lengths)
    for s in range(4):
        am, logits = model.forward_batch(seqs, toks, offsets, want_logits=True)
        for b, ref in enumerate(refs):
            want = ref.forward([toks[b]], offsets[b])
            assert np.abs(logits[b] - want).max() < 2e-3, (s, b)
            assert am[b] == reference_choice(logits[b])
            check_greedy(int(am[b]), want, 2e-3, f"step {s} sequence {b}")
            toks[b] = reference_choice(want)
            offsets[b] += 1
    model.close()


def test_llama_q8_decode_matches_oracle(tmp_path):
    """A bias-free family through the quantised GEMVs (per-position prefill,
    q8 codes from the device quantiser)."""
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import TINY_LLAMA, write_prepared
    root = write_prepared(tmp_path / "llama", TINY_LLAMA, seed=3)
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    ref = O.OracleModel(pm, cfg, "q8")
    model = R.CudaModel(root, quant="q8", max_positions=512)
    seq = model.new_sequence()
    prompt = _tokens(24, cfg["vocab_size"], 8)
    want = ref.forward(prompt, 0)
    assert np.abs(seq.forward(prompt, 0) - want).max() < 2e-3
    tok, pos = reference_choice(want), len(prompt)
    for step in range(8):
        want = ref.forward([tok], pos)
        got = np.empty_like(want)
        am = seq.forward_greedy([tok], pos, logits_out=got)
        assert np.abs(got - want).max() < 2e-3, f"step {step}"
        check_greedy(am, want, 2e-3, f"step {step}")
        tok, pos = reference_choice(want), pos + 1
    model.close()
