"""Decoder parity on the GPU through the `ModelForward` mirror (C-ABI
model/sequence entries) against the CPU oracle, plus the reference's own
forward properties (`decoder.rs:1710-1938`) on the CUDA backend."""

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


def _pair(root, kv_dtype="f32", quant="bf16", max_positions=2048):
    from cheetah_b200 import runtime as R
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    ref = O.OracleModel(pm, cfg, quant)
    model = R.CudaModel(root, quant=quant, kv_dtype=kv_dtype, max_positions=max_positions)
    return cfg, ref, model


def _tokens(n, vocab, seed=1):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_prefill_and_greedy_decode_match_oracle(fixture, kv_dtype, request):
    root = request.getfixturevalue(fixture)
    cfg, ref, model = _pair(root, kv_dtype)
    seq = model.new_sequence()
    prompt = _tokens(40, cfg["vocab_size"])
    got = seq.forward(prompt, 0)
    want = ref.forward(prompt, 0)
    tol = 1e-4 if kv_dtype == "f32" else 2e-3
    assert np.abs(got - want).max() < tol
    pos = len(prompt)
    check_greedy(int(np.argmax(got)), want, tol, "prompt")
    tok = reference_choice(want)
    for step in range(24):
        logits_ref = ref.forward([tok], pos)
        logits_gpu = np.empty_like(logits_ref)
        am = seq.forward_greedy([tok], pos, logits_out=logits_gpu)
        assert np.abs(logits_gpu - logits_ref).max() < tol
        # On-device argmax follows the engine's rule (`engine.rs:2247-2253`).
        assert am == reference_choice(logits_gpu)
        check_greedy(am, logits_ref, tol, f"step {step}")
        tok = reference_choice(logits_ref)
        pos += 1


def test_kv_cache_matches_oracle(tiny_prepared):
    cfg, ref, model = _pair(tiny_prepared, "f32")
    seq = model.new_sequence()
    prompt = _tokens(70, cfg["vocab_size"], 3)
    seq.forward(prompt, 0)
    ref.forward(prompt, 0)
    assert seq.positions() == ref.positions() == 70
    for layer in range(cfg["num_layers"]):
        gk, gv = seq.kv_layer(layer)
        rk, rv = ref.kv_layer(layer)
        assert np.abs(gk - rk).max() < 1e-5 and np.abs(gv - rv).max() < 1e-5


def test_continuation_snapshot_clone_and_clear_are_exact(tiny_prepared):
    # decoder.rs:1710 (continuation), :1795 (snapshot/restore), :1761 (clone),
    # :1733 (clear). Prompt rows take the tensor-core path and single tokens
    # the GEMV path, so prompt-vs-decode continuation agrees to tolerance;
    # every path is deterministic per row, so the rest is bit-exact.
    cfg, _, model = _pair(tiny_prepared, "bf16")
    toks = _tokens(90, cfg["vocab_size"], 5)
    a = model.new_sequence()
    full = a.forward(toks, 0)
    b = a.clone()
    assert b.positions() == 0
    b.forward(toks[:50], 0)
    for i in range(50, 90):
        step = b.forward(toks[i:i + 1], i)
    np.testing.assert_allclose(step, full, rtol=0, atol=2e-3)
    snap = a.kv_snapshot()
    assert snap.positions == 90
    c = model.new_sequence()
    c.restore_kv_prefix(snap, 65)
    assert c.positions() == 65
    np.testing.assert_array_equal(c.forward(toks[65:], 65), full)
    a.clear_cache()
    assert a.positions() == 0
    np.testing.assert_array_equal(a.forward(toks, 0), full)
    # Per-token continuation after a restore is bit-exact with itself.
    d = model.new_sequence()
    d.restore_kv_prefix(snap, 80)
    e = model.new_sequence()
    e.restore_kv_prefix(snap, 80)
    np.testing.assert_array_equal(d.forward([7], 80), e.forward([7], 80))


def test_snapshots_share_pages_and_copy_on_write(tiny_prepared):
    """Snapshots and restored sequences reference the source's KV pages
    instead of copying them; the first append into a shared partial page
    copies that page alone. Every holder stays independent: each restored
    sequence decodes bit-exactly like a sequence that prefilled the same
    prompt itself, while the source keeps decoding other tokens."""
    cfg, _, model = _pair(tiny_prepared, "bf16")
    total = model.info()["kv_pages_total"]
    toks = _tokens(100, cfg["vocab_size"], 12)  # two 64-token pages, the second partial
    a = model.new_sequence()
    a.forward(toks, 0)
    free0 = model.info()["kv_pages_free"]
    snap = a.kv_snapshot()
    assert model.info()["kv_pages_free"] == free0  # nothing copied
    clones = [model.new_sequence() for _ in range(3)]
    for c in clones:
        c.restore_kv_prefix(snap, 100)
    assert model.info()["kv_pages_free"] == free0  # still shared
    fresh = model.new_sequence()
    fresh.forward(toks, 0)
    free1 = model.info()["kv_pages_free"]
    # The source appends first (copy of its tail page), then every clone.
    a.forward([5], 100)
    outs = [c.forward([9], 100) for c in clones]
    assert model.info()["kv_pages_free"] == free1 - 1 - len(clones)
    want = fresh.forward([9], 100)
    for got in outs:
        np.testing.assert_array_equal(got, want)
    # Restoring a shorter prefix shares the pages below it; appends there
    # overwrite only the copy.
    d = model.new_sequence()
    d.restore_kv_prefix(snap, 70)
    e = model.new_sequence()
    e.forward(toks[:70], 0)
    np.testing.assert_array_equal(d.forward(toks[70:80], 70), e.forward(toks[70:80], 70))
    np.testing.assert_array_equal(clones[0].forward([3], 101), clones[1].forward([3], 101))
    # Pages go back to the pool once their last holder lets go.
    for seq in [a, fresh, d, e] + clones:
        seq.clear_cache()
    assert model.info()["kv_pages_free"] < total  # the snapshot still holds its pages
    del snap
    import gc
    gc.collect()
    assert model.info()["kv_pages_free"] == total


def test_forward_errors(tiny_prepared):
    from cheetah_b200 import runtime as R
    cfg, _, model = _pair(tiny_prepared, "bf16", max_positions=128)
    seq = model.new_sequence()
    with pytest.raises(R.CheetahCudaError, match="empty token input"):
        seq.forward([], 0)
    with pytest.raises(R.CheetahCudaError, match="exceeds the vocabulary size"):
        seq.forward([cfg["vocab_size"]], 0)
    with pytest.raises(R.CheetahCudaError, match="does not match"):
        seq.forward([1], 5)
    with pytest.raises(R.CheetahCudaError, match="capacity"):
        seq.forward(list(range(129)), 0)
    seq.forward([1, 2, 3], 0)  # still usable after errors
    assert seq.positions() == 3


def test_pool_exhaustion_is_an_error(tiny_prepared):
    from cheetah_b200 import runtime as R
    model = R.CudaModel(tiny_prepared, max_positions=1024, kv_pool_tokens=128)
    a = model.new_sequence()
    a.forward(list(range(128)), 0)
    b = model.new_sequence()
    with pytest.raises(R.CheetahCudaError, match="exhausted"):
        b.forward([1], 0)
    a.clear_cache()
    b.forward([1], 0)
    assert model.info()["kv_pages_total"] == 2


def test_qwen2_05b_greedy_64_steps_match_oracle():
    """Config 1 shape (Qwen2-0.5B architecture, seeded random-init bf16):
    512-token prompt, then greedy decode; tokens identical over 64 steps and
    logits within 2e-2 max-abs of the reference CPU path (bf16 KV)."""
    from cheetah_b200.prepared import cached_synthetic
    root = cached_synthetic("qwen2-0.5b")
    cfg, ref, model = _pair(root, "bf16", max_positions=1024)
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], 512).astype(np.uint32)
    seq = model.new_sequence()
    got = seq.forward(prompt, 0)
    want = ref.forward(prompt, 0)
    worst = np.abs(got - want).max()
    check_greedy(int(np.argmax(got)), want, 2e-2, "prompt")
    tok = reference_choice(want)
    pos = 512
    exact = 0
    for step in range(64):
        want = ref.forward([tok], pos)
        got = np.empty_like(want)
        tok_gpu = seq.forward_greedy([tok], pos, logits_out=got)
        exact += check_greedy(tok_gpu, want, 2e-2, f"step {step}")
        tok = reference_choice(want)
        worst = max(worst, np.abs(got - want).max())
        pos += 1
    assert worst < 2e-2, worst
    assert exact >= 62, f"only {exact} of 64 greedy tokens identical"


def test_device_greedy_chain_equals_per_token_greedy(tiny_prepared):
    """`generate_greedy` (no host round trip per token) produces the same
    tokens and KV as stepping `forward_greedy` token by token."""
    cfg, _, model = _pair(tiny_prepared, "bf16")
    prompt = _tokens(33, cfg["vocab_size"], 9)
    a = model.new_sequence()
    first = int(np.argmax(a.forward(prompt, 0)))
    chain = a.generate_greedy(first, 33, 40)
    b = model.new_sequence()
    b.forward(prompt, 0)
    tok, expect = first, []
    for i in range(40):
        tok = b.forward_greedy([tok], 33 + i)
        expect.append(tok)
    assert chain.tolist() == expect
    ka, va = a.kv_layer(1)
    kb, vb = b.kv_layer(1)
    np.testing.assert_array_equal(ka, kb)
    np.testing.assert_array_equal(va, vb)
    # The sequence keeps working after a chain (page table and positions).
    np.testing.assert_array_equal(a.forward([5], 73), b.forward([5], 73))


def test_bulk_prefetch_gemv_decode_path(tiny_prepared, monkeypatch):
    """The bulk-prefetch GEMV variant (pair-interleaved QKV rows) keeps parity."""
    monkeypatch.setenv("CHEETAH_CUDA_TMA_GEMV", "1")
    cfg, ref, model = _pair(tiny_prepared, "f32")
    seq = model.new_sequence()
    prompt = _tokens(20, cfg["vocab_size"], 12)
    assert np.abs(seq.forward(prompt, 0) - ref.forward(prompt, 0)).max() < 1e-4
    for i in range(5):
        assert np.abs(seq.forward([i + 3], 20 + i) - ref.forward([i + 3], 20 + i)).max() < 1e-4
