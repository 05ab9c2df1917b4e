"""Chunked prefill on the tensor cores (tcgen05 GEMMs + causal attention)
against the CPU oracle's chunked forward (`qwen2.rs:193-426`) and against
the CUDA backend's own per-token path."""

import numpy as np
import pytest

import oracle as O
from cheetah_b200.prepared import PreparedModel, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

# bf16 activations feed the tensor cores (f32 accumulation): logits stay
# within 2e-3 of the f32 oracle on the tiny models (contract: 2e-2).
TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _models(root, max_positions=4096):
    from cheetah_b200 import runtime as R
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    return cfg, O.OracleModel(pm, cfg), R.CudaModel(root, max_positions=max_positions)


def _toks(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
@pytest.mark.parametrize("n", [2, 17, 128, 300])
def test_prefill_logits_match_oracle(fixture, n, request):
    cfg, ref, model = _models(request.getfixturevalue(fixture))
    toks = _toks(n, cfg["vocab_size"], n)
    seq = model.new_sequence()
    got = seq.forward(toks, 0)
    want = ref.forward(toks, 0, chunk_rows=256)
    assert np.abs(got - want).max() < TOL
    # The KV rows the chunk appended track the oracle's f32 cache.
    for layer in range(cfg["num_layers"]):
        gk, gv = seq.kv_layer(layer)
        rk, rv = ref.kv_layer(layer)
        assert np.abs(gk - rk).max() < 2e-2 * max(1.0, np.abs(rk).max())
        assert np.abs(gv - rv).max() < 2e-2 * max(1.0, np.abs(rv).max())


@pytest.mark.parametrize("chunk", ["48", "256"])
def test_prefill_with_cached_prefix_and_several_chunks(tiny_prepared, chunk, monkeypatch):
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", chunk)
    cfg, ref, model = _models(tiny_prepared)
    toks = _toks(200, cfg["vocab_size"], 3)
    seq = model.new_sequence()
    seq.forward(toks[:70], 0)                     # cached prefix
    got = seq.forward(toks[70:], 70)              # prompt at a non-zero offset
    ref.forward(toks[:70], 0)
    want = ref.forward(toks[70:], 70)
    assert np.abs(got - want).max() < TOL
    tok = int(np.argmax(want))
    for i in range(6):                            # decode continues from it
        want = ref.forward([tok], 200 + i)
        got = seq.forward([tok], 200 + i)
        assert np.abs(got - want).max() < TOL
        tok = int(np.argmax(want))


def test_prefill_is_independent_of_chunking(tiny_prepared, monkeypatch):
    cfg, _, model = _models(tiny_prepared)
    toks = _toks(180, cfg["vocab_size"], 8)
    a = model.new_sequence()
    full = a.forward(toks, 0)
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", "32")
    b = model.new_sequence()
    np.testing.assert_array_equal(b.forward(toks, 0), full)


def test_config3_shape_chunked_equals_stepwise(monkeypatch):
    """Config 3 (0.5B shape): 2048-token cached prefix, then a prompt in
    512-token chunks; the tensor-core path agrees with the per-token GEMV
    path on the last logits and on the cache contents."""
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import cached_synthetic
    root = cached_synthetic("qwen2-0.5b")
    cfg = resolve_config(PreparedModel(root))
    model = R.CudaModel(root, max_positions=8192)
    toks = _toks(2048 + 1024, cfg["vocab_size"], 11)
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", "512")
    a = model.new_sequence()
    a.forward(toks[:2048], 0)
    la = a.forward(toks[2048:], 2048)
    monkeypatch.setenv("CHEETAH_CUDA_STEPWISE_PREFILL", "1")
    b = model.new_sequence()
    b.forward(toks[:2048], 0)
    lb = b.forward(toks[2048:], 2048)
    assert np.abs(la - lb).max() < 2e-2
    ka, _ = a.kv_layer(23)
    kb, _ = b.kv_layer(23)
    assert np.abs(ka - kb).max() < 5e-2 * max(1.0, np.abs(kb).max())


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
@pytest.mark.parametrize("chunk", ["256", "512"])
def test_prefill_attention_key_splits_match_oracle(fixture, chunk, monkeypatch, request):
    """A long cached prefix at an odd offset, then a multi-chunk prompt: the
    tensor-core attention splits each row block's key range over several CTAs
    (merged afterwards) and crosses 128-key tiles and 64-token pages
    mid-chunk, for head_dim 64 and 128. Checked against the oracle and
    against the mma.sync kernel (CHEETAH_PREFILL_TC=0)."""
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", chunk)
    cfg, ref, model = _models(request.getfixturevalue(fixture))
    toks = _toks(1700, cfg["vocab_size"], 19)
    seq = model.new_sequence()
    seq.forward(toks[:1003], 0)
    ref.forward(toks[:1003], 0)
    got = seq.forward(toks[1003:], 1003)
    want = ref.forward(toks[1003:], 1003)
    assert np.abs(got - want).max() < TOL
    monkeypatch.setenv("CHEETAH_PREFILL_TC", "0")
    other = model.new_sequence()
    other.forward(toks[:1003], 0)
    assert np.abs(other.forward(toks[1003:], 1003) - got).max() < TOL


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
def test_prefill_sliding_window_matches_oracle(fixture, monkeypatch, request):
    """A 150-token sliding window (not a multiple of the 128-key tile) over a
    cached prefix and two chunks: keys below the window are masked per row in
    the tensor-core attention (`ops.rs:1366-1372`)."""
    from cheetah_b200 import runtime as R
    monkeypatch.setenv("CHEETAH_PREFILL_CHUNK", "256")
    root = request.getfixturevalue(fixture)
    pm = PreparedModel(root)
    cfg = dict(resolve_config(pm, 2048))
    cfg["sliding_window"] = 150
    ref = O.OracleModel(pm, cfg)
    model = R.CudaModel(root, config=cfg)
    toks = _toks(900, cfg["vocab_size"], 23)
    seq = model.new_sequence()
    seq.forward(toks[:300], 0)
    ref.forward(toks[:300], 0)
    got = seq.forward(toks[300:], 300)
    want = ref.forward(toks[300:], 300)
    assert np.abs(got - want).max() < TOL
    model.close()
