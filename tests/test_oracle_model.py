"""The oracle's Qwen2 forward pinned the way the reference pins its own
(`src/chat/native/decoder.rs:1710-1938`: continuation, snapshot/restore,
chunked prefill ≡ per-position, all bit-exact) plus a torch fp32 third
opinion on the same seeded weights."""

import numpy as np
import pytest

import oracle as O
from cheetah_b200.prepared import PreparedModel, resolve_config


def _model(root, quant="bf16"):
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    return pm, cfg, O.OracleModel(pm, cfg, quant)


def _tokens(n, vocab, seed=1):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


def test_kv_continuation_equals_full_prefill(tiny_prepared):  # decoder.rs:1710
    _, cfg, m = _model(tiny_prepared)
    toks = _tokens(12, cfg["vocab_size"])
    full = m.forward(toks, 0, chunk_rows=1)
    m.clear_cache()
    m.forward(toks[:7], 0, chunk_rows=1)
    for i in range(7, 12):
        step = m.forward(toks[i:i + 1], i)
    np.testing.assert_array_equal(step, full)


def test_chunked_prefill_equals_per_position(tiny_prepared):  # decoder.rs:1824
    _, cfg, m = _model(tiny_prepared)
    toks = _tokens(53, cfg["vocab_size"])
    per_pos = m.forward(toks, 0, chunk_rows=1)
    for chunk in (16, 8, 53):
        m.clear_cache()
        np.testing.assert_array_equal(m.forward(toks, 0, chunk_rows=chunk), per_pos)
    # Non-zero offset: prefix per-position, then a chunked tail.
    m.clear_cache()
    m.forward(toks[:20], 0, chunk_rows=1)
    tail = m.forward(toks[20:], 20, chunk_rows=8)
    np.testing.assert_array_equal(tail, per_pos)


def test_snapshot_restore_then_continue_equals_full_prefill(tiny_prepared):  # decoder.rs:1795
    _, cfg, m = _model(tiny_prepared)
    toks = _tokens(10, cfg["vocab_size"])
    full = m.forward(toks, 0, chunk_rows=4)
    snap = m.kv_snapshot()
    m.clear_cache()
    m.restore_kv_prefix(snap, 6)
    assert m.positions() == 6
    cont = m.forward(toks[6:], 6, chunk_rows=4)
    np.testing.assert_array_equal(cont, full)


def test_clear_cache_isolates_generations(tiny_prepared):  # decoder.rs:1733
    _, cfg, m = _model(tiny_prepared)
    a = m.forward(_tokens(5, cfg["vocab_size"], 3), 0)
    m.forward(_tokens(9, cfg["vocab_size"], 4), 0)
    m.clear_cache()
    np.testing.assert_array_equal(m.forward(_tokens(5, cfg["vocab_size"], 3), 0), a)


def test_token_validation_errors(tiny_prepared):  # ops.rs:1065-1078
    _, cfg, m = _model(tiny_prepared)
    with pytest.raises(RuntimeError, match="empty token input"):
        m.forward([], 0)
    with pytest.raises(RuntimeError, match="exceeds the vocabulary size"):
        m.forward([cfg["vocab_size"]], 0)


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
def test_oracle_matches_torch_fp32(fixture, request):
    torch = pytest.importorskip("torch")
    from tests.torch_ref import TorchQwen2

    root = request.getfixturevalue(fixture)
    pm, cfg, m = _model(root)
    toks = _tokens(24, cfg["vocab_size"], 7)
    ref = TorchQwen2(pm, cfg).forward(toks.tolist())
    got = m.forward(toks, 0, chunk_rows=8)
    np.testing.assert_allclose(got, ref[-1].numpy(), rtol=0, atol=2e-5)
    m.clear_cache()
    for i, t in enumerate(toks):
        step = m.forward([t], i)
        np.testing.assert_allclose(step, ref[i].numpy(), rtol=0, atol=2e-5)


def test_family_oracle_matches_torch_fp32(family_prepared):
    """llama / mistral / qwen3 compositions (`llama.rs:431-560`,
    `mistral.rs`, `qwen3.rs:441-585`): the oracle's chunked and per-position
    forwards against the torch fp32 decoder, 80 tokens so mistral's 48-token
    window is engaged."""
    pytest.importorskip("torch")
    from tests.torch_ref import TorchDecoder

    pm, cfg, m = _model(family_prepared)
    toks = _tokens(80, cfg["vocab_size"], 9)
    ref = TorchDecoder(pm, cfg).forward(toks.tolist())
    got = m.forward(toks, 0, chunk_rows=32)
    np.testing.assert_allclose(got, ref[-1].numpy(), rtol=0, atol=2e-5)
    m.clear_cache()
    for i, t in enumerate(toks):
        step = m.forward([t], i)
        np.testing.assert_allclose(step, ref[i].numpy(), rtol=0, atol=2e-5)


@pytest.mark.parametrize("quant", ["q8", "q4"])
def test_quantised_forward_matches_dequantised_math(tiny_prepared, quant):
    # ops.rs:1180-1237: quantised linears compute scale*code*x; compare to the
    # torch forward run over the oracle's own dequantised weights.
    torch = pytest.importorskip("torch")
    from tests.torch_ref import TorchQwen2

    pm, cfg, m = _model(tiny_prepared, quant)
    ref = TorchQwen2(pm, cfg)
    for name in list(ref.w):
        if name.endswith("_proj.weight"):
            rows, cols = ref.w[name].shape
            w = pm.unit(name).f32().reshape(-1)
            buf = (O.quantize_q8 if quant == "q8" else O.quantize_q4)(w, rows, cols)
            ref.w[name] = torch.from_numpy(O.dequant_matrix(buf, rows, cols, quant))
    toks = _tokens(9, cfg["vocab_size"], 2)
    got = m.forward(toks, 0, chunk_rows=4)
    np.testing.assert_allclose(got, ref.forward(toks.tolist())[-1].numpy(), rtol=0, atol=2e-5)
