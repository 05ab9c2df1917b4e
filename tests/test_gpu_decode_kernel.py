"""The persistent single-sequence decode kernel (one cooperative launch per
step, or per run of greedy steps) against the CPU oracle and against the
multi-kernel decode path, through the C-ABI sequence entries.

The persistent kernel serves bf16-weight, bf16-KV models whose shapes fit
its shared-memory tiles; `CHEETAH_CUDA_MEGAKERNEL=0` at model open selects
the multi-kernel path for the same model."""

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


def _model(root, monkeypatch, persistent, max_positions=2048, config=None):
    from cheetah_b200 import runtime as R
    monkeypatch.setenv("CHEETAH_CUDA_MEGAKERNEL", "1" if persistent else "0")
    model = R.CudaModel(root, kv_dtype="bf16", max_positions=max_positions, config=config)
    assert model.info()["persistent_decode"] == (1 if persistent else 0)
    return model


def _tokens(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.uint32)


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared", "tiny15b_prepared"])
def test_persistent_decode_matches_oracle_and_multikernel_path(fixture, request, monkeypatch):
    root = request.getfixturevalue(fixture)
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    ref = O.OracleModel(pm, cfg, "bf16")
    fast = _model(root, monkeypatch, True)
    slow = _model(root, monkeypatch, False)
    prompt = _tokens(45, cfg["vocab_size"], 3)
    a, b = fast.new_sequence(), slow.new_sequence()
    la, lb = a.forward(prompt, 0), b.forward(prompt, 0)
    want = ref.forward(prompt, 0)
    tok = reference_choice(want)
    check_greedy(int(np.argmax(la)), want, 2e-3, "prompt (persistent)")
    check_greedy(int(np.argmax(lb)), want, 2e-3, "prompt (multi-kernel)")
    pos = len(prompt)
    for step in range(20):
        want = ref.forward([tok], pos)
        ga, gb = np.empty_like(want), np.empty_like(want)
        ta = a.forward_greedy([tok], pos, logits_out=ga)
        tb = b.forward_greedy([tok], pos, logits_out=gb)
        assert np.abs(ga - want).max() < 2e-3, f"step {step}"
        assert np.abs(ga - gb).max() < 2e-3, f"step {step}"
        check_greedy(ta, want, 2e-3, f"step {step} (persistent)")
        check_greedy(tb, want, 2e-3, f"step {step} (multi-kernel)")
        # Packed-key argmax keeps the larger index on ties (`engine.rs:2247-2253`).
        assert ta == int(np.nonzero(ga == ga.max())[0][-1])
        tok = ta
        pos += 1
    # Both paths appended the same K/V rows for the decoded positions.
    ka, va = a.kv_layer(1)
    kb, vb = b.kv_layer(1)
    assert np.abs(ka - kb).max() < 2e-2 and np.abs(va - vb).max() < 2e-2


def test_persistent_chain_equals_per_token_and_is_reproducible(tiny_prepared, monkeypatch):
    """One launch for 48 greedy steps gives the per-token launches' tokens;
    the arithmetic is in fixed order, so logits repeat bit for bit."""
    model = _model(tiny_prepared, monkeypatch, True)
    cfg = model.cfg
    prompt = _tokens(70, cfg["vocab_size"], 5)
    a = model.new_sequence()
    first = int(np.argmax(a.forward(prompt, 0)))
    chain = a.generate_greedy(first, 70, 48)
    b = model.new_sequence()
    b.forward(prompt, 0)
    tok, expect = first, []
    for i in range(48):
        tok = b.forward_greedy([tok], 70 + i)
        expect.append(tok)
    assert chain.tolist() == expect
    ka, va = a.kv_layer(0)
    kb, vb = b.kv_layer(0)
    np.testing.assert_array_equal(ka, kb)
    np.testing.assert_array_equal(va, vb)
    np.testing.assert_array_equal(a.forward([7], 118), b.forward([7], 118))
    runs = []
    for _ in range(2):
        c = model.new_sequence()
        c.forward(prompt, 0)
        runs.append(c.forward([first], 70))
    np.testing.assert_array_equal(runs[0], runs[1])


def test_persistent_decode_long_context_and_window(tiny_prepared, monkeypatch):
    """Key chunks spread over many pages (1.5k positions), and a sliding
    window that hides the early keys (`ops.rs:1366-1372`)."""
    pm = PreparedModel(tiny_prepared)
    for window in (0, 200):
        cfg = dict(resolve_config(pm, 2048))
        cfg["sliding_window"] = window
        ref = O.OracleModel(pm, cfg, "bf16")
        model = _model(tiny_prepared, monkeypatch, True, config=cfg)
        seq = model.new_sequence()
        prompt = _tokens(1500, cfg["vocab_size"], 11 + window)
        seq.forward(prompt, 0)
        ref.forward(prompt, 0)
        for i, tok in enumerate([3, 99, 512]):
            got = seq.forward([tok], 1500 + i)
            want = ref.forward([tok], 1500 + i)
            assert np.abs(got - want).max() < 2e-3, (window, i)
        model.close()


def test_persistent_decode_qwen2_05b_chain_matches_oracle(monkeypatch):
    """Config 1 shape: a 512-token prompt, then 64 greedy steps in one launch;
    tokens identical to the reference CPU path."""
    from cheetah_b200.prepared import cached_synthetic
    root = cached_synthetic("qwen2-0.5b")
    pm = PreparedModel(root)
    cfg = resolve_config(pm, 1024)
    ref = O.OracleModel(pm, cfg, "bf16")
    model = _model(root, monkeypatch, True, max_positions=1024)
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], 512).astype(np.uint32)
    seq = model.new_sequence()
    first = int(np.argmax(seq.forward(prompt, 0)))
    check_greedy(first, ref.forward(prompt, 0), 2e-2, "prompt")
    chain = seq.generate_greedy(first, 512, 64).tolist()
    # The oracle follows the chain's own tokens; each chained token must be
    # the oracle's greedy choice (or the other side of a near-tie).
    tok, exact = first, 0
    for i in range(64):
        exact += check_greedy(chain[i], ref.forward([tok], 512 + i), 2e-2, f"step {i}")
        tok = chain[i]
    assert exact >= 62, f"only {exact} of 64 greedy tokens identical"


def test_persistent_decode_appends_kv_at_page_boundaries(tiny_prepared, monkeypatch):
    """Tokens whose positions open a new KV page (installed by the kernel
    itself, positions 0 and 64) land in every layer's cache as on the
    multi-kernel path."""
    fast = _model(tiny_prepared, monkeypatch, True)
    slow = _model(tiny_prepared, monkeypatch, False)
    cfg = fast.cfg
    width = cfg["kv_heads"] * cfg["head_dim"]
    for prompt_len in (0, 64):
        a, b = fast.new_sequence(), slow.new_sequence()
        if prompt_len:
            prompt = _tokens(prompt_len, cfg["vocab_size"], 13)
            a.forward(prompt, 0)
            b.forward(prompt, 0)
        ga = a.forward([7], prompt_len)
        gb = b.forward([7], prompt_len)
        assert np.abs(ga - gb).max() < 2e-3
        for layer in range(cfg["num_layers"]):
            ka, va = (x.reshape(-1, width) for x in a.kv_layer(layer))
            kb, vb = (x.reshape(-1, width) for x in b.kv_layer(layer))
            # the page-opening position's row is written, and matches
            assert np.abs(ka[prompt_len]).max() > 0 and np.abs(va[prompt_len]).max() > 0, layer
            assert np.abs(ka - kb).max() < 1e-2 and np.abs(va - vb).max() < 1e-2, layer


def test_logits_into_pinned_and_pageable_host_buffers_agree(tiny_prepared, monkeypatch):
    """forward_ex writes logits straight into a page-locked caller buffer and
    through its own staging buffer otherwise; both give the same values."""
    model = _model(tiny_prepared, monkeypatch, True)
    cfg = model.cfg
    prompt = _tokens(33, cfg["vocab_size"], 21)
    a, b = model.new_sequence(), model.new_sequence()
    a.forward(prompt, 0)
    b.forward(prompt, 0)
    pinned = torch.empty(cfg["vocab_size"], dtype=torch.float32, pin_memory=True).numpy()
    pageable = np.empty(cfg["vocab_size"], dtype=np.float32)
    tok = 5
    for i in range(4):
        ta = a.forward_greedy([tok], 33 + i, logits_out=pinned)
        tb = b.forward_greedy([tok], 33 + i, logits_out=pageable)
        np.testing.assert_array_equal(pinned, pageable)
        assert ta == tb == int(np.nonzero(pageable == pageable.max())[0][-1])
        tok = ta


def test_persistent_decode_wait_timeout_reports_error_and_recovers(tiny_prepared, monkeypatch):
    """The kernel's bounded waits, exercised without a fault: the test hook
    CHEETAH_CUDA_TEST_STALL_WAIT=1 makes the run's first attention wait target
    a count nothing reaches, with a 20 ms bound (no copy is left waiting: the
    weight copies already issued land and are drained). The call returns the
    device guard's error with the kernel's code (0x4D4B01), the sequence keeps
    its positions, the error word and counters are reset, and the same
    sequence then decodes exactly as a sequence that never failed."""
    from cheetah_b200 import runtime as R
    model = _model(tiny_prepared, monkeypatch, True)
    cfg = model.cfg
    prompt = _tokens(40, cfg["vocab_size"], 13)
    seq, clean = model.new_sequence(), model.new_sequence()
    tok = int(np.argmax(seq.forward(prompt, 0)))
    clean.forward(prompt, 0)
    monkeypatch.setenv("CHEETAH_CUDA_TEST_STALL_WAIT", "1")
    with pytest.raises(R.CheetahCudaError, match=f"code {0x4D4B01}"):
        seq.forward_greedy([tok], 40)
    assert seq.positions() == 40
    with pytest.raises(R.CheetahCudaError, match=f"code {0x4D4B01}"):
        seq.generate_greedy(tok, 40, 4)
    assert seq.positions() == 40
    monkeypatch.delenv("CHEETAH_CUDA_TEST_STALL_WAIT")
    got, want = np.empty(cfg["vocab_size"], np.float32), np.empty(cfg["vocab_size"], np.float32)
    ta = seq.forward_greedy([tok], 40, logits_out=got)
    tb = clean.forward_greedy([tok], 40, logits_out=want)
    np.testing.assert_array_equal(got, want)
    assert ta == tb
    np.testing.assert_array_equal(seq.generate_greedy(ta, 41, 8), clean.generate_greedy(tb, 41, 8))
