"""Batched decode (`cheetah_cuda_forward_batch`): one token for each of B
sequences in one pass over the weights, against the oracle run sequence by
sequence (`ModelForward::forward`, `qwen2.rs:600-606`)."""

import numpy as np
import pytest

import oracle as O
from cheetah_b200.prepared import PreparedModel, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.parametrize("step", ["gemv", "gemm"])
@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared"])
def test_batched_decode_matches_per_sequence_oracle(fixture, step, request, monkeypatch):
    """Five sequences: the small-batch weight-streaming GEMV step, and the
    tensor-core GEMM step (CHEETAH_CUDA_BATCH_GEMV=0)."""
    from cheetah_b200 import runtime as R
    monkeypatch.setenv("CHEETAH_CUDA_BATCH_GEMV", "1" if step == "gemv" else "0")
    root = request.getfixturevalue(fixture)
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    model = R.CudaModel(root, max_positions=2048)
    lengths = [5, 70, 1, 130, 64]
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, cfg["vocab_size"], n).astype(np.uint32) for n in lengths]
    seqs, refs, toks = [], [], []
    for prompt in prompts:
        seq = model.new_sequence()
        ref = O.OracleModel(pm, cfg)
        want = ref.forward(prompt, 0)
        got = seq.forward(prompt, 0)
        assert np.abs(got - want).max() < 2e-3
        seqs.append(seq)
        refs.append(ref)
        toks.append(int(np.argmax(want)))
    offsets = list(lengths)
    for step in range(6):
        am, logits = model.forward_batch(seqs, toks, offsets, want_logits=True)
        for b, ref in enumerate(refs):
            want = ref.forward([toks[b]], offsets[b])
            assert np.abs(logits[b] - want).max() < 2e-3, (step, b)
            mx = logits[b].max()
            assert am[b] == int(np.nonzero(logits[b] == mx)[0][-1])
            toks[b] = int(np.argmax(want))
            offsets[b] += 1
    assert [s.positions() for s in seqs] == offsets
    # The sequences keep working one at a time afterwards.
    want = refs[0].forward([toks[0]], offsets[0])
    assert np.abs(seqs[0].forward([toks[0]], offsets[0]) - want).max() < 2e-3


def test_batched_decode_argmax_only_and_errors(tiny_prepared):
    from cheetah_b200 import runtime as R
    model = R.CudaModel(tiny_prepared, max_positions=512)
    a, b = model.new_sequence(), model.new_sequence()
    a.forward([1, 2, 3], 0)
    b.forward([4], 0)
    am = model.forward_batch([a, b], [5, 6], [3, 1])
    assert am.shape == (2,) and a.positions() == 4 and b.positions() == 2
    with pytest.raises(R.CheetahCudaError, match="does not match"):
        model.forward_batch([a, b], [5, 6], [3, 1])
    with pytest.raises(R.CheetahCudaError, match="repeated"):
        model.forward_batch([a, a], [5, 6], [4, 4])
    other = R.CudaModel(tiny_prepared, max_positions=512)
    c = other.new_sequence()
    with pytest.raises(R.CheetahCudaError, match="another model"):
        model.forward_batch([a, c], [5, 6], [4, 0])


@pytest.mark.parametrize("lengths,steps", [([5, 70, 1, 130, 64], 300), ([17], 40),
                                           ([3, 9, 33, 2, 15, 16, 47, 8, 100], 20)])
def test_chained_greedy_batch_matches_step_by_step(tiny_prepared, lengths, steps):
    """`cheetah_cuda_forward_batch_greedy` against `steps` calls of
    forward_batch fed their own ids (identical tokens: same kernels, same
    inputs), crossing page boundaries and, at 300 steps, the host's token-log
    chunk; the KV written by the chained steps is then checked against the
    oracle run over prompt + generated ids."""
    from cheetah_b200 import runtime as R
    pm = PreparedModel(tiny_prepared)
    cfg = resolve_config(pm)
    model = R.CudaModel(tiny_prepared, max_positions=1024)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg["vocab_size"], n).astype(np.uint32) for n in lengths]
    chained, stepped, first = [], [], []
    for prompt in prompts:
        a, b = model.new_sequence(), model.new_sequence()
        la, lb = a.forward(prompt, 0), b.forward(prompt, 0)
        assert np.array_equal(la, lb)
        chained.append(a)
        stepped.append(b)
        first.append(int(np.argmax(la)))
    out = model.forward_batch_greedy(chained, first, lengths, steps)
    assert out.shape == (len(lengths), steps)
    toks, offs, want = list(first), list(lengths), []
    for _ in range(steps):
        am = model.forward_batch(stepped, toks, offs)
        want.append(am.copy())
        toks = [int(t) for t in am]
        offs = [o + 1 for o in offs]
    assert np.array_equal(out, np.stack(want, axis=1))
    assert [s.positions() for s in chained] == [n + steps for n in lengths]
    # The chained steps' K/V: the next token's logits against the oracle.
    for b in {0, len(lengths) - 1}:
        ids = np.concatenate([prompts[b], [first[b]], out[b, :-1]]).astype(np.uint32)
        ref = O.OracleModel(pm, cfg)
        ref.forward(ids, 0)
        w = ref.forward([int(out[b, -1])], len(ids))
        g = chained[b].forward([int(out[b, -1])], len(ids))
        assert np.abs(g - w).max() < 2e-3


def test_chained_greedy_batch_errors(tiny_prepared):
    from cheetah_b200 import runtime as R
    model = R.CudaModel(tiny_prepared, max_positions=64)
    a = model.new_sequence()
    a.forward([1, 2, 3], 0)
    with pytest.raises(R.CheetahCudaError, match="capacity"):
        model.forward_batch_greedy([a], [4], [3], 62)
    with pytest.raises(R.CheetahCudaError, match="positive"):
        model.forward_batch_greedy([a], [4], [3], 0)
    with pytest.raises(R.CheetahCudaError, match="does not match"):
        model.forward_batch_greedy([a], [4], [2], 4)
    assert a.positions() == 3
    out = model.forward_batch_greedy([a], [4], [3], 61)
    assert out.shape == (1, 61) and a.positions() == 64


def test_concurrent_clone_forwards_are_batched_and_match_oracle(tiny_prepared, monkeypatch):
    """The batcher behind `forward`: eight threads, each owning a clone (a
    sequence of the one model), decode concurrently through the plain
    single-sequence call. Calls that meet while a step runs go out together
    as batched steps; every thread's logits stay within tolerance of the
    oracle and of the same clones run serially with batching off."""
    import threading
    from cheetah_b200 import runtime as R
    from tests.greedy import check_greedy, reference_choice
    monkeypatch.setenv("CHEETAH_CUDA_COALESCE_MIN", "2")
    pm = PreparedModel(tiny_prepared)
    cfg = resolve_config(pm)
    model = R.CudaModel(tiny_prepared, max_positions=1024)
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, cfg["vocab_size"], n).astype(np.uint32) for n in (3, 40, 64, 65, 100, 7, 130, 20)]
    steps = 10

    def run(concurrent):
        monkeypatch.setenv("CHEETAH_CUDA_COALESCE", "1" if concurrent else "0")
        seqs = [model.new_sequence() for _ in prompts]
        firsts = [reference_choice(s.forward(p, 0)) for s, p in zip(seqs, prompts)]
        logs = [[] for _ in prompts]
        barrier = threading.Barrier(len(prompts)) if concurrent else None
        errors = []

        def worker(i):
            try:
                tok, pos = firsts[i], len(prompts[i])
                for _ in range(steps):
                    if barrier:
                        barrier.wait()
                    logits = np.empty(cfg["vocab_size"], np.float32)
                    am = seqs[i].forward_greedy([tok], pos, logits_out=logits)
                    logs[i].append((tok, pos, logits, am))
                    tok, pos = reference_choice(logits), pos + 1
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append(e)
                if barrier:
                    barrier.abort()

        if not concurrent:  # serial calls, one sequence after another
            for i in range(len(prompts)):
                worker(i)
        else:
            threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(prompts))]
            for t in threads:
                t.start()
            for t in threads:
                t.join(timeout=120)
        assert not errors, errors
        return logs

    before = model.coalesce_stats()
    together = run(True)
    stats = model.coalesce_stats()
    assert stats["calls"] - before["calls"] == len(prompts) * steps
    assert stats["batched_calls"] - before["batched_calls"] > len(prompts) * steps // 2, stats
    alone = run(False)
    for i, prompt in enumerate(prompts):
        ref = O.OracleModel(pm, cfg)
        ref.forward(prompt, 0)
        for (tok, pos, logits, am), (tok2, pos2, logits2, _) in zip(together[i], alone[i]):
            want = ref.forward([tok], pos)
            assert np.abs(logits - want).max() < 2e-3, (i, pos)
            check_greedy(am, want, 2e-3, f"sequence {i} position {pos}")
            if (tok2, pos2) == (tok, pos):
                assert np.abs(logits - logits2).max() < 2e-3, (i, pos)
            else:
                break  # a near-tie sent the serial run down another path
    model.close()


def test_batch_of_one_is_the_single_sequence_path(tiny_prepared):
    """A batched call with one sequence runs the single-sequence path: its
    greedy chain equals `generate_greedy` on a twin sequence token for
    token, and a one-row `forward_batch` equals `forward` bit for bit."""
    from cheetah_b200 import runtime as R
    from tests.greedy import reference_choice
    pm = PreparedModel(tiny_prepared)
    cfg = resolve_config(pm)
    model = R.CudaModel(tiny_prepared, max_positions=512)
    prompt = np.random.default_rng(8).integers(0, cfg["vocab_size"], 37).astype(np.uint32)
    a, b, c, d = (model.new_sequence() for _ in range(4))
    first = int(np.argmax(a.forward(prompt, 0)))
    for s in (b, c, d):
        s.forward(prompt, 0)
    chained = model.forward_batch_greedy([a], [first], [37], 24)
    alone = b.generate_greedy(first, 37, 24)
    assert np.array_equal(chained[0], alone)
    ids, logits = model.forward_batch([c], [first], [37], want_logits=True)
    ref = d.forward([first], 37)
    np.testing.assert_array_equal(logits[0], ref)
    assert int(ids[0]) == reference_choice(ref)
