"""Ant VRAM tier on the GPU: a model opened with a residency plan
(`cheetah_cuda_model_open_ex`) streams its non-VRAM layer linears from
pinned host memory and must compute exactly what the HBM-resident model
computes (same kernels, same operands); units move between HBM and the host
at run time through `page_in_unit` / `evict_unit` (`AntTierControl`,
`registry.rs:88-93`) without changing results."""

import os

import numpy as np
import pytest

import oracle as O
from cheetah_b200.ant import plan_residency, units_of
from cheetah_b200.prepared import PreparedModel, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _plain(root, quant):
    """The HBM-resident model on the multi-kernel path (the path a planned
    model runs), for exact comparison."""
    from cheetah_b200 import runtime as R
    old = os.environ.get("CHEETAH_CUDA_MEGAKERNEL")
    os.environ["CHEETAH_CUDA_MEGAKERNEL"] = "0"
    try:
        return R.CudaModel(root, quant=quant, max_positions=1024)
    finally:
        if old is None:
            del os.environ["CHEETAH_CUDA_MEGAKERNEL"]
        else:
            os.environ["CHEETAH_CUDA_MEGAKERNEL"] = old


def _run(model, prompt, steps):
    """Prefill, `steps` greedy single-token forwards, then a device greedy
    chain and a batched step of two fresh sequences."""
    seq = model.new_sequence()
    out = [seq.forward(prompt, 0)]
    tok = int(np.argmax(out[0]))
    pos = len(prompt)
    for _ in range(steps):
        logits = np.empty_like(out[0])
        tok = seq.forward_greedy([tok], pos, logits_out=logits)
        out.append(logits)
        pos += 1
    chain = seq.generate_greedy(tok, pos, 6)
    if model.quant != "bf16":  # batched steps need bf16 weights
        return out, chain, None, None
    a, b = model.new_sequence(), model.new_sequence()
    a.forward(prompt[:9], 0)
    b.forward(prompt[:17], 0)
    ids, batch_logits = model.forward_batch([a, b], [int(prompt[9]), int(prompt[17])], [9, 17], want_logits=True)
    return out, chain, ids, batch_logits


@pytest.mark.parametrize("quant", ["bf16", "q8"])
def test_streamed_layers_match_the_resident_model(tiny_prepared, quant):
    from cheetah_b200 import runtime as R
    pm = PreparedModel(tiny_prepared)
    cfg = resolve_config(pm)
    units = units_of(pm)
    # VRAM pool = the layer-0 units: layer 1's linears are planned into RAM.
    pool = sum(u.bytes for u in units if u.layer_id == 0)
    plan = plan_residency(units, vram_pool_bytes=pool, ram_budget_bytes=1 << 40)
    assert plan["model.layers.1.mlp.gate_proj.weight"] == "ram"
    planned = R.CudaModel(tiny_prepared, quant=quant, max_positions=1024, residency=plan)
    res = planned.residency()
    assert res["planned"] == 1 and res["streamed_linears"] == 5 and res["resident_linears"] == 5
    assert res["streamed_linear_bytes"] > 0 and res["staging_bytes"] > 0
    plain = _plain(tiny_prepared, quant)
    assert planned.info()["weight_bytes"] < plain.info()["weight_bytes"]
    prompt = np.random.default_rng(11).integers(0, cfg["vocab_size"], 30).astype(np.uint32)
    got = _run(planned, prompt, 6)
    want = _run(plain, prompt, 6)
    for g, w in zip(got[0], want[0]):
        np.testing.assert_array_equal(g, w)
    np.testing.assert_array_equal(got[1], want[1])
    if quant == "bf16":
        np.testing.assert_array_equal(got[2], want[2])
        np.testing.assert_array_equal(got[3], want[3])
    # And the oracle agrees with both (bf16 KV tolerance).
    ref = O.OracleModel(pm, cfg, quant)
    assert np.abs(got[0][0] - ref.forward(prompt, 0)).max() < 2e-3


def test_page_in_and_evict_at_run_time(tiny_prepared):
    from cheetah_b200 import runtime as R
    pm = PreparedModel(tiny_prepared)
    cfg = resolve_config(pm)
    planned = R.CudaModel(tiny_prepared, max_positions=1024, residency={})  # planned, all in HBM
    plain = _plain(tiny_prepared, "bf16")
    full = planned.residency()
    assert full["streamed_linears"] == 0 and full["resident_linears"] == 10
    prompt = np.random.default_rng(12).integers(0, cfg["vocab_size"], 20).astype(np.uint32)
    s1, s2 = planned.new_sequence(), plain.new_sequence()
    np.testing.assert_array_equal(s1.forward(prompt, 0), s2.forward(prompt, 0))
    pos, tok = len(prompt), int(prompt[-1])

    def step():
        nonlocal pos, tok
        l1, l2 = np.empty(cfg["vocab_size"], np.float32), np.empty(cfg["vocab_size"], np.float32)
        a1 = s1.forward_greedy([tok], pos, logits_out=l1)
        a2 = s2.forward_greedy([tok], pos, logits_out=l2)
        np.testing.assert_array_equal(l1, l2)
        assert a1 == a2
        tok, pos = a1, pos + 1

    step()
    # Evicting one unit of the fused q/k/v linear streams the whole linear.
    assert planned.evict_unit("model.layers.0.self_attn.k_proj.weight")
    assert planned.evict_unit("model.layers.1.mlp.down_proj.weight")
    mid = planned.residency()
    assert mid["streamed_linears"] == 2 and mid["resident_linear_bytes"] < full["resident_linear_bytes"]
    step()
    step()
    # Paging q (already resident) changes nothing; paging k back restores the linear.
    assert planned.page_in_unit("model.layers.0.self_attn.q_proj.weight", 0)
    assert planned.residency()["streamed_linears"] == 2
    assert planned.page_in_unit("model.layers.0.self_attn.k_proj.weight", 0)
    assert planned.page_in_unit("model.layers.1.mlp.down_proj.weight", 0)
    assert planned.residency() == full
    step()
    # A host tier moves the unit out of HBM like an eviction.
    assert planned.page_in_unit("model.layers.1.mlp.up_proj.weight", 1)
    assert planned.residency()["streamed_linears"] == 1
    step()
    # Unknown units report False; units that always stay resident report True.
    assert not planned.evict_unit("model.layers.9.mlp.up_proj.weight")
    assert planned.evict_unit("model.norm.weight")
    assert planned.residency()["streamed_linears"] == 1
    step()


def test_residency_needs_a_plan(tiny_prepared):
    from cheetah_b200 import runtime as R
    model = R.CudaModel(tiny_prepared, max_positions=256)
    assert model.residency()["planned"] == 0
    with pytest.raises(R.CheetahCudaError, match="residency plan"):
        model.evict_unit("model.layers.0.mlp.up_proj.weight")
    with pytest.raises(R.CheetahCudaError, match="unknown Ant tier"):
        R.CudaModel(tiny_prepared, max_positions=256, residency={"model.layers.0.mlp.up_proj.weight": "hbm"})


def test_real_05b_shape_half_streamed_decodes_like_the_resident_model():
    """The 0.5B shape planned into a VRAM pool of half its bytes (17 layers
    partly streamed): prefill and 16 greedy steps give the resident model's
    logits bit for bit (same kernels, operands copied from host memory)."""
    from cheetah_b200 import runtime as R
    from cheetah_b200.ant import layer_residency_summary
    from cheetah_b200.prepared import cached_synthetic
    root = cached_synthetic("qwen2-0.5b")
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    units = units_of(pm)
    plan = plan_residency(units, vram_pool_bytes=sum(u.bytes for u in units) // 2, ram_budget_bytes=1 << 40)
    states = [e.state() for e in layer_residency_summary(units, plan)]
    assert "partial" in states and "full_vram" in states
    planned = R.CudaModel(root, max_positions=1024, residency=plan)
    assert planned.residency()["streamed_linears"] > 0
    plain = _plain(root, "bf16")
    prompt = np.random.default_rng(21).integers(0, cfg["vocab_size"], 200).astype(np.uint32)
    a, b = planned.new_sequence(), plain.new_sequence()
    la, lb = a.forward(prompt, 0), b.forward(prompt, 0)
    np.testing.assert_array_equal(la, lb)
    tok, pos = int(np.argmax(la)), len(prompt)
    for _ in range(16):
        ga, gb = np.empty_like(la), np.empty_like(lb)
        ta = a.forward_greedy([tok], pos, logits_out=ga)
        tb = b.forward_greedy([tok], pos, logits_out=gb)
        np.testing.assert_array_equal(ga, gb)
        assert ta == tb
        tok, pos = ta, pos + 1
