"""The prepared-model layout: the package's writer/reader against the
reference's own `cheetah init` (cheetah_init.c, compiled from the reference
sources into oracle/_ref by oracle/Makefile)."""

import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

from cheetah_b200.prepared import (ALIGNMENT, TINY, PreparedModel, resolve_config,
                                   tensor_specs, write_hf_source, write_prepared)

REF_SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libcheetah_init.so"


def _cheetah_init(src: Path, dst: Path) -> None:
    lib = C.CDLL(str(REF_SO))
    lib.cheetah_init_model.argtypes = [C.c_char_p, C.c_char_p]
    lib.cheetah_init_model.restype = C.c_int
    rc = lib.cheetah_init_model(str(src).encode(), str(dst).encode())
    assert rc == 0, "cheetah_init_model failed"


@pytest.fixture(scope="module")
def both_layouts(tmp_path_factory):
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libcheetah_init.so not built (reference tree absent)")
    base = tmp_path_factory.mktemp("layouts")
    write_hf_source(base / "hf", TINY, seed=0)
    _cheetah_init(base / "hf", base / "ref")
    write_prepared(base / "ours", TINY, seed=0)
    return PreparedModel(base / "ref"), PreparedModel(base / "ours")


def test_writer_matches_cheetah_init_units(both_layouts):
    ref, ours = both_layouts
    assert set(ref.units) == set(ours.units) == {n for n, _ in tensor_specs(TINY)}
    for uid, r in ref.units.items():
        o = ours.units[uid]
        assert (r.dtype, r.shape, r.nbytes, r.source_file, r.layer_id) == \
               (o.dtype, o.shape, o.nbytes, o.source_file, o.layer_id), uid
        np.testing.assert_array_equal(np.asarray(r.data), np.asarray(o.data))


def test_payloads_are_4096_aligned(both_layouts):
    for model in both_layouts:
        for unit in model.units.values():
            assert unit.source_offset % ALIGNMENT == 0
        weights = model.root / ".cheetah" / "weights"
        for shard in weights.iterdir():
            header_len = int.from_bytes(shard.read_bytes()[:8], "little")
            assert (8 + header_len) % ALIGNMENT == 0


def test_resolved_config_agrees(both_layouts):
    ref, ours = both_layouts
    a, b = resolve_config(ref), resolve_config(ours)
    assert a == b
    assert (a["hidden_size"], a["q_heads"], a["kv_heads"], a["head_dim"]) == (256, 14, 2, 64)
    assert a["sliding_window"] == 0 and a["tie_word_embeddings"] == 1


def test_reader_rejects_bad_manifests(tmp_path):
    (tmp_path / "cheetah_units.json").write_text("[]")
    with pytest.raises(ValueError, match="empty"):
        PreparedModel(tmp_path)
    (tmp_path / ".cheetah" / "weights").mkdir(parents=True)
    (tmp_path / ".cheetah" / "weights" / "global.safetensors").write_bytes(b"\x10" + b"\0" * 7 + b"{}")
    (tmp_path / "cheetah_units.json").write_text(json.dumps([{
        "unit_id": "x", "name": "x", "dtype": "BF16", "shape": [4], "bytes": 8,
        "source_file": "global.safetensors", "source_offset": 0, "shard": "s", "layer_id": 0}]))
    with pytest.raises(ValueError, match="header exceeds"):
        PreparedModel(tmp_path)


def _with_config(root: Path, **changes) -> PreparedModel:
    """The prepared directory at `root` with config.json fields replaced
    (None removes a field)."""
    cfg = json.loads((root / "config.json").read_text())
    for key, value in changes.items():
        if value is None:
            cfg.pop(key, None)
        else:
            cfg[key] = value
    (root / "config.json").write_text(json.dumps(cfg))
    return PreparedModel(root)


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-mistral", "tiny-qwen3"])
def test_family_configs_resolve_like_the_reference(tmp_path, name):
    """`decoder.rs:260-486` over each dense family's config: the written
    fields round-trip; absent fields fall back to the family constants
    (`llama.rs:66-82`, `mistral.rs:63-77`, `qwen3.rs:62-77`) and the
    manifest; `use_sliding_window` defaults to on (`decoder.rs:384-391`)."""
    from cheetah_b200.prepared import FAMILIES, SHAPES, write_prepared

    shape = SHAPES[name]
    root = write_prepared(tmp_path / "m", shape, seed=0)
    cfg = resolve_config(PreparedModel(root))
    assert (cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"]) == (shape.q_heads, shape.kv_heads, shape.head_dim)
    assert cfg["sliding_window"] == shape.sliding_window
    assert cfg["tie_word_embeddings"] == int(shape.tie_word_embeddings)
    fam = FAMILIES[shape.family]
    # Family constants when the config omits them; heads from the manifest.
    bare = resolve_config(_with_config(root, rope_theta=None, rms_norm_eps=None, tie_word_embeddings=None,
                                       num_key_value_heads=None, head_dim=None, intermediate_size=None))
    assert bare["rope_theta"] == fam["rope_theta"] and bare["rms_eps"] == pytest.approx(fam["rms_norm_eps"])
    assert bare["tie_word_embeddings"] == int(fam["tie_word_embeddings"])
    assert bare["head_dim"] == shape.q_dim // shape.q_heads
    assert bare["kv_heads"] == shape.kv_dim // bare["head_dim"]
    assert bare["intermediate_size"] == shape.intermediate_size
    # The window: on unless `use_sliding_window` is false.
    assert resolve_config(_with_config(root, sliding_window=4, use_sliding_window=None))["sliding_window"] == 4
    assert resolve_config(_with_config(root, sliding_window=4, use_sliding_window=True))["sliding_window"] == 4
    assert resolve_config(_with_config(root, sliding_window=4096, use_sliding_window=False))["sliding_window"] == 0
    # The family's context cap bounds max_position_embeddings (`engine.rs:1146-1162`).
    capped = resolve_config(_with_config(root, max_position_embeddings=10 ** 6))["max_positions"]
    assert capped == (fam["max_position_embeddings"] or 10 ** 6)


def test_architecture_selection_and_unserved_compositions(tmp_path):
    """The first `architectures` entry selects the family, else `model_type`
    (`chat/mod.rs:62-67`); no name at all resolves against the llama-shaped
    defaults (`decoder.rs:283-296`); other registered compositions are
    refused rather than resolved into a different model."""
    from cheetah_b200.prepared import DEFAULT_FAMILY, family_for, write_prepared

    assert family_for({"architectures": ["LlamaForCausalLM"], "model_type": "qwen2"})[0] == "llama"
    assert family_for({"model_type": "mistral"})[0] == "mistral"
    assert family_for({"architectures": [], "model_type": "qwen3"})[0] == "qwen3"
    assert family_for({}) == (None, DEFAULT_FAMILY)
    for arch in ("GemmaForCausalLM", "PhiForCausalLM", "MixtralForCausalLM"):
        with pytest.raises(ValueError, match="not served"):
            family_for({"architectures": [arch]})
    root = write_prepared(tmp_path / "m", TINY, seed=0)
    anon = resolve_config(_with_config(root, architectures=None, model_type=None, rope_theta=None,
                                       rms_norm_eps=None, tie_word_embeddings=None))
    assert (anon["rope_theta"], anon["tie_word_embeddings"]) == (1_000_000.0, 0)
    for field, value, match in (("num_local_experts", 8, "routed-expert"),
                                ("partial_rotary_factor", 0.5, "partial rotary"),
                                ("hidden_act", "gelu_pytorch_tanh", "GELU")):
        pm = _with_config(root, **{field: value})
        with pytest.raises(ValueError, match=match):
            resolve_config(pm)
        _with_config(root, **{field: None})
