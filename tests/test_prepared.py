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
