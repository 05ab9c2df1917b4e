"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def tiny_prepared(tmp_path_factory):
    """Seeded synthetic Qwen2 model with the 0.5B head geometry (14q/2kv/64)
    at a size the CPU oracle runs in milliseconds."""
    from cheetah_b200.prepared import TINY, write_prepared

    root = tmp_path_factory.mktemp("tiny_qwen2")
    write_prepared(root, TINY, seed=0)
    return root


@pytest.fixture(scope="session")
def tiny7b_prepared(tmp_path_factory):
    """Seeded synthetic model with the 7B head geometry (28q/4kv/128), untied."""
    from cheetah_b200.prepared import TINY_7B_HEADS, write_prepared

    root = tmp_path_factory.mktemp("tiny_qwen2_7bheads")
    write_prepared(root, TINY_7B_HEADS, seed=0)
    return root


@pytest.fixture(scope="session")
def tiny15b_prepared(tmp_path_factory):
    """Seeded synthetic model with the 1.5B width and head geometry
    (hidden 1536, 12q/2kv/128), untied, two layers."""
    from cheetah_b200.prepared import TINY_15B_HEADS, write_prepared

    root = tmp_path_factory.mktemp("tiny_qwen2_15bheads")
    write_prepared(root, TINY_15B_HEADS, seed=0)
    return root


@pytest.fixture(scope="session")
def tinywide_prepared(tmp_path_factory):
    """Seeded synthetic model with the 0.5B head geometry and a 16384-wide
    MLP: long down_proj rows (many steps per warp in the quantised GEMV)."""
    from cheetah_b200.prepared import TINY_WIDE_MLP, write_prepared

    root = tmp_path_factory.mktemp("tiny_qwen2_widemlp")
    write_prepared(root, TINY_WIDE_MLP, seed=0)
    return root


FAMILY_SHAPES = ("tiny-llama", "tiny-mistral", "tiny-qwen3")


@pytest.fixture(scope="session", params=FAMILY_SHAPES)
def family_prepared(request, tmp_path_factory):
    """Seeded synthetic models of the other dense families: llama (no
    biases, multi-head), mistral (sliding window 48) and qwen3 (per-head q/k
    norms, head_dim 128)."""
    from cheetah_b200.prepared import SHAPES, write_prepared

    root = tmp_path_factory.mktemp(request.param.replace("-", "_"))
    write_prepared(root, SHAPES[request.param], seed=0)
    return root
