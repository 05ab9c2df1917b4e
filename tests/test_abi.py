"""C-ABI library checks that need no GPU: it loads, exports every symbol the
header declares, and fails cleanly (status + message, no crash) when asked
for work it cannot do."""

import re
from pathlib import Path

import pytest

from cheetah_b200 import runtime as R

HEADER = Path(__file__).resolve().parent.parent / "include" / "cheetah_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"CHEETAH_CUDA_API\s+[\w\s\*]*?\b(cheetah_cuda_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "cheetah_cuda_forward" in names and "cheetah_cuda_op_decode_attention" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    lib = R.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_ctypes_signatures_cover_the_header():
    assert set(declared_symbols()) == set(R.SIGNATURES)


def test_abi_version():
    assert R.lib().cheetah_cuda_abi_version() == 2


def test_device_count_never_fails():
    assert R.device_count() >= 0


def test_open_reports_errors_without_crashing(tmp_path, tiny_prepared):
    if R.device_count() == 0:
        with pytest.raises(R.CheetahCudaError):
            R.CudaModel(tiny_prepared)
    with pytest.raises(R.CheetahCudaError):
        R.CudaModel(tmp_path, config={"hidden_size": 64, "num_layers": 1, "q_heads": 2, "kv_heads": 1,
                                      "head_dim": 64, "rotary_dim": 64, "intermediate_size": 64,
                                      "vocab_size": 10, "rms_eps": 1e-6, "rope_theta": 1e4,
                                      "tie_word_embeddings": 1, "sliding_window": 0,
                                      "max_positions": 16})


def test_null_arguments_are_rejected():
    lib = R.lib()
    assert lib.cheetah_cuda_forward(None, None, 0, 0, None) != 0
    assert b"null" in lib.cheetah_cuda_last_error() or b"empty" in lib.cheetah_cuda_last_error()
    assert lib.cheetah_cuda_model_info(None, None) != 0
    assert lib.cheetah_cuda_op_decode_attention(None, None) != 0
