"""bench.py's `prefill-attention-trace` post-processing (no GPU): the stamps
of a profiling build (-DCHEETAH_ATTN_TRACE) are read through the debug export
and summarised for the traced CTA (split 0 of query block 0, head 0, in the
last chunk of config 3)."""

from __future__ import annotations

from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture
def bench_module(monkeypatch):
    monkeypatch.syspath_prepend(str(ROOT))
    import bench
    return bench


class _TraceLib:
    """Stand-in for a trace build: tile j's event e at 1000 j + 50 e cycles."""

    def cheetah_cuda_debug_attn_trace(self, buf):
        for j in range(16):
            for e in range(16):
                buf[16 * j + e] = 1000 * j + 50 * e
        return 0

    def cheetah_cuda_last_error(self):
        return b""


class _PlainLib:
    def cheetah_cuda_last_error(self):
        return b""


class _R:
    def __init__(self, lib):
        self._lib = lib

    def lib(self):
        return self._lib


def test_trace_is_summarised_for_the_traced_cta(bench_module):
    cfg = {"q_heads": 14, "kv_heads": 2, "head_dim": 64}
    out = bench_module.attention_trace(_R(_TraceLib()), cfg, 148)
    # 2 query blocks x 14 heads = 28 blocks -> 5 splits; 46 key tiles -> 10 per split.
    assert out["key_tiles"] == 10
    assert "split 0 of 5" in out["launch"]
    assert len(out["events"]) == 10 and out["events"][3][2] == 3100
    m = out["median_cycles"]
    assert m["tile_pair"] == 1000
    assert m["A_max_pass"] == 50 and m["A_rescale"] == 50 and m["A_exp_pass"] == 50
    assert m["mma_issue_pv_a"] == 50 and m["mma_issue_s_b"] == 50 and m["mma_issue_pv_b"] == 50


def test_plain_build_is_refused_with_the_build_command(bench_module):
    with pytest.raises(SystemExit, match="CHEETAH_ATTN_TRACE"):
        bench_module.attention_trace(_R(_PlainLib()), {"q_heads": 14}, 148)
