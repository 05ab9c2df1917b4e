"""The allocation-free decode-attention entry point.

Some callers cannot let the library allocate device memory: code that records
its work into a CUDA graph (allocating is not allowed while a stream is being
captured), a host that keeps a fixed device-memory budget of its own, or a
latency-critical serving path that cannot absorb the synchronisation
cudaMalloc / cudaFree can cause. `cheetah_cuda_op_decode_attention_noalloc`
serves them: its split-merge scratch is a fixed array compiled into the
library instead of memory allocated on first use.

Checked here through the C-ABI: two calls in a row agree with the allocating
entry point (`cheetah_cuda_op_decode_attention`) to 1e-4, on the tensor-core
path (bf16 cache) and the CUDA-core path (f32 cache); a request beyond the
fixed capacity is refused with an error. This file sorts last so a run that
stops at its first failure has already run every other test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _paged(B, lengths, kv_heads, D, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    page = 64
    per = [(L + page - 1) // page for L in lengths]
    total = sum(per) + 2
    k = torch.randn(total, kv_heads, page, D, device="cuda", generator=g).to(dtype)
    v = torch.randn(total, kv_heads, page, D, device="cuda", generator=g).to(dtype)
    perm = torch.randperm(total, device="cuda", generator=g).to(torch.int32)
    table = torch.full((B, max(per)), -1, dtype=torch.int32, device="cuda")
    cursor = 0
    for b, n in enumerate(per):
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    return k, v, table, lens


@pytest.mark.parametrize("q_heads,kv_heads,D,dtype,lengths", [
    (14, 2, 64, torch.bfloat16, [1000, 3, 640]),      # tensor-core kernel
    (28, 4, 128, torch.bfloat16, [4097, 77]),         # tensor-core kernel, d=128
    (28, 4, 128, torch.float32, [2000, 129]),         # CUDA-core kernel
])
def test_noalloc_matches_allocating_entry_twice(q_heads, kv_heads, D, dtype, lengths):
    from cheetah_b200 import runtime as R
    B = len(lengths)
    k, v, table, lens = _paged(B, lengths, kv_heads, D, dtype, seed=sum(lengths))
    q = torch.randn(B, q_heads, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
    want = R.decode_attention(q, k, v, table, lens, max(lengths))
    for _ in range(2):  # the array keeps the previous call's contents
        got = R.decode_attention(q, k, v, table, lens, max(lengths), noalloc=True)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() < 1e-4


def test_noalloc_rejects_requests_beyond_its_capacity():
    from cheetah_b200 import runtime as R
    B, kv_heads = 600, 2  # 1200 (sequence, kv head) pairs > 1024
    k, v, table, lens = _paged(1, [64], kv_heads, 64, torch.bfloat16, seed=1)
    table = table.expand(B, -1).contiguous()
    lens = lens.expand(B).contiguous()
    q = torch.randn(B, 14, 64, device="cuda")
    with pytest.raises(R.CheetahCudaError, match="fixed scratch limit"):
        R.decode_attention(q, k, v, table, lens, 64, noalloc=True)
