"""The allocation-free decode-attention entry point.

Some callers cannot let the library allocate device memory: a host that
keeps a fixed device-memory budget of its own and hands the library only its
inputs and outputs, or a latency-critical serving path that cannot absorb the
device-wide synchronisation cudaMalloc / cudaFree can cause.
`cheetah_cuda_op_decode_attention_noalloc` serves them: its split-merge
scratch is a fixed array compiled into the library instead of memory
allocated on first use.

Checked here through the C-ABI: two calls in a row agree with the allocating
entry point (`cheetah_cuda_op_decode_attention`) to 1e-4, on the tensor-core
path (bf16 cache) and the CUDA-core path (f32 cache); at the array's limit
(batch x kv_heads = 1024, where the entry point reduces the key splits to fit)
two calls in a row agree with the allocating entry point to the 1e-2 contract
tolerance and with the CPU oracle; a request beyond the fixed capacity is
refused with an error. This file sorts last so a run that stops at its first
failure has already run every other test.
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


def test_noalloc_at_its_limit_reduces_splits_and_matches_oracle():
    """256 sequences x 4 KV heads = 1024 pairs: the split count drops to one
    key range per pair, where the allocating entry point splits further, so
    the two differ only by summation order (1e-2 contract tolerance)."""
    import oracle as O
    from cheetah_b200 import runtime as R
    B, q_heads, kv_heads, D = 256, 28, 4, 128
    rng = np.random.default_rng(41)
    lengths = rng.integers(1, 1500, B).tolist()
    lengths[0], lengths[1] = 1, 1499
    k, v, table, lens = _paged(B, lengths, kv_heads, D, torch.bfloat16, seed=42)
    q = torch.randn(B, q_heads, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(43))
    want = R.decode_attention(q, k, v, table, lens, max(lengths))
    for _ in range(2):
        got = R.decode_attention(q, k, v, table, lens, max(lengths), noalloc=True)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() < 1e-2
    kc, vc, tab, qc, out = k.float().cpu().numpy(), v.float().cpu().numpy(), table.cpu().numpy(), \
        q.cpu().numpy(), got.cpu().numpy()
    for b in (0, 1, 2, 100, B - 1):
        L = lengths[b]
        pages = tab[b, : (L + 63) // 64]
        kd = kc[pages].transpose(0, 2, 1, 3).reshape(-1, kv_heads * D)[:L]
        vd = vc[pages].transpose(0, 2, 1, 3).reshape(-1, kv_heads * D)[:L]
        ref = O.attention(np.ascontiguousarray(kd), np.ascontiguousarray(vd), qc[b].reshape(-1),
                          q_heads, kv_heads, D)
        assert np.abs(out[b].reshape(-1) - ref).max() < 1e-2, f"sequence {b}"


def test_noalloc_rejects_requests_beyond_its_capacity():
    from cheetah_b200 import runtime as R
    B, kv_heads = 600, 2  # 1200 (sequence, kv head) pairs > 1024
    k, v, table, lens = _paged(1, [64], kv_heads, 64, torch.bfloat16, seed=1)
    table = table.expand(B, -1).contiguous()
    lens = lens.expand(B).contiguous()
    q = torch.randn(B, 14, 64, device="cuda")
    with pytest.raises(R.CheetahCudaError, match="fixed scratch limit"):
        R.decode_attention(q, k, v, table, lens, 64, noalloc=True)
