"""Kernel parity on the GPU through the C-ABI op entries, against the CPU
oracle (the restatement of the reference math) on identical seeded inputs."""

import numpy as np
import pytest

import oracle as O
from cheetah_b200.prepared import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from cheetah_b200 import runtime
    runtime.lib()


def _gemv_case(rows, cols, batch, seed):
    from cheetah_b200 import runtime as R
    rng = np.random.default_rng(seed)
    wbits = f32_to_bf16_bits(rng.standard_normal(rows * cols, dtype=np.float32) * 0.02)
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    w_t = torch.from_numpy(wbits.view(np.int16).reshape(rows, cols)).view(torch.bfloat16).cuda()
    y = R.gemv_bf16(w_t, torch.from_numpy(x).cuda()).cpu().numpy()
    for b in range(batch):
        ref = O.gemv(wbits, rows, cols, x[b])
        scale = np.abs(bf16_bits_to_f32(wbits).reshape(rows, cols)) @ np.abs(x[b])
        err = np.abs(y[b] - ref)
        # f32 accumulation in a different order: a few ulps of sum |w||x|.
        assert np.all(err <= 1e-6 * scale + 1e-7), f"max err {err.max()}"


@pytest.mark.parametrize("kernel", ["bulk-prefetch", "register-stream"])
@pytest.mark.parametrize("rows,cols", [(1152, 896), (896, 896), (4864, 896), (896, 4864),
                                       (151936, 896), (3584, 3584), (18944, 3584), (3584, 18944),
                                       (1, 8), (3, 24), (257, 40)])
def test_gemv_bf16_matches_oracle(rows, cols, kernel, monkeypatch):
    monkeypatch.setenv("CHEETAH_CUDA_TMA_GEMV", "1" if kernel == "bulk-prefetch" else "0")
    _gemv_case(rows, cols, 1, rows + cols)


def test_gemv_bf16_batched():
    _gemv_case(1000, 896, 3, 7)


def test_gemv_rejects_bad_shapes():
    from cheetah_b200 import runtime as R
    w = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(R.CheetahCudaError, match="multiple of 8"):
        R.gemv_bf16(w, torch.zeros(1, 12, device="cuda"))


def make_paged_kv(B, L_list, kv_heads, D, page_tokens, kv_dtype, seed, extra_pages=3):
    """Random N(0,1) K/V in a shuffled paged pool + the dense f32 view the
    oracle reads ([L, kv_heads*D] per sequence)."""
    rng = np.random.default_rng(seed)
    pages_per = [(L + page_tokens - 1) // page_tokens for L in L_list]
    total = sum(pages_per) + extra_pages
    order = rng.permutation(total)
    max_pages = max(pages_per)
    table = np.full((B, max_pages), -1, np.int32)
    k_pool = np.zeros((total, kv_heads, page_tokens, D), np.float32)
    v_pool = np.zeros_like(k_pool)
    dense = []
    cursor = 0
    for b, L in enumerate(L_list):
        k = rng.standard_normal((L, kv_heads, D), dtype=np.float32)
        v = rng.standard_normal((L, kv_heads, D), dtype=np.float32)
        if kv_dtype == "bf16":
            k = bf16_bits_to_f32(f32_to_bf16_bits(k)).reshape(k.shape)
            v = bf16_bits_to_f32(f32_to_bf16_bits(v)).reshape(v.shape)
        for p in range(pages_per[b]):
            page = order[cursor]
            cursor += 1
            table[b, p] = page
            lo, hi = p * page_tokens, min(L, (p + 1) * page_tokens)
            k_pool[page, :, : hi - lo] = k[lo:hi].transpose(1, 0, 2)
            v_pool[page, :, : hi - lo] = v[lo:hi].transpose(1, 0, 2)
        dense.append((k.reshape(L, -1), v.reshape(L, -1)))
    tdt = torch.bfloat16 if kv_dtype == "bf16" else torch.float32
    kt = torch.from_numpy(k_pool).to(tdt).cuda()
    vt = torch.from_numpy(v_pool).to(tdt).cuda()
    return kt, vt, torch.from_numpy(table).cuda(), dense


# Tolerances: the CUDA-core kernel (f32 cache, or bf16 cache with the MMA
# path switched off) computes in f32 — 1e-4; the tensor-core kernel rounds q
# and the softmax weights to bf16 for the MMAs — the 1e-2 max-abs contract.
@pytest.mark.parametrize("q_heads,kv_heads,D", [(14, 2, 64), (28, 4, 128)])
@pytest.mark.parametrize("kernel", ["mma", "cuda-core-bf16", "cuda-core-f32"])
@pytest.mark.parametrize("L_list", [[1], [17], [64], [1000, 3], [4097, 65, 640]])
def test_decode_attention_matches_oracle(q_heads, kv_heads, D, kernel, L_list, monkeypatch):
    from cheetah_b200 import runtime as R
    kv_dtype = "f32" if kernel == "cuda-core-f32" else "bf16"
    if kernel == "cuda-core-bf16":
        monkeypatch.setenv("CHEETAH_CUDA_MMA_ATTENTION", "0")
    tol = 1e-2 if kernel == "mma" else 1e-4
    B = len(L_list)
    kt, vt, table, dense = make_paged_kv(B, L_list, kv_heads, D, 64, kv_dtype, seed=sum(L_list) + D)
    rng = np.random.default_rng(11)
    q = rng.standard_normal((B, q_heads, D), dtype=np.float32)
    lens = torch.tensor(L_list, dtype=torch.int32, device="cuda")
    out = R.decode_attention(torch.from_numpy(q).cuda(), kt, vt, table, lens, max(L_list)).cpu().numpy()
    for b in range(B):
        ref = O.attention(dense[b][0], dense[b][1], q[b].reshape(-1), q_heads, kv_heads, D)
        err = np.abs(out[b].reshape(-1) - ref).max()
        assert err < tol, f"b={b} max err {err}"


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_decode_attention_sliding_window(kv_dtype):
    from cheetah_b200 import runtime as R
    L, window = 700, 100
    kt, vt, table, dense = make_paged_kv(1, [L], 2, 64, 64, kv_dtype, seed=3)
    q = np.random.default_rng(4).standard_normal((1, 14, 64), dtype=np.float32)
    lens = torch.tensor([L], dtype=torch.int32, device="cuda")
    out = R.decode_attention(torch.from_numpy(q).cuda(), kt, vt, table, lens, L,
                             sliding_window=window).cpu().numpy()
    ref = O.attention(dense[0][0], dense[0][1], q[0].reshape(-1), 14, 2, 64, position=L - 1,
                      sliding_window=window)
    assert np.abs(out[0].reshape(-1) - ref).max() < (1e-4 if kv_dtype == "f32" else 1e-2)


def test_decode_attention_full_size_sampled():
    """Config-2 scale (B=8, L=32k, 14/2/64): full comparison on two sequences."""
    from cheetah_b200 import runtime as R
    B, L = 8, 32768
    kt, vt, table, dense = make_paged_kv(B, [L] * B, 2, 64, 64, "bf16", seed=5, extra_pages=0)
    q = np.random.default_rng(6).standard_normal((B, 14, 64), dtype=np.float32)
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = R.decode_attention(torch.from_numpy(q).cuda(), kt, vt, table, lens, L).cpu().numpy()
    for b in (0, B - 1):
        ref = O.attention(dense[b][0], dense[b][1], q[b].reshape(-1), 14, 2, 64)
        assert np.abs(out[b].reshape(-1) - ref).max() < 1e-2
    # Linearity property over the whole batch: a repeated call is identical.
    again = R.decode_attention(torch.from_numpy(q).cuda(), kt, vt, table, lens, L).cpu().numpy()
    np.testing.assert_array_equal(out, again)


# Prefill attention through its C-ABI op entry: query rows offset ..
# offset+T-1 each against the oracle's `attention` at that row's position
# (`ops.rs:1357-1421`; the chunk's own rows are already in the cache, as the
# per-row append-then-attend loop of `qwen2.rs:314-343` leaves them). q is
# bf16 (the GEMM epilogue's output), so the oracle reads the same rounded q.
@pytest.mark.parametrize("q_heads,kv_heads,D", [(14, 2, 64), (28, 4, 128), (8, 8, 64)])
@pytest.mark.parametrize("offset,T,window", [(0, 1, 0), (0, 130, 0), (700, 257, 0), (2048, 64, 0),
                                             (1024, 64, 0), (300, 200, 96), (5000, 77, 4096)])
def test_prefill_attention_op_matches_oracle(q_heads, kv_heads, D, offset, T, window):
    from cheetah_b200 import runtime as R
    from cheetah_b200.prepared import bf16_bits_to_f32, f32_to_bf16_bits
    L = offset + T
    kt, vt, table, dense = make_paged_kv(1, [L], kv_heads, D, 64, "bf16", seed=offset + T + D)
    rng = np.random.default_rng(7 + T)
    q = bf16_bits_to_f32(f32_to_bf16_bits(rng.standard_normal((T, q_heads, D), dtype=np.float32)))
    q = q.reshape(T, q_heads, D)
    qt = torch.from_numpy(q).to(torch.bfloat16).cuda()
    out = R.prefill_attention(qt, kt, vt, table[0].contiguous(), offset, sliding_window=window)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    k, v = dense[0]
    rows = sorted(set([0, T - 1] + list(np.random.default_rng(T).integers(0, T, 12))))
    for r in rows:
        pos = offset + r
        want = O.attention(k[:pos + 1], v[:pos + 1], q[r].reshape(-1), q_heads, kv_heads, D,
                           position=pos, sliding_window=window)
        err = np.abs(got[r].reshape(-1) - want).max()
        assert err < 1e-2, f"row {r} (position {pos}): max err {err}"
