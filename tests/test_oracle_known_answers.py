"""Pins the CPU oracle against the reference's own known-answer unit tests.

Each test restates one `#[test]` of the reference (file:line given) with the
same inputs, the same expected values and the same tolerance.
"""

import math

import numpy as np
import pytest

import oracle as O
from cheetah_b200.prepared import f32_to_bf16_bits


def bf16_trunc(values):
    """The reference tests build bf16 by truncation: `(value.to_bits() >> 16) as u16`."""
    return (np.asarray(values, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_bf16_widening_matches_bit_shift():  # ops.rs:1694
    from cheetah_b200.prepared import bf16_bits_to_f32
    assert bf16_bits_to_f32(np.array([0x3F80], np.uint16))[0] == 1.0
    assert bf16_bits_to_f32(np.array([0xC000], np.uint16))[0] == -2.0
    assert bf16_bits_to_f32(np.array([0x0000], np.uint16))[0] == 0.0


def test_gemv_multiplies_rows_in_parallel():  # ops.rs:1702
    w = np.array([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], np.float32)
    x = np.array([1.0, 0.0, -1.0], np.float32)
    assert O.gemv(w.view(np.uint8), 2, 3, x, dtype=O.F32).tolist() == [-2.0, -2.0]
    assert O.gemv(bf16_trunc(w), 2, 3, x, dtype=O.BF16).tolist() == [-2.0, -2.0]


def test_gemm_matches_per_row_gemv_bit_exact():  # ops.rs:1727
    rows, cols, n = 128 * 2 + 3, 8, 7
    weight = np.array([((i * 37 % 23) - 11.0) / 8.0 for i in range(rows * cols)], np.float32)
    x = np.array([((i * 11 % 17) - 8.0) / 4.0 for i in range(n * cols)], np.float32)
    wb = bf16_trunc(weight)
    y = O.gemm(wb, rows, cols, x)
    for t in range(n):
        np.testing.assert_array_equal(y[t], O.gemv(wb, rows, cols, x[t * cols:(t + 1) * cols]))
    y32 = O.gemm(weight.view(np.uint8), rows, cols, x, dtype=O.F32)
    for t in range(n):
        np.testing.assert_array_equal(
            y32[t], O.gemv(weight.view(np.uint8), rows, cols, x[t * cols:(t + 1) * cols], dtype=O.F32))


@pytest.mark.parametrize("cols", [896, 903, 4864])
def test_gemm_matches_gemv_bit_exact_at_model_widths(cols):
    rng = np.random.default_rng(5)
    rows, n = 300, 9
    wb = f32_to_bf16_bits(rng.standard_normal(rows * cols, dtype=np.float32))
    x = rng.standard_normal((n, cols), dtype=np.float32)
    y = O.gemm(wb, rows, cols, x)
    for t in range(n):
        np.testing.assert_array_equal(y[t], O.gemv(wb, rows, cols, x[t]))


def _q8_reference(weights, x):
    """ops.rs:1801 builds the buffer and the expected sums by hand."""
    rows, cols = len(weights), len(weights[0])
    row_bytes = (cols + 3) // 4 * 4
    buffer = np.zeros(rows * 4 + rows * row_bytes, np.uint8)
    expected = np.zeros(rows, np.float32)
    for r, row in enumerate(weights):
        max_abs = np.float32(max(abs(np.float32(v)) for v in row))
        scale = np.float32(max_abs / np.float32(127.0)) if max_abs > 0 else np.float32(1.0)
        buffer[r * 4:r * 4 + 4] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
        s = np.float32(0.0)
        for c, v in enumerate(row):
            q = np.float32(np.float32(v) / scale)
            code = int(np.clip(math.copysign(math.floor(abs(q) + 0.5), q), -127, 127))
            buffer[rows * 4 + r * row_bytes + c] = code & 0xFF
            s = np.float32(s + np.float32(np.float32(scale * np.float32(code)) * x[c]))
        expected[r] = s
    return buffer, expected


def test_gemv_q8_matches_rowwise_scale_code_reference():  # ops.rs:1801
    cols = 6
    x = np.array([0.5 - i * 0.1 for i in range(cols)], np.float32)
    weights = [[1.0, -2.0, 0.0, 3.5, -0.25, 2.0], [0.0] * 6, [-7.0, 7.0, -1.0, 1.0, -0.5, 0.5]]
    buffer, expected = _q8_reference(weights, x)
    y = O.gemv_q8(buffer, 3, cols, x)
    assert np.all(np.abs(y - expected) < 1e-5)
    # The oracle's quantiser writes the same buffer the test packs by hand.
    np.testing.assert_array_equal(O.quantize_q8(np.array(weights, np.float32), 3, cols), buffer)


def test_gemv_q4_matches_rowwise_scale_code_reference():  # ops.rs:1838
    cols = 9
    rows = 3
    x = np.array([0.5 - i * 0.1 for i in range(cols)], np.float32)
    weights = [[1.0, -2.0, 0.0, 3.5, -0.25, 2.0, -1.5, 0.75, 4.0], [0.0] * 9,
               [-7.0, 7.0, -1.0, 1.0, -0.5, 0.5, -3.0, 3.0, 0.0]]
    row_bytes = O.q4_row_bytes(cols)
    assert row_bytes == ((cols + 1 + 1) // 2 + 3) // 4 * 4
    buffer = np.zeros(rows * 4 + rows * row_bytes, np.uint8)
    expected = np.zeros(rows, np.float32)
    for r, row in enumerate(weights):
        max_abs = np.float32(max(abs(v) for v in row))
        scale = np.float32(max_abs / np.float32(7.0)) if max_abs > 0 else np.float32(1.0)
        buffer[r * 4:r * 4 + 4] = np.frombuffer(scale.tobytes(), np.uint8)
        s = np.float32(0.0)
        for c, v in enumerate(row):
            q = np.float32(np.float32(v) / scale)
            code = int(np.clip(math.copysign(math.floor(abs(q) + 0.5), q), -7, 7))
            buffer[rows * 4 + r * row_bytes + c // 2] |= ((code & 0x0F) << ((c % 2) * 4))
            s = np.float32(s + np.float32(np.float32(scale * np.float32(code)) * x[c]))
        expected[r] = s
    y = O.gemv_q4(buffer, rows, cols, x)
    assert np.all(np.abs(y - expected) < 1e-5)
    np.testing.assert_array_equal(O.quantize_q4(np.array(weights, np.float32), rows, cols), buffer)


@pytest.mark.parametrize("fmt", ["q4", "q8"])
def test_gemv_consumes_the_registered_quantize_output(fmt):  # ops.rs:1876, :1907
    rows, cols = 5, 9
    values = np.array([((i % 23) - 11.0) * 0.3 for i in range(rows * cols)], np.float32)
    quant = O.quantize_q4 if fmt == "q4" else O.quantize_q8
    gemv = O.gemv_q4 if fmt == "q4" else O.gemv_q8
    dq = O.q4_dequant if fmt == "q4" else O.q8_dequant
    buffer = quant(values, rows, cols)
    x = np.array([math.sin(i * 0.7 - 2.0) for i in range(cols)], np.float32)
    y = gemv(buffer, rows, cols, x)
    for r in range(rows):
        want = sum(dq(buffer, rows, cols, r, c) * float(x[c]) for c in range(cols))
        assert abs(y[r] - want) < 1e-4


def test_rmsnorm_matches_reference_computation():  # ops.rs:1935
    w = np.repeat(bf16_trunc(np.array([1.0], np.float32)), 2)
    y = O.rmsnorm(np.array([3.0, 4.0], np.float32), w, 1e-6)
    expected = 1.0 / np.sqrt(np.float32(12.5) + np.float32(1e-6))
    assert abs(y[0] - 3.0 * expected) < 1e-5 and abs(y[1] - 4.0 * expected) < 1e-5


def test_rope_preserves_magnitude_and_matches_reference():  # ops.rs:1947
    v = O.rope_in_place(np.array([3.0, 4.0], np.float32), 1, 2, 1, 1_000_000.0)
    assert abs(v[0] * v[0] + v[1] * v[1] - 25.0) < 1e-4
    c, s = math.cos(1.0), math.sin(1.0)
    assert abs(v[0] - (3.0 * c - 4.0 * s)) < 1e-5
    assert abs(v[1] - (4.0 * c + 3.0 * s)) < 1e-5


def test_rope_heads_rotates_leading_dims_of_every_head():  # ops.rs:1963
    values = O.rope_heads(np.array([1.0, 0.0, 9.0, 8.0, 0.0, 1.0, 7.0, 6.0], np.float32),
                          2, 4, 2, 1, 10_000.0)
    s, c = math.sin(1.0), math.cos(1.0)
    assert abs(values[0] - c) < 1e-5 and abs(values[1] - s) < 1e-5
    assert abs(values[4] + s) < 1e-5 and abs(values[5] - c) < 1e-5
    assert values[2:4].tolist() == [9.0, 8.0] and values[6:8].tolist() == [7.0, 6.0]


def test_silu_multiply_matches_reference():  # ops.rs:1981
    g = O.silu_multiply(np.array([1.0, -2.0], np.float32), np.array([2.0, 3.0], np.float32))
    silu = lambda x: x / (1.0 + math.exp(-x))
    assert abs(g[0] - silu(1.0) * 2.0) < 1e-6 and abs(g[1] - silu(-2.0) * 3.0) < 1e-6


def test_softmax_sums_to_one_and_is_shift_invariant():  # ops.rs:1990
    s = O.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(s.sum() - 1.0) < 1e-6 and s[2] > s[1] > s[0]
    shifted = O.softmax(np.array([1001.0, 1002.0, 1003.0], np.float32))
    assert abs(s[0] - shifted[0]) < 1e-5


def test_rope_matches_reference_rotate_half():  # ops.rs:2004
    head_dim, theta, half = 64, np.float32(1_000_000.0), 32
    inp = np.array([((i * 37 % 11) / 7.0) - 0.6 for i in range(head_dim)], np.float32)
    for position in range(1, 9):
        native = O.rope_in_place(inp, 1, head_dim, position, float(theta))
        expected = np.zeros(head_dim, np.float32)
        for i in range(half):
            freq = 1.0 / float(theta) ** (2.0 * i / head_dim)
            angle = position * freq
            expected[i] = inp[i] * math.cos(angle) - inp[i + half] * math.sin(angle)
            expected[i + half] = inp[i + half] * math.cos(angle) + inp[i] * math.sin(angle)
        assert np.max(np.abs(native - expected)) < 1e-4


def test_dot_row_bf16_fused_matches_dequant_dot():  # ops.rs:2040
    cols = 8
    row = bf16_trunc(np.array([float(i % 251) for i in range(cols)], np.float32))
    x = np.array([(i % 17) / 8.0 - 1.0 for i in range(cols)], np.float32)
    fused = O.gemv(row, 1, cols, x)[0]
    naive = float(np.dot((row.astype(np.uint32) << 16).view(np.float32), x))
    assert abs(fused - naive) < 1e-2


def test_dot_row_bf16_fused_full_width_matches_reference():  # ops.rs:2067
    cols = 896
    row = bf16_trunc(np.array([(i % 251) * 0.5 - 60.0 for i in range(cols)], np.float32))
    x = np.array([(i % 31) * 0.25 - 4.0 for i in range(cols)], np.float32)
    fused = O.gemv(row, 1, cols, x)[0]
    ref = float(np.dot((row.astype(np.uint32) << 16).view(np.float32).astype(np.float64), x))
    assert abs(fused - ref) / max(abs(ref), 1.0) < 1e-5


def test_q8_buffer_layout_matches_ffi_contract():  # q8.rs:209
    for rows, cols in [(3, 5), (8, 64), (128, 151936 // 128)]:
        values = np.array([(i % 17) - 8.0 for i in range(rows * cols)], np.float32)
        buf = O.quantize_q8(values, rows, cols)
        assert buf.size == rows * 4 + rows * ((cols + 3) // 4 * 4)


def test_q4_buffer_layout_matches_ffi_contract():  # q4.rs:246
    for rows, cols in [(3, 5), (8, 64), (128, 151936 // 128)]:
        values = np.array([(i % 17) - 8.0 for i in range(rows * cols)], np.float32)
        buf = O.quantize_q4(values, rows, cols)
        stride = -(-(-(-(cols + 1) // 2)) // 4) * 4
        assert buf.size == rows * 4 + rows * stride


def test_q4_row_stride_quirk_at_model_widths():
    # (cols + 1).div_ceil(2).div_ceil(4) * 4 over-pads even widths by 4 bytes.
    assert [O.q4_row_bytes(c) for c in (896, 3584, 4864, 18944)] == [452, 1796, 2436, 9476]
    assert [O.q8_row_bytes(c) for c in (896, 3584, 4864, 18944)] == [896, 3584, 4864, 18944]


@pytest.mark.parametrize("fmt,limit", [("q8", 127.0), ("q4", 7.0)])
def test_quantize_round_trip_within_one_step(fmt, limit):  # q8.rs:230, q4.rs:265
    rows = 2
    cols = 7 if fmt == "q8" else 9
    values = np.full(rows * cols, 0.25, np.float32)
    values[cols] = -40.0
    quant = O.quantize_q8 if fmt == "q8" else O.quantize_q4
    dq = O.q8_dequant if fmt == "q8" else O.q4_dequant
    buf = quant(values, rows, cols)
    scales = buf[:8].view(np.float32)
    assert abs(scales[0] - 0.25 / limit) < 1e-9 and abs(scales[1] - 40.0 / limit) < 1e-9
    for i, v in enumerate(values):
        r, c = divmod(i, cols)
        assert abs(dq(buf, rows, cols, r, c) - v) <= scales[r] / 2 + 1e-6


def test_q4_nibble_packing_matches_column_parity():  # q4.rs:292
    values = np.array([(i + 1.0) * 0.5 for i in range(8)], np.float32)
    buf = O.quantize_q4(values, 1, 8)
    scale = buf[:4].view(np.float32)[0]
    for c in range(8):
        code = int(np.clip(math.floor(values[c] / scale + 0.5), -7, 7))
        assert abs(O.q4_dequant(buf, 1, 8, 0, c) - code * scale) < 1e-6


def test_quantize_rejects_size_mismatch():  # q8.rs:254, q4.rs:317
    with pytest.raises(ValueError, match="expected 15 elements"):
        O.quantize_q8(np.zeros(10, np.float32), 3, 5)
    with pytest.raises(ValueError, match="expected 15 elements"):
        O.quantize_q4(np.zeros(10, np.float32), 3, 5)


def test_vectorised_dequant_matches_scalar_unpacking():
    rng = np.random.default_rng(3)
    rows, cols = 7, 37
    values = rng.standard_normal(rows * cols, dtype=np.float32)
    for fmt, quant, dq in [("q8", O.quantize_q8, O.q8_dequant), ("q4", O.quantize_q4, O.q4_dequant)]:
        buf = quant(values, rows, cols)
        mat = O.dequant_matrix(buf, rows, cols, fmt)
        for r in range(rows):
            for c in range(cols):
                assert mat[r, c] == np.float32(dq(buf, rows, cols, r, c))


def test_attention_single_key_returns_its_value():
    # One cached key: softmax weight 1, output equals the value row per head.
    q_heads, kv_heads, d = 4, 2, 8
    rng = np.random.default_rng(0)
    k = rng.standard_normal(kv_heads * d, dtype=np.float32)
    v = rng.standard_normal(kv_heads * d, dtype=np.float32)
    q = rng.standard_normal(q_heads * d, dtype=np.float32)
    out = O.attention(k, v, q, q_heads, kv_heads, d)
    for h in range(q_heads):
        np.testing.assert_array_equal(out[h * d:(h + 1) * d], v[(h // 2) * d:(h // 2 + 1) * d])
