"""q8 / q4 on the GPU: the device quantiser is byte-identical to the
reference's `q8::quantize` / `q4::quantize` (restated in the oracle), the
quantised GEMVs match `gemv_q8` / `gemv_q4`, and the quantised decoder
matches the oracle's quantised forward."""

import numpy as np
import pytest

import oracle as O
from tests.greedy import check_greedy
from cheetah_b200.prepared import PreparedModel, bf16_bits_to_f32, f32_to_bf16_bits, resolve_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _weights(rows, cols, seed, zero_rows=()):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * 0.02
    for r in zero_rows:
        w[r] = 0.0
    bits = f32_to_bf16_bits(w)
    return bits.reshape(rows, cols), bf16_bits_to_f32(bits).reshape(rows, cols)


def _to_dev(bits):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("rows,cols", [(3, 6), (3, 9), (5, 9), (64, 896), (130, 4864), (7, 3584), (2, 18944)])
def test_device_quantiser_is_byte_identical(fmt, rows, cols):
    from cheetah_b200 import runtime as R
    bits, values = _weights(rows, cols, rows * 7 + cols, zero_rows=(1,) if rows > 2 else ())
    got = R.quantize(_to_dev(bits), fmt).cpu().numpy()
    want = (O.quantize_q8 if fmt == "q8" else O.quantize_q4)(values.reshape(-1), rows, cols)
    assert got.size == want.size == R.quant_buffer_bytes(fmt, rows, cols)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("rows,cols", [(1152, 896), (4864, 896), (896, 4864), (512, 3584), (3584, 18944), (3, 8)])
def test_quantised_gemv_matches_oracle(fmt, rows, cols):
    from cheetah_b200 import runtime as R
    bits, values = _weights(rows, cols, rows + cols)
    buf = (O.quantize_q8 if fmt == "q8" else O.quantize_q4)(values.reshape(-1), rows, cols)
    x = np.random.default_rng(3).standard_normal(cols, dtype=np.float32)
    y = R.gemv_quant(torch.from_numpy(buf).cuda(), fmt, rows, cols, torch.from_numpy(x).cuda()).cpu().numpy()[0]
    ref = (O.gemv_q8 if fmt == "q8" else O.gemv_q4)(buf, rows, cols, x)
    dq = O.dequant_matrix(buf, rows, cols, fmt)
    scale = np.abs(dq) @ np.abs(x)
    assert np.all(np.abs(y - ref) <= 2e-6 * scale + 1e-7), np.abs(y - ref).max()


@pytest.mark.parametrize("fixture", ["tiny_prepared", "tiny7b_prepared", "tinywide_prepared"])
@pytest.mark.parametrize("quant", ["q8", "q4"])
def test_quantised_decoder_matches_oracle(fixture, quant, request):
    from cheetah_b200 import runtime as R
    root = request.getfixturevalue(fixture)
    pm = PreparedModel(root)
    cfg = resolve_config(pm)
    ref = O.OracleModel(pm, cfg, quant)
    model = R.CudaModel(root, quant=quant, kv_dtype="f32", max_positions=512)
    assert model.info()["quant"] == (1 if quant == "q8" else 2)
    seq = model.new_sequence()
    prompt = np.random.default_rng(4).integers(0, cfg["vocab_size"], 30).astype(np.uint32)
    got = seq.forward(prompt, 0)
    want = ref.forward(prompt, 0)
    assert np.abs(got - want).max() < 1e-4
    tok = int(np.argmax(want))
    for i in range(12):
        want = ref.forward([tok], 30 + i)
        got = np.empty_like(want)
        am = seq.forward_greedy([tok], 30 + i, logits_out=got)
        assert np.abs(got - want).max() < 1e-4
        check_greedy(am, want, 1e-4, f"step {i}")
        tok = am


def test_unknown_precision_is_rejected(tiny_prepared):
    from cheetah_b200 import runtime as R
    with pytest.raises(R.CheetahCudaError, match="no CUDA operator table"):
        R.CudaModel(tiny_prepared, quant="f16")
