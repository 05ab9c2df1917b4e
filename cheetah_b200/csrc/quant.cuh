// Per-row symmetric quantisers on the device, bit-identical to the
// reference's registered `q8::quantize` (`precision/q8.rs:91-125`) and
// `q4::quantize` (`precision/q4.rs:126-161`):
//   scale = max|w| / 127 (q4: / 7) as an IEEE f32 division, 1.0 for an
//   all-zero row; code = clamp(round_half_away(w / scale), -127, 127)
//   (q4: +-7); buffer = rows f32 scales || rows x row_bytes codes, padding
//   bytes zero; q4 packs two codes per byte, low nibble = even column.
// Input: the unit's bf16 weights (widened exactly, `ops.rs:634`
// dequant_values). One warp per row.
#pragma once

#include "common.cuh"

namespace cheetah {

__host__ __device__ inline long long q8_row_bytes(long long cols) { return (cols + 3) / 4 * 4; }
// q4.rs:50: (cols + 1).div_ceil(2).div_ceil(4) * 4 (over-pads even widths by 4).
__host__ __device__ inline long long q4_row_bytes(long long cols) { return ((cols + 2) / 2 + 3) / 4 * 4; }

// out_rb: bytes between output code rows; 0 = the reference row size. A
// smaller stride (q4 rows of cols / 2 bytes, 16-byte aligned for 128-bit
// loads) drops only the reference layout's padding bytes.
template <int BITS>
__global__ void quantize_rows_kernel(const uint16_t *__restrict__ w, int rows, int cols, uint8_t *__restrict__ out,
                                     long long out_rb = 0) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (warp >= rows) return;
    const uint16_t *row = w + (long long)warp * cols;
    float max_abs = 0.0f;
    for (int c = lane; c < cols; c += kWarp) max_abs = fmaxf(max_abs, fabsf(bf16_to_f32(row[c])));
    max_abs = warp_max(max_abs);
    const float limit = BITS == 8 ? 127.0f : 7.0f;
    const float scale = max_abs > 0.0f ? __fdiv_rn(max_abs, limit) : 1.0f;
    if (lane == 0) reinterpret_cast<float *>(out)[warp] = scale;
    const long long ref_rb = BITS == 8 ? q8_row_bytes(cols) : q4_row_bytes(cols);
    const long long rb = out_rb > 0 && out_rb < ref_rb ? out_rb : ref_rb;
    uint8_t *codes = out + (long long)rows * 4 + (long long)warp * rb;
    auto code_of = [&](int c) -> int {
        if (c >= cols) return 0;
        float q = roundf(__fdiv_rn(bf16_to_f32(row[c]), scale));
        q = fminf(fmaxf(q, -limit), limit);
        return (int)q;
    };
    if (BITS == 8) {
        for (long long byte = lane; byte < rb; byte += kWarp) codes[byte] = (uint8_t)(int8_t)code_of((int)byte);
    } else {
        for (long long byte = lane; byte < rb; byte += kWarp) {
            const int lo = code_of((int)(2 * byte));
            const int hi = code_of((int)(2 * byte + 1));
            codes[byte] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
        }
    }
}

}  // namespace cheetah
