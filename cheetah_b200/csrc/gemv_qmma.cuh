// Integer tensor-core GEMV for q8 / q4 weights (decode, one input vector).
//
// y = scale[r] * sum_k code[r][k] * x[k]  (`ops.rs:544-630`, per-row scales
// of `q8.rs:91-125` / `q4.rs:126-161`), computed with integer mma.sync:
//   A  16 weight rows x 32 codes as s8 (m16n8k32): q8 codes exactly as
//      stored, no widening instructions; q4 nibbles sign-extended to bytes
//      in registers (three ALU operations per four codes).
//   B  the input as a fixed-point integer x' = rint(x * 2^e), e chosen from
//      max|x| so that |x'| < 2^29, written as four signed base-256 digits,
//      one B column per digit: the bytes of (x' + 0x80808080) ^ 0x80808080
//      are the balanced signed digits of x'.
//   The int32 column sums S_n are exact; sum_n S_n * base^n is formed in 64
//   bits, partial sums of warps that split a row are added as integers (so
//   the result does not depend on the split), and the row result is
//   float(S) * 2^-e * scale. x' keeps 29 bits below max|x|, finer than the
//   f32 inputs' own rounding for every element within 2^5 of the largest.
//   The reduction index is permuted: each lane reads 16 contiguous bytes of
//   its two rows per step (128-bit streaming loads, no shared-memory staging
//   of weights); the digit table in shared memory follows the same order and
//   occupies exactly the bytes of x it was made from (x is staged with one
//   wave of cp.async and converted in place).
// Tiles of 16 rows follow the epilogue: QKV tiles hold 8 rotate-half pairs
// (rows g and g + 8 of the tile are partners), SwiGLU tiles 8 gate rows and
// the 8 up rows of the same indices, other tiles 16 consecutive rows. The
// epilogues are the register-streaming GEMV's (`epilogue_rows`).
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace cheetah {

constexpr int kQmThreads = 256;
constexpr int kQmWarps = kQmThreads / kWarp;

// Rows of tile position g: row_lo (tile row g) and row_hi (tile row g + 8).
template <int EPI>
__device__ __forceinline__ void qm_tile_rows(const GemvParams &p, int tile, int g, int &row_lo, int &row_hi) {
    if (EPI == kEpiQkv) {
        const int half = p.head_dim >> 1;
        const int pair = tile * 8 + g;
        const int head = pair / half, i = pair - head * half;
        row_lo = head * p.head_dim + i;
        row_hi = row_lo + half;
    } else if (EPI == kEpiSwiglu) {
        row_lo = row_hi = tile * 8 + g;  // gate row of w0, up row of w1
    } else {
        row_lo = tile * 16 + g;
        row_hi = row_lo + 8;
    }
}

__host__ __device__ inline int qm_num_tiles(int epi, int rows) { return epi == kEpiSwiglu ? rows / 8 : rows / 16; }

__device__ __forceinline__ void qm_imma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// Four 4-bit two's-complement codes (low nibbles of the bytes of u) as
// signed bytes: ((c ^ 8) + 0x78) ^ 0x80 per byte, no carries between bytes.
__device__ __forceinline__ uint32_t qm_nibbles_s8(uint32_t u) {
    return (((u & 0x0F0F0F0Fu) ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u;
}

__device__ __forceinline__ void qm_cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void qm_cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint4 qm_ldg(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// One step: 16 bytes of each of the lane's two rows (a0/a2 from row g,
// a1/a3 from row g + 8). `tab` is the step's part of the digit table:
// groups of 8 inputs, digit n as the 8-byte entry n of the group.
//   q8: 16 codes per lane, two MMAs; MMA h takes group 2q + h, whose b0/b1
//       are inputs 0-3 / 4-7.
//   q4: 32 codes per lane, four MMAs; MMA i takes word i: a0 = its even
//       codes (low nibbles), a2 = its odd codes, group 4q + i with b0/b1 =
//       inputs 0,2,4,6 / 1,3,5,7.
template <int WT>
__device__ __forceinline__ void qm_step(int (&acc0)[4], int (&acc1)[4], uint4 wlo, uint4 whi, const uint2 *tab,
                                        int lane) {
    const int n = lane >> 2, q = lane & 3;
    if (WT == kWQ8) {
        const uint2 b0 = n < 4 ? tab[(2 * q + 0) * 4 + n] : make_uint2(0u, 0u);
        const uint2 b1 = n < 4 ? tab[(2 * q + 1) * 4 + n] : make_uint2(0u, 0u);
        qm_imma(acc0, wlo.x, whi.x, wlo.y, whi.y, b0);
        qm_imma(acc1, wlo.z, whi.z, wlo.w, whi.w, b1);
    } else {
        const uint32_t lo[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
        const uint32_t hi[4] = {whi.x, whi.y, whi.z, whi.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint2 b = n < 4 ? tab[(4 * q + i) * 4 + n] : make_uint2(0u, 0u);
            const uint32_t a0 = qm_nibbles_s8(lo[i]), a2 = qm_nibbles_s8(lo[i] >> 4);
            const uint32_t a1 = qm_nibbles_s8(hi[i]), a3 = qm_nibbles_s8(hi[i] >> 4);
            if (i & 1) qm_imma(acc1, a0, a1, a2, a3, b);
            else qm_imma(acc0, a0, a1, a2, a3, b);
        }
    }
}

// Signed base-256 digits of rint(v) (|v| < 2^29), one per byte.
__device__ __forceinline__ uint32_t qm_digits(float v) {
    const uint32_t u = (uint32_t)__float2int_rn(v);
    return (u + 0x80808080u) ^ 0x80808080u;
}

// Digit n of four inputs' digit strings as one word (byte u = input u).
__device__ __forceinline__ void qm_transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&out)[4]) {
    const uint32_t t0 = __byte_perm(w0, w1, 0x5140), t1 = __byte_perm(w2, w3, 0x5140);
    const uint32_t t2 = __byte_perm(w0, w1, 0x7362), t3 = __byte_perm(w2, w3, 0x7362);
    out[0] = __byte_perm(t0, t1, 0x5410);
    out[1] = __byte_perm(t0, t1, 0x7632);
    out[2] = __byte_perm(t2, t3, 0x5410);
    out[3] = __byte_perm(t2, t3, 0x7632);
}

// Grid: CTAs over groups of kQmWarps / KS tiles (grid-stride); KS warps
// split a tile's steps and their partial sums are added as integers.
// Dynamic shared memory: x, converted in place into the digit table (4
// bytes per input element), then the RMSNorm weights when norm_w is set.
template <int EPI, int WT, int KS>
__global__ void __launch_bounds__(kQmThreads) gemv_qmma_kernel(const GemvParams p) {
    constexpr int kT = kQmWarps / KS;  // tiles per CTA pass
    constexpr int kElemsPerStep = WT == kWQ8 ? 64 : 128;
    constexpr int kDigits = 4;  // base-256 digits of x'
    // Steps of loads in flight per lane: a ring of 8, a slot refilled as
    // soon as it is consumed, for q4 (more MMA work per byte) and for tiles
    // split over 8 warps (few steps per warp: all of them in flight before
    // the dependency wait); batches of 4, the next batch issued before this
    // one's MMAs, for whole-row q8 tiles. Measured best for each.
    constexpr bool kRing = WT == kWQ4 || KS == 8;
    constexpr int kU = kRing ? 8 : 4;
    extern __shared__ __align__(16) float qm_x[];
    uint2 *qm_tab = reinterpret_cast<uint2 *>(qm_x);
    __shared__ float red[kQmWarps];
    __shared__ float redm[kQmWarps];
    __shared__ long long part[kQmWarps][16];
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int g = lane >> 2, q = lane & 3;
    const int tile_in = warp / KS, ks = warp % KS;
    const int K = p.cols;
    const int steps = K / kElemsPerStep;
    const int per = (steps + KS - 1) / KS;
    const int s_begin = min(steps, ks * per), s_end = min(steps, s_begin + per);
    const int tiles = qm_num_tiles(EPI, p.rows);
    const long long rs = p.row_stride;
    const uint8_t *w0 = reinterpret_cast<const uint8_t *>(p.w0);
    const uint8_t *w1 = reinterpret_cast<const uint8_t *>(EPI == kEpiSwiglu ? p.w1 : p.w0);

    int tile = blockIdx.x * kT + tile_in;
    const int tile_stride = gridDim.x * kT;
    const uint8_t *plo = nullptr, *phi = nullptr;
    auto set_rows = [&](int t) {
        int rl = 0, rh = 0;
        if (t < tiles) qm_tile_rows<EPI>(p, t, g, rl, rh);
        plo = w0 + (long long)rl * rs + 16 * q;
        phi = w1 + (long long)rh * rs + 16 * q;
    };
    uint4 la[kU], ha[kU];
    auto load = [&](int s0) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int s = s0 + u;
            if (s < s_end && tile < tiles) {
                la[u] = qm_ldg(plo + (long long)s * 64);
                ha[u] = qm_ldg(phi + (long long)s * 64);
            }
        }
    };

    // Weights and row scales do not depend on the previous kernel: start
    // streaming them.
    set_rows(tile);
    load(s_begin);
    float sc_lo = 0.0f, sc_hi = 0.0f;
    auto load_scales = [&](int t) {
        if (ks == 0 && q == 0 && t < tiles) {
            int rl, rh;
            qm_tile_rows<EPI>(p, t, g, rl, rh);
            sc_lo = p.scale0[rl];
            sc_hi = EPI == kEpiSwiglu ? p.scale1[rh] : p.scale0[rh];
        }
    };
    load_scales(tile);

    pdl_wait();
    pdl_launch_dependents();

    // Prologue: x (RMS-normalised when norm_w is set; the same arithmetic
    // as the register-streaming GEMV), as digits of rint(x * 2^e).
    float inv = 1.0f, inv_esc = 1.0f;
    {
        const float *nw = qm_x + K;
        const uint32_t xs = smem_u32(qm_x);
        for (int i = threadIdx.x; i < K / 4; i += kQmThreads) qm_cp_async16(xs + 16u * i, p.x + 4 * i);
        if (p.norm_w)
            for (int i = threadIdx.x; i < K / 4; i += kQmThreads) qm_cp_async16(xs + 16u * (K / 4 + i), p.norm_w + 4 * i);
        qm_cp_async_wait_all();
        __syncthreads();
        float ss = 0.0f, mx = 0.0f;
        for (int i = threadIdx.x; i < K; i += kQmThreads) {
            const float v = qm_x[i];
            ss = fmaf(v, v, ss);
            mx = fmaxf(mx, fabsf(p.norm_w ? v * nw[i] : v));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if (lane == 0) {
            red[warp] = ss;
            redm[warp] = mx;
        }
        __syncthreads();  // also: every read of x above is done before the in-place conversion
        float total = 0.0f, m = 0.0f;
#pragma unroll
        for (int w = 0; w < kQmWarps; ++w) {
            total += red[w];
            m = fmaxf(m, redm[w]);
        }
        if (p.norm_w) {
            inv = 1.0f / sqrtf(total / (float)K + p.eps);
            m *= inv;
        }
        // 2^e with m * 2^e in [2^27, 2^28): |x'| < 2^29 even where the
        // normalised product rounds above m, so the top digit stays small.
        int e = 0;
        if (m > 0.0f && isfinite(m)) {
            const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
            e = max(-100, min(100, 27 - ex));
        }
        const float esc = __uint_as_float((uint32_t)(127 + e) << 23);
        inv_esc = __uint_as_float((uint32_t)(127 - e) << 23);
        auto xv = [&](int i) -> float {
            const float v = p.norm_w ? __fmul_rn(qm_x[i], __fmul_rn(inv, nw[i])) : qm_x[i];
            return __fmul_rn(v, esc);
        };
        // Group of 8 inputs -> 4 entries (digit n): q8 b0/b1 = inputs 0-3 /
        // 4-7, q4 b0/b1 = inputs 0,2,4,6 / 1,3,5,7.
        for (int G = threadIdx.x; G < K / 8; G += kQmThreads) {
            uint32_t d[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) d[u] = qm_digits(xv(8 * G + u));
            uint32_t o0[4], o1[4];
            if (WT == kWQ8) {
                qm_transpose4(d[0], d[1], d[2], d[3], o0);
                qm_transpose4(d[4], d[5], d[6], d[7], o1);
            } else {
                qm_transpose4(d[0], d[2], d[4], d[6], o0);
                qm_transpose4(d[1], d[3], d[5], d[7], o1);
            }
#pragma unroll
            for (int n = 0; n < 4; ++n) qm_tab[4 * G + n] = make_uint2(o0[n], o1[n]);
        }
    }
    __syncthreads();

    unsigned long long best = 0ull;
    for (; tile - tile_in < tiles; tile += tile_stride) {
        int acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
        if (tile < tiles) {
            for (int s0 = s_begin; s0 < s_end; s0 += kU) {
                if constexpr (kRing) {
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        const int s = s0 + u;
                        if (s < s_end) {
                            qm_step<WT>(acc0, acc1, la[u], ha[u], qm_tab + (size_t)s * (kElemsPerStep / 2), lane);
                            if (s + kU < s_end) {
                                la[u] = qm_ldg(plo + (long long)(s + kU) * 64);
                                ha[u] = qm_ldg(phi + (long long)(s + kU) * 64);
                            }
                        }
                    }
                } else {
                    uint4 cl[kU], chh[kU];
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        cl[u] = la[u];
                        chh[u] = ha[u];
                    }
                    if (s0 + kU < s_end) load(s0 + kU);
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        if (s0 + u < s_end)
                            qm_step<WT>(acc0, acc1, cl[u], chh[u], qm_tab + (size_t)(s0 + u) * (kElemsPerStep / 2),
                                        lane);
                    }
                }
            }
        }
        // Next tile's first loads before the epilogue.
        const int next = tile + tile_stride;
        const float sl = sc_lo, sh = sc_hi;
        if (next - tile_in < tiles) {
            const int cur = tile;
            tile = next;
            set_rows(tile);
            load(s_begin);
            load_scales(tile);
            tile = cur;
        }
        // Lane q holds columns (digits) 2q and 2q + 1 of rows g and g + 8.
        long long vlo = 0, vhi = 0;
        if (2 * q < kDigits) {
            const int s0 = 8 * 2 * q, s1 = 8 * (2 * q + 1);
            vlo = ((long long)acc0[0] + acc1[0]) * (1ll << s0) + ((long long)acc0[1] + acc1[1]) * (1ll << s1);
            vhi = ((long long)acc0[2] + acc1[2]) * (1ll << s0) + ((long long)acc0[3] + acc1[3]) * (1ll << s1);
        }
        vlo += __shfl_xor_sync(0xFFFFFFFFu, vlo, 1);
        vhi += __shfl_xor_sync(0xFFFFFFFFu, vhi, 1);
        vlo += __shfl_xor_sync(0xFFFFFFFFu, vlo, 2);
        vhi += __shfl_xor_sync(0xFFFFFFFFu, vhi, 2);
        if (KS > 1) {
            if (q == 0) {
                part[warp][g] = vlo;
                part[warp][g + 8] = vhi;
            }
            __syncthreads();
            if (ks == 0 && q == 0) {
#pragma unroll
                for (int k = 1; k < KS; ++k) {
                    vlo += part[warp + k][g];
                    vhi += part[warp + k][g + 8];
                }
            }
            __syncthreads();
        }
        if (ks == 0 && q == 0 && tile < tiles) {
            int rl, rh;
            qm_tile_rows<EPI>(p, tile, g, rl, rh);
            const float flo = __fmul_rn(__fmul_rn(__ll2float_rn(vlo), inv_esc), sl);
            const float fhi = __fmul_rn(__fmul_rn(__ll2float_rn(vhi), inv_esc), sh);
            epilogue_rows<EPI>(p, 0, rl, rh, flo, fhi, best);
        }
    }
}

}  // namespace cheetah
