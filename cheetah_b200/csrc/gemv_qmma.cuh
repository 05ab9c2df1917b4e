// Tensor-core GEMV for q8 / q4 weights (decode, one input vector).
//
// y = scale[r] * sum_k code[r][k] * x[k]  (`ops.rs:544-630`, per-row scales
// of `q8.rs:91-125` / `q4.rs:126-161`), computed with mma.sync
// m16n8k16 f16 x f16 -> f32:
//   A  16 weight rows x 16 codes. int8 and int4 codes are exact in f16; a
//      code is widened by placing its biased value in the mantissa of 1024
//      (PRMT / LOP3) and subtracting the bias (one f16x2 subtraction per two
//      codes), so a q8 code costs about one instruction, not three.
//   B  the input vector as two f16 columns, hi = f16(x') and lo =
//      f16(x' - hi), x' = x * 2^e with e chosen from max|x| so that x' stays
//      far from the f16 overflow and subnormal ranges; hi + lo carries 22
//      significant bits of x', and the products are exact in the f32
//      accumulator. The result is scaled back by 2^-e (exact).
//   The reduction index is permuted: each lane reads 16 contiguous bytes of
//   its two rows per step (128-bit streaming loads, no shared-memory staging
//   of weights), and the table of B fragments in shared memory follows the
//   same permutation, so sum_k A[r][k] B[k] is the row dot product. The
//   table holds the fragments of a group of 4 (q8) or 8 (q4) inputs where
//   those inputs were: x is staged into shared memory with one wave of
//   cp.async and converted in place.
// Tiles of 16 rows follow the epilogue: QKV tiles hold 8 rotate-half pairs
// (rows g and g + 8 of the tile are partners), SwiGLU tiles 8 gate rows and
// the 8 up rows of the same indices, other tiles 16 consecutive rows. The
// epilogues are the register-streaming GEMV's (`epilogue_rows`).
#pragma once

#include <cuda_fp16.h>

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

__device__ __forceinline__ uint32_t qm_hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ void qm_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
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

// f16 pair (hi or lo part) of two scaled inputs.
__device__ __forceinline__ uint32_t qm_pack(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void qm_split(float v, float &hi, float &lo) {
    hi = __half2float(__float2half_rn(v));
    lo = __fsub_rn(v, hi);  // exact: v and hi agree in their top bits
}

// One step (64 bytes of each of the lane's two rows, 16 at this lane):
// MMAs over the codes in `wlo` (row g) and `whi` (row g + 8). `tab` is the
// step's part of the table; lane (n, q) = (lane / 4, lane % 4) of the B
// fragment reads the entry of input group 4q + j of the step, part n.
template <int WT>
__device__ __forceinline__ void qm_step(float (&acc0)[4], float (&acc1)[4], uint4 wlo, uint4 whi, const uint2 *tab,
                                        int lane) {
    const uint32_t lo[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
    const uint32_t hi[4] = {whi.x, whi.y, whi.z, whi.w};
    if (WT == kWQ8) {
        // word j: codes k0..k0+3, k0 = 64s + 16q + 4j; a0/a2 = (c0,c1)/(c2,c3).
        const uint32_t bias = 0x64806480u;  // f16 (1152, 1152) = 1024 + 128
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t bl = lo[j] ^ 0x80808080u, bh = hi[j] ^ 0x80808080u;
            const uint32_t a0 = qm_hsub2(__byte_perm(bl, 0x64646464u, 0x4140), bias);
            const uint32_t a2 = qm_hsub2(__byte_perm(bl, 0x64646464u, 0x4342), bias);
            const uint32_t a1 = qm_hsub2(__byte_perm(bh, 0x64646464u, 0x4140), bias);
            const uint32_t a3 = qm_hsub2(__byte_perm(bh, 0x64646464u, 0x4342), bias);
            const uint2 b = lane < 8 ? tab[2 * (4 * (lane & 3) + j) + (lane >> 2)] : make_uint2(0u, 0u);
            if (j & 1) qm_mma(acc1, a0, a1, a2, a3, b);
            else qm_mma(acc0, a0, a1, a2, a3, b);
        }
    } else {
        // word j: codes k0..k0+7, k0 = 128s + 32q + 8j (low nibble first);
        // half h: a0 = (c_2h, c_2h+4), a2 = (c_2h+1, c_2h+5).
        const uint32_t bias = 0x64086408u;  // f16 (1032, 1032) = 1024 + 8
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t bl = lo[j] ^ 0x88888888u, bh = hi[j] ^ 0x88888888u;
            uint32_t tl[4], th[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                tl[i] = qm_hsub2(((bl >> (4 * i)) & 0x000F000Fu) | 0x64006400u, bias);
                th[i] = qm_hsub2(((bh >> (4 * i)) & 0x000F000Fu) | 0x64006400u, bias);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint2 b = lane < 8 ? tab[4 * (4 * (lane & 3) + j) + 2 * h + (lane >> 2)] : make_uint2(0u, 0u);
                if (h) qm_mma(acc1, tl[2 * h], th[2 * h], tl[2 * h + 1], th[2 * h + 1], b);
                else qm_mma(acc0, tl[2 * h], th[2 * h], tl[2 * h + 1], th[2 * h + 1], b);
            }
        }
    }
}

// Grid: CTAs over groups of kQmWarps / KS tiles (grid-stride); KS warps
// split a tile's steps and their partials are summed in warp order.
// Dynamic shared memory: x, converted in place into the B table (4 bytes
// per input element), then the RMSNorm weights when norm_w is set.
template <int EPI, int WT, int KS>
__global__ void __launch_bounds__(kQmThreads) gemv_qmma_kernel(const GemvParams p) {
    constexpr int kT = kQmWarps / KS;                 // tiles per CTA pass
    constexpr int kElemsPerStep = WT == kWQ8 ? 64 : 128;
    constexpr int kU = 4;  // steps of loads in flight per lane
    extern __shared__ __align__(16) float qm_x[];
    uint2 *qm_tab = reinterpret_cast<uint2 *>(qm_x);
    __shared__ float red[kQmWarps];
    __shared__ float redm[kQmWarps];
    __shared__ float part[kQmWarps][16];
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
    // as the register-streaming GEMV), scaled by 2^e, as f16 hi/lo
    // fragments in the permuted order.
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
        // 2^e with m * 2^e in [2^13, 2^14): far below the f16 maximum (65504).
        int e = 0;
        if (m > 0.0f && isfinite(m)) {
            const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
            e = max(-100, min(100, 13 - ex));
        }
        const float esc = __uint_as_float((uint32_t)(127 + e) << 23);
        inv_esc = __uint_as_float((uint32_t)(127 - e) << 23);
        auto xv = [&](int i) -> float {
            const float v = p.norm_w ? __fmul_rn(qm_x[i], __fmul_rn(inv, nw[i])) : qm_x[i];
            return __fmul_rn(v, esc);
        };
        if (WT == kWQ8) {
            // group G = inputs 4G..4G+3 -> entries 2G (hi) and 2G + 1 (lo):
            // b0 = (x0, x1), b1 = (x2, x3) of MMA j = G % 4 of step G / 16,
            // quad q = G % 16 / 4.
            for (int G = threadIdx.x; G < K / 4; G += kQmThreads) {
                float h[4], l[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) qm_split(xv(4 * G + u), h[u], l[u]);
                qm_tab[2 * G] = make_uint2(qm_pack(h[0], h[1]), qm_pack(h[2], h[3]));
                qm_tab[2 * G + 1] = make_uint2(qm_pack(l[0], l[1]), qm_pack(l[2], l[3]));
            }
        } else {
            // group G = inputs 8G..8G+7 -> entries 4G + 2h + n: MMA 2j + h
            // takes b0 = (x_2h, x_2h+4), b1 = (x_2h+1, x_2h+5).
            for (int G = threadIdx.x; G < K / 8; G += kQmThreads) {
                float h[8], l[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) qm_split(xv(8 * G + u), h[u], l[u]);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int o = 2 * hh;
                    qm_tab[4 * G + 2 * hh] = make_uint2(qm_pack(h[o], h[o + 4]), qm_pack(h[o + 1], h[o + 5]));
                    qm_tab[4 * G + 2 * hh + 1] = make_uint2(qm_pack(l[o], l[o + 4]), qm_pack(l[o + 1], l[o + 5]));
                }
            }
        }
    }
    __syncthreads();

    unsigned long long best = 0ull;
    for (; tile - tile_in < tiles; tile += tile_stride) {
        float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (tile < tiles) {
            // The next batch's loads are issued before this batch's MMAs
            // (measured faster than refilling each slot as it is consumed).
            for (int s0 = s_begin; s0 < s_end; s0 += kU) {
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
                        qm_step<WT>(acc0, acc1, cl[u], chh[u], qm_tab + (size_t)(s0 + u) * (kElemsPerStep / 2), lane);
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
        // Columns 0 (hi) and 1 (lo) of lane q == 0: rows g and g + 8.
        float vlo = __fadd_rn(__fadd_rn(acc0[0], acc1[0]), __fadd_rn(acc0[1], acc1[1]));
        float vhi = __fadd_rn(__fadd_rn(acc0[2], acc1[2]), __fadd_rn(acc0[3], acc1[3]));
        if (KS > 1) {
            if (q == 0) {
                part[warp][g] = vlo;
                part[warp][g + 8] = vhi;
            }
            __syncthreads();
            if (ks == 0 && q == 0) {
                vlo = part[warp][g];
                vhi = part[warp][g + 8];
#pragma unroll
                for (int k = 1; k < KS; ++k) {
                    vlo = __fadd_rn(vlo, part[warp + k][g]);
                    vhi = __fadd_rn(vhi, part[warp + k][g + 8]);
                }
            }
            __syncthreads();
        }
        if (ks == 0 && q == 0 && tile < tiles) {
            int rl, rh;
            qm_tile_rows<EPI>(p, tile, g, rl, rh);
            vlo = __fmul_rn(__fmul_rn(vlo, inv_esc), sl);
            vhi = __fmul_rn(__fmul_rn(vhi, inv_esc), sh);
            epilogue_rows<EPI>(p, 0, rl, rh, vlo, vhi, best);
        }
    }
}

}  // namespace cheetah
