// Small-batch bf16 GEMV on the tensor cores: y[b] = W . x[b] for up to 8
// input rows at once (a batched decode step of <= 8 sequences), bf16 weights
// [rows, cols] (`ops.rs:202-278`, `gemm` `ops.rs:308` for several rows).
//
// mma.sync m16n8k16 (bf16 in, f32 accumulate):
//   A  16 weight rows x 16 columns, read straight from HBM: each lane loads
//      16 contiguous bytes of its two rows per step (128-bit streaming
//      loads); the reduction index is permuted so that those 8 weights are
//      A-fragment elements of two MMAs (elements 0-3 -> k {2c, 2c+1, 2c+8,
//      2c+9} of the first, 4-7 of the second).
//   B  the batch rows as the 8 MMA columns: x rounded to bf16 (optionally
//      RMS-normalised first) in a shared-memory table with padded rows, read
//      in the same permuted order (16 contiguous bytes per lane).
// Every weight byte is read once per step for all rows; 16-row tiles
// follow the register GEMV's epilogues (`epilogue_rows`): QKV tiles hold 8
// rotate-half pairs (tile rows g and g + 8 are partners), SwiGLU tiles 8
// gate rows and the 8 up rows of the same indices, other tiles 16
// consecutive rows. Many tiles: a warp per tile; few tiles: a CTA per
// (tile, K split), see gemv_mma_kernel. Persistent CTAs walk the work.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_qmma.cuh"

namespace cheetah {

constexpr int kGmThreads = 256;
constexpr int kGmWarps = kGmThreads / kWarp;
constexpr int kGmRows = 8;   // batch rows (MMA columns)
constexpr int kGmUnroll = 4; // steps of 32 columns in flight per lane

__device__ __forceinline__ void gm_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Tiles of a GEMV: QKV 8 pairs, SwiGLU 8 gate/up rows, else 16 rows (the
// last tile of those may be partial).
__host__ __device__ inline int gm_num_tiles(int epi, int rows) {
    if (epi == kEpiQkv) return rows / 16;
    if (epi == kEpiSwiglu) return (rows + 7) / 8;
    return (rows + 15) / 16;
}

// Dynamic shared memory: x table [8][cols + 8] bf16, then the K-split
// partials [warps][4][32] f32.
inline size_t gemv_mma_smem(int cols) { return (size_t)kGmRows * (cols + 8) * 2 + (size_t)kGmWarps * 4 * kWarp * 4; }

// KS == 1: one warp per 16-row tile over the whole K range (GEMVs with many
// tiles). KS == 8: one CTA per (tile, K split) item, the item's 32-column
// steps dealt round-robin to the 8 warps and summed in warp order; with
// p.splits > 1 every split writes its 16 x 8 partial and the tile's last
// split (a ticket, no waiting) adds them in split order and runs the
// epilogue, so results do not depend on which split finishes last.
template <int EPI, int KS>
__global__ void __launch_bounds__(kGmThreads) gemv_mma_kernel(const GemvParams p) {
    static_assert(KS == 1 || KS == kGmWarps, "warp per tile, or CTA per tile");
    extern __shared__ __align__(16) uint8_t gm_smem[];
    const int K = p.cols;
    const int xs_stride = K + 8;  // bf16 elements per table row (16-byte pad: no bank conflicts)
    uint16_t *xs = reinterpret_cast<uint16_t *>(gm_smem);
    float *part = reinterpret_cast<float *>(gm_smem + (size_t)kGmRows * xs_stride * 2);
    __shared__ unsigned long long best_s[kGmWarps][kGmRows];
    static_assert(kGmWarps == kGmRows, "one staging warp per batch row");

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int g = lane >> 2, c = lane & 3;
    const int steps = K / 32;
    const int tiles = gm_num_tiles(EPI, p.rows);
    const int splits = KS == 1 ? 1 : max(1, p.splits);
    const int per = (steps + splits - 1) / splits;
    // Work items: KS == 1, tiles of this warp; KS == 8, (tile, split) of the CTA.
    const int items = KS == 1 ? tiles : tiles * splits;
    const int item_stride = KS == 1 ? gridDim.x * kGmWarps : gridDim.x;
    int item = KS == 1 ? blockIdx.x * kGmWarps + warp : blockIdx.x;
    auto item_tile = [&](int it) { return KS == 1 ? it : it / splits; };
    // Steps of this warp in item it: j-th = first + j * stride, j < count.
    auto item_steps = [&](int it, int &first, int &stride, int &count) {
        if (KS == 1) {
            first = 0;
            stride = 1;
            count = steps;
        } else {
            const int sp = it % splits;
            const int a = sp * per, b = min(steps, a + per);
            first = a + warp;
            stride = kGmWarps;
            count = first < b ? (b - first + kGmWarps - 1) / kGmWarps : 0;
        }
    };

    // Weight vectors in two register sets: group j + 1 loads while group j
    // is multiplied.
    uint4 wl[2][kGmUnroll], wh[2][kGmUnroll];
    auto load = [&](int it, int j0, int buf) {
        const int t = item_tile(it);
        int rl, rh;
        qm_tile_rows<EPI>(p, t < tiles ? t : 0, g, rl, rh);
        const uint8_t *lo = reinterpret_cast<const uint8_t *>(p.w0) + (size_t)rl * K * 2;
        const uint8_t *hi = reinterpret_cast<const uint8_t *>(EPI == kEpiSwiglu ? p.w1 : p.w0) + (size_t)rh * K * 2;
        const bool vl = it < items && rl < p.rows, vh = it < items && rh < p.rows;
        int first, stride, count;
        item_steps(it, first, stride, count);
#pragma unroll
        for (int u = 0; u < kGmUnroll; ++u) {
            const int j = j0 + u;
            const size_t off = ((size_t)(first + j * stride) * 32 + 8 * c) * 2;
            wl[buf][u] = (j < count && vl) ? qm_ldg(lo + off) : make_uint4(0, 0, 0, 0);
            wh[buf][u] = (j < count && vh) ? qm_ldg(hi + off) : make_uint4(0, 0, 0, 0);
        }
    };
    load(item, 0, 0);

    pdl_wait();
    pdl_launch_dependents();

    // x table: batch rows (RMS-normalised when asked) as bf16, one warp per
    // row; each lane issues kV 16-byte loads at a time (rows up to 1024
    // columns stay in registers between the norm's two passes).
    {
        constexpr int kV = 8;
        const int b = warp;
        uint16_t *xo = xs + (size_t)b * xs_stride;
        const float *xin = p.x + (long long)b * p.x_stride;
        const bool live = b < p.batch;
        auto put = [&](int i, float4 n) {
            uint2 packed;
            packed.x = (uint32_t)f32_to_bf16_rne(n.x) | ((uint32_t)f32_to_bf16_rne(n.y) << 16);
            packed.y = (uint32_t)f32_to_bf16_rne(n.z) | ((uint32_t)f32_to_bf16_rne(n.w) << 16);
            *reinterpret_cast<uint2 *>(xo + i) = packed;
        };
        auto scale = [&](int i, float4 v, float inv) {
            const float4 w = *reinterpret_cast<const float4 *>(p.norm_w + i);
            return make_float4(__fmul_rn(v.x, __fmul_rn(inv, w.x)), __fmul_rn(v.y, __fmul_rn(inv, w.y)),
                               __fmul_rn(v.z, __fmul_rn(inv, w.z)), __fmul_rn(v.w, __fmul_rn(inv, w.w)));
        };
        if (live && p.norm_w && K <= kWarp * 4 * kV) {
            float4 v[kV];
            float ss = 0.0f;
#pragma unroll
            for (int u = 0; u < kV; ++u) {
                const int i = lane * 4 + u * kWarp * 4;
                v[u] = i < K ? __ldcg(reinterpret_cast<const float4 *>(xin + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kV; ++u) {
                ss = fmaf(v[u].x, v[u].x, ss);
                ss = fmaf(v[u].y, v[u].y, ss);
                ss = fmaf(v[u].z, v[u].z, ss);
                ss = fmaf(v[u].w, v[u].w, ss);
            }
            const float inv = 1.0f / sqrtf(warp_sum(ss) / (float)K + p.eps);
#pragma unroll
            for (int u = 0; u < kV; ++u) {
                const int i = lane * 4 + u * kWarp * 4;
                if (i < K) put(i, scale(i, v[u], inv));
            }
        } else if (live) {
            float inv = 1.0f;
            if (p.norm_w) {
                float ss = 0.0f;
                for (int i0 = lane * 4; i0 < K; i0 += kWarp * 4 * kV) {
                    float4 v[kV];
#pragma unroll
                    for (int u = 0; u < kV; ++u) {
                        const int i = i0 + u * kWarp * 4;
                        v[u] = i < K ? __ldcg(reinterpret_cast<const float4 *>(xin + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int u = 0; u < kV; ++u) {
                        ss = fmaf(v[u].x, v[u].x, ss);
                        ss = fmaf(v[u].y, v[u].y, ss);
                        ss = fmaf(v[u].z, v[u].z, ss);
                        ss = fmaf(v[u].w, v[u].w, ss);
                    }
                }
                inv = 1.0f / sqrtf(warp_sum(ss) / (float)K + p.eps);
            }
            for (int i0 = lane * 4; i0 < K; i0 += kWarp * 4 * kV) {
                float4 v[kV];
#pragma unroll
                for (int u = 0; u < kV; ++u) {
                    const int i = i0 + u * kWarp * 4;
                    v[u] = i < K ? __ldcg(reinterpret_cast<const float4 *>(xin + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kV; ++u) {
                    const int i = i0 + u * kWarp * 4;
                    if (i < K) put(i, p.norm_w ? scale(i, v[u], inv) : v[u]);
                }
            }
        } else {
            for (int i = lane * 4; i < K; i += kWarp * 4) *reinterpret_cast<uint2 *>(xo + i) = make_uint2(0u, 0u);
        }
    }
    __syncthreads();

    unsigned long long best[2] = {0ull, 0ull};
    const uint32_t xrow = smem_u32(xs + (size_t)g * xs_stride);
    // Loop bound uniform over the CTA (KS == 8 syncs inside).
    for (; (KS == 1 ? item - warp : item) < items; item += item_stride) {
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        int first, stride, count;
        item_steps(item, first, stride, count);
        // Register set 0 holds the group at j0, set 1 the next one (literal
        // indices, so the sets stay in registers).
        auto mul = [&](int bs, int jb) {
#pragma unroll
            for (int u = 0; u < kGmUnroll; ++u) {
                if (jb + u < count) {
                    uint4 xv;
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                                 : "r"(xrow + (uint32_t)(((first + (jb + u) * stride) * 32 + 8 * c) * 2)));
                    gm_mma(acc0, wl[bs][u].x, wh[bs][u].x, wl[bs][u].y, wh[bs][u].y, xv.x, xv.y);
                    gm_mma(acc1, wl[bs][u].z, wh[bs][u].z, wl[bs][u].w, wh[bs][u].w, xv.z, xv.w);
                }
            }
        };
        for (int j0 = 0; j0 < count; j0 += 2 * kGmUnroll) {
            if (j0 + kGmUnroll < count) load(item, j0 + kGmUnroll, 1);
            mul(0, j0);
            if (j0 + 2 * kGmUnroll < count) load(item, j0 + 2 * kGmUnroll, 0);
            mul(1, j0 + kGmUnroll);
        }
        float acc[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = acc0[e] + acc1[e];
        const int t = item_tile(item);
        // The next item's first vectors before the epilogue.
        if (item + item_stride < items) load(item + item_stride, 0, 0);
        bool run_epilogue = KS == 1 ? item < items : false;
        if (KS > 1) {
            // Sum the warps' partials in warp order (warp 0 holds the item's sum).
#pragma unroll
            for (int e = 0; e < 4; ++e) part[(warp * 4 + e) * kWarp + lane] = acc[e];
            __syncthreads();
            if (warp == 0) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = 0.0f;
#pragma unroll
                    for (int k = 0; k < kGmWarps; ++k) v += part[(k * 4 + e) * kWarp + lane];
                    acc[e] = v;
                }
                if (splits == 1) {
                    run_epilogue = true;
                } else {
                    // Publish this split; the tile's last split adds all of
                    // them in split order (no waiting on other CTAs).
                    float *mine = p.split_ws + ((size_t)item * 4) * kWarp;
#pragma unroll
                    for (int e = 0; e < 4; ++e) mine[e * kWarp + lane] = acc[e];
                    __threadfence();
                    __syncwarp();
                    unsigned old = 0;
                    if (lane == 0) old = atomicAdd(p.split_tickets + t, 1u);
                    old = __shfl_sync(0xFFFFFFFFu, old, 0);
                    if (old == (unsigned)splits - 1) {
                        __threadfence();
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[e] = 0.0f;
                        for (int sp = 0; sp < splits; ++sp) {
                            const float *src = p.split_ws + ((size_t)(t * splits + sp) * 4) * kWarp;
#pragma unroll
                            for (int e = 0; e < 4; ++e) acc[e] += __ldcg(src + e * kWarp + lane);
                        }
                        if (lane == 0) p.split_tickets[t] = 0u;
                        run_epilogue = true;
                    }
                }
            }
            __syncthreads();
        }
        if (run_epilogue) {
            int row_lo, row_hi;
            qm_tile_rows<EPI>(p, t, g, row_lo, row_hi);
            // Fragment: acc[0..1] = rows g, columns 2c, 2c + 1; acc[2..3] = rows g + 8.
            if (row_lo < p.rows) {
                const int rb = (EPI == kEpiQkv || EPI == kEpiSwiglu || row_hi < p.rows) ? row_hi : -1;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int b = 2 * c + e;
                    if (b < p.batch) epilogue_rows<EPI>(p, b, row_lo, rb, acc[e], acc[2 + e], best[e]);
                }
            }
        }
    }

    if (EPI == kEpiLogits && p.argmax) {
        // Per batch row (columns 2c, 2c + 1): max over the 8 fragment rows,
        // then over the warps.
#pragma unroll
        for (int e = 0; e < 2; ++e) {
#pragma unroll
            for (int o = 4; o < kWarp; o <<= 1) {
                const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best[e], o);
                best[e] = other > best[e] ? other : best[e];
            }
        }
        if (g == 0) {
            best_s[warp][2 * c] = best[0];
            best_s[warp][2 * c + 1] = best[1];
        }
        __syncthreads();
        if ((int)threadIdx.x < kGmRows && (int)threadIdx.x < p.batch) {
            unsigned long long m = 0ull;
#pragma unroll
            for (int w = 0; w < kGmWarps; ++w) m = best_s[w][threadIdx.x] > m ? best_s[w][threadIdx.x] : m;
            if (m) atomicMax(p.argmax + threadIdx.x, m);
        }
    }
}

}  // namespace cheetah
