// Paged GQA decode attention over a bf16 KV cache on the tensor cores.
//
// Same math as decode_attention_kernel (`OpsToolbox::attention_head`,
// `ops.rs:1424-1467`) with q and the softmax weights rounded to bf16 for the
// MMAs (f32 accumulation, f32 online softmax); tolerance-checked against the
// f32 oracle.
//
// Data movement: every warp streams its own tiles of TILE positions
// (TILE * head_dim * 2 bytes = 8 KB for K and 8 KB for V) from the paged
// pool into a 3-stage shared-memory ring with 2D TMA loads
// (cp.async.bulk.tensor, 128-byte swizzle, no multicast) completing on
// per-stage mbarriers; a tile never crosses a KV page, so one box per tile
// and per 64-column half of the row. Waits are bounded: on timeout the
// kernel records an error and skips the tile instead of hanging.
// Math: S[h][t] = Q[h] . K[t] with mma.m16n8k16 (query heads of the KV group
// stacked in M, padded to 16), online softmax on the accumulator fragments
// (row max/sum over the 4 lanes of a row), then O[h] += P[h][t] V[t] reusing
// the score fragments as the A operand; V fragments via ldmatrix.trans.
#pragma once

#include <cuda.h>

#include "attention.cuh"
#include "common.cuh"
#include "tma.cuh"

namespace cheetah {

constexpr int kMmaWarps = 4;
constexpr int kMmaThreads = kMmaWarps * kWarp;
constexpr int kMmaStages = 3;
constexpr int kTileBytes = 8192;  // one K (or V) tile: TILE rows x head_dim bf16

template <int HD>
struct MmaTile {
    static constexpr int kRows = kTileBytes / (HD * 2);  // 64 for d=64, 32 for d=128
    static constexpr int kNTiles = kRows / 8;            // score n-tiles per tile
    static constexpr int kKSteps = HD / 16;              // d k-steps for QK
    static constexpr int kChunks = HD / 8;               // 16-byte chunks per row
};

struct MmaAttnParams {
    AttnParams a;
    long long layer_row_offset;  // rows of the pool before this layer's pages
    int page_tokens;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128B-swizzled tile whose
// rows are split into 128-byte halves stored as separate sub-tiles.
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
    constexpr int kRows = MmaTile<HD>::kRows;
    return (uint32_t)((c >> 3) * (kRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(kMmaThreads, 1)
    decode_attention_mma_kernel(const __grid_constant__ CUtensorMap k_map,
                                const __grid_constant__ CUtensorMap v_map, const MmaAttnParams mp) {
    using T = MmaTile<HD>;
    constexpr int TILE = T::kRows;
    extern __shared__ __align__(1024) uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bars[kMmaWarps][kMmaStages];
    __shared__ float m_s[kMmaWarps][kMaxGroup];
    __shared__ float l_s[kMmaWarps][kMaxGroup];
    __shared__ __align__(16) float o_s[kMmaWarps][kMaxGroup][HD];
    __shared__ float w_s[kMaxSplits][kMaxGroup];
    __shared__ float big_l[kMaxGroup];
    __shared__ int is_last;
    __shared__ int page_s[kMmaWarps][kMmaStages];  // page of the tile in each stage

    const AttnParams &p = mp.a;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y;
    const int b = blockIdx.z;
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int g = lane >> 2;   // fragment row (query head within the group)
    const int c = lane & 3;    // fragment column pair
    const int group = p.q_heads / p.kv_heads;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
    uint8_t *warp_smem = base + warp * kMmaStages * 2 * kTileBytes;

    if (lane == 0) {
        for (int s = 0; s < kMmaStages; ++s) mbar_init(smem_u32(&bars[warp][s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    pdl_wait();
    pdl_launch_dependents();

    const int L = p.seq_lens[b];
    int ws = 0;
    if (p.window > 0) ws = L > p.window ? L - p.window : 0;
    if (ws > L - 1) ws = L > 0 ? L - 1 : 0;
    // Tile grid aligned to absolute positions (tiles never straddle a page).
    const int tile_lo = ws / TILE;
    const int tile_hi = L > 0 ? (L + TILE - 1) / TILE : tile_lo + 1;
    const int n_tiles = tile_hi - tile_lo;
    int per = (n_tiles + p.splits - 1) / p.splits;
    per = max(per, kMmaWarps);
    const int active = (n_tiles + per - 1) / per;
    if (split >= active) return;
    const int t_begin = tile_lo + split * per;
    const int t_end = min(tile_hi, t_begin + per);
    const int my_count = t_end - t_begin > warp ? (t_end - t_begin - warp + kMmaWarps - 1) / kMmaWarps : 0;
    const int32_t *table = p.page_table + (long long)b * p.max_pages;

    // Page of this warp's tiles i0 .. i0 + 31 (lane j: tile i0 + j): one
    // coalesced page-table read per 32 tiles, so issuing a tile's loads never
    // waits on a dependent global read. Called by all lanes, i warp-uniform.
    int pg_lane = -1, pg_i0 = -1;
    auto page_for = [&](int i) -> int {
        const int i0 = i & ~(kWarp - 1);
        if (i0 != pg_i0) {
            pg_i0 = i0;
            const int ti = i0 + lane;
            pg_lane = -1;
            if (ti < my_count) {
                const int pidx = (t_begin + warp + ti * kMmaWarps) * TILE / mp.page_tokens;
                pg_lane = pidx < p.max_pages ? table[pidx] : -1;
            }
        }
        return __shfl_sync(0xFFFFFFFFu, pg_lane, i & (kWarp - 1));
    };

    // Issue the TMA loads of this warp's i-th tile (on `page`) into stage
    // i % kMmaStages.
    auto issue = [&](int i, int page) {
        const int tile = t_begin + warp + i * kMmaWarps;
        const int stage = i % kMmaStages;
        const uint32_t bar = smem_u32(&bars[warp][stage]);
        const int pos0 = tile * TILE;
        const int pidx = pos0 / mp.page_tokens;
        page_s[warp][stage] = page;
        if (page < 0 || page >= p.num_pages) {
            if (p.error) *p.error = 1;
            mbar_arrive(bar);  // complete the phase without data; the tile is masked
            return;
        }
        const int row = (int)(mp.layer_row_offset + ((long long)page * p.kv_heads + kvh) * mp.page_tokens +
                              (pos0 - pidx * mp.page_tokens));
        uint8_t *ks = warp_smem + stage * 2 * kTileBytes;
        uint8_t *vs = ks + kTileBytes;
        mbar_expect_tx(bar, 2 * kTileBytes);
#pragma unroll
        for (int half = 0; half < HD / 64; ++half) {
            tma_load_2d(smem_u32(ks + half * TILE * 128), &k_map, half * 64, row, bar);
            tma_load_2d(smem_u32(vs + half * TILE * 128), &v_map, half * 64, row, bar);
        }
    };

    {
        int pg0[kMmaStages];
#pragma unroll
        for (int i = 0; i < kMmaStages; ++i) pg0[i] = page_for(i);
        if (lane == 0) {
            for (int i = 0; i < kMmaStages && i < my_count; ++i) issue(i, pg0[i]);
        }
        __syncwarp();
    }

    // Q as bf16 A fragments (rows >= group are zero padding).
    uint32_t qa[T::kKSteps][2];
    {
        const float *qrow = p.q + ((long long)b * p.q_heads + kvh * group + g) * HD;
        const bool real = g < group;
#pragma unroll
        for (int ks = 0; ks < T::kKSteps; ++ks) {
            float2 lo = real ? *reinterpret_cast<const float2 *>(qrow + ks * 16 + 2 * c) : make_float2(0.f, 0.f);
            float2 hi = real ? *reinterpret_cast<const float2 *>(qrow + ks * 16 + 8 + 2 * c) : make_float2(0.f, 0.f);
            qa[ks][0] = pack_bf16(lo.x, lo.y);
            qa[ks][1] = pack_bf16(hi.x, hi.y);
        }
    }
    const float scale_log2 = p.scale * 1.4426950408889634f;

    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_run = -INFINITY;  // in log2 units
    float l_run = 0.0f;
    bool failed = false;
    int fail_at = 0;

    for (int i = 0; i < my_count; ++i) {
        const int stage = i % kMmaStages;
        const uint32_t parity = (i / kMmaStages) & 1;
        const int tile = t_begin + warp + i * kMmaWarps;
        const int pos0 = tile * TILE;
        // Warp-uniform: once any lane saw the phase complete, it is complete.
        const bool ok = __any_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bars[warp][stage]), parity));
        if (!ok) {
            fail_at = i;
            if (p.error) *p.error = 2;
            failed = true;
            break;
        }
        const int page = page_s[warp][stage];
        const bool tile_ok = page >= 0 && page < p.num_pages;
        const uint32_t ks_base = smem_u32(warp_smem + stage * 2 * kTileBytes);
        const uint32_t vs_base = ks_base + kTileBytes;

        // S = Q K^T over the tile: kNTiles fragments of 8 positions.
        float s[T::kNTiles][4];
#pragma unroll
        for (int n = 0; n < T::kNTiles; ++n) {
            s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
            const int r = n * 8 + (lane & 7);
#pragma unroll
            for (int kc = 0; kc < T::kChunks; kc += 4) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(ks_base + swz<HD>(r, kc + (lane >> 3)), b0, b1, b2, b3);
                mma_bf16(s[n], qa[kc / 2][0], 0u, qa[kc / 2][1], 0u, b0, b1);
                mma_bf16(s[n], qa[kc / 2 + 1][0], 0u, qa[kc / 2 + 1][1], 0u, b2, b3);
            }
        }
        // Online softmax over this tile (row g; the 4 lanes of a row share it).
        float tmax = -INFINITY;
#pragma unroll
        for (int n = 0; n < T::kNTiles; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int pos = pos0 + n * 8 + 2 * c + e;
                const bool vis = tile_ok && pos >= ws && pos < L;
                const float v = vis ? s[n][e] * scale_log2 : -INFINITY;
                s[n][e] = v;
                tmax = fmaxf(tmax, v);
            }
        }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        const float corr = (m_new == -INFINITY) ? 1.0f : exp2f(m_run - m_new);
        float tsum = 0.0f;
        uint32_t pa[T::kNTiles];
#pragma unroll
        for (int n = 0; n < T::kNTiles; ++n) {
            const float p0 = (m_new == -INFINITY) ? 0.0f : exp2f(s[n][0] - m_new);
            const float p1 = (m_new == -INFINITY) ? 0.0f : exp2f(s[n][1] - m_new);
            tsum += p0 + p1;
            pa[n] = pack_bf16(p0, p1);
        }
        tsum += __shfl_xor_sync(0xFFFFFFFFu, tsum, 1);
        tsum += __shfl_xor_sync(0xFFFFFFFFu, tsum, 2);
        l_run = l_run * corr + tsum;
        m_run = m_new;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            o[j][0] *= corr;
            o[j][1] *= corr;
        }
        // O += P V: k-steps of 16 positions, V fragments by ldmatrix.trans.
#pragma unroll
        for (int kk = 0; kk < T::kNTiles / 2; ++kk) {
            const int blk = lane >> 3;
            const int r = kk * 16 + (lane & 7) + 8 * (blk & 1);
#pragma unroll
            for (int j = 0; j < HD / 8; j += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vs_base + swz<HD>(r, j + (blk >> 1)), b0, b1, b2, b3);
                mma_bf16(o[j], pa[2 * kk], 0u, pa[2 * kk + 1], 0u, b0, b1);
                mma_bf16(o[j + 1], pa[2 * kk], 0u, pa[2 * kk + 1], 0u, b2, b3);
            }
        }
        __syncwarp();
        if (i + kMmaStages < my_count) {
            const int pg = page_for(i + kMmaStages);
            if (lane == 0) issue(i + kMmaStages, pg);
            __syncwarp();
        }
    }
    if (failed) {
        // Drain this warp's loads still in flight (bounded) before exiting.
        if (lane == 0) {
            const int issued = min(my_count, fail_at + kMmaStages);
            for (int k = fail_at; k < issued; ++k) {
                (void)mbar_wait(smem_u32(&bars[warp][k % kMmaStages]), (k / kMmaStages) & 1);
            }
        }
        m_run = -INFINITY;
        l_run = 0.0f;
    }

    // Per-warp results -> shared memory, then the split merge.
    if (c == 0) {
        if (g < kMaxGroup) {
            m_s[warp][g] = m_run == -INFINITY ? -INFINITY : m_run / 1.4426950408889634f;
            l_s[warp][g] = l_run;
        }
    }
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
        if (g < kMaxGroup) {
            o_s[warp][g][j * 8 + 2 * c] = failed ? 0.0f : o[j][0];
            o_s[warp][g][j * 8 + 2 * c + 1] = failed ? 0.0f : o[j][1];
        }
    }
    __syncthreads();
    merge_splits<HD, kMmaWarps>(p, b, kvh, split, active, group, m_s, l_s, o_s, w_s, big_l, &is_last);
}

inline size_t mma_attention_smem() { return (size_t)kMmaWarps * kMmaStages * 2 * kTileBytes + 1024; }

}  // namespace cheetah
