// Causal GQA attention for a prefill chunk over the paged KV cache (cached
// prefix + the chunk's own keys), the batched form of the reference's
// per-row loop `forward_layer_chunk` (`qwen2.rs:314-343`: append row r's K/V,
// then attend position r) — equal up to rounding: q and the softmax weights
// are bf16 for the MMAs, f32 accumulation and online softmax.
//
// CTA = 16 consecutive tokens x one KV head; warp w serves query head
// kv_head * group + w over those 16 tokens (the mma M dimension), so each
// K/V tile is fetched once (TMA, 128-byte swizzle, 3-stage ring completed
// on mbarriers, bounded waits) and used by every query head of the group.
// S = Q K^T and O += P V with mma.m16n8k16 (bf16 -> f32), causal and window
// masks applied per (token, key) on the score fragments. A CTA barrier after
// each tile frees its stage for the next TMA load. The key range of a token
// block splits over blockIdx.z so the grid covers every SM; the splits are
// merged by prefill_merge_kernel.
#pragma once

#include "attention_mma.cuh"

namespace cheetah {

constexpr int kPrefillStages = 3;
constexpr int kPrefillWarps = 8;
constexpr int kPrefillMaxSplits = 8;

struct PrefillAttnParams {
    const uint16_t *q;        // bf16 [T][q_heads * head_dim], RoPE applied
    uint16_t *out;            // bf16 [T][q_heads * head_dim]
    int T;
    int offset;               // absolute position of token 0
    int q_heads, kv_heads;
    const int32_t *page_table;
    int max_pages, num_pages, page_tokens;
    long long layer_row_offset;
    int window;
    float scale;
    int *error;
    // Key-range split: blockIdx.z of `splits` takes a contiguous share of the
    // key tiles; with splits > 1 the CTA writes unnormalised partials
    // (O, and m in log2 units, l) that prefill_merge_kernel combines.
    int splits;
    float *part_o;            // [splits][T][q_heads][head_dim]
    float *part_ml;           // [splits][T][q_heads][2]
};

template <int HD>
__global__ void __launch_bounds__(kPrefillWarps * kWarp, HD == 64 ? 2 : 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
                             const PrefillAttnParams p) {
    using TL = MmaTile<HD>;
    constexpr int TILE = TL::kRows;
    extern __shared__ __align__(1024) uint8_t psmem[];
    __shared__ __align__(8) uint64_t full_bar[kPrefillStages];

    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(psmem) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int g = lane >> 2, c = lane & 3;
    const int group = p.q_heads / p.kv_heads;
    const int kvh = blockIdx.y;
    const int t0 = blockIdx.x * 16;
    const int t_last = min(p.T, t0 + 16) - 1;
    const int head = kvh * group + warp;
    const bool active = warp < group;
    const int q_stride = p.q_heads * HD;

    const int pos_first = p.offset + t0;
    const int pos_last = p.offset + t_last;
    int ws = 0;
    if (p.window > 0) ws = max(0, pos_first + 1 - p.window);
    const int all_lo = ws / TILE;
    const int all_hi = pos_last / TILE + 1;
    const int per_split = (all_hi - all_lo + p.splits - 1) / p.splits;
    const int split = blockIdx.z;
    const int tile_lo = all_lo + split * per_split;
    const int tile_hi = min(all_hi, tile_lo + per_split);
    const int n_tiles = max(0, tile_hi - tile_lo);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPrefillStages; ++s) mbar_init(smem_u32(&full_bar[s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();

    auto issue = [&](int i) {
        const int tile = tile_lo + i;
        const int s = i % kPrefillStages;
        const uint32_t bar = smem_u32(&full_bar[s]);
        const int pos0 = tile * TILE;
        const int pidx = pos0 / p.page_tokens;
        const int page = pidx < p.max_pages ? p.page_table[pidx] : -1;
        if (page < 0 || page >= p.num_pages) {
            if (p.error) *p.error = 6;
            mbar_arrive(bar);
            return;
        }
        const int row = (int)(p.layer_row_offset + ((long long)page * p.kv_heads + kvh) * p.page_tokens +
                              (pos0 - pidx * p.page_tokens));
        uint8_t *ks = ring + s * 2 * kTileBytes;
        uint8_t *vs = ks + kTileBytes;
        mbar_expect_tx(bar, 2 * kTileBytes);
#pragma unroll
        for (int half = 0; half < HD / 64; ++half) {
            tma_load_2d(smem_u32(ks + half * TILE * 128), &k_map, half * 64, row, bar);
            tma_load_2d(smem_u32(vs + half * TILE * 128), &v_map, half * 64, row, bar);
        }
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < kPrefillStages && i < n_tiles; ++i) issue(i);
    }

    // Q fragments (rows = tokens t0 + g and t0 + g + 8).
    uint32_t qa[TL::kKSteps][4];
    {
        const bool r0 = active && t0 + g <= t_last;
        const bool r1 = active && t0 + g + 8 <= t_last;
        const uint16_t *q0 = p.q + (long long)(t0 + g) * q_stride + head * HD;
        const uint16_t *q1 = p.q + (long long)(t0 + g + 8) * q_stride + head * HD;
#pragma unroll
        for (int ks = 0; ks < TL::kKSteps; ++ks) {
            qa[ks][0] = r0 ? *reinterpret_cast<const uint32_t *>(q0 + ks * 16 + 2 * c) : 0u;
            qa[ks][1] = r1 ? *reinterpret_cast<const uint32_t *>(q1 + ks * 16 + 2 * c) : 0u;
            qa[ks][2] = r0 ? *reinterpret_cast<const uint32_t *>(q0 + ks * 16 + 8 + 2 * c) : 0u;
            qa[ks][3] = r1 ? *reinterpret_cast<const uint32_t *>(q1 + ks * 16 + 8 + 2 * c) : 0u;
        }
    }
    const float scale_log2 = p.scale * 1.4426950408889634f;
    const int qpos0 = p.offset + t0 + g;  // query position of fragment row g
    const int qpos1 = qpos0 + 8;

    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    bool failed = false;

    for (int i = 0; i < n_tiles; ++i) {
        const int s = i % kPrefillStages;
        const uint32_t round = i / kPrefillStages;
        if (!__syncthreads_or(mbar_wait(smem_u32(&full_bar[s]), round & 1))) {
            failed = true;
            break;
        }
        const int pos0 = (tile_lo + i) * TILE;
        if (active) {
            const uint32_t ks_base = smem_u32(ring + s * 2 * kTileBytes);
            const uint32_t vs_base = ks_base + kTileBytes;
            float sc[TL::kNTiles][4];
#pragma unroll
            for (int n = 0; n < TL::kNTiles; ++n) {
                sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
                const int r = n * 8 + (lane & 7);
#pragma unroll
                for (int kc = 0; kc < TL::kChunks; kc += 4) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(ks_base + swz<HD>(r, kc + (lane >> 3)), b0, b1, b2, b3);
                    mma_bf16(sc[n], qa[kc / 2][0], qa[kc / 2][1], qa[kc / 2][2], qa[kc / 2][3], b0, b1);
                    mma_bf16(sc[n], qa[kc / 2 + 1][0], qa[kc / 2 + 1][1], qa[kc / 2 + 1][2], qa[kc / 2 + 1][3], b2, b3);
                }
            }
            float tmax0 = -INFINITY, tmax1 = -INFINITY;
#pragma unroll
            for (int n = 0; n < TL::kNTiles; ++n) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int kp = pos0 + n * 8 + 2 * c + e;
                    const bool vis0 = kp <= qpos0 && kp >= ws && (p.window == 0 || kp > qpos0 - p.window);
                    const bool vis1 = kp <= qpos1 && kp >= ws && (p.window == 0 || kp > qpos1 - p.window);
                    sc[n][e] = vis0 ? sc[n][e] * scale_log2 : -INFINITY;
                    sc[n][2 + e] = vis1 ? sc[n][2 + e] * scale_log2 : -INFINITY;
                    tmax0 = fmaxf(tmax0, sc[n][e]);
                    tmax1 = fmaxf(tmax1, sc[n][2 + e]);
                }
            }
            tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xFFFFFFFFu, tmax0, 1));
            tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xFFFFFFFFu, tmax0, 2));
            tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xFFFFFFFFu, tmax1, 1));
            tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xFFFFFFFFu, tmax1, 2));
            const float mn0 = fmaxf(m0, tmax0), mn1 = fmaxf(m1, tmax1);
            const float cr0 = mn0 == -INFINITY ? 1.0f : exp2f(m0 - mn0);
            const float cr1 = mn1 == -INFINITY ? 1.0f : exp2f(m1 - mn1);
            float s0 = 0.0f, s1 = 0.0f;
            uint32_t pa[TL::kNTiles][2];
#pragma unroll
            for (int n = 0; n < TL::kNTiles; ++n) {
                const float p00 = mn0 == -INFINITY ? 0.0f : exp2f(sc[n][0] - mn0);
                const float p01 = mn0 == -INFINITY ? 0.0f : exp2f(sc[n][1] - mn0);
                const float p10 = mn1 == -INFINITY ? 0.0f : exp2f(sc[n][2] - mn1);
                const float p11 = mn1 == -INFINITY ? 0.0f : exp2f(sc[n][3] - mn1);
                s0 += p00 + p01;
                s1 += p10 + p11;
                pa[n][0] = pack_bf16(p00, p01);
                pa[n][1] = pack_bf16(p10, p11);
            }
            s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 1);
            s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 2);
            s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
            s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 2);
            l0 = l0 * cr0 + s0;
            l1 = l1 * cr1 + s1;
            m0 = mn0;
            m1 = mn1;
#pragma unroll
            for (int j = 0; j < HD / 8; ++j) {
                o[j][0] *= cr0;
                o[j][1] *= cr0;
                o[j][2] *= cr1;
                o[j][3] *= cr1;
            }
#pragma unroll
            for (int kk = 0; kk < TL::kNTiles / 2; ++kk) {
                const int blk = lane >> 3;
                const int r = kk * 16 + (lane & 7) + 8 * (blk & 1);
#pragma unroll
                for (int j = 0; j < HD / 8; j += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(vs_base + swz<HD>(r, j + (blk >> 1)), b0, b1, b2, b3);
                    mma_bf16(o[j], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
                    mma_bf16(o[j + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b2, b3);
                }
            }
        }
        __syncthreads();  // every warp is done with stage s
        if (threadIdx.x == 0 && i + kPrefillStages < n_tiles) issue(i + kPrefillStages);
    }
    if (failed) {
        if (p.error) *p.error = 8;
        return;
    }
    if (!active) return;
    if (p.splits > 1) {
        const bool r0 = t0 + g <= t_last, r1 = t0 + g + 8 <= t_last;
        const long long base0 = (((long long)split * p.T + t0 + g) * p.q_heads + head);
        const long long base1 = (((long long)split * p.T + t0 + g + 8) * p.q_heads + head);
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            if (r0) *reinterpret_cast<float2 *>(p.part_o + base0 * HD + j * 8 + 2 * c) = make_float2(o[j][0], o[j][1]);
            if (r1) *reinterpret_cast<float2 *>(p.part_o + base1 * HD + j * 8 + 2 * c) = make_float2(o[j][2], o[j][3]);
        }
        if (c == 0) {
            if (r0) *reinterpret_cast<float2 *>(p.part_ml + base0 * 2) = make_float2(m0, l0);
            if (r1) *reinterpret_cast<float2 *>(p.part_ml + base1 * 2) = make_float2(m1, l1);
        }
        return;
    }
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f;
    const float inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    const bool r0 = t0 + g <= t_last, r1 = t0 + g + 8 <= t_last;
    uint16_t *out0 = p.out + (long long)(t0 + g) * q_stride + head * HD;
    uint16_t *out1 = p.out + (long long)(t0 + g + 8) * q_stride + head * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
        if (r0) *reinterpret_cast<uint32_t *>(out0 + j * 8 + 2 * c) = pack_bf16(o[j][0] * inv0, o[j][1] * inv0);
        if (r1) *reinterpret_cast<uint32_t *>(out1 + j * 8 + 2 * c) = pack_bf16(o[j][2] * inv1, o[j][3] * inv1);
    }
}

// Combine the key-range splits of prefill_attention_kernel: per (token, head)
// O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, written as bf16. The
// split loops are unrolled to kPrefillMaxSplits (guarded by p.splits) so a
// thread's loads of every split are in flight together; the arithmetic runs
// in split order.
template <int HD>
__global__ void prefill_merge_kernel(const PrefillAttnParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const long long rows = (long long)p.T * p.q_heads;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rows * (HD / 4);
         i += (long long)gridDim.x * blockDim.x) {
        const long long rh = i / (HD / 4);
        const int d4 = (int)(i % (HD / 4));
        float2 ml[kPrefillMaxSplits];
        float4 v[kPrefillMaxSplits];
#pragma unroll
        for (int s = 0; s < kPrefillMaxSplits; ++s) {
            if (s < p.splits) {
                ml[s] = *reinterpret_cast<const float2 *>(p.part_ml + ((long long)s * rows + rh) * 2);
                v[s] = reinterpret_cast<const float4 *>(p.part_o + ((long long)s * rows + rh) * HD)[d4];
            }
        }
        float m = -INFINITY;
#pragma unroll
        for (int s = 0; s < kPrefillMaxSplits; ++s) {
            if (s < p.splits) m = fmaxf(m, ml[s].x);
        }
        float l = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kPrefillMaxSplits; ++s) {
            if (s < p.splits) {
                const float w = m == -INFINITY ? 0.0f : exp2f(ml[s].x - m);
                l += w * ml[s].y;
                acc.x = fmaf(w, v[s].x, acc.x); acc.y = fmaf(w, v[s].y, acc.y);
                acc.z = fmaf(w, v[s].z, acc.z); acc.w = fmaf(w, v[s].w, acc.w);
            }
        }
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        uint16_t *out = p.out + rh * HD + d4 * 4;
        const uint32_t lo = (uint32_t)f32_to_bf16_rne(acc.x * inv) | ((uint32_t)f32_to_bf16_rne(acc.y * inv) << 16);
        const uint32_t hi = (uint32_t)f32_to_bf16_rne(acc.z * inv) | ((uint32_t)f32_to_bf16_rne(acc.w * inv) << 16);
        *reinterpret_cast<uint2 *>(out) = make_uint2(lo, hi);
    }
}

inline size_t prefill_attention_smem() { return (size_t)kPrefillStages * 2 * kTileBytes + 1024; }

// RMSNorm of f32 rows (`ops.rs:646-652`) into bf16 rows for the tensor cores.
__global__ void norm_rows_bf16_kernel(const float *__restrict__ x, int rows, int cols, const float *__restrict__ w,
                                      float eps, uint16_t *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float *xr = x + (long long)r * cols;
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) total += red[i];
    const float inv = 1.0f / sqrtf(total / (float)cols + eps);
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        out[(long long)r * cols + i] = f32_to_bf16_rne(__fmul_rn(xr[i], __fmul_rn(inv, w[i])));
    }
}

// Embedding rows of a chunk (`ops.rs:1083-1099`) into the f32 residual rows.
__global__ void embed_rows_kernel(const uint16_t *__restrict__ table, int hidden, const int32_t *__restrict__ tokens,
                                  int rows, float *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.x;
    if (r >= rows) return;
    const uint16_t *src = table + (long long)tokens[r] * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) out[(long long)r * hidden + i] = bf16_to_f32(src[i]);
}

}  // namespace cheetah
