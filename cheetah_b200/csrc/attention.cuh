// Paged GQA decode attention (split-K flash-decode), one query per sequence.
//
// Math of `OpsToolbox::attention_head` (`ops.rs:1424-1467`): per query head
// h (kv head h / group) scores = (q . k) * 1/sqrt(d) over the visible window
// (`ops.rs:1366-1372`), softmax (max-subtract, exp, normalise), weighted sum
// of V. Computed as an online softmax (running max / sum, rescaled partial
// outputs) so the KV length can split across CTAs; equal to the reference up
// to rounding.
//
// Grid (splits, kv_heads, batch): each CTA walks a contiguous span of
// positions for one KV head and serves all `group` query heads that share
// it, so every K/V byte is read once. Lane-per-position scores (the whole K
// row requested with 128-bit loads before use, q broadcast from shared
// memory), lane-per-dimension value mix (16 V rows in flight). The active
// split count follows the live length (>= 128 positions per CTA); CTAs past
// it exit. The last CTA of each (sequence, kv head) to finish merges the
// split partials (threadfence + atomic ticket, no spin-wait) and resets the
// ticket for the next launch. This CUDA-core kernel serves the f32 cache;
// the bf16 cache takes the tensor-core kernel in attention_mma.cuh.
#pragma once

#include "common.cuh"

namespace cheetah {

struct AttnParams {
    const float *q;            // [batch][q_heads][head_dim]
    const void *k_pool;        // [pages][kv_heads][page_tokens][head_dim]
    const void *v_pool;
    const int32_t *page_table; // [batch][max_pages]
    const int32_t *seq_lens;   // [batch]
    int max_pages;
    int num_pages;
    int page_tokens;
    int batch;
    int q_heads;
    int kv_heads;
    int window;
    int splits;
    float scale;
    float *out;                // [batch][q_heads][head_dim]
    // scratch (global memory beyond inputs/outputs)
    float *part_o;             // [batch][kv_heads][splits][kMaxGroup][head_dim]
    float *part_ml;            // [batch][kv_heads][splits][kMaxGroup][2]
    unsigned int *tickets;     // [batch][kv_heads], zero between launches
    int *error;                // nullable: set to 1 on an out-of-range page id
    uint16_t *out_bf16;        // nullable: write the result as bf16 here instead of `out`
};

__device__ __forceinline__ void store_attn_out(const AttnParams &p, long long index, float value) {
    if (p.out_bf16) p.out_bf16[index] = f32_to_bf16_rne(value);
    else p.out[index] = value;
}

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / kWarp;
constexpr int kMaxGroup = 8;
constexpr int kMinChunk = kAttnWarps * kWarp;  // positions per CTA at least
constexpr int kMaxSplits = 256;

template <int HD, bool KV_F32>
__device__ __forceinline__ void load_k_chunk(const void *pool, long long row, int c, float *out8) {
    if (KV_F32) {
        const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(pool) + row * HD + c * 8);
        const float4 a = __ldg(src), b = __ldg(src + 1);
        out8[0] = a.x; out8[1] = a.y; out8[2] = a.z; out8[3] = a.w;
        out8[4] = b.x; out8[5] = b.y; out8[6] = b.z; out8[7] = b.w;
    } else {
        const uint4 w = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(pool) + row * HD + c * 8));
        out8[0] = bf16_lo(w.x); out8[1] = bf16_hi(w.x);
        out8[2] = bf16_lo(w.y); out8[3] = bf16_hi(w.y);
        out8[4] = bf16_lo(w.z); out8[5] = bf16_hi(w.z);
        out8[6] = bf16_lo(w.w); out8[7] = bf16_hi(w.w);
    }
}

template <int HD, bool KV_F32>
__device__ __forceinline__ void load_v_lane(const void *pool, long long row, int lane, float *out) {
    constexpr int DPL = HD / kWarp;  // 2 or 4 dims per lane
    if (KV_F32) {
        const float *src = static_cast<const float *>(pool) + row * HD + lane * DPL;
        if (DPL == 2) {
            const float2 v = __ldg(reinterpret_cast<const float2 *>(src));
            out[0] = v.x; out[1] = v.y;
        } else {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(src));
            out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
        }
    } else {
        const uint16_t *src = static_cast<const uint16_t *>(pool) + row * HD + lane * DPL;
        if (DPL == 2) {
            const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(src));
            out[0] = bf16_lo(w); out[1] = bf16_hi(w);
        } else {
            const uint2 w = __ldg(reinterpret_cast<const uint2 *>(src));
            out[0] = bf16_lo(w.x); out[1] = bf16_hi(w.x); out[2] = bf16_lo(w.y); out[3] = bf16_hi(w.y);
        }
    }
}

// Active split count for a visible span: at least kMinChunk positions per
// CTA (one 32-position tile per warp), at most `splits`. Every CTA of a
// (sequence, kv head) derives the same value from the same length.
__device__ __forceinline__ void split_range(int span, int splits, int split, int &active, int &chunk) {
    chunk = (span + splits - 1) / splits;
    chunk = (chunk + kWarp - 1) / kWarp * kWarp;
    chunk = max(chunk, kMinChunk);
    active = span > 0 ? (span + chunk - 1) / chunk : 1;
}

// Merge this CTA's partial (m, l, o) into the per-split scratch, then the
// last CTA to arrive merges all active splits into `out`.
template <int HD, int NW = kAttnWarps>
__device__ __forceinline__ void merge_splits(const AttnParams &p, int b, int kvh, int split, int active,
                                             int group, float (*m_s)[kMaxGroup], float (*l_s)[kMaxGroup],
                                             float (*o_s)[kMaxGroup][HD], float (*w_s)[kMaxGroup],
                                             float *big_l, int *is_last) {
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const long long base = ((long long)b * p.kv_heads + kvh) * p.splits;
    const long long part = base + split;
    for (int i = threadIdx.x; i < group * HD; i += (NW * kWarp)) {
        const int g = i / HD, d = i % HD;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) m = fmaxf(m, m_s[w][g]);
        float l = 0.0f, o = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float f = (m == -INFINITY) ? 0.0f : expf(m_s[w][g] - m);
            l += l_s[w][g] * f;
            o += o_s[w][g][d] * f;
        }
        if (active == 1) {
            store_attn_out(p, ((long long)b * p.q_heads + kvh * group + g) * HD + d, l > 0.0f ? o / l : 0.0f);
        } else {
            p.part_o[(part * kMaxGroup + g) * HD + d] = o;
            if (d == 0) {
                p.part_ml[(part * kMaxGroup + g) * 2 + 0] = m;
                p.part_ml[(part * kMaxGroup + g) * 2 + 1] = l;
            }
        }
    }
    if (active == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int *ticket = p.tickets + (long long)b * p.kv_heads + kvh;
        const unsigned int prev = atomicAdd(ticket, 1u);
        *is_last = (prev == (unsigned)active - 1);
        if (*is_last) *ticket = 0u;
    }
    __syncthreads();
    if (!*is_last) return;
    __threadfence();
    // Per-head global max and split weights (warp g handles heads g, g+4):
    // every split's (m, l) is loaded at once (kMaxSplits / 32 per lane), so
    // the pass costs one L2 round trip; each lane folds its splits in split
    // order before the warp sum.
    constexpr int kPerLane = kMaxSplits / kWarp;
    for (int g = warp; g < group; g += NW) {
        float ms[kPerLane], ls[kPerLane];
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const int s2 = lane + k * kWarp;
            const bool in = s2 < active;
            ms[k] = in ? __ldcg(&p.part_ml[((base + s2) * kMaxGroup + g) * 2]) : -INFINITY;
            ls[k] = in ? __ldcg(&p.part_ml[((base + s2) * kMaxGroup + g) * 2 + 1]) : 0.0f;
        }
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) m = fmaxf(m, ms[k]);
        m = warp_max(m);
        float l = 0.0f;
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            const int s2 = lane + k * kWarp;
            if (s2 < active) {
                const float w = (m == -INFINITY) ? 0.0f : expf(ms[k] - m);
                w_s[s2][g] = w;
                l += w * ls[k];
            }
        }
        l = warp_sum(l);
        if (lane == 0) big_l[g] = l;
    }
    __syncthreads();
    // Weighted sum of the split outputs, four dimensions per thread, split
    // order; 16 splits' loads in flight at a time.
    for (int i = threadIdx.x; i < group * (HD / 4); i += (NW * kWarp)) {
        const int g = i / (HD / 4), d4 = i % (HD / 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 *src = reinterpret_cast<const float4 *>(p.part_o + ((base * kMaxGroup) + g) * HD) + d4;
        const long long stride4 = (long long)kMaxGroup * HD / 4;
        constexpr int kB = 16;
        for (int s2 = 0; s2 < active; s2 += kB) {
            float4 v[kB];
#pragma unroll
            for (int u = 0; u < kB; ++u)
                v[u] = s2 + u < active ? __ldcg(src + (s2 + u) * stride4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < kB; ++u) {
                if (s2 + u < active) {
                    const float w = w_s[s2 + u][g];
                    acc.x = fmaf(w, v[u].x, acc.x); acc.y = fmaf(w, v[u].y, acc.y);
                    acc.z = fmaf(w, v[u].z, acc.z); acc.w = fmaf(w, v[u].w, acc.w);
                }
            }
        }
        const float l = big_l[g];
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        float4 r = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        if (!(l > 0.0f)) r = make_float4(0.f, 0.f, 0.f, 0.f);
        const long long o0 = ((long long)b * p.q_heads + kvh * group + g) * HD + d4 * 4;
        if (p.out_bf16) {
            store_attn_out(p, o0, r.x);
            store_attn_out(p, o0 + 1, r.y);
            store_attn_out(p, o0 + 2, r.z);
            store_attn_out(p, o0 + 3, r.w);
        } else {
            reinterpret_cast<float4 *>(p.out + o0)[0] = r;
        }
    }
}

template <int HD, bool KV_F32>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(const AttnParams p) {
    constexpr int DPL = HD / kWarp;
    constexpr int CHUNKS = HD / 8;  // 8-element chunks per row
    __shared__ __align__(16) float q_s[kMaxGroup][HD];
    __shared__ __align__(16) float p_s[kAttnWarps][kWarp][kMaxGroup];
    __shared__ float m_s[kAttnWarps][kMaxGroup];
    __shared__ float l_s[kAttnWarps][kMaxGroup];
    __shared__ __align__(16) float o_s[kAttnWarps][kMaxGroup][HD];
    __shared__ float w_s[kMaxSplits][kMaxGroup];
    __shared__ float big_l[kMaxGroup];
    __shared__ int is_last;

    const int split = blockIdx.x;
    const int kvh = blockIdx.y;
    const int b = blockIdx.z;
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int group = p.q_heads / p.kv_heads;

    pdl_wait();
    pdl_launch_dependents();

    const int L = p.seq_lens[b];
    int ws = 0;
    if (p.window > 0) ws = L > p.window ? L - p.window : 0;
    if (ws > L - 1) ws = L > 0 ? L - 1 : 0;
    const int span = L - ws;
    int active, chunk;
    split_range(span, p.splits, split, active, chunk);
    if (split >= active) return;
    const int begin = ws + split * chunk;
    const int end = min(L, begin + chunk);

    for (int i = threadIdx.x; i < group * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        q_s[g][d] = p.q[((long long)b * p.q_heads + kvh * group + g) * HD + d];
    }
    __syncthreads();

    float m_run[kMaxGroup], l_run[kMaxGroup], o_run[kMaxGroup][DPL];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o_run[g][e] = 0.0f;
    }

    const int32_t *table = p.page_table + (long long)b * p.max_pages;
    for (int t0 = begin + warp * kWarp; t0 < end; t0 += kAttnWarps * kWarp) {
        const int pos = t0 + lane;
        const bool valid = pos < end;
        long long row = 0;
        if (valid) {
            const int page = pos / p.page_tokens < p.max_pages ? table[pos / p.page_tokens] : -1;
            if (page < 0 || page >= p.num_pages) {
                if (p.error) *p.error = 1;
            } else {
                row = ((long long)page * p.kv_heads + kvh) * p.page_tokens + (pos % p.page_tokens);
            }
        }
        // Scores: the whole K row is requested before any arithmetic.
        float s[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) s[g] = 0.0f;
        if (valid) {
#pragma unroll
            for (int c0 = 0; c0 < CHUNKS; c0 += 8) {
                float k8[8][8];
#pragma unroll
                for (int c = 0; c < 8; ++c) load_k_chunk<HD, KV_F32>(p.k_pool, row, c0 + c, k8[c]);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
#pragma unroll
                    for (int g = 0; g < kMaxGroup; ++g) {
                        if (g < group) {
                            const float4 qa = *reinterpret_cast<const float4 *>(&q_s[g][(c0 + c) * 8]);
                            const float4 qb = *reinterpret_cast<const float4 *>(&q_s[g][(c0 + c) * 8 + 4]);
                            float acc = s[g];
                            acc = fmaf(k8[c][0], qa.x, acc); acc = fmaf(k8[c][1], qa.y, acc);
                            acc = fmaf(k8[c][2], qa.z, acc); acc = fmaf(k8[c][3], qa.w, acc);
                            acc = fmaf(k8[c][4], qb.x, acc); acc = fmaf(k8[c][5], qb.y, acc);
                            acc = fmaf(k8[c][6], qb.z, acc); acc = fmaf(k8[c][7], qb.w, acc);
                            s[g] = acc;
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
            if (g < group) {
                const float score = valid ? s[g] * p.scale : -INFINITY;
                const float m_new = fmaxf(m_run[g], warp_max(score));
                const float pr = (valid && m_new != -INFINITY) ? expf(score - m_new) : 0.0f;
                const float corr = (m_new == -INFINITY) ? 1.0f : expf(m_run[g] - m_new);
                l_run[g] = l_run[g] * corr + warp_sum(pr);
#pragma unroll
                for (int e = 0; e < DPL; ++e) o_run[g][e] *= corr;
                m_run[g] = m_new;
                p_s[warp][lane][g] = pr;
            }
        }
        __syncwarp();
        // Value mix: 16 V rows requested at a time, then the FMAs.
        const int count = min(kWarp, end - t0);
#pragma unroll
        for (int j0 = 0; j0 < kWarp; j0 += 16) {
            if (j0 < count) {
                float v[16][DPL];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const long long vrow = __shfl_sync(0xFFFFFFFFu, row, j0 + j);
                    if (j0 + j < count) {
                        load_v_lane<HD, KV_F32>(p.v_pool, vrow, lane, v[j]);
                    } else {
#pragma unroll
                        for (int e = 0; e < DPL; ++e) v[j][e] = 0.0f;
                    }
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 pa = *reinterpret_cast<const float4 *>(&p_s[warp][j0 + j][0]);
                    const float4 pb = *reinterpret_cast<const float4 *>(&p_s[warp][j0 + j][4]);
                    const float pj[kMaxGroup] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                    for (int g = 0; g < kMaxGroup; ++g) {
                        if (g < group) {
#pragma unroll
                            for (int e = 0; e < DPL; ++e) o_run[g][e] = fmaf(pj[g], v[j][e], o_run[g][e]);
                        }
                    }
                }
            }
        }
        __syncwarp();
    }

    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
            m_s[warp][g] = m_run[g];
            l_s[warp][g] = l_run[g];
        }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
#pragma unroll
        for (int e = 0; e < DPL; ++e) o_s[warp][g][lane * DPL + e] = o_run[g][e];
    }
    __syncthreads();
    merge_splits<HD>(p, b, kvh, split, active, group, m_s, l_s, o_s, w_s, big_l, &is_last);
}

}  // namespace cheetah
