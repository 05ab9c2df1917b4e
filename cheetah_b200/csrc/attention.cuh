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
// it, so every K/V byte is read once. Lane-per-position scores (K row read
// with 128-bit loads, q broadcast from shared memory), lane-per-dimension
// value mix. The last CTA of each (sequence, kv head) to finish merges the
// split partials (threadfence + atomic ticket, no spin-wait) and resets the
// ticket for the next launch.
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
};

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / kWarp;
constexpr int kMaxGroup = 8;

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

template <int HD, bool KV_F32>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(const AttnParams p) {
    constexpr int DPL = HD / kWarp;
    __shared__ __align__(16) float q_s[kMaxGroup][HD];
    __shared__ __align__(16) float p_s[kAttnWarps][kWarp][kMaxGroup];
    __shared__ float m_s[kAttnWarps][kMaxGroup];
    __shared__ float l_s[kAttnWarps][kMaxGroup];
    __shared__ __align__(16) float o_s[kAttnWarps][kMaxGroup][HD];
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
    int chunk = (span + p.splits - 1) / p.splits;
    chunk = (chunk + kWarp - 1) / kWarp * kWarp;
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
        float s[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) s[g] = 0.0f;
        if (valid) {
#pragma unroll 2
            for (int c = 0; c < HD / 8; ++c) {
                float k8[8];
                load_k_chunk<HD, KV_F32>(p.k_pool, row, c, k8);
#pragma unroll
                for (int g = 0; g < kMaxGroup; ++g) {
                    if (g < group) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&q_s[g][c * 8]);
                        const float4 qb = *reinterpret_cast<const float4 *>(&q_s[g][c * 8 + 4]);
                        float acc = s[g];
                        acc = fmaf(k8[0], qa.x, acc); acc = fmaf(k8[1], qa.y, acc);
                        acc = fmaf(k8[2], qa.z, acc); acc = fmaf(k8[3], qa.w, acc);
                        acc = fmaf(k8[4], qb.x, acc); acc = fmaf(k8[5], qb.y, acc);
                        acc = fmaf(k8[6], qb.z, acc); acc = fmaf(k8[7], qb.w, acc);
                        s[g] = acc;
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
        const int count = min(kWarp, end - t0);
        for (int j = 0; j < count; ++j) {
            const long long vrow = __shfl_sync(0xFFFFFFFFu, row, j);
            float v[DPL];
            load_v_lane<HD, KV_F32>(p.v_pool, vrow, lane, v);
            const float4 pa = *reinterpret_cast<const float4 *>(&p_s[warp][j][0]);
            const float4 pb = *reinterpret_cast<const float4 *>(&p_s[warp][j][4]);
            const float pj[kMaxGroup] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
            for (int g = 0; g < kMaxGroup; ++g) {
                if (g < group) {
#pragma unroll
                    for (int e = 0; e < DPL; ++e) o_run[g][e] = fmaf(pj[g], v[e], o_run[g][e]);
                }
            }
        }
        __syncwarp();
    }

    // Merge the warps of this CTA.
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

    const long long part = ((long long)b * p.kv_heads + kvh) * p.splits + split;
    for (int i = threadIdx.x; i < group * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) m = fmaxf(m, m_s[w][g]);
        float l = 0.0f, o = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = (m == -INFINITY) ? 0.0f : expf(m_s[w][g] - m);
            l += l_s[w][g] * f;
            o += o_s[w][g][d] * f;
        }
        p.part_o[(part * kMaxGroup + g) * HD + d] = o;
        if (d == 0) {
            p.part_ml[(part * kMaxGroup + g) * 2 + 0] = m;
            p.part_ml[(part * kMaxGroup + g) * 2 + 1] = l;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int *ticket = p.tickets + (long long)b * p.kv_heads + kvh;
        const unsigned int prev = atomicAdd(ticket, 1u);
        is_last = (prev == (unsigned)p.splits - 1);
        if (is_last) *ticket = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // Last CTA: merge all splits of this (sequence, kv head).
    const long long base = ((long long)b * p.kv_heads + kvh) * p.splits;
    for (int i = threadIdx.x; i < group * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        float m = -INFINITY;
        for (int s2 = 0; s2 < p.splits; ++s2) m = fmaxf(m, __ldcg(&p.part_ml[((base + s2) * kMaxGroup + g) * 2]));
        float l = 0.0f, o = 0.0f;
        for (int s2 = 0; s2 < p.splits; ++s2) {
            const float ms = __ldcg(&p.part_ml[((base + s2) * kMaxGroup + g) * 2]);
            const float f = (m == -INFINITY) ? 0.0f : expf(ms - m);
            l += __ldcg(&p.part_ml[((base + s2) * kMaxGroup + g) * 2 + 1]) * f;
            o += __ldcg(&p.part_o[((base + s2) * kMaxGroup + g) * HD + d]) * f;
        }
        p.out[((long long)b * p.q_heads + kvh * group + g) * HD + d] = l > 0.0f ? o / l : 0.0f;
    }
}

}  // namespace cheetah
