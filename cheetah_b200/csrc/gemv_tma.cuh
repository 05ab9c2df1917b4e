// Decode GEMV with bulk-copy prefetch (one CTA per SM).
//
// Same arithmetic and epilogues as gemv_bf16_kernel (`ops::gemv`,
// `ops.rs:202-278`, plus the fused norm / bias / residual / SwiGLU / RoPE +
// KV append / argmax epilogues). What changes is how the weights arrive:
//   * each CTA owns a contiguous range of row chunks (8/KS rows each) and
//     streams them with 1D bulk copies (cp.async.bulk) into a shared-memory
//     ring completed by mbarriers (bounded waits);
//   * the first ring-full of chunks is requested BEFORE griddepcontrol.wait:
//     weights never depend on the previous kernel, so under programmatic
//     dependent launch a layer's weights stream while its predecessor still
//     runs (at Qwen2-0.5B sizes a CTA's whole slice fits the ring);
//   * 1 CTA per SM, <= 128 registers and ~100 KB of shared memory, so the
//     next kernel's CTAs fit beside it and can start their own prefetch;
//   * the input vector (normed in the prologue) lives in registers: lane l of
//     k-slice s always multiplies the same 16-byte vectors of every row.
// QKV rows are stored pair-interleaved (row 2j, 2j+1 of a head = logical
// rows j, j + head_dim/2), so a chunk holds whole RoPE pairs.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace cheetah {

__device__ __forceinline__ void fma8r(float &acc, uint4 w, const float (&x)[8]) {
    acc = fmaf(bf16_lo(w.x), x[0], acc);
    acc = fmaf(bf16_hi(w.x), x[1], acc);
    acc = fmaf(bf16_lo(w.y), x[2], acc);
    acc = fmaf(bf16_hi(w.y), x[3], acc);
    acc = fmaf(bf16_lo(w.z), x[4], acc);
    acc = fmaf(bf16_hi(w.z), x[5], acc);
    acc = fmaf(bf16_lo(w.w), x[6], acc);
    acc = fmaf(bf16_hi(w.w), x[7], acc);
}

constexpr int kTmaGemvThreads = 256;
constexpr int kTmaGemvWarps = 8;
constexpr int kTmaGemvMaxSlots = 8;

template <int EPI, int KS, int NX>
__global__ void __launch_bounds__(kTmaGemvThreads, 2)
    gemv_tma_kernel(const GemvParams p, int slots, int slot_bytes) {
    constexpr int RT = kTmaGemvWarps / KS;  // rows per chunk
    extern __shared__ __align__(128) uint8_t tsmem[];
    __shared__ __align__(8) uint64_t bars[kTmaGemvMaxSlots];
    __shared__ float partial[2][kTmaGemvWarps][2];
    __shared__ float red[kTmaGemvWarps];

    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int row_bytes = p.cols * 2;
    const int nvec = p.cols >> 3;
    const int slice_len = (nvec + KS - 1) / KS;
    const int r_local = warp / KS;
    const int kslice = warp % KS;
    const int v_begin = kslice * slice_len;
    const int v_end = min(nvec, v_begin + slice_len);
    const int total_chunks = (p.rows + RT - 1) / RT;
    const int c_begin = (int)(((long long)blockIdx.x * total_chunks) / gridDim.x);
    const int c_end = (int)(((long long)(blockIdx.x + 1) * total_chunks) / gridDim.x);
    const int n = c_end - c_begin;
    uint8_t *ring = tsmem;
    float *xs = reinterpret_cast<float *>(tsmem + (size_t)slots * slot_bytes);

    auto issue = [&](int k) {
        const int chunk = c_begin + k;
        const int slot = k % slots;
        const uint32_t bar = smem_u32(&bars[slot]);
        const int rows_in = min(RT, p.rows - chunk * RT);
        const uint32_t bytes = (uint32_t)rows_in * row_bytes;
        uint8_t *dst = ring + (size_t)slot * slot_bytes;
        const uint8_t *src0 = reinterpret_cast<const uint8_t *>(p.w0) + (long long)chunk * RT * row_bytes;
        if (EPI == kEpiSwiglu) {
            mbar_expect_tx(bar, 2 * bytes);
            bulk_load(smem_u32(dst), src0, bytes, bar);
            const uint8_t *src1 = reinterpret_cast<const uint8_t *>(p.w1) + (long long)chunk * RT * row_bytes;
            bulk_load(smem_u32(dst + (size_t)RT * row_bytes), src1, bytes, bar);
        } else {
            mbar_expect_tx(bar, bytes);
            bulk_load(smem_u32(dst), src0, bytes, bar);
        }
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < slots; ++s) mbar_init(smem_u32(&bars[s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < slots && k < n; ++k) issue(k);  // before the dependency wait
    }

    pdl_wait();
    pdl_launch_dependents();

    // Prologue: x (optionally RMS-normalised, `ops.rs:646-652`) -> shared -> registers.
    {
        const float *xin = p.x;
        if (p.norm_w) {
            float ss = 0.0f;
            for (int i = threadIdx.x; i < p.cols; i += kTmaGemvThreads) {
                const float v = xin[i];
                ss = fmaf(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float total = 0.0f;
#pragma unroll
            for (int w = 0; w < kTmaGemvWarps; ++w) total += red[w];
            const float inv = 1.0f / sqrtf(total / (float)p.cols + p.eps);
            for (int i = threadIdx.x; i < p.cols; i += kTmaGemvThreads) {
                xs[i] = __fmul_rn(xin[i], __fmul_rn(inv, p.norm_w[i]));
            }
        } else {
            for (int i = threadIdx.x; i < p.cols; i += kTmaGemvThreads) xs[i] = xin[i];
        }
    }
    __syncthreads();
    float xr[NX][8];
#pragma unroll
    for (int u = 0; u < NX; ++u) {
        const int v = v_begin + lane + u * kWarp;
        if (v < v_end) {
            const float4 a = *reinterpret_cast<const float4 *>(xs + v * 8);
            const float4 b = *reinterpret_cast<const float4 *>(xs + v * 8 + 4);
            xr[u][0] = a.x; xr[u][1] = a.y; xr[u][2] = a.z; xr[u][3] = a.w;
            xr[u][4] = b.x; xr[u][5] = b.y; xr[u][6] = b.z; xr[u][7] = b.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) xr[u][e] = 0.0f;
        }
    }

    unsigned long long best = 0ull;
    bool failed = false;
    int fail_at = 0;
    for (int k = 0; k < n; ++k) {
        const int slot = k % slots;
        const int chunk = c_begin + k;
        const int rows_in = min(RT, p.rows - chunk * RT);
        if (!__syncthreads_or(mbar_wait(smem_u32(&bars[slot]), (k / slots) & 1))) {
            failed = true;
            fail_at = k;
            break;
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        if (r_local < rows_in) {
            const uint4 *wa = reinterpret_cast<const uint4 *>(ring + (size_t)slot * slot_bytes + (size_t)r_local * row_bytes);
            const uint4 *wb = reinterpret_cast<const uint4 *>(ring + (size_t)slot * slot_bytes +
                                                               (size_t)(RT + r_local) * row_bytes);
#pragma unroll
            for (int u = 0; u < NX; ++u) {
                const int v = v_begin + lane + u * kWarp;
                if (v < v_end) {
                    fma8r(acc_a, wa[v], xr[u]);
                    if (EPI == kEpiSwiglu) fma8r(acc_b, wb[v], xr[u]);
                }
            }
        }
        acc_a = warp_sum(acc_a);
        if (EPI == kEpiSwiglu) acc_b = warp_sum(acc_b);
        if (lane == 0) {
            partial[k & 1][warp][0] = acc_a;
            partial[k & 1][warp][1] = acc_b;
        }
        __syncthreads();  // slot consumed, partials visible
        if (threadIdx.x == 0 && k + slots < n) issue(k + slots);
        if (EPI == kEpiQkv) {
            if (RT >= 2 && (int)threadIdx.x < RT / 2) {
                const int j = threadIdx.x;
                float da = 0.0f, db = 0.0f;
#pragma unroll
                for (int s = 0; s < KS; ++s) {
                    da += partial[k & 1][(2 * j) * KS + s][0];
                    db += partial[k & 1][(2 * j + 1) * KS + s][0];
                }
                if (2 * j < rows_in) {
                    const int srow = chunk * RT + 2 * j;  // storage row (pair-interleaved)
                    const int head = srow / p.head_dim;
                    const int i = (srow - head * p.head_dim) >> 1;
                    const int row_a = head * p.head_dim + i;
                    epilogue_rows<EPI>(p, 0, row_a, row_a + (p.head_dim >> 1), da, db, best);
                }
            }
        } else if (threadIdx.x < rows_in) {
            const int r = threadIdx.x;
            float da = 0.0f, db = 0.0f;
#pragma unroll
            for (int s = 0; s < KS; ++s) {
                da += partial[k & 1][r * KS + s][0];
                db += partial[k & 1][r * KS + s][1];
            }
            const int row = chunk * RT + r;
            epilogue_rows<EPI>(p, 0, row, EPI == kEpiSwiglu ? row : -1, da, db, best);
        }
    }
    if (failed) {
        if (p.error) *p.error = 3;
        if (threadIdx.x == 0) {
            const int issued = min(n, fail_at + slots);
            for (int k = fail_at; k < issued; ++k) (void)mbar_wait(smem_u32(&bars[k % slots]), (k / slots) & 1);
        }
        return;
    }
    if (EPI == kEpiLogits && p.argmax) {
        // Epilogue threads are warp 0's first RT lanes.
        if (warp == 0) {
            unsigned long long m = best;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, m, o);
                m = other > m ? other : m;
            }
            if (lane == 0 && m != 0ull) atomicMax(p.argmax, m);
        }
    }
}

}  // namespace cheetah
