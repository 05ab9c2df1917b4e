// Weight-streaming GEMV kernels for decode (one token per sequence).
//
// y = W . x over bf16 row-major weights [rows, cols], f32 input/accumulate,
// exactly the arithmetic of `ops::gemv` / `dot_row_bf16_avx2`
// (`ops.rs:202-278`) up to summation order. HBM-bound: every weight byte is
// read once per step with 128-bit streaming loads (L1 no-allocate), 2 row
// streams x 4 vectors in flight per lane, CTAs persistent over row groups.
// Fusions (one launch instead of the reference's separate passes):
//   prologue  RMSNorm of the input (`ops.rs:646`) into shared memory;
//   epilogues bias add (`ops.rs:1156`), residual add (`qwen2.rs:442-463`),
//             SiLU(gate)*up (`ops.rs:743`), rotate-half RoPE + paged KV
//             append (`ops.rs:722`, `ops.rs:1329`), greedy argmax
//             (`engine.rs:2247-2253`).
// The first weight vectors are loaded before griddepcontrol.wait, so under
// programmatic dependent launch they stream while the previous kernel drains.
#pragma once

#include "common.cuh"

namespace cheetah {

enum GemvEpilogue : int {
    kEpiStore = 0,     // y[r] = acc + bias[r]
    kEpiResidual = 1,  // y[r] += acc + bias[r]
    kEpiSwiglu = 2,    // y[r] = silu(acc_gate) * acc_up  (rows of w0 and w1)
    kEpiQkv = 3,       // bias, RoPE, q out / K,V into the paged cache
    kEpiLogits = 4,    // y[r] = acc, plus packed argmax
};

struct GemvParams {
    const uint16_t *w0;      // bf16 [rows, cols], or q8/q4 codes (reference layout rows)
    const uint16_t *w1;      // up_proj for kEpiSwiglu
    long long row_stride;    // bytes between weight rows (q8/q4); 0 = cols * 2 (bf16)
    const float *scale0;     // q8/q4 per-row scales of w0 (nullptr for bf16)
    const float *scale1;     // q8/q4 per-row scales of w1
    int wt;                  // WeightFormat of w0/w1
    int rows;                // output rows (for kEpiSwiglu: intermediate size)
    int cols;                // multiple of 8
    int batch;               // input vectors (NB template bound)
    const float *x;          // [batch][cols]
    long long x_stride;      // floats between batch rows
    const float *norm_w;     // nullptr: no RMSNorm prologue
    float eps;
    const float *bias;       // nullptr: none
    float *y;                // [batch][y_stride]
    long long y_stride;
    // kEpiQkv
    int q_heads, kv_heads, head_dim;
    const float *rope_cos;   // [max_positions][head_dim/2]
    const float *rope_sin;
    const int32_t *positions;   // [batch] absolute position of each query
    const int32_t *page_table;  // [batch][max_pages]
    int max_pages;
    int num_pages;           // pool pages (bounds guard)
    int page_tokens;
    void *k_cache;           // this layer's pool: [pages][kv_heads][page_tokens][head_dim]
    void *v_cache;
    int kv_f32;              // 1: f32 cache, 0: bf16
    // kEpiLogits
    unsigned long long *argmax;  // [batch] packed (order key << 32 | index), nullable
    int *error;                  // nullable: set when a bounded wait gives up
    // Cross-CTA K splits of the small-batch tensor-core GEMV (gemv_mma.cuh):
    // per-(tile, split) partials and per-tile tickets (zero between launches).
    int splits;
    float *split_ws;
    unsigned *split_tickets;
    // kEpiQkv for families with per-head q/k norms: the biased projections
    // go to qk_raw [batch][rows] and `qk_norm_rope_kernel` finishes them.
    float *qk_raw;
};

template <int NB>
struct Acc2 {
    float a[NB];
    float b[NB];
};

__device__ __forceinline__ void fma8(float &acc, uint4 w, const float *x) {
    const float4 x0 = *reinterpret_cast<const float4 *>(x);
    const float4 x1 = *reinterpret_cast<const float4 *>(x + 4);
    acc = fmaf(bf16_lo(w.x), x0.x, acc);
    acc = fmaf(bf16_hi(w.x), x0.y, acc);
    acc = fmaf(bf16_lo(w.y), x0.z, acc);
    acc = fmaf(bf16_hi(w.y), x0.w, acc);
    acc = fmaf(bf16_lo(w.z), x1.x, acc);
    acc = fmaf(bf16_hi(w.z), x1.y, acc);
    acc = fmaf(bf16_lo(w.w), x1.z, acc);
    acc = fmaf(bf16_hi(w.w), x1.w, acc);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    // ops.rs:743-747: g * (u / (1 + exp(-g)))
    return __fmul_rn(g, __fdiv_rn(u, __fadd_rn(1.0f, expf(-g))));
}

// Row-group -> the two weight rows a warp streams.
template <int EPI>
__device__ __forceinline__ void group_rows(const GemvParams &p, int group, int &row_a, int &row_b) {
    if (EPI == kEpiQkv) {
        const int half = p.head_dim >> 1;
        const int head = group / half;
        const int i = group - head * half;
        row_a = head * p.head_dim + i;
        row_b = row_a + half;
    } else if (EPI == kEpiSwiglu) {
        row_a = group;
        row_b = group;
    } else {
        row_a = 2 * group;
        row_b = 2 * group + 1 < p.rows ? 2 * group + 1 : -1;
    }
}

template <int EPI>
__device__ __forceinline__ int num_groups(const GemvParams &p) {
    if (EPI == kEpiQkv) return (p.rows >> 1);
    if (EPI == kEpiSwiglu) return p.rows;
    return (p.rows + 1) >> 1;
}

template <int NB>
__device__ __forceinline__ void store_kv(const GemvParams &p, int b, int kv_head, int d, float value,
                                         bool is_k) {
    const int pos = p.positions[b];
    if (pos < 0 || pos / p.page_tokens >= p.max_pages) return;
    const int page = p.page_table[(long long)b * p.max_pages + pos / p.page_tokens];
    if (page < 0 || page >= p.num_pages) return;  // no page installed: drop the write
    const int slot = pos - (pos / p.page_tokens) * p.page_tokens;
    const long long index =
        (((long long)page * p.kv_heads + kv_head) * p.page_tokens + slot) * p.head_dim + d;
    void *base = is_k ? p.k_cache : p.v_cache;
    if (p.kv_f32) {
        static_cast<float *>(base)[index] = value;
    } else {
        static_cast<uint16_t *>(base)[index] = f32_to_bf16_rne(value);
    }
}

// Epilogue for one output row pair of batch row b once the dot products
// are known. row_b < 0: single row. kEpiQkv: (row_a, row_b) are the logical
// rope partners (i, i + head_dim/2) of one head.
template <int EPI>
__device__ __forceinline__ void epilogue_rows(const GemvParams &p, int b, int row_a, int row_b, float acc_a,
                                              float acc_b, unsigned long long &best) {
    float *y = p.y + (long long)b * p.y_stride;
    if (EPI == kEpiStore || EPI == kEpiResidual) {
        float va = acc_a;
        if (p.bias) va = __fadd_rn(va, p.bias[row_a]);
        if (EPI == kEpiResidual) va = __fadd_rn(y[row_a], va);
        y[row_a] = va;
        if (row_b >= 0) {
            float vb = acc_b;
            if (p.bias) vb = __fadd_rn(vb, p.bias[row_b]);
            if (EPI == kEpiResidual) vb = __fadd_rn(y[row_b], vb);
            y[row_b] = vb;
        }
    } else if (EPI == kEpiSwiglu) {
        y[row_a] = silu_mul(acc_a, acc_b);
    } else if (EPI == kEpiLogits) {
        y[row_a] = acc_a;
        unsigned long long key = ((unsigned long long)total_order_key(acc_a) << 32) | (unsigned)row_a;
        if (row_b >= 0) {
            y[row_b] = acc_b;
            unsigned long long kb = ((unsigned long long)total_order_key(acc_b) << 32) | (unsigned)row_b;
            key = kb > key ? kb : key;
        }
        best = key > best ? key : best;
    } else {  // kEpiQkv
        const int hd = p.head_dim;
        const int half = hd >> 1;
        const int head = row_a / hd;
        const int i = row_a - head * hd;
        float va = __fadd_rn(acc_a, p.bias ? p.bias[row_a] : 0.0f);
        float vb = __fadd_rn(acc_b, p.bias ? p.bias[row_b] : 0.0f);
        if (p.qk_raw) {
            float *raw = p.qk_raw + (long long)b * p.rows;
            raw[row_a] = va;
            raw[row_b] = vb;
            return;
        }
        if (head < p.q_heads + p.kv_heads) {
            // ops.rs:693-715: a' = a*cos - b*sin, b' = b*cos + a*sin
            const int pos = p.positions[b];
            const float c = p.rope_cos[(long long)pos * half + i];
            const float s = p.rope_sin[(long long)pos * half + i];
            const float ra = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
            const float rb = __fadd_rn(__fmul_rn(vb, c), __fmul_rn(va, s));
            va = ra;
            vb = rb;
        }
        if (head < p.q_heads) {
            y[row_a] = va;
            y[row_b] = vb;
        } else if (head < p.q_heads + p.kv_heads) {
            store_kv<1>(p, b, head - p.q_heads, i, va, true);
            store_kv<1>(p, b, head - p.q_heads, i + half, vb, true);
        } else {
            store_kv<1>(p, b, head - p.q_heads - p.kv_heads, i, va, false);
            store_kv<1>(p, b, head - p.q_heads - p.kv_heads, i + half, vb, false);
        }
    }
}

// Epilogue for one row group once the full dot products are known.
template <int NB, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, int group, const float *acc_a,
                                              const float *acc_b, unsigned long long *best) {
    int row_a, row_b;
    group_rows<EPI>(p, group, row_a, row_b);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= p.batch) break;
        epilogue_rows<EPI>(p, b, row_a, EPI == kEpiSwiglu ? row_a : row_b, acc_a[b], acc_b[b], best[b]);
    }
}

// Weight formats of the register-streaming GEMV. bf16: 128-bit vectors of 8
// weights. q8 / q4 (`precision/q8.rs`, `precision/q4.rs` row layouts): 32-bit
// words of 4 int8 / 8 int4 codes, unpacked in registers; the per-row scale
// is applied once to the finished dot product.
enum WeightFormat : int { kWBf16 = 0, kWQ8 = 1, kWQ4 = 2 };

template <int WT>
struct WeightTraits;

template <>
struct WeightTraits<kWBf16> {
    using Vec = uint4;
    static constexpr int kElems = 8;
    static constexpr int kUnroll = 4;
    static __device__ __forceinline__ Vec load(const Vec *p) { return ldg_stream(p); }
    static __device__ __forceinline__ Vec zero() { return make_uint4(0, 0, 0, 0); }
    static __device__ __forceinline__ void fma(float &acc, Vec w, const float *x) { fma8(acc, w, x); }
};

__device__ __forceinline__ uint32_t ldg_stream_u32(const uint32_t *ptr) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(ptr));
    return v;
}

// int8 code -> exact float: (code + 128) in the low mantissa bits of 2^23.
__device__ __forceinline__ float q8_code(uint32_t biased, int byte) {
    return __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7440u + byte)) - 8388736.0f;
}

template <>
struct WeightTraits<kWQ8> {
    using Vec = uint32_t;
    static constexpr int kElems = 4;
    static constexpr int kUnroll = 8;
    static __device__ __forceinline__ Vec load(const Vec *p) { return ldg_stream_u32(p); }
    static __device__ __forceinline__ Vec zero() { return 0u; }
    static __device__ __forceinline__ void fma(float &acc, Vec w, const float *x) {
        const uint32_t b = w ^ 0x80808080u;
        const float4 xv = *reinterpret_cast<const float4 *>(x);
        acc = fmaf(q8_code(b, 0), xv.x, acc);
        acc = fmaf(q8_code(b, 1), xv.y, acc);
        acc = fmaf(q8_code(b, 2), xv.z, acc);
        acc = fmaf(q8_code(b, 3), xv.w, acc);
    }
};

// int4 code (low nibble = even column, `q4.rs:59-66`) -> exact float.
__device__ __forceinline__ float q4_code(uint32_t biased, int nibble) {
    return __uint_as_float(0x4B000000u | ((biased >> (4 * nibble)) & 0xFu)) - 8388616.0f;
}

template <>
struct WeightTraits<kWQ4> {
    using Vec = uint32_t;
    static constexpr int kElems = 8;
    static constexpr int kUnroll = 8;
    static __device__ __forceinline__ Vec load(const Vec *p) { return ldg_stream_u32(p); }
    static __device__ __forceinline__ Vec zero() { return 0u; }
    static __device__ __forceinline__ void fma(float &acc, Vec w, const float *x) {
        const uint32_t b = w ^ 0x88888888u;
        const float4 x0 = *reinterpret_cast<const float4 *>(x);
        const float4 x1 = *reinterpret_cast<const float4 *>(x + 4);
        acc = fmaf(q4_code(b, 0), x0.x, acc);
        acc = fmaf(q4_code(b, 1), x0.y, acc);
        acc = fmaf(q4_code(b, 2), x0.z, acc);
        acc = fmaf(q4_code(b, 3), x0.w, acc);
        acc = fmaf(q4_code(b, 4), x1.x, acc);
        acc = fmaf(q4_code(b, 5), x1.y, acc);
        acc = fmaf(q4_code(b, 6), x1.z, acc);
        acc = fmaf(q4_code(b, 7), x1.w, acc);
    }
};

// Quantised rows: dot = scale[row] * sum(code * x).
template <int NB, int EPI>
__device__ __forceinline__ void apply_row_scales(const GemvParams &p, int group, float *acc_a, float *acc_b) {
    int row_a, row_b;
    group_rows<EPI>(p, group, row_a, row_b);
    const float sa = p.scale0[row_a];
    const float sb = EPI == kEpiSwiglu ? p.scale1[row_a] : (row_b >= 0 ? p.scale0[row_b] : 0.0f);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        acc_a[b] *= sa;
        acc_b[b] *= sb;
    }
}

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / kWarp;
constexpr int kGemvUnroll = 4;

// Dynamic shared memory: x [NB][cols] f32, partials [warps][2][NB], argmax [warps][NB].
template <int NB, int EPI, int KSPLIT, int WT = kWBf16>
__global__ void __launch_bounds__(kGemvThreads) gemv_bf16_kernel(const GemvParams p) {
    using W = WeightTraits<WT>;
    using Vec = typename W::Vec;
    constexpr int kU = W::kUnroll;
    extern __shared__ __align__(16) float smem[];
    float *xs = smem;
    float *partial = smem + (size_t)NB * p.cols;
    __shared__ float red[kGemvWarps];
    __shared__ unsigned long long best_s[kGemvWarps][NB];

    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    constexpr int kGroupsPerCta = kGemvWarps / KSPLIT;
    const int group_in_cta = warp / KSPLIT;
    const int kslice = warp % KSPLIT;
    const int nvec = p.cols / W::kElems;
    const long long row_stride = p.row_stride ? p.row_stride : (long long)p.cols * 2;
    const int slice_len = (nvec + KSPLIT - 1) / KSPLIT;
    const int v_begin = kslice * slice_len;
    const int v_end = min(nvec, v_begin + slice_len);
    const int groups = num_groups<EPI>(p);
    const int group_stride = gridDim.x * kGroupsPerCta;

    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;

    int group = blockIdx.x * kGroupsPerCta + group_in_cta;

    // Stage the first weight vectors before waiting on the previous kernel.
    Vec wa[kU], wb[kU];
    auto load_batch = [&](int g, int base) {
        int ra, rb;
        group_rows<EPI>(p, g, ra, rb);
        const Vec *pa = reinterpret_cast<const Vec *>(reinterpret_cast<const uint8_t *>(p.w0) + (long long)ra * row_stride);
        const uint16_t *wsrc_b = (EPI == kEpiSwiglu) ? p.w1 : p.w0;
        const Vec *pb = reinterpret_cast<const Vec *>(reinterpret_cast<const uint8_t *>(wsrc_b) +
                                                      (long long)(rb < 0 ? ra : rb) * row_stride);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int v = base + u * kWarp + lane;
            if (v < v_end && g < groups) {
                wa[u] = W::load(pa + v);
                wb[u] = W::load(pb + v);
            } else {
                wa[u] = W::zero();
                wb[u] = W::zero();
            }
        }
    };
    load_batch(group, v_begin);

    pdl_wait();
    pdl_launch_dependents();

    // Prologue: x (optionally RMS-normalised) into shared memory.
    for (int b = 0; b < NB && b < p.batch; ++b) {
        const float *xin = p.x + (long long)b * p.x_stride;
        float *xo = xs + (size_t)b * p.cols;
        if (p.norm_w) {
            float ss = 0.0f;
            for (int i = threadIdx.x; i < p.cols; i += kGemvThreads) {
                const float v = xin[i];
                ss = fmaf(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float total = 0.0f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) total += red[w];
            const float inv = 1.0f / sqrtf(total / (float)p.cols + p.eps);
            for (int i = threadIdx.x; i < p.cols; i += kGemvThreads) {
                xo[i] = __fmul_rn(xin[i], __fmul_rn(inv, p.norm_w[i]));
            }
            __syncthreads();
        } else {
            for (int i = threadIdx.x; i < p.cols; i += kGemvThreads) xo[i] = xin[i];
        }
    }
    __syncthreads();

    for (; group - group_in_cta < groups; group += group_stride) {
        float acc_a[NB], acc_b[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc_a[b] = acc_b[b] = 0.0f;
        const bool active = group < groups;
        for (int base = v_begin; base < v_end; base += kWarp * kU) {
            if (base != v_begin) load_batch(group, base);
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int v = base + u * kWarp + lane;
                if (v < v_end) {
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        if (b < p.batch) {
                            const float *xv = xs + (size_t)b * p.cols + v * W::kElems;
                            W::fma(acc_a[b], wa[u], xv);
                            W::fma(acc_b[b], wb[u], xv);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            acc_a[b] = warp_sum(acc_a[b]);
            acc_b[b] = warp_sum(acc_b[b]);
        }
        // Prefetch the next group's first vectors before the epilogue.
        const int next = group + group_stride;
        if (next - group_in_cta < groups) load_batch(next, v_begin);

        if (KSPLIT > 1) {
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    partial[(warp * 2 + 0) * NB + b] = acc_a[b];
                    partial[(warp * 2 + 1) * NB + b] = acc_b[b];
                }
            }
            __syncthreads();
            if (kslice == 0 && lane == 0 && active) {
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    float sa = 0.0f, sb = 0.0f;
#pragma unroll
                    for (int k = 0; k < KSPLIT; ++k) {
                        sa += partial[((warp + k) * 2 + 0) * NB + b];
                        sb += partial[((warp + k) * 2 + 1) * NB + b];
                    }
                    acc_a[b] = sa;
                    acc_b[b] = sb;
                }
                if (WT != kWBf16) apply_row_scales<NB, EPI>(p, group, acc_a, acc_b);
                gemv_epilogue<NB, EPI>(p, group, acc_a, acc_b, best);
            }
            __syncthreads();
        } else if (lane == 0 && active) {
            if (WT != kWBf16) apply_row_scales<NB, EPI>(p, group, acc_a, acc_b);
            gemv_epilogue<NB, EPI>(p, group, acc_a, acc_b, best);
        }
    }

    if (EPI == kEpiLogits && p.argmax) {
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < NB; ++b) best_s[warp][b] = best[b];
        }
        __syncthreads();
        if (threadIdx.x < NB && threadIdx.x < p.batch) {
            unsigned long long m = 0ull;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) m = best_s[w][threadIdx.x] > m ? best_s[w][threadIdx.x] : m;
            atomicMax(p.argmax + threadIdx.x, m);
        }
    }
}

// Per-head RMSNorm of q and k (`ops.rs:1130-1152`, the qwen3 family), then
// RoPE and the q store / paged K,V append of the kEpiQkv epilogue, over the
// biased projections a kEpiQkv GEMV left in p.qk_raw. One warp per (head,
// batch row): grid (q_heads + 2 kv_heads, batch), 32 threads. A null norm
// weight leaves that head un-normalised (the reference's absent unit).
__global__ void __launch_bounds__(32) qk_norm_rope_kernel(const GemvParams p, const float *q_norm,
                                                          const float *k_norm) {
    const int head = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
    const int hd = p.head_dim, half = hd >> 1;
    pdl_wait();  // the QKV GEMV's rows
    pdl_launch_dependents();
    const float *raw = p.qk_raw + (long long)b * p.rows + (long long)head * hd;
    const bool is_q = head < p.q_heads;
    const bool is_k = !is_q && head < p.q_heads + p.kv_heads;
    const float *nw = is_q ? q_norm : (is_k ? k_norm : nullptr);
    float inv = 1.0f;
    if (nw) {
        // rmsnorm (`ops.rs:646-652`): x * (1/sqrt(mean(x^2) + eps) * w)
        float ss = 0.0f;
        for (int d = lane; d < hd; d += 32) ss = fmaf(raw[d], raw[d], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)hd), p.eps));
    }
    const int pos = p.positions[b];
    float *y = p.y + (long long)b * p.y_stride;
    for (int i = lane; i < half; i += 32) {
        float va = raw[i], vb = raw[i + half];
        if (nw) {
            va = __fmul_rn(va, __fmul_rn(inv, nw[i]));
            vb = __fmul_rn(vb, __fmul_rn(inv, nw[i + half]));
        }
        if (is_q || is_k) {
            const float c = p.rope_cos[(long long)pos * half + i];
            const float s = p.rope_sin[(long long)pos * half + i];
            const float ra = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
            const float rb = __fadd_rn(__fmul_rn(vb, c), __fmul_rn(va, s));
            va = ra;
            vb = rb;
        }
        if (is_q) {
            y[head * hd + i] = va;
            y[head * hd + i + half] = vb;
        } else {
            const int kvh = is_k ? head - p.q_heads : head - p.q_heads - p.kv_heads;
            store_kv<1>(p, b, kvh, i, va, is_k);
            store_kv<1>(p, b, kvh, i + half, vb, is_k);
        }
    }
}

}  // namespace cheetah
