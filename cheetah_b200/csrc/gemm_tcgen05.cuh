// Chunked-prefill linear layers on the 5th-generation tensor cores.
//
// D[M, N] = A[M, K] . B[N, K]^T with A the chunk's bf16 activations (rows =
// tokens) and B a layer's bf16 weights (rows = output features), both
// K-major — the batched form of `ops::gemm` (`ops.rs:308-354`, the per-row
// dot of `dot_row_bf16_avx2`) with the activations rounded to bf16 for the
// tensor cores (f32 accumulation; tolerance-checked against the f32 oracle).
//
// One CTA per 128 x BN output tile, warp-specialised:
//   warp 0      TMA producer: 128x64 A and BNx64 B boxes (128-byte swizzle,
//               no multicast) into a kStages-deep shared-memory ring;
//   warp 1      allocates BN TMEM columns; lane 0 issues tcgen05.mma
//               (kind::f16, M=128, N=BN, K=16 per instruction, f32
//               accumulators in TMEM) and tcgen05.commit to free each stage;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows (warp w reads
//               TMEM lanes 32*(w%4)..+31 = tile rows), fused epilogue, global
//               stores.
// All mbarrier waits are bounded: on a timeout the CTA sets the error flag,
// waits (bounded) for its own bulk copies and MMAs in flight, frees its TMEM
// and exits.
// Fused epilogues:
//   kPgQkv      + bias, rotate-half RoPE (`ops.rs:693-715`, host rotary
//               table), q rows -> bf16, K/V rows -> the paged cache
//               (`ops.rs:1329` cache_append);
//   kPgResidual + bias, then residual add into the f32 hidden rows
//               (`qwen2.rs:442-463`);
//   kPgSwiglu   B tile = 64 gate rows || 64 up rows; silu(g) * u
//               (`ops.rs:743`) -> bf16.
// Split-K (gridDim.z = S > 1, for grids far smaller than the SM count, as in
// batched decode): CTA z accumulates k-blocks [z*KB/S, (z+1)*KB/S), writes
// its f32 tile to a workspace and takes a ticket; the tile's last CTA sums
// the S partial tiles in split order (deterministic), stores the sum into its
// own TMEM accumulator and runs the epilogue above unchanged. The last CTA
// resets the ticket, so tickets are zero between launches.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace cheetah {

enum PrefillEpilogue : int { kPgQkv = 0, kPgResidual = 1, kPgSwiglu = 2, kPgLogits = 3 };

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;

struct PrefillGemmParams {
    int M, N, K;              // N counts output features (kPgSwiglu: intermediate size)
    // epilogue inputs
    const float *bias;        // [N] or nullptr
    float *out_f32;           // kPgResidual: hidden [M][ld_out]
    uint16_t *out_bf16;       // kPgQkv: q [M][q_dim]; kPgSwiglu: act [M][N]
    int ld_out;
    // kPgQkv
    int q_heads, kv_heads, head_dim;
    int offset;               // absolute position of row 0
    const float *rope_cos, *rope_sin;  // [max_positions][head_dim/2]
    const int32_t *page_table;
    int max_pages, num_pages, page_tokens;
    void *k_cache, *v_cache;  // this layer's pool base
    int kv_f32;
    int *error;
    // Batched decode: row r is sequence r at position row_pos[r] with its page
    // table at page_table + r * table_stride; q rows go out as f32.
    const int32_t *row_pos;   // nullptr: position = offset + row (prefill)
    int table_stride;
    float *out_q_f32;         // kPgQkv: q [M][q_dim] f32 instead of bf16
    // kPgQkv per-head RMSNorm of q / k before RoPE (qwen3, `ops.rs:1130`):
    // f32 [head_dim] weights, nullptr = none.
    const float *q_norm, *k_norm;
    float eps;
    // kPgLogits: logits [M][ld_out] f32 + per-row packed argmax
    unsigned long long *argmax;
    // Split-K (gridDim.z > 1): [splits][tiles][128][BN] f32 partial tiles
    // and one ticket per tile (zero between launches).
    float *split_ws;
    unsigned *split_tickets;
};

__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t addr) {
    // K-major, 128-byte swizzle: 8-row atoms of 128 B (SBO = 1024 B), LBO
    // unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
    uint64_t desc = 0;
    desc |= (uint64_t)((addr >> 4) & 0x3FFF);
    desc |= (uint64_t)1 << 16;
    desc |= (uint64_t)(1024 >> 4) << 32;
    desc |= (uint64_t)1 << 46;
    desc |= (uint64_t)2 << 61;
    return desc;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Split-K exchange by the four epilogue warps (thread = tile row `r`): this
// CTA's partial tile to the workspace, then a ticket; the last of the S
// CTAs of the tile sums the partials in split order into its TMEM
// accumulator. Returns true in that CTA.
template <int BN>
__device__ __forceinline__ bool split_k_reduce(const PrefillGemmParams &p, uint32_t lane_addr, int r, int *last_s) {
    const int S = gridDim.z;
    const int tiles = gridDim.x * gridDim.y;
    const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
    const size_t split_stride = (size_t)tiles * kGemmBM * BN;
    float *row_base = p.split_ws + ((size_t)tile_id * kGemmBM + r) * BN;
    // Only rows below M carry results; the others are never read.
    const bool live = blockIdx.y * kGemmBM + r < p.M;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(lane_addr + c0, v);
        float4 *d4 = reinterpret_cast<float4 *>(row_base + blockIdx.z * split_stride + c0);
        if (live) {
#pragma unroll
            for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
    __threadfence();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (threadIdx.x == 2 * kWarp) {
        const unsigned old = atomicAdd(p.split_tickets + tile_id, 1u);
        const int last = old == (unsigned)S - 1u;
        if (last) p.split_tickets[tile_id] = 0u;
        *last_s = last;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!*last_s) return false;
    __threadfence();
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        const float4 *s0 = reinterpret_cast<const float4 *>(row_base + c0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = live ? __ldcg(s0 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
        }
        for (int z = 1; z < S && live; ++z) {
            const float4 *sz = reinterpret_cast<const float4 *>(row_base + z * split_stride + c0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 a = __ldcg(sz + i);
                v[4 * i] = __fadd_rn(v[4 * i], a.x);
                v[4 * i + 1] = __fadd_rn(v[4 * i + 1], a.y);
                v[4 * i + 2] = __fadd_rn(v[4 * i + 2], a.z);
                v[4 * i + 3] = __fadd_rn(v[4 * i + 3], a.w);
            }
        }
        tmem_st32(lane_addr + c0, v);
    }
    return true;
}

// 16 consecutive values as bf16 (two 16-byte stores; dst 16-byte aligned).
__device__ __forceinline__ void store_bf16x16(uint16_t *dst, const float (&v)[16]) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = (uint32_t)f32_to_bf16_rne(v[2 * i]) | ((uint32_t)f32_to_bf16_rne(v[2 * i + 1]) << 16);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__device__ __forceinline__ void store_f32x16(float *dst, const float (&v)[16]) {
    float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int EPI, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                        const __grid_constant__ CUtensorMap b2_map, const PrefillGemmParams p) {
    constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
    constexpr int kBBytes = BN * kGemmBK * 2;
    constexpr int kStageBytes = kABytes + kBBytes;
    constexpr uint32_t kIdesc = umma_idesc_bf16(kGemmBM, BN);
    extern __shared__ __align__(1024) uint8_t gsmem[];
    __shared__ __align__(8) uint64_t full_bar[kGemmStages];
    __shared__ __align__(8) uint64_t empty_bar[kGemmStages];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    __shared__ int split_last_s;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsmem) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int n_tile = blockIdx.x;
    const int m_tile = blockIdx.y;
    const int k_total = (p.K + kGemmBK - 1) / kGemmBK;
    // This CTA's k-blocks (all of them without split-K).
    const int kb0 = (int)(((long long)k_total * blockIdx.z) / gridDim.z);
    const int kb1 = (int)(((long long)k_total * (blockIdx.z + 1)) / gridDim.z);
    const int k_blocks = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(&done_bar), 1);
        mbar_init(smem_u32(&drain_bar), 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"((uint32_t)BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_wait();
    pdl_launch_dependents();

    int issued = 0;  // k-blocks the producer has requested
    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < k_blocks; ++kb) {
                const int s = kb % kGemmStages;
                const uint32_t round = kb / kGemmStages;
                if (!mbar_wait(smem_u32(&empty_bar[s]), (round & 1) ^ 1)) {
                    abort_s = 1;
                    break;
                }
                uint8_t *a_dst = base + s * kStageBytes;
                uint8_t *b_dst = a_dst + kABytes;
                const uint32_t bar = smem_u32(&full_bar[s]);
                mbar_expect_tx(bar, kStageBytes);
                const int kx = (kb0 + kb) * kGemmBK;
                tma_load_2d(smem_u32(a_dst), &a_map, kx, m_tile * kGemmBM, bar);
                if (EPI == kPgSwiglu) {
                    tma_load_2d(smem_u32(b_dst), &b_map, kx, n_tile * (BN / 2), bar);
                    tma_load_2d(smem_u32(b_dst + kBBytes / 2), &b2_map, kx, n_tile * (BN / 2), bar);
                } else {
                    // Weight maps use 64-row boxes; a BN-row tile is BN/64 boxes.
#pragma unroll
                    for (int r = 0; r < BN / 64; ++r) {
                        tma_load_2d(smem_u32(b_dst + r * 64 * 128), &b_map, kx, n_tile * BN + r * 64, bar);
                    }
                }
                issued = kb + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < k_blocks; ++kb) {
                const int s = kb % kGemmStages;
                const uint32_t round = kb / kGemmStages;
                if (!mbar_wait(smem_u32(&full_bar[s]), round & 1)) {
                    abort_s = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(base + s * kStageBytes);
                const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                for (int k = 0; k < kGemmBK / 16; ++k) {
                    umma_bf16(tmem, umma_smem_desc(a_addr + k * 32), umma_smem_desc(b_addr + k * 32), kIdesc,
                              (kb > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(smem_u32(&empty_bar[s]));
            }
            umma_commit(smem_u32(&done_bar));
        }
    } else {
        // Epilogue warps 2..5: TMEM lane quadrant = warp % 4; thread = tile row.
        const int quad = warp % 4;
        const int row = m_tile * kGemmBM + quad * 32 + lane;
        const bool live = row < p.M;
        // 64-column residual tiles: the row's residual slice is loaded while
        // the MMAs run (it does not depend on them).
        constexpr bool kPrefetch = EPI == kPgResidual && BN == 64;
        float4 res_pre[kPrefetch ? 16 : 1];
        if (kPrefetch && live && n_tile * BN < p.N) {
            const float4 *s4 = reinterpret_cast<const float4 *>(p.out_f32 + (long long)row * p.ld_out + n_tile * BN);
#pragma unroll
            for (int i = 0; i < (kPrefetch ? 16 : 1); ++i) res_pre[i] = s4[i];
        }
        const bool ok = mbar_wait(smem_u32(&done_bar), 0);
        tc_fence_after();
        const uint32_t acc_addr = tmem + ((uint32_t)(quad * 32) << 16);
        const bool run = ok && (gridDim.z == 1 || split_k_reduce<BN>(p, acc_addr, quad * 32 + lane, &split_last_s));
        if (!ok) {
            if (p.error) *p.error = 4;
            abort_s = 1;
        } else if (run) {
            const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
            if (EPI == kPgResidual) {
                // hidden[row][n] += acc (+ bias): 32 columns per step, float4 traffic.
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(lane_addr + c0, v);
                    const int n0 = n_tile * BN + c0;
                    if (live && n0 < p.N) {
                        float4 *d4 = reinterpret_cast<float4 *>(p.out_f32 + (long long)row * p.ld_out + n0);
                        float4 r[8];
                        if (kPrefetch) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) r[i] = res_pre[(c0 / 4 + i) % (kPrefetch ? 16 : 1)];
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; ++i) r[i] = d4[i];
                        }
                        if (p.bias) {
                            const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + n0);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const float4 b = b4[i];
                                v[4 * i] = __fadd_rn(v[4 * i], b.x);
                                v[4 * i + 1] = __fadd_rn(v[4 * i + 1], b.y);
                                v[4 * i + 2] = __fadd_rn(v[4 * i + 2], b.z);
                                v[4 * i + 3] = __fadd_rn(v[4 * i + 3], b.w);
                            }
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            r[i].x = __fadd_rn(r[i].x, v[4 * i]);
                            r[i].y = __fadd_rn(r[i].y, v[4 * i + 1]);
                            r[i].z = __fadd_rn(r[i].z, v[4 * i + 2]);
                            r[i].w = __fadd_rn(r[i].w, v[4 * i + 3]);
                            d4[i] = r[i];
                        }
                    }
                }
            } else if (EPI == kPgSwiglu) {
#pragma unroll 1
                for (int c0 = 0; c0 < BN / 2; c0 += 16) {
                    float g[16], u[16];
                    tmem_ld16(lane_addr + c0, g);
                    tmem_ld16(lane_addr + BN / 2 + c0, u);
                    const int n0 = n_tile * (BN / 2) + c0;
                    if (live && n0 < p.N) {
                        uint32_t packed[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            // silu(g) * u = g * u / (1 + e^-g), rounded to bf16.
                            const float a0 = g[2 * i] * u[2 * i] *
                                             fast_rcp(1.0f + fast_exp2(g[2 * i] * -1.4426950408889634f));
                            const float a1 = g[2 * i + 1] * u[2 * i + 1] *
                                             fast_rcp(1.0f + fast_exp2(g[2 * i + 1] * -1.4426950408889634f));
                            packed[i] = (uint32_t)f32_to_bf16_rne(a0) | ((uint32_t)f32_to_bf16_rne(a1) << 16);
                        }
                        uint4 *dst = reinterpret_cast<uint4 *>(p.out_bf16 + (long long)row * p.ld_out + n0);
                        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    }
                }
            } else if (EPI == kPgLogits) {
                // Logits rows + greedy argmax per row (`engine.rs:2247-2253`).
                unsigned long long best = 0ull;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(lane_addr + c0, v);
                    const int n0 = n_tile * BN + c0;
                    if (live && n0 < p.N) {
                        float *dst = p.out_f32 ? p.out_f32 + (long long)row * p.ld_out + n0 : nullptr;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (n0 + i < p.N) {
                                if (dst) dst[i] = v[i];
                                const unsigned long long key =
                                    ((unsigned long long)total_order_key(v[i]) << 32) | (unsigned)(n0 + i);
                                best = key > best ? key : best;
                            }
                        }
                    }
                }
                if (live && best != 0ull) atomicMax(p.argmax + row, best);
            } else {  // kPgQkv: BN covers whole heads
                const int hd = p.head_dim;
                const int half = hd >> 1;
                const int pos = p.row_pos ? (live ? p.row_pos[row] : 0) : p.offset + row;
                const int32_t *table = p.page_table + (p.row_pos ? (long long)row * p.table_stride : 0);
                // The row's KV slot, resolved once.
                long long slot_base = -1;  // element index of (page, kv head 0, slot, d 0)
                if (live) {
                    const int pidx = pos / p.page_tokens;
                    const int page = pidx < p.max_pages ? table[pidx] : -1;
                    if (page >= 0 && page < p.num_pages) {
                        slot_base = ((long long)page * p.kv_heads * p.page_tokens + (pos - pidx * p.page_tokens)) * hd;
                    } else if (p.error) {
                        *p.error = 9;
                    }
                }
                const long long head_stride = (long long)p.page_tokens * hd;  // elements between kv heads of a page
#pragma unroll 1
                for (int hb = 0; hb < BN; hb += hd) {
                    const int col0 = n_tile * BN + hb;  // first output feature of this head
                    const int head = col0 / hd;
                    // Per-head q/k norm: a first pass over the head's
                    // accumulators (bias included) for the sum of squares.
                    const float *nw = head < p.q_heads ? p.q_norm
                                                       : (head < p.q_heads + p.kv_heads ? p.k_norm : nullptr);
                    float inv = 1.0f;
                    if (nw) {
                        float ss = 0.0f;
#pragma unroll 1
                        for (int j = 0; j < hd; j += 16) {
                            float a[16];
                            tmem_ld16(lane_addr + hb + j, a);
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                const float v = p.bias ? __fadd_rn(a[e], p.bias[col0 + j + e]) : a[e];
                                ss = fmaf(v, v, ss);
                            }
                        }
                        inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)hd), p.eps));
                    }
#pragma unroll 1
                    for (int j = 0; j < half; j += 16) {
                        float a[16], b[16];
                        tmem_ld16(lane_addr + hb + j, a);
                        tmem_ld16(lane_addr + hb + half + j, b);
                        if (!live || col0 >= p.N) continue;
                        if (p.bias) {
                            const float4 *ba = reinterpret_cast<const float4 *>(p.bias + col0 + j);
                            const float4 *bb = reinterpret_cast<const float4 *>(p.bias + col0 + half + j);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float4 x = ba[i], y = bb[i];
                                a[4 * i] = __fadd_rn(a[4 * i], x.x); a[4 * i + 1] = __fadd_rn(a[4 * i + 1], x.y);
                                a[4 * i + 2] = __fadd_rn(a[4 * i + 2], x.z); a[4 * i + 3] = __fadd_rn(a[4 * i + 3], x.w);
                                b[4 * i] = __fadd_rn(b[4 * i], y.x); b[4 * i + 1] = __fadd_rn(b[4 * i + 1], y.y);
                                b[4 * i + 2] = __fadd_rn(b[4 * i + 2], y.z); b[4 * i + 3] = __fadd_rn(b[4 * i + 3], y.w);
                            }
                        }
                        if (nw) {
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                a[e] = __fmul_rn(a[e], __fmul_rn(inv, nw[j + e]));
                                b[e] = __fmul_rn(b[e], __fmul_rn(inv, nw[half + j + e]));
                            }
                        }
                        if (head < p.q_heads + p.kv_heads) {
                            // ops.rs:693-715: a' = a*cos - b*sin, b' = b*cos + a*sin
                            const float4 *c4 = reinterpret_cast<const float4 *>(p.rope_cos + (long long)pos * half + j);
                            const float4 *s4 = reinterpret_cast<const float4 *>(p.rope_sin + (long long)pos * half + j);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float4 cv = c4[i], sv = s4[i];
                                const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
                                const float ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float va = a[4 * i + e], vb = b[4 * i + e];
                                    a[4 * i + e] = __fsub_rn(__fmul_rn(va, cc[e]), __fmul_rn(vb, ss[e]));
                                    b[4 * i + e] = __fadd_rn(__fmul_rn(vb, cc[e]), __fmul_rn(va, ss[e]));
                                }
                            }
                        }
                        if (head < p.q_heads) {
                            if (p.out_q_f32) {
                                float *q = p.out_q_f32 + (long long)row * p.ld_out + head * hd;
                                store_f32x16(q + j, a);
                                store_f32x16(q + half + j, b);
                            } else {
                                uint16_t *q = p.out_bf16 + (long long)row * p.ld_out + head * hd;
                                store_bf16x16(q + j, a);
                                store_bf16x16(q + half + j, b);
                            }
                        } else if (slot_base >= 0) {
                            const bool is_k = head < p.q_heads + p.kv_heads;
                            const int kvh = is_k ? head - p.q_heads : head - p.q_heads - p.kv_heads;
                            void *cache = is_k ? p.k_cache : p.v_cache;
                            const long long e0 = slot_base + kvh * head_stride;
                            if (p.kv_f32) {
                                float *dst = static_cast<float *>(cache) + e0;
                                store_f32x16(dst + j, a);
                                store_f32x16(dst + half + j, b);
                            } else {
                                uint16_t *dst = static_cast<uint16_t *>(cache) + e0;
                                store_bf16x16(dst + j, a);
                                store_bf16x16(dst + half + j, b);
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (abort_s) {
        // A wait gave up: let this CTA's copies and MMAs still in flight land
        // before its shared memory and TMEM are released (bounded waits).
        if (warp == 0 && lane == 0) {
            for (int kb = max(0, issued - kGemmStages); kb < issued; ++kb) {
                mbar_wait(smem_u32(&full_bar[kb % kGemmStages]), (kb / kGemmStages) & 1);
            }
        } else if (warp == 1 && lane == 0) {
            umma_commit(smem_u32(&drain_bar));
            mbar_wait(smem_u32(&drain_bar), 0);
        }
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && p.error && *p.error == 0) *p.error = 5;
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN));
    }
}

template <int BN>
constexpr size_t prefill_gemm_smem() {
    return (size_t)kGemmStages * (kGemmBM * kGemmBK * 2 + BN * kGemmBK * 2) + 1024;
}

}  // namespace cheetah
