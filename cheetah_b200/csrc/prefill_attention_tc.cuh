// Causal GQA attention for a prefill chunk on the 5th-generation tensor cores
// (head_dim 64, bf16 paged KV cache, pages of a multiple of 64 tokens): the
// same contract and results as prefill_attention_kernel (the batched form of
// `forward_layer_chunk`, `qwen2.rs:314-343`), with S = Q K^T and O = P V as
// tcgen05.mma (kind::f16, f32 accumulation in TMEM).
//
// CTA = 128 consecutive tokens x one query head; 192 threads:
//   warp 0      TMA producer: the Q tile once, then 128-key K and V tiles
//               (two 64-key boxes each, 128-byte swizzle, no multicast)
//               through a kTcStages-deep ring;
//   warp 1      allocates 512 TMEM columns; lane 0 issues the MMAs:
//               S_j = Q K_j^T (M=128, N=128 keys, K=64) into S buffer j%2,
//               then, once the softmax has written P_j, O_t = P_j V_j
//               (M=128, N=64, K=128 keys; V read MN-major) into the O_t
//               columns. S_{j+1} is issued before PV_j, so the tensor core
//               computes the next scores while the softmax runs;
//   warps 2-5   softmax, one thread per query row (its TMEM lane): load the
//               S row, causal/window mask, online max and sum in log2 units,
//               P_j as bf16 into shared memory in the K-major swizzled
//               layout the MMA reads, and O = O * alpha_{j-1} + O_t(j-1) in
//               registers as each PV completes.
// Key-range splits over blockIdx.z write unnormalised partials (O, m in log2
// units, l) in prefill_attention_kernel's format, combined by
// prefill_merge_kernel. All mbarrier waits are bounded: on a timeout the CTA
// sets the error flag, waits (bounded) for its own copies and MMAs in flight,
// frees its TMEM and exits.
#pragma once

#include "gemm_tcgen05.cuh"
#include "prefill_attention.cuh"

namespace cheetah {

constexpr int kTcRows = 128;       // query rows per CTA
constexpr int kTcKeys = 128;       // keys per tile
constexpr int kTcStages = 3;       // K/V ring depth
constexpr int kTcThreads = 192;
constexpr int kTcTmemCols = 512;   // S0 | S1 | O_t (64) | unused
constexpr int kTcOtCol = 2 * kTcKeys;
constexpr int kTcQBytes = kTcRows * 64 * 2;        // 16 KB
constexpr int kTcKvBytes = kTcKeys * 64 * 2;       // 16 KB per K or V tile
constexpr int kTcPBytes = kTcRows * kTcKeys * 2;   // 32 KB

inline size_t prefill_attention_tc_smem() {
    return (size_t)kTcQBytes + (size_t)kTcStages * 2 * kTcKvBytes + kTcPBytes + 1024;
}

// MN-major operand with 128-byte swizzle (rows of 128 B along N, 8-row atoms
// along K, SBO = 1024 B between K atoms); one 64-element atom along N.
__device__ __forceinline__ uint64_t umma_smem_desc_mn(uint32_t addr) {
    uint64_t desc = 0;
    desc |= (uint64_t)((addr >> 4) & 0x3FFF);
    desc |= (uint64_t)1 << 16;
    desc |= (uint64_t)(1024 >> 4) << 32;
    desc |= (uint64_t)1 << 46;
    desc |= (uint64_t)2 << 61;
    return desc;
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Pool rows of key tile `tile`'s two 64-key spans for KV head `kvh` (a span
// never crosses a page: page_tokens is a multiple of 64). A span past the
// chunk's last position `pos_last` holds only masked keys: it re-reads span 0
// (always in range) so the K/V ring holds finite values. A page-table entry
// out of range sets error 6 where its span holds visible keys.
__device__ __forceinline__ void kv_tile_rows(const PrefillAttnParams &p, int tile, int kvh, int pos_last,
                                             int (&rows)[2]) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int pos0 = tile * kTcKeys + b * 64;
        const int pidx = pos0 / p.page_tokens;
        const int page = pidx < p.max_pages ? p.page_table[pidx] : -1;
        if (page < 0 || page >= p.num_pages) {
            if (b == 0 || pos0 <= pos_last) {
                if (p.error) *p.error = 6;
            }
            rows[b] = b == 0 ? (int)p.layer_row_offset : rows[0];
        } else {
            rows[b] = (int)(p.layer_row_offset + ((long long)page * p.kv_heads + kvh) * p.page_tokens +
                            (pos0 - pidx * p.page_tokens));
        }
        if (b == 1 && pos0 > pos_last) rows[1] = rows[0];
    }
}

__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                                const __grid_constant__ CUtensorMap v_map, const PrefillAttnParams p) {
    constexpr int HD = 64;
    constexpr uint32_t kIdescS = umma_idesc_bf16(kTcRows, kTcKeys);
    constexpr uint32_t kIdescPV = umma_idesc_bf16(kTcRows, HD) | (1u << 16);  // B (V) MN-major
    extern __shared__ __align__(1024) uint8_t attn_tc_smem[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t kv_full[kTcStages];
    __shared__ __align__(8) uint64_t kv_empty[kTcStages];
    __shared__ __align__(8) uint64_t s_full[2];
    __shared__ __align__(8) uint64_t s_empty[2];
    __shared__ __align__(8) uint64_t p_full;
    __shared__ __align__(8) uint64_t o_full;
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(attn_tc_smem) + 1023) & ~uintptr_t(1023));
    uint8_t *q_s = base;
    uint8_t *ring = q_s + kTcQBytes;
    uint8_t *p_s = ring + kTcStages * 2 * kTcKvBytes;
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int group = p.q_heads / p.kv_heads;
    const int head = blockIdx.y;
    const int kvh = head / group;
    const int t0 = blockIdx.x * kTcRows;
    const int t_last = min(p.T, t0 + kTcRows) - 1;
    const int pos_first = p.offset + t0;
    const int pos_last = p.offset + t_last;
    int ws = 0;
    if (p.window > 0) ws = max(0, pos_first + 1 - p.window);
    const int all_lo = ws / kTcKeys;
    const int all_hi = pos_last / kTcKeys + 1;
    const int per_split = (all_hi - all_lo + p.splits - 1) / p.splits;
    const int split = blockIdx.z;
    const int tile_lo = all_lo + split * per_split;
    const int tile_hi = min(all_hi, tile_lo + per_split);
    const int n_tiles = max(0, tile_hi - tile_lo);

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&q_full), 1);
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(smem_u32(&kv_full[s]), 1);
            mbar_init(smem_u32(&kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&s_full[b]), 1);
            mbar_init(smem_u32(&s_empty[b]), kTcRows);
        }
        mbar_init(smem_u32(&p_full), kTcRows);
        mbar_init(smem_u32(&o_full), 1);
        mbar_init(smem_u32(&drain_bar), 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"((uint32_t)kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_wait();
    pdl_launch_dependents();

    int issued = 0;  // K/V tiles the producer has requested
    if (warp == 0) {
        if (lane == 0 && n_tiles > 0) {
            mbar_expect_tx(smem_u32(&q_full), kTcQBytes);
            tma_load_2d(smem_u32(q_s), &q_map, head * HD, t0, smem_u32(&q_full));
            for (int j = 0; j < n_tiles; ++j) {
                const int s = j % kTcStages;
                if (!mbar_wait(smem_u32(&kv_empty[s]), ((j / kTcStages) & 1) ^ 1)) {
                    abort_s = 1;
                    break;
                }
                const int tile = tile_lo + j;
                int rows[2];
                kv_tile_rows(p, tile, kvh, pos_last, rows);
                uint8_t *ks = ring + s * 2 * kTcKvBytes;
                uint8_t *vs = ks + kTcKvBytes;
                const uint32_t bar = smem_u32(&kv_full[s]);
                mbar_expect_tx(bar, 2 * kTcKvBytes);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    tma_load_2d(smem_u32(ks + b * 64 * 128), &k_map, 0, rows[b], bar);
                    tma_load_2d(smem_u32(vs + b * 64 * 128), &v_map, 0, rows[b], bar);
                }
                issued = j + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && n_tiles > 0) {
            const uint32_t q_addr = smem_u32(q_s);
            const uint32_t p_addr = smem_u32(p_s);
            bool ok = mbar_wait(smem_u32(&q_full), 0);
            auto issue_s = [&](int j) -> bool {
                const int s = j % kTcStages;
                if (!mbar_wait(smem_u32(&kv_full[s]), (j / kTcStages) & 1)) return false;
                if (!mbar_wait(smem_u32(&s_empty[j & 1]), ((j >> 1) & 1) ^ 1)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(ring + s * 2 * kTcKvBytes);
                const uint32_t d = tmem + (uint32_t)((j & 1) * kTcKeys);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    umma_bf16(d, umma_smem_desc(q_addr + k * 32), umma_smem_desc(k_addr + k * 32), kIdescS,
                              k > 0 ? 1u : 0u);
                }
                umma_commit(smem_u32(&s_full[j & 1]));
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < n_tiles; ++j) {
                if (j + 1 < n_tiles && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait(smem_u32(&p_full), j & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int s = j % kTcStages;
                const uint32_t v_addr = smem_u32(ring + s * 2 * kTcKvBytes + kTcKvBytes);
#pragma unroll
                for (int k = 0; k < kTcKeys / 16; ++k) {
                    umma_bf16(tmem + kTcOtCol, umma_smem_desc(p_addr + (k >> 2) * (kTcRows * 128) + (k & 3) * 32),
                              umma_smem_desc_mn(v_addr + k * 2048), kIdescPV, k > 0 ? 1u : 0u);
                }
                umma_commit(smem_u32(&o_full));
                umma_commit(smem_u32(&kv_empty[s]));
            }
            if (!ok) abort_s = 1;
        }
    } else {
        // Softmax warps 2..5: TMEM lane quadrant = warp % 4; thread = query row.
        const int quad = warp % 4;
        const int r = quad * 32 + lane;
        const int t = t0 + r;
        const int qpos = p.offset + t;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const float scale_log2 = p.scale * 1.4426950408889634f;
        float o[HD];
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = 0.0f;
        float m_run = -INFINITY, l_run = 0.0f, alpha_prev = 1.0f;
        bool ok = true;
        // O = O * alpha + O_t, 32 columns at a time.
        auto fold = [&](float alpha) {
#pragma unroll
            for (int h = 0; h < HD / 32; ++h) {
                float ot[32];
                tmem_ld32_nowait(tmem + lane_off + kTcOtCol + h * 32, ot);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[h * 32 + i] = fmaf(o[h * 32 + i], alpha, ot[i]);
            }
        };
        uint8_t *p_row0 = p_s + r * 128;
        for (int j = 0; j < n_tiles; ++j) {
            if (!mbar_wait(smem_u32(&s_full[j & 1]), (j >> 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sc[kTcKeys];
            const uint32_t s_addr = tmem + lane_off + (uint32_t)((j & 1) * kTcKeys);
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c) tmem_ld32_nowait(s_addr + c * 32, sc + c * 32);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(smem_u32(&s_empty[j & 1]));
            const int kp0 = (tile_lo + j) * kTcKeys;
            // Tiles wholly at or below the CTA's first position need no mask
            // (no window); otherwise key i is visible iff wlo < i <= lim.
            if (p.window > 0 || kp0 + kTcKeys - 1 > pos_first) {
                const int lim = qpos - kp0;
                const int wlo = p.window > 0 ? lim - p.window : -1;
#pragma unroll
                for (int i = 0; i < kTcKeys; ++i) sc[i] = (i <= lim && i > wlo) ? sc[i] : -INFINITY;
            }
            // Row max of the raw scores (scale > 0), eight partial chains.
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = sc[k];
#pragma unroll
            for (int i = 8; i < kTcKeys; ++i) mx[i & 7] = fmaxf(mx[i & 7], sc[i]);
#pragma unroll
            for (int k = 0; k < 4; ++k) mx[k] = fmaxf(mx[k], mx[k + 4]);
            const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            const float m_new = fmaxf(m_run, tmax * scale_log2);
            const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
            // p = 2^(s * scale_log2 - m_new); a masked key (-inf) gives 0.
            const float neg_m = m_new == -INFINITY ? 0.0f : -m_new;
            float sums[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) sums[k] = 0.0f;
            uint32_t packed[kTcKeys / 2];
#pragma unroll
            for (int i = 0; i < kTcKeys / 2; ++i) {
                const float e0 = fast_exp2(fmaf(sc[2 * i], scale_log2, neg_m));
                const float e1 = fast_exp2(fmaf(sc[2 * i + 1], scale_log2, neg_m));
                sums[i & 7] += e0 + e1;
                packed[i] = pack_bf16(e0, e1);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) sums[k] += sums[k + 4];
            const float rsum = (sums[0] + sums[1]) + (sums[2] + sums[3]);
            l_run = l_run * alpha + rsum;
            m_run = m_new;
            if (j > 0) {
                // PV_{j-1} done: fold O_t into O; P's buffer is free again.
                if (!mbar_wait(smem_u32(&o_full), (j - 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                fold(alpha_prev);
                tc_fence_before();
            }
            // P_j row r, K-major with 128-byte swizzle: keys 64b..64b+63 in
            // block b, 16-byte chunk c of the row at (c ^ (r & 7)).
#pragma unroll
            for (int c = 0; c < kTcKeys / 8; ++c) {
                const int blk = c >> 3, cc = c & 7;
                uint4 *dst = reinterpret_cast<uint4 *>(p_row0 + blk * (kTcRows * 128) + ((cc ^ (r & 7)) << 4));
                *dst = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(smem_u32(&p_full));
            alpha_prev = alpha;
        }
        if (ok && n_tiles > 0) {
            if (mbar_wait(smem_u32(&o_full), (n_tiles - 1) & 1)) {
                tc_fence_after();
                fold(alpha_prev);
            } else {
                ok = false;
            }
        }
        if (!ok) {
            abort_s = 1;
        } else if (t <= t_last) {
            if (p.splits > 1) {
                const long long rh = ((long long)split * p.T + t) * p.q_heads + head;
                float4 *dst = reinterpret_cast<float4 *>(p.part_o + rh * HD);
#pragma unroll
                for (int i = 0; i < HD / 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                *reinterpret_cast<float2 *>(p.part_ml + rh * 2) = make_float2(m_run, l_run);
            } else {
                const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + (long long)t * p.q_heads * HD + head * HD);
#pragma unroll
                for (int i = 0; i < HD / 8; ++i) {
                    dst[i] = make_uint4(pack_bf16(o[8 * i] * inv, o[8 * i + 1] * inv),
                                        pack_bf16(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                                        pack_bf16(o[8 * i + 4] * inv, o[8 * i + 5] * inv),
                                        pack_bf16(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (abort_s) {
        // A wait gave up: let this CTA's copies and MMAs still in flight land
        // before its shared memory and TMEM are released (bounded waits).
        if (warp == 0 && lane == 0 && n_tiles > 0) {
            mbar_wait(smem_u32(&q_full), 0);
            for (int j = max(0, issued - kTcStages); j < issued; ++j) {
                mbar_wait(smem_u32(&kv_full[j % kTcStages]), (j / kTcStages) & 1);
            }
        } else if (warp == 1 && lane == 0) {
            umma_commit(smem_u32(&drain_bar));
            mbar_wait(smem_u32(&drain_bar), 0);
        }
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && p.error) *p.error = 8;
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcTmemCols));
    }
}

// ---- O accumulated in TMEM (head_dim 64 and 128) ---------------------------
// The same contract with O kept in TMEM instead of registers. Differences from
// the kernel above: Q and every K / V tile are two 64-dimension halves
// (K-major, 128-byte swizzle), loaded as 32-row boxes of the cache's tensor
// maps; S = Q K^T takes eight K=16 steps across the halves; O = P V is two
// N=64 MMAs (one per V half) that accumulate into one 128-column O in TMEM
// across all key tiles. A softmax thread keeps no O in registers: when its
// warp's running max grows (alpha < 1 for some row) it rescales its O row in
// TMEM (load, multiply, store) before releasing P_j; rows whose max did not
// grow are multiplied by 1 (exact). The last tile's O is read back once,
// normalised and stored. At head_dim 128: two K/V stages of 64 KB (Q 32 KB, ring
// 128 KB, P 32 KB); at 64: three of 32 KB. The library launches it for
// head_dim 128; head_dim 64 runs prefill_attention_tc_pair_kernel below (two
// query tiles per CTA), or the kernel above when that is switched off.
template <int HD>
struct Tc2 {
    static constexpr int kStages = HD == 64 ? 3 : 2;
    static constexpr int kHalves = HD / 64;
    static constexpr int kHalf = kTcKeys * 128;       // bytes of one 64-dimension half (128 rows x 128 B)
    static constexpr int kQBytes = kTcRows * HD * 2;  // 16 / 32 KB
    static constexpr int kKvBytes = kTcKeys * HD * 2; // per K or V tile
    static constexpr int kOCol = 2 * kTcKeys;         // O: HD TMEM columns after S0 | S1
};

template <int HD>
inline size_t prefill_attention_tc2_smem() {
    using C = Tc2<HD>;
    return (size_t)C::kQBytes + (size_t)C::kStages * 2 * C::kKvBytes + kTcPBytes + 1024;
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attention_tc2_kernel(const __grid_constant__ CUtensorMap q_map,
                                 const __grid_constant__ CUtensorMap k_map,
                                 const __grid_constant__ CUtensorMap v_map, const PrefillAttnParams p) {
    using C = Tc2<HD>;
    constexpr int kTc2Stages = C::kStages;
    constexpr int kTc2QBytes = C::kQBytes;
    constexpr int kTc2KvBytes = C::kKvBytes;
    constexpr int kTc2Half = C::kHalf;
    constexpr int kTc2OCol = C::kOCol;
    constexpr int kBoxRows = kTileBytes / (HD * 2);  // rows of one cache-map box: 64 (d=64) or 32 (d=128)
    constexpr uint32_t kIdescS = umma_idesc_bf16(kTcRows, kTcKeys);
    constexpr uint32_t kIdescPV = umma_idesc_bf16(kTcRows, 64) | (1u << 16);  // B (V) MN-major
    extern __shared__ __align__(1024) uint8_t attn_tc2_smem[];
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t kv_full[kTc2Stages];
    __shared__ __align__(8) uint64_t kv_empty[kTc2Stages];
    __shared__ __align__(8) uint64_t s_full[2];
    __shared__ __align__(8) uint64_t s_empty[2];
    __shared__ __align__(8) uint64_t p_full;
    __shared__ __align__(8) uint64_t o_full;
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(attn_tc2_smem) + 1023) & ~uintptr_t(1023));
    uint8_t *q_s = base;
    uint8_t *ring = q_s + kTc2QBytes;
    uint8_t *p_s = ring + kTc2Stages * 2 * kTc2KvBytes;
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int group = p.q_heads / p.kv_heads;
    const int head = blockIdx.y;
    const int kvh = head / group;
    const int t0 = blockIdx.x * kTcRows;
    const int t_last = min(p.T, t0 + kTcRows) - 1;
    const int pos_first = p.offset + t0;
    const int pos_last = p.offset + t_last;
    int ws = 0;
    if (p.window > 0) ws = max(0, pos_first + 1 - p.window);
    const int all_lo = ws / kTcKeys;
    const int all_hi = pos_last / kTcKeys + 1;
    const int per_split = (all_hi - all_lo + p.splits - 1) / p.splits;
    const int split = blockIdx.z;
    const int tile_lo = all_lo + split * per_split;
    const int tile_hi = min(all_hi, tile_lo + per_split);
    const int n_tiles = max(0, tile_hi - tile_lo);

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&q_full), 1);
        for (int s = 0; s < kTc2Stages; ++s) {
            mbar_init(smem_u32(&kv_full[s]), 1);
            mbar_init(smem_u32(&kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&s_full[b]), 1);
            mbar_init(smem_u32(&s_empty[b]), kTcRows);
        }
        mbar_init(smem_u32(&p_full), kTcRows);
        mbar_init(smem_u32(&o_full), 1);
        mbar_init(smem_u32(&drain_bar), 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"((uint32_t)kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_wait();
    pdl_launch_dependents();

    int issued = 0;  // K/V tiles the producer has requested
    if (warp == 0) {
        if (lane == 0 && n_tiles > 0) {
            mbar_expect_tx(smem_u32(&q_full), kTc2QBytes);
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h)
                tma_load_2d(smem_u32(q_s + h * kTc2Half), &q_map, head * HD + h * 64, t0, smem_u32(&q_full));
            for (int j = 0; j < n_tiles; ++j) {
                const int s = j % kTc2Stages;
                if (!mbar_wait(smem_u32(&kv_empty[s]), ((j / kTc2Stages) & 1) ^ 1)) {
                    abort_s = 1;
                    break;
                }
                const int tile = tile_lo + j;
                int rows[2];
                kv_tile_rows(p, tile, kvh, pos_last, rows);
                uint8_t *ks = ring + s * 2 * kTc2KvBytes;
                uint8_t *vs = ks + kTc2KvBytes;
                const uint32_t bar = smem_u32(&kv_full[s]);
                mbar_expect_tx(bar, 2 * kTc2KvBytes);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
#pragma unroll
                    for (int r = 0; r < 64 / kBoxRows; ++r) {
                        const uint32_t row_off = (uint32_t)((b * 64 + r * kBoxRows) * 128);
#pragma unroll
                        for (int h = 0; h < C::kHalves; ++h) {
                            tma_load_2d(smem_u32(ks + h * kTc2Half + row_off), &k_map, h * 64, rows[b] + r * kBoxRows,
                                        bar);
                            tma_load_2d(smem_u32(vs + h * kTc2Half + row_off), &v_map, h * 64, rows[b] + r * kBoxRows,
                                        bar);
                        }
                    }
                }
                issued = j + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && n_tiles > 0) {
            const uint32_t q_addr = smem_u32(q_s);
            const uint32_t p_addr = smem_u32(p_s);
            bool ok = mbar_wait(smem_u32(&q_full), 0);
            auto issue_s = [&](int j) -> bool {
                const int s = j % kTc2Stages;
                if (!mbar_wait(smem_u32(&kv_full[s]), (j / kTc2Stages) & 1)) return false;
                if (!mbar_wait(smem_u32(&s_empty[j & 1]), ((j >> 1) & 1) ^ 1)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(ring + s * 2 * kTc2KvBytes);
                const uint32_t d = tmem + (uint32_t)((j & 1) * kTcKeys);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t off = (uint32_t)((k >> 2) * kTc2Half + (k & 3) * 32);
                    umma_bf16(d, umma_smem_desc(q_addr + off), umma_smem_desc(k_addr + off), kIdescS, k > 0 ? 1u : 0u);
                }
                umma_commit(smem_u32(&s_full[j & 1]));
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < n_tiles; ++j) {
                if (j + 1 < n_tiles && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait(smem_u32(&p_full), j & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int s = j % kTc2Stages;
                const uint32_t v_addr = smem_u32(ring + s * 2 * kTc2KvBytes + kTc2KvBytes);
#pragma unroll
                for (int h = 0; h < C::kHalves; ++h) {
#pragma unroll
                    for (int k = 0; k < kTcKeys / 16; ++k) {
                        umma_bf16(tmem + kTc2OCol + h * 64,
                                  umma_smem_desc(p_addr + (k >> 2) * (kTcRows * 128) + (k & 3) * 32),
                                  umma_smem_desc_mn(v_addr + h * kTc2Half + k * 2048), kIdescPV,
                                  (j > 0 || k > 0) ? 1u : 0u);
                    }
                }
                umma_commit(smem_u32(&o_full));
                umma_commit(smem_u32(&kv_empty[s]));
            }
            if (!ok) abort_s = 1;
        }
    } else {
        // Softmax warps 2..5: TMEM lane quadrant = warp % 4; thread = query row.
        const int quad = warp % 4;
        const int r = quad * 32 + lane;
        const int t = t0 + r;
        const int qpos = p.offset + t;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t o_addr = tmem + lane_off + kTc2OCol;
        const float scale_log2 = p.scale * 1.4426950408889634f;
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        uint8_t *p_row0 = p_s + r * 128;
        for (int j = 0; j < n_tiles; ++j) {
            // Waits decide warp-uniformly (the TMEM accesses below are warp-wide).
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&s_full[j & 1]), (j >> 1) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sc[kTcKeys];
            const uint32_t s_addr = tmem + lane_off + (uint32_t)((j & 1) * kTcKeys);
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c) tmem_ld32_nowait(s_addr + c * 32, sc + c * 32);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(smem_u32(&s_empty[j & 1]));
            const int kp0 = (tile_lo + j) * kTcKeys;
            if (p.window > 0 || kp0 + kTcKeys - 1 > pos_first) {
                const int lim = qpos - kp0;
                const int wlo = p.window > 0 ? lim - p.window : -1;
#pragma unroll
                for (int i = 0; i < kTcKeys; ++i) sc[i] = (i <= lim && i > wlo) ? sc[i] : -INFINITY;
            }
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = sc[k];
#pragma unroll
            for (int i = 8; i < kTcKeys; ++i) mx[i & 7] = fmaxf(mx[i & 7], sc[i]);
#pragma unroll
            for (int k = 0; k < 4; ++k) mx[k] = fmaxf(mx[k], mx[k + 4]);
            const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            const float m_new = fmaxf(m_run, tmax * scale_log2);
            const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
            const float neg_m = m_new == -INFINITY ? 0.0f : -m_new;
            float sums[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) sums[k] = 0.0f;
            uint32_t packed[kTcKeys / 2];
#pragma unroll
            for (int i = 0; i < kTcKeys / 2; ++i) {
                const float e0 = fast_exp2(fmaf(sc[2 * i], scale_log2, neg_m));
                const float e1 = fast_exp2(fmaf(sc[2 * i + 1], scale_log2, neg_m));
                sums[i & 7] += e0 + e1;
                packed[i] = pack_bf16(e0, e1);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) sums[k] += sums[k + 4];
            const float rsum = (sums[0] + sums[1]) + (sums[2] + sums[3]);
            l_run = l_run * alpha + rsum;
            m_run = m_new;
            if (j > 0) {
                // PV_{j-1} done: P's buffer is free and O holds tiles < j.
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&o_full), (j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // O *= alpha where any row of the warp's max grew (warp-wide
                // TMEM access; alpha == 1 rows are unchanged).
                if (__any_sync(0xFFFFFFFFu, alpha < 1.0f)) {
#pragma unroll 1
                    for (int c = 0; c < HD / 32; ++c) {
                        float ov[32];
                        tmem_ld32_nowait(o_addr + c * 32, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                        tmem_st32(o_addr + c * 32, ov);
                    }
                }
                tc_fence_before();
            }
#pragma unroll
            for (int c = 0; c < kTcKeys / 8; ++c) {
                const int blk = c >> 3, cc = c & 7;
                uint4 *dst = reinterpret_cast<uint4 *>(p_row0 + blk * (kTcRows * 128) + ((cc ^ (r & 7)) << 4));
                *dst = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(smem_u32(&p_full));
        }
        if (ok && n_tiles > 0) {
            if (__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&o_full), (n_tiles - 1) & 1))) {
                tc_fence_after();
            } else {
                ok = false;
            }
        }
        if (!ok) {
            abort_s = 1;
        } else if (n_tiles > 0) {
            // O row from TMEM (warp-wide loads), then partial or output.
            const bool live = t <= t_last;
            const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
            const long long rh = ((long long)split * p.T + t) * p.q_heads + head;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float ov[32];
                tmem_ld32_nowait(o_addr + c * 32, ov);
                tmem_wait_ld();
                if (!live) continue;
                if (p.splits > 1) {
                    float4 *dst = reinterpret_cast<float4 *>(p.part_o + rh * HD + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i) dst[i] = make_float4(ov[4 * i], ov[4 * i + 1], ov[4 * i + 2], ov[4 * i + 3]);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + (long long)t * p.q_heads * HD + head * HD + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        dst[i] = make_uint4(pack_bf16(ov[8 * i] * inv, ov[8 * i + 1] * inv),
                                            pack_bf16(ov[8 * i + 2] * inv, ov[8 * i + 3] * inv),
                                            pack_bf16(ov[8 * i + 4] * inv, ov[8 * i + 5] * inv),
                                            pack_bf16(ov[8 * i + 6] * inv, ov[8 * i + 7] * inv));
                    }
                }
            }
            if (live && p.splits > 1) *reinterpret_cast<float2 *>(p.part_ml + rh * 2) = make_float2(m_run, l_run);
        } else if (t <= t_last) {
            // A key split with no tiles (the split count rounds up): an empty
            // partial (O = 0, m = -inf, l = 0) that the merge weighs by zero.
            const long long rh = ((long long)split * p.T + t) * p.q_heads + head;
            if (p.splits > 1) {
                float4 *dst = reinterpret_cast<float4 *>(p.part_o + rh * HD);
#pragma unroll
                for (int i = 0; i < HD / 4; ++i) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float2 *>(p.part_ml + rh * 2) = make_float2(-INFINITY, 0.0f);
            } else {
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + (long long)t * p.q_heads * HD + head * HD);
#pragma unroll
                for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (abort_s) {
        // A wait gave up: let this CTA's copies and MMAs still in flight land
        // before its shared memory and TMEM are released (bounded waits).
        if (warp == 0 && lane == 0 && n_tiles > 0) {
            mbar_wait(smem_u32(&q_full), 0);
            for (int j = max(0, issued - kTc2Stages); j < issued; ++j) {
                mbar_wait(smem_u32(&kv_full[j % kTc2Stages]), (j / kTc2Stages) & 1);
            }
        } else if (warp == 1 && lane == 0) {
            umma_commit(smem_u32(&drain_bar));
            mbar_wait(smem_u32(&drain_bar), 0);
        }
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && p.error) *p.error = 8;
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcTmemCols));
    }
}

// ---- two query tiles per CTA (head_dim 64) --------------------------------
// 256 query rows x one head per CTA: two softmax groups (warps 2-5 and 6-9,
// each covering the four TMEM lane quadrants) work on the two 128-row query
// tiles A and B against the same K/V tiles, so while one group runs its
// softmax the tensor core computes the other group's S or P.V.
//
// S tiles rotate through three 128-column TMEM buffers in the order S_A(0),
// S_B(0), S_A(1), S_B(1), ... (S tile n = 2j + g in buffer n % 3), so a
// group's next S is computed while it still runs the softmax of the current
// one: per key tile j the MMA thread issues PV_A(j), S_B(j+1), PV_B(j) (the
// K/V stage is then free), S_A(j+2). Each S buffer has its own full/empty
// barriers, so no barrier can run two phases ahead of its consumer. O of each
// group is accumulated in TMEM (columns 384 and 448) and rescaled only when a
// row's running max grows by more than 2^8 (until then the old max is kept:
// P <= 256, and O and l use the same max, so the normalised result is the
// same softmax). A softmax thread reads its S row from TMEM twice, 64 columns
// at a time (the row max, then the exponentials), which keeps it within the
// 168 registers a thread of a 10-warp CTA can have. Shared memory: Q_A, Q_B
// (16 KB each), four 32 KB K/V stages, P_A, P_B (32 KB each): 225 KB.
// Optional per-key-tile timeline of one CTA (query block 0, head 0, split 0
// of the layer-0 launches; the last such launch's stamps remain), for
// profiling builds (-DCHEETAH_ATTN_TRACE): clock64 cycles since the CTA
// started. Events of tile j: 0-3 softmax group A (S landed, row max done,
// O rescaled, P released), 4-7 the same for group B, 8 MMA thread saw P_A,
// 9 issued P.V_A, 10 issued S_B(j+1), 11 saw P_B, 12 issued P.V_B, 13 issued
// S_A(j+2), 14 producer issued tile j's loads.
constexpr int kAttnTraceTiles = 16;
constexpr int kAttnTraceEvents = 16;
#ifdef CHEETAH_ATTN_TRACE
__device__ long long g_attn_trace[kAttnTraceTiles][kAttnTraceEvents];
#define ATTN_TRACE(cond, j, ev)                                                  \
    do {                                                                         \
        if ((cond) && (j) < kAttnTraceTiles) g_attn_trace[(j)][(ev)] = clock64() - trace_t0; \
    } while (0)
#else
#define ATTN_TRACE(cond, j, ev) \
    do {                        \
    } while (0)
#endif

constexpr int kTpRows = 2 * kTcRows;  // query rows per CTA
constexpr int kTpThreads = 320;       // producer, MMA, 2 x 4 softmax warps
constexpr int kTpStages = 4;
constexpr int kTpSBufs = 3;
constexpr int kTpQBytes = kTcRows * 64 * 2;   // per query tile
constexpr int kTpKvBytes = kTcKeys * 64 * 2;  // per K or V tile
constexpr int kTpOCol = kTpSBufs * kTcKeys;   // O_A at 384, O_B at 448
constexpr float kTpRescaleLog2 = 8.0f;        // keep the running max until it grows by 2^8
static_assert(kTpOCol + 2 * 64 <= kTcTmemCols, "TMEM columns");

inline size_t prefill_attention_tc_pair_smem() {
    return (size_t)2 * kTpQBytes + (size_t)kTpStages * 2 * kTpKvBytes + 2 * (size_t)kTcPBytes + 1024;
}

__global__ void __launch_bounds__(kTpThreads, 1)
    prefill_attention_tc_pair_kernel(const __grid_constant__ CUtensorMap q_map,
                                     const __grid_constant__ CUtensorMap k_map,
                                     const __grid_constant__ CUtensorMap v_map, const PrefillAttnParams p) {
    constexpr int HD = 64;
    constexpr uint32_t kIdescS = umma_idesc_bf16(kTcRows, kTcKeys);
    constexpr uint32_t kIdescPV = umma_idesc_bf16(kTcRows, HD) | (1u << 16);  // B (V) MN-major
    extern __shared__ __align__(1024) uint8_t attn_tp_smem[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t kv_full[kTpStages];
    __shared__ __align__(8) uint64_t kv_empty[kTpStages];
    __shared__ __align__(8) uint64_t s_full[kTpSBufs];  // per S buffer
    __shared__ __align__(8) uint64_t s_empty[kTpSBufs];
    __shared__ __align__(8) uint64_t p_full[2];  // per group
    __shared__ __align__(8) uint64_t o_full[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(attn_tp_smem) + 1023) & ~uintptr_t(1023));
    uint8_t *q_s = base;                                // Q_A | Q_B
    uint8_t *ring = q_s + 2 * kTpQBytes;
    uint8_t *p_s = ring + kTpStages * 2 * kTpKvBytes;  // P_A | P_B
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int group = p.q_heads / p.kv_heads;
    const int head = blockIdx.y;
    const int kvh = head / group;
    const int t0 = blockIdx.x * kTpRows;
    const int t_last = min(p.T, t0 + kTpRows) - 1;
    const int pos_first = p.offset + t0;
    const int pos_last = p.offset + t_last;
    int ws = 0;
    if (p.window > 0) ws = max(0, pos_first + 1 - p.window);
    const int all_lo = ws / kTcKeys;
    const int all_hi = pos_last / kTcKeys + 1;
    const int per_split = (all_hi - all_lo + p.splits - 1) / p.splits;
    const int split = blockIdx.z;
    const int tile_lo = all_lo + split * per_split;
    const int tile_hi = min(all_hi, tile_lo + per_split);
    const int n_tiles = max(0, tile_hi - tile_lo);
#ifdef CHEETAH_ATTN_TRACE
    const long long trace_t0 = clock64();
    const bool trace = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && p.layer_row_offset == 0;
#endif

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&q_full), 1);
        for (int s = 0; s < kTpStages; ++s) {
            mbar_init(smem_u32(&kv_full[s]), 1);
            mbar_init(smem_u32(&kv_empty[s]), 1);
        }
        for (int b = 0; b < kTpSBufs; ++b) {
            mbar_init(smem_u32(&s_full[b]), 1);
            mbar_init(smem_u32(&s_empty[b]), kTcRows);
        }
        for (int g = 0; g < 2; ++g) {
            mbar_init(smem_u32(&p_full[g]), kTcRows);
            mbar_init(smem_u32(&o_full[g]), 1);
        }
        mbar_init(smem_u32(&drain_bar), 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"((uint32_t)kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_wait();
    pdl_launch_dependents();

    int issued = 0;  // K/V tiles the producer has requested
    if (warp == 0) {
        if (lane == 0 && n_tiles > 0) {
            // Both query tiles (rows past the chunk read whatever the buffer
            // holds; their rows are computed but never stored).
            mbar_expect_tx(smem_u32(&q_full), 2 * kTpQBytes);
#pragma unroll
            for (int g = 0; g < 2; ++g)
                tma_load_2d(smem_u32(q_s + g * kTpQBytes), &q_map, head * HD, t0 + g * kTcRows, smem_u32(&q_full));
            for (int j = 0; j < n_tiles; ++j) {
                const int s = j % kTpStages;
                if (!mbar_wait(smem_u32(&kv_empty[s]), ((j / kTpStages) & 1) ^ 1)) {
                    abort_s = 1;
                    break;
                }
                const int tile = tile_lo + j;
                int rows[2];
                kv_tile_rows(p, tile, kvh, pos_last, rows);
                uint8_t *ks = ring + s * 2 * kTpKvBytes;
                uint8_t *vs = ks + kTpKvBytes;
                const uint32_t bar = smem_u32(&kv_full[s]);
                mbar_expect_tx(bar, 2 * kTpKvBytes);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    tma_load_2d(smem_u32(ks + b * 64 * 128), &k_map, 0, rows[b], bar);
                    tma_load_2d(smem_u32(vs + b * 64 * 128), &v_map, 0, rows[b], bar);
                }
                issued = j + 1;
                ATTN_TRACE(trace, j, 14);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && n_tiles > 0) {
            const uint32_t q_addr = smem_u32(q_s);
            const uint32_t p_addr = smem_u32(p_s);
            bool ok = mbar_wait(smem_u32(&q_full), 0);
            // S_g(j) = Q_g K_j^T into S buffer (2j + g) % 3.
            auto issue_s = [&](int g, int j) -> bool {
                const int n = 2 * j + g, sb = n % kTpSBufs;
                const int s = j % kTpStages;
                if (!mbar_wait(smem_u32(&kv_full[s]), (j / kTpStages) & 1)) return false;
                if (!mbar_wait(smem_u32(&s_empty[sb]), ((n / kTpSBufs) & 1) ^ 1)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(ring + s * 2 * kTpKvBytes);
                const uint32_t qg = q_addr + (uint32_t)(g * kTpQBytes);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    umma_bf16(tmem + (uint32_t)(sb * kTcKeys), umma_smem_desc(qg + k * 32),
                              umma_smem_desc(k_addr + k * 32), kIdescS, k > 0 ? 1u : 0u);
                }
                umma_commit(smem_u32(&s_full[sb]));
                return true;
            };
            // O_g += P_g(j) V_j.
            auto issue_pv = [&](int g, int j) -> bool {
                if (!mbar_wait(smem_u32(&p_full[g]), j & 1)) return false;
                ATTN_TRACE(trace, j, 8 + 3 * g);
                tc_fence_after();
                const int s = j % kTpStages;
                const uint32_t v_addr = smem_u32(ring + s * 2 * kTpKvBytes + kTpKvBytes);
                const uint32_t pg = p_addr + (uint32_t)(g * kTcPBytes);
#pragma unroll
                for (int k = 0; k < kTcKeys / 16; ++k) {
                    umma_bf16(tmem + kTpOCol + (uint32_t)(g * HD),
                              umma_smem_desc(pg + (k >> 2) * (kTcRows * 128) + (k & 3) * 32),
                              umma_smem_desc_mn(v_addr + k * 2048), kIdescPV, (j > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(smem_u32(&o_full[g]));
                ATTN_TRACE(trace, j, 9 + 3 * g);
                return true;
            };
            // S_B(j+1) reuses S_A(j)'s buffer and S_A(j+2) S_B(j)'s: both are
            // released (s_empty) before the P they follow (p_full).
            if (ok) ok = issue_s(0, 0) && issue_s(1, 0) && (n_tiles < 2 || issue_s(0, 1));
            for (int j = 0; ok && j < n_tiles; ++j) {
                ok = issue_pv(0, j);
                if (ok && j + 1 < n_tiles) ok = issue_s(1, j + 1);
                ATTN_TRACE(trace, j, 10);
                if (ok) ok = issue_pv(1, j);
                if (ok) umma_commit(smem_u32(&kv_empty[j % kTpStages]));
                if (ok && j + 2 < n_tiles) ok = issue_s(0, j + 2);
                ATTN_TRACE(trace, j, 13);
            }
            if (!ok) abort_s = 1;
        }
    } else {
        // Softmax group g (warps 2-5: tile A, 6-9: tile B); TMEM lane quadrant
        // = warp % 4; thread = query row of its tile.
        const int g = (warp - 2) / 4;
        const int quad = warp % 4;
        const int r = quad * 32 + lane;
        const int t = t0 + g * kTcRows + r;
        const int qpos = p.offset + t;
        const int gpos_first = pos_first + g * kTcRows;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t o_addr = tmem + lane_off + kTpOCol + (uint32_t)(g * HD);
        const float scale_log2 = p.scale * 1.4426950408889634f;
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        uint8_t *p_row0 = p_s + g * kTcPBytes + r * 128;
        for (int j = 0; j < n_tiles; ++j) {
            const int n = 2 * j + g, sb = n % kTpSBufs;
            const uint32_t s_addr = tmem + lane_off + (uint32_t)(sb * kTcKeys);
            // Waits decide warp-uniformly (the TMEM accesses below are warp-wide).
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&s_full[sb]), (n / kTpSBufs) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            ATTN_TRACE(trace && lane == 0 && quad == 2, j, 4 * g);
            const int kp0 = (tile_lo + j) * kTcKeys;
            // Tiles wholly at or below the group's first position need no mask
            // (no window); otherwise key i is visible iff wlo < i <= lim.
            const bool masked = p.window > 0 || kp0 + kTcKeys - 1 > gpos_first;
            const int lim = qpos - kp0;
            const int wlo = p.window > 0 ? lim - p.window : -1;
            // Pass 1: the row max of the raw scores (scale > 0), eight chains.
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float sc[64];
                tmem_ld32_nowait(s_addr + h * 64, sc);
                tmem_ld32_nowait(s_addr + h * 64 + 32, sc + 32);
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) sc[i] = (h * 64 + i <= lim && h * 64 + i > wlo) ? sc[i] : -INFINITY;
                }
#pragma unroll
                for (int i = 0; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], sc[i]);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) mx[k] = fmaxf(mx[k], mx[k + 4]);
            const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            // The running max moves only when it grows by more than 2^8 (from
            // -inf it always moves; -inf + 8 stays -inf).
            const float m_cand = fmaxf(m_run, tmax * scale_log2);
            const float m_new = m_cand > m_run + kTpRescaleLog2 ? m_cand : m_run;
            const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
            const float neg_m = m_new == -INFINITY ? 0.0f : -m_new;
            ATTN_TRACE(trace && lane == 0 && quad == 2, j, 4 * g + 1);
            if (j > 0) {
                // PV_g(j-1) done: P_g's buffer is free and O_g holds tiles < j.
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&o_full[g]), (j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xFFFFFFFFu, alpha < 1.0f)) {
#pragma unroll 1
                    for (int c = 0; c < HD / 32; ++c) {
                        float ov[32];
                        tmem_ld32_nowait(o_addr + c * 32, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                        tmem_st32(o_addr + c * 32, ov);
                    }
                }
            }
            ATTN_TRACE(trace && lane == 0 && quad == 2, j, 4 * g + 2);
            // Pass 2: p = 2^(s * scale_log2 - m_new) (a masked key gives 0)
            // into P_g row r, K-major with 128-byte swizzle: keys 64h..64h+63
            // in block h, 16-byte chunk c of the row at (c ^ (r & 7)).
            float sums[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) sums[k] = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float sc[64];
                tmem_ld32_nowait(s_addr + h * 64, sc);
                tmem_ld32_nowait(s_addr + h * 64 + 32, sc + 32);
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) sc[i] = (h * 64 + i <= lim && h * 64 + i > wlo) ? sc[i] : -INFINITY;
                }
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float e0 = fast_exp2(fmaf(sc[8 * c + 2 * q], scale_log2, neg_m));
                        const float e1 = fast_exp2(fmaf(sc[8 * c + 2 * q + 1], scale_log2, neg_m));
                        sums[(4 * c + q) & 7] += e0 + e1;
                        w[q] = pack_bf16(e0, e1);
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(p_row0 + h * (kTcRows * 128) + ((c ^ (r & 7)) << 4));
                    *dst = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&s_empty[sb]));
#pragma unroll
            for (int k = 0; k < 4; ++k) sums[k] += sums[k + 4];
            const float rsum = (sums[0] + sums[1]) + (sums[2] + sums[3]);
            l_run = l_run * alpha + rsum;
            m_run = m_new;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(smem_u32(&p_full[g]));
            ATTN_TRACE(trace && lane == 0 && quad == 2, j, 4 * g + 3);
        }
        if (ok && n_tiles > 0) {
            if (__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&o_full[g]), (n_tiles - 1) & 1))) {
                tc_fence_after();
            } else {
                ok = false;
            }
        }
        const bool live = t <= t_last;
        const long long rh = ((long long)split * p.T + t) * p.q_heads + head;
        if (!ok) {
            abort_s = 1;
        } else if (n_tiles > 0) {
            const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float ov[32];
                tmem_ld32_nowait(o_addr + c * 32, ov);
                tmem_wait_ld();
                if (!live) continue;
                if (p.splits > 1) {
                    float4 *dst = reinterpret_cast<float4 *>(p.part_o + rh * HD + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i) dst[i] = make_float4(ov[4 * i], ov[4 * i + 1], ov[4 * i + 2], ov[4 * i + 3]);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + (long long)t * p.q_heads * HD + head * HD + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        dst[i] = make_uint4(pack_bf16(ov[8 * i] * inv, ov[8 * i + 1] * inv),
                                            pack_bf16(ov[8 * i + 2] * inv, ov[8 * i + 3] * inv),
                                            pack_bf16(ov[8 * i + 4] * inv, ov[8 * i + 5] * inv),
                                            pack_bf16(ov[8 * i + 6] * inv, ov[8 * i + 7] * inv));
                    }
                }
            }
            if (live && p.splits > 1) *reinterpret_cast<float2 *>(p.part_ml + rh * 2) = make_float2(m_run, l_run);
        } else if (live) {
            // A key split with no tiles: an empty partial (O = 0, m = -inf,
            // l = 0) that the merge weighs by zero.
            if (p.splits > 1) {
                float4 *dst = reinterpret_cast<float4 *>(p.part_o + rh * HD);
#pragma unroll
                for (int i = 0; i < HD / 4; ++i) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float2 *>(p.part_ml + rh * 2) = make_float2(-INFINITY, 0.0f);
            } else {
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + (long long)t * p.q_heads * HD + head * HD);
#pragma unroll
                for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (abort_s) {
        // A wait gave up: let this CTA's copies and MMAs still in flight land
        // before its shared memory and TMEM are released (bounded waits).
        if (warp == 0 && lane == 0 && n_tiles > 0) {
            mbar_wait(smem_u32(&q_full), 0);
            for (int j = max(0, issued - kTpStages); j < issued; ++j) {
                mbar_wait(smem_u32(&kv_full[j % kTpStages]), (j / kTpStages) & 1);
            }
        } else if (warp == 1 && lane == 0) {
            umma_commit(smem_u32(&drain_bar));
            mbar_wait(smem_u32(&drain_bar), 0);
        }
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && p.error) *p.error = 8;
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcTmemCols));
    }
}

}  // namespace cheetah
