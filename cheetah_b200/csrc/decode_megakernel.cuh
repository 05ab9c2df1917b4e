// Persistent single-sequence decode kernel: B = 1, bf16 weights, bf16 KV.
//
// One CTA per SM runs a whole decode step, or a whole run of greedy steps.
// Every CTA owns a fixed slice of every weight matrix. A producer warp
// streams those slices, in exactly the order the CTA consumes them, through
// a ring of 32 KB shared-memory slots with 1D bulk copies (cp.async.bulk,
// L2 evict-first). The weight stream does not depend on activations, so it
// runs ahead across phase boundaries, layers and steps: HBM stays busy while
// the CTAs order themselves along the activation chain. Eight consumer warps
// compute from the slots.
//
// Phases of one layer (`Qwen2Native::forward_layer`, qwen2.rs:430-465):
//   QKV   RMSNorm(ln1) (`ops.rs:646-652`); q/k/v rows (a copy with the first
//         rows of all rotate-half pairs, then the partners, so a warp computes
//         one pair); bias (`ops.rs:1156`), RoPE (`ops.rs:693-740`); K/V
//         appended to the paged cache (`ops.rs:1329`), q to global. [all CTAs]
//   ATT   unit (q head h, key chunk j), S chunks per head. Keys written by
//         earlier steps are staged into shared memory with bulk copies while
//         the CTA waits for QKV; online-softmax partial over the chunk
//         (`ops.rs:1357-1467`); the S CTAs of a head wait for each other, each
//         merges the S partials in the same order, then multiplies its row
//         block of W_o[:, head h] (head-major copy) by the head output:
//         per-head o_proj partials.
//   RES   each CTA sums the heads' partials of the residual rows it owns
//         (+ o bias, + residual, qwen2.rs:442-449) and publishes them.
//   GU    RMSNorm(ln2) of the new residual; gate/up rows; SiLU(gate)*up
//         (`ops.rs:743-747`).                                      [all CTAs]
//   DOWN  down rows; residual add (qwen2.rs:459-463).               [all CTAs]
// After the last layer, LM: final RMSNorm and lm_head rows (`ops.rs:1513`),
// greedy argmax as a packed (total-order key, index) atomicMax, which keeps
// the larger index on ties like `Iterator::max_by` (engine.rs:2247-2253).
// The next step embeds that argmax.
//
// Ordering: monotonic arrival counters in global memory. Release = consumer
// barrier, then one thread's red.release.gpu add; acquire = one thread spins
// with ld.acquire.gpu, then the consumer barrier. All reductions run in a
// fixed order, so results are reproducible run to run. The last CTA to finish
// the run resets the counters. Every wait is bounded by %globaltimer: on a
// timeout the CTA records the error word and switches to abort mode (waits
// return at once, work continues over in-bounds addresses only, no new copies
// are issued), the producer drains the copies already in flight, and the CTA
// returns. Other CTAs see the error word and abort too.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "gemv.cuh"
#include "kernels_misc.cuh"
#include "tma.cuh"

namespace cheetah {

constexpr int kMkConsumerWarps = 8;
constexpr int kMkConsumers = kMkConsumerWarps * kWarp;
constexpr int kMkThreads = kMkConsumers + kWarp;  // + one producer warp
constexpr int kMkSlotBytes = 32768;
constexpr int kMkMaxSlots = 8;
constexpr int kMkMaxHeads = 64;
constexpr int kMkCtrlWords = 8 + kMkMaxHeads;
constexpr unsigned long long kMkTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr int kMkErrWait = 0x4D4B01;   // a counter or slot wait timed out
constexpr int kMkErrToken = 0x4D4B02;  // argmax outside the vocabulary

// Optional phase timestamps (first step, first layers) for profiling builds.
#ifdef CHEETAH_MK_TRACE
__device__ unsigned long long g_mk_trace[256][128];
#define MK_TRACE(step, ev)                                                                     \
    do {                                                                                        \
        if ((step) == 0 && threadIdx.x == 0 && (ev) < 128) {                                     \
            unsigned long long t__;                                                             \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t__));                            \
            g_mk_trace[blockIdx.x][(ev)] = t__;                                                 \
        }                                                                                       \
    } while (0)
// Cycle stamps of consumer thread 0 (SM clock) in layer 1 of the first step.
__device__ long long g_mk_cycles[256][32];
#define MK_CYC(step, layer, ev)                                                              \
    do {                                                                                      \
        if ((step) == 0 && (layer) == 1 && threadIdx.x == 0 && (ev) < 32)                      \
            g_mk_cycles[blockIdx.x][(ev)] = clock64();                                       \
    } while (0)
#else
#define MK_CYC(step, layer, ev) \
    do {                        \
    } while (0)
#define MK_TRACE(step, ev) \
    do {                   \
    } while (0)
#endif

enum MkCounter : int {
    kMkCntQkv = 0,
    kMkCntO = 1,
    kMkCntGu = 2,
    kMkCntDown = 3,
    kMkCntLm = 4,
    kMkCntRes = 5,  // residual rows after o_proj published
    kMkCntHead = 8
};

struct MkLayer {
    const uint16_t *wqkv;   // [q+2kv dims][H]: first rows of all rotate-half pairs, then the partners
    const float *bqkv;      // [q+2kv dims] in [q; k; v] order, or nullptr
    const uint16_t *wo;     // [q_heads][H][head_dim]: W_o[:, head] row blocks
    const float *bo;        // nullptr when absent
    const uint16_t *wgate;  // [I][H]
    const uint16_t *wup;    // [I][H]
    const uint16_t *wdown;  // [H][I]
    const float *ln1;
    const float *ln2;
};

struct MkParams {
    const MkLayer *layers;
    int num_layers, H, I, q_heads, kv_heads, hd, vocab;
    int window, att_splits, slots, xcap;
    // Bulk copies in flight per CTA (issued, not landed): during the layers,
    // and during the lm_head stream. Deeper queues raise the latency of every
    // other load on the chain (Little's law), the layers' weights only need a
    // fraction of HBM bandwidth, and lm_head needs all of it.
    int inflight_layers, inflight_lm;
    float eps, scale_log2;  // 1/sqrt(d) * log2(e)
    const uint16_t *embed;
    const uint16_t *lm_head;  // [vocab][H]
    const float *final_norm;
    const float *rope_cos, *rope_sin;  // [max_positions][d/2]
    uint8_t *k_pool, *v_pool;          // [layer][page][kv_head][page_tokens][d] bf16
    long long layer_stride_bytes;
    int num_pages, page_tokens, max_pages;
    int32_t *page_table;
    const StepState *step;  // token and position of the first step, optional page install
    int steps;
    float *hidden;    // [H] residual
    float *q;         // [q_heads * d]
    float *opart;     // [q_heads][H] per-head o_proj partials
    float *hnew;      // [H] residual after o_proj (+ bias), reduced by the rows' owners
    float *act;       // [I]
    float *att_part;  // [q_heads][S][2 + d]: m (log2 domain), l, o[d]
    unsigned *ctrl;   // kMkCtrlWords arrival counters, zero between runs
    unsigned long long *argmax_slots;  // [2], alternating per step
    unsigned long long *argmax_out;    // packed key of the last step
    int32_t *token_log;                // [steps] greedy token of each step, nullable
    float *logits;                     // [vocab] logits of the last step, nullable
    int *error;
};

struct MkShared {
    unsigned long long full[kMkMaxSlots];
    unsigned long long empty[kMkMaxSlots];
    unsigned long long kv_bar;  // staged K/V rows of the attention chunk
    volatile int abort;
    int token;
    int staged;    // positions [a, staged) of the chunk are in shared memory
    int kv_uses;   // completed kv_bar phases + the one in flight
    float norm_red[kMkConsumerWarps];
    unsigned long long best8[kMkConsumerWarps];
};

__device__ __forceinline__ unsigned long long mk_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned mk_ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long mk_ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mk_consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kMkConsumers) : "memory");
}

__device__ __forceinline__ uint64_t mk_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void mk_bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                             uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}

__device__ __forceinline__ bool mk_bar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded mbarrier wait; gives up on abort or after the timeout.
__device__ __forceinline__ bool mk_bar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                            bool honour_abort) {
    if (mk_bar_test(bar, parity)) return true;
    const unsigned long long t0 = mk_now();
    while (true) {
        if (mk_bar_test(bar, parity)) return true;
        if (honour_abort && *abort_flag) return false;
        if (mk_now() - t0 > kMkTimeoutNs) return false;
    }
}

__device__ __forceinline__ void mk_flag_error(MkShared &sh, int *error, int code) {
    sh.abort = 1;
    atomicCAS(error, 0, code);
}

// Counter wait by consumer thread 0, broadcast through the consumer barrier.
// Returns false in abort mode.
__device__ __forceinline__ bool mk_wait_count(const unsigned *cnt, unsigned target, MkShared &sh, int *error,
                                              int trace_step = 1, int trace_ev = 64) {
    if (threadIdx.x == 0 && !sh.abort) {
        if ((int)(mk_ld_acquire(cnt) - target) < 0) {
            const unsigned long long t0 = mk_now();
            unsigned polls = 0;
            while ((int)(mk_ld_acquire(cnt) - target) < 0) {
                ++polls;
                if (polls > 256) __nanosleep(40);
                if ((polls & 31u) == 0) {
                    if (*(volatile int *)error != 0) {
                        sh.abort = 1;
                        break;
                    }
                    if (mk_now() - t0 > kMkTimeoutNs) {
                        mk_flag_error(sh, error, kMkErrWait);
                        break;
                    }
                }
            }
        }
        MK_TRACE(trace_step, trace_ev);
    }
    // ld.acquire.gpu by thread 0, then the CTA barrier: every consumer
    // thread's later loads are ordered after the producers' writes.
    mk_consumer_sync();
    return !sh.abort;
}

// Arrival after this CTA's writes of the phase: the CTA barrier orders
// every consumer thread's writes before thread 0's release-add at gpu scope
// (cumulative), which the thread issues without waiting for it.
__device__ __forceinline__ void mk_arrive(unsigned *cnt) {
    mk_consumer_sync();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
}

// Arrival that returns the previous count (acq_rel) on consumer thread 0.
__device__ __forceinline__ unsigned mk_arrive_fetch(unsigned *cnt) {
    mk_consumer_sync();
    unsigned old = 0;
    if (threadIdx.x == 0)
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
    return old;
}

__device__ __forceinline__ int mk_split(int n, int parts, int i) {
    return (int)(((long long)n * i) / parts);
}

// ---- the static weight schedule (producer and consumers walk it alike) ----
// Weight rows are contiguous bf16 rows in HBM and in the tiles.
__device__ __forceinline__ int mk_row_stride(int K) { return 2 * K; }

struct MkTiles {
    int begin, end, per_tile;  // unit range of this CTA and units per tile
    __device__ int count() const { return end > begin ? (end - begin + per_tile - 1) / per_tile : 0; }
    __device__ int lo(int k) const { return begin + k * per_tile; }
    __device__ int hi(int k) const { return min(end, begin + (k + 1) * per_tile); }
};

// QKV: units are rotate-half pairs; a tile holds up to 8 pairs (one per
// consumer warp), the first rows of its n pairs at tile rows 0..n-1 and their
// partners from row per_tile on.
__device__ __forceinline__ MkTiles mk_qkv_tiles(const MkParams &p, int cta, int grid) {
    const int pairs = (p.q_heads + 2 * p.kv_heads) * p.hd / 2;
    return {mk_split(pairs, grid, cta), mk_split(pairs, grid, cta + 1),
            min(8, kMkSlotBytes / (2 * mk_row_stride(p.H)))};
}
__device__ __forceinline__ bool mk_att_unit(const MkParams &p, int cta) {
    return cta < p.q_heads * p.att_splits;
}
// ATT: rows of W_o[:, head] (head-major copy, head_dim elements each), contiguous.
__device__ __forceinline__ MkTiles mk_att_tiles(const MkParams &p, int cta) {
    if (!mk_att_unit(p, cta)) return {0, 0, 1};
    const int j = cta % p.att_splits;
    return {mk_split(p.H, p.att_splits, j), mk_split(p.H, p.att_splits, j + 1), kMkSlotBytes / (2 * p.hd)};
}
// GU: units are intermediate rows; gate rows first, up rows from per_tile on.
__device__ __forceinline__ MkTiles mk_gu_tiles(const MkParams &p, int cta, int grid) {
    return {mk_split(p.I, grid, cta), mk_split(p.I, grid, cta + 1), min(8, kMkSlotBytes / (2 * mk_row_stride(p.H)))};
}
__device__ __forceinline__ MkTiles mk_down_tiles(const MkParams &p, int cta, int grid) {
    return {mk_split(p.H, grid, cta), mk_split(p.H, grid, cta + 1), min(16, kMkSlotBytes / mk_row_stride(p.I))};
}
__device__ __forceinline__ MkTiles mk_lm_tiles(const MkParams &p, int cta, int grid) {
    return {mk_split(p.vocab, grid, cta), mk_split(p.vocab, grid, cta + 1), min(16, kMkSlotBytes / mk_row_stride(p.H))};
}
// QKV pair i -> its two rows of the [q; k; v] matrix (rotate-half partners).
__device__ __forceinline__ int mk_pair_row(const MkParams &p, int pair, int which) {
    const int half = p.hd / 2;
    const int head = pair / half;
    return head * p.hd + (pair - head * half) + which * half;
}

// ---- producer ----
__device__ void mk_producer(const MkParams &p, uint8_t *ring, MkShared &sh) {
    if ((threadIdx.x % kWarp) != 0) return;
    const int cta = blockIdx.x, grid = gridDim.x;
    const uint64_t pol = mk_evict_first_policy();
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t rs_h = (uint32_t)mk_row_stride(p.H), rs_i = (uint32_t)mk_row_stride(p.I);
    uint32_t seq = 0;
    bool ok = true;
    // Claim the next slot (free, and the copy `inflight` tiles back landed)
    // and arm its barrier with the tile's byte count.
    auto begin_tile = [&](uint32_t bytes, int inflight) -> uint32_t {
        if (!ok) return 0;
        const int s = (int)(seq % (uint32_t)p.slots);
        const uint32_t n = seq / (uint32_t)p.slots;
        if (sh.abort || (n > 0 && !mk_bar_wait(smem_u32(&sh.empty[s]), (n - 1) & 1u, &sh.abort, true))) {
            ok = false;
            return 0;
        }
        if (seq >= (uint32_t)inflight) {
            const uint32_t old = seq - (uint32_t)inflight;
            if (!mk_bar_wait(smem_u32(&sh.full[old % (uint32_t)p.slots]), (old / (uint32_t)p.slots) & 1u, &sh.abort,
                             true)) {
                ok = false;
                return 0;
            }
        }
        mbar_expect_tx(smem_u32(&sh.full[s]), bytes);
        return ring_s + (uint32_t)s * kMkSlotBytes;
    };
    auto copy = [&](uint32_t dst, const void *src, uint32_t bytes) {
        mk_bulk_load(dst, src, bytes, smem_u32(&sh.full[seq % (uint32_t)p.slots]), pol);
    };
    const MkTiles tq = mk_qkv_tiles(p, cta, grid), ta = mk_att_tiles(p, cta), tg = mk_gu_tiles(p, cta, grid),
                  td = mk_down_tiles(p, cta, grid), tl = mk_lm_tiles(p, cta, grid);
    const int head = mk_att_unit(p, cta) ? cta / p.att_splits : 0;
    for (int t = 0; t < p.steps && ok; ++t) {
        for (int l = 0; l < p.num_layers && ok; ++l) {
            const MkLayer &w = p.layers[l];
            const int q = p.inflight_layers;
            const int pairs = (p.q_heads + 2 * p.kv_heads) * p.hd / 2;
            const uint8_t *wqkv = reinterpret_cast<const uint8_t *>(w.wqkv);
            for (int k = 0; k < tq.count() && ok; ++k) {
                const uint32_t n = (uint32_t)(tq.hi(k) - tq.lo(k));
                const uint32_t base = begin_tile(2u * n * rs_h, q);
                if (!ok) break;
                copy(base, wqkv + (size_t)tq.lo(k) * rs_h, n * rs_h);
                copy(base + (uint32_t)tq.per_tile * rs_h, wqkv + (size_t)(pairs + tq.lo(k)) * rs_h, n * rs_h);
                ++seq;
            }
            for (int k = 0; k < ta.count() && ok; ++k) {
                const uint32_t bytes = (uint32_t)(ta.hi(k) - ta.lo(k)) * 2u * p.hd;
                const uint32_t base = begin_tile(bytes, q);
                if (!ok) break;
                copy(base, w.wo + ((size_t)head * p.H + ta.lo(k)) * p.hd, bytes);
                ++seq;
            }
            for (int k = 0; k < tg.count() && ok; ++k) {
                const uint32_t n = (uint32_t)(tg.hi(k) - tg.lo(k));
                const uint32_t base = begin_tile(2u * n * rs_h, q);
                if (!ok) break;
                copy(base, reinterpret_cast<const uint8_t *>(w.wgate) + (size_t)tg.lo(k) * rs_h, n * rs_h);
                copy(base + (uint32_t)tg.per_tile * rs_h, reinterpret_cast<const uint8_t *>(w.wup) + (size_t)tg.lo(k) * rs_h,
                     n * rs_h);
                ++seq;
            }
            for (int k = 0; k < td.count() && ok; ++k) {
                const uint32_t n = (uint32_t)(td.hi(k) - td.lo(k));
                const uint32_t base = begin_tile(n * rs_i, q);
                if (!ok) break;
                copy(base, reinterpret_cast<const uint8_t *>(w.wdown) + (size_t)td.lo(k) * rs_i, n * rs_i);
                ++seq;
            }
        }
        for (int k = 0; k < tl.count() && ok; ++k) {
            const uint32_t n = (uint32_t)(tl.hi(k) - tl.lo(k));
            const uint32_t base = begin_tile(n * rs_h, p.inflight_lm);
            if (!ok) break;
            copy(base, reinterpret_cast<const uint8_t *>(p.lm_head) + (size_t)tl.lo(k) * rs_h, n * rs_h);
            ++seq;
        }
    }
    // Drain: the newest copy of every slot must have landed before the CTA exits.
    for (int s = 0; s < p.slots; ++s) {
        if (seq <= (uint32_t)s) break;
        const uint32_t n_last = (seq - 1 - (uint32_t)s) / (uint32_t)p.slots;
        mk_bar_wait(smem_u32(&sh.full[s]), n_last & 1u, &sh.abort, false);
    }
}

// ---- consumer building blocks ----
struct MkRing {
    uint8_t *base;
    MkShared *sh;
    int slots;
    uint32_t seq;
    int *error;

    // Wait for the tile `ahead` tiles past the next one; returns its slot.
    __device__ uint8_t *acquire(int ahead = 0) {
        const uint32_t q = seq + (uint32_t)ahead;
        const int s = (int)(q % (uint32_t)slots);
        if (!sh->abort) {
            const uint32_t parity = (q / (uint32_t)slots) & 1u;
            if (!mk_bar_wait(smem_u32(&sh->full[s]), parity, &sh->abort, true) && !sh->abort)
                mk_flag_error(*sh, error, kMkErrWait);
        }
        return base + (size_t)s * kMkSlotBytes;
    }
    // This warp is done reading the next `count` tiles.
    __device__ void release(int count = 1) {
        __syncwarp();
        for (int k = 0; k < count; ++k) {
            const int s = (int)((seq + (uint32_t)k) % (uint32_t)slots);
            if ((threadIdx.x % kWarp) == 0 && !sh->abort) mbar_arrive(smem_u32(&sh->empty[s]));
        }
        seq += (uint32_t)count;
    }
};

// Pool row of (position, KV head) through the sequence's page table, or -1
// when the page is not installed or out of range (the access is skipped).
__device__ __forceinline__ long long mk_kv_row(const MkParams &p, int pos, int kv_head) {
    const int page_slot = pos / p.page_tokens;
    if (page_slot >= p.max_pages) return -1;
    const int page = __ldcg(p.page_table + page_slot);
    if (page < 0 || page >= p.num_pages) return -1;
    return ((long long)page * p.kv_heads + kv_head) * p.page_tokens + (pos - page_slot * p.page_tokens);
}

// Elements i = tid + u * kMkConsumers (u < kMkV) of a vector of width <= 1024,
// held in registers so that all of a thread's loads are in flight together.
constexpr int kMkV = (1024 + kMkConsumers - 1) / kMkConsumers;
struct MkV4 {
    float v[kMkV];
};

template <bool CG>
__device__ __forceinline__ MkV4 mk_ld4(const float *src, int n) {
    MkV4 r;
#pragma unroll
    for (int u = 0; u < kMkV; ++u) {
        const int i = (int)threadIdx.x + u * kMkConsumers;
        r.v[u] = i < n ? (CG ? __ldcg(src + i) : src[i]) : 0.0f;
    }
    return r;
}

__device__ __forceinline__ float mk_block_sum(float v, MkShared &sh) {
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    v = warp_sum(v);
    if (lane == 0) sh.norm_red[warp] = v;
    mk_consumer_sync();
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < kMkConsumerWarps; ++k) total += sh.norm_red[k];
    return total;
}

// RMSNorm (`ops.rs:646-652`) of register-held x (width <= 1024) with
// register-held weights into xs.
__device__ __forceinline__ void mk_rmsnorm4(const MkV4 &x, const MkV4 &w, int n, float eps, float *xs,
                                            MkShared &sh) {
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < kMkV; ++u) {
        if ((int)threadIdx.x + u * kMkConsumers < n) ss = fmaf(x.v[u], x.v[u], ss);
    }
    const float total = mk_block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(total / (float)n + eps);
#pragma unroll
    for (int u = 0; u < kMkV; ++u) {
        const int i = (int)threadIdx.x + u * kMkConsumers;
        if (i < n) xs[i] = __fmul_rn(x.v[u], __fmul_rn(inv, w.v[u]));
    }
    mk_consumer_sync();
}

// The same for any width: x is global memory another CTA wrote during this
// kernel (GLOBAL, read through L2), a bf16 row (BF16), or shared memory.
template <int SRC>  // 0 shared f32, 1 global f32, 2 global bf16
__device__ __forceinline__ void mk_rmsnorm_any(const void *x, const float *w, int n, float eps, float *xs,
                                               MkShared &sh) {
    auto load = [&](int i) -> float {
        if (SRC == 0) return static_cast<const float *>(x)[i];
        if (SRC == 1) return __ldcg(static_cast<const float *>(x) + i);
        return bf16_to_f32(static_cast<const uint16_t *>(x)[i]);
    };
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += kMkConsumers) {
        const float v = load(i);
        ss = fmaf(v, v, ss);
    }
    const float total = mk_block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(total / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += kMkConsumers) xs[i] = __fmul_rn(load(i), __fmul_rn(inv, w[i]));
    mk_consumer_sync();
}

// Global f32 vector (written by other CTAs) into shared memory, kU loads in
// flight per thread.
__device__ __forceinline__ void mk_gather(float *dst, const float *src, int n) {
    constexpr int kU = 22;
    for (int base = threadIdx.x; base < n; base += kU * kMkConsumers) {
        float v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int i = base + u * kMkConsumers;
            v[u] = i < n ? __ldcg(src + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int i = base + u * kMkConsumers;
            if (i < n) dst[i] = v[u];
        }
    }
    mk_consumer_sync();
}

// A lane's share of an f32 vector of width K (8-element chunks lane,
// lane + 32, ...), held in registers across all rows of a phase. XC chunks
// cover K <= XC * 256.
template <int XC>
struct MkXReg {
    float v[XC][8];
    __device__ __forceinline__ void load(const float *xs, int K) {
        const int lane = threadIdx.x % kWarp;
#pragma unroll
        for (int c = 0; c < XC; ++c) {
            const int idx = lane + c * kWarp;
            if (idx < K / 8) {
                const float4 a = *reinterpret_cast<const float4 *>(xs + idx * 8);
                const float4 b = *reinterpret_cast<const float4 *>(xs + idx * 8 + 4);
                v[c][0] = a.x; v[c][1] = a.y; v[c][2] = a.z; v[c][3] = a.w;
                v[c][4] = b.x; v[c][5] = b.y; v[c][6] = b.z; v[c][7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[c][e] = 0.0f;
            }
        }
    }
};

__device__ __forceinline__ void mk_fma8r(float &acc, uint4 w, const float *x) {
    acc = fmaf(bf16_lo(w.x), x[0], acc);
    acc = fmaf(bf16_hi(w.x), x[1], acc);
    acc = fmaf(bf16_lo(w.y), x[2], acc);
    acc = fmaf(bf16_hi(w.y), x[3], acc);
    acc = fmaf(bf16_lo(w.z), x[4], acc);
    acc = fmaf(bf16_hi(w.z), x[5], acc);
    acc = fmaf(bf16_lo(w.w), x[6], acc);
    acc = fmaf(bf16_hi(w.w), x[7], acc);
}

// Two dot products of bf16 rows (shared memory) with the register vector.
template <int XC>
__device__ __forceinline__ void mk_dot2r(const uint8_t *wa, const uint8_t *wb, const MkXReg<XC> &x, int K,
                                         float &ra, float &rb) {
    const int lane = threadIdx.x % kWarp;
    const uint4 *pa = reinterpret_cast<const uint4 *>(wa);
    const uint4 *pb = reinterpret_cast<const uint4 *>(wb);
    uint4 ua[XC], ub[XC];
#pragma unroll
    for (int c = 0; c < XC; ++c) {
        const int idx = lane + c * kWarp;
        const bool in = idx < K / 8;
        ua[c] = in ? pa[idx] : make_uint4(0, 0, 0, 0);
        ub[c] = in ? pb[idx] : make_uint4(0, 0, 0, 0);
    }
    float a = 0.0f, b = 0.0f;
#pragma unroll
    for (int c = 0; c < XC; ++c) {
        mk_fma8r(a, ua[c], x.v[c]);
        mk_fma8r(b, ub[c], x.v[c]);
    }
    ra = warp_sum(a);
    rb = warp_sum(b);
}

// Two dot products of bf16 rows (shared memory) with an f32 vector in shared memory.
__device__ __forceinline__ void mk_dot2(const uint8_t *wa, const uint8_t *wb, const float *x, int K, float &ra,
                                        float &rb) {
    const int lane = threadIdx.x % kWarp;
    const uint4 *pa = reinterpret_cast<const uint4 *>(wa);
    const uint4 *pb = reinterpret_cast<const uint4 *>(wb);
    float a = 0.0f, b = 0.0f;
#pragma unroll 2
    for (int v = lane; v < K / 8; v += kWarp) {
        const uint4 ua = pa[v], ub = pb[v];
        fma8(a, ua, x + v * 8);
        fma8(b, ub, x + v * 8);
    }
    ra = warp_sum(a);
    rb = warp_sum(b);
}

// One long dot product (four accumulators) of a bf16 row with an f32 vector, both in shared memory.
__device__ __forceinline__ float mk_dot(const uint8_t *wa, const float *x, int K) {
    const int lane = threadIdx.x % kWarp;
    const uint4 *pa = reinterpret_cast<const uint4 *>(wa);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int v = lane;
    for (; v + 3 * kWarp < K / 8; v += 4 * kWarp) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = pa[v + u * kWarp];
#pragma unroll
        for (int u = 0; u < 4; ++u) fma8(acc[u], w[u], x + (v + u * kWarp) * 8);
    }
    for (; v < K / 8; v += kWarp) fma8(acc[0], pa[v], x + v * 8);
    return warp_sum(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])));
}

__device__ __forceinline__ uint32_t mk_lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 mk_lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// Online-softmax partial of one head over key positions [a, b) (log2
// domain). Positions [a, sb) were staged in shared memory (stK / stV rows,
// row = position - a); later ones (this step's position among them) are read
// from the pool through L2. Lane = key position for the scores (each lane
// walks its K row's 16-byte chunks in a lane-rotated order, so the staged
// rows are read without bank conflicts), lane = head dims for P.V. Writes
// the CTA's (m, l, o[HD]) to `out`.
template <int HD>
__device__ void mk_attention_chunk(const MkParams &p, int layer, int head, int a, int b, int sb,
                                   const uint16_t *stK, const uint16_t *stV, const float *qh, float *attw,
                                   float *out) {
    constexpr int kDims = HD / kWarp;  // dims per lane in P.V
    constexpr int kChunks = HD / 8;    // 16-byte chunks per K row
    constexpr int kPre = HD == 64 ? 32 : 8;
    using VT = typename std::conditional<HD == 64, uint32_t, uint2>::type;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int kvh = head / (p.q_heads / p.kv_heads);
    const uint16_t *kbase = reinterpret_cast<const uint16_t *>(p.k_pool + (long long)layer * p.layer_stride_bytes);
    const uint16_t *vbase = reinterpret_cast<const uint16_t *>(p.v_pool + (long long)layer * p.layer_stride_bytes);
    const uint32_t stV_s = smem_u32(stV);
    float m = -INFINITY, l = 0.0f;
    float o[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) o[d] = 0.0f;
    for (int blk = a + warp * kWarp; blk < b; blk += kMkConsumers) {
        const int pos = blk + lane;
        const int n = min(kWarp, b - blk);
        const bool staged = pos < sb;
        long long row = -1;
        if (pos < b && !staged) row = mk_kv_row(p, pos, kvh);
        float s = -INFINITY;
        if (pos < b && (staged || row >= 0)) {
            const uint4 *ks = reinterpret_cast<const uint4 *>(stK + (size_t)(pos - a) * HD);
            const uint4 *kg = reinterpret_cast<const uint4 *>(kbase + row * HD);
            uint4 kr[kChunks];
#pragma unroll
            for (int v = 0; v < kChunks; ++v) {
                const int c = (v + lane) & (kChunks - 1);
                kr[v] = staged ? ks[c] : __ldcg(kg + c);
            }
            float acc = 0.0f;
#pragma unroll
            for (int v = 0; v < kChunks; ++v) fma8(acc, kr[v], qh + ((v + lane) & (kChunks - 1)) * 8);
            s = acc * p.scale_log2;
        }
        const float bm = warp_max(s);
        const float m_new = fmaxf(m, bm);
        if (m_new == -INFINITY) continue;  // nothing visible in this block
        const float corr = exp2f(m - m_new);
        const float pr = s == -INFINITY ? 0.0f : exp2f(s - m_new);
        l = l * corr + warp_sum(pr);
#pragma unroll
        for (int d = 0; d < kDims; ++d) o[d] *= corr;
        m = m_new;
        if (blk + n <= sb) {
            // Every position of the block is staged: V rows straight from
            // shared memory, probabilities broadcast from their lanes.
            const uint32_t vrow = stV_s + (uint32_t)(((blk - a) * HD + lane * kDims) * 2);
#pragma unroll
            for (int k = 0; k < kWarp; ++k) {
                const float pk = __shfl_sync(0xFFFFFFFFu, pr, k);
                if (k < n) {
                    const uint32_t va = vrow + (uint32_t)(k * HD * 2);
                    if constexpr (HD == 64) {
                        const uint32_t v = mk_lds32(va);
                        o[0] = fmaf(pk, bf16_lo(v), o[0]);
                        o[1] = fmaf(pk, bf16_hi(v), o[1]);
                    } else {
                        const uint2 v = mk_lds64(va);
                        o[0] = fmaf(pk, bf16_lo(v.x), o[0]);
                        o[1] = fmaf(pk, bf16_hi(v.x), o[1]);
                        o[2] = fmaf(pk, bf16_lo(v.y), o[2]);
                        o[3] = fmaf(pk, bf16_hi(v.y), o[3]);
                    }
                }
            }
            continue;
        }
        for (int k0 = 0; k0 < n; k0 += kPre) {
            VT vv[kPre];
#pragma unroll
            for (int k = 0; k < kPre; ++k) {
                const int idx = (k0 + k) & (kWarp - 1);
                const long long rk = __shfl_sync(0xFFFFFFFFu, row, idx);
                const int pk = blk + k0 + k;
                vv[k] = VT{};
                if (k0 + k < n) {
                    if (pk < sb) {
                        vv[k] = *reinterpret_cast<const VT *>(stV + (size_t)(pk - a) * HD + lane * kDims);
                    } else if (rk >= 0) {
                        vv[k] = __ldcg(reinterpret_cast<const VT *>(vbase + rk * HD + lane * kDims));
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kPre; ++k) {
                const float pk = __shfl_sync(0xFFFFFFFFu, pr, (k0 + k) & (kWarp - 1));
                if constexpr (HD == 64) {
                    o[0] = fmaf(pk, bf16_lo(vv[k]), o[0]);
                    o[1] = fmaf(pk, bf16_hi(vv[k]), o[1]);
                } else {
                    o[0] = fmaf(pk, bf16_lo(vv[k].x), o[0]);
                    o[1] = fmaf(pk, bf16_hi(vv[k].x), o[1]);
                    o[2] = fmaf(pk, bf16_lo(vv[k].y), o[2]);
                    o[3] = fmaf(pk, bf16_hi(vv[k].y), o[3]);
                }
            }
        }
    }
    float *mine = attw + warp * (2 + HD);
    if (lane == 0) {
        mine[0] = m;
        mine[1] = l;
    }
#pragma unroll
    for (int d = 0; d < kDims; ++d) mine[2 + lane * kDims + d] = o[d];
    mk_consumer_sync();
    if (warp == 0) {
        float mm = -INFINITY;
#pragma unroll
        for (int w = 0; w < kMkConsumerWarps; ++w) mm = fmaxf(mm, attw[w * (2 + HD)]);
        float ll = 0.0f;
        float oo[kDims];
#pragma unroll
        for (int d = 0; d < kDims; ++d) oo[d] = 0.0f;
        if (mm != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kMkConsumerWarps; ++w) {
                const float *ws = attw + w * (2 + HD);
                if (ws[0] == -INFINITY) continue;
                const float c = exp2f(ws[0] - mm);
                ll = fmaf(c, ws[1], ll);
#pragma unroll
                for (int d = 0; d < kDims; ++d) oo[d] = fmaf(c, ws[2 + lane * kDims + d], oo[d]);
            }
        }
        if (lane == 0) {
            out[0] = mm;
            out[1] = ll;
        }
#pragma unroll
        for (int d = 0; d < kDims; ++d) out[2 + lane * kDims + d] = oo[d];
    }
}

// Stage K and V rows of positions [a, min(b, limit, a + cap)) of one KV head
// into shared memory with bulk copies on `sh.kv_bar` (one thread). Rows of a
// page are contiguous in the pool, so each page is one copy per tensor.
// Publishes the staged end in sh.staged (a when nothing was staged).
template <int HD>
__device__ __forceinline__ void mk_stage_kv(const MkParams &p, int layer, int kvh, int a, int b, int limit, int cap,
                                            uint16_t *stK, uint16_t *stV, MkShared &sh) {
    constexpr int kMaxSegs = 4;
    int sb = min(min(b, limit), a + cap);
    long long rows[kMaxSegs];
    int segs = 0;
    for (int p0 = a; p0 < sb && segs < kMaxSegs; ++segs) {
        const int slot = p0 / p.page_tokens;
        const int p1 = min(sb, (slot + 1) * p.page_tokens);
        rows[segs] = mk_kv_row(p, p0, kvh);
        if (rows[segs] < 0) break;
        p0 = p1;
    }
    // Stop at the first unresolved page or after kMaxSegs pages.
    {
        int p0 = a, ok_end = a;
        for (int k = 0; k < segs; ++k) {
            if (rows[k] < 0) break;
            const int slot = p0 / p.page_tokens;
            const int p1 = min(sb, (slot + 1) * p.page_tokens);
            ok_end = p1;
            p0 = p1;
        }
        sb = ok_end;
    }
    if (sb > a && !sh.abort) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t bar = smem_u32(&sh.kv_bar);
        mbar_expect_tx(bar, (uint32_t)(sb - a) * HD * 2u * 2u);
        const uint8_t *kb = p.k_pool + (long long)layer * p.layer_stride_bytes;
        const uint8_t *vb = p.v_pool + (long long)layer * p.layer_stride_bytes;
        int p0 = a;
        for (int k = 0; p0 < sb; ++k) {
            const int slot = p0 / p.page_tokens;
            const int p1 = min(sb, (slot + 1) * p.page_tokens);
            const uint32_t bytes = (uint32_t)(p1 - p0) * HD * 2u;
            bulk_load(smem_u32(stK + (size_t)(p0 - a) * HD), kb + rows[k] * HD * 2, bytes, bar);
            bulk_load(smem_u32(stV + (size_t)(p0 - a) * HD), vb + rows[k] * HD * 2, bytes, bar);
            p0 = p1;
        }
        sh.kv_uses += 1;
    } else {
        sb = a;
    }
    sh.staged = sb;
}

// Floats of the per-warp attention partials, rounded up to 16 bytes so the
// vectors after them stay float4-aligned.
__host__ __device__ constexpr int mk_attw_floats(int hd) { return (kMkConsumerWarps * (2 + hd) + 3) / 4 * 4; }

// ---- the kernel ----
// SMALL: hidden <= 1024, so per-thread slices of hidden-width vectors are
// held in registers (all loads of a slice in flight together).
template <int HD, bool SMALL>
__global__ void __launch_bounds__(kMkThreads, 1) decode_megakernel(const MkParams p) {
    constexpr int XC = SMALL ? 4 : 1;  // register chunks of hidden-width inputs (SMALL only)
    extern __shared__ __align__(128) uint8_t mk_smem[];
    __shared__ MkShared sh;
    const int cta = blockIdx.x, grid = gridDim.x;
    const int warp = threadIdx.x / kWarp;
    uint8_t *ring = mk_smem;
    float *xs = reinterpret_cast<float *>(mk_smem + (size_t)p.slots * kMkSlotBytes);  // [xcap] layer input
    float *hn = xs + p.xcap;                                                         // [H] residual after o_proj
    float *attw = hn + p.H;                                                          // [warps][2 + HD]
    float *qh = attw + mk_attw_floats(HD);  // [HD], 16-byte aligned for float4 reads
    float *ah = qh + HD;                                                             // [HD]

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.slots; ++s) {
            mbar_init(smem_u32(&sh.full[s]), 1);
            mbar_init(smem_u32(&sh.empty[s]), kMkConsumerWarps);
        }
        mbar_init(smem_u32(&sh.kv_bar), 1);
        sh.kv_uses = 0;
        sh.staged = 0;
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == kMkConsumerWarps) {
        mk_producer(p, ring, sh);
        return;
    }

    MkRing ring_c{ring, &sh, p.slots, 0u, p.error};
    const MkTiles tq = mk_qkv_tiles(p, cta, grid), ta = mk_att_tiles(p, cta), tg = mk_gu_tiles(p, cta, grid),
                  td = mk_down_tiles(p, cta, grid), tl = mk_lm_tiles(p, cta, grid);
    const bool unit = mk_att_unit(p, cta);
    const int S = p.att_splits;
    const int head = unit ? cta / S : 0, chunk = unit ? cta % S : 0;
    const int NL = p.num_layers, H = p.H, I = p.I, half = HD / 2;
    const unsigned G = (unsigned)grid;
    const int pos0 = p.step->position;
    unsigned *ctrl = p.ctrl;
    const size_t rs_h = (size_t)mk_row_stride(H), rs_i = (size_t)mk_row_stride(I);
    const int lane = threadIdx.x % kWarp;
    MkXReg<XC> xr;
    // Two rows of hidden width against the normalised input in xs.
    auto dot2h = [&](const uint8_t *wa, const uint8_t *wb, float &ra, float &rb) {
        if constexpr (SMALL) {
            mk_dot2r<XC>(wa, wb, xr, H, ra, rb);
        } else {
            mk_dot2(wa, wb, xs, H, ra, rb);
        }
    };

    MK_TRACE(0, 0);
    for (int t = 0; t < p.steps; ++t) {
        const int pos = pos0 + t;
        for (int l = 0; l < NL; ++l) {
            const MkLayer &w = p.layers[l];
            const unsigned lg = (unsigned)(t * NL + l);
            const int tb = l < 3 ? 1 + 32 * l : 128;  // trace event base
            // ---------------- QKV ----------------
            // Constants first (norm weights; this thread's pair of the first
            // tile: bias and rotary factors), so only activations wait.
            MkV4 wln{};
            if constexpr (SMALL) wln = mk_ld4<false>(w.ln1, H);
            float pre_ba = 0.0f, pre_bb = 0.0f, pre_c = 1.0f, pre_s = 0.0f;
            // The K/V append row is resolved here too, except in the first
            // layer of the run's first step, where this CTA may still install
            // the position's page (below): there it is resolved at use.
            long long pre_row = -2;
            const bool page_may_change = t == 0 && l == 0;
            if (lane == 0 && tq.count() > 0 && warp < tq.hi(0) - tq.lo(0)) {
                const int pair = tq.lo(0) + warp;
                const int hh = pair / half, i = pair - hh * half;
                if (hh >= p.q_heads && !page_may_change) {
                    const int kvh = hh < p.q_heads + p.kv_heads ? hh - p.q_heads : hh - p.q_heads - p.kv_heads;
                    pre_row = mk_kv_row(p, pos, kvh);
                }
                if (w.bqkv) {
                    pre_ba = w.bqkv[mk_pair_row(p, pair, 0)];
                    pre_bb = w.bqkv[mk_pair_row(p, pair, 1)];
                }
                if (hh < p.q_heads + p.kv_heads) {
                    pre_c = p.rope_cos[(long long)pos * half + i];
                    pre_s = p.rope_sin[(long long)pos * half + i];
                }
            }
            if (l == 0) {
                if (t > 0) mk_wait_count(&ctrl[kMkCntLm], (unsigned)t * G, sh, p.error);
                if (threadIdx.x == 0) {
                    int token = t == 0 ? p.step->token
                                       : (int)(mk_ld_relaxed_u64(&p.argmax_slots[(t - 1) & 1]) & 0xFFFFFFFFull);
                    if (token < 0 || token >= p.vocab) {
                        if (!sh.abort) mk_flag_error(sh, p.error, kMkErrToken);
                        token = 0;
                    }
                    sh.token = token;
                    if (cta == 0 && t > 0 && p.token_log) p.token_log[t - 1] = token;
                    if (t == 0 && p.step->page_index >= 0 && p.step->page_index < p.max_pages)
                        p.page_table[p.step->page_index] = p.step->page_id;
                }
                mk_consumer_sync();
                const uint16_t *row = p.embed + (size_t)sh.token * H;
                for (int i = td.begin + (int)threadIdx.x; i < td.end; i += kMkConsumers) p.hidden[i] = bf16_to_f32(row[i]);
                if constexpr (SMALL) {
                    MkV4 xv;
#pragma unroll
                    for (int u = 0; u < kMkV; ++u) {
                        const int i = (int)threadIdx.x + u * kMkConsumers;
                        xv.v[u] = i < H ? bf16_to_f32(row[i]) : 0.0f;
                    }
                    mk_rmsnorm4(xv, wln, H, p.eps, xs, sh);
                } else {
                    mk_rmsnorm_any<2>(row, w.ln1, H, p.eps, xs, sh);
                }
            } else {
                mk_wait_count(&ctrl[kMkCntDown], lg * G, sh, p.error);
                if constexpr (SMALL) {
                    mk_rmsnorm4(mk_ld4<true>(p.hidden, H), wln, H, p.eps, xs, sh);
                } else {
                    mk_rmsnorm_any<1>(p.hidden, w.ln1, H, p.eps, xs, sh);
                }
            }
            MK_TRACE(t, tb + 0);
            if constexpr (SMALL) xr.load(xs, H);
            for (int k = 0; k < tq.count(); ++k) {
                const uint8_t *base = ring_c.acquire();
                const int n = tq.hi(k) - tq.lo(k);
                for (int e = warp; e < n; e += kMkConsumerWarps) {
                    float va, vb;
                    dot2h(base + (size_t)e * rs_h, base + (size_t)(tq.per_tile + e) * rs_h, va, vb);
                    if (lane == 0) {
                        const int pair = tq.lo(k) + e;
                        const int hh = pair / half, i = pair - hh * half;
                        const int ra = mk_pair_row(p, pair, 0), rb = mk_pair_row(p, pair, 1);
                        const bool pre = k == 0 && e == warp;
                        va = __fadd_rn(va, pre ? pre_ba : (w.bqkv ? w.bqkv[ra] : 0.0f));
                        vb = __fadd_rn(vb, pre ? pre_bb : (w.bqkv ? w.bqkv[rb] : 0.0f));
                        if (hh < p.q_heads + p.kv_heads) {
                            const float c = pre ? pre_c : p.rope_cos[(long long)pos * half + i];
                            const float s = pre ? pre_s : p.rope_sin[(long long)pos * half + i];
                            const float ra2 = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
                            const float rb2 = __fadd_rn(__fmul_rn(vb, c), __fmul_rn(va, s));
                            va = ra2;
                            vb = rb2;
                        }
                        if (hh < p.q_heads) {
                            p.q[hh * HD + i] = va;
                            p.q[hh * HD + i + half] = vb;
                        } else {
                            const bool is_k = hh < p.q_heads + p.kv_heads;
                            const int kvh = is_k ? hh - p.q_heads : hh - p.q_heads - p.kv_heads;
                            const long long row = (pre && pre_row != -2) ? pre_row : mk_kv_row(p, pos, kvh);
                            if (row >= 0) {
                                uint16_t *cache = reinterpret_cast<uint16_t *>(
                                    (is_k ? p.k_pool : p.v_pool) + (long long)l * p.layer_stride_bytes);
                                cache[row * HD + i] = f32_to_bf16_rne(va);
                                cache[row * HD + i + half] = f32_to_bf16_rne(vb);
                            }
                        }
                    }
                }
                ring_c.release();
            }
            MK_TRACE(t, tb + 19);
            mk_arrive(&ctrl[kMkCntQkv]);
            MK_TRACE(t, tb + 1);

            // ---------------- ATT + o_proj partials ----------------
            if (unit) {
                MK_TRACE(t, tb + 13);
                const int L = pos + 1;
                const int lo = (p.window > 0 && L > p.window) ? L - p.window : 0;
                const int cs = (L - lo + S - 1) / S;
                const int a = min(L, lo + chunk * cs), b = min(L, a + cs);
                const int kvh = head / (p.q_heads / p.kv_heads);
                // Keys before this step's position do not depend on the QKV
                // phase: one thread stages them into the idle activation
                // buffers (xs, hn) while thread 0 waits. The QKV phase's
                // reads of xs ended at the barrier of its arrival.
                uint16_t *stK = reinterpret_cast<uint16_t *>(xs);
                const int cap = (int)(((size_t)p.xcap + H) * 4 / (4 * HD));
                uint16_t *stV = stK + (size_t)cap * HD;
                if (threadIdx.x == kWarp) mk_stage_kv<HD>(p, l, kvh, a, b, pos, cap, stK, stV, sh);
                // This step's key (the last position) joins the staged rows
                // once QKV has written it: its pool row is resolved now.
                const bool has_cur = pos >= a && pos < b && pos - a < cap;
                const long long cur_row = has_cur ? mk_kv_row(p, pos, kvh) : -1;
                MK_TRACE(t, tb + 11);
                mk_wait_count(&ctrl[kMkCntQkv], (lg + 1) * G, sh, p.error, t, tb + 12);
                MK_TRACE(t, tb + 2);
                for (int d = threadIdx.x; d < HD; d += kMkConsumers) qh[d] = __ldcg(p.q + head * HD + d);
                const int sbulk = sh.staged;  // end of the bulk-staged rows
                int sb = sbulk;
                if (has_cur && cur_row >= 0 && sb == pos && !sh.abort) {
                    const uint16_t *kc = reinterpret_cast<const uint16_t *>(p.k_pool + (long long)l * p.layer_stride_bytes);
                    const uint16_t *vc = reinterpret_cast<const uint16_t *>(p.v_pool + (long long)l * p.layer_stride_bytes);
                    for (int d = threadIdx.x; d < HD; d += kMkConsumers) {
                        stK[(size_t)(pos - a) * HD + d] = __ldcg(kc + cur_row * HD + d);
                        stV[(size_t)(pos - a) * HD + d] = __ldcg(vc + cur_row * HD + d);
                    }
                    sb = pos + 1;
                }
                if (sbulk > a && !sh.abort) {
                    if (!mk_bar_wait(smem_u32(&sh.kv_bar), (uint32_t)(sh.kv_uses - 1) & 1u, &sh.abort, true) &&
                        !sh.abort)
                        mk_flag_error(sh, p.error, kMkErrWait);
                }
                mk_consumer_sync();
                MK_TRACE(t, tb + 24);
                float *part = p.att_part + ((size_t)head * S + chunk) * (2 + HD);
                mk_attention_chunk<HD>(p, l, head, a, b, sh.abort ? a : sb, stK, stV, qh, attw, part);
                MK_TRACE(t, tb + 3);
                mk_arrive(&ctrl[kMkCntHead + head]);
                mk_wait_count(&ctrl[kMkCntHead + head], (lg + 1) * (unsigned)S, sh, p.error);
                MK_TRACE(t, tb + 4);
                // Merge the S partials of this head (same order in every CTA,
                // one round trip): each thread loads every chunk's (m, l) and
                // its dims of o, and forms the weights itself.
                const float *ph = p.att_part + (size_t)head * S * (2 + HD);
                for (int d = threadIdx.x; d < HD; d += kMkConsumers) {
                    float mm = -INFINITY, ll = 0.0f, oo = 0.0f;
                    for (int j0 = 0; j0 < S; j0 += 16) {
                        float mj[16], lj[16], oj[16];
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const float *pj = ph + (size_t)(j0 + k) * (2 + HD);
                            const bool in = j0 + k < S;
                            mj[k] = in ? __ldcg(pj) : -INFINITY;
                            lj[k] = in ? __ldcg(pj + 1) : 0.0f;
                            oj[k] = in ? __ldcg(pj + 2 + d) : 0.0f;
                        }
                        // running rescale keeps one pass; order is j ascending
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            if (mj[k] == -INFINITY) continue;
                            const float m_new = fmaxf(mm, mj[k]);
                            const float c_old = mm == -INFINITY ? 0.0f : exp2f(mm - m_new);
                            const float c_new = exp2f(mj[k] - m_new);
                            ll = fmaf(c_new, lj[k], ll * c_old);
                            oo = fmaf(c_new, oj[k], oo * c_old);
                            mm = m_new;
                        }
                    }
                    ah[d] = ll > 0.0f ? __fdiv_rn(oo, ll) : 0.0f;
                }
                mk_consumer_sync();
                MK_TRACE(t, tb + 20);
                for (int k = 0; k < ta.count(); ++k) {
                    const uint8_t *base = ring_c.acquire();
                    const int n = ta.hi(k) - ta.lo(k);
                    // 8 lanes per row, 4 rows per warp pass.
                    const int sub = lane >> 3, sl = lane & 7;
                    constexpr int kVec = HD / 64;  // 16-byte vectors per lane
                    for (int r0 = warp * 4; r0 < n; r0 += 4 * kMkConsumerWarps) {
                        const int r = r0 + sub;
                        float acc = 0.0f;
                        if (r < n) {
                            const uint4 *wr = reinterpret_cast<const uint4 *>(base + (size_t)r * HD * 2) + sl * kVec;
#pragma unroll
                            for (int u = 0; u < kVec; ++u) fma8(acc, wr[u], ah + (sl * kVec + u) * 8);
                        }
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 4);
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 2);
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 1);
                        if (sl == 0 && r < n) p.opart[(size_t)head * H + ta.lo(k) + r] = acc;
                    }
                    ring_c.release();
                }
            }
            mk_arrive(&ctrl[kMkCntO]);
            MK_TRACE(t, tb + 5);

            // ---------------- residual rows after o_proj ----------------
            // Each CTA owns the residual rows it updates in DOWN: it sums the
            // heads' o_proj partials of those rows (head order), adds the o
            // bias and the residual, keeps them in hn and publishes them.
            {
                const int rows = td.end - td.begin;
                float bo_r = 0.0f;
                const int r = (int)threadIdx.x;
                if (r < rows && w.bo) bo_r = w.bo[td.begin + r];
                mk_wait_count(&ctrl[kMkCntO], (lg + 1) * G, sh, p.error);
                MK_TRACE(t, tb + 6);
                if (r < rows) {
                    const int row = td.begin + r;
                    float part[16];
                    float sv = 0.0f;
                    for (int h0 = 0; h0 < p.q_heads; h0 += 16) {
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            part[k] = h0 + k < p.q_heads ? __ldcg(p.opart + (size_t)(h0 + k) * H + row) : 0.0f;
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            if (h0 + k < p.q_heads) sv = __fadd_rn(sv, part[k]);
                    }
                    if (w.bo) sv = __fadd_rn(sv, bo_r);
                    const float v = __fadd_rn(__ldcg(p.hidden + row), sv);
                    hn[row] = v;
                    p.hnew[row] = v;
                }
                mk_arrive(&ctrl[kMkCntRes]);
            }

            // ---------------- GU ----------------
            MkV4 wln2{};
            if constexpr (SMALL) wln2 = mk_ld4<false>(w.ln2, H);
            mk_wait_count(&ctrl[kMkCntRes], (lg + 1) * G, sh, p.error);
            MK_TRACE(t, tb + 10);
            if constexpr (SMALL) {
                mk_rmsnorm4(mk_ld4<true>(p.hnew, H), wln2, H, p.eps, xs, sh);
            } else {
                mk_rmsnorm_any<1>(p.hnew, w.ln2, H, p.eps, xs, sh);
            }
            MK_TRACE(t, tb + 14);
            if (l == 0 && cta == 0 && threadIdx.x == 0) p.argmax_slots[t & 1] = 0ull;
            if constexpr (SMALL) xr.load(xs, H);
            for (int k = 0; k < tg.count(); ++k) {
                const uint8_t *base = ring_c.acquire();
                if (k == 0) MK_TRACE(t, tb + 16);
                const int n = tg.hi(k) - tg.lo(k);
                for (int e = warp; e < n; e += kMkConsumerWarps) {
                    float g, u;
                    dot2h(base + (size_t)e * rs_h, base + (size_t)(tg.per_tile + e) * rs_h, g, u);
                    if (lane == 0) p.act[tg.lo(k) + e] = silu_mul(g, u);
                }
                ring_c.release();
            }
            MK_TRACE(t, tb + 17);
            mk_arrive(&ctrl[kMkCntGu]);
            MK_TRACE(t, tb + 7);

            // ---------------- DOWN ----------------
            mk_wait_count(&ctrl[kMkCntGu], (lg + 1) * G, sh, p.error);
            MK_TRACE(t, tb + 8);
            mk_gather(xs, p.act, I);
            MK_TRACE(t, tb + 15);
            for (int k = 0; k < td.count(); ++k) {
                const uint8_t *base = ring_c.acquire();
                if (k == 0) MK_TRACE(t, tb + 21);
                const int n = td.hi(k) - td.lo(k);
                for (int r = warp; r < n; r += kMkConsumerWarps) {
                    const float acc = mk_dot(base + (size_t)r * rs_i, xs, I);
                    if (lane == 0) {
                        const int row = td.lo(k) + r;
                        p.hidden[row] = __fadd_rn(hn[row], acc);
                    }
                }
                ring_c.release();
            }
            MK_TRACE(t, tb + 18);
            mk_arrive(&ctrl[kMkCntDown]);
            MK_TRACE(t, tb + 9);
        }

        // ---------------- LM head + argmax ----------------
        MkV4 wfn{};
        if constexpr (SMALL) wfn = mk_ld4<false>(p.final_norm, H);
        mk_wait_count(&ctrl[kMkCntDown], (unsigned)(t * NL + NL) * G, sh, p.error);
        MK_TRACE(t, 120);
        if constexpr (SMALL) {
            mk_rmsnorm4(mk_ld4<true>(p.hidden, H), wfn, H, p.eps, xs, sh);
        } else {
            mk_rmsnorm_any<1>(p.hidden, p.final_norm, H, p.eps, xs, sh);
        }
        const bool want_logits = p.logits != nullptr && t == p.steps - 1;
        if constexpr (SMALL) xr.load(xs, H);
        unsigned long long best = 0ull;
        for (int k = 0; k < tl.count(); ++k) {
            const uint8_t *base = ring_c.acquire();
            const int n = tl.hi(k) - tl.lo(k);
            // Rows r and r + 8 per warp pass.
            for (int r = warp; r < n; r += 2 * kMkConsumerWarps) {
                const int r2 = r + kMkConsumerWarps;
                const bool two = r2 < n;
                float a0, a1;
                dot2h(base + (size_t)r * rs_h, base + (size_t)(two ? r2 : r) * rs_h, a0, a1);
                if (lane == 0) {
                    const int row = tl.lo(k) + r;
                    if (want_logits) p.logits[row] = a0;
                    unsigned long long key = ((unsigned long long)total_order_key(a0) << 32) | (unsigned)row;
                    if (two) {
                        if (want_logits) p.logits[row + kMkConsumerWarps] = a1;
                        const unsigned long long k1 =
                            ((unsigned long long)total_order_key(a1) << 32) | (unsigned)(row + kMkConsumerWarps);
                        key = k1 > key ? k1 : key;
                    }
                    best = key > best ? key : best;
                }
            }
            ring_c.release();
        }
        if (lane == 0) sh.best8[warp] = best;
        mk_consumer_sync();
        if (threadIdx.x == 0) {
            unsigned long long b = 0ull;
#pragma unroll
            for (int k = 0; k < kMkConsumerWarps; ++k) b = sh.best8[k] > b ? sh.best8[k] : b;
            if (b) atomicMax(&p.argmax_slots[t & 1], b);
        }
        const unsigned old = mk_arrive_fetch(&ctrl[kMkCntLm]);
        MK_TRACE(t, 121);
        if (t == p.steps - 1 && threadIdx.x == 0 && old == (unsigned)p.steps * G - 1u) {
            // Last CTA of the run: publish the final token, reset the counters.
            const unsigned long long key = mk_ld_relaxed_u64(&p.argmax_slots[t & 1]);
            *p.argmax_out = key;
            if (p.token_log) p.token_log[t] = (int32_t)(key & 0xFFFFFFFFull);
            for (int k = 0; k < kMkCtrlWords; ++k) ctrl[k] = 0u;
            __threadfence();
        }
    }
    // A K/V staging copy still in flight (abort mode) must land before exit.
    if (threadIdx.x == kWarp && sh.kv_uses > 0)
        mk_bar_wait(smem_u32(&sh.kv_bar), (uint32_t)(sh.kv_uses - 1) & 1u, &sh.abort, false);
}

// Dynamic shared memory of the kernel for `slots` ring slots: ring, the
// hi/lo split (xcap floats' worth), hn [hidden], per-warp attention
// partials, qh and ah [hd] each. xcap and hidden are multiples of 16, so
// every region starts 16-byte aligned.
inline size_t mk_smem_bytes(int slots, int xcap, int hidden, int hd) {
    return (size_t)slots * kMkSlotBytes + 4 * ((size_t)xcap + hidden + (size_t)mk_attw_floats(hd) + 2 * (size_t)hd);
}

}  // namespace cheetah
