// Persistent single-sequence decode kernel: B = 1, bf16 weights, bf16 KV.
//
// One CTA per SM runs a whole decode step, or a whole run of greedy steps.
// Every CTA owns fixed slices of every weight matrix. A producer warp streams
// those slices, in exactly the order the CTA consumes them, through a ring of
// 32 KB shared-memory slots: weights with 1D bulk copies (cp.async.bulk, L2
// evict-first), earlier steps' K/V with 2D tensor-map loads (128-byte
// swizzle, no multicast). Neither depends on this step's activations, so the
// stream runs ahead across phase boundaries, layers and steps: HBM stays busy
// while the CTAs order themselves along the activation chain. Eight consumer
// warps compute from the slots.
//
// Phases of one layer (`Qwen2Native::forward_layer`, qwen2.rs:430-465), four
// grid-wide hand-offs:
//   QKV   RMSNorm(ln1) (`ops.rs:646-652`) of the residual; q/k/v rows (a copy
//         with the first rows of all rotate-half pairs, then the partners, so
//         a warp computes one pair); bias (`ops.rs:1156`), RoPE
//         (`ops.rs:693-740`); K/V appended to the paged cache
//         (`ops.rs:1329`), q to global.                           [all CTAs]
//   ATT   every CTA is an attention unit of one query head and owns a block
//         of that head's o_proj rows. A unit computes its head's attention
//         (`ops.rs:1357-1467`) over the K/V tiles the producer streamed, with
//         all 256 consumer threads: scores one key per thread, a block-wide
//         softmax (log2 domain), P V one dimension pair x key group per
//         thread, the groups summed in a fixed order; this step's own key
//         (written by QKV, read through L2) joins the scores. Short
//         contexts: every unit of the head computes the whole attention
//         itself (no hand-off). Long contexts: the keys split over the
//         head's first units, whose partials every unit of the head merges
//         after a head-local hand-off. Then the unit's o_proj rows of
//         W_o[:, head]: per-head partials.
//   GU    every CTA sums residual + the heads' o_proj partials (+ o bias,
//         qwen2.rs:442-449) for all rows itself, in one fixed order (so all
//         CTAs hold the same values); RMSNorm(ln2); gate/up rows; SiLU(gate)
//         * up (`ops.rs:743-747`).                                [all CTAs]
//   DOWN  down rows (each row's dot split over idle warps, summed in warp
//         order); residual add (qwen2.rs:459-463).                [all CTAs]
// After the last layer, LM: final RMSNorm and lm_head rows (`ops.rs:1513`),
// greedy argmax as a packed (total-order key, index) atomicMax, which keeps
// the larger index on ties like `Iterator::max_by` (engine.rs:2247-2253).
// The next step embeds that argmax.
//
// Ordering: monotonic arrival counters in global memory. Release = consumer
// barrier, then one thread's red.release.gpu add; acquire = one thread spins
// with ld.acquire.gpu, then the consumer barrier. The producer acquires the
// QKV counter of the step that wrote a key before it streams that key, and
// orders the acquired writes before its tensor-map reads with a proxy fence.
// All reductions run in a fixed order, so results are reproducible run to
// run. The last CTA to finish the run resets the counters. Every wait is
// bounded by %globaltimer: on a timeout the CTA records the error word and
// switches to abort mode (waits return at once, work continues over
// in-bounds addresses only, no new copies are issued), the producer drains
// the copies already in flight, and the CTA returns. Other CTAs see the error
// word and abort too.
#pragma once

#include <algorithm>
#include <type_traits>

#include "attention_mma.cuh"
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
constexpr int kMkMaxHeads = 64;  // query heads
constexpr int kMkCtrlWords = 8 + kMkMaxHeads;
constexpr int kMkKvRows = 64;       // sub-tile pool rows of a step cached in shared memory
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
__device__ long long g_mk_cycles[256][32];
// Producer issue times of the tiles of layer 1 in the first step.
__device__ unsigned long long g_mk_ptrace[256][32];
#define MK_PTRACE(step, layer, k)                                                               \
    do {                                                                                        \
        if ((step) == 0 && (layer) == 1 && (k) < 32) {                                           \
            unsigned long long t__;                                                             \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t__));                            \
            g_mk_ptrace[blockIdx.x][(k)] = t__;                                                 \
        }                                                                                       \
    } while (0)
#else
#define MK_PTRACE(step, layer, k) \
    do {                          \
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
    kMkCntHead = 8  // + query head: key-split partials of the head published
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
    int window, slots, xcap;
    // Bulk copies in flight per CTA (issued, not landed): during the layers,
    // and during the lm_head stream.
    int inflight_layers, inflight_lm;
    float eps, scale_log2;  // 1/sqrt(d) * log2(e)
    const uint16_t *embed;
    const uint16_t *lm_head;  // [vocab][H]
    const float *final_norm;
    const float *rope_cos, *rope_sin;  // [max_positions][d/2]
    uint8_t *k_pool, *v_pool;          // [layer][page][kv_head][page_tokens][d] bf16
    long long layer_stride_bytes;
    long long layer_rows;              // tensor-map rows per layer (pages * kv_heads * page_tokens)
    int num_pages, page_tokens, max_pages;
    int32_t *page_table;
    const StepState *step;  // token and position of the first step, optional page install
    int steps;
    float *hidden;    // [H] residual
    float *q;         // [q_heads * d]
    float *opart;     // [q_heads][H] o_proj partials
    float *act;       // [I]
    float *att_part;  // [q_heads][units per head][2 + d]: m (log2 domain), l, o[d] of key splits
    int att_part_units;
    unsigned *ctrl;   // kMkCtrlWords arrival counters, zero between runs
    unsigned long long *argmax_slots;  // [2], alternating per step
    unsigned long long *argmax_out;    // packed key of the last step
    int32_t *token_log;                // [steps] greedy token of each step, nullable
    float *logits;                     // [vocab] logits of the last step, nullable
    int *error;
    unsigned long long timeout_ns;     // bound of every wait
    int stall_test;                    // test hook: the first attention wait targets a count never reached
};

struct MkShared {
    unsigned long long full[kMkMaxSlots];
    unsigned long long empty[kMkMaxSlots];
    unsigned long long kv_bar;  // staged K/V sub-tile of the attention
    // Pool row of the first position of the unit's K/V sub-tiles s0 + i
    // (i < kMkKvRows) for the current step, -1 when the page is missing;
    // written by the staging thread, read by all after the consumer barrier.
    long long kv_rows[kMkKvRows];
    int kv_uses;    // kv_bar phases completed + the one in flight
    int kv_staged;  // the current sub-tile was staged (its page exists)
    volatile int abort;
    int token;
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
                                            bool honour_abort, unsigned long long timeout_ns, int sleep_ns = 0) {
    if (mk_bar_test(bar, parity)) return true;
    const unsigned long long t0 = mk_now();
    while (true) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (mk_bar_test(bar, parity)) return true;
        if (honour_abort && *abort_flag) return false;
        if (mk_now() - t0 > timeout_ns) return false;
    }
}

__device__ __forceinline__ void mk_flag_error(MkShared &sh, int *error, int code) {
    sh.abort = 1;
    atomicCAS(error, 0, code);
}

// Bounded spin of one thread until *cnt reaches target. Returns false when
// the run aborts (another CTA's error, or this wait's timeout, recorded).
__device__ __forceinline__ bool mk_poll_count(const unsigned *cnt, unsigned target, MkShared &sh, int *error,
                                              unsigned long long timeout_ns) {
    if (sh.abort) return false;
    if ((int)(mk_ld_acquire(cnt) - target) >= 0) return true;
    const unsigned long long t0 = mk_now();
    unsigned polls = 0;
    while ((int)(mk_ld_acquire(cnt) - target) < 0) {
        ++polls;
        if (polls > 256) __nanosleep(40);
        if ((polls & 31u) == 0) {
            if (*(volatile int *)error != 0) {
                sh.abort = 1;
                return false;
            }
            if (mk_now() - t0 > timeout_ns) {
                mk_flag_error(sh, error, kMkErrWait);
                return false;
            }
        }
    }
    return true;
}

// Counter wait by consumer thread 0, broadcast through the consumer barrier.
// Returns false in abort mode.
__device__ __forceinline__ bool mk_wait_count(const unsigned *cnt, unsigned target, MkShared &sh, int *error,
                                              unsigned long long timeout_ns) {
    if (threadIdx.x == 0) mk_poll_count(cnt, target, sh, error, timeout_ns);
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

// Arrival nobody orders data by (a count kept in step with the others).
__device__ __forceinline__ void mk_arrive_relaxed(unsigned *cnt) {
    mk_consumer_sync();
    if (threadIdx.x == 0) asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
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

// The attention unit of a CTA: query head h (contiguous CTA ranges per
// head), its KV head, index u within the head's U units.
struct MkUnit {
    int h, kvh, u, U;
};
__device__ __forceinline__ MkUnit mk_unit(const MkParams &p, int cta, int grid) {
    const int h = (int)(((long long)cta * p.q_heads) / grid);
    const int b0 = (int)(((long long)h * grid + p.q_heads - 1) / p.q_heads);
    const int b1 = (int)(((long long)(h + 1) * grid + p.q_heads - 1) / p.q_heads);
    return {h, h / (p.q_heads / p.kv_heads), cta - b0, b1 - b0};
}

// o_proj rows of a unit: rows of W_o[:, head] ([H][head_dim] block).
__device__ __forceinline__ MkTiles mk_wo_tiles(const MkParams &p, const MkUnit &un) {
    return {mk_split(p.H, un.U, un.u), mk_split(p.H, un.U, un.u + 1), kMkSlotBytes / (2 * p.hd)};
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

// The attention plan of one step: the visible keys before this step's
// position are [lo, pos), covered by sub-tiles of T positions aligned to
// absolute positions (a sub-tile never crosses a KV page). They split over
// the head's first `splits` units, `per` sub-tiles each (a unit stages and
// folds them one at a time); the last split also folds in this step's key.
struct MkAttPlan {
    int lo, st_lo, n_st, splits, per;
};
__device__ __forceinline__ MkAttPlan mk_att_plan(const MkParams &p, int pos, int units) {
    MkAttPlan a;
    const int T = kTileBytes / (p.hd * 2);
    const int L = pos + 1;
    a.lo = (p.window > 0 && L > p.window) ? L - p.window : 0;
    a.st_lo = a.lo / T;
    const int st_hi = (pos + T - 1) / T;
    a.n_st = max(0, st_hi - a.st_lo);
    if (a.n_st <= 1) {
        a.splits = 1;
        a.per = a.n_st;
    } else {
        a.splits = min(units, a.n_st);
        a.per = (a.n_st + a.splits - 1) / a.splits;
        a.splits = (a.n_st + a.per - 1) / a.per;
    }
    return a;
}
// Sub-tiles [s0, s1) this unit computes (empty for units past the splits).
struct MkKvRange {
    int s0, s1;
    bool computes;  // the unit runs the attention math (it may have no old keys)
    bool has_cur;   // it folds in this step's own key
};
__device__ __forceinline__ MkKvRange mk_kv_range(const MkAttPlan &a, const MkUnit &un) {
    MkKvRange r;
    if (a.splits == 1) {
        r.s0 = a.st_lo;
        r.s1 = a.st_lo + a.n_st;
        r.computes = true;
        r.has_cur = true;
    } else if (un.u < a.splits) {
        r.s0 = a.st_lo + un.u * a.per;
        r.s1 = min(a.st_lo + a.n_st, r.s0 + a.per);
        r.computes = true;
        r.has_cur = un.u == a.splits - 1;
    } else {
        r.s0 = r.s1 = 0;
        r.computes = false;
        r.has_cur = false;
    }
    return r;
}

// Pool row of (position, KV head) through the sequence's page table, or -1
// when the page is not installed or out of range (the access is skipped).
__device__ __forceinline__ long long mk_kv_row(const MkParams &p, int pos, int kv_head) {
    const int page_slot = pos / p.page_tokens;
    if (page_slot >= p.max_pages || page_slot < 0) return -1;
    const int page = __ldcg(p.page_table + page_slot);
    if (page < 0 || page >= p.num_pages) return -1;
    return ((long long)page * p.kv_heads + kv_head) * p.page_tokens + (pos - page_slot * p.page_tokens);
}

// ---- producer ----
__device__ void mk_producer(const MkParams &p, uint8_t *ring, MkShared &sh) {
    if ((threadIdx.x % kWarp) != 0) return;
    const int cta = blockIdx.x, grid = gridDim.x;
    const uint64_t pol = mk_evict_first_policy();
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t rs_h = (uint32_t)mk_row_stride(p.H), rs_i = (uint32_t)mk_row_stride(p.I);
    const unsigned G = (unsigned)grid;
    uint32_t seq = 0;
    int cur_t = 0, cur_l = 0;  // position in the schedule (trace builds)
    uint32_t layer_seq0 = 0;   // seq of the layer's first tile (trace builds)
    (void)layer_seq0;
    (void)cur_t;
    (void)cur_l;
    bool ok = true;
    // Claim the next slot (free, and the copy `inflight` tiles back landed)
    // and arm its barrier with the tile's byte count.
    auto begin_tile = [&](uint32_t bytes, int inflight) -> uint32_t {
        if (!ok) return 0;
        const int s = (int)(seq % (uint32_t)p.slots);
        const uint32_t n = seq / (uint32_t)p.slots;
        // The producer backs off between polls: its spin shares an issue
        // slot with two consumer warps.
        if (sh.abort ||
            (n > 0 && !mk_bar_wait(smem_u32(&sh.empty[s]), (n - 1) & 1u, &sh.abort, true, p.timeout_ns, 128))) {
            ok = false;
            return 0;
        }
        if (seq >= (uint32_t)inflight) {
            const uint32_t old = seq - (uint32_t)inflight;
            if (!mk_bar_wait(smem_u32(&sh.full[old % (uint32_t)p.slots]), (old / (uint32_t)p.slots) & 1u, &sh.abort,
                             true, p.timeout_ns, 128)) {
                ok = false;
                return 0;
            }
        }
        mbar_expect_tx(smem_u32(&sh.full[s]), bytes);
        MK_PTRACE(cur_t, cur_l, (int)(seq - layer_seq0));
        return ring_s + (uint32_t)s * kMkSlotBytes;
    };
    auto copy = [&](uint32_t dst, const void *src, uint32_t bytes) {
        mk_bulk_load(dst, src, bytes, smem_u32(&sh.full[seq % (uint32_t)p.slots]), pol);
    };

    const MkTiles tq = mk_qkv_tiles(p, cta, grid), tg = mk_gu_tiles(p, cta, grid), td = mk_down_tiles(p, cta, grid),
                  tl = mk_lm_tiles(p, cta, grid);
    const MkUnit un = mk_unit(p, cta, grid);
    const MkTiles tw = mk_wo_tiles(p, un);
    const uint32_t wo_row = (uint32_t)(2 * p.hd);
    for (int t = 0; t < p.steps && ok; ++t) {
        for (int l = 0; l < p.num_layers && ok; ++l) {
            const MkLayer &w = p.layers[l];
            const int q = p.inflight_layers;
            layer_seq0 = seq;
            cur_t = t;
            cur_l = l;
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
            for (int k = 0; k < tw.count() && ok; ++k) {
                const uint32_t n = (uint32_t)(tw.hi(k) - tw.lo(k));
                const uint32_t base = begin_tile(n * wo_row, q);
                if (!ok) break;
                copy(base, reinterpret_cast<const uint8_t *>(w.wo) + ((size_t)un.h * p.H + tw.lo(k)) * wo_row,
                     n * wo_row);
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
        mk_bar_wait(smem_u32(&sh.full[s]), n_last & 1u, &sh.abort, false, p.timeout_ns);
    }
}

// ---- consumer building blocks ----
struct MkRing {
    uint8_t *base;
    MkShared *sh;
    int slots;
    uint32_t seq;
    int *error;
    unsigned long long timeout_ns;

    // Wait for the tile `ahead` tiles past the next one; returns its slot.
    __device__ uint8_t *acquire(int ahead = 0) {
        const uint32_t q = seq + (uint32_t)ahead;
        const int s = (int)(q % (uint32_t)slots);
        if (!sh->abort) {
            const uint32_t parity = (q / (uint32_t)slots) & 1u;
            if (!mk_bar_wait(smem_u32(&sh->full[s]), parity, &sh->abort, true, timeout_ns) && !sh->abort)
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

// N dot products of bf16 rows (shared memory) with the register vector, all
// rows' loads issued before the math, N independent accumulators; the N
// warp reductions are interleaved.
template <int XC, int N>
__device__ __forceinline__ void mk_dotNr(const uint8_t *const (&rows)[N], const MkXReg<XC> &x, int K, float (&r)[N]) {
    const int lane = threadIdx.x % kWarp;
    uint4 u[N][XC];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const uint4 *pr = reinterpret_cast<const uint4 *>(rows[n]);
#pragma unroll
        for (int c = 0; c < XC; ++c) {
            const int idx = lane + c * kWarp;
            u[n][c] = idx < K / 8 ? pr[idx] : make_uint4(0, 0, 0, 0);
        }
    }
    float acc[N];
#pragma unroll
    for (int n = 0; n < N; ++n) acc[n] = 0.0f;
#pragma unroll
    for (int c = 0; c < XC; ++c) {
#pragma unroll
        for (int n = 0; n < N; ++n) mk_fma8r(acc[n], u[n][c], x.v[c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int n = 0; n < N; ++n) acc[n] += __shfl_xor_sync(0xFFFFFFFFu, acc[n], o);
    }
#pragma unroll
    for (int n = 0; n < N; ++n) r[n] = acc[n];
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

// Partial dot product of a bf16 row with an f32 vector (both shared memory)
// over 16-byte chunks [c0, c1), four accumulators, summed within the warp.
__device__ __forceinline__ float mk_dot_range(const uint8_t *wa, const float *x, int c0, int c1) {
    const int lane = threadIdx.x % kWarp;
    const uint4 *pa = reinterpret_cast<const uint4 *>(wa);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int v = c0 + lane;
    for (; v + 3 * kWarp < c1; v += 4 * kWarp) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = pa[v + u * kWarp];
#pragma unroll
        for (int u = 0; u < 4; ++u) fma8(acc[u], w[u], x + (v + u * kWarp) * 8);
    }
    for (; v < c1; v += kWarp) fma8(acc[0], pa[v], x + v * 8);
    return warp_sum(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])));
}

// Shared memory of the attention in xs: the staged K | V sub-tile (16 KB),
// then the scratch floats: scores of the sub-tile's keys (+ this step's
// key), 16 reduction words, P V partials [8][64] or [4][128].
constexpr int kMkAttStageFloats = 2 * kTileBytes / 4;
__host__ __device__ constexpr int mk_att_scratch_floats(int hd) {
    return kMkAttStageFloats + (kTileBytes / (hd * 2)) + 4 + 16 + 512;
}

// Byte offset of dims [d, d + 8) (d % 8 == 0) of row r in a K or V sub-tile
// of T rows stored by the 128-byte-swizzled tensor-map load (64-dim halves).
template <int HD>
__device__ __forceinline__ uint32_t mk_kv_off(int r, int d) {
    constexpr int T = kTileBytes / (HD * 2);
    const int c = d >> 3;
    return (uint32_t)((c >> 3) * (T * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// ---- the kernel ----
// SMALL: hidden <= 1024, so per-thread slices of hidden-width vectors are
// held in registers (all loads of a slice in flight together).
template <int HD, bool SMALL>
__global__ void __launch_bounds__(kMkThreads, 1)
    decode_megakernel(const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
                      const MkParams p) {
    constexpr int XC = SMALL ? 4 : 1;  // register chunks of hidden-width inputs (SMALL only)
    constexpr int T = kTileBytes / (HD * 2);  // positions per K/V sub-tile
    extern __shared__ __align__(1024) uint8_t mk_smem_raw[];
    __shared__ MkShared sh;
    const int cta = blockIdx.x, grid = gridDim.x;
    const int warp = threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    // The ring starts on a 1024-byte boundary (128-byte-swizzled K/V tiles).
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(mk_smem_raw) + 1023) & ~uintptr_t(1023));
    float *xs = reinterpret_cast<float *>(ring + (size_t)p.slots * kMkSlotBytes);  // [xcap] layer input / merge buffer
    float *hn = xs + p.xcap;                                                      // [H] residual after o_proj
    float *ah = hn + p.H;                                                         // [8][HD]: o of the head | q
    float *kvc = ah + 8 * HD;                                                     // [2][HD] this step's K, V row

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.slots; ++s) {
            mbar_init(smem_u32(&sh.full[s]), 1);
            mbar_init(smem_u32(&sh.empty[s]), kMkConsumerWarps);
        }
        mbar_init(smem_u32(&sh.kv_bar), 1);
        sh.kv_uses = 0;
        sh.kv_staged = 0;
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == kMkConsumerWarps) {
        mk_producer(p, ring, sh);
        return;
    }

    MkRing ring_c{ring, &sh, p.slots, 0u, p.error, p.timeout_ns};
    const MkTiles tq = mk_qkv_tiles(p, cta, grid), tg = mk_gu_tiles(p, cta, grid), td = mk_down_tiles(p, cta, grid),
                  tl = mk_lm_tiles(p, cta, grid);
    const MkUnit un = mk_unit(p, cta, grid);
    const MkTiles tw = mk_wo_tiles(p, un);
    const int NL = p.num_layers, H = p.H, I = p.I, half = HD / 2;
    const unsigned G = (unsigned)grid;
    const int pos0 = p.step->position;
    unsigned *ctrl = p.ctrl;
    const size_t rs_h = (size_t)mk_row_stride(H), rs_i = (size_t)mk_row_stride(I);
    const unsigned long long tmo = p.timeout_ns;
    MkXReg<XC> xr;

    MK_TRACE(0, 0);
    for (int t = 0; t < p.steps; ++t) {
        const int pos = pos0 + t;
        const MkAttPlan plan = mk_att_plan(p, pos, un.U);
        const MkKvRange kr = mk_kv_range(plan, un);
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
                if (t > 0) mk_wait_count(&ctrl[kMkCntLm], (unsigned)t * G, sh, p.error, tmo);
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
                mk_wait_count(&ctrl[kMkCntDown], lg * G, sh, p.error, tmo);
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
                    if constexpr (SMALL) {
                        const uint8_t *rows[2] = {base + (size_t)e * rs_h, base + (size_t)(tq.per_tile + e) * rs_h};
                        float r2[2];
                        mk_dotNr<XC, 2>(rows, xr, H, r2);
                        va = r2[0];
                        vb = r2[1];
                    } else {
                        mk_dot2(base + (size_t)e * rs_h, base + (size_t)(tq.per_tile + e) * rs_h, xs, H, va, vb);
                    }
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
            {
                uint8_t *kvst = reinterpret_cast<uint8_t *>(xs);    // staged K | V sub-tile
                const uint32_t kvst_s = smem_u32(kvst);
                float *sc = xs + kMkAttStageFloats;                 // [T + 1] scores, then probabilities
                float *red = sc + T + 4;                            // [16] block reductions
                float *opv = red + 16;                              // [key groups][HD] P V partials
                float *qs = ah + HD;                                // [HD] q of the head
                const int nsub = kr.s1 - kr.s0;
                // One thread stages the unit's first K/V sub-tile into the
                // idle activation buffer while the others wait for QKV (xs's
                // last generic reads ended at QKV's arrival barrier). The K/V
                // of earlier steps were acquired through earlier waits.
                auto stage = [&](int i) -> int {
                    const long long row = i < kMkKvRows ? sh.kv_rows[i] : mk_kv_row(p, (kr.s0 + i) * T, un.kvh);
                    if (row < 0 || sh.abort) return 0;
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    const uint32_t bar = smem_u32(&sh.kv_bar);
                    const int y = (int)((long long)l * p.layer_rows + row);
                    mbar_expect_tx(bar, 2u * kTileBytes);
#pragma unroll
                    for (int hf = 0; hf < HD / 64; ++hf) {
                        tma_load_2d(kvst_s + (uint32_t)(hf * T * 128), &k_map, hf * 64, y, bar);
                        tma_load_2d(kvst_s + kTileBytes + (uint32_t)(hf * T * 128), &v_map, hf * 64, y, bar);
                    }
                    sh.kv_uses += 1;
                    return 1;
                };
                if (threadIdx.x == kWarp) {
                    if (l == 0) {
                        // The step's page lookups for all layers, loads in flight together.
                        for (int i0 = 0; i0 < min(nsub, kMkKvRows); i0 += 16) {
                            int pg[16];
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int slot = (kr.s0 + i0 + k) * T / p.page_tokens;
                                pg[k] = (i0 + k < nsub && slot < p.max_pages) ? __ldcg(p.page_table + slot) : -1;
                            }
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int i = i0 + k;
                                if (i >= kMkKvRows) break;
                                const int ppos = (kr.s0 + i) * T, slot = ppos / p.page_tokens;
                                sh.kv_rows[i] = (pg[k] >= 0 && pg[k] < p.num_pages)
                                                    ? ((long long)pg[k] * p.kv_heads + un.kvh) * p.page_tokens +
                                                          (ppos - slot * p.page_tokens)
                                                    : -1;
                            }
                        }
                    }
                    sh.kv_staged = (kr.computes && nsub > 0) ? stage(0) : 0;
                }
                // This step's own K/V row is resolved before the wait.
                const long long cur_row = kr.has_cur ? mk_kv_row(p, pos, un.kvh) : -1;
                const unsigned stall = (p.stall_test && t == 0 && l == 0) ? 0x40000000u : 0u;
                mk_wait_count(&ctrl[kMkCntQkv], (lg + 1) * G + stall, sh, p.error, tmo);
                MK_TRACE(t, tb + 2);
                const uint16_t *kc = reinterpret_cast<const uint16_t *>(p.k_pool + (long long)l * p.layer_stride_bytes);
                const uint16_t *vc = reinterpret_cast<const uint16_t *>(p.v_pool + (long long)l * p.layer_stride_bytes);
                // This step's K/V row and the head's q, one load per thread.
                for (int d = threadIdx.x; d < 3 * HD; d += kMkConsumers) {
                    float v = 0.0f;
                    if (!sh.abort) {
                        if (d < 2 * HD) {
                            if (cur_row >= 0) v = bf16_to_f32(__ldcg((d < HD ? kc : vc) + cur_row * HD + (d % HD)));
                        } else {
                            v = __ldcg(p.q + (size_t)un.h * HD + (d - 2 * HD));
                        }
                    }
                    if (d < 2 * HD) kvc[d] = v;
                    else qs[d - 2 * HD] = v;
                }
                mk_consumer_sync();
                MK_TRACE(t, tb + 11);
                // Sub-tile by sub-tile (staged one at a time); running
                // softmax state per dimension (threads d < HD).
                constexpr int kTpk = kMkConsumers / T;      // threads per key in the scores
                constexpr int kDpt = HD / kTpk;             // dims per thread (16)
                constexpr int kPairs = HD / 2;
                constexpr int kKg = kMkConsumers / kPairs;  // key groups in P V
                float run_m = -INFINITY, run_l = 0.0f, run_o = 0.0f;
                const int rounds = kr.computes ? max(1, nsub) : 0;
                for (int rd = 0; rd < rounds; ++rd) {
                    const bool cur_here = kr.has_cur && rd == rounds - 1;
                    const bool have = rd < nsub && sh.kv_staged;
                    if (have && !sh.abort) {
                        if (!mk_bar_wait(smem_u32(&sh.kv_bar), (uint32_t)(sh.kv_uses - 1) & 1u, &sh.abort, true, tmo) &&
                            !sh.abort)
                            mk_flag_error(sh, p.error, kMkErrWait);
                    }
                    if (rd == 0) MK_TRACE(t, tb + 10);
                    // Scores (log2 domain): kTpk threads per key.
                    float lmax = -INFINITY;
                    {
                        const int key = threadIdx.x / kTpk, qt = threadIdx.x % kTpk;
                        const int ppos = (kr.s0 + rd) * T + key;
                        const bool vis = have && !sh.abort && ppos >= plan.lo && ppos < pos;
                        float acc = 0.0f;
                        if (vis) {
#pragma unroll
                            for (int d = qt * kDpt; d < (qt + 1) * kDpt; d += 8) {
                                uint4 kv;
                                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                             : "=r"(kv.x), "=r"(kv.y), "=r"(kv.z), "=r"(kv.w)
                                             : "r"(kvst_s + mk_kv_off<HD>(key, d)));
                                fma8(acc, kv, qs + d);
                            }
                        }
#pragma unroll
                        for (int o = 1; o < kTpk; o <<= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
                        if (qt == 0) {
                            const float sv = vis ? acc * p.scale_log2 : -INFINITY;
                            sc[key] = sv;
                            lmax = sv;
                        }
                    }
                    if (warp == 0) {
                        // This step's own key.
                        float acc = 0.0f;
                        if (cur_here && cur_row >= 0) {
                            for (int d = lane; d < HD; d += kWarp) acc = fmaf(qs[d], kvc[d], acc);
                        }
                        acc = warp_sum(acc);
                        if (lane == 0) {
                            const float sv = (cur_here && cur_row >= 0) ? acc * p.scale_log2 : -INFINITY;
                            sc[T] = sv;
                            lmax = fmaxf(lmax, sv);
                        }
                    }
                    lmax = warp_max(lmax);
                    if (lane == 0) red[warp] = lmax;
                    mk_consumer_sync();
                    float mr = red[0];
#pragma unroll
                    for (int w8 = 1; w8 < kMkConsumerWarps; ++w8) mr = fmaxf(mr, red[w8]);
                    // Probabilities (`softmax`, ops.rs:770-781, as exp2 of
                    // log2-domain scores) and their sum in warp order.
                    float lsum = 0.0f;
                    if ((int)threadIdx.x <= T) {
                        const float sk = sc[threadIdx.x];
                        const float pk = (mr == -INFINITY || sk == -INFINITY) ? 0.0f : exp2f(sk - mr);
                        sc[threadIdx.x] = pk;
                        lsum = pk;
                    }
                    lsum = warp_sum(lsum);
                    if (lane == 0) red[8 + warp] = lsum;
                    mk_consumer_sync();
                    // P V: this thread's dimension pair over key group kg
                    // (keys kg, kg + kKg, ...); zero weights are skipped
                    // (`ops.rs:1457`). Warps are uniform in their key.
                    {
                        const int dp = threadIdx.x % kPairs, kg = threadIdx.x / kPairs;
                        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 4
                        for (int k = kg; k < T; k += kKg) {
                            const float pk = sc[k];
                            if (pk != 0.0f) {
                                uint32_t w2;
                                asm volatile("ld.shared.u32 %0, [%1];"
                                             : "=r"(w2)
                                             : "r"(kvst_s + kTileBytes + mk_kv_off<HD>(k, (2 * dp) & ~7) +
                                                   (uint32_t)(((2 * dp) & 7) * 2)));
                                a0 = fmaf(pk, bf16_lo(w2), a0);
                                a1 = fmaf(pk, bf16_hi(w2), a1);
                            }
                        }
                        if (kg == 0) {
                            const float pk = sc[T];
                            if (pk != 0.0f) {
                                a0 = fmaf(pk, kvc[HD + 2 * dp], a0);
                                a1 = fmaf(pk, kvc[HD + 2 * dp + 1], a1);
                            }
                        }
                        opv[kg * HD + 2 * dp] = a0;
                        opv[kg * HD + 2 * dp + 1] = a1;
                    }
                    mk_consumer_sync();
                    // The staged sub-tile is read: stage the next one.
                    if (threadIdx.x == kWarp && rd + 1 < nsub) sh.kv_staged = stage(rd + 1);
                    if ((int)threadIdx.x < HD) {
                        float lr = 0.0f;
#pragma unroll
                        for (int w8 = 0; w8 < kMkConsumerWarps; ++w8) lr += red[8 + w8];
                        float o = 0.0f;
#pragma unroll
                        for (int g = 0; g < kKg; ++g) o += opv[g * HD + threadIdx.x];
                        const float m_new = fmaxf(run_m, mr);
                        if (m_new != -INFINITY) {
                            const float ca = run_m == -INFINITY ? 0.0f : exp2f(run_m - m_new);
                            const float cb = mr == -INFINITY ? 0.0f : exp2f(mr - m_new);
                            run_l = run_l * ca + lr * cb;
                            run_o = run_o * ca + o * cb;
                            run_m = m_new;
                        }
                    }
                    mk_consumer_sync();  // the scratch is reused by the next round
                }
                MK_TRACE(t, tb + 3);
                if (plan.splits == 1) {
                    if ((int)threadIdx.x < HD) ah[threadIdx.x] = run_l > 0.0f ? run_o / run_l : 0.0f;
                    // The head counter advances every layer (one arrival per
                    // unit), so its target is the same whatever the split count.
                    mk_arrive_relaxed(&ctrl[kMkCntHead + un.h]);
                } else {
                    // Key splits: the head's units exchange partials, and
                    // every unit merges them in split order.
                    if (kr.computes && (int)threadIdx.x < HD) {
                        float *part = p.att_part + ((size_t)un.h * p.att_part_units + un.u) * (2 + HD);
                        if (threadIdx.x == 0) {
                            part[0] = run_m;
                            part[1] = run_l;
                        }
                        part[2 + threadIdx.x] = run_o;
                    }
                    mk_arrive(&ctrl[kMkCntHead + un.h]);
                    mk_wait_count(&ctrl[kMkCntHead + un.h], (lg + 1) * (unsigned)un.U, sh, p.error, tmo);
                    if ((int)threadIdx.x < HD) {
                        // Every split's (m, l, o[d]) loaded at once, then
                        // combined in split order.
                        const int d = threadIdx.x;
                        float mm = -INFINITY, ll = 0.0f, oo = 0.0f;
                        constexpr int kJ = 16;
                        for (int j0 = 0; j0 < plan.splits; j0 += kJ) {
                            float mj[kJ], lj[kJ], oj[kJ];
#pragma unroll
                            for (int k = 0; k < kJ; ++k) {
                                const float *pj = p.att_part + ((size_t)un.h * p.att_part_units + j0 + k) * (2 + HD);
                                const bool in = j0 + k < plan.splits && !sh.abort;
                                mj[k] = in ? __ldcg(pj) : -INFINITY;
                                lj[k] = in ? __ldcg(pj + 1) : 0.0f;
                                oj[k] = in ? __ldcg(pj + 2 + d) : 0.0f;
                            }
#pragma unroll
                            for (int k = 0; k < kJ; ++k) {
                                if (mj[k] == -INFINITY) continue;
                                const float m_new = fmaxf(mm, mj[k]);
                                const float c_old = mm == -INFINITY ? 0.0f : exp2f(mm - m_new);
                                const float c_new = exp2f(mj[k] - m_new);
                                ll = fmaf(c_new, lj[k], ll * c_old);
                                oo = fmaf(c_new, oj[k], oo * c_old);
                                mm = m_new;
                            }
                        }
                        ah[d] = ll > 0.0f ? oo / ll : 0.0f;
                    }
                    mk_consumer_sync();
                }
                MK_TRACE(t, tb + 4);
                // o_proj rows of this unit: W_o[r, head] . o (8 lanes per row,
                // four rows per warp pass).
                for (int k = 0; k < tw.count(); ++k) {
                    const uint8_t *base = ring_c.acquire();
                    const int n = tw.hi(k) - tw.lo(k);
                    const int sub = lane >> 3, sl8 = lane & 7;
                    constexpr int kVec = HD / 64;  // 16-byte vectors per lane
                    for (int r0 = warp * 4; r0 < n; r0 += 4 * kMkConsumerWarps) {
                        const int r = r0 + sub;
                        float acc = 0.0f;
                        if (r < n) {
                            const uint4 *wr = reinterpret_cast<const uint4 *>(base + (size_t)r * HD * 2) + sl8 * kVec;
#pragma unroll
                            for (int u = 0; u < kVec; ++u) fma8(acc, wr[u], ah + (sl8 * kVec + u) * 8);
                        }
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 4);
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 2);
                        acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 1);
                        if (sl8 == 0 && r < n) p.opart[(size_t)un.h * H + tw.lo(k) + r] = acc;
                    }
                    ring_c.release();
                }
            }
            mk_arrive(&ctrl[kMkCntO]);
            MK_TRACE(t, tb + 5);

            // ---------------- GU ----------------
            // Every CTA forms the residual after o_proj for all rows (same
            // order everywhere): residual + head partials in head order +
            // o bias. hn keeps it for DOWN's residual add.
            MkV4 wln2{};
            if constexpr (SMALL) wln2 = mk_ld4<false>(w.ln2, H);
            mk_wait_count(&ctrl[kMkCntO], (lg + 1) * G, sh, p.error, tmo);
            MK_TRACE(t, tb + 6);
            {
                // kU elements per thread, each with its (1 + heads) loads,
                // all issued before any sum (16 heads per round).
                constexpr int kU = 4, kG = 16;
                for (int i0 = threadIdx.x; i0 < H; i0 += kU * kMkConsumers) {
                    float hv[kU], part[kU][kG];
                    for (int g0 = 0; g0 < p.q_heads; g0 += kG) {
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            const int i = i0 + u * kMkConsumers;
                            if (g0 == 0) hv[u] = i < H ? __ldcg(p.hidden + i) : 0.0f;
#pragma unroll
                            for (int k = 0; k < kG; ++k)
                                part[u][k] = (i < H && g0 + k < p.q_heads) ? __ldcg(p.opart + (size_t)(g0 + k) * H + i)
                                                                             : 0.0f;
                        }
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            float sv = 0.0f;
#pragma unroll
                            for (int k = 0; k < kG; ++k)
                                if (g0 + k < p.q_heads) sv = __fadd_rn(sv, part[u][k]);
                            // Head partials summed in head order, 16 at a time.
                            hv[u] = __fadd_rn(hv[u], sv);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        const int i = i0 + u * kMkConsumers;
                        if (i < H) hn[i] = w.bo ? __fadd_rn(hv[u], w.bo[i]) : hv[u];
                    }
                }
                mk_consumer_sync();
            }
            if constexpr (SMALL) {
                mk_rmsnorm4(mk_ld4<false>(hn, H), wln2, H, p.eps, xs, sh);
            } else {
                mk_rmsnorm_any<0>(hn, w.ln2, H, p.eps, xs, sh);
            }
            MK_TRACE(t, tb + 14);
            if (l == 0 && cta == 0 && threadIdx.x == 0) p.argmax_slots[t & 1] = 0ull;
            if constexpr (SMALL) xr.load(xs, H);
            for (int k = 0; k < tg.count(); ++k) {
                const uint8_t *base = ring_c.acquire();
                const int n = tg.hi(k) - tg.lo(k);
                for (int e = warp; e < n; e += kMkConsumerWarps) {
                    float g, u;
                    if constexpr (SMALL) {
                        const uint8_t *rows[2] = {base + (size_t)e * rs_h, base + (size_t)(tg.per_tile + e) * rs_h};
                        float r2[2];
                        mk_dotNr<XC, 2>(rows, xr, H, r2);
                        g = r2[0];
                        u = r2[1];
                    } else {
                        mk_dot2(base + (size_t)e * rs_h, base + (size_t)(tg.per_tile + e) * rs_h, xs, H, g, u);
                    }
                    if (lane == 0) p.act[tg.lo(k) + e] = silu_mul(g, u);
                }
                ring_c.release();
            }
            MK_TRACE(t, tb + 17);
            mk_arrive(&ctrl[kMkCntGu]);
            MK_TRACE(t, tb + 7);

            // ---------------- DOWN ----------------
            mk_wait_count(&ctrl[kMkCntGu], (lg + 1) * G, sh, p.error, tmo);
            MK_TRACE(t, tb + 8);
            mk_gather(xs, p.act, I);
            MK_TRACE(t, tb + 15);
            {
                // All of the phase's tiles at once when they fit the ring (a
                // warp per row across the tiles), else tile by tile.
                const int nt = td.count();
                const int batch = nt <= p.slots - 1 ? nt : 1;
                for (int k0 = 0; k0 < nt; k0 += batch) {
                    const int kn = min(batch, nt - k0);
                    const uint8_t *bases[8];
                    int rows_total = 0;
                    if (k0 == 0) MK_TRACE(t, tb + 29);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        bases[k] = k < kn ? ring_c.acquire(k) : nullptr;
                        if (k < kn) rows_total += td.hi(k0 + k) - td.lo(k0 + k);
                    }
                    if (k0 == 0) MK_TRACE(t, tb + 30);
                    for (int rr = warp; rr < rows_total; rr += kMkConsumerWarps) {
                        int k = 0, r = rr;
                        while (r >= td.hi(k0 + k) - td.lo(k0 + k)) {
                            r -= td.hi(k0 + k) - td.lo(k0 + k);
                            ++k;
                        }
                        const uint8_t *base = bases[0];
#pragma unroll
                        for (int kk = 1; kk < 8; ++kk)
                            if (kk == k) base = bases[kk];
                        const float acc = mk_dot_range(base + (size_t)r * rs_i, xs, 0, I / 8);
                        if (lane == 0) {
                            const int row = td.lo(k0 + k) + r;
                            p.hidden[row] = __fadd_rn(hn[row], acc);
                        }
                    }
                    ring_c.release(kn);
                }
            }
            MK_TRACE(t, tb + 18);
            mk_arrive(&ctrl[kMkCntDown]);
            MK_TRACE(t, tb + 9);
        }

        // ---------------- LM head + argmax ----------------
        MkV4 wfn{};
        if constexpr (SMALL) wfn = mk_ld4<false>(p.final_norm, H);
        mk_wait_count(&ctrl[kMkCntDown], (unsigned)(t * NL + NL) * G, sh, p.error, tmo);
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
                if constexpr (SMALL) {
                    const uint8_t *rows[2] = {base + (size_t)r * rs_h, base + (size_t)(two ? r2 : r) * rs_h};
                    float rr[2];
                    mk_dotNr<XC, 2>(rows, xr, H, rr);
                    a0 = rr[0];
                    a1 = rr[1];
                } else {
                    mk_dot2(base + (size_t)r * rs_h, base + (size_t)(two ? r2 : r) * rs_h, xs, H, a0, a1);
                }
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
        mk_bar_wait(smem_u32(&sh.kv_bar), (uint32_t)(sh.kv_uses - 1) & 1u, &sh.abort, false, tmo);
}

// Dynamic shared memory of the kernel for `slots` ring slots: 1024 bytes of
// alignment slack, the ring, xs (xcap floats), hn [hidden], ah [8][hd] and
// this step's K/V row [2][hd]. xcap covers the attention merge buffer and the
// DOWN partials after the activations.
inline int mk_xcap(int hidden, int inter, int hd) {
    return std::max({hidden, inter + 16, mk_att_scratch_floats(hd)});
}
inline size_t mk_smem_bytes(int slots, int xcap, int hidden, int hd) {
    return 1024 + (size_t)slots * kMkSlotBytes + 4 * ((size_t)xcap + hidden + 8 * (size_t)hd + 2 * (size_t)hd);
}

}  // namespace cheetah
