// libcheetah_cuda: the C-ABI backend (include/cheetah_cuda.h).
//
// Model: every unit of a prepared directory HBM-resident (QKV rows fused into
// one [q+2kv, hidden] matrix, norms/biases widened to f32), a rotary table
// built with the reference's own float math (`ops.rs:693-715`: powf, then
// position*freq, sinf/cosf) and a paged KV pool shared by all sequences.
// Sequence: page table + activations + one captured CUDA graph per sequence
// for the decode step (embed -> 24 x [qkv, attention, o_proj, gate/up, down]
// -> lm_head), launched with programmatic dependent launch so each kernel's
// weight stream starts while its predecessor drains.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "cheetah_cuda.h"
#include "attention.cuh"
#include "attention_mma.cuh"
#include "common.cuh"
#include "decode_megakernel.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"
#include "kernels_misc.cuh"
#include "quant.cuh"
#include "gemv_qmma.cuh"
#include "gemv_mma.cuh"
#include "gemm_tcgen05.cuh"
#include "prefill_attention.cuh"
#include "prefill_attention_tc.cuh"
#include "store.h"

namespace cheetah {

namespace {
thread_local std::string g_last_error;
}
void set_error(const std::string &message) { g_last_error = message; }
const char *last_error() { return g_last_error.c_str(); }

// Chained batched greedy steps run in chunks of at most this many steps
// between host reads of the token log.
constexpr int kChainSteps = 256;
constexpr int kBatchGemvRows = 8;  // padded batch rows up to which a batched step streams weights through GEMVs

namespace {

bool env_flag(const char *name, bool fallback) {
    const char *v = std::getenv(name);
    if (v == nullptr || v[0] == '\0') return fallback;
    return !(v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F');
}

int env_int(const char *name, int fallback) {
    const char *v = std::getenv(name);
    if (v == nullptr || v[0] == '\0') return fallback;
    const int x = std::atoi(v);
    return x > 0 ? x : fallback;
}

int sm_count(int device) {
    int count = 0;
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
    return count > 0 ? count : 148;
}

template <typename Kernel, typename... Args>
cudaError_t launch_ex(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      bool pdl, Args... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    config.attrs = attr;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, args...);
}

int pick_ksplit(int cols) {
    const int nvec = cols / 8;
    if (nvec <= 160) return 1;
    if (nvec <= 320) return 2;
    if (nvec <= 640) return 4;
    return 8;
}

template <int NB, int EPI, int KS, int WT>
int launch_gemv_ks(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    auto kernel = gemv_bf16_kernel<NB, EPI, KS, WT>;
    const size_t smem = (size_t)NB * p.cols * sizeof(float) + (size_t)kGemvWarps * 2 * NB * sizeof(float);
    if (smem > 48 * 1024) {
        CH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    int per_sm = 0;
    CH_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGemvThreads, smem));
    per_sm = std::max(1, std::min(per_sm, 4));
    const int groups_per_cta = kGemvWarps / KS;
    int groups;
    if (EPI == kEpiQkv) groups = p.rows / 2;
    else if (EPI == kEpiSwiglu) groups = p.rows;
    else groups = (p.rows + 1) / 2;
    const int needed = (groups + groups_per_cta - 1) / groups_per_cta;
    const int grid = std::max(1, std::min(needed, sms * per_sm));
    CH_CUDA_TRY(launch_ex(kernel, dim3(grid), dim3(kGemvThreads), smem, stream, pdl, p));
    return 0;
}

template <int NB, int EPI, int WT>
int launch_gemv_wt(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    const int elems = WT == kWBf16 ? 8 : (WT == kWQ8 ? 4 : 8);
    switch (pick_ksplit(p.cols / elems * 8)) {
    case 1: return launch_gemv_ks<NB, EPI, 1, WT>(p, stream, pdl, sms);
    case 2: return launch_gemv_ks<NB, EPI, 2, WT>(p, stream, pdl, sms);
    case 4: return launch_gemv_ks<NB, EPI, 4, WT>(p, stream, pdl, sms);
    default: return launch_gemv_ks<NB, EPI, 8, WT>(p, stream, pdl, sms);
    }
}

// Small-batch decode GEMV (<= 8 rows) on the tensor cores. Enough tiles for
// every warp of the GPU: a warp per tile. Otherwise a CTA per tile, its K
// range split over up to `max_tickets` CTAs (at least 16 steps of 32
// columns per split) until about two items per SM.
template <int EPI>
int launch_gemv_mma(GemvParams p, cudaStream_t stream, bool pdl, int sms, int max_tickets) {
    const int steps = p.cols / 32, tiles = gm_num_tiles(EPI, p.rows);
    const size_t smem = gemv_mma_smem(p.cols);
    const bool per_warp = tiles >= sms * kGmWarps / 2;
    auto kernel = per_warp ? gemv_mma_kernel<EPI, 1> : gemv_mma_kernel<EPI, kGmWarps>;
    if (smem > 48 * 1024) CH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    CH_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGmThreads, smem));
    per_sm = std::max(1, std::min(per_sm, 4));
    int items;
    if (per_warp) {
        p.splits = 1;
        items = (tiles + kGmWarps - 1) / kGmWarps;
    } else {
        int splits = 1;
        if (tiles <= max_tickets && p.split_ws != nullptr && p.split_tickets != nullptr)
            splits = std::max(1, std::min((2 * sms + tiles - 1) / tiles, steps / 16));
        p.splits = splits;
        items = tiles * splits;
    }
    const int grid = std::max(1, std::min(items, sms * per_sm));
    CH_CUDA_TRY(launch_ex(kernel, dim3(grid), dim3(kGmThreads), smem, stream, pdl, p));
    return 0;
}

template <int NB, int EPI>
int launch_gemv(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    if (p.wt == kWQ8) return launch_gemv_wt<NB, EPI, kWQ8>(p, stream, pdl, sms);
    if (p.wt == kWQ4) return launch_gemv_wt<NB, EPI, kWQ4>(p, stream, pdl, sms);
    return launch_gemv_wt<NB, EPI, kWBf16>(p, stream, pdl, sms);
}

// Launch plan of the bulk-prefetch GEMV for one weight shape; false when the
// shape needs the register-streaming kernel instead.
struct TmaGemvPlan {
    int ks = 1, nx = 4, slots = 2, chunk_bytes = 0;
    size_t smem = 0;
};

bool plan_tma_gemv(int epi, int rows, int cols, TmaGemvPlan *plan) {
    // Off by default: in the per-kernel decode graph the register-streaming
    // kernel is faster (measured 0.73 vs 0.85 ms per 0.5B token).
    if (!env_flag("CHEETAH_CUDA_TMA_GEMV", false)) return false;
    if (cols % 8 != 0 || rows <= 0) return false;
    const int nvec = cols / 8;
    for (int ks = 1; ks <= 8; ks *= 2) {
        const int rt = kTmaGemvWarps / ks;
        if (epi == kEpiQkv && rt % 2 != 0) continue;
        const int slice = (nvec + ks - 1) / ks;
        const int nx = (slice + kWarp - 1) / kWarp;
        if (nx > 8) continue;
        const int chunk = rt * cols * 2 * (epi == kEpiSwiglu ? 2 : 1);
        const int xs_bytes = cols * 4;
        const int budget = 100 * 1024 - xs_bytes;
        if (budget < 2 * chunk) return false;
        plan->ks = ks;
        plan->nx = nx <= 4 ? 4 : 8;
        plan->chunk_bytes = chunk;
        plan->slots = std::min(kTmaGemvMaxSlots, budget / chunk);
        plan->smem = (size_t)plan->slots * chunk + xs_bytes;
        return true;
    }
    return false;
}

template <int EPI, int KS, int NX>
int launch_tma_ks(const GemvParams &p, const TmaGemvPlan &plan, cudaStream_t stream, bool pdl, int sms) {
    auto kernel = gemv_tma_kernel<EPI, KS, NX>;
    CH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem));
    const int rt = kTmaGemvWarps / KS;
    const int chunks = (p.rows + rt - 1) / rt;
    const int grid = std::max(1, std::min(chunks, sms));
    CH_CUDA_TRY(launch_ex(kernel, dim3(grid), dim3(kTmaGemvThreads), plan.smem, stream, pdl, p, plan.slots,
                          plan.chunk_bytes));
    return 0;
}

template <int EPI>
int launch_tma_gemv(const GemvParams &p, const TmaGemvPlan &plan, cudaStream_t stream, bool pdl, int sms) {
    const int key = plan.ks * 16 + plan.nx;
    switch (key) {
    case 1 * 16 + 4: return launch_tma_ks<EPI, 1, 4>(p, plan, stream, pdl, sms);
    case 1 * 16 + 8: return launch_tma_ks<EPI, 1, 8>(p, plan, stream, pdl, sms);
    case 2 * 16 + 4: return launch_tma_ks<EPI, 2, 4>(p, plan, stream, pdl, sms);
    case 2 * 16 + 8: return launch_tma_ks<EPI, 2, 8>(p, plan, stream, pdl, sms);
    case 4 * 16 + 4: return launch_tma_ks<EPI, 4, 4>(p, plan, stream, pdl, sms);
    case 4 * 16 + 8: return launch_tma_ks<EPI, 4, 8>(p, plan, stream, pdl, sms);
    case 8 * 16 + 4: return launch_tma_ks<EPI, 8, 4>(p, plan, stream, pdl, sms);
    default: return launch_tma_ks<EPI, 8, 8>(p, plan, stream, pdl, sms);
    }
}

// Tensor-core q8/q4 GEMV: one input vector, dense 16-byte aligned code rows
// (q8: cols bytes, q4: cols / 2 bytes), widths a multiple of one 64-byte
// step, whole 16-row tiles.
bool qmma_eligible(int epi, const GemvParams &p) {
    if (!env_flag("CHEETAH_CUDA_QMMA", true)) return false;
    if (p.batch != 1 || (p.wt != kWQ8 && p.wt != kWQ4) || p.scale0 == nullptr || epi == kEpiLogits) return false;
    const int step = p.wt == kWQ8 ? 64 : 128;
    if (p.cols % step != 0 || p.cols > 48 * 1024) return false;
    if (p.row_stride != (p.wt == kWQ8 ? (long long)p.cols : (long long)p.cols / 2)) return false;
    if (((uintptr_t)p.w0 & 15) != 0 || (epi == kEpiSwiglu && ((uintptr_t)p.w1 & 15) != 0)) return false;
    if (epi == kEpiSwiglu ? p.rows % 8 != 0 : p.rows % 16 != 0) return false;
    if (epi == kEpiQkv && (p.head_dim / 2) % 8 != 0) return false;
    return true;
}

template <int EPI, int WT, int KS>
int launch_qmma_ks(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    auto kernel = gemv_qmma_kernel<EPI, WT, KS>;
    const size_t smem = (size_t)p.cols * 4 * (p.norm_w ? 2 : 1);
    if (smem > 48 * 1024)
        CH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    CH_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kQmThreads, smem));
    per_sm = std::max(1, std::min(per_sm, 4));
    const int tiles = qm_num_tiles(EPI, p.rows);
    const int per_cta = kQmWarps / KS;
    const int needed = (tiles + per_cta - 1) / per_cta;
    const int grid = std::max(1, std::min(needed, sms * per_sm));
    CH_CUDA_TRY(launch_ex(kernel, dim3(grid), dim3(kQmThreads), smem, stream, pdl, p));
    return 0;
}

// Warps per tile: enough warps in all (about 16 per SM) to keep HBM busy,
// at least two 64-byte steps per warp.
template <int EPI, int WT>
int launch_qmma(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    const int tiles = qm_num_tiles(EPI, p.rows);
    const int steps = p.cols / (WT == kWQ8 ? 64 : 128);
    int ks = 1;
    while (ks < 8 && tiles * ks < 16 * sms && steps >= 4 * ks) ks *= 2;
    switch (ks) {
    case 1: return launch_qmma_ks<EPI, WT, 1>(p, stream, pdl, sms);
    case 2: return launch_qmma_ks<EPI, WT, 2>(p, stream, pdl, sms);
    case 4: return launch_qmma_ks<EPI, WT, 4>(p, stream, pdl, sms);
    default: return launch_qmma_ks<EPI, WT, 8>(p, stream, pdl, sms);
    }
}

// Decode GEMV dispatch: the tensor-core kernel for q8/q4 shapes it covers,
// the bulk-prefetch kernel when its plan exists, the register-streaming
// kernel otherwise.
template <int EPI>
int run_gemv(const GemvParams &p, cudaStream_t stream, bool pdl, int sms) {
    if constexpr (EPI != kEpiLogits) {
        if (qmma_eligible(EPI, p))
            return p.wt == kWQ8 ? launch_qmma<EPI, kWQ8>(p, stream, pdl, sms) : launch_qmma<EPI, kWQ4>(p, stream, pdl, sms);
    }
    TmaGemvPlan plan;
    if (p.batch == 1 && p.wt == kWBf16 && plan_tma_gemv(EPI, p.rows, p.cols, &plan)) {
        return launch_tma_gemv<EPI>(p, plan, stream, pdl, sms);
    }
    return launch_gemv<1, EPI>(p, stream, pdl, sms);
}

int launch_attention(const AttnParams &p, int head_dim, bool kv_f32, cudaStream_t stream, bool pdl) {
    dim3 grid(p.splits, p.kv_heads, p.batch);
    cudaError_t err;
    if (head_dim == 64) {
        err = kv_f32 ? launch_ex(decode_attention_kernel<64, true>, grid, dim3(kAttnThreads), 0, stream, pdl, p)
                     : launch_ex(decode_attention_kernel<64, false>, grid, dim3(kAttnThreads), 0, stream, pdl, p);
    } else {
        err = kv_f32 ? launch_ex(decode_attention_kernel<128, true>, grid, dim3(kAttnThreads), 0, stream, pdl, p)
                     : launch_ex(decode_attention_kernel<128, false>, grid, dim3(kAttnThreads), 0, stream, pdl, p);
    }
    CH_CUDA_TRY(err);
    return 0;
}

int attention_splits(int batch, int kv_heads, int max_len, int sms) {
    const int target = std::max(1, (2 * sms) / std::max(1, batch * kv_heads));
    const int by_len = std::max(1, (max_len + kWarp - 1) / kWarp);
    return std::max(1, std::min(std::min(target, by_len), kMaxSplits));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
    });
    return fn;
}

// 2D map over a bf16 KV pool viewed as [rows][head_dim]: 64-column boxes of
// `tile_rows` rows, 128-byte swizzle (the layout the MMA kernel's ldmatrix
// addressing undoes).
int make_kv_tensor_map(CUtensorMap *map, const void *base, unsigned long long rows, int head_dim) {
    auto encode = tensor_map_encoder();
    CH_REQUIRE(encode != nullptr, "CUDA backend: cuTensorMapEncodeTiled is unavailable");
    CH_REQUIRE(((uintptr_t)base & 15) == 0, "CUDA backend: KV pool must be 16-byte aligned");
    const int tile_rows = kTileBytes / (head_dim * 2);
    cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)tile_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CH_REQUIRE(r == CUDA_SUCCESS, "CUDA backend: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return 0;
}

// 2D map over a bf16 row-major matrix [rows][cols]: 64-column x box_rows
// boxes, 128-byte swizzle (the K-major UMMA operand layout).
int make_bf16_tensor_map(CUtensorMap *map, const void *base, unsigned long long rows, unsigned long long cols,
                         int box_rows) {
    auto encode = tensor_map_encoder();
    CH_REQUIRE(encode != nullptr, "CUDA backend: cuTensorMapEncodeTiled is unavailable");
    CH_REQUIRE(((uintptr_t)base & 15) == 0 && (cols * 2) % 16 == 0, "CUDA backend: operand must be 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CH_REQUIRE(r == CUDA_SUCCESS, "CUDA backend: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return 0;
}

bool mma_attention_eligible(int head_dim, int page_tokens) {
    if (!env_flag("CHEETAH_CUDA_MMA_ATTENTION", true)) return false;
    if (head_dim != 64 && head_dim != 128) return false;
    return page_tokens % (kTileBytes / (head_dim * 2)) == 0;
}

int launch_attention_mma(const CUtensorMap &k_map, const CUtensorMap &v_map, const MmaAttnParams &mp,
                         int head_dim, cudaStream_t stream, bool pdl) {
    const size_t smem = mma_attention_smem();
    dim3 grid(mp.a.splits, mp.a.kv_heads, mp.a.batch);
    if (head_dim == 64) {
        CH_CUDA_TRY(cudaFuncSetAttribute(decode_attention_mma_kernel<64>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        CH_CUDA_TRY(launch_ex(decode_attention_mma_kernel<64>, grid, dim3(kMmaThreads), smem, stream, pdl,
                              k_map, v_map, mp));
    } else {
        CH_CUDA_TRY(cudaFuncSetAttribute(decode_attention_mma_kernel<128>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        CH_CUDA_TRY(launch_ex(decode_attention_mma_kernel<128>, grid, dim3(kMmaThreads), smem, stream, pdl,
                              k_map, v_map, mp));
    }
    return 0;
}

int mma_attention_splits(int batch, int kv_heads, int sms) {
    return std::max(1, std::min(kMaxSplits, sms / std::max(1, batch * kv_heads)));
}

// One linear's device weights: bf16 rows, or a q8/q4 buffer in the
// reference interchange layout (rows f32 scales, then the code rows).
struct QuantMatrix {
    const uint16_t *codes = nullptr;  // bf16 rows or code rows
    const float *scales = nullptr;    // nullptr for bf16
    long long row_stride = 0;         // bytes between rows
};

struct LayerWeights {
    const uint16_t *wqkv = nullptr;
    const uint16_t *wo = nullptr;
    const uint16_t *wgate = nullptr;
    const uint16_t *wup = nullptr;
    const uint16_t *wdown = nullptr;
    QuantMatrix qqkv, qo, qgate, qup, qdown;
    // Tensor maps of the bf16 linears for the prefill GEMMs.
    CUtensorMap map_qkv{}, map_o{}, map_gate{}, map_up{}, map_down{};
    const float *ln1 = nullptr;
    const float *ln2 = nullptr;
    const float *bqkv = nullptr;
    const float *bo = nullptr;
    // Per-head q/k RMSNorm weights (qwen3's `self_attn.{q,k}_norm`), f32 [head_dim].
    const float *q_norm = nullptr;
    const float *k_norm = nullptr;
    // Persistent decode kernel copies: QKV rows as all first rows of the
    // rotate-half pairs, then all partner rows (a tile of pairs is two
    // contiguous bulk copies); W_o as head-major [q_heads][hidden][head_dim]
    // blocks.
    const uint16_t *mk_qkv = nullptr;
    const uint16_t *mk_wo = nullptr;
};

// Ant residency of one streamable linear of a layer (the fused q/k/v
// matrix, o_proj, gate_proj, up_proj, down_proj) in a model opened with a
// residency plan. The pinned host copy is authoritative (as the reference's
// GPU backend keeps its host `WeightData`, `vulkan/transformer.rs:484-489`):
// a resident linear also has its own HBM allocation, a streamed one is copied
// into the layer's staging slot before every use.
struct LinearHome {
    uint8_t *dev = nullptr;     // HBM copy while resident
    uint8_t *host = nullptr;    // pinned host copy
    size_t bytes = 0;           // bf16 rows, or f32 row scales + code rows
    size_t codes_off = 0;       // code rows' offset in the buffer (q8/q4)
    size_t slot_off = 0;        // offset in a staging slot
    size_t rows = 0, cols = 0;  // logical shape
    int units = 1;              // reference units fused into the linear (q/k/v: 3)
    unsigned unit_bits = 1;     // units planned into HBM (all set: resident)
    bool resident = true;
};
constexpr int kHomeQkv = 0, kHomeO = 1, kHomeGate = 2, kHomeUp = 3, kHomeDown = 4, kHomes = 5;

}  // namespace

struct Seq;

// One single-token forward waiting to be folded into a batched step.
struct CoalescedCall {
    Seq *s = nullptr;
    uint32_t token = 0;
    size_t offset = 0;
    float *logits = nullptr;
    uint32_t *argmax = nullptr;
    int status = 0;
    std::string error;
    bool done = false;
};

struct Model {
    CheetahCudaConfig cfg{};
    int device = 0;
    int quant = 0;
    int sms = 148;
    bool pdl = true;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0;
    size_t arena_used = 0;
    std::vector<LayerWeights> layers;
    const uint16_t *embed = nullptr;
    const uint16_t *lm_head = nullptr;
    const float *final_norm = nullptr;
    float *rope_cos = nullptr;
    float *rope_sin = nullptr;
    uint8_t *k_pool = nullptr;
    uint8_t *v_pool = nullptr;
    long long page_bytes = 0;
    long long layer_stride_bytes = 0;
    int num_pages = 0;
    int page_tokens = 64;
    int kv_f32 = 0;
    bool use_mma_attention = false;
    bool qkv_interleaved = false;  // QKV rows stored pair-interleaved (bulk-prefetch GEMV)
    bool gemm_prefill = false;     // bf16 weights with tensor maps: tensor-core chunked prefill
    bool batch_gemv = false;       // batched steps of <= kBatchGemvRows rows run as weight-streaming GEMVs
    CUtensorMap map_lm_head{};
    // Persistent B=1 decode kernel (bf16 weights, bf16 KV): ring slots,
    // attention key chunks per head, dynamic shared memory, layer table.
    bool mk_enabled = false;
    // Per-head q/k RMSNorm units present (qwen3): the QKV epilogues normalise
    // each q and k head before RoPE; the persistent decode kernel is off.
    bool qk_norm = false;
    int mk_slots = 0;
    int mk_group_units = 1;  // attention units of a query head (CTAs per head, rounded up)
    size_t mk_smem = 0;
    size_t mk_copy_bytes = 0;  // arena bytes of the decode-kernel weight copies
    MkLayer *mk_layers = nullptr;
    // Ant VRAM tier (model opened with a residency plan): per layer, the
    // streamable linears' homes; two staging slots (layer parity) that
    // streamed linears are copied into before their layer runs. Planned
    // models run without graphs, PDL or the persistent kernel, and their
    // forwards are serialised (plan_mutex on the host, plan_event across
    // streams) because every stream shares the staging slots.
    bool planned = false;
    std::vector<std::array<LinearHome, kHomes>> homes;
    uint8_t *stage = nullptr;
    size_t stage_slot_bytes = 0;
    std::recursive_mutex plan_mutex;
    cudaEvent_t plan_event = nullptr;
    std::set<std::string> unit_ids;  // every unit of the prepared directory
    // Batched decode workspace (one batch at a time per model).
    std::mutex batch_mutex;
    int batch_cap = 0;
    int batch_table_cap = 0;
    cudaStream_t batch_stream = nullptr;
    int32_t *b_meta = nullptr;        // tokens[cap] | pos[cap] | lens[cap] | table[cap][table_cap]
    int32_t *h_meta = nullptr;        // pinned staging of b_meta
    float *b_hid = nullptr, *b_q = nullptr, *b_logits = nullptr;
    uint16_t *b_xb = nullptr, *b_ab = nullptr, *b_act = nullptr;
    // f32 attention output and SwiGLU activations of the small-batch GEMV step.
    float *b_attn_f32 = nullptr, *b_act_f32 = nullptr;
    float *b_qk_raw = nullptr;  // [cap][q + 2 kv dims] biased QKV rows (per-head q/k norm families)
    unsigned long long *b_argmax = nullptr, *h_argmax = nullptr;
    float *b_part_o = nullptr, *b_part_ml = nullptr;
    unsigned int *b_tickets = nullptr;
    // Split-K GEMM partial tiles (SMs x 128 x 128 f32) and tile tickets.
    float *b_split_ws = nullptr;
    unsigned *b_split_tickets = nullptr;
    int *b_error = nullptr;
    // Chained greedy steps: [0] live rows, [1] step index within the chunk;
    // token log [kChainSteps][cap] and its pinned host copy.
    int32_t *b_chain = nullptr, *h_chain = nullptr;  // h_chain: [0..1] chain state, [2] error word read-back
    int32_t *b_log = nullptr, *h_log = nullptr;
    CUtensorMap map_bxb{}, map_bab{}, map_bact{};
    std::map<uint64_t, cudaGraphExec_t> batch_graphs;  // (rows, table stride, logits, chained) -> captured step
    CUtensorMap k_map{};
    CUtensorMap v_map{};
    std::mutex pool_mutex;
    std::vector<int> free_pages;
    // Holders of each KV page (sequences and snapshots); 0 = free. A page
    // with more than one holder is never written: a sequence about to append
    // into one first takes a private copy (make_tail_page_private).
    std::vector<int> page_refs;
    std::atomic<int> refs{1};
    // Continuous batching behind the per-sequence forward: single-token
    // calls that arrive while a step runs are folded into the next one.
    std::mutex co_mutex;
    std::condition_variable co_cv;
    std::vector<CoalescedCall *> co_pending;
    bool co_running = false;
    size_t co_last_group = 0;  // calls in the previous group (how many callers are active)
    std::atomic<unsigned long long> co_calls{0}, co_batched_calls{0}, co_batches{0};

    void free_batch() {
        for (auto &kv : batch_graphs) cudaGraphExecDestroy(kv.second);
        batch_graphs.clear();
        cudaFree(b_meta);
        cudaFreeHost(h_meta);
        cudaFree(b_hid);
        cudaFree(b_q);
        cudaFree(b_logits);
        cudaFree(b_xb);
        cudaFree(b_ab);
        cudaFree(b_act);
        cudaFree(b_attn_f32);
        cudaFree(b_act_f32);
        cudaFree(b_qk_raw);
        b_attn_f32 = b_act_f32 = b_qk_raw = nullptr;
        cudaFree(b_argmax);
        cudaFreeHost(h_argmax);
        cudaFree(b_part_o);
        cudaFree(b_part_ml);
        cudaFree(b_tickets);
        cudaFree(b_split_ws);
        cudaFree(b_split_tickets);
        cudaFree(b_error);
        cudaFree(b_chain);
        cudaFreeHost(h_chain);
        cudaFree(b_log);
        cudaFreeHost(h_log);
        b_chain = h_chain = b_log = h_log = nullptr;
        b_meta = h_meta = nullptr;
        b_hid = b_q = b_logits = nullptr;
        b_xb = b_ab = b_act = nullptr;
        b_argmax = h_argmax = nullptr;
        b_part_o = b_part_ml = nullptr;
        b_tickets = nullptr;
        b_split_ws = nullptr;
        b_split_tickets = nullptr;
        b_error = nullptr;
        batch_cap = batch_table_cap = 0;
    }

    void *take(size_t bytes) {
        size_t offset = (arena_used + 255) & ~size_t(255);
        if (offset + bytes > arena_bytes) return nullptr;
        arena_used = offset + bytes;
        return arena + offset;
    }

    int alloc_page() {
        std::lock_guard<std::mutex> lock(pool_mutex);
        if (free_pages.empty()) return -1;
        int page = free_pages.back();
        free_pages.pop_back();
        page_refs[page] = 1;
        return page;
    }

    // Drops one hold on each page; a page nobody holds returns to the pool.
    void release_pages(std::vector<int> &pages) {
        std::lock_guard<std::mutex> lock(pool_mutex);
        for (int page : pages) {
            if (--page_refs[page] == 0) free_pages.push_back(page);
        }
        pages.clear();
    }

    void retain_pages(const std::vector<int> &pages) {
        std::lock_guard<std::mutex> lock(pool_mutex);
        for (int page : pages) ++page_refs[page];
    }

    int page_holders(int page) {
        std::lock_guard<std::mutex> lock(pool_mutex);
        return page_refs[page];
    }

    ~Model() {
        cudaSetDevice(device);
        free_batch();
        if (batch_stream) cudaStreamDestroy(batch_stream);
        cudaFree(arena);
        cudaFree(rope_cos);
        cudaFree(rope_sin);
        cudaFree(k_pool);
        cudaFree(v_pool);
        cudaFree(mk_layers);
        for (auto &layer : homes) {
            for (LinearHome &h : layer) {
                cudaFree(h.dev);
                cudaFreeHost(h.host);
            }
        }
        cudaFree(stage);
        if (plan_event) cudaEventDestroy(plan_event);
    }
};

void model_unref(Model *m) {
    if (m != nullptr && m->refs.fetch_sub(1) == 1) delete m;
}

// ---- Ant VRAM tier -----------------------------------------------------------
// Where linear `j` of `layer` is read from now: its own HBM copy while
// resident, the layer's staging slot (layer parity) while streamed. Sets the
// layer's pointers and, for models with tensor-core prefill operands,
// re-encodes the linear's tensor map.
int bind_linear(Model &m, uint32_t layer, int j, bool encode_map) {
    LinearHome &h = m.homes[layer][j];
    LayerWeights &w = m.layers[layer];
    uint8_t *base = h.resident ? h.dev : m.stage + (layer % 2) * m.stage_slot_bytes + h.slot_off;
    QuantMatrix *q[kHomes] = {&w.qqkv, &w.qo, &w.qgate, &w.qup, &w.qdown};
    const uint16_t **raw[kHomes] = {&w.wqkv, &w.wo, &w.wgate, &w.wup, &w.wdown};
    CUtensorMap *map[kHomes] = {&w.map_qkv, &w.map_o, &w.map_gate, &w.map_up, &w.map_down};
    if (m.quant == kWBf16) {
        q[j]->codes = reinterpret_cast<const uint16_t *>(base);
        q[j]->scales = nullptr;
    } else {
        q[j]->scales = reinterpret_cast<const float *>(base);
        q[j]->codes = reinterpret_cast<const uint16_t *>(base + h.codes_off);
    }
    *raw[j] = q[j]->codes;
    if (encode_map && m.quant == kWBf16)
        return make_bf16_tensor_map(map[j], q[j]->codes, (unsigned long long)h.rows, (unsigned long long)h.cols, 64);
    return 0;
}

// Copies the streamed linears of `layer` into its staging slot, in stream
// order before the layer's kernels (the slot's previous user, layer - 2,
// precedes them in the same stream).
int stage_layer(Model &m, uint32_t layer, cudaStream_t st) {
    if (!m.planned) return 0;
    for (int j = 0; j < kHomes; ++j) {
        const LinearHome &h = m.homes[layer][j];
        if (h.resident) continue;
        CH_CUDA_TRY(cudaMemcpyAsync(m.stage + (layer % 2) * m.stage_slot_bytes + h.slot_off, h.host, h.bytes,
                                    cudaMemcpyHostToDevice, st));
    }
    return 0;
}

// Serialises the forwards of a planned model: one host thread at a time
// enqueues, and each forward's device work starts after the previous one's
// (whatever stream that ran on), since all of them share the staging slots.
struct PlanGuard {
    Model &m;
    cudaStream_t st;
    bool on;
    PlanGuard(Model &model, cudaStream_t stream) : m(model), st(stream), on(model.planned) {
        if (!on) return;
        m.plan_mutex.lock();
        cudaStreamWaitEvent(st, m.plan_event, 0);
    }
    ~PlanGuard() {
        if (!on) return;
        cudaEventRecord(m.plan_event, st);
        m.plan_mutex.unlock();
    }
};

struct Seq {
    Model *m = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<int> pages;
    size_t positions = 0;
    int max_pages = 0;
    int32_t *page_table = nullptr;
    float *hidden = nullptr, *q = nullptr, *attn_out = nullptr, *act = nullptr, *logits = nullptr;
    float *qk_raw = nullptr;  // [q + 2 kv dims] biased QKV (per-head q/k norm families)
    unsigned long long *argmax = nullptr;
    StepState *d_step = nullptr;
    StepState *h_step = nullptr;
    float *h_logits = nullptr;
    unsigned long long *h_argmax = nullptr;
    int *h_error = nullptr;  // pinned copy of d_error, read with the step's results
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned int *tickets = nullptr;
    int *d_error = nullptr;
    int splits = 1;
    int mma_splits = 1;
    int scratch_splits = 1;
    int32_t *token_log = nullptr;
    // Chunked-prefill buffers (allocated on the first prompt): token ids,
    // f32 residual rows, bf16 normed / q / attention / SwiGLU rows.
    int chunk_cap = 0;
    int32_t *ptokens = nullptr;
    float *phid = nullptr;
    uint16_t *pxb = nullptr, *pqb = nullptr, *pab = nullptr, *pact = nullptr;
    float *ppart_o = nullptr, *ppart_ml = nullptr;  // prefill attention key-range splits
    float *psplit_ws = nullptr;                     // prefill split-K GEMM partial tiles
    unsigned *psplit_tickets = nullptr;
    CUtensorMap map_xb{}, map_ab{}, map_act{};
    CUtensorMap map_qb{};  // q rows in 128-row boxes (tensor-core prefill attention)
    cudaGraphExec_t graph = nullptr;
    cudaGraphExec_t chain_graph = nullptr;
    // Persistent decode kernel scratch (allocated on first use).
    float *mk_opart = nullptr, *mk_att_part = nullptr;
    unsigned *mk_ctrl = nullptr;
    unsigned long long *mk_argmax = nullptr;

    ~Seq() {
        cudaSetDevice(m->device);
        if (stream) cudaStreamSynchronize(stream);
        if (graph) cudaGraphExecDestroy(graph);
        if (chain_graph) cudaGraphExecDestroy(chain_graph);
        cudaFree(token_log);
        cudaFree(ptokens);
        cudaFree(phid);
        cudaFree(pxb);
        cudaFree(pqb);
        cudaFree(pab);
        cudaFree(pact);
        cudaFree(ppart_o);
        cudaFree(ppart_ml);
        cudaFree(psplit_ws);
        cudaFree(psplit_tickets);
        cudaFree(mk_opart);
        cudaFree(mk_att_part);
        cudaFree(mk_ctrl);
        cudaFree(mk_argmax);
        if (stream) cudaStreamDestroy(stream);
        cudaFree(page_table);
        cudaFree(hidden);
        cudaFree(q);
        cudaFree(qk_raw);
        cudaFree(attn_out);
        cudaFree(act);
        cudaFree(logits);
        cudaFree(argmax);
        cudaFree(d_step);
        cudaFree(part_o);
        cudaFree(part_ml);
        cudaFree(tickets);
        cudaFree(d_error);
        cudaFreeHost(h_step);
        cudaFreeHost(h_logits);
        cudaFreeHost(h_argmax);
        cudaFreeHost(h_error);
        m->release_pages(pages);
        model_unref(m);
    }
};

struct Snapshot {
    Model *m = nullptr;
    std::vector<int> pages;
    size_t positions = 0;
    ~Snapshot() {
        m->release_pages(pages);
        model_unref(m);
    }
};

namespace {

// Enqueue one decode step (B = 1) on the sequence stream.
// The persistent decode kernel instance for a model shape: head dim, and
// per-thread hidden-width slices in registers when hidden <= 1024.
using MkKernel = void (*)(const CUtensorMap, const CUtensorMap, const MkParams);
MkKernel mk_kernel_for(const CheetahCudaConfig &c) {
    const bool small = c.hidden_size <= 1024;
    if (c.head_dim == 64) return small ? decode_megakernel<64, true> : decode_megakernel<64, false>;
    return small ? decode_megakernel<128, true> : decode_megakernel<128, false>;
}

int ensure_mk_buffers(Seq &s) {
    if (s.mk_ctrl != nullptr) return 0;
    const Model &m = *s.m;
    const CheetahCudaConfig &c = m.cfg;
    const size_t parts = (size_t)c.q_heads * m.mk_group_units * (2 + c.head_dim);
    bool ok = cudaMalloc(&s.mk_opart, (size_t)c.q_heads * c.hidden_size * 4) == cudaSuccess &&
              cudaMalloc(&s.mk_att_part, parts * 4) == cudaSuccess &&
              cudaMalloc(&s.mk_ctrl, kMkCtrlWords * 4) == cudaSuccess &&
              cudaMalloc(&s.mk_argmax, 2 * 8) == cudaSuccess;
    if (!ok) {
        set_error("CUDA backend: decode kernel scratch allocation failed.");
        return -1;
    }
    // Stream-ordered before the kernel's first launch on this sequence
    // (a plain cudaMemset would run on the legacy stream, unordered with
    // the sequence's non-blocking stream).
    CH_CUDA_TRY(cudaMemsetAsync(s.mk_ctrl, 0, kMkCtrlWords * 4, s.stream));
    CH_CUDA_TRY(cudaMemsetAsync(s.mk_argmax, 0, 2 * 8, s.stream));
    CH_CUDA_TRY(cudaMemsetAsync(s.mk_att_part, 0, parts * 4, s.stream));
    CH_CUDA_TRY(cudaMemsetAsync(s.mk_opart, 0, (size_t)c.q_heads * c.hidden_size * 4, s.stream));
    return 0;
}

// One cooperative launch of the persistent decode kernel for `steps` greedy
// steps starting from s.d_step (token, position, optional page install).
int launch_megakernel(Seq &s, int steps, float *logits, int32_t *token_log) {
    Model &m = *s.m;
    const CheetahCudaConfig &c = m.cfg;
    MkParams p = {};
    p.layers = m.mk_layers;
    p.num_layers = (int)c.num_layers;
    p.H = (int)c.hidden_size;
    p.I = (int)c.intermediate_size;
    p.q_heads = (int)c.q_heads;
    p.kv_heads = (int)c.kv_heads;
    p.hd = (int)c.head_dim;
    p.vocab = (int)c.vocab_size;
    p.window = (int)c.sliding_window;
    p.slots = m.mk_slots;
    p.xcap = mk_xcap((int)c.hidden_size, (int)c.intermediate_size, (int)c.head_dim);
    p.inflight_layers = std::min(m.mk_slots, env_int("CHEETAH_MK_INFLIGHT", 1));
    p.inflight_lm = std::min(m.mk_slots, env_int("CHEETAH_MK_INFLIGHT_LM", 3));
    p.eps = c.rms_eps;
    p.scale_log2 = (1.0f / sqrtf((float)c.head_dim)) * 1.4426950408889634f;
    p.embed = m.embed;
    p.lm_head = m.lm_head;
    p.final_norm = m.final_norm;
    p.rope_cos = m.rope_cos;
    p.rope_sin = m.rope_sin;
    p.k_pool = m.k_pool;
    p.v_pool = m.v_pool;
    p.layer_stride_bytes = m.layer_stride_bytes;
    p.layer_rows = (long long)m.num_pages * c.kv_heads * m.page_tokens;
    p.num_pages = m.num_pages;
    p.page_tokens = m.page_tokens;
    p.max_pages = s.max_pages;
    p.page_table = s.page_table;
    p.step = s.d_step;
    p.steps = steps;
    p.hidden = s.hidden;
    p.q = s.q;
    p.opart = s.mk_opart;
    p.att_part_units = m.mk_group_units;
    p.act = s.act;
    p.att_part = s.mk_att_part;
    p.ctrl = s.mk_ctrl;
    p.argmax_slots = s.mk_argmax;
    p.argmax_out = s.argmax;
    p.token_log = token_log;
    p.logits = logits;
    p.error = s.d_error;
    // Every wait is bounded (2 s). CHEETAH_CUDA_TEST_STALL_WAIT=1 is a test
    // hook: the run's first attention wait targets a count nothing reaches,
    // with a 20 ms bound, to exercise the timeout path.
    p.stall_test = env_flag("CHEETAH_CUDA_TEST_STALL_WAIT", false) ? 1 : 0;
    p.timeout_ns = p.stall_test ? 20000000ull : 2000000000ull;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m.sms);
    cfg.blockDim = dim3(kMkThreads);
    cfg.dynamicSmemBytes = m.mk_smem;
    cfg.stream = s.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CH_CUDA_TRY(cudaLaunchKernelEx(&cfg, mk_kernel_for(c), m.k_map, m.v_map, p));
    return 0;
}

int enqueue_decode_step(Seq &s, bool chain) {
    Model &m = *s.m;
    if (m.mk_enabled && !chain) {
        if (ensure_mk_buffers(s) != 0) return -1;
        return launch_megakernel(s, 1, s.logits, nullptr);
    }
    const CheetahCudaConfig &c = m.cfg;
    const int hidden = c.hidden_size, inter = c.intermediate_size;
    const int q_dim = c.q_heads * c.head_dim, kv_dim = c.kv_heads * c.head_dim;
    const bool pdl = m.pdl;
    cudaStream_t st = s.stream;

    CH_CUDA_TRY(launch_ex(embed_kernel, dim3(1), dim3(256), 0, st, pdl, m.embed, hidden, s.d_step,
                          s.hidden, s.argmax, s.page_table, chain ? 1 : 0, s.token_log));
    const int32_t *positions = &s.d_step->position;
    const int32_t *seq_lens = &s.d_step->seq_len;

    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        if (stage_layer(m, layer, st) != 0) return -1;
        const LayerWeights &w = m.layers[layer];
        uint8_t *k_layer = m.k_pool + layer * m.layer_stride_bytes;
        uint8_t *v_layer = m.v_pool + layer * m.layer_stride_bytes;

        GemvParams qkv = {};
        qkv.w0 = w.wqkv;
        qkv.wt = m.quant;
        qkv.scale0 = w.qqkv.scales;
        qkv.row_stride = w.qqkv.row_stride;
        qkv.rows = q_dim + 2 * kv_dim;
        qkv.cols = hidden;
        qkv.batch = 1;
        qkv.x = s.hidden;
        qkv.x_stride = hidden;
        qkv.norm_w = w.ln1;
        qkv.eps = c.rms_eps;
        qkv.bias = w.bqkv;
        qkv.y = s.q;
        qkv.y_stride = q_dim;
        qkv.q_heads = c.q_heads;
        qkv.kv_heads = c.kv_heads;
        qkv.head_dim = c.head_dim;
        qkv.rope_cos = m.rope_cos;
        qkv.rope_sin = m.rope_sin;
        qkv.positions = positions;
        qkv.page_table = s.page_table;
        qkv.max_pages = s.max_pages;
        qkv.num_pages = m.num_pages;
        qkv.page_tokens = m.page_tokens;
        qkv.k_cache = k_layer;
        qkv.v_cache = v_layer;
        qkv.kv_f32 = m.kv_f32;
        if (m.qk_norm) qkv.qk_raw = s.qk_raw;
        if (run_gemv<kEpiQkv>(qkv, st, pdl, m.sms) != 0) return -1;
        if (m.qk_norm) {
            CH_CUDA_TRY(launch_ex(qk_norm_rope_kernel, dim3(c.q_heads + 2 * c.kv_heads, 1), dim3(32), 0, st, pdl,
                                  qkv, w.q_norm, w.k_norm));
        }

        AttnParams at = {};
        at.q = s.q;
        at.k_pool = k_layer;
        at.v_pool = v_layer;
        at.page_table = s.page_table;
        at.seq_lens = seq_lens;
        at.max_pages = s.max_pages;
        at.num_pages = m.num_pages;
        at.page_tokens = m.page_tokens;
        at.batch = 1;
        at.q_heads = c.q_heads;
        at.kv_heads = c.kv_heads;
        at.window = c.sliding_window;
        at.splits = s.splits;
        at.scale = 1.0f / sqrtf((float)c.head_dim);
        at.out = s.attn_out;
        at.part_o = s.part_o;
        at.part_ml = s.part_ml;
        at.tickets = s.tickets;
        at.error = s.d_error;
        if (m.use_mma_attention) {
            MmaAttnParams mp = {};
            mp.a = at;
            mp.a.splits = s.mma_splits;
            mp.layer_row_offset = (long long)layer * m.num_pages * c.kv_heads * m.page_tokens;
            mp.page_tokens = m.page_tokens;
            if (launch_attention_mma(m.k_map, m.v_map, mp, c.head_dim, st, pdl) != 0) return -1;
        } else if (launch_attention(at, c.head_dim, m.kv_f32 != 0, st, pdl) != 0) {
            return -1;
        }

        GemvParams o = {};
        o.w0 = w.wo;
        o.wt = m.quant;
        o.scale0 = w.qo.scales;
        o.row_stride = w.qo.row_stride;
        o.rows = hidden;
        o.cols = q_dim;
        o.batch = 1;
        o.x = s.attn_out;
        o.x_stride = q_dim;
        o.bias = w.bo;
        o.y = s.hidden;
        o.y_stride = hidden;
        if (run_gemv<kEpiResidual>(o, st, pdl, m.sms) != 0) return -1;

        GemvParams gu = {};
        gu.w0 = w.wgate;
        gu.w1 = w.wup;
        gu.wt = m.quant;
        gu.scale0 = w.qgate.scales;
        gu.scale1 = w.qup.scales;
        gu.row_stride = w.qgate.row_stride;
        gu.rows = inter;
        gu.cols = hidden;
        gu.batch = 1;
        gu.x = s.hidden;
        gu.x_stride = hidden;
        gu.norm_w = w.ln2;
        gu.eps = c.rms_eps;
        gu.y = s.act;
        gu.y_stride = inter;
        if (run_gemv<kEpiSwiglu>(gu, st, pdl, m.sms) != 0) return -1;

        GemvParams dn = {};
        dn.w0 = w.wdown;
        dn.wt = m.quant;
        dn.scale0 = w.qdown.scales;
        dn.row_stride = w.qdown.row_stride;
        dn.rows = hidden;
        dn.cols = inter;
        dn.batch = 1;
        dn.x = s.act;
        dn.x_stride = inter;
        dn.y = s.hidden;
        dn.y_stride = hidden;
        if (run_gemv<kEpiResidual>(dn, st, pdl, m.sms) != 0) return -1;
    }

    GemvParams lm = {};
    lm.w0 = m.lm_head;
    lm.rows = c.vocab_size;
    lm.cols = hidden;
    lm.batch = 1;
    lm.x = s.hidden;
    lm.x_stride = hidden;
    lm.norm_w = m.final_norm;
    lm.eps = c.rms_eps;
    lm.y = s.logits;
    lm.y_stride = c.vocab_size;
    lm.argmax = s.argmax;
    return run_gemv<kEpiLogits>(lm, st, pdl, m.sms);
}

// chain = false: per-token graph (step state copied from pinned host memory).
// chain = true: greedy-chain graph (step state advanced on the device).
int build_decode_graph(Seq &s, bool chain, cudaGraphExec_t *exec) {
    cudaGraph_t graph = nullptr;
    CH_CUDA_TRY(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t copy = chain ? cudaSuccess
                             : cudaMemcpyAsync(s.d_step, s.h_step, sizeof(StepState), cudaMemcpyHostToDevice, s.stream);
    int rc = copy == cudaSuccess ? enqueue_decode_step(s, chain) : -1;
    cudaError_t end = cudaStreamEndCapture(s.stream, &graph);
    if (copy != cudaSuccess) {
        set_error(std::string("step state copy failed: ") + cudaGetErrorString(copy));
        rc = -1;
    }
    if (rc != 0 || end != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        if (rc == 0) set_error(std::string("graph capture failed: ") + cudaGetErrorString(end));
        return -1;
    }
    cudaError_t inst = cudaGraphInstantiate(exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
        set_error(std::string("graph instantiate failed: ") + cudaGetErrorString(inst));
        *exec = nullptr;
        return -1;
    }
    return 0;
}

// Make sure the page holding `position` exists; fills the step's page fields.
int ensure_page(Seq &s, size_t position) {
    const size_t index = position / s.m->page_tokens;
    s.h_step->page_index = -1;
    s.h_step->page_id = -1;
    if (index < s.pages.size()) return 0;
    if ((int)index >= s.max_pages) {
        set_error("CUDA backend: position " + std::to_string(position) +
                  " exceeds the sequence capacity " + std::to_string(s.m->cfg.max_positions) + ".");
        return -1;
    }
    const int page = s.m->alloc_page();
    if (page < 0) {
        set_error("CUDA backend: KV page pool exhausted (raise kv_pool_tokens).");
        return -1;
    }
    s.pages.push_back(page);
    s.h_step->page_index = (int32_t)index;
    s.h_step->page_id = page;
    return 0;
}

int run_decode_step(Seq &s, uint32_t token, size_t position) {
    if (ensure_page(s, position) != 0) return -1;
    s.h_step->token = (int32_t)token;
    s.h_step->position = (int32_t)position;
    s.h_step->seq_len = (int32_t)(position + 1);
    if (s.m->mk_enabled) {
        // One cooperative launch per step, issued directly (no graph).
        CH_CUDA_TRY(cudaMemcpyAsync(s.d_step, s.h_step, sizeof(StepState), cudaMemcpyHostToDevice, s.stream));
        if (enqueue_decode_step(s, false) != 0) return -1;
        s.positions = position + 1;
        return 0;
    }
    if (s.graph == nullptr) {
        if (env_flag("CHEETAH_CUDA_GRAPH", true) && !s.m->planned) {
            if (build_decode_graph(s, false, &s.graph) != 0) return -1;
        }
    }
    if (s.graph != nullptr) {
        CH_CUDA_TRY(cudaGraphLaunch(s.graph, s.stream));
    } else {
        CH_CUDA_TRY(cudaMemcpyAsync(s.d_step, s.h_step, sizeof(StepState), cudaMemcpyHostToDevice, s.stream));
        if (enqueue_decode_step(s, false) != 0) return -1;
    }
    s.positions = position + 1;
    return 0;
}

// Host rotary table with the reference's float arithmetic (`ops.rs:693-715`).
void build_rope_table(int max_positions, int head_dim, float theta, std::vector<float> &cos_t,
                      std::vector<float> &sin_t) {
    const int half = head_dim / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i) {
        const float exponent = (-2.0f * (float)i) / (float)head_dim;
        freq[i] = powf(theta, exponent);
    }
    cos_t.resize((size_t)max_positions * half);
    sin_t.resize((size_t)max_positions * half);
    for (int pos = 0; pos < max_positions; ++pos) {
        for (int i = 0; i < half; ++i) {
            const volatile float angle = (float)pos * freq[i];
            cos_t[(size_t)pos * half + i] = cosf(angle);
            sin_t[(size_t)pos * half + i] = sinf(angle);
        }
    }
}

float bf16_bits_to_float(uint16_t bits) {
    uint32_t w = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &w, 4);
    return f;
}

// Tier of a unit in a residency plan ("vram" when the plan does not list it).
bool plan_in_vram(const std::map<std::string, std::string> *plan, const std::string &unit) {
    if (plan == nullptr) return true;
    auto it = plan->find(unit);
    return it == plan->end() || it->second == "vram";
}

int open_model(const char *prepared_dir, const CheetahCudaConfig *config, const char *quant,
               int device, Model **out, const std::map<std::string, std::string> *plan = nullptr) {
    CH_REQUIRE(prepared_dir != nullptr && config != nullptr && out != nullptr,
               "cheetah_cuda_model_open: null argument");
    const std::string q = quant ? quant : "bf16";
    CH_REQUIRE(q == "bf16" || q == "q8" || q == "q4",
               "Weight precision '" + q + "' has no CUDA operator table (expected bf16, q8 or q4).");
    const int wfmt = q == "q8" ? kWQ8 : (q == "q4" ? kWQ4 : kWBf16);
    CheetahCudaConfig c = *config;
    if (c.rotary_dim == 0) c.rotary_dim = c.head_dim;
    if (c.kv_page_tokens == 0) {
        const char *env = std::getenv("CHEETAH_CUDA_KV_PAGE");
        c.kv_page_tokens = env ? (uint32_t)std::atoi(env) : 64;
    }
    if (c.max_positions == 0) c.max_positions = 32768;
    CH_REQUIRE(c.head_dim == 64 || c.head_dim == 128, "CUDA backend: head_dim must be 64 or 128.");
    CH_REQUIRE(c.rotary_dim == c.head_dim, "CUDA backend: partial rotary is not supported.");
    CH_REQUIRE(c.kv_heads > 0 && c.q_heads % c.kv_heads == 0 && c.q_heads / c.kv_heads <= kMaxGroup,
               "CUDA backend: q_heads must be a multiple of kv_heads with at most 8 per group.");
    CH_REQUIRE(c.hidden_size % 8 == 0 && c.intermediate_size % 8 == 0 && (c.q_heads * c.head_dim) % 8 == 0,
               "CUDA backend: hidden/intermediate/q widths must be multiples of 8.");
    CH_REQUIRE(c.kv_page_tokens >= 16 && c.kv_page_tokens % 16 == 0,
               "CUDA backend: kv_page_tokens must be a positive multiple of 16.");
    CH_REQUIRE(c.kv_dtype == CHEETAH_CUDA_KV_BF16 || c.kv_dtype == CHEETAH_CUDA_KV_F32,
               "CUDA backend: unknown kv_dtype.");
    int count = 0;
    CH_CUDA_TRY(cudaGetDeviceCount(&count));
    CH_REQUIRE(device >= 0 && device < count, "CUDA backend: no such device " + std::to_string(device));
    CH_CUDA_TRY(cudaSetDevice(device));

    PreparedStore store;
    std::string error;
    if (!store.open(prepared_dir, &error)) {
        set_error(error);
        return -1;
    }

    Model *m = new Model();
    m->cfg = c;
    m->device = device;
    m->sms = sm_count(device);
    m->pdl = env_flag("CHEETAH_CUDA_PDL", true);
    m->page_tokens = (int)c.kv_page_tokens;
    m->kv_f32 = c.kv_dtype == CHEETAH_CUDA_KV_F32;
    m->quant = wfmt;
    m->planned = plan != nullptr;
    if (m->planned) {
        // Streamed layers put host copies between kernels: plain stream order.
        m->pdl = false;
        for (const auto &kv : *plan) {
            if (kv.second != "vram" && kv.second != "ram" && kv.second != "disk") {
                set_error("CUDA backend: unknown Ant tier '" + kv.second + "' for unit '" + kv.first +
                          "' (expected vram, ram or disk).");
                delete m;
                return -1;
            }
        }
    }
    for (const std::string &id : store.unit_ids()) m->unit_ids.insert(id);

    const size_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
    const size_t QD = (size_t)c.q_heads * c.head_dim, KD = (size_t)c.kv_heads * c.head_dim;
    auto fail = [&](const std::string &msg) {
        set_error(msg);
        delete m;
        return -1;
    };
    auto check_unit = [&](const std::string &id, std::vector<uint64_t> shape, const uint8_t **bytes) -> bool {
        const UnitRecord *rec = store.record(id);
        if (rec == nullptr) {
            error = "Native backend: unknown unit '" + id + "'.";
            return false;
        }
        if (rec->dtype != "BF16" && rec->dtype != "bf16") {
            error = "CUDA backend: unit '" + id + "' is " + rec->dtype + "; bf16 weights are required.";
            return false;
        }
        if (rec->shape != shape) {
            error = "CUDA backend: unit '" + id + "' has an unexpected shape.";
            return false;
        }
        *bytes = store.slice(id, &error);
        return *bytes != nullptr;
    };

    // Size the arena: layer linears (bf16, or q8/q4 buffers in the reference
    // layout), bf16 embedding / lm_head, f32 norms and biases.
    const bool tied = c.tie_word_embeddings != 0;
    size_t total = V * H * 2 + (tied ? 0 : V * H * 2) + H * 4 + 4096;
    auto linear_bytes = [&](size_t rows, size_t cols) -> size_t {
        if (wfmt == kWQ8) return rows * 4 + rows * (size_t)q8_row_bytes((long long)cols) + 256;
        if (wfmt == kWQ4) return rows * 4 + rows * (size_t)q4_row_bytes((long long)cols) + 256;
        return rows * cols * 2 + 256;
    };
    // Persistent decode kernel: bf16 weights and KV, a 4-pair QKV tile and a
    // down row fit a 32 KB slot, and at least three slots fit beside the
    // activation vectors in shared memory of a cooperative 1-CTA-per-SM grid.
    {
        int coop = 0, optin = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        const int xcap = mk_xcap((int)H, (int)I, (int)c.head_dim);
        const size_t fixed = mk_smem_bytes(0, xcap, (int)H, (int)c.head_dim);
        const size_t budget = optin > 4096 ? (size_t)optin - 4096 : 0;  // static shared state
        const int slots = budget > fixed ? (int)std::min<size_t>(kMkMaxSlots, (budget - fixed) / kMkSlotBytes) : 0;
        // The K/V tiles arrive by 128-byte-swizzled tensor-map loads (the bf16
        // cache's maps): pages a whole number of tiles; every query head
        // gets at least one attention unit.
        m->qk_norm = store.contains("model.layers.0.self_attn.q_norm.weight") ||
                     store.contains("model.layers.0.self_attn.k_norm.weight");
        m->mk_enabled = env_flag("CHEETAH_CUDA_MEGAKERNEL", true) && coop != 0 && wfmt == kWBf16 && !m->kv_f32 &&
                        !m->qk_norm && !m->planned &&
                        4 * H <= (size_t)kMkSlotBytes && 2 * I <= (size_t)kMkSlotBytes &&
                        c.q_heads <= (uint32_t)kMkMaxHeads && c.q_heads <= (uint32_t)m->sms &&
                        mma_attention_eligible((int)c.head_dim, m->page_tokens) && slots >= 3;
        if (m->mk_enabled) {
            m->mk_slots = slots;
            m->mk_smem = mk_smem_bytes(slots, xcap, (int)H, (int)c.head_dim);
            m->mk_group_units = (m->sms + (int)c.q_heads - 1) / (int)c.q_heads;
        }
    }
    // A planned model's linears live outside the arena (own HBM copies, or
    // host copies streamed through the staging slots).
    size_t per_layer = (m->planned ? 0
                                   : linear_bytes(QD + 2 * KD, H) + linear_bytes(H, QD) + 2 * linear_bytes(I, H) +
                                         linear_bytes(H, I)) +
                       (2 * H + (QD + 2 * KD) + H) * 4 + 8 * 256;
    if (m->mk_enabled) per_layer += H * QD * 2 + (QD + 2 * KD) * H * 2 + 2 * 256;
    total += per_layer * c.num_layers;
    cudaError_t err = cudaMalloc(&m->arena, total);
    if (err != cudaSuccess) return fail(std::string("CUDA backend: weight allocation failed: ") + cudaGetErrorString(err));
    m->arena_bytes = total;

    auto upload = [&](void *dst, const void *src, size_t bytes) -> bool {
        cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            error = std::string("CUDA backend: weight upload failed: ") + cudaGetErrorString(e);
            return false;
        }
        return true;
    };
    auto upload_f32_from_bf16 = [&](float *dst, const uint8_t *src, size_t n) -> bool {
        std::vector<float> tmp(n);
        for (size_t i = 0; i < n; ++i) {
            uint16_t bits;
            memcpy(&bits, src + 2 * i, 2);
            tmp[i] = bf16_bits_to_float(bits);
        }
        return upload(dst, tmp.data(), n * 4);
    };

    const uint8_t *bytes = nullptr;
    if (!check_unit("model.embed_tokens.weight", {V, H}, &bytes)) return fail(error);
    uint16_t *embed = (uint16_t *)m->take(V * H * 2);
    if (!upload(embed, bytes, V * H * 2)) return fail(error);
    m->embed = embed;
    if (tied) {
        m->lm_head = embed;
    } else {
        if (!check_unit("lm_head.weight", {V, H}, &bytes)) {
            return fail("Native backend: neither tied embeddings nor a separate 'lm_head.weight' tensor are present.");
        }
        uint16_t *head = (uint16_t *)m->take(V * H * 2);
        if (!upload(head, bytes, V * H * 2)) return fail(error);
        m->lm_head = head;
    }
    if (!check_unit("model.norm.weight", {H}, &bytes)) return fail(error);
    float *fn = (float *)m->take(H * 4);
    if (!upload_f32_from_bf16(fn, bytes, H)) return fail(error);
    m->final_norm = fn;

    {
        TmaGemvPlan plan;
        m->qkv_interleaved = wfmt == kWBf16 && plan_tma_gemv(kEpiQkv, (int)(QD + 2 * KD), (int)H, &plan);
    }
    // Quantised formats stage each bf16 matrix on the device once and
    // quantise it there into the arena (bit-identical to the reference's
    // load-time quantisation, `ops.rs:1199-1226`).
    uint16_t *staging = nullptr;
    if (wfmt != kWBf16) {
        const size_t max_elems = std::max(std::max((QD + 2 * KD) * H, H * QD), std::max(I * H, H * I));
        if (cudaMalloc(&staging, max_elems * 2) != cudaSuccess) return fail("CUDA backend: staging allocation failed");
    }
    // Planned models: quantised buffers are built in a device scratch buffer,
    // then copied to the pinned host copy (and to an own HBM copy when the
    // linear is resident).
    uint8_t *qtmp = nullptr;
    if (m->planned && wfmt != kWBf16) {
        const size_t max_elems = std::max(std::max((QD + 2 * KD) * H, H * QD), std::max(I * H, H * I));
        if (cudaMalloc(&qtmp, max_elems + 8 * std::max(std::max(QD + 2 * KD, H), I) + 4096) != cudaSuccess)
            return fail("CUDA backend: quantisation scratch allocation failed");
    }
    auto place_home = [&](const uint16_t *host, size_t rows, size_t cols, QuantMatrix *out, LinearHome *home) -> bool {
        home->rows = rows;
        home->cols = cols;
        const uint8_t *src_dev = nullptr;  // device bytes to copy from (quantised formats)
        if (wfmt == kWBf16) {
            home->bytes = rows * cols * 2;
            home->codes_off = 0;
            out->row_stride = (long long)cols * 2;
        } else {
            if (!upload(staging, host, rows * cols * 2)) return false;
            long long rb = wfmt == kWQ8 ? q8_row_bytes((long long)cols) : q4_row_bytes((long long)cols);
            if (wfmt == kWQ4 && cols % 128 == 0) rb = (long long)cols / 2;
            const int blocks = (int)((rows * kWarp + 255) / 256);
            if (wfmt == kWQ8) quantize_rows_kernel<8><<<blocks, 256>>>(staging, (int)rows, (int)cols, qtmp, rb);
            else quantize_rows_kernel<4><<<blocks, 256>>>(staging, (int)rows, (int)cols, qtmp, rb);
            home->bytes = rows * 4 + rows * (size_t)rb;
            home->codes_off = rows * 4;
            out->row_stride = rb;
            src_dev = qtmp;
        }
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(&home->host), home->bytes, cudaHostAllocDefault);
        if (e == cudaSuccess) {
            if (src_dev) e = cudaMemcpy(home->host, src_dev, home->bytes, cudaMemcpyDeviceToHost);
            else memcpy(home->host, host, home->bytes);
        }
        if (e == cudaSuccess && home->resident) {
            e = cudaMalloc(reinterpret_cast<void **>(&home->dev), home->bytes);
            if (e == cudaSuccess)
                e = cudaMemcpy(home->dev, src_dev ? (const void *)src_dev : (const void *)home->host, home->bytes,
                               src_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) {
            error = std::string("CUDA backend: Ant residency placement failed: ") + cudaGetErrorString(e);
            return false;
        }
        return true;
    };
    auto place_linear = [&](const uint16_t *host, size_t rows, size_t cols, QuantMatrix *out,
                            LinearHome *home = nullptr) -> bool {
        if (home != nullptr) return place_home(host, rows, cols, out, home);
        if (wfmt == kWBf16) {
            uint16_t *dst = (uint16_t *)m->take(rows * cols * 2);
            if (!upload(dst, host, rows * cols * 2)) return false;
            out->codes = dst;
            out->scales = nullptr;
            out->row_stride = (long long)cols * 2;
            return true;
        }
        if (!upload(staging, host, rows * cols * 2)) return false;
        // q4 rows whose width is a multiple of 128 are stored cols / 2 bytes
        // apart (16-byte aligned for the tensor-core GEMV) instead of the
        // reference's padded row size; the codes and scales are the same.
        long long rb = wfmt == kWQ8 ? q8_row_bytes((long long)cols) : q4_row_bytes((long long)cols);
        if (wfmt == kWQ4 && cols % 128 == 0) rb = (long long)cols / 2;
        uint8_t *buf = (uint8_t *)m->take(rows * 4 + rows * (size_t)rb);
        const int blocks = (int)((rows * kWarp + 255) / 256);
        if (wfmt == kWQ8) quantize_rows_kernel<8><<<blocks, 256>>>(staging, (int)rows, (int)cols, buf, rb);
        else quantize_rows_kernel<4><<<blocks, 256>>>(staging, (int)rows, (int)cols, buf, rb);
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            error = std::string("CUDA backend: quantisation failed: ") + cudaGetErrorString(e);
            return false;
        }
        out->codes = reinterpret_cast<const uint16_t *>(buf + rows * 4);
        out->scales = reinterpret_cast<const float *>(buf);
        out->row_stride = rb;
        return true;
    };
    // Device copy of host rows for the persistent decode kernel.
    auto place_copy = [&](const void *src, size_t rows, size_t cols, const uint16_t **out) -> bool {
        uint8_t *dst = (uint8_t *)m->take(rows * cols * 2);
        if (dst == nullptr) {
            error = "CUDA backend: decode kernel weight arena exhausted";
            return false;
        }
        if (!upload(dst, src, rows * cols * 2)) return false;
        m->mk_copy_bytes += rows * cols * 2;
        *out = reinterpret_cast<const uint16_t *>(dst);
        return true;
    };
    m->layers.resize(c.num_layers);
    // Residency of each streamable linear: resident when every reference
    // unit fused into it is planned into HBM ("vram" or absent from the plan).
    static const char *kHomeUnits[kHomes][3] = {
        {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"},
        {"self_attn.o_proj.weight", nullptr, nullptr},
        {"mlp.gate_proj.weight", nullptr, nullptr},
        {"mlp.up_proj.weight", nullptr, nullptr},
        {"mlp.down_proj.weight", nullptr, nullptr}};
    if (m->planned) {
        m->homes.resize(c.num_layers);
        for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
            const std::string p = "model.layers." + std::to_string(layer) + ".";
            for (int j = 0; j < kHomes; ++j) {
                LinearHome &h = m->homes[layer][j];
                h.units = j == kHomeQkv ? 3 : 1;
                h.unit_bits = 0;
                for (int u = 0; u < h.units; ++u)
                    if (plan_in_vram(plan, p + kHomeUnits[j][u])) h.unit_bits |= 1u << u;
                h.resident = h.unit_bits == (1u << h.units) - 1;
            }
        }
    }
    auto home = [&](uint32_t layer, int j) -> LinearHome * {
        return m->planned ? &m->homes[layer][j] : nullptr;
    };
    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        const std::string p = "model.layers." + std::to_string(layer) + ".";
        LayerWeights &w = m->layers[layer];
        {
            // Host staging of [q; k; v]; for the bulk-prefetch kernel the rows
            // are pair-interleaved per head (storage rows 2i, 2i+1 = logical
            // rows i, i + d/2).
            std::vector<uint16_t> staged((QD + 2 * KD) * H);
            const char *names[3] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"};
            const size_t rows_of[3] = {QD, KD, KD};
            size_t row0 = 0;
            for (int k = 0; k < 3; ++k) {
                if (!check_unit(p + names[k], {rows_of[k], H}, &bytes)) return fail(error);
                memcpy(staged.data() + row0 * H, bytes, rows_of[k] * H * 2);
                row0 += rows_of[k];
            }
            if (m->mk_enabled) {
                // Pair order: first rows (head * d + i, i < d/2) of every
                // head, then the partners (+ d/2).
                const size_t hd = c.head_dim, half = hd / 2, pairs = (QD + 2 * KD) / 2;
                std::vector<uint16_t> order(staged.size());
                for (size_t i = 0; i < pairs; ++i) {
                    const size_t row = (i / half) * hd + (i % half);
                    memcpy(order.data() + i * H, staged.data() + row * H, H * 2);
                    memcpy(order.data() + (pairs + i) * H, staged.data() + (row + half) * H, H * 2);
                }
                if (!place_copy(order.data(), QD + 2 * KD, H, &w.mk_qkv)) return fail(error);
            }
            if (m->qkv_interleaved) {
                const size_t hd = c.head_dim, half = hd / 2, heads = (QD + 2 * KD) / hd;
                std::vector<uint16_t> perm(staged.size());
                for (size_t h = 0; h < heads; ++h) {
                    for (size_t i = 0; i < half; ++i) {
                        memcpy(perm.data() + (h * hd + 2 * i) * H, staged.data() + (h * hd + i) * H, H * 2);
                        memcpy(perm.data() + (h * hd + 2 * i + 1) * H, staged.data() + (h * hd + i + half) * H, H * 2);
                    }
                }
                staged.swap(perm);
            }
            if (!place_linear(staged.data(), QD + 2 * KD, H, &w.qqkv, home(layer, kHomeQkv))) return fail(error);
        }
        if (!check_unit(p + "self_attn.o_proj.weight", {H, QD}, &bytes) ||
            !place_linear((const uint16_t *)bytes, H, QD, &w.qo, home(layer, kHomeO))) return fail(error);
        if (m->mk_enabled) {
            // W_o[:, head] blocks, head-major: [q_heads][H][head_dim].
            const size_t hd = c.head_dim;
            std::vector<uint16_t> heads_major(H * QD);
            const uint16_t *src = (const uint16_t *)bytes;
            for (size_t h = 0; h < c.q_heads; ++h)
                for (size_t r = 0; r < H; ++r)
                    memcpy(heads_major.data() + (h * H + r) * hd, src + r * QD + h * hd, hd * 2);
            uint16_t *dst = (uint16_t *)m->take(heads_major.size() * 2);
            if (dst == nullptr || !upload(dst, heads_major.data(), heads_major.size() * 2))
                return fail("CUDA backend: decode kernel weight upload failed");
            w.mk_wo = dst;
            m->mk_copy_bytes += heads_major.size() * 2;
        }
        if (!check_unit(p + "mlp.gate_proj.weight", {I, H}, &bytes) ||
            !place_linear((const uint16_t *)bytes, I, H, &w.qgate, home(layer, kHomeGate))) return fail(error);
        if (!check_unit(p + "mlp.up_proj.weight", {I, H}, &bytes) ||
            !place_linear((const uint16_t *)bytes, I, H, &w.qup, home(layer, kHomeUp))) return fail(error);
        if (!check_unit(p + "mlp.down_proj.weight", {H, I}, &bytes) ||
            !place_linear((const uint16_t *)bytes, H, I, &w.qdown, home(layer, kHomeDown))) return fail(error);
        w.wqkv = w.qqkv.codes;
        w.wo = w.qo.codes;
        w.wgate = w.qgate.codes;
        w.wup = w.qup.codes;
        w.wdown = w.qdown.codes;
        float *ln1 = (float *)m->take(H * 4);
        if (!check_unit(p + "input_layernorm.weight", {H}, &bytes) || !upload_f32_from_bf16(ln1, bytes, H)) return fail(error);
        w.ln1 = ln1;
        float *ln2 = (float *)m->take(H * 4);
        if (!check_unit(p + "post_attention_layernorm.weight", {H}, &bytes) || !upload_f32_from_bf16(ln2, bytes, H)) return fail(error);
        w.ln2 = ln2;
        // Biases are unit-optional (`ops.rs:1156-1166`); absent ones add zero.
        const bool has_qkv_bias = store.contains(p + "self_attn.q_proj.bias") ||
                                  store.contains(p + "self_attn.k_proj.bias") ||
                                  store.contains(p + "self_attn.v_proj.bias");
        if (has_qkv_bias) {
            std::vector<float> b(QD + 2 * KD, 0.0f);
            const char *names[3] = {"self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"};
            const size_t offs[3] = {0, QD, QD + KD};
            const size_t lens[3] = {QD, KD, KD};
            for (int k = 0; k < 3; ++k) {
                if (!store.contains(p + names[k])) continue;
                if (!check_unit(p + names[k], {lens[k]}, &bytes)) return fail(error);
                for (size_t i = 0; i < lens[k]; ++i) {
                    uint16_t bits;
                    memcpy(&bits, bytes + 2 * i, 2);
                    b[offs[k] + i] = bf16_bits_to_float(bits);
                }
            }
            float *bq = (float *)m->take(b.size() * 4);
            if (!upload(bq, b.data(), b.size() * 4)) return fail(error);
            w.bqkv = bq;
        }
        if (store.contains(p + "self_attn.o_proj.bias")) {
            if (!check_unit(p + "self_attn.o_proj.bias", {H}, &bytes)) return fail(error);
            float *bo = (float *)m->take(H * 4);
            if (!upload_f32_from_bf16(bo, bytes, H)) return fail(error);
            w.bo = bo;
        }
        // Per-head q/k norms are unit-optional as well (`ops.rs:1130-1152`).
        const char *norm_names[2] = {"self_attn.q_norm.weight", "self_attn.k_norm.weight"};
        const float **norm_dst[2] = {&w.q_norm, &w.k_norm};
        for (int k = 0; k < 2; ++k) {
            if (!store.contains(p + norm_names[k])) continue;
            if (!m->qk_norm) return fail("CUDA backend: per-head q/k norms must start at layer 0");
            if (!check_unit(p + norm_names[k], {(size_t)c.head_dim}, &bytes)) return fail(error);
            float *nw = (float *)m->take((size_t)c.head_dim * 4);
            if (!upload_f32_from_bf16(nw, bytes, c.head_dim)) return fail(error);
            *norm_dst[k] = nw;
        }
    }

    cudaFree(staging);
    cudaFree(qtmp);

    if (m->planned) {
        // Staging slots: every streamable linear of a layer at a fixed
        // offset, two slots (layer parity).
        size_t off = 0;
        for (int j = 0; j < kHomes; ++j) {
            const size_t slot_off = off;
            for (auto &layer : m->homes) layer[j].slot_off = slot_off;
            off += (m->homes[0][j].bytes + 255) & ~size_t(255);
        }
        m->stage_slot_bytes = off;
        cudaError_t e = cudaMalloc(&m->stage, 2 * off);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->plan_event, cudaEventDisableTiming);
        if (e != cudaSuccess) return fail(std::string("CUDA backend: Ant staging allocation failed: ") + cudaGetErrorString(e));
        for (uint32_t layer = 0; layer < c.num_layers; ++layer)
            for (int j = 0; j < kHomes; ++j) bind_linear(*m, layer, j, false);
    }

    if (m->mk_enabled) {
        std::vector<MkLayer> table(c.num_layers);
        for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
            const LayerWeights &w = m->layers[layer];
            table[layer] = MkLayer{w.mk_qkv, w.bqkv, w.mk_wo, w.bo, w.wgate, w.wup, w.wdown, w.ln1, w.ln2};
        }
        cudaError_t e = cudaMalloc(&m->mk_layers, table.size() * sizeof(MkLayer));
        if (e == cudaSuccess) e = cudaMemcpy(m->mk_layers, table.data(), table.size() * sizeof(MkLayer), cudaMemcpyHostToDevice);
        const MkKernel kernel = mk_kernel_for(c);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->mk_smem);
        int per_sm = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kMkThreads, m->mk_smem);
        if (e != cudaSuccess) return fail(std::string("CUDA backend: decode kernel setup failed: ") + cudaGetErrorString(e));
        if (per_sm < 1) m->mk_enabled = false;  // the multi-kernel decode path runs instead
    }

    // Prefill GEMM operands (bf16 models with the standard QKV row order).
    bool weight_maps_ok = false;
    if (wfmt == kWBf16 && !m->qkv_interleaved && env_flag("CHEETAH_CUDA_GEMM_PREFILL", true)) {
        bool ok = true;
        for (uint32_t layer = 0; layer < c.num_layers && ok; ++layer) {
            LayerWeights &w = m->layers[layer];
            ok = make_bf16_tensor_map(&w.map_qkv, w.wqkv, QD + 2 * KD, H, 64) == 0 &&
                 make_bf16_tensor_map(&w.map_o, w.wo, H, QD, 64) == 0 &&
                 make_bf16_tensor_map(&w.map_gate, w.wgate, I, H, 64) == 0 &&
                 make_bf16_tensor_map(&w.map_up, w.wup, I, H, 64) == 0 &&
                 make_bf16_tensor_map(&w.map_down, w.wdown, H, I, 64) == 0;
        }
        if (!ok) {
            delete m;
            return -1;
        }
        ok = ok && make_bf16_tensor_map(&m->map_lm_head, m->lm_head, V, H, 64) == 0;
        if (!ok) {
            delete m;
            return -1;
        }
        weight_maps_ok = true;
    }

    // Rotary table.
    std::vector<float> cos_t, sin_t;
    build_rope_table((int)c.max_positions, (int)c.head_dim, c.rope_theta, cos_t, sin_t);
    if (cudaMalloc(&m->rope_cos, cos_t.size() * 4) != cudaSuccess ||
        cudaMalloc(&m->rope_sin, sin_t.size() * 4) != cudaSuccess ||
        !upload(m->rope_cos, cos_t.data(), cos_t.size() * 4) ||
        !upload(m->rope_sin, sin_t.data(), sin_t.size() * 4)) {
        return fail(error.empty() ? "CUDA backend: rotary table allocation failed" : error);
    }

    // KV pool.
    uint32_t pool_tokens = c.kv_pool_tokens ? c.kv_pool_tokens : std::max<uint32_t>(c.max_positions, 65536);
    m->num_pages = (int)((pool_tokens + m->page_tokens - 1) / m->page_tokens);
    const size_t elem = m->kv_f32 ? 4 : 2;
    m->page_bytes = (long long)c.kv_heads * m->page_tokens * c.head_dim * elem;
    m->layer_stride_bytes = m->page_bytes * m->num_pages;
    const size_t pool_bytes = (size_t)m->layer_stride_bytes * c.num_layers;
    if (cudaMalloc(&m->k_pool, pool_bytes) != cudaSuccess || cudaMalloc(&m->v_pool, pool_bytes) != cudaSuccess) {
        return fail("CUDA backend: KV pool allocation failed (" + std::to_string(pool_bytes * 2) + " bytes).");
    }
    cudaMemset(m->k_pool, 0, pool_bytes);
    cudaMemset(m->v_pool, 0, pool_bytes);
    if (!m->kv_f32 && mma_attention_eligible((int)c.head_dim, m->page_tokens)) {
        const unsigned long long rows = (unsigned long long)c.num_layers * m->num_pages * c.kv_heads * m->page_tokens;
        if (make_kv_tensor_map(&m->k_map, m->k_pool, rows, (int)c.head_dim) != 0 ||
            make_kv_tensor_map(&m->v_map, m->v_pool, rows, (int)c.head_dim) != 0) {
            delete m;
            return -1;
        }
        m->use_mma_attention = true;
    }
    // Tensor-core chunked prefill needs the bf16 weight maps and the bf16 KV maps.
    // Vectorised epilogues: residual widths in 32-column groups, SwiGLU in 16.
    m->gemm_prefill = weight_maps_ok && m->use_mma_attention && (c.head_dim == 64 || c.head_dim == 128) &&
                      c.hidden_size % 32 == 0 && c.intermediate_size % 16 == 0;
    // Small batches: every weight byte streamed once per step by GEMVs over
    // all SMs (tensor-core tiles would put a few dozen CTAs on the weights).
    m->batch_gemv = m->gemm_prefill && !m->qkv_interleaved && env_flag("CHEETAH_CUDA_BATCH_GEMV", true) &&
                    H % 32 == 0 && I % 32 == 0 && QD % 32 == 0 && ((QD + 2 * KD) / 2) % 8 == 0;
    m->free_pages.reserve(m->num_pages);
    for (int i = m->num_pages - 1; i >= 0; --i) m->free_pages.push_back(i);
    m->page_refs.assign(m->num_pages, 0);
    err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return fail(std::string("CUDA backend: ") + cudaGetErrorString(err));
    *out = m;
    return 0;
}

int new_seq(Model *m, Seq **out) {
    CH_REQUIRE(m != nullptr && out != nullptr, "cheetah_cuda_seq_new: null argument");
    CH_CUDA_TRY(cudaSetDevice(m->device));
    const CheetahCudaConfig &c = m->cfg;
    Seq *s = new Seq();
    m->refs.fetch_add(1);
    s->m = m;
    s->max_pages = (int)((c.max_positions + m->page_tokens - 1) / m->page_tokens);
    s->splits = attention_splits(1, c.kv_heads, c.max_positions, m->sms);
    s->mma_splits = mma_attention_splits(1, c.kv_heads, m->sms);
    s->scratch_splits = std::max(s->splits, s->mma_splits);
    const size_t QD = (size_t)c.q_heads * c.head_dim;
    bool ok = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMalloc(&s->page_table, s->max_pages * sizeof(int32_t)) == cudaSuccess &&
              cudaMalloc(&s->hidden, c.hidden_size * 4) == cudaSuccess &&
              cudaMalloc(&s->q, QD * 4) == cudaSuccess &&
              cudaMalloc(&s->qk_raw, (QD + 2 * (size_t)c.kv_heads * c.head_dim) * 4) == cudaSuccess &&
              cudaMalloc(&s->attn_out, QD * 4) == cudaSuccess &&
              cudaMalloc(&s->act, c.intermediate_size * 4) == cudaSuccess &&
              cudaMalloc(&s->logits, (size_t)c.vocab_size * 4) == cudaSuccess &&
              cudaMalloc(&s->argmax, 8) == cudaSuccess &&
              cudaMalloc(&s->d_step, sizeof(StepState)) == cudaSuccess &&
              cudaMalloc(&s->part_o, (size_t)c.kv_heads * s->scratch_splits * kMaxGroup * c.head_dim * 4) == cudaSuccess &&
              cudaMalloc(&s->part_ml, (size_t)c.kv_heads * s->scratch_splits * kMaxGroup * 2 * 4) == cudaSuccess &&
              cudaMalloc(&s->tickets, c.kv_heads * 4) == cudaSuccess &&
              cudaMalloc(&s->d_error, 4) == cudaSuccess &&
              cudaMalloc(&s->token_log, (size_t)c.max_positions * 4) == cudaSuccess &&
              cudaMallocHost(&s->h_step, sizeof(StepState)) == cudaSuccess &&
              cudaMallocHost(&s->h_logits, (size_t)c.vocab_size * 4) == cudaSuccess &&
              cudaMallocHost(&s->h_argmax, 8) == cudaSuccess && cudaMallocHost(&s->h_error, 4) == cudaSuccess;
    if (!ok) {
        delete s;
        set_error("CUDA backend: sequence allocation failed.");
        return -1;
    }
    cudaMemset(s->page_table, 0xFF, s->max_pages * sizeof(int32_t));
    cudaMemset(s->tickets, 0, c.kv_heads * 4);
    cudaMemset(s->d_error, 0, 4);
    cudaMemset(s->hidden, 0, c.hidden_size * 4);
    memset(s->h_step, 0, sizeof(StepState));
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        delete s;
        set_error(std::string("CUDA backend: ") + cudaGetErrorString(err));
        return -1;
    }
    *out = s;
    return 0;
}

int prefill_chunk_rows();
int run_prefill_chunk(Seq &s, const uint32_t *tokens, int M, size_t offset, bool last);
int check_device_error(Seq &s);

int make_tail_page_private(Seq &s);

int forward(Seq *s, const uint32_t *tokens, size_t n, size_t offset, float *logits_out,
            uint32_t *argmax_out) {
    CH_REQUIRE(s != nullptr, "cheetah_cuda_forward: null sequence");
    const CheetahCudaConfig &c = s->m->cfg;
    CH_REQUIRE(n > 0 && tokens != nullptr, "Native backend: empty token input.");
    for (size_t i = 0; i < n; ++i) {
        if (tokens[i] >= c.vocab_size) {
            set_error("Native backend: token id " + std::to_string(tokens[i]) +
                      " exceeds the vocabulary size " + std::to_string(c.vocab_size) + ".");
            return -1;
        }
    }
    CH_REQUIRE(offset == s->positions,
               "CUDA backend: offset " + std::to_string(offset) + " does not match the " +
                   std::to_string(s->positions) + " cached positions.");
    CH_REQUIRE(offset + n <= c.max_positions,
               "CUDA backend: position " + std::to_string(offset + n - 1) +
                   " exceeds the sequence capacity " + std::to_string(c.max_positions) + ".");
    CH_CUDA_TRY(cudaSetDevice(s->m->device));
    PlanGuard plan_guard(*s->m, s->stream);
    if (make_tail_page_private(*s) != 0) return -1;
    const bool chunked = n > 1 && s->m->gemm_prefill && std::getenv("CHEETAH_CUDA_STEPWISE_PREFILL") == nullptr;
    if (chunked) {
        const size_t chunk = (size_t)prefill_chunk_rows();
        for (size_t start = 0; start < n; start += chunk) {
            const size_t rows = std::min(chunk, n - start);
            if (run_prefill_chunk(*s, tokens + start, (int)rows, offset + start, start + rows == n) != 0) return -1;
        }
    } else {
        for (size_t i = 0; i < n; ++i) {
            if (run_decode_step(*s, tokens[i], offset + i) != 0) return -1;
            if (i + 1 < n) CH_CUDA_TRY(cudaStreamSynchronize(s->stream));  // h_step is reused
        }
    }
    // Results and the device error word come back in one stream round trip;
    // logits go straight into a caller buffer in pinned (page-locked or
    // registered) host memory, through the sequence's pinned buffer otherwise.
    bool direct = false;
    if (logits_out) {
        cudaPointerAttributes attr{};
        direct = cudaPointerGetAttributes(&attr, logits_out) == cudaSuccess && attr.type == cudaMemoryTypeHost;
        if (!direct) cudaGetLastError();
        CH_CUDA_TRY(cudaMemcpyAsync(direct ? logits_out : s->h_logits, s->logits, (size_t)c.vocab_size * 4,
                                    cudaMemcpyDeviceToHost, s->stream));
    }
    if (argmax_out) {
        CH_CUDA_TRY(cudaMemcpyAsync(s->h_argmax, s->argmax, 8, cudaMemcpyDeviceToHost, s->stream));
    }
    CH_CUDA_TRY(cudaMemcpyAsync(s->h_error, s->d_error, 4, cudaMemcpyDeviceToHost, s->stream));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (*s->h_error != 0 && check_device_error(*s) != 0) {
        // The call's K/V rows are not trusted: the sequence keeps the
        // positions it had, so the same call can be repeated.
        s->positions = offset;
        return -1;
    }
    if (logits_out && !direct) memcpy(logits_out, s->h_logits, (size_t)c.vocab_size * 4);
    if (argmax_out) *argmax_out = (uint32_t)(*s->h_argmax & 0xFFFFFFFFull);
    return 0;
}

int copy_pages(Model *m, const std::vector<int> &src, const std::vector<int> &dst, cudaStream_t stream) {
    if (src.empty()) return 0;
    int32_t *d_ids = nullptr;
    CH_CUDA_TRY(cudaMalloc(&d_ids, src.size() * 2 * sizeof(int32_t)));
    std::vector<int32_t> ids(src.begin(), src.end());
    ids.insert(ids.end(), dst.begin(), dst.end());
    cudaError_t err = cudaMemcpyAsync(d_ids, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, stream);
    if (err == cudaSuccess) {
        copy_pages_kernel<<<4 * m->sms, 256, 0, stream>>>(
            d_ids, d_ids + src.size(), (int)src.size(), m->k_pool, m->v_pool, m->layer_stride_bytes,
            (int)m->cfg.num_layers, m->page_bytes);
        err = cudaGetLastError();
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    cudaFree(d_ids);
    CH_CUDA_TRY(err);
    return 0;
}

// Copy-on-write of the page a sequence appends into next: the page holding
// position `positions` when a snapshot or another sequence also holds it
// (the pages before it are full and never written again).
int make_tail_page_private(Seq &s) {
    const size_t index = s.positions / s.m->page_tokens;
    if (index >= s.pages.size()) return 0;
    const int shared = s.pages[index];
    if (s.m->page_holders(shared) <= 1) return 0;
    const int page = s.m->alloc_page();
    if (page < 0) {
        set_error("CUDA backend: KV page pool exhausted (raise kv_pool_tokens).");
        return -1;
    }
    std::vector<int> dst{page};
    if (copy_pages(s.m, {shared}, dst, s.stream) != 0) {
        s.m->release_pages(dst);
        return -1;
    }
    std::vector<int> old{shared};
    s.m->release_pages(old);
    s.pages[index] = page;
    const int32_t id = page;
    CH_CUDA_TRY(cudaMemcpy(s.page_table + index, &id, 4, cudaMemcpyHostToDevice));
    return 0;
}

// Allocate pages so positions [0, end) are backed; new entries are written
// to the device page table.
int ensure_pages_upto(Seq &s, size_t end) {
    const size_t need = (end + s.m->page_tokens - 1) / s.m->page_tokens;
    if (need > (size_t)s.max_pages) {
        set_error("CUDA backend: position " + std::to_string(end - 1) + " exceeds the sequence capacity " +
                  std::to_string(s.m->cfg.max_positions) + ".");
        return -1;
    }
    const size_t first = s.pages.size();
    while (s.pages.size() < need) {
        const int page = s.m->alloc_page();
        if (page < 0) {
            set_error("CUDA backend: KV page pool exhausted (raise kv_pool_tokens).");
            return -1;
        }
        s.pages.push_back(page);
    }
    if (need > first) {
        std::vector<int32_t> ids(s.pages.begin() + first, s.pages.end());
        CH_CUDA_TRY(cudaMemcpyAsync(s.page_table + first, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, s.stream));
        CH_CUDA_TRY(cudaStreamSynchronize(s.stream));
    }
    return 0;
}

int prefill_chunk_rows() {
    const char *env = std::getenv("CHEETAH_PREFILL_CHUNK");  // ops.rs:523-535 (default 256)
    const int v = env ? std::atoi(env) : 0;
    return v > 0 ? v : 256;
}

int ensure_prefill_buffers(Seq &s, int rows) {
    if (rows <= s.chunk_cap) return 0;
    Model &m = *s.m;
    const CheetahCudaConfig &c = m.cfg;
    const size_t H = c.hidden_size, I = c.intermediate_size, QD = (size_t)c.q_heads * c.head_dim;
    cudaFree(s.ptokens);
    cudaFree(s.phid);
    cudaFree(s.pxb);
    cudaFree(s.pqb);
    cudaFree(s.pab);
    cudaFree(s.pact);
    cudaFree(s.ppart_o);
    cudaFree(s.ppart_ml);
    cudaFree(s.psplit_ws);
    cudaFree(s.psplit_tickets);
    s.psplit_ws = nullptr;
    s.psplit_tickets = nullptr;
    s.chunk_cap = 0;
    const size_t R = (size_t)rows;
    bool ok = cudaMalloc(&s.ptokens, R * 4) == cudaSuccess && cudaMalloc(&s.phid, R * H * 4) == cudaSuccess &&
              cudaMalloc(&s.pxb, R * H * 2) == cudaSuccess && cudaMalloc(&s.pqb, R * QD * 2) == cudaSuccess &&
              cudaMalloc(&s.pab, R * QD * 2) == cudaSuccess && cudaMalloc(&s.pact, R * I * 2) == cudaSuccess &&
              cudaMalloc(&s.ppart_o, (size_t)kPrefillMaxSplits * R * QD * 4) == cudaSuccess &&
              cudaMalloc(&s.ppart_ml, (size_t)kPrefillMaxSplits * R * c.q_heads * 2 * 4) == cudaSuccess &&
              cudaMalloc(&s.psplit_ws, (size_t)m.sms * kGemmBM * 128 * 4) == cudaSuccess &&
              cudaMalloc(&s.psplit_tickets, (size_t)m.sms * 4) == cudaSuccess;
    if (!ok) {
        set_error("CUDA backend: prefill buffer allocation failed.");
        return -1;
    }
    CH_CUDA_TRY(cudaMemsetAsync(s.psplit_tickets, 0, (size_t)m.sms * 4, s.stream));
    if (make_bf16_tensor_map(&s.map_xb, s.pxb, R, H, kGemmBM) != 0 ||
        make_bf16_tensor_map(&s.map_ab, s.pab, R, QD, kGemmBM) != 0 ||
        make_bf16_tensor_map(&s.map_act, s.pact, R, I, kGemmBM) != 0 ||
        make_bf16_tensor_map(&s.map_qb, s.pqb, R, QD, kTcRows) != 0) {
        return -1;
    }
    s.chunk_cap = rows;
    return 0;
}

template <int EPI, int BN>
int launch_prefill_gemm_bn(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &b2,
                           const PrefillGemmParams &p, cudaStream_t st, bool pdl, int splits = 1) {
    auto kernel = prefill_gemm_kernel<EPI, BN>;
    const size_t smem = prefill_gemm_smem<BN>();
    // The attribute is per function and device; set it once per device.
    static std::atomic<uint32_t> attr_devices{0};
    int dev = 0;
    CH_CUDA_TRY(cudaGetDevice(&dev));
    const uint32_t bit = dev < 32 ? 1u << dev : 0u;
    if (bit == 0 || !(attr_devices.load() & bit)) {
        CH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_devices.fetch_or(bit);
    }
    const int n_tiles = EPI == kPgSwiglu ? (p.N + BN / 2 - 1) / (BN / 2) : (p.N + BN - 1) / BN;
    dim3 grid(n_tiles, (p.M + kGemmBM - 1) / kGemmBM, splits);
    CH_CUDA_TRY(launch_ex(kernel, grid, dim3(kGemmThreads), smem, st, pdl, a, b, b2, p));
    return 0;
}

// Tile width: 64-column tiles double the CTA count of the narrow GEMMs
// (QKV, o_proj, down at chunk sizes of a few hundred rows). With a split-K
// workspace (batched decode: one row tile), a grid of fewer than half the
// SMs is split along K into up to SMs / tiles parts of at least eight
// k-blocks each (the workspace holds SMs tiles of 128 x 128 f32).
template <int EPI>
int launch_prefill_gemm(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &b2, const PrefillGemmParams &p,
                        cudaStream_t st, bool pdl, int sms) {
    const int m_tiles = (p.M + kGemmBM - 1) / kGemmBM;
    const bool narrow = EPI != kPgSwiglu && (EPI != kPgQkv || p.head_dim == 64) &&
                        ((p.N + 127) / 128) * m_tiles < sms;
    const int bn = narrow ? 64 : 128;
    const int tiles = m_tiles * (EPI == kPgSwiglu ? (p.N + bn / 2 - 1) / (bn / 2) : (p.N + bn - 1) / bn);
    int splits = 1;
    if (p.split_ws != nullptr && p.split_tickets != nullptr && 2 * tiles <= sms &&
        env_flag("CHEETAH_CUDA_GEMM_SPLITK", true)) {
        const int k_total = (p.K + kGemmBK - 1) / kGemmBK;
        splits = std::max(1, std::min(k_total / 8, sms / tiles));
    }
    if (narrow) return launch_prefill_gemm_bn<EPI, 64>(a, b, b2, p, st, pdl, splits);
    return launch_prefill_gemm_bn<EPI, 128>(a, b, b2, p, st, pdl, splits);
}

// Blocks of 256 threads for prefill_merge_kernel: one (row, head, 4 dims)
// item per thread, capped at 8 blocks per SM (all resident; a larger grid
// strides).
inline int merge_blocks(const PrefillAttnParams &ap, int head_dim, int sms) {
    const long long items = (long long)ap.T * ap.q_heads * (head_dim / 4);
    return (int)std::max(1LL, std::min((items + 255) / 256, 8LL * sms));
}

// Causal prefill attention over the paged bf16 cache (`ops.rs:1357-1421`
// for each query row; the rows' own K/V are already appended): tcgen05
// kernels, two 128-row query tiles per CTA for head_dim 64 and one for 128
// (CHEETAH_PREFILL_TC=0 selects the mma.sync kernel for both). Key-range
// splits fill the SMs when the query rows alone do not; a merge kernel then
// combines the partials (ap.part_o / ap.part_ml sized for kPrefillMaxSplits).
int launch_prefill_attention(PrefillAttnParams ap, const CUtensorMap &q_map, const CUtensorMap &k_map,
                             const CUtensorMap &v_map, int head_dim, size_t offset, int sms, cudaStream_t st,
                             bool pdl) {
    const int M = ap.T;
    if (head_dim == 64 && env_flag("CHEETAH_PREFILL_TC", true) && env_flag("CHEETAH_PREFILL_TC_PAIR", true)) {
        // Two 128-row query tiles per CTA; the same split rule over its blocks.
        const int blocks = ((M + kTpRows - 1) / kTpRows) * ap.q_heads;
        const int key_tiles = (int)((offset + M + kTcKeys - 1) / kTcKeys);
        ap.splits = std::max(1, std::min(std::min(kPrefillMaxSplits, sms / blocks), key_tiles / 2));
        const size_t tsmem = prefill_attention_tc_pair_smem();
        CH_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_tc_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem));
        dim3 tgrid((M + kTpRows - 1) / kTpRows, ap.q_heads, ap.splits);
        CH_CUDA_TRY(launch_ex(prefill_attention_tc_pair_kernel, tgrid, dim3(kTpThreads), tsmem, st, pdl, q_map,
                              k_map, v_map, ap));
        if (ap.splits > 1) {
            CH_CUDA_TRY(launch_ex(prefill_merge_kernel<64>, dim3(merge_blocks(ap, 64, sms)), dim3(256), 0, st, pdl, ap));
        }
        return 0;
    }
    if (head_dim == 64 && env_flag("CHEETAH_PREFILL_TC", true)) {
        // Tensor-core attention: one CTA per SM (512 TMEM columns each);
        // key-range splits fill the SMs, each split >= 2 key tiles.
        const int blocks = ((M + kTcRows - 1) / kTcRows) * ap.q_heads;
        const int key_tiles = (int)((offset + M + kTcKeys - 1) / kTcKeys);
        ap.splits = std::max(1, std::min(std::min(kPrefillMaxSplits, sms / blocks), key_tiles / 2));
        const size_t tsmem = prefill_attention_tc_smem();
        CH_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)tsmem));
        dim3 tgrid((M + kTcRows - 1) / kTcRows, ap.q_heads, ap.splits);
        CH_CUDA_TRY(launch_ex(prefill_attention_tc_kernel, tgrid, dim3(kTcThreads), tsmem, st, pdl, q_map, k_map,
                              v_map, ap));
        if (ap.splits > 1) {
            CH_CUDA_TRY(launch_ex(prefill_merge_kernel<64>, dim3(merge_blocks(ap, 64, sms)), dim3(256), 0, st, pdl, ap));
        }
        return 0;
    }
    if (head_dim == 128 && env_flag("CHEETAH_PREFILL_TC", true)) {
        // The same split rule for head_dim 128 (O accumulated in TMEM).
        const int blocks = ((M + kTcRows - 1) / kTcRows) * ap.q_heads;
        const int key_tiles = (int)((offset + M + kTcKeys - 1) / kTcKeys);
        ap.splits = std::max(1, std::min(std::min(kPrefillMaxSplits, sms / blocks), key_tiles / 2));
        const size_t tsmem = prefill_attention_tc2_smem<128>();
        CH_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_tc2_kernel<128>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem));
        dim3 tgrid((M + kTcRows - 1) / kTcRows, ap.q_heads, ap.splits);
        CH_CUDA_TRY(launch_ex(prefill_attention_tc2_kernel<128>, tgrid, dim3(kTcThreads), tsmem, st, pdl, q_map,
                              k_map, v_map, ap));
        if (ap.splits > 1) {
            CH_CUDA_TRY(launch_ex(prefill_merge_kernel<128>, dim3(merge_blocks(ap, 128, sms)), dim3(256), 0, st, pdl, ap));
        }
        return 0;
    }
    const size_t asmem = prefill_attention_smem();
    // Key-range splits: about two CTAs per SM (each CTA covers >= 4 key tiles).
    const int blocks = ((M + 15) / 16) * ap.kv_heads;
    const int key_tiles = (int)((offset + M + 63) / 64);
    ap.splits = std::max(1, std::min(std::min(kPrefillMaxSplits, (2 * sms + blocks - 1) / blocks),
                                     std::max(1, key_tiles / 4)));
    dim3 agrid((M + 15) / 16, ap.kv_heads, ap.splits);
    if (head_dim == 64) {
        CH_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)asmem));
        CH_CUDA_TRY(launch_ex(prefill_attention_kernel<64>, agrid, dim3(kPrefillWarps * kWarp), asmem, st, pdl,
                              k_map, v_map, ap));
        if (ap.splits > 1) {
            CH_CUDA_TRY(launch_ex(prefill_merge_kernel<64>, dim3(merge_blocks(ap, 64, sms)), dim3(256), 0, st, pdl, ap));
        }
    } else {
        CH_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)asmem));
        CH_CUDA_TRY(launch_ex(prefill_attention_kernel<128>, agrid, dim3(kPrefillWarps * kWarp), asmem, st, pdl,
                              k_map, v_map, ap));
        if (ap.splits > 1) {
            CH_CUDA_TRY(launch_ex(prefill_merge_kernel<128>, dim3(merge_blocks(ap, 128, sms)), dim3(256), 0, st, pdl, ap));
        }
    }
    return 0;
}

// One prompt chunk through every layer on the tensor cores
// (`Qwen2Native::forward_chunk`, `qwen2.rs:208-233`): embeddings, then per
// layer norm -> QKV GEMM (+bias, RoPE, KV append) -> causal attention ->
// o_proj GEMM (+bias, residual) -> norm -> gate/up GEMM (SwiGLU) -> down
// GEMM (residual). With `last`, the final row's norm + lm_head follow.
int run_prefill_chunk(Seq &s, const uint32_t *tokens, int M, size_t offset, bool last) {
    Model &m = *s.m;
    const CheetahCudaConfig &c = m.cfg;
    const int H = c.hidden_size, I = c.intermediate_size, QD = c.q_heads * c.head_dim, KD = c.kv_heads * c.head_dim;
    const bool pdl = m.pdl;
    cudaStream_t st = s.stream;
    if (ensure_prefill_buffers(s, std::max(M, prefill_chunk_rows())) != 0) return -1;
    if (ensure_pages_upto(s, offset + M) != 0) return -1;
    std::vector<int32_t> ids(tokens, tokens + M);
    CH_CUDA_TRY(cudaMemcpyAsync(s.ptokens, ids.data(), (size_t)M * 4, cudaMemcpyHostToDevice, st));
    CH_CUDA_TRY(launch_ex(embed_rows_kernel, dim3(M), dim3(256), 0, st, pdl, m.embed, H, (const int32_t *)s.ptokens, M,
                          s.phid));
    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        if (stage_layer(m, layer, st) != 0) return -1;
        const LayerWeights &w = m.layers[layer];
        uint8_t *k_layer = m.k_pool + layer * m.layer_stride_bytes;
        uint8_t *v_layer = m.v_pool + layer * m.layer_stride_bytes;
        CH_CUDA_TRY(launch_ex(norm_rows_bf16_kernel, dim3(M), dim3(256), 0, st, pdl, (const float *)s.phid, M, H,
                              w.ln1, c.rms_eps, s.pxb));
        PrefillGemmParams g = {};
        g.M = M;
        g.N = QD + 2 * KD;
        g.K = H;
        g.bias = w.bqkv;
        g.q_norm = w.q_norm;
        g.k_norm = w.k_norm;
        g.eps = c.rms_eps;
        g.out_bf16 = s.pqb;
        g.ld_out = QD;
        g.q_heads = c.q_heads;
        g.kv_heads = c.kv_heads;
        g.head_dim = c.head_dim;
        g.offset = (int)offset;
        g.rope_cos = m.rope_cos;
        g.rope_sin = m.rope_sin;
        g.page_table = s.page_table;
        g.max_pages = s.max_pages;
        g.num_pages = m.num_pages;
        g.page_tokens = m.page_tokens;
        g.k_cache = k_layer;
        g.v_cache = v_layer;
        g.kv_f32 = m.kv_f32;
        g.error = s.d_error;
        if (launch_prefill_gemm<kPgQkv>(s.map_xb, w.map_qkv, w.map_qkv, g, st, pdl, m.sms) != 0) return -1;

        PrefillAttnParams ap = {};
        ap.q = s.pqb;
        ap.out = s.pab;
        ap.T = M;
        ap.offset = (int)offset;
        ap.q_heads = c.q_heads;
        ap.kv_heads = c.kv_heads;
        ap.page_table = s.page_table;
        ap.max_pages = s.max_pages;
        ap.num_pages = m.num_pages;
        ap.page_tokens = m.page_tokens;
        ap.layer_row_offset = (long long)layer * m.num_pages * c.kv_heads * m.page_tokens;
        ap.window = c.sliding_window;
        ap.scale = 1.0f / sqrtf((float)c.head_dim);
        ap.error = s.d_error;
        ap.part_o = s.ppart_o;
        ap.part_ml = s.ppart_ml;
        if (launch_prefill_attention(ap, s.map_qb, m.k_map, m.v_map, (int)c.head_dim, offset, m.sms, st, pdl) != 0)
            return -1;

        PrefillGemmParams o = {};
        o.M = M;
        o.N = H;
        o.K = QD;
        o.bias = w.bo;
        o.out_f32 = s.phid;
        o.ld_out = H;
        o.error = s.d_error;
        if (launch_prefill_gemm<kPgResidual>(s.map_ab, w.map_o, w.map_o, o, st, pdl, m.sms) != 0) return -1;

        CH_CUDA_TRY(launch_ex(norm_rows_bf16_kernel, dim3(M), dim3(256), 0, st, pdl, (const float *)s.phid, M, H,
                              w.ln2, c.rms_eps, s.pxb));
        PrefillGemmParams gu = {};
        gu.M = M;
        gu.N = I;
        gu.K = H;
        gu.out_bf16 = s.pact;
        gu.ld_out = I;
        gu.error = s.d_error;
        if (launch_prefill_gemm<kPgSwiglu>(s.map_xb, w.map_gate, w.map_up, gu, st, pdl, m.sms) != 0) return -1;

        PrefillGemmParams dn = {};
        dn.M = M;
        dn.N = H;
        dn.K = I;
        dn.out_f32 = s.phid;
        dn.ld_out = H;
        dn.error = s.d_error;
        dn.split_ws = s.psplit_ws;
        dn.split_tickets = s.psplit_tickets;
        if (launch_prefill_gemm<kPgResidual>(s.map_act, w.map_down, w.map_down, dn, st, pdl, m.sms) != 0) return -1;
    }
    if (last) {
        CH_CUDA_TRY(cudaMemsetAsync(s.argmax, 0, 8, st));
        GemvParams lm = {};
        lm.w0 = m.lm_head;
        lm.rows = c.vocab_size;
        lm.cols = H;
        lm.batch = 1;
        lm.x = s.phid + (size_t)(M - 1) * H;
        lm.x_stride = H;
        lm.norm_w = m.final_norm;
        lm.eps = c.rms_eps;
        lm.y = s.logits;
        lm.y_stride = c.vocab_size;
        lm.argmax = s.argmax;
        if (run_gemv<kEpiLogits>(lm, st, pdl, m.sms) != 0) return -1;
    }
    s.positions = offset + M;
    return 0;
}

// Device-side guards (bounded waits, page-table checks) record a code in the
// sequence's error word; report and clear it after each synchronising call.
int check_device_error(Seq &s) {
    int code = 0;
    CH_CUDA_TRY(cudaMemcpy(&code, s.d_error, 4, cudaMemcpyDeviceToHost));
    if (code != 0) {
        cudaMemsetAsync(s.d_error, 0, 4, s.stream);
        if (s.mk_ctrl) cudaMemsetAsync(s.mk_ctrl, 0, kMkCtrlWords * 4, s.stream);
        if (s.psplit_tickets) cudaMemsetAsync(s.psplit_tickets, 0, (size_t)s.m->sms * 4, s.stream);
        set_error("CUDA backend: device-side guard tripped (code " + std::to_string(code) +
                  "): a bounded wait timed out or a KV page id was out of range.");
        return -1;
    }
    return 0;
}

// Batched decode workspace for up to `cap` sequences and page tables of
// `table_cap` entries.
int ensure_batch_workspace(Model &m, int cap, int table_cap) {
    if (cap <= m.batch_cap && table_cap <= m.batch_table_cap) return 0;
    CH_CUDA_TRY(cudaSetDevice(m.device));
    if (m.batch_stream) CH_CUDA_TRY(cudaStreamSynchronize(m.batch_stream));
    cap = std::max(cap, m.batch_cap);
    table_cap = std::max(table_cap, m.batch_table_cap);
    m.free_batch();
    const CheetahCudaConfig &c = m.cfg;
    const size_t R = (size_t)std::max(cap, 1), H = c.hidden_size, I = c.intermediate_size;
    const size_t QD = (size_t)c.q_heads * c.head_dim, V = c.vocab_size;
    const size_t meta = R * 3 + R * (size_t)table_cap;
    // Split partials for any batch <= cap: batch * kv_heads * splits <= max(SMs, batch * kv_heads).
    const size_t parts = std::max((size_t)m.sms, R * c.kv_heads) + 8;
    if (!m.batch_stream) CH_CUDA_TRY(cudaStreamCreateWithFlags(&m.batch_stream, cudaStreamNonBlocking));
    bool ok = cudaMalloc(&m.b_meta, meta * 4) == cudaSuccess && cudaMallocHost(&m.h_meta, meta * 4) == cudaSuccess &&
              cudaMalloc(&m.b_hid, R * H * 4) == cudaSuccess && cudaMalloc(&m.b_q, R * QD * 4) == cudaSuccess &&
              cudaMalloc(&m.b_logits, R * V * 4) == cudaSuccess && cudaMalloc(&m.b_xb, R * H * 2) == cudaSuccess &&
              cudaMalloc(&m.b_ab, R * QD * 2) == cudaSuccess && cudaMalloc(&m.b_act, R * I * 2) == cudaSuccess &&
              cudaMalloc(&m.b_attn_f32, R * QD * 4) == cudaSuccess && cudaMalloc(&m.b_act_f32, R * I * 4) == cudaSuccess &&
              cudaMalloc(&m.b_qk_raw, R * (QD + 2 * (size_t)c.kv_heads * c.head_dim) * 4) == cudaSuccess &&
              cudaMalloc(&m.b_argmax, R * 8) == cudaSuccess && cudaMallocHost(&m.h_argmax, R * 8) == cudaSuccess &&
              cudaMalloc(&m.b_part_o, parts * kMaxGroup * c.head_dim * 4) == cudaSuccess &&
              cudaMalloc(&m.b_part_ml, parts * kMaxGroup * 2 * 4) == cudaSuccess &&
              cudaMalloc(&m.b_tickets, R * c.kv_heads * 4) == cudaSuccess && cudaMalloc(&m.b_error, 4) == cudaSuccess &&
              cudaMalloc(&m.b_split_ws, (size_t)m.sms * kGemmBM * 128 * 4) == cudaSuccess &&
              cudaMalloc(&m.b_split_tickets, (size_t)m.sms * 4) == cudaSuccess &&
              cudaMalloc(&m.b_chain, 2 * 4) == cudaSuccess && cudaMallocHost(&m.h_chain, 4 * 4) == cudaSuccess &&
              cudaMalloc(&m.b_log, (size_t)kChainSteps * R * 4) == cudaSuccess &&
              cudaMallocHost(&m.h_log, (size_t)kChainSteps * R * 4) == cudaSuccess;
    if (!ok) {
        m.free_batch();
        set_error("CUDA backend: batch workspace allocation failed.");
        return -1;
    }
    cudaMemsetAsync(m.b_tickets, 0, R * c.kv_heads * 4, m.batch_stream);
    cudaMemsetAsync(m.b_split_tickets, 0, (size_t)m.sms * 4, m.batch_stream);
    cudaMemsetAsync(m.b_error, 0, 4, m.batch_stream);
    if (make_bf16_tensor_map(&m.map_bxb, m.b_xb, R, H, kGemmBM) != 0 ||
        make_bf16_tensor_map(&m.map_bab, m.b_ab, R, QD, kGemmBM) != 0 ||
        make_bf16_tensor_map(&m.map_bact, m.b_act, R, I, kGemmBM) != 0) {
        m.free_batch();
        return -1;
    }
    m.batch_cap = cap;
    m.batch_table_cap = table_cap;
    return 0;
}

// After a chained batched step: every row's next token is its greedy id (the
// padding rows copy row 0), its position and length advance by one, and the
// live rows' ids are logged at the chunk's step index.
__global__ void batch_advance_kernel(const unsigned long long *__restrict__ argmax, int32_t *__restrict__ meta,
                                     int cap, int rows, int32_t *__restrict__ chain, int32_t *__restrict__ log,
                                     int max_steps) {
    const int r = threadIdx.x;
    const int live = chain[0];
    const int step = chain[1];
    if (r < rows) {
        const int32_t tok = (int32_t)(argmax[r < live ? r : 0] & 0xFFFFFFFFull);
        meta[r] = tok;
        meta[cap + r] += 1;
        meta[2 * cap + r] += 1;
        if (r < live && step < max_steps) log[(long long)step * cap + r] = tok;
    }
    __syncthreads();
    if (r == 0) chain[1] = step + 1;
}

// Enqueue one padded batched decode step (M rows) on the model's batch
// stream: metadata upload, embeddings, every layer, final norm, lm_head +
// argmax. A chained step skips the upload (the metadata is already on the
// device) and ends with batch_advance_kernel, so the next step consumes this
// step's greedy ids.
// The same step for M <= kBatchGemvRows padded rows as weight-streaming
// tensor-core GEMVs over all M rows at once (gemv_mma.cuh: every weight byte
// streamed once, the rows as the MMA columns): RMSNorm prologues, QKV with
// RoPE and the paged K/V append of each row's position, batched tensor-core
// attention (f32 output), o_proj / down with residual epilogues, gate/up
// with SwiGLU, lm_head with per-row argmax. f32 activations between the
// kernels, rounded to bf16 as MMA operands (as the GEMM step's are).
int enqueue_batch_step_gemv(Model &m, int M, int table_stride, bool want_logits, bool chained) {
    cudaStream_t st = m.batch_stream;
    const bool pdl = m.pdl;
    const int cap = m.batch_cap;
    const CheetahCudaConfig &c = m.cfg;
    const int H = c.hidden_size, I = c.intermediate_size, QD = c.q_heads * c.head_dim, KD = c.kv_heads * c.head_dim;
    if (!chained) {
        CH_CUDA_TRY(cudaMemcpyAsync(m.b_meta, m.h_meta, (size_t)(3 * cap + M * table_stride) * 4,
                                    cudaMemcpyHostToDevice, st));
    }
    const int32_t *d_tok = m.b_meta, *d_pos = m.b_meta + cap, *d_len = m.b_meta + 2 * cap;
    const int32_t *d_tab = m.b_meta + 3 * cap;
    CH_CUDA_TRY(cudaMemsetAsync(m.b_argmax, 0, (size_t)M * 8, st));
    CH_CUDA_TRY(launch_ex(embed_rows_kernel, dim3(M), dim3(256), 0, st, pdl, m.embed, H, d_tok, M, m.b_hid));
    const int splits = mma_attention_splits(M, c.kv_heads, m.sms);
    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        if (stage_layer(m, layer, st) != 0) return -1;
        const LayerWeights &w = m.layers[layer];
        GemvParams q = {};
        q.w0 = w.wqkv;
        q.wt = kWBf16;
        q.rows = QD + 2 * KD;
        q.cols = H;
        q.batch = M;
        q.x = m.b_hid;
        q.x_stride = H;
        q.norm_w = w.ln1;
        q.eps = c.rms_eps;
        q.bias = w.bqkv;
        q.y = m.b_q;
        q.y_stride = QD;
        q.q_heads = c.q_heads;
        q.kv_heads = c.kv_heads;
        q.head_dim = c.head_dim;
        q.rope_cos = m.rope_cos;
        q.rope_sin = m.rope_sin;
        q.positions = d_pos;
        q.page_table = d_tab;
        q.max_pages = table_stride;
        q.num_pages = m.num_pages;
        q.page_tokens = m.page_tokens;
        q.k_cache = m.k_pool + layer * m.layer_stride_bytes;
        q.v_cache = m.v_pool + layer * m.layer_stride_bytes;
        q.kv_f32 = m.kv_f32;
        q.error = m.b_error;
        q.split_ws = m.b_split_ws;
        q.split_tickets = m.b_split_tickets;
        if (m.qk_norm) q.qk_raw = m.b_qk_raw;
        if (launch_gemv_mma<kEpiQkv>(q, st, pdl, m.sms, m.sms) != 0) return -1;
        if (m.qk_norm) {
            CH_CUDA_TRY(launch_ex(qk_norm_rope_kernel, dim3(c.q_heads + 2 * c.kv_heads, M), dim3(32), 0, st, pdl,
                                  q, w.q_norm, w.k_norm));
        }

        MmaAttnParams ap = {};
        ap.a.q = m.b_q;
        ap.a.page_table = d_tab;
        ap.a.seq_lens = d_len;
        ap.a.max_pages = table_stride;
        ap.a.num_pages = m.num_pages;
        ap.a.page_tokens = m.page_tokens;
        ap.a.batch = M;
        ap.a.q_heads = c.q_heads;
        ap.a.kv_heads = c.kv_heads;
        ap.a.window = c.sliding_window;
        ap.a.splits = splits;
        ap.a.scale = 1.0f / sqrtf((float)c.head_dim);
        ap.a.out = m.b_attn_f32;
        ap.a.part_o = m.b_part_o;
        ap.a.part_ml = m.b_part_ml;
        ap.a.tickets = m.b_tickets;
        ap.a.error = m.b_error;
        ap.layer_row_offset = (long long)layer * m.num_pages * c.kv_heads * m.page_tokens;
        ap.page_tokens = m.page_tokens;
        if (launch_attention_mma(m.k_map, m.v_map, ap, c.head_dim, st, pdl) != 0) return -1;

        GemvParams o = {};
        o.w0 = w.wo;
        o.wt = kWBf16;
        o.rows = H;
        o.cols = QD;
        o.batch = M;
        o.x = m.b_attn_f32;
        o.x_stride = QD;
        o.bias = w.bo;
        o.y = m.b_hid;
        o.y_stride = H;
        o.error = m.b_error;
        o.split_ws = m.b_split_ws;
        o.split_tickets = m.b_split_tickets;
        if (launch_gemv_mma<kEpiResidual>(o, st, pdl, m.sms, m.sms) != 0) return -1;

        GemvParams gu = {};
        gu.w0 = w.wgate;
        gu.w1 = w.wup;
        gu.wt = kWBf16;
        gu.rows = I;
        gu.cols = H;
        gu.batch = M;
        gu.x = m.b_hid;
        gu.x_stride = H;
        gu.norm_w = w.ln2;
        gu.eps = c.rms_eps;
        gu.y = m.b_act_f32;
        gu.y_stride = I;
        gu.error = m.b_error;
        gu.split_ws = m.b_split_ws;
        gu.split_tickets = m.b_split_tickets;
        if (launch_gemv_mma<kEpiSwiglu>(gu, st, pdl, m.sms, m.sms) != 0) return -1;

        GemvParams dn = {};
        dn.w0 = w.wdown;
        dn.wt = kWBf16;
        dn.rows = H;
        dn.cols = I;
        dn.batch = M;
        dn.x = m.b_act_f32;
        dn.x_stride = I;
        dn.y = m.b_hid;
        dn.y_stride = H;
        dn.error = m.b_error;
        dn.split_ws = m.b_split_ws;
        dn.split_tickets = m.b_split_tickets;
        if (launch_gemv_mma<kEpiResidual>(dn, st, pdl, m.sms, m.sms) != 0) return -1;
    }
    GemvParams lm = {};
    lm.w0 = m.lm_head;
    lm.wt = kWBf16;
    lm.rows = c.vocab_size;
    lm.cols = H;
    lm.batch = M;
    lm.x = m.b_hid;
    lm.x_stride = H;
    lm.norm_w = m.final_norm;
    lm.eps = c.rms_eps;
    lm.y = m.b_logits;  // always written (the rows' argmax reads the same pass)
    lm.y_stride = c.vocab_size;
    lm.argmax = m.b_argmax;
    lm.error = m.b_error;
    lm.split_ws = m.b_split_ws;
        lm.split_tickets = m.b_split_tickets;
        if (launch_gemv_mma<kEpiLogits>(lm, st, pdl, m.sms, m.sms) != 0) return -1;
    (void)want_logits;
    if (chained) {
        batch_advance_kernel<<<1, 128, 0, st>>>(m.b_argmax, m.b_meta, cap, M, m.b_chain, m.b_log, kChainSteps);
        CH_CUDA_TRY(cudaGetLastError());
    }
    return 0;
}

int enqueue_batch_step(Model &m, int M, int table_stride, bool want_logits, bool chained = false) {
    if (m.batch_gemv && M <= kBatchGemvRows) return enqueue_batch_step_gemv(m, M, table_stride, want_logits, chained);
    cudaStream_t st = m.batch_stream;
    const bool pdl = m.pdl;
    const int cap = m.batch_cap;
    const CheetahCudaConfig &c = m.cfg;
    const int H = c.hidden_size, I = c.intermediate_size, QD = c.q_heads * c.head_dim, KD = c.kv_heads * c.head_dim;
    if (!chained) {
        CH_CUDA_TRY(cudaMemcpyAsync(m.b_meta, m.h_meta, (size_t)(3 * cap + M * table_stride) * 4,
                                    cudaMemcpyHostToDevice, st));
    }
    const int32_t *d_tok = m.b_meta, *d_pos = m.b_meta + cap, *d_len = m.b_meta + 2 * cap;
    const int32_t *d_tab = m.b_meta + 3 * cap;
    CH_CUDA_TRY(cudaMemsetAsync(m.b_argmax, 0, (size_t)M * 8, st));
    CH_CUDA_TRY(launch_ex(embed_rows_kernel, dim3(M), dim3(256), 0, st, pdl, m.embed, H, d_tok, M, m.b_hid));
    const int splits = mma_attention_splits(M, c.kv_heads, m.sms);
    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        if (stage_layer(m, layer, st) != 0) return -1;
        const LayerWeights &w = m.layers[layer];
        CH_CUDA_TRY(launch_ex(norm_rows_bf16_kernel, dim3(M), dim3(256), 0, st, pdl, (const float *)m.b_hid, M, H,
                              w.ln1, c.rms_eps, m.b_xb));
        PrefillGemmParams g = {};
        g.M = M;
        g.N = QD + 2 * KD;
        g.K = H;
        g.bias = w.bqkv;
        g.q_norm = w.q_norm;
        g.k_norm = w.k_norm;
        g.eps = c.rms_eps;
        g.out_q_f32 = m.b_q;
        g.ld_out = QD;
        g.q_heads = c.q_heads;
        g.kv_heads = c.kv_heads;
        g.head_dim = c.head_dim;
        g.rope_cos = m.rope_cos;
        g.rope_sin = m.rope_sin;
        g.page_table = d_tab;
        g.row_pos = d_pos;
        g.table_stride = table_stride;
        g.max_pages = table_stride;
        g.num_pages = m.num_pages;
        g.page_tokens = m.page_tokens;
        g.k_cache = m.k_pool + layer * m.layer_stride_bytes;
        g.v_cache = m.v_pool + layer * m.layer_stride_bytes;
        g.kv_f32 = m.kv_f32;
        g.error = m.b_error;
        g.split_ws = m.b_split_ws;
        g.split_tickets = m.b_split_tickets;
        if (launch_prefill_gemm<kPgQkv>(m.map_bxb, w.map_qkv, w.map_qkv, g, st, pdl, m.sms) != 0) return -1;

        MmaAttnParams ap = {};
        ap.a.q = m.b_q;
        ap.a.page_table = d_tab;
        ap.a.seq_lens = d_len;
        ap.a.max_pages = table_stride;
        ap.a.num_pages = m.num_pages;
        ap.a.page_tokens = m.page_tokens;
        ap.a.batch = M;
        ap.a.q_heads = c.q_heads;
        ap.a.kv_heads = c.kv_heads;
        ap.a.window = c.sliding_window;
        ap.a.splits = splits;
        ap.a.scale = 1.0f / sqrtf((float)c.head_dim);
        ap.a.out_bf16 = m.b_ab;
        ap.a.part_o = m.b_part_o;
        ap.a.part_ml = m.b_part_ml;
        ap.a.tickets = m.b_tickets;
        ap.a.error = m.b_error;
        ap.layer_row_offset = (long long)layer * m.num_pages * c.kv_heads * m.page_tokens;
        ap.page_tokens = m.page_tokens;
        if (launch_attention_mma(m.k_map, m.v_map, ap, c.head_dim, st, pdl) != 0) return -1;

        PrefillGemmParams o = {};
        o.M = M;
        o.N = H;
        o.K = QD;
        o.bias = w.bo;
        o.out_f32 = m.b_hid;
        o.ld_out = H;
        o.error = m.b_error;
        o.split_ws = m.b_split_ws;
        o.split_tickets = m.b_split_tickets;
        if (launch_prefill_gemm<kPgResidual>(m.map_bab, w.map_o, w.map_o, o, st, pdl, m.sms) != 0) return -1;
        CH_CUDA_TRY(launch_ex(norm_rows_bf16_kernel, dim3(M), dim3(256), 0, st, pdl, (const float *)m.b_hid, M, H,
                              w.ln2, c.rms_eps, m.b_xb));
        PrefillGemmParams gu = {};
        gu.M = M;
        gu.N = I;
        gu.K = H;
        gu.out_bf16 = m.b_act;
        gu.ld_out = I;
        gu.error = m.b_error;
        gu.split_ws = m.b_split_ws;
        gu.split_tickets = m.b_split_tickets;
        if (launch_prefill_gemm<kPgSwiglu>(m.map_bxb, w.map_gate, w.map_up, gu, st, pdl, m.sms) != 0) return -1;
        PrefillGemmParams dn = {};
        dn.M = M;
        dn.N = H;
        dn.K = I;
        dn.out_f32 = m.b_hid;
        dn.ld_out = H;
        dn.error = m.b_error;
        dn.split_ws = m.b_split_ws;
        dn.split_tickets = m.b_split_tickets;
        if (launch_prefill_gemm<kPgResidual>(m.map_bact, w.map_down, w.map_down, dn, st, pdl, m.sms) != 0) return -1;
    }
    CH_CUDA_TRY(launch_ex(norm_rows_bf16_kernel, dim3(M), dim3(256), 0, st, pdl, (const float *)m.b_hid, M, H,
                          m.final_norm, c.rms_eps, m.b_xb));
    PrefillGemmParams lm = {};
    lm.M = M;
    lm.N = c.vocab_size;
    lm.K = H;
    lm.out_f32 = want_logits ? m.b_logits : nullptr;
    lm.ld_out = c.vocab_size;
    lm.argmax = m.b_argmax;
    lm.error = m.b_error;
    if (launch_prefill_gemm_bn<kPgLogits, 128>(m.map_bxb, m.map_lm_head, m.map_lm_head, lm, st, pdl) != 0) return -1;
    if (chained) {
        batch_advance_kernel<<<1, 128, 0, st>>>(m.b_argmax, m.b_meta, cap, M, m.b_chain, m.b_log, kChainSteps);
        CH_CUDA_TRY(cudaGetLastError());
    }
    return 0;
}

// Validate a batch, give every sequence pages up to offsets[b] + steps, size
// the workspace and stage the padded metadata in h_meta. Rows are padded to a
// multiple of 8 with copies of row 0 (they recompute and rewrite row 0's K/V
// bit for bit), so a handful of captured graphs serve every batch size.
int prepare_batch(Model &m, Seq *const *seqs, const uint32_t *tokens, const size_t *offsets, size_t B, size_t steps,
                  const char *api, int *M_out, int *table_stride_out) {
    const CheetahCudaConfig &c = m.cfg;
    CH_REQUIRE(B > 0 && B <= 128, std::string(api) + ": batch must be 1..128");
    CH_REQUIRE(m.gemm_prefill, std::string(api) + ": needs bf16 weights and a bf16 KV cache");
    CH_CUDA_TRY(cudaSetDevice(m.device));
    size_t max_pages_used = 1;
    for (size_t b = 0; b < B; ++b) {
        Seq *s = seqs[b];
        CH_REQUIRE(s != nullptr && s->m == &m, std::string(api) + ": sequence of another model");
        for (size_t b2 = 0; b2 < b; ++b2) CH_REQUIRE(seqs[b2] != s, std::string(api) + ": sequence repeated");
        CH_REQUIRE(tokens[b] < c.vocab_size, "Native backend: token id " + std::to_string(tokens[b]) +
                                                 " exceeds the vocabulary size " + std::to_string(c.vocab_size) + ".");
        CH_REQUIRE(offsets[b] == s->positions, "CUDA backend: offset " + std::to_string(offsets[b]) +
                                                   " does not match the " + std::to_string(s->positions) +
                                                   " cached positions.");
        CH_REQUIRE(offsets[b] + steps <= c.max_positions,
                   "CUDA backend: position " + std::to_string(offsets[b] + steps - 1) +
                       " exceeds the sequence capacity " + std::to_string(c.max_positions) + ".");
        CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
        if (make_tail_page_private(*s) != 0 || ensure_pages_upto(*s, offsets[b] + steps) != 0) return -1;
        max_pages_used = std::max(max_pages_used, s->pages.size());
    }
    const int table_stride = (int)((max_pages_used + 15) / 16 * 16);
    const int M = (int)((B + 7) / 8 * 8);
    if (ensure_batch_workspace(m, std::max(M, 8), table_stride) != 0) return -1;
    // Metadata: tokens | positions | lengths | page tables (stride table_stride).
    const int cap = m.batch_cap;
    int32_t *h_tok = m.h_meta, *h_pos = m.h_meta + cap, *h_len = m.h_meta + 2 * cap, *h_tab = m.h_meta + 3 * cap;
    for (int r = 0; r < M; ++r) {
        const size_t b = r < (int)B ? (size_t)r : 0;
        h_tok[r] = (int32_t)tokens[b];
        h_pos[r] = (int32_t)offsets[b];
        h_len[r] = (int32_t)offsets[b] + 1;
        const Seq *s = seqs[b];
        for (int i = 0; i < table_stride; ++i) h_tab[r * table_stride + i] = i < (int)s->pages.size() ? s->pages[i] : -1;
    }
    *M_out = M;
    *table_stride_out = table_stride;
    return 0;
}

// The captured graph of one batched step for (rows, table stride, logits,
// chained), or nullptr when graphs are switched off.
int batch_graph(Model &m, int M, int table_stride, bool want_logits, bool chained, cudaGraphExec_t *out) {
    *out = nullptr;
    const uint64_t key = ((uint64_t)M << 40) | ((uint64_t)table_stride << 8) | (chained ? 2u : 0u) |
                         (want_logits ? 1u : 0u);
    auto it = m.batch_graphs.find(key);
    if (it == m.batch_graphs.end() && env_flag("CHEETAH_CUDA_GRAPH", true) && !m.planned) {
        cudaGraph_t graph = nullptr;
        CH_CUDA_TRY(cudaStreamBeginCapture(m.batch_stream, cudaStreamCaptureModeThreadLocal));
        const int rc = enqueue_batch_step(m, M, table_stride, want_logits, chained);
        const cudaError_t end_err = cudaStreamEndCapture(m.batch_stream, &graph);
        if (rc != 0 || end_err != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            if (rc == 0) set_error(std::string("batch graph capture failed: ") + cudaGetErrorString(end_err));
            return -1;
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        CH_REQUIRE(inst == cudaSuccess, std::string("batch graph instantiate failed: ") + cudaGetErrorString(inst));
        it = m.batch_graphs.emplace(key, exec).first;
    }
    if (it != m.batch_graphs.end()) *out = it->second;
    return 0;
}

// Report and clear the batch error word after a synchronising call.
int check_batch_error(Model &m) {
    int code = 0;
    CH_CUDA_TRY(cudaMemcpy(&code, m.b_error, 4, cudaMemcpyDeviceToHost));
    if (code != 0) {
        cudaMemsetAsync(m.b_error, 0, 4, m.batch_stream);
        // A split whose wait gave up never took its ticket: start them over.
        cudaMemsetAsync(m.b_split_tickets, 0, (size_t)m.sms * 4, m.batch_stream);
        set_error("CUDA backend: device-side guard tripped in a batched step (code " + std::to_string(code) + ").");
        return -1;
    }
    return 0;
}

// One decode token for each of B sequences (`ModelForward::forward` with a
// single token, B times), batched into GEMMs on the tensor cores: the weight
// stream is shared by the batch; attention reads each sequence's own pages.
// The step is replayed from a CUDA graph cached per (padded rows, page-table
// stride, logits wanted).
// row_logits: nullptr, or one host destination per row (nullptr rows get no
// copy); each row is copied straight into its destination.
int forward_batch_rows(Model *mp, Seq *const *seqs, const uint32_t *tokens, const size_t *offsets, size_t B,
                       float *const *row_logits, uint32_t *argmax_out) {
    CH_REQUIRE(mp != nullptr && seqs != nullptr && tokens != nullptr && offsets != nullptr,
               "cheetah_cuda_forward_batch: null argument");
    Model &m = *mp;
    const CheetahCudaConfig &c = m.cfg;
    if (B == 1) {
        // A batch of one: the single-sequence step (see forward_batch_greedy).
        CH_REQUIRE(seqs[0] != nullptr && seqs[0]->m == &m, "cheetah_cuda_forward_batch: sequence of another model");
        CH_REQUIRE(m.gemm_prefill, "cheetah_cuda_forward_batch: needs bf16 weights and a bf16 KV cache");
        return forward(seqs[0], tokens, 1, offsets[0], row_logits ? row_logits[0] : nullptr, argmax_out);
    }
    std::lock_guard<std::mutex> lock(m.batch_mutex);
    int M = 0, table_stride = 0;
    if (prepare_batch(m, seqs, tokens, offsets, B, 1, "cheetah_cuda_forward_batch", &M, &table_stride) != 0) return -1;
    PlanGuard plan_guard(m, m.batch_stream);
    bool want_logits = false;
    for (size_t b = 0; row_logits != nullptr && b < B; ++b) want_logits |= row_logits[b] != nullptr;
    cudaGraphExec_t exec = nullptr;
    if (batch_graph(m, M, table_stride, want_logits, false, &exec) != 0) return -1;
    cudaStream_t st = m.batch_stream;
    if (exec != nullptr) {
        CH_CUDA_TRY(cudaGraphLaunch(exec, st));
    } else if (enqueue_batch_step(m, M, table_stride, want_logits) != 0) {
        return -1;
    }
    for (size_t b = 0; want_logits && b < B; ++b) {
        if (row_logits[b] == nullptr) continue;
        CH_CUDA_TRY(cudaMemcpyAsync(row_logits[b], m.b_logits + b * c.vocab_size, (size_t)c.vocab_size * 4,
                                    cudaMemcpyDeviceToHost, st));
    }
    CH_CUDA_TRY(cudaMemcpyAsync(m.h_argmax, m.b_argmax, (size_t)B * 8, cudaMemcpyDeviceToHost, st));
    CH_CUDA_TRY(cudaStreamSynchronize(st));
    if (check_batch_error(m) != 0) return -1;
    for (size_t b = 0; b < B; ++b) {
        seqs[b]->positions = offsets[b] + 1;
        if (argmax_out) argmax_out[b] = (uint32_t)(m.h_argmax[b] & 0xFFFFFFFFull);
    }
    return 0;
}

int forward_batch(Model *mp, Seq *const *seqs, const uint32_t *tokens, const size_t *offsets, size_t B,
                  float *logits_out, uint32_t *argmax_out) {
    CH_REQUIRE(mp != nullptr, "cheetah_cuda_forward_batch: null argument");
    if (logits_out == nullptr) return forward_batch_rows(mp, seqs, tokens, offsets, B, nullptr, argmax_out);
    CH_REQUIRE(B > 0 && B <= 128, "cheetah_cuda_forward_batch: batch must be 1..128");
    float *rows[128];
    for (size_t b = 0; b < B; ++b) rows[b] = logits_out + b * mp->cfg.vocab_size;
    return forward_batch_rows(mp, seqs, tokens, offsets, B, rows, argmax_out);
}

// ---- Continuous batching behind the per-sequence forward -----------------
// The reference serves concurrent generations by giving each one a clone of
// the model (`engine.rs:1872-1876`, `ModelForwardClone`) whose `forward`
// runs on its own thread. Here every clone is a sequence of one shared model,
// and single-token forwards that reach the model while a step is running
// queue up and run together as the next batched step (tensor-core GEMMs or
// weight-streaming GEMVs shared by the batch): the first waiting caller runs
// everything queued, the others sleep until their results are in. One caller
// alone runs at once, without waiting for company. Groups smaller than
// CHEETAH_CUDA_COALESCE_MIN (default 3) run one by one on the single-sequence
// path, which beats a batched step that small.

// Validates one call alone (the checks `forward` makes), so a bad call fails
// by itself instead of failing the calls batched with it.
bool coalesced_call_valid(CoalescedCall &call) {
    const CheetahCudaConfig &c = call.s->m->cfg;
    if (call.token >= c.vocab_size) {
        call.error = "Native backend: token id " + std::to_string(call.token) + " exceeds the vocabulary size " +
                     std::to_string(c.vocab_size) + ".";
    } else if (call.offset != call.s->positions) {
        call.error = "CUDA backend: offset " + std::to_string(call.offset) + " does not match the " +
                     std::to_string(call.s->positions) + " cached positions.";
    } else if (call.offset + 1 > c.max_positions) {
        call.error = "CUDA backend: position " + std::to_string(call.offset) + " exceeds the sequence capacity " +
                     std::to_string(c.max_positions) + ".";
    } else {
        return true;
    }
    call.status = -1;
    return false;
}

void run_coalesced(Model &m, const std::vector<CoalescedCall *> &calls) {
    std::vector<CoalescedCall *> ok;
    for (CoalescedCall *call : calls) {
        if (coalesced_call_valid(*call)) ok.push_back(call);
    }
    const size_t min_batch = (size_t)std::max(2, env_int("CHEETAH_CUDA_COALESCE_MIN", 3));
    if (ok.size() < min_batch) {
        for (CoalescedCall *call : ok) {
            call->status = forward(call->s, &call->token, 1, call->offset, call->logits, call->argmax);
            if (call->status != 0) call->error = last_error();
        }
        return;
    }
    constexpr size_t kMaxRows = 128;  // forward_batch's limit
    for (size_t b0 = 0; b0 < ok.size(); b0 += kMaxRows) {
        const size_t B = std::min(kMaxRows, ok.size() - b0);
        std::vector<Seq *> seqs(B);
        std::vector<uint32_t> tokens(B), argmax(B);
        std::vector<size_t> offsets(B);
        std::vector<float *> rows(B);
        for (size_t b = 0; b < B; ++b) {
            CoalescedCall *call = ok[b0 + b];
            seqs[b] = call->s;
            tokens[b] = call->token;
            offsets[b] = call->offset;
            rows[b] = call->logits;  // each caller's buffer, written by the device
        }
        const int rc = forward_batch_rows(&m, seqs.data(), tokens.data(), offsets.data(), B, rows.data(),
                                          argmax.data());
        const std::string err = rc != 0 ? std::string(last_error()) : std::string();
        for (size_t b = 0; b < B; ++b) {
            CoalescedCall *call = ok[b0 + b];
            call->status = rc;
            if (rc != 0) {
                call->error = err;
                continue;
            }
            if (call->argmax) *call->argmax = argmax[b];
        }
        if (rc == 0) {
            m.co_batches.fetch_add(1);
            m.co_batched_calls.fetch_add(B);
        }
    }
}

int coalesced_forward(Seq *s, uint32_t token, size_t offset, float *logits_out, uint32_t *argmax_out) {
    Model &m = *s->m;
    m.co_calls.fetch_add(1);
    CoalescedCall me;
    me.s = s;
    me.token = token;
    me.offset = offset;
    me.logits = logits_out;
    me.argmax = argmax_out;
    std::unique_lock<std::mutex> lock(m.co_mutex);
    m.co_pending.push_back(&me);
    if (m.co_pending.size() >= m.co_last_group) m.co_cv.notify_all();  // a leader may be gathering
    while (!me.done) {
        if (m.co_running) {
            m.co_cv.wait(lock);
            continue;
        }
        // Lead: run everything queued (this call included). When the last
        // group was larger, its callers are likely on their way back: give
        // them a short window (CHEETAH_CUDA_COALESCE_WAIT_US, default 200)
        // to join, ending as soon as they all have.
        m.co_running = true;
        if (m.co_pending.size() < m.co_last_group) {
            const auto until = std::chrono::steady_clock::now() +
                               std::chrono::microseconds(std::max(0, env_int("CHEETAH_CUDA_COALESCE_WAIT_US", 200)));
            while (m.co_pending.size() < m.co_last_group &&
                   m.co_cv.wait_until(lock, until) != std::cv_status::timeout) {
            }
        }
        std::vector<CoalescedCall *> take;
        take.swap(m.co_pending);
        m.co_last_group = take.size();
        lock.unlock();
        run_coalesced(m, take);
        lock.lock();
        for (CoalescedCall *call : take) call->done = true;
        m.co_running = false;
        m.co_cv.notify_all();
    }
    lock.unlock();
    if (me.status != 0) {
        set_error(me.error);
        return -1;
    }
    return 0;
}

// Single-token forwards go through the batcher when the model can run
// batched steps (bf16 weights and KV cache) and CHEETAH_CUDA_COALESCE is on.
int forward_entry(Seq *s, const uint32_t *tokens, size_t n, size_t offset, float *logits_out, uint32_t *argmax_out) {
    if (s != nullptr && n == 1 && tokens != nullptr && s->m->gemm_prefill && env_flag("CHEETAH_CUDA_COALESCE", true)) {
        CH_CUDA_TRY(cudaSetDevice(s->m->device));
        return coalesced_forward(s, tokens[0], offset, logits_out, argmax_out);
    }
    return forward(s, tokens, n, offset, logits_out, argmax_out);
}

// `steps` greedy tokens for each of B sequences with no host round trip
// between steps: the metadata is uploaded once, and each replayed step ends
// by feeding its greedy ids to the next (batch_advance_kernel). The host
// reads the token log every kChainSteps steps. tokens_out[b * steps + i] is
// sequence b's greedy token after consuming position offsets[b] + i.
int generate_greedy(Seq *s, uint32_t first_token, size_t offset, size_t steps, uint32_t *tokens_out);

int forward_batch_greedy(Model *mp, Seq *const *seqs, const uint32_t *tokens, const size_t *offsets, size_t B,
                         size_t steps, uint32_t *tokens_out) {
    CH_REQUIRE(mp != nullptr && seqs != nullptr && tokens != nullptr && offsets != nullptr && tokens_out != nullptr,
               "cheetah_cuda_forward_batch_greedy: null argument");
    CH_REQUIRE(steps > 0, "cheetah_cuda_forward_batch_greedy: steps must be positive");
    Model &m = *mp;
    // A batch of one runs the single-sequence greedy chain (the persistent
    // decode kernel where the model has it): a batched step pays the fixed
    // cost of ~5 launches per layer whatever its row count.
    if (B == 1) {
        CH_REQUIRE(seqs[0] != nullptr && seqs[0]->m == &m,
                   "cheetah_cuda_forward_batch_greedy: sequence of another model");
        return generate_greedy(seqs[0], tokens[0], offsets[0], steps, tokens_out);
    }
    std::lock_guard<std::mutex> lock(m.batch_mutex);
    int M = 0, table_stride = 0;
    if (prepare_batch(m, seqs, tokens, offsets, B, steps, "cheetah_cuda_forward_batch_greedy", &M, &table_stride) != 0)
        return -1;
    PlanGuard plan_guard(m, m.batch_stream);
    cudaGraphExec_t exec = nullptr;
    if (batch_graph(m, M, table_stride, false, true, &exec) != 0) return -1;
    cudaStream_t st = m.batch_stream;
    const int cap = m.batch_cap;
    CH_CUDA_TRY(cudaMemcpyAsync(m.b_meta, m.h_meta, (size_t)(3 * cap + M * table_stride) * 4, cudaMemcpyHostToDevice,
                                st));
    for (size_t done = 0; done < steps;) {
        const size_t n = std::min(steps - done, (size_t)kChainSteps);
        m.h_chain[0] = (int32_t)B;
        m.h_chain[1] = 0;
        CH_CUDA_TRY(cudaMemcpyAsync(m.b_chain, m.h_chain, 2 * 4, cudaMemcpyHostToDevice, st));
        for (size_t i = 0; i < n; ++i) {
            if (exec != nullptr) {
                CH_CUDA_TRY(cudaGraphLaunch(exec, st));
            } else if (enqueue_batch_step(m, M, table_stride, false, true) != 0) {
                return -1;
            }
        }
        CH_CUDA_TRY(cudaMemcpyAsync(m.h_log, m.b_log, n * (size_t)cap * 4, cudaMemcpyDeviceToHost, st));
        // The error word travels with the chunk's token log: a chunk that
        // tripped a device guard is reported before any of its ids are used.
        CH_CUDA_TRY(cudaMemcpyAsync(&m.h_chain[2], m.b_error, 4, cudaMemcpyDeviceToHost, st));
        CH_CUDA_TRY(cudaStreamSynchronize(st));
        if (m.h_chain[2] != 0) {
            check_batch_error(m);  // sets the message, resets the word and the tickets
            return -1;
        }
        for (size_t i = 0; i < n; ++i)
            for (size_t b = 0; b < B; ++b) tokens_out[b * steps + done + i] = (uint32_t)m.h_log[i * cap + b];
        done += n;
    }
    if (check_batch_error(m) != 0) return -1;
    for (size_t b = 0; b < B; ++b) seqs[b]->positions = offsets[b] + steps;
    return 0;
}

// Greedy decode entirely on the device: step i consumes the argmax of step
// i-1 (step 0 consumes `first_token`) at position offset+i. Pages for the
// whole run are allocated up front; nothing returns to the host between steps.
int generate_greedy(Seq *s, uint32_t first_token, size_t offset, size_t steps, uint32_t *tokens_out) {
    CH_REQUIRE(s != nullptr, "cheetah_cuda_generate_greedy: null sequence");
    const CheetahCudaConfig &c = s->m->cfg;
    CH_REQUIRE(steps > 0, "cheetah_cuda_generate_greedy: steps must be positive");
    CH_REQUIRE(first_token < c.vocab_size,
               "Native backend: token id " + std::to_string(first_token) + " exceeds the vocabulary size " +
                   std::to_string(c.vocab_size) + ".");
    CH_REQUIRE(offset == s->positions,
               "CUDA backend: offset " + std::to_string(offset) + " does not match the " +
                   std::to_string(s->positions) + " cached positions.");
    CH_REQUIRE(offset + steps <= c.max_positions,
               "CUDA backend: position " + std::to_string(offset + steps - 1) +
                   " exceeds the sequence capacity " + std::to_string(c.max_positions) + ".");
    CH_CUDA_TRY(cudaSetDevice(s->m->device));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (make_tail_page_private(*s) != 0) return -1;
    // Pages for every position of the run.
    const size_t first_page = s->pages.size();
    const size_t last_page = (offset + steps - 1) / s->m->page_tokens;
    for (size_t p = first_page; p <= last_page; ++p) {
        const int page = s->m->alloc_page();
        if (page < 0) {
            set_error("CUDA backend: KV page pool exhausted (raise kv_pool_tokens).");
            return -1;
        }
        s->pages.push_back(page);
    }
    if (last_page + 1 > first_page) {
        std::vector<int32_t> ids(s->pages.begin() + first_page, s->pages.end());
        CH_CUDA_TRY(cudaMemcpy(s->page_table + first_page, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice));
    }
    PlanGuard plan_guard(*s->m, s->stream);
    if (s->m->mk_enabled) {
        // One cooperative launch runs every step; token i is logged at i.
        if (ensure_mk_buffers(*s) != 0) return -1;
        StepState first = {};
        first.token = (int32_t)first_token;
        first.position = (int32_t)offset;
        first.seq_len = (int32_t)offset + 1;
        first.page_index = -1;
        first.page_id = -1;
        *s->h_step = first;
        CH_CUDA_TRY(cudaMemcpyAsync(s->d_step, s->h_step, sizeof(StepState), cudaMemcpyHostToDevice, s->stream));
        if (launch_megakernel(*s, (int)steps, nullptr, s->token_log) != 0) return -1;
        s->positions = offset + steps;
        if (tokens_out == nullptr) return 0;  // asynchronous: caller synchronises the stream
        std::vector<int32_t> log(steps);
        CH_CUDA_TRY(cudaMemcpyAsync(log.data(), s->token_log, steps * 4, cudaMemcpyDeviceToHost, s->stream));
        CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
        if (check_device_error(*s) != 0) {
            s->positions = offset;  // the run's K/V rows are not trusted
            return -1;
        }
        for (size_t i = 0; i < steps; ++i) tokens_out[i] = (uint32_t)log[i];
        return 0;
    }
    const bool eager = s->m->planned || !env_flag("CHEETAH_CUDA_GRAPH", true);
    if (!eager && s->chain_graph == nullptr && build_decode_graph(*s, true, &s->chain_graph) != 0) return -1;
    StepState init = {};
    init.token = (int32_t)first_token;
    init.position = (int32_t)offset - 1;
    init.seq_len = (int32_t)offset;
    init.page_index = -1;
    init.page_id = -1;
    init.chain_index = 0;
    const unsigned long long seed_key = (0xFFFFFFFFull << 32) | first_token;
    *s->h_step = init;
    *s->h_argmax = seed_key;
    CH_CUDA_TRY(cudaMemcpyAsync(s->d_step, s->h_step, sizeof(StepState), cudaMemcpyHostToDevice, s->stream));
    CH_CUDA_TRY(cudaMemcpyAsync(s->argmax, s->h_argmax, 8, cudaMemcpyHostToDevice, s->stream));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    for (size_t i = 0; i < steps; ++i) {
        if (eager) {
            if (enqueue_decode_step(*s, true) != 0) return -1;
        } else {
            CH_CUDA_TRY(cudaGraphLaunch(s->chain_graph, s->stream));
        }
    }
    s->positions = offset + steps;
    if (tokens_out == nullptr) return 0;  // asynchronous: caller synchronises the stream
    std::vector<int32_t> log(steps);
    CH_CUDA_TRY(cudaMemcpyAsync(log.data(), s->token_log, steps * 4, cudaMemcpyDeviceToHost, s->stream));
    CH_CUDA_TRY(cudaMemcpyAsync(s->h_argmax, s->argmax, 8, cudaMemcpyDeviceToHost, s->stream));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (check_device_error(*s) != 0) {
        s->positions = offset;  // the run's K/V rows are not trusted
        return -1;
    }
    for (size_t i = 0; i + 1 < steps; ++i) tokens_out[i] = (uint32_t)log[i + 1];
    tokens_out[steps - 1] = (uint32_t)(*s->h_argmax & 0xFFFFFFFFull);
    return 0;
}

// Layer, linear and unit bit of a streamable unit id
// ("model.layers.<n>.<suffix>"); false for every other unit.
bool parse_home_unit(const Model &m, const std::string &id, uint32_t *layer, int *j, int *bit) {
    static const char *kPrefix = "model.layers.";
    if (id.compare(0, 13, kPrefix) != 0) return false;
    size_t pos = 13, end = id.find('.', pos);
    if (end == std::string::npos || end == pos) return false;
    uint32_t n = 0;
    for (size_t i = pos; i < end; ++i) {
        if (id[i] < '0' || id[i] > '9') return false;
        n = n * 10 + (uint32_t)(id[i] - '0');
    }
    if (n >= m.cfg.num_layers) return false;
    const std::string suffix = id.substr(end + 1);
    static const struct {
        const char *suffix;
        int j, bit;
    } kMap[] = {{"self_attn.q_proj.weight", kHomeQkv, 0}, {"self_attn.k_proj.weight", kHomeQkv, 1},
                {"self_attn.v_proj.weight", kHomeQkv, 2}, {"self_attn.o_proj.weight", kHomeO, 0},
                {"mlp.gate_proj.weight", kHomeGate, 0},  {"mlp.up_proj.weight", kHomeUp, 0},
                {"mlp.down_proj.weight", kHomeDown, 0}};
    for (const auto &e : kMap) {
        if (suffix == e.suffix) {
            *layer = n;
            *j = e.j;
            *bit = e.bit;
            return true;
        }
    }
    return false;
}

// AntTierControl (`registry.rs:88-93`): moves one unit into HBM (resident)
// or out of it (streamed from its pinned host copy). A fused linear (q/k/v)
// is resident only while all of its units are. Units outside the layer
// linears (embedding, lm_head, norms, biases) always stay resident.
int set_unit_residency(Model *m, const char *unit_id, bool resident, int *known) {
    CH_REQUIRE(m != nullptr && unit_id != nullptr, "cheetah_cuda_model_set_residency: null argument");
    const std::string id(unit_id);
    const bool exists = m->unit_ids.count(id) != 0;
    if (known) *known = exists ? 1 : 0;
    if (!exists) return 0;
    uint32_t layer = 0;
    int j = 0, bit = 0;
    if (!parse_home_unit(*m, id, &layer, &j, &bit)) return 0;
    CH_REQUIRE(m->planned,
               "CUDA backend: the model was opened without a residency plan (cheetah_cuda_model_open_ex).");
    std::lock_guard<std::recursive_mutex> lock(m->plan_mutex);
    CH_CUDA_TRY(cudaSetDevice(m->device));
    CH_CUDA_TRY(cudaEventSynchronize(m->plan_event));  // the last forward's device work is done
    LinearHome &h = m->homes[layer][j];
    const unsigned old_bits = h.unit_bits;
    if (resident) h.unit_bits |= 1u << bit;
    else h.unit_bits &= ~(1u << bit);
    const bool want = h.unit_bits == (1u << h.units) - 1;
    if (want == h.resident) return 0;
    if (want) {
        cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&h.dev), h.bytes);
        if (e == cudaSuccess) e = cudaMemcpy(h.dev, h.host, h.bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(h.dev);
            h.dev = nullptr;
            h.unit_bits = old_bits;
            set_error(std::string("CUDA backend: Ant page-in failed: ") + cudaGetErrorString(e));
            return -1;
        }
        h.resident = true;
        return bind_linear(*m, layer, j, true);
    }
    h.resident = false;
    if (bind_linear(*m, layer, j, true) != 0) return -1;
    cudaFree(h.dev);
    h.dev = nullptr;
    return 0;
}

}  // namespace
}  // namespace cheetah

using cheetah::Model;
using cheetah::Seq;
using cheetah::Snapshot;

extern "C" {

const char *cheetah_cuda_last_error(void) { return cheetah::last_error(); }
int cheetah_cuda_abi_version(void) { return CHEETAH_CUDA_ABI_VERSION; }

#ifdef CHEETAH_MK_TRACE
// Profiling builds only: copy the persistent decode kernel's phase timestamps
// (global timer) and cycle stamps.
__attribute__((visibility("default"))) int cheetah_cuda_debug_mk_trace(unsigned long long *out) {
    CH_CUDA_TRY(cudaMemcpyFromSymbol(out, cheetah::g_mk_trace, sizeof(cheetah::g_mk_trace)));
    return 0;
}
__attribute__((visibility("default"))) int cheetah_cuda_debug_mk_cycles(long long *out) {
    CH_CUDA_TRY(cudaMemcpyFromSymbol(out, cheetah::g_mk_cycles, sizeof(cheetah::g_mk_cycles)));
    return 0;
}
__attribute__((visibility("default"))) int cheetah_cuda_debug_mk_ptrace(unsigned long long *out) {
    CH_CUDA_TRY(cudaMemcpyFromSymbol(out, cheetah::g_mk_ptrace, sizeof(cheetah::g_mk_ptrace)));
    return 0;
}
#endif

#ifdef CHEETAH_ATTN_TRACE
// Profiling builds only: copy the two-tile prefill attention kernel's
// per-key-tile timeline (kAttnTraceTiles x kAttnTraceEvents cycle stamps).
__attribute__((visibility("default"))) int cheetah_cuda_debug_attn_trace(long long *out) {
    CH_CUDA_TRY(cudaMemcpyFromSymbol(out, cheetah::g_attn_trace, sizeof(cheetah::g_attn_trace)));
    return 0;
}
#endif

int cheetah_cuda_device_count(int *count) {
    CH_REQUIRE(count != nullptr, "cheetah_cuda_device_count: null argument");
    int n = 0;
    cudaError_t err = cudaGetDeviceCount(&n);
    if (err != cudaSuccess) n = 0;
    *count = n;
    return 0;
}

int cheetah_cuda_model_open(const char *prepared_dir, const CheetahCudaConfig *config, const char *quant,
                            int device, CheetahCudaModel **out) {
    Model *m = nullptr;
    if (cheetah::open_model(prepared_dir, config, quant, device, &m) != 0) return -1;
    *out = reinterpret_cast<CheetahCudaModel *>(m);
    return 0;
}

int cheetah_cuda_model_open_ex(const char *prepared_dir, const CheetahCudaConfig *config, const char *quant,
                               int device, const CheetahCudaResidency *plan, CheetahCudaModel **out) {
    std::map<std::string, std::string> tiers;
    if (plan != nullptr) {
        CH_REQUIRE(plan->count == 0 || (plan->unit_ids != nullptr && plan->tiers != nullptr),
                   "cheetah_cuda_model_open_ex: null plan arrays");
        for (size_t i = 0; i < plan->count; ++i) {
            CH_REQUIRE(plan->unit_ids[i] != nullptr && plan->tiers[i] != nullptr,
                       "cheetah_cuda_model_open_ex: null plan entry");
            tiers[plan->unit_ids[i]] = plan->tiers[i];
        }
    }
    Model *m = nullptr;
    if (cheetah::open_model(prepared_dir, config, quant, device, &m, plan ? &tiers : nullptr) != 0) return -1;
    *out = reinterpret_cast<CheetahCudaModel *>(m);
    return 0;
}

int cheetah_cuda_model_page_in_unit(CheetahCudaModel *model, const char *unit_id, int tier, int *known) {
    CH_REQUIRE(tier >= 0 && tier <= 2, "cheetah_cuda_model_page_in_unit: tier must be 0 (vram), 1 (ram) or 2 (disk)");
    return cheetah::set_unit_residency(reinterpret_cast<Model *>(model), unit_id, tier == 0, known);
}

int cheetah_cuda_model_evict_unit(CheetahCudaModel *model, const char *unit_id, int *known) {
    return cheetah::set_unit_residency(reinterpret_cast<Model *>(model), unit_id, false, known);
}

int cheetah_cuda_model_residency(const CheetahCudaModel *model, CheetahCudaResidencyInfo *info) {
    CH_REQUIRE(model != nullptr && info != nullptr, "cheetah_cuda_model_residency: null argument");
    Model *m = const_cast<Model *>(reinterpret_cast<const Model *>(model));
    std::lock_guard<std::recursive_mutex> lock(m->plan_mutex);
    *info = CheetahCudaResidencyInfo{};
    info->planned = m->planned ? 1 : 0;
    info->staging_bytes = m->planned ? 2 * (uint64_t)m->stage_slot_bytes : 0;
    for (auto &layer : m->homes) {
        for (const cheetah::LinearHome &h : layer) {
            if (h.resident) {
                info->resident_linear_bytes += h.bytes;
                info->resident_linears += 1;
            } else {
                info->streamed_linear_bytes += h.bytes;
                info->streamed_linears += 1;
            }
        }
    }
    return 0;
}

int cheetah_cuda_model_free(CheetahCudaModel *model) {
    if (model != nullptr) cheetah::model_unref(reinterpret_cast<Model *>(model));
    return 0;
}

int cheetah_cuda_model_info(const CheetahCudaModel *model, CheetahCudaModelInfo *info) {
    CH_REQUIRE(model != nullptr && info != nullptr, "cheetah_cuda_model_info: null argument");
    Model *m = const_cast<Model *>(reinterpret_cast<const Model *>(model));
    info->weight_bytes = m->arena_used - m->mk_copy_bytes;  // distinct weights, not the decode-kernel copies
    {
        std::lock_guard<std::recursive_mutex> lock(m->plan_mutex);
        for (auto &layer : m->homes)
            for (const cheetah::LinearHome &h : layer)
                if (h.resident) info->weight_bytes += h.bytes;  // planned models' HBM-resident linears
    }
    info->kv_pool_bytes = (uint64_t)m->layer_stride_bytes * m->cfg.num_layers * 2;
    info->kv_pages_total = (uint32_t)m->num_pages;
    {
        std::lock_guard<std::mutex> lock(m->pool_mutex);
        info->kv_pages_free = (uint32_t)m->free_pages.size();
    }
    info->device = m->device;
    info->quant = m->quant;
    info->persistent_decode = m->mk_enabled ? 1 : 0;
    info->reserved = 0;
    return 0;
}

int cheetah_cuda_seq_new(CheetahCudaModel *model, CheetahCudaSeq **out) {
    Seq *s = nullptr;
    if (cheetah::new_seq(reinterpret_cast<Model *>(model), &s) != 0) return -1;
    *out = reinterpret_cast<CheetahCudaSeq *>(s);
    return 0;
}

int cheetah_cuda_seq_free(CheetahCudaSeq *seq) {
    delete reinterpret_cast<Seq *>(seq);
    return 0;
}

int cheetah_cuda_seq_clear(CheetahCudaSeq *seq) {
    CH_REQUIRE(seq != nullptr, "cheetah_cuda_seq_clear: null sequence");
    Seq *s = reinterpret_cast<Seq *>(seq);
    CH_CUDA_TRY(cudaSetDevice(s->m->device));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    s->m->release_pages(s->pages);
    s->positions = 0;
    return 0;
}

int cheetah_cuda_seq_positions(const CheetahCudaSeq *seq, size_t *positions) {
    CH_REQUIRE(seq != nullptr && positions != nullptr, "cheetah_cuda_seq_positions: null argument");
    *positions = reinterpret_cast<const Seq *>(seq)->positions;
    return 0;
}

int cheetah_cuda_forward(CheetahCudaSeq *seq, const uint32_t *tokens, size_t n, size_t offset,
                         float *logits_out) {
    return cheetah::forward_entry(reinterpret_cast<Seq *>(seq), tokens, n, offset, logits_out, nullptr);
}

int cheetah_cuda_forward_ex(CheetahCudaSeq *seq, const uint32_t *tokens, size_t n, size_t offset,
                            float *logits_out, uint32_t *argmax_out) {
    return cheetah::forward_entry(reinterpret_cast<Seq *>(seq), tokens, n, offset, logits_out, argmax_out);
}

int cheetah_cuda_model_coalesce_stats(const CheetahCudaModel *model, uint64_t *calls, uint64_t *batched_calls,
                                      uint64_t *batches) {
    CH_REQUIRE(model != nullptr && calls != nullptr && batched_calls != nullptr && batches != nullptr,
               "cheetah_cuda_model_coalesce_stats: null argument");
    const Model *m = reinterpret_cast<const Model *>(model);
    *calls = m->co_calls.load();
    *batched_calls = m->co_batched_calls.load();
    *batches = m->co_batches.load();
    return 0;
}

int cheetah_cuda_forward_batch(CheetahCudaModel *model, CheetahCudaSeq *const *seqs, const uint32_t *tokens,
                               const size_t *offsets, size_t batch, float *logits_out, uint32_t *argmax_out) {
    return cheetah::forward_batch(reinterpret_cast<Model *>(model), reinterpret_cast<Seq *const *>(seqs), tokens,
                                  offsets, batch, logits_out, argmax_out);
}

int cheetah_cuda_forward_batch_greedy(CheetahCudaModel *model, CheetahCudaSeq *const *seqs, const uint32_t *tokens,
                                      const size_t *offsets, size_t batch, size_t steps, uint32_t *tokens_out) {
    return cheetah::forward_batch_greedy(reinterpret_cast<Model *>(model), reinterpret_cast<Seq *const *>(seqs),
                                         tokens, offsets, batch, steps, tokens_out);
}

int cheetah_cuda_generate_greedy(CheetahCudaSeq *seq, uint32_t first_token, size_t offset, size_t steps,
                                 uint32_t *tokens_out) {
    return cheetah::generate_greedy(reinterpret_cast<Seq *>(seq), first_token, offset, steps, tokens_out);
}

int cheetah_cuda_seq_stream(const CheetahCudaSeq *seq, void **stream) {
    CH_REQUIRE(seq != nullptr && stream != nullptr, "cheetah_cuda_seq_stream: null argument");
    *stream = reinterpret_cast<const Seq *>(seq)->stream;
    return 0;
}

int cheetah_cuda_model_batch_stream(const CheetahCudaModel *model, void **stream) {
    CH_REQUIRE(model != nullptr && stream != nullptr, "cheetah_cuda_model_batch_stream: null argument");
    *stream = reinterpret_cast<const Model *>(model)->batch_stream;
    return 0;
}

int cheetah_cuda_seq_snapshot(const CheetahCudaSeq *seq, CheetahCudaSnapshot **out) {
    CH_REQUIRE(seq != nullptr && out != nullptr, "cheetah_cuda_seq_snapshot: null argument");
    Seq *s = const_cast<Seq *>(reinterpret_cast<const Seq *>(seq));
    CH_CUDA_TRY(cudaSetDevice(s->m->device));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));  // the captured rows are written
    // The snapshot holds the pages of the cached positions: no copy. Whoever
    // appends into the last (partial) page later copies it first.
    Snapshot *snap = new Snapshot();
    snap->m = s->m;
    s->m->refs.fetch_add(1);
    snap->positions = s->positions;
    const size_t n = (s->positions + s->m->page_tokens - 1) / s->m->page_tokens;
    snap->pages.assign(s->pages.begin(), s->pages.begin() + n);
    s->m->retain_pages(snap->pages);
    *out = reinterpret_cast<CheetahCudaSnapshot *>(snap);
    return 0;
}

int cheetah_cuda_snapshot_positions(const CheetahCudaSnapshot *snapshot, size_t *positions) {
    CH_REQUIRE(snapshot != nullptr && positions != nullptr, "cheetah_cuda_snapshot_positions: null argument");
    *positions = reinterpret_cast<const Snapshot *>(snapshot)->positions;
    return 0;
}

int cheetah_cuda_seq_restore_prefix(CheetahCudaSeq *seq, const CheetahCudaSnapshot *snapshot, size_t positions) {
    CH_REQUIRE(seq != nullptr && snapshot != nullptr, "cheetah_cuda_seq_restore_prefix: null argument");
    Seq *s = reinterpret_cast<Seq *>(seq);
    const Snapshot *snap = reinterpret_cast<const Snapshot *>(snapshot);
    CH_REQUIRE(snap->m == s->m, "CUDA backend: snapshot belongs to another model.");
    CH_CUDA_TRY(cudaSetDevice(s->m->device));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    s->m->release_pages(s->pages);
    s->positions = 0;
    // The sequence shares the snapshot's pages of the kept positions.
    const size_t keep = std::min(positions, snap->positions);
    const size_t pages = (keep + s->m->page_tokens - 1) / s->m->page_tokens;
    s->pages.assign(snap->pages.begin(), snap->pages.begin() + pages);
    s->m->retain_pages(s->pages);
    std::vector<int32_t> table(s->pages.begin(), s->pages.end());
    if (!table.empty()) {
        CH_CUDA_TRY(cudaMemcpy(s->page_table, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
    }
    s->positions = keep;
    return 0;
}

int cheetah_cuda_snapshot_free(CheetahCudaSnapshot *snapshot) {
    delete reinterpret_cast<Snapshot *>(snapshot);
    return 0;
}

int cheetah_cuda_seq_export_kv(const CheetahCudaSeq *seq, size_t layer, float *k_out, float *v_out) {
    CH_REQUIRE(seq != nullptr && k_out != nullptr && v_out != nullptr, "cheetah_cuda_seq_export_kv: null argument");
    const Seq *s = reinterpret_cast<const Seq *>(seq);
    const Model *m = s->m;
    CH_REQUIRE(layer < m->cfg.num_layers, "cheetah_cuda_seq_export_kv: layer out of range");
    CH_CUDA_TRY(cudaSetDevice(m->device));
    CH_CUDA_TRY(cudaStreamSynchronize(s->stream));
    const size_t n = s->positions * m->cfg.kv_heads * m->cfg.head_dim;
    if (n == 0) return 0;
    float *d_out = nullptr;
    int32_t *d_pages = nullptr;
    CH_CUDA_TRY(cudaMalloc(&d_out, n * 4));
    cudaError_t err = cudaMalloc(&d_pages, s->pages.size() * 4);
    std::vector<int32_t> pages(s->pages.begin(), s->pages.end());
    if (err == cudaSuccess) err = cudaMemcpy(d_pages, pages.data(), pages.size() * 4, cudaMemcpyHostToDevice);
    for (int which = 0; which < 2 && err == cudaSuccess; ++which) {
        const uint8_t *pool = (which ? m->v_pool : m->k_pool) + layer * m->layer_stride_bytes;
        cheetah::export_kv_kernel<<<256, 256, 0, s->stream>>>(pool, m->kv_f32, d_pages, (int)s->positions,
                                                              (int)m->cfg.kv_heads, m->page_tokens,
                                                              (int)m->cfg.head_dim, d_out);
        err = cudaGetLastError();
        if (err == cudaSuccess) err = cudaStreamSynchronize(s->stream);
        if (err == cudaSuccess) err = cudaMemcpy(which ? v_out : k_out, d_out, n * 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(d_out);
    cudaFree(d_pages);
    CH_CUDA_TRY(err);
    return 0;
}

int cheetah_cuda_op_gemv_bf16(const void *weight, size_t rows, size_t cols, const float *x, size_t batch,
                              float *y, void *stream) {
    CH_REQUIRE(weight != nullptr && x != nullptr && y != nullptr, "cheetah_cuda_op_gemv_bf16: null argument");
    CH_REQUIRE(cols % 8 == 0 && cols > 0 && rows > 0, "cheetah_cuda_op_gemv_bf16: cols must be a positive multiple of 8");
    CH_REQUIRE(((uintptr_t)weight & 15) == 0 && ((uintptr_t)x & 15) == 0,
               "cheetah_cuda_op_gemv_bf16: weight and x must be 16-byte aligned");
    CH_REQUIRE(rows < (1u << 31) && cols < (1u << 24), "cheetah_cuda_op_gemv_bf16: shape too large");
    int device = 0;
    CH_CUDA_TRY(cudaGetDevice(&device));
    const int sms = cheetah::sm_count(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (size_t b0 = 0; b0 < batch; ++b0) {
        cheetah::GemvParams p = {};
        p.w0 = static_cast<const uint16_t *>(weight);
        p.rows = (int)rows;
        p.cols = (int)cols;
        p.batch = 1;
        p.x = x + b0 * cols;
        p.x_stride = (long long)cols;
        p.y = y + b0 * rows;
        p.y_stride = (long long)rows;
        if (cheetah::run_gemv<cheetah::kEpiStore>(p, st, false, sms) != 0) return -1;
    }
    return 0;
}

int cheetah_cuda_quant_buffer_bytes(const char *format, size_t rows, size_t cols, size_t *bytes) {
    CH_REQUIRE(format != nullptr && bytes != nullptr, "cheetah_cuda_quant_buffer_bytes: null argument");
    const std::string f = format;
    if (f == "q8") *bytes = rows * 4 + rows * (size_t)cheetah::q8_row_bytes((long long)cols);
    else if (f == "q4") *bytes = rows * 4 + rows * (size_t)cheetah::q4_row_bytes((long long)cols);
    else CH_REQUIRE(false, "cheetah_cuda_quant_buffer_bytes: format must be q8 or q4");
    return 0;
}

static int op_quantize(int bits, const void *weight, size_t rows, size_t cols, void *out, void *stream) {
    CH_REQUIRE(weight != nullptr && out != nullptr, "cheetah_cuda_op_quantize: null argument");
    CH_REQUIRE(rows > 0 && cols > 0 && rows < (1u << 30) && cols < (1u << 30), "cheetah_cuda_op_quantize: bad shape");
    CH_REQUIRE(((uintptr_t)out & 3) == 0, "cheetah_cuda_op_quantize: output must be 4-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int blocks = (int)((rows * cheetah::kWarp + 255) / 256);
    if (bits == 8) {
        cheetah::quantize_rows_kernel<8><<<blocks, 256, 0, st>>>(static_cast<const uint16_t *>(weight), (int)rows, (int)cols,
                                                                  static_cast<uint8_t *>(out));
    } else {
        cheetah::quantize_rows_kernel<4><<<blocks, 256, 0, st>>>(static_cast<const uint16_t *>(weight), (int)rows, (int)cols,
                                                                  static_cast<uint8_t *>(out));
    }
    CH_CUDA_TRY(cudaGetLastError());
    return 0;
}

int cheetah_cuda_op_quantize_q8(const void *weight, size_t rows, size_t cols, void *out, void *stream) {
    return op_quantize(8, weight, rows, cols, out, stream);
}

int cheetah_cuda_op_quantize_q4(const void *weight, size_t rows, size_t cols, void *out, void *stream) {
    return op_quantize(4, weight, rows, cols, out, stream);
}

static int op_gemv_quant(int wt, const void *buffer, size_t rows, size_t cols, const float *x, size_t batch, float *y,
                         void *stream) {
    CH_REQUIRE(buffer != nullptr && x != nullptr && y != nullptr, "cheetah_cuda_op_gemv_q: null argument");
    CH_REQUIRE(cols % 8 == 0 && cols > 0 && rows > 0, "cheetah_cuda_op_gemv_q: cols must be a positive multiple of 8");
    CH_REQUIRE(rows < (1u << 30) && cols < (1u << 24), "cheetah_cuda_op_gemv_q: shape too large");
    CH_REQUIRE(((uintptr_t)buffer & 3) == 0 && ((uintptr_t)x & 15) == 0,
               "cheetah_cuda_op_gemv_q: buffer must be 4-byte and x 16-byte aligned");
    int device = 0;
    CH_CUDA_TRY(cudaGetDevice(&device));
    const int sms = cheetah::sm_count(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long rb = wt == cheetah::kWQ8 ? cheetah::q8_row_bytes((long long)cols) : cheetah::q4_row_bytes((long long)cols);
    for (size_t b0 = 0; b0 < batch; ++b0) {
        cheetah::GemvParams p = {};
        p.w0 = reinterpret_cast<const uint16_t *>(static_cast<const uint8_t *>(buffer) + rows * 4);
        p.scale0 = static_cast<const float *>(buffer);
        p.row_stride = rb;
        p.wt = wt;
        p.rows = (int)rows;
        p.cols = (int)cols;
        p.batch = 1;
        p.x = x + b0 * cols;
        p.x_stride = (long long)cols;
        p.y = y + b0 * rows;
        p.y_stride = (long long)rows;
        if (cheetah::run_gemv<cheetah::kEpiStore>(p, st, false, sms) != 0) return -1;
    }
    return 0;
}

int cheetah_cuda_op_gemv_q8(const void *buffer, size_t rows, size_t cols, const float *x, size_t batch, float *y,
                            void *stream) {
    return op_gemv_quant(cheetah::kWQ8, buffer, rows, cols, x, batch, y, stream);
}

int cheetah_cuda_op_gemv_q4(const void *buffer, size_t rows, size_t cols, const float *x, size_t batch, float *y,
                            void *stream) {
    return op_gemv_quant(cheetah::kWQ4, buffer, rows, cols, x, batch, y, stream);
}

// Split-merge scratch for the op entry, cached per (device, stream) and grown
// on demand; calls on one stream are ordered, so they may share it. Merge
// tickets live in their own buffer, zeroed when (re)allocated: every launch
// returns the tickets it used to zero, so any later layout finds zeros.
struct OpScratch {
    uint8_t *partials = nullptr;
    size_t partial_bytes = 0;
    unsigned int *tickets = nullptr;
    size_t ticket_count = 0;
};
static std::mutex g_op_scratch_mutex;
static std::map<std::pair<int, cudaStream_t>, OpScratch> g_op_scratch;

static int op_scratch(int device, cudaStream_t stream, size_t partial_bytes, size_t tickets,
                      uint8_t **partials_out, unsigned int **tickets_out) {
    std::lock_guard<std::mutex> lock(g_op_scratch_mutex);
    OpScratch &s = g_op_scratch[{device, stream}];
    if (s.partial_bytes < partial_bytes || s.ticket_count < tickets) {
        CH_CUDA_TRY(cudaStreamSynchronize(stream));
    }
    if (s.partial_bytes < partial_bytes) {
        cudaFree(s.partials);
        s.partials = nullptr;
        s.partial_bytes = 0;
        CH_CUDA_TRY(cudaMalloc(&s.partials, partial_bytes));
        s.partial_bytes = partial_bytes;
    }
    if (s.ticket_count < tickets) {
        cudaFree(s.tickets);
        s.tickets = nullptr;
        s.ticket_count = 0;
        CH_CUDA_TRY(cudaMalloc(&s.tickets, tickets * sizeof(unsigned int)));
        CH_CUDA_TRY(cudaMemsetAsync(s.tickets, 0, tickets * sizeof(unsigned int), stream));
        s.ticket_count = tickets;
    }
    *partials_out = s.partials;
    *tickets_out = s.tickets;
    return 0;
}

int cheetah_cuda_op_decode_attention(const CheetahCudaDecodeAttention *a, void *stream) {
    CH_REQUIRE(a != nullptr && a->q && a->k_pool && a->v_pool && a->page_table && a->seq_lens && a->out,
               "cheetah_cuda_op_decode_attention: null argument");
    CH_REQUIRE(a->head_dim == 64 || a->head_dim == 128, "cheetah_cuda_op_decode_attention: head_dim must be 64 or 128");
    CH_REQUIRE(a->kv_heads > 0 && a->q_heads % a->kv_heads == 0 && a->q_heads / a->kv_heads <= (uint32_t)cheetah::kMaxGroup,
               "cheetah_cuda_op_decode_attention: q_heads must be a multiple of kv_heads (group <= 8)");
    CH_REQUIRE(a->page_tokens > 0 && a->batch > 0 && a->num_pages > 0, "cheetah_cuda_op_decode_attention: empty shape");
    CH_REQUIRE(a->kv_dtype == CHEETAH_CUDA_KV_BF16 || a->kv_dtype == CHEETAH_CUDA_KV_F32,
               "cheetah_cuda_op_decode_attention: unknown kv_dtype");
    CH_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->out & 15) == 0,
               "cheetah_cuda_op_decode_attention: q and out must be 16-byte aligned");
    int device = 0;
    CH_CUDA_TRY(cudaGetDevice(&device));
    const int sms = cheetah::sm_count(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool mma = a->kv_dtype == CHEETAH_CUDA_KV_BF16 &&
                     cheetah::mma_attention_eligible((int)a->head_dim, (int)a->page_tokens);
    cheetah::AttnParams p = {};
    p.q = a->q;
    p.k_pool = a->k_pool;
    p.v_pool = a->v_pool;
    p.page_table = a->page_table;
    p.seq_lens = a->seq_lens;
    p.max_pages = (int)a->max_pages_per_seq;
    p.num_pages = (int)a->num_pages;
    p.page_tokens = (int)a->page_tokens;
    p.batch = (int)a->batch;
    p.q_heads = (int)a->q_heads;
    p.kv_heads = (int)a->kv_heads;
    p.window = (int)a->sliding_window;
    p.splits = mma ? cheetah::mma_attention_splits((int)a->batch, (int)a->kv_heads, sms)
                   : cheetah::attention_splits((int)a->batch, (int)a->kv_heads,
                                               (int)std::max<uint32_t>(1, a->max_seq_len), sms);
    p.scale = 1.0f / sqrtf((float)a->head_dim);
    p.out = a->out;
    const size_t parts = (size_t)a->batch * a->kv_heads * p.splits;
    const size_t o_bytes = (parts * cheetah::kMaxGroup * a->head_dim * 4 + 255) & ~size_t(255);
    const size_t ml_bytes = (parts * cheetah::kMaxGroup * 2 * 4 + 255) & ~size_t(255);
    uint8_t *scratch = nullptr;
    unsigned int *tickets = nullptr;
    if (op_scratch(device, st, o_bytes + ml_bytes, (size_t)a->batch * a->kv_heads, &scratch, &tickets) != 0) {
        return -1;
    }
    p.part_o = reinterpret_cast<float *>(scratch);
    p.part_ml = reinterpret_cast<float *>(scratch + o_bytes);
    p.tickets = tickets;
    p.error = nullptr;
    if (!mma) return cheetah::launch_attention(p, (int)a->head_dim, a->kv_dtype == CHEETAH_CUDA_KV_F32, st, true);
    CUtensorMap k_map, v_map;
    const unsigned long long rows = (unsigned long long)a->num_pages * a->kv_heads * a->page_tokens;
    if (cheetah::make_kv_tensor_map(&k_map, a->k_pool, rows, (int)a->head_dim) != 0 ||
        cheetah::make_kv_tensor_map(&v_map, a->v_pool, rows, (int)a->head_dim) != 0) {
        return -1;
    }
    cheetah::MmaAttnParams mp = {};
    mp.a = p;
    mp.layer_row_offset = 0;
    mp.page_tokens = (int)a->page_tokens;
    // Programmatic dependent launch: the kernel sets up its barriers while
    // the stream's previous kernel drains, and reads nothing before that
    // kernel has completed (griddepcontrol.wait).
    return cheetah::launch_attention_mma(k_map, v_map, mp, (int)a->head_dim, st, true);
}

int cheetah_cuda_op_prefill_attention(const CheetahCudaPrefillAttention *a, void *stream) {
    CH_REQUIRE(a != nullptr && a->q && a->k_pool && a->v_pool && a->page_table && a->out,
               "cheetah_cuda_op_prefill_attention: null argument");
    CH_REQUIRE(a->head_dim == 64 || a->head_dim == 128, "cheetah_cuda_op_prefill_attention: head_dim must be 64 or 128");
    CH_REQUIRE(a->kv_heads > 0 && a->q_heads % a->kv_heads == 0 && a->q_heads / a->kv_heads <= (uint32_t)cheetah::kMaxGroup,
               "cheetah_cuda_op_prefill_attention: q_heads must be a multiple of kv_heads (group <= 8)");
    CH_REQUIRE(a->tokens > 0 && a->num_pages > 0 && a->max_pages > 0,
               "cheetah_cuda_op_prefill_attention: empty shape");
    CH_REQUIRE(a->page_tokens > 0 && a->page_tokens % 64 == 0,
               "cheetah_cuda_op_prefill_attention: page_tokens must be a multiple of 64");
    CH_REQUIRE((uint64_t)a->offset + a->tokens <= (uint64_t)a->max_pages * a->page_tokens,
               "cheetah_cuda_op_prefill_attention: query rows past the page table");
    CH_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->out & 15) == 0 && ((uintptr_t)a->k_pool & 15) == 0 &&
                   ((uintptr_t)a->v_pool & 15) == 0,
               "cheetah_cuda_op_prefill_attention: q, out and the pools must be 16-byte aligned");
    int device = 0;
    CH_CUDA_TRY(cudaGetDevice(&device));
    const int sms = cheetah::sm_count(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t T = a->tokens, QD = (size_t)a->q_heads * a->head_dim;
    const size_t o_bytes = ((size_t)cheetah::kPrefillMaxSplits * T * QD * 4 + 255) & ~size_t(255);
    const size_t ml_bytes = ((size_t)cheetah::kPrefillMaxSplits * T * a->q_heads * 2 * 4 + 255) & ~size_t(255);
    uint8_t *scratch = nullptr;
    unsigned int *tickets = nullptr;
    if (op_scratch(device, st, o_bytes + ml_bytes, 1, &scratch, &tickets) != 0) return -1;
    CUtensorMap q_map, k_map, v_map;
    const unsigned long long rows = (unsigned long long)a->num_pages * a->kv_heads * a->page_tokens;
    if (cheetah::make_bf16_tensor_map(&q_map, a->q, T, QD, cheetah::kTcRows) != 0 ||
        cheetah::make_kv_tensor_map(&k_map, a->k_pool, rows, (int)a->head_dim) != 0 ||
        cheetah::make_kv_tensor_map(&v_map, a->v_pool, rows, (int)a->head_dim) != 0) {
        return -1;
    }
    cheetah::PrefillAttnParams ap = {};
    ap.q = static_cast<const uint16_t *>(a->q);
    ap.out = static_cast<uint16_t *>(a->out);
    ap.T = (int)T;
    ap.offset = (int)a->offset;
    ap.q_heads = (int)a->q_heads;
    ap.kv_heads = (int)a->kv_heads;
    ap.page_table = a->page_table;
    ap.max_pages = (int)a->max_pages;
    ap.num_pages = (int)a->num_pages;
    ap.page_tokens = (int)a->page_tokens;
    ap.layer_row_offset = 0;
    ap.window = (int)a->sliding_window;
    ap.scale = 1.0f / sqrtf((float)a->head_dim);
    ap.error = nullptr;
    ap.part_o = reinterpret_cast<float *>(scratch);
    ap.part_ml = reinterpret_cast<float *>(scratch + o_bytes);
    return cheetah::launch_prefill_attention(ap, q_map, k_map, v_map, (int)a->head_dim, a->offset, sms, st, false);
}

// ---- Decode attention without allocation ----------------------------------
// Some callers cannot let the library allocate device memory: a caller that
// manages a fixed device-memory budget itself, or a latency-critical caller
// that cannot absorb the device-wide synchronisation cudaMalloc / cudaFree
// may cause. This entry point computes
// the same attention as cheetah_cuda_op_decode_attention, but its split-merge
// scratch is a fixed array compiled into the library (held by every GPU that
// loads it, until exit) instead of memory allocated on first use.
constexpr int kNoAllocMaxParts = 1024;  // (sequence, kv head, split) partials
constexpr int kNoAllocMaxPairs = 1024;  // (sequence, kv head) merge tickets
constexpr size_t kNoAllocOBytes = (size_t)kNoAllocMaxParts * cheetah::kMaxGroup * 128 * sizeof(float);
constexpr size_t kNoAllocMlBytes = (size_t)kNoAllocMaxParts * cheetah::kMaxGroup * 2 * sizeof(float);
constexpr size_t kNoAllocTicketBytes = (size_t)kNoAllocMaxPairs * sizeof(unsigned int);
constexpr size_t kNoAllocScratchBytes = kNoAllocOBytes + kNoAllocMlBytes + kNoAllocTicketBytes;  // ~4.1 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (the host-side symbol is only a stand-in, not an address).
static std::mutex g_noalloc_mutex;
static std::map<int, uint8_t *> g_noalloc_ptrs;

static int noalloc_scratch(int device, uint8_t **out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    auto it = g_noalloc_ptrs.find(device);
    if (it == g_noalloc_ptrs.end()) {
        void *ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        CH_REQUIRE(err == cudaSuccess && ptr != nullptr,
                   std::string("cheetah_cuda_op_decode_attention_noalloc: cudaGetSymbolAddress failed: ") +
                       cudaGetErrorString(err));
        it = g_noalloc_ptrs.emplace(device, static_cast<uint8_t *>(ptr)).first;
    }
    *out = it->second;
    return 0;
}

int cheetah_cuda_op_decode_attention_noalloc(const CheetahCudaDecodeAttention *a, void *stream) {
    CH_REQUIRE(a != nullptr && a->q && a->k_pool && a->v_pool && a->page_table && a->seq_lens && a->out,
               "cheetah_cuda_op_decode_attention_noalloc: null argument");
    CH_REQUIRE(a->head_dim == 64 || a->head_dim == 128,
               "cheetah_cuda_op_decode_attention_noalloc: head_dim must be 64 or 128");
    CH_REQUIRE(a->kv_heads > 0 && a->q_heads % a->kv_heads == 0 && a->q_heads / a->kv_heads <= (uint32_t)cheetah::kMaxGroup,
               "cheetah_cuda_op_decode_attention_noalloc: q_heads must be a multiple of kv_heads (group <= 8)");
    CH_REQUIRE(a->page_tokens > 0 && a->batch > 0 && a->num_pages > 0,
               "cheetah_cuda_op_decode_attention_noalloc: empty shape");
    CH_REQUIRE(a->kv_dtype == CHEETAH_CUDA_KV_BF16 || a->kv_dtype == CHEETAH_CUDA_KV_F32,
               "cheetah_cuda_op_decode_attention_noalloc: unknown kv_dtype");
    CH_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->out & 15) == 0,
               "cheetah_cuda_op_decode_attention_noalloc: q and out must be 16-byte aligned");
    const size_t pairs = (size_t)a->batch * a->kv_heads;
    CH_REQUIRE(pairs <= (size_t)kNoAllocMaxPairs,
               "cheetah_cuda_op_decode_attention_noalloc: batch * kv_heads = " + std::to_string(pairs) +
                   " exceeds the fixed scratch limit of " + std::to_string(kNoAllocMaxPairs) + " sequence-head pairs");
    int device = 0;
    CH_CUDA_TRY(cudaGetDevice(&device));
    uint8_t *scratch = nullptr;
    if (noalloc_scratch(device, &scratch) != 0) return -1;
    const int sms = cheetah::sm_count(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool mma = a->kv_dtype == CHEETAH_CUDA_KV_BF16 &&
                     cheetah::mma_attention_eligible((int)a->head_dim, (int)a->page_tokens);
    cheetah::AttnParams p = {};
    p.q = a->q;
    p.k_pool = a->k_pool;
    p.v_pool = a->v_pool;
    p.page_table = a->page_table;
    p.seq_lens = a->seq_lens;
    p.max_pages = (int)a->max_pages_per_seq;
    p.num_pages = (int)a->num_pages;
    p.page_tokens = (int)a->page_tokens;
    p.batch = (int)a->batch;
    p.q_heads = (int)a->q_heads;
    p.kv_heads = (int)a->kv_heads;
    p.window = (int)a->sliding_window;
    int splits = mma ? cheetah::mma_attention_splits((int)a->batch, (int)a->kv_heads, sms)
                     : cheetah::attention_splits((int)a->batch, (int)a->kv_heads,
                                                 (int)std::max<uint32_t>(1, a->max_seq_len), sms);
    splits = std::max(1, std::min(splits, (int)(kNoAllocMaxParts / pairs)));  // fit the fixed partials
    p.splits = splits;
    p.scale = 1.0f / sqrtf((float)a->head_dim);
    p.out = a->out;
    p.part_o = reinterpret_cast<float *>(scratch);
    p.part_ml = reinterpret_cast<float *>(scratch + kNoAllocOBytes);
    p.tickets = reinterpret_cast<unsigned int *>(scratch + kNoAllocOBytes + kNoAllocMlBytes);
    p.error = nullptr;
    // The array keeps whatever the previous call left: clear the tickets this
    // call counts on (every completed launch also returns them to zero).
    CH_CUDA_TRY(cudaMemsetAsync(p.tickets, 0, pairs * sizeof(unsigned int), st));
    if (!mma) return cheetah::launch_attention(p, (int)a->head_dim, a->kv_dtype == CHEETAH_CUDA_KV_F32, st, false);
    CUtensorMap k_map, v_map;
    const unsigned long long rows = (unsigned long long)a->num_pages * a->kv_heads * a->page_tokens;
    if (cheetah::make_kv_tensor_map(&k_map, a->k_pool, rows, (int)a->head_dim) != 0 ||
        cheetah::make_kv_tensor_map(&v_map, a->v_pool, rows, (int)a->head_dim) != 0) {
        return -1;
    }
    cheetah::MmaAttnParams mp = {};
    mp.a = p;
    mp.layer_row_offset = 0;
    mp.page_tokens = (int)a->page_tokens;
    return cheetah::launch_attention_mma(k_map, v_map, mp, (int)a->head_dim, st, false);
}

}  // extern "C"
