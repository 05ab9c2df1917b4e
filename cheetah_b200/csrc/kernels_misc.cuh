// Small kernels around the decode step: embedding gather, KV page copies.
#pragma once

#include "common.cuh"

namespace cheetah {

// Step state shared by the captured decode graphs. The per-token graph copies
// it from pinned host memory as its first node; the greedy-chain graph
// advances it on the device (position + 1, token = previous argmax).
struct StepState {
    int32_t token;
    int32_t position;    // absolute position of this token
    int32_t seq_len;     // position + 1
    int32_t page_index;  // page-table slot to set this step, or -1
    int32_t page_id;     // pool page for that slot
    int32_t chain_index; // greedy chain: steps taken so far
    int32_t pad[2];
};

// `OpsToolbox::embedding_row_into` (`ops.rs:1083-1099`): widen one bf16 row to
// the f32 residual stream. Also resets the step's argmax slot and installs a
// freshly allocated KV page in the page table. In chain mode the input token
// is the previous step's greedy argmax (`engine.rs:2247-2253`) and the
// position advances on the device. One CTA, so the argmax slot is read
// before it is reset.
__global__ void embed_kernel(const uint16_t *table, int hidden, StepState *step, float *out,
                             unsigned long long *argmax, int32_t *page_table, int chain,
                             int32_t *token_log) {
    __shared__ long long token_s;
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        int32_t token;
        if (chain) {
            token = (int32_t)(*argmax & 0xFFFFFFFFull);
            const int32_t pos = step->position + 1;
            step->position = pos;
            step->seq_len = pos + 1;
            step->token = token;
            if (token_log) token_log[step->chain_index] = token;
            step->chain_index += 1;
        } else {
            token = step->token;
            if (step->page_index >= 0) page_table[step->page_index] = step->page_id;
        }
        token_s = token;
        if (argmax) *argmax = 0ull;
    }
    __syncthreads();
    const uint16_t *row = table + token_s * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) out[i] = bf16_to_f32(row[i]);
}

// Copy whole KV pages (every layer, K and V) from src ids to dst ids.
// Pool layout per layer: [pages][page_elems].
__global__ void copy_pages_kernel(const int32_t *src, const int32_t *dst, int count,
                                  uint8_t *k_pool, uint8_t *v_pool, long long layer_stride_bytes,
                                  int layers, long long page_bytes) {
    const long long vec_per_page = page_bytes / 16;
    const long long total = (long long)count * layers * 2 * vec_per_page;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long v = i % vec_per_page;
        long long rest = i / vec_per_page;
        const int which = rest % 2;
        rest /= 2;
        const int layer = rest % layers;
        const int n = static_cast<int>(rest / layers);
        uint8_t *pool = which ? v_pool : k_pool;
        const uint4 *s = reinterpret_cast<const uint4 *>(pool + layer * layer_stride_bytes + src[n] * page_bytes) + v;
        uint4 *d = reinterpret_cast<uint4 *>(pool + layer * layer_stride_bytes + dst[n] * page_bytes) + v;
        *d = *s;
    }
}

// Widen a layer's paged cache into a dense f32 [positions][kv_heads*head_dim]
// view (diagnostics / parity tests).
__global__ void export_kv_kernel(const void *pool, int kv_f32, const int32_t *pages, int positions,
                                 int kv_heads, int page_tokens, int head_dim, float *out) {
    const long long total = (long long)positions * kv_heads * head_dim;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int d = i % head_dim;
        const int h = (i / head_dim) % kv_heads;
        const int pos = static_cast<int>(i / ((long long)head_dim * kv_heads));
        const int page = pages[pos / page_tokens];
        const long long idx = (((long long)page * kv_heads + h) * page_tokens + pos % page_tokens) * head_dim + d;
        out[i] = kv_f32 ? static_cast<const float *>(pool)[idx]
                        : bf16_to_f32(static_cast<const uint16_t *>(pool)[idx]);
    }
}

}  // namespace cheetah
