/* cheetah_cuda — B200 (sm_100a) backend for Cheetah's decoder hot path.
 *
 * A C-ABI shared library (libcheetah_cuda.so) that the reference's Rust host
 * binds beside its Vulkan substrate (`src/native.rs:927` `mod vulkan` is the
 * sibling; this is `mod cuda`). Style follows `cheetah_vulkan.h`: opaque
 * handles, `int` status (0 = success, negative = failure) and a thread-local
 * last-error string. No function aborts or exits the process.
 *
 * Two layers:
 *  - Model / sequence entries implement the reference's `ModelForward`
 *    boundary (`src/chat/registry.rs:57-85`): `forward(tokens, offset)` returns
 *    the final position's vocabulary logits; `clear_cache`, `kv_snapshot`,
 *    `restore_kv_prefix`. Host buffers in and out; the library owns all
 *    device memory (weights HBM-resident, paged KV pool).
 *  - Op entries (`cheetah_cuda_op_*`) expose single kernels over caller-owned
 *    DEVICE buffers on a caller stream (`cudaStream_t` passed as void*), one
 *    per reference math kernel they replace.
 */
#ifndef CHEETAH_CUDA_H
#define CHEETAH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHEETAH_CUDA_ABI_VERSION 2

#if defined(__GNUC__)
#define CHEETAH_CUDA_API __attribute__((visibility("default")))
#else
#define CHEETAH_CUDA_API
#endif

/* KV cache element types. BF16 halves KV traffic; F32 mirrors the
 * reference's f32 cache (`ops.rs:995-999`) for parity runs. */
enum { CHEETAH_CUDA_KV_BF16 = 0, CHEETAH_CUDA_KV_F32 = 1 };

/* Resolved decoder hyper-parameters. Replaces the fields of the reference's
 * `DecoderConfig` (`src/chat/native/decoder.rs:29-92`) that the Qwen2 path
 * reads; the Rust loader fills it from `DecoderConfig::resolve`
 * (`decoder.rs:260-486`). */
typedef struct CheetahCudaConfig {
    uint32_t hidden_size;
    uint32_t num_layers;
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t rotary_dim;
    uint32_t intermediate_size;
    uint32_t vocab_size;
    float rms_eps;
    float rope_theta;
    int32_t tie_word_embeddings;
    uint32_t sliding_window;   /* 0 = full attention */
    uint32_t max_positions;    /* per-sequence capacity (rope table, page table) */
    uint32_t kv_page_tokens;   /* tokens per KV page; 0 = 64 (CHEETAH_CUDA_KV_PAGE) */
    uint32_t kv_pool_tokens;   /* KV pool size in tokens; 0 = default */
    int32_t kv_dtype;          /* CHEETAH_CUDA_KV_* */
} CheetahCudaConfig;

typedef struct CheetahCudaModel CheetahCudaModel;
typedef struct CheetahCudaSeq CheetahCudaSeq;
typedef struct CheetahCudaSnapshot CheetahCudaSnapshot;

typedef struct CheetahCudaModelInfo {
    uint64_t weight_bytes;    /* bytes of weights resident in HBM */
    uint64_t kv_pool_bytes;   /* bytes of the KV page pool */
    uint32_t kv_pages_total;
    uint32_t kv_pages_free;
    int32_t device;
    int32_t quant;            /* 0 bf16, 1 q8, 2 q4 */
    int32_t persistent_decode; /* 1: single-sequence decode runs as one persistent kernel */
    int32_t reserved;
} CheetahCudaModelInfo;

/* Thread-local description of the last failure on this thread
 * (mirrors `check_native_result`, `src/native.rs:1860-1870`). */
CHEETAH_CUDA_API const char *cheetah_cuda_last_error(void);
CHEETAH_CUDA_API int cheetah_cuda_abi_version(void);
CHEETAH_CUDA_API int cheetah_cuda_device_count(int *count);

/* Open a prepared model directory (`cheetah init` layout: cheetah_units.json
 * + .cheetah/weights/*.safetensors, read as `store.rs:74-157` does) and make
 * every unit HBM-resident on `device`. `quant` is "bf16", "q8" or "q4"
 * (selected like `CHEETAH_QUANT_Q8/Q4`, `precision.rs:348`). Replaces
 * `qwen2_native_loader` (`qwen2.rs:654`) + `OpsToolbox::open` (`ops.rs:1051`). */
CHEETAH_CUDA_API int cheetah_cuda_model_open(const char *prepared_dir, const CheetahCudaConfig *config,
                            const char *quant, int device, CheetahCudaModel **out);
CHEETAH_CUDA_API int cheetah_cuda_model_free(CheetahCudaModel *model);
CHEETAH_CUDA_API int cheetah_cuda_model_info(const CheetahCudaModel *model, CheetahCudaModelInfo *info);

/* Ant residency plan: the loader's `plan` argument (unit id -> "vram" /
 * "ram" / "disk", `BackendLoader` `registry.rs:138-146`, produced by
 * `Ant::plan_residency` `ant.rs:655-710`). Units it does not list are "vram". */
typedef struct CheetahCudaResidency {
    const char *const *unit_ids;
    const char *const *tiers;
    size_t count;
} CheetahCudaResidency;

/* `cheetah_cuda_model_open` with the Ant VRAM tier (`ant.rs:667-710`,
 * `cheetah_memory.h:12-16`; the reference's GPU backend buckets weights the
 * same way, `vulkan/transformer.rs:484-560`). The layer linears (q/k/v fused,
 * o, gate, up, down) planned into "vram" get their own HBM copy; the others
 * are kept in pinned host memory and streamed into one of two per-model
 * staging slots (layer parity) before their layer runs, in every forward.
 * A fused q/k/v linear is resident only when all three units are. The
 * embedding, lm_head, norms and biases are always HBM-resident. A planned
 * model runs without CUDA graphs, programmatic dependent launch or the
 * persistent decode kernel, and serialises its forwards (the staging slots
 * are shared). plan == NULL is `cheetah_cuda_model_open`. */
CHEETAH_CUDA_API int cheetah_cuda_model_open_ex(const char *prepared_dir, const CheetahCudaConfig *config,
                                                const char *quant, int device, const CheetahCudaResidency *plan,
                                                CheetahCudaModel **out);
/* `AntTierControl::page_in_unit` / `evict_unit` (`registry.rs:88-93`):
 * tier 0 (CHEETAH_ANT_TIER_VRAM) uploads the unit's linear into its own HBM
 * copy, tiers 1/2 and eviction release it (the pinned host copy stays
 * authoritative, so later forwards stream it). *known = 0 for a unit id the
 * units manifest does not list (no error); units that always stay resident
 * report known = 1 and do not move. Only for models opened with a plan. */
CHEETAH_CUDA_API int cheetah_cuda_model_page_in_unit(CheetahCudaModel *model, const char *unit_id, int tier,
                                                     int *known);
CHEETAH_CUDA_API int cheetah_cuda_model_evict_unit(CheetahCudaModel *model, const char *unit_id, int *known);
typedef struct CheetahCudaResidencyInfo {
    uint64_t resident_linear_bytes; /* layer linears with their own HBM copy */
    uint64_t streamed_linear_bytes; /* layer linears streamed from pinned host memory */
    uint64_t staging_bytes;         /* the two staging slots */
    uint32_t resident_linears;
    uint32_t streamed_linears;
    int32_t planned;                /* 1: opened with a residency plan */
    int32_t reserved;
} CheetahCudaResidencyInfo;
CHEETAH_CUDA_API int cheetah_cuda_model_residency(const CheetahCudaModel *model, CheetahCudaResidencyInfo *info);

/* A sequence: an empty KV cache that shares the model's weights — the
 * `ModelForwardClone` contract (`registry.rs:95-117`, pinned by
 * `decoder.rs:1761`). One thread uses a sequence at a time. */
CHEETAH_CUDA_API int cheetah_cuda_seq_new(CheetahCudaModel *model, CheetahCudaSeq **out);
CHEETAH_CUDA_API int cheetah_cuda_seq_free(CheetahCudaSeq *seq);
/* `ModelForward::clear_cache` (`registry.rs:63`, `ops.rs:1610`). */
CHEETAH_CUDA_API int cheetah_cuda_seq_clear(CheetahCudaSeq *seq);
CHEETAH_CUDA_API int cheetah_cuda_seq_positions(const CheetahCudaSeq *seq, size_t *positions);

/* `ModelForward::forward` (`registry.rs:60`, `qwen2.rs:600-606`): run
 * `tokens[0..n)` at absolute positions `offset..offset+n` and write the final
 * position's `vocab_size` f32 logits to `logits_out` (host memory). `offset`
 * must equal the sequence's cached position count. Errors: empty input, a
 * token id >= vocab (`ops.rs:1065-1078`), capacity exceeded. A `logits_out`
 * in page-locked host memory (cudaMallocHost / cudaHostRegister) is written
 * by the device directly; any other host buffer receives a copy from the
 * sequence's own page-locked buffer (one extra host memcpy per call). */
CHEETAH_CUDA_API int cheetah_cuda_forward(CheetahCudaSeq *seq, const uint32_t *tokens, size_t n, size_t offset,
                         float *logits_out);
/* As above; `logits_out` may be NULL (no logits copy) and `argmax_out`
 * (nullable) receives the greedy token chosen as the engine does
 * (`engine.rs:2247-2253`: max by total order, last maximum wins). */
CHEETAH_CUDA_API int cheetah_cuda_forward_ex(CheetahCudaSeq *seq, const uint32_t *tokens, size_t n,
                            size_t offset, float *logits_out, uint32_t *argmax_out);

/* Continuous batching behind cheetah_cuda_forward / _ex. Each concurrent
 * generation owns a sequence of one shared model (the clone of the
 * reference's per-generation `ModelForward`, `engine.rs:1872-1876`) and calls
 * forward from its own thread. Single-token calls (n == 1) that arrive while
 * a step runs wait and run together as the next batched step: one pass over
 * the weights for all of them, each with its own pages, results and errors
 * (an invalid call fails alone). A lone caller runs at once. Groups below
 * CHEETAH_CUDA_COALESCE_MIN calls (default 3) run one at a time on the
 * single-sequence path; CHEETAH_CUDA_COALESCE=0 switches batching off. Needs
 * bf16 weights and a bf16 KV cache (other models run every call alone).
 * Counters: single-token calls seen, calls that ran in batched steps, and
 * batched steps run. */
CHEETAH_CUDA_API int cheetah_cuda_model_coalesce_stats(const CheetahCudaModel *model, uint64_t *calls,
                                                       uint64_t *batched_calls, uint64_t *batches);

/* One decode token for each of `batch` (1..128) sequences of `model`: seqs[b]
 * consumes tokens[b] at position offsets[b] (= its cached position count).
 * The batch shares one pass over the weights (tensor-core GEMMs); attention
 * reads each sequence's own pages. logits_out (nullable, host) receives
 * batch x vocab f32; argmax_out (nullable, host) each row's greedy token
 * (`engine.rs:2247-2253`). The batched form of `ModelForward::forward`
 * (`registry.rs:60`) for concurrent sequences (serve: `engine.rs:1874`,
 * `serve/queue.rs:48-67`). Needs bf16 weights and a bf16 KV cache. A
 * batch of one runs the single-sequence step on the sequence's stream. */
CHEETAH_CUDA_API int cheetah_cuda_forward_batch(CheetahCudaModel *model, CheetahCudaSeq *const *seqs,
                                                const uint32_t *tokens, const size_t *offsets, size_t batch,
                                                float *logits_out, uint32_t *argmax_out);

/* `steps` greedy tokens for each of `batch` sequences, kept on the device:
 * step i of sequence b consumes its greedy token of step i-1 (step 0 consumes
 * tokens[b]) at position offsets[b] + i, so there is no host round trip
 * between steps; tokens_out[b * steps + i] receives that step's greedy token.
 * The same results as `steps` calls of cheetah_cuda_forward_batch, each fed
 * the previous call's ids: the serving loop's greedy batch
 * (`engine.rs:1874`, `engine.rs:1920-1958`) between changes of the batch.
 * Needs bf16 weights and a bf16 KV cache. A batch of one runs
 * cheetah_cuda_generate_greedy (the persistent decode kernel where the model
 * has it) on the sequence's stream. */
CHEETAH_CUDA_API int cheetah_cuda_forward_batch_greedy(CheetahCudaModel *model, CheetahCudaSeq *const *seqs,
                                                       const uint32_t *tokens, const size_t *offsets,
                                                       size_t batch, size_t steps, uint32_t *tokens_out);

/* Greedy decode kept on the device: step i consumes the greedy token of step
 * i-1 (step 0 consumes `first_token`) at position `offset + i`; tokens_out[i]
 * receives step i's greedy token. No host round trip between steps — the
 * device-resident form of the engine's greedy loop (`engine.rs:1920-1958`).
 * With tokens_out == NULL the steps are only enqueued on the sequence stream
 * (see cheetah_cuda_seq_stream) and the call returns without waiting. */
CHEETAH_CUDA_API int cheetah_cuda_generate_greedy(CheetahCudaSeq *seq, uint32_t first_token, size_t offset,
                                                  size_t steps, uint32_t *tokens_out);
/* The sequence's CUDA stream (cudaStream_t) for event timing / synchronisation. */
CHEETAH_CUDA_API int cheetah_cuda_seq_stream(const CheetahCudaSeq *seq, void **stream);
/* The model's batch stream (cudaStream_t), on which cheetah_cuda_forward_batch
 * and cheetah_cuda_forward_batch_greedy run batches of two or more, for
 * event timing. Created by the
 * first batched call; *stream is NULL before it. A harness accessor: the
 * reference times `forward` on the host (no counterpart in `registry.rs`). */
CHEETAH_CUDA_API int cheetah_cuda_model_batch_stream(const CheetahCudaModel *model, void **stream);

/* `ModelForward::kv_snapshot` / `restore_kv_prefix` (`registry.rs:68-79`,
 * `ops.rs:1575-1607`) without copying: a snapshot holds a reference on each
 * KV page of the cached positions, and a restored sequence references the
 * snapshot's pages. Shared pages are never written: the first append into a
 * shared partial page copies that one page (copy on write), so the source
 * sequence, the snapshot and every restored sequence stay independent.
 * Pages return to the pool when their last holder lets go. */
CHEETAH_CUDA_API int cheetah_cuda_seq_snapshot(const CheetahCudaSeq *seq, CheetahCudaSnapshot **out);
CHEETAH_CUDA_API int cheetah_cuda_snapshot_positions(const CheetahCudaSnapshot *snapshot, size_t *positions);
CHEETAH_CUDA_API int cheetah_cuda_seq_restore_prefix(CheetahCudaSeq *seq, const CheetahCudaSnapshot *snapshot,
                                    size_t positions);
CHEETAH_CUDA_API int cheetah_cuda_snapshot_free(CheetahCudaSnapshot *snapshot);
/* Test/diagnostic view of one layer's cache as f32 [positions][kv_heads*head_dim]
 * (host buffers of positions*kv_dim floats each). */
CHEETAH_CUDA_API int cheetah_cuda_seq_export_kv(const CheetahCudaSeq *seq, size_t layer, float *k_out,
                               float *v_out);

/* ---- Op entries: caller-owned device buffers, caller stream ---- */

/* y[b] = W . x[b] for b < batch. W: bf16 row-major [rows, cols] (cols % 8 == 0,
 * 16-byte aligned), x: f32 [batch, cols], y: f32 [batch, rows].
 * Replaces `ops::gemv` (`ops.rs:246`) / `bf16::gemv` (`precision/bf16.rs:54`). */
CHEETAH_CUDA_API int cheetah_cuda_op_gemv_bf16(const void *weight, size_t rows, size_t cols, const float *x,
                              size_t batch, float *y, void *stream);

/* Bytes of a q8 / q4 buffer in the reference interchange layout
 * (`precision/q8.rs:8-21`, `precision/q4.rs:9-36`): rows f32 scales, then
 * rows x row_bytes codes (q8 row_bytes = (cols+3)/4*4; q4 row_bytes =
 * (cols+1).div_ceil(2).div_ceil(4)*4). `format` is "q8" or "q4". */
CHEETAH_CUDA_API int cheetah_cuda_quant_buffer_bytes(const char *format, size_t rows, size_t cols, size_t *bytes);

/* Per-row quantisation of bf16 weights [rows, cols] (device) into `out`
 * (device, the reference layout above), bit-identical to `q8::quantize`
 * (`precision/q8.rs:91`) / `q4::quantize` (`precision/q4.rs:126`) applied to
 * the exactly widened values. */
CHEETAH_CUDA_API int cheetah_cuda_op_quantize_q8(const void *weight, size_t rows, size_t cols, void *out,
                                                 void *stream);
CHEETAH_CUDA_API int cheetah_cuda_op_quantize_q4(const void *weight, size_t rows, size_t cols, void *out,
                                                 void *stream);

/* y[b] = W . x[b] over a q8 / q4 buffer in the reference layout (device):
 * codes unpacked in registers, f32 accumulation, the row scale applied to the
 * finished dot. cols % 8 == 0. Replaces `gemv_q8` / `gemv_q4` (`ops.rs:544`,
 * `ops.rs:586`). */
CHEETAH_CUDA_API int cheetah_cuda_op_gemv_q8(const void *buffer, size_t rows, size_t cols, const float *x,
                                             size_t batch, float *y, void *stream);
CHEETAH_CUDA_API int cheetah_cuda_op_gemv_q4(const void *buffer, size_t rows, size_t cols, const float *x,
                                             size_t batch, float *y, void *stream);

/* Paged GQA decode attention for `batch` sequences, one query position each
 * (the newest), over a paged KV pool. Replaces `OpsToolbox::attention` /
 * `attention_head` (`ops.rs:1357-1467`) for one position of every head. */
typedef struct CheetahCudaDecodeAttention {
    const float *q;            /* [batch][q_heads][head_dim], RoPE applied */
    const void *k_pool;        /* [num_pages][kv_heads][page_tokens][head_dim] */
    const void *v_pool;        /* same layout as k_pool */
    int32_t kv_dtype;          /* CHEETAH_CUDA_KV_* */
    const int32_t *page_table; /* [batch][max_pages_per_seq] page ids */
    uint32_t max_pages_per_seq;
    const int32_t *seq_lens;   /* [batch] cached positions incl. the query's */
    uint32_t max_seq_len;      /* host upper bound on seq_lens (work split) */
    uint32_t num_pages;        /* pages in the pool (bounds check) */
    uint32_t page_tokens;
    uint32_t batch;
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;         /* 64 or 128 */
    uint32_t sliding_window;   /* 0 = full */
    float *out;                /* [batch][q_heads][head_dim] */
} CheetahCudaDecodeAttention;
CHEETAH_CUDA_API int cheetah_cuda_op_decode_attention(const CheetahCudaDecodeAttention *args, void *stream);

/* Causal attention of a prefill chunk: query rows offset .. offset+tokens-1
 * of one sequence, each over its cached keys up to and including its own
 * position (less the sliding window), over a paged bf16 pool that already
 * holds those rows' K/V. Replaces `OpsToolbox::attention` (`ops.rs:1357-1421`)
 * as the per-row loop of `forward_layer_chunk` (`qwen2.rs:314-343`) calls it.
 * Tensor cores for head_dim 64 (tcgen05) and 128. Asynchronous on `stream`;
 * split scratch is allocated on first use per (device, stream). */
typedef struct CheetahCudaPrefillAttention {
    const void *q;             /* bf16 [tokens][q_heads][head_dim], RoPE applied */
    const void *k_pool;        /* bf16 [num_pages][kv_heads][page_tokens][head_dim] */
    const void *v_pool;        /* same layout as k_pool */
    const int32_t *page_table; /* [max_pages] the sequence's page ids */
    uint32_t max_pages;
    uint32_t num_pages;        /* pages in the pool (bounds check) */
    uint32_t page_tokens;      /* a multiple of 64 */
    uint32_t tokens;           /* query rows */
    uint32_t offset;           /* absolute position of query row 0 */
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;         /* 64 or 128 */
    uint32_t sliding_window;   /* 0 = full */
    void *out;                 /* bf16 [tokens][q_heads][head_dim] */
} CheetahCudaPrefillAttention;
CHEETAH_CUDA_API int cheetah_cuda_op_prefill_attention(const CheetahCudaPrefillAttention *args, void *stream);

/* Decode attention for callers that cannot let the library allocate device
 * memory — e.g. a host that runs a fixed device-memory budget of its own and
 * hands the library only inputs and outputs, or a latency-critical path that
 * cannot absorb the device-wide synchronisation of cudaMalloc / cudaFree.
 * Same arguments and result as cheetah_cuda_op_decode_attention; the
 * split-merge scratch is a fixed ~4.1 MiB array compiled into the library,
 * held by every GPU that loads it until the process exits. Limits:
 * batch * kv_heads <= 1024 (larger requests fail with an error); the KV split
 * count is reduced so batch * kv_heads * splits <= 1024. The first call on a
 * device looks the array's device address up (cudaGetSymbolAddress); make
 * that first call before any stream capture. All calls share the one array:
 * calls that overlap on the GPU (different streams, no ordering) race.
 * No counterpart in the reference. */
CHEETAH_CUDA_API int cheetah_cuda_op_decode_attention_noalloc(const CheetahCudaDecodeAttention *args,
                                                              void *stream);

#ifdef __cplusplus
}
#endif

#endif
