/* TEST INFRASTRUCTURE ONLY — the CPU oracle for the Cheetah decoder hot path.
 *
 * A C++ restatement of the reference native CPU backend (Rust):
 *   src/chat/native/ops.rs            math kernels + OpsToolbox state
 *   src/chat/registrations/qwen2.rs   Qwen2 layer order (per-position + chunked)
 *   src/chat/precision/q8.rs, q4.rs   per-row quantisers and buffer layouts
 * The reference cannot be compiled in this image (no Rust toolchain), so this
 * restatement is the checker for the CUDA backend and the timed CPU baseline.
 * It is pinned against the reference's own known-answer unit tests
 * (ops.rs:1690-2092, q8.rs:209-266, q4.rs:239-327), restated in
 * tests/test_oracle_*.py.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library. The product path (libcheetah_cuda) never links it.
 */
#ifndef CHEETAH_ORACLE_REF_CPU_H
#define CHEETAH_ORACLE_REF_CPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight storage dtypes, as WeightDType in src/chat/native/store.rs:14-18. */
enum { ORACLE_BF16 = 0, ORACLE_F16 = 1, ORACLE_F32 = 2 };
/* Quantisation selection, as CHEETAH_QUANT_Q8 / CHEETAH_QUANT_Q4. */
enum { ORACLE_QUANT_NONE = 0, ORACLE_QUANT_Q8 = 1, ORACLE_QUANT_Q4 = 2 };

void oracle_set_threads(int threads);
int oracle_get_threads(void);
int oracle_has_avx2(void);

/* ops.rs:246 gemv over stored-precision rows (bf16 takes the AVX2 fused dot). */
void oracle_gemv(const uint8_t *weight, int dtype, size_t rows, size_t cols,
                 const float *x, float *y);
/* ops.rs:308 gemm: y[n, rows] = x[n, cols] . W^T, bit-identical per element. */
void oracle_gemm(const uint8_t *weight, int dtype, size_t rows, size_t cols,
                 const float *x, size_t n, float *y);
/* ops.rs:544 / ops.rs:586 quantised matvecs over the q8 / q4 interchange layout. */
void oracle_gemv_q8(const uint8_t *buffer, size_t rows, size_t cols,
                    const float *x, float *y);
void oracle_gemv_q4(const uint8_t *buffer, size_t rows, size_t cols,
                    const float *x, float *y);
/* q8.rs:91 / q4.rs:126 quantisers; out must hold oracle_q*_bytes(rows, cols). */
size_t oracle_q8_row_bytes(size_t cols);
size_t oracle_q4_row_bytes(size_t cols);
size_t oracle_q8_bytes(size_t rows, size_t cols);
size_t oracle_q4_bytes(size_t rows, size_t cols);
int oracle_quantize_q8(const float *values, size_t rows, size_t cols, uint8_t *out);
int oracle_quantize_q4(const float *values, size_t rows, size_t cols, uint8_t *out);
/* Dequantised element (q8.rs:66 / q4.rs:107 dequant_value). */
float oracle_q8_dequant(const uint8_t *buffer, size_t rows, size_t cols, size_t row, size_t col);
float oracle_q4_dequant(const uint8_t *buffer, size_t rows, size_t cols, size_t row, size_t col);

/* ops.rs:646 rmsnorm, in place. */
void oracle_rmsnorm(float *x, size_t n, const uint8_t *weight, int dtype, float eps);
/* ops.rs:693 / :722 rotate-half rope. */
void oracle_rope_in_place(float *values, size_t heads, size_t head_dim,
                          size_t position, float theta);
void oracle_rope_heads(float *values, size_t heads, size_t head_dim,
                       size_t rotary_dim, size_t position, float theta);
/* ops.rs:743 silu(gate) * up written into gate; ops.rs:770 softmax. */
void oracle_silu_multiply(float *gate, const float *up, size_t n);
void oracle_softmax(float *scores, size_t n);
/* ops.rs:1357 GQA attention for one query position over an f32 cache laid
 * out [pos][kv_heads][head_dim]; out is [q_heads][head_dim]. */
void oracle_attention(const float *keys, const float *values, size_t cache_len,
                      size_t position, const float *q, size_t q_heads,
                      size_t kv_heads, size_t head_dim, size_t sliding_window,
                      float *out);

/* ---- Qwen2 decoder (qwen2.rs:92-635 over OpsToolbox ops.rs:987-1690) ---- */
typedef struct OracleConfig {
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
    uint32_t sliding_window;
    int32_t quant; /* ORACLE_QUANT_* */
} OracleConfig;

typedef struct OracleModel OracleModel;

OracleModel *oracle_model_new(const OracleConfig *cfg);
void oracle_model_free(OracleModel *model);
/* Register one unit's bytes (borrowed; must outlive the model). */
int oracle_model_set_unit(OracleModel *model, const char *unit_id,
                          const uint8_t *data, int dtype, size_t bytes);
/* Quantise every layer linear up front (same result as the reference's lazy
 * first-use quantisation, ops.rs:1199-1226). */
int oracle_model_prepare(OracleModel *model);
/* ModelForward::forward: logits of the final position (vocab floats).
 * chunk_rows is the prefill chunk (qwen2.rs:138-157); 0 = 256. */
int oracle_model_forward(OracleModel *model, const uint32_t *tokens, size_t n,
                         size_t offset, size_t chunk_rows, float *logits);
void oracle_model_clear(OracleModel *model);
size_t oracle_model_positions(const OracleModel *model);
/* Copy layer KV ([positions][kv_dim] f32) out / restore a prefix in. */
int oracle_model_kv_export(const OracleModel *model, size_t layer, float *k, float *v);
int oracle_model_kv_restore(OracleModel *model, size_t positions,
                            const float *const *k_layers, const float *const *v_layers);
/* Final normed hidden of the last forward (tests). */
int oracle_model_hidden(const OracleModel *model, float *out);
const char *oracle_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
