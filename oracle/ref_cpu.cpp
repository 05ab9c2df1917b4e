// TEST INFRASTRUCTURE ONLY — CPU oracle for the Cheetah decoder hot path.
//
// A restatement of the reference native backend (Rust, not buildable here):
// every function cites the reference file:line whose arithmetic it follows.
// Floating-point order is kept exactly: compiled with -ffp-contract=off so
// that a*b+c stays two roundings (Rust never contracts), the AVX2 dot uses the
// same intrinsics/lane structure as ops.rs:202-237, sums are sequential folds
// starting at -0.0 (Rust's `Iterator::sum` for f32), and transcendentals are
// glibc's expf/sinf/cosf/powf (what Rust's f32 methods call on Linux).
// The product path never links this file; it is the checker and the timed
// CPU baseline only.

#include "ref_cpu.h"

#include <immintrin.h>

#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_error;

void set_error(const std::string &message) { g_error = message; }

// ---------------------------------------------------------------------------
// Thread pool: stands in for rayon's global pool (one worker per core,
// engine.rs:859-869). parallel_for hands out indices with an atomic counter.
// ---------------------------------------------------------------------------
class Pool {
  public:
    explicit Pool(int threads) { resize(threads); }
    ~Pool() { stop(); }

    int threads() const { return static_cast<int>(workers_.size()) + 1; }

    void resize(int threads) {
        stop();
        if (threads < 1) threads = 1;
        stopping_ = false;
        for (int i = 0; i < threads - 1; ++i) {
            workers_.emplace_back([this] { worker(); });
        }
    }

    void parallel_for(size_t count, const std::function<void(size_t)> &fn) {
        if (count == 0) return;
        if (workers_.empty() || count == 1) {
            for (size_t i = 0; i < count; ++i) fn(i);
            return;
        }
        std::lock_guard<std::mutex> serial(dispatch_);
        {
            std::lock_guard<std::mutex> lock(mutex_);
            task_ = &fn;
            count_ = count;
            next_.store(0);
            pending_.store(static_cast<int>(workers_.size()));
            ++generation_;
        }
        cv_.notify_all();
        run_indices(fn, count);
        // Wait for every worker to leave this generation.
        while (pending_.load(std::memory_order_acquire) != 0) {
            _mm_pause();
        }
        task_ = nullptr;
    }

  private:
    void run_indices(const std::function<void(size_t)> &fn, size_t count) {
        for (;;) {
            size_t index = next_.fetch_add(1);
            if (index >= count) break;
            fn(index);
        }
    }

    void worker() {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(size_t)> *task = nullptr;
            size_t count = 0;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                cv_.wait(lock, [&] { return stopping_ || generation_ != seen; });
                if (stopping_) return;
                seen = generation_;
                task = task_;
                count = count_;
            }
            run_indices(*task, count);
            pending_.fetch_sub(1, std::memory_order_release);
        }
    }

    void stop() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            stopping_ = true;
        }
        cv_.notify_all();
        for (auto &worker : workers_) worker.join();
        workers_.clear();
    }

    std::vector<std::thread> workers_;
    std::mutex mutex_;
    std::mutex dispatch_;
    std::condition_variable cv_;
    const std::function<void(size_t)> *task_ = nullptr;
    size_t count_ = 0;
    std::atomic<size_t> next_{0};
    std::atomic<int> pending_{0};
    uint64_t generation_ = 0;
    bool stopping_ = false;
};

Pool &pool() {
    static Pool instance(static_cast<int>(std::thread::hardware_concurrency()));
    return instance;
}

bool cpu_has_avx2_fma() {
    static const bool value = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    return value;
}

// ops.rs:59-62: bf16 widening is a 16-bit shift.
inline float bf16_f32(uint16_t bits) {
    uint32_t word = static_cast<uint32_t>(bits) << 16;
    float value;
    std::memcpy(&value, &word, 4);
    return value;
}

// ops.rs:70-72: f16 widening (half::f16::to_f32 is exact; so is F16C).
inline float f16_f32(uint16_t bits) { return _cvtsh_ss(bits); }

inline uint16_t load_u16(const uint8_t *bytes) {
    return static_cast<uint16_t>(bytes[0] | (bytes[1] << 8));
}

// ops.rs:84-95 scalar_at.
inline float scalar_at(const uint8_t *bytes, size_t index, int dtype) {
    switch (dtype) {
    case ORACLE_BF16: return bf16_f32(load_u16(bytes + 2 * index));
    case ORACLE_F16: return f16_f32(load_u16(bytes + 2 * index));
    default: {
        float value;
        std::memcpy(&value, bytes + 4 * index, 4);
        return value;
    }
    }
}

inline size_t element_size(int dtype) { return dtype == ORACLE_F32 ? 4 : 2; }

// Rust `Iterator::<f32>::sum` is a sequential fold from -0.0.
inline float seq_sum(const float *values, size_t n) {
    float sum = -0.0f;
    for (size_t i = 0; i < n; ++i) sum += values[i];
    return sum;
}

// ops.rs:121-135 dot_f32: 8 lane accumulators, then lane sum, then tail.
float dot_f32(const float *a, const float *b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t chunks = n / 8;
    for (size_t c = 0; c < chunks; ++c) {
        for (int lane = 0; lane < 8; ++lane) {
            float product = a[c * 8 + lane] * b[c * 8 + lane];
            acc[lane] += product;
        }
    }
    float sum = seq_sum(acc, 8);
    for (size_t i = chunks * 8; i < n; ++i) {
        float product = a[i] * b[i];
        sum += product;
    }
    return sum;
}

// ops.rs:173-192 portable fused bf16 dot (4 accumulators over 8-byte chunks).
float dot_row_bf16_portable(const uint8_t *row, const float *x, size_t cols) {
    size_t chunks = cols / 4;
    float acc[4] = {0, 0, 0, 0};
    for (size_t c = 0; c < chunks; ++c) {
        for (int lane = 0; lane < 4; ++lane) {
            float product = bf16_f32(load_u16(row + c * 8 + lane * 2)) * x[c * 4 + lane];
            acc[lane] += product;
        }
    }
    float sum = acc[0] + acc[1];
    sum = sum + acc[2];
    sum = sum + acc[3];
    for (size_t i = chunks * 4; i < cols; ++i) {
        float product = bf16_f32(load_u16(row + 2 * i)) * x[i];
        sum += product;
    }
    return sum;
}

// ops.rs:202-237 AVX2+FMA bf16 dot: per 16-element chunk acc0 += lo8*x[0..8],
// acc1 += hi8*x[8..16] (fused), then sum(acc0 lanes)+sum(acc1 lanes)+tail.
__attribute__((target("avx2,fma"))) float dot_row_bf16_avx2(const uint8_t *row, const float *x,
                                                             size_t cols) {
    size_t full = cols / 16;
    __m256 acc0 = _mm256_setzero_ps();
    __m256 acc1 = _mm256_setzero_ps();
    for (size_t c = 0; c < full; ++c) {
        __m256i w = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(row + c * 32));
        __m128i lo = _mm256_castsi256_si128(w);
        __m128i hi = _mm256_extracti128_si256(w, 1);
        __m256 f_lo = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(lo), 16));
        __m256 f_hi = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(hi), 16));
        __m256 x0 = _mm256_loadu_ps(x + c * 16);
        __m256 x1 = _mm256_loadu_ps(x + c * 16 + 8);
        acc0 = _mm256_fmadd_ps(f_lo, x0, acc0);
        acc1 = _mm256_fmadd_ps(f_hi, x1, acc1);
    }
    alignas(32) float lanes0[8];
    alignas(32) float lanes1[8];
    _mm256_store_ps(lanes0, acc0);
    _mm256_store_ps(lanes1, acc1);
    float total = seq_sum(lanes0, 8) + seq_sum(lanes1, 8);
    float tail_total = 0.0f;  // `let mut tail_total = 0f32`
    for (size_t i = full * 16; i < cols; ++i) {
        float product = bf16_f32(load_u16(row + 2 * i)) * x[i];
        tail_total += product;
    }
    return total + tail_total;
}

inline float dot_row_bf16(const uint8_t *row, const float *x, size_t cols) {
    if (cpu_has_avx2_fma()) return dot_row_bf16_avx2(row, x, cols);
    return dot_row_bf16_portable(row, x, cols);
}

// ops.rs:432-504: one bf16 row against up to 4 token rows. Per element the
// accumulation order equals dot_row_bf16_avx2 (the gemm≡gemv contract).
__attribute__((target("avx2,fma"))) void dot_row_bf16_avx2_multi(const uint8_t *row,
                                                                  const float *x, size_t cols,
                                                                  size_t token_start,
                                                                  size_t token_count,
                                                                  float *out) {
    size_t full = cols / 16;
    __m256 acc[4][2];
    for (int t = 0; t < 4; ++t) acc[t][0] = acc[t][1] = _mm256_setzero_ps();
    const float *base[4];
    for (size_t t = 0; t < 4; ++t) {
        base[t] = x + (token_start + (t < token_count ? t : 0)) * cols;
    }
    for (size_t c = 0; c < full; ++c) {
        __m256i w = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(row + c * 32));
        __m128i lo = _mm256_castsi256_si128(w);
        __m128i hi = _mm256_extracti128_si256(w, 1);
        __m256 f_lo = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(lo), 16));
        __m256 f_hi = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(hi), 16));
        for (int t = 0; t < 4; ++t) {
            acc[t][0] = _mm256_fmadd_ps(f_lo, _mm256_loadu_ps(base[t] + c * 16), acc[t][0]);
            acc[t][1] = _mm256_fmadd_ps(f_hi, _mm256_loadu_ps(base[t] + c * 16 + 8), acc[t][1]);
        }
    }
    for (size_t t = 0; t < token_count; ++t) {
        const float *x_row = x + (token_start + t) * cols;
        float tail_total = 0.0f;
        for (size_t i = full * 16; i < cols; ++i) {
            float product = bf16_f32(load_u16(row + 2 * i)) * x_row[i];
            tail_total += product;
        }
        alignas(32) float lanes0[8];
        alignas(32) float lanes1[8];
        _mm256_store_ps(lanes0, acc[t][0]);
        _mm256_store_ps(lanes1, acc[t][1]);
        float total = seq_sum(lanes0, 8) + seq_sum(lanes1, 8);
        out[t] = total + tail_total;
    }
}

constexpr size_t kGemvChunkRows = 128;   // ops.rs:51
constexpr size_t kGemmBlockRows = 64;    // ops.rs:285
constexpr size_t kGemmTokenGroup = 4;    // ops.rs:288
constexpr size_t kAttentionParallelMinCache = 384;  // ops.rs:291
constexpr size_t kPrefillChunkRows = 256;  // ops.rs:535
constexpr size_t kLmHeadChunkRows = 16384; // ops.rs:1543

float dot_row_any(const uint8_t *row, int dtype, const float *x, size_t cols,
                  std::vector<float> &scratch) {
    if (dtype == ORACLE_BF16) return dot_row_bf16(row, x, cols);
    scratch.resize(cols);
    for (size_t i = 0; i < cols; ++i) scratch[i] = scalar_at(row, i, dtype);
    return dot_f32(scratch.data(), x, cols);
}

// ops.rs:246-278.
void gemv_impl(const uint8_t *weight, int dtype, size_t rows, size_t cols, const float *x,
               float *y) {
    size_t row_stride = cols * element_size(dtype);
    auto run_rows = [&](size_t start, size_t end) {
        std::vector<float> scratch;
        for (size_t row = start; row < end; ++row) {
            y[row] = dot_row_any(weight + row * row_stride, dtype, x, cols, scratch);
        }
    };
    if (rows <= kGemvChunkRows) {
        run_rows(0, rows);
        return;
    }
    size_t chunks = (rows + kGemvChunkRows - 1) / kGemvChunkRows;
    pool().parallel_for(chunks, [&](size_t chunk) {
        size_t start = chunk * kGemvChunkRows;
        size_t end = std::min(rows, start + kGemvChunkRows);
        run_rows(start, end);
    });
}

// ops.rs:361-386 gemm_row_block.
void gemm_row_block(const uint8_t *weight, size_t cols, const float *x, size_t n,
                    size_t row_start, size_t block_rows, float *out) {
    size_t row_stride = cols * 2;
    for (size_t token_start = 0; token_start < n; token_start += kGemmTokenGroup) {
        size_t token_count = std::min(kGemmTokenGroup, n - token_start);
        for (size_t r = 0; r < block_rows; ++r) {
            const uint8_t *row = weight + (row_start + r) * row_stride;
            float *out_row = out + r * n;
            if (cpu_has_avx2_fma()) {
                dot_row_bf16_avx2_multi(row, x, cols, token_start, token_count,
                                        out_row + token_start);
            } else {
                for (size_t t = 0; t < token_count; ++t) {
                    out_row[token_start + t] =
                        dot_row_bf16_portable(row, x + (token_start + t) * cols, cols);
                }
            }
        }
    }
}

// ops.rs:308-354.
void gemm_impl(const uint8_t *weight, int dtype, size_t rows, size_t cols, const float *x,
               size_t n, float *y) {
    if (n == 1 || dtype != ORACLE_BF16) {
        for (size_t t = 0; t < n; ++t) gemv_impl(weight, dtype, rows, cols, x + t * cols, y + t * rows);
        return;
    }
    std::vector<float> y_t(rows * n, 0.0f);
    size_t block_rows = std::min(kGemmBlockRows, rows);
    if (rows <= block_rows) {
        gemm_row_block(weight, cols, x, n, 0, rows, y_t.data());
    } else {
        size_t blocks = (rows + block_rows - 1) / block_rows;
        pool().parallel_for(blocks, [&](size_t block) {
            size_t start = block * block_rows;
            size_t count = std::min(block_rows, rows - start);
            gemm_row_block(weight, cols, x, n, start, count, y_t.data() + start * n);
        });
    }
    for (size_t row = 0; row < rows; ++row) {
        for (size_t t = 0; t < n; ++t) y[t * rows + row] = y_t[row * n + t];
    }
}

inline float load_f32(const uint8_t *bytes) {
    float value;
    std::memcpy(&value, bytes, 4);
    return value;
}

// ops.rs:544-577: sum += scale * (code as f32) * x, left to right.
void gemv_q8_impl(const uint8_t *weight, size_t rows, size_t cols, const float *x, float *y) {
    size_t row_bytes = (cols + 3) / 4 * 4;
    size_t head = rows * 4;
    auto dot = [&](size_t row) {
        float scale = load_f32(weight + row * 4);
        const int8_t *codes = reinterpret_cast<const int8_t *>(weight + head + row * row_bytes);
        float sum = 0.0f;
        for (size_t c = 0; c < cols; ++c) {
            float scaled = scale * static_cast<float>(codes[c]);
            float product = scaled * x[c];
            sum += product;
        }
        return sum;
    };
    if (rows <= kGemvChunkRows) {
        for (size_t r = 0; r < rows; ++r) y[r] = dot(r);
        return;
    }
    size_t chunks = (rows + kGemvChunkRows - 1) / kGemvChunkRows;
    pool().parallel_for(chunks, [&](size_t chunk) {
        size_t start = chunk * kGemvChunkRows;
        size_t end = std::min(rows, start + kGemvChunkRows);
        for (size_t r = start; r < end; ++r) y[r] = dot(r);
    });
}

// q4.rs:59-66 decode_code: nibble >= 8 sign-extends (nibble - 16).
inline int q4_code(uint8_t byte, size_t half) {
    int nibble = half == 0 ? (byte & 0x0F) : (byte >> 4);
    return nibble >= 8 ? nibble - 16 : nibble;
}

size_t q4_row_bytes(size_t cols) {
    // q4.rs:50: (cols + 1).div_ceil(2).div_ceil(4) * 4
    size_t a = (cols + 1 + 1) / 2;
    size_t b = (a + 3) / 4;
    return b * 4;
}

// ops.rs:586-630.
void gemv_q4_impl(const uint8_t *weight, size_t rows, size_t cols, const float *x, float *y) {
    size_t row_bytes = q4_row_bytes(cols);
    size_t head = rows * 4;
    auto dot = [&](size_t row) {
        float scale = load_f32(weight + row * 4);
        const uint8_t *payload = weight + head + row * row_bytes;
        float sum = 0.0f;
        for (size_t c = 0; c < cols; ++c) {
            int code = q4_code(payload[c / 2], c % 2);
            float scaled = scale * static_cast<float>(code);
            float product = scaled * x[c];
            sum += product;
        }
        return sum;
    };
    if (rows <= kGemvChunkRows) {
        for (size_t r = 0; r < rows; ++r) y[r] = dot(r);
        return;
    }
    size_t chunks = (rows + kGemvChunkRows - 1) / kGemvChunkRows;
    pool().parallel_for(chunks, [&](size_t chunk) {
        size_t start = chunk * kGemvChunkRows;
        size_t end = std::min(rows, start + kGemvChunkRows);
        for (size_t r = start; r < end; ++r) y[r] = dot(r);
    });
}

// Rust `f32::round`: half away from zero == C roundf. `clamp` then `as i8`.
inline int8_t quant_code(float value, float scale, float limit) {
    float q = std::roundf(value / scale);
    if (q < -limit) q = -limit;
    if (q > limit) q = limit;
    return static_cast<int8_t>(q);
}

// Rust `fold(0f32, |acc, v| acc.max(v.abs()))`.
inline float row_max_abs(const float *values, size_t cols) {
    float max_abs = 0.0f;
    for (size_t c = 0; c < cols; ++c) max_abs = std::fmax(max_abs, std::fabs(values[c]));
    return max_abs;
}

// ops.rs:646-652 rmsnorm: sum of squares sequential, inv = 1/sqrt(mean+eps),
// x *= inv * w.
void rmsnorm_impl(float *x, size_t n, const uint8_t *weight, int dtype, float eps) {
    float sum = -0.0f;
    for (size_t i = 0; i < n; ++i) {
        float square = x[i] * x[i];
        sum += square;
    }
    float mean_square = sum / static_cast<float>(n);
    float inv = 1.0f / std::sqrt(mean_square + eps);
    for (size_t i = 0; i < n; ++i) {
        float scale = inv * scalar_at(weight, i, dtype);
        x[i] *= scale;
    }
}

// ops.rs:693-715 rope_in_place.
void rope_in_place_impl(float *values, size_t heads, size_t head_dim, size_t position,
                        float theta) {
    size_t half = head_dim / 2;
    for (size_t head = 0; head < heads; ++head) {
        size_t base = head * head_dim;
        for (size_t i = 0; i < half; ++i) {
            float exponent = (-2.0f * static_cast<float>(i)) / static_cast<float>(head_dim);
            float freq = powf(theta, exponent);
            float angle = static_cast<float>(position) * freq;
            float s = sinf(angle);
            float c = cosf(angle);
            size_t first = base + i;
            size_t second = base + half + i;
            float a = values[first];
            float b = values[second];
            float ac = a * c, bs = b * s, bc = b * c, as = a * s;
            values[first] = ac - bs;
            values[second] = bc + as;
        }
    }
}

// ops.rs:722-740 rope_heads.
void rope_heads_impl(float *values, size_t heads, size_t head_dim, size_t rotary_dim,
                     size_t position, float theta) {
    for (size_t head = 0; head < heads; ++head) {
        rope_in_place_impl(values + head * head_dim, 1, rotary_dim, position, theta);
    }
}

// ops.rs:743-747: g *= u / (1 + exp(-g)).
void silu_multiply_impl(float *gate, const float *up, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float denom = 1.0f + expf(-gate[i]);
        float factor = up[i] / denom;
        gate[i] *= factor;
    }
}

// ops.rs:770-781.
void softmax_impl(float *scores, size_t n) {
    float max = -INFINITY;
    for (size_t i = 0; i < n; ++i) max = std::fmax(max, scores[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        scores[i] = expf(scores[i] - max);
        sum += scores[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; ++i) scores[i] *= inv;
}

// ops.rs:1424-1467 attention_head.
void attention_head(const float *keys, const float *values, const float *q, size_t cache_len,
                    size_t window_start, size_t kv_dim, size_t head_group, size_t head_dim,
                    float scale, size_t head, float *out_head) {
    size_t kv_head = head / head_group;
    const float *qh = q + head * head_dim;
    size_t kv_base = kv_head * head_dim;
    std::vector<float> scores(cache_len, -INFINITY);
    for (size_t pos = window_start; pos < cache_len; ++pos) {
        const float *k = keys + pos * kv_dim + kv_base;
        float score = -0.0f;
        for (size_t d = 0; d < head_dim; ++d) {
            float product = k[d] * qh[d];
            score += product;
        }
        scores[pos] = score * scale;
    }
    softmax_impl(scores.data(), cache_len);
    for (size_t d = 0; d < head_dim; ++d) out_head[d] = 0.0f;
    for (size_t pos = window_start; pos < cache_len; ++pos) {
        float weight = scores[pos];
        if (weight == 0.0f) continue;
        const float *v = values + pos * kv_dim + kv_base;
        for (size_t d = 0; d < head_dim; ++d) {
            float product = weight * v[d];
            out_head[d] += product;
        }
    }
}

// ops.rs:1357-1421 attention.
void attention_impl(const float *keys, const float *values, size_t cache_len, size_t position,
                    const float *q, size_t q_heads, size_t kv_heads, size_t head_dim,
                    size_t sliding_window, float *out) {
    size_t kv_dim = kv_heads * head_dim;
    size_t head_group = q_heads / kv_heads;
    float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
    size_t window_start = 0;
    if (sliding_window != 0) {
        window_start = (position + 1) > sliding_window ? (position + 1) - sliding_window : 0;
    }
    size_t clamp_to = cache_len > 0 ? cache_len - 1 : 0;
    if (window_start > clamp_to) window_start = clamp_to;
    bool parallel = q_heads > 1 && cache_len >= kAttentionParallelMinCache;
    auto run = [&](size_t head) {
        attention_head(keys, values, q, cache_len, window_start, kv_dim, head_group, head_dim,
                       scale, head, out + head * head_dim);
    };
    if (parallel) {
        pool().parallel_for(q_heads, run);
    } else {
        for (size_t head = 0; head < q_heads; ++head) run(head);
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// C API: single ops.
// ---------------------------------------------------------------------------
extern "C" {

void oracle_set_threads(int threads) { pool().resize(threads); }
int oracle_get_threads(void) { return pool().threads(); }
int oracle_has_avx2(void) { return cpu_has_avx2_fma() ? 1 : 0; }
const char *oracle_last_error(void) { return g_error.c_str(); }

void oracle_gemv(const uint8_t *weight, int dtype, size_t rows, size_t cols, const float *x,
                 float *y) {
    gemv_impl(weight, dtype, rows, cols, x, y);
}

void oracle_gemm(const uint8_t *weight, int dtype, size_t rows, size_t cols, const float *x,
                 size_t n, float *y) {
    gemm_impl(weight, dtype, rows, cols, x, n, y);
}

void oracle_gemv_q8(const uint8_t *buffer, size_t rows, size_t cols, const float *x, float *y) {
    gemv_q8_impl(buffer, rows, cols, x, y);
}

void oracle_gemv_q4(const uint8_t *buffer, size_t rows, size_t cols, const float *x, float *y) {
    gemv_q4_impl(buffer, rows, cols, x, y);
}

size_t oracle_q8_row_bytes(size_t cols) { return (cols + 3) / 4 * 4; }
size_t oracle_q4_row_bytes(size_t cols) { return q4_row_bytes(cols); }
size_t oracle_q8_bytes(size_t rows, size_t cols) { return rows * 4 + rows * oracle_q8_row_bytes(cols); }
size_t oracle_q4_bytes(size_t rows, size_t cols) { return rows * 4 + rows * q4_row_bytes(cols); }

// q8.rs:91-125.
int oracle_quantize_q8(const float *values, size_t rows, size_t cols, uint8_t *out) {
    size_t row_bytes = oracle_q8_row_bytes(cols);
    std::memset(out, 0, oracle_q8_bytes(rows, cols));
    for (size_t row = 0; row < rows; ++row) {
        const float *v = values + row * cols;
        float max_abs = row_max_abs(v, cols);
        float scale = max_abs > 0.0f ? max_abs / 127.0f : 1.0f;
        std::memcpy(out + row * 4, &scale, 4);
        for (size_t c = 0; c < cols; ++c) {
            int8_t code = quant_code(v[c], scale, 127.0f);
            out[rows * 4 + row * row_bytes + c] = static_cast<uint8_t>(code);
        }
    }
    return 0;
}

// q4.rs:126-161.
int oracle_quantize_q4(const float *values, size_t rows, size_t cols, uint8_t *out) {
    size_t row_bytes = q4_row_bytes(cols);
    std::memset(out, 0, oracle_q4_bytes(rows, cols));
    for (size_t row = 0; row < rows; ++row) {
        const float *v = values + row * cols;
        float max_abs = row_max_abs(v, cols);
        float scale = max_abs > 0.0f ? max_abs / 7.0f : 1.0f;
        std::memcpy(out + row * 4, &scale, 4);
        for (size_t c = 0; c < cols; ++c) {
            int8_t code = quant_code(v[c], scale, 7.0f);
            size_t index = rows * 4 + row * row_bytes + c / 2;
            out[index] |= static_cast<uint8_t>((static_cast<uint8_t>(code) & 0x0F) << ((c % 2) * 4));
        }
    }
    return 0;
}

float oracle_q8_dequant(const uint8_t *buffer, size_t rows, size_t cols, size_t row, size_t col) {
    float scale = load_f32(buffer + row * 4);
    int8_t code = static_cast<int8_t>(buffer[rows * 4 + row * oracle_q8_row_bytes(cols) + col]);
    return scale * static_cast<float>(code);
}

float oracle_q4_dequant(const uint8_t *buffer, size_t rows, size_t cols, size_t row, size_t col) {
    float scale = load_f32(buffer + row * 4);
    uint8_t byte = buffer[rows * 4 + row * q4_row_bytes(cols) + col / 2];
    return scale * static_cast<float>(q4_code(byte, col % 2));
}

void oracle_rmsnorm(float *x, size_t n, const uint8_t *weight, int dtype, float eps) {
    rmsnorm_impl(x, n, weight, dtype, eps);
}

void oracle_rope_in_place(float *values, size_t heads, size_t head_dim, size_t position,
                          float theta) {
    rope_in_place_impl(values, heads, head_dim, position, theta);
}

void oracle_rope_heads(float *values, size_t heads, size_t head_dim, size_t rotary_dim,
                       size_t position, float theta) {
    rope_heads_impl(values, heads, head_dim, rotary_dim, position, theta);
}

void oracle_silu_multiply(float *gate, const float *up, size_t n) { silu_multiply_impl(gate, up, n); }
void oracle_softmax(float *scores, size_t n) { softmax_impl(scores, n); }

void oracle_attention(const float *keys, const float *values, size_t cache_len, size_t position,
                      const float *q, size_t q_heads, size_t kv_heads, size_t head_dim,
                      size_t sliding_window, float *out) {
    attention_impl(keys, values, cache_len, position, q, q_heads, kv_heads, head_dim,
                   sliding_window, out);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Qwen2 decoder: qwen2.rs:92-635 over the OpsToolbox state (ops.rs:987-1690).
// ---------------------------------------------------------------------------
struct OracleUnitRef {
    const uint8_t *data = nullptr;
    int dtype = ORACLE_BF16;
    size_t bytes = 0;
};

struct OracleModel {
    OracleConfig cfg{};
    std::unordered_map<std::string, OracleUnitRef> units;
    std::unordered_map<std::string, std::vector<uint8_t>> quant;  // unit -> packed buffer
    std::vector<std::vector<float>> kv_k, kv_v;
    // Scratch (ops.rs:800 Scratch): hidden is the persistent residual stream.
    std::vector<float> hidden, normed, q, k, v, attn_out, attn_projected, gate, up, mlp_out;
    // ChunkScratch (ops.rs:873).
    std::vector<float> c_hidden, c_normed, c_q, c_k, c_v, c_attn_out, c_attn_projected, c_gate,
        c_up, c_mlp_out;

    const OracleUnitRef *find(const std::string &id) const {
        auto it = units.find(id);
        return it == units.end() ? nullptr : &it->second;
    }

    size_t kv_dim() const { return cfg.kv_heads * cfg.head_dim; }
    size_t q_dim() const { return cfg.q_heads * cfg.head_dim; }

    bool require(const std::string &id, const OracleUnitRef **out) const {
        *out = find(id);
        if (*out == nullptr) {
            set_error("Native backend: unknown unit '" + id + "'.");
            return false;
        }
        return true;
    }

    // ops.rs:1102 rmsnorm against {unit}.weight.
    bool rmsnorm(const std::string &unit, float *target) const {
        const OracleUnitRef *w;
        if (!require(unit + ".weight", &w)) return false;
        rmsnorm_impl(target, cfg.hidden_size, w->data, w->dtype, cfg.rms_eps);
        return true;
    }

    // ops.rs:1156-1166 add_bias (no-op without the unit).
    void add_bias(float *values, size_t n, const std::string &unit) const {
        const OracleUnitRef *b = find(unit + ".bias");
        if (b == nullptr || b->bytes == 0) return;
        for (size_t i = 0; i < n; ++i) values[i] += scalar_at(b->data, i, b->dtype);
    }

    // ops.rs:1130-1152 qk_norm: per-head RMSNorm of q or k against
    // {unit}.weight (qwen3); a no-op when the unit is absent.
    void qk_norm(float *values, size_t heads, const std::string &unit) const {
        const OracleUnitRef *w = find(unit + ".weight");
        if (w == nullptr || w->bytes == 0) return;
        for (size_t head = 0; head < heads; ++head)
            rmsnorm_impl(values + head * cfg.head_dim, cfg.head_dim, w->data, w->dtype, cfg.rms_eps);
    }

    // ops.rs:1180-1237 linear (quantised buffer if prepared).
    bool linear(const std::string &unit, size_t rows, size_t cols, const float *x, float *y) const {
        auto qit = quant.find(unit);
        if (qit != quant.end()) {
            if (cfg.quant == ORACLE_QUANT_Q8) gemv_q8_impl(qit->second.data(), rows, cols, x, y);
            else gemv_q4_impl(qit->second.data(), rows, cols, x, y);
            return true;
        }
        const OracleUnitRef *w;
        if (!require(unit, &w)) return false;
        if (w->bytes != rows * cols * element_size(w->dtype)) {
            set_error("Linear unit '" + unit + "' does not match its shape.");
            return false;
        }
        gemv_impl(w->data, w->dtype, rows, cols, x, y);
        return true;
    }

    // ops.rs:1244-1326 linear_batch.
    bool linear_batch(const std::string &unit, size_t rows, size_t cols, const float *x, size_t n,
                      float *y) const {
        auto qit = quant.find(unit);
        if (qit != quant.end()) {
            for (size_t t = 0; t < n; ++t) {
                if (cfg.quant == ORACLE_QUANT_Q8) gemv_q8_impl(qit->second.data(), rows, cols, x + t * cols, y + t * rows);
                else gemv_q4_impl(qit->second.data(), rows, cols, x + t * cols, y + t * rows);
            }
            return true;
        }
        const OracleUnitRef *w;
        if (!require(unit, &w)) return false;
        if (w->dtype == ORACLE_BF16) {
            gemm_impl(w->data, w->dtype, rows, cols, x, n, y);
        } else {
            for (size_t t = 0; t < n; ++t) gemv_impl(w->data, w->dtype, rows, cols, x + t * cols, y + t * rows);
        }
        return true;
    }

    // ops.rs:1083-1099 embedding_row_into.
    bool embedding_row(size_t token, float *out) const {
        const OracleUnitRef *e;
        if (!require("model.embed_tokens.weight", &e)) return false;
        size_t base = token * cfg.hidden_size;
        for (size_t i = 0; i < cfg.hidden_size; ++i) out[i] = scalar_at(e->data, base + i, e->dtype);
        return true;
    }

    void cache_append(size_t layer, const float *kr, const float *vr) {
        kv_k[layer].insert(kv_k[layer].end(), kr, kr + kv_dim());
        kv_v[layer].insert(kv_v[layer].end(), vr, vr + kv_dim());
    }

    void attention(size_t layer, size_t position, const float *qv, float *out) const {
        size_t cache_len = kv_k[layer].size() / kv_dim();
        attention_impl(kv_k[layer].data(), kv_v[layer].data(), cache_len, position, qv,
                       cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.sliding_window, out);
    }

    // qwen2.rs:470-559 forward_attention.
    bool forward_attention(const std::string &prefix, size_t layer, size_t position) {
        size_t qd = q_dim(), kd = kv_dim();
        q.assign(qd, 0.0f);
        if (!linear(prefix + "self_attn.q_proj.weight", qd, cfg.hidden_size, normed.data(), q.data())) return false;
        add_bias(q.data(), qd, prefix + "self_attn.q_proj");
        k.assign(kd, 0.0f);
        if (!linear(prefix + "self_attn.k_proj.weight", kd, cfg.hidden_size, normed.data(), k.data())) return false;
        add_bias(k.data(), kd, prefix + "self_attn.k_proj");
        v.assign(kd, 0.0f);
        if (!linear(prefix + "self_attn.v_proj.weight", kd, cfg.hidden_size, normed.data(), v.data())) return false;
        add_bias(v.data(), kd, prefix + "self_attn.v_proj");
        // qwen3.rs:505-528: per-head q/k norms between the bias and rope.
        qk_norm(q.data(), cfg.q_heads, prefix + "self_attn.q_norm");
        qk_norm(k.data(), cfg.kv_heads, prefix + "self_attn.k_norm");
        rope_heads_impl(q.data(), cfg.q_heads, cfg.head_dim, cfg.rotary_dim, position, cfg.rope_theta);
        rope_heads_impl(k.data(), cfg.kv_heads, cfg.head_dim, cfg.rotary_dim, position, cfg.rope_theta);
        cache_append(layer, k.data(), v.data());
        attn_out.assign(qd, 0.0f);
        attention(layer, position, q.data(), attn_out.data());
        attn_projected.assign(cfg.hidden_size, 0.0f);
        if (!linear(prefix + "self_attn.o_proj.weight", cfg.hidden_size, qd, attn_out.data(), attn_projected.data())) return false;
        add_bias(attn_projected.data(), cfg.hidden_size, prefix + "self_attn.o_proj");
        return true;
    }

    // qwen2.rs:562-597 forward_mlp.
    bool forward_mlp(const std::string &prefix) {
        size_t inter = cfg.intermediate_size;
        gate.assign(inter, 0.0f);
        if (!linear(prefix + "mlp.gate_proj.weight", inter, cfg.hidden_size, normed.data(), gate.data())) return false;
        up.assign(inter, 0.0f);
        if (!linear(prefix + "mlp.up_proj.weight", inter, cfg.hidden_size, normed.data(), up.data())) return false;
        silu_multiply_impl(gate.data(), up.data(), inter);
        mlp_out.assign(cfg.hidden_size, 0.0f);
        return linear(prefix + "mlp.down_proj.weight", cfg.hidden_size, inter, gate.data(), mlp_out.data());
    }

    // qwen2.rs:430-465 forward_layer.
    bool forward_layer(size_t layer, size_t position) {
        std::string prefix = "model.layers." + std::to_string(layer) + ".";
        normed = hidden;
        if (!rmsnorm(prefix + "input_layernorm", normed.data())) return false;
        if (!forward_attention(prefix, layer, position)) return false;
        for (size_t i = 0; i < cfg.hidden_size; ++i) hidden[i] += attn_projected[i];
        normed = hidden;
        if (!rmsnorm(prefix + "post_attention_layernorm", normed.data())) return false;
        if (!forward_mlp(prefix)) return false;
        for (size_t i = 0; i < cfg.hidden_size; ++i) hidden[i] += mlp_out[i];
        return true;
    }

    // qwen2.rs:174-185 forward_position.
    bool forward_position(size_t token, size_t position) {
        hidden.assign(cfg.hidden_size, 0.0f);
        if (!embedding_row(token, hidden.data())) return false;
        for (size_t layer = 0; layer < cfg.num_layers; ++layer) {
            if (!forward_layer(layer, position)) return false;
        }
        return rmsnorm("model.norm", hidden.data());
    }

    // qwen2.rs:240-426 forward_layer_chunk.
    bool forward_layer_chunk(size_t layer, size_t offset, size_t rows) {
        size_t qd = q_dim(), kd = kv_dim(), hs = cfg.hidden_size, inter = cfg.intermediate_size;
        std::string prefix = "model.layers." + std::to_string(layer) + ".";
        c_normed = c_hidden;
        for (size_t r = 0; r < rows; ++r) {
            if (!rmsnorm(prefix + "input_layernorm", c_normed.data() + r * hs)) return false;
        }
        c_q.assign(rows * qd, 0.0f);
        if (!linear_batch(prefix + "self_attn.q_proj.weight", qd, hs, c_normed.data(), rows, c_q.data())) return false;
        c_k.assign(rows * kd, 0.0f);
        if (!linear_batch(prefix + "self_attn.k_proj.weight", kd, hs, c_normed.data(), rows, c_k.data())) return false;
        c_v.assign(rows * kd, 0.0f);
        if (!linear_batch(prefix + "self_attn.v_proj.weight", kd, hs, c_normed.data(), rows, c_v.data())) return false;
        for (size_t r = 0; r < rows; ++r) {
            add_bias(c_q.data() + r * qd, qd, prefix + "self_attn.q_proj");
            add_bias(c_k.data() + r * kd, kd, prefix + "self_attn.k_proj");
            add_bias(c_v.data() + r * kd, kd, prefix + "self_attn.v_proj");
        }
        // qwen3.rs:301-318: per-row q/k norms after the bias adds.
        for (size_t r = 0; r < rows; ++r) {
            qk_norm(c_q.data() + r * qd, cfg.q_heads, prefix + "self_attn.q_norm");
            qk_norm(c_k.data() + r * kd, cfg.kv_heads, prefix + "self_attn.k_norm");
        }
        c_attn_out.assign(rows * qd, 0.0f);
        for (size_t r = 0; r < rows; ++r) {
            size_t position = offset + r;
            rope_heads_impl(c_q.data() + r * qd, cfg.q_heads, cfg.head_dim, cfg.rotary_dim, position, cfg.rope_theta);
            rope_heads_impl(c_k.data() + r * kd, cfg.kv_heads, cfg.head_dim, cfg.rotary_dim, position, cfg.rope_theta);
            cache_append(layer, c_k.data() + r * kd, c_v.data() + r * kd);
            attention(layer, position, c_q.data() + r * qd, c_attn_out.data() + r * qd);
        }
        c_attn_projected.assign(rows * hs, 0.0f);
        if (!linear_batch(prefix + "self_attn.o_proj.weight", hs, qd, c_attn_out.data(), rows, c_attn_projected.data())) return false;
        for (size_t r = 0; r < rows; ++r) add_bias(c_attn_projected.data() + r * hs, hs, prefix + "self_attn.o_proj");
        for (size_t i = 0; i < rows * hs; ++i) c_hidden[i] += c_attn_projected[i];
        c_normed = c_hidden;
        for (size_t r = 0; r < rows; ++r) {
            if (!rmsnorm(prefix + "post_attention_layernorm", c_normed.data() + r * hs)) return false;
        }
        c_gate.assign(rows * inter, 0.0f);
        if (!linear_batch(prefix + "mlp.gate_proj.weight", inter, hs, c_normed.data(), rows, c_gate.data())) return false;
        c_up.assign(rows * inter, 0.0f);
        if (!linear_batch(prefix + "mlp.up_proj.weight", inter, hs, c_normed.data(), rows, c_up.data())) return false;
        for (size_t r = 0; r < rows; ++r) silu_multiply_impl(c_gate.data() + r * inter, c_up.data() + r * inter, inter);
        c_mlp_out.assign(rows * hs, 0.0f);
        if (!linear_batch(prefix + "mlp.down_proj.weight", hs, inter, c_gate.data(), rows, c_mlp_out.data())) return false;
        for (size_t i = 0; i < rows * hs; ++i) c_hidden[i] += c_mlp_out[i];
        return true;
    }

    // qwen2.rs:208-233 forward_chunk.
    bool forward_chunk(const uint32_t *tokens, size_t rows, size_t offset) {
        size_t hs = cfg.hidden_size;
        c_hidden.assign(rows * hs, 0.0f);
        for (size_t r = 0; r < rows; ++r) {
            if (!embedding_row(tokens[r], c_hidden.data() + r * hs)) return false;
        }
        for (size_t layer = 0; layer < cfg.num_layers; ++layer) {
            if (!forward_layer_chunk(layer, offset, rows)) return false;
        }
        hidden.assign(c_hidden.begin() + (rows - 1) * hs, c_hidden.begin() + rows * hs);
        return rmsnorm("model.norm", hidden.data());
    }

    // qwen2.rs:160-170 + ops.rs:1513-1563 lm_head (16384-row chunks).
    bool lm_head(float *logits) const {
        std::string head_unit = cfg.tie_word_embeddings ? "model.embed_tokens.weight" : "lm_head.weight";
        const OracleUnitRef *w = find(head_unit);
        if (w == nullptr) {
            set_error("Native backend: neither tied embeddings nor a separate '" + head_unit + "' tensor are present.");
            return false;
        }
        size_t row_stride = cfg.hidden_size * element_size(w->dtype);
        for (size_t start = 0; start < cfg.vocab_size; start += kLmHeadChunkRows) {
            size_t end = std::min<size_t>(cfg.vocab_size, start + kLmHeadChunkRows);
            gemv_impl(w->data + start * row_stride, w->dtype, end - start, cfg.hidden_size,
                      hidden.data(), logits + start);
        }
        return true;
    }
};

extern "C" {

OracleModel *oracle_model_new(const OracleConfig *cfg) {
    auto *model = new OracleModel();
    model->cfg = *cfg;
    model->kv_k.assign(cfg->num_layers, {});
    model->kv_v.assign(cfg->num_layers, {});
    return model;
}

void oracle_model_free(OracleModel *model) { delete model; }

int oracle_model_set_unit(OracleModel *model, const char *unit_id, const uint8_t *data, int dtype,
                          size_t bytes) {
    OracleUnitRef ref;
    ref.data = data;
    ref.dtype = dtype;
    ref.bytes = bytes;
    model->units[unit_id] = ref;
    return 0;
}

int oracle_model_prepare(OracleModel *model) {
    if (model->cfg.quant == ORACLE_QUANT_NONE) return 0;
    const OracleConfig &c = model->cfg;
    struct Lin { const char *name; size_t rows, cols; };
    size_t qd = c.q_heads * c.head_dim, kd = c.kv_heads * c.head_dim;
    const Lin lins[] = {
        {"self_attn.q_proj.weight", qd, c.hidden_size},
        {"self_attn.k_proj.weight", kd, c.hidden_size},
        {"self_attn.v_proj.weight", kd, c.hidden_size},
        {"self_attn.o_proj.weight", c.hidden_size, qd},
        {"mlp.gate_proj.weight", c.intermediate_size, c.hidden_size},
        {"mlp.up_proj.weight", c.intermediate_size, c.hidden_size},
        {"mlp.down_proj.weight", c.hidden_size, c.intermediate_size},
    };
    for (uint32_t layer = 0; layer < c.num_layers; ++layer) {
        for (const Lin &lin : lins) {
            std::string id = "model.layers." + std::to_string(layer) + "." + lin.name;
            const OracleUnitRef *w = model->find(id);
            if (w == nullptr) {
                set_error("Native backend: unknown unit '" + id + "'.");
                return -1;
            }
            if (w->bytes != lin.rows * lin.cols * element_size(w->dtype)) {
                set_error("Linear unit '" + id + "' does not match its shape.");
                return -1;
            }
            // ops.rs:634 dequant_values then the registered quantiser.
            std::vector<float> values(lin.rows * lin.cols);
            for (size_t i = 0; i < values.size(); ++i) values[i] = scalar_at(w->data, i, w->dtype);
            std::vector<uint8_t> buffer;
            if (c.quant == ORACLE_QUANT_Q8) {
                buffer.resize(oracle_q8_bytes(lin.rows, lin.cols));
                oracle_quantize_q8(values.data(), lin.rows, lin.cols, buffer.data());
            } else {
                buffer.resize(oracle_q4_bytes(lin.rows, lin.cols));
                oracle_quantize_q4(values.data(), lin.rows, lin.cols, buffer.data());
            }
            model->quant[id] = std::move(buffer);
        }
    }
    return 0;
}

// qwen2.rs:138-157 forward_with_chunk.
int oracle_model_forward(OracleModel *model, const uint32_t *tokens, size_t n, size_t offset,
                         size_t chunk_rows, float *logits) {
    // ops.rs:1065-1078 validate_tokens.
    if (n == 0) {
        set_error("Native backend: empty token input.");
        return -1;
    }
    for (size_t i = 0; i < n; ++i) {
        if (tokens[i] >= model->cfg.vocab_size) {
            set_error("Native backend: token id " + std::to_string(tokens[i]) +
                      " exceeds the vocabulary size " + std::to_string(model->cfg.vocab_size) + ".");
            return -1;
        }
    }
    if (chunk_rows == 0) chunk_rows = kPrefillChunkRows;
    bool ok;
    if (n == 1) {
        ok = model->forward_position(tokens[0], offset);
    } else {
        ok = true;
        for (size_t start = 0; ok && start < n; start += chunk_rows) {
            size_t end = std::min(n, start + chunk_rows);
            ok = model->forward_chunk(tokens + start, end - start, offset + start);
        }
    }
    if (!ok) return -1;
    return model->lm_head(logits) ? 0 : -1;
}

void oracle_model_clear(OracleModel *model) {
    for (auto &layer : model->kv_k) layer.clear();
    for (auto &layer : model->kv_v) layer.clear();
}

size_t oracle_model_positions(const OracleModel *model) {
    if (model->kv_k.empty()) return 0;
    return model->kv_k[0].size() / model->kv_dim();
}

int oracle_model_kv_export(const OracleModel *model, size_t layer, float *k, float *v) {
    if (layer >= model->kv_k.size()) return -1;
    std::memcpy(k, model->kv_k[layer].data(), model->kv_k[layer].size() * 4);
    std::memcpy(v, model->kv_v[layer].data(), model->kv_v[layer].size() * 4);
    return 0;
}

// ops.rs:1593-1607 restore_kv_prefix.
int oracle_model_kv_restore(OracleModel *model, size_t positions, const float *const *k_layers,
                            const float *const *v_layers) {
    size_t count = positions * model->kv_dim();
    for (size_t layer = 0; layer < model->kv_k.size(); ++layer) {
        model->kv_k[layer].assign(k_layers[layer], k_layers[layer] + count);
        model->kv_v[layer].assign(v_layers[layer], v_layers[layer] + count);
    }
    return 0;
}

int oracle_model_hidden(const OracleModel *model, float *out) {
    std::memcpy(out, model->hidden.data(), model->hidden.size() * 4);
    return static_cast<int>(model->hidden.size());
}

}  // extern "C"
