/*
 * snb_oracle.c — TEST INFRASTRUCTURE ONLY. A CPU restatement of the reference's arithmetic for the GEMM hot path,
 * used as the parity checker by tests/, by __graft_entry__.smoke() and as bench.py's CPU baseline. Nothing in the
 * product library links, loads or calls this file.
 *
 * Reference: arpanpathak/staleynet (Rust). Its CPU reference cannot be built here (no Rust toolchain), so every
 * function below restates one reference function and cites it (paths relative to the reference repository).
 * Parity pin: the known-answer tests of crates/staleynet-cuda/src/reference.rs:177-366 (tests/golden/) and the
 * published SplitMix64 output sequence (Steele, Lea & Flood 2014; the reference's random.rs:4-50 uses it).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../include/snb_matmul.h"

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------------------------------------------
 * GEMM: reference::matmul (crates/staleynet-cuda/src/reference.rs:18-38). For each batch, row and col: an f32
 * accumulator summed over `inner` in increasing order, then `scale*sum` (overwrite) or `C + scale*sum`
 * (accumulate). The reference reads operands through `logical()` (reference.rs:10-16), i.e. through Storage; the
 * general stride form used by the kernels (`Operand::at`, kernels/matmul.rs:120-125) is identical for those
 * layouts and is what is restated here.
 * ------------------------------------------------------------------------------------------------------------- */
static inline float operand_at(const float* values, const snb_operand* op, uint64_t batch, uint64_t row, uint64_t col) {
    return values[batch * op->batch_stride + row * op->row_stride + col * op->col_stride];
}

/* Rows [row_begin, row_end) of every matrix of the batch. */
void snb_oracle_matmul_rows(const snb_product* p, uint64_t count, const float* left, const float* right,
                            float* output, uint64_t row_begin, uint64_t row_end) {
    for (uint64_t batch = 0; batch < count; ++batch) {
        for (uint64_t row = row_begin; row < row_end && row < p->rows; ++row) {
            for (uint64_t col = 0; col < p->cols; ++col) {
                float sum = 0.0f;
                for (uint64_t step = 0; step < p->inner; ++step) {
                    sum += operand_at(left, &p->left, batch, row, step) * operand_at(right, &p->right, batch, step, col);
                }
                float* slot = &output[batch * p->output_batch_stride + row * p->cols + col];
                *slot = p->accumulate ? *slot + p->scale * sum : p->scale * sum;
            }
        }
    }
}

/* The whole product, single-threaded: exactly reference::matmul. */
void snb_oracle_matmul(const snb_product* p, uint64_t count, const float* left, const float* right, float* output) {
    snb_oracle_matmul_rows(p, count, left, right, output, 0, p->rows);
}

/* The same loop over the output block [row_begin, row_end) x [0, cols), output elements split over `threads`
 * OpenMP threads (0 = all). Each output element is still the reference's sequential f32 sum, so results are
 * bit-identical to snb_oracle_matmul. Used as the all-cores CPU baseline. Returns the thread count used. */
int snb_oracle_matmul_parallel(const snb_product* p, uint64_t count, const float* left, const float* right,
                               float* output, uint64_t row_begin, uint64_t row_end, int threads) {
    int used = 1;
    const int64_t begin = (int64_t)row_begin, end = (int64_t)(row_end < p->rows ? row_end : p->rows);
    const int64_t cols = (int64_t)p->cols;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
    used = threads;
#pragma omp parallel for collapse(3) num_threads(threads) schedule(static)
#endif
    for (int64_t batch = 0; batch < (int64_t)count; ++batch) {
        for (int64_t row = begin; row < end; ++row) {
            for (int64_t col = 0; col < cols; ++col) {
                float sum = 0.0f;
                for (uint64_t step = 0; step < p->inner; ++step) {
                    sum += operand_at(left, &p->left, (uint64_t)batch, (uint64_t)row, step) *
                           operand_at(right, &p->right, (uint64_t)batch, step, (uint64_t)col);
                }
                float* slot = &output[batch * p->output_batch_stride + row * p->cols + col];
                *slot = p->accumulate ? *slot + p->scale * sum : p->scale * sum;
            }
        }
    }
#ifndef _OPENMP
    (void)threads;
#endif
    return used;
}

/* The same product with an f64 accumulator (the "exact" reference for error measurements). */
void snb_oracle_matmul_f64(const snb_product* p, uint64_t count, const float* left, const float* right,
                           double* output) {
    for (uint64_t batch = 0; batch < count; ++batch) {
        for (uint64_t row = 0; row < p->rows; ++row) {
            for (uint64_t col = 0; col < p->cols; ++col) {
                double sum = 0.0;
                for (uint64_t step = 0; step < p->inner; ++step) {
                    sum += (double)operand_at(left, &p->left, batch, row, step) *
                           (double)operand_at(right, &p->right, batch, step, col);
                }
                double* slot = &output[batch * p->output_batch_stride + row * p->cols + col];
                *slot = p->accumulate ? *slot + (double)p->scale * sum : (double)p->scale * sum;
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Input rounding, to build the expected result of reduced-precision tensor-core arithmetic.
 * ------------------------------------------------------------------------------------------------------------- */

/* f32 -> TF32 with round-to-nearest, ties away from zero: what `cvt.rna.tf32.f32` does to every staged value in
 * the reference's tensor-core kernel (kernels/matmul.rs:397-398). Keeps 10 mantissa bits. */
void snb_oracle_round_tf32(const float* input, float* output, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t bits;
        memcpy(&bits, &input[i], 4);
        if ((bits & 0x7f800000u) != 0x7f800000u) { /* finite: add half an ulp of the kept precision, truncate */
            bits += 0x1000u;
            bits &= 0xffffe000u;
        }
        memcpy(&output[i], &bits, 4);
    }
}

/* f32 -> bf16 with round-to-nearest-even (IEEE default), returned as f32 values and as raw bf16 bits. */
void snb_oracle_round_bf16(const float* input, float* output, uint16_t* bits_out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t bits;
        memcpy(&bits, &input[i], 4);
        uint32_t rounded;
        if ((bits & 0x7f800000u) == 0x7f800000u) {
            rounded = (bits & 0xffff0000u) | ((bits & 0xffffu) ? 0x400000u : 0u); /* keep inf; NaN stays NaN */
        } else {
            rounded = (bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u;
        }
        if (output) memcpy(&output[i], &rounded, 4);
        if (bits_out) bits_out[i] = (uint16_t)(rounded >> 16);
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Seeded inputs: SplitMix64 + Box-Muller, restating crates/staleynet-model/src/random.rs:27-70.
 * ------------------------------------------------------------------------------------------------------------- */
#define SNB_GOLDEN_GAMMA 0x9E3779B97F4A7C15ull
#define SNB_MIX_1 0xBF58476D1CE4E5B9ull
#define SNB_MIX_2 0x94D049BB133111EBull

/* `Random::next_u64` (random.rs:39-46). */
uint64_t snb_oracle_next_u64(uint64_t* state) {
    *state += SNB_GOLDEN_GAMMA;
    uint64_t mixed = *state;
    mixed = (mixed ^ (mixed >> 30)) * SNB_MIX_1;
    mixed = (mixed ^ (mixed >> 27)) * SNB_MIX_2;
    return mixed ^ (mixed >> 31);
}

/* `Random::uniform` (random.rs:49-51): the top 24 bits over 2^24, in [0, 1). */
float snb_oracle_uniform(uint64_t* state) {
    return (float)(snb_oracle_next_u64(state) >> 40) / (float)(1u << 24);
}

/* `Random::below` (random.rs:54-56). */
uint64_t snb_oracle_below(uint64_t* state, uint64_t bound) {
    return snb_oracle_next_u64(state) % bound;
}

/* `Random::normal` (random.rs:64-68): radius from a uniform clamped below at 1e-7, angle 2*pi*uniform, in f32. */
float snb_oracle_normal(uint64_t* state) {
    float u = snb_oracle_uniform(state);
    if (u < 1e-7f) u = 1e-7f;
    float radius = sqrtf(-2.0f * logf(u));
    float angle = 6.28318530717958647692f * snb_oracle_uniform(state);
    return radius * cosf(angle);
}

/* `Init::Normal(std)` (crates/staleynet-model/src/parameter.rs:54): n draws of normal()*std, in order. */
void snb_oracle_fill_normal(uint64_t* state, float std, float* output, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) output[i] = snb_oracle_normal(state) * std;
}

/* Uniform integer targets in [0, bound), as the reference's bench batches (bench.rs:152-154). */
void snb_oracle_fill_below(uint64_t* state, uint64_t bound, uint32_t* output, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) output[i] = (uint32_t)snb_oracle_below(state, bound);
}

/* The parity tests' input generator: Knuth's MMIX LCG mapped to roughly [-1, 1]
 * (crates/staleynet-cuda/tests/kernels_match_reference.rs:26-38). */
void snb_oracle_fill_lcg(uint64_t seed, float* output, uint64_t n) {
    uint64_t state = seed * 6364136223846793005ull + 1442695040888963407ull;
    for (uint64_t i = 0; i < n; ++i) {
        state = state * 6364136223846793005ull + 1442695040888963407ull;
        output[i] = ((float)(state >> 40) / (float)(1ull << 24)) * 2.0f - 1.0f;
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * The elementwise neighbours of the GEMMs (their contracts fix what the fused epilogues must produce).
 * ------------------------------------------------------------------------------------------------------------- */
#define SNB_GELU_SQRT_2_OVER_PI 0.7978846f /* kernels/elementwise.rs:9 */
#define SNB_GELU_CUBIC 0.044715f           /* kernels/elementwise.rs:12 */

/* reference::gelu (reference.rs:40-43), tanh approximation. */
float snb_oracle_gelu(float x) {
    return 0.5f * x * (1.0f + tanhf(SNB_GELU_SQRT_2_OVER_PI * (x + SNB_GELU_CUBIC * x * x * x)));
}

/* reference::gelu_derivative (reference.rs:45-49). */
float snb_oracle_gelu_derivative(float x) {
    float t = tanhf(SNB_GELU_SQRT_2_OVER_PI * (x + SNB_GELU_CUBIC * x * x * x));
    return 0.5f * (1.0f + t) +
           0.5f * x * (1.0f - t * t) * SNB_GELU_SQRT_2_OVER_PI * (1.0f + 3.0f * SNB_GELU_CUBIC * x * x);
}

void snb_oracle_gelu_fill(const float* input, float* output, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) output[i] = snb_oracle_gelu(input[i]);
}

void snb_oracle_gelu_derivative_fill(const float* input, float* output, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) output[i] = snb_oracle_gelu_derivative(input[i]);
}

/* reference::causal_softmax (reference.rs:100-120), in place over [rows, keys]. */
void snb_oracle_causal_softmax(float* scores, uint64_t rows, uint64_t queries, uint64_t keys, float scale,
                               uint64_t query_offset) {
    for (uint64_t row = 0; row < rows; ++row) {
        float* values = scores + row * keys;
        uint64_t visible = row % queries + query_offset + 1;
        if (visible > keys) visible = keys;
        float maximum = -INFINITY;
        for (uint64_t k = 0; k < visible; ++k) maximum = fmaxf(maximum, values[k] * scale);
        for (uint64_t k = 0; k < visible; ++k) values[k] = expf(values[k] * scale - maximum);
        float total = 0.0f;
        for (uint64_t k = 0; k < visible; ++k) total += values[k];
        for (uint64_t k = 0; k < visible; ++k) values[k] /= total;
        for (uint64_t k = visible; k < keys; ++k) values[k] = 0.0f;
    }
}

/* reference::softmax_backward (reference.rs:122-137), in place on grad. */
void snb_oracle_softmax_backward(const float* probabilities, float* grad, uint64_t rows, uint64_t cols) {
    for (uint64_t row = 0; row < rows; ++row) {
        const float* p = probabilities + row * cols;
        float* g = grad + row * cols;
        float projection = 0.0f;
        for (uint64_t c = 0; c < cols; ++c) projection += g[c] * p[c];
        for (uint64_t c = 0; c < cols; ++c) g[c] = p[c] * (g[c] - projection);
    }
}

/* reference::cross_entropy (reference.rs:139-166) for one head: per row, loss = log_partition - z[target] and the
 * head's gradient columns ((exp(z - log_partition) - onehot) * grad_scale), f32 throughout; rows whose target is
 * EMPTY_TOKEN (u32::MAX, kernels/mod.rs:46) get loss 0 and a zero gradient. Other columns are left untouched. */
void snb_oracle_cross_entropy(const float* logits, const uint32_t* targets, uint64_t rows, uint64_t cols,
                              uint64_t column_offset, uint64_t classes, uint64_t target_stride, uint64_t target_offset,
                              float grad_scale, float* losses, float* logits_grad) {
    for (uint64_t row = 0; row < rows; ++row) {
        const float* z = logits + row * cols + column_offset;
        float* g = logits_grad + row * cols + column_offset;
        const uint32_t target = targets[row * target_stride + target_offset];
        if (target == 0xFFFFFFFFu) {
            losses[row] = 0.0f;
            for (uint64_t c = 0; c < classes; ++c) g[c] = 0.0f;
            continue;
        }
        float maximum = -INFINITY;
        for (uint64_t c = 0; c < classes; ++c) maximum = fmaxf(maximum, z[c]);
        float total = 0.0f;
        for (uint64_t c = 0; c < classes; ++c) total += expf(z[c] - maximum);
        const float log_partition = maximum + logf(total);
        losses[row] = log_partition - z[target];
        for (uint64_t c = 0; c < classes; ++c) {
            const float one_hot = (uint64_t)target == c ? 1.0f : 0.0f;
            g[c] = (expf(z[c] - log_partition) - one_hot) * grad_scale;
        }
    }
}

/* reference::rms_norm_forward (reference.rs:60-77): per row s = 1 / sqrt(mean(x^2) + epsilon), y = x * s * g. */
void snb_oracle_rms_norm_forward(const float* input, const float* gain, uint64_t rows, uint64_t cols, float epsilon,
                                 float* output, float* inv_rms) {
    for (uint64_t row = 0; row < rows; ++row) {
        const float* x = input + row * cols;
        float square_sum = 0.0f;
        for (uint64_t c = 0; c < cols; ++c) square_sum += x[c] * x[c];
        const float inverse = 1.0f / sqrtf(square_sum / (float)cols + epsilon);
        for (uint64_t c = 0; c < cols; ++c) output[row * cols + c] = x[c] * inverse * gain[c];
        inv_rms[row] = inverse;
    }
}

/* reference::rms_norm_backward (reference.rs:79-98): dx = s g dy - x s^3 / cols * sum(dy g x); gain_grad += dy x s
 * (added to, as the GPU kernel accumulates). */
void snb_oracle_rms_norm_backward(const float* output_grad, const float* input, const float* gain,
                                  const float* inv_rms, uint64_t rows, uint64_t cols, float* input_grad,
                                  float* gain_grad) {
    for (uint64_t row = 0; row < rows; ++row) {
        const float* dy = output_grad + row * cols;
        const float* x = input + row * cols;
        const float inverse = inv_rms[row];
        float projection = 0.0f;
        for (uint64_t c = 0; c < cols; ++c) projection += dy[c] * gain[c] * x[c];
        const float correction = inverse * inverse * inverse * projection / (float)cols;
        for (uint64_t c = 0; c < cols; ++c) {
            input_grad[row * cols + c] = inverse * gain[c] * dy[c] - x[c] * correction;
            gain_grad[c] += dy[c] * x[c] * inverse;
        }
    }
}

/* The AdamW update of the reference's kernel (kernels/optimizer.rs:47-71) and its parity test
 * (tests/kernels_match_reference.rs:299-327), with first_correction = 1 - beta1^step and
 * second_correction = 1 - beta2^step as ops/optimizer.rs:44-54 computes them. */
void snb_oracle_adamw_step(float* parameter, const float* gradient, float* first_moment, float* second_moment,
                           uint64_t count, float learning_rate, float beta1, float beta2, float epsilon,
                           float weight_decay, uint32_t step) {
    float b1 = 1.0f, b2 = 1.0f;
    for (uint32_t i = 0; i < step; ++i) {
        b1 *= beta1;
        b2 *= beta2;
    }
    const float first_correction = 1.0f - b1, second_correction = 1.0f - b2;
    for (uint64_t i = 0; i < count; ++i) {
        const float grad = gradient[i];
        const float mean = beta1 * first_moment[i] + (1.0f - beta1) * grad;
        const float variance = beta2 * second_moment[i] + (1.0f - beta2) * grad * grad;
        first_moment[i] = mean;
        second_moment[i] = variance;
        const float mean_hat = mean / first_correction;
        const float variance_hat = variance / second_correction;
        const float weight = parameter[i];
        const float update = mean_hat / (sqrtf(variance_hat) + epsilon) + weight_decay * weight;
        parameter[i] = weight - learning_rate * update;
    }
}

/* sum of squares in f64 (the reference sums its f32 partial sums as f64, ops/optimizer.rs:72-85). */
double snb_oracle_sum_of_squares(const float* values, uint64_t count) {
    double sum = 0.0;
    for (uint64_t i = 0; i < count; ++i) sum += (double)values[i] * (double)values[i];
    return sum;
}

int snb_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
