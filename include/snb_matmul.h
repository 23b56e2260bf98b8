/*
 * snb_matmul.h — C ABI of the B200 (sm_100a) dense-contraction library.
 *
 * This is the drop-in boundary for StaleyNET's GEMM hot path. Every entry point here replaces one entry point of
 * the reference crate `staleynet-cuda` (paths below are relative to the reference repository):
 *
 *   snb_product / snb_operand   <- `Product` / `Operand`, crates/staleynet-cuda/src/kernels/matmul.rs:108-157
 *   snb_matmul                  <- `Gpu::matmul`, crates/staleynet-cuda/src/ops/matmul.rs:144-172
 *   snb_matmul_bf16             <- `Gpu::matmul` with bf16 operands (no reference counterpart: the reference has
 *                                  only f32 tensors, device.rs:245-275; this is the bf16 tensor-core variant)
 *   snb_gemm                    <- `Gpu::matmul` followed by the elementwise pass a caller runs on its output:
 *                                  `add_row_bias` (ops/elementwise.rs, kernels/elementwise.rs:62),
 *                                  `gelu_forward`/`gelu_backward` (kernels/elementwise.rs:139-159) and
 *                                  `add_scaled` residual adds (kernels/elementwise.rs:37), fused into the epilogue
 *   snb_causal_softmax          <- `Gpu::causal_softmax`, crates/staleynet-cuda/src/ops/attention.rs:61-81
 *   snb_softmax_backward        <- `Gpu::softmax_backward`, crates/staleynet-cuda/src/ops/attention.rs:84-100
 *   snb_head_layout             <- `HeadLayout`, crates/staleynet-cuda/src/kernels/attention.rs:19-41
 *   snb_split_heads             <- `Gpu::split_heads`, crates/staleynet-cuda/src/ops/attention.rs:20-36
 *   snb_merge_heads             <- `Gpu::merge_heads`, crates/staleynet-cuda/src/ops/attention.rs:38-52
 *
 * Conventions shared by every entry point:
 *   - All pointers are caller-owned device pointers; nothing is allocated or freed inside a call.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream). Calls are asynchronous and
 *     ordered on that stream, like the reference's single `Gpu::stream` (device.rs:129-145). The tensor-core GEMM
 *     kernels use programmatic dependent launch: each waits (griddepcontrol.wait) for the previous kernel of the
 *     stream to complete before touching global memory, and lets the next one be scheduled early
 *     (griddepcontrol.launch_dependents). A caller's own kernel launched right after with programmatic stream
 *     serialisation must therefore call griddepcontrol.wait before reading a GEMM's output; ordinary launches,
 *     events and copies are ordered exactly as without it.
 *   - Lengths are element counts, the `len()` of the reference's `Tensor` (device.rs:262-265).
 *   - Return value: SNB_OK or a positive SNB_ERR_* code. The reference panics on undersized operands
 *     (ops/matmul.rs:147-149) and returns `DriverError` on launch failure; here both become status codes, and
 *     snb_last_error() gives the message of the last failure on the calling thread.
 */
#ifndef SNB_MATMUL_H
#define SNB_MATMUL_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SNB_API __attribute__((visibility("default")))
#else
#define SNB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element (row, col) of matrix b of a batch is values[b*batch_stride + row*row_stride + col*col_stride].
 * Same fields and order as `Operand` (kernels/matmul.rs:108-126); Rust's usize is uint64_t on LP64. */
typedef struct snb_operand {
    uint64_t row_stride;
    uint64_t col_stride;
    uint64_t batch_stride;
} snb_operand;

/* One batched product C_b = scale * A_b * B_b (+ C_b), A_b [rows, inner], B_b [inner, cols], C_b row-major
 * [rows, cols] at b*output_batch_stride. Byte-identical to `Product` (kernels/matmul.rs:128-157): 88 bytes. */
typedef struct snb_product {
    uint64_t rows;
    uint64_t cols;
    uint64_t inner;
    snb_operand left;
    snb_operand right;
    uint64_t output_batch_stride;
    float scale;
    uint32_t accumulate; /* 1: C += scale*A*B; 0: C = scale*A*B (`WriteMode::flag`, ops/mod.rs:36-43) */
} snb_product;

/* Where a group of attention heads lives in two layouts. Packed: [batch * time, width], head h of a row at columns
 * column_offset + h * head_dim ..; head-major: [batch, heads, time_capacity, head_dim], the moved time steps at
 * rows time_offset .. (which lets the same copy append to a key/value cache). Byte-identical to the reference's
 * `HeadLayout` (crates/staleynet-cuda/src/kernels/attention.rs:19-41, repr(C), 8 x usize = 64 bytes). */
typedef struct snb_head_layout {
    uint64_t batch;
    uint64_t time;
    uint64_t heads;
    uint64_t head_dim;
    uint64_t width;
    uint64_t column_offset;
    uint64_t time_capacity;
    uint64_t time_offset;
} snb_head_layout;

/* Arithmetic of a product. Maps `MatmulKernel` (device.rs:38-67): Naive/Tiled/Blocked compute exact f32
 * (tolerance 1e-5) -> SNB_PRECISION_F32; TensorCore rounds inputs to TF32 (tolerance 2e-3) -> SNB_PRECISION_TF32.
 * SNB_PRECISION_BF16 is the bf16 tensor-core path and needs bf16 operands (snb_matmul_bf16 / snb_gemm). */
enum {
    SNB_PRECISION_F32 = 0,
    SNB_PRECISION_TF32 = 1,
    SNB_PRECISION_BF16 = 2
};

/* Element types of snb_gemm operands and outputs. */
enum {
    SNB_TYPE_F32 = 0,
    SNB_TYPE_BF16 = 1
};

/* Elementwise function applied in the epilogue of snb_gemm, after scale and bias. */
enum {
    SNB_ACTIVATION_NONE = 0,
    SNB_ACTIVATION_GELU = 1,     /* out = gelu(x); x optionally stored to pre_activation (feed_forward.rs:55-59) */
    SNB_ACTIVATION_GELU_GRAD = 2 /* out = x * gelu'(gelu_input) (`gelu_backward`, kernels/elementwise.rs:153) */
};

/* Causal structure of a batched attention product, so the kernel can skip work the causal softmax makes void.
 * Query q of each matrix sees keys 0..=q+offset (`causal_softmax`, kernels/attention.rs:153-180); masked scores
 * are never read by the softmax and masked probabilities are 0.
 *   SKIP_MASKED_OUTPUT  output is a [queries, keys] score matrix (Q*K^T, dO*V^T): tiles whose every element is
 *                       masked are not computed and keep their previous contents.
 *   LEFT_MASKED         left operand is a [queries, keys] probability-like matrix, zero after key q+offset
 *                       (P*V, dS*K): the sum over keys stops there.
 *   LEFT_T_MASKED       left operand is such a matrix transposed, [keys, queries] (P^T*dO, dS^T*Q): the sum
 *                       over queries starts at key-offset.
 * The SIMT kernel ignores the hint (it computes every element, which the hint's contract allows). */
enum {
    SNB_CAUSAL_NONE = 0,
    SNB_CAUSAL_SKIP_MASKED_OUTPUT = 1,
    SNB_CAUSAL_LEFT_MASKED = 2,
    SNB_CAUSAL_LEFT_T_MASKED = 3
};

/* Status codes. */
enum {
    SNB_OK = 0,
    SNB_ERR_LEFT_TOO_SMALL = 1,   /* "matmul: left operand too small" (ops/matmul.rs:147) */
    SNB_ERR_RIGHT_TOO_SMALL = 2,  /* "matmul: right operand too small" (ops/matmul.rs:148) */
    SNB_ERR_OUTPUT_TOO_SMALL = 3, /* "matmul: output too small" (ops/matmul.rs:149) */
    SNB_ERR_INVALID_ARGUMENT = 4, /* null pointer, zero batch count, unknown enum value, bad shape */
    SNB_ERR_UNSUPPORTED = 5,      /* combination this build does not implement (message says which) */
    SNB_ERR_CUDA = 6,             /* a CUDA runtime/driver call failed (message carries the CUDA error) */
    SNB_ERR_DEVICE_TIMEOUT = 7    /* a kernel's bounded wait gave up; see snb_device_status() */
};

/* Which kernel family ran the last successful call on this thread (for tests and tracing). */
enum {
    SNB_PATH_NONE = 0,
    SNB_PATH_TENSOR_CORE = 1, /* tcgen05 + TMA persistent kernel */
    SNB_PATH_SIMT = 2,        /* strided SIMT kernel: any strides and alignments, exact f32 FMA */
    SNB_PATH_EMPTY = 3,       /* nothing to compute (rows or cols is 0) */
    SNB_PATH_TENSOR_CORE_PAIR = 4 /* tcgen05 kernel on CTA pairs (cta_group::2, 256 x 256 tiles) */
};

/* Batched strided GEMM on f32 operands: replaces `Gpu::matmul` (ops/matmul.rs:146-171).
 * `count` is `BatchStrides::count` (the reference passes it as the grid's z extent, launch.rs:28-48).
 * precision: SNB_PRECISION_F32 or SNB_PRECISION_TF32.
 * Checks, in the reference's order, left_len/right_len/output_len >= the elements the batch addresses. */
SNB_API int snb_matmul(void* stream, const snb_product* product, uint64_t count,
               const float* left, uint64_t left_len,
               const float* right, uint64_t right_len,
               float* output, uint64_t output_len,
               int32_t precision);

/* As snb_matmul, with bf16 operands (raw 16-bit bf16 bit patterns) and an f32 output; always bf16 tensor cores
 * (or the SIMT kernel on bf16 inputs when strides or alignment rule out TMA). No reference counterpart. */
SNB_API int snb_matmul_bf16(void* stream, const snb_product* product, uint64_t count,
                    const uint16_t* left, uint64_t left_len,
                    const uint16_t* right, uint64_t right_len,
                    float* output, uint64_t output_len);

/* A product with its caller's elementwise follow-up fused into the epilogue. For each output element
 *   x   = scale * (A*B)[r,c] + (bias ? bias[c] : 0)
 *   y   = activation(x)                      (pre_activation[r,c] = x when requested)
 *   out = y + (residual ? residual[r,c] : 0) (+ out[r,c] when product->accumulate)
 * Same meaning as `Linear::forward` (linear.rs:43-48) + `gelu_forward` + `add_scaled(1.0, residual, out)`
 * (block.rs:182,188), done in one pass over the output. */
typedef struct snb_gemm_args {
    snb_product product;
    uint64_t count;
    int32_t left_type;   /* SNB_TYPE_F32 (with precision F32/TF32) or SNB_TYPE_BF16 (precision BF16) */
    int32_t right_type;  /* must equal left_type */
    int32_t output_type; /* SNB_TYPE_F32 or SNB_TYPE_BF16 (bf16 output needs accumulate == 0) */
    int32_t precision;   /* SNB_PRECISION_* */
    const void* left;
    uint64_t left_len;
    const void* right;
    uint64_t right_len;
    void* output;
    uint64_t output_len;
    const float* bias;          /* [cols] or NULL */
    int32_t activation;         /* SNB_ACTIVATION_* */
    int32_t aux_type;           /* element type of pre_activation / gelu_input: SNB_TYPE_F32 or SNB_TYPE_BF16 */
    void* pre_activation;       /* GELU: receives x, laid out like the output; or NULL */
    const void* gelu_input;     /* GELU_GRAD: the forward pre-activation, laid out like the output */
    const void* residual;       /* laid out like the output, same type as the output; or NULL */
    int32_t causal;             /* SNB_CAUSAL_*: structure of a batched attention product (work it may skip) */
    int32_t flags;              /* SNB_GEMM_* bits; 0 for the default behaviour */
    int64_t causal_offset;      /* query q sees keys 0..=q+causal_offset (the softmax's query_offset) */
    const float* row_scale;     /* [rows] multiplier of each output row before the bias (count 1 only), or NULL:
                                 * with the RMSNorm gain folded into the right operand (snb_scale_rows) and
                                 * row_scale = the rows' 1/rms (snb_rms_norm_stats), left * right = rms_norm(left)
                                 * times the unscaled right operand, without a normalised copy of left. */
    /* Head-major operands (count 1; NULL = off), which fuse the reference's split_heads / merge_heads permutes
     * (crates/staleynet-model/src/layers/attention.rs:201-214, 233, 262-264) into the products around attention.
     * left_heads: `left` is the head-major form ([batch, heads, time_capacity, head_dim]) of the packed tensor
     * [batch * time, width] (width = heads * head_dim, column_offset 0) that product->left describes, RowMajor
     * (rows = batch * time, inner = width) or Transposed (rows = width, inner = batch * time); left_len counts the
     * head-major tensor. E.g. the attention output projection reading the attention context, and its weight
     * gradient. Needs head_dim a multiple of 64 (bf16) / 32 (tf32) and time a multiple of 128 (RowMajor) or
     * 64 (bf16) / 32 (tf32) (Transposed).
     * output_heads: the output [rows, cols] = [batch * time, cols] is written as cols / (heads * head_dim)
     * head-major tensors [batch, heads, time_capacity, head_dim] one after the other (output_heads->width = cols,
     * column_offset 0): column (p * heads + h) * head_dim + d of row b * time + s goes to element
     * ((b * heads + h) * time_capacity + time_offset + s) * head_dim + d of tensor p. E.g. the fused QKV
     * projection writing queries, keys and values head-major. Needs an overwrite without residual,
     * pre-activation or GELU input, head_dim a multiple of 64 (bf16 output) / 32 (f32) and time a multiple of 32;
     * output_len counts all the head-major tensors.
     * Both run on the tensor-core kernel only; other shapes return SNB_ERR_UNSUPPORTED (use snb_permute_heads). */
    const snb_head_layout* left_heads;
    const snb_head_layout* output_heads;
} snb_gemm_args;

SNB_API int snb_gemm(void* stream, const snb_gemm_args* args);

/* snb_gemm_args.flags bits.
 * Run-to-run reproducibility. By default a product whose K range the tensor-core kernel splits across CTAs (f32
 * outputs without activation, when its cost model finds idle SMs otherwise, e.g. weight gradients with K = tokens)
 * adds the splits' partial sums into the output with TMA reduce-adds in arrival order, so two runs on the same
 * inputs can differ in the last bits of those outputs. The reference's sum is a fixed-order f32 loop
 * (crates/staleynet-cuda/src/reference.rs:18-38). With SNB_GEMM_DETERMINISTIC every output element is summed in a
 * fixed order: each split stores its partial tile into its own slab of a stream-ordered workspace (cudaMallocAsync /
 * cudaFreeAsync on the call's stream, splits x rows x cols floats), then one kernel adds the slabs into the output
 * in split order (after the output's previous contents when accumulating); batched products (count > 1) are not
 * split at all. Results are then bit-identical between runs on the same device; the cost is the slabs' traffic.
 * Unsplit products, the SIMT kernel and the attention-product paths are deterministic either way. */
enum {
    SNB_GEMM_DETERMINISTIC = 1
};

/* Caps, for the calling thread, the SMs that the persistent tensor-core GEMM grid of later snb_matmul,
 * snb_matmul_bf16 and snb_gemm calls may occupy (sms <= 0: all of them, the default). The GEMM kernels keep one CTA
 * (or CTA pair) per SM for the whole launch and assign work units to CTAs statically, so a kernel that holds some SMs
 * meanwhile (a collective on another stream) stretches every GEMM by a whole CTA's share of work; with a budget the
 * GEMM leaves those SMs free. Returns the previous setting. No reference counterpart. */
SNB_API int snb_set_sm_budget(int32_t sms);

/* Sets, for the calling thread, whether snb_matmul, snb_matmul_bf16 and snb_gemm run as with SNB_GEMM_DETERMINISTIC
 * (enabled != 0) — the switch for callers of the f32 drop-in, which has no flags argument. Returns the previous
 * setting (0 or 1). Off by default. No reference counterpart. */
SNB_API int snb_set_deterministic(int32_t enabled);

/* In-place causal softmax of scores [rows, keys] (rows = matrices * queries): query q of each matrix sees keys
 * 0..=q+query_offset, scaled by `scale`, later keys become 0. Replaces `Gpu::causal_softmax`
 * (ops/attention.rs:61-81; kernel kernels/attention.rs:153-180). scores_len must be >= rows*keys. */
SNB_API int snb_causal_softmax(void* stream, float* scores, uint64_t scores_len, uint64_t rows, uint64_t queries,
                       uint64_t keys, float scale, uint64_t query_offset);

/* In place on grad [rows, cols]: grad = p * (grad - sum(grad * p)) per row. Replaces `Gpu::softmax_backward`
 * (ops/attention.rs:84-100; kernel kernels/attention.rs:190-207). */
SNB_API int snb_softmax_backward(void* stream, const float* probabilities, float* grad, uint64_t rows, uint64_t cols);

/* snb_causal_softmax that also writes the probabilities as bf16 into probabilities_bf16 ([rows, keys], may be
 * NULL), the operand of bf16 tensor-core P*V and P^T*dO products. No reference counterpart (the reference keeps
 * f32 only). */
SNB_API int snb_causal_softmax_bf16(void* stream, float* scores, uint64_t scores_len, uint64_t rows, uint64_t queries,
                                    uint64_t keys, float scale, uint64_t query_offset, uint16_t* probabilities_bf16);

/* softmax_backward for causal probabilities: row r (query q = r % queries) reads only its visible keys
 * 0..=q+query_offset, where p can be non-zero, and writes grad = p * (grad - sum) there and 0 after; masked grad
 * entries are never read (a SKIP_MASKED_OUTPUT dO*V^T leaves them unwritten). Equal to snb_softmax_backward
 * wherever the latter's inputs are finite. Optionally also writes grad as bf16 (grad_bf16, may be NULL). */
SNB_API int snb_causal_softmax_backward(void* stream, const float* probabilities, float* grad, uint64_t rows,
                                        uint64_t queries, uint64_t cols, uint64_t query_offset, uint16_t* grad_bf16);

/* Packed columns -> head-major tensor (f32): replaces `Gpu::split_heads` (crates/staleynet-cuda/src/ops/attention.rs:
 * 20-36; kernel kernels/attention.rs:112-121). Element (b, h, s, d) moves from packed[(b * time + s) * width +
 * column_offset + h * head_dim + d] to head_major[((b * heads + h) * time_capacity + time_offset + s) * head_dim + d].
 * The reference's checks (`check_layout`, ops/attention.rs:11-18) in its order and words, each returning
 * SNB_ERR_INVALID_ARGUMENT: "HeadLayout: time range exceeds capacity" (time_offset + time > time_capacity),
 * "HeadLayout: packed tensor too small" (packed_len < batch * time * width), "HeadLayout: head-major tensor too
 * small" (head_major_len < batch * heads * time_capacity * head_dim). Also refused: a head that does not fit in the
 * packed row (column_offset + heads * head_dim > width). */
SNB_API int snb_split_heads(void* stream, const float* packed, uint64_t packed_len, float* head_major,
                            uint64_t head_major_len, const snb_head_layout* layout);

/* Head-major tensor -> packed columns (f32), other columns untouched: replaces `Gpu::merge_heads`
 * (ops/attention.rs:38-52; kernel kernels/attention.rs:129-138). The same checks as snb_split_heads, in the same
 * order (the reference runs one check_layout for both directions). */
SNB_API int snb_merge_heads(void* stream, const float* head_major, uint64_t head_major_len, float* packed,
                            uint64_t packed_len, const snb_head_layout* layout);

/* Directions of snb_permute_heads. */
enum {
    SNB_HEADS_SPLIT = 0, /* packed -> head-major */
    SNB_HEADS_MERGE = 1  /* head-major -> packed */
};

/* snb_split_heads / snb_merge_heads with element types of their own: src_type and dst_type SNB_TYPE_F32 or
 * SNB_TYPE_BF16 (f32 -> bf16 rounds to nearest even). E.g. the f32 query/key/value gradients of
 * snb_causal_attention_backward merged into the bf16 packed gradient of the QKV projection. Same checks as the two
 * drop-ins. No reference counterpart. */
SNB_API int snb_permute_heads(void* stream, int32_t direction, const void* src, int32_t src_type, uint64_t src_len,
                              void* dst, int32_t dst_type, uint64_t dst_len, const snb_head_layout* layout);

/* Message of the last failed call on the calling thread ("" if none). Valid until the next call. */
SNB_API const char* snb_last_error(void);

/* Kernel family used by the last successful snb_matmul/snb_matmul_bf16/snb_gemm call on this thread. */
SNB_API int snb_last_path(void);

/* Reads and clears the device-side status word of the current device: 0 if every bounded wait since the last
 * read completed, else SNB_ERR_DEVICE_TIMEOUT. Synchronizes the device. */
SNB_API int snb_device_status(void);

/* Causal attention forward in one tcgen05 kernel, without materialising the scores:
 *   out[b, q, :] = sum over keys k <= q + query_offset (k < keys) of softmax_k(scale * Q[b,q].K[b,k]) V[b,k,:]
 * — the reference's QK^T product, causal_softmax and P.V product (layers/attention.rs:206-213) composed — and
 * lse[b, q] = log sum_k exp(scale * Q[b,q].K[b,k]) over the same keys (may be NULL), from which a backward pass can
 * rebuild the probabilities. q is [count, queries, 64], k and v are [count, keys, 64], all bf16 (16-byte aligned);
 * out is [count, queries, 64] of out_type (SNB_TYPE_F32 or SNB_TYPE_BF16). head_dim must be 64 and scale positive
 * and finite (SNB_ERR_INVALID_ARGUMENT otherwise). Probabilities are
 * rounded to bf16 for the P.V product (as the bf16 attention products do). No reference counterpart: the reference
 * always materialises the [queries, keys] scores. */
SNB_API int snb_causal_attention_forward(void* stream, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                         uint64_t count, uint64_t queries, uint64_t keys, uint64_t head_dim,
                                         float scale, uint64_t query_offset, void* out, int32_t out_type, float* lse);

/* Causal attention backward in tcgen05 kernels, without materialising the [queries, keys] probabilities or their
 * gradients: given the forward's q, k, v, out (= snb_causal_attention_forward's output, out_type f32 or bf16) and
 * lse, and the output gradient d_out (bf16, [count, queries, 64]), writes
 *   dq = scale dS K, dk = scale dS^T Q, dv = P^T dO,  dS = P * (dO V^T - rowsum(dO * out)),
 * P the causal softmax probabilities rebuilt from lse — the reference's backward (layers/attention.rs:220-267,
 * kernels/attention.rs:182-207) with rowsum(P * dP) taken as rowsum(dO * out). dq is [count, queries, 64], dk and dv
 * [count, keys, 64], all f32 and overwritten. P and dS are rounded to bf16 for the products (as the bf16 attention
 * products do). Uses a stream-ordered scratch buffer of count * queries * 8 bytes (cudaMallocAsync / cudaFreeAsync
 * on `stream`). No reference counterpart: the reference materialises P and dS. */
SNB_API int snb_causal_attention_backward(void* stream, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                          const void* out, int32_t out_type, const uint16_t* d_out, const float* lse,
                                          uint64_t count, uint64_t queries, uint64_t keys, uint64_t head_dim,
                                          float scale, uint64_t query_offset, float* dq, float* dk, float* dv);

/* snb_causal_attention_backward without any allocation: the same arguments, kernels and results, but the
 * row-statistics scratch is a fixed 8 MiB __device__ array of the library (its address looked up once per device)
 * instead of a stream-ordered allocation, and nothing else is allocated. Returns SNB_ERR_INVALID_ARGUMENT, before
 * touching any buffer, when count * queries * 8 bytes (rounded up per matrix) exceed that array. The array is shared
 * by every call on a device: calls that overlap in time (on different streams or threads) race on it and must be
 * serialised by the caller. No reference counterpart. */
SNB_API int snb_causal_attention_backward_noalloc(void* stream, const uint16_t* q, const uint16_t* k,
                                                  const uint16_t* v, const void* out, int32_t out_type,
                                                  const uint16_t* d_out, const float* lse, uint64_t count,
                                                  uint64_t queries, uint64_t keys, uint64_t head_dim, float scale,
                                                  uint64_t query_offset, float* dq, float* dk, float* dv);

/* One classifier head of the output layer, laid out like the reference's `CrossEntropyHead` (ops/loss.rs:14-30):
 * the head owns logit columns column_offset .. column_offset + classes of every row and reads its target at
 * target_offset within each row of target_stride targets; grad_scale multiplies its gradient. */
typedef struct snb_cross_entropy_head {
    uint64_t column_offset;
    uint64_t classes;
    uint64_t target_stride;
    uint64_t target_offset;
    float grad_scale;
    uint32_t reserved; /* 0 */
} snb_cross_entropy_head;

/* Softmax cross-entropy of one head with its gradient. Replaces `Gpu::cross_entropy` (ops/loss.rs:35-71; kernel
 * kernels/loss.rs:54-94): for each of `rows` rows of logits [rows, cols] (f32), losses[row] = logsumexp(z) - z[target]
 * and the head's columns of logits_grad [rows, cols] (f32) = (softmax(z) - onehot(target)) * grad_scale; a target of
 * 0xFFFFFFFF (EMPTY_TOKEN) gives loss 0 and a zero gradient; other columns of logits_grad are left untouched. The
 * reference's three checks are status codes in its order and words: "head exceeds logits"
 * (column_offset + classes > cols), "losses too small" (losses_len < rows), "too few targets"
 * (targets_len < rows * target_stride, or the last target beyond targets_len). A target >= classes (which the
 * reference would read outside the row) gives a NaN loss and gradient instead of a fault. */
SNB_API int snb_cross_entropy(void* stream, const float* logits, uint64_t rows, uint64_t cols,
                              const uint32_t* targets, uint64_t targets_len, const snb_cross_entropy_head* head,
                              float* losses, uint64_t losses_len, float* logits_grad);

/* The output layer's forward and loss in two launches: `head` (a snb_gemm, count 1, writing logits [rows, codebooks *
 * codebook_size] row-major to head->output as f32 or bf16, bias included) then the cross-entropy of every codebook
 * head c (columns c * codebook_size .., target c of each row of `codebooks` targets, gradient scale grad_scales[c],
 * a device array) in one launch. loss_sums[c] (device, [codebooks]) receives the sum of head c's row losses (it is
 * zeroed first), so one small copy replaces the reference's per-codebook loss downloads (training.rs:209-235).
 * logits_grad ([rows, codebooks * codebook_size] of grad_type) may be head->output itself when grad_type equals
 * head->output_type: the gradient then overwrites the logits in place, each logit read once. No f32 logits need
 * exist. No reference counterpart as one call: it replaces Linear::forward of the head plus `codebook_losses`. */
SNB_API int snb_head_cross_entropy(void* stream, const snb_gemm_args* head, const uint32_t* targets,
                                   uint64_t targets_len, uint64_t codebooks, uint64_t codebook_size,
                                   const float* grad_scales, float* loss_sums, void* logits_grad, int32_t grad_type);

/* The loss half of snb_head_cross_entropy on logits a caller has already computed: every codebook's softmax
 * cross-entropy of logits [rows, codebooks * codebook_size] (logits_type SNB_TYPE_F32 or SNB_TYPE_BF16) in one
 * launch, with the same targets, grad_scales, loss_sums (zeroed first) and logits_grad (may be logits itself when
 * grad_type equals logits_type) as snb_head_cross_entropy. Replaces the reference's `codebook_losses` loop of one
 * `Gpu::cross_entropy` and one host download per codebook (crates/staleynet-model/src/training.rs:209-235). */
SNB_API int snb_codebook_cross_entropy(void* stream, const void* logits, int32_t logits_type, uint64_t rows,
                                       uint64_t codebooks, uint64_t codebook_size, const uint32_t* targets,
                                       uint64_t targets_len, const float* grad_scales, float* loss_sums,
                                       void* logits_grad, int32_t grad_type);

/* ---------------------------------------------------------------------------------------------- RMSNorm, AdamW */

/* RMSNorm forward (`Gpu::rms_norm_forward`, ops/normalization.rs; kernel kernels/normalization.rs:27-51): for each
 * row of input [rows, cols] (f32), inv_rms[row] = 1/sqrt(mean(x^2) + epsilon) and output = x * inv_rms * gain.
 * The reference's checks as status codes: "gain length" (gain_len != cols), "inv_rms too small". */
SNB_API int snb_rms_norm_forward(void* stream, const float* input, uint64_t rows, uint64_t cols, const float* gain,
                                 uint64_t gain_len, float* output, float* inv_rms, uint64_t inv_rms_len, float epsilon);

/* RMSNorm backward (`Gpu::rms_norm_backward`; kernels/normalization.rs:53-127): input_grad = s g dy - x s^3 / cols *
 * sum(dy g x) per row, and gain_grad[c] += sum over rows of dy x s ("gain_grad length" if gain_grad_len != cols). */
SNB_API int snb_rms_norm_backward(void* stream, const float* output_grad, const float* input, const float* gain,
                                  const float* inv_rms, float* input_grad, float* gain_grad, uint64_t gain_grad_len,
                                  uint64_t rows, uint64_t cols);

/* The RMSNorm statistics of the fused prologue: inv_rms[row] of input [rows, cols] (input_type f32 or bf16) and,
 * when output is not NULL, the normalised rows x * inv_rms * gain as output_type. With output NULL, the GEMM
 * left * (gain-scaled right, snb_scale_rows) with row_scale = inv_rms computes rms_norm(left) * right without the
 * normalised tensor. No reference counterpart. */
SNB_API int snb_rms_norm_stats(void* stream, const void* input, int32_t input_type, uint64_t rows, uint64_t cols,
                               float epsilon, float* inv_rms, const float* gain, void* output, int32_t output_type);

/* output[k, :] = scale[k] * input[k, :] for row-major [rows, cols] (types f32 or bf16; may be in place when the
 * types match): folds an RMSNorm gain into the weight matrix that follows it. No reference counterpart. */
SNB_API int snb_scale_rows(void* stream, const float* scale, const void* input, int32_t input_type, void* output,
                           int32_t output_type, uint64_t rows, uint64_t cols);

/* AdamWHyperparameters (ops/optimizer.rs:9-28). */
typedef struct snb_adamw_hyper {
    float learning_rate;
    float beta1;
    float beta2;
    float epsilon;
    float weight_decay; /* snb_adamw_step only; snb_adamw_step_multi takes it per tensor */
    uint32_t step;      /* 1-based, for the bias corrections 1 - beta^step */
} snb_adamw_hyper;

/* One parameter tensor of snb_adamw_step_multi (48 bytes). */
typedef struct snb_adamw_tensor {
    float* parameter;
    const float* gradient;
    float* first_moment;
    float* second_moment;
    uint64_t count;
    float weight_decay; /* 0 for gains, biases and embeddings (the reference's Decay::Exempt) */
    uint32_t reserved;
} snb_adamw_tensor;

/* One AdamW step of one tensor (`Gpu::adamw_step`, ops/optimizer.rs:32-66; kernel kernels/optimizer.rs:47-71). */
SNB_API int snb_adamw_step(void* stream, float* parameter, const float* gradient, float* first_moment,
                           float* second_moment, uint64_t count, const snb_adamw_hyper* hyper);

/* *result (device, one double) = sum of values[i]^2 (`Gpu::sum_of_squares`, ops/optimizer.rs:68-85, which reduces
 * the block sums on the host instead). */
SNB_API int snb_sum_of_squares(void* stream, const float* values, uint64_t count, double* result);

/* The optimizer step of `AdamW::step` (model optimizer.rs:125-177) over up to 256 tensors in two launches and no
 * host round trip: *gradient_square_sum (device double) = the sum of every gradient's squares; the clip factor
 * max_gradient_norm / norm (when the norm exceeds it) and the AdamW update of every tensor follow on the device.
 * Unlike the reference, the gradients themselves are left unscaled. No reference counterpart as one call. */
SNB_API int snb_adamw_step_multi(void* stream, const snb_adamw_tensor* tensors, uint64_t tensor_count,
                                 const snb_adamw_hyper* hyper, float max_gradient_norm, double* gradient_square_sum);

/* Seeded inputs on the device, the reference's generator (`Random`, crates/staleynet-model/src/random.rs:27-70):
 * SplitMix64 whose k-th draw (k = 1, 2, ...) from Random::new(seed) is its output for state seed + k * 0x9E3779B97F4A7C15.
 * output[i] = std * normal() computed from draws first_draw + 2i + 1 and + 2 (random.rs:64-68, two draws per value),
 * i.e. what `Init::Normal(std)` (parameter.rs:54) writes from a Random that has already made first_draw draws; a
 * following fill continues at first_draw + 2 * count. output_type SNB_TYPE_F32, or SNB_TYPE_BF16 (the f32 value
 * rounded to nearest even). The device's logf / cosf may differ from the host libm's in an f32's last bit. No
 * reference counterpart as a device call. */
SNB_API int snb_random_normal(void* stream, void* output, int32_t output_type, uint64_t count, uint64_t seed,
                              uint64_t first_draw, float std);

/* output[i] = `Random::below(bound)` (random.rs:54-56) from draw first_draw + i + 1 (one draw per value). */
SNB_API int snb_random_below(void* stream, uint32_t* output, uint64_t count, uint64_t seed, uint64_t first_draw,
                             uint64_t bound);

/* Failure-detection self-test: launches a one-thread kernel that waits on an mbarrier nothing completes, through
 * the bounded wait every tensor-core pipeline wait uses. The wait gives up after limit_ns (at most 1 s), records a
 * timeout in the device status word and the kernel returns normally; a following snb_device_status() reports
 * SNB_ERR_DEVICE_TIMEOUT and the context stays usable. No reference counterpart (the reference's kernels have no
 * bounded waits). */
SNB_API int snb_selftest_bounded_wait(void* stream, uint64_t limit_ns);

/* Version of this ABI (major*100 + minor). */
SNB_API int snb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SNB_MATMUL_H */
