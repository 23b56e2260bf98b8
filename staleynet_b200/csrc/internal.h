// internal.h — declarations shared by the library's translation units (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <string>

#include "snb_matmul.h"

namespace snb {

// One product with its epilogue, after argument validation; element types are SNB_TYPE_*.
struct GemmRequest {
    snb_product p;
    uint64_t count;
    int a_type, b_type, c_type;
    int precision;
    const void* A;
    const void* B;
    void* C;
    const float* bias;
    int activation;
    int aux_type;
    void* pre;
    const void* gelu_input;
    const void* residual;
    int causal;
    int64_t causal_offset;
    const float* row_scale;   // [rows] output-row multipliers (count 1), or nullptr
    bool deterministic;       // split-K partials summed in a fixed order (SNB_GEMM_DETERMINISTIC)
    const snb_head_layout* a_heads;  // left operand read from its head-major form, or nullptr (snb_gemm_args)
    const snb_head_layout* c_heads;  // output written head-major, or nullptr
    int sm_budget;            // SMs the persistent grid may occupy (0: all; snb_set_sm_budget)
};

struct DeviceInfo {
    int device;
    int sm_count;
    int major, minor;
};

// Properties of the current device (cached per device).
int current_device_info(DeviceInfo* info, std::string* err);

// Runs the product on a tcgen05 kernel if its layout allows TMA (unit strides, 16-byte alignment); *launched
// says whether it did and *path which kernel (SNB_PATH_TENSOR_CORE or SNB_PATH_TENSOR_CORE_PAIR). Returns SNB_OK
// or an error code (with *err set).
int tc_gemm_try(cudaStream_t stream, const GemmRequest& r, bool* launched, int* path, std::string* err);

// Runs the product on the strided SIMT kernel (any layout).
int simt_gemm(cudaStream_t stream, const GemmRequest& r, std::string* err);

int causal_softmax(cudaStream_t stream, float* scores, uint64_t rows, uint64_t queries, uint64_t keys, float scale,
                   uint64_t query_offset, uint16_t* probs_bf16, std::string* err);
int softmax_backward(cudaStream_t stream, const float* probabilities, float* grad, uint64_t rows, uint64_t cols,
                     std::string* err);
int causal_softmax_backward(cudaStream_t stream, const float* probabilities, float* grad, uint64_t rows,
                            uint64_t queries, uint64_t cols, uint64_t query_offset, uint16_t* grad_bf16,
                            std::string* err);

// Fused causal attention forward (tcgen05; head_dim 64; bf16 q/k/v [count, rows, 64]).
int fused_attention_forward(cudaStream_t stream, const void* q, const void* k, const void* v, uint64_t count,
                            uint64_t queries, uint64_t keys, float scale, uint64_t query_offset, void* out,
                            int out_type, float* lse, std::string* err);
// Softmax cross-entropy with its gradient over `heads` classifiers side by side (cross_entropy.cu): head h owns
// columns column_offset + h * classes .. and target target_offset + h of each target row. row_losses
// ([rows * heads], head fastest) and loss_sums ([heads], added to) may be null; grad may alias logits when the
// element types match.
int cross_entropy_launch(cudaStream_t stream, const void* logits, int logits_type, uint64_t rows, uint64_t row_width,
                         const uint32_t* targets, uint64_t target_stride, uint64_t heads, uint64_t column_offset,
                         uint64_t classes, uint64_t target_offset, const float* grad_scales, float grad_scale,
                         float* row_losses, float* loss_sums, void* grad, int grad_type, std::string* err);

// RMSNorm and optimizer launches (norm_optim.cu).
int rms_norm_forward_launch(cudaStream_t s, const void* input, int input_type, const float* gain, void* output,
                            int output_type, float* inv_rms, uint64_t rows, uint64_t cols, float epsilon,
                            std::string* err);
int rms_norm_backward_launch(cudaStream_t s, const float* dy, const float* x, const float* gain, const float* inv_rms,
                             float* dx, float* gain_grad, uint64_t rows, uint64_t cols, std::string* err);
int scale_rows_launch(cudaStream_t s, const float* scale, const void* in, int in_type, void* out, int out_type,
                      uint64_t rows, uint64_t cols, std::string* err);
int adamw_launch(cudaStream_t s, float* parameter, const float* gradient, float* first, float* second, uint64_t count,
                 const snb_adamw_hyper& h, std::string* err);
int sum_of_squares_launch(cudaStream_t s, const float* values, uint64_t count, double* total, std::string* err);
int adamw_multi_launch(cudaStream_t s, const snb_adamw_tensor* tensors, uint64_t n, const snb_adamw_hyper& h,
                       float max_gradient_norm, double* square_sum, std::string* err);

// Fused causal attention backward (attention_fused_bwd.cuh): dq [count, queries, 64], dk and dv [count, keys, 64],
// all f32 and overwritten, from bf16 q, k, v, d_out, the forward's output (f32 or bf16) and its log-sum-exp. The
// row-statistics scratch comes from cudaMallocAsync on `stream`, or with static_scratch_only from a fixed
// __device__ array (no allocation; SNB_ERR_INVALID_ARGUMENT when it is too small; concurrent calls share it).
int fused_attention_backward(cudaStream_t stream, const void* q, const void* k, const void* v, const void* out,
                             int out_type, const void* d_out, const float* lse, uint64_t count, uint64_t queries,
                             uint64_t keys, float scale, uint64_t query_offset, float* dq, float* dk, float* dv,
                             bool static_scratch_only, std::string* err);

// The attention head permutes (heads.cu): split = packed -> head-major, else head-major -> packed; element types
// SNB_TYPE_*; the layout is checked by the caller.
int permute_heads_launch(cudaStream_t stream, bool split, const void* src, int src_type, void* dst, int dst_type,
                         const snb_head_layout& layout, std::string* err);

// Launches a one-thread kernel whose mbarrier wait nothing completes; it gives up after limit_ns.
int bounded_wait_probe(cudaStream_t stream, uint64_t limit_ns, std::string* err);

// Reads and clears the tensor-core kernels' device status word on the current device (synchronizes first).
int read_and_clear_device_status(unsigned int* status, std::string* err);

std::string cuda_message(const char* what, cudaError_t e);

// The reference's seeded stream on the device (random.cu): normal values (f32 or bf16 output) and below(bound)
// integers from draw first_draw + 1 on.
int random_normal_launch(cudaStream_t s, void* out, int out_type, uint64_t count, uint64_t seed, uint64_t first_draw,
                         float stddev, std::string* err);
int random_below_launch(cudaStream_t s, uint32_t* out, uint64_t count, uint64_t seed, uint64_t first_draw,
                        uint64_t bound, std::string* err);

}  // namespace snb
