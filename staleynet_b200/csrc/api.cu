// api.cu — the extern "C" entry points of include/snb_matmul.h: argument checks in the reference's order
// (crates/staleynet-cuda/src/ops/matmul.rs:146-149), choice of kernel family, and per-thread error reporting.
#include <cuda_runtime.h>

#include <mutex>
#include <cmath>
#include <string>
#include <vector>

#include "internal.h"

namespace snb {

namespace {

thread_local std::string t_last_error;
thread_local int t_last_path = SNB_PATH_NONE;
thread_local bool t_deterministic = false;   // snb_set_deterministic
thread_local int t_sm_budget = 0;            // snb_set_sm_budget

int fail(int code, const std::string& message) {
    t_last_error = message;
    return code;
}

// Elements an operand must hold: the largest index the batch addresses, plus one. For the reference's
// RowMajor/Transposed layouts this is `MatmulSpec::required_len` (ops/matmul.rs:138-141):
// (count-1)*batch_stride + rows*cols.
uint64_t required_len(uint64_t count, uint64_t batch_stride, uint64_t rows, uint64_t cols, uint64_t row_stride,
                      uint64_t col_stride) {
    if (rows == 0 || cols == 0) return 0;
    return (count - 1) * batch_stride + (rows - 1) * row_stride + (cols - 1) * col_stride + 1;
}

int run(cudaStream_t stream, const GemmRequest& r, uint64_t left_len, uint64_t right_len, uint64_t output_len) {
    const snb_product& p = r.p;
    if (r.count == 0) return fail(SNB_ERR_INVALID_ARGUMENT, "matmul: batch count must be at least 1");
    if (left_len < required_len(r.count, p.left.batch_stride, p.rows, p.inner, p.left.row_stride, p.left.col_stride))
        return fail(SNB_ERR_LEFT_TOO_SMALL, "matmul: left operand too small");
    if (right_len <
        required_len(r.count, p.right.batch_stride, p.inner, p.cols, p.right.row_stride, p.right.col_stride))
        return fail(SNB_ERR_RIGHT_TOO_SMALL, "matmul: right operand too small");
    if (output_len < required_len(r.count, p.output_batch_stride, p.rows, p.cols, p.cols, 1))
        return fail(SNB_ERR_OUTPUT_TOO_SMALL, "matmul: output too small");
    if (p.rows == 0 || p.cols == 0) {
        t_last_path = SNB_PATH_EMPTY;
        return SNB_OK;
    }
    if (r.C == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "matmul: output pointer is null");
    if (p.inner > 0 && (r.A == nullptr || r.B == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "matmul: operand pointer is null");
    if (r.activation == SNB_ACTIVATION_GELU_GRAD && r.gelu_input == nullptr)
        return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: GELU_GRAD needs gelu_input");
    if (r.pre != nullptr && r.activation != SNB_ACTIVATION_GELU)
        return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: pre_activation is only written with GELU");
    if (r.c_type == SNB_TYPE_BF16 && p.accumulate)
        return fail(SNB_ERR_UNSUPPORTED, "gemm: accumulating into a bf16 output is not supported");

    std::string err;
    bool launched = false;
    int path = SNB_PATH_NONE;
    int rc = tc_gemm_try(stream, r, &launched, &path, &err);
    if (rc != SNB_OK) return fail(rc, err);
    if (launched) {
        t_last_path = path;
        return SNB_OK;
    }
    if (r.a_heads != nullptr || r.c_heads != nullptr)
        return fail(SNB_ERR_UNSUPPORTED,
                    err.empty() ? "gemm: head-major operands run on the sm_100 tensor-core kernel only (bf16 or tf32 "
                                  "operands with unit-stride, 16-byte aligned layouts)"
                                : "gemm: " + err);
    rc = simt_gemm(stream, r, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

std::mutex g_info_mu;
std::vector<DeviceInfo> g_info;

// a * b, or false when it overflows 64 bits.
bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) { return !__builtin_mul_overflow(a, b, out); }

// Elements of a head-major tensor [batch, heads, time_capacity, head_dim], or false on overflow.
bool head_major_elements(const snb_head_layout& L, uint64_t* n) {
    uint64_t t = 0;
    return mul_ok(L.batch, L.heads, &t) && mul_ok(t, L.time_capacity, &t) && mul_ok(t, L.head_dim, n);
}

// The reference's check_layout (crates/staleynet-cuda/src/ops/attention.rs:11-18), in its order and words, plus the
// packed row holding the heads; empty string when the layout is usable.
std::string check_head_layout(const snb_head_layout& L, uint64_t packed_len, uint64_t head_major_len) {
    if (L.time_offset > L.time_capacity || L.time > L.time_capacity - L.time_offset)
        return "HeadLayout: time range exceeds capacity";
    uint64_t packed = 0, head_major = 0, span = 0;
    if (!mul_ok(L.batch, L.time, &packed) || !mul_ok(packed, L.width, &packed) || packed_len < packed)
        return "HeadLayout: packed tensor too small";
    if (!head_major_elements(L, &head_major) || head_major_len < head_major)
        return "HeadLayout: head-major tensor too small";
    if (!mul_ok(L.heads, L.head_dim, &span) || L.column_offset > L.width || span > L.width - L.column_offset)
        return "HeadLayout: heads exceed the packed row";
    return "";
}

}  // namespace

std::string cuda_message(const char* what, cudaError_t e) {
    return std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
}

int current_device_info(DeviceInfo* info, std::string* err) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *err = cuda_message("cudaGetDevice", e);
        return SNB_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_info_mu);
    for (const DeviceInfo& d : g_info) {
        if (d.device == dev) {
            *info = d;
            return SNB_OK;
        }
    }
    DeviceInfo d{dev, 0, 0, 0};
    if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) {
        *err = cuda_message("cudaDeviceGetAttribute", e);
        return SNB_ERR_CUDA;
    }
    g_info.push_back(d);
    *info = d;
    return SNB_OK;
}

}  // namespace snb

using namespace snb;

extern "C" {

int snb_abi_version(void) { return 106; }

const char* snb_last_error(void) { return t_last_error.c_str(); }

int snb_last_path(void) { return t_last_path; }

int snb_matmul(void* stream, const snb_product* product, uint64_t count, const float* left, uint64_t left_len,
               const float* right, uint64_t right_len, float* output, uint64_t output_len, int32_t precision) {
    t_last_path = SNB_PATH_NONE;
    if (product == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "matmul: product is null");
    if (precision != SNB_PRECISION_F32 && precision != SNB_PRECISION_TF32)
        return fail(SNB_ERR_INVALID_ARGUMENT,
                    "matmul: precision must be SNB_PRECISION_F32 or SNB_PRECISION_TF32 for f32 operands");
    GemmRequest r{};
    r.p = *product;
    r.count = count;
    r.a_type = r.b_type = r.c_type = SNB_TYPE_F32;
    r.precision = precision;
    r.A = left;
    r.B = right;
    r.C = output;
    r.aux_type = SNB_TYPE_F32;
    r.deterministic = t_deterministic;
    r.sm_budget = t_sm_budget;
    return run(static_cast<cudaStream_t>(stream), r, left_len, right_len, output_len);
}

int snb_matmul_bf16(void* stream, const snb_product* product, uint64_t count, const uint16_t* left,
                    uint64_t left_len, const uint16_t* right, uint64_t right_len, float* output, uint64_t output_len) {
    t_last_path = SNB_PATH_NONE;
    if (product == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "matmul: product is null");
    GemmRequest r{};
    r.p = *product;
    r.count = count;
    r.a_type = r.b_type = SNB_TYPE_BF16;
    r.c_type = SNB_TYPE_F32;
    r.precision = SNB_PRECISION_BF16;
    r.A = left;
    r.B = right;
    r.C = output;
    r.aux_type = SNB_TYPE_F32;
    r.deterministic = t_deterministic;
    r.sm_budget = t_sm_budget;
    return run(static_cast<cudaStream_t>(stream), r, left_len, right_len, output_len);
}

int snb_set_sm_budget(int32_t sms) {
    const int previous = t_sm_budget;
    t_sm_budget = sms > 0 ? sms : 0;
    return previous;
}

int snb_set_deterministic(int32_t enabled) {
    const int previous = t_deterministic ? 1 : 0;
    t_deterministic = enabled != 0;
    return previous;
}

int snb_gemm(void* stream, const snb_gemm_args* a) {
    t_last_path = SNB_PATH_NONE;
    if (a == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: args is null");
    const bool types_ok = (a->left_type == SNB_TYPE_F32 || a->left_type == SNB_TYPE_BF16) &&
                          a->right_type == a->left_type &&
                          (a->output_type == SNB_TYPE_F32 || a->output_type == SNB_TYPE_BF16) &&
                          (a->aux_type == SNB_TYPE_F32 || a->aux_type == SNB_TYPE_BF16);
    if (!types_ok) return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: unknown or mismatched element types");
    const bool prec_ok = a->left_type == SNB_TYPE_BF16
                             ? a->precision == SNB_PRECISION_BF16
                             : (a->precision == SNB_PRECISION_F32 || a->precision == SNB_PRECISION_TF32);
    if (!prec_ok) return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: precision does not match the operand type");
    if (a->activation < SNB_ACTIVATION_NONE || a->activation > SNB_ACTIVATION_GELU_GRAD)
        return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: unknown activation");
    if (a->causal < SNB_CAUSAL_NONE || a->causal > SNB_CAUSAL_LEFT_T_MASKED || a->causal_offset < 0)
        return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: unknown causal mode or negative offset");
    if (a->row_scale != nullptr && a->count != 1)
        return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: row_scale needs count 1");
    if ((a->flags & ~SNB_GEMM_DETERMINISTIC) != 0) return fail(SNB_ERR_INVALID_ARGUMENT, "gemm: unknown flags");
    const snb_product& gp = a->product;
    if (a->left_heads != nullptr) {
        const snb_head_layout& L = *a->left_heads;
        uint64_t tokens = 0, n = 0;
        const bool geometry = L.column_offset == 0 && L.heads > 0 && L.head_dim > 0 &&
                              L.width == L.heads * L.head_dim && L.time_offset <= L.time_capacity &&
                              L.time <= L.time_capacity - L.time_offset && mul_ok(L.batch, L.time, &tokens);
        const bool row_major = gp.left.row_stride == L.width && gp.left.col_stride == 1 && gp.rows == tokens &&
                               gp.inner == L.width;
        const bool transposed = gp.left.row_stride == 1 && gp.left.col_stride == L.width && gp.rows == L.width &&
                                gp.inner == tokens;
        if (a->count != 1 || !geometry || !(row_major || transposed))
            return fail(SNB_ERR_INVALID_ARGUMENT,
                        "gemm: left_heads must describe the packed left operand [batch * time, heads * head_dim] "
                        "(RowMajor or Transposed, column_offset 0, count 1)");
        if (!head_major_elements(L, &n) || a->left_len < n)
            return fail(SNB_ERR_LEFT_TOO_SMALL, "matmul: left operand too small");
    }
    if (a->output_heads != nullptr) {
        const snb_head_layout& L = *a->output_heads;
        uint64_t tokens = 0, n = 0, span = 0;
        const bool geometry = L.column_offset == 0 && L.heads > 0 && L.head_dim > 0 && L.width == gp.cols &&
                              mul_ok(L.heads, L.head_dim, &span) && gp.cols % span == 0 &&
                              L.time_offset <= L.time_capacity && L.time <= L.time_capacity - L.time_offset &&
                              mul_ok(L.batch, L.time, &tokens) && gp.rows == tokens;
        if (a->count != 1 || !geometry)
            return fail(SNB_ERR_INVALID_ARGUMENT,
                        "gemm: output_heads must describe the output [batch * time, P * heads * head_dim] "
                        "(width = cols, column_offset 0, count 1)");
        if (!head_major_elements(L, &n) || !mul_ok(n, gp.cols / span, &n) || a->output_len < n)
            return fail(SNB_ERR_OUTPUT_TOO_SMALL, "matmul: output too small");
    }
    GemmRequest r{};
    r.p = a->product;
    r.count = a->count;
    r.a_type = a->left_type;
    r.b_type = a->right_type;
    r.c_type = a->output_type;
    r.precision = a->precision;
    r.A = a->left;
    r.B = a->right;
    r.C = a->output;
    r.bias = a->bias;
    r.activation = a->activation;
    r.aux_type = a->aux_type;
    r.pre = a->pre_activation;
    r.gelu_input = a->gelu_input;
    r.residual = a->residual;
    r.causal = a->causal;
    r.causal_offset = a->causal_offset;
    r.row_scale = a->row_scale;
    r.deterministic = t_deterministic || (a->flags & SNB_GEMM_DETERMINISTIC) != 0;
    r.a_heads = a->left_heads;
    r.c_heads = a->output_heads;
    r.sm_budget = t_sm_budget;
    return run(static_cast<cudaStream_t>(stream), r, a->left_len, a->right_len, a->output_len);
}

namespace {

int permute_heads_entry(const char* name, void* stream, bool split, const void* src, int32_t src_type,
                        uint64_t src_len, void* dst, int32_t dst_type, uint64_t dst_len, const snb_head_layout* layout) {
    t_last_path = SNB_PATH_NONE;
    if (layout == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": layout is null");
    if ((src_type != SNB_TYPE_F32 && src_type != SNB_TYPE_BF16) || (dst_type != SNB_TYPE_F32 && dst_type != SNB_TYPE_BF16))
        return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": unknown element type");
    const uint64_t packed_len = split ? src_len : dst_len;
    const uint64_t head_major_len = split ? dst_len : src_len;
    const std::string bad = check_head_layout(*layout, packed_len, head_major_len);
    if (!bad.empty()) return fail(SNB_ERR_INVALID_ARGUMENT, bad);
    const snb_head_layout& L = *layout;
    if (L.batch == 0 || L.time == 0 || L.heads == 0 || L.head_dim == 0) {
        t_last_path = SNB_PATH_EMPTY;
        return SNB_OK;
    }
    if (src == nullptr || dst == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
    std::string err;
    const int rc = permute_heads_launch(static_cast<cudaStream_t>(stream), split, src, src_type, dst, dst_type, L, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

}  // namespace

int snb_split_heads(void* stream, const float* packed, uint64_t packed_len, float* head_major, uint64_t head_major_len,
                    const snb_head_layout* layout) {
    return permute_heads_entry("split_heads", stream, true, packed, SNB_TYPE_F32, packed_len, head_major, SNB_TYPE_F32,
                               head_major_len, layout);
}

int snb_merge_heads(void* stream, const float* head_major, uint64_t head_major_len, float* packed, uint64_t packed_len,
                    const snb_head_layout* layout) {
    return permute_heads_entry("merge_heads", stream, false, head_major, SNB_TYPE_F32, head_major_len, packed,
                               SNB_TYPE_F32, packed_len, layout);
}

int snb_permute_heads(void* stream, int32_t direction, const void* src, int32_t src_type, uint64_t src_len, void* dst,
                      int32_t dst_type, uint64_t dst_len, const snb_head_layout* layout) {
    if (direction != SNB_HEADS_SPLIT && direction != SNB_HEADS_MERGE)
        return fail(SNB_ERR_INVALID_ARGUMENT, "permute_heads: unknown direction");
    return permute_heads_entry("permute_heads", stream, direction == SNB_HEADS_SPLIT, src, src_type, src_len, dst,
                               dst_type, dst_len, layout);
}

int snb_causal_softmax_bf16(void* stream, float* scores, uint64_t scores_len, uint64_t rows, uint64_t queries,
                            uint64_t keys, float scale, uint64_t query_offset, uint16_t* probabilities_bf16) {
    if (queries == 0 || rows % queries != 0)
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_softmax: rows must be a multiple of queries");
    if (scores_len < rows * keys) return fail(SNB_ERR_OUTPUT_TOO_SMALL, "causal_softmax: scores too small");
    if (rows > 0 && keys > 0 && scores == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "causal_softmax: null scores");
    if (keys == 0) return SNB_OK;
    std::string err;
    int rc = snb::causal_softmax(static_cast<cudaStream_t>(stream), scores, rows, queries, keys, scale, query_offset,
                                 probabilities_bf16, &err);
    return rc == SNB_OK ? rc : fail(rc, err);
}

int snb_causal_softmax(void* stream, float* scores, uint64_t scores_len, uint64_t rows, uint64_t queries,
                       uint64_t keys, float scale, uint64_t query_offset) {
    return snb_causal_softmax_bf16(stream, scores, scores_len, rows, queries, keys, scale, query_offset, nullptr);
}

int snb_causal_softmax_backward(void* stream, const float* probabilities, float* grad, uint64_t rows,
                                uint64_t queries, uint64_t cols, uint64_t query_offset, uint16_t* grad_bf16) {
    if (queries == 0 || rows % queries != 0)
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_softmax_backward: rows must be a multiple of queries");
    if (rows > 0 && cols > 0 && (probabilities == nullptr || grad == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_softmax_backward: null pointer");
    if (cols == 0) return SNB_OK;
    std::string err;
    int rc = snb::causal_softmax_backward(static_cast<cudaStream_t>(stream), probabilities, grad, rows, queries, cols,
                                          query_offset, grad_bf16, &err);
    return rc == SNB_OK ? rc : fail(rc, err);
}

int snb_softmax_backward(void* stream, const float* probabilities, float* grad, uint64_t rows, uint64_t cols) {
    if (rows > 0 && cols > 0 && (probabilities == nullptr || grad == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "softmax_backward: null pointer");
    if (cols == 0) return SNB_OK;
    std::string err;
    int rc = snb::softmax_backward(static_cast<cudaStream_t>(stream), probabilities, grad, rows, cols, &err);
    return rc == SNB_OK ? rc : fail(rc, err);
}

int snb_causal_attention_forward(void* stream, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                 uint64_t count, uint64_t queries, uint64_t keys, uint64_t head_dim, float scale,
                                 uint64_t query_offset, void* out, int32_t out_type, float* lse) {
    t_last_path = SNB_PATH_NONE;
    if (head_dim != 64) return fail(SNB_ERR_UNSUPPORTED, "causal_attention_forward: head_dim must be 64");
    if (out_type != SNB_TYPE_F32 && out_type != SNB_TYPE_BF16)
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_attention_forward: unknown output type");
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_attention_forward: scale must be positive and finite");
    if (count > 0 && queries > 0 && (q == nullptr || k == nullptr || v == nullptr || out == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "causal_attention_forward: null pointer");
    std::string err;
    int rc = fused_attention_forward(static_cast<cudaStream_t>(stream), q, k, v, count, queries, keys, scale,
                                     query_offset, out, out_type, lse, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_TENSOR_CORE;
    return SNB_OK;
}

namespace {

int attention_backward_entry(const char* name, bool static_scratch_only, void* stream, const uint16_t* q,
                             const uint16_t* k, const uint16_t* v, const void* out, int32_t out_type,
                             const uint16_t* d_out, const float* lse, uint64_t count, uint64_t queries, uint64_t keys,
                             uint64_t head_dim, float scale, uint64_t query_offset, float* dq, float* dk, float* dv) {
    t_last_path = SNB_PATH_NONE;
    // (Messages are built on the error paths only: the no-alloc entry allocates nothing when it succeeds.)
    if (head_dim != 64) return fail(SNB_ERR_UNSUPPORTED, std::string(name) + ": head_dim must be 64");
    if (out_type != SNB_TYPE_F32 && out_type != SNB_TYPE_BF16)
        return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": unknown output type");
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": scale must be positive and finite");
    if (count > 0 && ((queries > 0 && (q == nullptr || d_out == nullptr || out == nullptr || lse == nullptr ||
                                       dq == nullptr)) ||
                      (keys > 0 && (k == nullptr || v == nullptr || dk == nullptr || dv == nullptr))))
        return fail(SNB_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
    std::string err;
    int rc = fused_attention_backward(static_cast<cudaStream_t>(stream), q, k, v, out, out_type, d_out, lse, count,
                                      queries, keys, scale, query_offset, dq, dk, dv, static_scratch_only, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_TENSOR_CORE;
    return SNB_OK;
}

}  // namespace

int snb_causal_attention_backward(void* stream, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                  const void* out, int32_t out_type, const uint16_t* d_out, const float* lse,
                                  uint64_t count, uint64_t queries, uint64_t keys, uint64_t head_dim, float scale,
                                  uint64_t query_offset, float* dq, float* dk, float* dv) {
    return attention_backward_entry("causal_attention_backward", false, stream, q, k, v, out, out_type, d_out, lse,
                                    count, queries, keys, head_dim, scale, query_offset, dq, dk, dv);
}

int snb_causal_attention_backward_noalloc(void* stream, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                          const void* out, int32_t out_type, const uint16_t* d_out, const float* lse,
                                          uint64_t count, uint64_t queries, uint64_t keys, uint64_t head_dim,
                                          float scale, uint64_t query_offset, float* dq, float* dk, float* dv) {
    return attention_backward_entry("causal_attention_backward_noalloc", true, stream, q, k, v, out, out_type, d_out,
                                    lse, count, queries, keys, head_dim, scale, query_offset, dq, dk, dv);
}

int snb_cross_entropy(void* stream, const float* logits, uint64_t rows, uint64_t cols, const uint32_t* targets,
                      uint64_t targets_len, const snb_cross_entropy_head* head, float* losses, uint64_t losses_len,
                      float* logits_grad) {
    t_last_path = SNB_PATH_NONE;
    if (head == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "cross_entropy: head is null");
    // The reference's checks (ops/loss.rs:43-47), in its order and words.
    if (head->column_offset > cols || head->classes > cols - head->column_offset)
        return fail(SNB_ERR_INVALID_ARGUMENT, "cross_entropy: head exceeds logits");
    if (losses_len < rows) return fail(SNB_ERR_INVALID_ARGUMENT, "cross_entropy: losses too small");
    if (rows > 0 && (head->target_stride == 0 || targets_len / head->target_stride < rows ||
                     (rows - 1) * head->target_stride + head->target_offset >= targets_len))
        return fail(SNB_ERR_INVALID_ARGUMENT, "cross_entropy: too few targets");
    if (rows == 0 || head->classes == 0) return SNB_OK;
    if (logits == nullptr || targets == nullptr || losses == nullptr || logits_grad == nullptr)
        return fail(SNB_ERR_INVALID_ARGUMENT, "cross_entropy: null pointer");
    std::string err;
    int rc = cross_entropy_launch(static_cast<cudaStream_t>(stream), logits, SNB_TYPE_F32, rows, cols, targets,
                                  head->target_stride, 1, head->column_offset, head->classes, head->target_offset,
                                  nullptr, head->grad_scale, losses, nullptr, logits_grad, SNB_TYPE_F32, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

namespace {

// The loss half of the output layer: every codebook's cross-entropy of logits [rows, codebooks * codebook_size]
// (logits_type) in one launch, loss_sums zeroed first. Arguments are checked by the callers.
int codebook_losses(cudaStream_t s, const void* logits, int32_t logits_type, uint64_t rows, uint64_t codebooks,
                    uint64_t codebook_size, const uint32_t* targets, const float* grad_scales, float* loss_sums,
                    void* logits_grad, int32_t grad_type) {
    cudaError_t e = cudaMemsetAsync(loss_sums, 0, codebooks * sizeof(float), s);
    if (e != cudaSuccess) return fail(SNB_ERR_CUDA, cuda_message("cudaMemsetAsync(loss_sums)", e));
    std::string err;
    const int rc = cross_entropy_launch(s, logits, logits_type, rows, codebooks * codebook_size, targets, codebooks,
                                        codebooks, 0, codebook_size, 0, grad_scales, 0.0f, nullptr, loss_sums,
                                        logits_grad, grad_type, &err);
    if (rc != SNB_OK) return fail(rc, err);
    return SNB_OK;
}

// Checks shared by snb_head_cross_entropy and snb_codebook_cross_entropy (messages prefixed with `name`).
int check_codebook_args(const char* name, uint64_t rows, uint64_t cols, const void* logits, int32_t logits_type,
                        const uint32_t* targets, uint64_t targets_len, uint64_t codebooks, uint64_t codebook_size,
                        const float* grad_scales, const float* loss_sums, const void* logits_grad,
                        int32_t grad_type) {
    const std::string n(name);
    if (codebooks == 0 || codebook_size == 0 || cols / codebooks != codebook_size || cols % codebooks != 0)
        return fail(SNB_ERR_INVALID_ARGUMENT, n + ": logits columns differ from codebooks * codebook_size");
    if (grad_type != SNB_TYPE_F32 && grad_type != SNB_TYPE_BF16)
        return fail(SNB_ERR_INVALID_ARGUMENT, n + ": unknown gradient type");
    if (logits_grad == logits && grad_type != logits_type)
        return fail(SNB_ERR_INVALID_ARGUMENT, n + ": an in-place gradient must have the logits' element type");
    if (rows > 0 && targets_len / codebooks < rows) return fail(SNB_ERR_INVALID_ARGUMENT, n + ": too few targets");
    if (rows > 0 && (targets == nullptr || grad_scales == nullptr || loss_sums == nullptr || logits_grad == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, n + ": null pointer");
    return SNB_OK;
}

}  // namespace

int snb_head_cross_entropy(void* stream, const snb_gemm_args* head, const uint32_t* targets, uint64_t targets_len,
                           uint64_t codebooks, uint64_t codebook_size, const float* grad_scales, float* loss_sums,
                           void* logits_grad, int32_t grad_type) {
    t_last_path = SNB_PATH_NONE;
    if (head == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "head_cross_entropy: head is null");
    const snb_product& p = head->product;
    if (head->count != 1) return fail(SNB_ERR_INVALID_ARGUMENT, "head_cross_entropy: the head GEMM must have count 1");
    int rc = check_codebook_args("head_cross_entropy", p.rows, p.cols, head->output, head->output_type, targets,
                                 targets_len, codebooks, codebook_size, grad_scales, loss_sums, logits_grad, grad_type);
    if (rc != SNB_OK) return rc;
    rc = snb_gemm(stream, head);
    if (rc != SNB_OK) return rc;   // (snb_gemm has set the message)
    const int gemm_path = t_last_path;
    rc = codebook_losses(static_cast<cudaStream_t>(stream), head->output, head->output_type, p.rows, codebooks,
                         codebook_size, targets, grad_scales, loss_sums, logits_grad, grad_type);
    if (rc != SNB_OK) return rc;
    t_last_path = gemm_path;
    return SNB_OK;
}

int snb_codebook_cross_entropy(void* stream, const void* logits, int32_t logits_type, uint64_t rows,
                               uint64_t codebooks, uint64_t codebook_size, const uint32_t* targets,
                               uint64_t targets_len, const float* grad_scales, float* loss_sums, void* logits_grad,
                               int32_t grad_type) {
    t_last_path = SNB_PATH_NONE;
    if (logits_type != SNB_TYPE_F32 && logits_type != SNB_TYPE_BF16)
        return fail(SNB_ERR_INVALID_ARGUMENT, "codebook_cross_entropy: unknown logits type");
    if (rows > 0 && logits == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "codebook_cross_entropy: null pointer");
    int rc = check_codebook_args("codebook_cross_entropy", rows, codebooks * codebook_size, logits, logits_type,
                                 targets, targets_len, codebooks, codebook_size, grad_scales, loss_sums, logits_grad,
                                 grad_type);
    if (rc != SNB_OK) return rc;
    if (rows == 0) {
        if (loss_sums == nullptr) return SNB_OK;
        const cudaError_t e = cudaMemsetAsync(loss_sums, 0, codebooks * sizeof(float), static_cast<cudaStream_t>(stream));
        return e == cudaSuccess ? SNB_OK : fail(SNB_ERR_CUDA, cuda_message("cudaMemsetAsync(loss_sums)", e));
    }
    rc = codebook_losses(static_cast<cudaStream_t>(stream), logits, logits_type, rows, codebooks, codebook_size,
                         targets, grad_scales, loss_sums, logits_grad, grad_type);
    if (rc != SNB_OK) return rc;
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_rms_norm_forward(void* stream, const float* input, uint64_t rows, uint64_t cols, const float* gain,
                         uint64_t gain_len, float* output, float* inv_rms, uint64_t inv_rms_len, float epsilon) {
    t_last_path = SNB_PATH_NONE;
    // The reference's checks (ops/normalization.rs), in its order and words.
    if (gain_len != cols) return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_forward: gain length");
    if (inv_rms_len < rows) return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_forward: inv_rms too small");
    if (rows > 0 && (input == nullptr || gain == nullptr || output == nullptr || inv_rms == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_forward: null pointer");
    std::string err;
    int rc = rms_norm_forward_launch(static_cast<cudaStream_t>(stream), input, SNB_TYPE_F32, gain, output,
                                     SNB_TYPE_F32, inv_rms, rows, cols, epsilon, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_rms_norm_backward(void* stream, const float* output_grad, const float* input, const float* gain,
                          const float* inv_rms, float* input_grad, float* gain_grad, uint64_t gain_grad_len,
                          uint64_t rows, uint64_t cols) {
    t_last_path = SNB_PATH_NONE;
    if (gain_grad_len != cols) return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_backward: gain_grad length");
    if (rows > 0 && (output_grad == nullptr || input == nullptr || gain == nullptr || inv_rms == nullptr ||
                     input_grad == nullptr || gain_grad == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_backward: null pointer");
    std::string err;
    int rc = rms_norm_backward_launch(static_cast<cudaStream_t>(stream), output_grad, input, gain, inv_rms,
                                      input_grad, gain_grad, rows, cols, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_rms_norm_stats(void* stream, const void* input, int32_t input_type, uint64_t rows, uint64_t cols,
                       float epsilon, float* inv_rms, const float* gain, void* output, int32_t output_type) {
    t_last_path = SNB_PATH_NONE;
    const bool types_ok = (input_type == SNB_TYPE_F32 || input_type == SNB_TYPE_BF16) &&
                          (output == nullptr || output_type == SNB_TYPE_F32 || output_type == SNB_TYPE_BF16);
    if (!types_ok) return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_stats: unknown element type");
    if (rows > 0 && (input == nullptr || inv_rms == nullptr || (output != nullptr && gain == nullptr)))
        return fail(SNB_ERR_INVALID_ARGUMENT, "rms_norm_stats: null pointer");
    std::string err;
    int rc = rms_norm_forward_launch(static_cast<cudaStream_t>(stream), input, input_type, gain, output, output_type,
                                     inv_rms, rows, cols, epsilon, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_scale_rows(void* stream, const float* scale, const void* input, int32_t input_type, void* output,
                   int32_t output_type, uint64_t rows, uint64_t cols) {
    t_last_path = SNB_PATH_NONE;
    const bool types_ok = (input_type == SNB_TYPE_F32 || input_type == SNB_TYPE_BF16) &&
                          (output_type == SNB_TYPE_F32 || output_type == SNB_TYPE_BF16);
    if (!types_ok) return fail(SNB_ERR_INVALID_ARGUMENT, "scale_rows: unknown element type");
    if (input == output && input_type != output_type)
        return fail(SNB_ERR_INVALID_ARGUMENT, "scale_rows: in place needs one element type");
    if (rows > 0 && cols > 0 && (scale == nullptr || input == nullptr || output == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "scale_rows: null pointer");
    std::string err;
    int rc = scale_rows_launch(static_cast<cudaStream_t>(stream), scale, input, input_type, output, output_type, rows,
                               cols, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_adamw_step(void* stream, float* parameter, const float* gradient, float* first_moment, float* second_moment,
                   uint64_t count, const snb_adamw_hyper* hyper) {
    t_last_path = SNB_PATH_NONE;
    if (hyper == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "adamw_step: hyper is null");
    if (count > 0 && (parameter == nullptr || gradient == nullptr || first_moment == nullptr || second_moment == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "adamw_step: null pointer");
    std::string err;
    int rc = adamw_launch(static_cast<cudaStream_t>(stream), parameter, gradient, first_moment, second_moment, count,
                          *hyper, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_random_normal(void* stream, void* output, int32_t output_type, uint64_t count, uint64_t seed,
                      uint64_t first_draw, float std) {
    t_last_path = SNB_PATH_NONE;
    if (count > 0 && output == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "random_normal: null output");
    if (output_type != SNB_TYPE_F32 && output_type != SNB_TYPE_BF16)
        return fail(SNB_ERR_INVALID_ARGUMENT, "random_normal: output_type must be SNB_TYPE_F32 or SNB_TYPE_BF16");
    std::string err;
    int rc = random_normal_launch(static_cast<cudaStream_t>(stream), output, output_type, count, seed, first_draw, std,
                                  &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_random_below(void* stream, uint32_t* output, uint64_t count, uint64_t seed, uint64_t first_draw,
                     uint64_t bound) {
    t_last_path = SNB_PATH_NONE;
    if (count > 0 && output == nullptr) return fail(SNB_ERR_INVALID_ARGUMENT, "random_below: null output");
    if (bound == 0) return fail(SNB_ERR_INVALID_ARGUMENT, "random_below: bound must be positive");
    std::string err;
    int rc = random_below_launch(static_cast<cudaStream_t>(stream), output, count, seed, first_draw, bound, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_sum_of_squares(void* stream, const float* values, uint64_t count, double* result) {
    t_last_path = SNB_PATH_NONE;
    if (result == nullptr || (count > 0 && values == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "sum_of_squares: null pointer");
    std::string err;
    int rc = sum_of_squares_launch(static_cast<cudaStream_t>(stream), values, count, result, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_adamw_step_multi(void* stream, const snb_adamw_tensor* tensors, uint64_t tensor_count,
                         const snb_adamw_hyper* hyper, float max_gradient_norm, double* gradient_square_sum) {
    t_last_path = SNB_PATH_NONE;
    if (hyper == nullptr || gradient_square_sum == nullptr || (tensor_count > 0 && tensors == nullptr))
        return fail(SNB_ERR_INVALID_ARGUMENT, "adamw_step_multi: null pointer");
    for (uint64_t i = 0; i < tensor_count; ++i) {
        const snb_adamw_tensor& t = tensors[i];
        if (t.count > 0 && (t.parameter == nullptr || t.gradient == nullptr || t.first_moment == nullptr ||
                            t.second_moment == nullptr))
            return fail(SNB_ERR_INVALID_ARGUMENT, "adamw_step_multi: null pointer in tensor " + std::to_string(i));
    }
    if (!(max_gradient_norm > 0.0f)) return fail(SNB_ERR_INVALID_ARGUMENT, "adamw_step_multi: max_gradient_norm <= 0");
    std::string err;
    int rc = adamw_multi_launch(static_cast<cudaStream_t>(stream), tensors, tensor_count, *hyper, max_gradient_norm,
                                gradient_square_sum, &err);
    if (rc != SNB_OK) return fail(rc, err);
    t_last_path = SNB_PATH_SIMT;
    return SNB_OK;
}

int snb_selftest_bounded_wait(void* stream, uint64_t limit_ns) {
    if (limit_ns == 0 || limit_ns > 1000000000ull)
        return fail(SNB_ERR_INVALID_ARGUMENT, "selftest: limit_ns must lie in (0, 1 s]");
    std::string err;
    int rc = bounded_wait_probe(static_cast<cudaStream_t>(stream), limit_ns, &err);
    return rc == SNB_OK ? rc : fail(rc, err);
}

int snb_device_status(void) {
    unsigned int status = 0;
    std::string err;
    int rc = read_and_clear_device_status(&status, &err);
    if (rc != SNB_OK) return fail(rc, err);
    if (status != 0) return fail(SNB_ERR_DEVICE_TIMEOUT, "a tensor-core kernel's bounded wait timed out");
    return SNB_OK;
}

}  // extern "C"
