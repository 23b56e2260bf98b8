// norm_optim.cu — RMSNorm and the optimizer step of the training loop, around the GEMMs:
//   RMSNorm forward / backward (crates/staleynet-cuda/src/kernels/normalization.rs:27-127): per row
//     s = 1 / sqrt(mean(x^2) + epsilon), y = x s g;  dx = s g dy - x s^3 / cols sum(dy g x);  dg += sum_rows dy x s.
//   The fused prologue of a GEMM on normalised rows: the statistics s alone (rms_norm_stats), and the gain folded
//   into the right operand (scale_rows: W_g[k, :] = g[k] W[k, :]), so that rms_norm(x) W = diag(s) x W_g is one GEMM
//   with row_scale = s and no normalised copy of x.
//   AdamW (kernels/optimizer.rs:47-71) for one tensor, the sum of squares of the gradient-norm clip
//   (kernels/optimizer.rs:80-113; reduced to one f64 on the device instead of on the host), and both over every
//   parameter tensor of a model in one launch each, the clip factor computed on the device from the global norm
//   (model optimizer.rs:125-177 does this per tensor with a host round trip and a separate scaling pass).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>

#include "internal.h"

namespace snb {
namespace {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    return v;
}

__device__ __forceinline__ float load_elem(const void* base, int64_t i, bool bf16) {
    return bf16 ? __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(base)[i]) << 16)
                : reinterpret_cast<const float*>(base)[i];
}

__device__ __forceinline__ void store_elem(void* base, int64_t i, float x, bool bf16) {
    if (bf16) {
        const uint32_t u = __float_as_uint(x);
        reinterpret_cast<uint16_t*>(base)[i] = static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
    } else {
        reinterpret_cast<float*>(base)[i] = x;
    }
}

// Eight consecutive elements from 16 bytes of bf16 (or four from f32; the rest of `v` is left alone).
__device__ __forceinline__ void unpack16(uint4 q, bool bf16, float (&v)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (bf16) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = __uint_as_float(w[k] << 16);
            v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __uint_as_float(w[k]);
    }
}

// The row computation of rms_norm_forward_kernel (one warp).
__device__ __forceinline__ void rms_norm_row(const void* input, int in_bf16, const float* gain, void* output,
                                             int out_bf16, float* inv_rms, int64_t row, int64_t cols, float epsilon,
                                             int vec, int lane) {
    const int64_t base = row * cols;
    const int per = in_bf16 ? 8 : 4;   // elements per 16 bytes of input
    float square_sum = 0.0f;
    if (vec) {
        const uint4* src = reinterpret_cast<const uint4*>(
            reinterpret_cast<const uint8_t*>(input) + base * (in_bf16 ? 2 : 4));
        const int64_t pieces = cols / per;
#pragma unroll 4
        for (int64_t k = lane; k < pieces; k += 32) {
            float v[8];
            unpack16(__ldg(src + k), in_bf16, v);
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (e < per) square_sum += v[e] * v[e];
        }
    } else {
        for (int64_t c = lane; c < cols; c += 32) {
            const float x = load_elem(input, base + c, in_bf16);
            square_sum += x * x;
        }
    }
    const float inverse = 1.0f / sqrtf(warp_sum_f(square_sum) / static_cast<float>(cols) + epsilon);
    // The normalised output, one element per lane so that a warp's stores are contiguous.
    if (output != nullptr) {
        for (int64_t c = lane; c < cols; c += 32)
            store_elem(output, base + c, load_elem(input, base + c, in_bf16) * inverse * gain[c], out_bf16);
    }
    if (lane == 0) inv_rms[row] = inverse;
}

// One warp per row (the launch gives every row its own warp: a grid of fewer, row-looping warps measured slower,
// since a warp reduces one row before it loads the next): inv_rms[row] = s and, when `output` is given,
// output = x s g (of out_bf16's type). With `vec`
// (every row of the input starts on a 16-byte boundary) each lane reads 16-byte pieces of the row for the sum of
// squares (the same f32 values added in a different order).
__global__ void rms_norm_forward_kernel(const void* input, int in_bf16, const float* gain, void* output, int out_bf16,
                                        float* inv_rms, int64_t rows, int64_t cols, float epsilon, int vec) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps)
        rms_norm_row(input, in_bf16, gain, output, out_bf16, inv_rms, row, cols, epsilon, vec, lane);
}

// One warp per row: dx = s g dy - x s^3 / cols sum(dy g x).
__global__ void rms_norm_backward_input_kernel(const float* dy, const float* x, const float* gain,
                                               const float* inv_rms, float* dx, int64_t rows, int64_t cols) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t base = row * cols;
    const float inverse = inv_rms[row];
    float projection = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) projection += dy[base + c] * gain[c] * x[base + c];
    const float correction = inverse * inverse * inverse * warp_sum_f(projection) / static_cast<float>(cols);
    for (int64_t c = lane; c < cols; c += 32)
        dx[base + c] = inverse * gain[c] * dy[base + c] - x[base + c] * correction;
}

constexpr int64_t kGainRowsPerBlock = 256;

// gain_grad[c] += sum over rows of dy x s: block (bx, by) sums rows [256 bx, 256 bx + 256) for the columns its
// threads stride over, then adds with one atomic per column.
__global__ void rms_norm_backward_gain_kernel(const float* dy, const float* x, const float* inv_rms, float* gain_grad,
                                              int64_t rows, int64_t cols) {
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kGainRowsPerBlock;
    const int64_t r1 = r0 + kGainRowsPerBlock < rows ? r0 + kGainRowsPerBlock : rows;
    for (int64_t c = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x; c < cols;
         c += static_cast<int64_t>(gridDim.y) * blockDim.x) {
        float sum = 0.0f;
        for (int64_t r = r0; r < r1; ++r) sum += dy[r * cols + c] * x[r * cols + c] * inv_rms[r];
        atomicAdd(gain_grad + c, sum);
    }
}

// out[k, n] = scale[k] * in[k, n] for a row-major [rows, cols] matrix.
__global__ void scale_rows_kernel(const float* scale, const void* in, int in_bf16, void* out, int out_bf16,
                                  int64_t rows, int64_t cols) {
    const int64_t total = rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        store_elem(out, i, scale[i / cols] * load_elem(in, i, in_bf16), out_bf16);
}

struct AdamWArgs {
    float learning_rate, beta1, beta2, epsilon;
    float first_correction, second_correction;
};

// The reference's per-element update (kernels/optimizer.rs:57-70), on the gradient times `clip`, in registers.
__device__ __forceinline__ void adamw_value(float& weight, float gradient, float& first, float& second,
                                            const AdamWArgs& a, float weight_decay, float clip) {
    const float grad = gradient * clip;
    const float mean = a.beta1 * first + (1.0f - a.beta1) * grad;
    const float variance = a.beta2 * second + (1.0f - a.beta2) * grad * grad;
    first = mean;
    second = variance;
    const float mean_hat = mean / a.first_correction;
    const float variance_hat = variance / a.second_correction;
    const float update = mean_hat / (sqrtf(variance_hat) + a.epsilon) + weight_decay * weight;
    weight = weight - a.learning_rate * update;
}

__device__ __forceinline__ void adamw_element(float* parameter, const float* gradient, float* first, float* second,
                                              int64_t i, const AdamWArgs& a, float weight_decay, float clip) {
    float w = parameter[i], m = first[i], v = second[i];
    adamw_value(w, gradient[i], m, v, a, weight_decay, clip);
    first[i] = m;
    second[i] = v;
    parameter[i] = w;
}

// Arrays that start on 16-byte boundaries are read and written as float4 vectors, four elements per access, which
// keeps four times as many bytes in flight per thread (the streaming kernels here are bound by HBM latency times
// bandwidth, not arithmetic).
__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ void adamw_vector(float* parameter, const float* gradient, float* first, float* second,
                                             int64_t j, const AdamWArgs& a, float weight_decay, float clip) {
    float4 pv = reinterpret_cast<float4*>(parameter)[j], mv = reinterpret_cast<float4*>(first)[j];
    float4 vv = reinterpret_cast<float4*>(second)[j];
    const float4 gv = reinterpret_cast<const float4*>(gradient)[j];
    adamw_value(pv.x, gv.x, mv.x, vv.x, a, weight_decay, clip);
    adamw_value(pv.y, gv.y, mv.y, vv.y, a, weight_decay, clip);
    adamw_value(pv.z, gv.z, mv.z, vv.z, a, weight_decay, clip);
    adamw_value(pv.w, gv.w, mv.w, vv.w, a, weight_decay, clip);
    reinterpret_cast<float4*>(parameter)[j] = pv;
    reinterpret_cast<float4*>(first)[j] = mv;
    reinterpret_cast<float4*>(second)[j] = vv;
}

__global__ void adamw_kernel(float* parameter, const float* gradient, float* first, float* second, int64_t count,
                             AdamWArgs a, float weight_decay) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t scalar_begin = 0;
    if (aligned16(parameter) && aligned16(gradient) && aligned16(first) && aligned16(second)) {
        for (int64_t j = tid; j < count / 4; j += stride) adamw_vector(parameter, gradient, first, second, j, a,
                                                                      weight_decay, 1.0f);
        scalar_begin = count / 4 * 4;
    }
    for (int64_t i = scalar_begin + tid; i < count; i += stride)
        adamw_element(parameter, gradient, first, second, i, a, weight_decay, 1.0f);
}

// Block sums of squares added into one f64 (`total`, zeroed by the host).
__device__ __forceinline__ void add_block_sum(float v, double* total) {
    __shared__ float warp_sums[8];
    v = warp_sum_f(v);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += static_cast<double>(warp_sums[w]);
        atomicAdd(total, s);
    }
}

__global__ void __launch_bounds__(256) sum_of_squares_kernel(const float* values, int64_t count, double* total) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    float sum = 0.0f;
    int64_t scalar_begin = 0;
    if (aligned16(values)) {
        const float4* v4 = reinterpret_cast<const float4*>(values);
        for (int64_t j = tid; j < count / 4; j += stride) {
            const float4 v = v4[j];
            sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        scalar_begin = count / 4 * 4;
    }
    for (int64_t i = scalar_begin + tid; i < count; i += stride) sum += values[i] * values[i];
    add_block_sum(sum, total);
}

// Every parameter tensor of a model in one launch: block b takes chunk b of the concatenation of the tensors
// (chunk_start[t] = first chunk of tensor t), kMultiChunk elements per chunk.
constexpr int kMultiMax = 256;
constexpr int64_t kMultiChunk = 16384;

struct MultiTensors {
    int32_t n;
    snb_adamw_tensor t[kMultiMax];
    int64_t chunk_start[kMultiMax + 1];
};

__device__ __forceinline__ int tensor_of_chunk(const MultiTensors& m, int64_t chunk) {
    int lo = 0, hi = m.n - 1;
    while (lo < hi) {   // last t with chunk_start[t] <= chunk
        const int mid = (lo + hi + 1) >> 1;
        if (m.chunk_start[mid] <= chunk) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Chunks start at multiples of kMultiChunk (a multiple of 4), so a tensor whose arrays are 16-byte aligned is
// read and written in float4 vectors (see aligned16); the last count % 4 elements and unaligned tensors take the
// scalar path.

__global__ void __launch_bounds__(256) multi_sum_of_squares_kernel(const __grid_constant__ MultiTensors m,
                                                                   double* total) {
    const int64_t chunk = blockIdx.x;
    const int t = tensor_of_chunk(m, chunk);
    const int64_t begin = (chunk - m.chunk_start[t]) * kMultiChunk;
    const int64_t end = begin + kMultiChunk < static_cast<int64_t>(m.t[t].count) ? begin + kMultiChunk
                                                                                   : static_cast<int64_t>(m.t[t].count);
    const float* g = m.t[t].gradient;
    float sum = 0.0f;
    int64_t scalar_begin = begin;
    if (aligned16(g)) {
        const int64_t n4 = (end - begin) >> 2;
        const float4* g4 = reinterpret_cast<const float4*>(g + begin);
        for (int64_t j = threadIdx.x; j < n4; j += blockDim.x) {
            const float4 v = g4[j];
            sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        scalar_begin = begin + 4 * n4;
    }
    for (int64_t i = scalar_begin + threadIdx.x; i < end; i += blockDim.x) sum += g[i] * g[i];
    add_block_sum(sum, total);
}

__global__ void __launch_bounds__(256) multi_adamw_kernel(const __grid_constant__ MultiTensors m, AdamWArgs a,
                                                          const double* square_sum, float max_norm) {
    const float norm = static_cast<float>(sqrt(*square_sum));
    const float clip = norm > max_norm ? max_norm / norm : 1.0f;   // model optimizer.rs:127
    const int64_t chunk = blockIdx.x;
    const int t = tensor_of_chunk(m, chunk);
    const int64_t begin = (chunk - m.chunk_start[t]) * kMultiChunk;
    const int64_t end = begin + kMultiChunk < static_cast<int64_t>(m.t[t].count) ? begin + kMultiChunk
                                                                                   : static_cast<int64_t>(m.t[t].count);
    const snb_adamw_tensor& x = m.t[t];
    int64_t scalar_begin = begin;
    if (aligned16(x.parameter) && aligned16(x.gradient) && aligned16(x.first_moment) && aligned16(x.second_moment)) {
        const int64_t n4 = (end - begin) >> 2;
        for (int64_t j = threadIdx.x; j < n4; j += blockDim.x)
            adamw_vector(x.parameter + begin, x.gradient + begin, x.first_moment + begin, x.second_moment + begin, j,
                         a, x.weight_decay, clip);
        scalar_begin = begin + 4 * n4;
    }
    for (int64_t i = scalar_begin + threadIdx.x; i < end; i += blockDim.x)
        adamw_element(x.parameter, x.gradient, x.first_moment, x.second_moment, i, a, x.weight_decay, clip);
}

AdamWArgs adamw_args(const snb_adamw_hyper& h) {
    AdamWArgs a{};
    a.learning_rate = h.learning_rate;
    a.beta1 = h.beta1;
    a.beta2 = h.beta2;
    a.epsilon = h.epsilon;
    // 1 - beta^step as ops/optimizer.rs:44-54 computes it (f32 powi: repeated multiplication).
    float b1 = 1.0f, b2 = 1.0f;
    for (uint32_t i = 0; i < h.step; ++i) {
        b1 *= h.beta1;
        b2 *= h.beta2;
    }
    a.first_correction = 1.0f - b1;
    a.second_correction = 1.0f - b2;
    return a;
}

int launch_status(const char* what, std::string* err) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message(what, e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

unsigned warp_rows_grid(int64_t rows) { return static_cast<unsigned>((rows + 7) / 8); }

}  // namespace

int rms_norm_forward_launch(cudaStream_t s, const void* input, int input_type, const float* gain, void* output,
                            int output_type, float* inv_rms, uint64_t rows, uint64_t cols, float epsilon,
                            std::string* err) {
    if (rows == 0) return SNB_OK;
    if (rows > (1ull << 34)) {
        *err = "rms_norm: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    const uint64_t row_bytes = cols * (input_type == SNB_TYPE_BF16 ? 2 : 4);
    const int vec = (reinterpret_cast<uintptr_t>(input) % 16 == 0 && row_bytes % 16 == 0) ? 1 : 0;
    rms_norm_forward_kernel<<<warp_rows_grid(static_cast<int64_t>(rows)), 256, 0, s>>>(
        input, input_type == SNB_TYPE_BF16, gain, output, output_type == SNB_TYPE_BF16, inv_rms,
        static_cast<int64_t>(rows), static_cast<int64_t>(cols), epsilon, vec);
    return launch_status("rms_norm_forward_kernel launch", err);
}

int rms_norm_backward_launch(cudaStream_t s, const float* dy, const float* x, const float* gain, const float* inv_rms,
                             float* dx, float* gain_grad, uint64_t rows, uint64_t cols, std::string* err) {
    if (rows == 0 || cols == 0) return SNB_OK;
    if (rows > (1ull << 34)) {
        *err = "rms_norm: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    rms_norm_backward_input_kernel<<<warp_rows_grid(static_cast<int64_t>(rows)), 256, 0, s>>>(
        dy, x, gain, inv_rms, dx, static_cast<int64_t>(rows), static_cast<int64_t>(cols));
    int rc = launch_status("rms_norm_backward_input_kernel launch", err);
    if (rc != SNB_OK) return rc;
    const int64_t bx = (static_cast<int64_t>(rows) + kGainRowsPerBlock - 1) / kGainRowsPerBlock;
    const int64_t by = (static_cast<int64_t>(cols) + 255) / 256;
    rms_norm_backward_gain_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by < 65535 ? by : 65535)),
                                    256, 0, s>>>(dy, x, inv_rms, gain_grad, static_cast<int64_t>(rows),
                                                 static_cast<int64_t>(cols));
    return launch_status("rms_norm_backward_gain_kernel launch", err);
}

int scale_rows_launch(cudaStream_t s, const float* scale, const void* in, int in_type, void* out, int out_type,
                      uint64_t rows, uint64_t cols, std::string* err) {
    if (rows == 0 || cols == 0) return SNB_OK;
    scale_rows_kernel<<<148 * 8, 256, 0, s>>>(scale, in, in_type == SNB_TYPE_BF16, out, out_type == SNB_TYPE_BF16,
                                              static_cast<int64_t>(rows), static_cast<int64_t>(cols));
    return launch_status("scale_rows_kernel launch", err);
}

int adamw_launch(cudaStream_t s, float* parameter, const float* gradient, float* first, float* second, uint64_t count,
                 const snb_adamw_hyper& h, std::string* err) {
    if (count == 0) return SNB_OK;
    adamw_kernel<<<148 * 8, 256, 0, s>>>(parameter, gradient, first, second, static_cast<int64_t>(count),
                                         adamw_args(h), h.weight_decay);
    return launch_status("adamw_kernel launch", err);
}

int sum_of_squares_launch(cudaStream_t s, const float* values, uint64_t count, double* total, std::string* err) {
    cudaError_t e = cudaMemsetAsync(total, 0, sizeof(double), s);
    if (e != cudaSuccess) {
        *err = cuda_message("cudaMemsetAsync(sum of squares)", e);
        return SNB_ERR_CUDA;
    }
    if (count == 0) return SNB_OK;
    sum_of_squares_kernel<<<148 * 4, 256, 0, s>>>(values, static_cast<int64_t>(count), total);
    return launch_status("sum_of_squares_kernel launch", err);
}

int adamw_multi_launch(cudaStream_t s, const snb_adamw_tensor* tensors, uint64_t n, const snb_adamw_hyper& h,
                       float max_gradient_norm, double* square_sum, std::string* err) {
    cudaError_t e = cudaMemsetAsync(square_sum, 0, sizeof(double), s);
    if (e != cudaSuccess) {
        *err = cuda_message("cudaMemsetAsync(gradient square sum)", e);
        return SNB_ERR_CUDA;
    }
    if (n == 0) return SNB_OK;
    if (n > static_cast<uint64_t>(kMultiMax)) {
        *err = "adamw_step_multi: at most " + std::to_string(kMultiMax) + " tensors per call";
        return SNB_ERR_UNSUPPORTED;
    }
    MultiTensors m{};
    m.n = static_cast<int32_t>(n);
    int64_t chunks = 0;
    for (uint64_t i = 0; i < n; ++i) {
        m.t[i] = tensors[i];
        m.chunk_start[i] = chunks;
        chunks += (static_cast<int64_t>(tensors[i].count) + kMultiChunk - 1) / kMultiChunk;
    }
    m.chunk_start[n] = chunks;
    if (chunks == 0) return SNB_OK;
    if (chunks > 0x7fffffff) {
        *err = "adamw_step_multi: too many elements";
        return SNB_ERR_UNSUPPORTED;
    }
    // Empty tensors own no chunk; a block never lands on one because chunk_start repeats their start.
    multi_sum_of_squares_kernel<<<static_cast<unsigned>(chunks), 256, 0, s>>>(m, square_sum);
    int rc = launch_status("multi_sum_of_squares_kernel launch", err);
    if (rc != SNB_OK) return rc;
    multi_adamw_kernel<<<static_cast<unsigned>(chunks), 256, 0, s>>>(m, adamw_args(h), square_sum, max_gradient_norm);
    return launch_status("multi_adamw_kernel launch", err);
}

}  // namespace snb
