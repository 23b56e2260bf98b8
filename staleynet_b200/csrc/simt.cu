// simt.cu — kernels that run on the SM's CUDA cores:
//  * the strided GEMM for layouts TMA cannot read (no unit stride, strides not 16-byte multiples, ragged sizes
//    such as the reference test's 17x33x9) and for exact f32 arithmetic (`MatmulKernel::{Naive,Tiled,Blocked}`,
//    crates/staleynet-cuda/src/device.rs:38-67). Each output is one f32 sum over k in increasing order, like
//    reference::matmul (reference.rs:18-38), tiled 64x64 with a 4x4 block per thread.
//  * the causal softmax and its backward between the attention products
//    (crates/staleynet-cuda/src/kernels/attention.rs:153-207).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "internal.h"

namespace snb {

namespace {

constexpr int ST_TILE = 64;
constexpr int ST_DEPTH = 16;
constexpr int ST_THREADS = 256;

struct SimtParams {
    int64_t M, N, K;
    int64_t a_rs, a_cs, a_bs;
    int64_t b_rs, b_cs, b_bs;
    int64_t c_bs;
    int64_t count;
    float scale;
    int accumulate;
    int a_bf16, b_bf16, c_bf16;
    const float* bias;
    int activation;
    int aux_bf16;
    void* pre;
    const void* gelu_input;
    const void* residual;
};

__device__ __forceinline__ float load_any(const void* base, int64_t index, int is_bf16) {
    if (is_bf16) {
        const unsigned short bits = reinterpret_cast<const unsigned short*>(base)[index];
        return __uint_as_float(static_cast<uint32_t>(bits) << 16);
    }
    return reinterpret_cast<const float*>(base)[index];
}

__device__ __forceinline__ void store_any(void* base, int64_t index, float v, int is_bf16) {
    if (is_bf16) {
        reinterpret_cast<__nv_bfloat16*>(base)[index] = __float2bfloat16_rn(v);
    } else {
        reinterpret_cast<float*>(base)[index] = v;
    }
}

__device__ __forceinline__ float gelu_f(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978846f * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float gelu_df(float x) {
    const float t = tanhf(0.7978846f * (x + 0.044715f * x * x * x));
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978846f * (1.0f + 3.0f * 0.044715f * x * x);
}

__global__ void __launch_bounds__(ST_THREADS) simt_gemm_kernel(const void* __restrict__ A, const void* __restrict__ B,
                                                                void* C, const SimtParams p) {
    __shared__ float As[ST_DEPTH][ST_TILE + 4];  // [k][m]
    __shared__ float Bs[ST_DEPTH][ST_TILE + 4];  // [k][n]
    const int tx = threadIdx.x % 16;
    const int ty = threadIdx.x / 16;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * ST_TILE;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * ST_TILE;
    // Consecutive threads walk the operand's contiguous direction so global reads coalesce.
    const bool a_m_fast = p.a_rs == 1 && p.a_cs != 1;
    const bool b_n_fast = !(p.b_rs == 1 && p.b_cs != 1);

    for (int64_t b = blockIdx.z; b < p.count; b += gridDim.z) {
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

        for (int64_t k0 = 0; k0 < p.K; k0 += ST_DEPTH) {
#pragma unroll
            for (int l = 0; l < (ST_TILE * ST_DEPTH) / ST_THREADS; ++l) {
                const int lin = threadIdx.x + l * ST_THREADS;
                int am, ak, bn, bk;
                if (a_m_fast) { am = lin % ST_TILE; ak = lin / ST_TILE; } else { ak = lin % ST_DEPTH; am = lin / ST_DEPTH; }
                if (b_n_fast) { bn = lin % ST_TILE; bk = lin / ST_TILE; } else { bk = lin % ST_DEPTH; bn = lin / ST_DEPTH; }
                const int64_t gm = m0 + am, gk = k0 + ak;
                As[ak][am] = (gm < p.M && gk < p.K) ? load_any(A, b * p.a_bs + gm * p.a_rs + gk * p.a_cs, p.a_bf16) : 0.0f;
                const int64_t gn = n0 + bn, gk2 = k0 + bk;
                Bs[bk][bn] = (gn < p.N && gk2 < p.K) ? load_any(B, b * p.b_bs + gk2 * p.b_rs + gn * p.b_cs, p.b_bf16) : 0.0f;
            }
            __syncthreads();
            const int depth = static_cast<int>(p.K - k0 < ST_DEPTH ? p.K - k0 : ST_DEPTH);
            for (int k = 0; k < depth; ++k) {
                float a[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
                for (int j = 0; j < 4; ++j) bv[j] = Bs[k][tx + 16 * j];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
            }
            __syncthreads();
        }

#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t row = m0 + ty + 16 * i;
                const int64_t col = n0 + tx + 16 * j;
                if (row < p.M && col < p.N) {
                    const int64_t idx = b * p.c_bs + row * p.N + col;
                    float x = p.scale * acc[i][j];
                    if (p.bias) x += p.bias[col];
                    if (p.pre) store_any(p.pre, idx, x, p.c_bf16);
                    if (p.activation == SNB_ACTIVATION_GELU) x = gelu_f(x);
                    else if (p.activation == SNB_ACTIVATION_GELU_GRAD) x *= gelu_df(load_any(p.gelu_input, idx, p.aux_bf16));
                    if (p.residual) x += load_any(p.residual, idx, p.c_bf16);
                    if (p.accumulate) x += load_any(C, idx, p.c_bf16);
                    store_any(C, idx, x, p.c_bf16);
                }
            }
        }
    }
}

// One warp per row (kernels/attention.rs:153-180): max of the scaled visible scores, exponentials, normalisation;
// keys after q + query_offset become 0 and are never read. With probs_bf16 the probabilities are also written as
// bf16 (the operand of bf16 P*V and P^T*dO products).
__global__ void causal_softmax_kernel(float* scores, int64_t rows, int64_t queries, int64_t keys, float scale,
                                      int64_t query_offset, __nv_bfloat16* probs_bf16) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    float* values = scores + row * keys;
    int64_t visible = row % queries + query_offset + 1;
    if (visible > keys) visible = keys;
    float maximum = -3.0e38f;
    for (int64_t k = lane; k < visible; k += 32) maximum = fmaxf(maximum, values[k] * scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maximum = fmaxf(maximum, __shfl_xor_sync(0xffffffffu, maximum, o));
    float total = 0.0f;
    for (int64_t k = lane; k < visible; k += 32) {
        const float e = expf(values[k] * scale - maximum);
        values[k] = e;
        total += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    const float normaliser = 1.0f / total;
    __nv_bfloat16* out16 = probs_bf16 ? probs_bf16 + row * keys : nullptr;
    for (int64_t k = lane; k < keys; k += 32) {
        const float p = k < visible ? values[k] * normaliser : 0.0f;
        values[k] = p;
        if (out16) out16[k] = __float2bfloat16_rn(p);
    }
}

// grad <- p * (grad - sum(grad * p)) per row, one warp per row (kernels/attention.rs:190-207).
__global__ void softmax_backward_kernel(const float* probabilities, float* grad, int64_t rows, int64_t cols) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    const float* p = probabilities + row * cols;
    float* g = grad + row * cols;
    float projection = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) projection += g[c] * p[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) projection += __shfl_xor_sync(0xffffffffu, projection, o);
    for (int64_t c = lane; c < cols; c += 32) g[c] = p[c] * (g[c] - projection);
}

// The same for causal probabilities: only the visible keys 0..=q+query_offset are read (p is 0 after them, so the
// sum and the result are unchanged), masked gradient entries are never read and become 0; optional bf16 copy.
__global__ void causal_softmax_backward_kernel(const float* probabilities, float* grad, int64_t rows,
                                               int64_t queries, int64_t cols, int64_t query_offset,
                                               __nv_bfloat16* grad_bf16) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    const float* p = probabilities + row * cols;
    float* g = grad + row * cols;
    int64_t visible = row % queries + query_offset + 1;
    if (visible > cols) visible = cols;
    float projection = 0.0f;
    for (int64_t c = lane; c < visible; c += 32) projection += g[c] * p[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) projection += __shfl_xor_sync(0xffffffffu, projection, o);
    __nv_bfloat16* out16 = grad_bf16 ? grad_bf16 + row * cols : nullptr;
    for (int64_t c = lane; c < cols; c += 32) {
        const float d = c < visible ? p[c] * (g[c] - projection) : 0.0f;
        g[c] = d;
        if (out16) out16[c] = __float2bfloat16_rn(d);
    }
}

}  // namespace

int simt_gemm(cudaStream_t stream, const GemmRequest& r, std::string* err) {
    SimtParams p{};
    p.M = static_cast<int64_t>(r.p.rows);
    p.N = static_cast<int64_t>(r.p.cols);
    p.K = static_cast<int64_t>(r.p.inner);
    p.a_rs = static_cast<int64_t>(r.p.left.row_stride);
    p.a_cs = static_cast<int64_t>(r.p.left.col_stride);
    p.a_bs = static_cast<int64_t>(r.p.left.batch_stride);
    p.b_rs = static_cast<int64_t>(r.p.right.row_stride);
    p.b_cs = static_cast<int64_t>(r.p.right.col_stride);
    p.b_bs = static_cast<int64_t>(r.p.right.batch_stride);
    p.c_bs = static_cast<int64_t>(r.p.output_batch_stride);
    p.count = static_cast<int64_t>(r.count);
    p.scale = r.p.scale;
    p.accumulate = r.p.accumulate != 0;
    p.a_bf16 = r.a_type == SNB_TYPE_BF16;
    p.b_bf16 = r.b_type == SNB_TYPE_BF16;
    p.c_bf16 = r.c_type == SNB_TYPE_BF16;
    p.bias = r.bias;
    p.activation = r.activation;
    p.aux_bf16 = r.aux_type == SNB_TYPE_BF16;
    p.pre = r.pre;
    p.gelu_input = r.gelu_input;
    p.residual = r.residual;
    const int64_t gx = (p.N + ST_TILE - 1) / ST_TILE;
    const int64_t gy = (p.M + ST_TILE - 1) / ST_TILE;
    if (gx > 0x7fffffff || gy > 65535) {
        *err = "matmul: rows exceed the SIMT kernel's grid (" + std::to_string(p.M) + ")";
        return SNB_ERR_UNSUPPORTED;
    }
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(std::min<int64_t>(p.count, 65535)));
    simt_gemm_kernel<<<grid, ST_THREADS, 0, stream>>>(r.A, r.B, r.C, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("simt_gemm_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

int causal_softmax(cudaStream_t stream, float* scores, uint64_t rows, uint64_t queries, uint64_t keys, float scale,
                   uint64_t query_offset, uint16_t* probs_bf16, std::string* err) {
    if (rows == 0) return SNB_OK;
    const int threads = 256;
    const uint64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffffull) {
        *err = "causal_softmax: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    causal_softmax_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        scores, static_cast<int64_t>(rows), static_cast<int64_t>(queries), static_cast<int64_t>(keys), scale,
        static_cast<int64_t>(query_offset), reinterpret_cast<__nv_bfloat16*>(probs_bf16));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("causal_softmax_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

int causal_softmax_backward(cudaStream_t stream, const float* probabilities, float* grad, uint64_t rows,
                            uint64_t queries, uint64_t cols, uint64_t query_offset, uint16_t* grad_bf16,
                            std::string* err) {
    if (rows == 0) return SNB_OK;
    const int threads = 256;
    const uint64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffffull) {
        *err = "causal_softmax_backward: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    causal_softmax_backward_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        probabilities, grad, static_cast<int64_t>(rows), static_cast<int64_t>(queries), static_cast<int64_t>(cols),
        static_cast<int64_t>(query_offset), reinterpret_cast<__nv_bfloat16*>(grad_bf16));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("causal_softmax_backward_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

int softmax_backward(cudaStream_t stream, const float* probabilities, float* grad, uint64_t rows, uint64_t cols,
                     std::string* err) {
    if (rows == 0) return SNB_OK;
    const int threads = 256;
    const uint64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffffull) {
        *err = "softmax_backward: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    softmax_backward_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        probabilities, grad, static_cast<int64_t>(rows), static_cast<int64_t>(cols));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("softmax_backward_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

}  // namespace snb
