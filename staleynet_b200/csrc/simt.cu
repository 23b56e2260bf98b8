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
    const float* row_scale;   // [M] output-row multipliers (one matrix), or nullptr
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
                    float x = (p.row_scale ? p.scale * p.row_scale[row] : p.scale) * acc[i][j];
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

// Online (max, sum) pair of a softmax: sum of exp(x - max) over the values seen so far.
struct MaxSum {
    float m, s;
};

__device__ __forceinline__ MaxSum maxsum_add(MaxSum a, float x) {
    if (x > a.m) return {x, a.s * expf(a.m - x) + 1.0f};
    return {a.m, a.s + expf(x - a.m)};
}

__device__ __forceinline__ MaxSum maxsum_merge(MaxSum a, MaxSum b) {
    const float m = fmaxf(a.m, b.m);
    const float s = (a.s > 0.0f ? a.s * expf(a.m - m) : 0.0f) + (b.s > 0.0f ? b.s * expf(b.m - m) : 0.0f);
    return {m, s};
}

// One warp per row (kernels/attention.rs:153-180): p = exp(s*x - max) / sum over the visible keys
// 0..=q+query_offset, 0 after them; masked scores are never read. One read pass accumulates (max, sum) online,
// a second reads the visible scores again and writes the whole row (f32 in place and, with probs_bf16, bf16).
// VEC = 4 moves 16 bytes per lane and step (rows start 16-byte aligned).
template <int VEC>
__global__ void causal_softmax_kernel(float* scores, int64_t rows, int64_t queries, int64_t keys, float scale,
                                      int64_t query_offset, __nv_bfloat16* probs_bf16) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    float* values = scores + row * keys;
    int64_t visible = row % queries + query_offset + 1;
    if (visible > keys) visible = keys;
    MaxSum acc{-3.0e38f, 0.0f};
    for (int64_t k0 = static_cast<int64_t>(lane) * VEC; k0 < visible; k0 += 32 * VEC) {
        float x[VEC];
        if constexpr (VEC == 4) {
            const float4 v = *reinterpret_cast<const float4*>(values + k0);
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
            x[0] = values[k0];
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i)
            if (k0 + i < visible) acc = maxsum_add(acc, x[i] * scale);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        MaxSum other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
        acc = maxsum_merge(acc, other);
    }
    const float normaliser = 1.0f / acc.s;
    __nv_bfloat16* out16 = probs_bf16 ? probs_bf16 + row * keys : nullptr;
    for (int64_t k0 = static_cast<int64_t>(lane) * VEC; k0 < keys; k0 += 32 * VEC) {
        float p[VEC];
        if (k0 < visible) {
            float x[VEC];
            if constexpr (VEC == 4) {
                const float4 v = *reinterpret_cast<const float4*>(values + k0);
                x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
            } else {
                x[0] = values[k0];
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) p[i] = k0 + i < visible ? expf(x[i] * scale - acc.m) * normaliser : 0.0f;
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) p[i] = 0.0f;
        }
        if constexpr (VEC == 4) {
            *reinterpret_cast<float4*>(values + k0) = make_float4(p[0], p[1], p[2], p[3]);
            if (out16) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(p[0], p[1]);
                __nv_bfloat162 hi = __floats2bfloat162_rn(p[2], p[3]);
                uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
                *reinterpret_cast<uint2*>(out16 + k0) = packed;
            }
        } else {
            values[k0] = p[0];
            if (out16) out16[k0] = __float2bfloat16_rn(p[0]);
        }
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
template <int VEC>
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
    for (int64_t c0 = static_cast<int64_t>(lane) * VEC; c0 < visible; c0 += 32 * VEC) {
        if constexpr (VEC == 4) {
            const float4 pv = *reinterpret_cast<const float4*>(p + c0);
            const float4 gv = *reinterpret_cast<const float4*>(g + c0);
            const float pp[4] = {pv.x, pv.y, pv.z, pv.w};
            const float gg[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (c0 + i < visible) projection += gg[i] * pp[i];
        } else {
            projection += g[c0] * p[c0];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) projection += __shfl_xor_sync(0xffffffffu, projection, o);
    __nv_bfloat16* out16 = grad_bf16 ? grad_bf16 + row * cols : nullptr;
    for (int64_t c0 = static_cast<int64_t>(lane) * VEC; c0 < cols; c0 += 32 * VEC) {
        float d[VEC];
        if (c0 < visible) {
            if constexpr (VEC == 4) {
                const float4 pv = *reinterpret_cast<const float4*>(p + c0);
                const float4 gv = *reinterpret_cast<const float4*>(g + c0);
                const float pp[4] = {pv.x, pv.y, pv.z, pv.w};
                const float gg[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) d[i] = c0 + i < visible ? pp[i] * (gg[i] - projection) : 0.0f;
            } else {
                d[0] = p[c0] * (g[c0] - projection);
            }
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) d[i] = 0.0f;
        }
        if constexpr (VEC == 4) {
            *reinterpret_cast<float4*>(g + c0) = make_float4(d[0], d[1], d[2], d[3]);
            if (out16) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(d[0], d[1]);
                __nv_bfloat162 hi = __floats2bfloat162_rn(d[2], d[3]);
                *reinterpret_cast<uint2*>(out16 + c0) =
                    make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
            }
        } else {
            g[c0] = d[0];
            if (out16) out16[c0] = __float2bfloat16_rn(d[0]);
        }
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
    p.row_scale = r.row_scale;
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
    const bool vec = keys % 4 == 0 && reinterpret_cast<uintptr_t>(scores) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(probs_bf16) % 8 == 0;
    if (vec)
        causal_softmax_kernel<4><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            scores, static_cast<int64_t>(rows), static_cast<int64_t>(queries), static_cast<int64_t>(keys), scale,
            static_cast<int64_t>(query_offset), reinterpret_cast<__nv_bfloat16*>(probs_bf16));
    else
        causal_softmax_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
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
    const bool vec = cols % 4 == 0 && reinterpret_cast<uintptr_t>(probabilities) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(grad) % 16 == 0 && reinterpret_cast<uintptr_t>(grad_bf16) % 8 == 0;
    if (vec)
        causal_softmax_backward_kernel<4><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            probabilities, grad, static_cast<int64_t>(rows), static_cast<int64_t>(queries),
            static_cast<int64_t>(cols), static_cast<int64_t>(query_offset),
            reinterpret_cast<__nv_bfloat16*>(grad_bf16));
    else
        causal_softmax_backward_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            probabilities, grad, static_cast<int64_t>(rows), static_cast<int64_t>(queries),
            static_cast<int64_t>(cols), static_cast<int64_t>(query_offset),
            reinterpret_cast<__nv_bfloat16*>(grad_bf16));
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
