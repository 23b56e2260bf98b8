// cross_entropy.cu — softmax cross-entropy with its gradient, for one classifier head or for every codebook head of
// the output layer in one launch: the reference's `cross_entropy` kernel (crates/staleynet-cuda/src/kernels/loss.rs:
// 54-94, CPU form reference.rs:139-166). Per (row, head): log_partition = max + log(sum exp(z - max)),
// loss = log_partition - z[target], gradient = (exp(z - log_partition) - onehot(target)) * grad_scale; rows whose
// target is EMPTY_TOKEN get loss 0 and a zero gradient; columns of other heads are left untouched.
//
// One warp per (row, head), 8 warps per block, each warp taking CE_ROWS_PER_WARP rows of one head. When a head's
// classes are a multiple of 256 (up to 2048) and its rows are 16-byte aligned, each lane keeps its classes/32 logits
// in registers, so every logit is read once and its gradient written once (the gradient may overwrite the logits in
// place), with base-2 exponentials (ex2.approx, relative error ~2^-22); otherwise three lane-strided passes over the
// row with expf/logf, as the reference does. Per-head loss sums are reduced
// per block and added with one atomic per block, so a whole training step's losses reach the host in one copy.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>
#include <type_traits>

#include "internal.h"

namespace snb {
namespace {

constexpr uint32_t kEmptyToken = 0xFFFFFFFFu;   // EMPTY_TOKEN (kernels/mod.rs:46)
constexpr float kNegativeLarge = -3.0e38f;      // NEGATIVE_LARGE (kernels/mod.rs:49), the running max's start
constexpr int CE_WARPS = 8;
constexpr int CE_ROWS_PER_WARP = 8;

struct CeParams {
    const void* logits;
    int32_t logits_bf16;
    int32_t grad_bf16;
    uint64_t rows, row_width;       // logits and gradient: [rows, row_width]
    const uint32_t* targets;
    uint64_t target_stride;
    uint64_t column_offset;         // first column of head 0; head h starts at column_offset + h * classes
    uint64_t classes;
    uint64_t target_offset;         // head h's target sits at target_offset + h within a target row
    const float* grad_scales;       // per head, or nullptr: grad_scale for every head
    float grad_scale;
    float* row_losses;              // [rows * heads] (head fastest), or nullptr
    float* loss_sums;               // [heads], added to, or nullptr
    void* grad;
};

__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
    return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x with subnormal results flushed to zero (one special-function-unit operation; relative error ~2^-22).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Two floats rounded to nearest-even bf16, `lo` in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float load_logit(const CeParams& p, uint64_t i) {
    return p.logits_bf16 ? bf16_to_f32(static_cast<const uint16_t*>(p.logits)[i]) : static_cast<const float*>(p.logits)[i];
}

__device__ __forceinline__ void store_grad(const CeParams& p, uint64_t i, float g) {
    if (p.grad_bf16) static_cast<uint16_t*>(p.grad)[i] = f32_to_bf16_rne(g);
    else static_cast<float*>(p.grad)[i] = g;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    return v;
}

// NV > 0: the register path with NV 8-element vectors per lane (classes == 256 * NV), logits and gradient of the
// element types IN_BF16 / OUT_BF16; NV == 0: three passes over the row (types read from the parameters).
template <int NV, bool IN_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(CE_WARPS * 32, NV >= 8 ? 2 : 4) cross_entropy_kernel(const CeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t head = blockIdx.y;
    const float scale = p.grad_scales ? p.grad_scales[head] : p.grad_scale;
    const uint64_t heads = gridDim.y;
    float loss_acc = 0.0f;
    for (int k = 0; k < CE_ROWS_PER_WARP; ++k) {
        const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * CE_WARPS + warp) * CE_ROWS_PER_WARP + k;
        if (row >= p.rows) break;
        const uint64_t base = row * p.row_width + p.column_offset + head * p.classes;
        const uint32_t target = p.targets[row * p.target_stride + p.target_offset + head];
        float loss = 0.0f;
        if (target == kEmptyToken) {
            for (uint64_t c = lane; c < p.classes; c += 32) store_grad(p, base + c, 0.0f);
        } else if (target >= p.classes) {
            // Not a class of this head (the reference would read outside the row): NaN loss and gradient.
            loss = __uint_as_float(0x7FC00000u);
            for (uint64_t c = lane; c < p.classes; c += 32) store_grad(p, base + c, loss);
        } else {
            // The target's logit, read before any gradient may overwrite it in place.
            const float z_target = load_logit(p, base + target);
            if constexpr (NV > 0) {
                // Base-2 arithmetic: u = z log2(e), so exp(z - m) = 2^(u - m log2(e)) by one ex2.approx each.
                float v[NV * 8];
#pragma unroll
                for (int b = 0; b < NV; ++b) {
                    const uint64_t c0 = base + static_cast<uint64_t>(b * 32 + lane) * 8;
                    if constexpr (IN_BF16) {
                        const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.logits) + c0);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            v[b * 8 + 2 * i] = __uint_as_float(ws[i] << 16) * kLog2e;
                            v[b * 8 + 2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u) * kLog2e;
                        }
                    } else {
                        const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(p.logits) + c0);
                        const float4 a = f[0], b4 = f[1];
                        v[b * 8 + 0] = a.x * kLog2e; v[b * 8 + 1] = a.y * kLog2e;
                        v[b * 8 + 2] = a.z * kLog2e; v[b * 8 + 3] = a.w * kLog2e;
                        v[b * 8 + 4] = b4.x * kLog2e; v[b * 8 + 5] = b4.y * kLog2e;
                        v[b * 8 + 6] = b4.z * kLog2e; v[b * 8 + 7] = b4.w * kLog2e;
                    }
                }
                float maximum = kNegativeLarge;
#pragma unroll
                for (int i = 0; i < NV * 8; ++i) maximum = fmaxf(maximum, v[i]);
                maximum = warp_max(maximum);
                float total = 0.0f;
#pragma unroll
                for (int i = 0; i < NV * 8; ++i) total += exp2_approx(v[i] - maximum);
                const float log2_partition = maximum + __log2f(warp_sum(total));
                loss = log2_partition * kLn2 - z_target;
#pragma unroll
                for (int b = 0; b < NV; ++b) {
                    const uint32_t first = static_cast<uint32_t>(b * 32 + lane) * 8;   // class of v[b * 8]
                    float g[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) g[i] = exp2_approx(v[b * 8 + i] - log2_partition) * scale;
                    if (target - first < 8u) {
                        // This lane holds the target: subtract the one-hot term there.
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            if (first + i == target) g[i] -= scale;
                    }
                    const uint64_t c0 = base + first;
                    if constexpr (OUT_BF16) {
                        const uint4 w = make_uint4(pack_bf16x2_rn(g[0], g[1]), pack_bf16x2_rn(g[2], g[3]),
                                                   pack_bf16x2_rn(g[4], g[5]), pack_bf16x2_rn(g[6], g[7]));
                        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.grad) + c0) = w;
                    } else {
                        float4* f = reinterpret_cast<float4*>(static_cast<float*>(p.grad) + c0);
                        f[0] = make_float4(g[0], g[1], g[2], g[3]);
                        f[1] = make_float4(g[4], g[5], g[6], g[7]);
                    }
                }
            } else {
                float maximum = kNegativeLarge;
                for (uint64_t c = lane; c < p.classes; c += 32) maximum = fmaxf(maximum, load_logit(p, base + c));
                maximum = warp_max(maximum);
                float total = 0.0f;
                for (uint64_t c = lane; c < p.classes; c += 32) total += expf(load_logit(p, base + c) - maximum);
                const float log_partition = maximum + logf(warp_sum(total));
                loss = log_partition - z_target;
                for (uint64_t c = lane; c < p.classes; c += 32) {
                    const float probability = expf(load_logit(p, base + c) - log_partition);
                    store_grad(p, base + c, (probability - (c == target ? 1.0f : 0.0f)) * scale);
                }
            }
        }
        if (lane == 0) {
            if (p.row_losses) p.row_losses[row * heads + head] = loss;
            loss_acc += loss;
        }
    }
    if (p.loss_sums) {
        __shared__ float partial[CE_WARPS];
        if (lane == 0) partial[warp] = loss_acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f;
            for (int w = 0; w < CE_WARPS; ++w) s += partial[w];
            atomicAdd(&p.loss_sums[head], s);
        }
    }
}

}  // namespace

int cross_entropy_launch(cudaStream_t stream, const void* logits, int logits_type, uint64_t rows, uint64_t row_width,
                         const uint32_t* targets, uint64_t target_stride, uint64_t heads, uint64_t column_offset,
                         uint64_t classes, uint64_t target_offset, const float* grad_scales, float grad_scale,
                         float* row_losses, float* loss_sums, void* grad, int grad_type, std::string* err) {
    if (rows == 0 || heads == 0 || classes == 0) return SNB_OK;
    if (heads > 65535) {
        *err = "cross_entropy: more than 65535 heads";
        return SNB_ERR_UNSUPPORTED;
    }
    CeParams p{};
    p.logits = logits;
    p.logits_bf16 = logits_type == SNB_TYPE_BF16;
    p.grad_bf16 = grad_type == SNB_TYPE_BF16;
    p.rows = rows;
    p.row_width = row_width;
    p.targets = targets;
    p.target_stride = target_stride;
    p.column_offset = column_offset;
    p.classes = classes;
    p.target_offset = target_offset;
    p.grad_scales = grad_scales;
    p.grad_scale = grad_scale;
    p.row_losses = row_losses;
    p.loss_sums = loss_sums;
    p.grad = grad;
    // Register path: classes = 256 * NV, every head's row 16-byte aligned in both tensors.
    const uint64_t in_es = p.logits_bf16 ? 2 : 4, out_es = p.grad_bf16 ? 2 : 4;
    const bool aligned = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && reinterpret_cast<uintptr_t>(grad) % 16 == 0 &&
                         (row_width * in_es) % 16 == 0 && (row_width * out_es) % 16 == 0 &&
                         (column_offset * in_es) % 16 == 0 && (column_offset * out_es) % 16 == 0;
    const int nv = (aligned && classes % 256 == 0 && classes <= 2048) ? static_cast<int>(classes / 256) : 0;
    // (NV values without an instantiation below fall back to the three-pass path.)
    const uint64_t rows_per_block = static_cast<uint64_t>(CE_WARPS) * CE_ROWS_PER_WARP;
    const uint64_t bx = (rows + rows_per_block - 1) / rows_per_block;
    if (bx > 0x7fffffffull) {
        *err = "cross_entropy: too many rows";
        return SNB_ERR_UNSUPPORTED;
    }
    const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(heads));
    const int threads = CE_WARPS * 32;
    // Register path instantiated for the codebook sizes in use (classes = 256 * NV, NV in {1, 2, 4, 8}); any other
    // size takes the three-pass path.
    auto launch = [&](auto nv_c, auto in_c, auto out_c) {
        cross_entropy_kernel<decltype(nv_c)::value, decltype(in_c)::value, decltype(out_c)::value>
            <<<grid, threads, 0, stream>>>(p);
    };
    auto with_types = [&](auto nv_c) {
        using T = std::true_type;
        using F = std::false_type;
        if (p.logits_bf16 && p.grad_bf16) launch(nv_c, T{}, T{});
        else if (p.logits_bf16) launch(nv_c, T{}, F{});
        else if (p.grad_bf16) launch(nv_c, F{}, T{});
        else launch(nv_c, F{}, F{});
    };
    switch (nv) {
        case 1: with_types(std::integral_constant<int, 1>{}); break;
        case 2: with_types(std::integral_constant<int, 2>{}); break;
        case 4: with_types(std::integral_constant<int, 4>{}); break;
        case 8: with_types(std::integral_constant<int, 8>{}); break;
        default: launch(std::integral_constant<int, 0>{}, std::false_type{}, std::false_type{}); break;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("cross_entropy_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

}  // namespace snb
