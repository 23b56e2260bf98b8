// random.cu — the reference's seeded input stream generated on the device.
//
// `Random` (crates/staleynet-model/src/random.rs:27-70) is SplitMix64: every draw adds the golden-ratio increment to
// the state and mixes it, so the k-th draw (k = 1, 2, ...) of `Random::new(seed)` is mix(seed + k * gamma) and
// depends on nothing else. `normal()` (random.rs:64-68) takes two fresh draws per value (Box-Muller without the
// second sample), `below(bound)` one. Element i of a fill is therefore computed on its own thread, from draw numbers
// first_draw + 2i + 1, + 2 (normal) or first_draw + i + 1 (below), with the same f32 operations in the same order
// as the reference: a 24-bit uniform, max(u, 1e-7), sqrt(-2 ln u), TAU * u', radius * cos(angle), then * std for
// `Init::Normal(std)` (parameter.rs:54). The library is built without fast-math, so logf, sqrtf and cosf are CUDA's
// accurate versions; they may differ from the host's libm in the last bit of an f32 (the tests bound that), and a
// bf16 output is the f32 value rounded to nearest even.
#include <cuda_bf16.h>
#include <cstdint>

#include "internal.h"

namespace snb {

namespace {

constexpr uint64_t kGoldenGamma = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kMix1 = 0xBF58476D1CE4E5B9ull;
constexpr uint64_t kMix2 = 0x94D049BB133111EBull;

// The k-th draw (k >= 1) of Random::new(seed).
__device__ __forceinline__ uint64_t draw(uint64_t seed, uint64_t k) {
    uint64_t m = seed + k * kGoldenGamma;
    m = (m ^ (m >> 30)) * kMix1;
    m = (m ^ (m >> 27)) * kMix2;
    return m ^ (m >> 31);
}

// Random::uniform from draw k: the top 24 bits over 2^24.
__device__ __forceinline__ float uniform(uint64_t seed, uint64_t k) {
    return static_cast<float>(draw(seed, k) >> 40) / 16777216.0f;
}

template <bool OUT_BF16>
__global__ void random_normal_kernel(void* out, uint64_t count, uint64_t seed, uint64_t first_draw, float stddev) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        const uint64_t k = first_draw + 2 * i + 1;
        const float radius = sqrtf(-2.0f * logf(fmaxf(uniform(seed, k), 1e-7f)));
        const float angle = 6.28318530717958647692f * uniform(seed, k + 1);
        const float v = radius * cosf(angle) * stddev;
        if constexpr (OUT_BF16) reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
        else reinterpret_cast<float*>(out)[i] = v;
    }
}

__global__ void random_below_kernel(uint32_t* out, uint64_t count, uint64_t seed, uint64_t first_draw, uint64_t bound) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
        out[i] = static_cast<uint32_t>(draw(seed, first_draw + i + 1) % bound);
}

int launched(const char* what, std::string* err) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message(what, e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

unsigned fill_grid(uint64_t count) {
    const uint64_t blocks = (count + 255) / 256;
    return static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16);
}

}  // namespace

int random_normal_launch(cudaStream_t s, void* out, int out_type, uint64_t count, uint64_t seed, uint64_t first_draw,
                         float stddev, std::string* err) {
    if (count == 0) return SNB_OK;
    if (out_type == SNB_TYPE_BF16)
        random_normal_kernel<true><<<fill_grid(count), 256, 0, s>>>(out, count, seed, first_draw, stddev);
    else
        random_normal_kernel<false><<<fill_grid(count), 256, 0, s>>>(out, count, seed, first_draw, stddev);
    return launched("random_normal_kernel launch", err);
}

int random_below_launch(cudaStream_t s, uint32_t* out, uint64_t count, uint64_t seed, uint64_t first_draw,
                        uint64_t bound, std::string* err) {
    if (count == 0) return SNB_OK;
    random_below_kernel<<<fill_grid(count), 256, 0, s>>>(out, count, seed, first_draw, bound);
    return launched("random_below_kernel launch", err);
}

}  // namespace snb
