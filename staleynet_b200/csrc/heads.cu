// heads.cu — the attention head permutes between the packed layout [batch * time, width] and the head-major layout
// [batch, heads, time_capacity, head_dim]: the reference's split_heads / merge_heads (crates/staleynet-cuda/src/
// kernels/attention.rs:112-138, one thread per element), here as 16-byte moves.
//
// In both layouts the head_dim elements of one (batch, head, time step) are contiguous, so the permute moves whole
// runs of head_dim elements. A thread moves 8 consecutive elements of a run (32 bytes of f32 or 16 of bf16) with
// vector loads and stores, converting the element type on the way when the two sides differ; threads are laid out
// so that consecutive threads cover consecutive runs of the destination, which makes the writes fully coalesced and
// each read a contiguous run. Layouts whose runs do not start on 8-element boundaries (head_dim, width or
// column_offset not multiples of 8, or bases not 16-byte aligned) take a one-element-per-thread kernel.
// HBM-bound: one read and one write of every moved element.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "internal.h"

namespace snb {

namespace {

struct HeadGeometry {
    int64_t batch, time, heads, head_dim, width, column_offset, capacity, time_offset;
};

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Copies between identical types move the bits (no round trip through f32 for bf16 -> bf16).
__device__ __forceinline__ void move8(const float* s, float* d) {
    *reinterpret_cast<float4*>(d) = *reinterpret_cast<const float4*>(s);
    *reinterpret_cast<float4*>(d + 4) = *reinterpret_cast<const float4*>(s + 4);
}
__device__ __forceinline__ void move8(const __nv_bfloat16* s, __nv_bfloat16* d) {
    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
}
template <typename S, typename D>
__device__ __forceinline__ void move8(const S* s, D* d) {
    float v[8];
    load8(s, v);
    store8(d, v);
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void from_f32(float x, float* d) { *d = x; }
__device__ __forceinline__ void from_f32(float x, __nv_bfloat16* d) { *d = __float2bfloat16_rn(x); }

// Run r of the destination order -> (batch, head, step). Split writes head-major runs, so r walks (batch, head,
// step); merge writes packed runs, so r walks (batch, step, head).
template <bool SPLIT>
__device__ __forceinline__ void run_coords(const HeadGeometry& g, int64_t r, int64_t& b, int64_t& h, int64_t& s) {
    if (SPLIT) {
        s = r % g.time;
        const int64_t bh = r / g.time;
        h = bh % g.heads;
        b = bh / g.heads;
    } else {
        h = r % g.heads;
        const int64_t bs = r / g.heads;
        s = bs % g.time;
        b = bs / g.time;
    }
}

// One thread per 8-element piece: piece q of run r, q = 0 .. head_dim / 8 - 1.
template <typename S, typename D, bool SPLIT>
__global__ void permute_heads_vec_kernel(const S* __restrict__ src, D* __restrict__ dst, HeadGeometry g,
                                         int64_t pieces) {
    const int64_t per_run = g.head_dim / 8;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < pieces;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_run;
        const int64_t d = (i - r * per_run) * 8;
        int64_t b, h, s;
        run_coords<SPLIT>(g, r, b, h, s);
        const int64_t packed = (b * g.time + s) * g.width + g.column_offset + h * g.head_dim + d;
        const int64_t head_major = ((b * g.heads + h) * g.capacity + g.time_offset + s) * g.head_dim + d;
        if (SPLIT) move8(src + packed, dst + head_major);
        else move8(src + head_major, dst + packed);
    }
}

// One thread per element (the reference's form): any layout and alignment.
template <typename S, typename D, bool SPLIT>
__global__ void permute_heads_kernel(const S* __restrict__ src, D* __restrict__ dst, HeadGeometry g,
                                     int64_t elements) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < elements;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / g.head_dim;
        const int64_t d = i - r * g.head_dim;
        int64_t b, h, s;
        run_coords<SPLIT>(g, r, b, h, s);
        const int64_t packed = (b * g.time + s) * g.width + g.column_offset + h * g.head_dim + d;
        const int64_t head_major = ((b * g.heads + h) * g.capacity + g.time_offset + s) * g.head_dim + d;
        if (SPLIT) from_f32(to_f32(src[packed]), dst + head_major);
        else from_f32(to_f32(src[head_major]), dst + packed);
    }
}

template <typename S, typename D>
int launch_typed(cudaStream_t stream, bool split, const void* src, void* dst, const HeadGeometry& g, int sm_count,
                 std::string* err) {
    const int64_t elements = g.batch * g.heads * g.time * g.head_dim;
    const bool aligned = reinterpret_cast<uintptr_t>(src) % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0;
    const bool vec = aligned && g.head_dim % 8 == 0 && g.width % 8 == 0 && g.column_offset % 8 == 0;
    const int64_t items = vec ? elements / 8 : elements;
    const int64_t blocks = std::min<int64_t>((items + 255) / 256, static_cast<int64_t>(sm_count) * 16);
    const S* s = static_cast<const S*>(src);
    D* d = static_cast<D*>(dst);
    if (vec) {
        if (split) permute_heads_vec_kernel<S, D, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(s, d, g, items);
        else permute_heads_vec_kernel<S, D, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(s, d, g, items);
    } else {
        if (split) permute_heads_kernel<S, D, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(s, d, g, items);
        else permute_heads_kernel<S, D, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(s, d, g, items);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("permute_heads launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

}  // namespace

int permute_heads_launch(cudaStream_t stream, bool split, const void* src, int src_type, void* dst, int dst_type,
                         const snb_head_layout& L, std::string* err) {
    DeviceInfo dev;
    int rc = current_device_info(&dev, err);
    if (rc != SNB_OK) return rc;
    const HeadGeometry g{static_cast<int64_t>(L.batch),    static_cast<int64_t>(L.time),
                         static_cast<int64_t>(L.heads),    static_cast<int64_t>(L.head_dim),
                         static_cast<int64_t>(L.width),    static_cast<int64_t>(L.column_offset),
                         static_cast<int64_t>(L.time_capacity), static_cast<int64_t>(L.time_offset)};
    const bool sf = src_type == SNB_TYPE_F32, df = dst_type == SNB_TYPE_F32;
    if (sf && df) return launch_typed<float, float>(stream, split, src, dst, g, dev.sm_count, err);
    if (sf) return launch_typed<float, __nv_bfloat16>(stream, split, src, dst, g, dev.sm_count, err);
    if (df) return launch_typed<__nv_bfloat16, float>(stream, split, src, dst, g, dev.sm_count, err);
    return launch_typed<__nv_bfloat16, __nv_bfloat16>(stream, split, src, dst, g, dev.sm_count, err);
}

}  // namespace snb
