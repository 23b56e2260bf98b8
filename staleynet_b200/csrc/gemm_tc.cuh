// gemm_tc.cuh — the tensor-core GEMM for sm_100a: C_b = scale * A_b * B_b (+ epilogue) for every matrix of a
// batch, computing the same product as the reference's `matmul_*` kernels (crates/staleynet-cuda/src/kernels/
// matmul.rs:216-448) with tcgen05 tensor cores.
//
// Structure (one persistent CTA of 320 threads per SM, work units strided over the grid):
//   warp 0     TMA producer: one elected thread streams 128-byte-wide K slices of A and B into a STAGES-deep
//              shared-memory ring (128B swizzle), completion tracked by `full` mbarriers; it also prefetches each
//              tile's epilogue inputs (residual, GELU input) into L2 and, in SB kernels, copies the tile's bias into
//              one of two shared-memory buffers (a 1-D bulk copy) once the epilogue has released that buffer.
//   warp 1     allocates / frees TMEM (2*BN columns); one elected thread issues tcgen05.mma (M=128, N=BN,
//              K=32 bytes per instruction) into one of two TMEM accumulators and frees ring slots with
//              tcgen05.commit on `empty` mbarriers.
//   warps 2-9  epilogue: a warp may read the 32 TMEM lanes of its quadrant (warp % 4) = 32 output rows; the two
//              warps of a quadrant take alternate 128-byte column chunks. Per chunk a warp loads 32 columns at a
//              time (tcgen05.ld 32x32b.x32), applies scale / bias / GELU / residual, writes a swizzled 32x128-byte
//              box to shared memory and stores it with a TMA store, or a TMA reduce-add when accumulating into C.
//              The second accumulator lets the epilogue of one tile overlap the main loop of the next; eight
//              warps (two per scheduler) hide the latency of TMEM and global loads. When a bf16 output reads one
//              bf16 auxiliary input (GELU input or residual), each warp TMA-loads that input's chunks into its
//              staging boxes as soon as its previous tile's stores have read them, and the output overwrites the
//              input in place.
//
// Operand layouts: each operand is either K-major (K contiguous) or MN-major (M or N contiguous); both are loaded
// by TMA in their stored order and described to the tensor core by the major bits of the instruction descriptor,
// so the four storage combinations of the reference (`Storage::{RowMajor,Transposed}`, ops/matmul.rs:16-33) run
// without any transposition pass. Every operand uses a 128-byte swizzle with 16-byte atoms except MN-major tf32
// operands, which the tensor core reads only with 32-byte atoms (TMA's SWIZZLE_128B_ATOM_32B).
//
// Split-K: a work unit may cover only part of K; partial sums then reach C through TMA reduce-add, which adds
// element-wise in L2 in arrival order (C must be pre-zeroed by the host for an overwrite), or, in the deterministic
// mode (split_slabs), each split stores its partial into its own workspace slab and the host sums the slabs into C
// in split order afterwards.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace snb {

constexpr int TC_BM = 128;
constexpr int TC_EPI_WARP0 = 2;   // warps 2..9 drain the accumulator
constexpr int TC_EPI_WARPS = 8;   // two per TMEM lane quadrant, splitting the tile's columns
constexpr int TC_THREADS = 32 * (TC_EPI_WARP0 + TC_EPI_WARPS);
constexpr int TC_EPI_BOX_BYTES = 32 * 128;  // one staged output box: 32 rows x 128 bytes

struct TcParams {
    int32_t M, N, K;          // rows, cols, inner of each product
    int32_t count;            // matrices in the batch
    int32_t a_mn_major;       // 1: A stored with M contiguous; 0: K contiguous
    int32_t b_mn_major;       // 1: B stored with N contiguous; 0: K contiguous
    int32_t a_batched;        // 0: one A shared by every matrix (batch stride 0)
    int32_t b_batched;
    int32_t m_tiles, n_tiles; // output tiles per matrix
    int32_t k_blocks;         // 128-byte K slices per product
    int32_t splits;           // K splits per tile (>= 1)
    int32_t m_fastest;        // unit order: 1 = M tile index fastest, 0 = N tile index fastest
    int32_t k_blocks_per_split;
    int32_t num_units;        // count * m_tiles * n_tiles * splits
    float scale;
    int32_t reduce;           // 1: C += result via TMA reduce-add (accumulate or split-K); 0: TMA store
    int32_t activation;       // SNB_ACTIVATION_*
    int32_t aux_bf16;         // element type of gelu_input (pre_activation always has the output's type)
    int32_t has_pre;          // pre-activation store through the second output map
    const float* bias;        // [N] or nullptr
    const void* residual;     // laid out like C (type of C) or nullptr
    const void* gelu_input;   // laid out like C (aux type) or nullptr
    int64_t out_batch_stride; // elements between output matrices (for residual / gelu_input addressing)
    int32_t causal;           // SNB_CAUSAL_* work-skipping hint of a batched attention product
    int64_t causal_offset;    // query q sees keys 0..=q+causal_offset
    const float* row_scale;   // [M] output-row multipliers (one matrix), or nullptr
    int32_t split_slabs;      // 1: split s of the K range stores its partial tile into slab s of the output map (a
                              // [splits, M, N] workspace, count 1), summed later in split order; 0: C itself
    // Head-major operands (count 1). A packed activation [batch * time, heads * head_dim] whose heads are stored
    // head-major, [batch, heads, capacity, head_dim] with time step s at row time_offset + s (the reference's
    // HeadLayout, crates/staleynet-cuda/src/kernels/attention.rs:19-41), is read or written through 4-D / 5-D tensor
    // maps instead of a packed copy: a_heads = A is such a tensor (tm_a 4-D: head_dim, capacity, heads, batch;
    // K-major = tokens are A's rows, MN-major = tokens are the K index); c_heads = C is written to P such tensors
    // side by side (tm_c 5-D: head_dim, capacity, heads, batch, P), columns (p * heads + h) * head_dim + d.
    int32_t a_heads, a_hd, a_time, a_toff;
    int32_t c_heads, c_hd, c_nheads, c_time, c_toff;
};

// Epilogue staging modes (see epilogue_tile); the host picks one per launch.
constexpr int TC_EPI_ONE_BOX = 1;
constexpr int TC_EPI_TWO_BOX = 2;
constexpr int TC_EPI_AUX_BOX = 3;
constexpr int tc_epi_boxes(int epi) { return epi == TC_EPI_ONE_BOX ? 1 : 2; }

// Shared memory of one sm_100 CTA available to a kernel.
constexpr int TC_SMEM_LIMIT = 232448;

// NBOX = staging boxes per epilogue warp: 2 lets a chunk be staged while the previous chunk's TMA store still reads
// its box (worth it for GELU epilogues), at the price of one ring stage for BN = 256. SB = the tile's bias is
// copied into shared memory (one BN-float buffer per accumulator) instead of being read from global memory by every
// epilogue warp; the ring keeps as many stages as still fit.
template <int BN, int NBOX, bool SB = false>
struct TcConfig {
    static constexpr int STAGE_A = TC_BM * 128;
    static constexpr int STAGE_B = BN * 128;
    static constexpr int STAGE = STAGE_A + STAGE_B;
    static constexpr int EPI_BYTES = TC_EPI_WARPS * NBOX * TC_EPI_BOX_BYTES;
    static constexpr int BIAS_BYTES = SB ? 2 * BN * 4 : 0;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int BARRIER_BYTES = 512;
    static constexpr int BASE_STAGES = BN == 256 ? (NBOX == 2 ? 3 : 4) : (BN == 128 ? 4 : 6);
    static constexpr int FIT_STAGES = (TC_SMEM_LIMIT - 1024 - EPI_BYTES - BIAS_BYTES - BARRIER_BYTES) / STAGE;
    static constexpr int STAGES = BASE_STAGES < FIT_STAGES ? BASE_STAGES : FIT_STAGES;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE + EPI_BYTES + BIAS_BYTES + BARRIER_BYTES;
    static_assert(SMEM_BYTES <= TC_SMEM_LIMIT, "shared memory budget of one sm_100 CTA");
    static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation is a power of two");
};

struct TcUnit {
    int32_t batch, m0, n0, kb_begin, kb_end, split;
    bool skip;  // every output of the tile is a masked score (SNB_CAUSAL_SKIP_MASKED_OUTPUT): no work at all
};

// The unit at output tile (mt, nt) of matrix `batch` in K split `split`: its output origin and K-slice range, cut
// by the causal hints of a batched attention product.
__device__ __forceinline__ TcUnit tc_make_unit(const TcParams& p, int32_t split, int32_t batch, int32_t mt, int32_t nt,
                                               int BN, int BK, int BM) {
    TcUnit u;
    u.split = split;
    u.batch = batch;
    u.m0 = mt * BM;
    u.n0 = nt * BN;
    u.kb_begin = u.split * p.k_blocks_per_split;
    u.kb_end = min(p.k_blocks, u.kb_begin + p.k_blocks_per_split);
    u.skip = false;
    // Causal attention products (never split): skip work whose operands or results the causal softmax voids.
    if (p.causal == 1) {
        // all (row, col) of the tile masked: the tile's smallest col - row exceeds the offset
        u.skip = static_cast<int64_t>(u.n0) - (u.m0 + TC_BM - 1) > p.causal_offset;
    } else if (p.causal == 2) {
        // left[row, key] is zero for key > row + offset: stop after the last key any row of the tile sees
        const int64_t last_key = static_cast<int64_t>(u.m0) + TC_BM - 1 + p.causal_offset;
        const int64_t lim = last_key / BK + 1;
        if (lim < u.kb_end) u.kb_end = static_cast<int32_t>(lim);
    } else if (p.causal == 3) {
        // left[key, query] is zero for query < key - offset: start at the first query any row of the tile sees
        const int64_t first_query = static_cast<int64_t>(u.m0) - p.causal_offset;
        if (first_query > 0) u.kb_begin = max(u.kb_begin, static_cast<int32_t>(first_query / BK));
    }
    // Keep at least one K slice (its masked contributions are zero) so the accumulator is always written.
    if (u.kb_begin >= u.kb_end) u.kb_begin = u.kb_end - 1;
    return u;
}

// Work-unit order: K split outermost (the tiles of one split run side by side, so concurrent CTAs share operand
// slices in L2 and the splits of one tile never reduce into C at the same time), then the batch, then output tiles
// with the M or the N tile index fastest, whichever keeps the larger operand streaming through DRAM once: unit
// = ((split * count + batch) * n_slow + slow) * n_fast + fast, with (fast, slow) = (mt, nt) when p.m_fastest, else
// (nt, mt). A CTA walks units first, first + step, ... with a TcCursor, which keeps these digits
// and adds the step's digits with carries: the integer divisions happen once per CTA, not once per tile, where
// they kept the single MMA-issuing thread busy for about a thousand cycles between tiles while the tensor pipe ran
// dry (measured on K=768 products: ~1,100 idle cycles per 6,144-cycle tile).
struct TcCursor {
    int32_t unit, step;
    int32_t split, batch, slow, fast;
    int32_t d_split, d_batch, d_slow, d_fast;
    int32_t n_slow, n_fast;
};

__device__ __forceinline__ void tc_digits(const TcParams& p, int32_t x, int32_t n_slow, int32_t n_fast, int32_t& split,
                                          int32_t& batch, int32_t& slow, int32_t& fast) {
    fast = x % n_fast;
    x /= n_fast;
    slow = x % n_slow;
    x /= n_slow;
    batch = x % p.count;
    split = x / p.count;
}

__device__ __forceinline__ TcCursor tc_cursor(const TcParams& p, int32_t first, int32_t step) {
    TcCursor c;
    c.unit = first;
    c.step = step;
    c.n_fast = p.m_fastest ? p.m_tiles : p.n_tiles;
    c.n_slow = p.m_fastest ? p.n_tiles : p.m_tiles;
    tc_digits(p, first, c.n_slow, c.n_fast, c.split, c.batch, c.slow, c.fast);
    tc_digits(p, step, c.n_slow, c.n_fast, c.d_split, c.d_batch, c.d_slow, c.d_fast);
    return c;
}

__device__ __forceinline__ void tc_advance(const TcParams& p, TcCursor& c) {
    c.unit += c.step;
    c.fast += c.d_fast;
    int32_t carry = c.fast >= c.n_fast ? 1 : 0;
    c.fast -= carry * c.n_fast;
    c.slow += c.d_slow + carry;
    carry = c.slow >= c.n_slow ? 1 : 0;
    c.slow -= carry * c.n_slow;
    c.batch += c.d_batch + carry;
    carry = c.batch >= p.count ? 1 : 0;
    c.batch -= carry * p.count;
    c.split += c.d_split + carry;
}

__device__ __forceinline__ TcUnit tc_cursor_unit(const TcParams& p, const TcCursor& c, int BN, int BK, int BM = TC_BM) {
    return p.m_fastest ? tc_make_unit(p, c.split, c.batch, c.fast, c.slow, BN, BK, BM)
                       : tc_make_unit(p, c.split, c.batch, c.slow, c.fast, BN, BK, BM);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Loads 32 consecutive elements (f32: 8 x 16 bytes; bf16: 4 x 16 bytes) of one row starting at element `index`,
// zero where `valid` (columns left in the row) runs out or the row is dead. The host guarantees 16-byte alignment
// of every row start and that the row length is a multiple of 16 bytes.
__device__ __forceinline__ void load_row_32(const void* base, int64_t index, int is_bf16, int valid, bool live,
                                            uint4 (&r)[8]) {
    if (is_bf16) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + index);
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = (live && 8 * j < valid) ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(base) + index);
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = (live && 4 * j < valid) ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
    }
}

// tanh for the GELU epilogues. Outputs rounded to bf16 use the hardware's tanh.approx.f32 (one MUFU instruction,
// relative error about 2^-11, below the 2^-9 rounding of bf16), which keeps a GELU epilogue off the critical path;
// f32 outputs use the accurate tanhf.
template <bool FAST>
__device__ __forceinline__ float tanh_epilogue(float x) {
    if constexpr (FAST) {
        float y;
        asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
        return y;
    } else {
        return tanhf(x);
    }
}

// GELU, tanh approximation (the reference's gelu_forward, crates/staleynet-cuda/src/kernels/elementwise.rs:14-17)
// and its derivative (kernels/elementwise.rs:20-24), on pairs of values with Blackwell's packed f32x2 arithmetic:
//   t = tanh(c (x + a x^3)),  gelu = 0.5 x (1 + t),  gelu' = 0.5 (1 + t) + 0.5 x (1 - t^2) (c + 3 a c x^2)
// with c = sqrt(2/pi) and a = 0.044715.
constexpr float GELU_C = 0.7978846f;
constexpr float GELU_A = 0.044715f;

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

template <bool FAST>
__device__ __forceinline__ float2 gelu_tanh_arg(float2 x, float2& x2) {
    x2 = __fmul2_rn(x, x);
    const float2 x3 = __fmul2_rn(x2, x);
    const float2 inner = __ffma2_rn(f2(GELU_A), x3, x);
    const float2 arg = __fmul2_rn(f2(GELU_C), inner);
    return make_float2(tanh_epilogue<FAST>(arg.x), tanh_epilogue<FAST>(arg.y));
}

template <bool FAST>
__device__ __forceinline__ float2 gelu2(float2 x) {
    float2 x2;
    const float2 t = gelu_tanh_arg<FAST>(x, x2);
    const float2 hx = __fmul2_rn(f2(0.5f), x);
    return __ffma2_rn(hx, t, hx);
}

template <bool FAST>
__device__ __forceinline__ float2 gelu2_derivative(float2 x) {
    float2 x2;
    const float2 t = gelu_tanh_arg<FAST>(x, x2);
    const float2 half_1pt = __ffma2_rn(f2(0.5f), t, f2(0.5f));
    const float2 one_m_t2 = __ffma2_rn(make_float2(-t.x, -t.y), t, f2(1.0f));
    const float2 poly = __ffma2_rn(f2(3.0f * GELU_A * GELU_C), x2, f2(GELU_C));
    const float2 q = __fmul2_rn(__fmul2_rn(f2(0.5f), x), one_m_t2);
    return __ffma2_rn(q, poly, half_1pt);
}

// Unpacks 32 auxiliary values loaded by load_row_32 into 16 pairs.
__device__ __forceinline__ void unpack_row_32x2(const uint4 (&r)[8], int is_bf16, float2 (&v)[16]) {
    if (is_bf16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t u[4] = {r[j].x, r[j].y, r[j].z, r[j].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) v[4 * j + k] = make_float2(__uint_as_float(u[k] << 16), __uint_as_float(u[k] & 0xffff0000u));
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[2 * j] = make_float2(__uint_as_float(r[j].x), __uint_as_float(r[j].y));
            v[2 * j + 1] = make_float2(__uint_as_float(r[j].z), __uint_as_float(r[j].w));
        }
    }
}

// Writes 32 values (one tcgen05.ld of a lane) into this lane's row of the 128B-swizzled staging box: f32 fills
// 16-byte chunks [0, 8) (a 32-column box), bf16 fills chunks [4h, 4h + 4) of a 64-column box. Chunk j of row r
// sits at position j ^ (r % 8), the layout a SWIZZLE_128B tensor map expects.
template <bool OUT_BF16>
__device__ __forceinline__ void stage_half(uint8_t* box, int lane, int h, const float2 (&v)[16]) {
    uint8_t* row = box + lane * 128;
    if constexpr (OUT_BF16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 q4 = make_uint4(pack_bf16x2(v[4 * j].x, v[4 * j].y), pack_bf16x2(v[4 * j + 1].x, v[4 * j + 1].y),
                                        pack_bf16x2(v[4 * j + 2].x, v[4 * j + 2].y),
                                        pack_bf16x2(v[4 * j + 3].x, v[4 * j + 3].y));
            *reinterpret_cast<uint4*>(row + (((4 * h + j) ^ (lane & 7)) << 4)) = q4;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 q4 = make_uint4(__float_as_uint(v[2 * j].x), __float_as_uint(v[2 * j].y),
                                        __float_as_uint(v[2 * j + 1].x), __float_as_uint(v[2 * j + 1].y));
            *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) = q4;
        }
    }
}

// The epilogue function for 32 columns [col, col + 32) of one output row, starting from the TMEM accumulator:
//   x = scale * row_scale[row] * acc + bias;  (x staged into pre_box when given);  pre_only: return x;
//   y = activation(x) (+ residual).
// The first auxiliary input (GELU input, else residual) is requested before waiting for TMEM so the two latencies
// overlap; only when both are present is the residual read afterwards. With `aux_box` the first auxiliary input is
// already in shared memory (TMA-loaded into the 128B-swizzled staging box this half is staged into) and is read
// from this lane's row of it. SB: the bias of these 32 columns is read from shared memory at `bias_s` (the tile's
// bias buffer, offset to column `col`), a broadcast read, instead of from global memory.
template <bool OUT_BF16, bool SB = false>
__device__ __forceinline__ void epilogue_half(const TcParams& p, uint32_t taddr, int32_t col, int32_t row,
                                              int64_t out_base, bool first_split, uint8_t* pre_box, int h,
                                              float2 (&v)[16], bool pre_only, const uint8_t* aux_box = nullptr,
                                              uint32_t bias_s = 0) {
    uint32_t x[32];
    tmem_load_32x32b_x32(taddr, x);
    const int valid = p.N - col;  // columns of this piece inside the matrix (a multiple of 4 or 8)
    const bool row_live = row < p.M;
    const bool want_gin = !pre_only && p.activation == 2;
    const bool want_res = !pre_only && p.residual != nullptr && first_split;
    uint4 raux[8];
    if (aux_box != nullptr) {
        const int lane = threadIdx.x & 31;
        const uint32_t rowp = smem_addr(aux_box) + lane * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 f = ld_shared_f4(rowp + (((4 * h + j) ^ (lane & 7)) << 4));
            raux[j] = make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
        }
    } else if (want_gin) {
        load_row_32(p.gelu_input, out_base + col, p.aux_bf16, valid, row_live, raux);
    } else if (want_res) {
        load_row_32(p.residual, out_base + col, OUT_BF16, valid, row_live, raux);
    }
    tmem_load_wait();

#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = make_float2(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1]));
    const float s = p.row_scale != nullptr ? p.scale * (row_live ? __ldg(p.row_scale + row) : 0.0f) : p.scale;
    if (s != 1.0f) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __fmul2_rn(f2(s), v[j]);
    }
    if (p.bias != nullptr && first_split) {
        const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (4 * j < valid) b = SB ? ld_shared_f4(bias_s + 16 * j) : __ldg(b4 + j);
            v[2 * j] = __fadd2_rn(v[2 * j], make_float2(b.x, b.y));
            v[2 * j + 1] = __fadd2_rn(v[2 * j + 1], make_float2(b.z, b.w));
        }
    }
    if (pre_box != nullptr) stage_half<OUT_BF16>(pre_box, threadIdx.x & 31, h, v);  // x before the activation
    if (pre_only) return;
    if (p.activation == 1) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gelu2<OUT_BF16>(v[j]);
    } else if (p.activation == 2) {
        float2 gi[16];
        unpack_row_32x2(raux, p.aux_bf16, gi);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __fmul2_rn(v[j], gelu2_derivative<OUT_BF16>(gi[j]));
        if (want_res) load_row_32(p.residual, out_base + col, OUT_BF16, valid, row_live, raux);
    }
    if (want_res) {
        float2 r[16];
        unpack_row_32x2(raux, OUT_BF16, r);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __fadd2_rn(v[j], r[j]);
    }
}

// Stores (or reduce-adds) one staged output box at column col0, row row0 of matrix/slab cz: through the 3-D map of
// C, or, with c_heads, through the 5-D map of the head-major output (the box's 32 rows lie in one sequence and its
// columns in one head: the host checks time % 32 == 0 and head_dim % box columns == 0).
__device__ __forceinline__ void store_c_box(const TcParams& p, const CUtensorMap* tm_c, uint32_t box, int32_t col0,
                                            int32_t row0, int32_t cz) {
    if (p.c_heads) {
        const int32_t head = col0 / p.c_hd;
        tma_store_5d(tm_c, box, col0 - head * p.c_hd, p.c_toff + row0 % p.c_time, head % p.c_nheads,
                     row0 / p.c_time, head / p.c_nheads);
    } else if (p.reduce) {
        tma_reduce_add_3d(tm_c, box, col0, row0, cz);
    } else {
        tma_store_3d(tm_c, box, col0, row0, cz);
    }
}

// Loads A's K slice k0 for the 128 output rows from m0 into the ring slot at `sa` (completion on `bar`): one box of
// 128 rows x BK for a K-major A, 128 / MN_BOX boxes of MN_BOX x BK for an MN-major A; with a_heads the boxes come
// from the head-major 4-D map (a K-major box stays inside one head and one sequence: head_dim % BK == 0 and
// time % 128 == 0; an MN-major box likewise with head_dim % MN_BOX == 0 and time % BK == 0, checked by the host).
// PAIR: the load completes on the CTA pair's leader barrier.
template <int BK, int MN_BOX, bool PAIR>
__device__ __forceinline__ void load_a_slice(const TcParams& p, const CUtensorMap* tm_a, uint32_t sa, uint32_t bar,
                                             int32_t m0, int32_t k0, int32_t ba) {
    if (!p.a_heads) {
        if (!p.a_mn_major) {
            if constexpr (PAIR) tma_load_3d_pair(sa, tm_a, bar, k0, m0, ba);
            else tma_load_3d(sa, tm_a, bar, k0, m0, ba);
        } else {
#pragma unroll
            for (int j = 0; j < 128 / MN_BOX; ++j) {
                if constexpr (PAIR) tma_load_3d_pair(sa + j * (BK * 128), tm_a, bar, m0 + j * MN_BOX, k0, ba);
                else tma_load_3d(sa + j * (BK * 128), tm_a, bar, m0 + j * MN_BOX, k0, ba);
            }
        }
        return;
    }
    if (!p.a_mn_major) {
        // rows = tokens (batch-major, then time), K = head * head_dim + d
        const int32_t h = k0 / p.a_hd;
        const int32_t b = m0 / p.a_time;
        const int32_t s = p.a_toff + (m0 - b * p.a_time);
        if constexpr (PAIR) tma_load_4d_pair(sa, tm_a, bar, k0 - h * p.a_hd, s, h, b);
        else tma_load_4d(sa, tm_a, bar, k0 - h * p.a_hd, s, h, b);
    } else {
        // rows = head * head_dim + d, K = tokens
        const int32_t b = k0 / p.a_time;
        const int32_t s = p.a_toff + (k0 - b * p.a_time);
#pragma unroll
        for (int j = 0; j < 128 / MN_BOX; ++j) {
            const int32_t m = m0 + j * MN_BOX;
            const int32_t h = m / p.a_hd;
            if constexpr (PAIR) tma_load_4d_pair(sa + j * (BK * 128), tm_a, bar, m - h * p.a_hd, s, h, b);
            else tma_load_4d(sa + j * (BK * 128), tm_a, bar, m - h * p.a_hd, s, h, b);
        }
    }
}

// Requests, on one lane, the auxiliary input of every column chunk an epilogue warp will stage for tile `u` (the
// chunks epilogue_tile visits, box j for the j-th): one TMA load of a 32-row box per chunk into staging box j,
// completing on aux_bar[j]. The boxes must no longer be read by earlier TMA stores.
template <bool OUT_BF16, int BN>
__device__ __forceinline__ void request_aux_boxes(const TcParams& p, const CUtensorMap* tm_aux, const TcUnit& u,
                                                  int32_t row0, int group, uint8_t* boxes, uint64_t* aux_bar) {
    constexpr int CHUNK = OUT_BF16 ? 64 : 32;
    int j = 0;
    for (int c = group * CHUNK; c < BN && row0 < p.M && u.n0 + c < p.N; c += 2 * CHUNK, ++j) {
        const uint32_t bar = smem_addr(&aux_bar[j]);
        mbar_arrive_expect_tx(bar, TC_EPI_BOX_BYTES);
        tma_load_3d(smem_addr(boxes + j * TC_EPI_BOX_BYTES), tm_aux, bar, u.n0 + c, row0, u.batch);
    }
}

// One epilogue warp's share of a finished accumulator tile: the column chunks c = group*CHUNK, +2*CHUNK, ... of
// its 32 rows. Each chunk is staged in a 128-byte-row box and written by a TMA store (or reduce-add). How the boxes
// are used is the staging mode EPI (a template parameter, so each kernel carries one path):
//   TC_EPI_ONE_BOX   one box per warp; a kept pre-activation is staged and stored first, then the output from a
//                    second TMEM read.
//   TC_EPI_TWO_BOX   two boxes that alternate, so staging one chunk overlaps the TMA engine's read of the previous
//                    one; a kept pre-activation fills both boxes from one TMEM read.
//   TC_EPI_AUX_BOX   two boxes; chunk j's one bf16 auxiliary input (GELU input or residual, map tm_aux) was
//                    TMA-loaded into box j by request_aux_boxes and its output overwrites it in place.
//   SB               the tile's bias is in shared memory at bias_tile (BN floats).
template <bool OUT_BF16, int BN, int EPI, bool SB = false>
__device__ __forceinline__ void epilogue_tile(const TcParams& p, const CUtensorMap* tm_c, const CUtensorMap* tm_pre,
                                              const TcUnit& u, int32_t row0, uint32_t t_lane, int group,
                                              uint8_t* boxes, int& ebox, uint64_t* aux_bar, uint32_t& aux_phase,
                                              uint32_t bias_tile = 0) {
    constexpr int CHUNK = OUT_BF16 ? 64 : 32;
    const int lane = threadIdx.x & 31;
    const int32_t row = row0 + lane;
    const bool first_split = u.split == 0;
    const int64_t out_base = static_cast<int64_t>(u.batch) * p.out_batch_stride + static_cast<int64_t>(row) * p.N;
    const int32_t cz = p.split_slabs ? u.split : u.batch;  // third coordinate of the output map
    int j = 0;
    for (int c = group * CHUNK; c < BN && row0 < p.M && u.n0 + c < p.N; c += 2 * CHUNK, ++j) {
        const int32_t col0 = u.n0 + c;
        if constexpr (EPI == TC_EPI_AUX_BOX) {
            uint8_t* box = boxes + j * TC_EPI_BOX_BYTES;
            // A timed-out wait has already set the device status; the tile is finished with whatever the box holds
            // so that every barrier still completes.
            mbar_wait(smem_addr(&aux_bar[j]), (aux_phase >> j) & 1u);
            __syncwarp();
            aux_phase ^= 1u << j;
#pragma unroll
            for (int h = 0; h < CHUNK / 32; ++h) {
                float2 v[16];
                epilogue_half<OUT_BF16, SB>(p, t_lane + c + 32 * h, col0 + 32 * h, row, out_base, first_split,
                                            nullptr, h, v, false, box, bias_tile + 4 * (c + 32 * h));
                stage_half<OUT_BF16>(box, lane, h, v);
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
                store_c_box(p, tm_c, smem_addr(box), col0, row0, u.batch);
                bulk_commit_group();
            }
        } else if constexpr (EPI == TC_EPI_TWO_BOX) {
            uint8_t* box = boxes + ebox * TC_EPI_BOX_BYTES;
            uint8_t* pre_box = p.has_pre ? boxes + (ebox ^ 1) * TC_EPI_BOX_BYTES : nullptr;
            if (lane == 0) {
                if (p.has_pre) bulk_wait_group_read<0>();  // both boxes are rewritten
                else bulk_wait_group_read<1>();            // only the store before last used this box
            }
            __syncwarp();
#pragma unroll
            for (int h = 0; h < CHUNK / 32; ++h) {
                float2 v[16];
                epilogue_half<OUT_BF16, SB>(p, t_lane + c + 32 * h, col0 + 32 * h, row, out_base, first_split,
                                            pre_box, h, v, false, nullptr, bias_tile + 4 * (c + 32 * h));
                stage_half<OUT_BF16>(box, lane, h, v);
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
                if (pre_box != nullptr) tma_store_3d(tm_pre, smem_addr(pre_box), col0, row0, u.batch);
                store_c_box(p, tm_c, smem_addr(box), col0, row0, cz);
                bulk_commit_group();
            }
            if (!p.has_pre) ebox ^= 1;
        } else {
            uint8_t* box = boxes;
            for (int pass = p.has_pre ? 0 : 1; pass < 2; ++pass) {
                if (lane == 0) bulk_wait_group_read<0>();  // the box's previous TMA store has read it
                __syncwarp();
#pragma unroll
                for (int h = 0; h < CHUNK / 32; ++h) {
                    float2 v[16];
                    epilogue_half<OUT_BF16, SB>(p, t_lane + c + 32 * h, col0 + 32 * h, row, out_base, first_split,
                                                nullptr, h, v, pass == 0, nullptr, bias_tile + 4 * (c + 32 * h));
                    stage_half<OUT_BF16>(box, lane, h, v);
                }
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    if (pass == 0) tma_store_3d(tm_pre, smem_addr(box), col0, row0, u.batch);
                    else store_c_box(p, tm_c, smem_addr(box), col0, row0, cz);
                    bulk_commit_group();
                }
            }
        }
    }
}

// The bias feed of SB kernels: the producer copies tile t's BN bias values into buffer t & 1 of `bias_s` once the
// epilogue warps have released that buffer from tile t - 2 (bias_empty), completion on bias_full[t & 1].
template <int BN>
__device__ __forceinline__ void issue_tile_bias(const TcParams& p, int32_t n0, uint32_t bias_s, uint64_t* bias_full,
                                                int buf) {
    const uint32_t bytes = 4u * static_cast<uint32_t>(min(BN, p.N - n0));  // N % 4 == 0: a multiple of 16
    const uint32_t bar = smem_addr(&bias_full[buf]);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load_1d(bias_s + static_cast<uint32_t>(buf * BN * 4), p.bias + n0, bytes, bar);
}

template <typename E, int BN, bool OUT_BF16, int EPI, bool SB = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_pre,
                   const __grid_constant__ CUtensorMap tm_res, const __grid_constant__ CUtensorMap tm_gin,
                   const __grid_constant__ CUtensorMap tm_aux, const TcParams p) {
    constexpr int NBOX = tc_epi_boxes(EPI);
    using Cfg = TcConfig<BN, NBOX, SB>;
    constexpr int ESIZE = sizeof(E);
    constexpr int BK = 128 / ESIZE;      // K elements per ring slot (one 128-byte swizzle row)
    constexpr int UMMA_K = 32 / ESIZE;   // K elements per tcgen05.mma (32 bytes)
    constexpr int MN_BOX = 128 / ESIZE;  // M/N elements per 128-byte row of an MN-major box
    constexpr bool IS_BF16 = ESIZE == 2;
    constexpr uint32_t FORMAT = IS_BF16 ? 1u : 2u;  // instruction-descriptor A/B format: bf16 = 1, tf32 = 2

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* epi = smem + Cfg::STAGES * Cfg::STAGE;
    const uint32_t bias_s = smem_addr(epi + Cfg::EPI_BYTES);  // SB: two BN-float bias buffers
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi + Cfg::EPI_BYTES + Cfg::BIAS_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + Cfg::STAGES;
    uint64_t* acc_full = bars + 2 * Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* aux_bars = drain + 1;  // two per epilogue warp
    uint64_t* bias_full = aux_bars + 2 * TC_EPI_WARPS;
    uint64_t* bias_empty = bias_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bias_empty + 2);
    const bool feed_bias = SB && p.bias != nullptr;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // The next GEMM of the stream may start its set-up as this grid's CTAs finish (programmatic dependent launch);
    // it touches no global memory before its own griddep_wait below.
    griddep_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_addr(&acc_full[a]), 1);
            mbar_init(smem_addr(&acc_empty[a]), TC_EPI_WARPS);  // one arrival per epilogue warp
            mbar_init(smem_addr(&bias_full[a]), 1);
            mbar_init(smem_addr(&bias_empty[a]), TC_EPI_WARPS);
        }
        mbar_init(smem_addr(drain), 1);
        for (int b = 0; b < 2 * TC_EPI_WARPS; ++b) mbar_init(smem_addr(&aux_bars[b]), 1);
        fence_mbarrier_init();
        fence_proxy_async_shared();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_descriptor(&tm_a);
        tma_prefetch_descriptor(&tm_b);
        tma_prefetch_descriptor(&tm_c);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish_alloc_permit();
    }
    tcgen05_fence_before_sync();
    __syncthreads();
    tcgen05_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above is local set-up; the operands, epilogue inputs and outputs may belong to the previous kernel.
    griddep_wait();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int tile = 0;
            for (TcCursor cur = tc_cursor(p, blockIdx.x, gridDim.x); cur.unit < p.num_units && ok; tc_advance(p, cur)) {
                const TcUnit u = tc_cursor_unit(p, cur, BN, BK);
                if (u.skip) continue;
                const int32_t ba = p.a_batched ? u.batch : 0;
                const int32_t bb = p.b_batched ? u.batch : 0;
                // The tile's bias is copied as soon as its buffer is free, checked between K slices without
                // blocking the operand loads (the buffer's previous tile is finished long before this tile's).
                const int bbuf = tile & 1;
                const uint32_t bpar = ((tile >> 1) & 1) ^ 1u;
                bool bias_pending = feed_bias;
                // Bring this tile's epilogue inputs into L2 now; the epilogue reads them one main loop later.
                if (u.split == 0) {
                    if (p.residual != nullptr) tma_prefetch_l2_3d(&tm_res, u.n0, u.m0, u.batch);
                    if (p.activation == 2) tma_prefetch_l2_3d(&tm_gin, u.n0, u.m0, u.batch);
                }
                for (int32_t kb = u.kb_begin; kb < u.kb_end; ++kb) {
                    const uint32_t fb = smem_addr(&full[stage]);
                    if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1u)) { ok = false; break; }
                    mbar_arrive_expect_tx(fb, Cfg::STAGE);
                    const uint32_t sa = smem_addr(ring + stage * Cfg::STAGE);
                    const uint32_t sb = sa + Cfg::STAGE_A;
                    const int32_t k0 = kb * BK;
                    load_a_slice<BK, MN_BOX, false>(p, &tm_a, sa, fb, u.m0, k0, ba);
                    if (!p.b_mn_major) {
                        tma_load_3d(sb, &tm_b, fb, k0, u.n0, bb);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / MN_BOX; ++j)
                            tma_load_3d(sb + j * (BK * 128), &tm_b, fb, u.n0 + j * MN_BOX, k0, bb);
                    }
                    if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1u; }
                    if (bias_pending && mbar_test_wait(smem_addr(&bias_empty[bbuf]), bpar)) {
                        issue_tile_bias<BN>(p, u.n0, bias_s, bias_full, bbuf);
                        bias_pending = false;
                    }
                }
                if (!ok) break;
                if (bias_pending) {
                    if (!mbar_wait(smem_addr(&bias_empty[bbuf]), bpar)) { ok = false; break; }
                    issue_tile_bias<BN>(p, u.n0, bias_s, bias_full, bbuf);
                }
                ++tile;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (elect_one()) {
            const uint32_t idesc = make_instr_desc(FORMAT, p.a_mn_major, p.b_mn_major, TC_BM, BN);
            // Byte offsets of the canonical 128-byte-swizzled layouts: K-major rows are 128 bytes apart and groups
            // of 8 rows 1024 bytes apart (SBO). MN-major slices have 128-byte K rows and successive 128-byte MN
            // chunks one box (BK rows) apart (LBO); their K rows group by 8 (16-byte swizzle atoms, bf16, SBO 1024)
            // or by 4 (32-byte atoms, tf32, SBO 512).
            constexpr uint32_t MN_LAYOUT = IS_BF16 ? SNB_LAYOUT_SWIZZLE_128B : SNB_LAYOUT_SWIZZLE_128B_BASE32B;
            constexpr uint32_t MN_SBO = IS_BF16 ? 1024 : 512;
            const uint32_t a_lbo = p.a_mn_major ? BK * 128 : 16;
            const uint32_t b_lbo = p.b_mn_major ? BK * 128 : 16;
            const uint32_t a_sbo = p.a_mn_major ? MN_SBO : 1024;
            const uint32_t b_sbo = p.b_mn_major ? MN_SBO : 1024;
            const uint32_t a_layout = p.a_mn_major ? MN_LAYOUT : SNB_LAYOUT_SWIZZLE_128B;
            const uint32_t b_layout = p.b_mn_major ? MN_LAYOUT : SNB_LAYOUT_SWIZZLE_128B;
            const uint32_t a_kstep = p.a_mn_major ? UMMA_K * 128 : 32;
            const uint32_t b_kstep = p.b_mn_major ? UMMA_K * 128 : 32;
            int stage = 0;
            uint32_t phase = 0;
            int iter = 0;
            bool ok = true;
            bool issued = false;
            for (TcCursor cur = tc_cursor(p, blockIdx.x, gridDim.x); cur.unit < p.num_units && ok; tc_advance(p, cur)) {
                const TcUnit u = tc_cursor_unit(p, cur, BN, BK);
                if (u.skip) continue;
                const int acc = iter & 1;
                const uint32_t acc_phase = (iter >> 1) & 1;
                if (!mbar_wait(smem_addr(&acc_empty[acc]), acc_phase ^ 1u)) { ok = false; break; }
                tcgen05_fence_after_sync();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int32_t kb = u.kb_begin; kb < u.kb_end; ++kb) {
                    if (!mbar_wait(smem_addr(&full[stage]), phase)) { ok = false; break; }
                    tcgen05_fence_after_sync();
                    const uint32_t sa = smem_addr(ring + stage * Cfg::STAGE);
                    const uint32_t sb = sa + Cfg::STAGE_A;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        const uint64_t ad = make_smem_desc(sa + k * a_kstep, a_lbo, a_sbo, a_layout);
                        const uint64_t bd = make_smem_desc(sb + k * b_kstep, b_lbo, b_sbo, b_layout);
                        const uint32_t accumulate = (kb > u.kb_begin || k > 0) ? 1u : 0u;
                        if (IS_BF16) umma_bf16(d_tmem, ad, bd, idesc, accumulate);
                        else umma_tf32(d_tmem, ad, bd, idesc, accumulate);
                    }
                    issued = true;
                    umma_commit(smem_addr(&empty[stage]));
                    if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                umma_commit(smem_addr(&acc_full[acc]));
                ++iter;
            }
            if (!ok && issued) {
                // Let every MMA already issued finish before TMEM is released.
                umma_commit(smem_addr(drain));
                mbar_wait(smem_addr(drain), 0);
            }
        }
        __syncwarp();
    } else if (warp >= TC_EPI_WARP0) {
        // ------------------------------------------------------------------ epilogue
        // A warp may read only the TMEM lanes of its quadrant (warp % 4): 32 output rows. The two warps of a
        // quadrant take alternate chunks of the tile's columns.
        const int q = warp & 3;
        const int group = (warp - TC_EPI_WARP0) >> 2;
        uint8_t* boxes = epi + (warp - TC_EPI_WARP0) * NBOX * TC_EPI_BOX_BYTES;
        uint64_t* aux_bar = aux_bars + 2 * (warp - TC_EPI_WARP0);
        // The host picks TC_EPI_AUX_BOX only for bf16 outputs of products without causal skipping.
        constexpr bool box_aux = EPI == TC_EPI_AUX_BOX;
        uint32_t aux_phase = 0;
        int ebox = 0;
        int iter = 0;
        TcCursor cur = tc_cursor(p, blockIdx.x, gridDim.x);
        if (box_aux && lane == 0 && cur.unit < p.num_units) {
            const TcUnit u0 = tc_cursor_unit(p, cur, BN, BK);
            request_aux_boxes<OUT_BF16, BN>(p, &tm_aux, u0, u0.m0 + q * 32, group, boxes, aux_bar);
        }
        for (; cur.unit < p.num_units; tc_advance(p, cur)) {
            const TcUnit u = tc_cursor_unit(p, cur, BN, BK);
            if (u.skip) continue;
            const int acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            if (!mbar_wait(smem_addr(&acc_full[acc]), acc_phase)) break;
            tcgen05_fence_after_sync();
            if (feed_bias && !mbar_wait(smem_addr(&bias_full[acc]), acc_phase)) break;
            const int32_t row0 = u.m0 + q * 32;
            const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;

            epilogue_tile<OUT_BF16, BN, EPI, SB>(p, &tm_c, &tm_pre, u, row0, t_lane, group, boxes, ebox, aux_bar,
                                                 aux_phase, bias_s + static_cast<uint32_t>(acc * BN * 4));
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_addr(&acc_empty[acc]));
                if (feed_bias) mbar_arrive(smem_addr(&bias_empty[acc]));
            }
            ++iter;
            // The next tile's auxiliary input is requested as soon as this tile's stores have read the boxes, so
            // its loads overlap the next main loop.
            TcCursor next = cur;
            tc_advance(p, next);
            if (box_aux && lane == 0 && next.unit < p.num_units) {
                bulk_wait_group_read<0>();
                const TcUnit un = tc_cursor_unit(p, next, BN, BK);
                request_aux_boxes<OUT_BF16, BN>(p, &tm_aux, un, un.m0 + q * 32, group, boxes, aux_bar);
            }
            __syncwarp();
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tcgen05_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tcgen05_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace snb
