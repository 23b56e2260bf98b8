// attention_fused.cuh — causal attention forward in one kernel on tcgen05, without materialising the scores:
//   out[q] = sum_k softmax_k(scale * Q[q].K[k]) V[k]  over the visible keys k <= q + offset (k < keys),
// the composition of the reference's QK^T product, `causal_softmax` and P.V product
// (crates/staleynet-model/src/layers/attention.rs:206-213, crates/staleynet-cuda/src/kernels/attention.rs:153-180),
// plus the per-query log-sum-exp, from which a backward pass can rebuild the probabilities.
//
// One CTA of 384 threads per pair of 128-query tiles of one (batch, head) matrix; head_dim 64; keys in steps of 128:
//   warp 0     TMA: both query tiles once, then K/V tiles through a 2-stage ring.
//   warp 1     allocates TMEM (S0, S1: 128 columns each, O0, O1: 64 each) and, on one elected thread, issues
//              S_t = Q_t K_j^T (M=128, N=128, K=64) and O_t += P_t V_j (M=128, N=64, K=128) for both tiles t.
//   warps 4-7  / 8-11: online softmax of tile 0 / tile 1, one thread per query row: row max over S_t (TMEM), exponentials
//              with ex2.approx, P_t written as bf16 into a 128B-swizzled shared-memory operand, O_t rescaled in TMEM
//              when the row max grows; finally O_t / l written out and the log-sum-exp saved.
// Every mbarrier wait is bounded (see sm100_ptx.cuh).
#pragma once

#include "gemm_tc.cuh"

namespace snb {

constexpr int FA_BM = 128;   // queries per tile (two tiles per CTA)
constexpr int FA_BN = 128;   // keys per step
constexpr int FA_D = 64;     // head dimension
constexpr int FA_THREADS = 384;
constexpr int FA_TMEM_COLS = 512;
constexpr float FA_RESCALE_SLACK = 8.0f;  // log2 of the largest unnormalised probability the softmax lets stand

struct FaParams {
    int32_t count, sq, sk;   // matrices; queries and keys per matrix
    int32_t pairs;           // query-tile pairs per matrix
    int64_t offset;          // query q sees keys 0..=q+offset
    float scale_log2;        // scale * log2(e)
    int32_t out_bf16;
    void* out;               // [count, sq, 64]
    int64_t out_stride;      // elements between matrices of out
    float* lse;              // [count, sq] natural-log log-sum-exp, or nullptr
};

struct FaSmem {
    static constexpr int Q = FA_BM * 128;           // one query tile: 128 rows x 64 bf16
    static constexpr int KV = FA_BN * 128;          // one K or V tile
    static constexpr int P = FA_BM * FA_BN * 2;     // one P tile: two 64-key slices of 128 rows x 128 bytes
    static constexpr int BYTES = 1024 + 2 * Q + 2 * 2 * KV + 2 * P + 256;
    static_assert(BYTES <= 232448, "shared memory budget of one sm_100 CTA");
};

__device__ __forceinline__ int64_t imin64(int64_t x, int64_t y) { return x < y ? x : y; }

// mbar_wait agreed by the whole warp: tcgen05.ld/st are warp-collective (.sync.aligned), so every branch around
// them must be taken by all 32 lanes together.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Keys steps a query tile needs: through the last key any of its rows sees.
__device__ __forceinline__ int32_t fa_steps(const FaParams& p, int32_t q0) {
    if (q0 >= p.sq) return 0;
    const int64_t last_key = imin64(static_cast<int64_t>(p.sk) - 1, static_cast<int64_t>(q0) + FA_BM - 1 + p.offset);
    return static_cast<int32_t>(last_key / FA_BN + 1);
}

__global__ void __launch_bounds__(FA_THREADS, 1)
    fa_forward_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const FaParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* q_s = smem;                                  // 2 query tiles
    uint8_t* kv_s = q_s + 2 * FaSmem::Q;                  // 2 stages x (K, V)
    uint8_t* p_s = kv_s + 4 * FaSmem::KV;                 // 2 P tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + 2 * FaSmem::P);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;    // [2]
    uint64_t* kv_empty = bars + 3;   // [2]
    uint64_t* s_full = bars + 5;     // [2] per tile
    uint64_t* s_empty = bars + 7;    // [2]
    uint64_t* p_full = bars + 9;     // [2]
    uint64_t* o_done = bars + 11;    // [2]
    uint64_t* drain = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Heavier (later) query tiles first.
    const int32_t pair = p.pairs - 1 - static_cast<int32_t>(blockIdx.x % p.pairs);
    const int32_t matrix = static_cast<int32_t>(blockIdx.x / p.pairs);
    const int32_t q_first = pair * 2 * FA_BM;  // tile t covers queries q_first + 128 t ...
    const int32_t steps0 = fa_steps(p, q_first), steps1 = fa_steps(p, q_first + FA_BM);
    const int32_t nsteps = max(steps0, steps1);

    if (threadIdx.x == 0) {
        mbar_init(smem_addr(q_full), 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&kv_full[i]), 1);
            mbar_init(smem_addr(&kv_empty[i]), 1);
            mbar_init(smem_addr(&s_full[i]), 1);
            mbar_init(smem_addr(&s_empty[i]), 4);
            mbar_init(smem_addr(&p_full[i]), 4);
            mbar_init(smem_addr(&o_done[i]), 1);
        }
        mbar_init(smem_addr(drain), 1);
        fence_mbarrier_init();
        fence_proxy_async_shared();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), FA_TMEM_COLS);
        tmem_relinquish_alloc_permit();
    }
    tcgen05_fence_before_sync();
    __syncthreads();
    tcgen05_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (elect_one()) {
            bool ok = true;
            const uint32_t qb = smem_addr(q_full);
            mbar_arrive_expect_tx(qb, 2 * FaSmem::Q);
            tma_load_3d(smem_addr(q_s), &tm_q, qb, 0, q_first, matrix);
            tma_load_3d(smem_addr(q_s + FaSmem::Q), &tm_q, qb, 0, q_first + FA_BM, matrix);
            for (int32_t j = 0; j < nsteps && ok; ++j) {
                const int s = j & 1;
                if (!mbar_wait(smem_addr(&kv_empty[s]), ((j >> 1) & 1) ^ 1u)) { ok = false; break; }
                const uint32_t fb = smem_addr(&kv_full[s]);
                mbar_arrive_expect_tx(fb, 2 * FaSmem::KV);
                uint8_t* kt = kv_s + s * 2 * FaSmem::KV;
                tma_load_3d(smem_addr(kt), &tm_k, fb, 0, j * FA_BN, matrix);
                tma_load_3d(smem_addr(kt + FaSmem::KV), &tm_v, fb, 0, j * FA_BN, matrix);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (elect_one()) {
            const uint32_t idesc_s = make_instr_desc(1u, 0u, 0u, FA_BM, FA_BN);    // Q K-major, K K-major
            const uint32_t idesc_o = make_instr_desc(1u, 0u, 1u, FA_BM, FA_D);     // P K-major, V N-major
            bool ok = mbar_wait(smem_addr(q_full), 0);
            bool issued = false;
            auto issue_pv = [&](int32_t jj) {
                // O_t += P_t V_jj for both tiles that still need step jj, then free the K/V stage.
                const int s = jj & 1;
                const uint32_t vb = smem_addr(kv_s + s * 2 * FaSmem::KV + FaSmem::KV);
                for (int t = 0; t < 2 && ok; ++t) {
                    if (jj >= (t == 0 ? steps0 : steps1)) continue;
                    if (!mbar_wait(smem_addr(&p_full[t]), jj & 1)) { ok = false; break; }
                    tcgen05_fence_after_sync();
                    const uint32_t pb = smem_addr(p_s + t * FaSmem::P);
                    const uint32_t o_tmem = tmem_base + 2 * FA_BN + t * FA_D;
#pragma unroll
                    for (int kk = 0; kk < FA_BN / 16; ++kk) {
                        const uint64_t ad = make_smem_desc(pb + (kk / 4) * (FaSmem::P / 2) + (kk % 4) * 32, 16, 1024,
                                                           SNB_LAYOUT_SWIZZLE_128B);
                        const uint64_t bd = make_smem_desc(vb + kk * 16 * 128, FaSmem::KV, 1024, SNB_LAYOUT_SWIZZLE_128B);
                        umma_bf16(o_tmem, ad, bd, idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
                    }
                    issued = true;
                    umma_commit(smem_addr(&o_done[t]));
                }
                if (ok) umma_commit(smem_addr(&kv_empty[s]));
            };
            for (int32_t j = 0; j < nsteps && ok; ++j) {
                const int s = j & 1;
                if (!mbar_wait(smem_addr(&kv_full[s]), (j >> 1) & 1)) { ok = false; break; }
                tcgen05_fence_after_sync();
                const uint32_t kb = smem_addr(kv_s + s * 2 * FaSmem::KV);
                for (int t = 0; t < 2 && ok; ++t) {
                    if (j >= (t == 0 ? steps0 : steps1)) continue;
                    // S_t is free once the softmax has read step j-1's scores.
                    if (!mbar_wait(smem_addr(&s_empty[t]), (j & 1) ^ 1u)) { ok = false; break; }
                    tcgen05_fence_after_sync();
                    const uint32_t qb = smem_addr(q_s + t * FaSmem::Q);
                    const uint32_t s_tmem = tmem_base + t * FA_BN;
#pragma unroll
                    for (int k = 0; k < FA_D / 16; ++k) {
                        const uint64_t ad = make_smem_desc(qb + k * 32, 16, 1024, SNB_LAYOUT_SWIZZLE_128B);
                        const uint64_t bd = make_smem_desc(kb + k * 32, 16, 1024, SNB_LAYOUT_SWIZZLE_128B);
                        umma_bf16(s_tmem, ad, bd, idesc_s, k > 0 ? 1u : 0u);
                    }
                    issued = true;
                    umma_commit(smem_addr(&s_full[t]));
                }
                if (ok && j >= 1) issue_pv(j - 1);
            }
            if (ok && nsteps >= 1) issue_pv(nsteps - 1);
            if (!ok && issued) {
                // Let every MMA already issued finish before TMEM is released.
                umma_commit(smem_addr(drain));
                mbar_wait(smem_addr(drain), 0);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ------------------------------------------------------------------ softmax (one thread per query row)
        const int t = (warp - 4) >> 2;   // query tile of this warpgroup
        const int q = warp & 3;          // TMEM lane quadrant
        const int r = q * 32 + lane;     // row within the tile
        const int32_t tsteps = t == 0 ? steps0 : steps1;
        const int64_t query = static_cast<int64_t>(q_first) + t * FA_BM + r;
        // Keys [0, row_end) are visible to this row: key <= query + offset and key < sk (row_end >= 1).
        const int32_t row_end = static_cast<int32_t>(imin64(query + p.offset, static_cast<int64_t>(p.sk) - 1) + 1);
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t s_tmem = tmem_base + lane_base + t * FA_BN;
        const uint32_t o_tmem = tmem_base + lane_base + 2 * FA_BN + t * FA_D;
        uint8_t* p_tile = p_s + t * FaSmem::P;
        const float c = p.scale_log2;
        const float2 c2 = make_float2(c, c);
        // Running max m (in units of log2: scale*log2(e)*score) and running sum l of 2^(x - m). m may lag the true
        // row max by up to FA_RESCALE_SLACK: O and l are only rescaled when some row of the warp outgrows it, which
        // keeps every exponent <= 2^FA_RESCALE_SLACK and leaves O / l unchanged.
        float m = -1.0e30f;
        float l = 0.0f;
        bool ok = true;
        for (int32_t j = 0; j < tsteps && ok; ++j) {
            if (!warp_wait(smem_addr(&s_full[t]), j & 1)) { ok = false; break; }
            tcgen05_fence_after_sync();
            const int32_t vis = row_end - j * FA_BN;   // visible keys of this step (>= FA_BN: all)
            // Pass 1: row max of the raw scores (scale > 0, so it commutes with the scaling).
            float mr[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
            for (int c0 = 0; c0 < FA_BN; c0 += 64) {
                uint32_t xs[2][32];
                tmem_load_32x32b_x32(s_tmem + c0, xs[0]);
                tmem_load_32x32b_x32(s_tmem + c0 + 32, xs[1]);
                tmem_load_wait();
const auto X = [&](int i) { return __uint_as_float(xs[i >> 5][i & 31]); };
                if (vis >= c0 + 64) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) mr[i & 3] = fmaxf(mr[i & 3], X(i));
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (c0 + i < vis) mr[i & 3] = fmaxf(mr[i & 3], X(i));
                }
            }
            const float mx = fmaxf(m, fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3])) * c);
            const bool rescale = __any_sync(0xffffffffu, mx > m + FA_RESCALE_SLACK);
            const float m_use = rescale ? mx : m;
            // P_t may be rewritten (and O_t rescaled) once step j-1's P.V product has finished.
            if (j > 0 && !warp_wait(smem_addr(&o_done[t]), (j - 1) & 1)) { ok = false; break; }
            // Pass 2: 2^(x - m), their sum, and the bf16 operand of P.V.
            const float2 nm2 = make_float2(-m_use, -m_use);
            float2 sa = make_float2(0.0f, 0.0f), sb = make_float2(0.0f, 0.0f);
#pragma unroll 1
            for (int c0 = 0; c0 < FA_BN; c0 += 64) {
                uint32_t xs[2][32];
                tmem_load_32x32b_x32(s_tmem + c0, xs[0]);
                tmem_load_32x32b_x32(s_tmem + c0 + 32, xs[1]);
                tmem_load_wait();
const auto X = [&](int i) { return __uint_as_float(xs[i >> 5][i & 31]); };
                uint32_t w[32];
                if (vis >= c0 + 64) {
#pragma unroll
                    for (int i = 0; i < 64; i += 4) {
                        float2 e0 = __ffma2_rn(make_float2(X(i), X(i + 1)), c2, nm2);
                        float2 e1 = __ffma2_rn(make_float2(X(i + 2), X(i + 3)), c2, nm2);
                        e0.x = exp2_hw(e0.x);
                        e0.y = exp2_hw(e0.y);
                        e1.x = exp2_hw(e1.x);
                        e1.y = exp2_hw(e1.y);
                        sa = __fadd2_rn(sa, e0);
                        sb = __fadd2_rn(sb, e1);
                        w[i / 2] = pack_bf16x2(e0.x, e0.y);
                        w[i / 2 + 1] = pack_bf16x2(e1.x, e1.y);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 64; i += 2) {
                        const float e0 = (c0 + i < vis) ? exp2_hw(fmaf(X(i), c, -m_use)) : 0.0f;
                        const float e1 = (c0 + i + 1 < vis) ? exp2_hw(fmaf(X(i + 1), c, -m_use)) : 0.0f;
                        sa = __fadd2_rn(sa, make_float2(e0, e1));
                        w[i / 2] = pack_bf16x2(e0, e1);
                    }
                }
                // Row r of the K-major 128B-swizzled operand: keys [64s, 64s+64) live in slice s.
                uint8_t* row = p_tile + (c0 / 64) * (FaSmem::P / 2) + r * 128;
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    *reinterpret_cast<uint4*>(row + ((g ^ (r & 7)) << 4)) =
                        make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
            }
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&s_empty[t]));  // S_t may take the next step's scores
            if (rescale) {
                const float alpha = exp2_hw(m - m_use);
                if (j > 0) {
                    // O_t *= alpha for the rows of this warp (alpha = 1 for rows whose max did not grow).
                    for (int c0 = 0; c0 < FA_D; c0 += 32) {
                        uint32_t o[32];
                        tmem_load_32x32b_x32(o_tmem + c0, o);
                        tmem_load_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_store_32x32b_x32(o_tmem + c0, o);
                    }
                    tmem_store_wait();
                }
                l *= alpha;
                m = m_use;
            }
            l += (sa.x + sa.y) + (sb.x + sb.y);
            fence_proxy_async_shared();  // P_t writes -> the tensor core's reads
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&p_full[t]));
        }
        if (ok && tsteps > 0 && warp_wait(smem_addr(&o_done[t]), (tsteps - 1) & 1)) {
            tcgen05_fence_after_sync();
            const float inv = 1.0f / l;
            const bool live = query < p.sq;
            const int64_t base = static_cast<int64_t>(matrix) * p.out_stride + query * FA_D;
            for (int c0 = 0; c0 < FA_D; c0 += 32) {
                uint32_t o[32];
                tmem_load_32x32b_x32(o_tmem + c0, o);
                tmem_load_wait();
                if (!live) continue;
                if (p.out_bf16) {
                    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base + c0);
#pragma unroll
                    for (int g = 0; g < 4; ++g)
                        dst[g] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * g]) * inv, __uint_as_float(o[8 * g + 1]) * inv),
                                            pack_bf16x2(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv),
                                            pack_bf16x2(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv),
                                            pack_bf16x2(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv));
                } else {
                    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + base + c0);
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        dst[g] = make_float4(__uint_as_float(o[4 * g]) * inv, __uint_as_float(o[4 * g + 1]) * inv,
                                             __uint_as_float(o[4 * g + 2]) * inv, __uint_as_float(o[4 * g + 3]) * inv);
                }
            }
            if (live && p.lse != nullptr)
                p.lse[static_cast<int64_t>(matrix) * p.sq + query] = (m + __log2f(l)) * 0.69314718f;
        }
    }

    tcgen05_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tcgen05_fence_after_sync();
        tmem_dealloc(tmem_base, FA_TMEM_COLS);
    }
}

}  // namespace snb
