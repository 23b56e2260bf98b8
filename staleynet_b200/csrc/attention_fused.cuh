// attention_fused.cuh — causal attention forward in one kernel on tcgen05, without materialising the scores:
//   out[q] = sum_k softmax_k(scale * Q[q].K[k]) V[k]  over the visible keys k <= q + offset (k < keys),
// the composition of the reference's QK^T product, `causal_softmax` and P.V product
// (crates/staleynet-model/src/layers/attention.rs:206-213, crates/staleynet-cuda/src/kernels/attention.rs:153-180),
// plus the per-query log-sum-exp, from which a backward pass can rebuild the probabilities.
//
// One CTA of 576 threads per pair of 128-query tiles of one (batch, head) matrix; head_dim 64; keys in steps of 128:
//   warps 0-15 softmax, two threads per query row: warp w serves tile w / 8, key half (w / 4) % 2 (64 of the step's
//              128 scores, held in registers) and TMEM lane quadrant w % 4. The two halves of a row exchange their
//              partial maxima through shared memory under a 64-thread named barrier; exponentials by ex2.approx;
//              each half stores its 64 keys of P_t as bf16 into TMEM (tcgen05.st) and rescales its 32 columns of
//              O_t in TMEM when a row max outgrows the running one; finally O_t / l is written out and the
//              log-sum-exp saved.
//   warp 16    TMA: both query tiles once, then K/V tiles through a FA_KV_STAGES-deep ring.
//   warp 17    allocates TMEM (S0, S1: 128 f32 columns each; O0, O1: 64 each; P0, P1: 64 columns of bf16 pairs each)
//              and, on one elected thread, issues per key step j, tile by tile: S_t(j) = Q_t K_j^T (M=128, N=128,
//              K=64, both operands from shared memory), then O_t += P_t(j-1) V_{j-1} (M=128, N=64, K=128, P from
//              TMEM), so that each tile's softmax runs while the other tile's products execute. Keeping P in TMEM
//              spares shared memory 128 KB of traffic per key step (the P stores and the product's reads of them).
// Every mbarrier wait is bounded (see sm100_ptx.cuh); the two warps of a row pair agree on every timeout before
// either leaves its loop, so no named barrier is left waiting for a warp that gave up.
#pragma once

#include "gemm_tc.cuh"

namespace snb {

constexpr int FA_BM = 128;   // queries per tile (two tiles per CTA)
constexpr int FA_BN = 128;   // keys per step
constexpr int FA_D = 64;     // head dimension
constexpr int FA_SOFTMAX_WARPS = 16;
constexpr int FA_PRODUCER_WARP = 16;
constexpr int FA_MMA_WARP = 17;
constexpr int FA_THREADS = 18 * 32;
constexpr int FA_TMEM_COLS = 512;
constexpr int FA_KV_STAGES = 3;
constexpr int FA_O_COL = 2 * FA_BN;          // TMEM columns: S0, S1 at 0 and 128; O0, O1 at 256 and 320;
constexpr int FA_P_COL = 2 * FA_BN + 2 * FA_D; // P0, P1 at 384 and 448
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
    static constexpr int BARS = 256;
    // Row-pair exchange: [step parity][tile][key half][row] partial maxima, then [parity][tile][half][quadrant] flags.
    static constexpr int XMAX = 2 * 2 * 2 * FA_BM * 4;
    static constexpr int XFLAG = 2 * 2 * 2 * 4 * 4;
    static constexpr int BYTES = 1024 + 2 * Q + FA_KV_STAGES * 2 * KV + BARS + XMAX + XFLAG;
    static_assert(BYTES <= 232448, "shared memory budget of one sm_100 CTA");
};

__device__ __forceinline__ int64_t imin64(int64_t x, int64_t y) { return x < y ? x : y; }

// mbar_wait agreed by the whole warp: tcgen05.ld/st are warp-collective (.sync.aligned), so every branch around
// them must be taken by all 32 lanes together.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Named barrier over the two warps (64 threads) that share a row quadrant of a tile.
__device__ __forceinline__ void pair_barrier(int id) {
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
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
    uint8_t* kv_s = q_s + 2 * FaSmem::Q;                  // FA_KV_STAGES stages x (K, V)
    uint64_t* bars = reinterpret_cast<uint64_t*>(kv_s + FA_KV_STAGES * 2 * FaSmem::KV);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;                   // [FA_KV_STAGES]
    uint64_t* kv_empty = kv_full + FA_KV_STAGES;    // [FA_KV_STAGES]
    uint64_t* s_full = kv_empty + FA_KV_STAGES;     // [2] per tile
    uint64_t* s_empty = s_full + 2;                 // [2]
    uint64_t* p_full = s_empty + 2;                 // [2]
    uint64_t* o_done = p_full + 2;                  // [2]
    uint64_t* drain = o_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    float* xmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + FaSmem::BARS);
    int32_t* xflag = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(xmax) + FaSmem::XMAX);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Longest first over the whole grid: the last query-tile pair of every matrix, then the one before, ...
    const int32_t pair = p.pairs - 1 - static_cast<int32_t>(blockIdx.x / p.count);
    const int32_t matrix = static_cast<int32_t>(blockIdx.x % p.count);
    const int32_t q_first = pair * 2 * FA_BM;  // tile t covers queries q_first + 128 t ...
    const int32_t steps0 = fa_steps(p, q_first), steps1 = fa_steps(p, q_first + FA_BM);
    const int32_t nsteps = max(steps0, steps1);
    constexpr uint32_t kSoftmaxArrivals = FA_SOFTMAX_WARPS / 2;  // warps per tile

    // The producer starts Q and the first K/V stages before the CTA-wide barrier: it prefetches the tensor maps,
    // initialises the barriers of its own loads and issues them, so that they overlap the other barriers' set-up
    // and the TMEM allocation.
    bool producer = false;
    if (warp == FA_PRODUCER_WARP) producer = elect_one();
    int pstage = 0;
    uint32_t pphase = 0;
    int32_t pj = 0;   // key steps whose K and V are requested
    auto load_kv = [&](int32_t j) {
        const uint32_t fb = smem_addr(&kv_full[pstage]);
        mbar_arrive_expect_tx(fb, 2 * FaSmem::KV);
        uint8_t* kt = kv_s + pstage * 2 * FaSmem::KV;
        tma_load_3d(smem_addr(kt), &tm_k, fb, 0, j * FA_BN, matrix);
        tma_load_3d(smem_addr(kt + FaSmem::KV), &tm_v, fb, 0, j * FA_BN, matrix);
        if (++pstage == FA_KV_STAGES) { pstage = 0; pphase ^= 1u; }
    };
    if (producer) {
        for (const CUtensorMap* m : {&tm_q, &tm_k, &tm_v}) tma_prefetch_descriptor(m);
        mbar_init(smem_addr(q_full), 1);
        for (int i = 0; i < FA_KV_STAGES; ++i) {
            mbar_init(smem_addr(&kv_full[i]), 1);
            mbar_init(smem_addr(&kv_empty[i]), 1);
        }
        fence_mbarrier_init();
        const uint32_t qb = smem_addr(q_full);
        mbar_arrive_expect_tx(qb, 2 * FaSmem::Q);
        tma_load_3d(smem_addr(q_s), &tm_q, qb, 0, q_first, matrix);
        tma_load_3d(smem_addr(q_s + FaSmem::Q), &tm_q, qb, 0, q_first + FA_BM, matrix);
        for (; pj < nsteps && pj < FA_KV_STAGES; ++pj) load_kv(pj);   // the ring starts empty
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&s_full[i]), 1);
            mbar_init(smem_addr(&s_empty[i]), kSoftmaxArrivals);
            mbar_init(smem_addr(&p_full[i]), kSoftmaxArrivals);
            mbar_init(smem_addr(&o_done[i]), 1);
        }
        mbar_init(smem_addr(drain), 1);
        fence_mbarrier_init();
        fence_proxy_async_shared();
    }
    if (warp == FA_MMA_WARP) {
        tmem_alloc(smem_addr(tmem_slot), FA_TMEM_COLS);
        tmem_relinquish_alloc_permit();
    }
    tcgen05_fence_before_sync();
    __syncthreads();
    tcgen05_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == FA_PRODUCER_WARP) {
        // ------------------------------------------------------------------ TMA producer
        if (producer) {
            for (; pj < nsteps; ++pj) {
                if (!mbar_wait(smem_addr(&kv_empty[pstage]), pphase ^ 1u)) break;
                load_kv(pj);
            }
        }
        __syncwarp();
    } else if (warp == FA_MMA_WARP) {
        // ------------------------------------------------------------------ MMA issuer
        if (elect_one()) {
            const uint32_t idesc_s = make_instr_desc(1u, 0u, 0u, FA_BM, FA_BN);    // Q K-major, K K-major
            const uint32_t idesc_o = make_instr_desc(1u, 0u, 1u, FA_BM, FA_D);     // P K-major, V N-major
            bool ok = mbar_wait(smem_addr(q_full), 0);
            bool issued = false;
            int stage = 0, prev_stage = 0;
            uint32_t phase = 0;
            for (int32_t j = 0; j <= nsteps && ok; ++j) {
                if (j < nsteps) {
                    if (!mbar_wait(smem_addr(&kv_full[stage]), phase)) { ok = false; break; }
                    tcgen05_fence_after_sync();
                }
                const uint32_t kb = smem_addr(kv_s + stage * 2 * FaSmem::KV);
                const uint32_t vb = smem_addr(kv_s + prev_stage * 2 * FaSmem::KV + FaSmem::KV);
                for (int t = 0; t < 2 && ok; ++t) {
                    const int32_t tsteps = t == 0 ? steps0 : steps1;
                    if (j < tsteps) {
                        // S_t(j) = Q_t K_j^T once the softmax has read S_t(j-1).
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
                    if (j >= 1 && j - 1 < tsteps) {
                        // O_t += P_t(j-1) V_{j-1} once the softmax has written P_t(j-1).
                        if (!mbar_wait(smem_addr(&p_full[t]), (j - 1) & 1)) { ok = false; break; }
                        tcgen05_fence_after_sync();
                        const uint32_t p_tmem = tmem_base + FA_P_COL + t * (FA_BN / 2);
                        const uint32_t o_tmem = tmem_base + FA_O_COL + t * FA_D;
#pragma unroll
                        for (int kk = 0; kk < FA_BN / 16; ++kk) {
                            // Keys 16kk..16kk+15 of P: 8 TMEM columns of bf16 pairs.
                            const uint64_t bd = make_smem_desc(vb + kk * 16 * 128, FaSmem::KV, 1024,
                                                               SNB_LAYOUT_SWIZZLE_128B);
                            umma_bf16_tmem_a(o_tmem, p_tmem + 8 * kk, bd, idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
                        }
                        issued = true;
                        umma_commit(smem_addr(&o_done[t]));
                    }
                }
                // Stage j-1 (K read by S(j-1), V by P.V(j-1)) is free once those products finish.
                if (ok && j >= 1) umma_commit(smem_addr(&kv_empty[prev_stage]));
                prev_stage = stage;
                if (j < nsteps && ++stage == FA_KV_STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok && issued) {
                // Let every MMA already issued finish before TMEM is released.
                umma_commit(smem_addr(drain));
                mbar_wait(smem_addr(drain), 0);
            }
        }
        __syncwarp();
    } else if (warp < FA_SOFTMAX_WARPS) {
        // ------------------------------------------------------------------ softmax (two threads per query row)
        const int t = warp >> 3;          // query tile
        const int h = (warp >> 2) & 1;    // key half of every step: keys [64h, 64h + 64)
        const int q = warp & 3;           // TMEM lane quadrant
        const int r = q * 32 + lane;      // row within the tile
        const int pair_bar = 1 + t * 4 + q;   // named barrier of this row pair (0 is __syncthreads)
        const int32_t tsteps = t == 0 ? steps0 : steps1;
        const int64_t query = static_cast<int64_t>(q_first) + t * FA_BM + r;
        // Keys [0, row_end) are visible to this row: key <= query + offset and key < sk (row_end >= 1).
        const int32_t row_end = static_cast<int32_t>(imin64(query + p.offset, static_cast<int64_t>(p.sk) - 1) + 1);
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t s_tmem = tmem_base + lane_base + t * FA_BN + 64 * h;
        const uint32_t o_tmem = tmem_base + lane_base + FA_O_COL + t * FA_D + 32 * h;
        const uint32_t p_tmem = tmem_base + lane_base + FA_P_COL + t * (FA_BN / 2) + 32 * h;
        const float c = p.scale_log2;
        const float2 c2 = make_float2(c, c);
        // Running max m (in units of log2: scale*log2(e)*score), the same in both halves of a row, and this half's
        // running sum l of 2^(x - m). m may lag the true row max by up to FA_RESCALE_SLACK: O and l are only
        // rescaled when some row of the warp outgrows it, which keeps every exponent <= 2^FA_RESCALE_SLACK and leaves
        // O / l unchanged.
        float m = -1.0e30f;
        float l = 0.0f;
        bool ok = true;
        for (int32_t j = 0; j < tsteps; ++j) {
            bool ready = warp_wait(smem_addr(&s_full[t]), j & 1);
            tcgen05_fence_after_sync();
            uint32_t xs[2][32];
            tmem_load_32x32b_x32(s_tmem, xs[0]);
            tmem_load_32x32b_x32(s_tmem + 32, xs[1]);
            tmem_load_wait();
            // S_t is free for the next step's scores as soon as it sits in registers.
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&s_empty[t]));
            const int32_t vis = row_end - j * FA_BN - 64 * h;   // visible keys of this half-step
            if (vis < 64) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (i >= vis) xs[i >> 5][i & 31] = 0xff800000u;   // -inf: exponential 0
            }
            float mr[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 64; ++i) mr[i & 3] = fmaxf(mr[i & 3], __uint_as_float(xs[i >> 5][i & 31]));
            // P_t may be rewritten (and O_t rescaled) once the P.V product of step j-1 has finished.
            if (j > 0 && ready) ready = warp_wait(smem_addr(&o_done[t]), (j - 1) & 1);
            // Exchange partial maxima and readiness with the other half of the row.
            const int slot = j & 1;
            xmax[((slot * 2 + t) * 2 + h) * FA_BM + r] = fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3]));
            if (lane == 0) xflag[((slot * 2 + t) * 2 + h) * 4 + q] = ready ? 1 : 0;
            pair_barrier(pair_bar);
            const float other = xmax[((slot * 2 + t) * 2 + (h ^ 1)) * FA_BM + r];
            const bool other_ready = xflag[((slot * 2 + t) * 2 + (h ^ 1)) * 4 + q] != 0;
            if (!(ready && other_ready)) { ok = false; break; }
            // scale > 0, so the max commutes with the scaling.
            const float mx = fmaxf(m, fmaxf(fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3])), other) * c);
            const bool rescale = __any_sync(0xffffffffu, mx > m + FA_RESCALE_SLACK);
            const float m_use = rescale ? mx : m;
            const float2 nm2 = make_float2(-m_use, -m_use);
            float2 sa = make_float2(0.0f, 0.0f), sb = make_float2(0.0f, 0.0f);
            // 2^(x - m) as bf16 pairs, 32 keys at a time: w[i/2] holds keys 32b + i, 32b + i + 1 of this half.
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float2 e0 = __ffma2_rn(make_float2(__uint_as_float(xs[b][i]), __uint_as_float(xs[b][i + 1])), c2, nm2);
                    float2 e1 = __ffma2_rn(make_float2(__uint_as_float(xs[b][i + 2]), __uint_as_float(xs[b][i + 3])), c2,
                                           nm2);
                    e0.x = exp2_ftz(e0.x);
                    e0.y = exp2_ftz(e0.y);
                    e1.x = exp2_ftz(e1.x);
                    e1.y = exp2_ftz(e1.y);
                    sa = __fadd2_rn(sa, e0);
                    sb = __fadd2_rn(sb, e1);
                    w[i / 2] = pack_bf16x2(e0.x, e0.y);
                    w[i / 2 + 1] = pack_bf16x2(e1.x, e1.y);
                }
                tmem_store_32x32b_x16(p_tmem + 16 * b, w);
            }
            if (rescale) {
                const float alpha = exp2_ftz(m - m_use);
                if (j > 0) {
                    // This half's 32 columns of O_t *= alpha (alpha = 1 for rows whose max did not grow).
                    uint32_t o[32];
                    tmem_load_32x32b_x32(o_tmem, o);
                    tmem_load_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_store_32x32b_x32(o_tmem, o);
                }
                l *= alpha;
                m = m_use;
            }
            l += (sa.x + sa.y) + (sb.x + sb.y);
            tmem_store_wait();           // P_t (and O_t) stores complete before the product that reads them
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&p_full[t]));
        }
        // Final sums: both halves' l, and whether both saw the last product finish.
        bool done = ok && tsteps > 0 && warp_wait(smem_addr(&o_done[t]), (tsteps - 1) & 1);
        if (ok) {
            // (A pair that left its loop on a timeout skips this exchange together.) The slot of parity tsteps & 1
            // was last read by the partner before the final step's barrier, so it may be overwritten now.
            const int slot = tsteps & 1;
            xmax[((slot * 2 + t) * 2 + h) * FA_BM + r] = l;
            if (lane == 0) xflag[((slot * 2 + t) * 2 + h) * 4 + q] = done ? 1 : 0;
            pair_barrier(pair_bar);
            const float l_row = l + xmax[((slot * 2 + t) * 2 + (h ^ 1)) * FA_BM + r];
            done = done && xflag[((slot * 2 + t) * 2 + (h ^ 1)) * 4 + q] != 0;
            if (done) {
                tcgen05_fence_after_sync();
                const float inv = 1.0f / l_row;
                const bool live = query < p.sq;
                const int64_t base = static_cast<int64_t>(matrix) * p.out_stride + query * FA_D + 32 * h;
                uint32_t o[32];
                tmem_load_32x32b_x32(o_tmem, o);
                tmem_load_wait();
                if (live) {
                    if (p.out_bf16) {
                        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base);
#pragma unroll
                        for (int g = 0; g < 4; ++g)
                            dst[g] = make_uint4(
                                pack_bf16x2(__uint_as_float(o[8 * g]) * inv, __uint_as_float(o[8 * g + 1]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv));
                    } else {
                        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + base);
#pragma unroll
                        for (int g = 0; g < 8; ++g)
                            dst[g] = make_float4(__uint_as_float(o[4 * g]) * inv, __uint_as_float(o[4 * g + 1]) * inv,
                                                 __uint_as_float(o[4 * g + 2]) * inv, __uint_as_float(o[4 * g + 3]) * inv);
                    }
                    if (h == 0 && p.lse != nullptr)
                        p.lse[static_cast<int64_t>(matrix) * p.sq + query] = (m + __log2f(l_row)) * 0.69314718f;
                }
            }
        }
    }

    tcgen05_fence_before_sync();
    __syncthreads();
    if (warp == FA_MMA_WARP) {
        tcgen05_fence_after_sync();
        tmem_dealloc(tmem_base, FA_TMEM_COLS);
    }
}

}  // namespace snb
