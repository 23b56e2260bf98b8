// attention_fused_bwd.cuh — causal attention backward on tcgen05 without materialising the [queries, keys] scores,
// probabilities or their gradients: the backward of the reference's QK^T product, `causal_softmax` and P.V product
// (crates/staleynet-model/src/layers/attention.rs:220-267, kernels/attention.rs:182-207):
//   dP = dO V^T, dV = P^T dO, dS = P * (dP - rowsum(P * dP)), dQ = scale dS K, dK = scale dS^T Q,
// with P rebuilt per tile from the forward's log-sum-exp (P = exp(scale S - lse)) and rowsum(P * dP) taken as
// D = rowsum(dO * O), which equals it because O = P V.
//
// Two kernels:
//   fb_rowstats_kernel   per query: (-lse * log2(e), D) into a scratch buffer, one warp per query row.
//   fb_backward_kernel   one CTA of 448 threads per 128-key tile of one matrix, looping over the query tiles whose
//                        queries see any of its keys. Keys sit on the TMEM lanes:
//     warp 12      TMA: K_j, V_j once; then Q_i, dO_i and the row statistics of tile i through a 3-stage ring
//                  (K_j, V_j and the first stages requested before the CTA's set-up barrier).
//     warp 13      allocates TMEM (S^T, dP^T: 128 f32 columns each; dV, dK, dQ: 64 each; P^T: 64 columns of bf16
//                  pairs) and, on one elected thread, issues per query tile i:
//                    S^T = K_j Q_i^T, dP^T = V_j dO_i^T          (M=128 keys, N=128 queries, K=64)
//                    dV += P^T dO_i (P^T from TMEM), dK += dS^T Q_i (M=128 keys, N=64, K=128 queries)
//                    dQ_i = dS K_j                               (M=128 queries, N=64, K=128 keys)
//                  dS^T lives once in shared memory as a 128B-swizzled tile whose rows are keys: the dK product reads
//                  it K-major, the dQ product reads the same bytes M-major (queries contiguous).
//     warps 0-11   per key row (TMEM lane quadrant warp % 4) and query group (warp / 4: 48, 48 and 32 of the 128
//                  queries): P = 2^(S c + nl), dS = P (dP - D), causal and range masks applied, P^T stored bf16 into
//                  TMEM, dS^T into shared memory; at the end warps 0-3 write dV and warps 8-11 scale * dK through
//                  the dS^T buffer with TMA stores.
//     warps 4-11   also drain dQ_{i-1} after their share of tile i (queries on lanes; warps 4-7 columns 0-31, warps
//                  8-11 columns 32-63): scale it and add it into the global dQ (f32, zeroed by the host) with TMA
//                  reduce-add, each warp through its own 128B-swizzled 32x32 staging box, while dV and dK of tile i
//                  run.
// Every mbarrier wait is bounded (see sm100_ptx.cuh).
#pragma once

#include "attention_fused.cuh"

namespace snb {

constexpr int FB_BK = 128;   // keys per CTA (TMEM lanes of S^T, dP^T, dV, dK)
constexpr int FB_BQ = 128;   // queries per iteration
constexpr int FB_D = 64;
constexpr int FB_STAGES = 3;
constexpr int FB_ELEM_WARPS = 12;   // warps 0-11: P and dS; warps 4-11 also drain dQ
constexpr int FB_PRODUCER_WARP = 12;
constexpr int FB_MMA_WARP = 13;
constexpr int FB_THREADS = 14 * 32;
constexpr int FB_TMEM_COLS = 512;
constexpr int FB_S_COL = 0, FB_DP_COL = 128, FB_DV_COL = 256, FB_DK_COL = 320, FB_DQ_COL = 384, FB_P_COL = 448;

struct FbParams {
    int32_t count, sq, sk;   // matrices; queries and keys per matrix
    int32_t q_tiles;         // query tiles per matrix
    int32_t k_tiles;         // key tiles per matrix
    int32_t group;           // matrices per scheduling group (see the block order in fb_backward_kernel)
    int64_t offset;          // query q sees keys 0..=q+offset
    float scale;             // softmax scale
    float scale_log2;        // scale * log2(e)
};

struct FbSmem {
    static constexpr int KV = FB_BK * 128;          // K_j or V_j: 128 rows x 64 bf16
    static constexpr int QT = FB_BQ * 128;          // Q_i or dO_i
    static constexpr int STATS = FB_BQ * 8;         // (-lse * log2(e), D) per query
    static constexpr int STAGE = 2 * QT + STATS;    // 33 KB, a multiple of 1 KB
    static constexpr int DS = FB_BK * FB_BQ * 2;    // dS^T: two 64-query slices of 128 key rows x 128 bytes
    static constexpr int DQ = FB_BQ * FB_D * 4;     // dQ staging: per dQ warp two 32x32 f32 boxes (4 KB each)
    static constexpr int BARS = 256;
    static constexpr int BYTES = 1024 + 2 * KV + FB_STAGES * STAGE + DS + DQ + BARS;
    static_assert(STAGE % 1024 == 0, "swizzled tiles need 1 KB alignment");
    static_assert(BYTES <= 232448, "shared memory budget of one sm_100 CTA");
};

// Row statistics of the backward: stats[m, 2q] = -lse[m, q] * log2(e), stats[m, 2q + 1] = D[m, q] =
// sum_d dO[m, q, d] O[m, q, d]. One warp per (matrix, query) row; rows of stats are `stride` floats apart.
__global__ void fb_rowstats_kernel(const void* out, int32_t out_bf16, const uint16_t* d_out, const float* lse,
                                   float* stats, int64_t rows, int32_t sq, int64_t stride) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float o0, o1;
    if (out_bf16) {
        const uint32_t w = reinterpret_cast<const uint32_t*>(out)[row * 32 + lane];
        o0 = __uint_as_float(w << 16);
        o1 = __uint_as_float(w & 0xFFFF0000u);
    } else {
        const float2 f = reinterpret_cast<const float2*>(out)[row * 32 + lane];
        o0 = f.x;
        o1 = f.y;
    }
    const uint32_t g = reinterpret_cast<const uint32_t*>(d_out)[row * 32 + lane];
    float d = fmaf(__uint_as_float(g << 16), o0, __uint_as_float(g & 0xFFFF0000u) * o1);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) d += __shfl_xor_sync(0xffffffffu, d, s);
    if (lane == 0) {
        const int64_t m = row / sq, q = row % sq;
        stats[m * stride + 2 * q] = -lse[row] * 1.4426950408889634f;
        stats[m * stride + 2 * q + 1] = d;
    }
}

// fb_rowstats_kernel with eight lanes per row and 16-byte loads (out and d_out 16-byte aligned): each lane reads
// eight elements of dO and of O, so a warp keeps six times the bytes in flight of the one-warp-per-row form. The
// 64 products are summed in a different order.
__global__ void fb_rowstats_vec_kernel(const void* out, int32_t out_bf16, const uint16_t* d_out, const float* lse,
                                       float* stats, int64_t rows, int32_t sq, int64_t stride) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
    const int sub = threadIdx.x & 7;
    float d = 0.0f;
    if (row < rows) {   // every lane reaches the shuffles below
        const uint4 g = reinterpret_cast<const uint4*>(d_out + row * FB_D)[sub];
        const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
        float o[8];
        if (out_bf16) {
            const uint4 q = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(out) + row * FB_D)[sub];
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                o[2 * k] = __uint_as_float(qw[k] << 16);
                o[2 * k + 1] = __uint_as_float(qw[k] & 0xFFFF0000u);
            }
        } else {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(out) + row * FB_D) + 2 * sub;
            const float4 a = src[0], b = src[1];
            o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
            o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            d = fmaf(__uint_as_float(gw[k] << 16), o[2 * k], d);
            d = fmaf(__uint_as_float(gw[k] & 0xFFFF0000u), o[2 * k + 1], d);
        }
    }
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    if (row < rows && sub == 0) {
        const int64_t m = row / sq, q = row % sq;
        stats[m * stride + 2 * q] = -lse[row] * 1.4426950408889634f;
        stats[m * stride + 2 * q + 1] = d;
    }
}

__global__ void __launch_bounds__(FB_THREADS, 1)
    fb_backward_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_stats, const __grid_constant__ CUtensorMap tm_dq,
                       const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                       const FbParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* k_s = smem;
    uint8_t* v_s = k_s + FbSmem::KV;
    uint8_t* stage_s = v_s + FbSmem::KV;                        // FB_STAGES x (Q_i, dO_i, stats)
    uint8_t* ds_s = stage_s + FB_STAGES * FbSmem::STAGE;
    uint8_t* dq_s = ds_s + FbSmem::DS;
    uint64_t* bars = reinterpret_cast<uint64_t*>(dq_s + FbSmem::DQ);
    uint64_t* kv_full = bars;
    uint64_t* qdo_full = bars + 1;                // [FB_STAGES]
    uint64_t* qdo_empty = qdo_full + FB_STAGES;   // [FB_STAGES]
    uint64_t* sdp_full = qdo_empty + FB_STAGES;   // S^T and dP^T computed
    uint64_t* sdp_empty = sdp_full + 1;           // ... and read by the elementwise warps
    uint64_t* pds_full = sdp_empty + 1;           // P^T (TMEM) and dS^T (shared) written
    uint64_t* pds_empty = pds_full + 1;           // ... and read by the dV, dK, dQ products
    uint64_t* dq_full = pds_empty + 1;
    uint64_t* dq_empty = dq_full + 1;
    uint64_t* acc_done = dq_empty + 1;            // every product finished: dK, dV final
    uint64_t* drain = acc_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Block order: matrices in groups of p.group, and within a group the longest key tiles first (key tile 0 of
    // every matrix of the group is seen by the most query tiles). The CTAs running at one time then share a few
    // matrices, whose Q, dO and dQ (re-read or reduced into once per key tile) stay in L2, while the short tiles
    // of each group still come last.
    const int32_t per_group = p.group * p.k_tiles;
    const int32_t grp = static_cast<int32_t>(blockIdx.x / per_group);
    const int32_t in_group = static_cast<int32_t>(blockIdx.x % per_group);
    const int32_t gsz = min(p.group, p.count - grp * p.group);   // the last group may hold fewer matrices
    const int32_t key_tile = in_group / gsz;
    const int32_t matrix = grp * p.group + in_group % gsz;
    const int32_t key0 = key_tile * FB_BK;
    // Query tiles with a query q >= key0 - offset (a query that sees some key of this tile), if any query does.
    const int64_t q_lo = static_cast<int64_t>(key0) - p.offset;
    const int32_t i_first = q_lo <= 0 ? 0 : static_cast<int32_t>(q_lo / FB_BQ);
    const int32_t n_iter = q_lo > static_cast<int64_t>(p.sq) - 1 ? 0 : p.q_tiles - i_first;

    // The producer starts K, V and the first Q, dO stages before the CTA-wide barrier: it prefetches the tensor
    // maps, initialises the barriers of its own loads and issues them, so that they overlap the other barriers'
    // set-up and the TMEM allocation.
    bool producer = false;
    if (warp == FB_PRODUCER_WARP) producer = elect_one();
    int pstage = 0;
    uint32_t pphase = 0;
    int32_t pn = 0;   // query tiles whose Q, dO and statistics are requested
    auto load_stage = [&](int32_t n) {
        const int32_t q0 = (i_first + n) * FB_BQ;
        const uint32_t fb = smem_addr(&qdo_full[pstage]);
        uint8_t* st = stage_s + pstage * FbSmem::STAGE;
        mbar_arrive_expect_tx(fb, FbSmem::STAGE);
        tma_load_3d(smem_addr(st), &tm_q, fb, 0, q0, matrix);
        tma_load_3d(smem_addr(st + FbSmem::QT), &tm_do, fb, 0, q0, matrix);
        tma_load_3d(smem_addr(st + 2 * FbSmem::QT), &tm_stats, fb, 2 * q0, matrix, 0);
        if (++pstage == FB_STAGES) { pstage = 0; pphase ^= 1u; }
    };
    if (producer) {
        for (const CUtensorMap* m : {&tm_k, &tm_v, &tm_q, &tm_do, &tm_stats, &tm_dq, &tm_dk, &tm_dv})
            tma_prefetch_descriptor(m);
        mbar_init(smem_addr(kv_full), 1);
        for (int s = 0; s < FB_STAGES; ++s) {
            mbar_init(smem_addr(&qdo_full[s]), 1);
            mbar_init(smem_addr(&qdo_empty[s]), 1);
        }
        fence_mbarrier_init();
        if (n_iter > 0) {
            const uint32_t kb = smem_addr(kv_full);
            mbar_arrive_expect_tx(kb, 2 * FbSmem::KV);
            tma_load_3d(smem_addr(k_s), &tm_k, kb, 0, key0, matrix);
            tma_load_3d(smem_addr(v_s), &tm_v, kb, 0, key0, matrix);
            for (; pn < n_iter && pn < FB_STAGES; ++pn) load_stage(pn);   // the ring starts empty
        }
    }
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(sdp_full), 1);
        mbar_init(smem_addr(sdp_empty), FB_ELEM_WARPS);
        mbar_init(smem_addr(pds_full), FB_ELEM_WARPS);
        mbar_init(smem_addr(pds_empty), 1);
        mbar_init(smem_addr(dq_full), 1);
        mbar_init(smem_addr(dq_empty), 8);   // the eight draining warps (groups 1 and 2) have loaded dQ
        mbar_init(smem_addr(acc_done), 1);
        mbar_init(smem_addr(drain), 1);
        fence_mbarrier_init();
        fence_proxy_async_shared();
    }
    if (warp == FB_MMA_WARP) {
        tmem_alloc(smem_addr(tmem_slot), FB_TMEM_COLS);
        tmem_relinquish_alloc_permit();
    }
    tcgen05_fence_before_sync();
    __syncthreads();
    tcgen05_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == FB_PRODUCER_WARP) {
        // ------------------------------------------------------------------ TMA producer: the remaining stages
        if (producer) {
            for (; pn < n_iter; ++pn) {
                if (!mbar_wait(smem_addr(&qdo_empty[pstage]), pphase ^ 1u)) break;
                load_stage(pn);
            }
        }
        __syncwarp();
    } else if (warp == FB_MMA_WARP) {
        // ------------------------------------------------------------------ MMA issuer
        if (elect_one()) {
            constexpr uint32_t idesc_s = make_instr_desc(1u, 0u, 0u, FB_BK, FB_BQ);   // K-major x K-major
            constexpr uint32_t idesc_kv = make_instr_desc(1u, 0u, 1u, FB_BK, FB_D);   // K-major x N-major
            constexpr uint32_t idesc_q = make_instr_desc(1u, 1u, 1u, FB_BQ, FB_D);    // M-major x N-major
            const uint32_t ks = smem_addr(k_s), vs = smem_addr(v_s), dss = smem_addr(ds_s);
            bool ok = n_iter == 0 || mbar_wait(smem_addr(kv_full), 0);
            bool issued = false;
            // S^T(n) = K_j Q_i^T and dP^T(n) = V_j dO_i^T for the tile in `stage`.
            auto issue_scores = [&](int st) {
                const uint32_t qs = smem_addr(stage_s + st * FbSmem::STAGE);
                const uint32_t dos = qs + FbSmem::QT;
                tcgen05_fence_after_sync();
#pragma unroll
                for (int k = 0; k < FB_D / 16; ++k) {
                    umma_bf16(tmem_base + FB_S_COL, make_smem_desc(ks + 32 * k, 16, 1024, SNB_LAYOUT_SWIZZLE_128B),
                              make_smem_desc(qs + 32 * k, 16, 1024, SNB_LAYOUT_SWIZZLE_128B), idesc_s, k > 0 ? 1u : 0u);
                    umma_bf16(tmem_base + FB_DP_COL, make_smem_desc(vs + 32 * k, 16, 1024, SNB_LAYOUT_SWIZZLE_128B),
                              make_smem_desc(dos + 32 * k, 16, 1024, SNB_LAYOUT_SWIZZLE_128B), idesc_s, k > 0 ? 1u : 0u);
                }
                issued = true;
                umma_commit(smem_addr(sdp_full));
            };
            int stage = 0;
            uint32_t phase = 0;
            if (ok && n_iter > 0) {
                ok = mbar_wait(smem_addr(&qdo_full[0]), 0);
                if (ok) issue_scores(0);
            }
            for (int32_t n = 0; n < n_iter && ok; ++n) {
                const int next_stage = stage + 1 == FB_STAGES ? 0 : stage + 1;
                const uint32_t next_phase = next_stage == 0 ? phase ^ 1u : phase;
                // The next tile's scores as soon as the elementwise warps hold this tile's in registers, so that
                // they overlap this tile's remaining products.
                if (n + 1 < n_iter) {
                    if (!mbar_wait(smem_addr(sdp_empty), n & 1) ||
                        !mbar_wait(smem_addr(&qdo_full[next_stage]), next_phase)) { ok = false; break; }
                    issue_scores(next_stage);
                }
                const uint32_t qs = smem_addr(stage_s + stage * FbSmem::STAGE);
                const uint32_t dos = qs + FbSmem::QT;
                if (!mbar_wait(smem_addr(pds_full), n & 1)) { ok = false; break; }
                tcgen05_fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < FB_BQ / 16; ++kk) {
                    // dV += P^T dO_i: queries 16kk..16kk+15 of P^T are TMEM columns 8kk..8kk+7.
                    umma_bf16_tmem_a(tmem_base + FB_DV_COL, tmem_base + FB_P_COL + 8 * kk,
                                     make_smem_desc(dos + kk * 2048, FbSmem::QT, 1024, SNB_LAYOUT_SWIZZLE_128B), idesc_kv,
                                     (n > 0 || kk > 0) ? 1u : 0u);
                    // dK += dS^T Q_i: dS^T K-major (queries contiguous, 64-query slices 16 KB apart).
                    umma_bf16(tmem_base + FB_DK_COL,
                              make_smem_desc(dss + (kk / 4) * (FbSmem::DS / 2) + (kk % 4) * 32, 16, 1024,
                                             SNB_LAYOUT_SWIZZLE_128B),
                              make_smem_desc(qs + kk * 2048, FbSmem::QT, 1024, SNB_LAYOUT_SWIZZLE_128B), idesc_kv,
                              (n > 0 || kk > 0) ? 1u : 0u);
                }
                if (!mbar_wait(smem_addr(dq_empty), (n & 1) ^ 1u)) { ok = false; break; }
                tcgen05_fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < FB_BK / 16; ++kk) {
                    // dQ_i = dS K_j: dS M-major from the dS^T tile (keys 16kk.. are rows, the two 64-query slices are
                    // the M atoms 16 KB apart); K_j N-major (keys are rows).
                    umma_bf16(tmem_base + FB_DQ_COL,
                              make_smem_desc(dss + kk * 2048, FbSmem::DS / 2, 1024, SNB_LAYOUT_SWIZZLE_128B),
                              make_smem_desc(ks + kk * 2048, FbSmem::KV, 1024, SNB_LAYOUT_SWIZZLE_128B), idesc_q,
                              kk > 0 ? 1u : 0u);
                }
                umma_commit(smem_addr(dq_full));
                umma_commit(smem_addr(pds_empty));
                umma_commit(smem_addr(&qdo_empty[stage]));
                stage = next_stage;
                phase = next_phase;
            }
            if (ok) {
                if (issued) umma_commit(smem_addr(acc_done));   // after every product above
                else mbar_arrive(smem_addr(acc_done));          // no query tile sees these keys
            } else if (issued) {
                // Let every product already issued finish before TMEM is released.
                umma_commit(smem_addr(drain));
                mbar_wait(smem_addr(drain), 0);
            }
        }
        __syncwarp();
    } else if (warp < FB_ELEM_WARPS) {
        // ------------------------------------------------------------------ P and dS (one key row per thread)
        // Warp w serves TMEM lane quadrant w % 4 and query group w / 4: 16-query chunks 0-2, 3-5 or 6-7 of every
        // tile. The last group's warps also drain dQ, one tile behind, while dV and dK of the current tile run.
        const int quad = warp & 3;
        const int group = warp >> 2;
        const int ch0 = 3 * group;                 // first chunk of the group
        const int nch = group == 2 ? 2 : 3;        // chunks of the group
        const int gc0 = 16 * ch0, gw = 16 * nch;   // first query column and width of the group
        const int r = quad * 32 + lane;            // key row within the tile
        const int64_t key = static_cast<int64_t>(key0) + r;
        const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
        const uint32_t ds_row = smem_addr(ds_s + r * 128);   // row r of slice 0; slice s is DS/2 * s further
        const float c = p.scale_log2;
        // dQ is drained by groups 1 and 2, group 1 taking columns 0-31 and group 2 columns 32-63 of its quadrant's 32
        // queries: split this way the drain adds ~500 cycles to both groups instead of ~1,000 to group 2 alone, whose
        // two score chunks plus the whole drain were the longest path of a query tile.
        const bool drains = group >= 1;
        const int dq_half = group - 1;
        uint8_t* box = dq_s + quad * (FbSmem::DQ / 4) + (drains ? dq_half : 0) * (FbSmem::DQ / 8);
        // This warp's half of dQ of tile m: scale it and add it into the global dQ through its 32x32 f32 staging box.
        auto drain = [&](int32_t m) -> bool {
            if (!warp_wait(smem_addr(dq_full), m & 1)) return false;
            tcgen05_fence_after_sync();
            uint32_t da[32];
            tmem_load_32x32b_x32(tmem_base + lane_base + FB_DQ_COL + 32 * dq_half, da);
            tmem_load_wait();
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(dq_empty));
            // The staging box is free once this warp's previous reduction has read it.
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            const uint32_t row0 = smem_addr(box + lane * 128);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const uint32_t off = (g ^ (lane & 7)) << 4;
                st_shared_v4(row0 + off, __float_as_uint(__uint_as_float(da[4 * g]) * p.scale),
                             __float_as_uint(__uint_as_float(da[4 * g + 1]) * p.scale),
                             __float_as_uint(__uint_as_float(da[4 * g + 2]) * p.scale),
                             __float_as_uint(__uint_as_float(da[4 * g + 3]) * p.scale));
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
                const int32_t q0 = (i_first + m) * FB_BQ + 32 * quad;
                tma_reduce_add_3d(&tm_dq, smem_addr(box), 32 * dq_half, q0, matrix);
                bulk_commit_group();
            }
            return true;
        };
        bool ok = true;
        int stage = 0;
        uint32_t phase = 0;
        for (int32_t n = 0; n < n_iter; ++n) {
            const int64_t qg = static_cast<int64_t>(i_first + n) * FB_BQ + gc0;   // first query of this group
            // Visible columns j of this group: qg + j >= key - offset, qg + j < sq, and key < sk.
            const int64_t lo64 = key < p.sk ? key - p.offset - qg : gw;
            const int64_t hi64 = static_cast<int64_t>(p.sq) - qg;
            const int32_t lo = static_cast<int32_t>(lo64 < 0 ? 0 : (lo64 > gw ? gw : lo64));
            const int32_t hi = static_cast<int32_t>(hi64 < 0 ? 0 : (hi64 > gw ? gw : hi64));
            if (!warp_wait(smem_addr(sdp_full), n & 1) || !warp_wait(smem_addr(&qdo_full[stage]), phase)) {
                ok = false;
                break;
            }
            tcgen05_fence_after_sync();
            // (nl, D) of query 2k, 2k+1 of this group at stats + 16 k bytes, read with explicit shared loads.
            const uint32_t stats = smem_addr(stage_s + stage * FbSmem::STAGE + 2 * FbSmem::QT) + 8 * gc0;
            // Off the diagonal and the ragged edges every column of every row of the warp is visible.
            const bool unmasked = __all_sync(0xffffffffu, lo == 0 && hi == gw);
            // Scores and their gradients in 16-column chunks, the next chunk's TMEM loads in flight while this one
            // is computed.
            uint32_t s[2][16], dp[2][16];
            tmem_load_32x32b_x16(tmem_base + lane_base + FB_S_COL + gc0, s[0]);
            tmem_load_32x32b_x16(tmem_base + lane_base + FB_DP_COL + gc0, dp[0]);
            tmem_load_wait();
#pragma unroll
            for (int cc = 0; cc < 3; ++cc) {
                if (cc >= nch) break;
                const int b = cc & 1;
                const int ch = ch0 + cc;
                if (cc + 1 < nch) {
                    tmem_load_32x32b_x16(tmem_base + lane_base + FB_S_COL + 16 * (ch + 1), s[b ^ 1]);
                    tmem_load_32x32b_x16(tmem_base + lane_base + FB_DP_COL + 16 * (ch + 1), dp[b ^ 1]);
                }
                uint32_t pw[8], dw[8];
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const float4 nd = ld_shared_f4(stats + 8 * (16 * cc + j));   // (nl, D, nl, D) of columns j, j+1
                    const int col = 16 * cc + j;
                    float p0 = exp2_ftz(fmaf(__uint_as_float(s[b][j]), c, nd.x));
                    float p1 = exp2_ftz(fmaf(__uint_as_float(s[b][j + 1]), c, nd.z));
                    if (!unmasked) {
                        p0 = (col >= lo && col < hi) ? p0 : 0.0f;
                        p1 = (col + 1 >= lo && col + 1 < hi) ? p1 : 0.0f;
                    }
                    pw[j / 2] = pack_bf16x2(p0, p1);
                    dw[j / 2] = pack_bf16x2(p0 * (__uint_as_float(dp[b][j]) - nd.y),
                                            p1 * (__uint_as_float(dp[b][j + 1]) - nd.w));
                }
                if (cc == 0 && n > 0 && !warp_wait(smem_addr(pds_empty), (n - 1) & 1)) {
                    // (P^T and dS^T of the previous tile are free once its dV, dK, dQ products finished.)
                    ok = false;
                }
                if (ok) {
                    tmem_store_32x32b_x8(tmem_base + lane_base + FB_P_COL + 8 * ch, pw);
                    // dS^T row r, queries 16 ch ..: slice ch / 4, 16-byte chunks 2 (ch % 4), +1 of its 128-byte row.
                    const uint32_t row = ds_row + (ch / 4) * (FbSmem::DS / 2);
                    st_shared_v4(row + (((2 * (ch % 4)) ^ (r & 7)) << 4), dw[0], dw[1], dw[2], dw[3]);
                    st_shared_v4(row + (((2 * (ch % 4) + 1) ^ (r & 7)) << 4), dw[4], dw[5], dw[6], dw[7]);
                }
                if (cc + 1 < nch) tmem_load_wait();
                if (cc + 2 == nch) {
                    // S^T and dP^T are all in registers: the next tile's products may overwrite them.
                    tcgen05_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_addr(sdp_empty));
                }
            }
            if (!ok) break;
            tmem_store_wait();
            fence_proxy_async_shared();   // dS^T writes -> the tensor core's reads
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(pds_full));
            if (++stage == FB_STAGES) { stage = 0; phase ^= 1u; }
            if (drains && n > 0 && !drain(n - 1)) { ok = false; break; }
        }
        if (drains) {
            if (ok && n_iter > 0) ok = drain(n_iter - 1);
            // The reductions complete on their own; the CTA only has to keep its staging boxes until they are read.
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
        }
        if (group != 1 && ok && warp_wait(smem_addr(acc_done), 0)) {
            // dV (group 0) or scale * dK (group 2, whose last drain ends before group 1's) of this warp's 32 key rows
            // (zero when no query sees them), staged as two 128B-swizzled 32 x 32 f32 boxes through this warp's 4 KB
            // of the dS^T buffer (free: every product has finished) and written with TMA stores, which clip the rows
            // past the last key.
            const int h = group == 0 ? 0 : 1;
            tcgen05_fence_after_sync();
            const float mul = h == 0 ? 1.0f : p.scale;
            uint8_t* wbox = ds_s + (4 * h + quad) * 4096;
            const uint32_t wrow = smem_addr(wbox + lane * 128);
            for (int c0 = 0; c0 < FB_D; c0 += 32) {
                uint32_t o[32];
                tmem_load_32x32b_x32(tmem_base + lane_base + (h == 0 ? FB_DV_COL : FB_DK_COL) + c0, o);
                tmem_load_wait();
                if (c0 > 0) {
                    if (lane == 0) bulk_wait_group_read<0>();   // the first box has been read
                    __syncwarp();
                }
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    // (n_iter == 0: TMEM holds no product; an explicit zero keeps stale bits out.)
                    const uint32_t off = (g ^ (lane & 7)) << 4;
                    if (n_iter == 0) {
                        st_shared_v4(wrow + off, 0u, 0u, 0u, 0u);
                    } else {
                        st_shared_v4(wrow + off, __float_as_uint(__uint_as_float(o[4 * g]) * mul),
                                     __float_as_uint(__uint_as_float(o[4 * g + 1]) * mul),
                                     __float_as_uint(__uint_as_float(o[4 * g + 2]) * mul),
                                     __float_as_uint(__uint_as_float(o[4 * g + 3]) * mul));
                    }
                }
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(h == 0 ? &tm_dv : &tm_dk, smem_addr(wbox), c0, key0 + 32 * quad, matrix);
                    bulk_commit_group();
                }
            }
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
        }
    }

    tcgen05_fence_before_sync();
    __syncthreads();
    if (warp == FB_MMA_WARP) {
        tcgen05_fence_after_sync();
        tmem_dealloc(tmem_base, FB_TMEM_COLS);
    }
}

}  // namespace snb
