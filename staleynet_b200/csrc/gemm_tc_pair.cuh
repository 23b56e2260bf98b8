// gemm_tc_pair.cuh — the tensor-core GEMM on CTA pairs: one tcgen05.mma.cta_group::2 computes a 256 x 256 tile
// for a cluster of two CTAs (one per SM). Each CTA stages its own 128 rows of A and its own 128 columns of B, so a
// K slice costs each SM 32 KB of L2 traffic instead of the 48 KB of a 128 x 256 single-CTA tile: a third less
// L2 -> SM traffic per FLOP, which is what limits the single-CTA kernel's main loop on B200.
//
// Roles per CTA (320 threads, as the single-CTA kernel):
//   warp 0     TMA producer in both CTAs: loads this CTA's A rows and B columns into its ring (4-6 stages by
//              staging mode); the completion bytes of both CTAs are counted on the first CTA's `full` barrier
//              (cta_group::2 loads). In SB kernels it also copies each tile's 256 bias values into this CTA's
//              shared memory (two buffers, local barriers), as in the single-CTA kernel.
//   warp 1     allocates / frees the pair's TMEM (cta_group::2) in both CTAs; in the first CTA one elected thread
//              issues the pair MMAs and commits each ring slot back to both CTAs' `empty` barriers and each
//              finished accumulator to both CTAs' `acc_full` barriers (one plain commit per CTA).
//   warps 2-9  epilogue in both CTAs, on this CTA's 128 rows x 256 columns of the accumulator (same code as the
//              single-CTA kernel); every warp of both CTAs arrives on the first CTA's `acc_empty` barrier.
#pragma once

#include "gemm_tc.cuh"

namespace snb {

constexpr int TC2_BM = 256;  // rows per CTA pair (128 per CTA)
constexpr int TC2_BN = 256;  // columns per pair tile (128 staged per CTA)

// NBOX = staging boxes per epilogue warp, as in the single-CTA kernel: two boxes (GELU epilogues) cost one ring
// stage. SB = the tile's bias staged in shared memory (each CTA holds its own copy of the tile's 256 values per
// accumulator), which costs one more stage.
template <int NBOX, bool SB = false>
struct Tc2Config {
    static constexpr int STAGE_A = 128 * 128;
    static constexpr int STAGE_B = (TC2_BN / 2) * 128;
    static constexpr int STAGE = STAGE_A + STAGE_B;
    static constexpr int EPI_BYTES = TC_EPI_WARPS * NBOX * TC_EPI_BOX_BYTES;
    static constexpr int BIAS_BYTES = SB ? 2 * TC2_BN * 4 : 0;
    static constexpr int TMEM_COLS = 2 * TC2_BN;
    static constexpr int BARRIER_BYTES = 512;
    static constexpr int BASE_STAGES = NBOX == 2 ? 5 : 6;
    static constexpr int FIT_STAGES = (TC_SMEM_LIMIT - 1024 - EPI_BYTES - BIAS_BYTES - BARRIER_BYTES) / STAGE;
    static constexpr int STAGES = BASE_STAGES < FIT_STAGES ? BASE_STAGES : FIT_STAGES;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE + EPI_BYTES + BIAS_BYTES + BARRIER_BYTES;
    static_assert(SMEM_BYTES <= TC_SMEM_LIMIT, "shared memory budget of one sm_100 CTA");
};

template <typename E, bool OUT_BF16, int EPI, bool SB = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_pre,
                        const __grid_constant__ CUtensorMap tm_res, const __grid_constant__ CUtensorMap tm_gin,
                        const __grid_constant__ CUtensorMap tm_aux, const TcParams p) {
    constexpr int NBOX = tc_epi_boxes(EPI);
    using Cfg = Tc2Config<NBOX, SB>;
    constexpr int BN = TC2_BN;
    constexpr int ESIZE = sizeof(E);
    constexpr int BK = 128 / ESIZE;
    constexpr int UMMA_K = 32 / ESIZE;
    constexpr int MN_BOX = 128 / ESIZE;
    constexpr bool IS_BF16 = ESIZE == 2;
    constexpr uint32_t FORMAT = IS_BF16 ? 1u : 2u;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* epi = smem + Cfg::STAGES * Cfg::STAGE;
    const uint32_t bias_s = smem_addr(epi + Cfg::EPI_BYTES);  // SB: two 256-float bias buffers of this CTA
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi + Cfg::EPI_BYTES + Cfg::BIAS_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + Cfg::STAGES;
    uint64_t* acc_full = bars + 2 * Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* aux_bars = drain + 1;  // two per epilogue warp
    uint64_t* bias_full = aux_bars + 2 * TC_EPI_WARPS;  // this CTA's bias feed (local barriers)
    uint64_t* bias_empty = bias_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bias_empty + 2);
    const bool feed_bias = SB && p.bias != nullptr;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_cta_rank();
    const bool leader = rank == 0;
    const int32_t first_unit = static_cast<int32_t>(blockIdx.x >> 1);
    const int32_t unit_step = static_cast<int32_t>(gridDim.x >> 1);
    griddep_launch_dependents();   // as in the single-CTA kernel

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_addr(&acc_full[a]), 1);
            mbar_init(smem_addr(&acc_empty[a]), 2 * TC_EPI_WARPS);  // every epilogue warp of both CTAs
            mbar_init(smem_addr(&bias_full[a]), 1);
            mbar_init(smem_addr(&bias_empty[a]), TC_EPI_WARPS);      // this CTA's epilogue warps
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
        tmem_alloc_pair(smem_addr(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish_alloc_permit_pair();
    }
    tcgen05_fence_before_sync();
    cluster_sync();  // both CTAs' barriers exist before either CTA signals the other's
    tcgen05_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // no global memory before the previous kernel of the stream has completed

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer (both CTAs)
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int tile = 0;
            for (TcCursor cur = tc_cursor(p, first_unit, unit_step); cur.unit < p.num_units && ok; tc_advance(p, cur)) {
                const TcUnit u = tc_cursor_unit(p, cur, BN, BK, TC2_BM);
                const int bbuf = tile & 1;
                const uint32_t bpar = ((tile >> 1) & 1) ^ 1u;
                bool bias_pending = feed_bias;
                const int32_t ba = p.a_batched ? u.batch : 0;
                const int32_t bb = p.b_batched ? u.batch : 0;
                const int32_t m0 = u.m0 + 128 * static_cast<int32_t>(rank);  // this CTA's rows
                const int32_t n0 = u.n0 + (BN / 2) * static_cast<int32_t>(rank);  // this CTA's columns of B
                if (u.split == 0) {
                    if (p.residual != nullptr) tma_prefetch_l2_3d(&tm_res, u.n0, m0, u.batch);
                    if (p.activation == 2) tma_prefetch_l2_3d(&tm_gin, u.n0, m0, u.batch);
                }
                for (int32_t kb = u.kb_begin; kb < u.kb_end; ++kb) {
                    if (!mbar_wait_cluster(smem_addr(&empty[stage]), phase ^ 1u)) { ok = false; break; }
                    const uint32_t fb_local = smem_addr(&full[stage]);
                    if (leader) mbar_arrive_expect_tx(fb_local, 2 * Cfg::STAGE);  // both CTAs' bytes
                    const uint32_t fb = map_to_cta(fb_local, 0);
                    const uint32_t sa = smem_addr(ring + stage * Cfg::STAGE);
                    const uint32_t sb = sa + Cfg::STAGE_A;
                    const int32_t k0 = kb * BK;
                    load_a_slice<BK, MN_BOX, true>(p, &tm_a, sa, fb, m0, k0, ba);
                    if (!p.b_mn_major) {
                        tma_load_3d_pair(sb, &tm_b, fb, k0, n0, bb);
                    } else {
#pragma unroll
                        for (int j = 0; j < (BN / 2) / MN_BOX; ++j)
                            tma_load_3d_pair(sb + j * (BK * 128), &tm_b, fb, n0 + j * MN_BOX, k0, bb);
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
        // ------------------------------------------------------------------ MMA issuer (first CTA)
        if (leader && elect_one()) {
            const uint32_t idesc = make_instr_desc(FORMAT, p.a_mn_major, p.b_mn_major, TC2_BM, BN);
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
            for (TcCursor cur = tc_cursor(p, first_unit, unit_step); cur.unit < p.num_units && ok; tc_advance(p, cur)) {
                const TcUnit u = tc_cursor_unit(p, cur, BN, BK, TC2_BM);
                const int acc = iter & 1;
                const uint32_t acc_phase = (iter >> 1) & 1;
                if (!mbar_wait_cluster(smem_addr(&acc_empty[acc]), acc_phase ^ 1u)) { ok = false; break; }
                tcgen05_fence_after_sync();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int32_t kb = u.kb_begin; kb < u.kb_end; ++kb) {
                    if (!mbar_wait_cluster(smem_addr(&full[stage]), phase)) { ok = false; break; }
                    tcgen05_fence_after_sync();
                    const uint32_t sa = smem_addr(ring + stage * Cfg::STAGE);
                    const uint32_t sb = sa + Cfg::STAGE_A;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        const uint64_t ad = make_smem_desc(sa + k * a_kstep, a_lbo, a_sbo, a_layout);
                        const uint64_t bd = make_smem_desc(sb + k * b_kstep, b_lbo, b_sbo, b_layout);
                        const uint32_t accumulate = (kb > u.kb_begin || k > 0) ? 1u : 0u;
                        if (IS_BF16) umma_bf16_pair(d_tmem, ad, bd, idesc, accumulate);
                        else umma_tf32_pair(d_tmem, ad, bd, idesc, accumulate);
                    }
                    issued = true;
                    const uint32_t eb = smem_addr(&empty[stage]);
                    umma_commit_pair(map_to_cta(eb, 0));
                    umma_commit_pair(map_to_cta(eb, 1));
                    if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                const uint32_t fb = smem_addr(&acc_full[acc]);
                umma_commit_pair(map_to_cta(fb, 0));
                umma_commit_pair(map_to_cta(fb, 1));
                ++iter;
            }
            if (!ok && issued) {
                umma_commit_pair(map_to_cta(smem_addr(drain), 0));
                mbar_wait(smem_addr(drain), 0);
            }
        }
        __syncwarp();
    } else if (warp >= TC_EPI_WARP0) {
        // ------------------------------------------------------------------ epilogue (both CTAs)
        const int q = warp & 3;
        const int group = (warp - TC_EPI_WARP0) >> 2;
        uint8_t* boxes = epi + (warp - TC_EPI_WARP0) * NBOX * TC_EPI_BOX_BYTES;
        uint64_t* aux_bar = aux_bars + 2 * (warp - TC_EPI_WARP0);
        constexpr bool box_aux = EPI == TC_EPI_AUX_BOX;
        const int32_t row_off = 128 * static_cast<int32_t>(rank) + q * 32;  // this warp's rows within a pair tile
        uint32_t aux_phase = 0;
        int ebox = 0;
        int iter = 0;
        TcCursor cur = tc_cursor(p, first_unit, unit_step);
        if (box_aux && lane == 0 && cur.unit < p.num_units) {
            const TcUnit u0 = tc_cursor_unit(p, cur, BN, BK, TC2_BM);
            request_aux_boxes<OUT_BF16, BN>(p, &tm_aux, u0, u0.m0 + row_off, group, boxes, aux_bar);
        }
        for (; cur.unit < p.num_units; tc_advance(p, cur)) {
            const TcUnit u = tc_cursor_unit(p, cur, BN, BK, TC2_BM);
            const int acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            if (!mbar_wait_cluster(smem_addr(&acc_full[acc]), acc_phase)) break;
            tcgen05_fence_after_sync();
            if (feed_bias && !mbar_wait(smem_addr(&bias_full[acc]), acc_phase)) break;
            const int32_t row0 = u.m0 + row_off;
            const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;

            epilogue_tile<OUT_BF16, BN, EPI, SB>(p, &tm_c, &tm_pre, u, row0, t_lane, group, boxes, ebox, aux_bar,
                                                 aux_phase, bias_s + static_cast<uint32_t>(acc * BN * 4));
            tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_cluster(map_to_cta(smem_addr(&acc_empty[acc]), 0));
                if (feed_bias) mbar_arrive(smem_addr(&bias_empty[acc]));
            }
            ++iter;
            TcCursor next = cur;
            tc_advance(p, next);
            if (box_aux && lane == 0 && next.unit < p.num_units) {
                bulk_wait_group_read<0>();
                const TcUnit un = tc_cursor_unit(p, next, BN, BK, TC2_BM);
                request_aux_boxes<OUT_BF16, BN>(p, &tm_aux, un, un.m0 + row_off, group, boxes, aux_bar);
            }
            __syncwarp();
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tcgen05_fence_before_sync();
    cluster_sync();  // both CTAs are done with the pair's TMEM and with each other's barriers
    if (warp == 1) {
        tcgen05_fence_after_sync();
        tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace snb
