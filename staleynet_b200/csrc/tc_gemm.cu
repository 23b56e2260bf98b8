// tc_gemm.cu — host side of the tcgen05 GEMM: eligibility (TMA needs a unit stride and 16-byte aligned strides),
// tensor-map encoding, tile-width and split-K choice, and the launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <utility>
#include <mutex>

#include "attention_fused.cuh"
#include "attention_fused_bwd.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc_pair.cuh"
#include "internal.h"

namespace snb {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// How one operand is read: `mn_major` = the M (or N) index is contiguous; `ld` = elements between consecutive
// rows of the other index; `batched` = distinct matrix per batch entry.
struct OperandLayout {
    bool ok;
    bool mn_major;
    uint64_t ld;
    bool batched;
};

// Decides the layout of an operand with logical extents (mn, k): element (i, kk) at
// b*batch + i*mn_stride + kk*k_stride.
OperandLayout classify(uint64_t mn, uint64_t k, uint64_t mn_stride, uint64_t k_stride, uint64_t batch_stride,
                       uint64_t count, int esize, const void* base) {
    OperandLayout L{false, false, 0, false};
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return L;
    // The contiguous dimension must have more than one element; with a single row the other stride is never
    // used for addressing, so it is replaced by the row length.
    if (k > 1 && k_stride == 1) {
        L.mn_major = false;
        L.ld = (mn == 1) ? k : mn_stride;
        if (L.ld < k) return L;
    } else if (mn > 1 && mn_stride == 1) {
        L.mn_major = true;
        L.ld = (k == 1) ? mn : k_stride;
        if (L.ld < mn) return L;
    } else {
        return L;  // no unit stride (or a 1x1 matrix): the SIMT kernel handles it
    }
    const uint64_t outer = L.mn_major ? k : mn;
    if (outer == 1) L.ld = ((L.ld * esize + 15) / 16) * 16 / esize;  // pad the unused stride to 16 bytes
    if ((L.ld * esize) % 16 != 0) return L;
    L.batched = count > 1 && batch_stride != 0;
    if (L.batched) {
        if ((batch_stride * esize) % 16 != 0) return L;
        if (batch_stride < L.ld * outer) return L;
    }
    L.ok = true;
    return L;
}

bool encode_3d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t d0, uint64_t d1,
               uint64_t d2, uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box0, uint32_t box1,
               std::string* err, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
        return false;
    }
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {stride1_elems * esize, stride2_elems * esize};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
        return false;
    }
    return true;
}

// A tiled map of rank 4 or 5 (head-major operands): dims[0] contiguous, strides in elements for dims 1.., box
// extents per dim.
bool encode_nd(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, int rank, const uint64_t* dims,
               const uint64_t* strides_elems, const uint32_t* box, std::string* err,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
        return false;
    }
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t b[5];
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        if (i > 0) st[i - 1] = strides_elems[i - 1] * esize;
    }
    CUresult r = fn(map, dt, rank, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled (rank " + std::to_string(rank) + ") failed with CUresult " +
               std::to_string(static_cast<int>(r));
        return false;
    }
    return true;
}

// Launches a GEMM kernel with programmatic stream serialisation: its CTAs may be scheduled while the previous
// kernel of the stream finishes (the kernels call griddepcontrol.wait before touching global memory, and let their
// own dependents start early with griddepcontrol.launch_dependents), so the set-up of one GEMM (barriers, TMEM,
// tensor-map prefetch) overlaps the tail of the one before.
template <typename... KArgs, typename... Args>
cudaError_t launch_with_dependents(void (*kernel)(KArgs...), int grid, int threads, int smem, cudaStream_t stream,
                                   Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename E, int BN, bool OUT_BF16, int EPI, bool SB = false>
int launch(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
           const CUtensorMap& tp, const CUtensorMap& tr, const CUtensorMap& tg, const CUtensorMap& tx,
           const TcParams& p, int grid, std::string* err) {
    constexpr int smem = TcConfig<BN, tc_epi_boxes(EPI), SB>::SMEM_BYTES;
    static int configured_device = -1;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(mu);
        // cudaFuncSetAttribute is per device; redo it when the current device changes.
        if (configured_device != dev) {
            cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<E, BN, OUT_BF16, EPI, SB>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) {
                *err = cuda_message("cudaFuncSetAttribute(tc_gemm_kernel)", e);
                return SNB_ERR_CUDA;
            }
            configured_device = dev;
        }
    }
    cudaError_t e = launch_with_dependents(tc_gemm_kernel<E, BN, OUT_BF16, EPI, SB>, grid, TC_THREADS, smem, stream,
                                           ta, tb, tc, tp, tr, tg, tx, p);
    if (e != cudaSuccess) {
        *err = cuda_message("tc_gemm_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

// Narrow tiles (BN 64, 128) always stage through two boxes; BN = 256 tiles take the staging mode `epi` (two-box
// modes cost one of the four ring stages). The auxiliary-box mode exists for bf16 outputs of bf16 products only.
template <typename E, bool OUT_BF16>
int launch_bn(int bn, int epi, cudaStream_t s, const CUtensorMap* m, const TcParams& p, int grid, std::string* err) {
#define SNB_LAUNCH(BN_, EPI_) launch<E, BN_, OUT_BF16, EPI_>(s, m[0], m[1], m[2], m[3], m[4], m[5], m[6], p, grid, err)
    if (bn == 64) return SNB_LAUNCH(64, TC_EPI_TWO_BOX);
    if (bn == 128) return SNB_LAUNCH(128, TC_EPI_TWO_BOX);
    if constexpr (OUT_BF16 && sizeof(E) == 2) {
        if (epi == TC_EPI_AUX_BOX) return SNB_LAUNCH(256, TC_EPI_AUX_BOX);
    }
    if (epi == TC_EPI_ONE_BOX) return SNB_LAUNCH(256, TC_EPI_ONE_BOX);
    return SNB_LAUNCH(256, TC_EPI_TWO_BOX);
#undef SNB_LAUNCH
}

template <typename E, bool OUT_BF16, int EPI, bool SB = false>
int launch_pair(cudaStream_t stream, const CUtensorMap* m, const TcParams& p, int grid, std::string* err) {
    constexpr int smem = Tc2Config<tc_epi_boxes(EPI), SB>::SMEM_BYTES;
    static int configured_device = -1;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(mu);
        if (configured_device != dev) {
            cudaError_t e = cudaFuncSetAttribute(tc_gemm_pair_kernel<E, OUT_BF16, EPI, SB>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) {
                *err = cuda_message("cudaFuncSetAttribute(tc_gemm_pair_kernel)", e);
                return SNB_ERR_CUDA;
            }
            configured_device = dev;
        }
    }
    cudaError_t e = launch_with_dependents(tc_gemm_pair_kernel<E, OUT_BF16, EPI, SB>, grid, TC_THREADS, smem, stream,
                                           m[0], m[1], m[2], m[3], m[4], m[5], m[6], p);
    if (e != cudaSuccess) {
        *err = cuda_message("tc_gemm_pair_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

// The deterministic split-K reduction: C = (accumulate ? C : 0) + slab_0 + slab_1 + ... in that order, for C
// [n] f32 and `splits` slabs of n floats each (16-byte aligned, n a multiple of 4). Every element is summed by one
// thread in a fixed order, so the result does not depend on scheduling.
__global__ void split_slab_sum_kernel(const float4* __restrict__ slabs, int64_t slab4, int32_t splits, float4* c,
                                      int32_t accumulate, int64_t n4) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 acc = accumulate ? c[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int32_t s = 0; s < splits; ++s) {
            const float4 v = __ldcs(slabs + s * slab4 + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        c[i] = acc;
    }
}

// K splits for a problem of `tiles` output tiles and `kb` K slices on `workers` SMs (or SM pairs): minimises the
// critical path ceil(tiles*s/workers) * ceil(kb/s) (waves times slices per unit, in slice times of one worker),
// keeping at least 4 K slices per split, plus what a split costs in output traffic at HBM speed in the same units:
// every partial beyond the first is one more reduce-add into C, and an overwritten C is zeroed first.
int choose_splits(int64_t tiles, int64_t kb, int workers, double slice_flops, double worker_flops, double out_bytes,
                  bool overwrite) {
    if (kb < 8) return 1;
    constexpr double kHbmBytesPerSecond = 6.5e12;
    const double slices_per_byte = worker_flops / (kHbmBytesPerSecond * slice_flops);
    int best = 1;
    double best_cost = static_cast<double>((tiles + workers - 1) / workers) * static_cast<double>(kb);
    for (int s = 2; s <= 32; ++s) {
        const int64_t per = (kb + s - 1) / s;
        if (per < 4) break;
        const double extra = slices_per_byte * out_bytes * static_cast<double>((s - 1) + (overwrite ? 1 : 0));
        const double cost = static_cast<double>((tiles * s + workers - 1) / workers) * static_cast<double>(per) + extra;
        if (cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

}  // namespace

int tc_gemm_try(cudaStream_t stream, const GemmRequest& r, bool* launched, int* path, std::string* err) {
    *launched = false;
    *path = SNB_PATH_TENSOR_CORE;
    const snb_product& p = r.p;
    if (p.inner == 0 || p.rows == 0 || p.cols == 0) return SNB_OK;
    if (r.precision != SNB_PRECISION_TF32 && r.precision != SNB_PRECISION_BF16) return SNB_OK;
    const bool bf16_in = r.a_type == SNB_TYPE_BF16;
    if (bf16_in != (r.precision == SNB_PRECISION_BF16)) return SNB_OK;
    const bool out_bf16 = r.c_type == SNB_TYPE_BF16;
    if (!bf16_in && out_bf16) return SNB_OK;  // f32 operands run with an f32 output only
    // 32-bit tile coordinates.
    const uint64_t lim = (1ull << 31) - 256;
    if (p.rows > lim || p.cols > lim || p.inner > lim || r.count > lim) return SNB_OK;

    DeviceInfo dev;
    int rc = current_device_info(&dev, err);
    if (rc != SNB_OK) return rc;
    if (dev.major != 10) return SNB_OK;  // the tcgen05 kernels are built for sm_100a only

    const int esize = bf16_in ? 2 : 4;
    const OperandLayout la = classify(p.rows, p.inner, p.left.row_stride, p.left.col_stride, p.left.batch_stride,
                                      r.count, esize, r.A);
    const OperandLayout lb = classify(p.cols, p.inner, p.right.col_stride, p.right.row_stride, p.right.batch_stride,
                                      r.count, esize, r.B);
    if (!la.ok || !lb.ok) return SNB_OK;
    // Head-major operands (checked against the product by snb_gemm): the TMA boxes must not straddle a head or a
    // sequence. A K-major A box is BK features x 128 tokens, an MN-major one MN_BOX features x BK tokens; an output
    // box is 64 (bf16) or 32 (f32) columns x 32 rows.
    const snb_head_layout* ah = r.a_heads;
    const snb_head_layout* ch = r.c_heads;
    if (ah != nullptr) {
        const uint64_t need_hd = 128 / esize;  // BK or MN_BOX elements (128 bytes)
        const uint64_t need_time = la.mn_major ? 128 / esize : TC_BM;
        if (r.count != 1 || ah->head_dim % need_hd != 0 || ah->time % need_time != 0) {
            *err = "head-major left operand: needs count 1, head_dim a multiple of " + std::to_string(need_hd) +
                   " and time a multiple of " + std::to_string(need_time) + " for this storage";
            return SNB_OK;
        }
    }
    if (ch != nullptr) {
        const uint64_t chunk_cols = r.c_type == SNB_TYPE_BF16 ? 64 : 32;
        if (r.count != 1 || p.accumulate != 0 || r.residual != nullptr || r.gelu_input != nullptr ||
            r.pre != nullptr || r.causal != SNB_CAUSAL_NONE || ch->head_dim % chunk_cols != 0 || ch->time % 32 != 0) {
            *err = "head-major output: needs count 1, an overwrite without residual, GELU input or pre-activation, "
                   "head_dim a multiple of " + std::to_string(chunk_cols) + " and time a multiple of 32";
            return SNB_OK;
        }
    }

    // Output (and every tensor laid out like it): row-major [rows, cols] with rows `cols` apart.
    const int csize = out_bf16 ? 2 : 4;
    if ((p.cols * csize) % 16 != 0) return SNB_OK;
    if (reinterpret_cast<uintptr_t>(r.C) % 16 != 0) return SNB_OK;
    if (r.pre && reinterpret_cast<uintptr_t>(r.pre) % 16 != 0) return SNB_OK;
    if (r.pre && r.aux_type != r.c_type) return SNB_OK;
    // The epilogue reads bias, residual and GELU input with 16-byte vector loads: every row start must be
    // 16-byte aligned.
    const int aux_size = r.aux_type == SNB_TYPE_BF16 ? 2 : 4;
    if (r.bias && reinterpret_cast<uintptr_t>(r.bias) % 16 != 0) return SNB_OK;
    if (r.residual && reinterpret_cast<uintptr_t>(r.residual) % 16 != 0) return SNB_OK;
    if (r.gelu_input && (reinterpret_cast<uintptr_t>(r.gelu_input) % 16 != 0 || (p.cols * aux_size) % 16 != 0 ||
                         (r.count > 1 && (p.output_batch_stride * aux_size) % 16 != 0)))
        return SNB_OK;
    const bool c_batched = r.count > 1;
    if (c_batched && ((p.output_batch_stride * csize) % 16 != 0 || p.output_batch_stride < p.rows * p.cols))
        return SNB_OK;

    const int bn = p.cols <= 64 ? 64 : (p.cols <= 128 ? 128 : 256);
    const int bk = 128 / esize;
    // Tall products wider than 128 columns run on CTA pairs (256 x 256 tiles, a third less L2 traffic per FLOP, and a
    // 6-stage ring that covers the longer load latency while output stores are in flight) when K is long, and for
    // bf16 products also when they are at most 1,024 columns wide. Measured on the training step's K=768 shapes:
    // pairs are 3-7 % faster at 768 columns (output.fwd, output.dX) but 3-7 % slower at 2,304 and 3,072 (project.dX;
    // qkv.fwd and expand.fwd too while each epilogue warp read the bias from global memory), where the pair's main
    // loop waits for the slower of two epilogues. The causal attention hints are implemented by the single-CTA
    // kernel only.
    constexpr int64_t kPairMinKBytes = 4096;  // K >= 2048 bf16 / 1024 f32
    constexpr int64_t kPairMaxNarrowCols = 1024;
    // SMs the persistent grid may occupy: all of them, or the caller's budget (which leaves the rest to kernels on
    // other streams, e.g. a collective running beside the backward pass).
    const int sms = r.sm_budget > 0 ? std::min(r.sm_budget, dev.sm_count) : dev.sm_count;
    // A short-K bf16 product with a bias and a bf16 output runs on pairs with the bias staged in shared memory (SB
    // kernels, one ring stage fewer). Long-K products keep the deeper ring and read the bias from global memory.
    const bool bias_pair = bf16_in && out_bf16 && r.bias != nullptr &&
                           static_cast<int64_t>(p.inner) * esize < kPairMinKBytes;
    // TF32 products move twice the operand bytes per FLOP of bf16 ones while their epilogue stays the same, so pairs
    // pay at every K except where the epilogue reads an f32 GELU input row by row (project.dX): measured on the
    // step's K=768 shapes, qkv.fwd +18 %, head.fwd +24 %, output.dX +18 %, expand.fwd +4 %, project.dX -8 %.
    const bool tf32_pair = !bf16_in && r.activation != SNB_ACTIVATION_GELU_GRAD;
    const bool pair = bn == 256 && p.rows > TC_BM && r.causal == SNB_CAUSAL_NONE && sms >= 2 &&
                      (tf32_pair || static_cast<int64_t>(p.inner) * esize >= kPairMinKBytes ||
                       (bf16_in && static_cast<int64_t>(p.cols) <= kPairMaxNarrowCols) || bias_pair);
    const int bm = pair ? TC2_BM : TC_BM;
    const int workers = pair ? sms / 2 : sms;
    const int64_t m_tiles = (p.rows + bm - 1) / bm;
    const int64_t n_tiles = (p.cols + bn - 1) / bn;
    const int64_t k_blocks = (p.inner + bk - 1) / bk;
    const int64_t tiles = static_cast<int64_t>(r.count) * m_tiles * n_tiles;
    if (tiles > (1ll << 30)) return SNB_OK;
    const bool plain_epilogue = !out_bf16 && r.activation == SNB_ACTIVATION_NONE && r.pre == nullptr &&
                                r.causal == SNB_CAUSAL_NONE && ch == nullptr;
    // Tensor rate of one worker (one SM, or an SM pair) and the FLOPs of one K slice of one tile.
    const double sm_flops = (bf16_in ? 8192.0 : 4096.0) * 1.8e9;
    const double slice_flops = 2.0 * bm * bn * bk;
    const double out_bytes = static_cast<double>(r.count) * static_cast<double>(p.rows) * static_cast<double>(p.cols) *
                             static_cast<double>(csize);
    // The deterministic mode gives each split its own workspace slab (count 1 only): a split then costs its output
    // bytes twice (slab store, then the ordered sum's read), and C is read and written once more.
    const bool slab_mode = r.deterministic && r.count == 1;
    const int splits = plain_epilogue && (!r.deterministic || slab_mode)
                           ? choose_splits(tiles, k_blocks, workers, slice_flops, pair ? 2.0 * sm_flops : sm_flops,
                                           slab_mode ? 2.0 * out_bytes : out_bytes, slab_mode || p.accumulate == 0)
                           : 1;
    const int64_t kb_per_split = (k_blocks + splits - 1) / splits;
    const int64_t splits_used = (k_blocks + kb_per_split - 1) / kb_per_split;  // every split has >= 1 slice
    const bool slabs = slab_mode && splits_used > 1;

    CUtensorMap maps[7];
    CUtensorMap &ta = maps[0], &tb = maps[1], &tc = maps[2], &tp = maps[3], &tr = maps[4], &tg = maps[5],
                &tx = maps[6];
    const CUtensorMapDataType in_dt = bf16_in ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_TFLOAT32;
    const uint32_t mn_box = 128 / esize;
    // MN-major tf32 slices use 32-byte swizzle atoms (the only MN-major layout the tensor core reads for 32-bit
    // operands); everything else 16-byte atoms.
    const CUtensorMapSwizzle mn_swizzle = bf16_in ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    // A: (mn = rows, k = inner)
    if (ah != nullptr) {
        // [batch, heads, capacity, head_dim] -> dims (head_dim, capacity, heads, batch)
        const uint64_t dims[4] = {ah->head_dim, ah->time_capacity, ah->heads, ah->batch};
        const uint64_t strides[3] = {ah->head_dim, ah->time_capacity * ah->head_dim,
                                     ah->heads * ah->time_capacity * ah->head_dim};
        const uint32_t box_k[4] = {static_cast<uint32_t>(bk), TC_BM, 1, 1};
        const uint32_t box_mn[4] = {mn_box, static_cast<uint32_t>(bk), 1, 1};
        if (!encode_nd(&ta, in_dt, esize, r.A, 4, dims, strides, la.mn_major ? box_mn : box_k, err,
                       la.mn_major ? mn_swizzle : CU_TENSOR_MAP_SWIZZLE_128B))
            return SNB_OK;
    } else if (la.mn_major) {
        if (!encode_3d(&ta, in_dt, esize, r.A, p.rows, p.inner, la.batched ? r.count : 1, la.ld,
                       la.batched ? p.left.batch_stride : la.ld * p.inner, mn_box, bk, err, mn_swizzle))
            return SNB_OK;
    } else {
        if (!encode_3d(&ta, in_dt, esize, r.A, p.inner, p.rows, la.batched ? r.count : 1, la.ld,
                       la.batched ? p.left.batch_stride : la.ld * p.rows, bk, TC_BM, err))
            return SNB_OK;
    }
    // B: (mn = cols, k = inner)
    if (lb.mn_major) {
        if (!encode_3d(&tb, in_dt, esize, r.B, p.cols, p.inner, lb.batched ? r.count : 1, lb.ld,
                       lb.batched ? p.right.batch_stride : lb.ld * p.inner, mn_box, bk, err, mn_swizzle))
            return SNB_OK;
    } else {
        if (!encode_3d(&tb, in_dt, esize, r.B, p.inner, p.cols, lb.batched ? r.count : 1, lb.ld,
                       lb.batched ? p.right.batch_stride : lb.ld * p.cols, bk, static_cast<uint32_t>(pair ? bn / 2 : bn),
                       err))
            return SNB_OK;
    }
    const CUtensorMapDataType out_dt = out_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const uint32_t chunk = out_bf16 ? 64 : 32;
    const uint64_t c_bstride = c_batched ? p.output_batch_stride : p.rows * p.cols;
    // Deterministic split-K: the splits' partial tiles go to slabs [splits, rows, cols] of a stream-ordered
    // workspace, freed (stream-ordered) when this call returns, after the kernels that use it are queued.
    float* slab_base = nullptr;
    struct SlabRelease {
        float*& ptr;
        cudaStream_t stream;
        ~SlabRelease() {
            if (ptr != nullptr) cudaFreeAsync(ptr, stream);
        }
    } slab_release{slab_base, stream};
    if (slabs) {
        uint64_t slab_bytes = 0;
        if (__builtin_mul_overflow(static_cast<uint64_t>(splits_used), p.rows * p.cols * sizeof(float), &slab_bytes))
            return SNB_OK;
        cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&slab_base), slab_bytes, stream);
        if (e != cudaSuccess) {
            slab_base = nullptr;
            *err = cuda_message("cudaMallocAsync(split-K slabs)", e);
            return SNB_ERR_CUDA;
        }
        if (!encode_3d(&tc, out_dt, csize, slab_base, p.cols, p.rows, static_cast<uint64_t>(splits_used), p.cols,
                       p.rows * p.cols, chunk, 32, err))
            return SNB_OK;
    } else if (ch != nullptr) {
        // P head-major tensors [batch, heads, capacity, head_dim] side by side -> dims (head_dim, capacity, heads,
        // batch, P)
        const uint64_t per = ch->batch * ch->heads * ch->time_capacity * ch->head_dim;
        const uint64_t dims[5] = {ch->head_dim, ch->time_capacity, ch->heads, ch->batch,
                                  p.cols / (ch->heads * ch->head_dim)};
        const uint64_t strides[4] = {ch->head_dim, ch->time_capacity * ch->head_dim,
                                     ch->heads * ch->time_capacity * ch->head_dim, per};
        const uint32_t box[5] = {chunk, 32, 1, 1, 1};
        if (!encode_nd(&tc, out_dt, csize, r.C, 5, dims, strides, box, err)) return SNB_OK;
    } else if (!encode_3d(&tc, out_dt, csize, r.C, p.cols, p.rows, c_batched ? r.count : 1, p.cols, c_bstride, chunk,
                          32, err)) {
        return SNB_OK;
    }
    if (r.pre) {
        if (!encode_3d(&tp, out_dt, csize, r.pre, p.cols, p.rows, c_batched ? r.count : 1, p.cols, c_bstride, chunk,
                       32, err))
            return SNB_OK;
    } else {
        tp = tc;
    }
    // Residual and GELU-input maps serve only the L2 prefetch of each tile (box: the whole tile, no swizzle).
    const uint32_t pf_cols = static_cast<uint32_t>(std::min(bn, 256));
    tr = tc;
    tg = tc;
    if (r.residual &&
        !encode_3d(&tr, out_dt, csize, r.residual, p.cols, p.rows, c_batched ? r.count : 1, p.cols, c_bstride,
                   pf_cols, TC_BM, err, CU_TENSOR_MAP_SWIZZLE_NONE))
        return SNB_OK;
    if (r.activation == SNB_ACTIVATION_GELU_GRAD) {
        const CUtensorMapDataType gdt =
            r.aux_type == SNB_TYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        if (!encode_3d(&tg, gdt, aux_size, r.gelu_input, p.cols, p.rows, c_batched ? r.count : 1, p.cols, c_bstride,
                       pf_cols, TC_BM, err, CU_TENSOR_MAP_SWIZZLE_NONE))
            return SNB_OK;
    }

    // A bf16 output of a BN = 256 tile whose epilogue reads exactly one bf16 auxiliary input (the GELU input of a
    // GELU', or a residual) gets that input by TMA loads into the output's own staging boxes (map tx: box = one
    // 64-column x 32-row chunk, 128B swizzle like the output map), which replaces 32 uncoalesced 16-byte loads per
    // warp instruction with one asynchronous copy per chunk (measured on the training step's K=768 products:
    // project.dX 8 % and output.fwd 9 % faster). Such epilogues stage through two boxes per warp.
    const bool gin_only =
        r.activation == SNB_ACTIVATION_GELU_GRAD && r.aux_type == SNB_TYPE_BF16 && r.residual == nullptr;
    const bool res_only = r.activation != SNB_ACTIVATION_GELU_GRAD && r.residual != nullptr;
    const bool aux_box = out_bf16 && bf16_in && bn == 256 && r.pre == nullptr && r.causal == SNB_CAUSAL_NONE &&
                         splits_used == 1 && (gin_only || res_only);
    tx = tc;
    if (aux_box && !encode_3d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gin_only ? r.gelu_input : r.residual, p.cols,
                              p.rows, c_batched ? r.count : 1, p.cols, c_bstride, chunk, 32, err))
        return SNB_OK;

    // An overwrite computed in several K splits reaches C by reduce-add, so C starts at zero (slab stores need no
    // zeroing: the ordered sum writes C).
    const bool reduce = !slabs && (p.accumulate != 0 || splits_used > 1);
    if (!slabs && p.accumulate == 0 && splits_used > 1) {
        cudaError_t e;
        if (!c_batched || p.output_batch_stride == p.rows * p.cols) {
            e = cudaMemsetAsync(r.C, 0, r.count * p.rows * p.cols * csize, stream);
        } else {
            e = cudaMemset2DAsync(r.C, p.output_batch_stride * csize, 0, p.rows * p.cols * csize, r.count, stream);
        }
        if (e != cudaSuccess) {
            *err = cuda_message("zeroing the split-K output", e);
            return SNB_ERR_CUDA;
        }
    }

    TcParams kp{};
    kp.M = static_cast<int32_t>(p.rows);
    kp.N = static_cast<int32_t>(p.cols);
    kp.K = static_cast<int32_t>(p.inner);
    kp.count = static_cast<int32_t>(r.count);
    kp.a_mn_major = la.mn_major;
    kp.b_mn_major = lb.mn_major;
    kp.a_batched = la.batched;
    kp.b_batched = lb.batched;
    kp.m_tiles = static_cast<int32_t>(m_tiles);
    kp.n_tiles = static_cast<int32_t>(n_tiles);
    kp.k_blocks = static_cast<int32_t>(k_blocks);
    kp.splits = static_cast<int32_t>(splits_used);
    // Stream the larger operand once: with the N tile index fastest a wave shares A's rows and re-reads all of B
    // per wave (right when B is small, e.g. weights); with M fastest it is the other way round.
    const double a_bytes = static_cast<double>(p.rows) * p.inner;
    const double b_bytes = static_cast<double>(p.cols) * p.inner;
    kp.m_fastest = b_bytes > a_bytes ? 1 : 0;
    kp.k_blocks_per_split = static_cast<int32_t>(kb_per_split);
    const int64_t units = tiles * splits_used;
    if (units > (1ll << 31) - 1) return SNB_OK;
    kp.num_units = static_cast<int32_t>(units);
    kp.scale = p.scale;
    kp.reduce = reduce;
    kp.activation = r.activation;
    kp.aux_bf16 = r.aux_type == SNB_TYPE_BF16;
    kp.has_pre = r.pre != nullptr;
    kp.bias = r.bias;
    kp.row_scale = r.row_scale;
    kp.residual = r.residual;
    kp.gelu_input = r.gelu_input;
    kp.out_batch_stride = static_cast<int64_t>(c_batched ? p.output_batch_stride : 0);
    kp.causal = r.causal;
    kp.causal_offset = r.causal_offset;
    kp.split_slabs = slabs ? 1 : 0;
    if (ah != nullptr) {
        kp.a_heads = 1;
        kp.a_hd = static_cast<int32_t>(ah->head_dim);
        kp.a_time = static_cast<int32_t>(ah->time);
        kp.a_toff = static_cast<int32_t>(ah->time_offset);
    }
    if (ch != nullptr) {
        kp.c_heads = 1;
        kp.c_hd = static_cast<int32_t>(ch->head_dim);
        kp.c_nheads = static_cast<int32_t>(ch->heads);
        kp.c_time = static_cast<int32_t>(ch->time);
        kp.c_toff = static_cast<int32_t>(ch->time_offset);
    }
    // After the GEMM, the slabs are summed into C in split order.
    auto sum_slabs = [&]() -> int {
        if (!slabs) return SNB_OK;
        const int64_t n4 = static_cast<int64_t>(p.rows * p.cols / 4);
        const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(dev.sm_count) * 8);
        split_slab_sum_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            reinterpret_cast<const float4*>(slab_base), n4, static_cast<int32_t>(splits_used),
            reinterpret_cast<float4*>(r.C), p.accumulate != 0 ? 1 : 0, n4);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            *err = cuda_message("split_slab_sum_kernel launch", e);
            return SNB_ERR_CUDA;
        }
        return SNB_OK;
    };

    // Staging mode of the epilogue (gemm_tc.cuh, epilogue_tile).
    const bool heavy = r.activation != SNB_ACTIVATION_NONE;
    int epi = heavy ? TC_EPI_TWO_BOX : TC_EPI_ONE_BOX;
    if (aux_box) epi = TC_EPI_AUX_BOX;
    if (pair) {
        const int grid = 2 * static_cast<int>(std::min<int64_t>(units, workers));
        if (bias_pair) {
            if (epi == TC_EPI_AUX_BOX)
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_AUX_BOX, true>(stream, maps, kp, grid, err);
            else if (epi == TC_EPI_TWO_BOX)
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_TWO_BOX, true>(stream, maps, kp, grid, err);
            else
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_ONE_BOX, true>(stream, maps, kp, grid, err);
        } else if (bf16_in && out_bf16) {
            if (epi == TC_EPI_AUX_BOX)
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_AUX_BOX>(stream, maps, kp, grid, err);
            else if (epi == TC_EPI_TWO_BOX)
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_TWO_BOX>(stream, maps, kp, grid, err);
            else
                rc = launch_pair<__nv_bfloat16, true, TC_EPI_ONE_BOX>(stream, maps, kp, grid, err);
        } else if (bf16_in) {
            rc = heavy ? launch_pair<__nv_bfloat16, false, TC_EPI_TWO_BOX>(stream, maps, kp, grid, err)
                       : launch_pair<__nv_bfloat16, false, TC_EPI_ONE_BOX>(stream, maps, kp, grid, err);
        } else {
            rc = launch_pair<float, false, TC_EPI_ONE_BOX>(stream, maps, kp, grid, err);
        }
        if (rc == SNB_OK) rc = sum_slabs();
        if (rc == SNB_OK) {
            *launched = true;
            *path = SNB_PATH_TENSOR_CORE_PAIR;
        }
        return rc;
    }
    const int grid = static_cast<int>(std::min<int64_t>(units, sms));
    if (bf16_in) {
        rc = out_bf16 ? launch_bn<__nv_bfloat16, true>(bn, epi, stream, maps, kp, grid, err)
                      : launch_bn<__nv_bfloat16, false>(bn, epi, stream, maps, kp, grid, err);
    } else {
        rc = launch_bn<float, false>(bn, epi, stream, maps, kp, grid, err);
    }
    if (rc == SNB_OK) rc = sum_slabs();
    if (rc == SNB_OK) *launched = true;
    return rc;
}

int fused_attention_forward(cudaStream_t stream, const void* q, const void* k, const void* v, uint64_t count,
                            uint64_t queries, uint64_t keys, float scale, uint64_t query_offset, void* out,
                            int out_type, float* lse, std::string* err) {
    if (count == 0 || queries == 0) return SNB_OK;
    DeviceInfo dev;
    int rc = current_device_info(&dev, err);
    if (rc != SNB_OK) return rc;
    if (dev.major != 10) {
        *err = "fused attention needs an sm_100 device";
        return SNB_ERR_UNSUPPORTED;
    }
    const uint64_t lim = (1ull << 31) - 256;
    if (count > lim || queries > lim || keys > lim || keys == 0) {
        *err = "fused attention: sizes out of range";
        return SNB_ERR_INVALID_ARGUMENT;
    }
    for (const void* ptr : {q, k, v, static_cast<const void*>(out)}) {
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
            *err = "fused attention: q, k, v and out must be 16-byte aligned";
            return SNB_ERR_INVALID_ARGUMENT;
        }
    }
    CUtensorMap tq, tk, tv;
    // [count, rows, 64] bf16, rows 128 bytes apart; boxes of 128 rows x 64 (one 128-byte swizzle row each).
    if (!encode_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, FA_D, queries, count, FA_D, queries * FA_D, FA_D,
                   FA_BM, err) ||
        !encode_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, FA_D, keys, count, FA_D, keys * FA_D, FA_D, FA_BN,
                   err) ||
        !encode_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, v, FA_D, keys, count, FA_D, keys * FA_D, FA_D, FA_BN,
                   err))
        return SNB_ERR_INVALID_ARGUMENT;
    FaParams fp{};
    fp.count = static_cast<int32_t>(count);
    fp.sq = static_cast<int32_t>(queries);
    fp.sk = static_cast<int32_t>(keys);
    const int64_t q_tiles = (static_cast<int64_t>(queries) + FA_BM - 1) / FA_BM;
    fp.pairs = static_cast<int32_t>((q_tiles + 1) / 2);
    fp.offset = static_cast<int64_t>(query_offset);
    fp.scale_log2 = scale * 1.4426950408889634f;
    fp.out_bf16 = out_type == SNB_TYPE_BF16;
    fp.out = out;
    fp.out_stride = static_cast<int64_t>(queries) * FA_D;
    fp.lse = lse;
    const int64_t grid = static_cast<int64_t>(fp.pairs) * static_cast<int64_t>(count);
    if (grid > 0x7fffffff) {
        *err = "fused attention: grid too large";
        return SNB_ERR_UNSUPPORTED;
    }
    static int configured_device = -1;
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (configured_device != dev.device) {
            cudaError_t e = cudaFuncSetAttribute(fa_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 FaSmem::BYTES);
            if (e != cudaSuccess) {
                *err = cuda_message("cudaFuncSetAttribute(fa_forward_kernel)", e);
                return SNB_ERR_CUDA;
            }
            configured_device = dev.device;
        }
    }
    fa_forward_kernel<<<static_cast<unsigned>(grid), FA_THREADS, FaSmem::BYTES, stream>>>(tq, tk, tv, fp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("fa_forward_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

namespace {

// Scratch of the no-alloc backward entry point: the row statistics live here instead of in a stream-ordered
// allocation. One array per device image of the library, shared by every call on that device.
constexpr uint64_t kStaticScratchBytes = 8ull << 20;
static __device__ __align__(256) float g_attention_scratch[kStaticScratchBytes / sizeof(float)];

// The scratch array's device address on the current device, looked up once per device (the first no-alloc call
// on a device does it). A cudaDeviceReset of that device unloads the library's module from it, so the cached address
// is no longer valid afterwards: a process that resets a device does not use the no-alloc entry point on it again.
int static_scratch(float** ptr, std::string* err) {
    static std::mutex mu;
    static float* cached[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *err = cuda_message("cudaGetDevice", e);
        return SNB_ERR_CUDA;
    }
    if (dev < 0 || dev >= 64) {
        *err = "no-alloc scratch: device ordinal " + std::to_string(dev) + " is beyond the 64 devices it tracks";
        return SNB_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess) {
            *err = cuda_message("cudaGetSymbolAddress(scratch)", e);
            return SNB_ERR_CUDA;
        }
        cached[dev] = static_cast<float*>(p);
    }
    *ptr = cached[dev];
    return SNB_OK;
}

}  // namespace

int fused_attention_backward(cudaStream_t stream, const void* q, const void* k, const void* v, const void* out,
                             int out_type, const void* d_out, const float* lse, uint64_t count, uint64_t queries,
                             uint64_t keys, float scale, uint64_t query_offset, float* dq, float* dk, float* dv,
                             bool static_scratch_only, std::string* err) {
    if (count == 0) return SNB_OK;
    // Sizes and alignment are checked before any CUDA call, so a refused call touches neither the device nor a
    // buffer.
    const uint64_t lim = (1ull << 31) - 256;
    if (count > lim || queries > lim || keys > lim) {
        *err = "fused attention backward: sizes out of range";
        return SNB_ERR_INVALID_ARGUMENT;
    }
    // Scratch: per query (-lse * log2(e), D), matrices `stride` floats apart (16-byte multiple for the tensor map).
    // Every byte count below is formed with overflow checks: count and queries may each be close to 2^31, and a
    // wrapped product would pass the size check of the static scratch or ask for a too-small allocation.
    const uint64_t stride = (2 * queries + 3) / 4 * 4;
    uint64_t scratch_bytes = 0, dq_bytes = 0, dkv_bytes = 0;
    if (__builtin_mul_overflow(count, stride, &scratch_bytes) ||
        __builtin_mul_overflow(scratch_bytes, sizeof(float), &scratch_bytes) ||
        __builtin_mul_overflow(count, queries, &dq_bytes) ||
        __builtin_mul_overflow(dq_bytes, FB_D * sizeof(float), &dq_bytes) ||
        __builtin_mul_overflow(count, keys, &dkv_bytes) ||
        __builtin_mul_overflow(dkv_bytes, FB_D * sizeof(float), &dkv_bytes)) {
        *err = "fused attention backward: count * queries (or keys) * head size overflows 64 bits";
        return SNB_ERR_INVALID_ARGUMENT;
    }
    if (static_scratch_only && queries > 0 && keys > 0 && scratch_bytes > kStaticScratchBytes) {
        *err = "fused attention backward (no-alloc): needs " + std::to_string(scratch_bytes) +
               " bytes of row statistics (count * queries * 8, rounded), the static scratch holds " +
               std::to_string(kStaticScratchBytes);
        return SNB_ERR_INVALID_ARGUMENT;
    }
    for (const void* ptr : {q, k, v, out, d_out, static_cast<const void*>(dq), static_cast<const void*>(dk),
                            static_cast<const void*>(dv)}) {
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
            *err = "fused attention backward: q, k, v, out, d_out, dq, dk and dv must be 16-byte aligned";
            return SNB_ERR_INVALID_ARGUMENT;
        }
    }
    DeviceInfo dev;
    int rc = current_device_info(&dev, err);
    if (rc != SNB_OK) return rc;
    if (dev.major != 10) {
        *err = "fused attention needs an sm_100 device";
        return SNB_ERR_UNSUPPORTED;
    }
    auto memset_or_fail = [&](void* ptr, uint64_t bytes, const char* what) -> int {
        if (bytes == 0) return SNB_OK;
        cudaError_t e = cudaMemsetAsync(ptr, 0, bytes, stream);
        if (e != cudaSuccess) {
            *err = cuda_message(what, e);
            return SNB_ERR_CUDA;
        }
        return SNB_OK;
    };
    // dQ is accumulated into by TMA reductions; with no queries or no keys every gradient is zero.
    rc = memset_or_fail(dq, dq_bytes, "cudaMemsetAsync(dq)");
    if (rc != SNB_OK) return rc;
    if (queries == 0 || keys == 0) {
        rc = memset_or_fail(dk, dkv_bytes, "cudaMemsetAsync(dk)");
        if (rc == SNB_OK) rc = memset_or_fail(dv, dkv_bytes, "cudaMemsetAsync(dv)");
        return rc;
    }
    // The row-statistics grid covers count * queries rows, 32 per block (8 for the scalar form).
    if (count * queries > 8ull * 0x7fffffffull) {
        *err = "fused attention backward: count * queries exceeds the row-statistics grid";
        return SNB_ERR_INVALID_ARGUMENT;
    }
    float* stats = nullptr;
    cudaError_t e = cudaSuccess;
    if (static_scratch_only) {
        rc = static_scratch(&stats, err);
        if (rc != SNB_OK) return rc;
    } else {
        e = cudaMallocAsync(reinterpret_cast<void**>(&stats), scratch_bytes, stream);
        if (e != cudaSuccess) {
            *err = cuda_message("cudaMallocAsync(row statistics)", e);
            return SNB_ERR_CUDA;
        }
    }
    auto release = [&]() {
        if (!static_scratch_only) cudaFreeAsync(stats, stream);
    };
    const uint64_t rows = count * queries;
    if (reinterpret_cast<uintptr_t>(out) % 16 == 0 && reinterpret_cast<uintptr_t>(d_out) % 16 == 0) {
        fb_rowstats_vec_kernel<<<static_cast<unsigned>((rows + 31) / 32), 256, 0, stream>>>(
            out, out_type == SNB_TYPE_BF16 ? 1 : 0, static_cast<const uint16_t*>(d_out), lse, stats,
            static_cast<int64_t>(rows), static_cast<int32_t>(queries), static_cast<int64_t>(stride));
    } else {
        fb_rowstats_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
            out, out_type == SNB_TYPE_BF16 ? 1 : 0, static_cast<const uint16_t*>(d_out), lse, stats,
            static_cast<int64_t>(rows), static_cast<int32_t>(queries), static_cast<int64_t>(stride));
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        release();
        *err = cuda_message("fb_rowstats_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    CUtensorMap tq, tk, tv, tdo, tst, tdq, tdk, tdv;
    // [count, rows, 64] bf16 tiles of 128 rows (one 128-byte swizzle row each); the statistics as 256-float rows
    // (128 queries); dQ, dK and dV as f32 boxes of 32 columns x 32 rows (128-byte swizzle rows).
    if (!encode_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, FB_D, queries, count, FB_D, queries * FB_D, FB_D,
                   FB_BQ, err) ||
        !encode_3d(&tdo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d_out, FB_D, queries, count, FB_D, queries * FB_D, FB_D,
                   FB_BQ, err) ||
        !encode_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, FB_D, keys, count, FB_D, keys * FB_D, FB_D, FB_BK,
                   err) ||
        !encode_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, v, FB_D, keys, count, FB_D, keys * FB_D, FB_D, FB_BK,
                   err) ||
        !encode_3d(&tst, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, stats, 2 * queries, count, 1, stride, stride * count,
                   2 * FB_BQ, 1, err, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_3d(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dq, FB_D, queries, count, FB_D, queries * FB_D, 32, 32,
                   err) ||
        !encode_3d(&tdk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dk, FB_D, keys, count, FB_D, keys * FB_D, 32, 32, err) ||
        !encode_3d(&tdv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dv, FB_D, keys, count, FB_D, keys * FB_D, 32, 32, err)) {
        release();
        return SNB_ERR_INVALID_ARGUMENT;
    }
    FbParams fp{};
    fp.count = static_cast<int32_t>(count);
    fp.sq = static_cast<int32_t>(queries);
    fp.sk = static_cast<int32_t>(keys);
    fp.q_tiles = static_cast<int32_t>((queries + FB_BQ - 1) / FB_BQ);
    fp.k_tiles = static_cast<int32_t>((keys + FB_BK - 1) / FB_BK);
    // Scheduling groups of 8 matrices: a group's Q, dO, dQ and K, V (0.8 MB each per matrix at 3,072 x 64) fit in
    // L2 many times over while one wave of CTAs covers about a group.
    fp.group = static_cast<int32_t>(std::min<uint64_t>(count, 8));
    fp.offset = static_cast<int64_t>(query_offset);
    fp.scale = scale;
    fp.scale_log2 = scale * 1.4426950408889634f;
    const int64_t grid = static_cast<int64_t>((keys + FB_BK - 1) / FB_BK) * static_cast<int64_t>(count);
    if (grid > 0x7fffffff) {
        release();
        *err = "fused attention backward: grid too large";
        return SNB_ERR_UNSUPPORTED;
    }
    static int configured_device = -1;
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (configured_device != dev.device) {
            e = cudaFuncSetAttribute(fb_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FbSmem::BYTES);
            if (e != cudaSuccess) {
                release();
                *err = cuda_message("cudaFuncSetAttribute(fb_backward_kernel)", e);
                return SNB_ERR_CUDA;
            }
            configured_device = dev.device;
        }
    }
    fb_backward_kernel<<<static_cast<unsigned>(grid), FB_THREADS, FbSmem::BYTES, stream>>>(tq, tk, tv, tdo, tst, tdq,
                                                                                           tdk, tdv, fp);
    e = cudaGetLastError();
    release();
    if (e != cudaSuccess) {
        *err = cuda_message("fb_backward_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

namespace {

// Waits on an mbarrier that nothing ever completes, through the same bounded wait the GEMM pipeline uses: the wait
// must give up after `limit_ns`, flag the device status and let the kernel return normally.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(smem_addr(&bar), 1);
    fence_mbarrier_init();
    mbar_wait(smem_addr(&bar), 0, limit_ns);
}

}  // namespace

int bounded_wait_probe(cudaStream_t stream, uint64_t limit_ns, std::string* err) {
    bounded_wait_probe_kernel<<<1, 32, 0, stream>>>(limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = cuda_message("bounded_wait_probe_kernel launch", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

int read_and_clear_device_status(unsigned int* status, std::string* err) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        *err = cuda_message("cudaDeviceSynchronize", e);
        return SNB_ERR_CUDA;
    }
    e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned int));
    if (e != cudaSuccess) {
        *err = cuda_message("reading the device status", e);
        return SNB_ERR_CUDA;
    }
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int));
    if (e != cudaSuccess) {
        *err = cuda_message("clearing the device status", e);
        return SNB_ERR_CUDA;
    }
    return SNB_OK;
}

}  // namespace snb
