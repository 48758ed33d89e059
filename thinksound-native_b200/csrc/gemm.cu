// gemm.cu — instantiations and host launch of the tcgen05 GEMM (gemm_tc.cuh), plus the TMA
// tensor-map encoders (driver entry point fetched through the runtime, no -lcuda needed).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <map>
#include <mutex>

#include "gemm_2sm.cuh"
#include "kernels.h"

namespace tsn {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool encoder() {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q{};
        void * fn = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = (PFN_cuTensorMapEncodeTiled_v12000) fn;
    });
    return g_encode != nullptr;
}
} // namespace

bool make_act_map(CUtensorMap * m, const void * base, uint64_t K_in, uint64_t rows, uint64_t B,
                  uint32_t bt, uint32_t bb, int bf16) {
    if (!encoder() || ((uintptr_t) base & 15) || (K_in % 64) || bt * bb > 128 || (bt * bb) % 8) return false;
    const cuuint64_t dims[3] = {K_in, rows, B};
    const cuuint64_t strides[2] = {K_in * 2, rows * K_in * 2};
    const cuuint32_t box[3] = {64, bt, bb};
    const cuuint32_t es[3] = {1, 1, 1};
    return g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *) base,
                    dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_act_map_rows(CUtensorMap * m, const void * base, uint64_t K_in, uint64_t rows, uint64_t B, uint32_t box_rows) {
    if (!encoder() || ((uintptr_t) base & 15) || (K_in % 64) || box_rows == 0 || box_rows > 256) return false;
    const cuuint64_t dims[3] = {K_in, rows, B};
    const cuuint64_t strides[2] = {K_in * 2, rows * K_in * 2};
    const cuuint32_t box[3] = {64, box_rows, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *) base, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_head_map(CUtensorMap * m, const void * base, uint64_t rows, uint32_t box_rows, uint64_t lo_elems) {
    if (!encoder() || ((uintptr_t) base & 15) || box_rows > 256) return false;
    const cuuint64_t dims[3] = {64, rows, 2};
    const cuuint64_t strides[2] = {128, (lo_elems ? lo_elems : rows * 64) * 2};
    const cuuint32_t box[3] = {64, box_rows, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *) base, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_w_map(CUtensorMap * m, const void * base, uint64_t K, uint64_t N, uint32_t bn, int bf16) {
    if (!encoder() || ((uintptr_t) base & 15) || (K % 64) || bn > 256) return false;
    const cuuint64_t dims[2] = {K, N};
    const cuuint64_t strides[1] = {K * 2};
    const cuuint32_t box[2] = {64, bn};
    const cuuint32_t es[2] = {1, 1};
    return g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *) base,
                    dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_out_map_f32(CUtensorMap * m, void * base, uint64_t N, uint64_t rows, uint64_t B, uint64_t Z, uint64_t ldo,
                      uint64_t out_bs, uint64_t z_stride) {
    if (!encoder() || ((uintptr_t) base & 15) || ldo < N || (ldo * 4) % 16 || (out_bs * 4) % 16 || (z_stride * 4) % 16 ||
        !N || !rows || !B || !Z)
        return false;
    const cuuint64_t dims[4] = {N, rows, B, Z};
    const cuuint64_t strides[3] = {ldo * 4, out_bs * 4, z_stride * 4};
    const cuuint32_t box[4] = {32, 32, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Pipeline depth: as many stages as fit in the 227 KB of shared memory a CTA may use (the qkv
// epilogue also stages RoPE rows, which costs the 192-wide split tile one stage).
constexpr int stages_for(int bn, bool split, int epi) {
    return split ? (bn == 256 ? 3 : bn == 192 || bn == 176 ? (epi == EPI_QKV ? 3 : 4) : bn == 128 ? 4 : 5)
                 : (bn == 256 ? 4 : bn == 192 ? 5 : bn == 128 ? 6 : 8);
}
int gemm_stages(int bn, bool split, int epi) { return stages_for(bn, split, epi); }

namespace {
template <int BN, bool SPLIT, int EPI>
constexpr int smem_total() { return GemmSmem<BN, stages_for(BN, SPLIT, EPI), SPLIT, EPI>::TOTAL; }
template <int BN, bool SPLIT>
size_t smem_of(int epi) {
    switch (epi) {
        case EPI_F32: return smem_total<BN, SPLIT, EPI_F32>();
        case EPI_F16: return smem_total<BN, SPLIT, EPI_F16>();
        case EPI_F16_SILU: return smem_total<BN, SPLIT, EPI_F16_SILU>();
        case EPI_SWIGLU: return smem_total<BN, SPLIT, EPI_SWIGLU>();
        case EPI_QKV: return smem_total<BN, SPLIT, EPI_QKV>();
        case EPI_GEGLU: return smem_total<BN, SPLIT, EPI_GEGLU>();
    }
    return 0;
}
} // namespace

// Dynamic shared memory of one configuration: the kernel's own layout constant (single source).
size_t gemm_smem_bytes(int bn, bool split, int epi) {
    switch (bn) {
        case 64: return split ? smem_of<64, true>(epi) : smem_of<64, false>(epi);
        case 128: return split ? smem_of<128, true>(epi) : smem_of<128, false>(epi);
        case 192: return split ? smem_of<192, true>(epi) : smem_of<192, false>(epi);
        case 256: return split ? smem_of<256, true>(epi) : smem_of<256, false>(epi);
        case 176: return split && epi == EPI_SWIGLU ? smem_total<176, true, EPI_SWIGLU>() : 0;
    }
    return 0;
}

constexpr int persist_stages(int bn) { return bn == 128 ? 4 : 3; }
size_t gemm_persistent_smem_bytes(int bn) {
    switch (bn) {
        case 128: return PersistSmem<128, persist_stages(128)>::TOTAL;
        case 192: return PersistSmem<192, persist_stages(192)>::TOTAL;
        case 256: return PersistSmem<256, persist_stages(256)>::TOTAL;
    }
    return 0;
}

constexpr int stages2(int nt, bool split) {
    return split ? (nt == 256 ? 4 : nt == 192 ? 5 : nt == 128 ? 6 : nt == 96 ? 7 : 8) : (nt == 256 ? 6 : nt == 192 ? 7 : 8);
}
size_t gemm2_smem_bytes(int nt, bool split) {
    switch (nt * 2 + (split ? 1 : 0)) {
        case 64 * 2: return Gemm2Smem<64, stages2(64, false), false>::TOTAL;
        case 64 * 2 + 1: return Gemm2Smem<64, stages2(64, true), true>::TOTAL;
        case 96 * 2: return Gemm2Smem<96, stages2(96, false), false>::TOTAL;
        case 96 * 2 + 1: return Gemm2Smem<96, stages2(96, true), true>::TOTAL;
        case 128 * 2: return Gemm2Smem<128, stages2(128, false), false>::TOTAL;
        case 128 * 2 + 1: return Gemm2Smem<128, stages2(128, true), true>::TOTAL;
        case 192 * 2: return Gemm2Smem<192, stages2(192, false), false>::TOTAL;
        case 192 * 2 + 1: return Gemm2Smem<192, stages2(192, true), true>::TOTAL;
        case 256 * 2: return Gemm2Smem<256, stages2(256, false), false>::TOTAL;
        case 256 * 2 + 1: return Gemm2Smem<256, stages2(256, true), true>::TOTAL;
    }
    return 0;
}

namespace {
using Kernel2Fn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs);
template <int NT, int EPI, bool SPLIT>
Kernel2Fn pick2() {
    static_assert(Gemm2Smem<NT, stages2(NT, SPLIT), SPLIT>::TOTAL <= 232448, "smem budget");
    return (Kernel2Fn) gemm2_kernel<NT, EPI, stages2(NT, SPLIT), SPLIT>;
}
template <int NT>
Kernel2Fn pick2_epi(int epi, bool split) {
    if (epi == EPI_F32) return split ? pick2<NT, EPI_F32, true>() : pick2<NT, EPI_F32, false>();
    if (epi == EPI_SWIGLU) return split ? pick2<NT, EPI_SWIGLU, true>() : pick2<NT, EPI_SWIGLU, false>();
    return nullptr;
}
Kernel2Fn gemm2_for(int nt, int epi, bool split) {
    switch (nt) {
        case 64: return pick2_epi<64>(epi, split);
        case 96: return pick2_epi<96>(epi, split);   // 188 tokens of one arm as 96 + 92
        case 128: return pick2_epi<128>(epi, split);
        case 192: return pick2_epi<192>(epi, split);
        case 256: return pick2_epi<256>(epi, split);
    }
    return nullptr;
}
} // namespace

namespace {
using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs, int);

template <int BN>
KernelFn pick_persistent() {
    static_assert(PersistSmem<BN, persist_stages(BN)>::TOTAL <= 232448, "smem budget");
    return (KernelFn) gemm_tc_persistent<BN, persist_stages(BN)>;
}
KernelFn persistent_for(int bn) {
    switch (bn) {
        case 128: return pick_persistent<128>();
        case 192: return pick_persistent<192>();
        case 256: return pick_persistent<256>();
    }
    return nullptr;
}

using TileFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs, int);

template <int BN, int EPI, bool SPLIT>
TileFn pick() {
    constexpr int ST = stages_for(BN, SPLIT, EPI);
    static_assert(GemmSmem<BN, ST, SPLIT, EPI>::TOTAL <= 232448, "smem budget");
    return (TileFn) gemm_tc_kernel<BN, EPI, ST, SPLIT>;
}

template <int BN, bool SPLIT>
TileFn pick_epi(int epi) {
    switch (epi) {
        case EPI_F32: return pick<BN, EPI_F32, SPLIT>();
        case EPI_F16: return pick<BN, EPI_F16, SPLIT>();
        case EPI_F16_SILU: return pick<BN, EPI_F16_SILU, SPLIT>();
        case EPI_SWIGLU: return pick<BN, EPI_SWIGLU, SPLIT>();
        case EPI_QKV: return pick<BN, EPI_QKV, SPLIT>();
        case EPI_GEGLU: return pick<BN, EPI_GEGLU, SPLIT>();
    }
    return nullptr;
}

TileFn kernel_for(int bn, int epi, bool split) {
    switch (bn) {
        case 64: return split ? pick_epi<64, true>(epi) : pick_epi<64, false>(epi);
        case 128: return split ? pick_epi<128, true>(epi) : pick_epi<128, false>(epi);
        case 192: return split ? pick_epi<192, true>(epi) : pick_epi<192, false>(epi);
        case 256: return split ? pick_epi<256, true>(epi) : pick_epi<256, false>(epi);
        // 11 column groups of [8 w1 | 8 w3]: the SwiGLU GEMMs whose 8192-wide output in 192-wide
        // tiles leaves SMs idle (376 x 8192: 141 CTAs instead of 129)
        case 176: return split && epi == EPI_SWIGLU ? pick<176, EPI_SWIGLU, true>() : nullptr;
    }
    return nullptr;
}
using GroupFn = void (*)(GroupMaps, GroupArgs, int);
template <int BN, int EPI, bool SPLIT>
GroupFn pick_group() {
    return (GroupFn) gemm_tc_group<BN, EPI, stages_for(BN, SPLIT, EPI), SPLIT>;
}
// the grouped instantiations the joint blocks use: qkv, swiglu (split operands), f32 (both)
template <int BN>
GroupFn group_epi(int epi, bool split) {
    if (epi == EPI_QKV && split) return pick_group<BN, EPI_QKV, true>();
    if (epi == EPI_SWIGLU && split) return pick_group<BN, EPI_SWIGLU, true>();
    if (epi == EPI_F32) return split ? pick_group<BN, EPI_F32, true>() : pick_group<BN, EPI_F32, false>();
    return nullptr;
}
// the grouped SwiGLU launch whose shallow member runs as 208-wide persistent tile lists
constexpr int GROUP_P_BN = 208, GROUP_P_STAGES = 3;
GroupFn group_p_for(int bn, int epi, bool split) {
    if (bn == 256 && epi == EPI_SWIGLU && split)
        return (GroupFn) gemm_tc_group_p<256, GROUP_P_BN, EPI_SWIGLU, stages_for(256, true, EPI_SWIGLU), GROUP_P_STAGES, true>;
    return nullptr;
}
GroupFn group_for(int bn, int epi, bool split) {
    switch (bn) {
        case 64: return group_epi<64>(epi, split);
        case 128: return group_epi<128>(epi, split);
        case 192: return group_epi<192>(epi, split);
        case 256: return group_epi<256>(epi, split);
    }
    return nullptr;
}
} // namespace

bool gemm_group_supported(int bn, int epi, bool split) { return group_for(bn, epi, split) != nullptr; }

// ---- split activations x split weights (gemm_ws_kernel): the VAE decoder ----
namespace {
constexpr int stages_ws(int bn) { return bn == 256 ? 2 : bn == 128 ? 3 : 4; }
using KernelWsFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs);
template <int BN, int EPI>
KernelWsFn pick_ws() {
    static_assert(GemmSmem<BN, stages_ws(BN), true, EPI, true>::TOTAL <= 232448, "smem budget");
    return (KernelWsFn) gemm_ws_kernel<BN, EPI, stages_ws(BN)>;
}
template <int BN>
KernelWsFn ws_epi(int epi) {
    switch (epi) {
        case EPI_F32: return pick_ws<BN, EPI_F32>();
        case EPI_F16_SNAKE: return pick_ws<BN, EPI_F16_SNAKE>();
        case EPI_RESID_SNAKE: return pick_ws<BN, EPI_RESID_SNAKE>();
        case EPI_F32_SNAKE2: return pick_ws<BN, EPI_F32_SNAKE2>();
        case EPI_QKV: return pick_ws<BN, EPI_QKV>();
        case EPI_F16_GELUQ: return pick_ws<BN, EPI_F16_GELUQ>();
    }
    return nullptr;
}
KernelWsFn ws_for(int bn, int epi) {
    switch (bn) {
        case 64: return ws_epi<64>(epi);
        case 128: return ws_epi<128>(epi);
        case 256: return ws_epi<256>(epi);
    }
    return nullptr;
}
} // namespace

namespace {
template <int BN>
size_t ws_smem_of(int epi) {
    switch (epi) {
        case EPI_F32: return GemmSmem<BN, stages_ws(BN), true, EPI_F32, true>::TOTAL;
        case EPI_F16_SNAKE: return GemmSmem<BN, stages_ws(BN), true, EPI_F16_SNAKE, true>::TOTAL;
        case EPI_RESID_SNAKE: return GemmSmem<BN, stages_ws(BN), true, EPI_RESID_SNAKE, true>::TOTAL;
        case EPI_F32_SNAKE2: return GemmSmem<BN, stages_ws(BN), true, EPI_F32_SNAKE2, true>::TOTAL;
        case EPI_QKV: return GemmSmem<BN, stages_ws(BN), true, EPI_QKV, true>::TOTAL;
        case EPI_F16_GELUQ: return GemmSmem<BN, stages_ws(BN), true, EPI_F16_GELUQ, true>::TOTAL;
    }
    return 0;
}
} // namespace

size_t gemm_ws_smem_bytes(int bn, int epi) {
    switch (bn) {
        case 64: return ws_smem_of<64>(epi);
        case 128: return ws_smem_of<128>(epi);
        case 256: return ws_smem_of<256>(epi);
    }
    return 0;
}

namespace {
template <int BN, int EPI>
KernelWsFn pick_wsp() {
    static_assert(PersistWsSmem<BN, stages_ws(BN), EPI>::TOTAL <= 232448, "smem budget");
    return (KernelWsFn) gemm_ws_persistent<BN, EPI, stages_ws(BN)>;
}
template <int BN>
KernelWsFn wsp_epi(int epi) {
    switch (epi) {
        case EPI_F32: return pick_wsp<BN, EPI_F32>();
        case EPI_F16_SNAKE: return pick_wsp<BN, EPI_F16_SNAKE>();
        case EPI_RESID_SNAKE: return pick_wsp<BN, EPI_RESID_SNAKE>();
        case EPI_F32_SNAKE2: return pick_wsp<BN, EPI_F32_SNAKE2>();
    }
    return nullptr;
}
KernelWsFn wsp_for(int bn, int epi) {
    switch (bn) {
        case 64: return wsp_epi<64>(epi);
        case 128: return wsp_epi<128>(epi);
        case 256: return wsp_epi<256>(epi);
    }
    return nullptr;
}
template <int BN>
size_t wsp_smem_of(int epi) {
    switch (epi) {
        case EPI_F32: return PersistWsSmem<BN, stages_ws(BN), EPI_F32>::TOTAL;
        case EPI_F16_SNAKE: return PersistWsSmem<BN, stages_ws(BN), EPI_F16_SNAKE>::TOTAL;
        case EPI_RESID_SNAKE: return PersistWsSmem<BN, stages_ws(BN), EPI_RESID_SNAKE>::TOTAL;
        case EPI_F32_SNAKE2: return PersistWsSmem<BN, stages_ws(BN), EPI_F32_SNAKE2>::TOTAL;
    }
    return 0;
}
} // namespace

size_t gemm_ws_persistent_smem_bytes(int bn, int epi) {
    switch (bn) {
        case 64: return wsp_smem_of<64>(epi);
        case 128: return wsp_smem_of<128>(epi);
        case 256: return wsp_smem_of<256>(epi);
    }
    return 0;
}

// CTAs of the split-weight kernel that fit at once in clusters of `cluster` along z
int gemm_ws_capacity(int bn, int epi, int cluster) {
    KernelWsFn fn = ws_for(bn, epi);
    if (!fn) return 0;
    if (cluster <= 1) {
        int per_sm = 0, sms = 0, d = 0;
        cudaGetDevice(&d);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 192, gemm_ws_smem_bytes(bn, epi)) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return per_sm * sms;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1, 1, (unsigned) std::max(cluster, 1));
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = gemm_ws_smem_bytes(bn, epi);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned) std::max(cluster, 1);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n * std::max(cluster, 1);
}

cudaError_t launch_gemm_ws(const GemmLaunch & g, cudaStream_t s) {
    if (g.persistent) {
        KernelWsFn fn = wsp_for(g.bn, g.epi);
        if (!fn || !g.split || g.args.splits != 1) return cudaErrorInvalidValue;
        return launch_ex(fn, g.grid, dim3(192), g.smem, s, 1u, g.ta, g.ta2, g.tb, g.tb2, g.args);
    }
    KernelWsFn fn = ws_for(g.bn, g.epi);
    if (!fn || !g.split) return cudaErrorInvalidValue;
    return launch_ex(fn, g.grid, dim3(192), g.smem, s, g.args.splits > 1 ? (unsigned) g.args.splits : 1u, g.ta, g.ta2,
                     g.tb, g.tb2, g.args);
}

// Set the dynamic shared-memory limit of every instantiation once, outside any stream capture.
cudaError_t configure_gemm_kernels() {
    for (int split = 0; split < 2; ++split)
        for (int bn : {64, 128, 176, 192, 256})
            for (int epi = 0; epi <= EPI_F16_GELUQ; ++epi) {
                TileFn fn = kernel_for(bn, epi, split != 0);
                if (!fn) continue;
                cudaError_t e = cudaFuncSetAttribute((const void *) fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int) gemm_smem_bytes(bn, split != 0, epi));
                if (e != cudaSuccess) return e;
            }
    for (int split = 0; split < 2; ++split)
        for (int bn : {64, 128, 192, 256})
            for (int epi = 0; epi < 6; ++epi) {
                GroupFn fn = group_for(bn, epi, split != 0);
                if (!fn) continue;
                cudaError_t e = cudaFuncSetAttribute((const void *) fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int) gemm_smem_bytes(bn, split != 0, epi));
                if (e != cudaSuccess) return e;
            }
    for (int bn : {64, 128, 256})
        for (int epi : {(int) EPI_F32, (int) EPI_F16_SNAKE, (int) EPI_RESID_SNAKE, (int) EPI_F32_SNAKE2, (int) EPI_QKV,
                        (int) EPI_F16_GELUQ}) {
            cudaError_t e = cudaFuncSetAttribute((const void *) ws_for(bn, epi), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int) gemm_ws_smem_bytes(bn, epi));
            if (e == cudaSuccess && wsp_for(bn, epi))
                e = cudaFuncSetAttribute((const void *) wsp_for(bn, epi), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int) gemm_ws_persistent_smem_bytes(bn, epi));
            if (e != cudaSuccess) return e;
        }
    {
        cudaError_t e = cudaFuncSetAttribute((const void *) group_p_for(256, EPI_SWIGLU, true),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int) gemm_group_persist_smem_bytes(256, EPI_SWIGLU, true));
        if (e != cudaSuccess) return e;
    }
    for (int bn : {128, 192, 256}) {
        cudaError_t e = cudaFuncSetAttribute((const void *) persistent_for(bn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int) gemm_persistent_smem_bytes(bn));
        if (e != cudaSuccess) return e;
    }
    for (int nt : {64, 96, 128, 192, 256})
        for (int epi : {(int) EPI_F32, (int) EPI_SWIGLU})
            for (int split = 0; split < 2; ++split) {
                cudaError_t e = cudaFuncSetAttribute((const void *) gemm2_for(nt, epi, split != 0),
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int) gemm2_smem_bytes(nt, split != 0));
                if (e != cudaSuccess) return e;
            }
    return cudaSuccess;
}

bool pdl_enabled() {
    static const bool on = std::getenv("TSN_NO_PDL") == nullptr;
    return on;
}

cudaError_t launch_gemm(const GemmLaunch & g, cudaStream_t s) {
    if (g.pair_nt) {
        Kernel2Fn fn = gemm2_for(g.pair_nt, g.epi, g.split);
        if (!fn || g.grid.x % 2) return cudaErrorInvalidValue;
        return launch_cl(fn, g.grid, dim3(192), g.smem, s, dim3(2, 1, 1), g.tb, g.ta, g.ta2, g.args.tma_out ? g.to : g.tb,
                         g.args);
    }
    if (g.persistent) {
        KernelFn fn = persistent_for(g.bn);
        if (!fn || g.epi != EPI_F32 || !g.split || g.args.splits != 1) return cudaErrorInvalidValue;
        return launch_ex(fn, g.grid, dim3(192), g.smem, s, 1u, g.ta, g.ta2, g.tb, g.args, g.ab_bf16);
    }
    TileFn fn = kernel_for(g.bn, g.epi, g.split);
    if (!fn) return cudaErrorInvalidValue;
    if (g.bn % 32 && g.args.splits != 1) return cudaErrorInvalidValue;   // cluster reductions: 32-column units
    // split-K: the K slices of one output tile form a cluster along grid.z
    return launch_ex(fn, g.grid, dim3(192), g.smem, s, g.args.splits > 1 ? (unsigned) g.args.splits : 1u,
                     g.ta, g.split ? g.ta2 : g.ta, g.tb, g.args.tma_out ? g.to : g.tb, g.args, g.ab_bf16);
}

int gemm_group_persist_bn(int bn, int epi, bool split) { return group_p_for(bn, epi, split) ? GROUP_P_BN : 0; }
size_t gemm_group_persist_smem_bytes(int bn, int epi, bool split) {
    if (!group_p_for(bn, epi, split)) return 0;
    return std::max(gemm_smem_bytes(bn, split, epi), (size_t) PersistListSmem<GROUP_P_BN, GROUP_P_STAGES, true>::TOTAL);
}

cudaError_t launch_gemm_group(const GroupLaunch & g, cudaStream_t s) {
    GroupFn fn = g.args.persist_q >= 0 ? group_p_for(g.bn, g.epi, g.split) : group_for(g.bn, g.epi, g.split);
    const int n = g.args.n;
    if (!fn || n < 1 || n > MAX_GROUP || g.cluster < 1 || g.cluster > 8) return cudaErrorInvalidValue;
    for (int q = 0; q < n; ++q) {
        const int begin = q ? g.args.cta_end[q - 1] : 0;
        if (g.args.cta_end[q] <= begin || g.args.slices[q] < 1 || g.args.m_tiles[q] < 1) return cudaErrorInvalidValue;
        // clusters never straddle two problems, and a cluster is exactly one tile's K slices
        if (g.cluster > 1 && (begin % g.cluster || g.args.slices[q] != g.cluster || g.args.p[q].splits != g.cluster))
            return cudaErrorInvalidValue;
        if (g.cluster == 1 && g.args.p[q].splits != 1) return cudaErrorInvalidValue;
    }
    if (g.args.persist_q >= 0) {   // the persistent member: its own CTA range, one CTA per tile run
        const int q = g.args.persist_q, begin = q ? g.args.cta_end[q - 1] : 0;
        if (q >= n || g.cluster != 1 || g.args.persist_ctas < 1 || g.args.persist_tiles < 1 ||
            g.args.cta_end[q] - begin != g.args.persist_ctas)
            return cudaErrorInvalidValue;
    }
    return launch_cl(fn, dim3((unsigned) g.args.cta_end[n - 1]), dim3(192), g.smem, s, dim3((unsigned) g.cluster, 1, 1),
                     g.maps, g.args, g.ab_bf16);
}

// CTAs of the 2-SM kernel that can run at once (in pairs)
int gemm2_capacity(int nt, int epi, bool split) {
    static std::mutex mu;
    static std::map<int, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const int key = ((dev * 512 + nt) * 8 + epi) * 2 + (split ? 1 : 0);
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    Kernel2Fn fn = gemm2_for(nt, epi, split);
    int cap = 0;
    if (fn) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(192, 1, 1);
        cfg.dynamicSmemBytes = gemm2_smem_bytes(nt, split);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, (const void *) fn, &cfg) == cudaSuccess) cap = 2 * clusters;
        else cudaGetLastError();
    }
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = cap;
    return cap;
}

int cluster_capacity_uncached(int bn, int epi, bool split, int cluster);

// How many CTAs of this configuration can run at once when grouped in clusters of `cluster`.
int gemm_cluster_capacity(int bn, int epi, bool split, int cluster) {
    static std::mutex mu;
    static std::map<int, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const int key = ((dev * 512 + bn) * 8 + epi) * 64 + (split ? 32 : 0) + cluster;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    const int cap = cluster_capacity_uncached(bn, epi, split, cluster);
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = cap;
    return cap;
}

int cluster_capacity_uncached(int bn, int epi, bool split, int cluster) {
    TileFn fn = kernel_for(bn, epi, split);
    if (!fn) return 0;
    if (cluster <= 1) {
        int per_sm = 0, sms = 0, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 192, gemm_smem_bytes(bn, split, epi)) != cudaSuccess)
            return 0;
        return per_sm * sms;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1, 1, (unsigned) cluster);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = gemm_smem_bytes(bn, split, epi);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned) cluster;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n * cluster;
}

} // namespace tsn
