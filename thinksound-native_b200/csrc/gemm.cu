// gemm.cu — instantiations and host launch of the tcgen05 GEMM (gemm_tc.cuh), plus the TMA
// tensor-map encoders (driver entry point fetched through the runtime, no -lcuda needed).
#include <cudaTypedefs.h>

#include <mutex>

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
    if (!encoder() || ((uintptr_t) base & 15) || (K_in % 64) || bt * bb != 128) return false;
    const cuuint64_t dims[3] = {K_in, rows, B};
    const cuuint64_t strides[2] = {K_in * 2, rows * K_in * 2};
    const cuuint32_t box[3] = {64, bt, bb};
    const cuuint32_t es[3] = {1, 1, 1};
    return g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *) base,
                    dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

int gemm_stages(int bn) { return bn == 256 ? 4 : bn == 128 ? 6 : 8; }

size_t gemm_smem_bytes(int bn, int stages) {
    return (size_t) stages * (128 * 128 + bn * 128) + 256 + 1024;
}

namespace {
using KernelFn = void (*)(CUtensorMap, CUtensorMap, GemmArgs, int);

template <int BN, int EPI>
KernelFn pick() {
    constexpr int ST = BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static_assert(GemmSmem<BN, ST>::TOTAL <= 232448, "smem budget");
    return (KernelFn) gemm_tc_kernel<BN, EPI, ST>;
}

template <int BN>
KernelFn pick_epi(int epi) {
    switch (epi) {
        case EPI_F32: return pick<BN, EPI_F32>();
        case EPI_F16: return pick<BN, EPI_F16>();
        case EPI_F16_SILU: return pick<BN, EPI_F16_SILU>();
        case EPI_SWIGLU: if constexpr (BN % 128 == 0) return pick<BN, EPI_SWIGLU>(); else return nullptr;
        case EPI_GATE: return pick<BN, EPI_GATE>();
        case EPI_QKV: return pick<BN, EPI_QKV>();
    }
    return nullptr;
}

KernelFn kernel_for(int bn, int epi) {
    switch (bn) {
        case 64: return pick_epi<64>(epi);
        case 128: return pick_epi<128>(epi);
        case 256: return pick_epi<256>(epi);
    }
    return nullptr;
}
} // namespace

// Set the dynamic shared-memory limit of every instantiation once, outside any stream capture.
cudaError_t configure_gemm_kernels() {
    for (int bn : {64, 128, 256})
        for (int epi = 0; epi < 6; ++epi) {
            KernelFn fn = kernel_for(bn, epi);
            if (!fn) continue;
            cudaError_t e = cudaFuncSetAttribute((const void *) fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int) gemm_smem_bytes(bn, gemm_stages(bn)));
            if (e != cudaSuccess) return e;
        }
    return cudaSuccess;
}

cudaError_t launch_gemm(const GemmLaunch & g, cudaStream_t s) {
    KernelFn fn = kernel_for(g.bn, g.epi);
    if (!fn) return cudaErrorInvalidValue;
    fn<<<g.grid, 192, g.smem, s>>>(g.ta, g.tb, g.args, g.ab_bf16);
    return cudaGetLastError();
}

} // namespace tsn
