// gemm_lo8.cu — a split-operand GEMM whose low-order product runs on the 8-bit tensor path.
//
// The library's split GEMM computes X·W^T as Xh·W + Xl·W with Xh = f16(X), Xl = f16(X - Xh), both
// products on the f16 tensor path (kind::f16), which doubles the tensor work of a single-operand
// GEMM. Here the low-order product uses e4m3 operands instead:
//   Xl8 = e4m3(2^12 (X - Xh)),  W8 = e4m3(2^wexp W)   (per-tensor power-of-two scales)
//   Y   = acc_hi + 2^-(12 + wexp) acc_lo,  acc_hi = Xh·W (kind::f16), acc_lo = Xl8·W8 (kind::f8f6f4)
// An e4m3 product of K = 32 issues in the time of an f16 product of K = 16, so the tensor work per
// 64-wide K block falls from eight f16 instruction times to six. The low-order term is ~2^-12 of X
// and e4m3 keeps it to ~2^-4, so the product is exact to ~2^-16 of X·W against ~2^-12 for a single
// f16 operand. Xl8 saturates for |X| >= 2^8 (|X - Xh| * 2^12 > 448) and W8 for |W| * 2^wexp > 448.
//
// Warp-specialised like gemm_tc_kernel: warp 4 issues the TMA loads of a stage (Xh and W with
// 128-byte swizzle, Xl8 and W8 with 64-byte swizzle), warp 5's elected thread issues the UMMAs into
// two TMEM accumulators (hi at column 0, lo at column BN), warps 0-3 combine them and store f32
// rows. Every wait is bounded; a CTA that gives up lets its issued UMMAs complete (bounded) before
// the TMEM is freed. Reached through tsn_selftest_gemm_lo8 only: no model path uses it. The file
// also holds gemm_splitkb_kernel, the split f16 product with 64- or 32-wide K blocks, the control
// these experiments are timed against. Measured at the step's GEMM shapes, neither form beats
// the production kernel's 64-wide K blocks and 4-stage ring at 176-wide tiles.
#include <cudaTypedefs.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <functional>
#include <string>

#include "kernels.h"
#include "runtime.h"

namespace tsn {

namespace {

constexpr int LO8_X_EXP = 12;

#define LO8_CK(expr)                                                                              \
    do {                                                                                          \
        cudaError_t e_ = (expr);                                                                  \
        if (e_ != cudaSuccess) return fail(TSN_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

template <int BN> struct Lo8Smem {
    static constexpr int AH = 128 * 128;             // Xh: 128 rows x 64 f16, 128-byte rows
    static constexpr int BH = BN * 128;              // W: BN rows x 64 f16
    static constexpr int A8 = 128 * 64;              // Xl8: 128 rows x 64 e4m3, 64-byte rows
    static constexpr int B8 = BN * 64;               // W8: BN rows x 64 e4m3
    static constexpr int OFF_BH = AH, OFF_A8 = AH + BH, OFF_B8 = AH + BH + A8;
    static constexpr int STAGE = AH + BH + A8 + B8;
    static_assert(OFF_BH % 1024 == 0 && OFF_A8 % 1024 == 0 && OFF_B8 % 1024 == 0 && STAGE % 1024 == 0,
                  "every operand tile starts on a 1024-byte boundary (the swizzle atoms' alignment)");
};
template <int BN, int STAGES> constexpr size_t lo8_smem_bytes() {
    return (size_t) STAGES * Lo8Smem<BN>::STAGE + 256 + 1024;   // barriers, slot, flag; alignment slack
}

// Shared-memory matrix descriptor, K-major, 64-byte swizzle: 64-byte rows, 8-row core groups 512 B
// apart (the layout a CU_TENSOR_MAP_SWIZZLE_64B load with a 64-byte inner box leaves).
__device__ __forceinline__ uint64_t umma_desc_sw64(const void * smem_tile) {
    const uint32_t a = smem_u32(smem_tile);
    uint64_t d = 0;
    d |= (uint64_t) ((a & 0x3FFFFu) >> 4);          // start address   [0,14)
    d |= (uint64_t) 1u << 16;                        // LBO (unused for swizzled K-major)
    d |= (uint64_t) (512u >> 4) << 32;               // SBO = 512 B     [32,46)
    d |= (uint64_t) 1u << 46;                        // descriptor version (sm100)
    d |= (uint64_t) 4u << 61;                        // layout: SWIZZLE_64B
    return d;
}

// D[tmem] (+)= A[smem] · B[smem]^T with e4m3 operands, M = 128, one elected thread issues. The
// instruction descriptor's format fields read E4M3 = 0 for A and B.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

struct Lo8Args {
    int M, N, k_blocks;
    float out_scale;          // 2^-(12 + wexp)
    const float * bias;       // [N] or null
    float * y;                // [M][ldy]
    int ldy;
    int * err;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_lo8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA8,
                const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB8, const Lo8Args a) {
    using L = Lo8Smem<BN>;
    constexpr uint32_t TCOLS = 2 * BN <= 256 ? 256u : 512u;
    static_assert(2 * BN <= 512 && BN % 16 == 0, "two BN-column accumulators must fit in TMEM");
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + STAGES * L::STAGE);
    uint64_t * empty = full + STAGES;
    uint64_t * tfull = empty + STAGES;
    uint64_t * drain = tfull + 1;
    uint32_t * tslot = (uint32_t *) (drain + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128, nk = a.k_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmA8); tma_prefetch(&tmB); tma_prefetch(&tmB8); }
    if (warp == 5) tmem_alloc(tslot, TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t acc_hi = tmem, acc_lo = tmem + (uint32_t) BN;
    int issued = 0;   // warp 4, lane 0: stages whose loads were issued

    if (warp == 4) {
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY))
                    break;
                uint8_t * sa = smem + s * L::STAGE;
                mbar_expect_tx(&full[s], (uint32_t) L::STAGE);
                tma_load_3d(sa, &tmA, &full[s], i * 64, m0, 0);   // {K, rows, 1} view
                tma_load_2d(sa + L::OFF_BH, &tmB, &full[s], i * 64, n0);
                tma_load_2d(sa + L::OFF_A8, &tmA8, &full[s], i * 64, m0);
                tma_load_2d(sa + L::OFF_B8, &tmB8, &full[s], i * 64, n0);
                issued = i + 1;
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            // f16 x f16 and e4m3 x e4m3 share the descriptor: format code 0 for A and B in both kinds
            const uint32_t idesc = umma_idesc_f16(BN, 0);
            bool ok = true;
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (!(ok = mbar_wait(&full[s], (i / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL))) break;
                tc_fence_after();
                const uint8_t * sa = smem + s * L::STAGE;
                const uint64_t ad = umma_desc_sw128(sa), bd = umma_desc_sw128(sa + L::OFF_BH);
                const uint64_t a8 = umma_desc_sw64(sa + L::OFF_A8), b8 = umma_desc_sw64(sa + L::OFF_B8);
#pragma unroll
                for (int k = 0; k < 4; ++k)   // K = 16 f16 per instruction: 32 bytes along the row
                    umma_f16(acc_hi, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (i | k) != 0);
#pragma unroll
                for (int k = 0; k < 2; ++k)   // K = 32 e4m3 per instruction: 32 bytes along the row
                    umma_f8(acc_lo, a8 + (uint64_t) (2 * k), b8 + (uint64_t) (2 * k), idesc, (i | k) != 0);
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(tfull);
            else {   // let every UMMA issued so far complete before the TMEM is freed
                umma_commit(drain);
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000ull) {}
            }
        }
    } else {
        pdl_wait();
        const bool ok = mbar_wait(tfull, 0, abort_flag, a.err, DEV_TIMEOUT_TMEM) && !*abort_flag;
        tc_fence_after();
        if (ok) {
            const int row = m0 + warp * 32 + lane;
            const uint32_t lane_off = (uint32_t) (warp * 32) << 16;
            float * yr = a.y + (size_t) row * a.ldy;
            const bool vec = (a.ldy % 4) == 0 && ((uintptr_t) a.y & 15) == 0;
            for (int c = 0; c < BN; c += 32) {
                float h[32], l[32];
                const int w = c + 32 <= BN ? 32 : 16;   // the same for every lane: the loads are warp-collective
                if (w == 32) {
                    tmem_ld32(acc_hi + lane_off + (uint32_t) c, h);
                    tmem_ld32(acc_lo + lane_off + (uint32_t) c, l);
                } else {
                    tmem_ld16(acc_hi + lane_off + (uint32_t) c, h);
                    tmem_ld16(acc_lo + lane_off + (uint32_t) c, l);
                }
                if (row < a.M) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        if (e >= w) break;
                        const int n = n0 + c + e;
                        float v[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            v[q] = fmaf(l[e + q], a.out_scale, h[e + q]) + (a.bias && n + q < a.N ? a.bias[n + q] : 0.0f);
                        if (vec && n + 3 < a.N) *(float4 *) (yr + n) = make_float4(v[0], v[1], v[2], v[3]);
                        else
                            for (int q = 0; q < 4; ++q)
                                if (n + q < a.N) yr[n + q] = v[q];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && warp == 4 && lane == 0) {
        // loads issued for stages nobody consumed must land before this CTA's shared memory is reused
        const uint64_t t0 = global_ns();
        for (int i = issued - STAGES < 0 ? 0 : issued - STAGES; i < issued; ++i)
            while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && global_ns() - t0 < 1000000ull) {}
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TCOLS);
    }
}

// The same split f16 product as the library's GEMM (Xh·W + Xl·W into one accumulator) with the K
// block as a parameter, to measure the stage ring's depth against its stage size: KB = 64 keeps
// 128-byte rows (128-byte swizzle), KB = 32 keeps 64-byte rows (64-byte swizzle) and fits twice the
// stages in the same shared memory. Epilogue and roles as gemm_lo8_kernel.
template <int BN, int KB> struct SplitKbSmem {
    static constexpr int ROW = KB * 2;
    static constexpr int AT = 128 * ROW, BT = BN * ROW;
    static constexpr int OFF_AL = AT, OFF_B = 2 * AT;
    static constexpr int STAGE = 2 * AT + BT;
    static_assert(AT % 1024 == 0 && BT % 1024 == 0, "operand tiles start on 1024-byte boundaries");
};
template <int BN, int KB, int STAGES> constexpr size_t splitkb_smem_bytes() {
    return (size_t) STAGES * SplitKbSmem<BN, KB>::STAGE + 256 + 1024;
}

template <int BN, int KB, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_splitkb_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                    const __grid_constant__ CUtensorMap tmB, const Lo8Args a) {
    using L = SplitKbSmem<BN, KB>;
    static_assert(KB == 64 || KB == 32, "K blocks of 64 (128-byte rows) or 32 (64-byte rows)");
    constexpr uint32_t TCOLS = BN <= 128 ? 128u : 256u;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + STAGES * L::STAGE);
    uint64_t * empty = full + STAGES;
    uint64_t * tfull = empty + STAGES;
    uint64_t * drain = tfull + 1;
    uint32_t * tslot = (uint32_t *) (drain + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128, nk = a.k_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmA2); tma_prefetch(&tmB); }
    if (warp == 5) tmem_alloc(tslot, TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    int issued = 0;

    if (warp == 4) {
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY))
                    break;
                uint8_t * sa = smem + s * L::STAGE;
                mbar_expect_tx(&full[s], (uint32_t) L::STAGE);
                tma_load_2d(sa, &tmA, &full[s], i * KB, m0);
                tma_load_2d(sa + L::OFF_AL, &tmA2, &full[s], i * KB, m0);
                tma_load_2d(sa + L::OFF_B, &tmB, &full[s], i * KB, n0);
                issued = i + 1;
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(BN, 0);
            bool ok = true;
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (!(ok = mbar_wait(&full[s], (i / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL))) break;
                tc_fence_after();
                const uint8_t * sa = smem + s * L::STAGE;
                const uint64_t ad = KB == 64 ? umma_desc_sw128(sa) : umma_desc_sw64(sa);
                const uint64_t al = KB == 64 ? umma_desc_sw128(sa + L::OFF_AL) : umma_desc_sw64(sa + L::OFF_AL);
                const uint64_t bd = KB == 64 ? umma_desc_sw128(sa + L::OFF_B) : umma_desc_sw64(sa + L::OFF_B);
#pragma unroll
                for (int k = 0; k < KB / 16; ++k) {   // K = 16 f16 per instruction: 32 bytes along the row
                    umma_f16(tmem, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (i | k) != 0);
                    umma_f16(tmem, al + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, 1u);
                }
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(tfull);
            else {
                umma_commit(drain);
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000ull) {}
            }
        }
    } else {
        pdl_wait();
        const bool ok = mbar_wait(tfull, 0, abort_flag, a.err, DEV_TIMEOUT_TMEM) && !*abort_flag;
        tc_fence_after();
        if (ok) {
            const int row = m0 + warp * 32 + lane;
            const uint32_t lane_off = (uint32_t) (warp * 32) << 16;
            float * yr = a.y + (size_t) row * a.ldy;
            const bool vec = (a.ldy % 4) == 0 && ((uintptr_t) a.y & 15) == 0;
            for (int c = 0; c < BN; c += 32) {
                float h[32];
                const int w = c + 32 <= BN ? 32 : 16;
                if (w == 32) tmem_ld32(tmem + lane_off + (uint32_t) c, h);
                else tmem_ld16(tmem + lane_off + (uint32_t) c, h);
                if (row < a.M) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        if (e >= w) break;
                        const int n = n0 + c + e;
                        float v[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) v[q] = h[e + q] + (a.bias && n + q < a.N ? a.bias[n + q] : 0.0f);
                        if (vec && n + 3 < a.N) *(float4 *) (yr + n) = make_float4(v[0], v[1], v[2], v[3]);
                        else
                            for (int q = 0; q < 4; ++q)
                                if (n + q < a.N) yr[n + q] = v[q];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && warp == 4 && lane == 0) {
        const uint64_t t0 = global_ns();
        for (int i = issued - STAGES < 0 ? 0 : issued - STAGES; i < issued; ++i)
            while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && global_ns() - t0 < 1000000ull) {}
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TCOLS);
    }
}

// X f32 [M][K] -> Xh f16 [M][K] and Xl8 = e4m3(2^12 (X - Xh)) [M][K]
__global__ void k_split_lo8(const float * x, long long n, __half * xh, __nv_fp8_storage_t * xl8) {
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const float v = x[i];
        const __half h = __float2half_rn(v);
        xh[i] = h;
        xl8[i] = __nv_cvt_float_to_fp8((v - __half2float(h)) * (float) (1 << LO8_X_EXP), __NV_SATFINITE, __NV_E4M3);
    }
}
// X f32 [M][K] -> the library's split f16 operand: hi [M][K], lo [M][K] right after it
__global__ void k_split_f16(const float * x, long long n, __half * out) {
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const float v = x[i];
        const __half h = __float2half_rn(v);
        out[i] = h;
        out[i + n] = __float2half_rn(v - __half2float(h));
    }
}
// W f16 [N][K] -> W8 = e4m3(2^wexp W)
__global__ void k_w8(const __half * w, long long n, float scale, __nv_fp8_storage_t * w8) {
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x)
        w8[i] = __nv_cvt_float_to_fp8(__half2float(w[i]) * scale, __NV_SATFINITE, __NV_E4M3);
}

// 2-D tensor map over a row-major [rows][K] array of esize-byte elements; box {inner, box_rows}
bool make_map_2d(CUtensorMap * m, const void * base, CUtensorMapDataType dt, uint32_t esize, uint64_t K, uint64_t rows,
                 uint32_t inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    // looked up once; a function-local static is initialised once even when threads race to it
    static const PFN_cuTensorMapEncodeTiled_v12000 enc = [] {
        cudaDriverEntryPointQueryResult q{};
        void * fn = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000) fn;
    }();
    if (!enc || ((uintptr_t) base & 15) || (K * esize) % 16 || K % inner || box_rows == 0 || box_rows > 256) return false;
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {K * esize};
    const cuuint32_t box[2] = {inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, dt, 2, (void *) base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
bool make_u8_map(CUtensorMap * m, const void * base, uint64_t K, uint64_t rows, uint32_t box_rows) {
    // 64 bytes inner: one 64-byte swizzle span
    return make_map_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, rows, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_64B);
}
bool make_f16_map(CUtensorMap * m, const void * base, uint64_t K, uint64_t rows, uint32_t kb, uint32_t box_rows) {
    return make_map_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, rows, kb, box_rows,
                       kb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

template <int BN, int KB, int STAGES>
cudaError_t launch_splitkb(const CUtensorMap & ta, const CUtensorMap & ta2, const CUtensorMap & tb, const Lo8Args & a,
                           cudaStream_t s) {
    const size_t smem = splitkb_smem_bytes<BN, KB, STAGES>();
    cudaError_t e = cudaFuncSetAttribute(gemm_splitkb_kernel<BN, KB, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    gemm_splitkb_kernel<BN, KB, STAGES><<<dim3((a.N + BN - 1) / BN, (a.M + 127) / 128), 192, smem, s>>>(ta, ta2, tb, a);
    return cudaGetLastError();
}

template <int BN, int STAGES>
cudaError_t launch_lo8(const CUtensorMap & ta, const CUtensorMap & ta8, const CUtensorMap & tb, const CUtensorMap & tb8,
                       const Lo8Args & a, cudaStream_t s) {
    const size_t smem = lo8_smem_bytes<BN, STAGES>();
    cudaError_t e = cudaFuncSetAttribute(gemm_lo8_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    gemm_lo8_kernel<BN, STAGES><<<dim3((a.N + BN - 1) / BN, (a.M + 127) / 128), 192, smem, s>>>(ta, ta8, tb, tb8, a);
    return cudaGetLastError();
}

struct DevBuf {
    void * p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
};

} // namespace

// mode 0: the e4m3 low-order GEMM (tile width bn in {128, 176, 256}); mode 1: the library's split
// f16 GEMM (gemm_tc_kernel, f32 output, bn in {128, 256}); modes 2 and 3: gemm_splitkb_kernel with
// K blocks of 64 and 32 (bn in {128, 176, 256}); + 4: no L2 eviction between launches.
// Operands are prepared outside the timed region; each of the reps launches is timed alone with
// CUDA events, after a write of 256 MiB that evicts L2 unless mode has bit 2 set, and *ms receives
// the mean.
int selftest_gemm_lo8(DeviceCtx & c, const void * W, const void * X, void * Y, const void * bias, uint32_t M, uint32_t N,
                      uint32_t K, int wexp, int mode, int bn, int reps, float * ms) {
    const bool warm = (mode & 4) != 0;   // no L2-evicting write between the timed launches
    mode &= 3;
    if (!W || !X || !Y || !M || !N || K % 64 || K > 65536 || reps < 1 || reps > 100 || wexp < -8 || wexp > 24)
        return fail(TSN_ERR_ARG, "selftest_gemm_lo8: bad arguments");
    if (mode == 1 ? (bn != 128 && bn != 256) || N % bn : (bn != 128 && bn != 176 && bn != 256))
        return fail(TSN_ERR_ARG, "selftest_gemm_lo8: bad mode or tile width (mode 1 needs N a multiple of bn)");
    const long long nx = (long long) M * K, nw = (long long) N * K;
    DevBuf xa, w8, flush;
    if (cudaMalloc(&xa.p, (size_t) nx * 4) != cudaSuccess || (mode == 0 && cudaMalloc(&w8.p, (size_t) nw) != cudaSuccess) ||
        cudaMalloc(&flush.p, (size_t) 256 << 20) != cudaSuccess)
        return fail(TSN_ERR_OOM, "selftest_gemm_lo8: scratch");
    const unsigned gx = (unsigned) std::min<long long>((nx + 255) / 256, 4096), gw = (unsigned) std::min<long long>((nw + 255) / 256, 4096);
    cudaStream_t s = c.stream;
    std::function<cudaError_t()> run;
    CUtensorMap ta{}, ta8{}, tb{}, tb8{};
    Lo8Args la{};
    GemmLaunch g{};
    if (mode == 0) {
        __half * xh = (__half *) xa.p;
        __nv_fp8_storage_t * xl8 = (__nv_fp8_storage_t *) (xh + nx);
        k_split_lo8<<<gx, 256, 0, s>>>((const float *) X, nx, xh, xl8);
        k_w8<<<gw, 256, 0, s>>>((const __half *) W, nw, ldexpf(1.0f, wexp), (__nv_fp8_storage_t *) w8.p);
        if (!make_act_map(&ta, xh, K, M, 1, 128, 1, 0) || !make_u8_map(&ta8, xl8, K, M, 128) ||
            !make_w_map(&tb, W, K, N, (uint32_t) bn, 0) || !make_u8_map(&tb8, w8.p, K, N, (uint32_t) bn))
            return fail(TSN_ERR_CUDA, "selftest_gemm_lo8: tensor maps");
        la = Lo8Args{(int) M, (int) N, (int) (K / 64), ldexpf(1.0f, -(LO8_X_EXP + wexp)), (const float *) bias, (float *) Y,
                     (int) N, c.d_err};
        run = [&]() {
            return bn == 128 ? launch_lo8<128, 4>(ta, ta8, tb, tb8, la, s)
                 : bn == 176 ? launch_lo8<176, 3>(ta, ta8, tb, tb8, la, s)
                             : launch_lo8<256, 3>(ta, ta8, tb, tb8, la, s);
        };
    } else if (mode >= 2) {
        const uint32_t kb = mode == 2 ? 64u : 32u;
        __half * xs = (__half *) xa.p;
        k_split_f16<<<gx, 256, 0, s>>>((const float *) X, nx, xs);
        if (!make_f16_map(&ta, xs, K, M, kb, 128) || !make_f16_map(&ta8, xs + nx, K, M, kb, 128) ||
            !make_f16_map(&tb, W, K, N, kb, (uint32_t) bn))
            return fail(TSN_ERR_CUDA, "selftest_gemm_lo8: tensor maps");
        la = Lo8Args{(int) M, (int) N, (int) (K / kb), 1.0f, (const float *) bias, (float *) Y, (int) N, c.d_err};
        if (mode == 2)
            run = [&]() {
                return bn == 128 ? launch_splitkb<128, 64, 4>(ta, ta8, tb, la, s)
                     : bn == 176 ? launch_splitkb<176, 64, 4>(ta, ta8, tb, la, s)
                                 : launch_splitkb<256, 64, 3>(ta, ta8, tb, la, s);
            };
        else
            run = [&]() {
                return bn == 128 ? launch_splitkb<128, 32, 8>(ta, ta8, tb, la, s)
                     : bn == 176 ? launch_splitkb<176, 32, 8>(ta, ta8, tb, la, s)
                                 : launch_splitkb<256, 32, 6>(ta, ta8, tb, la, s);
            };
    } else {
        __half * xs = (__half *) xa.p;
        k_split_f16<<<gx, 256, 0, s>>>((const float *) X, nx, xs);
        g.bn = bn; g.epi = EPI_F32; g.split = true; g.smem = gemm_smem_bytes(bn, true, EPI_F32); g.ab_bf16 = 0;
        g.grid = dim3(N / bn + (N % bn ? 1 : 0), (M + 127) / 128, 1);
        if (!make_act_map(&g.ta, xs, K, M, 1, 128, 1, 0) || !make_act_map(&g.ta2, xs + nx, K, M, 1, 128, 1, 0) ||
            !make_w_map(&g.tb, W, K, N, (uint32_t) bn, 0))
            return fail(TSN_ERR_CUDA, "selftest_gemm_lo8: tensor maps");
        GemmArgs & ga = g.args;
        ga.rows = (int) M; ga.B = 1; ga.bt = 128; ga.bb = 1; ga.m_tiles_t = (int) ((M + 127) / 128); ga.N = (int) N;
        ga.k_blocks = (int) (K / 64); ga.ic_blocks = (int) (K / 64); ga.pad = 0; ga.splits = 1; ga.kb_per_split = ga.k_blocks;
        ga.err = c.d_err; ga.bias = (const float *) bias; ga.out = Y; ga.ldo = N; ga.out_bs = 0;
        run = [&]() { return launch_gemm(g, s); };
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("selftest_gemm_lo8 prep: ") + cudaGetErrorString(e));
    cudaEvent_t e0, e1;
    LO8_CK(cudaEventCreate(&e0));
    LO8_CK(cudaEventCreate(&e1));
    double total = 0.0;
    for (int r = 0; r < reps && e == cudaSuccess; ++r) {
        if (!warm) e = cudaMemsetAsync(flush.p, r & 0xFF, (size_t) 256 << 20, s);
        if (e == cudaSuccess) e = cudaEventRecord(e0, s);
        if (e == cudaSuccess) e = run();
        if (e == cudaSuccess) e = cudaEventRecord(e1, s);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float t = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
        total += t;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("selftest_gemm_lo8: ") + cudaGetErrorString(e));
    if (int rc = c.sync()) return rc;
    if (ms) *ms = (float) (total / reps);
    return TSN_OK;
}

} // namespace tsn
