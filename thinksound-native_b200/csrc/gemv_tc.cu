// gemv_tc.cu — the step's clip/text adaLN modulation GEMVs on the tensor cores.
//
// Every joint block's clip and text streams take their adaLN modulation from one gemv_h each
// (shaders/gemm_attn.metal:48-64, called at src/dit_fwd.cpp:195-207): y_b = W · silu(global_c_b) + bias
// for the CFG arms b, W f16 [6H][H] (2H for the last block). At the 8 s geometry the 14 jobs stream
// 159 MB of weights per step, so the bound is HBM. Here the weights are the M operand of a tcgen05
// product instead of a CUDA-core dot product:
//   * each 128-row weight tile x 64-wide K block is one TMA load (128-byte swizzle) into a ring of
//     GTC_STAGES stages, 160 KB in flight per SM;
//   * the arms form the N operand: row 2b holds f16(x_b), row 2b + 1 its residual f16(x_b - f16(x_b)),
//     so each arm's product is exact to ~2^-22 of x as in the library's split GEMMs. The 16 x K tile is
//     built in shared memory once per CTA (128-byte swizzle by hand) and stays resident;
//   * one CTA per SM walks the 128-row tiles of all jobs (tile t, t + grid, ...); the accumulator
//     (16 columns) is double-buffered in TMEM so a tile's epilogue overlaps the next tile's products;
//     y_b[row] = acc[row][2b] + acc[row][2b + 1] + bias[row].
// Warp 4 issues the TMA loads (weights do not depend on the upstream kernel: no wait), warp 5's
// elected thread the UMMAs (after the N tile is built), warps 0-3 build the N tile and run the
// epilogue. Every wait is bounded; a CTA that gives up waits (bounded) for its issued copies and
// UMMAs before it frees its TMEM.
#include <cudaTypedefs.h>

#include <algorithm>

#include "kernels.h"

namespace tsn {

namespace {

constexpr int GTC_STAGES = 10;
constexpr int GTC_A_BYTES = 128 * 128;                     // 128 weight rows x 64 f16
constexpr int GTC_B_KB_BYTES = 16 * 128;                   // 16 N rows x 64 f16, per K block
constexpr int GTC_RING = GTC_STAGES * GTC_A_BYTES;
constexpr int GTC_B_OFF = GTC_RING;                         // N tile: K / 64 blocks of GTC_B_KB_BYTES
constexpr int GTC_BAR_OFF = GTC_B_OFF + (GEMV_MAX_K / 64) * GTC_B_KB_BYTES;
constexpr size_t GTC_SMEM = (size_t) GTC_BAR_OFF + 256 + 1024;

struct GemvTcMaps { CUtensorMap w[GEMV_MAX_JOBS]; };
struct GemvTcArgs {
    int njobs, K, nb, total_tiles;
    int tile_end[GEMV_MAX_JOBS];      // 128-row tiles of jobs 0..q
    float * y[GEMV_MAX_JOBS];
    long long y_bs[GEMV_MAX_JOBS];
    const float * bias[GEMV_MAX_JOBS];
    int N[GEMV_MAX_JOBS];
    const float * x;                  // arm b at x + b * x_bs, K floats
    long long x_bs;
    int * err;
    unsigned long long * trace;       // 3 stamps per CTA (entry, upstream done, exit), or null
};

__global__ void __launch_bounds__(192, 1) gemv_tc_kernel(const __grid_constant__ GemvTcMaps maps,
                                                         const __grid_constant__ GemvTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + GTC_BAR_OFF);
    uint64_t * empty = full + GTC_STAGES;
    uint64_t * accf = empty + GTC_STAGES;      // [2] accumulator buffer ready for the epilogue
    uint64_t * acce = accf + 2;                // [2] accumulator buffer read by the epilogue (4 arrivals)
    uint64_t * bready = acce + 2;              // N tile built (128 arrivals)
    uint64_t * drain = bready + 1;
    uint32_t * tslot = (uint32_t *) (drain + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = a.K / 64;
    unsigned long long * tr = a.trace ? a.trace + 3 * blockIdx.x : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();

    if (threadIdx.x == 0) {
        for (int s = 0; s < GTC_STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 4); }
        mbar_init(bready, 128);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4 && lane == 0) for (int q = 0; q < a.njobs; ++q) tma_prefetch(&maps.w[q]);
    if (warp == 5) tmem_alloc(tslot, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_trigger();
    const uint32_t tmem = *tslot;
    int issued = 0;

    if (warp == 4) {
        if (lane == 0) {
            int g = 0, q = 0;
            for (int t = blockIdx.x; t < a.total_tiles; t += gridDim.x) {
                while (q + 1 < a.njobs && t >= a.tile_end[q]) ++q;
                const int row0 = (t - (q ? a.tile_end[q - 1] : 0)) * 128;
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % GTC_STAGES;
                    if (g >= GTC_STAGES &&
                        !(ok = mbar_wait(&empty[s], ((g / GTC_STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY)))
                        break;
                    mbar_expect_tx(&full[s], (uint32_t) GTC_A_BYTES);
                    tma_load_2d(smem + s * GTC_A_BYTES, &maps.w[q], &full[s], kb * 64, row0);
                    issued = g + 1;
                }
                if (!ok) break;
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(16, 0);
            bool ok = mbar_wait(bready, 0, abort_flag, a.err, DEV_TIMEOUT_FULL);
            int g = 0, lt = 0;
            for (int t = blockIdx.x; t < a.total_tiles && ok; t += gridDim.x, ++lt) {
                const int buf = lt & 1;
                if (lt >= 2 && !(ok = mbar_wait(&acce[buf], ((lt >> 1) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)))
                    break;
                tc_fence_after();
                const uint32_t d = tmem + 16u * (uint32_t) buf;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % GTC_STAGES;
                    if (!(ok = mbar_wait(&full[s], (g / GTC_STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL))) break;
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem + s * GTC_A_BYTES);
                    const uint64_t bd = umma_desc_sw128(smem + GTC_B_OFF + kb * GTC_B_KB_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_f16(d, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (kb | k) != 0);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&accf[buf]);
            }
            if (!ok) {   // let every UMMA issued so far complete before the TMEM is freed
                umma_commit(drain);
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000ull) {}
            }
        }
    } else {
        pdl_wait();   // x is the upstream kernel's output
        if (tr && threadIdx.x == 0) tr[1] = global_ns();
        {   // the N tile: row 2b = f16(x_b), row 2b + 1 = its residual, rows 2 nb.. zero; K-major,
            // 128-byte rows per K block, 16-byte chunk c of row r at chunk c ^ (r & 7)
            uint8_t * bt = smem + GTC_B_OFF;
            const int chunks = 16 * (a.K / 8);
            for (int i = threadIdx.x; i < chunks; i += 128) {
                const int r = i / (a.K / 8), c8 = i % (a.K / 8);
                const int k0 = c8 * 8, kb = k0 >> 6, c = (k0 & 63) >> 3;
                const int arm = r >> 1;
                __align__(16) __half h[8];
                if (arm < a.nb) {
                    const float4 v0 = *(const float4 *) (a.x + arm * a.x_bs + k0);
                    const float4 v1 = *(const float4 *) (a.x + arm * a.x_bs + k0 + 4);
                    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const __half hi = __float2half_rn(v[e]);
                        h[e] = (r & 1) ? __float2half_rn(v[e] - __half2float(hi)) : hi;
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(0.0f);
                }
                *(uint4 *) (bt + kb * GTC_B_KB_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) = *(const uint4 *) h;
            }
            fence_proxy_async_smem();   // this thread's writes, visible to the tensor core's reads
            mbar_arrive(bready);
        }
        const uint32_t lane_off = (uint32_t) (warp * 32) << 16;
        int q = 0, lt = 0;
        for (int t = blockIdx.x; t < a.total_tiles; t += gridDim.x, ++lt) {
            while (q + 1 < a.njobs && t >= a.tile_end[q]) ++q;
            const int buf = lt & 1;
            if (!mbar_wait(&accf[buf], (lt >> 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
            tc_fence_after();
            float v[16];
            tmem_ld16(tmem + lane_off + 16u * (uint32_t) buf, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[buf]);
            const int row = (t - (q ? a.tile_end[q - 1] : 0)) * 128 + warp * 32 + lane;
            if (row < a.N[q]) {
                const float bias = a.bias[q] ? a.bias[q][row] : 0.0f;
                for (int b = 0; b < a.nb; ++b) a.y[q][b * a.y_bs[q] + row] = (v[2 * b] + v[2 * b + 1]) + bias;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && warp == 4 && lane == 0) {
        // copies issued for stages nobody consumed must land before this CTA's shared memory is reused
        const uint64_t t0 = global_ns();
        for (int i = std::max(0, issued - GTC_STAGES); i < issued; ++i)
            while (!mbar_try_wait(&full[i % GTC_STAGES], (i / GTC_STAGES) & 1) && global_ns() - t0 < 1000000ull) {}
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
    if (tr && threadIdx.x == 0) tr[2] = global_ns();
}

} // namespace

cudaError_t configure_gemv_tc() {
    return cudaFuncSetAttribute(gemv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) GTC_SMEM);
}

int gemv_tc_blocks(const GemvJob * jobs, int njobs, int sms) {
    long long tiles = 0;
    for (int q = 0; q < njobs; ++q) tiles += (jobs[q].N + 127) / 128;
    return (int) std::min<long long>(tiles, sms);
}

cudaError_t launch_gemv_tc(const GemvJob * jobs, int njobs, int sms, int * err, cudaStream_t s,
                           unsigned long long * trace) {
    if (njobs < 1 || njobs > GEMV_MAX_JOBS || sms < 1) return cudaErrorInvalidValue;
    GemvTcMaps maps{};
    GemvTcArgs a{};
    a.njobs = njobs;
    a.K = jobs[0].K;
    a.nb = jobs[0].nb;
    a.x = jobs[0].x;
    a.x_bs = jobs[0].x_bs;
    a.err = err;
    a.trace = trace;
    if (a.K < 64 || a.K > GEMV_MAX_K || a.K % 64 || a.nb < 1 || a.nb > 8 || ((uintptr_t) a.x & 15) || a.x_bs % 4)
        return cudaErrorInvalidValue;
    int tiles = 0;
    for (int q = 0; q < njobs; ++q) {
        const GemvJob & j = jobs[q];
        if (j.K != a.K || j.nb != a.nb || j.x != a.x || j.x_bs != a.x_bs || j.x_step || j.act || j.N < 1 ||
            !make_w_map(&maps.w[q], j.W, (uint64_t) a.K, (uint64_t) j.N, 128, 0))
            return cudaErrorInvalidValue;
        tiles += (j.N + 127) / 128;
        a.tile_end[q] = tiles;
        a.y[q] = j.y;
        a.y_bs[q] = j.y_bs;
        a.bias[q] = j.bias;
        a.N[q] = j.N;
    }
    a.total_tiles = tiles;
    const int grid = std::min(tiles, sms);
    return launch_ex(gemv_tc_kernel, dim3(grid), dim3(192), GTC_SMEM, s, 1u, maps, a);
}

} // namespace tsn
