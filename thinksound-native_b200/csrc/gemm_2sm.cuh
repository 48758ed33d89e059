// gemm_2sm.cuh — the CTA-pair (cta_group::2) tcgen05 GEMM with weights on the M side.
//
// Same product as gemm_tc.cuh, Y[token][n] = sum_k X[token][k] W[n][k], but computed as
// D[n][token] = W · X^T so that the large output-feature dimension is the MMA's M and the few
// tokens (2 CFG arms x 188 rows at 8 s) its N. Two CTAs on neighbouring SMs form a cluster pair:
// each loads 128 weight rows (its half of M = 256) and half of the NT-token activation tile
// (f16, split hi + lo or plain), and the pair leader issues tcgen05.mma.cta_group::2 over both CTAs' shared
// memory into both CTAs' TMEM (split f16 activations: a hi and a lo UMMA per K step; plain f16 for
// the FFN down-projection). Per SM and per MMA cycle this moves ~30 % fewer operand bytes than
// the single-CTA kernel (which holds a whole weight tile per SM), so the same ring depth hides
// more of the weight-tile latency. Each CTA's epilogue owns its 128 output features: lanes are
// consecutive features, so every store instruction writes one token's contiguous feature run.
//
//   warp 4 (both CTAs)  TMA: weight rows and activation half-tile per 64-wide K block into a
//                       STAGES-deep ring; the bytes of both CTAs are counted on the leader's barrier
//   warp 5 (leader)     M=256 x N=NT x K=16 UMMAs (hi, then lo) into TMEM; commits release the
//                       stage in both CTAs and finally signal both CTAs' epilogues
//   warps 0-3           tcgen05.ld of the CTA's 128 feature rows x NT tokens; f32 (+bias, or
//                       split-K partial tile) or SwiGLU f16 output
// Split-K (grid.z) gives independent K slices, each writing its own partial tile (EPI_F32 with
// part_stride); there is no in-kernel split-K reduction. No TMA load uses multicast.
#pragma once
#include "gemm_tc.cuh"

namespace tsn {

template <int NT, int STAGES, bool SPLIT>
struct Gemm2Smem {
    static constexpr int W_BYTES = 128 * 128;              // 128 weight rows x 64 K f16
    static constexpr int X_BYTES = (NT / 2) * 128;         // this CTA's NT/2 tokens x 64 K f16, one half
    static constexpr int X_OFF = W_BYTES;
    static constexpr int STAGE = W_BYTES + (SPLIT ? 2 : 1) * X_BYTES;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int TOTAL = BAR_OFF + 256 + 1024;    // barriers, TMEM slot, abort flag + alignment slack
    static_assert(X_BYTES % 1024 == 0, "activation half-tiles must stay 1024-byte aligned");
};

template <int NT, int EPI, int STAGES, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
gemm2_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
             const __grid_constant__ CUtensorMap tmX2, const __grid_constant__ CUtensorMap tmY, const GemmArgs a) {
    using L = Gemm2Smem<NT, STAGES, SPLIT>;
    static_assert(EPI == EPI_F32 || EPI == EPI_SWIGLU, "2-SM epilogues: f32 / partial f32, SwiGLU");
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + L::BAR_OFF);    // used on the leader only
    uint64_t * empty = full + STAGES;
    uint64_t * tfull = empty + STAGES;
    uint32_t * tslot = (uint32_t *) (tfull + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();                  // 0: pair leader
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    unsigned long long * tr = a.trace ? a.trace + (size_t) cta * TRACE_SLOTS : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    const int n0 = (blockIdx.x >> 1) * 256 + (int) rank * 128;      // this CTA's 128 weight rows
    const int b = blockIdx.y / a.m_tiles_t, t0 = (blockIdx.y % a.m_tiles_t) * NT;   // the pair's token tile
    const int tx = t0 + (int) rank * (NT / 2);             // this CTA's half of the tokens
    const int kb_begin = blockIdx.z * a.kb_per_split;
    const int kb_end = min(a.k_blocks, kb_begin + a.kb_per_split);
    const int nk = kb_end - kb_begin;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 0) pdl_trigger();
    if (warp == 4 && lane == 0) {
        tma_prefetch(&tmW);
        tma_prefetch(&tmX);
        if (SPLIT) tma_prefetch(&tmX2);
    }
    if (warp == 5) tmem_alloc2(tslot, TmemCols<NT>::N);
    // both CTAs' barriers are initialised and their TMEM allocated before either side proceeds
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tr && threadIdx.x == 0) tr[1] = global_ns();

    if (warp == 4) {
        if (lane == 0) {
            uint32_t full_leader[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) full_leader[s] = dsmem_map(smem_u32(&full[s]), 0);
            // weights do not depend on the upstream kernel: issue the first stages' weight rows now
            const int pre = nk < STAGES ? nk : STAGES;
            for (int i = 0; i < pre; ++i) {
                if (rank == 0) mbar_expect_tx(&full[i], 2 * L::STAGE);
                tma_load_2d_cg2(smem + i * L::STAGE, &tmW, full_leader[i], (kb_begin + i) * 64, n0);
            }
            pdl_wait();
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY))
                    break;
                const int kb = kb_begin + i;
                const int tap = kb / a.ic_blocks, ic0 = (kb % a.ic_blocks) * 64;
                uint8_t * st = smem + s * L::STAGE;
                if (i >= pre) {
                    if (rank == 0) mbar_expect_tx(&full[s], 2 * L::STAGE);
                    tma_load_2d_cg2(st, &tmW, full_leader[s], kb * 64, n0);
                }
                const int row = tx + tap * (a.dil > 1 ? a.dil : 1) - a.pad;
                tma_load_3d_cg2(st + L::X_OFF, &tmX, full_leader[s], ic0, row, b);
                if (SPLIT) tma_load_3d_cg2(st + L::X_OFF + L::X_BYTES, &tmX2, full_leader[s], ic0, row, b);
            }
        }
    } else if (warp == 5) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = umma_idesc_f16(NT, 0, 0, 256);
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&full[s], (i / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL)) break;
                if (tr && i == 0) tr[2] = global_ns();
                tc_fence_after();
                const uint8_t * st = smem + s * L::STAGE;
                const uint64_t wd = umma_desc_sw128(st), xh = umma_desc_sw128(st + L::X_OFF),
                               xl = umma_desc_sw128(st + L::X_OFF + L::X_BYTES);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    umma2_f16(tmem, wd + (uint64_t) (2 * k), xh + (uint64_t) (2 * k), idesc, (i | k) != 0);
                    if (SPLIT) umma2_f16(tmem, wd + (uint64_t) (2 * k), xl + (uint64_t) (2 * k), idesc, 1u);
                }
                umma2_commit_pair(&empty[s]);
            }
            umma2_commit_pair(tfull);
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        pdl_wait();
        const bool ok = mbar_wait(tfull, 0, abort_flag, a.err, DEV_TIMEOUT_TMEM) && !*abort_flag;
        tc_fence_after();
        if (tr && threadIdx.x == 0) tr[3] = global_ns();
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        if constexpr (EPI == EPI_F32) {
          static_assert(NT / 32 * 4096 * 4 <= STAGES * L::STAGE, "TMA output boxes must fit in the operand ring");
          if (a.tma_out) {
            // each 32-token chunk of this warp's 32 features goes to its own 4 KB box in shared memory
            // (the operand ring is free: every MMA of the pair has completed) as [token][feature],
            // 128-byte rows in the 128-byte swizzle (16-byte chunk j of row t at chunk j ^ (t & 7);
            // a store instruction writes one token's 32 features, one per bank), then one TMA store
            // writes the box; the stores drain while the next chunks are read from TMEM
            const int f0 = n0 + warp * 32;
            const float bl = a.bias && f0 + lane < a.N ? a.bias[f0 + lane] : 0.0f;
            uint8_t * boxes = smem + warp * (NT / 32) * 4096;
            const uint32_t chunk = (uint32_t) (lane >> 2), word = (uint32_t) (lane & 3) * 4;
#pragma unroll
            for (int ci = 0; ci < NT / 32; ++ci) {
                const int c = ci * 32;
                float cur[32];
                tmem_ld32(trow + c, cur);
                uint8_t * box = boxes + ci * 4096;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    *(float *) (box + j * 128 + ((chunk ^ (uint32_t) (j & 7)) << 4) + word) = cur[j] + bl;
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && ok && f0 < a.N && t0 + c < a.rows) tma_store_4d(&tmY, box, f0, t0 + c, b, (int) blockIdx.z);
            }
            if (lane == 0) {
                bulk_commit();
                bulk_wait_read0();
            }
            __syncwarp();
          } else {
            // this warp's 32 features x 32 tokens per chunk go through a padded smem block (the
            // operand ring is free: every MMA of the pair has completed), so that each store
            // instruction writes four tokens' 128-byte runs of 32 consecutive features
            float * tb = (float *) smem + warp * (32 * 33);
            const int f0 = n0 + warp * 32, cq = (lane & 7) * 4;   // the warp's first feature; lane's 4
            float4 bl = make_float4(0.f, 0.f, 0.f, 0.f);
            if (a.bias && f0 + cq < a.N) bl = *(const float4 *) (a.bias + f0 + cq);
            float * ob = (float *) a.out + blockIdx.z * a.part_stride + (long long) b * a.out_bs + f0 + cq;
#pragma unroll 1
            for (int c = 0; c < NT; c += 32) {
                float v[32];
                tmem_ld32(trow + c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = v[j];   // [feature][token]
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int tk = 4 * i + (lane >> 3), t = t0 + c + tk;   // token of this store
                    if (ok && f0 + cq < a.N && t < a.rows)
                        *(float4 *) (ob + (long long) t * a.ldo) =
                            make_float4(tb[cq * 33 + tk] + bl.x, tb[(cq + 1) * 33 + tk] + bl.y,
                                        tb[(cq + 2) * 33 + tk] + bl.z, tb[(cq + 3) * 33 + tk] + bl.w);
                }
                __syncwarp();
            }
          }
        } else {
            // SwiGLU: weight rows come in groups of 16 = [8 w1 | 8 w3]; a warp's 32 rows hold two
            // groups and give 16 consecutive output features (16 warp .. 16 warp + 15 of the CTA's
            // 64, which start at n0 / 2). Per chunk of 32 tokens the warp turns its 32 x 32 block
            // around through padded shared memory (the operand ring is free: every MMA of the pair
            // has completed), so that lane j then holds token c + j: it forms its 16 outputs
            // silu(w1)·w3 and puts them, 32 bytes, into an f16 tile [NT tokens][64 features]. Once
            // every chunk is in, the four warps write the tile as whole 128-byte token rows.
            float * xb = (float *) smem + warp * (32 * 33);          // [row][token], rows padded to 33
            __half * ot = (__half *) (smem + 4 * 32 * 33 * 4);      // [NT][64]
#pragma unroll 1
            for (int c = 0; c < NT; c += 32) {
                float v[32];
                tmem_ld32(trow + c, v);                             // weight row `lane`, tokens c .. c+31
#pragma unroll
                for (int j = 0; j < 32; ++j) xb[lane * 33 + j] = v[j];
                __syncwarp();
                __align__(16) __half h[16];
#pragma unroll
                for (int g = 0; g < 2; ++g)
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        h[8 * g + e] = __float2half_rn(silu_f(xb[(16 * g + e) * 33 + lane]) * xb[(16 * g + 8 + e) * 33 + lane]);
                uint4 * dst = (uint4 *) (ot + (c + lane) * 64 + 16 * warp);
                dst[0] = *(const uint4 *) h;
                dst[1] = *(const uint4 *) (h + 8);
                __syncwarp();
            }
            epi_bar();
            const int f0 = n0 >> 1;                                  // the CTA's first output feature
            const int nf = min(64, (a.N - n0) / 2);                  // output features of weight rows < N
            if (ok && nf > 0) {
                __half * ob = (__half *) a.out + (long long) b * a.out_bs + f0;
                for (int i = threadIdx.x; i < NT * 8; i += 128) {
                    const int tk = i >> 3, ch = i & 7, t = t0 + tk;
                    if (t < a.rows && ch * 8 < nf)
                        *(uint4 *) (ob + (long long) t * a.ldo + ch * 8) = *(const uint4 *) (ot + tk * 64 + ch * 8);
                }
            }
        }
    }
    // every thread of both CTAs: TMEM reads and peer shared-memory traffic are over before the
    // pair releases its TMEM
    tc_fence_before();
    cluster_sync_all();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc2(tmem, TmemCols<NT>::N);
    }
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
    if (*abort_flag && threadIdx.x == 0) {
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}

} // namespace tsn
