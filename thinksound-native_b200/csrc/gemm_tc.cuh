// gemm_tc.cuh — the BF16/F16 tcgen05 GEMM and implicit-GEMM conv1d of the DiT path.
//
// Replaces the reference's im2col + MetalPerformancePrimitives matmul2d pair
// (shaders/ops_conv.metal:265-283 + shaders/gemm_mpp.metal:18-60, driven by Runtime::gemm /
// Runtime::conv, src/net.mm:14-49): Y = X·W^T (+bias), f32 accumulate, for every dense
// projection and every stride-1 conv of the forward.
//
// Layout. Activations are [B][rows][K_in] (B = CFG arms), read through a 3-D TMA view
// {K_in, rows, B} with a box {64, bt, bb}, bt*bb = 128: one 128-row M tile holds bb batches of bt
// consecutive time rows. A conv with `taps` taps and left padding `pad` walks its K loop over
// (tap, 64-channel block) and shifts the box by tap-pad rows; rows outside [0, rows) of each batch
// are zero-filled by TMA, which is exactly the conv's zero padding per batch — no im2col buffer.
// Weights are [N][taps*K_in], conv weights reordered at load from [OC][IC][K] to [OC][K][IC].
//
// Pipeline (one output tile per CTA, 192 threads):
//   warp 4      TMA producer: A box + B box per 64-wide K block into a STAGES-deep smem ring
//   warp 5      TMEM allocation + single-thread tcgen05.mma issue (M=128, N=BN, K=16 x 4)
//   warps 0-3   epilogue: tcgen05.ld rows from TMEM, fused op, global stores
// Split-K (grid.z = S) runs the S K-slices of a tile as one thread-block cluster: each CTA stages
// its f32 partial in its own shared memory, a cluster barrier publishes them, and CTA q reduces the
// q-th 1/S share of the tile by reading all S partials over distributed shared memory, in the fixed
// order 0..S-1 (deterministic), then applies the epilogue to that share. No global scratch.
//
// Split operands (SPLIT=true). The reference keeps activations in f32; one f16 rounding of every
// GEMM input costs ~2.8e-4 relative error per site and ~1.8e-3 on the 21-block flow. A split
// operand stores A = A_hi + A_lo with A_hi = f16(A), A_lo = f16(A - A_hi) (~22-bit mantissa);
// the kernel loads both tiles and issues hi and lo UMMAs into the same f32 TMEM accumulator
// against the same f16 weight tile, so the product equals the f32-activation GEMM to ~2^-22.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace tsn {

enum GemmEpi : int {
    EPI_F32 = 0,       // out f32 = acc (+bias)
    EPI_F16 = 1,       // out f16 = acc (+bias)
    EPI_F16_SILU = 2,  // out f16 = silu(acc + bias)
    EPI_SWIGLU = 3,    // columns in groups of 16 = [8 w1 | 8 w3] -> out f16 = silu(a)*b
    EPI_QKV = 5,       // bias, per-head RMSNorm(q,k), RoPE(q,k), f16 head-major q/k/v
    EPI_F16_SNAKE = 6, // out split f16 = snake(acc + bias) with per-column e^alpha, e^-beta (VAE;
                       // hardware __sinf: a few 1e-6 absolute, far below the f16 rounding of the output)
    EPI_RESID_SNAKE = 7,   // out f32 += acc + bias (residual, in place); out2 split f16 = snake(out)
    EPI_F32_SNAKE2 = 8,    // out f32 = acc + bias; out2 split f16 = snake(out)
    EPI_GEGLU = 9,     // columns in groups of 64 = [32 wi_0 | 32 wi_1] -> out split f16 = gelu_tanh(a)*b (T5 FFN)
    EPI_F16_GELUQ = 10,    // out split f16 = gelu_quick(acc + bias) (CLIP MLP)
};
constexpr bool epi_snake(int epi) { return epi == EPI_F16_SNAKE || epi == EPI_RESID_SNAKE || epi == EPI_F32_SNAKE2; }

struct GemmArgs {
    int rows, B, bt, bb, m_tiles_t, N, k_blocks, ic_blocks, pad, splits, kb_per_split;
    int * err;               // device error word
    const float * bias;      // [N] or null
    void * out;              // EPI_F32/F16*/SWIGLU output
    long long ldo, out_bs;   // row stride and batch stride of out (elements)
    // EPI_QKV
    const float * qn; const float * kn;   // per-head RMSNorm gains [64]
    const float2 * rope;                  // [rows][32] (cos, sin) or null (text stream)
    int H, s_off, S_pad, NH;
    __half * q; __half * k; __half * v;   // [B][NH][S_pad][64]
    long long out_lo;                     // element offset of the lo half of a split f16 output (0: none)
    unsigned long long * trace;           // optional per-CTA phase timestamps (tsn_dit_trace_op), else null
    long long part_stride;                // EPI_F32 split-K without a cluster: K slice z writes out + z*part_stride
    int m_fast;                           // grid.x walks the M tiles and grid.y the N tiles (else the reverse)
    int dil;                              // conv tap dilation: tap k reads row t + k*dil - pad (0 or 1: none)
    const float * snake_a; const float * snake_b;   // snake epilogues: [N] e^alpha, e^-beta
    void * out2; long long ldo2, out2_lo;           // EPI_RESID_SNAKE / EPI_F32_SNAKE2: split f16 [rows][ldo2] (B = 1)
    int a_rows;                                     // rows per activation tile the A views load (0: 128; tile kernel,
                                                    // bt * bb = a_rows): rows past it hold stale data, never stored
    int tma_out;                                    // EPI_F32 without a split-K cluster: store through the output
                                                    // tensor map (4-D {N, rows, B, K slice}, 32 x 32 f32 boxes)
};

// phase stamps per CTA when tracing: entry, setup done, first stage landed (MMA issuer),
// accumulator complete (epilogue), epilogue done, exit, and for split-K clusters: first cluster
// barrier passed, cluster reduction done (0 otherwise)
constexpr int TRACE_SLOTS = 8;

// RoPE rows staged for the qkv epilogue: 64 time rows of 32 (cos, sin) pairs, rows padded to 17
// float4 so that threads reading consecutive rows hit different banks
constexpr int ROPE_ROWS = 64, ROPE_STRIDE4 = 17;

template <int BN, int STAGES, bool SPLIT, int EPI, bool WS = false>
struct GemmSmem {
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int NA = SPLIT ? 2 : 1;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int B_OFF = NA * A_BYTES;
    static constexpr int B2_OFF = B_OFF + B_BYTES;        // WS: the weights' lo half
    static constexpr int STAGE = NA * A_BYTES + (WS ? 2 : 1) * B_BYTES;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int CONST_OFF = BAR_OFF + 256;       // epilogue constants: bias slice, q/k gains
    // bias (256) + q/k gains (64 + 64), or bias + snake e^alpha, e^-beta (256 each)
    static constexpr int CONST_BYTES = (EPI >= 6 && EPI <= 8 ? 3 * 256 : 256 + 64 + 64) * 4;
    static constexpr int ROPE_OFF = CONST_OFF + CONST_BYTES;
    static constexpr int ROPE_BYTES = EPI == 5 ? ROPE_ROWS * ROPE_STRIDE4 * 16 : 0;   // EPI_QKV only
    static constexpr int TOTAL = ROPE_OFF + ROPE_BYTES + 1024;   // + alignment slack
};

// SiLU with the fast exponential and division (relative error ~1e-7, far below the f16 operand
// rounding every downstream GEMM sees)
__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }


// Per-tile epilogue constants staged in shared memory before the accumulator is ready.
struct EpiConst {
    const float * bias;   // bias[n0 .. n0+BN) in shared memory, or null
    const float * qn;     // q RMSNorm gains (64), shared memory; EPI_F16_SNAKE: e^alpha[n0 ..]
    const float * kn;     // k RMSNorm gains (64), shared memory; EPI_F16_SNAKE: e^-beta[n0 ..]
    const float4 * rope;  // RoPE rows t0 .. t0+ROPE_ROWS-1 in shared memory (qkv with RoPE), or null
    int t0;
};

// store 8 f32 values as f16 at o, and their rounding residuals at o + lo (when lo != 0)
__device__ __forceinline__ void store8_split(__half * o, long long lo, const float * v) {
    __align__(16) __half h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(v[e]);
    *(uint4 *) o = *(const uint4 *) h;
    if (lo) {
        __align__(16) __half l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) l[e] = __float2half_rn(v[e] - __half2float(h[e]));
        *(uint4 *) (o + lo) = *(const uint4 *) l;
    }
}

// Columns one epilogue call handles: one 32-column chunk (for SwiGLU two [8 w1 | 8 w3] groups); a
// whole 64-column head for the qkv epilogue (RMSNorm + RoPE need it); a [32 wi_0 | 32 wi_1] group
// for GEGLU.
template <int EPI> struct EpiUnit {
    static constexpr int U = EPI == EPI_QKV || EPI == EPI_GEGLU ? 64 : 32;
};

// geglu_ (shaders/ops_conv.metal:15-24): tanh-approximated GELU of a, argument clamped to +-10
__device__ __forceinline__ float gelu_tanh_f(float v) {
    const float arg = 0.7978845608f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(fminf(fmaxf(arg, -10.0f), 10.0f)));
}
// gelu_quick_ (shaders/ops_conv.metal:25-29)
__device__ __forceinline__ float gelu_quick_f(float v) { return v / (1.0f + expf(-1.702f * v)); }

// TMEM columns for a BN-wide f32 accumulator (allocations are powers of two, at least 32)
template <int BN> struct TmemCols {
    static constexpr int N = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : BN <= 256 ? 256 : 512;
};

// Epilogue for tile row r, columns [u*U, (u+1)*U) of the tile. load32(c, v) returns the 32
// accumulated values of columns [c, c+32) of row r (from TMEM, or summed over the cluster's
// partials). In the TMEM path every lane must call load32 (warp-collective tcgen05.ld), so the
// validity test only guards the stores.
template <int EPI, typename Load>
__device__ __forceinline__ void epi_unit(const GemmArgs & a, const EpiConst & ec, int r, int u, int n0, int t0, int b0, int z,
                                         bool ok, Load && load32) {
    constexpr int U = EpiUnit<EPI>::U;
    const int b = b0 + r / a.bt, t = t0 + r % a.bt;
    const int c0 = u * U;
    // a tile may overhang N (tile widths that do not divide N): whole units beyond N are skipped
    const bool valid = ok && t < a.rows && b < a.B && n0 + c0 < a.N;
    if constexpr (EPI == EPI_GEGLU) {
        float va[32], vb[32];
        load32(c0, va);
        load32(c0 + 32, vb);
        if (valid) {
            __half * o = (__half *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + (n0 + c0) / 2;
#pragma unroll
            for (int e = 0; e < 32; ++e) va[e] = gelu_tanh_f(va[e]) * vb[e];
#pragma unroll
            for (int q = 0; q < 32; q += 8) store8_split(o + q, a.out_lo, va + q);
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        // 32 columns = two [8 w1 | 8 w3] groups -> 16 consecutive output features from (n0 + c0) / 2;
        // a tile that overhangs N may end inside the unit: only whole groups below N are stored
        float v[32];
        load32(c0, v);
        if (valid) {
            __half * o = (__half *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + (n0 + c0) / 2;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (n0 + c0 + 16 * g >= a.N) break;
                __align__(16) __half h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(silu_f(v[16 * g + e]) * v[16 * g + 8 + e]);
                *(uint4 *) (o + 8 * g) = *(const uint4 *) h;
            }
        }
    } else if constexpr (EPI == EPI_QKV) {
        float v[64];
        load32(c0, v);
        load32(c0 + 32, v + 32);
        if (!valid) return;
        const int n = n0 + c0, which = n / a.H, head = (n % a.H) >> 6;
        if (ec.bias) {
#pragma unroll
            for (int e = 0; e < 64; ++e) v[e] += ec.bias[c0 + e];
        }
        if (which < 2) {
            if (a.qn) {   // per-head RMSNorm (the DiT; the text encoders have none)
                const float * g = which == 0 ? ec.qn : ec.kn;
                float ss = 0.0f;
#pragma unroll
                for (int e = 0; e < 64; ++e) ss += v[e] * v[e];
                const float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
                for (int e = 0; e < 64; ++e) v[e] = v[e] * inv * g[e];
            }
            if (a.rope) {
                // this row's (cos, sin) pairs, two per float4: staged rows when the tile's time rows
                // fit the staged table, else straight from the global table
                const float4 * cs = t - ec.t0 < ROPE_ROWS ? ec.rope + (t - ec.t0) * ROPE_STRIDE4
                                                          : (const float4 *) (a.rope + (size_t) t * 32);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 w = cs[j];
                    float x0 = v[4 * j], x1 = v[4 * j + 1];
                    v[4 * j] = x0 * w.x - x1 * w.y;
                    v[4 * j + 1] = x0 * w.y + x1 * w.x;
                    x0 = v[4 * j + 2]; x1 = v[4 * j + 3];
                    v[4 * j + 2] = x0 * w.z - x1 * w.w;
                    v[4 * j + 3] = x0 * w.w + x1 * w.z;
                }
            }
        }
        __half * dst = which == 0 ? a.q : which == 1 ? a.k : a.v;
        dst += (((size_t) b * a.NH + head) * a.S_pad + a.s_off + t) * 64;
#pragma unroll
        for (int q = 0; q < 64; q += 8) store8_split(dst + q, a.out_lo, v + q);
    } else {
        float v[32];
        load32(c0, v);
        if (!valid) return;
        const int n = n0 + c0;
        if (ec.bias) {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] += ec.bias[c0 + e];
        }
        if constexpr (EPI == EPI_F32) {
            float * o = (float *) a.out + z * a.part_stride + (long long) b * a.out_bs + (long long) t * a.ldo + n;
#pragma unroll
            for (int q = 0; q < 32; q += 4) *(float4 *) (o + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
        } else if constexpr (EPI == EPI_F16 || EPI == EPI_F16_SILU || EPI == EPI_F16_SNAKE || EPI == EPI_F16_GELUQ) {
            __half * o = (__half *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + n;
            if (EPI == EPI_F16_SILU) {
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = silu_f(v[e]);
            }
            if (EPI == EPI_F16_GELUQ) {
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = gelu_quick_f(v[e]);
            }
            if (EPI == EPI_F16_SNAKE) {   // snake_ (shaders/ops_conv.metal:204-213) on acc + bias
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float sv = __sinf(v[e] * ec.qn[c0 + e]);
                    v[e] = v[e] + sv * sv * ec.kn[c0 + e];
                }
            }
#pragma unroll
            for (int q = 0; q < 32; q += 8) store8_split(o + q, a.out_lo, v + q);
        } else if constexpr (EPI == EPI_RESID_SNAKE || EPI == EPI_F32_SNAKE2) {
            float * xo = (float *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + n;
            if (EPI == EPI_RESID_SNAKE) {   // the residual add of src/vae.cpp:75
#pragma unroll
                for (int q = 0; q < 32; q += 4) {
                    const float4 r = *(const float4 *) (xo + q);
                    v[q] += r.x; v[q + 1] += r.y; v[q + 2] += r.z; v[q + 3] += r.w;
                }
            }
#pragma unroll
            for (int q = 0; q < 32; q += 4) *(float4 *) (xo + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
#pragma unroll
            for (int e = 0; e < 32; ++e) {   // snake_ (shaders/ops_conv.metal:204-213) of the new value
                const float sv = __sinf(v[e] * ec.qn[c0 + e]);
                v[e] = v[e] + sv * sv * ec.kn[c0 + e];
            }
            __half * ho = (__half *) a.out2 + (long long) t * a.ldo2 + n;
#pragma unroll
            for (int q = 0; q < 32; q += 8) store8_split(ho + q, a.out2_lo, v + q);
        }
    }
}

// One output tile (M tile mi, N tile ni, K slice z) computed by the whole CTA; `cta` indexes the
// trace rows. The tensor maps are kernel parameters (grid constants).
// WS: the weights are split too (W = W_hi + W_lo, tmB2 the lo half; the VAE's f32 weights): each
// K step issues A_hi·W_hi + A_lo·W_hi + A_hi·W_lo.
template <int BN, int EPI, int STAGES, bool SPLIT, bool WS = false>
__device__ __forceinline__ void gemm_tile(const CUtensorMap * tmA, const CUtensorMap * tmA2, const CUtensorMap * tmB,
                                          const GemmArgs & a, const int ab_bf16, const int mi, const int ni, const int z,
                                          const int cta, const CUtensorMap * tmB2 = nullptr,
                                          const CUtensorMap * tmO = nullptr) {
    using L = GemmSmem<BN, STAGES, SPLIT, EPI, WS>;
    static_assert(!WS || SPLIT, "split weights go with a split A operand");
    static_assert(BN % 32 == 0 || (BN % 16 == 0 && EPI == EPI_SWIGLU), "tile widths not a multiple of 32: SwiGLU only");
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + L::BAR_OFF);
    uint64_t * empty = full + STAGES;
    uint64_t * tfull = empty + STAGES;
    uint32_t * tslot = (uint32_t *) (tfull + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    float * cbias = (float *) (smem + L::CONST_OFF);      // BN floats
    float * cqn = cbias + 256, * ckn = cqn + (epi_snake(EPI) ? 256 : 64);   // q/k gains, or snake e^a, e^-b
    float4 * crope = (float4 *) (smem + L::ROPE_OFF);      // qkv: ROPE_ROWS x ROPE_STRIDE4

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long * tr = a.trace ? a.trace + (size_t) cta * TRACE_SLOTS : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    const int mt = mi % a.m_tiles_t, mb = mi / a.m_tiles_t;
    const int t0 = mt * a.bt, b0 = mb * a.bb, n0 = ni * BN;
    const int kb_begin = z * a.kb_per_split;
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
        tma_prefetch(tmA);
        if (SPLIT) tma_prefetch(tmA2);
        tma_prefetch(tmB);
    }
    if (warp == 5) tmem_alloc(tslot, TmemCols<BN>::N);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tr && threadIdx.x == 0) tr[1] = global_ns();

    if (warp == 4) {
        if (lane == 0) {
            // bytes per stage: activation tiles of a_rows rows leave the rest of the 128-row tile
            // unwritten (rows the epilogue never stores)
            const uint32_t stage_tx = L::STAGE - (a.a_rows ? (uint32_t) (128 - a.a_rows) * 128u * (SPLIT ? 2u : 1u) : 0u);
            // weights do not depend on the upstream kernel: start the first stages' weight loads,
            // then wait for upstream outputs before loading activations
            const int pre = nk < STAGES ? nk : STAGES;
            for (int i = 0; i < pre; ++i) {
                uint8_t * sa = smem + i * L::STAGE;
                mbar_expect_tx(&full[i], stage_tx);
                tma_load_2d(sa + L::B_OFF, tmB, &full[i], (kb_begin + i) * 64, n0);
                if (WS) tma_load_2d(sa + L::B2_OFF, tmB2, &full[i], (kb_begin + i) * 64, n0);
            }
            pdl_wait();
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY))
                    break;
                const int kb = kb_begin + i;
                const int tap = kb / a.ic_blocks, ic0 = (kb % a.ic_blocks) * 64;
                uint8_t * sa = smem + s * L::STAGE;
                if (i >= pre) {
                    mbar_expect_tx(&full[s], stage_tx);
                    tma_load_2d(sa + L::B_OFF, tmB, &full[s], kb * 64, n0);
                    if (WS) tma_load_2d(sa + L::B2_OFF, tmB2, &full[s], kb * 64, n0);
                }
                const int row = t0 + tap * (a.dil > 1 ? a.dil : 1) - a.pad;
                tma_load_3d(sa, tmA, &full[s], ic0, row, b0);
                if (SPLIT) tma_load_3d(sa + L::A_BYTES, tmA2, &full[s], ic0, row, b0);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(BN, ab_bf16);
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&full[s], (i / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL)) break;
                if (tr && i == 0) tr[2] = global_ns();
                tc_fence_after();
                const uint8_t * sa = smem + s * L::STAGE;
                const uint64_t ad = umma_desc_sw128(sa), bd = umma_desc_sw128(sa + L::B_OFF);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    umma_f16(tmem, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (i | k) != 0);
                    if (SPLIT) {
                        const uint64_t al = umma_desc_sw128(sa + L::A_BYTES);
                        umma_f16(tmem, al + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, 1u);
                    }
                    if (WS) {
                        const uint64_t b2 = umma_desc_sw128(sa + L::B2_OFF);
                        umma_f16(tmem, ad + (uint64_t) (2 * k), b2 + (uint64_t) (2 * k), idesc, 1u);
                    }
                }
                umma_commit(&empty[s]);
            }
            umma_commit(tfull);
        }
    } else {
        // ------------------------------------------------------------------ epilogue, part 1
        pdl_wait();
        {   // stage the tile's constants while the mainloop runs; warm L1 with this row's RoPE entries
            const int tid = threadIdx.x;
            if (a.bias)
                for (int i = tid; i < BN && n0 + i < a.N; i += 128) cbias[i] = a.bias[n0 + i];
            if (EPI == EPI_QKV && a.qn && tid < 64) { cqn[tid] = a.qn[tid]; ckn[tid] = a.kn[tid]; }
            if (epi_snake(EPI))
                for (int i = tid; i < BN && n0 + i < a.N; i += 128) { cqn[i] = a.snake_a[n0 + i]; ckn[i] = a.snake_b[n0 + i]; }
            if (EPI == EPI_QKV && a.rope)
                for (int i = tid; i < ROPE_ROWS * 16; i += 128) {
                    const int rr = i >> 4, c4 = i & 15;
                    if (t0 + rr < a.rows) crope[rr * ROPE_STRIDE4 + c4] = __ldg((const float4 *) (a.rope + (size_t) (t0 + rr) * 32) + c4);
                }
            epi_bar();
        }
        const EpiConst ec{a.bias ? cbias : nullptr, cqn, ckn, crope, t0};
        const bool ok = mbar_wait(tfull, 0, abort_flag, a.err, DEV_TIMEOUT_TMEM) && !*abort_flag;
        tc_fence_after();
        const int r = warp * 32 + lane;
        if (tr && r == 0) tr[3] = global_ns();
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        bool tma_done = false;
        if constexpr (EPI == EPI_F32) {
            if (a.splits == 1 && a.tma_out && tmO) {
                static_assert(BN / 32 * 4096 * 4 <= STAGES * L::STAGE, "TMA output boxes must fit in the operand ring");
                // each 32-column unit of the warp's 32 rows goes to its own 4 KB box in shared memory
                // (the operand ring is free: every TMA load was consumed and every MMA has completed),
                // a thread's row as 128 bytes in the 128-byte swizzle (16-byte chunk j at j ^ (row & 7)),
                // then one TMA store writes the box and drains while the next unit is read from TMEM.
                // The warp's rows are consecutive times of one arm: the host binds the view only when
                // bt is a multiple of 32.
                const int rw = warp * 32, bw = b0 + rw / a.bt, tw = t0 + rw % a.bt;
                uint8_t * boxes = smem + warp * (BN / 32) * 4096;
#pragma unroll
                for (int u = 0; u < BN / 32; ++u) {
                    float v[32];
                    tmem_ld32(trow + u * 32, v);
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] += ec.bias ? ec.bias[u * 32 + e] : 0.0f;
                    uint8_t * row = boxes + u * 4096 + lane * 128;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *(float4 *) (row + ((q ^ (lane & 7)) << 4)) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && ok && tw < a.rows && bw < a.B && n0 + u * 32 < a.N)
                        tma_store_4d(tmO, boxes + u * 4096, n0 + u * 32, tw, bw, z);
                }
                if (lane == 0) {
                    bulk_commit();
                    bulk_wait_read0();
                }
                __syncwarp();
                tma_done = true;
            }
        }
        if (tma_done) {
        } else if (a.splits == 1) {
            auto load_tmem = [&](int c, float * v) { tmem_ld32(trow + c, v); };
#pragma unroll 1
            for (int u = 0; u < BN / EpiUnit<EPI>::U; ++u) epi_unit<EPI>(a, ec, r, u, n0, t0, b0, z, ok, load_tmem);
            if constexpr (EPI == EPI_SWIGLU && BN % 32 == 16) {
                // the last [8 w1 | 8 w3] group of a tile width that is an odd multiple of 16
                constexpr int c0 = BN - 16;
                float v[16];
                tmem_ld16(trow + c0, v);
                const int b = b0 + r / a.bt, t = t0 + r % a.bt;
                if (ok && t < a.rows && b < a.B && n0 + c0 < a.N) {
                    __align__(16) __half h[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(silu_f(v[e]) * v[8 + e]);
                    *(uint4 *) ((__half *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + (n0 + c0) / 2) =
                        *(const uint4 *) h;
                }
            }
        } else {
            // stage this CTA's partial in its own shared memory as [BN/4][128] float4 (the stage ring
            // is free: every TMA load was consumed and every MMA has completed)
            float4 * part = (float4 *) smem;
            for (int c = 0; c < BN; c += 32) {
                float v[32];
                tmem_ld32(trow + c, v);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    part[(c / 4 + j) * 128 + r] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tr && threadIdx.x == 0) tr[4] = global_ns();
    if (a.splits > 1) {
        // ---------------------------------------------------------- epilogue, part 2 (cluster)
        cluster_sync_all();
        if (tr && threadIdx.x == 0) tr[6] = global_ns();
        if (warp < 4 && !*abort_flag) {
            const EpiConst ec2{a.bias ? cbias : nullptr, cqn, ckn, crope, t0};
            const int S = a.splits;
            const uint32_t q = cluster_rank();
            const uint32_t local = smem_u32(smem);
            uint32_t peer[8];
#pragma unroll
            for (int sp = 0; sp < 8; ++sp) peer[sp] = sp < S ? dsmem_map(local, (uint32_t) sp) : 0u;
            constexpr int U = EpiUnit<EPI>::U;
            const int items = (BN / U) * 128;
            const int lo = (int) ((long long) items * q / S), hi = (int) ((long long) items * (q + 1) / S);
            for (int it = lo + (int) threadIdx.x; it < hi; it += 128) {
                const int rr = it & 127, u = it >> 7;
                auto load_dsmem = [&](int c, float * v) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t off = (uint32_t) (((c / 4 + j) * 128 + rr) * 16);
                        float4 p[8];
#pragma unroll
                        for (int sp = 0; sp < 8; ++sp)
                            if (sp < S) p[sp] = dsmem_ld4(peer[sp] + off);
                        float4 acc = p[0];
#pragma unroll
                        for (int sp = 1; sp < 8; ++sp)
                            if (sp < S) { acc.x += p[sp].x; acc.y += p[sp].y; acc.z += p[sp].z; acc.w += p[sp].w; }
                        v[4 * j] = acc.x; v[4 * j + 1] = acc.y; v[4 * j + 2] = acc.z; v[4 * j + 3] = acc.w;
                    }
                };
                epi_unit<EPI>(a, ec2, rr, u, n0, t0, b0, z, true, load_dsmem);
            }
        }
        if (tr && threadIdx.x == 0) tr[7] = global_ns();
        cluster_sync_all();   // peers have finished reading this CTA's shared memory
    }
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TmemCols<BN>::N);
    }
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
    if (*abort_flag && threadIdx.x == 0) {
        // let TMA copies that were issued but never consumed land before the CTA's smem is reused
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}

template <int BN, int EPI, int STAGES, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
               const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmO,
               const __grid_constant__ GemmArgs a, const int ab_bf16) {
    // with m_fast the CTAs that share a weight tile are launched next to each other, so a weight
    // matrix larger than L2 is streamed from HBM once rather than once per M tile
    const int mi = a.m_fast ? blockIdx.x : blockIdx.y, ni = a.m_fast ? blockIdx.y : blockIdx.x;
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    gemm_tile<BN, EPI, STAGES, SPLIT>(&tmA, &tmA2, &tmB, a, ab_bf16, mi, ni, (int) blockIdx.z, cta, nullptr, &tmO);
}

// Split activations and split weights (the VAE decoder's f32 weights as W_hi + W_lo f16): grid
// as gemm_tc_kernel, tmB2 the weights' lo half.
template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
               const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB2,
               const __grid_constant__ GemmArgs a) {
    const int mi = a.m_fast ? blockIdx.x : blockIdx.y, ni = a.m_fast ? blockIdx.y : blockIdx.x;
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    gemm_tile<BN, EPI, STAGES, true, true>(&tmA, &tmA2, &tmB, a, 0, mi, ni, (int) blockIdx.z, cta, &tmB2);
}

// ------------------------------------------------------------------------------------------
// Grouped launch: up to MAX_GROUP independent GEMMs with one tile shape and epilogue kind (the
// latent, clip and text streams of a joint block run the same projection with their own weights,
// rows and outputs). grid.x is the concatenation of the problems' CTAs, problem q owning
// [cta_end[q-1], cta_end[q]); inside a problem consecutive CTAs are the K slices of one tile and
// tiles go M tile fastest. The slices either form a cluster along x (in-cluster split-K reduction:
// every problem then has `slices` equal to the cluster size and starts on a cluster boundary) or
// are independent partial tiles (EPI_F32 with part_stride, any slice count per problem). One
// launch fills the SMs with all three streams' tiles where three launches would contend for them.
constexpr int MAX_GROUP = 3;
struct GroupMaps {
    CUtensorMap a[MAX_GROUP], a2[MAX_GROUP], b[MAX_GROUP];
    CUtensorMap o[MAX_GROUP];    // f32 output views of members with GemmArgs::tma_out
};
struct GroupArgs {
    GemmArgs p[MAX_GROUP];
    int n;                     // problems in the group
    int cta_end[MAX_GROUP];    // exclusive end of each problem's CTA range in grid.x
    int slices[MAX_GROUP];     // K slices per tile
    int m_tiles[MAX_GROUP];    // M tiles per problem
    // gemm_tc_group_p only: problem persist_q runs on persist_ctas persistent CTAs, each taking an
    // equal run of its persist_tiles tiles (persist_bn wide, M tile fastest)
    int persist_q = -1, persist_ctas = 0, persist_tiles = 0;
};

template <int BN, int EPI, int STAGES, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
gemm_tc_group(const __grid_constant__ GroupMaps maps, const __grid_constant__ GroupArgs g, const int ab_bf16) {
    const int x = (int) blockIdx.x;
    int q = 0;
    while (q + 1 < g.n && x >= g.cta_end[q]) ++q;
    const int l = x - (q ? g.cta_end[q - 1] : 0);
    const int S = g.slices[q], z = l % S, tile = l / S;
    const int mi = tile % g.m_tiles[q], ni = tile / g.m_tiles[q];
    gemm_tile<BN, EPI, STAGES, SPLIT>(&maps.a[q], &maps.a2[q], &maps.b[q], g.p[q], ab_bf16, mi, ni, z, x, nullptr, &maps.o[q]);
}

// ------------------------------------------------------------------------------------------
// A run of output tiles [lo, hi) of one problem on one CTA (the shallow problem of a grouped
// launch whose deep tiles leave some SMs free): tile t is (M tile t % m_tiles, N tile
// t / m_tiles), PBN columns wide, no K slices. The operand ring runs on across tile boundaries and
// two TMEM accumulators (columns 0 and 256) let the epilogue of tile i overlap the mainloop of
// tile i + 1. Same warp roles as gemm_tile; epilogue through epi_unit (plus a 16-column tail for
// SwiGLU widths that are odd multiples of 16). Shared memory: PSTAGES stages of split A + PBN
// weight rows, then the barriers.
template <int PBN, int PSTAGES, bool SPLIT>
struct PersistListSmem {
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int NA = SPLIT ? 2 : 1;
    static constexpr int B_OFF = NA * A_BYTES;
    static constexpr int STAGE = NA * A_BYTES + PBN * 128;
    static constexpr int BAR_OFF = PSTAGES * STAGE;
    static constexpr int TOTAL = BAR_OFF + 256 + 1024;   // barriers, TMEM slot, abort flag + alignment slack
    static_assert(STAGE % 1024 == 0, "stages must stay 1024-byte aligned");
};

template <int PBN, int EPI, int PSTAGES, bool SPLIT>
__device__ __forceinline__ void gemm_tile_list(const CUtensorMap * tmA, const CUtensorMap * tmA2, const CUtensorMap * tmB,
                                               const GemmArgs & a, const int ab_bf16, const int m_tiles, const int lo,
                                               const int hi) {
    using L = PersistListSmem<PBN, PSTAGES, SPLIT>;
    constexpr int ACC = 256;
    static_assert(PBN <= ACC && PBN % 16 == 0, "tile width");
    static_assert(PBN % 32 == 0 || EPI == EPI_SWIGLU, "odd multiples of 16: SwiGLU only");
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + L::BAR_OFF);
    uint64_t * empty = full + PSTAGES;
    uint64_t * afull = empty + PSTAGES;      // [2] accumulator ready for the epilogue
    uint64_t * aempty = afull + 2;           // [2] accumulator drained (one arrival per epilogue warp)
    uint32_t * tslot = (uint32_t *) (aempty + 2);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = a.k_blocks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&afull[b], 1); mbar_init(&aempty[b], 4); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 0) pdl_trigger();
    if (warp == 4 && lane == 0) {
        tma_prefetch(tmA);
        if (SPLIT) tma_prefetch(tmA2);
        tma_prefetch(tmB);
    }
    if (warp == 5) tmem_alloc(tslot, 2 * ACC);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    auto coords = [&](int tile, int & t0, int & b0, int & n0) {
        const int mi = tile % m_tiles, ni = tile / m_tiles;
        t0 = (mi % a.m_tiles_t) * a.bt;
        b0 = (mi / a.m_tiles_t) * a.bb;
        n0 = ni * PBN;
    };
    if (warp == 4) {
        if (lane == 0) {
            const uint32_t stage_tx = L::STAGE - (a.a_rows ? (uint32_t) (128 - a.a_rows) * 128u * (SPLIT ? 2u : 1u) : 0u);
            int t0, b0, n0;
            coords(lo, t0, b0, n0);
            // the first tile's weight stages do not depend on the upstream kernel
            const int pre = lo < hi ? (nk < PSTAGES ? nk : PSTAGES) : 0;
            for (int i = 0; i < pre; ++i) {
                mbar_expect_tx(&full[i], stage_tx);
                tma_load_2d(smem + i * L::STAGE + L::B_OFF, tmB, &full[i], i * 64, n0);
            }
            pdl_wait();
            int g = 0;   // k blocks issued so far (ring position)
            bool stop = false;
            for (int tile = lo; tile < hi && !stop; ++tile) {
                coords(tile, t0, b0, n0);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % PSTAGES;
                    if (g >= PSTAGES && !mbar_wait(&empty[s], ((g / PSTAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
                    uint8_t * sa = smem + s * L::STAGE;
                    if (g >= pre) {
                        mbar_expect_tx(&full[s], stage_tx);
                        tma_load_2d(sa + L::B_OFF, tmB, &full[s], kb * 64, n0);
                    }
                    const int tap = kb / a.ic_blocks, ic0 = (kb % a.ic_blocks) * 64;
                    const int row = t0 + tap * (a.dil > 1 ? a.dil : 1) - a.pad;
                    tma_load_3d(sa, tmA, &full[s], ic0, row, b0);
                    if (SPLIT) tma_load_3d(sa + L::A_BYTES, tmA2, &full[s], ic0, row, b0);
                }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(PBN, ab_bf16);
            int g = 0, i = 0;
            bool stop = false;
            for (int tile = lo; tile < hi && !stop; ++tile, ++i) {
                const int buf = i & 1;
                if (i >= 2 && !mbar_wait(&aempty[buf], ((i >> 1) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t) (buf * ACC);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % PSTAGES;
                    if (!mbar_wait(&full[s], (g / PSTAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL)) { stop = true; break; }
                    tc_fence_after();
                    const uint8_t * sa = smem + s * L::STAGE;
                    const uint64_t ad = umma_desc_sw128(sa), bd = umma_desc_sw128(sa + L::B_OFF);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        umma_f16(d, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (kb | k) != 0);
                        if (SPLIT) {
                            const uint64_t al = umma_desc_sw128(sa + L::A_BYTES);
                            umma_f16(d, al + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, 1u);
                        }
                    }
                    umma_commit(&empty[s]);
                }
                if (!stop) umma_commit(&afull[buf]);
            }
        }
    } else {
        pdl_wait();
        const int r = warp * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        int i = 0;
        for (int tile = lo; tile < hi; ++tile, ++i) {
            const int buf = i & 1;
            const bool ok = mbar_wait(&afull[buf], (i >> 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM) && !*abort_flag;
            if (!ok) break;
            tc_fence_after();
            int t0, b0, n0;
            coords(tile, t0, b0, n0);
            const uint32_t tb = trow + (uint32_t) (buf * ACC);
            auto load_tmem = [&](int c, float * v) { tmem_ld32(tb + (uint32_t) c, v); };
            const EpiConst ec{a.bias ? a.bias + n0 : nullptr, nullptr, nullptr, nullptr, t0};
#pragma unroll 1
            for (int u = 0; u < PBN / EpiUnit<EPI>::U; ++u) epi_unit<EPI>(a, ec, r, u, n0, t0, b0, 0, true, load_tmem);
            if constexpr (EPI == EPI_SWIGLU && PBN % 32 == 16) {
                constexpr int c0 = PBN - 16;
                float v[16];
                tmem_ld16(tb + (uint32_t) c0, v);
                const int b = b0 + r / a.bt, t = t0 + r % a.bt;
                if (t < a.rows && b < a.B && n0 + c0 < a.N) {
                    __align__(16) __half h[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(silu_f(v[e]) * v[8 + e]);
                    *(uint4 *) ((__half *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + (n0 + c0) / 2) =
                        *(const uint4 *) h;
                }
            }
            // this warp is done reading accumulator `buf`
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&aempty[buf])) : "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ACC);
    }
    if (*abort_flag && threadIdx.x == 0) {
        // let TMA copies that were issued but never consumed land before the CTA's smem is reused
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}

// A grouped launch whose problem g.persist_q runs as a tile list on g.persist_ctas persistent CTAs
// (gemm_tile_list, PBN wide); the other problems' CTAs are ordinary tiles (gemm_tile, BN wide).
// Dynamic shared memory: the larger of the two layouts.
template <int BN, int PBN, int EPI, int STAGES, int PSTAGES, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
gemm_tc_group_p(const __grid_constant__ GroupMaps maps, const __grid_constant__ GroupArgs g, const int ab_bf16) {
    const int x = (int) blockIdx.x;
    int q = 0;
    while (q + 1 < g.n && x >= g.cta_end[q]) ++q;
    const int l = x - (q ? g.cta_end[q - 1] : 0);
    if (q == g.persist_q) {
        const int P = g.persist_ctas, T = g.persist_tiles;
        const int lo = (int) ((long long) T * l / P), hi = (int) ((long long) T * (l + 1) / P);
        gemm_tile_list<PBN, EPI, PSTAGES, SPLIT>(&maps.a[q], &maps.a2[q], &maps.b[q], g.p[q], ab_bf16, g.m_tiles[q], lo, hi);
        return;
    }
    const int S = g.slices[q], z = l % S, tile = l / S;
    const int mi = tile % g.m_tiles[q], ni = tile / g.m_tiles[q];
    gemm_tile<BN, EPI, STAGES, SPLIT>(&maps.a[q], &maps.a2[q], &maps.b[q], g.p[q], ab_bf16, mi, ni, z, x, nullptr, &maps.o[q]);
}

// ------------------------------------------------------------------------------------------
// Persistent variant for GEMMs with many more tiles than SMs (the step's latent modulation GEMM,
// 376 x 131072 x 1024: 2049 tiles). One CTA per SM walks the tiles blockIdx.x, +gridDim.x, ...
// (M tiles fastest, so the CTAs sharing a weight tile run together); the operand ring runs on
// across tile boundaries, and two TMEM accumulators let the epilogue of tile i (f32 + bias) overlap
// the mainloop of tile i+1. Split f16 A operand, f32 output.
template <int BN, int STAGES>
struct PersistSmem {
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_OFF = 2 * A_BYTES;
    static constexpr int STAGE = 2 * A_BYTES + BN * 128;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int XPOSE_OFF = BAR_OFF + 256;      // per epilogue warp: 32 rows x 33 floats (padded)
    static constexpr int TOTAL = XPOSE_OFF + 4 * 32 * 33 * 4 + 1024;   // + alignment slack
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_tc_persistent(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs a, const int ab_bf16) {
    using L = PersistSmem<BN, STAGES>;
    constexpr int ACC = 256;   // TMEM column offset of the second accumulator
    static_assert(BN <= ACC, "two accumulators must fit TMEM");
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + L::BAR_OFF);
    uint64_t * empty = full + STAGES;
    uint64_t * afull = empty + STAGES;       // [2] accumulator ready for the epilogue
    uint64_t * aempty = afull + 2;           // [2] accumulator drained (4 arrivals: one per epilogue warp)
    uint32_t * tslot = (uint32_t *) (aempty + 2);
    volatile int * abort_flag = (volatile int *) (tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long * tr = a.trace ? a.trace + (size_t) blockIdx.x * TRACE_SLOTS : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    const int MT = a.m_tiles_t * ((a.B + a.bb - 1) / a.bb), NT = (a.N + BN - 1) / BN;
    const int tiles = MT * NT, nk = a.k_blocks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&afull[b], 1); mbar_init(&aempty[b], 4); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 0) pdl_trigger();
    if (warp == 4 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmA2); tma_prefetch(&tmB); }
    if (warp == 5) tmem_alloc(tslot, 2 * ACC);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    auto tile_coords = [&](int tile, int & t0, int & b0, int & n0) {
        const int mi = tile % MT, ni = tile / MT;
        t0 = (mi % a.m_tiles_t) * a.bt;
        b0 = (mi / a.m_tiles_t) * a.bb;
        n0 = ni * BN;
    };

    if (warp == 4) {
        if (lane == 0) {
            // the first tile's weight stages do not depend on the upstream kernel
            int t0, b0, n0;
            tile_coords(blockIdx.x, t0, b0, n0);
            const int pre = blockIdx.x < tiles ? (nk < STAGES ? nk : STAGES) : 0;
            for (int i = 0; i < pre; ++i) {
                mbar_expect_tx(&full[i], L::STAGE);
                tma_load_2d(smem + i * L::STAGE + L::B_OFF, &tmB, &full[i], i * 64, n0);
            }
            pdl_wait();
            int g = 0;   // k blocks issued by this CTA so far (ring position)
            bool stop = false;
            for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
                tile_coords(tile, t0, b0, n0);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (g >= STAGES && !mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
                    uint8_t * sa = smem + s * L::STAGE;
                    if (g >= pre) {
                        mbar_expect_tx(&full[s], L::STAGE);
                        tma_load_2d(sa + L::B_OFF, &tmB, &full[s], kb * 64, n0);
                    }
                    tma_load_3d(sa, &tmA, &full[s], kb * 64, t0, b0);
                    tma_load_3d(sa + L::A_BYTES, &tmA2, &full[s], kb * 64, t0, b0);
                }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(BN, ab_bf16);
            int g = 0, i = 0;
            bool stop = false;
            for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x, ++i) {
                const int buf = i & 1;
                if (i >= 2 && !mbar_wait(&aempty[buf], ((i >> 1) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t) (buf * ACC);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(&full[s], (g / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL)) { stop = true; break; }
                    if (tr && g == 0) tr[2] = global_ns();
                    tc_fence_after();
                    const uint8_t * sa = smem + s * L::STAGE;
                    const uint64_t ad = umma_desc_sw128(sa), al = umma_desc_sw128(sa + L::A_BYTES),
                                   bd = umma_desc_sw128(sa + L::B_OFF);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        umma_f16(d, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (kb | k) != 0);
                        umma_f16(d, al + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, 1u);
                    }
                    umma_commit(&empty[s]);
                }
                if (!stop) umma_commit(&afull[buf]);
            }
        }
    } else {
        pdl_wait();
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        int i = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
            const int buf = i & 1;
            if (!mbar_wait(&afull[buf], (i >> 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
            tc_fence_after();
            int t0, b0, n0;
            tile_coords(tile, t0, b0, n0);
            // The output rows are far apart (the modulation GEMM's rows are 512 KB long): each
            // 32 x 32 chunk goes through this warp's padded smem block so that every store
            // instruction writes four whole 128-byte row segments.
            float * tb = (float *) (smem + L::XPOSE_OFF) + warp * (32 * 33);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                float v[32];
                tmem_ld32(trow + (uint32_t) (buf * ACC + c), v);
                const int n = n0 + c;
                if (n >= a.N) continue;                      // the same for the whole warp
#pragma unroll
                for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = v[j];
                __syncwarp();
                // store i: rows 4i .. 4i+3 of the block, 8 lanes per row, one float4 each
                const int cq = (lane & 7) * 4, col = n + cq;
                const bool col_ok = col < a.N;
                float4 bl = make_float4(0.f, 0.f, 0.f, 0.f);
                if (a.bias && col_ok) bl = __ldg((const float4 *) (a.bias + col));
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int rr = 4 * i + (lane >> 3), row = warp * 32 + rr, b = b0 + row / a.bt, t = t0 + row % a.bt;
                    const float * src = tb + rr * 33 + cq;
                    if (col_ok && t < a.rows && b < a.B)
                        *(float4 *) ((float *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + col) =
                            make_float4(src[0] + bl.x, src[1] + bl.y, src[2] + bl.z, src[3] + bl.w);
                }
                __syncwarp();
            }
            // this warp is done reading accumulator `buf`
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&aempty[buf])) : "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ACC);
    }
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
    if (*abort_flag && threadIdx.x == 0) {
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}


// ------------------------------------------------------------------------------------------
// Persistent split-activation x split-weight GEMM / implicit conv (the VAE decoder's convs, up to
// 3008 tiles per launch): one CTA per SM walks the tiles blockIdx.x, +gridDim.x, ... (M tiles
// fastest); the operand ring runs on across tiles and two TMEM accumulators let the epilogue of
// tile i (any epi_unit epilogue, constants read from global memory) overlap the mainloop of tile
// i + 1. Conv taps and dilation as in gemm_tile; no split-K (a.splits must be 1).
template <int BN, int STAGES, int EPI>
struct PersistWsSmem {
    using S = GemmSmem<BN, STAGES, true, EPI, true>;
    static constexpr int STAGE = S::STAGE, A_BYTES = S::A_BYTES, B_OFF = S::B_OFF, B2_OFF = S::B2_OFF;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int XPOSE_OFF = BAR_OFF + 256;      // per epilogue warp: 32 x 33 floats (padded)
    static constexpr int TOTAL = XPOSE_OFF + 4 * 32 * 33 * 4 + 1024;   // + alignment slack
};

template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_ws_persistent(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB2,
                   const __grid_constant__ GemmArgs a) {
    using L = PersistWsSmem<BN, STAGES, EPI>;
    constexpr uint32_t ACC = BN <= 128 ? 128 : 256;   // TMEM column offset of the second accumulator
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t * full = (uint64_t *) (smem + L::BAR_OFF);
    uint64_t * empty = full + STAGES;
    uint64_t * afull = empty + STAGES;       // [2] accumulator ready for the epilogue
    uint64_t * aempty = afull + 2;           // [2] accumulator drained (4 arrivals: one per epilogue warp)
    uint32_t * tslot = (uint32_t *) (aempty + 2);
    volatile int * abort_flag = (volatile int *) (tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long * tr = a.trace ? a.trace + (size_t) blockIdx.x * TRACE_SLOTS : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    const int MT = a.m_tiles_t * ((a.B + a.bb - 1) / a.bb), NT = (a.N + BN - 1) / BN;
    const int tiles = MT * NT, nk = a.k_blocks, dil = a.dil > 1 ? a.dil : 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&afull[b], 1); mbar_init(&aempty[b], 4); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 0) pdl_trigger();
    if (warp == 4 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmA2); tma_prefetch(&tmB); tma_prefetch(&tmB2); }
    if (warp == 5) tmem_alloc(tslot, 2 * ACC);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    auto tile_coords = [&](int tile, int & t0, int & b0, int & n0) {
        const int mi = tile % MT, ni = tile / MT;
        t0 = (mi % a.m_tiles_t) * a.bt;
        b0 = (mi / a.m_tiles_t) * a.bb;
        n0 = ni * BN;
    };

    if (warp == 4) {
        if (lane == 0) {
            // the first tile's weight stages do not depend on the upstream kernel
            int t0, b0, n0;
            tile_coords(blockIdx.x, t0, b0, n0);
            const int pre = blockIdx.x < tiles ? (nk < STAGES ? nk : STAGES) : 0;
            for (int i = 0; i < pre; ++i) {
                mbar_expect_tx(&full[i], L::STAGE);
                tma_load_2d(smem + i * L::STAGE + L::B_OFF, &tmB, &full[i], i * 64, n0);
                tma_load_2d(smem + i * L::STAGE + L::B2_OFF, &tmB2, &full[i], i * 64, n0);
            }
            pdl_wait();
            int g = 0;   // k blocks issued by this CTA so far (ring position)
            bool stop = false;
            for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
                tile_coords(tile, t0, b0, n0);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (g >= STAGES && !mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
                    uint8_t * sa = smem + s * L::STAGE;
                    if (g >= pre) {
                        mbar_expect_tx(&full[s], L::STAGE);
                        tma_load_2d(sa + L::B_OFF, &tmB, &full[s], kb * 64, n0);
                        tma_load_2d(sa + L::B2_OFF, &tmB2, &full[s], kb * 64, n0);
                    }
                    const int tap = kb / a.ic_blocks, ic0 = (kb % a.ic_blocks) * 64;
                    const int row = t0 + tap * dil - a.pad;
                    tma_load_3d(sa, &tmA, &full[s], ic0, row, b0);
                    tma_load_3d(sa + L::A_BYTES, &tmA2, &full[s], ic0, row, b0);
                }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(BN, 0);
            int g = 0, i = 0;
            bool stop = false;
            for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x, ++i) {
                const int buf = i & 1;
                if (i >= 2 && !mbar_wait(&aempty[buf], ((i >> 1) - 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t) (buf * ACC);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(&full[s], (g / STAGES) & 1, abort_flag, a.err, DEV_TIMEOUT_FULL)) { stop = true; break; }
                    if (tr && g == 0) tr[2] = global_ns();
                    tc_fence_after();
                    const uint8_t * sa = smem + s * L::STAGE;
                    const uint64_t ad = umma_desc_sw128(sa), al = umma_desc_sw128(sa + L::A_BYTES),
                                   bd = umma_desc_sw128(sa + L::B_OFF), b2 = umma_desc_sw128(sa + L::B2_OFF);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        umma_f16(d, ad + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, (kb | k) != 0);
                        umma_f16(d, al + (uint64_t) (2 * k), bd + (uint64_t) (2 * k), idesc, 1u);
                        umma_f16(d, ad + (uint64_t) (2 * k), b2 + (uint64_t) (2 * k), idesc, 1u);
                    }
                    umma_commit(&empty[s]);
                }
                if (!stop) umma_commit(&afull[buf]);
            }
        }
    } else {
        pdl_wait();
        const int r = warp * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        int i = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
            const int buf = i & 1;
            if (!mbar_wait(&afull[buf], (i >> 1) & 1, abort_flag, a.err, DEV_TIMEOUT_TMEM)) break;
            tc_fence_after();
            int t0, b0, n0;
            tile_coords(tile, t0, b0, n0);
            // the tile's constants straight from global memory (L1/L2-resident across tiles)
            const EpiConst ec{a.bias ? a.bias + n0 : nullptr, a.snake_a ? a.snake_a + n0 : nullptr,
                              a.snake_b ? a.snake_b + n0 : nullptr, nullptr, t0};
            if constexpr (EPI == EPI_F32 || EPI == EPI_RESID_SNAKE || EPI == EPI_F32_SNAKE2) {
                // rows are 512 B or more apart: each 32 x 32 chunk goes through this warp's padded
                // smem block, so every access instruction covers four whole 128-byte row segments
                // (the residual read, the f32 write and the split f16 write)
                float * tb = (float *) (smem + L::XPOSE_OFF) + warp * (32 * 33);
                const int cq = (lane & 7) * 4;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    float v[32];
                    tmem_ld32(trow + (uint32_t) (buf * ACC + c), v);
                    if (n0 + c >= a.N) continue;                  // the same for the whole warp
#pragma unroll
                    for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = v[j];
                    __syncwarp();
                    const int col = n0 + c + cq;
                    const bool col_ok = col < a.N;
                    float bl[4] = {0.f, 0.f, 0.f, 0.f}, ea[4] = {0.f, 0.f, 0.f, 0.f}, eb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (col_ok && ec.bias) bl[e] = __ldg(ec.bias + c + cq + e);
                        if (EPI != EPI_F32 && col_ok) { ea[e] = __ldg(ec.qn + c + cq + e); eb[e] = __ldg(ec.kn + c + cq + e); }
                    }
                    // the chunk's residual rows are read before any arithmetic: one memory round trip
                    float4 xr[8];
                    if (EPI == EPI_RESID_SNAKE) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int row = warp * 32 + 4 * i + (lane >> 3);
                            const int b = b0 + row / a.bt, t = t0 + row % a.bt;
                            xr[i] = col_ok && t < a.rows && b < a.B
                                        ? *(const float4 *) ((const float *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + col)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rr = 4 * i + (lane >> 3), row = warp * 32 + rr;
                        const int b = b0 + row / a.bt, t = t0 + row % a.bt;
                        if (!col_ok || t >= a.rows || b >= a.B) continue;
                        float y[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) y[e] = tb[rr * 33 + cq + e] + bl[e];
                        float * xo = (float *) a.out + (long long) b * a.out_bs + (long long) t * a.ldo + col;
                        if (EPI == EPI_RESID_SNAKE) {   // the residual add of src/vae.cpp:75
                            y[0] += xr[i].x; y[1] += xr[i].y; y[2] += xr[i].z; y[3] += xr[i].w;
                        }
                        *(float4 *) xo = make_float4(y[0], y[1], y[2], y[3]);
                        if constexpr (EPI != EPI_F32) {
                            __align__(8) __half hv[4], lv[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float sv = __sinf(y[e] * ea[e]);       // snake_, ops_conv.metal:204-213
                                const float z = y[e] + sv * sv * eb[e];
                                hv[e] = __float2half_rn(z);
                                lv[e] = __float2half_rn(z - __half2float(hv[e]));
                            }
                            __half * ho = (__half *) a.out2 + (long long) t * a.ldo2 + col;
                            *(uint2 *) ho = *(const uint2 *) hv;
                            *(uint2 *) (ho + a.out2_lo) = *(const uint2 *) lv;
                        }
                    }
                    __syncwarp();
                }
            } else {
                auto load_tmem = [&](int c, float * v) { tmem_ld32(trow + (uint32_t) (buf * ACC + c), v); };
#pragma unroll 1
                for (int u = 0; u < BN / EpiUnit<EPI>::U; ++u) epi_unit<EPI>(a, ec, r, u, n0, t0, b0, 0, true, load_tmem);
            }
            // this warp is done reading accumulator `buf`
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&aempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ACC);
    }
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
    if (*abort_flag && threadIdx.x == 0) {
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}

} // namespace tsn
