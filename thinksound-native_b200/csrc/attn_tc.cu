// attn_tc.cu — joint / latent attention on the tcgen05 tensor cores (sm_100a).
//
// Replaces attn_qk + softmax_rows + attn_pav (shaders/gemm_attn.metal:96-202) for the DiT path:
// O = softmax(Q·K^T / 8) · V per (arm, head), head dim 64, no mask, over the joint sequence. The
// [NH, S, S] f32 probability tensor of the reference never exists.
//
// One CTA per (128 query rows, head, arm), 192 threads, two CTAs per SM:
//   warp 4      TMA: the Q tile (hi and lo halves) once, then K (lane 0) and V (lane 1) 64-key
//               tiles into 2-stage rings; a K stage is free once its S product is done, a V stage
//               once its PV product is
//   warp 5      one thread issues the UMMAs: S_j = Qh·Kh^T + Qh·Kl^T + Ql·Kh^T (M 128, N 64,
//               K 64) into TMEM, one key tile ahead of the softmax, and O_j = P_j·Vh + P_j·Vl
//               (M 128, N 64, K 64; P read from TMEM, V MN-major from shared memory)
//   warps 0-3   one query row per thread: base-2 online softmax in f32 on the row of S_j read
//               from TMEM, P_j rounded to f16 and stored back into TMEM (the A operand of the PV
//               product), running O and row sum in registers, O / l written as the split f16
//               attention output of the row's stream.
// P and O_j are double-buffered in TMEM, so the softmax of tile j waits only for the PV product
// of tile j - 2: it overlaps the PV product of tile j - 1 instead of following it. O_j is folded
// into the register O two tiles later with the scale factors of both tiles. The arithmetic matches
// attn_kernel (same split products, P in f16, sums of the f32 p).
// Every mbarrier wait is bounded (ptx.cuh): a stalled pipeline ends the kernel with an error code.
#include "kernels.h"

namespace tsn {

namespace {

// 2^x by the hardware approximation (relative error ~2^-22, far below the f16 rounding of P)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr int Q_BYTES = 128 * 128;              // one half (hi or lo) of the 128 x 64 f16 Q tile
constexpr int KV_BYTES = 64 * 128;              // one half of a 64 x 64 f16 K or V tile
constexpr int OFF_Q = 0;                        // Q hi | Q lo
constexpr int OFF_K = 2 * Q_BYTES;              // [stage][hi | lo]
constexpr int OFF_V = OFF_K + 4 * KV_BYTES;     // [stage][hi | lo]
constexpr int OFF_BAR = OFF_V + 4 * KV_BYTES;
constexpr int SMEM_TOTAL = OFF_BAR + 256;       // the dynamic window starts 1024-aligned (checked)

// TMEM columns (256 allocated): S_j, O in two buffers, P (two f16 per column) in two buffers
constexpr uint32_t TM_S = 0, TM_O = 64, TM_P = 192;

// the split f16 attention output of joint row s_row (o unnormalised, l its row sum), into the
// output of the row's stream
__device__ __forceinline__ void store_row(const AttnArgs & a, int b, int h, int s_row, const float * o, float l) {
    if (s_row >= a.S) return;
    __half * dst;
    long long olo;
    if (s_row < a.n0) { dst = a.out0 + ((size_t) b * a.n0 + s_row) * a.H; olo = a.out_lo0; }
    else if (s_row < a.n0 + a.n1) { dst = a.out1 + ((size_t) b * a.n1 + (s_row - a.n0)) * a.H; olo = a.out_lo1; }
    else { dst = a.out2 + ((size_t) b * a.n2 + (s_row - a.n0 - a.n1)) * a.H; olo = a.out_lo2; }
    dst += h * 64;
    const float inv = 1.0f / l;
#pragma unroll
    for (int c = 0; c < 64; c += 8) {
        __align__(16) __half hv[8], lv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float v = o[c + e] * inv;
            hv[e] = __float2half_rn(v);
            lv[e] = __float2half_rn(v - __half2float(hv[e]));
        }
        *(uint4 *) (dst + c) = *(const uint4 *) hv;
        if (olo) *(uint4 *) (dst + olo + c) = *(const uint4 *) lv;
    }
}

// o = o * alpha + (this row's 64 columns of the O buffer at TMEM address t)
__device__ __forceinline__ void fold_o(float * o, float alpha, uint32_t t) {
#pragma unroll
    for (int c = 0; c < 64; c += 32) {
        float ot[32];
        tmem_ld32(t + c, ot);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c + e] = o[c + e] * alpha + ot[e];
    }
}

__global__ void __launch_bounds__(192, 2)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const AttnArgs a, int * err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long * tr = a.trace ? a.trace + 3 * ((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    if (smem_u32(smem) & 1023) {   // the swizzled tiles need 1024-byte alignment
        if (threadIdx.x == 0 && err) atomicCAS(err, 0, DEV_BAD_ARGS);
        return;
    }
    uint64_t * bar = (uint64_t *) (smem + OFF_BAR);
    uint64_t * q_full = bar;          // Q landed
    uint64_t * k_full = bar + 1;      // [2] K tile landed
    uint64_t * k_empty = bar + 3;     // [2] K tile consumed (after S)
    uint64_t * v_full = bar + 5;      // [2] V tile landed
    uint64_t * v_empty = bar + 7;     // [2] V tile consumed (after PV)
    uint64_t * s_full = bar + 9;      // S_j in TMEM
    uint64_t * s_free = bar + 10;     // S_j read by the softmax warps (4 arrivals)
    uint64_t * p_full = bar + 11;     // [2] P_j in TMEM buffer j & 1 (4 arrivals)
    uint64_t * pv_done = bar + 13;    // [2] O_j in TMEM buffer j & 1
    uint32_t * tslot = (uint32_t *) (bar + 15);
    volatile int * abort_flag = (volatile int *) (tslot + 1);

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int head_row = (b * a.NH + h) * a.S_pad;   // first row of this (arm, head) in the q/k/v views
    const int nkt = (a.S + 63) >> 6;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1);
            mbar_init(&p_full[s], 4); mbar_init(&pv_done[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 0) pdl_trigger();
    if (warp == 4 && lane == 0) { tma_prefetch(&tq); tma_prefetch(&tk); tma_prefetch(&tv); }
    if (warp == 5) tmem_alloc(tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 4) {
        if (lane < 2) {
            pdl_wait();
            if (lane == 0) {
                mbar_expect_tx(q_full, 2 * Q_BYTES);
                tma_load_3d(smem + OFF_Q, &tq, q_full, 0, head_row + qt * 128, 0);
                tma_load_3d(smem + OFF_Q + Q_BYTES, &tq, q_full, 0, head_row + qt * 128, 1);
            }
            // lane 0 streams K, lane 1 streams V
            const CUtensorMap * tm = lane == 0 ? &tk : &tv;
            uint64_t * full = lane == 0 ? k_full : v_full, * empty = lane == 0 ? k_empty : v_empty;
            uint8_t * ring = smem + (lane == 0 ? OFF_K : OFF_V);
            for (int j = 0; j < nkt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&empty[s], ((j >> 1) - 1) & 1, abort_flag, err, DEV_TIMEOUT_EMPTY)) break;
                uint8_t * t = ring + s * 2 * KV_BYTES;
                mbar_expect_tx(&full[s], 2 * KV_BYTES);
                tma_load_3d(t, tm, &full[s], 0, head_row + j * 64, 0);
                tma_load_3d(t + KV_BYTES, tm, &full[s], 0, head_row + j * 64, 1);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t id_s = umma_idesc_f16(64, 0), id_pv = umma_idesc_f16(64, 0, 1);
            const uint64_t qh = umma_desc_sw128(smem + OFF_Q), ql = umma_desc_sw128(smem + OFF_Q + Q_BYTES);
            bool ok = mbar_wait(q_full, 0, abort_flag, err, DEV_TIMEOUT_FULL);
            auto issue_s = [&](int j) {   // S_j = Qh Kh^T + Qh Kl^T + Ql Kh^T
                const int s = j & 1;
                if (!mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, err, DEV_TIMEOUT_FULL)) return false;
                if (j >= 1 && !mbar_wait(s_free, (j - 1) & 1, abort_flag, err, DEV_TIMEOUT_TMEM)) return false;
                if (tr && j == 0) tr[1] = global_ns();
                tc_fence_after();
                const uint8_t * k = smem + OFF_K + s * 2 * KV_BYTES;
                const uint64_t kh = umma_desc_sw128(k), kl = umma_desc_sw128(k + KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t o = (uint64_t) (2 * kk);
                    umma_f16(tmem + TM_S, qh + o, kh + o, id_s, kk != 0);
                    umma_f16(tmem + TM_S, qh + o, kl + o, id_s, 1u);
                    umma_f16(tmem + TM_S, ql + o, kh + o, id_s, 1u);
                }
                umma_commit(s_full);
                umma_commit(&k_empty[s]);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; j < nkt && ok; ++j) {
                if (j + 1 < nkt && !issue_s(j + 1)) break;
                // O_j = P_j (Vh + Vl) into O buffer j & 1, P_j from TMEM buffer j & 1
                const int pb = j & 1;
                if (!mbar_wait(&p_full[pb], (j >> 1) & 1, abort_flag, err, DEV_TIMEOUT_FULL)) break;
                if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, abort_flag, err, DEV_TIMEOUT_FULL)) break;
                tc_fence_after();
                const uint8_t * v = smem + OFF_V + (j & 1) * 2 * KV_BYTES;
                const uint32_t d = tmem + TM_O + 64 * pb, p = tmem + TM_P + 32 * pb;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t vh = umma_desc_sw128_mn(v + kk * 2048), vl = umma_desc_sw128_mn(v + KV_BYTES + kk * 2048);
                    umma_f16_ts(d, p + 8 * kk, vh, id_pv, kk != 0);
                    umma_f16_ts(d, p + 8 * kk, vl, id_pv, 1u);
                }
                umma_commit(&pv_done[pb]);
                umma_commit(&v_empty[j & 1]);
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warps
        pdl_wait();
        const int r = warp * 32 + lane;                          // query row within the tile
        const uint32_t trow = tmem + ((uint32_t) (warp * 32) << 16);
        float o[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0.0f;
        // m: running row max; a1, a2: the scale factors of tiles j - 1 and j - 2
        // (alpha_i = 2^(m_{i-1} - m_i)); O_{j-2} is folded at tile j with a2
        float m = -INFINITY, l = 0.0f, a1 = 1.0f, a2 = 1.0f;
        bool ok = true;
        for (int j = 0; j < nkt; ++j) {
            if (!mbar_wait(s_full, j & 1, abort_flag, err, DEV_TIMEOUT_TMEM)) { ok = false; break; }
            tc_fence_after();
            float p[64];
            tmem_ld32(trow + TM_S, p);
            tmem_ld32(trow + TM_S + 32, p + 32);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);                  // the MMA may overwrite S now
            // online softmax in base 2 on the scaled logits (scale > 0: max first, scale once);
            // keys >= S exist only in the last tile
            if (j * 64 + 64 > a.S) {
#pragma unroll
                for (int e = 0; e < 64; ++e)
                    if (j * 64 + e >= a.S) p[e] = -INFINITY;
            }
            // max and sum as four interleaved chains (one warp per SM sub-partition: the
            // softmax is latency-bound, not issue-bound)
            float mq[4] = {p[0], p[1], p[2], p[3]};
#pragma unroll
            for (int e = 4; e < 64; ++e) mq[e & 3] = fmaxf(mq[e & 3], p[e]);
            const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
            const float mn = fmaxf(m, mx * a.scale_log2);
            const float alpha = ex2(m - mn);
            m = mn;
            float sq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int e = 0; e < 64; ++e) {
                p[e] = ex2(fmaf(p[e], a.scale_log2, -mn));
                sq[e & 3] += p[e];
            }
            l = l * alpha + ((sq[0] + sq[1]) + (sq[2] + sq[3]));
            // buffer j & 1 is free once the PV product of tile j - 2 is done: fold O_{j-2}
            const int pb = j & 1;
            if (j >= 2) {
                if (!mbar_wait(&pv_done[pb], ((j - 2) >> 1) & 1, abort_flag, err, DEV_TIMEOUT_TMEM)) { ok = false; break; }
                tc_fence_after();
                fold_o(o, a2, trow + TM_O + 64 * pb);
            }
            // P_j as f16 pairs into TMEM buffer pb (column c holds elements 2c, 2c + 1)
            uint32_t pk[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const __half2 hv = __floats2half2_rn(p[2 * c], p[2 * c + 1]);
                pk[c] = *(const uint32_t *) &hv;
            }
            tmem_st32(trow + TM_P + 32 * pb, pk);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[pb]);
            a2 = a1;
            a1 = alpha;
        }
        // fold the last two tiles' O (tile nkt - 2 with its scale, then tile nkt - 1)
        for (int j = nkt >= 2 ? nkt - 2 : 0; ok && j < nkt; ++j) {
            const int pb = j & 1;
            if (!mbar_wait(&pv_done[pb], (j >> 1) & 1, abort_flag, err, DEV_TIMEOUT_TMEM)) { ok = false; break; }
            tc_fence_after();
            fold_o(o, j == nkt - 1 ? a1 : a2, trow + TM_O + 64 * pb);
        }
        if (ok) store_row(a, b, h, qt * 128 + r, o, l);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
    if (tr && threadIdx.x == 0) tr[2] = global_ns();
    if (*abort_flag && threadIdx.x == 0) {
        // let TMA copies that were issued but never consumed land before the CTA's smem is reused
        const uint64_t t1 = global_ns();
        while (global_ns() - t1 < 20000ull) {}
    }
}

// ================================================================================ short sequences
// attn_short_kernel: the same product for sequences of at most SHORT_MAX_KT * 64 = 384 keys (the DiT's
// 188-row fused blocks and 329-row joint blocks at the 8 s geometry, the encoders' 77 tokens), where
// every key and value tile of an (arm, head) fits in shared memory at once and the whole score row
// fits in TMEM. No online softmax: the UMMAs write S_j for key tile j as its K tile lands; the
// softmax takes the exact row maximum, writes P_j (f16 pairs) over the first half of S_j's columns,
// and the PV product of tile j starts as soon as P_j is written. One CTA per (128 query rows, head,
// arm), 448 threads:
//   warp 12     TMA: Q (hi, lo) and every K and V tile (hi, lo), each on its own barrier
//   warp 13     one thread issues S_j = Qh·Kh_j^T + Qh·Kl_j^T + Ql·Kh_j^T into TMEM columns
//               [64 j, 64 j + 64) (one commit per tile), then O = sum_j P_j·(Vh_j + Vl_j) with P_j
//               read from TMEM
//   warps 0-11  SHORT_G groups of four warps (warp w reads TMEM lanes 32 (w % 4) ..: one query row
//               per thread); group g owns key tiles g, g + SHORT_G, ...: the row maximum and row sum
//               of its tiles, combined across the groups through shared memory in group order (the
//               result does not depend on timing), p = 2^(s·scale_log2 + bias - max) in f32 (pairs
//               through the f32x2 FMA), P_j in f16 into TMEM; groups 0 and 1 write 32 columns each of
//               O / sum as the split f16 output.
// Spreading a row's keys over three warps per TMEM lane quadrant shortens the per-warp dependent
// chain of the softmax threefold; the exponentials are bound by the SFU rate (16 per cycle per SM).
// With an additive logit bias (the text encoders' T5 relative-position bias / pad mask, CLIP's causal
// and EOT mask; log2 units, -inf masks a key) the bias is added to the scaled logit of every key.
// Every wait is bounded; an aborted CTA waits (bounded) for its issued copies and UMMAs before it
// frees its TMEM and exits.
constexpr int SHORT_MAX_KT = 6;
constexpr int SHORT_G = 3;                             // softmax warp groups
constexpr int SHORT_THREADS = 32 * (4 * SHORT_G + 2);
constexpr int SH_OFF_K = 2 * Q_BYTES;                  // K: [hi tile 0 .. nkt-1][lo tile 0 .. nkt-1], then V the same way
__host__ __device__ constexpr int short_smem_bytes(int nkt) { return SH_OFF_K + 2 * nkt * 2 * KV_BYTES + 256; }

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float & a, float & b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
// (a0, a1) * (b0, b1) + (c0, c1), each lane rounded once
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__global__ void __launch_bounds__(SHORT_THREADS, 1)
attn_short_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const AttnArgs a, int * err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int W_TMA = 4 * SHORT_G, W_MMA = 4 * SHORT_G + 1;
    // stamps (globaltimer ns, 8 per CTA): 0 entry, 1 upstream done, 2 Q landed, 3 every S product
    // complete, 4 row maximum known, 5 exit, 6 every P written, 7 O complete
    unsigned long long * tr = a.trace ? a.trace + 8 * ((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    const int nkt = (a.S + 63) >> 6;
    if ((smem_u32(smem) & 1023) || nkt < 1 || nkt > SHORT_MAX_KT) {
        if (threadIdx.x == 0 && err) atomicCAS(err, 0, DEV_BAD_ARGS);
        return;
    }
    const int off_v = SH_OFF_K + nkt * 2 * KV_BYTES, off_bar = off_v + nkt * 2 * KV_BYTES;
    uint64_t * bar = (uint64_t *) (smem + off_bar);
    uint64_t * q_full = bar;                           // Q landed
    uint64_t * k_full = bar + 1;                       // [nkt] K tile j landed
    uint64_t * v_full = k_full + SHORT_MAX_KT;         // [nkt] V tile j landed
    uint64_t * s_full = v_full + SHORT_MAX_KT;         // [nkt] S_j in TMEM (and every S before it)
    uint64_t * p_ready = s_full + SHORT_MAX_KT;        // [nkt] P_j in TMEM (4 arrivals)
    uint64_t * o_full = p_ready + SHORT_MAX_KT;        // O complete
    uint64_t * drain = o_full + 1;                     // abort path: the issued UMMAs have completed
    uint32_t * tslot = (uint32_t *) (drain + 1);
    volatile int * abort_flag = (volatile int *) (tslot + 1);
    // per-row partial maxima and sums of the softmax groups, in the Q tile's space once every S
    // product (the only reader of Q) has completed
    float * red_max = (float *) smem;                  // [SHORT_G][128]
    float * red_sum = red_max + SHORT_G * 128;         // [SHORT_G][128]
    const uint32_t tcols = nkt <= 3 ? 256u : 512u;
    const uint32_t TM_OS = 64u * (uint32_t) nkt;      // O after the score columns

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int head_row = (b * a.NH + h) * a.S_pad;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int j = 0; j < SHORT_MAX_KT; ++j) {
            mbar_init(&k_full[j], 1); mbar_init(&v_full[j], 1); mbar_init(&s_full[j], 1); mbar_init(&p_ready[j], 4);
        }
        mbar_init(o_full, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        pdl_trigger();
    }
    if (warp == W_TMA && lane == 0) { tma_prefetch(&tq); tma_prefetch(&tk); tma_prefetch(&tv); }
    if (warp == W_MMA) tmem_alloc(tslot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == W_TMA) {
        if (lane == 0) {
            pdl_wait();
            if (tr) tr[1] = global_ns();
            mbar_expect_tx(q_full, 2 * Q_BYTES);
            tma_load_3d(smem, &tq, q_full, 0, head_row + qt * 128, 0);
            tma_load_3d(smem + Q_BYTES, &tq, q_full, 0, head_row + qt * 128, 1);
            for (int j = 0; j < nkt; ++j) {
                uint8_t * t = smem + SH_OFF_K + j * KV_BYTES;
                mbar_expect_tx(&k_full[j], 2 * KV_BYTES);
                tma_load_3d(t, &tk, &k_full[j], 0, head_row + j * 64, 0);
                tma_load_3d(t + nkt * KV_BYTES, &tk, &k_full[j], 0, head_row + j * 64, 1);
            }
            for (int j = 0; j < nkt; ++j) {
                uint8_t * t = smem + off_v + j * KV_BYTES;
                mbar_expect_tx(&v_full[j], 2 * KV_BYTES);
                tma_load_3d(t, &tv, &v_full[j], 0, head_row + j * 64, 0);
                tma_load_3d(t + nkt * KV_BYTES, &tv, &v_full[j], 0, head_row + j * 64, 1);
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            const uint32_t id_pv = umma_idesc_f16(64, 0, 1);
            const uint64_t qh = umma_desc_sw128(smem), ql = umma_desc_sw128(smem + Q_BYTES);
            bool ok = mbar_wait(q_full, 0, abort_flag, err, DEV_TIMEOUT_FULL);
            if (tr) tr[2] = global_ns();
            // S for key tiles [j0, j0 + w) in one set of UMMAs with N = 64 w (the hi and lo K tiles
            // are each contiguous, so w tiles form one K-major operand): nkt in chunks of at most
            // four, sizes as even as possible
            const int nch = (nkt + 3) / 4;
            for (int c = 0, j0 = 0; c < nch && ok; ++c) {
                const int w = (nkt - j0 + (nch - c) - 1) / (nch - c);
                for (int j = j0; j < j0 + w && ok; ++j) ok = mbar_wait(&k_full[j], 0, abort_flag, err, DEV_TIMEOUT_FULL);
                if (!ok) break;
                tc_fence_after();
                const uint8_t * k = smem + SH_OFF_K + j0 * KV_BYTES;
                const uint64_t kh = umma_desc_sw128(k), kl = umma_desc_sw128(k + nkt * KV_BYTES);
                const uint32_t id_s = umma_idesc_f16(64 * w, 0);
                const uint32_t d = tmem + 64u * (uint32_t) j0;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t o = (uint64_t) (2 * kk);
                    umma_f16(d, qh + o, kh + o, id_s, kk != 0);
                    umma_f16(d, qh + o, kl + o, id_s, 1u);
                    umma_f16(d, ql + o, kh + o, id_s, 1u);
                }
                for (int j = j0; j < j0 + w; ++j) umma_commit(&s_full[j]);
                j0 += w;
            }
            for (int j = 0; j < nkt && ok; ++j) {      // O += P_j (Vh_j + Vl_j) as P_j is written
                if (!(ok = mbar_wait(&p_ready[j], 0, abort_flag, err, DEV_TIMEOUT_TMEM))) break;
                if (!(ok = mbar_wait(&v_full[j], 0, abort_flag, err, DEV_TIMEOUT_FULL))) break;
                tc_fence_after();
                const uint8_t * v = smem + off_v + j * KV_BYTES;
                const uint32_t p = tmem + 32u * (uint32_t) j;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t vh = umma_desc_sw128_mn(v + kk * 2048), vl = umma_desc_sw128_mn(v + nkt * KV_BYTES + kk * 2048);
                    umma_f16_ts(tmem + TM_OS, p + 8 * kk, vh, id_pv, (j | kk) != 0);
                    umma_f16_ts(tmem + TM_OS, p + 8 * kk, vl, id_pv, 1u);
                }
            }
            if (ok) umma_commit(o_full);
            if (!ok) {   // let every UMMA issued so far complete before the TMEM is freed
                umma_commit(drain);
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000ull) {}
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warps
        pdl_wait();
        const int g = warp >> 2, qd = warp & 3;
        const int r = qd * 32 + lane;                            // query row within the tile
        const int row = qt * 128 + r;                            // joint row
        const uint32_t trow = tmem + ((uint32_t) (qd * 32) << 16);
        const float * lb = a.lbias ? a.lbias + (((size_t) b * a.NH + h) * a.S + (size_t) min(row, a.S - 1)) * a.S_pad
                                   : nullptr;
        bool ok = true;
        // pass 1: this group's maximum of the scaled (and biased) logits; keys >= S are masked
        float mloc = -INFINITY;
        for (int j = g; j < nkt && ok; j += SHORT_G) {
            if (!(ok = mbar_wait(&s_full[j], 0, abort_flag, err, DEV_TIMEOUT_TMEM))) break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float v[32];
                tmem_ld32(trow + 64u * (uint32_t) j + 32u * (uint32_t) c, v);
                const int key0 = j * 64 + c * 32;
                if (lb) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = fmaf(v[e], a.scale_log2, lb[key0 + e]);
                }
                if (key0 + 32 > a.S) {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (key0 + e >= a.S) v[e] = -INFINITY;
                }
                float mq[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
                for (int e = 4; e < 32; e += 8) {
                    mq[0] = max3f(mq[0], v[e], v[e + 1]);
                    mq[1] = max3f(mq[1], v[e + 2], v[e + 3]);
                    mq[2] = max3f(mq[2], v[e + 4], v[e + 5]);
                    mq[3] = max3f(mq[3], v[e + 6], v[e + 7]);
                }
                mloc = max3f(mloc, max3f(mq[0], mq[1], mq[2]), mq[3]);
            }
        }
        if (!lb && mloc != -INFINITY) mloc *= a.scale_log2;     // scale > 0: the max of the scaled logits
        // every S product is complete once the last tile's commit has arrived: Q's space is free
        if (ok) ok = mbar_wait(&s_full[nkt - 1], 0, abort_flag, err, DEV_TIMEOUT_TMEM);
        if (tr && warp == 0 && lane == 0) tr[3] = global_ns();
        if (ok) red_max[g * 128 + r] = mloc;
        epi_bar_n(128 * SHORT_G);
        if (tr && warp == 0 && lane == 0) tr[4] = global_ns();
        float m = -INFINITY;
        if (ok) {
#pragma unroll
            for (int q = 0; q < SHORT_G; ++q) m = fmaxf(m, red_max[q * 128 + r]);
            if (m == -INFINITY) m = 0.0f;                        // a row whose keys are all masked
        }
        // pass 2: p = 2^(x - m), the f32 row sum, P_j as f16 pairs over S_j's first half
        float lloc = 0.0f;
        const uint64_t sc2 = f2_pack(a.scale_log2, a.scale_log2), nm2 = f2_pack(-m, -m);
        for (int j = g; j < nkt && ok; j += SHORT_G) {
            float v[64];
            tmem_ld32(trow + 64u * (uint32_t) j, v);
            tmem_ld32(trow + 64u * (uint32_t) j + 32u, v + 32);
            uint64_t s2[4] = {0, 0, 0, 0};
            uint32_t pk[32];
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
                const int key = j * 64 + e;
                uint64_t x2 = lb ? fadd2(ffma2(f2_pack(v[e], v[e + 1]), sc2, f2_pack(lb[key], lb[key + 1])), nm2)
                                 : ffma2(f2_pack(v[e], v[e + 1]), sc2, nm2);
                float x0, x1;
                f2_unpack(x2, x0, x1);
                const float p0 = key < a.S ? ex2(x0) : 0.0f, p1 = key + 1 < a.S ? ex2(x1) : 0.0f;
                const uint64_t p2 = f2_pack(p0, p1);
                s2[(e >> 1) & 3] = fadd2(s2[(e >> 1) & 3], p2);
                const __half2 hv = __floats2half2_rn(p0, p1);
                pk[e >> 1] = *(const uint32_t *) &hv;
            }
            const uint64_t t2 = fadd2(fadd2(s2[0], s2[1]), fadd2(s2[2], s2[3]));
            float t0, t1;
            f2_unpack(t2, t0, t1);
            lloc += t0 + t1;
            tmem_st32(trow + 32u * (uint32_t) j, pk);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready[j]);
        }
        if (ok) red_sum[g * 128 + r] = lloc;
        epi_bar_n(128 * SHORT_G);
        if (tr && warp == 0 && lane == 0) tr[6] = global_ns();
        // O / l as split f16 halves, staged in shared memory over K and V (free once O is complete)
        // as [hi | lo][128 rows][64 cols], the 16-byte chunk c of a row at c ^ (row & 7), so that
        // the stores below write whole 128-byte row runs
        uint8_t * stage = smem + SH_OFF_K;
        if (ok && g < 2) {
            float l = 0.0f;
#pragma unroll
            for (int q = 0; q < SHORT_G; ++q) l += red_sum[q * 128 + r];
            if ((ok = mbar_wait(o_full, 0, abort_flag, err, DEV_TIMEOUT_TMEM))) {
                if (tr && warp == 0 && lane == 0) tr[7] = global_ns();
                tc_fence_after();
                float o[32];
                tmem_ld32(trow + TM_OS + 32u * (uint32_t) g, o);
                const float inv = 1.0f / l;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    __align__(16) __half hv[8], lv[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float v = o[c * 8 + e] * inv;
                        hv[e] = __float2half_rn(v);
                        lv[e] = __float2half_rn(v - __half2float(hv[e]));
                    }
                    const int pc = ((4 * g + c) ^ (r & 7)) << 4;
                    *(uint4 *) (stage + r * 128 + pc) = *(const uint4 *) hv;
                    *(uint4 *) (stage + 128 * 128 + r * 128 + pc) = *(const uint4 *) lv;
                }
            }
        }
        epi_bar_n(128 * SHORT_G);
        if (!*abort_flag) {
            // 256 row runs (hi and lo of 128 rows) of 128 bytes, four per warp instruction
            for (int seg = warp * 4 + (lane >> 3); seg < 256; seg += 4 * 4 * SHORT_G) {
                const int half = seg >> 7, rr = seg & 127, srow = qt * 128 + rr, ch = lane & 7;
                if (srow >= a.S) continue;
                __half * dst;
                long long olo;
                if (srow < a.n0) { dst = a.out0 + ((size_t) b * a.n0 + srow) * a.H; olo = a.out_lo0; }
                else if (srow < a.n0 + a.n1) { dst = a.out1 + ((size_t) b * a.n1 + (srow - a.n0)) * a.H; olo = a.out_lo1; }
                else { dst = a.out2 + ((size_t) b * a.n2 + (srow - a.n0 - a.n1)) * a.H; olo = a.out_lo2; }
                if (half && !olo) continue;
                const uint4 v = *(const uint4 *) (stage + half * 128 * 128 + rr * 128 + ((ch ^ (rr & 7)) << 4));
                *(uint4 *) (dst + (half ? olo : 0) + h * 64 + ch * 8) = v;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && warp == W_TMA && lane == 0) {
        // copies issued but never consumed must land before this CTA's shared memory is reused
        const uint64_t t0 = global_ns();
        bool landed = false;
        while (!landed && global_ns() - t0 < 1000000ull) {
            landed = mbar_try_wait(q_full, 0);
            for (int j = 0; j < nkt; ++j) landed = landed && mbar_try_wait(&k_full[j], 0) && mbar_try_wait(&v_full[j], 0);
        }
    }
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
    }
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
}

} // namespace

cudaError_t configure_attention_short() {
    return cudaFuncSetAttribute(attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                short_smem_bytes(SHORT_MAX_KT));
}

bool attention_short_fits(int S) { return S >= 1 && S <= SHORT_MAX_KT * 64; }

cudaError_t launch_attention_short(const AttnMaps & m, const AttnArgs & a, cudaStream_t s) {
    if (!attention_short_fits(a.S)) return cudaErrorInvalidValue;
    const int nkt = (a.S + 63) / 64;
    return launch_ex(attn_short_kernel, dim3((a.S + 127) / 128, a.NH, a.B), dim3(SHORT_THREADS), short_smem_bytes(nkt), s, 1u, m.q,
                     m.k, m.v, a, a.err);
}

cudaError_t configure_attention_tc() {
    return cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL);
}

cudaError_t launch_attention_tc(const AttnMaps & m, const AttnArgs & a, cudaStream_t s) {
    return launch_ex(attn_tc_kernel, dim3((a.S + 127) / 128, a.NH, a.B), dim3(192), SMEM_TOTAL, s, 1u, m.q, m.k, m.v, a,
                     a.err);
}

} // namespace tsn
