// oracle/kernels.cpp — scalar CPU restatement of the reference's Metal kernels
// (TEST INFRASTRUCTURE: the parity checker, never the product path).
//
// One function per kernel, each citing the shader lines it restates. Arithmetic is f32 with
// glibc expf/sqrtf/powf/cosf/sinf. Reductions keep the shader's own order where the shader
// fixes one; the MPP GEMM (shaders/gemm_mpp.metal:18-48, MetalPerformancePrimitives matmul2d)
// documents no order, so it is restated as a sequential k-order f32 fused-multiply-add chain,
// bias added after the sum (gemm_mpp.metal:36-44). Parallelism (OpenMP) is over independent
// outputs only, so results do not depend on the thread count.
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../include/tsn_synth.h"

namespace oracle {

float h2f(uint16_t h) { return tsn_f16_to_f32(h); }

// ---------------------------------------------------------------------------------------------
// GEMM  Y[M,N] = X[M,K] · W[N,K]^T (+ bias[n])      shaders/gemm_mpp.metal:18-48 (contract),
// dispatched by Runtime::gemm (src/net.mm:14-23).
// Blocked for speed (64 outputs of one row-block share a converted weight panel), but every
// output is one sequential fmaf chain over k = 0..K-1, so the blocking never changes a bit.
// ---------------------------------------------------------------------------------------------
template <typename WT, typename CVT>
static void gemm_core(const WT * W, const float * X, float * Y, const float * bias,
                      const GemmP & p, CVT cvt) {
    const int M = (int) p.M, N = (int) p.N, K = (int) p.K;
    const size_t ldx = p.ldx, ldw = p.ldw, ldy = p.ldy;
    constexpr int NB = 64, MB = 4;
    const int nblocks = (N + NB - 1) / NB;
#pragma omp parallel
    {
        std::vector<float> wt((size_t) K * NB);
#pragma omp for schedule(dynamic, 1)
        for (int nb = 0; nb < nblocks; ++nb) {
            const int n0 = nb * NB, nw = std::min(NB, N - n0);
            for (int k = 0; k < K; ++k)
                for (int j = 0; j < NB; ++j)
                    wt[(size_t) k * NB + j] = j < nw ? cvt(W[(size_t) (n0 + j) * ldw + k]) : 0.0f;
            for (int m0 = 0; m0 < M; m0 += MB) {
                const int mr = std::min(MB, M - m0);
                alignas(64) float acc[MB][NB];
                for (int r = 0; r < MB; ++r)
                    for (int j = 0; j < NB; ++j) acc[r][j] = 0.0f;
                for (int k = 0; k < K; ++k) {
                    const float * wk = &wt[(size_t) k * NB];
                    for (int r = 0; r < MB; ++r) {
                        const float xv = r < mr ? X[(size_t) (m0 + r) * ldx + k] : 0.0f;
                        for (int j = 0; j < NB; ++j) acc[r][j] = std::fmaf(xv, wk[j], acc[r][j]);
                    }
                }
                for (int r = 0; r < mr; ++r)
                    for (int j = 0; j < nw; ++j) {
                        float v = acc[r][j];
                        if (p.bias_mode) v += bias[n0 + j];
                        Y[(size_t) (m0 + r) * ldy + n0 + j] = v;
                    }
            }
        }
    }
}

void gemm_h(const uint16_t * W, const float * X, float * Y, const float * bias, const GemmP & p) {
    gemm_core(W, X, Y, bias, p, [](uint16_t h) { return tsn_f16_to_f32(h); });
}
void gemm_f(const float * W, const float * X, float * Y, const float * bias, const GemmP & p) {
    gemm_core(W, X, Y, bias, p, [](float f) { return f; });
}

// gemv: y[n] = bias[n] + Σ_k W[n,k]·x[k], sequential k      shaders/gemm_attn.metal:48-64
template <typename WT, typename CVT>
static void gemv_core(const WT * W, const float * X, float * Y, const float * bias,
                      const GemmP & p, CVT cvt) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < (int) p.N; ++n) {
        const WT * w = W + (size_t) n * p.ldw;
        float acc = p.bias_mode ? bias[n] : 0.0f;
        for (uint32_t k = 0; k < p.K; ++k) acc += cvt(w[k]) * X[k];
        Y[n] = acc;
    }
}
void gemv_h(const uint16_t * W, const float * X, float * Y, const float * bias, const GemmP & p) {
    gemv_core(W, X, Y, bias, p, [](uint16_t h) { return tsn_f16_to_f32(h); });
}
void gemv_f(const float * W, const float * X, float * Y, const float * bias, const GemmP & p) {
    gemv_core(W, X, Y, bias, p, [](float f) { return f; });
}

// ---------------------------------------------------------------------------------------------
// Attention, three passes                                   shaders/gemm_attn.metal:84-202
// ---------------------------------------------------------------------------------------------
// P[h,q,k] = scale·Σ_d Q[q,d]K[k,d] (+T5 bias / CLIP mask)   gemm_attn.metal:96-143
void attn_qk(const float * QKV, float * P, const int32_t * bkt, const float * rb, const AttnP & p) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < (int) p.nh; ++h)
        for (int q = 0; q < (int) p.Sq; ++q) {
            const float * qr = QKV + (size_t) q * p.ld + p.q_off + (size_t) h * p.hd;
            for (uint32_t k = 0; k < p.Sk; ++k) {
                const float * kr = QKV + (size_t) k * p.ld + p.k_off + (size_t) h * p.hd;
                float s = 0.0f;
                for (uint32_t d = 0; d < p.hd; ++d) s += qr[d] * kr[d];
                s *= p.scale;
                if (p.bias_mode == 1) {
                    const int32_t * pad = bkt + (size_t) p.Sq * p.Sk;
                    if (p.pad_on && pad[k] == 0) s = -INFINITY;
                    else s += rb[(size_t) bkt[(size_t) q * p.Sk + k] * p.nh + h];
                } else if (p.bias_mode == 2) {
                    if (!(k <= (uint32_t) q && k <= p.eot)) s = -INFINITY;
                }
                P[(size_t) p.p_off + ((size_t) h * p.Sq + q) * p.Sk + k] = s;
            }
        }
}

// in-place row softmax                                      gemm_attn.metal:145-157
void softmax_rows(float * P, const AttnP & p) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < (int) p.nh; ++h)
        for (int q = 0; q < (int) p.Sq; ++q) {
            float * row = P + (size_t) p.p_off + ((size_t) h * p.Sq + q) * p.Sk;
            float mx = -INFINITY;
            for (uint32_t k = 0; k < p.Sk; ++k) mx = std::max(mx, row[k]);
            float sum = 0.0f;
            for (uint32_t k = 0; k < p.Sk; ++k) { row[k] = std::exp(row[k] - mx); sum += row[k]; }
            const float inv = 1.0f / sum;
            for (uint32_t k = 0; k < p.Sk; ++k) row[k] *= inv;
        }
}

// O[q, h·hd+d] = Σ_k P[h,q,k]·V[k,d], summed in 32-key chunks   gemm_attn.metal:160-202
void attn_pav(const float * P, const float * QKV, float * O, const AttnP & p) {
    constexpr uint32_t KT = 32;
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < (int) p.nh; ++h)
        for (int q = 0; q < (int) p.Sq; ++q) {
            const float * prow = P + (size_t) p.p_off + ((size_t) h * p.Sq + q) * p.Sk;
            for (uint32_t d = 0; d < p.hd; ++d) {
                float acc = 0.0f;
                for (uint32_t k0 = 0; k0 < p.Sk; k0 += KT) {
                    float s = 0.0f;
                    for (uint32_t k = k0; k < std::min(k0 + KT, p.Sk); ++k)
                        s += prow[k] * QKV[(size_t) k * p.ld + p.v_off + (size_t) h * p.hd + d];
                    acc += s;
                }
                O[(size_t) q * p.ldo + p.o_off + (size_t) h * p.hd + d] = acc;
            }
        }
}

// ---------------------------------------------------------------------------------------------
// Convolution helpers                                      shaders/ops_conv.metal:215-283
// ---------------------------------------------------------------------------------------------
// col[r, ic·K+k] = x[ti(t0+r, k), ic], zero outside [0,T)   ops_conv.metal:265-283
void im2col(const float * x, float * col, const IcP & p, size_t n_threads) {
    const size_t KC = (size_t) p.IC * p.K;
    const size_t total = std::min(n_threads, (size_t) p.rows * KC);
#pragma omp parallel for schedule(static)
    for (long long gid = 0; gid < (long long) total; ++gid) {
        const uint32_t t = p.t0 + (uint32_t) (gid / KC), r = (uint32_t) (gid % KC);
        const uint32_t ic = r / p.K, k = r % p.K;
        int ti;
        bool ok;
        if (p.convt) {
            const int ui = (int) t - (int) p.pad + (int) k;
            ok = ui >= 0 && ui % (int) p.stride == 0;
            ti = ui / (int) p.stride;
        } else {
            ti = (int) (t * p.stride) - (int) p.pad + (int) (k * p.dil);
            ok = true;
        }
        ok = ok && ti >= 0 && ti < (int) p.T;
        col[gid] = ok ? x[(size_t) ti * p.ldx + ic] : 0.0f;
    }
}

// direct conv (VAE, OC < 32)                               ops_conv.metal:221-260
template <typename WT, typename CVT>
static void conv_core(const float * x, const WT * w, const float * bias, float * y,
                      const ConvP & p, CVT cvt) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < (int) p.OL; ++t)
        for (int oc = 0; oc < (int) p.OC; ++oc) {
            float acc = (p.use_bias && bias) ? bias[oc] : 0.0f;
            for (uint32_t ic = 0; ic < p.IC; ++ic)
                for (uint32_t k = 0; k < p.K; ++k) {
                    int ti;
                    if (p.convt) {
                        const int ui = t - (int) p.pad + (int) k;
                        if (ui < 0 || ui % (int) p.stride != 0) continue;
                        ti = ui / (int) p.stride;
                    } else {
                        ti = (int) (t * p.stride) - (int) p.pad + (int) (k * p.dil);
                    }
                    if (ti < 0 || ti >= (int) p.T) continue;
                    acc += x[(size_t) ti * p.ldx + ic] * cvt(w[((size_t) oc * p.IC + ic) * p.K + k]);
                }
            y[(size_t) t * p.ldy + oc] = acc;
        }
}
void conv1d_fwd_h(const float * x, const uint16_t * w, const float * bias, float * y, const ConvP & p) {
    conv_core(x, w, bias, y, p, [](uint16_t h) { return tsn_f16_to_f32(h); });
}
void conv1d_fwd_f(const float * x, const float * w, const float * bias, float * y, const ConvP & p) {
    conv_core(x, w, bias, y, p, [](float f) { return f; });
}

// ---------------------------------------------------------------------------------------------
// Elementwise                                               shaders/ops_conv.metal:9-57
// ---------------------------------------------------------------------------------------------
static inline float silu1(float v) { return v / (1.0f + std::exp(-v)); }

void silu_(float * x, uint32_t n) {                                    // :9-13
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) x[i] = silu1(x[i]);
}
void copy_(const float * x, float * y, uint32_t n) {                   // :30-34
    std::memmove(y, x, (size_t) n * 4);
}
void swiglu_(const float * a, const float * b, float * y, uint32_t n) { // :36-42
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) {
        const float va = a[i], vb = b[i];
        y[i] = (va / (1.0f + std::exp(-va))) * vb;
    }
}
void geglu_(const float * a, const float * b, float * y, uint32_t n) {  // :15-24
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) {
        const float v = a[i];
        const float arg = 0.7978845608f * (v + 0.044715f * v * v * v);
        y[i] = 0.5f * v * (1.0f + std::tanh(std::min(10.0f, std::max(-10.0f, arg)))) * b[i];
    }
}
void gelu_quick_(float * x, uint32_t n) {                              // :25-29
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) x[i] = x[i] / (1.0f + std::exp(-1.702f * x[i]));
}
void add_(const float * a, const float * b, float * y, uint32_t n) {    // :43-48
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) y[i] = a[i] + b[i];
}
void add_bcast_col(const float * x, const float * v, float * y, const CH & p) {   // :50-57
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) p.n; ++i) y[i] = x[i] + v[i % p.H];
}

// ---------------------------------------------------------------------------------------------
// Norms, adaLN, RoPE, qkv de-interleave                     shaders/ops_conv.metal:59-169
// ---------------------------------------------------------------------------------------------
// src col 3c+j -> dst block j·H + c at row row_off+y          ops_conv.metal:60-74
void qkv_split3(const float * src, float * dst, const QS3 & p, uint32_t rows) {
    const size_t ld = (size_t) 3 * p.H;
#pragma omp parallel for schedule(static)
    for (int y = 0; y < (int) rows; ++y)
        for (uint32_t c = 0; c < p.H; ++c)
            for (uint32_t j = 0; j < 3; ++j)
                dst[(size_t) (p.row_off + y) * ld + (size_t) j * p.H + c] = src[(size_t) y * ld + 3 * c + j];
}

static inline void ln_stats(const float * r, uint32_t H, float eps, float & mean, float & inv) {
    mean = 0.0f;
    for (uint32_t i = 0; i < H; ++i) mean += r[i];
    mean /= (float) H;
    float var = 0.0f;
    for (uint32_t i = 0; i < H; ++i) { const float d = r[i] - mean; var += d * d; }
    var /= (float) H;
    inv = 1.0f / std::sqrt(var + eps);
}

void ln_plain(const float * x, float * y, const HE & p, uint32_t rows) {       // :77-89
#pragma omp parallel for schedule(static)
    for (int g = 0; g < (int) rows; ++g) {
        const float * r = x + (size_t) g * p.H;
        float * o = y + (size_t) g * p.H;
        float mean, inv;
        ln_stats(r, p.H, p.eps, mean, inv);
        for (uint32_t i = 0; i < p.H; ++i) o[i] = (r[i] - mean) * inv;
    }
}
void ln_wb(const float * x, float * y, const float * w, const float * b, const HE & p, uint32_t rows) { // :90-103
#pragma omp parallel for schedule(static)
    for (int g = 0; g < (int) rows; ++g) {
        const float * r = x + (size_t) g * p.H;
        float * o = y + (size_t) g * p.H;
        float mean, inv;
        ln_stats(r, p.H, p.eps, mean, inv);
        for (uint32_t i = 0; i < p.H; ++i) o[i] = (r[i] - mean) * inv * w[i] + b[i];
    }
}
void rms_w(const float * x, float * y, const float * w, const HE & p, uint32_t rows) {   // :104-113
#pragma omp parallel for schedule(static)
    for (int g = 0; g < (int) rows; ++g) {
        const float * r = x + (size_t) g * p.H;
        float * o = y + (size_t) g * p.H;
        float ss = 0.0f;
        for (uint32_t i = 0; i < p.H; ++i) ss += r[i] * r[i];
        const float inv = 1.0f / std::sqrt(ss / (float) p.H + p.eps);
        for (uint32_t i = 0; i < p.H; ++i) o[i] = r[i] * inv * w[i];
    }
}

// per-head RMSNorm on a column slice, in place               ops_conv.metal:115-125
void rms_head(float * x, const float * w, const RH & p, uint32_t rows, uint32_t nh) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int g = 0; g < (int) rows; ++g)
        for (int h = 0; h < (int) nh; ++h) {
            float * r = x + (size_t) (p.row_off + g) * p.ld + p.col_off + (size_t) h * p.hd;
            float ss = 0.0f;
            for (uint32_t i = 0; i < p.hd; ++i) ss += r[i] * r[i];
            const float inv = 1.0f / std::sqrt(ss / (float) p.hd + p.eps);
            for (uint32_t i = 0; i < p.hd; ++i) r[i] = r[i] * inv * w[i];
        }
}

// y = LN(x)·(1 + m[base+H+i]) + m[base+i]                   ops_conv.metal:127-144
void adaln_ln(const float * x, const float * mod, float * y, const AD & p, uint32_t rows) {
#pragma omp parallel for schedule(static)
    for (int g = 0; g < (int) rows; ++g) {
        const float * r = x + (size_t) g * p.H;
        const float * m = mod + (p.per_row ? (size_t) g * p.chunks * p.H : 0) + p.base;
        float * o = y + (size_t) g * p.H;
        float mean, inv;
        ln_stats(r, p.H, p.eps, mean, inv);
        for (uint32_t i = 0; i < p.H; ++i) o[i] = (r[i] - mean) * inv * (1.0f + m[p.H + i]) + m[i];
    }
}

// y = x + f·mod[gate_idx·H + c] over every dispatched thread  ops_conv.metal:146-154
void gate_add(const float * x, const float * f, const float * mod, float * y, const GA & p, size_t n_threads) {
#pragma omp parallel for schedule(static)
    for (long long gid = 0; gid < (long long) n_threads; ++gid) {
        const uint32_t s = (uint32_t) (gid / p.H), c = (uint32_t) (gid % p.H);
        const float * m = mod + (p.per_row ? (size_t) s * p.chunks * p.H : 0);
        y[gid] = x[gid] + f[gid] * m[(size_t) p.gate_idx * p.H + c];
    }
}

// interleaved-pair RoPE per head                             ops_conv.metal:156-169
void rope_pairs(float * qkv, const int32_t * pos, const RP & p, uint32_t rows, uint32_t npairs_total) {
    const uint32_t npair = p.hd / 2;
#pragma omp parallel for collapse(2) schedule(static)
    for (int g = 0; g < (int) rows; ++g)
        for (int gy = 0; gy < (int) npairs_total; ++gy) {
            const uint32_t head = (uint32_t) gy / npair, j = (uint32_t) gy % npair;
            const float inv = std::pow(p.base, -2.0f * (float) j / (float) p.hd);
            const float ang = (float) (pos ? pos[g] : g) * p.fscale * inv;
            const float cs = std::cos(ang), sn = std::sin(ang);
            float * r = qkv + (size_t) (p.row_off + g) * p.ld + p.col_off + (size_t) head * p.hd;
            const float x0 = r[2 * j], x1 = r[2 * j + 1];
            r[2 * j] = x0 * cs - x1 * sn;
            r[2 * j + 1] = x0 * sn + x1 * cs;
        }
}

// column mean: 32 strided lane partials, then summed in lane order   ops_conv.metal:171-191
void mean_cols(const float * x, float * y, const SH & p) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < (int) p.H; ++c) {
        float partial[32];
        for (uint32_t lane = 0; lane < 32; ++lane) {
            float acc = 0.0f;
            for (uint32_t s = lane; s < p.S; s += 32) acc += x[(size_t) s * p.H + c];
            partial[lane] = acc;
        }
        float sum = 0.0f;
        for (uint32_t k = 0; k < 32; ++k) sum += partial[k];
        y[c] = sum / (float) p.S;
    }
}

// x += dt·(fu + (fc − fu)·cfg)                               ops_conv.metal:193-201
void cfg_euler(const float * fc, const float * fu, float * x, const CD & p) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) p.n; ++i) {
        const float v = fu[i] + (fc[i] - fu[i]) * p.cfg;
        x[i] += p.dt * v;
    }
}

// snake activation (VAE)                                     ops_conv.metal:203-213
void snake_(const float * x, float * y, const float * ab, const SH & p) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) p.S * p.H; ++i) {
        const uint32_t c = (uint32_t) (i % p.H);
        const float v = x[i];
        const float ea = std::exp(ab[c]), eb = std::exp(-ab[p.H + c]);
        const float s = std::sin(v * ea);
        y[i] = v + s * s * eb;
    }
}

// ---------------------------------------------------------------------------------------------
// dispatch by name with Metal grid semantics (src/gpu.mm:293-337)
// ---------------------------------------------------------------------------------------------
template <typename P>
static bool get(const void * params, size_t n, P & out) {
    if (!params || n < sizeof(P)) return false;
    std::memcpy(&out, params, sizeof(P));
    return true;
}

bool dispatch(const char * name_c, const Grid & g, const void * const * b, size_t nb,
              const void * params, size_t np) {
    const std::string name(name_c);
    const size_t threads = (size_t) g.gx * g.gy * g.gz * g.tx * g.ty * g.tz;
    auto F = [&](size_t i) { return (float *) (i < nb ? b[i] : nullptr); };
    auto U16 = [&](size_t i) { return (const uint16_t *) (i < nb ? b[i] : nullptr); };
    auto I32 = [&](size_t i) { return (const int32_t *) (i < nb ? b[i] : nullptr); };
    uint32_t n1 = 0;
    if (name == "gemm_mpp_h" || name == "gemm_mpp_h_rel" || name == "gemm_mpp_h_32x64" ||
        name == "gemm_mpp_h_64x64" || name == "gemm_h" || name == "gemm_t_h" || name == "gemm_t64_h") {
        GemmP p; if (!get(params, np, p)) return false;
        gemm_h(U16(0), F(1), F(2), F(3), p); return true;
    }
    if (name == "gemm_mpp_f" || name == "gemm_f" || name == "gemm_t_f") {
        GemmP p; if (!get(params, np, p)) return false;
        gemm_f(F(0), F(1), F(2), F(3), p); return true;
    }
    if (name == "gemv_h") { GemmP p; if (!get(params, np, p)) return false; gemv_h(U16(0), F(1), F(2), F(3), p); return true; }
    if (name == "gemv_f") { GemmP p; if (!get(params, np, p)) return false; gemv_f(F(0), F(1), F(2), F(3), p); return true; }
    if (name == "attn_qk") { AttnP p; if (!get(params, np, p)) return false; attn_qk(F(0), F(1), I32(2), F(3), p); return true; }
    if (name == "softmax_rows") { AttnP p; if (!get(params, np, p)) return false; softmax_rows(F(0), p); return true; }
    if (name == "attn_pav") { AttnP p; if (!get(params, np, p)) return false; attn_pav(F(0), F(1), F(2), p); return true; }
    if (name == "im2col") { IcP p; if (!get(params, np, p)) return false; im2col(F(0), F(1), p, threads); return true; }
    if (name == "conv1d_fwd") { ConvP p; if (!get(params, np, p)) return false; conv1d_fwd_h(F(0), U16(1), F(2), F(3), p); return true; }
    if (name == "conv1d_fwd_f") { ConvP p; if (!get(params, np, p)) return false; conv1d_fwd_f(F(0), F(1), F(2), F(3), p); return true; }
    if (name == "silu_") { if (!get(params, np, n1)) return false; silu_(F(0), n1); return true; }
    if (name == "copy_") { if (!get(params, np, n1)) return false; copy_(F(0), F(1), n1); return true; }
    if (name == "swiglu_") { if (!get(params, np, n1)) return false; swiglu_(F(0), F(1), F(2), n1); return true; }
    if (name == "geglu_") { if (!get(params, np, n1)) return false; geglu_(F(0), F(1), F(2), n1); return true; }
    if (name == "gelu_quick_") { if (!get(params, np, n1)) return false; gelu_quick_(F(0), n1); return true; }
    if (name == "add_") { if (!get(params, np, n1)) return false; add_(F(0), F(1), F(2), n1); return true; }
    if (name == "add_bcast_col") { CH p; if (!get(params, np, p)) return false; add_bcast_col(F(0), F(1), F(2), p); return true; }
    if (name == "qkv_split3") { QS3 p; if (!get(params, np, p)) return false; qkv_split3(F(0), F(1), p, g.gy * g.ty); return true; }
    if (name == "ln_plain") { HE p; if (!get(params, np, p)) return false; ln_plain(F(0), F(1), p, g.gx * g.tx); return true; }
    if (name == "ln_wb") { HE p; if (!get(params, np, p)) return false; ln_wb(F(0), F(1), F(2), F(3), p, g.gx * g.tx); return true; }
    if (name == "rms_w") { HE p; if (!get(params, np, p)) return false; rms_w(F(0), F(1), F(2), p, g.gx * g.tx); return true; }
    if (name == "rms_head") { RH p; if (!get(params, np, p)) return false; rms_head(F(0), F(1), p, g.gx * g.tx, g.gy * g.ty); return true; }
    if (name == "adaln_ln") { AD p; if (!get(params, np, p)) return false; adaln_ln(F(0), F(1), F(2), p, g.gx * g.tx); return true; }
    if (name == "gate_add") { GA p; if (!get(params, np, p)) return false; gate_add(F(0), F(1), F(2), F(3), p, threads); return true; }
    if (name == "rope_pairs") { RP p; if (!get(params, np, p)) return false; rope_pairs(F(0), I32(1), p, g.gx * g.tx, g.gy * g.ty); return true; }
    if (name == "mean_cols") { SH p; if (!get(params, np, p)) return false; mean_cols(F(0), F(1), p); return true; }
    if (name == "cfg_euler") { CD p; if (!get(params, np, p)) return false; cfg_euler(F(0), F(1), F(2), p); return true; }
    if (name == "snake_") { SH p; if (!get(params, np, p)) return false; snake_(F(0), F(1), F(2), p); return true; }
    return false;
}

} // namespace oracle
