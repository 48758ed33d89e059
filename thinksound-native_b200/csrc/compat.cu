// compat.cu — CUDA versions of the reference's named Metal kernels (see compat.h).
//
// Names and constant-block layouts accepted by compat_dispatch (reference file:line of each
// Metal kernel; struct layouts from src/gpu.h:52-78, src/dit_fwd.cpp:16-22, src/net.mm:44):
//   gemm_mpp_h / gemm_mpp_f / gemm_h / gemm_f  GemmP   shaders/gemm_mpp.metal:18-60, gemm_attn.metal:34-45
//   gemv_h / gemv_f                            GemmP   shaders/gemm_attn.metal:48-64
//   attn_qk / softmax_rows / attn_pav          AttnP   shaders/gemm_attn.metal:96-202
//   im2col                                     IcP     shaders/ops_conv.metal:265-283
//   conv1d_fwd / conv1d_fwd_f                  ConvP   shaders/ops_conv.metal:221-260
//   adaln_ln AD, gate_add GA, rms_head RH, rope_pairs RP, qkv_split3 QS3   ops_conv.metal:60-169
//   silu_ copy_ swiglu_ geglu_ gelu_quick_ add_ (N1), add_bcast_col CH, ln_plain/ln_wb/rms_w HE,
//   mean_cols SH, cfg_euler CD, snake_ SH                                  ops_conv.metal:9-213
// Thread-count semantics of the Metal dispatch (grid x threadgroup) are kept where the kernel
// depends on them (gate_add covers every dispatched thread; row counts come from the grid).
// Dense GEMMs whose shapes fit the tensor-core tiles (K, N multiples of 64) convert X to f16 and
// run the tcgen05 kernel; other shapes use a CUDA-core tiled GEMM.
#include <algorithm>
#include <cstring>
#include <string>

#include "compat.h"
#include "kernels.h"

namespace tsn {

namespace {
struct GemmP { uint32_t M, N, K, ldx, ldw, ldy, bias_mode, pad0; };
struct AttnP { uint32_t pad_on, Sq, Sk, hd, nh, ld, ldo, q_off, k_off, v_off, o_off, bias_mode, eot; float scale; uint32_t p_off; };
struct ConvP { uint32_t T, OL, IC, OC, K, stride, pad, dil, ldx, ldy, convt, use_bias; };
struct IcP { uint32_t T, rows, IC, K, stride, pad, dil, ldx, convt, t0; };
struct AD { uint32_t H, per_row, chunks, base; float eps; };
struct GA { uint32_t H, per_row, chunks, gate_idx; };
struct RH { uint32_t ld, hd, col_off, row_off; float eps; };
struct RP { uint32_t ld, hd, col_off, row_off; float fscale, base; };
struct QS3 { uint32_t H, row_off; };
struct CD { float cfg, dt; uint32_t n; };
struct CH { uint32_t H, n; };
struct SH { uint32_t S, H; };
struct HE { uint32_t H; float eps; };

__device__ __forceinline__ float ld_w(const void * w, int f16, size_t i) {
    return f16 ? __half2float(((const __half *) w)[i]) : ((const float *) w)[i];
}
__device__ __forceinline__ float silu1(float v) { return v / (1.0f + expf(-v)); }

#define GRID_STRIDE(i, n) for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < (long long) (n); i += (long long) gridDim.x * blockDim.x)

__global__ void k_unary(int op, float * x, const float * a, const float * b, float * y, long long n, uint32_t H) {
    GRID_STRIDE(i, n) {
        switch (op) {
            case 0: x[i] = silu1(x[i]); break;
            case 1: y[i] = a[i]; break;
            case 2: { const float va = a[i]; y[i] = (va / (1.0f + expf(-va))) * b[i]; } break;
            case 3: { const float v = a[i], arg = 0.7978845608f * (v + 0.044715f * v * v * v);
                      y[i] = 0.5f * v * (1.0f + tanhf(fminf(10.0f, fmaxf(-10.0f, arg)))) * b[i]; } break;
            case 4: x[i] = x[i] / (1.0f + expf(-1.702f * x[i])); break;
            case 5: y[i] = a[i] + b[i]; break;
            case 6: y[i] = a[i] + b[i % H]; break;
        }
    }
}

__global__ void k_qkv_split3(const float * src, float * dst, QS3 p, uint32_t rows) {
    GRID_STRIDE(i, (long long) rows * p.H) {
        const uint32_t y = (uint32_t) (i / p.H), c = (uint32_t) (i % p.H);
        const size_t ld = (size_t) 3 * p.H;
        for (uint32_t j = 0; j < 3; ++j) dst[(size_t) (p.row_off + y) * ld + (size_t) j * p.H + c] = src[(size_t) y * ld + 3 * c + j];
    }
}

// one warp per row: mode 0 ln_plain, 1 ln_wb, 2 rms_w, 3 adaln_ln
__global__ void k_rownorm(int mode, const float * x, float * y, const float * w, const float * bb, const float * mod,
                          uint32_t H, float eps, uint32_t per_row, uint32_t chunks, uint32_t base, uint32_t rows) {
    const uint32_t g = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (g >= rows) return;
    const float * r = x + (size_t) g * H;
    float * o = y + (size_t) g * H;
    float mean = 0.0f, inv;
    if (mode == 2) {
        float ss = 0.0f;
        for (uint32_t i = lane; i < H; i += 32) ss += r[i] * r[i];
        for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        inv = 1.0f / sqrtf(ss / (float) H + eps);
    } else {
        float s = 0.0f;
        for (uint32_t i = lane; i < H; i += 32) s += r[i];
        for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        mean = s / (float) H;
        float var = 0.0f;
        for (uint32_t i = lane; i < H; i += 32) { const float d = r[i] - mean; var += d * d; }
        for (int off = 16; off; off >>= 1) var += __shfl_xor_sync(0xffffffffu, var, off);
        inv = 1.0f / sqrtf(var / (float) H + eps);
    }
    const float * m = mod ? mod + (per_row ? (size_t) g * chunks * H : 0) + base : nullptr;
    for (uint32_t i = lane; i < H; i += 32) {
        switch (mode) {
            case 0: o[i] = (r[i] - mean) * inv; break;
            case 1: o[i] = (r[i] - mean) * inv * w[i] + bb[i]; break;
            case 2: o[i] = r[i] * inv * w[i]; break;
            case 3: o[i] = (r[i] - mean) * inv * (1.0f + m[H + i]) + m[i]; break;
        }
    }
}

__global__ void k_rms_head(float * x, const float * w, RH p, uint32_t rows, uint32_t nh) {
    GRID_STRIDE(i, (long long) rows * nh) {
        const uint32_t g = (uint32_t) (i / nh), h = (uint32_t) (i % nh);
        float * r = x + (size_t) (p.row_off + g) * p.ld + p.col_off + (size_t) h * p.hd;
        float ss = 0.0f;
        for (uint32_t k = 0; k < p.hd; ++k) ss += r[k] * r[k];
        const float inv = 1.0f / sqrtf(ss / (float) p.hd + p.eps);
        for (uint32_t k = 0; k < p.hd; ++k) r[k] = r[k] * inv * w[k];
    }
}

__global__ void k_rope(float * qkv, const int * pos, RP p, uint32_t rows, uint32_t npt) {
    const uint32_t npair = p.hd / 2;
    GRID_STRIDE(i, (long long) rows * npt) {
        const uint32_t g = (uint32_t) (i / npt), gy = (uint32_t) (i % npt);
        const uint32_t head = gy / npair, j = gy % npair;
        const float inv = powf(p.base, -2.0f * (float) j / (float) p.hd);
        const float ang = (float) (pos ? pos[g] : (int) g) * p.fscale * inv;
        const float cs = cosf(ang), sn = sinf(ang);
        float * r = qkv + (size_t) (p.row_off + g) * p.ld + p.col_off + (size_t) head * p.hd;
        const float x0 = r[2 * j], x1 = r[2 * j + 1];
        r[2 * j] = x0 * cs - x1 * sn;
        r[2 * j + 1] = x0 * sn + x1 * cs;
    }
}

__global__ void k_gate_add(const float * x, const float * f, const float * mod, float * y, GA p, long long nthreads) {
    GRID_STRIDE(i, nthreads) {
        const uint32_t s = (uint32_t) (i / p.H), c = (uint32_t) (i % p.H);
        const float * m = mod + (p.per_row ? (size_t) s * p.chunks * p.H : 0);
        y[i] = x[i] + f[i] * m[(size_t) p.gate_idx * p.H + c];
    }
}

__global__ void k_mean_cols(const float * x, float * y, SH p) {
    GRID_STRIDE(c, p.H) {
        float part[32];
        for (uint32_t lane = 0; lane < 32; ++lane) {
            float acc = 0.0f;
            for (uint32_t s = lane; s < p.S; s += 32) acc += x[(size_t) s * p.H + c];
            part[lane] = acc;
        }
        float sum = 0.0f;
        for (int k = 0; k < 32; ++k) sum += part[k];
        y[c] = sum / (float) p.S;
    }
}

__global__ void k_cfg_euler(const float * fc, const float * fu, float * x, CD p) {
    GRID_STRIDE(i, p.n) {
        const float v = __fadd_rn(fu[i], __fmul_rn(__fsub_rn(fc[i], fu[i]), p.cfg));
        x[i] = __fadd_rn(x[i], __fmul_rn(p.dt, v));
    }
}

__global__ void k_snake(const float * x, float * y, const float * ab, SH p) {
    GRID_STRIDE(i, (long long) p.S * p.H) {
        const uint32_t c = (uint32_t) (i % p.H);
        const float v = x[i], ea = expf(ab[c]), eb = expf(-ab[p.H + c]), s = sinf(v * ea);
        y[i] = v + s * s * eb;
    }
}

__global__ void k_im2col(const float * x, float * col, IcP p, long long nthreads) {
    const long long KC = (long long) p.IC * p.K;
    const long long total = nthreads < (long long) p.rows * KC ? nthreads : (long long) p.rows * KC;
    GRID_STRIDE(gid, total) {
        const uint32_t t = p.t0 + (uint32_t) (gid / KC), r = (uint32_t) (gid % KC), ic = r / p.K, k = r % p.K;
        int ti;
        bool ok;
        if (p.convt) { const int ui = (int) t - (int) p.pad + (int) k; ok = ui >= 0 && ui % (int) p.stride == 0; ti = ui / (int) p.stride; }
        else { ti = (int) (t * p.stride) - (int) p.pad + (int) (k * p.dil); ok = true; }
        ok = ok && ti >= 0 && ti < (int) p.T;
        col[gid] = ok ? x[(size_t) ti * p.ldx + ic] : 0.0f;
    }
}

__global__ void k_conv1d(const float * x, const void * w, int wf16, const float * bias, float * y, ConvP p) {
    GRID_STRIDE(i, (long long) p.OL * p.OC) {
        const uint32_t t = (uint32_t) (i / p.OC), oc = (uint32_t) (i % p.OC);
        float acc = (p.use_bias && bias) ? bias[oc] : 0.0f;
        for (uint32_t ic = 0; ic < p.IC; ++ic)
            for (uint32_t k = 0; k < p.K; ++k) {
                int ti;
                if (p.convt) { const int ui = (int) t - (int) p.pad + (int) k; if (ui < 0 || ui % (int) p.stride) continue; ti = ui / (int) p.stride; }
                else ti = (int) (t * p.stride) - (int) p.pad + (int) (k * p.dil);
                if (ti < 0 || ti >= (int) p.T) continue;
                acc += x[(size_t) ti * p.ldx + ic] * ld_w(w, wf16, ((size_t) oc * p.IC + ic) * p.K + k);
            }
        y[(size_t) t * p.ldy + oc] = acc;
    }
}

// warp per output row
__global__ void k_gemv(const void * W, int wf16, const float * X, float * Y, const float * bias, GemmP p) {
    const uint32_t n = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (n >= p.N) return;
    float acc = 0.0f;
    for (uint32_t k = lane; k < p.K; k += 32) acc += ld_w(W, wf16, (size_t) n * p.ldw + k) * X[k];
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) Y[n] = acc + (p.bias_mode ? bias[n] : 0.0f);
}

// CUDA-core tiled GEMM for shapes the tensor-core tiles do not cover
__global__ void k_gemm_simple(const void * W, int wf16, const float * X, float * Y, const float * bias, GemmP p) {
    __shared__ float xs[16][17], ws[16][17];
    const uint32_t tx = threadIdx.x, ty = threadIdx.y;
    const uint32_t m = blockIdx.y * 16 + ty, n = blockIdx.x * 16 + tx;
    float acc = 0.0f;
    for (uint32_t k0 = 0; k0 < p.K; k0 += 16) {
        xs[ty][tx] = (m < p.M && k0 + tx < p.K) ? X[(size_t) m * p.ldx + k0 + tx] : 0.0f;
        const uint32_t wn = blockIdx.x * 16 + ty;
        ws[ty][tx] = (wn < p.N && k0 + tx < p.K) ? ld_w(W, wf16, (size_t) wn * p.ldw + k0 + tx) : 0.0f;
        __syncthreads();
        for (int kk = 0; kk < 16; ++kk) acc += xs[ty][kk] * ws[tx][kk];
        __syncthreads();
    }
    if (m < p.M && n < p.N) Y[(size_t) m * p.ldy + n] = acc + (p.bias_mode ? bias[n] : 0.0f);
}

// f32 [M][ldx] -> split f16 operand: hi [M][K] at out, lo [M][K] at out + M*K
__global__ void k_f32_to_f16(const float * x, uint32_t M, uint32_t K, uint32_t ldx, __half * out) {
    GRID_STRIDE(i, (long long) M * K) {
        const uint32_t m = (uint32_t) (i / K), k = (uint32_t) (i % K);
        const float v = x[(size_t) m * ldx + k];
        const __half h = __float2half_rn(v);
        out[i] = h;
        out[i + (long long) M * K] = __float2half_rn(v - __half2float(h));
    }
}

__global__ void k_attn_qk(const float * QKV, float * P, const int * bkt, const float * rb, AttnP p) {
    GRID_STRIDE(i, (long long) p.nh * p.Sq * p.Sk) {
        const uint32_t k = (uint32_t) (i % p.Sk), q = (uint32_t) ((i / p.Sk) % p.Sq), h = (uint32_t) (i / ((long long) p.Sk * p.Sq));
        const float * qr = QKV + (size_t) q * p.ld + p.q_off + (size_t) h * p.hd;
        const float * kr = QKV + (size_t) k * p.ld + p.k_off + (size_t) h * p.hd;
        float s = 0.0f;
        for (uint32_t d = 0; d < p.hd; ++d) s += qr[d] * kr[d];
        s *= p.scale;
        if (p.bias_mode == 1) {
            const int * pad = bkt + (size_t) p.Sq * p.Sk;
            if (p.pad_on && pad[k] == 0) s = -INFINITY;
            else s += rb[(size_t) bkt[(size_t) q * p.Sk + k] * p.nh + h];
        } else if (p.bias_mode == 2) {
            if (!(k <= q && k <= p.eot)) s = -INFINITY;
        }
        P[(size_t) p.p_off + ((size_t) h * p.Sq + q) * p.Sk + k] = s;
    }
}

// warp per row
__global__ void k_softmax_rows(float * P, AttnP p) {
    const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (row >= p.nh * p.Sq) return;
    float * r = P + (size_t) p.p_off + (size_t) row * p.Sk;
    float mx = -INFINITY;
    for (uint32_t k = lane; k < p.Sk; k += 32) mx = fmaxf(mx, r[k]);
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (uint32_t k = lane; k < p.Sk; k += 32) { const float e = expf(r[k] - mx); r[k] = e; sum += e; }
    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = 1.0f / sum;
    for (uint32_t k = lane; k < p.Sk; k += 32) r[k] *= inv;
}

__global__ void k_attn_pav(const float * P, const float * QKV, float * O, AttnP p) {
    GRID_STRIDE(i, (long long) p.nh * p.Sq * p.hd) {
        const uint32_t d = (uint32_t) (i % p.hd), q = (uint32_t) ((i / p.hd) % p.Sq), h = (uint32_t) (i / ((long long) p.hd * p.Sq));
        const float * pr = P + (size_t) p.p_off + ((size_t) h * p.Sq + q) * p.Sk;
        float acc = 0.0f;
        for (uint32_t k = 0; k < p.Sk; ++k) acc += pr[k] * QKV[(size_t) k * p.ld + p.v_off + (size_t) h * p.hd + d];
        O[(size_t) q * p.ldo + p.o_off + (size_t) h * p.hd + d] = acc;
    }
}

inline unsigned nblk(long long n, int t = 256) {
    long long b = (n + t - 1) / t;
    return (unsigned) (b < 1 ? 1 : b > 65535 * 8 ? 65535 * 8 : b);
}

template <typename P>
bool get(const void * params, size_t n, P & out) {
    if (!params || n < sizeof(P)) return false;
    std::memcpy(&out, params, sizeof(P));
    return true;
}

int launched(const char * name) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("launch ") + name + ": " + cudaGetErrorString(e));
    return TSN_OK;
}

int ensure_scratch(DeviceCtx & c, size_t bytes) {
    if (c.scratch_bytes >= bytes) return TSN_OK;
    if (c.scratch) { cudaStreamSynchronize(c.stream); cudaFree(c.scratch); c.scratch = nullptr; }
    if (cudaMalloc(&c.scratch, bytes) != cudaSuccess) { c.scratch_bytes = 0; return fail(TSN_ERR_OOM, "compat scratch"); }
    c.scratch_bytes = bytes;
    return TSN_OK;
}

const char * const kNames[] = {"gemm_mpp_h", "gemm_mpp_f", "gemm_mpp_h_rel", "gemm_mpp_h_32x64", "gemm_mpp_h_64x64",
                                "gemm_h", "gemm_f", "gemv_h", "gemv_f", "attn_qk", "softmax_rows", "attn_pav",
                                "im2col", "conv1d_fwd", "conv1d_fwd_f", "adaln_ln", "gate_add", "rms_head",
                                "rope_pairs", "qkv_split3", "silu_", "copy_", "swiglu_", "geglu_", "gelu_quick_",
                                "add_", "add_bcast_col", "ln_plain", "ln_wb", "rms_w", "mean_cols", "cfg_euler", "snake_"};
} // namespace

bool compat_has(const char * name) {
    for (const char * n : kNames)
        if (!std::strcmp(n, name)) return true;
    return false;
}

int compat_gemm(DeviceCtx & c, int wf16, const void * W, const void * X, void * Y, const void * bias,
                uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy) {
    if (M == 0 || N == 0) return TSN_OK;
    GemmP p{M, N, K, ldx, ldw, ldy, bias ? 1u : 0u, 0};
    const bool tc = wf16 && K % 64 == 0 && N % 64 == 0 && (ldw * 2) % 16 == 0 && ((uintptr_t) W & 15) == 0;
    if (!tc) {
        dim3 grid((N + 15) / 16, (M + 15) / 16);
        k_gemm_simple<<<grid, dim3(16, 16), 0, c.stream>>>(W, wf16, (const float *) X, (float *) Y, (const float *) bias, p);
        return launched("gemm_simple");
    }
    // X -> split f16 operand (hi | lo), then the tcgen05 GEMM with one batch of 128-row tiles;
    // weights whose rows are ldw apart are first packed to a dense [N][K] copy for the TMA view.
    const size_t xa_bytes = ((size_t) 2 * M * K * 2 + 255) & ~(size_t) 255;
    int rc = ensure_scratch(c, xa_bytes + (ldw != K ? (size_t) N * K * 2 : 0));
    if (rc) return rc;
    __half * xa = (__half *) c.scratch;
    k_f32_to_f16<<<nblk((long long) M * K), 256, 0, c.stream>>>((const float *) X, M, K, ldx, xa);
    if ((rc = launched("f32_to_f16"))) return rc;
    const void * wd = W;
    if (ldw != K) {
        wd = (char *) c.scratch + xa_bytes;
        cudaError_t e = cudaMemcpy2DAsync((void *) wd, (size_t) K * 2, W, (size_t) ldw * 2, (size_t) K * 2, N,
                                          cudaMemcpyDefault, c.stream);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("compat gemm: pack W: ") + cudaGetErrorString(e));
    }
    const int bn = N % 256 == 0 ? 256 : N % 128 == 0 ? 128 : 64;
    GemmLaunch g{};
    g.bn = bn; g.epi = EPI_F32; g.split = true; g.smem = gemm_smem_bytes(bn, true, EPI_F32); g.ab_bf16 = 0;
    g.grid = dim3(N / bn, (M + 127) / 128, 1);
    if (!make_act_map(&g.ta, xa, K, M, 1, 128, 1, 0) || !make_act_map(&g.ta2, xa + (size_t) M * K, K, M, 1, 128, 1, 0) ||
        !make_w_map(&g.tb, wd, K, N, bn, 0))
        return fail(TSN_ERR_CUDA, "compat gemm: tensor maps");
    GemmArgs & a = g.args;
    a.rows = (int) M; a.B = 1; a.bt = 128; a.bb = 1; a.m_tiles_t = (int) ((M + 127) / 128); a.N = (int) N;
    a.k_blocks = (int) (K / 64); a.ic_blocks = (int) (K / 64); a.pad = 0; a.splits = 1; a.kb_per_split = a.k_blocks;
    a.err = c.d_err;
    a.bias = (const float *) bias;
    a.out = Y; a.ldo = ldy; a.out_bs = 0;
    cudaError_t e = launch_gemm(g, c.stream);
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("compat gemm: ") + cudaGetErrorString(e));
    return TSN_OK;
}

int compat_gemv(DeviceCtx & c, int wf16, const void * W, const void * X, void * Y, const void * bias, uint32_t N,
                uint32_t K, uint32_t ldw) {
    if (N == 0) return TSN_OK;
    // f16 weights with dense 16-byte-aligned rows of at most 1024: the weight-streaming GEMV
    if (wf16 && ldw == K && K % 8 == 0 && K <= (uint32_t) GEMV_MAX_K && ((uintptr_t) W & 15) == 0) {
        GemvJob j{W, (const float *) bias, (const float *) X, 0, nullptr, 0, (float *) Y, 0, (int) N, (int) K, 1, 0};
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.ordinal);
        cudaError_t e = launch_gemv(&j, 1, (int) N, 1, sms, 0, c.d_err, c.stream);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("gemv: ") + cudaGetErrorString(e));
        return TSN_OK;
    }
    GemmP p{1, N, K, K, ldw, N, bias ? 1u : 0u, 0};
    k_gemv<<<(N + 7) / 8, 256, 0, c.stream>>>(W, wf16, (const float *) X, (float *) Y, (const float *) bias, p);
    return launched("gemv");
}

// Runtime::conv (src/net.mm:25-49): pointwise -> GEMM; OC < 32 -> direct; else im2col + GEMM
int compat_conv(DeviceCtx & c, int wf16, const void * W, const void * bias, const void * x, void * y, uint32_t T,
                uint32_t OL, uint32_t IC, uint32_t OC, uint32_t K, uint32_t stride, uint32_t pad, uint32_t dil, int convt) {
    if (K == 1 && stride == 1 && pad == 0 && !convt && OL == T) return compat_gemm(c, wf16, W, x, y, bias, OL, OC, IC, IC, IC, OC);
    if (OC < 32) {
        ConvP p{T, OL, IC, OC, K, stride, pad, dil, IC, OC, convt ? 1u : 0u, bias ? 1u : 0u};
        k_conv1d<<<nblk((long long) OL * OC), 256, 0, c.stream>>>((const float *) x, W, wf16, (const float *) bias, (float *) y, p);
        return launched("conv1d");
    }
    // Runtime::conv's chunking (src/net.mm:36-47): output rows per chunk keep the col scratch at
    // most 16 M floats; the col buffer persists on the device context (grown only when a larger
    // chunk needs it, freed with the device), so a conv allocates nothing once the buffer is sized
    const size_t KC = (size_t) IC * K, max_elems = (size_t) 16 << 20;
    const uint32_t rows = (uint32_t) std::max<size_t>(1, std::min<size_t>(OL, max_elems / KC));
    const size_t need = (size_t) rows * KC * 4;
    if (c.col_bytes < need) {
        if (c.col) { cudaStreamSynchronize(c.stream); cudaFree(c.col); c.col = nullptr; c.col_bytes = 0; }
        if (cudaMalloc(&c.col, need) != cudaSuccess) return fail(TSN_ERR_OOM, "im2col buffer");
        c.col_bytes = need;
    }
    float * col = (float *) c.col;
    for (uint32_t t0 = 0; t0 < OL; t0 += rows) {
        const uint32_t n = std::min(rows, OL - t0);
        IcP ip{T, n, IC, K, stride, pad, dil, IC, convt ? 1u : 0u, t0};
        k_im2col<<<nblk((long long) n * KC), 256, 0, c.stream>>>((const float *) x, col, ip, (long long) n * KC);
        int rc = launched("im2col");
        if (!rc) rc = compat_gemm(c, wf16, W, col, (float *) y + (size_t) t0 * OC, bias, n, OC, (uint32_t) KC, (uint32_t) KC,
                                  (uint32_t) KC, OC);
        if (rc) return rc;
    }
    return TSN_OK;
}

int compat_elementwise(DeviceCtx & c, const char * name, const void * a, const void * b, void * y, size_t n,
                       uint32_t h, int) {
    const std::string s(name);
    const int op = s == "silu_" ? 0 : s == "copy_" ? 1 : s == "swiglu_" ? 2 : s == "geglu_" ? 3 : s == "gelu_quick_" ? 4
                 : s == "add_" ? 5 : s == "add_bcast_col" ? 6 : -1;
    if (op < 0) return fail(TSN_ERR_UNSUPPORTED, "elementwise " + s);
    float * xin = (float *) (op == 0 || op == 4 ? a : nullptr);
    k_unary<<<nblk((long long) n), 256, 0, c.stream>>>(op, xin, (const float *) a, (const float *) b, (float *) y, (long long) n, h ? h : 1);
    return launched(name);
}

int compat_cfg_euler(DeviceCtx & c, const void * fc, const void * fu, void * x, size_t n, float cfg, float dt) {
    CD p{cfg, dt, (uint32_t) n};
    k_cfg_euler<<<nblk((long long) n), 256, 0, c.stream>>>((const float *) fc, (const float *) fu, (float *) x, p);
    return launched("cfg_euler");
}

int compat_mean_cols(DeviceCtx & c, const void * x, void * y, uint32_t S, uint32_t H) {
    SH p{S, H};
    k_mean_cols<<<nblk(H), 256, 0, c.stream>>>((const float *) x, (float *) y, p);
    return launched("mean_cols");
}

int compat_dispatch(DeviceCtx & c, const char * name_c, const uint32_t grid[3], const uint32_t block[3],
                    const void * const * b, int nb, const void * params, size_t np) {
    const std::string name(name_c);
    const uint32_t gx = grid ? grid[0] : 1, gy = grid ? grid[1] : 1, gz = grid ? grid[2] : 1;
    const uint32_t tx = block ? block[0] : 1, ty = block ? block[1] : 1, tz = block ? block[2] : 1;
    const long long threads = (long long) gx * gy * gz * tx * ty * tz;
    auto B = [&](int i) { return i < nb ? (void *) b[i] : nullptr; };
    auto F = [&](int i) { return (float *) B(i); };
    uint32_t n1 = 0;
    auto short_params = [&]() { return fail(TSN_ERR_ARG, "short constant block for " + name); };
    if (name.rfind("gemm_mpp_h", 0) == 0 || name == "gemm_h" || name == "gemm_mpp_f" || name == "gemm_f") {
        GemmP p; if (!get(params, np, p)) return short_params();
        const int wf16 = name.find("_f") == std::string::npos || name.rfind("gemm_mpp_h", 0) == 0 ? 1 : 0;
        return compat_gemm(c, wf16, B(0), B(1), B(2), p.bias_mode ? B(3) : nullptr, p.M, p.N, p.K, p.ldx, p.ldw, p.ldy);
    }
    if (name == "gemv_h" || name == "gemv_f") {
        GemmP p; if (!get(params, np, p)) return short_params();
        k_gemv<<<(p.N + 7) / 8, 256, 0, c.stream>>>(B(0), name == "gemv_h", F(1), F(2), F(3), p);
        return launched(name_c);
    }
    if (name == "attn_qk") {
        AttnP p; if (!get(params, np, p)) return short_params();
        k_attn_qk<<<nblk((long long) p.nh * p.Sq * p.Sk), 256, 0, c.stream>>>(F(0), F(1), (const int *) B(2), F(3), p);
        return launched(name_c);
    }
    if (name == "softmax_rows") {
        AttnP p; if (!get(params, np, p)) return short_params();
        k_softmax_rows<<<(p.nh * p.Sq + 7) / 8, 256, 0, c.stream>>>(F(0), p);
        return launched(name_c);
    }
    if (name == "attn_pav") {
        AttnP p; if (!get(params, np, p)) return short_params();
        k_attn_pav<<<nblk((long long) p.nh * p.Sq * p.hd), 256, 0, c.stream>>>(F(0), F(1), F(2), p);
        return launched(name_c);
    }
    if (name == "im2col") {
        IcP p; if (!get(params, np, p)) return short_params();
        k_im2col<<<nblk((long long) p.rows * p.IC * p.K), 256, 0, c.stream>>>(F(0), F(1), p, threads);
        return launched(name_c);
    }
    if (name == "conv1d_fwd" || name == "conv1d_fwd_f") {
        ConvP p; if (!get(params, np, p)) return short_params();
        k_conv1d<<<nblk((long long) p.OL * p.OC), 256, 0, c.stream>>>(F(0), B(1), name == "conv1d_fwd", F(2), F(3), p);
        return launched(name_c);
    }
    if (name == "adaln_ln") {
        AD p; if (!get(params, np, p)) return short_params();
        const uint32_t rows = gx * tx;
        k_rownorm<<<(rows + 7) / 8, 256, 0, c.stream>>>(3, F(0), F(2), nullptr, nullptr, F(1), p.H, p.eps, p.per_row, p.chunks, p.base, rows);
        return launched(name_c);
    }
    if (name == "ln_plain" || name == "ln_wb" || name == "rms_w") {
        HE p; if (!get(params, np, p)) return short_params();
        const uint32_t rows = gx * tx;
        const int mode = name == "ln_plain" ? 0 : name == "ln_wb" ? 1 : 2;
        k_rownorm<<<(rows + 7) / 8, 256, 0, c.stream>>>(mode, F(0), F(1), F(2), F(3), nullptr, p.H, p.eps, 0, 0, 0, rows);
        return launched(name_c);
    }
    if (name == "gate_add") {
        GA p; if (!get(params, np, p)) return short_params();
        k_gate_add<<<nblk(threads), 256, 0, c.stream>>>(F(0), F(1), F(2), F(3), p, threads);
        return launched(name_c);
    }
    if (name == "rms_head") {
        RH p; if (!get(params, np, p)) return short_params();
        k_rms_head<<<nblk((long long) gx * tx * gy * ty), 256, 0, c.stream>>>(F(0), F(1), p, gx * tx, gy * ty);
        return launched(name_c);
    }
    if (name == "rope_pairs") {
        RP p; if (!get(params, np, p)) return short_params();
        k_rope<<<nblk((long long) gx * tx * gy * ty), 256, 0, c.stream>>>(F(0), (const int *) B(1), p, gx * tx, gy * ty);
        return launched(name_c);
    }
    if (name == "qkv_split3") {
        QS3 p; if (!get(params, np, p)) return short_params();
        k_qkv_split3<<<nblk((long long) gy * ty * p.H), 256, 0, c.stream>>>(F(0), F(1), p, gy * ty);
        return launched(name_c);
    }
    if (name == "mean_cols") { SH p; if (!get(params, np, p)) return short_params(); return compat_mean_cols(c, B(0), B(1), p.S, p.H); }
    if (name == "cfg_euler") { CD p; if (!get(params, np, p)) return short_params(); return compat_cfg_euler(c, B(0), B(1), B(2), p.n, p.cfg, p.dt); }
    if (name == "snake_") {
        SH p; if (!get(params, np, p)) return short_params();
        k_snake<<<nblk((long long) p.S * p.H), 256, 0, c.stream>>>(F(0), F(1), F(2), p);
        return launched(name_c);
    }
    if (name == "add_bcast_col") {
        CH p; if (!get(params, np, p)) return short_params();
        return compat_elementwise(c, "add_bcast_col", B(0), B(1), B(2), p.n, p.H, 0);
    }
    if (name == "silu_" || name == "gelu_quick_") {
        if (!get(params, np, n1)) return short_params();
        return compat_elementwise(c, name_c, B(0), nullptr, nullptr, n1, 0, 0);
    }
    if (name == "copy_") { if (!get(params, np, n1)) return short_params(); return compat_elementwise(c, name_c, B(0), nullptr, B(1), n1, 0, 0); }
    if (name == "swiglu_" || name == "geglu_" || name == "add_") {
        if (!get(params, np, n1)) return short_params();
        return compat_elementwise(c, name_c, B(0), B(1), B(2), n1, 0, 0);
    }
    return fail(TSN_ERR_UNSUPPORTED, "kernel " + name + " not provided");
}

} // namespace tsn
