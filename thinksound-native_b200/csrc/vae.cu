// vae.cu — the VAE decoder (VaeModel::decode, src/vae.cpp:17-86) on the GPU.
//
// The reference runs every conv as im2col + an f32-weight GEMM, transposed convs on a zero-stuffed
// input, and the snake activations and residual adds as separate passes over [T, C] buffers. Here:
//   * every conv is the tcgen05 implicit-GEMM (gemm_ws_kernel): TMA views of the [T, IC] split-f16
//     activations shifted by tap * dilation - pad (zero fill outside [0, T) is the conv padding);
//     the f32 weights are split into f16 hi + lo halves at load, and each K step issues
//     A_hi·W_hi + A_lo·W_hi + A_hi·W_lo, so the product follows the f32 weights to ~2^-22
//     (f16-rounded weights alone move the decoded audio by ~1.3e-3 rel-L2);
//   * a transposed conv of stride s runs as s stride-1 convs over the un-stuffed input (output
//     phase p = t mod s meets only the taps k = r_p + s j, r_p = (pad - p) mod s), written into
//     every s-th output row: no multiply by the stuffed zeros;
//   * the snake after each dilated conv is that GEMM's epilogue (EPI_F16_SNAKE); the snake before
//     a conv, with the residual add of the previous unit, is one elementwise pass writing the next
//     GEMM's split operand (vae_snake_kernel).
// The whole decode for a latent length is one CUDA graph.
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include "../../include/tsn_synth.h"
#include "gguf_io.h"
#include "kernels.h"
#include "runtime.h"

namespace tsn {

namespace {

#define VCK(expr)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) return fail(TSN_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define VRT(call) do { int rc_ = (call); if (rc_) return rc_; } while (0)

// One conv as split-weight implicit GEMMs: `phases` weight sets (s for a transposed conv of stride
// s, else 1), each [Npad][taps * IC] f16 hi, then the lo halves of all phases.
struct VConv {
    __half * w = nullptr;          // hi halves of every phase, then lo halves
    float * b = nullptr;           // [OC] or null
    int OC = 0, IC = 0, taps = 1, phases = 1, Npad = 0, dil = 1;
    int pad[8] = {0};              // per phase: the GEMM's left padding (negative: a right shift)
    size_t phase_elems() const { return (size_t) Npad * taps * IC; }
    const __half * hi(int p) const { return w + (size_t) p * phase_elems(); }
    const __half * lo(int p) const { return w + (size_t) (phases + p) * phase_elems(); }
};

struct VSnake { float * ea = nullptr, * eb = nullptr; int C = 0; };   // e^alpha, e^-beta per channel

// f32 tensor values of the VAE GGUF (mmap'd file, or the seeded synthetic values)
struct VSource {
    Gguf file;
    bool synthetic = false;
    VaeGeom geom;
    uint64_t seed = 0;
    std::map<std::string, TensorSpec> specs;
    int get(const std::string & name, std::vector<float> & out, std::vector<uint64_t> & ne) {
        if (synthetic) {
            auto it = specs.find(name);
            if (it == specs.end()) return fail(TSN_ERR_MISSING, "missing tensor " + name);
            const TensorSpec & s = it->second;
            out.resize(s.nelem());
            synth_fill_host(s, seed, out.data());
            ne.assign(s.ne, s.ne + s.n_dims);
            return TSN_OK;
        }
        const GgufTensorInfo * t = file.find(name);
        if (!t) return fail(TSN_ERR_MISSING, "missing tensor " + name);
        ne.assign(t->ne, t->ne + t->n_dims);
        out.resize(t->nelem());
        if (t->type == GG_F32) std::memcpy(out.data(), t->data, out.size() * 4);
        else if (t->type == GG_F16)
            for (size_t i = 0; i < out.size(); ++i) out[i] = tsn_f16_to_f32(((const uint16_t *) t->data)[i]);
        else if (t->type == GG_BF16)
            for (size_t i = 0; i < out.size(); ++i) out[i] = tsn_bf16_to_f32(((const uint16_t *) t->data)[i]);
        else return fail(TSN_ERR_MISSING, "tensor " + name + " has an unsupported type");
        return TSN_OK;
    }
};

// split an f32 value into f16 hi + lo (hi = f16(w), lo = f16(w - hi))
inline void split16(float w, uint16_t & hi, uint16_t & lo) {
    hi = tsn_ref_f32_to_f16(w);
    lo = tsn_ref_f32_to_f16(w - tsn_f16_to_f32(hi));
}

} // namespace

// ----------------------------------------------------------------------------- elementwise
// h = split f16 of snake(x + g) (snake_, shaders/ops_conv.metal:204-213; identity when ea is
// null), optionally writing x + g back to xo (the residual add, src/vae.cpp:75). h holds the hi
// halves [rows][C] followed by the lo halves.
__global__ void __launch_bounds__(256) vae_snake_kernel(const float * x, const float * g, float * xo, const float * ea,
                                                        const float * eb, __half * h, long long rows, int C) {
    pdl_trigger();
    pdl_wait();
    const long long n4 = rows * C / 4, lo = rows * C;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n4; i += (long long) gridDim.x * blockDim.x) {
        float4 v = ((const float4 *) x)[i];
        if (g) {
            const float4 d = ((const float4 *) g)[i];
            v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
        }
        if (xo) ((float4 *) xo)[i] = v;
        float y[4] = {v.x, v.y, v.z, v.w};
        if (ea) {
            const int c = (int) ((i * 4) % C);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float s = __sinf(y[e] * ea[c + e]);
                y[e] = y[e] + s * s * eb[c + e];
            }
        }
        __align__(8) __half hv[4], lv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            hv[e] = __float2half_rn(y[e]);
            lv[e] = __float2half_rn(y[e] - __half2float(hv[e]));
        }
        *(uint2 *) (h + i * 4) = *(const uint2 *) hv;
        *(uint2 *) (h + lo + i * 4) = *(const uint2 *) lv;
    }
}

struct VaeModel {
    DeviceCtx * dev = nullptr;
    VaeGeom g;
    VConv conv0, convT[5], c7[5][3], c1[5][3], fin;
    VSnake s_in[5], s_a[5][3], s_b[5][3], s_fin;
    std::vector<void *> weights;
    // per latent length
    int T = 0;
    size_t max_elems = 0;
    float * lat = nullptr, * x = nullptr, * audio = nullptr;
    __half * lat16 = nullptr, * hA = nullptr, * hB = nullptr, * hC = nullptr;   // split operands, rotated
    std::vector<void *> bufs;
    std::vector<std::function<cudaError_t(cudaStream_t)>> ops;
    std::vector<std::string> op_names;
    cudaGraphExec_t gx = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    double last_ms = 0.0;
    double flops = 0.0;   // algorithmic 2·M·N·K of every conv of the prepared length

    ~VaeModel() {
        if (dev) dev->activate();
        release();
        for (void * p : weights) cudaFree(p);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
    }
    void release() {
        if (gx) { cudaGraphExecDestroy(gx); gx = nullptr; }
        for (void * p : bufs) cudaFree(p);
        bufs.clear();
        T = 0;
    }
    template <typename P> int dalloc(P ** p, size_t bytes, std::vector<void *> & list) {
        void * q = nullptr;
        VCK(cudaMalloc(&q, std::max<size_t>(bytes, 16)));
        list.push_back(q);
        *p = (P *) q;
        return TSN_OK;
    }
    template <typename V> int upload(V ** dst, const std::vector<V> & src) {
        VRT(dalloc(dst, src.size() * sizeof(V), weights));
        VCK(cudaMemcpy(*dst, src.data(), src.size() * sizeof(V), cudaMemcpyHostToDevice));
        return TSN_OK;
    }
    int load_snake(VSource & src, const std::string & p, VSnake & s) {
        std::vector<float> a, b;
        std::vector<uint64_t> ne;
        VRT(src.get(p + ".alpha", a, ne));
        VRT(src.get(p + ".beta", b, ne));
        if (a.size() != b.size()) return fail(TSN_ERR_MISSING, p + ": alpha/beta sizes differ");
        std::vector<float> ea(a.size()), eb(a.size());
        for (size_t i = 0; i < a.size(); ++i) { ea[i] = (float) std::exp((double) a[i]); eb[i] = (float) std::exp(-(double) b[i]); }
        s.C = (int) a.size();
        VRT(upload(&s.ea, ea));
        return upload(&s.eb, eb);
    }
    // conv weight ne = {K, IC, OC} (w[oc][ic][k]) -> split GEMM weights [Npad][taps * IC], tap-major
    // K. A transposed conv of stride s (the converted kernel the reference applies to the stuffed
    // input, src/vae.cpp:65-66, shaders/ops_conv.metal:273-276) becomes s phase convs of K/s taps.
    int load_conv(VSource & src, const std::string & p, bool bias, int stride, int pad, int dil, VConv & cv) {
        std::vector<float> w, b;
        std::vector<uint64_t> ne;
        VRT(src.get(p + ".weight", w, ne));
        if (ne.size() != 3) return fail(TSN_ERR_MISSING, p + ": expected a 3-D conv weight");
        const int K = (int) ne[0], IC = (int) ne[1], OC = (int) ne[2];
        if (IC % 64) return fail(TSN_ERR_UNSUPPORTED, p + ": input channels must be a multiple of 64");
        cv.OC = OC; cv.IC = IC; cv.dil = dil;
        cv.Npad = OC < 64 ? 64 : OC;
        if (OC >= 64 && OC % 64) return fail(TSN_ERR_UNSUPPORTED, p + ": output channels must be a multiple of 64");
        cv.phases = stride;
        if (stride > 1) {
            if (K % stride || stride > 8) return fail(TSN_ERR_UNSUPPORTED, p + ": transposed conv kernel not a multiple of its stride");
            cv.taps = K / stride;
        } else {
            cv.taps = K;
        }
        const size_t pe = cv.phase_elems();
        std::vector<uint16_t> hw(2 * pe * cv.phases, 0);
        for (int ph = 0; ph < cv.phases; ++ph) {
            int r = 0;
            if (stride > 1) {
                r = ((pad - ph) % stride + stride) % stride;   // the taps k = r + s j meet phase ph
                cv.pad[ph] = -((ph - pad + r) / stride);       // output row s q + ph reads q + c + j
            } else {
                cv.pad[ph] = pad;
            }
            uint16_t * hi = hw.data() + (size_t) ph * pe, * lo = hw.data() + (size_t) (cv.phases + ph) * pe;
            for (int n = 0; n < OC; ++n)
                for (int j = 0; j < cv.taps; ++j) {
                    const int k = stride > 1 ? r + stride * j : j;
                    for (int ic = 0; ic < IC; ++ic) {
                        const size_t o = ((size_t) n * cv.taps + j) * IC + ic;
                        split16(w[((size_t) n * IC + ic) * K + k], hi[o], lo[o]);
                    }
                }
        }
        VRT(dalloc(&cv.w, hw.size() * 2, weights));
        VCK(cudaMemcpy(cv.w, hw.data(), hw.size() * 2, cudaMemcpyHostToDevice));
        if (bias) {
            VRT(src.get(p + ".bias", b, ne));
            if ((int) b.size() != OC) return fail(TSN_ERR_MISSING, p + ": bias size");
            VRT(upload(&cv.b, b));
        }
        return TSN_OK;
    }

    int load(VSource & src) {
        VRT(load_conv(src, "decoder.layers.0", true, 1, 3, 1, conv0));                 // src/vae.cpp:59
        g.latent_dim = (uint32_t) conv0.IC;
        for (int n = 0; n < 5; ++n) {                                                   // src/vae.cpp:61-78
            const std::string bp = "decoder.layers." + std::to_string(n + 1);
            const int s = (int) VAE_STRIDES[n];
            VRT(load_snake(src, bp + ".layers.0", s_in[n]));
            std::vector<float> tmp;
            std::vector<uint64_t> ne;
            VRT(src.get(bp + ".layers.1.weight", tmp, ne));
            const int K = (int) ne[0];
            VRT(load_conv(src, bp + ".layers.1", true, s, K - 1 - s / 2, 1, convT[n]));
            for (int r = 0; r < 3; ++r) {
                const std::string rp = bp + ".layers." + std::to_string(r + 2);
                const int d = (int) VAE_DILS[r];
                VRT(load_snake(src, rp + ".layers.0", s_a[n][r]));
                VRT(load_conv(src, rp + ".layers.1", true, 1, 3 * d, d, c7[n][r]));
                VRT(load_snake(src, rp + ".layers.2", s_b[n][r]));
                VRT(load_conv(src, rp + ".layers.3", true, 1, 0, 1, c1[n][r]));
            }
        }
        VRT(load_snake(src, "decoder.layers.6", s_fin));                              // src/vae.cpp:80-81
        VRT(load_conv(src, "decoder.layers.7", false, 1, 3, 1, fin));
        g.out_channels = (uint32_t) fin.OC;
        if (fin.OC > 32) return fail(TSN_ERR_UNSUPPORTED, "more than 32 output channels");
        g.channels = (uint32_t) fin.IC;
        // chain checks: every conv reads the channels the previous one wrote
        int c = conv0.OC;
        for (int n = 0; n < 5; ++n) {
            if (convT[n].IC != c || s_in[n].C != c) return fail(TSN_ERR_MISSING, "VAE block widths do not chain");
            c = convT[n].OC;
            for (int r = 0; r < 3; ++r)
                if (c7[n][r].IC != c || c7[n][r].OC != c || c1[n][r].IC != c || c1[n][r].OC != c || s_a[n][r].C != c ||
                    s_b[n][r].C != c)
                    return fail(TSN_ERR_MISSING, "VAE residual unit widths do not chain");
        }
        if (fin.IC != c || s_fin.C != c) return fail(TSN_ERR_MISSING, "VAE final conv width");
        VCK(cudaEventCreate(&e0));
        VCK(cudaEventCreate(&e1));
        return TSN_OK;
    }

    // one phase of a conv as a split-weight GEMM over `rows` input rows of the split operand A
    // ([rows][IC] hi, then lo): tile width and K slices by the cost model of the DiT planner
    int conv_op(const std::string & name, const VConv & cv, int ph, const __half * A, int rows, void * out, long long ldo,
                int epi, const VSnake * snake, long long out_lo, void * out2 = nullptr, long long ldo2 = 0,
                long long out2_lo = 0) {
        const int kb = cv.taps * cv.IC / 64, mtt = (rows + 127) / 128;
        double best = 1e30;
        int bn = 0, sp = 1;
        for (int cb : {256, 128, 64}) {
            if (cv.Npad % cb) continue;
            const double kcost = cb == 256 ? 1.1 : cb == 128 ? 0.6 : 0.45;   // three UMMAs per K step
            const int tiles = mtt * (cv.Npad / cb);
            for (int s = 1; s <= 8 && s <= kb; ++s) {
                const int kbps = (kb + s - 1) / s;
                if ((kb + kbps - 1) / kbps != s) continue;
                const int cap = gemm_ws_capacity(cb, epi, s);
                if (cap <= 0) continue;
                const int waves = (tiles * s + cap - 1) / cap;
                const double cost = waves * (kbps * kcost + 1.5) + (s > 1 ? 1.5 * waves : 0.0);
                if (cost < best - 1e-9) { best = cost; bn = cb; sp = s; }
            }
        }
        if (!bn) return fail(TSN_ERR_ARG, name + ": no tile fits");
        GemmLaunch gl{};
        gl.bn = bn; gl.epi = epi; gl.split = true; gl.ab_bf16 = 0;
        gl.smem = gemm_ws_smem_bytes(bn, epi);
        gl.grid = dim3(mtt, cv.Npad / bn, sp);
        if (!make_act_map(&gl.ta, A, cv.IC, rows, 1, 128, 1, 0) ||
            !make_act_map(&gl.ta2, A + (size_t) rows * cv.IC, cv.IC, rows, 1, 128, 1, 0) ||
            !make_w_map(&gl.tb, cv.hi(ph), (uint64_t) cv.taps * cv.IC, cv.Npad, bn, 0) ||
            !make_w_map(&gl.tb2, cv.lo(ph), (uint64_t) cv.taps * cv.IC, cv.Npad, bn, 0))
            return fail(TSN_ERR_CUDA, name + ": tensor map encode failed");
        GemmArgs & a = gl.args;
        a.rows = rows; a.B = 1; a.bt = 128; a.bb = 1; a.m_tiles_t = mtt; a.N = cv.OC;
        a.k_blocks = kb; a.ic_blocks = cv.IC / 64; a.pad = cv.pad[ph]; a.dil = cv.dil;
        a.splits = sp; a.kb_per_split = (kb + sp - 1) / sp;
        a.err = dev->d_err;
        a.bias = cv.b;
        a.out = out; a.ldo = ldo; a.out_bs = 0; a.out_lo = out_lo;
        a.out2 = out2; a.ldo2 = ldo2; a.out2_lo = out2_lo;
        a.m_fast = 1;
        if (snake) { a.snake_a = snake->ea; a.snake_b = snake->eb; }
        // many waves of tiles: one persistent CTA per SM overlaps each tile's epilogue (the fused
        // residual and snake passes) with the next tile's mainloop
        const int tiles = mtt * (cv.Npad / bn);
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev->ordinal);
        if (sp == 1 && tiles > 2 * sms) {
            gl.persistent = true;
            gl.smem = gemm_ws_persistent_smem_bytes(bn, epi);
            gl.grid = dim3((unsigned) std::min(tiles, sms), 1, 1);
        }
        ops.push_back([gl](cudaStream_t s) { return launch_gemm_ws(gl, s); });
        op_names.push_back(name);
        flops += 2.0 * rows * (double) cv.OC * cv.taps * cv.IC;
        return TSN_OK;
    }
    void snake_op(const float * xin, const float * gin, float * xo, const VSnake * sn, __half * out, long long rows, int C) {
        const float * ea = sn ? sn->ea : nullptr, * eb = sn ? sn->eb : nullptr;
        const long long n4 = rows * C / 4;
        const unsigned blocks = (unsigned) std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 148 * 16));
        ops.push_back([=](cudaStream_t s) {
            return launch_ex(vae_snake_kernel, dim3(blocks), dim3(256), 0, s, 1u, xin, gin, xo, ea, eb, out, rows, C);
        });
        op_names.push_back("snake");
    }

    int prepare(int T_) {
        release();
        ops.clear();
        op_names.clear();
        flops = 0.0;
        // largest [rows][C] of any stage
        long long t = T_, mx = (long long) T_ * conv0.OC;
        for (int n = 0; n < 5; ++n) {
            t *= VAE_STRIDES[n];
            mx = std::max(mx, t * convT[n].OC);
        }
        const long long Ta = t;
        max_elems = (size_t) mx;
        VRT(dalloc(&lat, (size_t) T_ * conv0.IC * 4, bufs));
        VRT(dalloc(&lat16, (size_t) T_ * conv0.IC * 2 * 2, bufs));
        VRT(dalloc(&x, max_elems * 4, bufs));
        VRT(dalloc(&hA, max_elems * 2 * 2, bufs));
        VRT(dalloc(&hB, max_elems * 2 * 2, bufs));
        VRT(dalloc(&hC, max_elems * 2 * 2, bufs));
        VRT(dalloc(&audio, (size_t) Ta * 32 * 4, bufs));
        // VaeModel::decode, src/vae.cpp:57-81. Every snake except the latent split is a GEMM
        // epilogue: conv0 writes the first block's snake; each transposed conv writes x and the
        // first unit's snake; each unit's dilated conv applies its inner snake, and its k1 conv adds
        // the residual into x and writes the snake that follows (the next unit's, the next
        // block's, or the final one). hC feeds transposed convs and the final conv, hA dilated
        // convs, hB k1 convs, so no launch reads the buffer it writes.
        snake_op(lat, nullptr, nullptr, nullptr, lat16, T_, conv0.IC);
        VRT(conv_op("conv0", conv0, 0, lat16, T_, hC, conv0.OC, EPI_F16_SNAKE, &s_in[0], (long long) T_ * conv0.OC));
        long long rows = T_;
        for (int n = 0; n < 5; ++n) {
            const int s = (int) VAE_STRIDES[n], C = convT[n].OC;
            const long long out_rows = rows * s;
            for (int ph = 0; ph < s; ++ph)
                VRT(conv_op("convT" + std::to_string(n), convT[n], ph, hC, (int) rows, x + (size_t) ph * C, (long long) s * C,
                            EPI_F32_SNAKE2, &s_a[n][0], 0, hA + (size_t) ph * C, (long long) s * C, out_rows * C));
            rows = out_rows;
            for (int r = 0; r < 3; ++r) {
                const std::string nm = "res" + std::to_string(n) + std::to_string(r);
                const VSnake * next = r < 2 ? &s_a[n][r + 1] : n < 4 ? &s_in[n + 1] : &s_fin;
                __half * hn = r < 2 ? hA : hC;
                VRT(conv_op(nm + ".conv7", c7[n][r], 0, hA, (int) rows, hB, C, EPI_F16_SNAKE, &s_b[n][r], rows * C));
                VRT(conv_op(nm + ".conv1", c1[n][r], 0, hB, (int) rows, x, C, EPI_RESID_SNAKE, next, 0, hn, C, rows * C));
            }
        }
        VRT(conv_op("final", fin, 0, hC, (int) rows, audio, 32, EPI_F32, nullptr, 0));
        T = T_;
        // capture
        cudaGraph_t graph = nullptr;
        VCK(cudaStreamBeginCapture(dev->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = cudaSuccess;
        for (size_t i = 0; i < ops.size() && e == cudaSuccess; ++i) e = ops[i](dev->stream);
        cudaError_t e2 = cudaStreamEndCapture(dev->stream, &graph);
        if (e != cudaSuccess || e2 != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            return fail(TSN_ERR_CUDA, std::string("VAE graph capture: ") + cudaGetErrorString(e != cudaSuccess ? e : e2));
        }
        e = cudaGraphInstantiate(&gx, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("VAE graph instantiate: ") + cudaGetErrorString(e));
        return TSN_OK;
    }

    // the prepared decode eagerly, one line per launch: index, name, device ms
    int profile(std::string & rep) {
        if (!T) return fail(TSN_ERR_STATE, "decode once before profiling");
        std::vector<cudaEvent_t> ev(ops.size() + 1);
        for (auto & e : ev) VCK(cudaEventCreate(&e));
        VCK(cudaEventRecord(ev[0], dev->stream));
        for (size_t i = 0; i < ops.size(); ++i) {
            VCK(ops[i](dev->stream));
            VCK(cudaEventRecord(ev[i + 1], dev->stream));
        }
        int rc = dev->sync();
        char line[160];
        for (size_t i = 0; !rc && i < ops.size(); ++i) {
            float ms = 0;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            snprintf(line, sizeof line, "%4zu %-16s %8.4f ms\n", i, op_names[i].c_str(), ms);
            rep += line;
        }
        for (auto & e : ev) cudaEventDestroy(e);
        return rc;
    }

    long long audio_len(int T_) const {
        long long t = T_;
        for (int n = 0; n < 5; ++n) t *= VAE_STRIDES[n];
        return t;
    }

    // latent [T, latent_dim] and audio [T_audio, out_channels], host or device memory
    int decode(const float * latent, int T_, float * out, size_t out_cap, uint32_t * T_audio) {
        if (T_ < 1) return fail(TSN_ERR_ARG, "latent length must be positive");
        const long long Ta = audio_len(T_);
        if (T_audio) *T_audio = (uint32_t) Ta;
        if (!out || out_cap < (size_t) Ta * g.out_channels) return fail(TSN_ERR_ARG, "audio buffer too small");
        if (T_ != T) VRT(prepare(T_));
        VCK(cudaMemcpyAsync(lat, latent, (size_t) T_ * conv0.IC * 4, cudaMemcpyDefault, dev->stream));
        VCK(cudaEventRecord(e0, dev->stream));
        VCK(cudaGraphLaunch(gx, dev->stream));
        VCK(cudaEventRecord(e1, dev->stream));
        VCK(cudaMemcpy2DAsync(out, (size_t) g.out_channels * 4, audio, 32 * 4, (size_t) g.out_channels * 4, (size_t) Ta,
                              cudaMemcpyDefault, dev->stream));
        VRT(dev->sync());
        float ms = 0;
        VCK(cudaEventElapsedTime(&ms, e0, e1));
        last_ms = ms;
        return TSN_OK;
    }
};

} // namespace tsn

// ------------------------------------------------------------------------------- C ABI
struct tsn_vae { tsn::VaeModel m; };

using namespace tsn;

namespace {
int new_vae(tsn_device * dev, VSource & src, tsn_vae ** out) {
    if (!dev || !out) return fail(TSN_ERR_ARG, "null argument");
    *out = nullptr;
    VRT(dev->ctx.activate());
    std::unique_ptr<tsn_vae> v(new tsn_vae);
    v->m.dev = &dev->ctx;
    VRT(v->m.load(src));
    *out = v.release();
    return TSN_OK;
}
} // namespace

extern "C" {

int tsn_vae_load(tsn_device * dev, const char * gguf_path, tsn_vae ** out) {
    if (!gguf_path) return fail(TSN_ERR_ARG, "null path");
    VSource src;
    std::string err;
    if (!src.file.open(gguf_path, err)) return fail(TSN_ERR_IO, err);
    return new_vae(dev, src, out);
}

int tsn_vae_load_synthetic(tsn_device * dev, uint32_t latent_dim, uint32_t channels, uint32_t out_channels, uint64_t seed,
                           tsn_vae ** out) {
    if (!latent_dim || !channels || !out_channels) return fail(TSN_ERR_ARG, "bad VAE geometry");
    VSource src;
    src.synthetic = true;
    src.geom.latent_dim = latent_dim; src.geom.channels = channels; src.geom.out_channels = out_channels;
    src.seed = seed;
    for (const TensorSpec & s : vae_schema(src.geom)) src.specs[s.name] = s;
    return new_vae(dev, src, out);
}

int tsn_vae_decode(tsn_vae * v, const float * latent, uint32_t T, float * audio, size_t audio_cap, uint32_t * T_audio) {
    if (!v || !latent) return fail(TSN_ERR_ARG, "null argument");
    VRT(v->m.dev->activate());
    return v->m.decode(latent, (int) T, audio, audio_cap, T_audio);
}

double tsn_vae_last_ms(tsn_vae * v) { return v ? v->m.last_ms : 0.0; }

int tsn_vae_profile_ops(tsn_vae * v, char * out, size_t cap) {
    if (!v) return fail(TSN_ERR_ARG, "null argument");
    VRT(v->m.dev->activate());
    std::string rep;
    VRT(v->m.profile(rep));
    if (out && cap) { std::strncpy(out, rep.c_str(), cap - 1); out[cap - 1] = 0; }
    return TSN_OK;
}
double tsn_vae_flops(tsn_vae * v) { return v ? v->m.flops : 0.0; }
int tsn_vae_launches(tsn_vae * v) { return v ? (int) v->m.ops.size() : 0; }

int tsn_vae_free(tsn_vae * v) {
    if (v) { if (v->m.dev) cudaStreamSynchronize(v->m.dev->stream); delete v; }
    return TSN_OK;
}

} // extern "C"
