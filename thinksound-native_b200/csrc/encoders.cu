// encoders.cu — the two text encoders on the GPU: T5 v1.1 (T5Model::encode, src/t5.cpp:84-131)
// and MetaCLIP text (ClipModel::encode, src/clip.cpp:30-101).
//
// The reference runs each layer as separate q, k and v GEMMs into a [77, 3H] buffer, an attention
// that writes the f32 score tensor [NH, 77, 77] to memory three times (attn_qk, softmax_rows,
// attn_pav, shaders/gemm_attn.metal:96-202), then o/out GEMM + add_, norm, the FFN GEMMs, an
// activation pass and add_ again: 13 dispatches per layer, every activation in f32 through memory.
// Here a layer is seven launches:
//   norm    the previous GEMM's split-K partial sums (+ bias) added into the residual stream x,
//           then RMSNorm (T5) or LayerNorm (CLIP) written as the next GEMM's split f16 operand
//   qkv     one GEMM over [q | k | v] weights concatenated at load, whose epilogue scatters q, k, v
//           head-major as split f16 (EPI_QKV without the DiT's per-head norm and RoPE)
//   attn    the tcgen05 short-sequence attention (attn_short_kernel) with an additive logit-bias
//           table: T5's relative-position bias and pad mask, or CLIP's causal + EOT mask, built once
//           per encode from the token ids; no score tensor in memory
//   o/out   GEMM whose K slices write partial tiles; the next norm adds them (and the bias)
//   norm
//   up      T5: wi_0 / wi_1 interleaved in 32-row groups, one GEMM whose epilogue applies
//           gelu_tanh(a)·b (EPI_GEGLU); CLIP: fc1 + bias with gelu_quick in the epilogue
//   down    wo / fc2 as partial tiles
// Weights follow the reference's device types (WeightSet::load with keep_f32, src/net.mm:126-173):
// tensors stored as f32 in the file stay f32 and run as split-weight GEMMs (f16 hi + lo, three
// UMMAs per K step); any other type (the T5 file's Q8_0) becomes f16 by the reference's rounding
// rule. Activations are split f16 operands (~2^-22), so the GEMMs follow the f32 arithmetic.
// One CUDA graph per encoder.
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <thread>
#include <vector>

#include "../../include/tsn_synth.h"
#include "gguf_io.h"
#include "kernels.h"
#include "runtime.h"

namespace tsn {

namespace {

#define ECK(expr)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) return fail(TSN_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define ERT(call) do { int rc_ = (call); if (rc_) return rc_; } while (0)

constexpr float LOG2E = 1.4426950408889634f;

// T5's relative-position bucket (src/t5.cpp:7-20): bidirectional, half the buckets per sign, exact
// below max_exact = buckets/4, logarithmic up to max_dist. Host only, in double like the reference.
int t5_bucket(int rel, int num_buckets, int max_dist) {
    int ret = 0;
    num_buckets /= 2;
    if (rel > 0) ret += num_buckets;
    const int n = rel < 0 ? -rel : rel;
    const int max_exact = num_buckets / 2;
    if (n < max_exact) return ret + n;
    const int v = max_exact + (int) (std::log((double) n / max_exact) / std::log((double) max_dist / max_exact) *
                                     (num_buckets - max_exact));
    return ret + std::min(v, num_buckets - 1);
}

} // namespace

// ----------------------------------------------------------------------------------- kernels
// x[s][:] = tok[ids[s]][:] (+ pos[s][:]): the host-side embedding gathers of src/t5.cpp:92-98 and
// src/clip.cpp:33-40, from the device copy of the table.
__global__ void __launch_bounds__(256) enc_embed_kernel(const int * ids, const float * tok, const float * pos, float * x,
                                                        int n, int d) {
    pdl_trigger();
    pdl_wait();
    const long long n4 = (long long) n * d / 4;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n4; i += (long long) gridDim.x * blockDim.x) {
        const int s = (int) (i * 4 / d), c = (int) (i * 4 % d);
        float4 v = *(const float4 *) (tok + (size_t) ids[s] * d + c);
        if (pos) {
            const float4 p = *(const float4 *) (pos + (size_t) s * d + c);
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        ((float4 *) x)[i] = v;
    }
}

// Logit-bias table lb[h][q][k] (log2 units, [NH][n][S_pad]) of one encode. grid (n, NH), S_pad
// threads. mode 1 (T5, attn_qk bias_mode 1 with pad_on, shaders/gemm_attn.metal:131-136): key k
// masked where ids[k] == 0, else rel_bias[bucket[q][k]][h]. mode 2 (CLIP, bias_mode 2 :137-138):
// key k allowed iff k <= q and k <= eot, eot the first position of the largest id
// (src/clip.cpp:42-43), which block (0, 0) also stores for the pooled projection.
__global__ void enc_lbias_kernel(const int * ids, const int * bkt, const float * rb, float * lb, int * eot_out, int n,
                                 int S_pad, int NH, int mode) {
    pdl_trigger();
    pdl_wait();
    const int q = blockIdx.x, h = blockIdx.y, k = threadIdx.x;
    __shared__ int eot;
    if (mode == 2 && threadIdx.x == 0) {
        int e = 0, mx = ids[0];
        for (int i = 1; i < n; ++i)
            if (ids[i] > mx) { mx = ids[i]; e = i; }
        eot = e;
        if (q == 0 && h == 0 && eot_out) *eot_out = e;
    }
    __syncthreads();
    if (k >= S_pad) return;
    float v = 0.0f;
    if (k < n) {
        if (mode == 1) v = ids[k] == 0 ? -INFINITY : rb[bkt[q * n + k] * NH + h] * LOG2E;
        else v = (k <= q && k <= eot) ? 0.0f : -INFINITY;
    }
    lb[((size_t) h * n + q) * S_pad + k] = v;
}

// One residual row per block, d/4 threads holding 4 contiguous values each.
struct EncNormArgs {
    float * x;                       // [n][d] residual stream, updated in place
    const float * part; long long part_stride; int nparts;   // pending partial tiles (nparts 0: none)
    const float * pbias;             // pending bias [d] or null
    const float * w; const float * b;   // gains, LayerNorm bias (null for RMSNorm)
    int rms;                         // 1: rms_w (shaders/ops_conv.metal:104-114), 0: ln_wb (:90-102)
    float eps;
    __half * out16; long long out_lo;   // split f16 output (hi, lo at out16 + out_lo), or
    float * out32;                   // f32 output (the final norm)
    int d;
};

__device__ __forceinline__ float enc_block_sum(float v, float * red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();   // red is reused by consecutive reductions
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

__global__ void __launch_bounds__(1024) enc_norm_kernel(const EncNormArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int row = blockIdx.x, c = threadIdx.x * 4;
    float * xr = a.x + (size_t) row * a.d + c;
    float4 v = *(const float4 *) xr;
    if (a.nparts) {
        // add_ (shaders/ops_conv.metal:43-48) of the GEMM output: its K slices summed in slice order
        float4 g = *(const float4 *) (a.part + (size_t) row * a.d + c);
        for (int z = 1; z < a.nparts; ++z) {
            const float4 p = *(const float4 *) (a.part + z * a.part_stride + (size_t) row * a.d + c);
            g.x += p.x; g.y += p.y; g.z += p.z; g.w += p.w;
        }
        if (a.pbias) {
            const float4 bb = *(const float4 *) (a.pbias + c);
            g.x += bb.x; g.y += bb.y; g.z += bb.z; g.w += bb.w;
        }
        v.x += g.x; v.y += g.y; v.z += g.z; v.w += g.w;
        *(float4 *) xr = v;
    }
    const float inv_d = 1.0f / (float) a.d;
    float y[4];
    if (a.rms) {
        const float ss = enc_block_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w, red);
        const float inv = 1.0f / sqrtf(ss * inv_d + a.eps);
        const float4 w = *(const float4 *) (a.w + c);
        y[0] = v.x * inv * w.x; y[1] = v.y * inv * w.y; y[2] = v.z * inv * w.z; y[3] = v.w * inv * w.w;
    } else {
        const float mean = enc_block_sum(v.x + v.y + v.z + v.w, red) * inv_d;
        const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
        const float var = enc_block_sum(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3, red) * inv_d;
        const float inv = 1.0f / sqrtf(var + a.eps);
        const float4 w = *(const float4 *) (a.w + c), bb = *(const float4 *) (a.b + c);
        y[0] = d0 * inv * w.x + bb.x; y[1] = d1 * inv * w.y + bb.y; y[2] = d2 * inv * w.z + bb.z; y[3] = d3 * inv * w.w + bb.w;
    }
    if (a.out32) {
        *(float4 *) (a.out32 + (size_t) row * a.d + c) = make_float4(y[0], y[1], y[2], y[3]);
    } else {
        __align__(8) __half hv[4], lv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            hv[e] = __float2half_rn(y[e]);
            lv[e] = __float2half_rn(y[e] - __half2float(hv[e]));
        }
        __half * o = a.out16 + (size_t) row * a.d + c;
        *(uint2 *) o = *(const uint2 *) hv;
        *(uint2 *) (o + a.out_lo) = *(const uint2 *) lv;
    }
}

// global[j] = sum_k W[j][k] * x[eot][k]: the pooled projection gemv (src/clip.cpp:119-120,
// gemv_f, shaders/gemm_attn.metal:66-74) on the EOT row, f32 weights. One warp per output.
__global__ void __launch_bounds__(256) enc_pool_kernel(const float * W, const float * x, const int * eot, float * out, int H) {
    pdl_trigger();
    pdl_wait();
    const int j = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (j >= H) return;
    const float * xr = x + (size_t) *eot * H;
    const float * wr = W + (size_t) j * H;
    float acc = 0.0f;
    for (int k = lane * 4; k < H; k += 128) {
        const float4 w = *(const float4 *) (wr + k), v = *(const float4 *) (xr + k);
        acc += w.x * v.x + w.y * v.y + w.z * v.z + w.w * v.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[j] = acc;
}

// ------------------------------------------------------------------------------------ model
namespace {

// [N][K] weights as the GEMM reads them: f16 (the reference's f32 -> f16 rule), or f16 hi then lo
// halves of f32 weights (split: the split-weight kernel)
struct ELin {
    __half * w = nullptr;
    float * b = nullptr;
    int N = 0, K = 0;
    bool split = false;
    const __half * lo() const { return w + (size_t) N * K; }
    double bytes() const { return (split ? 4.0 : 2.0) * N * K; }
};

// f16 bits -> f32 as the reference's to_f32 reads them: subnormals flushed to signed zero
// (src/gguf.cpp:201-212, and the Q8_0 scale, :219-223)
inline float ref_f16_to_f32(uint16_t u) {
    const uint32_t sign = (u >> 15) & 1u, exp = (u >> 10) & 0x1Fu, man = u & 0x3FFu;
    uint32_t f;
    if (exp == 0) f = sign << 31;
    else if (exp == 31) f = (sign << 31) | 0x7F800000u | (man << 13);
    else f = (sign << 31) | ((exp + 112u) << 23) | (man << 13);
    float r;
    std::memcpy(&r, &f, 4);
    return r;
}

template <typename F> void parallel_for(size_t n, F && f) {
    const unsigned nth = n < (1u << 18) ? 1u : std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    if (nth == 1) { f((size_t) 0, n); return; }
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nth; ++t) th.emplace_back([&, t] { f(n * t / nth, n * (t + 1) / nth); });
    for (auto & x : th) x.join();
}

// A tensor's values as f32 (to_f32, src/gguf.cpp:193-234) and whether the reference's device
// keeps it in f32 (WeightSet::load with keep_f32: exactly the F32 tensors, src/net.mm:128-129).
int tensor_f32(const Gguf & file, const std::string & name, std::vector<float> & out, bool * is_f32,
               std::vector<uint64_t> * ne = nullptr) {
    const GgufTensorInfo * t = file.find(name);
    if (!t || !t->data) return fail(TSN_ERR_MISSING, "missing tensor " + name);
    if (ne) ne->assign(t->ne, t->ne + t->n_dims);
    const size_t n = (size_t) t->nelem();
    out.resize(n);
    if (is_f32) *is_f32 = t->type == GG_F32;
    const uint8_t * d = t->data;
    switch (t->type) {
        case GG_F32: std::memcpy(out.data(), d, n * 4); break;
        case GG_F16:
            parallel_for(n, [&](size_t lo, size_t hi) {
                for (size_t i = lo; i < hi; ++i) out[i] = ref_f16_to_f32(((const uint16_t *) d)[i]);
            });
            break;
        case GG_BF16:
            parallel_for(n, [&](size_t lo, size_t hi) {
                for (size_t i = lo; i < hi; ++i) out[i] = tsn_bf16_to_f32(((const uint16_t *) d)[i]);
            });
            break;
        case GG_Q8_0:
            parallel_for(n / 32, [&](size_t lo, size_t hi) {
                for (size_t bk = lo; bk < hi; ++bk) {
                    const uint8_t * blk = d + bk * 34;
                    uint16_t su;
                    std::memcpy(&su, blk, 2);
                    const float s = ref_f16_to_f32(su);
                    for (int k = 0; k < 32; ++k) out[bk * 32 + k] = s * (float) (int8_t) blk[2 + k];
                }
            });
            break;
        default: return fail(TSN_ERR_UNSUPPORTED, "tensor " + name + " has an unsupported type");
    }
    return TSN_OK;
}

} // namespace

struct EncModel {
    enum Kind { T5 = 1, CLIP = 2 };
    DeviceCtx * dev = nullptr;
    Kind kind = T5;
    int d = 0, F = 0, L = 0, NH = 0, n = 77, S_pad = 128, vocab = 0, n_bucket = 32, max_dist = 128;
    float eps = 1e-6f, scale = 1.0f;
    struct Layer { ELin qkv, o, up, down; float * n1w = nullptr, * n1b = nullptr, * n2w = nullptr, * n2b = nullptr; };
    std::vector<Layer> layers;
    float * fnw = nullptr, * fnb = nullptr;   // final norm
    float * tok = nullptr, * pos = nullptr;   // embedding tables (f32, as the reference's host copies)
    float * rel = nullptr;                    // T5 relative bias [n_bucket][NH]
    float * proj = nullptr;                   // CLIP text_proj [H][H] f32
    int * bkt = nullptr;                      // T5 bucket table [n][n]
    std::vector<void *> weights;
    // activations
    int * ids_d = nullptr, * eot_d = nullptr;
    float * x = nullptr, * part = nullptr, * lb = nullptr, * out = nullptr, * glob = nullptr;
    __half * a16 = nullptr, * qkv = nullptr, * att = nullptr, * h = nullptr;
    std::vector<std::function<cudaError_t(cudaStream_t)>> ops;
    std::vector<std::string> op_names;
    cudaGraphExec_t gx = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    double last_ms = 0.0, flops = 0.0, wbytes = 0.0;
    int last_splits = 1;   // K slices of the last planned GEMM (the partial tiles the next norm adds)

    ~EncModel() {
        if (dev) dev->activate();
        if (gx) cudaGraphExecDestroy(gx);
        for (void * p : weights) cudaFree(p);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
    }
    template <typename P> int dalloc(P ** p, size_t bytes) {
        void * q = nullptr;
        ECK(cudaMalloc(&q, std::max<size_t>(bytes, 16)));
        weights.push_back(q);
        *p = (P *) q;
        return TSN_OK;
    }
    template <typename V> int upload(V ** dst, const V * src, size_t count) {
        ERT(dalloc(dst, count * sizeof(V)));
        ECK(cudaMemcpy(*dst, src, count * sizeof(V), cudaMemcpyHostToDevice));
        return TSN_OK;
    }
    int vec(const Gguf & f, const std::string & name, int len, float ** dst) {
        std::vector<float> v;
        ERT(tensor_f32(f, name, v, nullptr));
        if ((int) v.size() != len) return fail(TSN_ERR_MISSING, name + ": expected " + std::to_string(len) + " values");
        return upload(dst, v.data(), v.size());
    }
    // Linear weights [N][K] from one or more tensors stacked along N; `interleave` (two parts)
    // orders rows in 32-row groups [part 0 | part 1] for the gated epilogues.
    int lin(const Gguf & f, const std::vector<std::string> & names, int K, bool interleave, ELin & W,
            const std::vector<std::string> & biases = {}) {
        std::vector<std::vector<float>> parts(names.size());
        bool f32 = false;
        int N = 0;
        for (size_t i = 0; i < names.size(); ++i) {
            bool t32 = false;
            std::vector<uint64_t> ne;
            ERT(tensor_f32(f, names[i], parts[i], &t32, &ne));
            if (ne.size() != 2 || (int) ne[0] != K) return fail(TSN_ERR_MISSING, names[i] + ": unexpected shape");
            if (i && t32 != f32) return fail(TSN_ERR_UNSUPPORTED, names[i] + ": fused tensors differ in type");
            f32 = t32;
            N += (int) ne[1];
        }
        if (interleave && (names.size() != 2 || parts[0].size() != parts[1].size() || (parts[0].size() / K) % 32))
            return fail(TSN_ERR_UNSUPPORTED, names[0] + ": gated halves must match in 32-row groups");
        if (K % 64 || N % 64) return fail(TSN_ERR_UNSUPPORTED, names[0] + ": dimensions must be multiples of 64");
        W.N = N; W.K = K; W.split = f32;
        const size_t nk = (size_t) N * K;
        std::vector<uint16_t> hw(f32 ? 2 * nk : nk);
        auto src_row = [&](int r) -> const float * {
            if (interleave) {
                const int g = r / 64, j = r % 64;
                return parts[j < 32 ? 0 : 1].data() + (size_t) (g * 32 + (j & 31)) * K;
            }
            for (auto & p : parts) {
                const int rows = (int) (p.size() / K);
                if (r < rows) return p.data() + (size_t) r * K;
                r -= rows;
            }
            return nullptr;
        };
        parallel_for((size_t) N, [&](size_t lo, size_t hi) {
            for (size_t r = lo; r < hi; ++r) {
                const float * s = src_row((int) r);
                for (int k = 0; k < K; ++k) {
                    const size_t o = r * K + k;
                    const uint16_t hv = tsn_ref_f32_to_f16(s[k]);
                    hw[o] = hv;
                    if (f32) hw[nk + o] = tsn_ref_f32_to_f16(s[k] - tsn_f16_to_f32(hv));
                }
            }
        });
        ERT(upload(&W.w, (const __half *) hw.data(), hw.size()));
        if (!biases.empty()) {
            std::vector<float> b;
            for (const std::string & bn : biases) {
                std::vector<float> v;
                ERT(tensor_f32(f, bn, v, nullptr));
                b.insert(b.end(), v.begin(), v.end());
            }
            if ((int) b.size() != N) return fail(TSN_ERR_MISSING, biases[0] + ": bias length");
            ERT(upload(&W.b, b.data(), b.size()));
        }
        wbytes += W.bytes();
        return TSN_OK;
    }

    // T5Model::load (src/t5.cpp:22-59) / ClipModel::load (src/clip.cpp:6-28): geometry from the KV
    // keys with the reference's defaults, every tensor the encode reads
    int load(const Gguf & f, Kind k) {
        kind = k;
        if (kind == T5) {
            d = (int) f.num("t5.d_model", 2048);
            F = (int) f.num("t5.d_ff", 5120);
            L = (int) f.num("t5.n_layers", 24);
            NH = (int) f.num("t5.n_heads", 32);
            n_bucket = (int) f.num("t5.rel_buckets", 32);
            max_dist = (int) f.num("t5.rel_max_dist", 128);
            eps = (float) f.num("t5.eps", 1e-6);
            n = (int) T5_CTX;
            vocab = (int) T5_VOCAB;
            scale = 1.0f;   // T5 folds 1/sqrt(d_kv) into its q weights (src/t5.cpp:73)
        } else {
            d = (int) f.num("clip.hidden", 1024);
            L = (int) f.num("clip.layers", 24);
            NH = (int) f.num("clip.heads", 16);
            n = (int) f.num("clip.ctx", 77);
            F = 4 * d;
            eps = 1e-5f;
            vocab = (int) CLIP_VOCAB;
        }
        if (NH <= 0 || d % NH || d / NH != 64) return fail(TSN_ERR_UNSUPPORTED, "text encoder: head size must be 64");
        if (d % 128 || d > 4096 || F % 64 || n < 1 || n > 256 || L < 1)
            return fail(TSN_ERR_UNSUPPORTED, "text encoder: unsupported geometry");
        if (kind == CLIP) scale = 1.0f / std::sqrt((float) (d / NH));   // src/clip.cpp:114
        S_pad = (n + 63) / 64 * 64;
        layers.resize(L);
        {
            std::vector<float> t;
            bool f32 = false;
            ERT(tensor_f32(f, "tok_emb", t, &f32));
            if (t.size() != (size_t) vocab * d) return fail(TSN_ERR_MISSING, "tok_emb: unexpected size");
            ERT(upload(&tok, t.data(), t.size()));
        }
        for (int l = 0; l < L; ++l) {
            const std::string bp = "blk." + std::to_string(l);
            Layer & y = layers[l];
            if (kind == T5) {                                                              // src/t5.cpp:104-127
                ERT(vec(f, bp + ".attn_norm", d, &y.n1w));
                ERT(lin(f, {bp + ".q", bp + ".k", bp + ".v"}, d, false, y.qkv));
                ERT(lin(f, {bp + ".o"}, d, false, y.o));
                ERT(vec(f, bp + ".ffn_norm", d, &y.n2w));
                ERT(lin(f, {bp + ".wi_0", bp + ".wi_1"}, d, true, y.up));
                ERT(lin(f, {bp + ".wo"}, F, false, y.down));
            } else {                                                                       // src/clip.cpp:50-94
                ERT(vec(f, bp + ".ln1.w", d, &y.n1w));
                ERT(vec(f, bp + ".ln1.b", d, &y.n1b));
                ERT(lin(f, {bp + ".q.w", bp + ".k.w", bp + ".v.w"}, d, false, y.qkv, {bp + ".q.b", bp + ".k.b", bp + ".v.b"}));
                ERT(lin(f, {bp + ".out.w"}, d, false, y.o, {bp + ".out.b"}));
                ERT(vec(f, bp + ".ln2.w", d, &y.n2w));
                ERT(vec(f, bp + ".ln2.b", d, &y.n2b));
                ERT(lin(f, {bp + ".fc1.w"}, d, false, y.up, {bp + ".fc1.b"}));
                ERT(lin(f, {bp + ".fc2.w"}, F, false, y.down, {bp + ".fc2.b"}));
            }
            if (y.qkv.N != 3 * d || y.o.N != d || y.up.N != (kind == T5 ? 2 * F : F) || y.down.N != d)
                return fail(TSN_ERR_MISSING, bp + ": projection shapes do not match the geometry");
        }
        if (kind == T5) {
            ERT(vec(f, "out_norm", d, &fnw));                                            // src/t5.cpp:129
            ERT(vec(f, "rel_bias", n_bucket * NH, &rel));
            std::vector<int> bk((size_t) n * n);                                           // src/t5.cpp:47-54
            for (int q = 0; q < n; ++q)
                for (int kk = 0; kk < n; ++kk) bk[(size_t) q * n + kk] = t5_bucket(kk - q, n_bucket, max_dist);
            ERT(upload(&bkt, bk.data(), bk.size()));
        } else {
            std::vector<float> p;
            ERT(tensor_f32(f, "pos_emb", p, nullptr));
            if (p.size() != (size_t) n * d) return fail(TSN_ERR_MISSING, "pos_emb: unexpected size");
            ERT(upload(&pos, p.data(), p.size()));
            ERT(vec(f, "out_ln.w", d, &fnw));                                            // src/clip.cpp:117
            ERT(vec(f, "out_ln.b", d, &fnb));
            std::vector<float> w;
            ERT(tensor_f32(f, "text_proj", w, nullptr));
            if (w.size() != (size_t) d * d) return fail(TSN_ERR_MISSING, "text_proj: unexpected size");
            ERT(upload(&proj, w.data(), w.size()));
            wbytes += 4.0 * d * d;
        }
        // activations
        ERT(dalloc(&ids_d, (size_t) n * 4));
        ERT(dalloc(&eot_d, 16));
        ERT(dalloc(&x, (size_t) n * d * 4));
        ERT(dalloc(&part, (size_t) MAX_PARTS * n * d * 4));
        ERT(dalloc(&lb, (size_t) NH * n * S_pad * 4));
        ERT(dalloc(&out, (size_t) n * d * 4));
        ERT(dalloc(&glob, (size_t) d * 4));
        ERT(dalloc(&a16, (size_t) 2 * n * d * 2));
        ERT(dalloc(&att, (size_t) 2 * n * d * 2));
        ERT(dalloc(&h, (size_t) 2 * n * F * 2));
        ERT(dalloc(&qkv, (size_t) 6 * d * S_pad * 2));
        ECK(cudaMemset(qkv, 0, (size_t) 6 * d * S_pad * 2));   // rows n .. S_pad-1 stay zero
        ECK(cudaEventCreate(&e0));
        ECK(cudaEventCreate(&e1));
        return prepare();
    }

    // One projection over the n token rows of the split operand A ([n][K] hi, then lo). Tile width
    // and K slices: timed at load over every valid configuration (once per GEMM role: qkv, o, up,
    // down share their shapes across layers), or the split-operand cost model with autotune off.
    // partial: independent K slices write partial tiles into `part`.
    std::map<std::string, std::pair<int, int>> tiles;   // role -> (tile width, K slices)
    bool autotune = true;

    std::vector<std::pair<int, int>> candidates(const ELin & W, int epi, bool partial) const {
        std::vector<std::pair<int, int>> c;
        const int kb = W.K / 64;
        for (int cb : {256, 128, 64}) {
            if (W.N % cb) continue;
            for (int s = 1; s <= (partial ? MAX_PARTS : 8) && s <= kb; ++s) {
                const int kbps = (kb + s - 1) / s;
                if ((kb + kbps - 1) / kbps != s) continue;
                const int cl = partial ? 1 : s;
                if ((W.split ? gemm_ws_capacity(cb, epi, cl) : gemm_cluster_capacity(cb, epi, true, cl)) > 0) c.push_back({cb, s});
            }
        }
        return c;
    }
    std::pair<int, int> cost_model(const ELin & W, int epi, bool partial) const {
        const int kb = W.K / 64;
        double best = 1e30;
        std::pair<int, int> r{0, 1};
        for (auto [cb, s] : candidates(W, epi, partial)) {
            const double kcost = W.split ? (cb == 256 ? 1.1 : cb == 128 ? 0.6 : 0.45) : (cb == 256 ? 0.74 : cb == 128 ? 0.40 : 0.30);
            const int kbps = (kb + s - 1) / s, cl = partial ? 1 : s;
            const int cap = W.split ? gemm_ws_capacity(cb, epi, cl) : gemm_cluster_capacity(cb, epi, true, cl);
            const int waves = (W.N / cb * s + cap - 1) / cap;
            const double cost = waves * (kbps * kcost + 1.5) + (s > 1 ? (partial ? 0.3 * s : 1.5 * waves) : 0.0);
            if (cost < best - 1e-9) { best = cost; r = {cb, s}; }
        }
        return r;
    }
    int build_gemm(const std::string & name, const ELin & W, const __half * A, int epi, bool partial, int bn, int sp,
                   const std::function<void(GemmArgs &)> & outs, GemmLaunch & gl) {
        const int kb = W.K / 64;
        gl = GemmLaunch{};
        gl.bn = bn; gl.epi = epi; gl.split = true; gl.ab_bf16 = 0;
        gl.smem = W.split ? gemm_ws_smem_bytes(bn, epi) : gemm_smem_bytes(bn, true, epi);
        gl.grid = dim3(1, W.N / bn, sp);
        // the 77 token rows as an 80-row activation box: rows 80..127 of each A tile are never loaded
        const int ar = (n + 15) / 16 * 16;
        if (!make_act_map(&gl.ta, A, W.K, n, 1, ar, 1, 0) || !make_act_map(&gl.ta2, A + (size_t) n * W.K, W.K, n, 1, ar, 1, 0) ||
            !make_w_map(&gl.tb, W.w, W.K, W.N, bn, 0) || (W.split && !make_w_map(&gl.tb2, W.lo(), W.K, W.N, bn, 0)))
            return fail(TSN_ERR_CUDA, name + ": tensor map encode failed");
        GemmArgs & a = gl.args;
        a.rows = n; a.B = 1; a.bt = ar; a.bb = 1; a.m_tiles_t = 1; a.N = W.N; a.a_rows = ar;
        a.k_blocks = kb; a.ic_blocks = kb; a.pad = 0;
        a.splits = partial ? 1 : sp; a.kb_per_split = (kb + sp - 1) / sp;
        a.err = dev->d_err;
        a.bias = partial ? nullptr : W.b;
        a.m_fast = 1;
        if (partial) { a.out = part; a.ldo = d; a.out_bs = 0; a.part_stride = (long long) n * d; }
        outs(a);
        return TSN_OK;
    }
    static cudaError_t run_gemm(const GemmLaunch & gl, bool ws, cudaStream_t s) {
        return ws ? launch_gemm_ws(gl, s) : launch_gemm(gl, s);
    }
    // mean device time of `reps` back-to-back launches (after warm-up), microseconds
    int time_gemm(const GemmLaunch & gl, bool ws, double & us) {
        for (int i = 0; i < 3; ++i) ECK(run_gemm(gl, ws, dev->stream));
        ECK(cudaEventRecord(e0, dev->stream));
        const int reps = 10;
        for (int i = 0; i < reps; ++i) ECK(run_gemm(gl, ws, dev->stream));
        ECK(cudaEventRecord(e1, dev->stream));
        ERT(dev->sync());
        float ms = 0;
        ECK(cudaEventElapsedTime(&ms, e0, e1));
        us = 1000.0 * ms / reps;
        return TSN_OK;
    }
    int gemm_op(const std::string & name, const ELin & W, const __half * A, int epi, bool partial,
                const std::function<void(GemmArgs &)> & outs) {
        const std::string role = name.substr(name.rfind('.') + 1);
        GemmLaunch gl;
        auto it = tiles.find(role);
        if (it == tiles.end()) {
            std::pair<int, int> pick = cost_model(W, epi, partial);
            if (!pick.first) return fail(TSN_ERR_ARG, name + ": no tile fits");
            if (autotune) {
                double best = 1e30;
                for (auto c : candidates(W, epi, partial)) {
                    double us = 0;
                    ERT(build_gemm(name, W, A, epi, partial, c.first, c.second, outs, gl));
                    ERT(time_gemm(gl, W.split, us));
                    if (us < best) { best = us; pick = c; }
                }
            }
            it = tiles.emplace(role, pick).first;
        }
        const int bn = it->second.first, sp = it->second.second;
        ERT(build_gemm(name, W, A, epi, partial, bn, sp, outs, gl));
        last_splits = sp;
        const bool ws = W.split;
        ops.push_back([gl, ws](cudaStream_t s) { return run_gemm(gl, ws, s); });
        op_names.push_back(name + "[" + std::to_string(bn) + "x" + std::to_string(sp) + "]");
        flops += 2.0 * n * (double) W.N * W.K;
        return TSN_OK;
    }

    void norm_op(const std::string & name, int nparts, const float * pbias, const float * w, const float * b,
                 __half * out16, float * out32) {
        EncNormArgs a{};
        a.x = x; a.part = part; a.part_stride = (long long) n * d; a.nparts = nparts; a.pbias = pbias;
        a.w = w; a.b = b; a.rms = kind == T5; a.eps = eps;
        a.out16 = out16; a.out_lo = (long long) n * d; a.out32 = out32; a.d = d;
        const int rows = n, threads = d / 4;
        ops.push_back([a, rows, threads](cudaStream_t s) {
            return launch_ex(enc_norm_kernel, dim3(rows), dim3(threads), 0, s, 1u, a);
        });
        op_names.push_back(name);
    }

    // the encode as launches (T5Model::encode, src/t5.cpp:84-131; ClipModel::encode,
    // src/clip.cpp:30-101), captured into one graph
    int prepare() {
        ops.clear();
        op_names.clear();
        flops = 0.0;
        {
            const long long n4 = (long long) n * d / 4;
            const unsigned blocks = (unsigned) std::min<long long>((n4 + 255) / 256, 148 * 4);
            const int * ids = ids_d; const float * tk = tok, * ps = pos; float * xx = x; const int nn = n, dd = d;
            ops.push_back([=](cudaStream_t s) {
                return launch_ex(enc_embed_kernel, dim3(blocks), dim3(256), 0, s, 1u, ids, tk, ps, xx, nn, dd);
            });
            op_names.push_back("embed");
            const int * bk = bkt; const float * rb = rel; float * lbb = lb; int * eo = eot_d;
            const int sp = S_pad, nh = NH, mode = kind == T5 ? 1 : 2;
            ops.push_back([=](cudaStream_t s) {
                return launch_ex(enc_lbias_kernel, dim3(nn, nh), dim3(sp), 0, s, 1u, ids, bk, rb, lbb, eo, nn, sp, nh, mode);
            });
            op_names.push_back("logit_bias");
        }
        const long long qkv_lo = 3LL * d * S_pad;
        __half * q = qkv, * k = qkv + (size_t) d * S_pad, * v = qkv + 2 * (size_t) d * S_pad;
        int nparts = 0;
        const float * pbias = nullptr;
        for (int l = 0; l < L; ++l) {
            const Layer & y = layers[l];
            const std::string bp = "blk." + std::to_string(l);
            norm_op(bp + ".norm1", nparts, pbias, y.n1w, y.n1b, a16, nullptr);
            ERT(gemm_op(bp + ".qkv", y.qkv, a16, EPI_QKV, false, [&](GemmArgs & a) {
                a.q = q; a.k = k; a.v = v; a.H = d; a.NH = NH; a.S_pad = S_pad; a.s_off = 0; a.out_lo = qkv_lo;
                a.qn = nullptr; a.kn = nullptr; a.rope = nullptr;
            }));
            {
                AttnArgs at{};
                at.q = q; at.k = k; at.v = v; at.B = 1; at.NH = NH; at.S = n; at.S_pad = S_pad;
                at.scale_log2 = scale * LOG2E;
                at.out0 = att; at.n0 = n; at.H = d; at.qkv_lo = qkv_lo; at.out_lo0 = (long long) n * d;
                at.err = dev->d_err;
                at.lbias = lb;
                // the tcgen05 short-sequence kernel with the logit-bias table (TSN_ATTN_KERNEL=mma:
                // the earlier mma.sync kernel, for comparison)
                AttnMaps mp{};
                const uint64_t rows = (uint64_t) NH * S_pad;
                const char * ak = std::getenv("TSN_ATTN_KERNEL");
                const bool tc = attention_short_fits(n) && !(ak && !strcmp(ak, "mma"));
                if (tc && !(make_head_map(&mp.q, q, rows, 128, (uint64_t) qkv_lo) &&
                            make_head_map(&mp.k, k, rows, 64, (uint64_t) qkv_lo) &&
                            make_head_map(&mp.v, v, rows, 64, (uint64_t) qkv_lo)))
                    return fail(TSN_ERR_CUDA, "encoder attention: tensor map encode failed");
                ops.push_back([at, mp, tc](cudaStream_t s) {
                    return tc ? launch_attention_short(mp, at, s) : launch_attention(at, s);
                });
                op_names.push_back(bp + ".attn");
                flops += 4.0 * n * (double) n * d;
            }
            ERT(gemm_op(bp + ".o", y.o, att, EPI_F32, true, [](GemmArgs &) {}));
            nparts = last_splits;
            pbias = y.o.b;
            norm_op(bp + ".norm2", nparts, pbias, y.n2w, y.n2b, a16, nullptr);
            ERT(gemm_op(bp + ".up", y.up, a16, kind == T5 ? EPI_GEGLU : EPI_F16_GELUQ, false, [&](GemmArgs & a) {
                a.out = h; a.ldo = F; a.out_bs = 0; a.out_lo = (long long) n * F;
            }));
            ERT(gemm_op(bp + ".down", y.down, h, EPI_F32, true, [](GemmArgs &) {}));
            nparts = last_splits;
            pbias = y.down.b;
        }
        norm_op("final_norm", nparts, pbias, fnw, fnb, nullptr, out);
        if (kind == CLIP) {
            const float * W = proj, * xo = out; const int * eo = eot_d; float * g = glob; const int H = d;
            ops.push_back([=](cudaStream_t s) {
                return launch_ex(enc_pool_kernel, dim3((H + 7) / 8), dim3(256), 0, s, 1u, W, xo, eo, g, H);
            });
            op_names.push_back("text_proj");
            flops += 2.0 * d * d;
        }
        if (gx) { cudaGraphExecDestroy(gx); gx = nullptr; }
        cudaGraph_t graph = nullptr;
        ECK(cudaStreamBeginCapture(dev->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = cudaSuccess;
        for (size_t i = 0; i < ops.size() && e == cudaSuccess; ++i) e = ops[i](dev->stream);
        cudaError_t e2 = cudaStreamEndCapture(dev->stream, &graph);
        if (e != cudaSuccess || e2 != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            return fail(TSN_ERR_CUDA, std::string("text encoder graph capture: ") + cudaGetErrorString(e != cudaSuccess ? e : e2));
        }
        e = cudaGraphInstantiate(&gx, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("text encoder graph instantiate: ") + cudaGetErrorString(e));
        return TSN_OK;
    }

    // ids: n token ids (host); per_token [n][d] and (CLIP) pooled [d], host or device pointers
    int encode(const int32_t * ids, float * per_token, size_t cap, float * pooled, size_t pooled_cap) {
        if (!ids || !per_token) return fail(TSN_ERR_ARG, "null argument");
        if (cap < (size_t) n * d) return fail(TSN_ERR_ARG, "output buffer too small");
        if (kind == CLIP && pooled && pooled_cap < (size_t) d) return fail(TSN_ERR_ARG, "pooled buffer too small");
        for (int i = 0; i < n; ++i)
            if (ids[i] < 0 || ids[i] >= vocab) return fail(TSN_ERR_ARG, "token id out of range");
        ECK(cudaMemcpyAsync(ids_d, ids, (size_t) n * 4, cudaMemcpyHostToDevice, dev->stream));
        ECK(cudaEventRecord(e0, dev->stream));
        ECK(cudaGraphLaunch(gx, dev->stream));
        ECK(cudaEventRecord(e1, dev->stream));
        ECK(cudaMemcpyAsync(per_token, out, (size_t) n * d * 4, cudaMemcpyDefault, dev->stream));
        if (kind == CLIP && pooled) ECK(cudaMemcpyAsync(pooled, glob, (size_t) d * 4, cudaMemcpyDefault, dev->stream));
        ERT(dev->sync());
        float ms = 0;
        ECK(cudaEventElapsedTime(&ms, e0, e1));
        last_ms = ms;
        return TSN_OK;
    }

    // the graph's launches once more eagerly, one line per launch: index, name, device ms
    int profile(std::string & rep) {
        std::vector<cudaEvent_t> ev(ops.size() + 1);
        for (auto & e : ev) ECK(cudaEventCreate(&e));
        ECK(cudaEventRecord(ev[0], dev->stream));
        for (size_t i = 0; i < ops.size(); ++i) {
            ECK(ops[i](dev->stream));
            ECK(cudaEventRecord(ev[i + 1], dev->stream));
        }
        int rc = dev->sync();
        char line[160];
        for (size_t i = 0; !rc && i < ops.size(); ++i) {
            float ms = 0;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            snprintf(line, sizeof line, "%4zu %-20s %8.4f ms\n", i, op_names[i].c_str(), ms);
            rep += line;
        }
        for (auto & e : ev) cudaEventDestroy(e);
        return rc;
    }
};

} // namespace tsn

// ------------------------------------------------------------------------------- C ABI
struct tsn_encoder { tsn::EncModel m; };

using namespace tsn;

namespace {
int new_encoder(tsn_device * dev, const char * path, EncModel::Kind kind, tsn_encoder ** out) {
    if (!dev || !path || !out) return fail(TSN_ERR_ARG, "null argument");
    *out = nullptr;
    ERT(dev->ctx.activate());
    Gguf f;
    std::string err;
    if (!f.open(path, err)) return fail(TSN_ERR_IO, err);
    std::unique_ptr<tsn_encoder> e(new tsn_encoder);
    e->m.dev = &dev->ctx;
    ERT(e->m.load(f, kind));
    *out = e.release();
    return TSN_OK;
}
} // namespace

extern "C" {

int tsn_t5_load(tsn_device * dev, const char * gguf_path, tsn_encoder ** out) {
    return new_encoder(dev, gguf_path, EncModel::T5, out);
}

int tsn_clip_load(tsn_device * dev, const char * gguf_path, tsn_encoder ** out) {
    return new_encoder(dev, gguf_path, EncModel::CLIP, out);
}

int tsn_encoder_info(tsn_encoder * e, uint32_t * width, uint32_t * ctx, uint32_t * layers) {
    if (!e) return fail(TSN_ERR_ARG, "null argument");
    if (width) *width = (uint32_t) e->m.d;
    if (ctx) *ctx = (uint32_t) e->m.n;
    if (layers) *layers = (uint32_t) e->m.L;
    return TSN_OK;
}

int tsn_encoder_encode(tsn_encoder * e, const int32_t * ids, uint32_t n_ids, float * per_token, size_t per_token_cap,
                       float * pooled, size_t pooled_cap) {
    if (!e || !ids) return fail(TSN_ERR_ARG, "null argument");
    if ((int) n_ids != e->m.n) return fail(TSN_ERR_ARG, "expected exactly ctx token ids");
    ERT(e->m.dev->activate());
    return e->m.encode(ids, per_token, per_token_cap, pooled, pooled_cap);
}

double tsn_encoder_last_ms(tsn_encoder * e) { return e ? e->m.last_ms : 0.0; }
double tsn_encoder_flops(tsn_encoder * e) { return e ? e->m.flops : 0.0; }
int tsn_encoder_launches(tsn_encoder * e) { return e ? (int) e->m.ops.size() : 0; }
double tsn_encoder_weight_bytes(tsn_encoder * e) { return e ? e->m.wbytes : 0.0; }

int tsn_encoder_profile_ops(tsn_encoder * e, char * out, size_t cap) {
    if (!e) return fail(TSN_ERR_ARG, "null argument");
    ERT(e->m.dev->activate());
    std::string rep;
    ERT(e->m.profile(rep));
    if (out && cap) { std::strncpy(out, rep.c_str(), cap - 1); out[cap - 1] = 0; }
    return TSN_OK;
}

int tsn_encoder_free(tsn_encoder * e) {
    if (e) { if (e->m.dev) cudaStreamSynchronize(e->m.dev->stream); delete e; }
    return TSN_OK;
}

int tsn_gguf_write_synthetic_t5(const char * path, uint32_t d_model, uint32_t d_ff, uint32_t layers, uint32_t heads,
                                uint64_t seed) {
    if (!path || !d_model || !d_ff || !layers || !heads) return fail(TSN_ERR_ARG, "bad T5 geometry");
    T5Geom g;
    g.d_model = d_model; g.d_ff = d_ff; g.layers = layers; g.heads = heads;
    std::string err;
    if (!write_synthetic_t5_gguf(path, g, seed, err)) return fail(TSN_ERR_IO, err);
    return TSN_OK;
}

int tsn_gguf_write_synthetic_clip(const char * path, uint32_t hidden, uint32_t layers, uint32_t heads, uint64_t seed) {
    if (!path || !hidden || !layers || !heads) return fail(TSN_ERR_ARG, "bad CLIP geometry");
    ClipGeom g;
    g.hidden = hidden; g.layers = layers; g.heads = heads;
    std::string err;
    if (!write_synthetic_clip_gguf(path, g, seed, err)) return fail(TSN_ERR_IO, err);
    return TSN_OK;
}

} // extern "C"
