// prep.cu — the once-per-generation conditioning on the GPU: DitModel::prep_conditioning and
// DitModel::prep_text_arm (src/dit.cpp:55-192).
//
// The reference runs these through its Runtime (gemm / conv / silu / swiglu / mean_cols / gemv)
// and round-trips through the host for the sync position embedding, the sync row gather and the
// clip_fc + text_fc sum. Here every step stays on the device: the same sequence runs on the
// library's runtime face (split-operand tcgen05 GEMMs, im2col conv, elementwise kernels) plus two
// small kernels for the position-embedding add and the gather, and the results land directly in
// the model's conditioning buffers (clip_pp, sync_gather, text_pp[arm], gcmlp[arm]) that the
// forward reads — no tsn_dit_set_conditioning needed.
#include <cmath>
#include <vector>

#include "compat.h"
#include "kernels.h"
#include "runtime.h"

namespace tsn {

#define CKR(expr)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) return fail(TSN_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

namespace {

// sbuf[s][c] = sync_f[s][c] + pos[s % 8][c]   (src/dit.cpp:93-99, on the host there)
__global__ void add_sync_pos_kernel(const float * sync_f, const float * pos, float * out, int sync_S) {
    const long long n = (long long) sync_S * 768;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const int s = (int) (i / 768), c = (int) (i % 768);
        out[i] = sync_f[i] + pos[(s % 8) * 768 + c];
    }
}

// dst[i][:] = src[idx[i]][:]   (src/dit.cpp:110-114)
__global__ void gather_rows_kernel(const float * src, const int * idx, float * dst, int rows, int H) {
    const long long n = (long long) rows * H;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const int r = (int) (i / H), c = (int) (i % H);
        dst[i] = src[(long long) idx[r] * H + c];
    }
}

unsigned grid_for(long long n) { return (unsigned) std::min<long long>((n + 255) / 256, 148 * 8); }

// device scratch owned by one prep call
struct Scratch {
    std::vector<void *> bufs;
    ~Scratch() { for (void * p : bufs) cudaFree(p); }
    template <typename T> int get(size_t n, T ** out) {
        void * p = nullptr;
        CKR(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
        bufs.push_back(p);
        *out = (T *) p;
        return TSN_OK;
    }
};

#define RT(call) do { int rc_ = (call); if (rc_) return rc_; } while (0)

// convmlp (src/dit.cpp:14-20): conv k3 w1, w3 -> swiglu -> conv k3 w2 into y (y may alias x)
int convmlp(DeviceCtx & c, const Lin & w1, const Lin & w3, const Lin & w2, const float * x, float * h1, float * h3,
            float * y, int T, int C, int F) {
    RT(compat_conv(c, 1, w1.w, nullptr, x, h1, T, T, C, F, 3, 1, 1, 1, 0));
    RT(compat_conv(c, 1, w3.w, nullptr, x, h3, T, T, C, F, 3, 1, 1, 1, 0));
    RT(compat_elementwise(c, "swiglu_", h1, h3, h1, (size_t) T * F, 0, 0));
    return compat_conv(c, 1, w2.w, nullptr, h1, y, T, T, F, C, 3, 1, 1, 1, 0);
}

// mlp (src/dit.cpp:21-27) on `rows` rows
int mlp(DeviceCtx & c, const Lin & w1, const Lin & w3, const Lin & w2, const float * x, float * h1, float * h3, float * y,
        int rows, int C, int F) {
    RT(compat_gemm(c, 1, w1.w, x, h1, nullptr, rows, F, C, C, C, F));
    RT(compat_gemm(c, 1, w3.w, x, h3, nullptr, rows, F, C, C, C, F));
    RT(compat_elementwise(c, "swiglu_", h1, h3, h1, (size_t) rows * F, 0, 0));
    return compat_gemm(c, 1, w2.w, h1, y, nullptr, rows, C, F, F, F, C);
}

} // namespace

int Model::prep_conditioning(const float * clip_f, const float * sync_f, int sync_S) {
    if (g.H != 1024) return fail(TSN_ERR_UNSUPPORTED, "prep_conditioning needs H = 1024 (its cond projections read 1024 inputs)");
    if (G != 1) return fail(TSN_ERR_UNSUPPORTED, "prep_conditioning serves models prepared for one generation");
    if (sync_S < 1) return fail(TSN_ERR_ARG, "sync_S must be positive");
    RT(load_prep(*this));
    DeviceCtx & c = *dev;
    const int H = (int) g.H, F = (int) g.F;
    const PrepW & w = pw;
    Scratch sc;
    float * clipf, * syncf, * sbuf, * smid, * h1, * h3, * cmean;
    int * idx;
    const int rows_max = std::max(sync_S, C);
    RT(sc.get((size_t) C * 1024, &clipf));
    RT(sc.get((size_t) sync_S * 768, &syncf));
    RT(sc.get((size_t) sync_S * 768, &sbuf));
    RT(sc.get((size_t) sync_S * H, &smid));
    RT(sc.get((size_t) rows_max * F, &h1));
    RT(sc.get((size_t) rows_max * F, &h3));
    RT(sc.get((size_t) H, &cmean));
    RT(sc.get((size_t) T, &idx));
    if (!clip_fc) CKR(cudaMalloc(&clip_fc, (size_t) H * 4));
    CKR(cudaMemcpyAsync(clipf, clip_f, (size_t) C * 1024 * 4, cudaMemcpyDefault, c.stream));
    CKR(cudaMemcpyAsync(syncf, sync_f, (size_t) sync_S * 768 * 4, cudaMemcpyDefault, c.stream));
    // sync: + position embedding per 8-frame segment, conv k7 + silu, convmlp, gather to T rows
    add_sync_pos_kernel<<<grid_for((long long) sync_S * 768), 256, 0, c.stream>>>(syncf, w.sync_pos, sbuf, sync_S);
    CKR(cudaGetLastError());
    RT(compat_conv(c, 1, w.sync0.w, w.sync0.b, sbuf, smid, sync_S, sync_S, 768, H, 7, 1, 3, 1, 0));
    RT(compat_elementwise(c, "silu_", smid, nullptr, smid, (size_t) sync_S * H, 0, 0));
    RT(convmlp(c, w.sync_w1, w.sync_w3, w.sync_w2, smid, h1, h3, smid, sync_S, H, F));
    std::vector<int> hidx(T);
    for (int i = 0; i < T; ++i) hidx[i] = (int) floorf(((float) i + 0.5f) * (float) sync_S / (float) T);   // dit.cpp:111
    CKR(cudaMemcpyAsync(idx, hidx.data(), (size_t) T * 4, cudaMemcpyHostToDevice, c.stream));
    gather_rows_kernel<<<grid_for((long long) T * H), 256, 0, c.stream>>>(smid, idx, sync_gather, T, H);
    CKR(cudaGetLastError());
    // clip: linear + silu + convmlp -> clip_pp; clip_fc = clip_cond_proj(mean over the clip rows)
    RT(compat_gemm(c, 1, w.clip0.w, clipf, clip_pp, w.clip0.b, C, H, 1024, 1024, 1024, H));
    RT(compat_elementwise(c, "silu_", clip_pp, nullptr, clip_pp, (size_t) C * H, 0, 0));
    RT(convmlp(c, w.clip_w1, w.clip_w3, w.clip_w2, clip_pp, h1, h3, clip_pp, C, H, F));
    RT(compat_mean_cols(c, clip_pp, cmean, C, H));
    RT(compat_gemv(c, 1, w.clip_cond.w, cmean, clip_fc, w.clip_cond.b, H, 1024, 1024));
    RT(dev->sync());   // the scratch buffers are freed on return
    clip_fc_valid = true;
    return TSN_OK;
}

int Model::prep_text_arm(int arm, const float * text_cat, const float * gtext) {
    if (arm < 0 || arm >= B) return fail(TSN_ERR_ARG, "arm out of range for the prepared model");
    if (!clip_fc_valid) return fail(TSN_ERR_STATE, "call tsn_dit_prep_conditioning first");
    RT(load_prep(*this));
    DeviceCtx & c = *dev;
    const int H = (int) g.H, F = (int) g.F;
    const PrepW & w = pw;
    Scratch sc;
    float * tcat, * gt, * f1, * f3, * tfc, * g1, * g3;
    RT(sc.get((size_t) TS * 2048, &tcat));
    RT(sc.get((size_t) 1024, &gt));
    RT(sc.get((size_t) TS * F, &f1));
    RT(sc.get((size_t) TS * F, &f3));
    RT(sc.get((size_t) H, &tfc));
    RT(sc.get((size_t) F, &g1));
    RT(sc.get((size_t) F, &g3));
    CKR(cudaMemcpyAsync(tcat, text_cat, (size_t) TS * 2048 * 4, cudaMemcpyDefault, c.stream));
    CKR(cudaMemcpyAsync(gt, gtext, (size_t) 1024 * 4, cudaMemcpyDefault, c.stream));
    float * tp = text_pp + (size_t) arm * TS * H;
    // text_pp = w2(swiglu(w1 x, w3 x)) with x = silu(text_input_proj.0(text_cat))
    RT(compat_gemm(c, 1, w.text0.w, tcat, tp, w.text0.b, TS, H, 2048, 2048, 2048, H));
    RT(compat_elementwise(c, "silu_", tp, nullptr, tp, (size_t) TS * H, 0, 0));
    RT(mlp(c, w.text_w1, w.text_w3, w.text_w2, tp, f1, f3, tp, TS, H, F));
    // gcmlp = global_cond_mlp(text_cond_proj(gtext) + clip_fc)
    RT(compat_gemv(c, 1, w.text_cond.w, gt, tfc, w.text_cond.b, H, 1024, 1024));
    RT(compat_elementwise(c, "add_", tfc, clip_fc, tfc, (size_t) H, 0, 0));
    RT(mlp(c, w.g_w1, w.g_w3, w.g_w2, tfc, g1, g3, gcmlp + (size_t) arm * H, 1, H, F));
    return dev->sync();
}

} // namespace tsn
