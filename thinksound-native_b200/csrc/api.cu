// api.cu — the C ABI of include/tsn.h over DeviceCtx / Model (runtime.h) and the named-kernel
// compat layer (compat.cu).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <unistd.h>

#include "compat.h"
#include "gguf_io.h"
#include "runtime.h"

using namespace tsn;

namespace tsn {
const std::string & last_error();
int gemm_noalloc(DeviceCtx & c, const void * W, const void * X, void * Y, const void * bias, uint32_t M, uint32_t N,
                 uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy);
int selftest_gemm_lo8(DeviceCtx & c, const void * W, const void * X, void * Y, const void * bias, uint32_t M, uint32_t N,
                      uint32_t K, int wexp, int mode, int bn, int reps, float * ms);
}

struct tsn_dit { Model m; };

#define CKR(expr)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) return fail(TSN_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define TRY(expr) do { int rc_ = (expr); if (rc_) return rc_; } while (0)

extern "C" {

const char * tsn_last_error(void) { return tsn::last_error().c_str(); }
int tsn_version(void) { return 1; }

// ------------------------------------------------------------------------------- device face
int tsn_device_create(int ordinal, tsn_device ** out) {
    if (!out) return fail(TSN_ERR_ARG, "null out");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(TSN_ERR_CUDA, "no CUDA device");
    if (ordinal < 0 || ordinal >= n) return fail(TSN_ERR_ARG, "device ordinal out of range");
    cudaDeviceProp prop{};
    CKR(cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major != 10) return fail(TSN_ERR_CUDA, std::string("needs an sm_100 (B200) device, found ") + prop.name);
    auto d = std::make_unique<tsn_device>();
    d->ctx.ordinal = ordinal;
    TRY(d->ctx.activate());
    CKR(cudaStreamCreateWithFlags(&d->ctx.stream, cudaStreamNonBlocking));
    d->ctx.own_stream = true;
    CKR(cudaMalloc(&d->ctx.d_err, 64));
    CKR(cudaMemset(d->ctx.d_err, 0, 64));
    CKR(cudaEventCreate(&d->ctx.ev0));
    CKR(cudaEventCreate(&d->ctx.ev1));
    CKR(configure_gemm_kernels());
    CKR(configure_attention());
    CKR(configure_attention_tc());
    CKR(configure_attention_short());
    CKR(configure_gemv());
    CKR(configure_gemv_tc());
    *out = d.release();
    return TSN_OK;
}

int tsn_device_destroy(tsn_device * dev) {
    if (!dev) return TSN_OK;
    DeviceCtx & c = dev->ctx;
    c.activate();
    cudaStreamSynchronize(c.stream);
    for (void * p : c.managed) cudaFree(p);
    for (auto & r : c.host_regs) cudaHostUnregister((void *) r.first);
    if (c.scratch) cudaFree(c.scratch);
    if (c.col) cudaFree(c.col);
    if (c.d_err) cudaFree(c.d_err);
    if (c.ev0) cudaEventDestroy(c.ev0);
    if (c.ev1) cudaEventDestroy(c.ev1);
    if (c.own_stream && c.stream) cudaStreamDestroy(c.stream);
    delete dev;
    return TSN_OK;
}

int tsn_device_set_stream(tsn_device * dev, void * s) {
    if (!dev) return fail(TSN_ERR_ARG, "null device");
    DeviceCtx & c = dev->ctx;
    if (c.own_stream && c.stream) { cudaStreamSynchronize(c.stream); cudaStreamDestroy(c.stream); }
    c.stream = (cudaStream_t) s;
    c.own_stream = false;
    return TSN_OK;
}

void * tsn_device_stream(tsn_device * dev) { return dev ? (void *) dev->ctx.stream : nullptr; }

int tsn_alloc(tsn_device * dev, size_t bytes, void ** out) {
    if (!dev || !out) return fail(TSN_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    TRY(dev->ctx.activate());
    if (bytes == 0) bytes = 16;
    void * p = nullptr;
    if (cudaMallocManaged(&p, bytes) != cudaSuccess) return fail(TSN_ERR_OOM, "managed allocation failed");
    CKR(cudaMemset(p, 0, bytes));
    CKR(cudaDeviceSynchronize());
    dev->ctx.managed.push_back(p);
    *out = p;
    return TSN_OK;
}

// Device::wrap (src/gpu.mm:66-87). Managed/device memory is used as is; host memory is pinned in
// place (no copy) page by page. Like the reference's registry lookup, a range inside memory an
// earlier wrap registered resolves through that registration; a range that reaches past it
// registers only the pages not yet registered (mapped host pages keep their host address on the
// device, so the pieces need not be one registration). Registrations end with the device.
int tsn_wrap(tsn_device * dev, const void * p, size_t bytes, void ** out) {
    if (!dev || !out || !p) return fail(TSN_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    const uintptr_t a = (uintptr_t) p, e = a + std::max<size_t>(bytes, 1);
    auto covering = [&](uintptr_t x) {   // the registration holding address x, or end()
        auto it = c.host_regs.upper_bound(x);
        if (it == c.host_regs.begin()) return c.host_regs.end();
        --it;
        return x < it->first + it->second.bytes ? it : c.host_regs.end();
    };
    auto hit = covering(a);
    if (hit != c.host_regs.end() && e <= hit->first + hit->second.bytes) {
        *out = (char *) hit->second.dev + (a - hit->first);
        return TSN_OK;
    }
    cudaPointerAttributes pa{};
    if (hit == c.host_regs.end() && cudaPointerGetAttributes(&pa, p) == cudaSuccess &&
        pa.type != cudaMemoryTypeUnregistered) {
        *out = (void *) p;
        return TSN_OK;
    }
    cudaGetLastError();
    int same_addr = 0;
    CKR(cudaDeviceGetAttribute(&same_addr, cudaDevAttrCanUseHostPointerForRegisteredMem, c.ordinal));
    const uintptr_t page = (uintptr_t) sysconf(_SC_PAGESIZE), lo = a & ~(page - 1), hi = (e + page - 1) & ~(page - 1);
    if (hit != c.host_regs.end() && !same_addr)
        return fail(TSN_ERR_ARG, "wrap range extends a registered range and this device cannot use host addresses");
    // register every run of pages in [lo, hi) that no earlier wrap holds
    for (uintptr_t x = lo; x < hi;) {
        auto r = covering(x);
        if (r != c.host_regs.end()) { x = r->first + r->second.bytes; continue; }
        auto next = c.host_regs.upper_bound(x);
        const uintptr_t run_end = next == c.host_regs.end() ? hi : std::min<uintptr_t>(hi, next->first);
        CKR(cudaHostRegister((void *) x, run_end - x, cudaHostRegisterMapped | cudaHostRegisterPortable));
        void * d = nullptr;
        CKR(cudaHostGetDevicePointer(&d, (void *) x, 0));
        c.host_regs[x] = DeviceCtx::HostReg{run_end - x, d};
        x = run_end;
    }
    if (same_addr) { *out = (void *) p; return TSN_OK; }
    hit = covering(a);
    *out = (char *) hit->second.dev + (a - hit->first);
    return TSN_OK;
}

int tsn_begin(tsn_device * dev) {
    if (!dev) return fail(TSN_ERR_ARG, "null device");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    if (dev->ctx.pending) TRY(dev->ctx.sync());
    dev->ctx.pending = false;
    return TSN_OK;
}

int tsn_dispatch(tsn_device * dev, const char * kernel, const uint32_t grid[3], const uint32_t block[3],
                 const void * const * bufs, int nbufs, const void * params, size_t nparams) {
    if (!dev || !kernel) return fail(TSN_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    if (!c.pending) { CKR(cudaEventRecord(c.ev0, c.stream)); c.pending = true; }
    return compat_dispatch(c, kernel, grid, block, bufs, nbufs, params, nparams);
}

int tsn_commit(tsn_device * dev) {
    if (!dev) return fail(TSN_ERR_ARG, "null device");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    if (!c.pending) return TSN_OK;
    CKR(cudaEventRecord(c.ev1, c.stream));
    TRY(c.sync());
    float ms = 0.0f;
    CKR(cudaEventElapsedTime(&ms, c.ev0, c.ev1));
    c.last_ms = ms;
    c.pending = false;
    return TSN_OK;
}

uint32_t tsn_exec_width(tsn_device * dev, const char * kernel) {
    return dev && kernel && compat_has(kernel) ? 32u : 0u;
}

double tsn_last_gpu_ms(tsn_device * dev) { return dev ? dev->ctx.last_ms : 0.0; }

int tsn_selftest_device_timeout(tsn_device * dev, uint32_t limit_us) {
    if (!dev) return fail(TSN_ERR_ARG, "null device");
    if (limit_us < 100 || limit_us > 1000000) return fail(TSN_ERR_ARG, "limit must lie in [100 us, 1 s]");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    TRY(c.sync());    // a timeout reported below is this call's own
    CKR(launch_wait_selftest(c.d_err, 1000ull * limit_us, c.stream));
    return c.sync();
}

int tsn_selftest_gemm_lo8(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias, uint32_t M,
                          uint32_t N, uint32_t K, int wexp, int mode, int bn, int reps, float * ms) {
    if (!dev) return fail(TSN_ERR_ARG, "null device");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    TRY(c.sync());
    return selftest_gemm_lo8(c, W, X, Y, bias, M, N, K, wexp, mode, bn, reps, ms);
}

int tsn_selftest_gemv_jobs(tsn_device * dev, const void * W, const void * bias, const void * x, void * Y,
                           const uint32_t * N, int njobs, uint32_t K, int nb, int nb_cap, int act, int blocks, int tc) {
    if (!dev || !W || !x || !Y || !N) return fail(TSN_ERR_ARG, "null argument");
    if (njobs < 1 || njobs > 64 || blocks < 1 || act < 0 || act > 1) return fail(TSN_ERR_ARG, "bad job count, blocks or act");
    std::lock_guard<std::mutex> lk(dev->ctx.mu);
    DeviceCtx & c = dev->ctx;
    TRY(c.activate());
    long long total = 0;
    uint32_t max_n = 0;
    for (int q = 0; q < njobs; ++q) { total += N[q]; max_n = std::max(max_n, N[q]); }
    std::vector<GemvJob> jobs((size_t) njobs);
    long long row = 0;
    for (int q = 0; q < njobs; ++q) {
        jobs[(size_t) q] = GemvJob{(const __half *) W + row * K, bias ? (const float *) bias + row : nullptr,
                                   (const float *) x, (long long) K, nullptr, 0, (float *) Y + row, total,
                                   (int) N[q], (int) K, nb, act};
        row += N[q];
    }
    if (tc) {
        if (act || njobs > GEMV_MAX_JOBS) return fail(TSN_ERR_ARG, "the tensor-core GEMV takes no act and at most 16 jobs");
        CKR(launch_gemv_tc(jobs.data(), njobs, blocks, c.d_err, c.stream));
    } else {
        CKR(launch_gemv(jobs.data(), njobs, (int) max_n, nb_cap, blocks, 0, c.d_err, c.stream));
    }
    return c.sync();
}

// ------------------------------------------------------------------------------- runtime face
#define RT_BEGIN                                                         \
    if (!dev) return fail(TSN_ERR_ARG, "null device");                  \
    std::lock_guard<std::mutex> lk(dev->ctx.mu);                        \
    DeviceCtx & c = dev->ctx;                                            \
    TRY(c.activate());                                                   \
    if (!c.pending) { CKR(cudaEventRecord(c.ev0, c.stream)); c.pending = true; }

int tsn_gemm(tsn_device * dev, int wf16, const void * W, const void * X, void * Y, const void * bias,
             uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy) {
    RT_BEGIN
    return compat_gemm(c, wf16, W, X, Y, bias, M, N, K, ldx ? ldx : K, ldw ? ldw : K, ldy ? ldy : N);
}
int tsn_gemm_noalloc(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias,
                     uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy) {
    RT_BEGIN
    return gemm_noalloc(c, W, X, Y, bias, M, N, K, ldx ? ldx : K, ldw ? ldw : K, ldy ? ldy : N);
}
int tsn_gemv(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias, uint32_t N, uint32_t K,
             uint32_t ldw, int wf16) {
    RT_BEGIN
    return compat_gemv(c, wf16, W, X, Y, bias, N, K, ldw ? ldw : K);
}
int tsn_conv(tsn_device * dev, int wf16, const void * W, const void * bias, const void * x, void * y, uint32_t T,
             uint32_t OL, uint32_t IC, uint32_t OC, uint32_t K, uint32_t stride, uint32_t pad, uint32_t dil, int convt) {
    RT_BEGIN
    return compat_conv(c, wf16, W, bias, x, y, T, OL, IC, OC, K, stride, pad, dil, convt);
}
int tsn_silu(tsn_device * dev, void * x, size_t n) { RT_BEGIN return compat_elementwise(c, "silu_", x, nullptr, nullptr, n, 0, 0); }
int tsn_copy(tsn_device * dev, const void * x, void * y, size_t n) { RT_BEGIN return compat_elementwise(c, "copy_", x, nullptr, y, n, 0, 0); }
int tsn_swiglu(tsn_device * dev, const void * a, const void * b, void * y, size_t n) { RT_BEGIN return compat_elementwise(c, "swiglu_", a, b, y, n, 0, 0); }
int tsn_add(tsn_device * dev, const void * a, const void * b, void * y, size_t n) { RT_BEGIN return compat_elementwise(c, "add_", a, b, y, n, 0, 0); }
int tsn_add_bcast_col(tsn_device * dev, const void * x, const void * v, void * y, uint32_t S, uint32_t H) {
    RT_BEGIN return compat_elementwise(c, "add_bcast_col", x, v, y, (size_t) S * H, H, 0);
}
int tsn_cfg_euler(tsn_device * dev, const void * fc, const void * fu, void * x, size_t n, float cfg, float dt) {
    RT_BEGIN return compat_cfg_euler(c, fc, fu, x, n, cfg, dt);
}
int tsn_mean_cols(tsn_device * dev, const void * x, void * y, uint32_t S, uint32_t H) {
    RT_BEGIN return compat_mean_cols(c, x, y, S, H);
}

// ------------------------------------------------------------------------------- model face
static int new_model(tsn_device * dev, int compute_type, tsn_dit ** out, const std::string * path,
                     const tsn_dit_geom * g, uint64_t seed) {
    if (!dev || !out) return fail(TSN_ERR_ARG, "null argument");
    if (compute_type == TSN_COMPUTE_BF16)
        return fail(TSN_ERR_UNSUPPORTED, "BF16 operands are not provided: the reference's device weights are f16 and "
                                         "BF16 rounding of activations misses the 1e-3 flow gate; use TSN_COMPUTE_F16");
    if (compute_type != TSN_COMPUTE_F16) return fail(TSN_ERR_ARG, "bad compute type");
    *out = nullptr;
    TRY(dev->ctx.activate());
    auto m = std::make_unique<tsn_dit>();
    m->m.dev = &dev->ctx;
    m->m.bf16 = compute_type;
    DitGeom dg;
    if (g) {
        dg.H = g->H; dg.NH = g->NH; dg.F = g->F; dg.depth = g->depth; dg.fused_depth = g->fused_depth;
        dg.latent_dim = g->latent_dim; dg.rope_theta = g->rope_theta; dg.t_max_period = g->t_max_period;
    }
    std::string err;
    TRY(load_model(m->m, path, g ? &dg : nullptr, seed, err));
    *out = m.release();
    return TSN_OK;
}

int tsn_dit_load(tsn_device * dev, const char * path, int compute_type, tsn_dit ** out) {
    if (!path) return fail(TSN_ERR_ARG, "null path");
    std::string p(path);
    return new_model(dev, compute_type, out, &p, nullptr, 0);
}

int tsn_dit_inspect(const char * path, tsn_dit_geom * geom, size_t * weight_bytes) {
    if (!path) return fail(TSN_ERR_ARG, "null path");
    DitGeom g;
    size_t wb = 0;
    TRY(inspect_model(path, g, wb));
    if (geom) *geom = tsn_dit_geom{g.H, g.NH, g.F, g.depth, g.fused_depth, g.latent_dim, g.rope_theta, g.t_max_period};
    if (weight_bytes) *weight_bytes = wb;
    return TSN_OK;
}

int tsn_dit_load_synthetic(tsn_device * dev, const tsn_dit_geom * g, uint64_t seed, int compute_type, tsn_dit ** out) {
    if (!g) return fail(TSN_ERR_ARG, "null geometry");
    return new_model(dev, compute_type, out, nullptr, g, seed);
}

int tsn_dit_free(tsn_dit * m) {
    if (m) { if (m->m.dev) cudaStreamSynchronize(m->m.dev->stream); delete m; }
    return TSN_OK;
}

int tsn_dit_get_geom(tsn_dit * m, tsn_dit_geom * o) {
    if (!m || !o) return fail(TSN_ERR_ARG, "null argument");
    const DitGeom & g = m->m.g;
    *o = tsn_dit_geom{g.H, g.NH, g.F, g.depth, g.fused_depth, g.latent_dim, g.rope_theta, g.t_max_period};
    return TSN_OK;
}

size_t tsn_dit_weight_bytes(tsn_dit * m) { return m ? m->m.arena_used : 0; }

#define M_BEGIN                                                        \
    if (!m) return fail(TSN_ERR_ARG, "null model");                    \
    Model & M = m->m;                                                  \
    TRY(M.dev->activate());
#define NEED_PREPARED if (!M.prepared) return fail(TSN_ERR_STATE, "call tsn_dit_prepare first");

int tsn_dit_prepare(tsn_dit * m, uint32_t T, uint32_t C, uint32_t TS, uint32_t arms) {
    M_BEGIN
    return M.prepare((int) T, (int) C, (int) TS, (int) arms);
}

int tsn_dit_set_conditioning(tsn_dit * m, const float * clip_pp, const float * sync_gather, const float * text_pp,
                             const float * gcmlp) {
    M_BEGIN NEED_PREPARED
    const size_t H = M.g.H;
    cudaStream_t s = M.dev->stream;
    CKR(cudaMemcpyAsync(M.clip_pp, clip_pp, (size_t) M.G * M.C * H * 4, cudaMemcpyDefault, s));
    CKR(cudaMemcpyAsync(M.sync_gather, sync_gather, (size_t) M.G * M.T * H * 4, cudaMemcpyDefault, s));
    CKR(cudaMemcpyAsync(M.text_pp, text_pp, (size_t) M.B * M.TS * H * 4, cudaMemcpyDefault, s));
    CKR(cudaMemcpyAsync(M.gcmlp, gcmlp, (size_t) M.B * H * 4, cudaMemcpyDefault, s));
    CKR(cudaStreamSynchronize(s));
    return TSN_OK;
}

int tsn_dit_get_conditioning(tsn_dit * m, float * clip_pp, float * sync_gather, float * text_pp, float * gcmlp) {
    M_BEGIN NEED_PREPARED
    const size_t H = M.g.H;
    cudaStream_t s = M.dev->stream;
    if (clip_pp) CKR(cudaMemcpyAsync(clip_pp, M.clip_pp, (size_t) M.G * M.C * H * 4, cudaMemcpyDefault, s));
    if (sync_gather) CKR(cudaMemcpyAsync(sync_gather, M.sync_gather, (size_t) M.G * M.T * H * 4, cudaMemcpyDefault, s));
    if (text_pp) CKR(cudaMemcpyAsync(text_pp, M.text_pp, (size_t) M.B * M.TS * H * 4, cudaMemcpyDefault, s));
    if (gcmlp) CKR(cudaMemcpyAsync(gcmlp, M.gcmlp, (size_t) M.B * H * 4, cudaMemcpyDefault, s));
    return M.dev->sync();
}

int tsn_dit_prep_conditioning(tsn_dit * m, const float * clip_f, const float * sync_f, int sync_S) {
    M_BEGIN NEED_PREPARED
    if (!clip_f || !sync_f) return fail(TSN_ERR_ARG, "null argument");
    return M.prep_conditioning(clip_f, sync_f, sync_S);
}

int tsn_dit_prep_text_arm(tsn_dit * m, int arm, const float * text_cat, const float * gtext) {
    M_BEGIN NEED_PREPARED
    if (!text_cat || !gtext) return fail(TSN_ERR_ARG, "null argument");
    return M.prep_text_arm(arm, text_cat, gtext);
}

int tsn_dit_set_x(tsn_dit * m, const float * x) {
    M_BEGIN NEED_PREPARED
    CKR(cudaMemcpyAsync(M.x, x, (size_t) M.G * M.T * M.g.latent_dim * 4, cudaMemcpyDefault, M.dev->stream));
    CKR(cudaStreamSynchronize(M.dev->stream));
    return TSN_OK;
}

int tsn_dit_get_x(tsn_dit * m, float * x) {
    M_BEGIN NEED_PREPARED
    CKR(cudaMemcpyAsync(x, M.x, (size_t) M.G * M.T * M.g.latent_dim * 4, cudaMemcpyDefault, M.dev->stream));
    return M.dev->sync();
}

int tsn_dit_forward(tsn_dit * m, float t, float * flow_out) {
    M_BEGIN NEED_PREPARED
    TRY(M.set_time(t, 0.0f));
    CKR(cudaGraphLaunch(M.gx_fwd, M.dev->stream));
    if (flow_out)
        CKR(cudaMemcpyAsync(flow_out, M.flow, (size_t) M.B * M.T * M.g.latent_dim * 4, cudaMemcpyDefault, M.dev->stream));
    return M.dev->sync();
}

int tsn_dit_forward_taps(tsn_dit * m, float t, float * flow_out) {
    M_BEGIN NEED_PREPARED
    std::vector<Op> ops;
    TRY(M.build_ops(ops, 2, 0.0f));
    TRY(M.set_time(t, 0.0f));
    TRY(M.run_ops(ops, true));
    if (flow_out)
        CKR(cudaMemcpyAsync(flow_out, M.flow, (size_t) M.B * M.T * M.g.latent_dim * 4, cudaMemcpyDefault, M.dev->stream));
    return M.dev->sync();
}

static int read_tap(Model & M, const std::string & name, int arm, std::vector<float> & out) {
    auto it = M.taps.find(name);
    if (it == M.taps.end()) return fail(TSN_ERR_ARG, "no tap " + name + " (run tsn_dit_forward_taps)");
    std::vector<uint8_t> raw(it->second.bytes);
    CKR(cudaMemcpy(raw.data(), it->second.dev, raw.size(), cudaMemcpyDeviceToHost));
    it->second.convert(raw, arm, out);
    return TSN_OK;
}

int tsn_dit_tap(tsn_dit * m, const char * name, int arm, float * out, size_t n, size_t * len) {
    M_BEGIN NEED_PREPARED
    if (!name || arm < 0 || arm >= M.B) return fail(TSN_ERR_ARG, "bad tap name or arm");
    TRY(M.dev->sync());
    std::vector<float> v;
    if (std::string(name) == "a0_out") {   // joint attention output rows [lat | clip | text]
        std::vector<float> a, b, c;
        TRY(read_tap(M, "a0_out_l", arm, a));
        TRY(read_tap(M, "a0_out_c", arm, b));
        TRY(read_tap(M, "a0_out_t", arm, c));
        v = a; v.insert(v.end(), b.begin(), b.end()); v.insert(v.end(), c.begin(), c.end());
    } else {
        TRY(read_tap(M, name, arm, v));
    }
    if (len) *len = v.size();
    if (out) std::memcpy(out, v.data(), std::min(n, v.size()) * 4);
    return TSN_OK;
}

static int ensure_step_graph(Model & M, float cfg) {
    if (M.gx_step && M.step_cfg == cfg) return TSN_OK;
    TRY(M.build_ops(M.ops_step, 1, cfg));
    TRY(M.capture(M.ops_step, &M.gx_step));
    M.step_cfg = cfg;
    return TSN_OK;
}

int tsn_dit_step(tsn_dit * m, float t, float cfg, float dt) {
    M_BEGIN NEED_PREPARED
    if (M.A != 2) return fail(TSN_ERR_STATE, "tsn_dit_step needs both CFG arms (arms = 2 per generation)");
    TRY(ensure_step_graph(M, cfg));
    TRY(M.set_time(t, dt));
    CKR(cudaGraphLaunch(M.gx_step, M.dev->stream));
    return M.dev->sync();
}

// the pipeline's schedule (src/pipeline.cpp:142-145) into the model's t-embedding and dt tables
static int fill_schedule(Model & M, int steps) {
    std::vector<float> tb((size_t) steps * M.g.H), dts(steps);
    for (int s = 0; s < steps; ++s) {
        float t_curr = 1.0f - (float) s / steps;
        float t_prev = 1.0f - (float) (s + 1) / steps;
        dts[s] = t_prev - t_curr;
        M.temb_host(t_curr, tb.data() + (size_t) s * M.g.H);
    }
    CKR(cudaMemcpy(M.temb_tab, tb.data(), tb.size() * 4, cudaMemcpyHostToDevice));
    CKR(cudaMemcpy(M.dt_tab, dts.data(), dts.size() * 4, cudaMemcpyHostToDevice));
    CKR(cudaMemsetAsync(M.step, 0, 4, M.dev->stream));
    M.sched_steps = steps;
    return TSN_OK;
}

int tsn_dit_schedule(tsn_dit * m, int steps, float cfg) {
    M_BEGIN NEED_PREPARED
    if (M.A != 2) return fail(TSN_ERR_STATE, "the sampler needs both CFG arms (arms = 2 per generation)");
    if (steps < 1 || steps > M.max_steps) return fail(TSN_ERR_ARG, "steps out of range");
    TRY(ensure_step_graph(M, cfg));
    return fill_schedule(M, steps);
}

int tsn_dit_split_schedule(tsn_dit * m, int steps) {
    M_BEGIN NEED_PREPARED
    if (M.A != 1) return fail(TSN_ERR_STATE, "the CFG split runs one arm per device (arms = 1)");
    if (steps < 1 || steps > M.max_steps) return fail(TSN_ERR_ARG, "steps out of range");
    TRY(fill_schedule(M, steps));
    return M.dev->sync();
}

int tsn_dit_split_forward(tsn_dit * m, float * flow_dev) {
    M_BEGIN NEED_PREPARED
    if (M.A != 1 || !M.sched_steps) return fail(TSN_ERR_STATE, "call tsn_dit_split_schedule on a one-arm model first");
    if (!flow_dev) return fail(TSN_ERR_ARG, "null flow");
    TRY(M.run_ops(M.ops_fwd));
    CKR(cudaMemcpyAsync(flow_dev, M.flow, (size_t) M.T * M.g.latent_dim * 4, cudaMemcpyDeviceToDevice, M.dev->stream));
    return TSN_OK;
}

int tsn_dit_split_update(tsn_dit * m, const float * flows2_dev, float cfg) {
    M_BEGIN NEED_PREPARED
    if (M.A != 1 || !M.sched_steps) return fail(TSN_ERR_STATE, "call tsn_dit_split_schedule on a one-arm model first");
    if (!flows2_dev) return fail(TSN_ERR_ARG, "null flows");
    CKR(launch_cfg_euler(flows2_dev, M.x, M.T * (int) M.g.latent_dim, 1, cfg, M.dt_tab, M.step, 0.0f, M.dev->stream));
    CKR(launch_step_advance(M.step, M.dev->stream));
    return TSN_OK;
}

int tsn_dit_run_steps(tsn_dit * m, int n) {
    M_BEGIN NEED_PREPARED
    if (!M.gx_step) return fail(TSN_ERR_STATE, "call tsn_dit_schedule first");
    for (int i = 0; i < n; ++i) CKR(cudaGraphLaunch(M.gx_step, M.dev->stream));
    return TSN_OK;
}

int tsn_dit_sample(tsn_dit * m, int steps, float cfg) {
    TRY(tsn_dit_schedule(m, steps, cfg));
    TRY(tsn_dit_run_steps(m, steps));
    return m->m.dev->sync();
}

int tsn_dit_step_host(tsn_dit * m, const float * x_in, float * x_out, float t, float cfg, float dt) {
    M_BEGIN NEED_PREPARED
    if (M.A != 2) return fail(TSN_ERR_STATE, "tsn_dit_step_host needs both CFG arms (arms = 2 per generation)");
    TRY(ensure_step_graph(M, cfg));
    const size_t bytes = (size_t) M.G * M.T * M.g.latent_dim * 4;
    std::vector<float> tb(M.g.H);
    M.temb_host(t, tb.data());
    cudaStream_t s = M.dev->stream;
    CKR(cudaMemcpyAsync(M.x, x_in, bytes, cudaMemcpyHostToDevice, s));
    CKR(cudaMemcpyAsync(M.temb_tab, tb.data(), M.g.H * 4, cudaMemcpyHostToDevice, s));
    CKR(cudaMemcpyAsync(M.dt_tab, &dt, 4, cudaMemcpyHostToDevice, s));
    CKR(cudaMemsetAsync(M.step, 0, 4, s));
    CKR(cudaGraphLaunch(M.gx_step, s));
    CKR(cudaMemcpyAsync(x_out, M.x, bytes, cudaMemcpyDeviceToHost, s));
    return M.dev->sync();
}

int tsn_dit_kernels_per_step(tsn_dit * m) {
    if (!m || !m->m.prepared) return 0;
    int n = 0;
    for (const Op & o : m->m.ops_fwd) n += o.evkind == 0;
    return n + 2;
}

int tsn_dit_profile_step(tsn_dit * m, double * out5) {
    M_BEGIN NEED_PREPARED
    if (!out5) return fail(TSN_ERR_ARG, "null out");
    const std::vector<Op> & ops = M.ops_fwd;
    std::vector<cudaEvent_t> ev(ops.size() + 1);
    for (auto & e : ev) CKR(cudaEventCreate(&e));
    cudaStream_t s = M.dev->stream;
    CKR(cudaEventRecord(ev[0], s));
    for (size_t i = 0; i < ops.size(); ++i) {
        cudaError_t e = ops[i].fn(s);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, "launch " + ops[i].name + ": " + cudaGetErrorString(e));
        CKR(cudaEventRecord(ev[i + 1], s));
    }
    TRY(M.dev->sync());
    double t[3] = {0, 0, 0}, fl = 0, n = 0;
    for (size_t i = 0; i < ops.size(); ++i) {
        float ms = 0;
        CKR(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        t[ops[i].kind] += ms;
        if (ops[i].kind == 0) { fl += ops[i].flops; n += 1; }
    }
    for (auto & e : ev) cudaEventDestroy(e);
    out5[0] = t[0]; out5[1] = t[1]; out5[2] = t[2]; out5[3] = fl; out5[4] = n;
    return TSN_OK;
}

int tsn_dit_profile_ops(tsn_dit * m, char * out, size_t cap) {
    M_BEGIN NEED_PREPARED
    const std::vector<Op> & ops = M.ops_fwd;
    std::vector<cudaEvent_t> ev(ops.size() + 1);
    for (auto & e : ev) CKR(cudaEventCreate(&e));
    cudaStream_t s = M.dev->stream;
    CKR(cudaEventRecord(ev[0], s));
    for (size_t i = 0; i < ops.size(); ++i) {
        cudaError_t e = ops[i].fn(s);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, "launch " + ops[i].name + ": " + cudaGetErrorString(e));
        CKR(cudaEventRecord(ev[i + 1], s));
    }
    TRY(M.dev->sync());
    std::string rep;
    char line[320];
    for (size_t i = 0; i < ops.size(); ++i) {
        float ms = 0;
        CKR(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        const double tf = ops[i].flops > 0 && ms > 0 ? ops[i].flops / (ms * 1e-3) / 1e12 : 0.0;
        snprintf(line, sizeof line, "%4zu %-14s %8.4f ms %8.1f TF/s  %s%sflops=%.0f\n", i, ops[i].name.c_str(), ms, tf,
                 ops[i].desc.c_str(), ops[i].desc.empty() ? "" : " ", ops[i].flops);
        rep += line;
    }
    for (auto & e : ev) cudaEventDestroy(e);
    if (out && cap) { std::strncpy(out, rep.c_str(), cap - 1); out[cap - 1] = 0; }
    return TSN_OK;
}

int tsn_dit_autotune(tsn_dit * m, char * report, size_t cap) {
    M_BEGIN NEED_PREPARED
    std::string rep;
    TRY(M.autotune(rep));
    if (report && cap) { std::strncpy(report, rep.c_str(), cap - 1); report[cap - 1] = 0; }
    return TSN_OK;
}

int tsn_dit_get_tiles(tsn_dit * m, int * out, int max_gemms, int * n_gemms) {
    M_BEGIN NEED_PREPARED
    int n = 0;
    for (const Op & o : M.ops_fwd) {
        if (o.kind != 0 || o.gemm_id < 0) continue;
        if (out && n < max_gemms) { out[3 * n] = o.gemm_id; out[3 * n + 1] = o.tile_bn; out[3 * n + 2] = o.tile_s; }
        ++n;
    }
    if (n_gemms) *n_gemms = n;
    return TSN_OK;
}

int tsn_dit_set_tiles(tsn_dit * m, const int * tiles, int n) {
    M_BEGIN NEED_PREPARED
    if (n < 0 || (n > 0 && !tiles)) return fail(TSN_ERR_ARG, "null tile table");
    std::map<int, std::pair<int, int>> t;
    for (int i = 0; i < n; ++i) t[tiles[3 * i]] = {tiles[3 * i + 1], tiles[3 * i + 2]};
    return M.set_tiles(t);
}

int tsn_dit_trace_op(tsn_dit * m, int op, unsigned long long * out, size_t max_ctas, int * n_ctas) {
    M_BEGIN NEED_PREPARED
    if (op < 0 || op >= (int) M.ops_fwd.size() || !M.ops_fwd[op].traced)
        return fail(TSN_ERR_ARG, "op is not a stamped launch");
    const Op & o = M.ops_fwd[op];
    const size_t slots = (size_t) o.trace_slots, n = (size_t) o.ctas * slots;
    unsigned long long * d = nullptr;
    CKR(cudaMalloc(&d, n * 8));
    CKR(cudaMemsetAsync(d, 0, n * 8, M.dev->stream));
    for (size_t i = 0; i < M.ops_fwd.size() && (int) i < op; ++i) M.ops_fwd[i].fn(M.dev->stream);   // inputs of op
    cudaError_t e = o.traced(M.dev->stream, d);
    int rc = e == cudaSuccess ? M.dev->sync() : fail(TSN_ERR_CUDA, cudaGetErrorString(e));
    if (!rc && out) {
        std::vector<unsigned long long> h(n);
        CKR(cudaMemcpy(h.data(), d, n * 8, cudaMemcpyDeviceToHost));
        const size_t rows = std::min((size_t) o.ctas, max_ctas);
        for (size_t r = 0; r < rows; ++r)
            for (size_t k = 0; k < (size_t) TRACE_SLOTS; ++k) out[r * TRACE_SLOTS + k] = k < slots ? h[r * slots + k] : 0;
    }
    cudaFree(d);
    if (n_ctas) *n_ctas = o.ctas;
    return rc;
}

int tsn_dit_timeline(tsn_dit * m, double * out, size_t max_rows, int * n_rows) {
    M_BEGIN NEED_PREPARED
    std::vector<double> rows;
    TRY(M.timeline(rows));
    const size_t n = rows.size() / 5;
    if (out) std::memcpy(out, rows.data(), std::min(n, max_rows) * 5 * sizeof(double));
    if (n_rows) *n_rows = (int) n;
    return TSN_OK;
}

int tsn_gguf_write_synthetic(const char * path, const tsn_dit_geom * g, uint64_t seed, int with_prep) {
    if (!path || !g) return fail(TSN_ERR_ARG, "null argument");
    DitGeom dg;
    dg.H = g->H; dg.NH = g->NH; dg.F = g->F; dg.depth = g->depth; dg.fused_depth = g->fused_depth;
    dg.latent_dim = g->latent_dim; dg.rope_theta = g->rope_theta; dg.t_max_period = g->t_max_period;
    std::string err;
    if (!write_synthetic_gguf(path, dg, seed, with_prep != 0, err)) return fail(TSN_ERR_IO, err);
    return TSN_OK;
}

int tsn_gguf_write_synthetic_vae(const char * path, uint32_t latent_dim, uint32_t channels, uint32_t out_channels,
                                 uint64_t seed) {
    if (!path || latent_dim == 0 || channels == 0 || out_channels == 0) return fail(TSN_ERR_ARG, "bad VAE geometry");
    VaeGeom v;
    v.latent_dim = latent_dim; v.channels = channels; v.out_channels = out_channels;
    std::string err;
    if (!write_synthetic_vae_gguf(path, v, seed, err)) return fail(TSN_ERR_IO, err);
    return TSN_OK;
}

} // extern "C"
