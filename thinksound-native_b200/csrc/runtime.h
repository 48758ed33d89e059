// runtime.h — host-side state behind the C ABI (include/tsn.h): the device context and the
// MMDiT model (weights in HBM, activation buffers, planned launches, CUDA graphs, taps).
#pragma once
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tsn.h"
#include "dit_schema.h"
#include "kernels.h"

namespace tsn {

int fail(int code, const std::string & msg);
void clear_error();

struct DeviceCtx {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    int * d_err = nullptr;           // device error word written by bounded waits
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    double last_ms = 0.0;
    bool pending = false;            // work issued since the last commit
    std::mutex mu;
    std::vector<void *> managed;     // tsn_alloc buffers (freed with the device)
    // tsn_wrap registrations of host memory: page-aligned [base, base + bytes) -> device address
    // (unregistered with the device)
    struct HostReg { size_t bytes; void * dev; };
    std::map<uintptr_t, HostReg> host_regs;
    // compat path scratch: f32 -> f16 operand staging, grown on demand
    void * scratch = nullptr;
    size_t scratch_bytes = 0;
    // runtime-face conv: im2col scratch of one chunk of output rows (at most 16 M floats)
    void * col = nullptr;
    size_t col_bytes = 0;
    int activate();                  // cudaSetDevice(ordinal)
    int check_device_error();        // after a sync: TSN_ERR_TIMEOUT if a kernel gave up
    int sync();                      // stream sync + device error word
};

struct Lin {
    uint16_t * w = nullptr;   // [N][taps*K_in] f16/bf16
    float * b = nullptr;      // [N] or null
    int N = 0, K_in = 0, taps = 1;
};

struct Blk {
    Lin ada, qkv, l1, w13, w2;
    float * qn = nullptr, * kn = nullptr;
    int chunks = 6;
    bool post = false, conv = true;
};

struct Op {
    std::function<cudaError_t(cudaStream_t)> fn;
    int kind = 2;          // 0 tensor-core GEMM, 1 attention, 2 other
    double flops = 0.0;
    std::string name;
    std::string desc;      // launch configuration, for profiles
    int gemm_id = -1;      // GEMM sequence number within the forward (kind 0)
    int tile_bn = 0, tile_s = 0;   // the GEMM's tile: width (2000 + NT: CTA pair) and K slices / cluster size
    std::string shape;     // GEMM shape key: ops with equal keys have the same candidate configs
    std::function<cudaError_t(cudaStream_t, unsigned long long *)> traced;   // launch with per-CTA stamps
    int ctas = 0;
    int trace_slots = TRACE_SLOTS;   // stamps per CTA of `traced` (GEMMs: TRACE_SLOTS; others: 3)
    double part_bytes = 0.0;         // partial-tile GEMMs: bytes of one K slice's f32 tile
    int stream = 0;        // 0 latent (the device stream), 1 clip, 2 text
    int evkind = 0;        // 0 kernel/copy, 1 record event `ev` on `stream`, 2 make `stream` wait on `ev`
    int ev = -1;
};

// Once-per-generation conditioning weights (DitModel::prep_conditioning / prep_text_arm,
// src/dit.cpp:55-192) in the reference's own layouts: linear [N][K], conv [OC][IC][K] f16 (the
// runtime face's im2col GEMM reads them as they are), biases and sync_pos_emb f32.
struct PrepW {
    float * sync_pos = nullptr;                         // [8][768]
    Lin sync0, sync_w1, sync_w3, sync_w2;               // conv k7 768->H; convmlp k3
    Lin clip0, clip_w1, clip_w3, clip_w2, clip_cond;    // linear 1024->H; convmlp k3; cond proj
    Lin text0, text_w1, text_w3, text_w2, text_cond;    // linear 2048->H; linear SwiGLU MLP; cond proj
    Lin g_w1, g_w3, g_w2;                               // global_cond_mlp
};

struct TapBuf {
    void * dev = nullptr;
    size_t bytes = 0;
    std::function<void(const std::vector<uint8_t> &, int, std::vector<float> &)> convert;
};

struct Model {
    DeviceCtx * dev = nullptr;
    DitGeom g;
    int bf16 = 0;
    Lin te0, te2, ain0, ain13, ain2, fada, fconv;
    // every latent adaLN modulation weight (joint blocks, fused blocks, final layer) in one
    // contiguous [N_all][H] matrix, so one GEMM per step computes all of them
    Lin mod_all;
    std::vector<int> mod_off;   // column offset of each block's 6H chunk (joint then fused), final last
    std::vector<Blk> jl, jc, jt, fb;
    void * arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    // the weights' source, for the once-per-generation conditioning weights loaded on first use
    std::string src_path;             // GGUF path, or empty for the synthetic generator
    uint64_t src_seed = 0;
    PrepW pw;
    void * prep_arena = nullptr;
    bool prep_loaded = false;
    float * clip_fc = nullptr;        // [H] clip_cond_proj(mean clip_pp) of the current generation
    bool clip_fc_valid = false;
    int prep_conditioning(const float * clip_f, const float * sync_f, int sync_S);
    int prep_text_arm(int arm, const float * text_cat, const float * gtext);

    // geometry (tsn_dit_prepare)
    bool prepared = false;
    int T = 0, C = 0, TS = 0, B = 0, S = 0, S_pad = 0;
    int A = 2, G = 1;     // B = G generations x A CFG arms (A = 1: one arm of a CFG split)

    std::vector<void *> act;
    float * x = nullptr, * clip_pp = nullptr, * sync_gather = nullptr, * text_pp = nullptr, * gcmlp = nullptr;
    float * te_h = nullptr, * te = nullptr, * gc_silu = nullptr, * lat = nullptr, * clip_s = nullptr, * text_s = nullptr;
    float * modl = nullptr, * modc = nullptr, * modt = nullptr, * flow = nullptr;   // modl: [B][T][N_all]
    __half * x16 = nullptr, * extc16 = nullptr, * xn_l = nullptr, * xn_c = nullptr, * xn_t = nullptr;
    __half * att_l = nullptr, * att_c = nullptr, * att_t = nullptr, * h_l = nullptr, * h_c = nullptr, * h_t = nullptr;
    float * part_l = nullptr, * part_c = nullptr, * part_t = nullptr;   // [MAX_PARTS][B][rows][H] split-K partials
    __half * q = nullptr, * k = nullptr, * v = nullptr;
    float2 * rope_l = nullptr, * rope_c = nullptr;
    float * temb_tab = nullptr, * dt_tab = nullptr;
    int * step = nullptr;
    int max_steps = 1024;
    std::vector<GemvJob> jobs;     // t-embed MLP, then the clip/text modulations of every joint block
    int n_mod_jobs = 0;
    float * tap_gc = nullptr, * tap_extc = nullptr;
    std::map<std::string, TapBuf> taps;

    // GEMM configuration overrides by GEMM sequence number in the forward: (tile width, splits)
    std::map<int, std::pair<int, int>> gemm_force;
    int gemm_seq = 0;
    std::vector<Op> ops_fwd, ops_step;
    cudaGraphExec_t gx_fwd = nullptr, gx_step = nullptr;
    float step_cfg = 0.0f;
    int sched_steps = 0;

    ~Model();
    void * arena_take(size_t bytes);
    int prepare(int T, int C, int TS, int B);
    int build_ops(std::vector<Op> & ops, int mode, float cfg);   // mode 0 forward, 1 step, 2 taps
    // serial: every op on the device stream in list order (taps, profiles); otherwise the clip and
    // text streams run on their own CUDA streams, joined by events
    int run_ops(const std::vector<Op> & ops, bool serial = false);
    int ensure_streams();
    cudaStream_t side[2] = {nullptr, nullptr};
    std::vector<cudaEvent_t> events;
    int n_events = 0;
    int capture(const std::vector<Op> & ops, cudaGraphExec_t * out);
    int autotune(std::string & report);
    int set_tiles(const std::map<int, std::pair<int, int>> & tiles);   // pin tiles, re-plan, re-capture
    int timeline(std::vector<double> & rows);
    int set_time(float t, float dt);
    void temb_host(float t, float * out) const;
    mutable std::vector<float> temb_fr;   // temb_host's frequencies (the geometry's, computed on first use)
    void release_activations();
};

int load_model(Model & m, const std::string * gguf_path, const DitGeom * synth_geom, uint64_t seed, std::string & err);
int load_prep(Model & m);   // loads PrepW from the model's source on first use
// Host-only check of a DiT GGUF: geometry and every tensor the forward reads (no device needed).
int inspect_model(const std::string & path, DitGeom & g, size_t & weight_bytes);

} // namespace tsn

struct tsn_device { tsn::DeviceCtx ctx; };   // the C ABI's device handle (include/tsn.h)
