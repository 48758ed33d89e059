// kernels.h — host-side launch wrappers of the DiT path's device kernels (see kernels.cu,
// gemm.cu). All launches are asynchronous on the given stream; none allocates.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <utility>

#include "gemm_tc.cuh"

namespace tsn {

// Launch with programmatic stream serialisation (the kernel may start while its predecessor on
// the stream runs; it calls pdl_wait() before touching upstream data) and an optional thread-block
// cluster shape. Setting TSN_NO_PDL in the environment launches with plain stream order instead.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_cl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, dim3 cluster,
                      Args &&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cluster of cluster_z CTAs along z (the split-K clusters)
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, unsigned cluster_z,
                      Args &&... args) {
    return launch_cl(kernel, grid, block, smem, s, dim3(1, 1, cluster_z), std::forward<Args>(args)...);
}

// ---- GEMM / implicit conv (gemm.cu) ----
struct GemmLaunch {
    CUtensorMap ta, ta2, tb, tb2; // A (hi), A lo half (split operands only), weights, weights' lo half (WS)
    CUtensorMap to;               // f32 output view of the CTA-pair kernel when GemmArgs::tma_out
    GemmArgs args;
    dim3 grid;
    int bn = 0, epi = 0, ab_bf16 = 0;
    bool split = false;
    bool persistent = false;      // gemm_tc_persistent (f32 out, split A, one CTA per SM over many tiles)
    int pair_nt = 0;              // > 0: gemm2_kernel (CTA pairs, weights on M) with NT-token tiles
    size_t smem = 0;
};
// Encode a 3-D TMA view {K_in, rows, B} of a [B][rows][K_in] 16-bit activation buffer with a
// {64, bt, bb} box; bt * bb = 128, or fewer (a multiple of 8) with GemmArgs::a_rows = bt * bb.
bool make_act_map(CUtensorMap * m, const void * base, uint64_t K_in, uint64_t rows, uint64_t B,
                  uint32_t bt, uint32_t bb, int bf16);
// Encode a 3-D TMA view {64, rows, 2} of a head-major [hi|lo][rows][64] f16 q/k/v buffer with a
// {64, box_rows, 1} box (rows = B * NH * S_pad); the lo half starts lo_elems elements after the hi
// half (0: right after it, rows * 64).
bool make_head_map(CUtensorMap * m, const void * base, uint64_t rows, uint32_t box_rows, uint64_t lo_elems = 0);
// Encode a 4-D TMA view {N, rows, B, Z} of an f32 output out[z][b][t][n] (strides ldo, out_bs and
// z_stride elements) with {32, 32, 1, 1} boxes of 128-byte rows in the 128-byte swizzle.
bool make_out_map_f32(CUtensorMap * m, void * base, uint64_t N, uint64_t rows, uint64_t B, uint64_t Z, uint64_t ldo,
                      uint64_t out_bs, uint64_t z_stride);
// Encode a 2-D TMA view {K, N} of an [N][K] 16-bit weight matrix with a {64, bn} box.
bool make_w_map(CUtensorMap * m, const void * base, uint64_t K, uint64_t N, uint32_t bn, int bf16);
cudaError_t launch_gemm(const GemmLaunch & g, cudaStream_t s);
// split activations x split weights (gemm_ws_kernel; EPI_F32 or EPI_F16_SNAKE; bn 64, 128, 256)
cudaError_t launch_gemm_ws(const GemmLaunch & g, cudaStream_t s);
size_t gemm_ws_smem_bytes(int bn, int epi);
size_t gemm_ws_persistent_smem_bytes(int bn, int epi);   // GemmLaunch::persistent with the split-weight kernel
int gemm_ws_capacity(int bn, int epi, int cluster);
// A grouped launch of up to MAX_GROUP GEMMs sharing tile width, epilogue and operand split
// (gemm_tc_group): grid.x = args.cta_end[args.n - 1] CTAs, clusters of `cluster` along x.
struct GroupLaunch {
    GroupMaps maps;
    GroupArgs args;
    int bn = 0, epi = 0, ab_bf16 = 0;
    bool split = false;
    int cluster = 1;
    size_t smem = 0;
};
cudaError_t launch_gemm_group(const GroupLaunch & g, cudaStream_t s);
// grouped launches with a persistent shallow member (GroupArgs::persist_q): its tile width (0: no
// such kernel for this tile width / epilogue) and the launch's dynamic shared memory
int gemm_group_persist_bn(int bn, int epi, bool split);
size_t gemm_group_persist_smem_bytes(int bn, int epi, bool split);
cudaError_t configure_gemm_kernels();
int gemm_cluster_capacity(int bn, int epi, bool split, int cluster);
bool gemm_group_supported(int bn, int epi, bool split);   // a grouped instantiation exists
size_t gemm_smem_bytes(int bn, bool split, int epi);
size_t gemm_persistent_smem_bytes(int bn);   // 0: no persistent kernel for this tile width
size_t gemm2_smem_bytes(int nt, bool split);   // 0: no 2-SM kernel for this token tile
int gemm2_capacity(int nt, int epi, bool split);   // 2-SM CTAs that fit on the device at once
// Encode a 3-D TMA view {K_in, rows, B} of a [B][rows][K_in] f16 activation buffer with a
// {64, box_rows, 1} box (the 2-SM GEMM's half token tile).
bool make_act_map_rows(CUtensorMap * m, const void * base, uint64_t K_in, uint64_t rows, uint64_t B, uint32_t box_rows);
int gemm_stages(int bn, bool split, int epi);

// ---- attention (kernels.cu) ----
struct AttnArgs {
    const __half * q; const __half * k; const __half * v;   // [B][NH][S_pad][64]
    int B, NH, S, S_pad;
    float scale_log2;                                        // softmax scale * log2(e)
    // output streams: joint row s < n0 -> out0 row s; s < n0+n1 -> out1; else out2
    __half * out0; __half * out1; __half * out2;             // [B][n_i][H]
    int n0, n1, n2, H;
    long long qkv_lo;                                        // element offset of the lo halves of q, k, v
    long long out_lo0, out_lo1, out_lo2;                     // ... and of each output (0: hi only)
    unsigned long long * trace;                              // optional per-CTA stamps (entry, upstream done, exit)
    int * err;                                               // device error word (attn_tc_kernel)
    // optional additive logit bias in log2 units, [B][NH][S][S_pad] (key fastest; -inf masks a key):
    // the text encoders' T5 relative-position bias and pad mask, or CLIP's causal + EOT mask
    // (attn_short_kernel and attn_kernel)
    const float * lbias;
};
cudaError_t configure_attention();
cudaError_t launch_attention(const AttnArgs & a, cudaStream_t s);
// tcgen05 attention (attn_tc.cu): q/k/v read through TMA views made by make_head_map
struct AttnMaps { CUtensorMap q, k, v; };
cudaError_t configure_attention_tc();
cudaError_t launch_attention_tc(const AttnMaps & m, const AttnArgs & a, cudaStream_t s);
// tcgen05 attention for S <= 384 (attn_tc.cu, attn_short_kernel): every key tile resident, exact
// row maximum, no online rescaling; optional additive logit bias (AttnArgs::lbias). q map box 128
// rows, k and v maps box 64 rows.
cudaError_t configure_attention_short();
bool attention_short_fits(int S);
cudaError_t launch_attention_short(const AttnMaps & m, const AttnArgs & a, cudaStream_t s);

// ---- adaLN LayerNorm + modulation -> f16 GEMM operand ----
constexpr int MAX_PARTS = 12;   // most split-K partial tiles a gated GEMM leaves for the next adaLN
struct AdaLnArgs {
    float * x; long long x_bs;              // [B][rows][H] f32 residual stream
    const float * mod; long long mod_bs, mod_ld; int per_row, base;   // shift at base, scale at base + H
    __half * out; long long out_bs;         // [B][rows][H] f16, or null: apply the pending update only
    int B, rows, H;
    float eps;
    long long out_lo;                       // element offset of the lo half (0: hi only)
    unsigned long long * trace;             // optional per-CTA stamps (entry, upstream done, exit)
    // Pending gated residual update of the GEMM before (gate_add, shaders/ops_conv.metal:146-154),
    // applied to x first and written back: x += gate * (part[0] + ... + part[nsplit-1] + pbias).
    const float * part; long long part_stride; int nsplit;   // part[z][B][rows][H]; null: none
    const float * pbias;                                     // [H]
    const float * gmod; long long gmod_bs, gmod_ld; int gper_row, goff;   // gate rows, like mod; null: gate 1
    int x_zero;                                              // the update starts the stream: x's old contents unused
};
cudaError_t launch_adaln(const AdaLnArgs & a, cudaStream_t s);
// several streams' adaLNs (same H) in one launch; stream q owns blocks [end[q-1], end[q])
struct AdaLnGroup {
    AdaLnArgs p[MAX_GROUP];
    int n;
    int end[MAX_GROUP];
};
cudaError_t launch_adaln_group(const AdaLnGroup & g, cudaStream_t s);
int adaln_threads(int H);   // threads per row (one row per block), 0 when H is unsupported

// ---- batched GEMV y[b][n] = act(W[n,:]·x[b,:] + bias[n]) ----
struct GemvJob {
    const void * W; const float * bias;
    const float * x; long long x_bs;
    const int * x_step; long long x_step_stride;   // x += (*x_step) * stride when x_step != null
    float * y; long long y_bs;
    int N, K, nb, act;                             // act: 0 none, 1 silu
};
// Jobs of one launch, passed by value as a kernel parameter.
constexpr int GEMV_MAX_JOBS = 16;
struct GemvBatch {
    GemvJob j[GEMV_MAX_JOBS];
    int slot_end[GEMV_MAX_JOBS];   // set by launch_gemv: slots (row groups) of jobs 0..q
};
constexpr int GEMV_MAX_K = 1024;
// jobs: host array (copied into the launch's parameters; more than GEMV_MAX_JOBS take several
// launches), all sharing x (and x_step), x_bs, K and nb; nb: the kernel's arm capacity (1..8, every
// job's nb <= it); every N <= max_n; K <= GEMV_MAX_K and a multiple of 8, W 16-byte aligned with
// rows K apart; sms: the device's SM count (one block per SM at most); err: device error word for
// wait timeouts
cudaError_t configure_gemv();
// trace: optional per-block stamps (3 per block: entry, upstream done, exit) of the first launch;
// gemv_blocks gives its block count
cudaError_t launch_gemv(const GemvJob * jobs, int njobs, int max_n, int nb, int sms, int ab_bf16, int * err, cudaStream_t s,
                        unsigned long long * trace = nullptr);
int gemv_blocks(const GemvJob * jobs, int njobs, int nb, int sms);
// The same jobs on the tensor cores (gemv_tc.cu): weights as the M operand in 128-row tiles, the
// arms' split x as a resident 16-row N operand, one CTA per SM over all jobs' tiles. Jobs share x,
// x_bs, K (64..GEMV_MAX_K, a multiple of 64) and nb (<= 8); f16 weights; no x_step, no act.
cudaError_t configure_gemv_tc();
cudaError_t launch_gemv_tc(const GemvJob * jobs, int njobs, int sms, int * err, cudaStream_t s,
                           unsigned long long * trace = nullptr);
int gemv_tc_blocks(const GemvJob * jobs, int njobs, int sms);

// ---- per-forward conditioning prologue (src/dit_fwd.cpp:131-140, 166-167) ----
// B batch rows = G generations x A CFG arms (A = 2, or 1 for a single-arm model); the per-
// generation inputs (sync_gather, clip_pp, x) are indexed by generation b / A.
struct CondArgs {
    const float * te;            // [H]  t_embed output
    const float * gcmlp;         // [B][H]
    const float * sync_gather;   // [G][T][H]
    const float * clip_pp;       // [G][C][H]
    const float * text_pp;       // [B][TS][H]
    const float * x;             // [G][T][L]
    float * gc_silu;             // [B][H]
    __half * extc16;             // [B][T][H]  silu(sync_gather + gcmlp + te)
    float * clip_s;              // [B][C][H]
    float * text_s;              // [B][TS][H]
    __half * x16;                // [B][T][L]
    float * tap_gc;              // [B][H]     global_c before silu (nullable)
    float * tap_extc;            // [B][T][H]  extended_c before silu (nullable)
    int B, T, C, TS, H, L;
    long long extc_lo, x_lo;     // element offsets of the lo halves of extc16 and x16
    int A;                       // CFG arms per generation
};
// part 0: all of it; 1: global_c / extended_c (needs t_emb); 2: the clip/text restart and x's split operand
cudaError_t launch_cond(const CondArgs & a, cudaStream_t s, int part = 0);

// ---- x += dt * (fu + cfg * (fc - fu)) (src/pipeline.cpp:148, shaders/ops_conv.metal:194-201) ----
// x[g] += dt (fu + cfg (fc - fu)) for g < gens, with fc = flow[2g], fu = flow[2g + 1], n floats each.
// With parts: the flow is first formed from nparts partial slices (slice z at parts + z *
// part_stride, the same layout as flow) plus bias[e % C], summed in slice order, and written to flow.
cudaError_t launch_cfg_euler(const float * flow2, float * x, int n, int gens, float cfg, const float * dt_table,
                             const int * step, float dt_const, cudaStream_t s, const float * parts = nullptr,
                             long long part_stride = 0, int nparts = 0, const float * bias = nullptr, int C = 0);
// flow[e] = parts[0][e] + ... + parts[nparts-1][e] + bias[e % C] for e < n (the final conv's K slices)
cudaError_t launch_flow_sum(float * flow, long long n, const float * parts, long long part_stride, int nparts,
                            const float * bias, int C, cudaStream_t s);
cudaError_t launch_step_advance(int * step, cudaStream_t s);
// failure-path self-test: one thread waits on an mbarrier that nothing arrives on, bounded by
// limit_ns; records DEV_TIMEOUT_FULL in err when the bound runs out
cudaError_t launch_wait_selftest(int * err, unsigned long long limit_ns, cudaStream_t s);

// ---- weight preparation ----
// dst[n][tap*IC + ic] = cvt(src[row(n)][ic][tap]) for conv sources ([OC][IC][K], K=taps) or
// dst[n][k] = cvt(src[row(n)][k]) for linear sources (taps = 1). row(n) by mode:
//   0 identity; 1 qkv de-interleave (row j*Hq + c <- 3c + j); 2 w1/w3 interleave in [8 w1 | 8 w3]
//   row groups.
// src_type: 0 f32, 1 f16, 30 bf16 (GGUF types); out_bf16 selects the compute operand type.
cudaError_t launch_prep_weight(void * dst, const void * src, const void * src2, int src_type, int out_bf16,
                               long long N, int IC, int taps, int mode, int Hq, cudaStream_t s);
// f32 vector copy with optional qkv permutation (mode 1) from any GGUF float type.
cudaError_t launch_prep_vec(float * dst, const void * src, int src_type, long long n, int mode, int Hq, cudaStream_t s);
// synthetic tensor values, bit-identical to synth_fill_host (include/tsn_synth.h)
cudaError_t launch_synth(void * dst, long long n, uint64_t key, int type, int init, float scale, cudaStream_t s);

} // namespace tsn
