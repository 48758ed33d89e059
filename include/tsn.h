/* tsn.h — C ABI of the B200 (sm_100a) MMDiT denoising path of thinksound-native.
 *
 * Three faces, each replacing one layer of the reference (paths relative to the reference repo):
 *   device face   tsn_device_* / tsn_alloc / tsn_dispatch / tsn_commit   -> src/gpu.h Device (src/gpu.mm)
 *   runtime face  tsn_gemm / tsn_gemv / tsn_conv / tsn_cfg_euler ...     -> src/net.h Runtime (src/net.mm)
 *   model face    tsn_dit_*                                              -> src/models.h DitModel
 *                 (src/dit.cpp, src/dit_fwd.cpp) and the sampler loop of src/pipeline.cpp:126-155
 *
 * Conventions: every call returns TSN_OK (0) or a TSN_ERR_* code; tsn_last_error() gives the
 * message of the last failure on the calling thread. Pointers named *_dev are device (or
 * managed) addresses; *_host are host addresses; "any" pointers may be either (cudaMemcpyDefault).
 * All work is issued on the device's stream (tsn_device_set_stream); calls that return results to
 * the host synchronise that stream. No entry point falls back to the CPU: without a usable
 * sm_100 device every compute call fails with TSN_ERR_CUDA.
 */
#ifndef TSN_H
#define TSN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TSN_OK = 0,
    TSN_ERR_ARG = 1,          /* bad argument or unsupported geometry */
    TSN_ERR_CUDA = 2,         /* CUDA runtime/driver error, or no usable device */
    TSN_ERR_IO = 3,           /* file not found / unreadable */
    TSN_ERR_FORMAT = 4,       /* malformed GGUF */
    TSN_ERR_MISSING = 5,      /* a tensor the DiT needs is absent or mis-shaped */
    TSN_ERR_OOM = 6,          /* device allocation failed */
    TSN_ERR_UNSUPPORTED = 7,  /* kernel name or mode not provided by this build */
    TSN_ERR_TIMEOUT = 8,      /* a device-side wait gave up (kernel reported through the error word) */
    TSN_ERR_STATE = 9         /* call out of order (e.g. forward before prepare) */
};

/* Operand type of the tensor-core GEMMs. F16 matches the reference's device weights
 * (BF16 GGUF values converted with the reference's f32->f16 rule, src/net.mm:141-168). */
enum { TSN_COMPUTE_F16 = 0, TSN_COMPUTE_BF16 = 1 };

const char * tsn_last_error(void);
int tsn_version(void);

/* ------------------------------------------------------------------ device face (src/gpu.h) */
typedef struct tsn_device tsn_device;

/* Device::init (src/gpu.h:25). Binds CUDA device `ordinal`; creates a private stream. */
int tsn_device_create(int ordinal, tsn_device ** out);
/* Device::~Device (src/gpu.h:22). Frees every buffer tsn_alloc returned (the reference has no free). */
int tsn_device_destroy(tsn_device * dev);
/* Use an external cudaStream_t (e.g. the caller's framework stream) for all later work. */
int tsn_device_set_stream(tsn_device * dev, void * cuda_stream);
void * tsn_device_stream(tsn_device * dev);
/* Device::alloc (src/gpu.h:26, src/gpu.mm:52-64): zeroed managed memory, so the pointer is
 * valid on host and device like the reference's unified-memory Buf.p. 0 bytes -> 16 bytes. */
int tsn_alloc(tsn_device * dev, size_t bytes, void ** out);
/* Device::wrap (src/gpu.h:28, src/gpu.mm:66-87): register caller memory without copying. */
int tsn_wrap(tsn_device * dev, const void * p, size_t bytes, void ** out);
/* Device::begin (src/gpu.h:31). */
int tsn_begin(tsn_device * dev);
/* Device::dispatch (src/gpu.h:34-38): run the reference kernel `kernel` by name with its Metal
 * param block. grid/block are advisory (Metal threadgroup semantics); each kernel uses its own
 * CUDA launch geometry. Unknown names -> TSN_ERR_UNSUPPORTED (the reference logs and skips). */
int tsn_dispatch(tsn_device * dev, const char * kernel, const uint32_t grid[3], const uint32_t block[3],
                 const void * const * bufs, int nbufs, const void * params, size_t nparams);
/* Device::commit (src/gpu.h:39): synchronise the stream; records the queue time for last_gpu_ms. */
int tsn_commit(tsn_device * dev);
/* Device::exec_width (src/gpu.h:40): 32 for every provided kernel, 0 for unknown names. */
uint32_t tsn_exec_width(tsn_device * dev, const char * kernel);
/* Device::last_gpu_ms (src/gpu.h:41). */
double tsn_last_gpu_ms(tsn_device * dev);
/* No counterpart in the reference (a test hook for the failure path). Launches one block whose
 * thread waits on an mbarrier that nothing ever arrives on, bounded by limit_us (100 us .. 1 s), the
 * way every pipeline wait of this library is bounded. Expected result: TSN_ERR_TIMEOUT, with the
 * device still usable afterwards. */
int tsn_selftest_device_timeout(tsn_device * dev, uint32_t limit_us);
/* No counterpart in the reference (a test hook for an experimental GEMM, not used by any model
 * path). Y[M,N] = X·W^T (+bias) with X f32 [M][K], W f16 [N][K], Y f32 [M][N]. mode 0: X split into
 * an f16 high part on the f16 tensor path and its residual, scaled by 2^12, as e4m3 against an e4m3
 * copy of W scaled by 2^wexp (tile width bn 128, 176 or 256); mode 1: the library's split f16 GEMM
 * (bn 128 or 256); modes 2 and 3: a split f16 GEMM with K blocks of 64 or 32, so twice the stages
 * (bn 128, 176 or 256); mode + 4: the same without the L2-evicting write between launches. Operands are
 * prepared outside the timing; each of reps launches (1..100) is timed alone, and *ms (may be null)
 * receives the mean. K a multiple of 64.
 * Allocates its scratch; synchronises. */
int tsn_selftest_gemm_lo8(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias, uint32_t M,
                          uint32_t N, uint32_t K, int wexp, int mode, int bn, int reps, float * ms);
/* No counterpart in the reference (a test hook for the batched GEMV that carries the t-embedding
 * and every clip/text modulation of a step; each job is one Runtime::gemv, src/net.mm:51-56).
 * njobs jobs (1..64), job q: Y_q[b][n] = act(sum_k W_q[n][k] x[b][k] + bias_q[n]) for b < nb,
 * n < N[q]; act 0 none, 1 SiLU. W: the jobs' f16 rows of K back to back (job q from row sum N[<q]);
 * bias: f32, laid out the same way, or null; x: [nb][K] f32; Y: [nb][sum N] f32, job q's arm b at
 * b * sum N + sum N[<q]. K a multiple of 8 up to 1024; nb <= nb_cap <= 8 (the kernel instance's arm
 * capacity); blocks: the grid's cap (>= 1; results do not depend on it). tc = 1: the tensor-core form
 * the model uses for its modulation jobs (K a multiple of 64, act 0, at most 16 jobs; nb_cap unused).
 * Synchronises. */
int tsn_selftest_gemv_jobs(tsn_device * dev, const void * W, const void * bias, const void * x, void * Y,
                           const uint32_t * N, int njobs, uint32_t K, int nb, int nb_cap, int act, int blocks, int tc);

/* ------------------------------------------------------------------ runtime face (src/net.h) */
/* Runtime::gemm (src/net.h:23-24): Y[M,N] = X[M,K]·W[N,K]^T (+bias), X/Y f32, W f16 (wf16=1) or
 * f32 (wf16=0), leading dimensions in elements (0 = dense). */
int tsn_gemm(tsn_device * dev, int wf16, const void * W, const void * X, void * Y, const void * bias,
             uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy);
/* No counterpart in the reference. The same product as tsn_gemm with f16 weights, for callers
 * that must not allocate device memory once running: an audio host's real-time render thread
 * (cudaMalloc can take a device-wide lock and synchronise the GPU mid-callback) or a process
 * whose device memory another framework's pool allocator divided up front. tsn_gemm grows a
 * cudaMalloc'd scratch buffer for its split f16 copy of X; this entry point uses a fixed 8 MiB
 * device array inside the library instead and calls no allocator. Limits: K and N multiples of
 * 64, and 4*M*K bytes (plus 2*N*K when ldw != K) at most 8 MiB, else TSN_ERR_ARG. The first call
 * on each device looks up the array's device address; make that first call before any stream
 * capture begins; the looked-up address does not survive cudaDeviceReset of that device. Every
 * call on a device shares the one array: calls that overlap on the GPU (other streams, other
 * threads) race on it, so serialise them. */
int tsn_gemm_noalloc(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias,
                     uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy);
/* Runtime::gemv (src/net.h:25-26). */
int tsn_gemv(tsn_device * dev, const void * W, const void * X, void * Y, const void * bias,
             uint32_t N, uint32_t K, uint32_t ldw, int wf16);
/* Runtime::conv (src/net.h:29-31): conv1d of x [T,IC] with W (GGUF [K,IC,OC], i.e. [OC][IC][K]). */
int tsn_conv(tsn_device * dev, int wf16, const void * W, const void * bias, const void * x, void * y,
             uint32_t T, uint32_t OL, uint32_t IC, uint32_t OC, uint32_t K, uint32_t stride, uint32_t pad,
             uint32_t dil, int convt);
/* Runtime elementwise helpers (src/net.h:36-48). */
int tsn_silu(tsn_device * dev, void * x, size_t n);
int tsn_copy(tsn_device * dev, const void * x, void * y, size_t n);
int tsn_swiglu(tsn_device * dev, const void * a, const void * b, void * y, size_t n);
int tsn_add(tsn_device * dev, const void * a, const void * b, void * y, size_t n);
int tsn_add_bcast_col(tsn_device * dev, const void * x, const void * v, void * y, uint32_t S, uint32_t H);
/* Runtime::cfg_euler (src/net.h:46-47): x += dt·(fu + cfg·(fc − fu)). */
int tsn_cfg_euler(tsn_device * dev, const void * fc, const void * fu, void * x, size_t n, float cfg, float dt);
int tsn_mean_cols(tsn_device * dev, const void * x, void * y, uint32_t S, uint32_t H);

/* ------------------------------------------------------------------ model face (src/models.h) */
typedef struct tsn_dit tsn_dit;

typedef struct tsn_dit_geom {
    uint32_t H, NH, F, depth, fused_depth, latent_dim;
    float rope_theta, t_max_period;
} tsn_dit_geom;

/* DitModel::load (src/models.h:67, src/dit.cpp:29-46): read the GGUF, upload its BF16 tensors to
 * HBM and convert them there (qkv rows de-interleaved, conv weights reordered to [OC][K][IC],
 * FFN w1/w3 interleaved). compute_type: TSN_COMPUTE_F16 or TSN_COMPUTE_BF16. */
int tsn_dit_load(tsn_device * dev, const char * gguf_path, int compute_type, tsn_dit ** out);
/* Host-only check of a DiT GGUF, no device needed: DitModel::load's geometry keys
 * (src/dit.cpp:29-46) and every tensor the forward reads, present with its expected shape
 * (WeightSet::need, src/net.mm:110-118). TSN_ERR_IO (unreadable), TSN_ERR_FORMAT (bad magic,
 * version, truncated header or tensor table, tensor data past the end of the file;
 * src/gguf.cpp:73-151), TSN_ERR_MISSING (a tensor absent or mis-shaped), TSN_ERR_ARG (geometry
 * this build does not provide). tsn_dit_load fails with the same codes. geom and weight_bytes (the
 * device bytes the weights take) may be null. */
int tsn_dit_inspect(const char * gguf_path, tsn_dit_geom * geom, size_t * weight_bytes);
/* Same model from the seeded synthetic fixture generated on the device: bit-identical to loading
 * the file tsn_gguf_write_synthetic writes for the same geometry and seed. */
int tsn_dit_load_synthetic(tsn_device * dev, const tsn_dit_geom * g, uint64_t seed, int compute_type, tsn_dit ** out);
int tsn_dit_free(tsn_dit * m);
int tsn_dit_get_geom(tsn_dit * m, tsn_dit_geom * out);
size_t tsn_dit_weight_bytes(tsn_dit * m);

/* Fix the sequence geometry and allocate every activation buffer (src/dit.cpp:63-88):
 * T latent rows, clip_S clip rows, text_S text rows. arms = 2 runs one generation's cond and uncond
 * arms batched in one forward (CFG); arms = 2G (4, 6, 8) batches G independent generations, each
 * with its two arms (cond at 2g, uncond at 2g + 1), all stepping on the same schedule; arms = 1
 * runs a single arm (the 2-GPU CFG split). */
int tsn_dit_prepare(tsn_dit * m, uint32_t T, uint32_t clip_S, uint32_t text_S, uint32_t arms);

/* Per-generation conditioning, the outputs of DitModel::prep_conditioning / prep_text_arm
 * (src/dit.cpp:55-192): clip_pp [G][C,H], sync_gather [G][T,H] shared by a generation's arms;
 * text_pp [arms][TS,H] and gcmlp [arms][H] per arm (cond first). Any-pointers; copied in. */
int tsn_dit_set_conditioning(tsn_dit * m, const float * clip_pp, const float * sync_gather,
                             const float * text_pp, const float * gcmlp);
/* Read back the model's conditioning buffers (the layouts of tsn_dit_set_conditioning); any
 * pointer may be null to skip that buffer. */
int tsn_dit_get_conditioning(tsn_dit * m, float * clip_pp, float * sync_gather, float * text_pp, float * gcmlp);
/* DitModel::prep_conditioning (src/dit.cpp:55-135) on the GPU for the prepared geometry:
 * clip_f [C][1024] (C = the prepared clip rows) and sync_f [sync_S][768] f32, host or device
 * pointers. Writes the model's clip_pp and sync_gather and keeps clip_fc for the text arms.
 * Needs the once-per-generation conditioning weights in the model's source (loaded on first use)
 * and H = 1024; one generation (arms 1 or 2). */
int tsn_dit_prep_conditioning(tsn_dit * m, const float * clip_f, const float * sync_f, int sync_S);
/* DitModel::prep_text_arm (src/dit.cpp:137-192) for CFG arm `arm` (< the prepared arms):
 * text_cat [TS][2048] and gtext [1024] f32 -> the model's text_pp[arm] and gcmlp[arm].
 * After tsn_dit_prep_conditioning; together they replace tsn_dit_set_conditioning. */
int tsn_dit_prep_text_arm(tsn_dit * m, int arm, const float * text_cat, const float * gtext);

/* Latent x [G][T,64] (any-pointer in / out). */
int tsn_dit_set_x(tsn_dit * m, const float * x);
int tsn_dit_get_x(tsn_dit * m, float * x_out);

/* DitModel::forward (src/dit_fwd.cpp:104-304) for every arm at once at flow time t; writes
 * flow [arms][T,64] to flow_out (any-pointer). Runs as a replayed CUDA graph. */
int tsn_dit_forward(tsn_dit * m, float t, float * flow_out);
/* The same forward run eagerly, keeping the reference's per-tap tensors (src/dit_fwd.cpp:151-301). */
int tsn_dit_forward_taps(tsn_dit * m, float t, float * flow_out);
/* Copy tap `name` of arm `arm` from the last tsn_dit_forward_taps, in the reference's row-major
 * layout, into out (n floats at most). Returns the tap length through *len. */
int tsn_dit_tap(tsn_dit * m, const char * name, int arm, float * out, size_t n, size_t * len);

/* One sampler step (src/pipeline.cpp:146-148): both forwards + cfg_euler, x updated in place on the
 * device. Requires arms = 2. */
int tsn_dit_step(tsn_dit * m, float t, float cfg, float dt);
/* The Euler loop of src/pipeline.cpp:142-155 (t = 1 - s/steps, dt = t_{s+1} - t_s) over `steps`. */
int tsn_dit_sample(tsn_dit * m, int steps, float cfg);
/* Run `n` more steps of the schedule installed by the last tsn_dit_schedule (for timing loops). */
int tsn_dit_schedule(tsn_dit * m, int steps, float cfg);
int tsn_dit_run_steps(tsn_dit * m, int n);
/* The sampler with the CFG pair split over two GPUs (src/pipeline.cpp:142-155 with the cond and
 * uncond forwards of each step on different devices, arms = 1 on each), as three calls that only
 * issue work on the device's stream (no synchronisation, no host copies, no allocation), so that a
 * caller can capture a whole step, its own flow exchange included (e.g. an NCCL all-gather on the
 * same stream), in one CUDA graph and replay it. Make one eager step before capturing (it loads
 * kernels and creates the library's side streams); tsn_dit_split_schedule then rewinds.
 * tsn_dit_split_schedule: install the t / dt schedule of src/pipeline.cpp:142-145 for `steps` steps
 *   and rewind it to step 0 (synchronises; not for capture).
 * tsn_dit_split_forward: this arm's forward at the schedule's current step; its flow [T,64] f32 is
 *   copied to flow_dev (device memory).
 * tsn_dit_split_update: x += dt_s (fu + cfg (fc - fu)) with fc, fu = flows2_dev[0], flows2_dev[1]
 *   ([2][T,64] f32, device) and the current step's dt (shaders/ops_conv.metal:194-201), then advance
 *   the schedule one step. */
int tsn_dit_split_schedule(tsn_dit * m, int steps);
int tsn_dit_split_forward(tsn_dit * m, float * flow_dev);
int tsn_dit_split_update(tsn_dit * m, const float * flows2_dev, float cfg);
/* End-to-end step through host memory: copy x_host_in to the device, one step, copy x back. */
int tsn_dit_step_host(tsn_dit * m, const float * x_host_in, float * x_host_out, float t, float cfg, float dt);
/* Number of kernels one step (forward + cfg_euler + schedule advance) launches. */
int tsn_dit_kernels_per_step(tsn_dit * m);
/* Per-kernel-class device time of one eagerly launched step, measured with CUDA events around
 * each launch: out[0] tensor-core GEMM ms, out[1] attention ms, out[2] other ms, out[3] GEMM
 * FLOPs, out[4] GEMM launches. */
int tsn_dit_profile_step(tsn_dit * m, double * out5);
/* The same eager forward with one line per launch (name, device ms, TFLOP/s, tile configuration,
 * algorithmic FLOPs) written into out (NUL-terminated, truncated to cap). */
int tsn_dit_profile_ops(tsn_dit * m, char * out, size_t cap);

/* Run the forward up to stamped launch `op` (index in tsn_dit_profile_ops) and that launch once more
 * with per-CTA phase timestamps (globaltimer ns): entry, setup done, first stage landed,
 * accumulator complete, epilogue done, exit, first cluster barrier passed, cluster reduction
 * done (the last two 0 without split-K) — 8 per CTA into out (max_ctas CTAs). adaLN and
 * attention launches stamp entry, upstream wait passed and exit in the first 3 of the 8. */
int tsn_dit_trace_op(tsn_dit * m, int op, unsigned long long * out, size_t max_ctas, int * n_ctas);

/* Run one forward eagerly on the graph's streams with every GEMM, adaLN and attention launch
 * stamping its CTAs (globaltimer ns). Per stamped launch, 5 doubles into out (max_rows rows): op
 * index (as in tsn_dit_profile_ops), earliest CTA entry, earliest start of work (GEMM: first operand
 * stage landed; others: upstream wait passed), latest exit, median exit — in ns from the earliest
 * entry. n_rows receives the number of stamped launches. */
int tsn_dit_timeline(tsn_dit * m, double * out, size_t max_rows, int * n_rows);

/* Time every valid tile configuration (tile width, cluster split-K factor) of each distinct GEMM
 * shape of the prepared forward on this device and keep the fastest (the default is a static cost
 * model). Results stay bit-identical between calls of this model; two processes that tune
 * differently may differ in the last bits. Writes one line per shape into report. */
int tsn_dit_autotune(tsn_dit * m, char * report, size_t cap);

/* The tile of every GEMM launch of the planned forward, 3 ints each into out (max_gemms entries):
 * GEMM index, tile width (2000 + NT for the CTA-pair kernel with NT-token tiles) and K slices (the
 * cluster size, or the partial-tile count of the deepest member of a grouped launch). n_gemms
 * receives the count. Saving this table after tsn_dit_autotune and passing it to
 * tsn_dit_set_tiles later reproduces the tuned forward without re-timing. */
int tsn_dit_get_tiles(tsn_dit * m, int * out, int max_gemms, int * n_gemms);

/* Pin GEMM tiles (n triples as tsn_dit_get_tiles writes them) and re-plan the forward; GEMMs not
 * listed, and entries that do not fit their GEMM, fall back to the static cost model. */
int tsn_dit_set_tiles(tsn_dit * m, const int * tiles, int n);

/* ------------------------------------------------------------------ VAE decoder */
/* VaeModel::decode (src/vae.cpp:17-86) on the GPU: latent [T, latent_dim] f32 -> interleaved audio
 * [T * 2048, out_channels] f32. The f32 weights are held as f16 hi + lo halves (split-weight
 * tcgen05 GEMMs); transposed convs run as polyphase stride-1 convs. */
typedef struct tsn_vae tsn_vae;
/* Load from a VAE GGUF (the tensor names of src/vae.cpp; f32, f16 or bf16 values). */
int tsn_vae_load(tsn_device * dev, const char * gguf_path, tsn_vae ** out);
/* The seeded synthetic VAE (the values tsn_gguf_write_synthetic_vae writes), generated in memory. */
int tsn_vae_load_synthetic(tsn_device * dev, uint32_t latent_dim, uint32_t channels, uint32_t out_channels, uint64_t seed,
                           tsn_vae ** out);
/* Decode latent [T, latent_dim] into audio [T_audio, out_channels] (host or device pointers;
 * audio_cap in floats). The first decode of a length plans and captures its graph. */
int tsn_vae_decode(tsn_vae * v, const float * latent, uint32_t T, float * audio, size_t audio_cap, uint32_t * T_audio);
/* Device time of the last decode (ms, graph only) and the algorithmic FLOPs (2·M·N·K over every
 * conv) of the prepared length. */
double tsn_vae_last_ms(tsn_vae * v);
/* The last decoded length once more, launch by launch, one line per launch (name, device ms). */
int tsn_vae_profile_ops(tsn_vae * v, char * out, size_t cap);
double tsn_vae_flops(tsn_vae * v);
/* Kernel launches in one decode graph of the prepared length. */
int tsn_vae_launches(tsn_vae * v);
int tsn_vae_free(tsn_vae * v);

/* ------------------------------------------------------------------ text encoders */
/* T5Model (src/t5.cpp, src/models.h:40-52) and ClipModel (src/clip.cpp, src/models.h:24-38) on the
 * GPU, one handle type for both. Loading follows WeightSet::load with keep_f32 (src/net.mm:126-173):
 * f32 tensors stay f32 (split-weight GEMMs), others (the T5 file's Q8_0) become f16 by the
 * reference's rounding rule. Returns TSN_ERR_UNSUPPORTED unless the head size is 64. */
typedef struct tsn_encoder tsn_encoder;
/* Replaces T5Model::load (src/t5.cpp:22-59): KV keys t5.* with the reference's defaults. */
int tsn_t5_load(tsn_device * dev, const char * gguf_path, tsn_encoder ** out);
/* Replaces ClipModel::load (src/clip.cpp:6-28): KV keys clip.*. */
int tsn_clip_load(tsn_device * dev, const char * gguf_path, tsn_encoder ** out);
/* Width (d_model / hidden), context (77) and layer count. */
int tsn_encoder_info(tsn_encoder * e, uint32_t * width, uint32_t * ctx, uint32_t * layers);
/* Replaces T5Model::encode (src/t5.cpp:84-131) and ClipModel::encode (src/clip.cpp:30-101): n_ids
 * must equal ctx (ids already padded, as the tokenizers return them); every id must lie inside the
 * vocabulary (TSN_ERR_ARG otherwise; the reference would read past its table). per_token [ctx, width]
 * f32; pooled [width] (CLIP's text_proj of the EOT row; ignored for T5, may be null). Host or device
 * pointers. One CUDA graph per encoder. */
int tsn_encoder_encode(tsn_encoder * e, const int32_t * ids, uint32_t n_ids, float * per_token, size_t per_token_cap,
                       float * pooled, size_t pooled_cap);
/* Device time of the last encode (ms), its algorithmic FLOPs and the weight bytes it streams. */
double tsn_encoder_last_ms(tsn_encoder * e);
double tsn_encoder_flops(tsn_encoder * e);
/* Kernel launches in one encode graph. */
int tsn_encoder_launches(tsn_encoder * e);
double tsn_encoder_weight_bytes(tsn_encoder * e);
/* The encode's launches once more eagerly, one line per launch (name, device ms). */
int tsn_encoder_profile_ops(tsn_encoder * e, char * out, size_t cap);
int tsn_encoder_free(tsn_encoder * e);

/* ------------------------------------------------------------------ fixtures */
/* Write the seeded synthetic DiT GGUF (with_prep adds the conditioning-prep tensors). Host only. */
int tsn_gguf_write_synthetic(const char * path, const tsn_dit_geom * g, uint64_t seed, int with_prep);
/* Write the seeded synthetic VAE decoder GGUF (f32 tensors: conv k7 latent_dim -> 16 channels,
 * five upsampling blocks at strides 8, 8, 4, 4, 2 with widths 8, 4, 2, 1, 1 x channels, final conv
 * to out_channels; tensor names of src/vae.cpp). Host only. */
int tsn_gguf_write_synthetic_vae(const char * path, uint32_t latent_dim, uint32_t channels, uint32_t out_channels,
                                 uint64_t seed);
/* Write the seeded synthetic T5 encoder GGUF (Q8_0 matrices and embedding, f32 norms and relative
 * bias; tensor names and KV keys of src/t5.cpp; vocabulary 32128). Host only. */
int tsn_gguf_write_synthetic_t5(const char * path, uint32_t d_model, uint32_t d_ff, uint32_t layers, uint32_t heads,
                                uint64_t seed);
/* Write the seeded synthetic MetaCLIP text encoder GGUF (f32; names and keys of src/clip.cpp;
 * vocabulary 49408, context 77). Host only. */
int tsn_gguf_write_synthetic_clip(const char * path, uint32_t hidden, uint32_t layers, uint32_t heads, uint64_t seed);

#ifdef __cplusplus
}
#endif

#endif /* TSN_H */
