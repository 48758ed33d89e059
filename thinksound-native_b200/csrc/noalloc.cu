// noalloc.cu — tsn_gemm_noalloc: the runtime-face GEMM with no device allocation.
//
// Some callers cannot call cudaMalloc once they are running: an audio host's real-time render
// thread (cudaMalloc may take a device-wide lock and synchronise the GPU in the middle of a
// callback), or a process whose device memory was divided up front by another framework's pool
// allocator. tsn_gemm converts X into a split f16 operand in a scratch buffer it grows with
// cudaMalloc; this variant keeps that scratch in a fixed file-scope device array instead, so a
// call never allocates. The array is NOALLOC_SCRATCH_BYTES (8 MiB) per device, held by every GPU
// that loads the library until the process exits.
#include <mutex>

#include "kernels.h"
#include "runtime.h"

namespace tsn {

constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t) 8 << 20;

namespace {

// Host code must not take this symbol's address directly: on the host it names a stand-in, not
// device memory. Its device address comes from cudaGetSymbolAddress (scratch_address below).
__device__ __align__(256) uint8_t g_scratch[NOALLOC_SCRATCH_BYTES];

// f32 [M][ldx] -> split f16 operand: hi [M][K] at out, lo [M][K] right after it
__global__ void k_split_operand(const float * x, uint32_t M, uint32_t K, uint32_t ldx, __half * out) {
    const long long n = (long long) M * K;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const uint32_t m = (uint32_t) (i / K), k = (uint32_t) (i % K);
        const float v = x[(size_t) m * ldx + k];
        const __half h = __float2half_rn(v);
        out[i] = h;
        out[i + n] = __float2half_rn(v - __half2float(h));
    }
}

std::mutex g_mu;
// Device address of g_scratch, per device ordinal, looked up once. The cache belongs to the
// device's primary context: after cudaDeviceReset on a device the module is loaded anew and the
// cached address is stale, so a process that resets a device must not call tsn_gemm_noalloc on it
// again.
void * g_addr[64] = {};

int scratch_address(int ordinal, void ** out) {
    if (ordinal < 0 || ordinal >= 64) return fail(TSN_ERR_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[ordinal]) {
        void * p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);   // the calling thread has this device current
        if (e != cudaSuccess || !p)
            return fail(TSN_ERR_CUDA, std::string("static scratch address lookup: ") + cudaGetErrorString(e));
        g_addr[ordinal] = p;
    }
    *out = g_addr[ordinal];
    return TSN_OK;
}

} // namespace

int gemm_noalloc(DeviceCtx & c, const void * W, const void * X, void * Y, const void * bias, uint32_t M, uint32_t N,
                 uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy) {
    if (M == 0 || N == 0) return TSN_OK;
    if (!W || !X || !Y) return fail(TSN_ERR_ARG, "null operand");
    if (K % 64 || N % 64) return fail(TSN_ERR_ARG, "tsn_gemm_noalloc needs K and N to be multiples of 64");
    if (ldx < K || ldw < K || ldy < N || (ldw * 2) % 16 || ((uintptr_t) W & 15))
        return fail(TSN_ERR_ARG, "tsn_gemm_noalloc: bad leading dimension or unaligned weights");
    const size_t xa_bytes = ((size_t) 2 * M * K * 2 + 255) & ~(size_t) 255;
    const size_t need = xa_bytes + (ldw != K ? (size_t) N * K * 2 : 0);
    if (need > NOALLOC_SCRATCH_BYTES)
        return fail(TSN_ERR_ARG, "tsn_gemm_noalloc: operands need " + std::to_string(need) +
                                     " bytes of scratch, more than its fixed 8 MiB (4*M*K, plus 2*N*K when ldw != K)");
    void * base = nullptr;
    int rc = scratch_address(c.ordinal, &base);
    if (rc) return rc;
    __half * xa = (__half *) base;
    const long long n = (long long) M * K;
    const unsigned blocks = (unsigned) std::min<long long>((n + 255) / 256, 4096);
    k_split_operand<<<blocks, 256, 0, c.stream>>>((const float *) X, M, K, ldx, xa);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("split operand: ") + cudaGetErrorString(e));
    const void * wd = W;
    if (ldw != K) {
        wd = (char *) base + xa_bytes;
        e = cudaMemcpy2DAsync((void *) wd, (size_t) K * 2, W, (size_t) ldw * 2, (size_t) K * 2, N, cudaMemcpyDefault, c.stream);
        if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("pack weights: ") + cudaGetErrorString(e));
    }
    const int bn = N % 256 == 0 ? 256 : N % 128 == 0 ? 128 : 64;
    GemmLaunch g{};
    g.bn = bn; g.epi = EPI_F32; g.split = true; g.smem = gemm_smem_bytes(bn, true, EPI_F32); g.ab_bf16 = 0;
    g.grid = dim3(N / bn, (M + 127) / 128, 1);
    if (!make_act_map(&g.ta, xa, K, M, 1, 128, 1, 0) || !make_act_map(&g.ta2, xa + n, K, M, 1, 128, 1, 0) ||
        !make_w_map(&g.tb, wd, K, N, bn, 0))
        return fail(TSN_ERR_CUDA, "tsn_gemm_noalloc: tensor maps");
    GemmArgs & a = g.args;
    a.rows = (int) M; a.B = 1; a.bt = 128; a.bb = 1; a.m_tiles_t = (int) ((M + 127) / 128); a.N = (int) N;
    a.k_blocks = (int) (K / 64); a.ic_blocks = (int) (K / 64); a.pad = 0; a.splits = 1; a.kb_per_split = a.k_blocks;
    a.err = c.d_err;
    a.bias = (const float *) bias;
    a.out = Y; a.ldo = ldy; a.out_bs = 0;
    e = launch_gemm(g, c.stream);
    if (e != cudaSuccess) return fail(TSN_ERR_CUDA, std::string("tsn_gemm_noalloc: ") + cudaGetErrorString(e));
    return TSN_OK;
}

} // namespace tsn
