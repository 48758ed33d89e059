// compat.h — the reference's named kernels on CUDA, for the device/runtime faces of the C ABI.
//
// src/dit_fwd.cpp and src/net.mm dispatch Metal kernels by name with a raw constant block
// (src/gpu.h:34-38). compat_dispatch accepts exactly those names and byte layouts (listed in
// compat.cu) and runs a CUDA kernel with the same semantics on the device's stream, reading the
// buffers through their (managed or device) pointers. This is the drop-in path that lets the
// reference's own host code run unmodified; the fused fast path is the model face (model.cu).
#pragma once
#include <cstddef>
#include <cstdint>

#include "runtime.h"

namespace tsn {

bool compat_has(const char * name);
int compat_dispatch(DeviceCtx & c, const char * name, const uint32_t grid[3], const uint32_t block[3],
                    const void * const * bufs, int nbufs, const void * params, size_t nparams);
int compat_gemm(DeviceCtx & c, int wf16, const void * W, const void * X, void * Y, const void * bias,
                uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw, uint32_t ldy);
int compat_gemv(DeviceCtx & c, int wf16, const void * W, const void * X, void * Y, const void * bias,
                uint32_t N, uint32_t K, uint32_t ldw);
int compat_conv(DeviceCtx & c, int wf16, const void * W, const void * bias, const void * x, void * y,
                uint32_t T, uint32_t OL, uint32_t IC, uint32_t OC, uint32_t K, uint32_t stride, uint32_t pad,
                uint32_t dil, int convt);
// name: silu_ (a in place), copy_ (a -> y), swiglu_/add_ (a, b -> y), add_bcast_col (a + b[i % h] -> y)
int compat_elementwise(DeviceCtx & c, const char * name, const void * a, const void * b, void * y, size_t n,
                       uint32_t h, int unused);
int compat_cfg_euler(DeviceCtx & c, const void * fc, const void * fu, void * x, size_t n, float cfg, float dt);
int compat_mean_cols(DeviceCtx & c, const void * x, void * y, uint32_t S, uint32_t H);

} // namespace tsn
