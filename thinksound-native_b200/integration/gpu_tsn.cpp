// gpu_tsn.cpp — the reference's device harness tn::gpu::Device (declared in its src/gpu.h:20-49)
// implemented over libtsn's C ABI: the drop-in replacement for src/gpu.mm.
//
// Compiled against the reference's own header, next to its unmodified host code (src/net.mm as
// C++, src/dit.cpp, src/dit_fwd.cpp, src/vae.cpp, src/t5.cpp, src/clip.cpp, src/gguf.cpp), it runs
// every named dispatch of that code (adaln_ln, qkv_split3, rms_head, rope_pairs, gate_add,
// attn_qk, softmax_rows, attn_pav, gemm_mpp_*, im2col, gemv_*, the elementwise kernels, ...) on
// the GPU with the reference's constant-block layouts. Buffers are managed memory, so Buf.p is
// both the host and the device address as on Apple unified memory (src/gpu.h:13-18).
//
// Error conventions of src/gpu.mm: init returns false on failure, alloc returns Buf{nullptr}, an
// unknown or failing dispatch is logged to stderr and skipped (src/gpu.mm:103,128-129), and
// commit waits for the queue (here: a stream synchronise that also reports a device-side wait
// that gave up).
#include "gpu.h"

#include <cstdio>

#include "tsn.h"

namespace tn::gpu {

struct Impl {
    tsn_device * d = nullptr;
};

Device::~Device() {
    if (!impl_) return;
    if (impl_->d) tsn_device_destroy(impl_->d);
    delete impl_;
}

bool Device::init(const std::string &) {
    if (!impl_) impl_ = new Impl();
    if (tsn_device_create(0, &impl_->d) != TSN_OK) {
        fprintf(stderr, "gpu: init failed: %s\n", tsn_last_error());
        impl_->d = nullptr;
        return false;
    }
    return true;
}

// src/gpu.mm:52-64: zero-length requests become 16 bytes; buffers start zeroed
Buf Device::alloc(size_t bytes) {
    Buf b;
    void * p = nullptr;
    if (!impl_ || !impl_->d) return b;
    if (tsn_alloc(impl_->d, bytes ? bytes : 16, &p) != TSN_OK) {
        fprintf(stderr, "gpu: alloc of %zu bytes failed: %s\n", bytes, tsn_last_error());
        return b;
    }
    b.p = p;
    b.bytes = bytes ? bytes : 16;
    return b;
}

// src/gpu.mm:66-87: no copy; the memory must stay alive
Buf Device::wrap(const void * p, size_t bytes) {
    Buf b;
    void * q = nullptr;
    if (!impl_ || !impl_->d || tsn_wrap(impl_->d, p, bytes, &q) != TSN_OK) return b;
    b.p = q;
    b.bytes = bytes;
    return b;
}

void Device::begin() {
    if (impl_ && impl_->d) tsn_begin(impl_->d);
}

void Device::dispatch(const std::string & kernel, uint32_t gx, uint32_t gy, uint32_t gz, uint32_t tx, uint32_t ty,
                      uint32_t tz, const std::vector<const void *> & buffers, const void * scalars, size_t scalar_bytes) {
    if (!impl_ || !impl_->d) return;
    const uint32_t g[3] = {gx, gy, gz}, t[3] = {tx, ty, tz};
    if (tsn_dispatch(impl_->d, kernel.c_str(), g, t, buffers.data(), (int) buffers.size(), scalars, scalar_bytes) != TSN_OK)
        fprintf(stderr, "gpu: dispatch %s skipped: %s\n", kernel.c_str(), tsn_last_error());
}

void Device::commit() {
    if (!impl_ || !impl_->d) return;
    if (tsn_commit(impl_->d) != TSN_OK) fprintf(stderr, "gpu: commit: %s\n", tsn_last_error());
    last_gpu_ms_ = tsn_last_gpu_ms(impl_->d);
}

uint32_t Device::exec_width(const std::string & kernel) {
    return impl_ && impl_->d ? tsn_exec_width(impl_->d, kernel.c_str()) : 0;
}

} // namespace tn::gpu
