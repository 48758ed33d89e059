// oracle/ref_cpu_device.cpp — a CPU implementation of the reference's tn::gpu::Device
// (TEST INFRASTRUCTURE).
//
// Compiled only against the reference's own header (src/gpu.h, found with -I on the reference
// tree) by oracle/Makefile, into oracle/_ref/. It replaces src/gpu.mm (the Metal harness):
// buffers are zeroed host allocations (host pointer == "device" pointer, like Apple unified
// memory, src/gpu.h:13-18) and dispatch(name, ...) runs the scalar restatement of that Metal
// kernel from oracle/kernels.cpp immediately. Everything above it — src/net.mm (Runtime,
// WeightSet), src/dit.cpp, src/dit_fwd.cpp, src/gguf.cpp — is the reference's unmodified code.
#include "gpu.h"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "kernels.h"

namespace tn::gpu {

struct Impl {
    std::vector<void *> allocs;
    std::mutex mutex;
};

Device::~Device() {
    if (!impl_) return;
    for (void * p : impl_->allocs) std::free(p);
    delete impl_;
}

bool Device::init(const std::string &) {
    impl_ = new Impl();
    return true;
}

// src/gpu.mm:52-64: zero-length requests become 16 bytes; Metal shared buffers start zeroed.
Buf Device::alloc(size_t bytes) {
    std::lock_guard<std::mutex> lk(impl_->mutex);
    Buf b;
    if (bytes == 0) bytes = 16;
    const size_t rounded = (bytes + 63) & ~(size_t) 63;
    void * p = std::aligned_alloc(64, rounded);
    if (!p) return b;
    std::memset(p, 0, rounded);
    impl_->allocs.push_back(p);
    b.p = p;
    b.bytes = bytes;
    return b;
}

// src/gpu.mm:66-87: wrap never copies.
Buf Device::wrap(const void * p, size_t bytes) {
    Buf b;
    b.p = const_cast<void *>(p);
    b.bytes = bytes;
    return b;
}

void Device::begin() {}

void Device::dispatch(const std::string & kernel, uint32_t gx, uint32_t gy, uint32_t gz,
                      uint32_t tx, uint32_t ty, uint32_t tz,
                      const std::vector<const void *> & buffers,
                      const void * scalars, size_t scalar_bytes) {
    std::lock_guard<std::mutex> lk(impl_->mutex);
    oracle::Grid g{gx, gy, gz, tx, ty, tz};
    if (!oracle::dispatch(kernel.c_str(), g, buffers.data(), buffers.size(), scalars, scalar_bytes))
        fprintf(stderr, "cpu-device: kernel %s not found or params short\n", kernel.c_str());
}

// Dispatches already ran; commit only records the (zero) queue drain time.
void Device::commit() { last_gpu_ms_ = 0.0; }

uint32_t Device::exec_width(const std::string &) { return 32; }

} // namespace tn::gpu
