// gguf_io.h — GGUF v2/v3 reader (mmap) and the synthetic-fixture writer.
//
// The reader parses the same container the reference reads (src/gguf.h:52-85,
// src/gguf.cpp:73-165): KV metadata, tensor infos, data section aligned to general.alignment
// (default 32). Unlike the reference it never converts on the host; the loader uploads the raw
// BF16/F16/F32 bytes and converts on the device.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "dit_schema.h"

namespace tsn {

struct GgufTensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0;
    const uint8_t * data = nullptr;
    uint64_t nbytes = 0;
    uint64_t nelem() const { uint64_t n = 1; for (uint32_t d = 0; d < n_dims; ++d) n *= ne[d]; return n; }
};

class Gguf {
public:
    ~Gguf();
    // Returns false and fills err on a missing file, bad magic, unsupported version,
    // truncated header or a tensor whose data runs past the end of the file.
    bool open(const std::string & path, std::string & err);
    bool has(const std::string & key) const { return num_.count(key) != 0; }
    double num(const std::string & key, double def) const;
    const GgufTensorInfo * find(const std::string & name) const;
    const std::map<std::string, GgufTensorInfo> & tensors() const { return tensors_; }

private:
    void * map_ = nullptr;
    uint64_t len_ = 0;
    std::map<std::string, double> num_;
    std::map<std::string, GgufTensorInfo> tensors_;
};

// Write the seeded synthetic DiT fixture (values from include/tsn_synth.h) as GGUF v3.
bool write_synthetic_gguf(const std::string & path, const DitGeom & g, uint64_t seed, bool with_prep,
                          std::string & err);
// The seeded synthetic VAE decoder fixture (f32 tensors of vae_schema).
bool write_synthetic_vae_gguf(const std::string & path, const VaeGeom & v, uint64_t seed, std::string & err);
// The seeded synthetic text encoders (t5_schema: Q8_0 matrices; clip_schema: f32).
bool write_synthetic_t5_gguf(const std::string & path, const T5Geom & g, uint64_t seed, std::string & err);
bool write_synthetic_clip_gguf(const std::string & path, const ClipGeom & g, uint64_t seed, std::string & err);

// Fill dst with the synthetic values of one tensor (F32 values, BF16 bits or Q8_0 blocks by spec.type).
void synth_fill_host(const TensorSpec & spec, uint64_t seed, void * dst);

} // namespace tsn
