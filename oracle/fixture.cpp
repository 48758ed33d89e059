// fixture.cpp — TEST INFRASTRUCTURE: the seeded synthetic DiT GGUF writer, exported from
// liboracle.so so that the CPU arms (bench.py --impl reference, the CPU baseline) can write their
// weight file without loading the GPU library. The writer itself is the package's host-only
// GGUF code (gguf_io.cpp, dit_schema.cpp), compiled into this library as well; the values come
// from include/tsn_synth.h, so the file is byte-identical to the one tsn_gguf_write_synthetic
// writes and to the weights tsn_dit_load_synthetic generates on the device.
#include <string>

#include "../thinksound-native_b200/csrc/gguf_io.h"

extern "C" {

// Same arguments as tsn_gguf_write_synthetic (include/tsn.h), geometry spelled out.
// Returns 0 on success, -1 on an I/O error (message to stderr).
int oracle_write_synthetic_gguf(const char * path, unsigned H, unsigned NH, unsigned F, unsigned depth,
                                unsigned fused_depth, unsigned latent_dim, float rope_theta, float t_max_period,
                                unsigned long long seed, int with_prep) {
    tsn::DitGeom g;
    g.H = H; g.NH = NH; g.F = F; g.depth = depth; g.fused_depth = fused_depth; g.latent_dim = latent_dim;
    g.rope_theta = rope_theta; g.t_max_period = t_max_period;
    std::string err;
    if (!tsn::write_synthetic_gguf(path, g, seed, with_prep != 0, err)) {
        fprintf(stderr, "oracle_write_synthetic_gguf: %s\n", err.c_str());
        return -1;
    }
    return 0;
}

} // extern "C"
