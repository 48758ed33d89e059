// dit_schema.h — the tensor inventory of the ThinkSound MMDiT GGUF and the synthetic fixture.
//
// Names, shapes (GGUF ne order: ne[0] fastest) and which tensors exist follow the reference's
// use of them: DitModel::forward (src/dit_fwd.cpp:104-304), DitModel::load (src/dit.cpp:29-46),
// prep_conditioning / prep_text_arm (src/dit.cpp:55-192) and the pipeline's empty features
// (src/pipeline.cpp:86-106). Linear weights [out,in] are ne = {in, out}; conv1d weights
// [OC,IC,K] are ne = {K, IC, OC} (src/net.h:109-110).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace tsn {

struct DitGeom {
    uint32_t H = 1024, NH = 16, F = 4096, depth = 21, fused_depth = 14, latent_dim = 64;
    float rope_theta = 10000.0f, t_max_period = 1.0f;
    uint32_t n_joint() const { return depth - fused_depth; }
    uint32_t hd() const { return H / NH; }
};

enum : uint32_t { GG_F32 = 0, GG_F16 = 1, GG_Q8_0 = 8, GG_BF16 = 30 };

struct TensorSpec {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = GG_BF16;
    int init = 0;          // tsn_init_kind
    float scale = 0.02f;
    uint64_t nelem() const { uint64_t n = 1; for (uint32_t d = 0; d < n_dims; ++d) n *= ne[d]; return n; }
};

// with_prep adds the once-per-generation conditioning weights (sync/clip/text projections,
// global_cond_mlp, empty features) that DitModel::prep_* and the pipeline read.
std::vector<TensorSpec> dit_schema(const DitGeom & g, bool with_prep);

// The VAE decoder (VaeModel::decode, src/vae.cpp:17-86): conv k7 latent -> 16C, five upsampling
// blocks (snake, transposed conv with kernel 2s at the strides below, three residual units with
// dilations 1, 3, 9), final snake and conv k7 C -> out_channels without bias. Widths follow the
// block order 16C, 8C, 4C, 2C, C, C. All tensors f32 (the reference keeps VAE weights in f32,
// src/vae.cpp:12-13); transposed-conv weights are stored converted, as the stride-1 conv kernel
// the reference applies to the zero-stuffed input.
struct VaeGeom {
    uint32_t latent_dim = 64, channels = 128, out_channels = 2;
};
constexpr uint32_t VAE_STRIDES[5] = {8, 8, 4, 4, 2};
constexpr uint32_t VAE_DILS[3] = {1, 3, 9};
inline uint32_t vae_width(const VaeGeom & v, int i) {   // channels after conv0 (i = 0) and block i
    static const uint32_t mult[6] = {16, 8, 4, 2, 1, 1};
    return v.channels * mult[i];
}
std::vector<TensorSpec> vae_schema(const VaeGeom & v);

// The T5 v1.1 text encoder (T5Model, src/t5.cpp:22-131): token embedding [32128, d_model], per
// layer RMSNorm gains, q/k/v/o [d,d], gated-GELU FFN wi_0/wi_1 [d_ff,d] and wo [d,d_ff], the
// relative-position bias table [n_bucket][NH] and the final RMSNorm. The reference's file is
// Q8_0 ("t5-q8.gguf", src/pipeline.cpp:62): matrices and the embedding are Q8_0 here too, norm
// gains and the bias table f32 (the bias is read as f32 by attn_qk, shaders/gemm_attn.metal:133-136).
struct T5Geom {
    uint32_t d_model = 2048, d_ff = 5120, layers = 24, heads = 32, rel_buckets = 32, rel_max_dist = 128;
};
constexpr uint32_t T5_VOCAB = 32128, T5_CTX = 77;
std::vector<TensorSpec> t5_schema(const T5Geom & g);

// The MetaCLIP text encoder (ClipModel, src/clip.cpp:6-123): token [49408, H] and position
// [ctx, H] embeddings, per layer LayerNorms, biased q/k/v/out [H,H], fc1 [4H,H], fc2 [H,4H], the
// final LayerNorm and the pooled projection text_proj [H,H]. All f32 ("metaclip-text-f32.gguf").
struct ClipGeom {
    uint32_t hidden = 1024, layers = 24, heads = 16, ctx = 77;
};
constexpr uint32_t CLIP_VOCAB = 49408;
std::vector<TensorSpec> clip_schema(const ClipGeom & g);

} // namespace tsn
