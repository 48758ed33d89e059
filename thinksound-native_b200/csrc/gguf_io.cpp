// gguf_io.cpp — GGUF reader and synthetic-fixture writer (see gguf_io.h).
#include "gguf_io.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>

#include "../../include/tsn_synth.h"

namespace tsn {

Gguf::~Gguf() {
    if (map_) munmap(map_, len_);
}

static uint64_t type_size(uint32_t t) { return t == GG_F32 ? 4 : (t == GG_F16 || t == GG_BF16) ? 2 : 0; }
// bytes of a tensor's data: plain types, or Q8_0 blocks of 32 values (f16 scale + 32 int8), the
// only quantised type the reference reads (src/gguf.cpp:46,216-228); 0 for any other type
static uint64_t tensor_bytes(uint32_t t, uint64_t nelem) {
    if (t == GG_Q8_0) return nelem % 32 ? 0 : nelem / 32 * 34;
    return nelem * type_size(t);
}

bool Gguf::open(const std::string & path, std::string & err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { err = "cannot open " + path; return false; }
    struct stat st{};
    if (fstat(fd, &st) != 0) { ::close(fd); err = "cannot stat " + path; return false; }
    len_ = (uint64_t) st.st_size;
    map_ = len_ ? mmap(nullptr, len_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    ::close(fd);
    if (map_ == MAP_FAILED) { map_ = nullptr; err = "cannot map " + path; return false; }
    const uint8_t * p = (const uint8_t *) map_, * end = p + len_;
    bool bad = false;
    auto raw = [&](void * dst, uint64_t n) {
        if (bad || (uint64_t) (end - p) < n) { bad = true; return; }
        if (dst) memcpy(dst, p, n);
        p += n;
    };
    auto u32 = [&]() { uint32_t v = 0; raw(&v, 4); return v; };
    auto u64 = [&]() { uint64_t v = 0; raw(&v, 8); return v; };
    auto str = [&]() {
        uint64_t n = u64();
        if (bad || n > (uint64_t) (end - p)) { bad = true; return std::string(); }
        std::string s((const char *) p, (size_t) n);
        p += n;
        return s;
    };
    const uint32_t magic = u32();
    if (bad || magic != 0x46554747u) { err = "bad GGUF magic"; return false; }
    const uint32_t version = u32();
    if (version < 2 || version > 3) { err = "unsupported GGUF version " + std::to_string(version); return false; }
    const uint64_t n_t = u64(), n_kv = u64();
    if (bad) { err = "truncated GGUF header"; return false; }
    static const uint8_t ssz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    for (uint64_t i = 0; i < n_kv && !bad; ++i) {
        const std::string key = str();
        const uint32_t ty = u32();
        if (ty == 8) { str(); continue; }
        if (ty == 9) {
            const uint32_t et = u32();
            const uint64_t n = u64();
            for (uint64_t k = 0; k < n && !bad; ++k) {
                if (et == 8) str();
                else if (et < 13 && ssz[et]) raw(nullptr, ssz[et]);
                else bad = true;
            }
            continue;
        }
        if (ty >= 13 || !ssz[ty]) { bad = true; break; }
        uint8_t b[8] = {0};
        raw(b, ssz[ty]);
        double v = 0;
        switch (ty) {
            case 0: v = b[0]; break;
            case 1: v = (int8_t) b[0]; break;
            case 2: { uint16_t x; memcpy(&x, b, 2); v = x; } break;
            case 3: { int16_t x; memcpy(&x, b, 2); v = x; } break;
            case 4: { uint32_t x; memcpy(&x, b, 4); v = x; } break;
            case 5: { int32_t x; memcpy(&x, b, 4); v = x; } break;
            case 6: { float x; memcpy(&x, b, 4); v = x; } break;
            case 7: v = b[0] != 0; break;
            case 10: { uint64_t x; memcpy(&x, b, 8); v = (double) x; } break;
            case 11: { int64_t x; memcpy(&x, b, 8); v = (double) x; } break;
            case 12: { double x; memcpy(&x, b, 8); v = x; } break;
        }
        num_[key] = v;
    }
    if (bad) { err = "truncated or malformed GGUF metadata"; return false; }
    const uint64_t align = num_.count("general.alignment") ? (uint64_t) num_["general.alignment"] : 32;
    if (align == 0 || (align & (align - 1))) { err = "bad general.alignment"; return false; }
    for (uint64_t i = 0; i < n_t && !bad; ++i) {
        GgufTensorInfo t;
        t.name = str();
        t.n_dims = u32();
        if (t.n_dims > 4) { err = "tensor " + t.name + " has more than 4 dims"; return false; }
        for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = u64();
        t.type = u32();
        t.offset = u64();
        t.nbytes = tensor_bytes(t.type, t.nelem());
        tensors_[t.name] = t;
    }
    if (bad) { err = "truncated GGUF tensor table"; return false; }
    const uint64_t hdr = (uint64_t) (p - (const uint8_t *) map_);
    const uint64_t data_start = (hdr + align - 1) & ~(align - 1);
    for (auto & [name, t] : tensors_) {
        if (t.nbytes == 0) continue;   // types the reference cannot read either
        if (data_start + t.offset + t.nbytes > len_) { err = "tensor " + name + " runs past end of file"; return false; }
        t.data = (const uint8_t *) map_ + data_start + t.offset;
    }
    return true;
}

double Gguf::num(const std::string & key, double def) const {
    auto it = num_.find(key);
    return it == num_.end() ? def : it->second;
}

const GgufTensorInfo * Gguf::find(const std::string & name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

void synth_fill_host(const TensorSpec & s, uint64_t seed, void * dst) {
    const uint64_t key = tsn_stream_key(s.name.c_str(), seed);
    const uint64_t n = s.nelem();
    const unsigned nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    auto work = [&](unsigned t) {
        const uint64_t lo = n * t / nth, hi = n * (t + 1) / nth;
        if (s.type == GG_Q8_0) {
            // ggml's Q8_0 quantiser: per block of 32, d = max|x| / 127, q = round(x / d)
            uint8_t * o = (uint8_t *) dst;
            const uint64_t nb = n / 32, b0 = nb * t / nth, b1 = nb * (t + 1) / nth;
            for (uint64_t bk = b0; bk < b1; ++bk) {
                float x[32], amax = 0.0f;
                for (int k = 0; k < 32; ++k) {
                    x[k] = tsn_init_value(key, bk * 32 + k, s.init, s.scale);
                    amax = std::max(amax, std::fabs(x[k]));
                }
                const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
                const uint16_t d16 = tsn_ref_f32_to_f16(d);
                uint8_t * blk = o + bk * 34;
                std::memcpy(blk, &d16, 2);
                for (int k = 0; k < 32; ++k) {
                    const long q = std::lrint(x[k] * id);
                    blk[2 + k] = (uint8_t) (int8_t) std::max(-127L, std::min(127L, q));
                }
            }
            return;
        }
        if (s.type == GG_F32) {
            float * o = (float *) dst;
            for (uint64_t i = lo; i < hi; ++i) o[i] = tsn_init_value(key, i, s.init, s.scale);
        } else {
            uint16_t * o = (uint16_t *) dst;
            for (uint64_t i = lo; i < hi; ++i) o[i] = tsn_f32_to_bf16(tsn_init_value(key, i, s.init, s.scale));
        }
    };
    if (n < (1u << 16)) { work(0); if (nth > 1) for (unsigned t = 1; t < nth; ++t) work(t); return; }
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nth; ++t) th.emplace_back(work, t);
    for (auto & x : th) x.join();
}

namespace {
struct KvU32 { std::string k; uint32_t v; };
struct KvF32 { std::string k; float v; };
// GGUF v3 file: the given scalar KV pairs plus architecture and seed, then every tensor of specs
// filled by synth_fill_host (bit-identical to the device fill)
bool write_gguf(const std::string & path, const std::vector<TensorSpec> & specs, const std::vector<KvU32> & u32s,
                const std::vector<KvF32> & f32s, const std::string & arch, uint64_t seed, std::string & err) {
    FILE * f = fopen(path.c_str(), "wb");
    if (!f) { err = "cannot create " + path; return false; }
    auto w = [&](const void * p, size_t n) { fwrite(p, 1, n, f); };
    auto w32 = [&](uint32_t v) { w(&v, 4); };
    auto w64 = [&](uint64_t v) { w(&v, 8); };
    auto ws = [&](const std::string & s) { w64(s.size()); w(s.data(), s.size()); };
    const uint64_t align = 32;
    w32(0x46554747u);            // "GGUF"
    w32(3);
    w64(specs.size());
    w64(1 + u32s.size() + f32s.size() + 2);
    ws("general.alignment"); w32(4); w32((uint32_t) align);
    for (const KvU32 & kv : u32s) { ws(kv.k); w32(4); w32(kv.v); }
    for (const KvF32 & kv : f32s) { ws(kv.k); w32(6); w(&kv.v, 4); }
    ws("general.architecture"); w32(8); ws(arch);
    ws("tsn.synthetic.seed"); w32(10); w64(seed);
    uint64_t off = 0;
    for (const TensorSpec & s : specs) {
        ws(s.name);
        w32(s.n_dims);
        for (uint32_t d = 0; d < s.n_dims; ++d) w64(s.ne[d]);
        w32(s.type);
        w64(off);
        off += (tensor_bytes(s.type, s.nelem()) + align - 1) & ~(align - 1);
    }
    long pos = ftell(f);
    const uint64_t pad = ((uint64_t) pos + align - 1) / align * align - (uint64_t) pos;
    static const uint8_t zeros[64] = {0};
    w(zeros, (size_t) pad);
    std::vector<uint8_t> buf;
    for (const TensorSpec & s : specs) {
        const uint64_t nb = tensor_bytes(s.type, s.nelem());
        buf.resize((size_t) nb);
        synth_fill_host(s, seed, buf.data());
        w(buf.data(), (size_t) nb);
        const uint64_t tail = ((nb + align - 1) & ~(align - 1)) - nb;
        w(zeros, (size_t) tail);
    }
    const bool ok = ferror(f) == 0;
    fclose(f);
    if (!ok) err = "write error on " + path;
    return ok;
}
} // namespace

bool write_synthetic_gguf(const std::string & path, const DitGeom & g, uint64_t seed, bool with_prep,
                          std::string & err) {
    return write_gguf(path, dit_schema(g, with_prep),
                      {{"dit.hidden_dim", g.H}, {"dit.num_heads", g.NH}, {"dit.depth", g.depth},
                       {"dit.fused_depth", g.fused_depth}, {"dit.latent_dim", g.latent_dim}},
                      {{"dit.rope_theta", g.rope_theta}, {"dit.t_embed_max_period", g.t_max_period}},
                      "thinksound-dit-synthetic", seed, err);
}

bool write_synthetic_vae_gguf(const std::string & path, const VaeGeom & v, uint64_t seed, std::string & err) {
    return write_gguf(path, vae_schema(v),
                      {{"vae.latent_dim", v.latent_dim}, {"vae.channels", v.channels}, {"vae.out_channels", v.out_channels}},
                      {}, "thinksound-vae-synthetic", seed, err);
}

// KV keys of T5Model::load (src/t5.cpp:22-33) and ClipModel::load (src/clip.cpp:6-12)
bool write_synthetic_t5_gguf(const std::string & path, const T5Geom & g, uint64_t seed, std::string & err) {
    return write_gguf(path, t5_schema(g),
                      {{"t5.d_model", g.d_model}, {"t5.d_ff", g.d_ff}, {"t5.n_layers", g.layers}, {"t5.n_heads", g.heads},
                       {"t5.d_kv", g.d_model / g.heads}, {"t5.rel_buckets", g.rel_buckets}, {"t5.rel_max_dist", g.rel_max_dist}},
                      {{"t5.eps", 1e-6f}}, "t5-synthetic", seed, err);
}

bool write_synthetic_clip_gguf(const std::string & path, const ClipGeom & g, uint64_t seed, std::string & err) {
    return write_gguf(path, clip_schema(g),
                      {{"clip.hidden", g.hidden}, {"clip.layers", g.layers}, {"clip.heads", g.heads}, {"clip.ctx", g.ctx}},
                      {}, "metaclip-text-synthetic", seed, err);
}

} // namespace tsn
