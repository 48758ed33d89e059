// oracle/port.cpp — CPU restatement of the reference's DiT denoising path
// (TEST INFRASTRUCTURE: the parity checker and the CPU baseline, never the product path).
//
// Restates, in order and op for op:
//   GGUF parsing            src/gguf.cpp:73-151, 193-234
//   WeightSet::load         src/net.mm:126-173 (1-D f32 kept; everything else bf16->f32->f16)
//   Runtime gemm/conv/gemv  src/net.mm:14-56 and the elementwise wrappers src/net.mm:58-106
//   DitModel::forward       src/dit_fwd.cpp:104-304 (pre_attn :24-49, post_attn :51-81,
//                           attention :83-102), including the reference's per-tap dumps
//   sampler step            src/pipeline.cpp:142-155
// over the scalar kernels of oracle/kernels.cpp. Because both this port and the reference's own
// host code (built into oracle/_ref/ by oracle/Makefile) call the same kernels in the same
// order, the two agree bit for bit; tests/test_oracle.py checks that.
//
// C ABI (ctypes): oracle_load, oracle_free, oracle_info, oracle_forward, oracle_step,
// oracle_tap, oracle_threads.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <memory>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/tsn_synth.h"
#include "kernels.h"

namespace {

using namespace oracle;

// ------------------------------------------------------------------------------------------
// GGUF v2/v3 reader (src/gguf.cpp:73-151): KV metadata, tensor infos, aligned data section.
// ------------------------------------------------------------------------------------------
struct Tensor {
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;      // 0 f32, 1 f16, 30 bf16
    const uint8_t * data = nullptr;
    uint64_t nelem() const { uint64_t n = 1; for (uint32_t d = 0; d < n_dims; ++d) n *= ne[d]; return n; }
};

struct Gguf {
    void * map = nullptr;
    size_t len = 0;
    std::map<std::string, double> num;   // numeric KV values
    std::map<std::string, Tensor> tensors;
    ~Gguf() { if (map) munmap(map, len); }

    bool open(const char * path) {
        int fd = ::open(path, O_RDONLY);
        if (fd < 0) return false;
        struct stat st{};
        if (fstat(fd, &st) != 0) { ::close(fd); return false; }
        len = (size_t) st.st_size;
        map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (map == MAP_FAILED) { map = nullptr; return false; }
        const uint8_t * p = (const uint8_t *) map, * end = p + len;
        bool bad = false;
        auto raw = [&](void * dst, size_t n) {
            if (bad || (size_t) (end - p) < n) { bad = true; return; }
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
        if (u32() != 0x46554747u) return false;              // "GGUF"
        uint32_t version = u32();
        if (version < 2 || version > 3) return false;
        uint64_t n_t = u64(), n_kv = u64();
        const size_t scalar_size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        for (uint64_t i = 0; i < n_kv && !bad; ++i) {
            std::string key = str();
            uint32_t ty = u32();
            if (ty == 8) { str(); continue; }
            if (ty == 9) {
                uint32_t et = u32(); uint64_t n = u64();
                for (uint64_t k = 0; k < n && !bad; ++k) {
                    if (et == 8) str();
                    else if (et < 13 && scalar_size[et]) raw(nullptr, scalar_size[et]);
                    else bad = true;
                }
                continue;
            }
            if (ty >= 13 || !scalar_size[ty]) return false;
            uint8_t buf[8] = {0};
            raw(buf, scalar_size[ty]);
            double v = 0;
            switch (ty) {
                case 0: v = buf[0]; break;
                case 1: v = (int8_t) buf[0]; break;
                case 2: { uint16_t x; memcpy(&x, buf, 2); v = x; break; }
                case 3: { int16_t x; memcpy(&x, buf, 2); v = x; break; }
                case 4: { uint32_t x; memcpy(&x, buf, 4); v = x; break; }
                case 5: { int32_t x; memcpy(&x, buf, 4); v = x; break; }
                case 6: { float x; memcpy(&x, buf, 4); v = x; break; }
                case 7: v = buf[0] != 0; break;
                case 10: { uint64_t x; memcpy(&x, buf, 8); v = (double) x; break; }
                case 11: { int64_t x; memcpy(&x, buf, 8); v = (double) x; break; }
                case 12: { double x; memcpy(&x, buf, 8); v = x; break; }
            }
            num[key] = v;
        }
        if (bad) return false;
        uint64_t align = num.count("general.alignment") ? (uint64_t) num["general.alignment"] : 32;
        std::vector<std::pair<std::string, uint64_t>> offs;
        for (uint64_t i = 0; i < n_t && !bad; ++i) {
            std::string name = str();
            Tensor t;
            t.n_dims = u32();
            if (t.n_dims > 4) return false;
            for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = u64();
            t.type = u32();
            uint64_t off = u64();
            tensors[name] = t;
            offs.emplace_back(name, off);
        }
        if (bad) return false;
        uint64_t hdr = (uint64_t) (p - (const uint8_t *) map);
        uint64_t data_start = (hdr + align - 1) & ~(align - 1);
        for (auto & [name, off] : offs) tensors[name].data = (const uint8_t *) map + data_start + off;
        return true;
    }
    double kv(const std::string & k, double def) const {
        auto it = num.find(k);
        return it == num.end() ? def : it->second;
    }
};

// to_f32 (src/gguf.cpp:193-234) for the types the DiT uses.
static std::vector<float> to_f32(const Tensor & t) {
    std::vector<float> out((size_t) t.nelem());
    const uint16_t * h = (const uint16_t *) t.data;
    if (t.type == 0) memcpy(out.data(), t.data, out.size() * 4);
    else if (t.type == 30) for (size_t i = 0; i < out.size(); ++i) out[i] = tsn_bf16_to_f32(h[i]);
    else if (t.type == 1) {
        for (size_t i = 0; i < out.size(); ++i) {     // the reference's f16 path flushes subnormals
            uint32_t u = h[i], sign = (u >> 15) & 1, exp = (u >> 10) & 0x1F, man = u & 0x3FF, f;
            if (exp == 0) f = sign << 31;
            else if (exp == 31) f = (sign << 31) | 0x7F800000u | (man << 13);
            else f = (sign << 31) | ((exp + 112) << 23) | (man << 13);
            memcpy(&out[i], &f, 4);
        }
    } else out.clear();
    return out;
}

// ------------------------------------------------------------------------------------------
// Weights as the reference's device sees them (src/net.mm:126-173)
// ------------------------------------------------------------------------------------------
struct Ent { std::vector<uint16_t> h; std::vector<float> f; bool f16 = true; };

struct Model {
    Gguf file;
    std::map<std::string, Ent> w;
    uint32_t H = 1024, NH = 16, hd = 64, depth = 21, fused_depth = 14, latent_dim = 64, H_ffn = 2816;
    float rope_theta = 10000.0f, t_max_period = 1.0f;
    uint32_t n_joint = 7;
    std::map<std::string, std::vector<float>> taps;
    bool want_taps = false;

    const void * W(const std::string & n) const {
        auto it = w.find(n);
        if (it == w.end()) { fprintf(stderr, "oracle: missing tensor %s\n", n.c_str()); return nullptr; }
        return it->second.f16 ? (const void *) it->second.h.data() : (const void *) it->second.f.data();
    }
};

bool load_model(Model & m, const char * path) {
    if (!m.file.open(path)) return false;
    for (auto & [name, t] : m.file.tensors) {
        Ent e;
        e.f16 = !(t.type == 0 && t.n_dims <= 1);
        std::vector<float> v = to_f32(t);
        if (v.empty() && t.nelem()) return false;
        if (e.f16) { e.h.resize(v.size()); for (size_t i = 0; i < v.size(); ++i) e.h[i] = tsn_ref_f32_to_f16(v[i]); }
        else e.f = std::move(v);
        m.w[name] = std::move(e);
    }
    // DitModel::load (src/dit.cpp:29-46)
    m.H = (uint32_t) m.file.kv("dit.hidden_dim", 1024);
    m.NH = (uint32_t) m.file.kv("dit.num_heads", 16);
    m.hd = m.H / m.NH;
    m.depth = (uint32_t) m.file.kv("dit.depth", 21);
    m.fused_depth = (uint32_t) m.file.kv("dit.fused_depth", 14);
    m.latent_dim = (uint32_t) m.file.kv("dit.latent_dim", 64);
    m.rope_theta = (float) m.file.kv("dit.rope_theta", 10000.0);
    m.t_max_period = (float) m.file.kv("dit.t_embed_max_period", 1.0);
    m.n_joint = m.depth - m.fused_depth;
    auto it = m.file.tensors.find("joint_blocks.0.latent_block.ffn.w1.weight");
    m.H_ffn = (it != m.file.tensors.end() && it->second.n_dims >= 3) ? (uint32_t) it->second.ne[2] : 2816;
    return true;
}

// ------------------------------------------------------------------------------------------
// Runtime wrappers (src/net.mm:14-106)
// ------------------------------------------------------------------------------------------
struct Rt {
    std::vector<float> col;
    void gemm(const void * W, const float * X, float * Y, const float * bias,
              uint32_t M, uint32_t N, uint32_t K, uint32_t ldx = 0, uint32_t ldw = 0, uint32_t ldy = 0) {
        GemmP p{M, N, K, ldx ? ldx : K, ldw ? ldw : K, ldy ? ldy : N, bias ? 1u : 0u, 0};
        gemm_h((const uint16_t *) W, X, Y, bias, p);
    }
    void gemv(const void * W, const float * X, float * Y, const float * bias, uint32_t N, uint32_t K, uint32_t ldw) {
        GemmP p{1, N, K, K, ldw ? ldw : K, N, bias ? 1u : 0u, 0};
        gemv_h((const uint16_t *) W, X, Y, bias, p);
    }
    // stride-1 conv, OL == T (the DiT's only form): im2col + GEMM, or direct when OC < 32
    void conv(const void * W, const float * bias, const float * x, float * y,
              uint32_t T, uint32_t IC, uint32_t OC, uint32_t K, uint32_t pad, uint32_t dil) {
        const uint32_t OL = T;
        if (K == 1 && pad == 0) { gemm(W, x, y, bias, OL, OC, IC); return; }
        if (OC < 32) {
            ConvP p{T, OL, IC, OC, K, 1, pad, dil, IC, OC, 0, bias ? 1u : 0u};
            conv1d_fwd_h(x, (const uint16_t *) W, bias, y, p);
            return;
        }
        const size_t KC = (size_t) IC * K, max_elems = (size_t) 16 << 20;
        const uint32_t rows = (uint32_t) std::max<size_t>(1, std::min<size_t>(OL, max_elems / KC));
        if (col.size() < (size_t) rows * KC) col.resize((size_t) rows * KC);
        for (uint32_t t0 = 0; t0 < OL; t0 += rows) {
            const uint32_t n = std::min(rows, OL - t0);
            IcP ic{T, n, IC, K, 1, pad, dil, IC, 0, t0};
            im2col(x, col.data(), ic, (size_t) n * KC);
            gemm(W, col.data(), y + (size_t) t0 * OC, bias, n, OC, (uint32_t) KC);
        }
    }
    void silu(float * x, size_t n) { silu_(x, (uint32_t) n); }
    void copy(const float * x, float * y, size_t n) { copy_(x, y, (uint32_t) n); }
    void swiglu(const float * a, const float * b, float * y, size_t n) { swiglu_(a, b, y, (uint32_t) n); }
    void add(const float * a, const float * b, float * y, size_t n) { add_(a, b, y, (uint32_t) n); }
    void add_bcast(const float * x, const float * v, float * y, uint32_t S, uint32_t H) {
        CH p{H, S * H}; add_bcast_col(x, v, y, p);
    }
};

// ------------------------------------------------------------------------------------------
// The forward: src/dit_fwd.cpp:104-304 over buffers sized as src/dit.cpp:63-88
// ------------------------------------------------------------------------------------------
struct Fwd {
    Model & m;
    Rt rt;
    uint32_t T, C, TS, S;
    std::vector<float> extc, extc_silu, x_in, jointq, sc_qkv, joint_att, mod_lat, mod_clip, mod_text,
        clip_s, text_s, mod_fin, te_out, gc_pre, global_c, probs, sc_l1, sc_r, sc_f1, sc_f3;
    std::vector<int32_t> pos_lat, pos_clip;

    Fwd(Model & model, uint32_t T_, uint32_t C_, uint32_t TS_) : m(model), T(T_), C(C_), TS(TS_) {
        const uint32_t H = m.H;
        S = T + C + TS;
        auto z = [](std::vector<float> & v, size_t n) { v.assign(n, 0.0f); };
        z(extc, (size_t) T * H); z(extc_silu, (size_t) T * H); z(x_in, (size_t) T * H);
        z(jointq, (size_t) S * 3 * H); z(sc_qkv, (size_t) S * 3 * H); z(joint_att, (size_t) S * H);
        z(mod_lat, (size_t) T * 6 * H); z(mod_clip, 6 * H); z(mod_text, 6 * H);
        z(clip_s, (size_t) C * H); z(text_s, (size_t) TS * H); z(mod_fin, (size_t) T * 2 * H);
        z(te_out, H); z(gc_pre, H); z(global_c, H); z(probs, (size_t) m.NH * S * S);
        z(sc_l1, (size_t) S * H); z(sc_r, (size_t) S * H); z(sc_f1, (size_t) S * m.H_ffn); z(sc_f3, (size_t) S * m.H_ffn);
        pos_lat.resize(T); pos_clip.resize(C);                   // dit_fwd.cpp:171-179
        for (uint32_t i = 0; i < T; ++i) pos_lat[i] = (int32_t) i;
        for (uint32_t i = 0; i < C; ++i) pos_clip[i] = (int32_t) i;
    }

    void tap(const char * name, const float * p, size_t n) {
        if (m.want_taps) m.taps[name].assign(p, p + n);
    }

    // dit_fwd.cpp:24-49
    void pre_attn(const std::string & bp, const float * x, const float * mod, bool per_row, uint32_t rows,
                  uint32_t row_off, float * qkv_dst, const int32_t * pos, float fscale, bool is_text, uint32_t chunks) {
        const uint32_t H = m.H;
        AD ad{H, per_row ? 1u : 0u, chunks, 0u, 1e-5f};
        adaln_ln(x, mod, sc_f1.data(), ad, rows);
        rt.gemm(m.W(bp + ".attn.qkv.weight"), sc_f1.data(), qkv_dst, (const float *) m.W(bp + ".attn.qkv.bias"),
                rows, 3 * H, H, H, H, 3 * H);
        QS3 qs{H, row_off};
        qkv_split3(qkv_dst, sc_qkv.data(), qs, rows);
        RH rq{3 * H, m.hd, 0, row_off, 1e-6f};
        rms_head(sc_qkv.data(), (const float *) m.W(bp + ".attn.q_norm.weight"), rq, rows, m.NH);
        RH rk{3 * H, m.hd, H, row_off, 1e-6f};
        rms_head(sc_qkv.data(), (const float *) m.W(bp + ".attn.k_norm.weight"), rk, rows, m.NH);
        if (!is_text) {
            RP pq{3 * H, m.hd, 0, row_off, fscale, m.rope_theta};
            rope_pairs(sc_qkv.data(), pos, pq, rows, H / 2);
            RP pk{3 * H, m.hd, H, row_off, fscale, m.rope_theta};
            rope_pairs(sc_qkv.data(), pos, pk, rows, H / 2);
        }
    }

    // dit_fwd.cpp:51-81
    void post_attn(const std::string & bp, float * x, const float * attn_out, const float * mod, bool per_row,
                   uint32_t rows, bool is_text) {
        const uint32_t H = m.H, F = m.H_ffn;
        if (is_text)
            rt.gemm(m.W(bp + ".linear1.weight"), attn_out, sc_l1.data(), (const float *) m.W(bp + ".linear1.bias"), rows, H, H);
        else
            rt.conv(m.W(bp + ".linear1.weight"), (const float *) m.W(bp + ".linear1.bias"), attn_out, sc_l1.data(), rows, H, H, 3, 1, 1);
        GA ga{H, per_row ? 1u : 0u, 6u, 2u};
        gate_add(x, sc_l1.data(), mod, x, ga, (size_t) (((size_t) rows * H + 255) / 256) * 256);
        AD ad{H, per_row ? 1u : 0u, 6u, 3u * H, 1e-5f};
        adaln_ln(x, mod, sc_r.data(), ad, rows);
        if (is_text) {
            rt.gemm(m.W(bp + ".ffn.w1.weight"), sc_r.data(), sc_f1.data(), nullptr, rows, F, H);
            rt.gemm(m.W(bp + ".ffn.w3.weight"), sc_r.data(), sc_f3.data(), nullptr, rows, F, H);
            rt.swiglu(sc_f1.data(), sc_f3.data(), sc_f1.data(), (size_t) rows * F);
            rt.gemm(m.W(bp + ".ffn.w2.weight"), sc_f1.data(), sc_f3.data(), nullptr, rows, H, F);
        } else {
            rt.conv(m.W(bp + ".ffn.w1.weight"), nullptr, sc_r.data(), sc_f1.data(), rows, H, F, 3, 1, 1);
            rt.conv(m.W(bp + ".ffn.w3.weight"), nullptr, sc_r.data(), sc_f3.data(), rows, H, F, 3, 1, 1);
            rt.swiglu(sc_f1.data(), sc_f3.data(), sc_f1.data(), (size_t) rows * F);
            rt.conv(m.W(bp + ".ffn.w2.weight"), nullptr, sc_f1.data(), sc_f3.data(), rows, F, H, 3, 1, 1);
        }
        GA gf{H, per_row ? 1u : 0u, 6u, 5u};
        gate_add(x, sc_f3.data(), mod, x, gf, (size_t) (((size_t) rows * H + 255) / 256) * 256);
    }

    // dit_fwd.cpp:83-102
    void attention(uint32_t S_) {
        AttnP p{};
        p.Sq = p.Sk = S_; p.hd = m.hd; p.nh = m.NH; p.ld = 3 * m.H; p.ldo = m.H; p.bias_mode = 0;
        p.scale = 1.0f / sqrtf((float) m.hd);
        p.q_off = 0; p.k_off = m.H; p.v_off = 2 * m.H; p.o_off = 0; p.p_off = 0;
        attn_qk(sc_qkv.data(), probs.data(), nullptr, nullptr, p);
        softmax_rows(probs.data(), p);
        attn_pav(probs.data(), sc_qkv.data(), joint_att.data(), p);
    }

    // dit_fwd.cpp:104-304
    // one joint block (dit_fwd.cpp:180-257) on lat [T,H] and the clip_s / text_s streams, with the
    // conditioning already in extc_silu and global_c (silu applied)
    void joint_block(uint32_t i, float * lat) {
        const uint32_t H = m.H;
        const float clip_fscale = (float) T / (float) C;
        const bool pre_only = (i == m.n_joint - 1);
        const std::string jb = "joint_blocks." + std::to_string(i);
        rt.gemm(m.W(jb + ".latent_block.adaLN_modulation.1.weight"), extc_silu.data(), mod_lat.data(),
                (const float *) m.W(jb + ".latent_block.adaLN_modulation.1.bias"), T, 6 * H, H);
        pre_attn(jb + ".latent_block", lat, mod_lat.data(), true, T, 0, jointq.data(), pos_lat.data(), 1.0f, false, 6);
        const uint32_t ct = pre_only ? 2u : 6u;
        rt.gemv(m.W(jb + ".clip_block.adaLN_modulation.1.weight"), global_c.data(), mod_clip.data(),
                (const float *) m.W(jb + ".clip_block.adaLN_modulation.1.bias"), ct * H, H, H);
        pre_attn(jb + ".clip_block", clip_s.data(), mod_clip.data(), false, C, T,
                 jointq.data() + (size_t) T * 3 * H, pos_clip.data(), clip_fscale, false, ct);
        rt.gemv(m.W(jb + ".text_block.adaLN_modulation.1.weight"), global_c.data(), mod_text.data(),
                (const float *) m.W(jb + ".text_block.adaLN_modulation.1.bias"), ct * H, H, H);
        pre_attn(jb + ".text_block", text_s.data(), mod_text.data(), false, TS, T + C,
                 jointq.data() + (size_t) (T + C) * 3 * H, nullptr, 1.0f, true, ct);
        if (i == 0 && m.want_taps) {                                                     // :211-233
            tap("text_xn", sc_f1.data(), (size_t) TS * H);
            std::vector<float> q((size_t) S * H), k((size_t) S * H), v((size_t) S * H);
            for (uint32_t s = 0; s < S; ++s) {
                memcpy(q.data() + (size_t) s * H, sc_qkv.data() + (size_t) s * 3 * H, H * 4);
                memcpy(k.data() + (size_t) s * H, sc_qkv.data() + (size_t) s * 3 * H + H, H * 4);
                memcpy(v.data() + (size_t) s * H, sc_qkv.data() + (size_t) s * 3 * H + 2 * H, H * 4);
            }
            tap("a0_q", q.data(), q.size()); tap("a0_k", k.data(), k.size()); tap("a0_v", v.data(), v.size());
        }
        attention(S);
        post_attn(jb + ".latent_block", lat, joint_att.data(), mod_lat.data(), true, T, false);
        if (!pre_only) {
            post_attn(jb + ".clip_block", clip_s.data(), joint_att.data() + (size_t) T * H, mod_clip.data(), false, C, false);
            post_attn(jb + ".text_block", text_s.data(), joint_att.data() + (size_t) (T + C) * H, mod_text.data(), false, TS, true);
        }
        if (i == 0) {                                                                    // :245-256
            tap("a0_out", joint_att.data(), (size_t) S * H);
            tap("jb0_lat", lat, (size_t) T * H);
            tap("jb0_clip", clip_s.data(), (size_t) C * H);
            tap("jb0_text", text_s.data(), (size_t) TS * H);
        }
    }

    void forward(const float * x, float t, const float * clip_pp, const float * sync_gather,
                 const float * text_pp, const float * gcmlp, float * flow) {
        const uint32_t H = m.H;
        // timestep embedding on the host                          dit_fwd.cpp:112-119
        std::vector<float> temb(H);
        const int half = H / 2;
        const float fscale_t = 10000.0f / m.t_max_period;
        for (int kk = 0; kk < half; ++kk) {
            float fr = fscale_t * powf(10000.0f, -2.0f * kk / (float) H);
            temb[kk] = cosf(t * fr);
            temb[half + kk] = sinf(t * fr);
        }
        std::vector<float> te_scr(H);
        rt.gemv(m.W("t_embed.mlp.0.weight"), temb.data(), te_out.data(), (const float *) m.W("t_embed.mlp.0.bias"), H, H, H);
        rt.silu(te_out.data(), H);
        rt.gemv(m.W("t_embed.mlp.2.weight"), te_out.data(), te_scr.data(), (const float *) m.W("t_embed.mlp.2.bias"), H, H, H);
        rt.add(gcmlp, te_scr.data(), global_c.data(), H);                                   // :131
        rt.copy(te_scr.data(), te_out.data(), H);
        rt.add_bcast(sync_gather, global_c.data(), extc.data(), T, H);                      // :135
        rt.copy(extc.data(), extc_silu.data(), (size_t) T * H);
        rt.silu(extc_silu.data(), (size_t) T * H);
        rt.copy(global_c.data(), gc_pre.data(), H);
        rt.silu(global_c.data(), H);
        // audio_input_proj                                         dit_fwd.cpp:143-149
        rt.conv(m.W("audio_input_proj.0.weight"), (const float *) m.W("audio_input_proj.0.bias"), x, x_in.data(),
                T, m.latent_dim, H, 3, 1, 1);
        rt.silu(x_in.data(), (size_t) T * H);
        rt.conv(m.W("audio_input_proj.2.w1.weight"), nullptr, x_in.data(), sc_f1.data(), T, H, m.H_ffn, 3, 1, 1);
        rt.conv(m.W("audio_input_proj.2.w3.weight"), nullptr, x_in.data(), sc_f3.data(), T, H, m.H_ffn, 3, 1, 1);
        rt.swiglu(sc_f1.data(), sc_f3.data(), sc_f1.data(), (size_t) T * m.H_ffn);
        rt.conv(m.W("audio_input_proj.2.w2.weight"), nullptr, sc_f1.data(), x_in.data(), T, m.H_ffn, H, 3, 1, 1);
        tap("t_emb", te_out.data(), H);                                                      // :151-162
        tap("global_c", gc_pre.data(), H);
        tap("extended_c", extc.data(), (size_t) T * H);
        tap("x_in", x_in.data(), (size_t) T * H);

        // joint blocks                                              dit_fwd.cpp:164-257
        rt.copy(clip_pp, clip_s.data(), (size_t) C * H);
        rt.copy(text_pp, text_s.data(), (size_t) TS * H);
        float * lat = x_in.data();
        for (uint32_t i = 0; i < m.n_joint; ++i) joint_block(i, lat);
        tap("after_joint", lat, (size_t) T * H);                                             // :259-265
        for (uint32_t i = 0; i < m.fused_depth; ++i) {                                       // :267-279
            const std::string fb = "fused_blocks." + std::to_string(i);
            rt.gemm(m.W(fb + ".adaLN_modulation.1.weight"), extc_silu.data(), mod_lat.data(),
                    (const float *) m.W(fb + ".adaLN_modulation.1.bias"), T, 6 * H, H);
            pre_attn(fb, lat, mod_lat.data(), true, T, 0, jointq.data(), pos_lat.data(), 1.0f, false, 6);
            attention(T);
            post_attn(fb, lat, joint_att.data(), mod_lat.data(), true, T, false);
        }
        tap("after_fused", lat, (size_t) T * H);
        // final layer                                               dit_fwd.cpp:287-303
        rt.gemm(m.W("final_layer.adaLN_modulation.1.weight"), extc_silu.data(), mod_fin.data(),
                (const float *) m.W("final_layer.adaLN_modulation.1.bias"), T, 2 * H, H);
        AD af{H, 1u, 2u, 0u, 1e-5f};
        adaln_ln(lat, mod_fin.data(), sc_l1.data(), af, T);
        tap("final_fx", sc_l1.data(), (size_t) T * H);
        tap("final_mod", mod_fin.data(), (size_t) T * 2 * H);
        rt.conv(m.W("final_layer.conv.weight"), (const float *) m.W("final_layer.conv.bias"), sc_l1.data(), flow,
                T, H, m.latent_dim, 7, 3, 1);
        tap("flow", flow, (size_t) T * m.latent_dim);
    }
};

// ------------------------------------------------------------------------------------------
// Per-generation conditioning: DitModel::prep_conditioning (src/dit.cpp:55-135) and
// DitModel::prep_text_arm (src/dit.cpp:137-192), with convmlp / mlp of src/dit.cpp:14-27.
// ------------------------------------------------------------------------------------------
struct Prep {
    Model & m;
    Rt rt;
    std::vector<float> h1, h3;
    std::vector<float> clip_fc;                                   // DitModel::clip_fc_host

    explicit Prep(Model & model) : m(model) {}

    // convmlp (src/dit.cpp:14-20): conv k3 w1, w3 -> swiglu -> conv k3 w2; y may alias x
    void convmlp(const std::string & pre, const float * x, float * y, uint32_t T, uint32_t C) {
        const uint32_t F = m.H_ffn;
        h1.assign((size_t) T * F, 0.0f);
        h3.assign((size_t) T * F, 0.0f);
        rt.conv(m.W(pre + ".w1.weight"), nullptr, x, h1.data(), T, C, F, 3, 1, 1);
        rt.conv(m.W(pre + ".w3.weight"), nullptr, x, h3.data(), T, C, F, 3, 1, 1);
        rt.swiglu(h1.data(), h3.data(), h1.data(), (size_t) T * F);
        rt.conv(m.W(pre + ".w2.weight"), nullptr, h1.data(), y, T, F, C, 3, 1, 1);
    }
    // mlp (src/dit.cpp:21-27)
    void mlp(const std::string & pre, const float * x, float * y, uint32_t rows, uint32_t C) {
        const uint32_t F = m.H_ffn;
        h1.assign((size_t) rows * F, 0.0f);
        h3.assign((size_t) rows * F, 0.0f);
        rt.gemm(m.W(pre + ".w1.weight"), x, h1.data(), nullptr, rows, F, C);
        rt.gemm(m.W(pre + ".w3.weight"), x, h3.data(), nullptr, rows, F, C);
        rt.swiglu(h1.data(), h3.data(), h1.data(), (size_t) rows * F);
        rt.gemm(m.W(pre + ".w2.weight"), h1.data(), y, nullptr, rows, C, F);
    }
    // src/dit.cpp:91-133
    void conditioning(uint32_t T, uint32_t clip_S, uint32_t sync_S, const float * clip_f, const float * sync_f,
                      float * clip_pp, float * sync_gather) {
        const uint32_t H = m.H;
        // sync: + sync_pos_emb per 8-frame segment (host f32), conv k7, silu, convmlp, gather to T
        auto pit = m.file.tensors.find("sync_pos_emb");
        const std::vector<float> spe = pit == m.file.tensors.end() ? std::vector<float>() : to_f32(pit->second);
        std::vector<float> sbuf(sync_f, sync_f + (size_t) sync_S * 768);
        for (uint32_t s = 0; s < sync_S && !spe.empty(); ++s)
            for (int c = 0; c < 768; ++c) sbuf[(size_t) s * 768 + c] += spe[(size_t) (s % 8) * 768 + c];
        std::vector<float> smid((size_t) sync_S * H, 0.0f);
        rt.conv(m.W("sync_input_proj.0.weight"), (const float *) m.W("sync_input_proj.0.bias"), sbuf.data(), smid.data(),
                sync_S, 768, H, 7, 3, 1);
        rt.silu(smid.data(), (size_t) sync_S * H);
        convmlp("sync_input_proj.2", smid.data(), smid.data(), sync_S, H);
        for (uint32_t i = 0; i < T; ++i) {
            const int32_t si = (int32_t) floorf(((float) i + 0.5f) * (float) sync_S / (float) T);
            memcpy(sync_gather + (size_t) i * H, smid.data() + (size_t) si * H, (size_t) H * 4);
        }
        // clip: linear + silu + convmlp -> clip_pp
        rt.gemm(m.W("clip_input_proj.0.weight"), clip_f, clip_pp, (const float *) m.W("clip_input_proj.0.bias"), clip_S, H,
                1024);
        rt.silu(clip_pp, (size_t) clip_S * H);
        convmlp("clip_input_proj.2", clip_pp, clip_pp, clip_S, H);
        // clip_fc = clip_cond_proj(mean over clip rows)
        std::vector<float> cmean(H, 0.0f);
        SH sh{clip_S, H};
        mean_cols(clip_pp, cmean.data(), sh);
        clip_fc.assign(H, 0.0f);
        rt.gemv(m.W("clip_cond_proj.weight"), cmean.data(), clip_fc.data(), (const float *) m.W("clip_cond_proj.bias"), H,
                1024, 1024);
    }
    // src/dit.cpp:137-192
    void text_arm(uint32_t text_S, const float * text_cat, const float * gtext, float * text_pp, float * gcmlp) {
        const uint32_t H = m.H, F = m.H_ffn;
        rt.gemm(m.W("text_input_proj.0.weight"), text_cat, text_pp, (const float *) m.W("text_input_proj.0.bias"), text_S, H,
                2048);
        rt.silu(text_pp, (size_t) text_S * H);
        std::vector<float> f1((size_t) text_S * F, 0.0f), f3((size_t) text_S * F, 0.0f);
        rt.gemm(m.W("text_input_proj.2.w1.weight"), text_pp, f1.data(), nullptr, text_S, F, H);
        rt.gemm(m.W("text_input_proj.2.w3.weight"), text_pp, f3.data(), nullptr, text_S, F, H);
        rt.swiglu(f1.data(), f3.data(), f1.data(), (size_t) text_S * F);
        rt.gemm(m.W("text_input_proj.2.w2.weight"), f1.data(), text_pp, nullptr, text_S, H, F);
        std::vector<float> tfc(H, 0.0f);
        rt.gemv(m.W("text_cond_proj.weight"), gtext, tfc.data(), (const float *) m.W("text_cond_proj.bias"), H, 1024, 1024);
        for (uint32_t i = 0; i < H; ++i) tfc[i] += clip_fc[i];                 // host f32 add (dit.cpp:186-187)
        mlp("global_cond_mlp", tfc.data(), gcmlp, 1, H);
    }
};

} // namespace

extern "C" {

// prep_conditioning + prep_text_arm for both CFG arms (needs H = 1024: the clip and text cond
// projections read 1024 inputs, src/dit.cpp:130-131, 181-182).
int oracle_prep(void * h, int T, int C, int TS, int sync_S, const float * clip_f, const float * sync_f,
                const float * text_cat_c, const float * gtext_c, const float * text_cat_u, const float * gtext_u,
                float * clip_pp, float * sync_gather, float * text_pp_c, float * gcmlp_c, float * text_pp_u,
                float * gcmlp_u) {
    Model * m = (Model *) h;
    if (m->H != 1024) return -1;
    Prep p(*m);
    p.conditioning((uint32_t) T, (uint32_t) C, (uint32_t) sync_S, clip_f, sync_f, clip_pp, sync_gather);
    p.text_arm((uint32_t) TS, text_cat_c, gtext_c, text_pp_c, gcmlp_c);
    p.text_arm((uint32_t) TS, text_cat_u, gtext_u, text_pp_u, gcmlp_u);
    return 0;
}

void * oracle_load(const char * gguf_path) {
    auto * m = new Model();
    if (!load_model(*m, gguf_path)) { delete m; return nullptr; }
    return m;
}

void oracle_free(void * h) { delete (Model *) h; }

// H, NH, F, depth, fused_depth, latent_dim
int oracle_info(void * h, int * out6) {
    Model * m = (Model *) h;
    out6[0] = (int) m->H; out6[1] = (int) m->NH; out6[2] = (int) m->H_ffn;
    out6[3] = (int) m->depth; out6[4] = (int) m->fused_depth; out6[5] = (int) m->latent_dim;
    return 0;
}

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// One arm's forward (dit_fwd.cpp:104-304). want_taps keeps the reference's tap set in memory.
int oracle_forward(void * h, int T, int C, int TS, const float * x, float t, const float * clip_pp,
                   const float * sync_gather, const float * text_pp, const float * gcmlp, float * flow,
                   int want_taps) {
    Model * m = (Model *) h;
    m->want_taps = want_taps != 0;
    m->taps.clear();
    Fwd f(*m, (uint32_t) T, (uint32_t) C, (uint32_t) TS);
    f.forward(x, t, clip_pp, sync_gather, text_pp, gcmlp, flow);
    return 0;
}

// One CFG sampler step (pipeline.cpp:146-148): x is updated in place; fc/fu receive the flows.
int oracle_step(void * h, int T, int C, int TS, float * x, float t, float cfg, float dt,
                const float * clip_pp, const float * sync_gather,
                const float * text_pp_c, const float * gcmlp_c, const float * text_pp_u, const float * gcmlp_u,
                float * fc, float * fu) {
    Model * m = (Model *) h;
    m->want_taps = false;
    Fwd f(*m, (uint32_t) T, (uint32_t) C, (uint32_t) TS);
    f.forward(x, t, clip_pp, sync_gather, text_pp_c, gcmlp_c, fc);
    f.forward(x, t, clip_pp, sync_gather, text_pp_u, gcmlp_u, fu);
    CD p{cfg, dt, (uint32_t) ((size_t) T * m->latent_dim)};
    cfg_euler(fc, fu, x, p);
    return 0;
}

// One full joint block (joint block 0, dit_fwd.cpp:180-257) for one arm: lat [T,H], clip [C,H] and
// text [TS,H] are updated in place; extc_silu [T,H] and global_c_silu [H] are the block's
// conditioning. Needs a model with at least two joint blocks (block 0 full).
int oracle_joint_block(void * h, int T, int C, int TS, float * lat, float * clip, float * text, const float * extc_silu,
                       const float * global_c_silu) {
    Model * m = (Model *) h;
    if (m->n_joint < 2) return -1;
    m->want_taps = false;
    Fwd f(*m, (uint32_t) T, (uint32_t) C, (uint32_t) TS);
    const size_t H = m->H;
    memcpy(f.extc_silu.data(), extc_silu, (size_t) T * H * 4);
    memcpy(f.global_c.data(), global_c_silu, H * 4);
    memcpy(f.clip_s.data(), clip, (size_t) C * H * 4);
    memcpy(f.text_s.data(), text, (size_t) TS * H * 4);
    f.joint_block(0, lat);
    memcpy(clip, f.clip_s.data(), (size_t) C * H * 4);
    memcpy(text, f.text_s.data(), (size_t) TS * H * 4);
    return 0;
}

// Copy a tap of the last forward into out (n floats at most); returns its length or -1.
long long oracle_tap(void * h, const char * name, float * out, long long n) {
    Model * m = (Model *) h;
    auto it = m->taps.find(name);
    if (it == m->taps.end()) return -1;
    const long long len = (long long) it->second.size();
    if (out) memcpy(out, it->second.data(), (size_t) std::min(n, len) * 4);
    return len;
}

} // extern "C"
