// oracle/ref_driver.cpp — runs the reference's own DiT host code on the CPU device
// (TEST INFRASTRUCTURE; built by oracle/Makefile into oracle/_ref/ts_ref_dit).
//
//   ts_ref_dit forward <gguf> <T> <C> <TS> <in_dir> <out_dir> <t> <arm>
//       one DitModel::forward (src/dit_fwd.cpp:104-304) with TN_DUMP_EARLY=<out_dir>, so the
//       reference writes its own per-tap dumps nat_*.bin; the flow goes to <out_dir>/flow.bin.
//   ts_ref_dit step <gguf> <T> <C> <TS> <in_dir> <out_dir> <t> <cfg> <dt> [reps]
//       one CFG step exactly as the sampler loop runs it (src/pipeline.cpp:146-148): forward
//       cond, forward uncond, Runtime::cfg_euler. Writes x_out.bin; prints a JSON timing line.
//   ts_ref_dit sample <gguf> <T> <C> <TS> <in_dir> <out_dir> <steps> <cfg> [x0_seed] [dump_steps]
//       the Euler loop of src/pipeline.cpp:142-155 from the given x; writes x_final.bin. With
//       x0_seed >= 0 the initial latent is drawn as generate_wav draws it (src/pipeline.cpp:126-132:
//       mt19937(seed), normal_distribution<float>, channel-major draws into [T,64]) instead of read
//       from x.bin, and written to x0.bin. dump_steps (comma-separated step indices) writes, for
//       each listed step s, its input x_s<s>.bin and the flows fc_s<s>.bin, fu_s<s>.bin.
//   ts_ref_dit prep <gguf> <T> <C> <TS> <in_dir> <out_dir> <sync_S>
//       DitModel::prep_conditioning (src/dit.cpp:55-135) on clip_f.bin [C,1024] and sync_f.bin
//       [sync_S,768], then DitModel::prep_text_arm (src/dit.cpp:137-192) on text_cat_<arm>.bin
//       [TS,2048] and gtext_<arm>.bin [1024] for arm = cond, unc; writes clip_pp.bin,
//       sync_gather.bin, text_pp_<arm>.bin, gcmlp_<arm>.bin.
//   ts_ref_dit vae <vae_gguf> <T> 0 0 <in_dir> <out_dir> [reps]
//       VaeModel::decode (src/vae.cpp:17-86) of latent.bin [T,64]; writes audio.bin
//       [T_audio,2] (interleaved stereo) and prints a JSON timing line.
//   ts_ref_dit t5 <t5_gguf> 0 0 0 <in_dir> <out_dir> [reps]
//       T5Model::encode (src/t5.cpp:84-131) of ids.bin (int32 [77]); writes out.bin [77,d_model].
//   ts_ref_dit clip <clip_gguf> 0 0 0 <in_dir> <out_dir> [reps]
//       ClipModel::encode (src/clip.cpp:30-101) of ids.bin (int32 [77]); writes per_token.bin
//       [77,H] and global.bin [H].
//
// Inputs in <in_dir> (f32, row-major): x.bin [T,64], clip_pp.bin [C,H], sync_gather.bin [T,H],
// text_pp_cond.bin / text_pp_unc.bin [TS,H], gcmlp_cond.bin / gcmlp_unc.bin [H].
// These are the per-generation outputs of DitModel::prep_conditioning / prep_text_arm; the
// driver takes them as given and only allocates the forward's buffers the way
// prep_conditioning does (src/dit.cpp:63-88).
#include "models.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <random>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

using namespace tn;

static bool read_into(const std::string & path, gpu::Buf & b, size_t n) {
    FILE * f = fopen(path.c_str(), "rb");
    if (!f) { fprintf(stderr, "missing %s\n", path.c_str()); return false; }
    size_t got = fread(b.p, 4, n, f);
    fclose(f);
    if (got != n) { fprintf(stderr, "short read %s (%zu of %zu)\n", path.c_str(), got, n); return false; }
    return true;
}
static void write_from(const std::string & path, const void * p, size_t n) {
    FILE * f = fopen(path.c_str(), "wb");
    if (!f) { fprintf(stderr, "cannot write %s\n", path.c_str()); return; }
    fwrite(p, 4, n, f);
    fclose(f);
}

// Buffer set of src/dit.cpp:63-88 (prep_conditioning), without the prep computations.
static bool alloc_forward_buffers(Runtime & rt, DitModel & m) {
    const uint32_t H = m.H;
    const size_t S = (size_t) m.T + m.clip_S + m.text_S;
    const size_t SM = S * H * 4, SM_ffn = S * m.H_ffn * 4;
    m.clip_pp = rt.dev.alloc((size_t) m.clip_S * H * 4);
    m.sync_gather = rt.dev.alloc((size_t) m.T * H * 4);
    m.extc = rt.dev.alloc((size_t) m.T * H * 4);
    m.extc_silu = rt.dev.alloc((size_t) m.T * H * 4);
    m.x_in = rt.dev.alloc((size_t) m.T * H * 4);
    m.jointq = rt.dev.alloc(S * 3 * H * 4);
    m.sc_qkv = rt.dev.alloc(S * 3 * H * 4);
    m.joint_att = rt.dev.alloc(SM);
    m.mod_lat = rt.dev.alloc((size_t) m.T * 6 * H * 4);
    m.mod_clip = rt.dev.alloc(6 * H * 4);
    m.mod_text = rt.dev.alloc(6 * H * 4);
    m.clip_s = rt.dev.alloc((size_t) m.clip_S * H * 4);
    m.text_s = rt.dev.alloc((size_t) m.text_S * H * 4);
    m.mod_fin = rt.dev.alloc((size_t) m.T * 2 * H * 4);
    m.te_out = rt.dev.alloc(H * 4);
    m.gc_pre = rt.dev.alloc(H * 4);
    m.global_c = rt.dev.alloc(H * 4);
    m.probs = rt.dev.alloc((size_t) m.NH * S * S * 4);
    m.sc_l1 = rt.dev.alloc(SM);
    m.sc_r = rt.dev.alloc(SM);
    m.sc_f1 = rt.dev.alloc(SM_ffn);
    m.sc_f3 = rt.dev.alloc(SM_ffn);
    return m.probs.ok() && m.jointq.ok() && m.sc_f1.ok();
}

int main(int argc, char ** argv) {
    if (argc < 9) {
        fprintf(stderr, "usage: ts_ref_dit {forward|step|sample} <gguf> <T> <C> <TS> <in_dir> <out_dir> ...\n");
        return 2;
    }
    const std::string mode = argv[1], gguf = argv[2];
    const uint32_t T = (uint32_t) atoi(argv[3]), C = (uint32_t) atoi(argv[4]), TS = (uint32_t) atoi(argv[5]);
    const std::string in = argv[6], out = argv[7];

    Runtime rt;
    if (!rt.init("")) return 1;
    if (mode == "vae") {
        VaeModel vae;
        if (!vae.load(rt, gguf)) { fprintf(stderr, "vae load failed\n"); return 1; }
        std::vector<float> lat((size_t) T * 64);
        {
            FILE * f = fopen((in + "/latent.bin").c_str(), "rb");
            if (!f || fread(lat.data(), 4, lat.size(), f) != lat.size()) { fprintf(stderr, "missing latent.bin\n"); return 1; }
            fclose(f);
        }
        const int reps = argc > 8 ? atoi(argv[8]) : 1;
        int threads = 1;
#ifdef _OPENMP
        threads = omp_get_max_threads();
#endif
        std::vector<float> audio;
        uint32_t Ta = 0;
        printf("{\"mode\": \"vae\", \"threads\": %d, \"seconds\": [", threads);
        for (int r = 0; r < reps; ++r) {
            const auto t0 = std::chrono::steady_clock::now();
            audio = vae.decode(rt, lat.data(), T, Ta);
            const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            printf("%s%.6f", r ? ", " : "", sec);
        }
        printf("], \"T_audio\": %u}\n", Ta);
        write_from(out + "/audio.bin", audio.data(), audio.size());
        return 0;
    }
    if (mode == "t5" || mode == "clip") {
        std::vector<int32_t> ids(77);
        {
            FILE * f = fopen((in + "/ids.bin").c_str(), "rb");
            if (!f || fread(ids.data(), 4, ids.size(), f) != ids.size()) { fprintf(stderr, "missing ids.bin\n"); return 1; }
            fclose(f);
        }
        const int reps = argc > 8 ? atoi(argv[8]) : 1;
        int threads = 1;
#ifdef _OPENMP
        threads = omp_get_max_threads();
#endif
        std::vector<double> secs;
        if (mode == "t5") {
            T5Model t5;
            if (!t5.load(rt, gguf)) { fprintf(stderr, "t5 load failed\n"); return 1; }
            gpu::Buf o = rt.dev.alloc((size_t) 77 * t5.d_model * 4);
            for (int r = 0; r < reps; ++r) {
                const auto t0 = std::chrono::steady_clock::now();
                t5.encode(rt, ids, o);
                rt.dev.commit();
                secs.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
            }
            write_from(out + "/out.bin", o.p, (size_t) 77 * t5.d_model);
        } else {
            ClipModel clip;
            if (!clip.load(rt, gguf)) { fprintf(stderr, "clip load failed\n"); return 1; }
            gpu::Buf pt = rt.dev.alloc((size_t) clip.ctx * clip.H * 4), gl = rt.dev.alloc((size_t) clip.H * 4);
            for (int r = 0; r < reps; ++r) {
                const auto t0 = std::chrono::steady_clock::now();
                clip.encode(rt, ids, pt, gl);
                rt.dev.commit();
                secs.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
            }
            write_from(out + "/per_token.bin", pt.p, (size_t) clip.ctx * clip.H);
            write_from(out + "/global.bin", gl.p, clip.H);
        }
        printf("{\"mode\": \"%s\", \"threads\": %d, \"seconds\": [", mode.c_str(), threads);
        for (size_t i = 0; i < secs.size(); ++i) printf("%s%.6f", i ? ", " : "", secs[i]);
        printf("]}\n");
        return 0;
    }
    DitModel dit;
    if (!dit.load(rt, gguf)) { fprintf(stderr, "dit load failed\n"); return 1; }
    if (mode == "prep") {
        if (argc < 9) { fprintf(stderr, "prep needs <sync_S>\n"); return 2; }
        const uint32_t sync_S = (uint32_t) atoi(argv[8]), H = dit.H;
        dit.text_S = TS;
        gpu::Buf clip_f = rt.dev.alloc((size_t) C * 1024 * 4), sync_f = rt.dev.alloc((size_t) sync_S * 768 * 4);
        if (!read_into(in + "/clip_f.bin", clip_f, (size_t) C * 1024) ||
            !read_into(in + "/sync_f.bin", sync_f, (size_t) sync_S * 768)) return 1;
        if (!dit.prep_conditioning(rt, clip_f, sync_f, T, C, sync_S)) { fprintf(stderr, "prep failed\n"); return 1; }
        write_from(out + "/clip_pp.bin", dit.clip_pp.p, (size_t) C * H);
        write_from(out + "/sync_gather.bin", dit.sync_gather.p, (size_t) T * H);
        for (const char * arm : {"cond", "unc"}) {
            gpu::Buf tc = rt.dev.alloc((size_t) TS * 2048 * 4), gt = rt.dev.alloc(1024 * 4);
            gpu::Buf tp = rt.dev.alloc((size_t) TS * H * 4), gc = rt.dev.alloc(H * 4);
            if (!read_into(in + "/text_cat_" + arm + ".bin", tc, (size_t) TS * 2048) ||
                !read_into(in + "/gtext_" + arm + ".bin", gt, 1024)) return 1;
            dit.prep_text_arm(rt, tc, gt, tp, gc);
            write_from(out + "/text_pp_" + std::string(arm) + ".bin", tp.p, (size_t) TS * H);
            write_from(out + "/gcmlp_" + std::string(arm) + ".bin", gc.p, H);
        }
        return 0;
    }
    dit.T = T; dit.clip_S = C; dit.text_S = TS; dit.sync_S = 0;
    if (!alloc_forward_buffers(rt, dit)) { fprintf(stderr, "alloc failed\n"); return 1; }
    const uint32_t H = dit.H, L = dit.latent_dim;

    gpu::Buf x = rt.dev.alloc((size_t) T * L * 4);
    gpu::Buf tp_c = rt.dev.alloc((size_t) TS * H * 4), tp_u = rt.dev.alloc((size_t) TS * H * 4);
    gpu::Buf gc_c = rt.dev.alloc(H * 4), gc_u = rt.dev.alloc(H * 4);
    gpu::Buf fc = rt.dev.alloc((size_t) T * L * 4), fu = rt.dev.alloc((size_t) T * L * 4);
    bool ok = read_into(in + "/x.bin", x, (size_t) T * L) &&
              read_into(in + "/clip_pp.bin", dit.clip_pp, (size_t) C * H) &&
              read_into(in + "/sync_gather.bin", dit.sync_gather, (size_t) T * H);
    if (!ok) return 1;

    if (mode == "forward") {
        const float t = (float) atof(argv[8]);
        const std::string arm = argc > 9 ? argv[9] : "cond";
        if (!read_into(in + "/text_pp_" + arm + ".bin", tp_c, (size_t) TS * H) ||
            !read_into(in + "/gcmlp_" + arm + ".bin", gc_c, H)) return 1;
        setenv("TN_DUMP_EARLY", out.c_str(), 1);
        dit.forward(rt, x, t, tp_c, gc_c, fc);
        rt.dev.commit();
        unsetenv("TN_DUMP_EARLY");
        write_from(out + "/flow.bin", fc.p, (size_t) T * L);
        return 0;
    }

    if (!read_into(in + "/text_pp_cond.bin", tp_c, (size_t) TS * H) ||
        !read_into(in + "/gcmlp_cond.bin", gc_c, H) ||
        !read_into(in + "/text_pp_unc.bin", tp_u, (size_t) TS * H) ||
        !read_into(in + "/gcmlp_unc.bin", gc_u, H)) return 1;
#ifdef _OPENMP
    const int threads = omp_get_max_threads();
#else
    const int threads = 1;
#endif

    if (mode == "step") {
        if (argc < 11) { fprintf(stderr, "step needs <t> <cfg> <dt> [reps]\n"); return 2; }
        const float t = (float) atof(argv[8]), cfg = (float) atof(argv[9]), dt = (float) atof(argv[10]);
        const int reps = argc > 11 ? atoi(argv[11]) : 1;
        std::vector<double> secs;
        for (int r = 0; r < reps; ++r) {
            auto t0 = std::chrono::steady_clock::now();
            dit.forward(rt, x, t, tp_c, gc_c, fc);                            // pipeline.cpp:146
            dit.forward(rt, x, t, tp_u, gc_u, fu);                            // pipeline.cpp:147
            rt.cfg_euler(fc.p, fu.p, x.p, (size_t) T * L, cfg, dt);           // pipeline.cpp:148
            rt.dev.commit();
            secs.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
        }
        write_from(out + "/x_out.bin", x.p, (size_t) T * L);
        write_from(out + "/flow_cond.bin", fc.p, (size_t) T * L);
        write_from(out + "/flow_unc.bin", fu.p, (size_t) T * L);
        printf("{\"mode\": \"step\", \"threads\": %d, \"seconds\": [", threads);
        for (size_t i = 0; i < secs.size(); ++i) printf("%s%.6f", i ? ", " : "", secs[i]);
        printf("]}\n");
        return 0;
    }

    if (mode == "sample") {
        const int steps = atoi(argv[8]);
        const float cfg = argc > 9 ? (float) atof(argv[9]) : 5.0f;
        const long long x0_seed = argc > 10 ? atoll(argv[10]) : -1;
        std::vector<int> dump;
        if (argc > 11)
            for (const char * p = argv[11]; *p;) {
                dump.push_back(atoi(p));
                while (*p && *p != ',') ++p;
                if (*p == ',') ++p;
            }
        if (x0_seed >= 0) {                                                   // pipeline.cpp:126-132
            std::mt19937 rng((uint32_t) x0_seed);
            std::normal_distribution<float> nd(0, 1);
            for (uint32_t c = 0; c < L; ++c)
                for (uint32_t t = 0; t < T; ++t) ((float *) x.p)[(size_t) t * L + c] = nd(rng);
            write_from(out + "/x0.bin", x.p, (size_t) T * L);
        }
        auto t0 = std::chrono::steady_clock::now();
        for (int s = 0; s < steps; ++s) {                                     // pipeline.cpp:142-155
            float t_curr = 1.0f - (float) s / steps;
            float t_prev = 1.0f - (float) (s + 1) / steps;
            float dt = t_prev - t_curr;
            const bool d = std::find(dump.begin(), dump.end(), s) != dump.end();
            if (d) write_from(out + "/x_s" + std::to_string(s) + ".bin", x.p, (size_t) T * L);
            dit.forward(rt, x, t_curr, tp_c, gc_c, fc);
            dit.forward(rt, x, t_curr, tp_u, gc_u, fu);
            if (d) {
                rt.dev.commit();
                write_from(out + "/fc_s" + std::to_string(s) + ".bin", fc.p, (size_t) T * L);
                write_from(out + "/fu_s" + std::to_string(s) + ".bin", fu.p, (size_t) T * L);
            }
            rt.cfg_euler(fc.p, fu.p, x.p, (size_t) T * L, cfg, dt);
        }
        rt.dev.commit();
        const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        write_from(out + "/x_final.bin", x.p, (size_t) T * L);
        printf("{\"mode\": \"sample\", \"threads\": %d, \"steps\": %d, \"seconds\": %.6f}\n", threads, steps, sec);
        return 0;
    }
    fprintf(stderr, "unknown mode %s\n", mode.c_str());
    return 2;
}
