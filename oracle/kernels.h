// oracle/kernels.h — CPU restatement of the reference's Metal kernels (TEST INFRASTRUCTURE).
//
// This directory is the parity checker, not the product: only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline / reference legs may load it.
//
// Every kernel below restates one Metal kernel of the reference's DiT path in scalar C++.
// Param structs mirror the byte layout of the reference's constant blocks, because the
// reference's host code (src/net.mm, src/dit_fwd.cpp) hands those bytes to dispatch():
//   GemmP  src/gpu.h:52-58, shaders/gemm_attn.metal:5-10     AttnP src/gpu.h:60-69
//   ConvP  src/gpu.h:72-78                                    IcP   src/net.mm:44
//   AD/GA/RH/RP  src/dit_fwd.cpp:16-19, shaders/ops_conv.metal:117,128,147,157
//   QS3 src/dit_fwd.cpp:22   CD shaders/ops_conv.metal:194   CH/SH/HE/N1 shaders/ops_conv.metal
#pragma once
#include <cstddef>
#include <cstdint>

namespace oracle {

struct GemmP { uint32_t M, N, K, ldx, ldw, ldy, bias_mode, pad0; };
struct AttnP {
    uint32_t pad_on, Sq, Sk, hd, nh, ld, ldo, q_off, k_off, v_off, o_off, bias_mode, eot;
    float scale;
    uint32_t p_off;
};
struct ConvP { uint32_t T, OL, IC, OC, K, stride, pad, dil, ldx, ldy, convt, use_bias; };
struct IcP { uint32_t T, rows, IC, K, stride, pad, dil, ldx, convt, t0; };
struct AD { uint32_t H, per_row, chunks, base; float eps; };
struct GA { uint32_t H, per_row, chunks, gate_idx; };
struct RH { uint32_t ld, hd, col_off, row_off; float eps; };
struct RP { uint32_t ld, hd, col_off, row_off; float fscale, base; };
struct QS3 { uint32_t H, row_off; };
struct CD { float cfg, dt; uint32_t n; };
struct CH { uint32_t H, n; };
struct SH { uint32_t S, H; };
struct HE { uint32_t H; float eps; };

// Metal dispatch geometry: threadgroups (gx,gy,gz) of (tx,ty,tz) threads (src/gpu.mm:160-161).
struct Grid { uint32_t gx, gy, gz, tx, ty, tz; };

// Run the named kernel over its whole dispatch. bufs are raw pointers (unified memory in the
// reference, host memory here). Returns false if the name is unknown or params are short.
bool dispatch(const char * name, const Grid & g, const void * const * bufs, size_t nbufs,
              const void * params, size_t nparams);

// Direct entry points (used by the port in oracle/port.cpp; dispatch() routes here too).
// W16 is IEEE half bits (the reference's device weight type), W32 is f32.
void gemm_h(const uint16_t * W, const float * X, float * Y, const float * bias, const GemmP & p);
void gemm_f(const float * W, const float * X, float * Y, const float * bias, const GemmP & p);
void gemv_h(const uint16_t * W, const float * X, float * Y, const float * bias, const GemmP & p);
void gemv_f(const float * W, const float * X, float * Y, const float * bias, const GemmP & p);
void attn_qk(const float * QKV, float * P, const int32_t * bkt, const float * rb, const AttnP & p);
void softmax_rows(float * P, const AttnP & p);
void attn_pav(const float * P, const float * QKV, float * O, const AttnP & p);
void im2col(const float * x, float * col, const IcP & p, size_t n_threads);
void conv1d_fwd_h(const float * x, const uint16_t * w, const float * bias, float * y, const ConvP & p);
void conv1d_fwd_f(const float * x, const float * w, const float * bias, float * y, const ConvP & p);
void silu_(float * x, uint32_t n);
void copy_(const float * x, float * y, uint32_t n);
void swiglu_(const float * a, const float * b, float * y, uint32_t n);
void geglu_(const float * a, const float * b, float * y, uint32_t n);
void gelu_quick_(float * x, uint32_t n);
void add_(const float * a, const float * b, float * y, uint32_t n);
void add_bcast_col(const float * x, const float * v, float * y, const CH & p);
void qkv_split3(const float * src, float * dst, const QS3 & p, uint32_t rows);
void ln_plain(const float * x, float * y, const HE & p, uint32_t rows);
void ln_wb(const float * x, float * y, const float * w, const float * b, const HE & p, uint32_t rows);
void rms_w(const float * x, float * y, const float * w, const HE & p, uint32_t rows);
void rms_head(float * x, const float * w, const RH & p, uint32_t rows, uint32_t nh);
void adaln_ln(const float * x, const float * mod, float * y, const AD & p, uint32_t rows);
void gate_add(const float * x, const float * f, const float * mod, float * y, const GA & p, size_t n_threads);
void rope_pairs(float * qkv, const int32_t * pos, const RP & p, uint32_t rows, uint32_t npairs_total);
void mean_cols(const float * x, float * y, const SH & p);
void cfg_euler(const float * fc, const float * fu, float * x, const CD & p);
void snake_(const float * x, float * y, const float * ab, const SH & p);

float h2f(uint16_t h);

} // namespace oracle
