/* tsn_synth.h — deterministic synthetic tensors shared by the GGUF writer, the on-device
 * weight generator and the CPU oracle.
 *
 * The reference ships no weights or golden dumps for its DiT path, so every parity test and
 * benchmark runs on seeded synthetic tensors. To let the host writer, the CUDA generator and
 * the oracle produce BIT-IDENTICAL values without sharing transcendental math (glibc and CUDA
 * logf/cosf differ in the last ulp), the normal deviate is an Irwin–Hall(12) sum of 16-bit
 * uniforms drawn from a splitmix64 counter stream:
 *
 *     z = (sum_{j<12} v_j - 393210) / 65536,   v_j in [0, 65535]
 *
 * Mean 0, variance (1 - 2^-32) ~ 1, support +-6. The numerator is an integer below 2^19 in
 * magnitude, so z is exact in f32; scaling by a standard deviation is one f32 multiply and the
 * BF16 rounding is round-to-nearest-even on the bit pattern — all deterministic on any IEEE
 * host or device.
 *
 * Streams are keyed by (seed, FNV-1a 64 of a tensor name); element i of a tensor uses counters
 * 3i, 3i+1, 3i+2 of its stream.
 */
#ifndef TSN_SYNTH_H
#define TSN_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define TSN_HD __host__ __device__ __forceinline__
#else
#define TSN_HD static inline
#endif

TSN_HD uint64_t tsn_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* FNV-1a 64 of a NUL-terminated name, mixed with the seed: the stream key of one tensor. */
TSN_HD uint64_t tsn_stream_key(const char * name, uint64_t seed) {
    uint64_t h = 1469598103934665603ull;
    for (const char * p = name; *p; ++p) { h ^= (uint8_t) *p; h *= 1099511628211ull; }
    return tsn_splitmix64(h ^ tsn_splitmix64(seed));
}

/* Irwin–Hall(12) standard normal deviate, element idx of stream key. Exact in f32. */
TSN_HD float tsn_normal(uint64_t key, uint64_t idx) {
    int32_t s = 0;
    for (int j = 0; j < 3; ++j) {
        uint64_t r = tsn_splitmix64(key + 3ull * idx + (uint64_t) j);
        s += (int32_t) (r & 0xFFFF) + (int32_t) ((r >> 16) & 0xFFFF) +
             (int32_t) ((r >> 32) & 0xFFFF) + (int32_t) (r >> 48);
    }
    return (float) (s - 393210) * (1.0f / 65536.0f);
}

/* f32 -> bf16 bits, round to nearest even (NaN kept quiet). */
TSN_HD uint16_t tsn_f32_to_bf16(float f) {
    union { float f; uint32_t u; } c; c.f = f;
    uint32_t u = c.u;
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t) ((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t) (u >> 16);
}

TSN_HD float tsn_bf16_to_f32(uint16_t h) {
    union { uint32_t u; float f; } c; c.u = (uint32_t) h << 16;
    return c.f;
}

/* The reference's weight conversion: f32 -> f16 bits with round-to-nearest-even on the 13
 * dropped mantissa bits, f32 zero/denormal flushed to signed zero, f16-subnormal results
 * truncated, overflow to inf (src/net.mm:144-164). Every DiT weight passes through this on the
 * reference's device, so the CUDA build applies the identical rule to the BF16 file values. */
TSN_HD uint16_t tsn_ref_f32_to_f16(float f) {
    union { float f; uint32_t u; } c; c.f = f;
    uint32_t x = c.u;
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t) ((x >> 23) & 0xFF) - 127 + 15;
    uint32_t man = x & 0x7FFFFFu;
    if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t) (sign | 0x7C00u | (man ? 0x200u : 0u));
    if (((x >> 23) & 0xFF) == 0) return (uint16_t) sign;
    if (exp >= 0x1F) return (uint16_t) (sign | 0x7C00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t) sign;
        man |= 0x800000u;
        uint32_t shift = (uint32_t) (1 - exp);
        uint32_t dm = man >> (shift + 13);
        return (uint16_t) (sign | dm);
    }
    uint16_t base = (uint16_t) (sign | ((uint32_t) exp << 10) | (man >> 13));
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (base & 1u))) base = (uint16_t) (base + 1u);
    return base;
}

/* IEEE f16 bits -> f32, subnormals included (what a GPU does when it reads `half`). */
TSN_HD float tsn_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) u = sign;
        else {                              /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400u));
            man &= 0x3FFu;
            u = sign | ((uint32_t) (127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) u = sign | 0x7F800000u | (man << 13);
    else u = sign | ((exp + 112u) << 23) | (man << 13);
    union { uint32_t u; float f; } c; c.u = u;
    return c.f;
}

/* Initialisation kinds used by the synthetic DiT fixture. */
enum tsn_init_kind {
    TSN_INIT_NORMAL = 0,      /* scale * N(0,1)              */
    TSN_INIT_ONE_PLUS = 1,    /* 1 + scale * N(0,1) (norm gains) */
};

/* One rounded multiply, then one rounded add: no fused multiply-add on either side (nvcc
 * contracts a*b+c by default; host builds of this header use -ffp-contract=off). */
TSN_HD float tsn_init_value(uint64_t key, uint64_t idx, int kind, float scale) {
#if defined(__CUDA_ARCH__)
    float z = __fmul_rn(tsn_normal(key, idx), scale);
    return kind == TSN_INIT_ONE_PLUS ? __fadd_rn(1.0f, z) : z;
#else
    volatile float z = tsn_normal(key, idx) * scale;
    return kind == TSN_INIT_ONE_PLUS ? 1.0f + z : z;
#endif
}

#endif /* TSN_SYNTH_H */
