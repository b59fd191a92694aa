// Counter-based synthetic IQ3_XXS weight generator.
//
// Every byte of a synthetic expert tensor is a pure function of
// (seed, stream, block index), so the device can fill tens of GB in place
// and the host can rebuild any slice of it bit for bit for a parity check.
//
// Per 98-byte block (the GGUF IQ3_XXS layout: fp16 d, 64 grid-index bytes,
// 8 little-endian u32 scale/sign words):
//   d   = fp16_rne(2e-4f + 1.8e-3f * u),  u = (w0 >> 40) * 2^-24   (uniform in [2e-4, 2e-3))
//   qs  = the 64 bytes of w1..w8          (uniform 0..255)
//   aux = the 32 bytes of w9..w12         (uniform u32)
// where w_j = gp_hash(seed, stream, 16*block + j).  The fp32 arithmetic is two
// correctly rounded operations (no fused multiply-add) on both sides.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define GP_HD __host__ __device__ __forceinline__
#else
#define GP_HD static inline
#endif

GP_HD uint64_t gp_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

GP_HD uint64_t gp_hash(uint64_t seed, uint64_t stream, uint64_t idx) {
    return gp_mix64(gp_mix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) + idx);
}

// IEEE binary32 -> binary16, round to nearest even (finite inputs in the
// normal fp16 range only, which is all the generator produces).
GP_HD uint16_t gp_f32_to_f16_rne(float f) {
    union { float f; uint32_t u; } v;
    v.f = f;
    const uint32_t sign = (v.u >> 16) & 0x8000u;
    const int32_t exp = (int32_t)((v.u >> 23) & 0xFFu) - 127 + 15;
    uint32_t man = v.u & 0x7FFFFFu;
    uint32_t h = sign | ((uint32_t)exp << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;  // carry may bump the exponent: still correct
    return (uint16_t)h;
}

GP_HD float gp_block_scale_f32(uint64_t w0) {
    const float u = (float)(uint32_t)(w0 >> 40) * (1.0f / 16777216.0f);  // exact: 24-bit integer * 2^-24
#if defined(__CUDA_ARCH__)
    return __fadd_rn(2e-4f, __fmul_rn(1.8e-3f, u));
#else
    volatile float p = 1.8e-3f * u;  // volatile: keep the product rounded (no contraction)
    return 2e-4f + p;
#endif
}

// Writes one 98-byte IQ3_XXS block for (seed, stream, block) into dst.
GP_HD void gp_synth_iq3xxs_block(uint64_t seed, uint64_t stream, uint64_t block, uint8_t* dst) {
    const uint64_t base = block * 16u;
    const uint64_t w0 = gp_hash(seed, stream, base);
    const uint16_t d = gp_f32_to_f16_rne(gp_block_scale_f32(w0));
    dst[0] = (uint8_t)(d & 0xFF);
    dst[1] = (uint8_t)(d >> 8);
    for (int j = 0; j < 12; ++j) {
        const uint64_t w = gp_hash(seed, stream, base + 1u + (uint64_t)j);
        for (int b = 0; b < 8; ++b) dst[2 + 8 * j + b] = (uint8_t)(w >> (8 * b));
    }
}
