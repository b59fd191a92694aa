// IQ3_XXS decode primitives for sm_100a.
//
// Block format (reference cpp/core/src/quant.cpp:186-210, 98 bytes / 256 weights):
//   d   : fp16 super-scale
//   qs  : 64 grid indices (one byte per 4 weights) into the 256-entry codebook
//   aux : 8 u32 words, one per 32-weight sub-block: bits 0..27 hold four 7-bit
//         sign fields (one per 8 weights; the 8th sign is the parity bit),
//         bits 28..31 the 4-bit sub-scale s.
//   w   = d * (0.5 + s) * 0.5 * grid_byte * (+-1)
//       = d * (2s+1)/4 * (+-grid_byte)                      (exact in fp32)
//
// The GEMV path keeps the weight an exact small integer (+-grid_byte, int8)
// and moves d*(2s+1)/4 out of the inner product.  Activations are quantised
// per 16- or 32-element lane unit to int16 (x ~= sx * q), so one sub-block dot
// is exact integer arithmetic via dp2a (16-bit x 8-bit pairs):
//   sum_j w_j x_j = d*(2s+1)/4 * sx * sum_j (+-g_j) q_j
// The relative error this adds is ~3e-5 (int16 activation rounding).
//
// Lookup tables live in shared memory, replicated 32 times so each lane of a
// warp reads its own bank (conflict-free random lookups):
//   row r (r = 0..255) at byte offset 256*r:
//     words  0..31 : codebook entry r (4 unsigned magnitudes)
//     words 32..63 : for r < 128, the two PRMT selectors that apply sign field
//                    k = r to a pair of codebook words: low half for weights
//                    0..3, high half for weights 4..7.
// A selector picks byte j from the magnitude word (nibble j) or from its
// bytewise negation (nibble j+4), giving signed int8 weights in one PRMT.
#pragma once
#include "common.cuh"
#include "iq3xxs_grid.h"

#define GP_IQ3_BLOCK_BYTES 98

// Device copy of the codebook (one per translation unit; read only while
// building shared-memory tables).
static __constant__ uint32_t gp_iq3xxs_grid_dev[256] = {GPEED_IQ3XXS_GRID_VALUES};
#define GP_IQ3_TABLE_BYTES 65536

// Fills the 64 KB lookup table at tbl (dynamic shared memory) cooperatively.
GP_DEVINL void iq3_build_tables(uint8_t* tbl, int tid, int nthreads) {
    uint32_t* w = reinterpret_cast<uint32_t*>(tbl);
    for (int i = tid; i < 256 * 64; i += nthreads) {
        const int r = i >> 6, c = i & 63;
        uint32_t v = 0;
        if (c < 32) {
            v = gp_iq3xxs_grid_dev[r];
        } else if (r < 128) {
            const uint32_t s = (uint32_t)r | ((uint32_t)(__popc(r) & 1) << 7);  // 8 sign bits
            uint32_t sel0 = 0x3210u, sel1 = 0x3210u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sel0 |= ((s >> j) & 1u) << (4 * j + 2);
                sel1 |= ((s >> (j + 4)) & 1u) << (4 * j + 2);
            }
            v = sel0 | (sel1 << 16);
        }
        w[i] = v;
    }
}

// The lookup tables sit at the start of the kernel's dynamic shared memory,
// whose shared-window address is GP_DSMEM_BASE for kernels without static
// shared memory (1 KB is reserved by the system below it).  Folding that
// constant into the load's immediate offset makes each lookup one PRMT (or
// LOP3) plus one LDS.  Kernels verify the base at entry (gp_tables_at_base).
#define GP_DSMEM_BASE 1024u
GP_DEVINL bool gp_tables_at_base(const void* dyn_smem) { return smem_u32(dyn_smem) == GP_DSMEM_BASE; }
GP_DEVINL uint32_t tbl_grid(uint32_t off) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1+1024];" : "=r"(v) : "r"(off));
    return v;
}
GP_DEVINL uint32_t tbl_sel(uint32_t off) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1+1152];" : "=r"(v) : "r"(off));  // words 32..63 of row k
    return v;
}


// Codebook word for the index in byte `m` of q (selector constant 0x55m4:
// byte0 <- lane offset, byte1 <- index, bytes 2,3 <- 0 => index*256 + lane*4).
template <int M>
GP_DEVINL uint32_t iq3_grid(const uint8_t* tbl, uint32_t q, uint32_t lane4) {
    (void)tbl;
    return tbl_grid(prmt(q, lane4, 0x5504u | (M << 4)));
}

// Table offset of the selectors for the 7-bit sign field at bits 8..14 of f
// (the caller moves the field there).
GP_DEVINL uint32_t iq3_sel_off(uint32_t f, uint32_t lane4) { return (f & 0x7F00u) | lane4; }

// x >> n as a multiply-high, which issues on the FMA pipe instead of the
// integer ALU pipe that the byte permutes and dot products saturate.
template <int N>
GP_DEVINL uint32_t shr_fma(uint32_t x) {
    uint32_t r;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(1u << (32 - N)));
    return r;
}

// Signed int8 weights for 4 positions: magnitudes g, selector sel (low 16 bits).
GP_DEVINL uint32_t iq3_apply_sign(uint32_t g, uint32_t sel) {
    // bytewise negation without borrows: (256 - g_j) per byte, g_j in [4, 62]
    const uint32_t ng = 0x01010100u - g;
    return prmt(g, ng, sel);
}

// Decodes one 8-weight sign group: indices in bytes (M, M+1) of q, sign field
// pre-shifted into bits 8..14 of f.  Writes two signed int8x4 words.
template <int M>
GP_DEVINL void iq3_group(const uint8_t* tbl, uint32_t q, uint32_t f, uint32_t lane4, uint32_t& s0,
                         uint32_t& s1) {
    const uint32_t g0 = iq3_grid<M>(tbl, q, lane4);
    const uint32_t g1 = iq3_grid<M + 1>(tbl, q, lane4);
    const uint32_t sel = tbl_sel(iq3_sel_off(f, lane4));
    s0 = iq3_apply_sign(g0, sel);
    s1 = iq3_apply_sign(g1, shr_fma<16>(sel));
}

// Full 32-weight sub-block: q0/q1 = its 8 index bytes, aux = its scale/sign
// word.  sw[0..7] = signed int8x4 weights in natural order.
GP_DEVINL void iq3_decode_sub32(const uint8_t* tbl, uint32_t q0, uint32_t q1, uint32_t aux, uint32_t lane4,
                                uint32_t (&sw)[8]) {
    iq3_group<0>(tbl, q0, aux << 8, lane4, sw[0], sw[1]);
    iq3_group<2>(tbl, q0, aux << 1, lane4, sw[2], sw[3]);
    iq3_group<0>(tbl, q1, shr_fma<6>(aux), lane4, sw[4], sw[5]);
    iq3_group<2>(tbl, q1, shr_fma<13>(aux), lane4, sw[6], sw[7]);
}

// Half sub-block (16 weights, sign groups 2h and 2h+1): q = the 4 index bytes
// of that half, auxh = aux >> (14*h).
GP_DEVINL void iq3_decode_sub16(const uint8_t* tbl, uint32_t q, uint32_t auxh, uint32_t lane4, uint32_t (&sw)[4]) {
    iq3_group<0>(tbl, q, auxh << 8, lane4, sw[0], sw[1]);
    iq3_group<2>(tbl, q, auxh << 1, lane4, sw[2], sw[3]);
}

// Integer dot of N signed int8x4 weight words with 2N packed int16 pairs.
template <int N>
GP_DEVINL int iq3_idot(const uint32_t (&sw)[N], const uint32_t* xq) {
    int acc = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        acc = dp2a_lo(xq[2 * i], sw[i], acc);
        acc = dp2a_hi(xq[2 * i + 1], sw[i], acc);
    }
    return acc;
}

// d * (2s+1) / 4 for a sub-block (exact in fp32: 11-bit d times a 5-bit odd integer).
GP_DEVINL float iq3_subscale(float d, uint32_t aux) {
    return d * (float)((aux >> 27) | 1u) * 0.25f;
}
// The odd factor 2s+1 of a sub-block; |isum * (2s+1)| < 2^31 for int16 activations.
// (2 * (aux >> 28) + 1, all on the FMA pipe.)
GP_DEVINL int iq3_oddscale(uint32_t aux) { return (int)(shr_fma<28>(aux) * 2u + 1u); }

// Quantises UNIT activations to int16 pairs; returns the scale sx (x ~= sx*q).
template <int UNIT>
GP_DEVINL float quant_i16(const float (&v)[UNIT], uint32_t* xq) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < UNIT; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
#pragma unroll
    for (int p = 0; p < UNIT / 2; ++p) {
        const int a = __float2int_rn(v[2 * p] * inv);
        const int b = __float2int_rn(v[2 * p + 1] * inv);
        xq[p] = (static_cast<uint32_t>(a) & 0xFFFFu) | (static_cast<uint32_t>(b) << 16);
    }
    return amax * (1.0f / 32767.0f);
}

// ---- bit-exact fp32 decode (the reference's blk_iq3_xxs arithmetic) ---------
// y = (d*(0.5+s)*0.5 * g) * sign with IEEE round-to-nearest multiplies.
GP_DEVINL float iq3_weight_f32(float db, uint32_t g_byte, bool neg) {
    const float w = __fmul_rn(db, (float)g_byte);
    return neg ? -w : w;
}
GP_DEVINL float iq3_db(float d, uint32_t aux) {
    return __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.5f);
}
