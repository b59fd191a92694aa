/* Oracle (TEST INFRASTRUCTURE ONLY): CPU restatement of the reference engine's
 * IQ3_XXS routed-expert MoE path.  Used as the checker by tests/, smoke() and
 * the CPU-baseline leg of bench.py; never by the product.  Each function names
 * the reference file:line it follows (paths inside the reference project).
 *
 * Pinned by tests/test_oracle.py against (a) the reference's own IQ3_XXS
 * known-answer vector (python/tools/make_test_gguf.py seed 1234, checked by
 * tests/gguf_selftest.cpp), committed under tests/golden/, and (b) outputs of
 * the reference's compiled quant.cpp (oracle/_ref) on seeded inputs. */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "../gpeed_b200/csrc/iq3xxs_grid.h"
#include "../gpeed_b200/csrc/quant_grids.h"
#include "../gpeed_b200/csrc/synth.h"

#define QK_K 256
#define IQ3XXS_BLOCK_BYTES 98

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Host threads the OpenMP loops use from here on (torchrun starts its ranks
 * with OMP_NUM_THREADS=1; the CPU baseline wants every core). */
void orc_set_num_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

/* quant.cpp:130-154: IEEE half -> float including subnormals. */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            uint32_t ex = 127 - 15 + 1;
            while ((m & 0x400u) == 0) { m <<= 1; --ex; }
            bits = sign | (ex << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint8_t sign_byte(uint32_t k7) {
    /* iq3xxs_tables.h:61-70 (kSignsIq2xs): k with even parity in bit 7. */
    return (uint8_t)(k7 | ((uint32_t)(__builtin_popcount(k7) & 1) << 7));
}

/* quant.cpp:186-210 (blk_iq3_xxs): one 98-byte block -> 256 floats.
 * y = (db * grid) * (+-1) with db = (d * (0.5 + s)) * 0.5, all fp32, no FMA. */
static void decode_block(const uint8_t* blk, float* y) {
    uint16_t dh;
    memcpy(&dh, blk, 2);
    const float d = orc_f16_to_f32(dh);
    const uint8_t* qs = blk + 2;
    const uint8_t* sas = blk + 2 + QK_K / 4;
    for (int ib = 0; ib < 8; ++ib) {
        uint32_t aux;
        memcpy(&aux, sas + 4 * ib, 4);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int l = 0; l < 4; ++l) {
            const uint8_t signs = sign_byte((aux >> (7 * l)) & 127u);
            const uint32_t g1 = gpeed_iq3xxs_grid[qs[8 * ib + 2 * l + 0]];
            const uint32_t g2 = gpeed_iq3xxs_grid[qs[8 * ib + 2 * l + 1]];
            for (int j = 0; j < 4; ++j) {
                const float a = db * (float)((g1 >> (8 * j)) & 0xFF);
                const float b = db * (float)((g2 >> (8 * j)) & 0xFF);
                y[32 * ib + 8 * l + j] = (signs >> j) & 1 ? -a : a;
                y[32 * ib + 8 * l + j + 4] = (signs >> (j + 4)) & 1 ? -b : b;
            }
        }
    }
}

/* quant.cpp:521-573. */
int orc_dequantize_iq3xxs(const uint8_t* src, float* dst, uint64_t n) {
    if (n % QK_K) return -1;
    const int64_t nb = (int64_t)(n / QK_K);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b) decode_block(src + (size_t)b * IQ3XXS_BLOCK_BYTES, dst + (size_t)b * QK_K);
    return 0;
}

/* simd.h:12-37: two 8-wide FMA accumulators over 16-element steps, one more
 * 8-wide step into the first, lane-wise a0+a1, then (l0+l4, ..) halves,
 * two horizontal adds, and a scalar tail. */
float orc_dot_f32(const float* a, const float* b, int n) {
    float a0[8] = {0}, a1[8] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int k = 0; k < 8; ++k) {
            a0[k] = fmaf(a[i + k], b[i + k], a0[k]);
            a1[k] = fmaf(a[i + 8 + k], b[i + 8 + k], a1[k]);
        }
    for (; i + 8 <= n; i += 8)
        for (int k = 0; k < 8; ++k) a0[k] = fmaf(a[i + k], b[i + k], a0[k]);
    float s[8], lo[4];
    for (int k = 0; k < 8; ++k) s[k] = a0[k] + a1[k];
    for (int k = 0; k < 4; ++k) lo[k] = s[k] + s[k + 4];
    const float h0 = lo[0] + lo[1], h1 = lo[2] + lo[3];
    float acc = h0 + h1;
    for (; i < n; ++i) acc += a[i] * b[i];
    return acc;
}

/* ---- the other GGUF codecs the reference decodes (quant.cpp:165-519) ------
 * One restated block decoder per type, writing the block's values in order.
 * Arithmetic follows the reference's products term by term, without
 * contraction (-ffp-contract=off here; the reference's -O3 -mavx2 -mfma build
 * of quant.cpp does not contract Q2_K's dl * q - ml either: the two agree bit
 * for bit on every type). */

static const uint64_t kOrcIq2sGrid[1024] = {GPEED_IQ2S_GRID_VALUES};
static const uint32_t kOrcIq3sGrid[512] = {GPEED_IQ3S_GRID_VALUES};
static const int8_t kOrcIq4nl[16] = {GPEED_IQ4NL_VALUES};

static inline float h2f_at(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

/* quant.cpp:165-184: y = d * q */
static void blk_q8_0_(const uint8_t* b, float* y) {
    const float d = h2f_at(b);
    for (int i = 0; i < 32; ++i) y[i] = d * (float)(int8_t)b[2 + i];
}

/* quant.cpp:212-307 (the scalar branch; the AVX2 branch forms the same products) */
static void blk_q6_k_(const uint8_t* b, float* y) {
    const float d = h2f_at(b + 208);
    for (int h = 0; h < 2; ++h) {
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(b + 192 + 8 * h);
        float* o = y + 128 * h;
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = (int)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
            const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            o[l] = d * (float)sc[is] * (float)q1;
            o[l + 32] = d * (float)sc[is + 2] * (float)q2;
            o[l + 64] = d * (float)sc[is + 4] * (float)q3;
            o[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

/* quant.cpp:309-335: y = dl * q - ml, 16 values per scale */
static void blk_q2_k_(const uint8_t* b, float* y) {
    const float d = h2f_at(b + 80), mn = h2f_at(b + 82);
    int is = 0;
    for (int h = 0; h < 2; ++h) {
        const uint8_t* q = b + 16 + 32 * h;
        for (int j = 0; j < 4; ++j) {
            const int shift = 2 * j;
            for (int half = 0; half < 2; ++half) {
                const uint8_t sc = b[is++];
                const float dl = d * (float)(sc & 0xF), ml = mn * (float)(sc >> 4);
                for (int l = 0; l < 16; ++l)
                    *y++ = dl * (float)((q[l + 16 * half] >> shift) & 3) - ml;
            }
        }
    }
}

/* quant.cpp:337-371: 6-bit scales unpacked from 12 bytes; high bit from hmask */
static void blk_q3_k_(const uint8_t* b, float* y) {
    const uint8_t* hm = b;
    uint32_t aux[4];
    memcpy(aux, b + 96, 12);
    const uint32_t m1 = 0x03030303u, m2 = 0x0f0f0f0fu, t = aux[2];
    aux[2] = ((aux[0] >> 4) & m2) | (((t >> 4) & m1) << 4);
    aux[3] = ((aux[1] >> 4) & m2) | (((t >> 6) & m1) << 4);
    aux[0] = (aux[0] & m2) | ((t & m1) << 4);
    aux[1] = (aux[1] & m2) | (((t >> 2) & m1) << 4);
    const int8_t* scales = (const int8_t*)aux;
    const float d_all = h2f_at(b + 108);
    int is = 0;
    uint8_t m = 1;
    for (int h = 0; h < 2; ++h) {
        const uint8_t* q = b + 32 + 32 * h;
        for (int j = 0; j < 4; ++j, m <<= 1) {
            const int shift = 2 * j;
            for (int half = 0; half < 2; ++half) {
                const float dl = d_all * (float)(scales[is++] - 32);
                for (int l = 16 * half; l < 16 * half + 16; ++l)
                    *y++ = dl * (float)((int)((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4));
            }
        }
    }
}

/* quant.cpp:373-419: 10-bit grid index (qs + 2 bits of qh), explicit sign bytes.
 * As the AVX2 branch the reference builds with: the sign negates the grid byte
 * before the product (dl * -g; the scalar branch's (dl * g) * -1 differs only
 * in the sign of a NaN). */
static void blk_iq2_s_(const uint8_t* b, float* y) {
    const float d = h2f_at(b);
    const uint8_t* qs = b + 2;
    const uint8_t* qh = b + 66;
    const uint8_t* scales = b + 74;
    const uint8_t* signs = b + 2 + 32;
    for (int ib = 0; ib < 8; ++ib) {
        const float db0 = d * (0.5f + (float)(scales[ib] & 0xf)) * 0.25f;
        const float db1 = d * (0.5f + (float)(scales[ib] >> 4)) * 0.25f;
        for (int l = 0; l < 4; ++l) {
            const float dl = l < 2 ? db0 : db1;
            const uint32_t idx = (uint32_t)qs[l] | (((uint32_t)qh[ib] << (8 - 2 * l)) & 0x300u);
            const uint64_t g = kOrcIq2sGrid[idx];
            for (int j = 0; j < 8; ++j)
                y[j] = dl * (float)((signs[l] >> j) & 1 ? -(int)(uint8_t)(g >> (8 * j)) : (int)(uint8_t)(g >> (8 * j)));
            y += 8;
        }
        qs += 4;
        signs += 4;
    }
}

/* quant.cpp:421-483: 9-bit grid index (qs + 1 bit of qh), explicit sign bytes;
 * signed grid byte times db, as the AVX2 branch */
static void blk_iq3_s_(const uint8_t* b, float* y) {
    const float d = h2f_at(b);
    const uint8_t* qs = b + 2;
    const uint8_t* qh = b + 66;
    const uint8_t* signs = b + 74;
    const uint8_t* scales = b + 106;
    for (int ib = 0; ib < 8; ib += 2) {
        const float db1 = d * (1.0f + 2.0f * (float)(scales[ib / 2] & 0xf));
        const float db2 = d * (1.0f + 2.0f * (float)(scales[ib / 2] >> 4));
        for (int pass = 0; pass < 2; ++pass) {
            const float db = pass == 0 ? db1 : db2;
            for (int l = 0; l < 4; ++l) {
                const uint32_t i1 = (uint32_t)qs[2 * l] | (((uint32_t)qh[pass] << (8 - 2 * l)) & 256u);
                const uint32_t i2 = (uint32_t)qs[2 * l + 1] | (((uint32_t)qh[pass] << (7 - 2 * l)) & 256u);
                const uint32_t g1 = kOrcIq3sGrid[i1], g2 = kOrcIq3sGrid[i2];
                for (int j = 0; j < 4; ++j) {
                    const int a1 = (uint8_t)(g1 >> (8 * j)), a2 = (uint8_t)(g2 >> (8 * j));
                    y[j] = db * (float)((signs[l] >> j) & 1 ? -a1 : a1);
                    y[j + 4] = db * (float)((signs[l] >> (j + 4)) & 1 ? -a2 : a2);
                }
                y += 8;
            }
            qs += 8;
            signs += 4;
        }
        qh += 2;
    }
}

/* quant.cpp:485-503: 6-bit block scales, non-linear 4-bit values */
static void blk_iq4_xs_(const uint8_t* b, float* y) {
    const float d = h2f_at(b);
    uint16_t sh;
    memcpy(&sh, b + 2, 2);
    const uint8_t* sl = b + 4;
    const uint8_t* qs = b + 8;
    for (int ib = 0; ib < 8; ++ib) {
        const int ls = ((sl[ib / 2] >> (4 * (ib % 2))) & 0xf) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        for (int j = 0; j < 16; ++j) {
            y[j] = dl * (float)kOrcIq4nl[qs[j] & 0xf];
            y[j + 16] = dl * (float)kOrcIq4nl[qs[j] >> 4];
        }
        y += 32;
        qs += 16;
    }
}

/* quant.cpp:521-573: F32 / F16 / BF16 element-wise, block types per block;
 * -1 for a count that is not a whole number of blocks, -2 for a type the
 * reference does not decode (it throws in both cases). */
int orc_dequantize(int type, const uint8_t* src, float* dst, uint64_t n) {
    void (*fn)(const uint8_t*, float*) = NULL;
    int bytes = 0, vals = 256;
    switch (type) {
        case 0: memcpy(dst, src, (size_t)n * 4); return 0;
        case 1:
            for (uint64_t i = 0; i < n; ++i) dst[i] = h2f_at(src + 2 * i);
            return 0;
        case 30:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                memcpy(&h, src + 2 * i, 2);
                const uint32_t bits = (uint32_t)h << 16;
                memcpy(dst + i, &bits, 4);
            }
            return 0;
        case 8: fn = blk_q8_0_; bytes = 34; vals = 32; break;
        case 10: fn = blk_q2_k_; bytes = 84; break;
        case 11: fn = blk_q3_k_; bytes = 110; break;
        case 14: fn = blk_q6_k_; bytes = 210; break;
        case 18: return orc_dequantize_iq3xxs(src, dst, n);
        case 21: fn = blk_iq3_s_; bytes = 110; break;
        case 22: fn = blk_iq2_s_; bytes = 82; break;
        case 23: fn = blk_iq4_xs_; bytes = 136; break;
        default: return -2;
    }
    if (n % (uint64_t)vals) return -1;
    const int64_t nb = (int64_t)(n / (uint64_t)vals);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nb; ++i) fn(src + (size_t)i * bytes, dst + (size_t)i * vals);
    return 0;
}

static size_t row_bytes(int in_dim) { return (size_t)(in_dim / QK_K) * IQ3XXS_BLOCK_BYTES; }

/* weights.cpp:167-203 (WeightStore::matvec_quant): decode each row, dot with x. */
int orc_matvec_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim,
                     const float* x, float* dst) {
    if (in_dim % QK_K) return -1;
    const size_t rb = row_bytes(in_dim);
    const uint8_t* src = w + row0 * rb;
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)in_dim);
#pragma omp for schedule(static)
        for (int j = 0; j < out_dim; ++j) {
            for (int b = 0; b < in_dim / QK_K; ++b)
                decode_block(src + rb * (size_t)j + (size_t)b * IQ3XXS_BLOCK_BYTES, row + b * QK_K);
            dst[j] = orc_dot_f32(row, x, in_dim);
        }
        free(row);
    }
    return 0;
}

/* weights.cpp:86-165 (WeightStore::matmul_quant).  Both of its regimes compute
 * Y[t][j] = dot_f32(decoded row j, X[t]); this restatement uses the
 * row-parallel form (weights.cpp:113-132). */
int orc_matmul_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim,
                     const float* X, int n_tok, float* Y) {
    if (n_tok <= 0 || out_dim <= 0) return 0;
    if (in_dim % QK_K) return -1;
    const size_t rb = row_bytes(in_dim);
    const uint8_t* src = w + row0 * rb;
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)in_dim);
#pragma omp for schedule(static)
        for (int j = 0; j < out_dim; ++j) {
            for (int b = 0; b < in_dim / QK_K; ++b)
                decode_block(src + rb * (size_t)j + (size_t)b * IQ3XXS_BLOCK_BYTES, row + b * QK_K);
            for (int t = 0; t < n_tok; ++t)
                Y[(size_t)t * out_dim + j] = orc_dot_f32(row, X + (size_t)t * in_dim, in_dim);
        }
        free(row);
    }
    return 0;
}

/* ops.h:16-17 */
static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
static inline float siluf_(float x) { return x / (1.0f + expf(-x)); }
static inline float minf_(float a, float b) { return b < a ? b : a; }
static inline float clampf_(float v, float lo, float hi) { return v < lo ? lo : (hi < v ? hi : v); }

/* simd.h:40-50 (axpy_f32 uses FMA: a += s*b). */
static void axpy_(float* a, const float* b, float s, int n) {
    for (int i = 0; i < n; ++i) a[i] = fmaf(s, b[i], a[i]);
}

/* std::partial_sort(idx, idx+K, idx+E, choice[a] > choice[b]) (model.cpp:714-716):
 * the K largest by choice, in descending order.  Ties (absent with continuous
 * random inputs) resolve to the lower expert id here. */
static void topk_desc(const float* choice, int E, int K, int* out) {
    for (int k = 0; k < K; ++k) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
            int taken = 0;
            for (int q = 0; q < k; ++q) taken |= (out[q] == e);
            if (taken) continue;
            if (best < 0 || choice[e] > choice[best]) best = e;
        }
        out[k] = best;
    }
}

static void swiglu_(const float* g, const float* u, float* h, int n, float lim) {
    for (int i = 0; i < n; ++i) {
        const float gi = minf_(g[i], lim);
        const float ui = clampf_(u[i], -lim, lim);
        h[i] = siluf_(gi) * ui;
    }
}

/* model.cpp:692-756 (Model::moe_forward). */
int orc_moe_forward(const orc_shape* s, const float* router_w, const float* corr,
                    const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                    const float* x, float* y, const int* forced, int* topk_out, float* topw_out) {
    const int H = s->hidden, I = s->inter, E = s->n_experts, K = s->top_k;
    if (H % QK_K || I % QK_K || K <= 0 || K > E) return -1;
    float* logits = (float*)malloc(sizeof(float) * E);
    float* scores = (float*)malloc(sizeof(float) * E);
    float* choice = (float*)malloc(sizeof(float) * E);
    int* idx = (int*)malloc(sizeof(int) * K);
    float* wsum = (float*)malloc(sizeof(float) * K);
    float* g = (float*)malloc(sizeof(float) * I);
    float* u = (float*)malloc(sizeof(float) * I);
    float* h = (float*)malloc(sizeof(float) * I);
    float* dn = (float*)malloc(sizeof(float) * H);

    /* router matvec (model.cpp:41-46, 702), sigmoid + bias (704-708) */
    for (int e = 0; e < E; ++e) logits[e] = orc_dot_f32(router_w + (size_t)e * H, x, H);
    for (int e = 0; e < E; ++e) {
        scores[e] = sigmoidf_(logits[e]);
        choice[e] = scores[e] + (corr ? corr[e] : 0.0f);
    }
    if (forced) memcpy(idx, forced, sizeof(int) * K);
    else topk_desc(choice, E, K, idx);
    /* renormalise and scale (model.cpp:718-725) */
    float denom = 1e-20f;
    for (int k = 0; k < K; ++k) { wsum[k] = scores[idx[k]]; denom += wsum[k]; }
    if (s->norm_topk) for (int k = 0; k < K; ++k) wsum[k] /= denom;
    for (int k = 0; k < K; ++k) wsum[k] *= s->routed_scale;

    for (int i = 0; i < H; ++i) y[i] = 0.0f;
    for (int k = 0; k < K; ++k) {   /* model.cpp:729-743 */
        const int e = idx[k];
        orc_matvec_quant(gate_exps, (uint64_t)e * I, H, I, x, g);
        orc_matvec_quant(up_exps, (uint64_t)e * I, H, I, x, u);
        swiglu_(g, u, h, I, s->swiglu_limit);
        orc_matvec_quant(down_exps, (uint64_t)e * H, I, H, h, dn);
        axpy_(y, dn, wsum[k], H);
    }
    if (gate_sh) {                   /* model.cpp:745-755 */
        orc_matvec_quant(gate_sh, 0, H, I, x, g);
        orc_matvec_quant(up_sh, 0, H, I, x, u);
        swiglu_(g, u, h, I, s->swiglu_limit);
        orc_matvec_quant(down_sh, 0, I, H, h, dn);
        for (int i = 0; i < H; ++i) y[i] += dn[i];
    }
    if (topk_out) memcpy(topk_out, idx, sizeof(int) * K);
    if (topw_out) memcpy(topw_out, wsum, sizeof(float) * K);
    free(logits); free(scores); free(choice); free(idx); free(wsum);
    free(g); free(u); free(h); free(dn);
    return 0;
}

/* model_batch.cpp:165-281 (Model::moe_batch). */
int orc_moe_batch(const orc_shape* s, const float* router_w, const float* corr,
                  const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                  const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                  const float* X, int n, float* Y, const int* forced, int* topk_out, float* topw_out) {
    const int H = s->hidden, I = s->inter, E = s->n_experts, K = s->top_k;
    if (H % QK_K || I % QK_K || K <= 0 || K > E || n < 0) return -1;
    if (n == 0) return 0;
    const size_t nk = (size_t)n * K;
    float* logit = (float*)malloc(sizeof(float) * (size_t)n * E);
    float* score = (float*)malloc(sizeof(float) * E);
    float* choice = (float*)malloc(sizeof(float) * E);
    int* idx = (int*)malloc(sizeof(int) * K);
    int* a_tok = (int*)malloc(sizeof(int) * nk);
    int* a_e = (int*)malloc(sizeof(int) * nk);
    float* a_w = (float*)malloc(sizeof(float) * nk);
    int* cnt = (int*)calloc((size_t)E, sizeof(int));
    int* eptr = (int*)malloc(sizeof(int) * (E + 1));
    int* cursor = (int*)malloc(sizeof(int) * E);
    int* b_tok = (int*)malloc(sizeof(int) * nk);
    float* b_wt = (float*)malloc(sizeof(float) * nk);

    /* 1. router for all tokens (model_batch.cpp:172) */
    for (int t = 0; t < n; ++t)
        for (int e = 0; e < E; ++e)
            logit[(size_t)t * E + e] = orc_dot_f32(router_w + (size_t)e * H, X + (size_t)t * H, H);
    /* 2. per-token top-k and assignment list (model_batch.cpp:184-203) */
    size_t na = 0;
    for (int t = 0; t < n; ++t) {
        const float* lg = logit + (size_t)t * E;
        for (int e = 0; e < E; ++e) {
            score[e] = 1.0f / (1.0f + expf(-lg[e]));
            choice[e] = score[e] + (corr ? corr[e] : 0.0f);
        }
        if (forced) memcpy(idx, forced + (size_t)t * K, sizeof(int) * K);
        else topk_desc(choice, E, K, idx);
        float denom = 1e-20f;
        for (int k = 0; k < K; ++k) denom += score[idx[k]];
        const float inv = s->norm_topk ? s->routed_scale / denom : s->routed_scale;
        for (int k = 0; k < K; ++k) {
            const int e = idx[k];
            a_tok[na] = t; a_e[na] = e; a_w[na] = score[e] * inv;
            if (topk_out) topk_out[(size_t)t * K + k] = e;
            if (topw_out) topw_out[(size_t)t * K + k] = score[e] * inv;
            ++na;
            ++cnt[e];
        }
    }
    /* histogram -> exclusive scan (model_batch.cpp:204-209) */
    int acc = 0;
    for (int e = 0; e < E; ++e) { eptr[e] = acc; acc += cnt[e]; }
    eptr[E] = acc;
    /* stable bucket sort by expert id (model_batch.cpp:211-219) */
    for (int e = 0; e < E; ++e) cursor[e] = eptr[e];
    for (size_t a = 0; a < na; ++a) {
        const int p = cursor[a_e[a]]++;
        b_tok[p] = a_tok[a];
        b_wt[p] = a_w[a];
    }
    for (size_t i = 0; i < (size_t)n * H; ++i) Y[i] = 0.0f;

    /* 3. one grouped pass per touched expert (model_batch.cpp:224-262) */
    int gmax = 0;
    for (int e = 0; e < E; ++e) if (cnt[e] > gmax) gmax = cnt[e];
    float* Xg = (float*)malloc(sizeof(float) * (size_t)(gmax ? gmax : 1) * H);
    float* Gg = (float*)malloc(sizeof(float) * (size_t)(gmax > n ? gmax : n) * I);
    float* Ug = (float*)malloc(sizeof(float) * (size_t)(gmax > n ? gmax : n) * I);
    float* Hg = (float*)malloc(sizeof(float) * (size_t)(gmax > n ? gmax : n) * I);
    float* Dg = (float*)malloc(sizeof(float) * (size_t)(gmax > n ? gmax : n) * H);
    for (int e = 0; e < E; ++e) {
        const int lo = eptr[e], hi = eptr[e + 1], gcount = hi - lo;
        if (gcount == 0) continue;
        for (int i = 0; i < gcount; ++i)
            memcpy(Xg + (size_t)i * H, X + (size_t)b_tok[lo + i] * H, sizeof(float) * H);
        orc_matmul_quant(gate_exps, (uint64_t)e * I, H, I, Xg, gcount, Gg);
        orc_matmul_quant(up_exps, (uint64_t)e * I, H, I, Xg, gcount, Ug);
        for (int i = 0; i < gcount * I; ++i) {
            const float gi = minf_(Gg[i], s->swiglu_limit);
            const float ui = clampf_(Ug[i], -s->swiglu_limit, s->swiglu_limit);
            Hg[i] = (gi / (1.0f + expf(-gi))) * ui;
        }
        orc_matmul_quant(down_exps, (uint64_t)e * H, I, H, Hg, gcount, Dg);
        for (int i = 0; i < gcount; ++i)
            axpy_(Y + (size_t)b_tok[lo + i] * H, Dg + (size_t)i * H, b_wt[lo + i], H);
    }
    /* 4. shared expert over all tokens (model_batch.cpp:264-280) */
    if (gate_sh) {
        orc_matmul_quant(gate_sh, 0, H, I, X, n, Gg);
        orc_matmul_quant(up_sh, 0, H, I, X, n, Ug);
        for (int i = 0; i < n * I; ++i) {
            const float gi = minf_(Gg[i], s->swiglu_limit);
            const float ui = clampf_(Ug[i], -s->swiglu_limit, s->swiglu_limit);
            Hg[i] = (gi / (1.0f + expf(-gi))) * ui;
        }
        orc_matmul_quant(down_sh, 0, I, H, Hg, n, Dg);
        for (size_t i = 0; i < (size_t)n * H; ++i) Y[i] += Dg[i];
    }
    free(Xg); free(Gg); free(Ug); free(Hg); free(Dg);
    free(logit); free(score); free(choice); free(idx); free(a_tok); free(a_e); free(a_w);
    free(cnt); free(eptr); free(cursor); free(b_tok); free(b_wt);
    return 0;
}

/* ---- mHC residual mixing around the MoE layer ----------------------------- */

/* ops.h rmsnorm: y = x * (1 / sqrt(mean(x^2) + eps)) [* w] */
static void rmsnorm_(float* out, const float* x, const float* w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    const float rstd = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = w ? x[i] * rstd * w[i] : x[i] * rstd;
}

/* model.cpp:49-59 softmax (max-subtracted) */
static void softmax_(float* s, int n) {
    float mx = s[0];
    for (int i = 1; i < n; ++i) mx = s[i] > mx ? s[i] : mx;
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        s[i] = expf(s[i] - mx);
        sum += s[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) s[i] *= inv;
}

/* model.cpp:205-263 (Model::hc_forward) then the ffn norm (model.cpp:292-296,
 * model_batch.cpp:374-384), per token */
int orc_mhc_pre(const float* streams, int n, int N, int H, int iters, float hc_eps, float rms_eps, const float* fn,
                const float* base, const float* scale, const float* norm_w, float* x, float* post, float* comb) {
    if (N < 1 || N > 8 || iters < 1) return -1;
    const int HN = N * H, W = (2 + N) * N;
    float* flat = (float*)malloc(sizeof(float) * (size_t)HN);
    float* mixed = (float*)malloc(sizeof(float) * (size_t)H);
    float w[80], pre[8], row[8];
    for (int t = 0; t < n; ++t) {
        const float* S = streams + (size_t)t * HN;
        float* po = post + (size_t)t * N;
        float* cb = comb + (size_t)t * N * N;
        rmsnorm_(flat, S, NULL, HN, rms_eps);
        for (int j = 0; j < W; ++j) w[j] = orc_dot_f32(fn + (size_t)j * HN, flat, HN);  /* matvec, model.cpp:41-46 */
        for (int i = 0; i < N; ++i) {
            pre[i] = 1.0f / (1.0f + expf(-(w[i] * scale[0] + base[i]))) + hc_eps;
            po[i] = 2.0f * (1.0f / (1.0f + expf(-(w[N + i] * scale[1] + base[N + i]))));
        }
        for (int i = 0; i < N; ++i) {
            for (int j = 0; j < N; ++j) row[j] = w[2 * N + i * N + j] * scale[2] + base[2 * N + i * N + j];
            softmax_(row, N);
            for (int j = 0; j < N; ++j) cb[i * N + j] = row[j] + hc_eps;
        }
        for (int j = 0; j < N; ++j) {  /* Sinkhorn: columns, then (iters - 1) x (rows, columns) */
            float d = 0.0f;
            for (int i = 0; i < N; ++i) d += cb[i * N + j];
            d += hc_eps;
            for (int i = 0; i < N; ++i) cb[i * N + j] /= d;
        }
        for (int it = 0; it < iters - 1; ++it) {
            for (int i = 0; i < N; ++i) {
                float d = 0.0f;
                for (int j = 0; j < N; ++j) d += cb[i * N + j];
                d += hc_eps;
                for (int j = 0; j < N; ++j) cb[i * N + j] /= d;
            }
            for (int j = 0; j < N; ++j) {
                float d = 0.0f;
                for (int i = 0; i < N; ++i) d += cb[i * N + j];
                d += hc_eps;
                for (int i = 0; i < N; ++i) cb[i * N + j] /= d;
            }
        }
        for (int d = 0; d < H; ++d) mixed[d] = 0.0f;
        for (int i = 0; i < N; ++i)
            for (int d = 0; d < H; ++d) mixed[d] += pre[i] * S[(size_t)i * H + d];
        rmsnorm_(x + (size_t)t * H, mixed, norm_w, H, rms_eps);
    }
    free(flat);
    free(mixed);
    return 0;
}

/* model.cpp:309-318 / model_batch.cpp:395-409: streams after the MLP */
int orc_mhc_post(const float* in, const float* mlp, const float* post, const float* comb, int n, int N, int H,
                 float* out) {
    for (int t = 0; t < n; ++t)
        for (int k = 0; k < N; ++k)
            for (int d = 0; d < H; ++d) {
                float acc = post[(size_t)t * N + k] * mlp[(size_t)t * H + d];
                for (int m = 0; m < N; ++m)
                    acc += comb[(size_t)t * N * N + m * N + k] * in[((size_t)t * N + m) * H + d];
                out[((size_t)t * N + k) * H + d] = acc;
            }
    return 0;
}

void orc_synth_iq3xxs(uint64_t seed, uint64_t stream, uint64_t block0, uint64_t nblocks, uint8_t* dst) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < (int64_t)nblocks; ++b)
        gp_synth_iq3xxs_block(seed, stream, block0 + (uint64_t)b, dst + (size_t)b * IQ3XXS_BLOCK_BYTES);
}
