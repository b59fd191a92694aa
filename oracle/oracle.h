/* Oracle for the IQ3_XXS routed-expert MoE path: a plain-C restatement of the
 * reference engine's CPU code, used ONLY as a checker by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg.  Nothing in the
 * product library links or calls it.
 *
 * Each function cites the reference file:line it restates (paths inside the
 * reference project).  The sibling oracle/_ref build links the reference's own
 * quant.cpp and exports the same entry points with a `ref_` prefix. */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_shape {
    int hidden;          /* H  (model_config.h:57-70 via ModelConfig) */
    int inter;           /* I  = moe_inter */
    int n_experts;       /* E */
    int top_k;           /* K */
    float routed_scale;  /* 2.5 */
    int norm_topk;       /* 1 */
    float swiglu_limit;  /* 10.0 */
} orc_shape;

/* quant.cpp:130-154 */
float orc_f16_to_f32(uint16_t h);
/* quant.cpp:521-573 (dequantize / dequantize_row for IQ3_XXS); returns -1 when
 * n is not a multiple of 256 (the reference throws, quant.cpp:523-524). */
int orc_dequantize_iq3xxs(const uint8_t* src, float* dst, uint64_t n);
/* quant.cpp:521-573 for every type the reference decodes: F32 (0), F16 (1),
 * Q8_0 (8), Q2_K (10), Q3_K (11), Q6_K (14), IQ3_XXS (18), IQ3_S (21),
 * IQ2_S (22), IQ4_XS (23), BF16 (30).  -1: n not a whole number of blocks;
 * -2: type not decoded by the reference. */
int orc_dequantize(int type, const uint8_t* src, float* dst, uint64_t n);
/* model.cpp:205-263 (Model::hc_forward) + the ffn RMSNorm, per token:
 * streams [n][N][H] -> x [n][H], post [n][N], comb [n][N][N]. */
int orc_mhc_pre(const float* streams, int n, int N, int H, int iters, float hc_eps, float rms_eps, const float* fn,
                const float* base, const float* scale, const float* norm_w, float* x, float* post, float* comb);
/* model.cpp:309-318: out[t][k] = post[t][k] mlp[t] + sum_m comb[t][m][k] in[t][m]. */
int orc_mhc_post(const float* in, const float* mlp, const float* post, const float* comb, int n, int N, int H,
                 float* out);
/* simd.h:12-37: AVX2 dot_f32 summation order, emulated with fmaf. */
float orc_dot_f32(const float* a, const float* b, int n);
/* weights.cpp:167-203: dst[j] = dot(decode(row row0+j), x). */
int orc_matvec_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim,
                     const float* x, float* dst);
/* weights.cpp:86-165: Y[t][j] for t < n_tok (numerically one dot per (t, j)). */
int orc_matmul_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim,
                     const float* X, int n_tok, float* Y);
/* model.cpp:692-756 (Model::moe_forward) for one token.  Expert tensors are
 * raw GGUF IQ3_XXS bytes laid out [E][rows][blocks]; the shared expert
 * pointers may be NULL (no shared expert).  forced (K ints) replaces the
 * top-k selection when not NULL.  topk_out / topw_out (K each) may be NULL. */
int orc_moe_forward(const orc_shape* s, const float* router_w, const float* corr,
                    const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                    const float* x, float* y, const int* forced, int* topk_out, float* topw_out);
/* model_batch.cpp:165-281 (Model::moe_batch) for n tokens; forced is n*K or
 * NULL; topk_out / topw_out are n*K or NULL (in per-token top-k order). */
int orc_moe_batch(const orc_shape* s, const float* router_w, const float* corr,
                  const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                  const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                  const float* X, int n, float* Y, const int* forced, int* topk_out, float* topw_out);
/* Host twin of the device synthetic generator (gpeed_b200/csrc/synth.h). */
void orc_synth_iq3xxs(uint64_t seed, uint64_t stream, uint64_t block0, uint64_t nblocks, uint8_t* dst);
int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
