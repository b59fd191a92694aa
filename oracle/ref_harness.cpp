// Reference harness (TEST INFRASTRUCTURE ONLY): links the reference engine's
// own codec (cpp/core/src/quant.cpp, compiled from the reference tree by
// oracle/Makefile into oracle/_ref/) and its header-only SIMD/activation
// helpers (simd.h, ops.h), and drives them with the loop structure of the
// reference's expert path.  Model::moe_forward / moe_batch are private members
// that need a whole GGUF model, so their control flow is restated here; every
// arithmetic step is the reference's own function:
//   decode  glm5::dequantize_row (quant.cpp:571, blk_iq3_xxs :186-210)
//   dot     glm5::dot_f32 (simd.h:12-37), axpy_f32 (:40-50), add_f32 (:53-62)
//   act     glm5::sigmoidf / siluf (ops.h:16-17)
// Exported with a ref_ prefix and the same signatures as oracle/oracle.h.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "glm5/ops.h"
#include "glm5/quant.h"
#include "glm5/simd.h"

#ifdef _OPENMP
#include <omp.h>
#endif

#include "oracle.h"

using namespace glm5;

namespace {

size_t row_bytes(int in_dim) { return static_cast<size_t>(in_dim / QK_K) * 98u; }

// weights.cpp:167-203 with the tensor payload already resident in RAM.
void matvec(const uint8_t* w, uint64_t row0, int in_dim, int out_dim, const float* x, float* dst) {
    const size_t rb = row_bytes(in_dim);
    const uint8_t* src = w + row0 * rb;
#pragma omp parallel
    {
        std::vector<float> row(static_cast<size_t>(in_dim));
#pragma omp for schedule(static)
        for (int j = 0; j < out_dim; ++j) {
            dequantize_row(DType::IQ3_XXS, src + rb * static_cast<size_t>(j), row.data(),
                           static_cast<uint64_t>(in_dim));
            dst[j] = dot_f32(row.data(), x, in_dim);
        }
    }
}

// weights.cpp:113-132 (row-parallel regime of matmul_quant).
void matmul(const uint8_t* w, uint64_t row0, int in_dim, int out_dim, const float* X, int n_tok,
            float* Y) {
    if (n_tok <= 0 || out_dim <= 0) return;
    const size_t rb = row_bytes(in_dim);
    const uint8_t* src = w + row0 * rb;
#pragma omp parallel
    {
        std::vector<float> row(static_cast<size_t>(in_dim));
#pragma omp for schedule(static)
        for (int j = 0; j < out_dim; ++j) {
            dequantize_row(DType::IQ3_XXS, src + rb * static_cast<size_t>(j), row.data(),
                           static_cast<uint64_t>(in_dim));
            for (int s = 0; s < n_tok; ++s)
                Y[static_cast<size_t>(s) * out_dim + j] =
                    dot_f32(row.data(), X + static_cast<size_t>(s) * in_dim, in_dim);
        }
    }
}

// model.cpp:41-46 (fp32 router matvec).
void matvec_f32(float* dst, const float* W, const float* x, int in_dim, int out_dim) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < out_dim; ++j) dst[j] = dot_f32(W + static_cast<size_t>(in_dim) * j, x, in_dim);
}

void topk(const std::vector<float>& choice, int E, int K, std::vector<int>& idx) {
    idx.resize(E);
    for (int e = 0; e < E; ++e) idx[e] = e;
    std::partial_sort(idx.begin(), idx.begin() + K, idx.end(),
                      [&](int a, int b) { return choice[a] > choice[b]; });
}

}  // namespace

extern "C" {

int ref_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// Host threads the reference's OpenMP loops use from here on (see oracle.c).
void ref_set_num_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

int ref_dequantize_iq3xxs(const uint8_t* src, float* dst, uint64_t n) {
    try {
        dequantize(DType::IQ3_XXS, src, dst, n);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

// any codec the reference decodes (quant.cpp:521-573 dispatch): type = ggml id
int ref_dequantize(int type, const uint8_t* src, float* dst, uint64_t n) {
    try {
        dequantize(static_cast<DType>(type), src, dst, n);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

float ref_dot_f32(const float* a, const float* b, int n) { return dot_f32(a, b, n); }

int ref_matvec_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim, const float* x,
                     float* dst) {
    if (in_dim % QK_K) return -1;
    matvec(w, row0, in_dim, out_dim, x, dst);
    return 0;
}

int ref_matmul_quant(const uint8_t* w, uint64_t row0, int in_dim, int out_dim, const float* X,
                     int n_tok, float* Y) {
    if (in_dim % QK_K) return -1;
    matmul(w, row0, in_dim, out_dim, X, n_tok, Y);
    return 0;
}

// model.cpp:692-756 (Model::moe_forward).
int ref_moe_forward(const orc_shape* s, const float* router_w, const float* corr,
                    const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                    const float* x, float* y, const int* forced, int* topk_out, float* topw_out) {
    const int H = s->hidden, I = s->inter, E = s->n_experts, K = s->top_k;
    if (H % QK_K || I % QK_K || K <= 0 || K > E) return -1;
    std::vector<float> logits(E), scores(E), choice(E);
    matvec_f32(logits.data(), router_w, x, H, E);
    for (int e = 0; e < E; ++e) {
        scores[e] = sigmoidf(logits[e]);
        choice[e] = scores[e] + (corr ? corr[e] : 0.0f);
    }
    std::vector<int> idx;
    if (forced) idx.assign(forced, forced + K);
    else topk(choice, E, K, idx);
    std::vector<float> wsum(K);
    float denom = 1e-20f;
    for (int k = 0; k < K; ++k) {
        wsum[k] = scores[idx[k]];
        denom += wsum[k];
    }
    if (s->norm_topk)
        for (int k = 0; k < K; ++k) wsum[k] /= denom;
    for (int k = 0; k < K; ++k) wsum[k] *= s->routed_scale;

    std::fill(y, y + H, 0.0f);
    const float lim = s->swiglu_limit;
    std::vector<float> g(I), u(I), h(I), dn(H);
    for (int k = 0; k < K; ++k) {
        const int e = idx[k];
        matvec(gate_exps, static_cast<uint64_t>(e) * I, H, I, x, g.data());
        matvec(up_exps, static_cast<uint64_t>(e) * I, H, I, x, u.data());
        for (int i = 0; i < I; ++i) h[i] = siluf(std::min(g[i], lim)) * std::clamp(u[i], -lim, lim);
        matvec(down_exps, static_cast<uint64_t>(e) * H, I, H, h.data(), dn.data());
        axpy_f32(y, dn.data(), wsum[k], H);
    }
    if (gate_sh) {
        matvec(gate_sh, 0, H, I, x, g.data());
        matvec(up_sh, 0, H, I, x, u.data());
        for (int i = 0; i < I; ++i) h[i] = siluf(std::min(g[i], lim)) * std::clamp(u[i], -lim, lim);
        matvec(down_sh, 0, I, H, h.data(), dn.data());
        add_f32(y, dn.data(), H);
    }
    if (topk_out) std::copy(idx.begin(), idx.begin() + K, topk_out);
    if (topw_out) std::copy(wsum.begin(), wsum.end(), topw_out);
    return 0;
}

// model_batch.cpp:165-281 (Model::moe_batch).
int ref_moe_batch(const orc_shape* s, const float* router_w, const float* corr,
                  const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                  const uint8_t* gate_sh, const uint8_t* up_sh, const uint8_t* down_sh,
                  const float* X, int n, float* Y, const int* forced, int* topk_out, float* topw_out) {
    const int H = s->hidden, I = s->inter, E = s->n_experts, K = s->top_k;
    if (H % QK_K || I % QK_K || K <= 0 || K > E || n < 0) return -1;
    if (n == 0) return 0;
    std::vector<float> logit(static_cast<size_t>(n) * E);
    for (int t = 0; t < n; ++t)
        matvec_f32(logit.data() + static_cast<size_t>(t) * E, router_w, X + static_cast<size_t>(t) * H, H, E);
    struct Assign { int tok, e; float w; };
    std::vector<Assign> asg;
    std::vector<int> cnt(E, 0), idx;
    std::vector<float> choice(E), score(E);
    for (int t = 0; t < n; ++t) {
        const float* lg = logit.data() + static_cast<size_t>(t) * E;
        for (int e = 0; e < E; ++e) {
            score[e] = 1.0f / (1.0f + std::exp(-lg[e]));
            choice[e] = score[e] + (corr ? corr[e] : 0.0f);
        }
        if (forced) idx.assign(forced + static_cast<size_t>(t) * K, forced + static_cast<size_t>(t + 1) * K);
        else topk(choice, E, K, idx);
        float denom = 1e-20f;
        for (int k = 0; k < K; ++k) denom += score[idx[k]];
        const float inv = s->norm_topk ? s->routed_scale / denom : s->routed_scale;
        for (int k = 0; k < K; ++k) {
            const int e = idx[k];
            asg.push_back({t, e, score[e] * inv});
            if (topk_out) topk_out[static_cast<size_t>(t) * K + k] = e;
            if (topw_out) topw_out[static_cast<size_t>(t) * K + k] = score[e] * inv;
            ++cnt[e];
        }
    }
    std::vector<int> eptr(E + 1);
    int acc = 0;
    for (int e = 0; e < E; ++e) { eptr[e] = acc; acc += cnt[e]; }
    eptr[E] = acc;
    std::vector<int> cursor(eptr.begin(), eptr.end() - 1), b_tok(asg.size());
    std::vector<float> b_wt(asg.size());
    for (size_t a = 0; a < asg.size(); ++a) {
        const int p = cursor[asg[a].e]++;
        b_tok[p] = asg[a].tok;
        b_wt[p] = asg[a].w;
    }
    std::fill(Y, Y + static_cast<size_t>(n) * H, 0.0f);
    const float lim = s->swiglu_limit;
    const int gmax = std::max(n, *std::max_element(cnt.begin(), cnt.end()));
    std::vector<float> Xg(static_cast<size_t>(gmax) * H), Gg(static_cast<size_t>(gmax) * I),
        Ug(static_cast<size_t>(gmax) * I), Hg(static_cast<size_t>(gmax) * I), Dg(static_cast<size_t>(gmax) * H);
    for (int e = 0; e < E; ++e) {
        const int lo = eptr[e], g = eptr[e + 1] - lo;
        if (g == 0) continue;
        for (int i = 0; i < g; ++i)
            std::memcpy(Xg.data() + static_cast<size_t>(i) * H, X + static_cast<size_t>(b_tok[lo + i]) * H,
                        sizeof(float) * H);
        matmul(gate_exps, static_cast<uint64_t>(e) * I, H, I, Xg.data(), g, Gg.data());
        matmul(up_exps, static_cast<uint64_t>(e) * I, H, I, Xg.data(), g, Ug.data());
        for (int i = 0; i < g * I; ++i) {
            const float gi = std::min(Gg[i], lim);
            const float ui = std::clamp(Ug[i], -lim, lim);
            Hg[i] = (gi / (1.0f + std::exp(-gi))) * ui;
        }
        matmul(down_exps, static_cast<uint64_t>(e) * H, I, H, Hg.data(), g, Dg.data());
        for (int i = 0; i < g; ++i)
            axpy_f32(Y + static_cast<size_t>(b_tok[lo + i]) * H, Dg.data() + static_cast<size_t>(i) * H,
                     b_wt[lo + i], H);
    }
    if (gate_sh) {
        matmul(gate_sh, 0, H, I, X, n, Gg.data());
        matmul(up_sh, 0, H, I, X, n, Ug.data());
        for (int i = 0; i < n * I; ++i) {
            const float gi = std::min(Gg[i], lim);
            const float ui = std::clamp(Ug[i], -lim, lim);
            Hg[i] = (gi / (1.0f + std::exp(-gi))) * ui;
        }
        matmul(down_sh, 0, I, H, Hg.data(), n, Dg.data());
        add_f32(Y, Dg.data(), n * H);
    }
    return 0;
}

}  // extern "C"
