// TEST INFRASTRUCTURE ONLY.  Drives the reference engine's own glm5::Model
// (cpp/core/src/model.cpp and the files it needs, compiled from the reference
// tree by oracle/Makefile into oracle/_ref/libgpeed_ref_model.so) on small
// synthetic GGUF models, to record golden outputs of two private members:
//
//   Model::hc_forward   (model.cpp:205-263) + the ffn RMSNorm that follows it
//                       in layer_forward (model.cpp:295-297): the mHC input
//                       of the MoE layer, with post[] and comb[]
//   Model::moe_forward  (model.cpp:692-756): one batch-1 MoE layer
//
// Both are private and need a complete Model, so this file includes the
// reference's model.h with `private` defined as `public`; the standard headers
// it pulls in are included first, so only the reference's classes see it.
// Nothing here is restated: the numbers come from the reference's code.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#define private public
#include "glm5/model.h"
#undef private
#include "glm5/gguf.h"
#include "glm5/ops.h"

namespace {

struct Loaded {
    std::string path;
    glm5::GgufModel gguf;
    std::unique_ptr<glm5::Model> model;
};
Loaded* g_loaded = nullptr;

glm5::Model* model_for(const char* path) {
    if (g_loaded && g_loaded->path == path) return g_loaded->model.get();
    delete g_loaded;
    g_loaded = new Loaded();
    g_loaded->path = path;
    g_loaded->gguf.load(glm5::GgufModel::discover_shards(path));
    glm5::ModelOptions o;
    o.max_ctx = 8;
    o.pin_nonexpert = false;  // tensors are read by name when used
    o.use_indexer = false;
    g_loaded->model.reset(new glm5::Model(g_loaded->gguf, o));
    return g_loaded->model.get();
}

std::string blk(int layer, const char* name) { return "blk." + std::to_string(layer) + "." + name; }

}  // namespace

extern "C" {

// Model config the harness saw: out[0..4] = hidden, hc_mult, n_experts, top_k, moe_inter.
int refm_config(const char* gguf, int* out) {
    try {
        const glm5::Model* m = model_for(gguf);
        out[0] = m->cfg_.hidden;
        out[1] = m->cfg_.hc_mult;
        out[2] = m->cfg_.n_experts;
        out[3] = m->cfg_.top_k;
        out[4] = m->cfg_.moe_inter;
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "refm_config: %s\n", e.what());
        return 1;
    }
}

// One token: streams [hc_mult][hidden] -> x [hidden] (the rms-normed MoE
// input), post [hc_mult], comb [hc_mult][hc_mult], pre [hc_mult].
int refm_hc_ffn(const char* gguf, int layer, const float* streams, float* x, float* post, float* comb, float* pre) {
    try {
        glm5::Model* m = model_for(gguf);
        const int H = m->cfg_.hidden, N = m->cfg_.hc_mult;
        std::copy(streams, streams + (size_t)N * H, m->streams_.begin());
        m->hc_forward(blk(layer, "hc_ffn_"), post, comb);
        std::copy(m->pre_.begin(), m->pre_.end(), pre);
        const float* fnorm = m->store_.get(blk(layer, "ffn_norm.weight"));
        glm5::rmsnorm(m->mixed_.data(), m->mixed_.data(), fnorm, H, m->cfg_.rms_eps);  // model.cpp:296-297
        std::copy(m->mixed_.begin(), m->mixed_.end(), x);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "refm_hc_ffn: %s\n", e.what());
        return 1;
    }
}

// One token: x [hidden] (the MoE input, as layer_forward leaves it in mixed_)
// -> y [hidden] = Model::moe_forward(layer)'s mlp_out_.
int refm_moe_forward(const char* gguf, int layer, const float* x, float* y) {
    try {
        glm5::Model* m = model_for(gguf);
        const int H = m->cfg_.hidden;
        std::copy(x, x + H, m->mixed_.begin());
        m->moe_forward(layer);
        std::copy(m->mlp_out_.begin(), m->mlp_out_.end(), y);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "refm_moe_forward: %s\n", e.what());
        return 1;
    }
}

}  // extern "C"
