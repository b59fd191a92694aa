// C++ shim with the reference engine's expert-op signatures on top of the C
// ABI (include/gpeed_moe.h).  A glm5::WeightStore user swaps
//   store.matvec_quant(name, row0, in_dim, out_dim, x, dst)
// (reference cpp/core/include/glm5/weights.h:38-48) for the same call on
// gpeed::WeightStore, with the same host buffers (matvec_quant_device and
// matmul_quant_device take device buffers and a stream).  Non-zero status codes
// become std::runtime_error carrying gpeed_last_error(), as the reference
// throws (weights.cpp:170-174, quant.cpp:523-554).  Header-only; link
// libgpeed_moe.so.
//
// gpeed::GgufModel opens a (sharded) GGUF model like glm5::GgufModel
// (gguf.h:122-150); a WeightStore built on one resolves tensor names in it on
// first use, as glm5::WeightStore(const GgufModel&, bool) does (weights.h:15-20),
// and keeps the device copy for later calls.
#pragma once
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../../include/gpeed_moe.h"

namespace gpeed {

inline void check(int rc) {
    if (rc != GPEED_OK) throw std::runtime_error(std::string("gpeed: ") + gpeed_last_error());
}

class GgufModel {
public:
    // any one shard path; the others are found by name (gguf.cpp:298-326)
    explicit GgufModel(const std::string& path) { check(gpeed_gguf_open(path.c_str(), &g_)); }
    ~GgufModel() { gpeed_gguf_close(g_); }
    GgufModel(const GgufModel&) = delete;
    GgufModel& operator=(const GgufModel&) = delete;

    gpeed_gguf* handle() const { return g_; }
    // nullptr-like false when absent (GgufModel::find_tensor)
    bool find_tensor(const std::string& name, gpeed_gguf_tensor* out) const {
        return gpeed_gguf_tensor_info(g_, name.c_str(), out) == GPEED_OK;
    }
    // GgufFile::read_at, inside one tensor
    void read_at(const std::string& name, uint64_t offset, size_t bytes, void* dst) const {
        check(gpeed_gguf_read(g_, name.c_str(), offset, bytes, dst));
    }

private:
    gpeed_gguf* g_ = nullptr;
};

class WeightStore {
public:
    explicit WeightStore(int device = 0) { check(gpeed_ctx_create(device, &ctx_)); }
    explicit WeightStore(const GgufModel& model, int device = 0) : model_(&model) {
        check(gpeed_ctx_create(device, &ctx_));
    }
    ~WeightStore() { gpeed_ctx_destroy(ctx_); }
    WeightStore(const WeightStore&) = delete;
    WeightStore& operator=(const WeightStore&) = delete;

    gpeed_ctx* ctx() const { return ctx_; }

    // Registers a raw IQ3_XXS tensor (rows x in_dim weights, GGUF block order),
    // the device counterpart of WeightStore::pin_nonexpert / payload().
    void add(const std::string& name, const void* raw, bool on_device, uint64_t rows, int in_dim) {
        int h = -1;
        check(gpeed_tensor_upload(ctx_, raw, on_device ? 1 : 0, GPEED_DTYPE_IQ3_XXS, rows, in_dim, &h));
        handles_[name] = h;
    }
    bool has(const std::string& name) const { return handles_.count(name) != 0; }

    // weights.h:38-41 and weights.h:43-48, with the reference's calling
    // convention: x / X and dst / Y are host buffers (its callers pass
    // std::vector data, model.cpp:733-754, model_batch.cpp:241-279) and the
    // call returns with dst / Y filled.  Throws like the reference.
    void matvec_quant(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* x, float* dst) {
        check(gpeed_matvec_quant_host(ctx_, handle(name), row0, in_dim, out_dim, x, dst));
    }
    void matmul_quant(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* X, int n_tok,
                      float* Y) {
        check(gpeed_matmul_quant_host(ctx_, handle(name), row0, in_dim, out_dim, X, n_tok, Y));
    }

    // The same on device buffers, asynchronous on `stream` (an engine that
    // keeps its activations on the GPU; device-side faults surface at
    // check_device()).
    void matvec_quant_device(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* x_dev,
                             float* dst_dev, void* stream = nullptr) {
        check(gpeed_matvec_quant(ctx_, handle(name), row0, in_dim, out_dim, x_dev, dst_dev, stream));
    }
    void matmul_quant_device(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* X_dev,
                             int n_tok, float* Y_dev, void* stream = nullptr) {
        check(gpeed_matmul_quant(ctx_, handle(name), row0, in_dim, out_dim, X_dev, n_tok, Y_dev, stream));
    }
    void check_device(void* stream = nullptr) { check(gpeed_ctx_check(ctx_, stream)); }

private:
    int handle(const std::string& name) {
        auto it = handles_.find(name);
        if (it != handles_.end()) return it->second;
        if (!model_) throw std::runtime_error("weights: missing tensor " + name);  // weights.cpp:170
        int h = -1;
        check(gpeed_tensor_upload_gguf(ctx_, model_->handle(), name.c_str(), &h));
        handles_[name] = h;
        return h;
    }
    const GgufModel* model_ = nullptr;
    gpeed_ctx* ctx_ = nullptr;
    std::unordered_map<std::string, int> handles_;
};

}  // namespace gpeed
