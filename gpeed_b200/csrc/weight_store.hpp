// C++ shim with the reference engine's expert-op signatures on top of the C
// ABI (include/gpeed_moe.h).  A glm5::WeightStore user swaps
//   store.matvec_quant(name, row0, in_dim, out_dim, x, dst)
// (reference cpp/core/include/glm5/weights.h:38-48) for the same call on
// gpeed::WeightStore, with x/dst in device memory.  Non-zero status codes
// become std::runtime_error carrying gpeed_last_error(), as the reference
// throws (weights.cpp:170-174, quant.cpp:523-554).  Header-only; link
// libgpeed_moe.so.
#pragma once
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../../include/gpeed_moe.h"

namespace gpeed {

inline void check(int rc) {
    if (rc != GPEED_OK) throw std::runtime_error(std::string("gpeed: ") + gpeed_last_error());
}

class WeightStore {
public:
    explicit WeightStore(int device = 0) { check(gpeed_ctx_create(device, &ctx_)); }
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

    // weights.h:38-41
    void matvec_quant(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* x, float* dst,
                      void* stream = nullptr) {
        check(gpeed_matvec_quant(ctx_, handle(name), row0, in_dim, out_dim, x, dst, stream));
    }
    // weights.h:43-48
    void matmul_quant(const std::string& name, uint64_t row0, int in_dim, int out_dim, const float* X, int n_tok,
                      float* Y, void* stream = nullptr) {
        check(gpeed_matmul_quant(ctx_, handle(name), row0, in_dim, out_dim, X, n_tok, Y, stream));
    }

private:
    int handle(const std::string& name) const {
        auto it = handles_.find(name);
        if (it == handles_.end()) throw std::runtime_error("weights: missing tensor " + name);  // weights.cpp:170
        return it->second;
    }
    gpeed_ctx* ctx_ = nullptr;
    std::unordered_map<std::string, int> handles_;
};

}  // namespace gpeed
