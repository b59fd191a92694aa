// GGUF model files: reader (metadata, tensor table, shards) and the MoE layer
// loader that feeds expert tensors from the file mapping to the device.
//
// Reference behaviour kept (paths inside the reference project):
//   parse         cpp/core/src/gguf.cpp:133-188   magic "GGUF", versions 2-3,
//                 u64 counts, typed key/values (nested arrays allowed),
//                 "general.alignment" (default 32) rounds the end of the
//                 tensor table up to the start of the tensor-data section
//   shards        gguf.cpp:255-326  "<stem>-NNNNN-of-MMMMM.gguf" expands to all
//                 MMMMM files (same zero padding); a tensor name resolves to
//                 the first shard listing it, a key to the first shard with it
//   values        gguf.cpp:85-117   permissive numeric coercion
//   type sizes    quant.cpp:52-116  ggml block sizes and bytes per block
//   MoE config    model_config.cpp:80-95 (keys and defaults)
//   tensor names  model.cpp:702-754 (blk.N.ffn_gate_inp.weight, exp_probs_b.bias,
//                 ffn_{gate,up,down}_exps.weight, ffn_{gate,up,down}_shexp.weight)
// Differences: files are memory-mapped on every platform (the reference maps
// only on Windows and otherwise reads through an ifstream); tensor ranges are
// checked against the file size before a read; at most 4 dimensions.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/gpeed_moe.h"
#include "host_error.h"

namespace {

int err(int code, const char* fmt, ...) {
    char buf[600];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return gp::set_error(code, buf);
}

// ggml (block elements, bytes per block); {0, 0} for ids the format table leaves open
struct TypeSize {
    int block;
    int bytes;
};
TypeSize type_size(int t) {
    switch (t) {
        case 0: return {1, 4};     // F32
        case 1: return {1, 2};     // F16
        case 2: return {32, 18};   // Q4_0
        case 3: return {32, 20};   // Q4_1
        case 6: return {32, 22};   // Q5_0
        case 7: return {32, 24};   // Q5_1
        case 8: return {32, 34};   // Q8_0
        case 9: return {32, 36};   // Q8_1
        case 10: return {256, 84};   // Q2_K
        case 11: return {256, 110};  // Q3_K
        case 12: return {256, 144};  // Q4_K
        case 13: return {256, 176};  // Q5_K
        case 14: return {256, 210};  // Q6_K
        case 15: return {256, 292};  // Q8_K
        case 16: return {256, 66};   // IQ2_XXS
        case 17: return {256, 74};   // IQ2_XS
        case 18: return {256, 98};   // IQ3_XXS
        case 19: return {256, 50};   // IQ1_S
        case 20: return {32, 18};    // IQ4_NL
        case 21: return {256, 110};  // IQ3_S
        case 22: return {256, 82};   // IQ2_S
        case 23: return {256, 136};  // IQ4_XS
        case 24: return {1, 1};      // I8
        case 25: return {1, 2};      // I16
        case 26: return {1, 4};      // I32
        case 27: return {1, 8};      // I64
        case 28: return {1, 8};      // F64
        case 30: return {1, 2};      // BF16
        default: return {0, 0};
    }
}

uint64_t payload_bytes(int type, uint64_t n_elements) {
    const TypeSize ts = type_size(type);
    if (!ts.bytes || n_elements % (uint64_t)ts.block) return 0;
    uint64_t bytes = 0;
    if (__builtin_mul_overflow(n_elements / (uint64_t)ts.block, (uint64_t)ts.bytes, &bytes)) return 0;
    return bytes;
}

enum VType : int { U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STR = 8, ARR = 9,
                   U64 = 10, I64 = 11, F64 = 12 };

struct Value {
    int type = U8;
    int elem_type = U8;
    uint64_t n = 0;            // array length
    uint64_t u = 0;            // integer scalars (two's complement for signed)
    double f = 0;              // float scalars
    std::string str;
    std::vector<double> nums;  // numeric array elements
};

double value_f64(const Value& v) {
    switch (v.type) {
        case F32: case F64: return v.f;
        case I8: case I16: case I32: case I64: return (double)(int64_t)v.u;
        default: return (double)v.u;
    }
}

struct Cursor {
    const uint8_t* p = nullptr;
    const uint8_t* end;
    bool ok = true;
    bool need(uint64_t n) {
        if (!ok || (uint64_t)(end - p) < n) ok = false;
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            std::memcpy(&v, p, sizeof(T));
            p += sizeof(T);
        }
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!need(n)) return {};
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
};

bool read_scalar(Cursor& c, int type, Value& v) {
    v.type = type;
    switch (type) {
        case U8: v.u = c.get<uint8_t>(); break;
        case I8: v.u = (uint64_t)(int64_t)c.get<int8_t>(); break;
        case U16: v.u = c.get<uint16_t>(); break;
        case I16: v.u = (uint64_t)(int64_t)c.get<int16_t>(); break;
        case U32: v.u = c.get<uint32_t>(); break;
        case I32: v.u = (uint64_t)(int64_t)c.get<int32_t>(); break;
        case F32: v.f = c.get<float>(); break;
        case BOOL: v.u = c.get<uint8_t>() != 0; break;
        case STR: v.str = c.str(); break;
        case U64: v.u = c.get<uint64_t>(); break;
        case I64: v.u = (uint64_t)c.get<int64_t>(); break;
        case F64: v.f = c.get<double>(); break;
        default: return false;
    }
    return c.ok;
}

// skips (nested arrays) or records (numeric elements) an array body
bool read_array(Cursor& c, Value& v, int depth) {
    v.type = ARR;
    v.elem_type = (int)c.get<uint32_t>();
    v.n = c.get<uint64_t>();
    if (!c.ok || depth > 8) return false;
    const bool numeric = v.elem_type != STR && v.elem_type != ARR;
    if (numeric) {
        const TypeSize w = v.elem_type == U8 || v.elem_type == I8 || v.elem_type == BOOL ? TypeSize{1, 1}
                           : v.elem_type == U16 || v.elem_type == I16                   ? TypeSize{1, 2}
                           : v.elem_type == U32 || v.elem_type == I32 || v.elem_type == F32 ? TypeSize{1, 4}
                           : v.elem_type == U64 || v.elem_type == I64 || v.elem_type == F64 ? TypeSize{1, 8}
                                                                                              : TypeSize{0, 0};
        if (!w.bytes || v.n > (uint64_t)(c.end - c.p) / (uint64_t)w.bytes) return false;
        v.nums.reserve((size_t)v.n);
    }
    for (uint64_t i = 0; i < v.n; ++i) {
        Value e;
        if (v.elem_type == ARR) {
            if (!read_array(c, e, depth + 1)) return false;
        } else {
            if (!read_scalar(c, v.elem_type, e)) return false;
            if (numeric) v.nums.push_back(value_f64(e));
        }
    }
    return c.ok;
}

struct Tensor {
    std::string name;
    int type = 0, n_dims = 0, shard = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t offset = 0, nbytes = 0;
};

struct Shard {
    std::string path;
    int fd = -1;
    const uint8_t* map = nullptr;
    uint64_t size = 0;
    uint64_t data_off = 0;
    std::unordered_map<std::string, Value> meta;
    std::vector<std::string> keys;
};

// "<prefix>-NNNNN-of-MMMMM<ext>" -> every shard path; anything else -> {path}
std::vector<std::string> shard_paths(const std::string& path) {
    const size_t slash = path.find_last_of('/');
    const std::string dir = slash == std::string::npos ? "" : path.substr(0, slash + 1);
    const std::string file = slash == std::string::npos ? path : path.substr(slash + 1);
    const size_t dot = file.find_last_of('.');
    const std::string stem = (dot == std::string::npos || dot == 0) ? file : file.substr(0, dot);
    const std::string ext = stem.size() == file.size() ? "" : file.substr(stem.size());
    const size_t of = stem.rfind("-of-");
    if (of == std::string::npos || of == 0) return {path};
    const size_t dash = stem.rfind('-', of - 1);
    if (dash == std::string::npos) return {path};
    const std::string num = stem.substr(dash + 1, of - dash - 1), tot = stem.substr(of + 4);
    if (num.empty() || tot.empty() || num.find_first_not_of("0123456789") != std::string::npos ||
        tot.find_first_not_of("0123456789") != std::string::npos || tot.size() > 6)
        return {path};
    const int total = std::stoi(tot), width = (int)num.size();
    std::vector<std::string> out;
    for (int i = 1; i <= total; ++i) {
        char b[16];
        std::snprintf(b, sizeof(b), "%0*d", width, i);
        out.push_back(dir + stem.substr(0, dash) + "-" + b + "-of-" + tot + ext);
    }
    return out;
}

}  // namespace

struct gpeed_gguf {
    std::vector<Shard> shards;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;  // first shard wins
    std::vector<std::string> names;
    std::vector<std::string> keys;                    // union, first-seen order

    ~gpeed_gguf() {
        for (auto& s : shards) {
            if (s.map) munmap(const_cast<uint8_t*>(s.map), (size_t)s.size);
            if (s.fd >= 0) close(s.fd);
        }
    }
    const Value* find(const std::string& key) const {
        for (const auto& s : shards) {
            auto it = s.meta.find(key);
            if (it != s.meta.end()) return &it->second;
        }
        return nullptr;
    }
    const Tensor* tensor(const std::string& name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : &tensors[it->second];
    }
};

namespace {

int open_shard(gpeed_gguf* g, const std::string& path, int index) {
    Shard s;
    s.path = path;
    s.fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (s.fd < 0) return err(GPEED_ERR_INVALID, "GGUF: cannot open %s: %s", path.c_str(), strerror(errno));
    g->shards.push_back(std::move(s));  // the destructor now owns the descriptor
    Shard& sh = g->shards.back();
    struct stat st {};
    if (fstat(sh.fd, &st) != 0 || st.st_size < 24) return err(GPEED_ERR_INVALID, "GGUF: %s is too short", path.c_str());
    sh.size = (uint64_t)st.st_size;
    void* m = mmap(nullptr, (size_t)sh.size, PROT_READ, MAP_SHARED, sh.fd, 0);
    if (m == MAP_FAILED) return err(GPEED_ERR_INVALID, "GGUF: cannot map %s: %s", path.c_str(), strerror(errno));
    sh.map = static_cast<const uint8_t*>(m);

    Cursor c{sh.map, sh.map + sh.size};
    if (c.get<uint32_t>() != 0x46554747u) return err(GPEED_ERR_INVALID, "GGUF: bad magic in %s", path.c_str());
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) return err(GPEED_ERR_UNSUPPORTED, "GGUF: unsupported version %u", version);
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        const int vt = (int)c.get<uint32_t>();
        Value v;
        const bool ok = vt == ARR ? read_array(c, v, 0) : read_scalar(c, vt, v);
        if (!ok) return err(GPEED_ERR_INVALID, "GGUF: bad value for key '%s' in %s", key.c_str(), path.c_str());
        if (key == "general.alignment" && vt != STR && vt != ARR) alignment = (uint64_t)value_f64(v);
        if (!sh.meta.count(key)) sh.keys.push_back(key);
        sh.meta[key] = std::move(v);
    }
    if (!c.ok) return err(GPEED_ERR_INVALID, "GGUF: unexpected end of metadata in %s", path.c_str());
    if (alignment == 0) return err(GPEED_ERR_INVALID, "GGUF: general.alignment is 0");
    const size_t first = g->tensors.size();
    for (uint64_t i = 0; i < n_tensors; ++i) {
        Tensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (!c.ok) break;
        if (nd == 0 || nd > 4) return err(GPEED_ERR_UNSUPPORTED, "GGUF: tensor '%s' has %u dims", t.name.c_str(), nd);
        t.n_dims = (int)nd;
        uint64_t ne = 1;
        bool wrapped = false;
        for (uint32_t d = 0; d < nd; ++d) {
            t.dims[d] = c.get<uint64_t>();
            wrapped |= __builtin_mul_overflow(ne, t.dims[d], &ne);
        }
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        t.shard = index;
        if (!c.ok) break;
        if (wrapped) return err(GPEED_ERR_INVALID, "GGUF: tensor '%s': element count overflows 64 bits", t.name.c_str());
        t.nbytes = payload_bytes(t.type, ne);
        // a known type whose element count is not a whole number of blocks, or
        // whose byte count overflows, describes no payload this reader can map
        if (type_size(t.type).bytes && ne && !t.nbytes)
            return err(GPEED_ERR_INVALID, "GGUF: tensor '%s': %llu elements do not form whole blocks of type %d",
                       t.name.c_str(), (unsigned long long)ne, t.type);
        g->tensors.push_back(std::move(t));
    }
    if (!c.ok) return err(GPEED_ERR_INVALID, "GGUF: unexpected end of tensor table in %s", path.c_str());
    const uint64_t consumed = (uint64_t)(c.p - sh.map);
    sh.data_off = (consumed + alignment - 1) / alignment * alignment;
    for (size_t i = first; i < g->tensors.size(); ++i) {
        const Tensor& t = g->tensors[i];
        if (g->by_name.emplace(t.name, i).second) g->names.push_back(t.name);
    }
    return GPEED_OK;
}

// bounds-checked pointer to [byte_off, byte_off + bytes) of tensor t
int tensor_span(const gpeed_gguf* g, const Tensor& t, uint64_t byte_off, uint64_t bytes, const uint8_t** out) {
    const Shard& s = g->shards[t.shard];
    const uint64_t start = s.data_off + t.offset + byte_off;
    if (byte_off > t.nbytes || bytes > t.nbytes - byte_off || start < s.data_off || start > s.size ||
        bytes > s.size - start)
        return err(GPEED_ERR_INVALID, "GGUF: range [%llu, +%llu) of tensor '%s' lies outside %s",
                   (unsigned long long)byte_off, (unsigned long long)bytes, t.name.c_str(), s.path.c_str());
    *out = s.map + start;
    return GPEED_OK;
}

std::string arch_key(const gpeed_gguf* g, const char* suffix) {
    const Value* a = g->find("general.architecture");
    const std::string arch = a && a->type == STR ? a->str : std::string("glm5-next");
    return arch + "." + suffix;
}

double meta_num(const gpeed_gguf* g, const char* suffix, double def) {
    const Value* v = g->find(arch_key(g, suffix));
    if (!v || v->type == STR) return def;
    if (v->type == ARR) return v->nums.empty() ? def : v->nums[0];
    return value_f64(*v);
}

std::string blk_name(int blk, const char* what) { return "blk." + std::to_string(blk) + "." + what; }

}  // namespace

extern "C" {

int gpeed_gguf_open(const char* path, gpeed_gguf** out) {
    if (!path || !out) return err(GPEED_ERR_INVALID, "GGUF: path or out is NULL");
    *out = nullptr;
    gpeed_gguf* g = new gpeed_gguf();
    const std::vector<std::string> paths = shard_paths(path);
    for (size_t i = 0; i < paths.size(); ++i) {
        const int rc = open_shard(g, paths[i], (int)i);
        if (rc) {
            delete g;
            return rc;
        }
    }
    for (const auto& s : g->shards)
        for (const auto& k : s.keys)
            if (g->find(k) == &s.meta.at(k)) g->keys.push_back(k);
    *out = g;
    return GPEED_OK;
}

int gpeed_gguf_close(gpeed_gguf* g) {
    delete g;
    return GPEED_OK;
}

int gpeed_gguf_counts(gpeed_gguf* g, int* n_shards, int64_t* n_tensors, int64_t* n_keys) {
    if (!g) return err(GPEED_ERR_INVALID, "GGUF: handle is NULL");
    if (n_shards) *n_shards = (int)g->shards.size();
    if (n_tensors) *n_tensors = (int64_t)g->names.size();
    if (n_keys) *n_keys = (int64_t)g->keys.size();
    return GPEED_OK;
}

int gpeed_gguf_tensor_name(gpeed_gguf* g, int64_t i, const char** name) {
    if (!g || !name) return err(GPEED_ERR_INVALID, "GGUF: handle or name is NULL");
    if (i < 0 || i >= (int64_t)g->names.size()) return err(GPEED_ERR_INVALID, "GGUF: tensor index %lld", (long long)i);
    *name = g->names[(size_t)i].c_str();
    return GPEED_OK;
}

int gpeed_gguf_key_name(gpeed_gguf* g, int64_t i, const char** name) {
    if (!g || !name) return err(GPEED_ERR_INVALID, "GGUF: handle or name is NULL");
    if (i < 0 || i >= (int64_t)g->keys.size()) return err(GPEED_ERR_INVALID, "GGUF: key index %lld", (long long)i);
    *name = g->keys[(size_t)i].c_str();
    return GPEED_OK;
}

int gpeed_gguf_tensor_info(gpeed_gguf* g, const char* name, gpeed_gguf_tensor* out) {
    if (!g || !name || !out) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Tensor* t = g->tensor(name);
    if (!t) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", name);
    out->dtype = t->type;
    out->n_dims = t->n_dims;
    for (int d = 0; d < 4; ++d) out->dims[d] = t->dims[d];
    out->offset = t->offset;
    out->nbytes = t->nbytes;
    out->shard = t->shard;
    return GPEED_OK;
}

int gpeed_gguf_read(gpeed_gguf* g, const char* name, uint64_t byte_off, uint64_t bytes, void* dst) {
    if (!g || !name || (!dst && bytes)) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Tensor* t = g->tensor(name);
    if (!t) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", name);
    if (!t->nbytes) return err(GPEED_ERR_UNSUPPORTED, "GGUF: tensor '%s' has type %d of unknown size", name, t->type);
    const uint8_t* p = nullptr;
    const int rc = tensor_span(g, *t, byte_off, bytes, &p);
    if (rc) return rc;
    if (bytes) std::memcpy(dst, p, (size_t)bytes);
    return GPEED_OK;
}

int gpeed_gguf_meta_type(gpeed_gguf* g, const char* key, int* type, int* elem_type, uint64_t* n) {
    if (!g || !key) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Value* v = g->find(key);
    if (!v) return err(GPEED_ERR_INVALID, "GGUF: missing metadata key %s", key);
    if (type) *type = v->type;
    if (elem_type) *elem_type = v->type == ARR ? v->elem_type : v->type;
    if (n) *n = v->type == ARR ? v->n : 1;
    return GPEED_OK;
}

int gpeed_gguf_meta_f64(gpeed_gguf* g, const char* key, uint64_t index, double* out) {
    if (!g || !key || !out) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Value* v = g->find(key);
    if (!v) return err(GPEED_ERR_INVALID, "GGUF: missing metadata key %s", key);
    if (v->type == STR || (v->type == ARR && v->nums.size() != v->n))
        return err(GPEED_ERR_INVALID, "GGUF: value is not numeric (%s)", key);
    if (v->type == ARR) {
        if (index >= v->n) return err(GPEED_ERR_INVALID, "GGUF: index %llu past the %llu elements of %s",
                                      (unsigned long long)index, (unsigned long long)v->n, key);
        *out = v->nums[(size_t)index];
        return GPEED_OK;
    }
    if (index) return err(GPEED_ERR_INVALID, "GGUF: %s is a scalar", key);
    *out = value_f64(*v);
    return GPEED_OK;
}

int gpeed_gguf_meta_u64(gpeed_gguf* g, const char* key, uint64_t* out) {
    if (!g || !key || !out) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Value* v = g->find(key);
    if (!v) return err(GPEED_ERR_INVALID, "GGUF: missing metadata key %s", key);
    if (v->type == STR || v->type == ARR) return err(GPEED_ERR_INVALID, "GGUF: value is not numeric (%s)", key);
    *out = (v->type == F32 || v->type == F64) ? (uint64_t)v->f : v->u;
    return GPEED_OK;
}

int gpeed_gguf_meta_str(gpeed_gguf* g, const char* key, const char** out) {
    if (!g || !key || !out) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const Value* v = g->find(key);
    if (!v) return err(GPEED_ERR_INVALID, "GGUF: missing metadata key %s", key);
    if (v->type != STR) return err(GPEED_ERR_INVALID, "GGUF: value is not a string (%s)", key);
    *out = v->str.c_str();
    return GPEED_OK;
}

int gpeed_gguf_moe_shape(gpeed_gguf* g, int blk, gpeed_moe_shape* out) {
    if (!g || !out) return err(GPEED_ERR_INVALID, "GGUF: NULL argument");
    const std::string gname = blk_name(blk, "ffn_gate_exps.weight");
    const Tensor* gt = g->tensor(gname);
    if (!gt) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", gname.c_str());
    if (gt->n_dims != 3) return err(GPEED_ERR_INVALID, "weights: not a 3D expert tensor: %s", gname.c_str());
    gpeed_moe_shape s{};
    s.hidden = (int)gt->dims[0];
    s.inter = (int)gt->dims[1];
    s.n_experts = (int)gt->dims[2];
    const double h_meta = meta_num(g, "embedding_length", s.hidden);
    const double i_meta = meta_num(g, "expert_feed_forward_length", s.inter);
    const double e_meta = meta_num(g, "expert_count", s.n_experts);
    if (h_meta != s.hidden || i_meta != s.inter || e_meta != s.n_experts)
        return err(GPEED_ERR_INVALID, "GGUF: %s is [%d, %d, %d] but the metadata says H %g, I %g, E %g", gname.c_str(),
                   s.hidden, s.inter, s.n_experts, h_meta, i_meta, e_meta);
    s.top_k = (int)meta_num(g, "expert_used_count", 8);
    s.n_shared = (int)meta_num(g, "expert_shared_count", 1);
    s.routed_scale = (float)meta_num(g, "expert_weights_scale", 2.5);
    s.norm_topk = meta_num(g, "expert_weights_norm", 1) != 0;
    {  // the first element of the per-layer array, as the reference reads it
        const Value* v = g->find(arch_key(g, "swiglu_clamp_exp"));
        s.swiglu_limit = v && v->type == ARR && !v->nums.empty() ? (float)v->nums[0] : 10.0f;
    }
    const int gating = (int)meta_num(g, "expert_gating_func", 2);
    if (gating != 2) return err(GPEED_ERR_UNSUPPORTED, "GGUF: expert_gating_func %d (only 2, sigmoid)", gating);
    *out = s;
    return GPEED_OK;
}

int gpeed_tensor_upload_gguf(gpeed_ctx* ctx, gpeed_gguf* g, const char* name, int* handle) {
    if (!ctx || !g || !name || !handle) return err(GPEED_ERR_INVALID, "NULL argument");
    const Tensor* t = g->tensor(name);
    if (!t) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", name);  // weights.cpp:170-171
    if (t->type != GPEED_DTYPE_IQ3_XXS)
        return err(GPEED_ERR_UNSUPPORTED, "weights: %s has type %d; the expert kernels take IQ3_XXS (18)", name, t->type);
    uint64_t rows = 1;
    for (int d = 1; d < t->n_dims; ++d) rows *= t->dims[d];
    if (t->dims[0] > (1u << 30)) return err(GPEED_ERR_UNSUPPORTED, "weights: %s rows of %llu weights", name,
                                            (unsigned long long)t->dims[0]);
    const uint8_t* p = nullptr;
    const int rc = tensor_span(g, *t, 0, t->nbytes, &p);
    if (rc) return rc;
    return gpeed_tensor_upload(ctx, p, 0, GPEED_DTYPE_IQ3_XXS, rows, (int)t->dims[0], handle);
}

int gpeed_moe_load_layer_gguf(gpeed_ctx* ctx, gpeed_gguf* g, int blk, int layer, int expert_begin, int expert_count,
                              gpeed_moe_shape* shape_out) {
    if (!ctx || !g) return err(GPEED_ERR_INVALID, "ctx or GGUF handle is NULL");
    gpeed_moe_shape s;
    int rc = gpeed_gguf_moe_shape(g, blk, &s);
    if (rc) return rc;
    if (expert_count < 0) expert_count = s.n_experts - expert_begin;
    if (expert_begin < 0 || expert_count < 0 || expert_begin + expert_count > s.n_experts)
        return err(GPEED_ERR_INVALID, "expert range [%d, %d) outside [0, %d)", expert_begin, expert_begin + expert_count,
                   s.n_experts);
    const int H = s.hidden, I = s.inter, E = s.n_experts;

    // expert tensors: IQ3_XXS, ggml ne = [in, out, E] routed / [in, out] shared
    const void* ptr[6] = {};
    const char* names[6] = {"ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight",
                            "ffn_gate_shexp.weight", "ffn_up_shexp.weight", "ffn_down_shexp.weight"};
    for (int m = 0; m < (s.n_shared ? 6 : 3); ++m) {
        const std::string nm = blk_name(blk, names[m]);
        const Tensor* t = g->tensor(nm);
        if (!t) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", nm.c_str());
        if (t->type != GPEED_DTYPE_IQ3_XXS)
            return err(GPEED_ERR_UNSUPPORTED, "weights: %s has type %d; the expert kernels take IQ3_XXS (18)",
                       nm.c_str(), t->type);
        const bool down = m % 3 == 2, shared = m >= 3;
        const uint64_t in = down ? I : H, rows = down ? H : I;
        if (t->n_dims != (shared ? 2 : 3) || t->dims[0] != in || t->dims[1] != rows || (!shared && t->dims[2] != (uint64_t)E))
            return err(GPEED_ERR_INVALID, "weights: %s has shape [%llu, %llu, %llu], want [%llu, %llu%s]", nm.c_str(),
                       (unsigned long long)t->dims[0], (unsigned long long)t->dims[1], (unsigned long long)t->dims[2],
                       (unsigned long long)in, (unsigned long long)rows, shared ? "" : ", E");
        const uint64_t per_expert = rows * (in / 256) * 98;
        const uint64_t off = shared ? 0 : per_expert * (uint64_t)expert_begin;
        const uint64_t len = shared ? per_expert : per_expert * (uint64_t)expert_count;
        const uint8_t* p = nullptr;
        if ((rc = tensor_span(g, *t, off, len, &p))) return rc;
        ptr[m] = p;
    }

    // router [E][H] (ggml ne = [H, E]) as fp32; F16 / BF16 widen exactly
    const std::string rn = blk_name(blk, "ffn_gate_inp.weight");
    const Tensor* rt = g->tensor(rn);
    if (!rt) return err(GPEED_ERR_INVALID, "weights: missing tensor %s", rn.c_str());
    if (rt->n_dims != 2 || rt->dims[0] != (uint64_t)H || rt->dims[1] != (uint64_t)E)
        return err(GPEED_ERR_INVALID, "weights: %s is not [H, E]", rn.c_str());
    if (rt->type != 0 && rt->type != 1 && rt->type != 30)
        return err(GPEED_ERR_UNSUPPORTED, "weights: %s has type %d (F32, F16 or BF16 expected)", rn.c_str(), rt->type);
    const uint8_t* rp = nullptr;
    if ((rc = tensor_span(g, *rt, 0, rt->nbytes, &rp))) return rc;
    std::vector<float> router;
    const float* router_ptr = reinterpret_cast<const float*>(rp);
    if (rt->type == 1 || rt->type == 30 || reinterpret_cast<uintptr_t>(rp) % 4) {
        router.resize((size_t)E * H);
        for (size_t i = 0; i < router.size(); ++i) {
            uint32_t bits;
            if (rt->type == 0) {
                std::memcpy(&router[i], rp + 4 * i, 4);
                continue;
            }
            uint16_t h;
            std::memcpy(&h, rp + 2 * i, 2);
            if (rt->type == 30) {
                bits = (uint32_t)h << 16;
            } else {  // IEEE half -> float, subnormals included (quant.cpp:130-154)
                const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
                if (ex == 0 && man == 0) {
                    bits = sign;
                } else if (ex == 0) {
                    uint32_t e = 113, m2 = man;
                    while (!(m2 & 0x400u)) { m2 <<= 1; --e; }
                    bits = sign | (e << 23) | ((m2 & 0x3ffu) << 13);
                } else if (ex == 31) {
                    bits = sign | 0x7f800000u | (man << 13);
                } else {
                    bits = sign | ((ex + 112) << 23) | (man << 13);
                }
            }
            std::memcpy(&router[i], &bits, 4);
        }
        router_ptr = router.data();
    }

    // correction bias [E] fp32, optional (model.cpp:703)
    const std::string cn = blk_name(blk, "exp_probs_b.bias");
    const Tensor* ct = g->tensor(cn);
    std::vector<float> corr;
    if (ct) {
        if (ct->type != 0 || ct->dims[0] != (uint64_t)E) return err(GPEED_ERR_INVALID, "weights: %s is not F32 [E]", cn.c_str());
        const uint8_t* cp = nullptr;
        if ((rc = tensor_span(g, *ct, 0, ct->nbytes, &cp))) return rc;
        corr.resize((size_t)E);
        std::memcpy(corr.data(), cp, sizeof(float) * E);
    }
    rc = gpeed_moe_load_layer_range(ctx, layer, &s, expert_begin, expert_count, router_ptr, ct ? corr.data() : nullptr,
                                    ptr[0], ptr[1], ptr[2], ptr[3], ptr[4], ptr[5], 0);
    if (!rc && shape_out) *shape_out = s;
    return rc;
}

}  // extern "C"
