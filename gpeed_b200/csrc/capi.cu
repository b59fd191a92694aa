// C ABI of libgpeed_moe.so (declared in include/gpeed_moe.h): context,
// weight registry, and the orchestration of the MoE layer forward
//   router -> route (top-k, histogram, permutation, slots)
//          -> gate/up GEMV + SwiGLU -> down GEMV -> weighted combine
// as a chain of kernels on one stream with programmatic dependent launch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/gpeed_moe.h"
#include "host_error.h"
#include "kernels.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define GP_CUDA(call)                                                                        \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) return fail(GPEED_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

struct Tensor {
    uint8_t* packed = nullptr;
    int64_t rows = 0;
    int in_dim = 0;
};

struct Layer {
    gpeed_moe_shape shape{};
    float* router = nullptr;
    float* corr = nullptr;
    uint8_t* gate = nullptr;  // repacked, (E + n_shared) experts x I rows of H
    uint8_t* up = nullptr;
    uint8_t* down = nullptr;  // (E + n_shared) experts x H rows of I
    int64_t gu_stride = 0, d_stride = 0;
    // the down projections again in the column-slab layout the persistent
    // decode kernel streams (launch_repack_cols), for shapes it serves
    uint8_t* down_col = nullptr;
    int64_t dc_stride = 0;
    // experts held here: routed [e_lo, e_lo + e_cnt) at local index e - e_lo,
    // then the shared expert at local index e_cnt (all of them unless the
    // layer was loaded for expert parallelism)
    int e_lo = 0, e_cnt = 0;
    // units of 32 intermediate rows of every routed expert held here: [u_lo,
    // u_lo + u_cnt) of inter / 32 (gpeed_moe_slice_units; all of them
    // otherwise).  A sliced layer keeps only the gate/up row groups and down
    // column slabs of those units, for the persistent decode kernel, and the
    // shared expert whole after them.
    int u_lo = 0, u_cnt = 0;
    bool sliced() const { return u_cnt != shape.inter / 32; }
    // the router weights split into bf16 hi/lo/lo2 rows for the tensor-core router (or nullptr)
    uint16_t* router_split = nullptr;
    int router_nb = 0;
};

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    int ensure(size_t want) {
        if (want <= n) return GPEED_OK;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        if (cudaMalloc(&p, want * sizeof(T)) != cudaSuccess)
            return fail(GPEED_ERR_CUDA, "cudaMalloc(%zu bytes) failed", want * sizeof(T));
        n = want;
        return GPEED_OK;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

int64_t padded_rows(int64_t rows) { return (rows + 7) / 8 * 8 + 32; }

}  // namespace

struct gpeed_ctx {
    int device = 0;
    int num_sms = 148;
    uint8_t* tables = nullptr;
    uint32_t* status = nullptr;
    std::vector<Tensor> tensors;
    std::map<int, Layer> layers;
    // forward scratch (grown on demand; grow before capturing a graph)
    DevBuf<float> partial, topk_w, h, D, mvout;
    DevBuf<int> topk_ids, perm, inv_pos, counts, nslots;
    DevBuf<gp::SlotDesc> slots;
    // batch-1 forward in one persistent kernel when the shape has a variant
    bool fused_decode = true;
    int fused_max_tokens = 12;         // batches up to this size: the fused kernel once per token
    bool fused_cooperative = false;
    uint32_t spin_limit = GPEED_SPIN_LIMIT_DEFAULT;  // polls before a wait of the fused kernel gives up
    int withhold_logit = -1;           // test hook (GPEED_OPT_TEST_WITHHOLD_LOGIT)
    int tc_min_tokens = 8;             // batches this large run the experts on tensor cores
    DevBuf<uint16_t> xp;               // fp16 token rows in expert-sorted order (tensor-core path)
    DevBuf<int> route_chunks;          // per-chunk expert counts of the large-batch stable sort
    DevBuf<unsigned long long> logits, hx;
    // expert-parallel exchange over peer memory (gpeed_ep_setup / _connect)
    struct Ep {
        int world = 0, rank = -1, hidden = 0;
        uint8_t* base = nullptr;                      // this rank's block (cudaMalloc, exported by IPC)
        uint8_t* peer[gp::kDecodeMaxTokens] = {};     // every rank's block (this rank's = base)
        bool connected = false;
    } ep;
    unsigned* sync = nullptr;  // grid counters of the persistent kernel (zero between launches)
    // optional per-stage timing of gpeed_moe_forward (CUDA events on its stream)
    bool prof = false;
    cudaEvent_t ev[6] = {};
    double prof_ms[5] = {0, 0, 0, 0, 0};
    long prof_calls = 0;
    DevBuf<float> mhc_partial;         // per-slice partial sums of the mHC dot products
    // pinned staging ring for weight uploads from pageable host memory
    uint8_t* stage[4] = {};
    cudaEvent_t stage_ev[4] = {};
    // host-pointer matvec/matmul: pinned in/out staging, device buffers, own stream
    std::mutex host_mu;
    float* host_pin = nullptr;
    size_t host_pin_n = 0;
    DevBuf<float> host_x, host_y;
    cudaStream_t host_stream = nullptr;
};

int gp::set_error(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

namespace {

int set_device(const gpeed_ctx* c) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != c->device) GP_CUDA(cudaSetDevice(c->device));
    return GPEED_OK;
}

// every row to local expert 0 with weight 1 (the dense MLP as a one-expert pass)
__global__ void fill_unit_kernel(int* ids, float* w, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        ids[i] = 0;
        w[i] = 1.f;
    }
}

__global__ void make_slots_kernel(gp::SlotDesc* slots, int* nslots, int n_tok, int nt) {
    const int ns = (n_tok + nt - 1) / nt;
    for (int i = threadIdx.x; i < ns; i += blockDim.x) {
        gp::SlotDesc s;
        s.expert = 0;
        s.begin = i * nt;
        s.ntok = min(nt, n_tok - i * nt);
        s.pad = 0;
        slots[i] = s;
    }
    if (threadIdx.x == 0) *nslots = ns;
}

// Pipeline depth that fits the opt-in shared memory (227 KB) next to the
// 64 KB decode tables, counting the per-stage partial sums.
int stages_for(int in_dim, int nm, int tile_rows, int nw, int nt) {
    const int per_stage = nm * tile_rows * 98 * (in_dim / 256) + nm * tile_rows * nw * nt * 4 + 12;
    const int budget = 227 * 1024 - 65536 - 1024;
    return std::min(8, budget / per_stage);
}

// GEMV geometry for a given K (in_dim), matrices per stage (nm) and tokens per
// slot (nt): the most consumer warps NW (the kernel's cap, gemv_max_warps) such
// that 32*NW is a multiple of the sub-blocks per row SB, then the largest tile
// TR (multiple of 8, <= 32) whose stage splits into P <= 8 whole passes, whose
// reduction fits one butterfly (P * rows-per-warp * nt <= 32), that leaves at
// least 3 stages, that divides rows_div (the rows of one expert, 0 = any),
// and that has an instantiated kernel.
struct Geo {
    int nwarps, tile_rows, passes, rpw, stages;
};

int pick_geo(int in_dim, int nm, int nt, int rows_div, Geo* g) {
    if (in_dim <= 0 || in_dim % 256) return fail(GPEED_ERR_UNSUPPORTED, "in_dim %d not a multiple of 256", in_dim);
    const int SB = in_dim / 32;
    const int maxw = gp::gemv_max_warps(nt, nm == 2);
    for (int nw = maxw; nw >= 1; --nw) {
        if ((32 * nw) % SB) continue;
        const int rowstep = 32 * nw / SB;
        int rpw = 1;
        for (int w = 0; w < nw; ++w) rpw = std::max(rpw, (w * 32 + 31) / SB - (w * 32) / SB + 1);
        for (int tr = 32; tr >= 8; tr -= 8) {
            if ((nm * tr) % rowstep || (rows_div && rows_div % tr)) continue;
            const int p = nm * tr / rowstep;
            if (p > 8 || p * rpw * nt > 32) continue;
            const int st = stages_for(in_dim, nm, tr, nw, nt);
            if (st < 3 || !gp::gemv_variant_exists(nt, nm == 2, p, rpw)) continue;
            if (nm * tr * 98 * (in_dim / 256) > 40 * 1024 && tr > 8) continue;  // keep stages small
            g->nwarps = nw;
            g->tile_rows = tr;
            g->passes = p;
            g->rpw = rpw;
            g->stages = st;
            return GPEED_OK;
        }
    }
    return fail(GPEED_ERR_UNSUPPORTED, "no expert GEMV geometry for in_dim %d, %d matrices, %d tokens per slot",
                in_dim, nm, nt);
}

int nt_for(int ntok) {
    if (ntok <= 1) return 1;
    if (ntok <= 2) return 2;
    return 4;
}

constexpr size_t kStageBytes = size_t(32) << 20;
constexpr int kStages = 4;

// memcpy split over up to `nthr` host threads (page-cache reads of a mapped
// file fault in page by page; several threads keep the H2D link busy)
void parallel_copy(uint8_t* dst, const uint8_t* src, size_t n, unsigned nthr) {
    if (n < (size_t(2) << 20) || nthr <= 1) {
        std::memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    const size_t part = (n / nthr + 4095) & ~size_t(4095);
    size_t done = 0;
    try {
        for (unsigned i = 0; i + 1 < nthr && done + part < n; ++i, done += part)
            th.emplace_back([=] { std::memcpy(dst + done, src + done, part); });
    } catch (...) {  // no thread to be had: the calling thread copies the rest
    }
    std::memcpy(dst + done, src + done, n - done);
    for (auto& t : th) t.join();
}

// Pageable host bytes (a file mapping or a caller's array) -> device through
// kStages pinned buffers: host threads fill one while the copy engine drains
// the others, so an upload runs at the slower of the host reads and the H2D
// link rather than through the driver's synchronous pageable staging.
int h2d_staged(gpeed_ctx* c, void* dst, const void* src, size_t bytes, cudaStream_t st) {
    if (!c->stage[0]) {
        for (int i = 0; i < kStages; ++i) {
            GP_CUDA(cudaHostAlloc(&c->stage[i], kStageBytes, cudaHostAllocDefault));
            GP_CUDA(cudaEventCreateWithFlags(&c->stage_ev[i], cudaEventDisableTiming));
        }
    }
    const unsigned nthr = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint8_t* d = static_cast<uint8_t*>(dst);
    size_t k = 0;
    for (size_t off = 0; off < bytes; off += kStageBytes, ++k) {
        const int b = (int)(k % kStages);
        const size_t n = std::min(kStageBytes, bytes - off);
        GP_CUDA(cudaEventSynchronize(c->stage_ev[b]));  // the copy that last read this buffer has ended
        parallel_copy(c->stage[b], s + off, n, nthr);
        GP_CUDA(cudaMemcpyAsync(d + off, c->stage[b], n, cudaMemcpyHostToDevice, st));
        GP_CUDA(cudaEventRecord(c->stage_ev[b], st));
    }
    return GPEED_OK;
}

// Raw GGUF IQ3_XXS rows (host or device) -> the row-group layout at dst and,
// when dst_cols is given, also the column-slab layout of n_mat stacked down
// projections of rows / n_mat rows each.
int upload_matrix(gpeed_ctx* c, const void* raw, int on_device, int64_t rows, int in_dim, uint8_t* dst,
                  cudaStream_t st, uint8_t* dst_cols = nullptr, int64_t n_mat = 1) {
    const size_t raw_bytes = (size_t)rows * (in_dim / 256) * 98;
    const uint8_t* src = static_cast<const uint8_t*>(raw);
    uint8_t* tmp = nullptr;
    if (!on_device) {
        GP_CUDA(cudaMalloc(&tmp, raw_bytes));
        int rc = h2d_staged(c, tmp, raw, raw_bytes, st);
        if (rc) {
            cudaStreamSynchronize(st);
            cudaFree(tmp);
            return rc;
        }
        src = tmp;
    }
    GP_CUDA(gp::launch_repack(src, dst, rows, in_dim, st));
    if (dst_cols) GP_CUDA(gp::launch_repack_cols(src, dst_cols, n_mat, (int)(rows / n_mat), in_dim, st));
    if (tmp) {
        GP_CUDA(cudaStreamSynchronize(st));
        GP_CUDA(cudaFree(tmp));
    }
    return GPEED_OK;
}

int check_shape(const gpeed_moe_shape* s) {
    if (!s) return fail(GPEED_ERR_INVALID, "shape is NULL");
    if (s->hidden <= 0 || s->hidden % 512 || s->inter <= 0 || s->inter % 512)
        return fail(GPEED_ERR_UNSUPPORTED, "hidden (%d) and inter (%d) must be positive multiples of 512", s->hidden,
                    s->inter);
    if (s->n_experts <= 0 || s->n_experts > 512) return fail(GPEED_ERR_UNSUPPORTED, "n_experts %d not in [1, 512]", s->n_experts);
    if (s->top_k <= 0 || s->top_k > 32 || s->top_k > s->n_experts)
        return fail(GPEED_ERR_INVALID, "top_k %d not in [1, min(32, n_experts)]", s->top_k);
    if (s->n_shared < 0 || s->n_shared > 1) return fail(GPEED_ERR_UNSUPPORTED, "n_shared must be 0 or 1");
    if (s->inter % 8 || s->hidden % 32) return fail(GPEED_ERR_UNSUPPORTED, "row tiling needs inter%%8 == hidden%%32 == 0");
    return GPEED_OK;
}

int alloc_layer(gpeed_ctx* c, int layer, const gpeed_moe_shape* s, int e_lo, int e_cnt, const float* router_w,
                const float* corr, int on_device, Layer** out) {
    const int H = s->hidden, I = s->inter, E = s->n_experts, NE = e_cnt + s->n_shared;
    auto it = c->layers.find(layer);
    if (it != c->layers.end()) {
        Layer& old = it->second;
        cudaFree(old.router); cudaFree(old.corr); cudaFree(old.gate); cudaFree(old.up); cudaFree(old.down);
        cudaFree(old.down_col);
        cudaFree(old.router_split);
        c->layers.erase(it);
    }
    Layer L;
    L.shape = *s;
    L.e_lo = e_lo;
    L.e_cnt = e_cnt;
    L.u_cnt = I / 32;
    L.gu_stride = gp::repacked_bytes(I, H);
    L.d_stride = gp::repacked_bytes(H, I);
    const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    GP_CUDA(cudaMalloc(&L.router, sizeof(float) * E * H));
    GP_CUDA(cudaMemcpy(L.router, router_w, sizeof(float) * E * H, kind));
    L.router_nb = gp::router_tc_nb(E, H);
    if (L.router_nb) {
        GP_CUDA(cudaMalloc(&L.router_split, sizeof(uint16_t) * 2 * L.router_nb * H));
        GP_CUDA(gp::launch_router_split(L.router, E, H, L.router_nb, L.router_split, 0));
        GP_CUDA(cudaStreamSynchronize(0));
    }
    if (corr) {
        GP_CUDA(cudaMalloc(&L.corr, sizeof(float) * E));
        GP_CUDA(cudaMemcpy(L.corr, corr, sizeof(float) * E, kind));
    }
    // + 32 spare rows of padding after the last expert (tiles never read past the allocation)
    GP_CUDA(cudaMalloc(&L.gate, L.gu_stride * NE + gp::repacked_bytes(32, H)));
    GP_CUDA(cudaMalloc(&L.up, L.gu_stride * NE + gp::repacked_bytes(32, H)));
    GP_CUDA(cudaMalloc(&L.down, L.d_stride * NE + gp::repacked_bytes(32, I)));
    if (gp::decode_layer_supported(H, I, E, s->top_k, s->n_shared)) {
        L.dc_stride = (int64_t)H * (I / 256) * 98;
        GP_CUDA(cudaMalloc(&L.down_col, L.dc_stride * NE));
    }
    c->layers[layer] = L;
    *out = &c->layers[layer];
    return GPEED_OK;
}

int ensure_scratch(gpeed_ctx* c, int n, int E, int K, int H, int I) {
    const size_t nk = (size_t)n * K, na = nk + n;
    const size_t max_slots = nk + E + n + 4;  // nt >= 1
    int rc;
    const int rs = gp::router_splits(n, H, E);  // logits, then the router's split partial sums
    if ((rc = c->partial.ensure((size_t)n * E * (rs > 1 ? 1 + rs : 1)))) return rc;
    if ((rc = c->topk_w.ensure(nk))) return rc;
    if ((rc = c->route_chunks.ensure(gp::route_chunk_ints(n, K, E) + 1))) return rc;
    if ((rc = c->topk_ids.ensure(nk))) return rc;
    if ((rc = c->perm.ensure(na))) return rc;
    if ((rc = c->inv_pos.ensure(nk))) return rc;
    if ((rc = c->counts.ensure(E))) return rc;
    if ((rc = c->slots.ensure(max_slots))) return rc;
    if ((rc = c->nslots.ensure(1))) return rc;
    if ((rc = c->h.ensure(na * I))) return rc;
    if ((rc = c->D.ensure(na * H))) return rc;
    return GPEED_OK;
}

// The batched path's expert work for n rows: route (or take the given top-k),
// gate/up with SwiGLU, down, and the weighted combine into y.  `ro` holds the
// routing inputs; the scratch and slot fields are filled in here.
template <typename Mark>
int expert_pass(gpeed_ctx* c, const Layer& L, const void* x, int x_bf16, gp::RouteArgs ro, int combine_shared,
                const float* d_shared, float* y, cudaStream_t st, Mark&& mark) {
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, n = ro.n, K = ro.K;
    int rc;
    ro.perm_tok = c->perm.p;
    ro.inv_pos = c->inv_pos.p;
    ro.counts = c->counts.p;
    ro.slots = c->slots.p;
    ro.max_slots = (int)c->slots.n;
    ro.nslots = c->nslots.p;
    ro.status = c->status;
    ro.chunk_counts = c->route_chunks.p;
    ro.chunk_cap = c->route_chunks.n;
    const int npos = n * K;
    if (npos >= c->tc_min_tokens && !ro.with_shared && gp::tc_moe_supported(H, I)) {
        // large batches: grouped GEMMs on the tensor cores over slots of <= 224 rows
        // (the same kernels as the whole-layer forward; here without the shared expert)
        ro.nt = gp::tc_moe_slot_tokens();
        GP_CUDA(gp::launch_route(ro, st, false));
        if ((rc = c->xp.ensure((size_t)npos * H))) return rc;
        GP_CUDA(gp::launch_gather_cast(x, x_bf16, c->perm.p, npos, H, c->xp.p, c->status, st));
        mark(2);
        const int El = L.e_cnt + s.n_shared;
        uint16_t* h16 = reinterpret_cast<uint16_t*>(c->h.p);  // npos x I fp16 fits the fp32 h scratch
        gp::TcArgs ga{c->slots.p, c->nslots.p, I / 128, H, I, s.swiglu_limit, h16, c->status};
        GP_CUDA(gp::launch_tc_moe(true, L.gate, L.up, (int64_t)El * I, c->xp.p, npos, ga, c->num_sms, st));
        mark(3);
        gp::TcArgs da{c->slots.p, c->nslots.p, H / 128, I, H, 0.f, c->D.p, c->status};
        GP_CUDA(gp::launch_tc_moe(false, L.down, nullptr, (int64_t)El * H, h16, npos, da, c->num_sms, st));
        mark(4);
        gp::CombineArgs cb{c->D.p, c->inv_pos.p, ro.topk_w, n, K, H, combine_shared, y, d_shared};
        GP_CUDA(gp::launch_combine(cb, st, false));
        return GPEED_OK;
    }
    Geo ggu, gd;
    // one slot list serves both expert kernels: its token count must suit both
    const int nt = nt_for(n);
    if ((rc = pick_geo(H, 2, nt, I, &ggu))) return rc;
    if ((rc = pick_geo(I, 1, nt, H, &gd))) return rc;
    ro.nt = nt;
    GP_CUDA(gp::launch_route(ro, st, !c->prof));
    mark(2);

    gp::GemvArgs a{};
    a.w0 = L.gate;
    a.w1 = L.up;
    a.expert_stride = L.gu_stride;
    a.in_dim = H;
    a.rows = I;
    a.tile_rows = ggu.tile_rows;
    a.nwarps = ggu.nwarps;
    a.stages = ggu.stages;
    a.slots = c->slots.p;
    a.nslots = c->nslots.p;
    a.perm_tok = c->perm.p;
    a.x = x;
    a.x_bf16 = x_bf16;
    a.out = c->h.p;
    a.limit = s.swiglu_limit;
    a.tables = c->tables;
    a.status = c->status;
    if (I % a.tile_rows) return fail(GPEED_ERR_UNSUPPORTED, "inter %% %d != 0", a.tile_rows);
    GP_CUDA(gp::launch_gemv(a, nt, true, ggu.passes, ggu.rpw, c->num_sms, st, !c->prof));
    mark(3);

    gp::GemvArgs d{};
    d.w0 = L.down;
    d.w1 = nullptr;
    d.expert_stride = L.d_stride;
    d.in_dim = I;
    d.rows = H;
    d.tile_rows = gd.tile_rows;
    d.nwarps = gd.nwarps;
    d.stages = gd.stages;
    d.slots = c->slots.p;
    d.nslots = c->nslots.p;
    d.perm_tok = nullptr;
    d.x = c->h.p;
    d.x_bf16 = 0;
    d.out = c->D.p;
    d.tables = c->tables;
    d.status = c->status;
    if (H % d.tile_rows) return fail(GPEED_ERR_UNSUPPORTED, "hidden %% %d != 0", d.tile_rows);
    GP_CUDA(gp::launch_gemv(d, nt, false, gd.passes, gd.rpw, c->num_sms, st, !c->prof));
    mark(4);

    gp::CombineArgs cb{c->D.p, c->inv_pos.p, ro.topk_w, n, K, H, combine_shared, y, d_shared};
    GP_CUDA(gp::launch_combine(cb, st, !c->prof));
    return GPEED_OK;
}

// Arguments of the persistent decode kernel (decode_layer.cu) for n_tok
// tokens of layer L, with the context's exchange buffers sized (and their
// tags zeroed) on first use.  Outside stream capture on first use.
int fused_args(gpeed_ctx* c, const Layer& L, const void* x, int x_dtype, int n_tok, int own_tok, float* y,
               const int* forced, int* topk_ids, float* topk_w, cudaStream_t st, gp::DecodeLayerArgs* out) {
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, E = s.n_experts, K = s.top_k;
    int rc;
    const size_t had = c->logits.n;
    if ((rc = c->logits.ensure(gp::decode_layer_logit_words(E)))) return rc;
    if (c->logits.n != had)  // tags must start below the first launch's
        GP_CUDA(cudaMemsetAsync(c->logits.p, 0, c->logits.n * sizeof(unsigned long long), st));
    const size_t had_h = c->hx.n;
    if ((rc = c->hx.ensure(gp::decode_layer_h_words(I)))) return rc;
    if (c->hx.n != had_h) GP_CUDA(cudaMemsetAsync(c->hx.p, 0, c->hx.n * sizeof(unsigned long long), st));
    gp::DecodeLayerArgs& da = *out;
    da = gp::DecodeLayerArgs{};
    da.router = L.router;
    da.corr = L.corr;
    if (!L.down_col) return fail(GPEED_ERR_UNSUPPORTED, "layer holds no column-slab copy of its down projections");
    da.gate = L.gate;
    da.up = L.up;
    da.down_col = L.down_col;
    da.gu_stride = L.gu_stride;
    da.dc_stride = L.dc_stride;
    da.H = H;
    da.I = I;
    da.E = E;
    da.K = K;
    da.routed_scale = s.routed_scale;
    da.norm_topk = s.norm_topk;
    da.limit = s.swiglu_limit;
    da.with_shared = s.n_shared;
    da.x = x;
    da.x_bf16 = x_dtype == GPEED_DTYPE_BF16;
    da.y = y;
    da.forced = forced;
    da.topk_ids = topk_ids;
    da.topk_w = topk_w;
    da.n_tok = n_tok;
    da.e_lo = L.e_lo;
    da.e_cnt = L.e_cnt;
    da.own_tok = own_tok;
    da.u_lo = L.u_lo;
    da.u_cnt = L.u_cnt;
    da.logits = c->logits.p;
    da.hx = c->hx.p;
    da.sync = c->sync;
    da.tables = c->tables;
    da.status = c->status;
    da.stages = 3;  // the deepest stage ring that fits next to the tables
    while (gp::decode_layer_smem(H, I, da.stages + 1, n_tok) <= 227u * 1024u && da.stages < 8) ++da.stages;
    da.cooperative = c->fused_cooperative;
    da.spin_limit = c->spin_limit;
    da.withhold_logit = c->withhold_logit;
    return GPEED_OK;
}

// One gpeed_matmul_quant call (WeightStore::matmul_quant, weights.cpp:86-165):
// the validated arguments and the GEMV geometry.  Both the allocating entry
// point and gpeed_matmul_quant_noalloc run exactly this plan; they differ only
// in where the work list and the staged output live (MatmulScratch).
struct MatmulPlan {
    bool empty = false;         // n_tok or out_dim <= 0: nothing to do (weights.cpp:88)
    const Tensor* t = nullptr;
    Geo g{};
    int nt = 1, ns = 0, n_tok = 0, in_dim = 0, out_dim = 0;
    int64_t g0 = 0, skip = 0, ntile = 0, rows_eff = 0;
    bool direct = true;         // output rows land in Y as they are (no staging)
    size_t staged_floats() const { return direct ? 0 : (size_t)n_tok * rows_eff; }
};

struct MatmulScratch {
    gp::SlotDesc* slots;        // >= plan.ns descriptors
    int* nslots;
    float* staged;              // >= plan.staged_floats(), or nullptr when direct
};

int plan_matmul(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* X, int n_tok,
                const float* Y, MatmulPlan* p) {
    if (!c || handle < 0 || handle >= (int)c->tensors.size()) return fail(GPEED_ERR_INVALID, "bad handle");
    if (n_tok <= 0 || out_dim <= 0) {
        p->empty = true;
        return GPEED_OK;
    }
    const Tensor& t = c->tensors[handle];
    if (in_dim != t.in_dim) return fail(GPEED_ERR_INVALID, "in_dim %d != tensor in_dim %d", in_dim, t.in_dim);
    if ((int64_t)row0 + out_dim > t.rows)
        return fail(GPEED_ERR_INVALID, "rows [%llu, %llu) past the tensor's %lld rows", (unsigned long long)row0,
                    (unsigned long long)row0 + out_dim, (long long)t.rows);
    if (!X || !Y || (reinterpret_cast<uintptr_t>(X) & 15)) return fail(GPEED_ERR_INVALID, "X must be a 16-byte aligned device pointer");
    int rc;
    if ((rc = set_device(c))) return rc;
    p->t = &t;
    p->nt = nt_for(n_tok);
    if ((rc = pick_geo(in_dim, 1, p->nt, 0, &p->g))) return rc;
    p->n_tok = n_tok;
    p->in_dim = in_dim;
    p->out_dim = out_dim;
    p->g0 = (int64_t)row0 / 8 * 8;
    p->skip = (int64_t)row0 - p->g0;
    p->ntile = (p->skip + out_dim + p->g.tile_rows - 1) / p->g.tile_rows;
    p->rows_eff = p->ntile * p->g.tile_rows;
    p->ns = (n_tok + p->nt - 1) / p->nt;
    p->direct = p->skip == 0 && p->rows_eff == out_dim;
    return GPEED_OK;
}

int run_matmul(gpeed_ctx* c, const MatmulPlan& p, const float* X, float* Y, const MatmulScratch& sc,
               cudaStream_t st) {
    make_slots_kernel<<<1, 256, 0, st>>>(sc.slots, sc.nslots, p.n_tok, p.nt);
    GP_CUDA(cudaGetLastError());
    gp::GemvArgs a{};
    a.w0 = p.t->packed + (p.g0 / 8) * 784 * (p.in_dim / 256);
    a.w1 = nullptr;
    a.expert_stride = 0;
    a.in_dim = p.in_dim;
    a.rows = (int)p.rows_eff;
    a.tile_rows = p.g.tile_rows;
    a.nwarps = p.g.nwarps;
    a.stages = p.g.stages;
    a.slots = sc.slots;
    a.nslots = sc.nslots;
    a.perm_tok = nullptr;
    a.x = X;
    a.x_bf16 = 0;
    a.out = p.direct ? Y : sc.staged;
    a.limit = 0.f;
    a.tables = c->tables;
    a.status = c->status;
    const int grid = (int)std::min<int64_t>(c->num_sms, p.ntile * p.ns);
    GP_CUDA(gp::launch_gemv(a, p.nt, false, p.g.passes, p.g.rpw, grid, st, false));
    if (!p.direct)
        GP_CUDA(cudaMemcpy2DAsync(Y, sizeof(float) * p.out_dim, sc.staged + p.skip, sizeof(float) * p.rows_eff,
                                  sizeof(float) * p.out_dim, p.n_tok, cudaMemcpyDeviceToDevice, st));
    return GPEED_OK;
}

}  // namespace

extern "C" {

const char* gpeed_last_error(void) { return g_err.c_str(); }
int gpeed_version(void) { return 1; }

int gpeed_ctx_create(int device, gpeed_ctx** out) {
    if (!out) return fail(GPEED_ERR_INVALID, "out is NULL");
    *out = nullptr;
    int ndev = 0;
    GP_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(GPEED_ERR_INVALID, "device %d not present (%d devices)", device, ndev);
    GP_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    GP_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(GPEED_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device,
                                      prop.major, prop.minor);
    gpeed_ctx* c = new gpeed_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if (cudaMalloc(&c->tables, 65536) != cudaSuccess || cudaMalloc(&c->status, sizeof(uint32_t)) != cudaSuccess) {
        delete c;
        return fail(GPEED_ERR_CUDA, "cudaMalloc failed in ctx_create");
    }
    cudaMemset(c->status, 0, sizeof(uint32_t));
    if (cudaMalloc(&c->sync, gp::kDecodeSyncWords * sizeof(unsigned)) != cudaSuccess) {
        cudaFree(c->tables);
        cudaFree(c->status);
        delete c;
        return fail(GPEED_ERR_CUDA, "cudaMalloc failed in ctx_create");
    }
    cudaMemset(c->sync, 0, gp::kDecodeSyncWords * sizeof(unsigned));
    cudaError_t e = gp::build_tables(c->tables, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(c->tables);
        cudaFree(c->status);
        delete c;
        return fail(GPEED_ERR_CUDA, "table build: %s", cudaGetErrorString(e));
    }
    *out = c;
    return GPEED_OK;
}

void ep_release(gpeed_ctx* c);  // (below, with the expert-parallel entry points)

int gpeed_ctx_destroy(gpeed_ctx* c) {
    if (!c) return GPEED_OK;
    set_device(c);
    cudaDeviceSynchronize();
    for (auto& t : c->tensors) cudaFree(t.packed);
    for (auto& kv : c->layers) {
        Layer& L = kv.second;
        cudaFree(L.router); cudaFree(L.corr); cudaFree(L.gate); cudaFree(L.up); cudaFree(L.down);
        cudaFree(L.down_col);
        cudaFree(L.router_split);
    }
    c->partial.release(); c->topk_w.release(); c->h.release(); c->D.release(); c->mvout.release();
    c->topk_ids.release(); c->perm.release(); c->inv_pos.release(); c->counts.release(); c->nslots.release();
    c->slots.release();
    for (auto& e : c->ev)
        if (e) cudaEventDestroy(e);
    c->logits.release();
    c->hx.release();
    ep_release(c);
    c->xp.release();
    c->route_chunks.release();
    c->mhc_partial.release();
    cudaFree(c->sync);
    cudaFree(c->tables);
    cudaFree(c->status);
    for (int i = 0; i < 4; ++i) {
        if (c->stage[i]) cudaFreeHost(c->stage[i]);
        if (c->stage_ev[i]) cudaEventDestroy(c->stage_ev[i]);
    }
    if (c->host_pin) cudaFreeHost(c->host_pin);
    c->host_x.release();
    c->host_y.release();
    if (c->host_stream) cudaStreamDestroy(c->host_stream);
    delete c;
    return GPEED_OK;
}

int gpeed_ctx_check(gpeed_ctx* c, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    int rc;
    if ((rc = set_device(c))) return rc;
    GP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    uint32_t st = 0;
    GP_CUDA(cudaMemcpy(&st, c->status, sizeof(st), cudaMemcpyDeviceToHost));
    if (st) {
        GP_CUDA(cudaMemset(c->status, 0, sizeof(uint32_t)));
        // a kernel that gave up may leave counters set; generation and logit
        // tags restart together
        GP_CUDA(cudaMemset(c->sync, 0, gp::kDecodeSyncWords * sizeof(unsigned)));
        if (c->logits.p) GP_CUDA(cudaMemset(c->logits.p, 0, c->logits.n * sizeof(unsigned long long)));
        if (c->hx.p) GP_CUDA(cudaMemset(c->hx.p, 0, c->hx.n * sizeof(unsigned long long)));
        // (an expert-parallel group whose step failed is set up again: its
        // counters are shared with the other ranks)
        return fail(GPEED_ERR_DEVICE, "device status 0x%x (1: stage wait timed out, 2: drain wait timed out, "
                                      "4: expert id out of range, 8: bad shape, 16: a token or h value past the fp16 range "
                                      "on the tensor-core path)", st);
    }
    return GPEED_OK;
}

int gpeed_ctx_set_option(gpeed_ctx* c, int option, int value) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    switch (option) {
        case GPEED_OPT_FUSED_DECODE: c->fused_decode = value != 0; return GPEED_OK;
        case GPEED_OPT_FUSED_MAX_TOKENS:
            if (value < 1) return fail(GPEED_ERR_INVALID, "GPEED_OPT_FUSED_MAX_TOKENS must be >= 1");
            c->fused_max_tokens = value;
            return GPEED_OK;
        case GPEED_OPT_FUSED_COOPERATIVE: c->fused_cooperative = value != 0; return GPEED_OK;
        case GPEED_OPT_SPIN_LIMIT:
            if (value < 1) return fail(GPEED_ERR_INVALID, "GPEED_OPT_SPIN_LIMIT must be >= 1");
            c->spin_limit = (uint32_t)value;
            return GPEED_OK;
        case GPEED_OPT_TEST_WITHHOLD_LOGIT: c->withhold_logit = value < 0 ? -1 : value; return GPEED_OK;
        case GPEED_OPT_TC_MIN_TOKENS:
            if (value < 1) return fail(GPEED_ERR_INVALID, "tensor-core threshold must be >= 1");
            c->tc_min_tokens = value;
            return GPEED_OK;
        default: return fail(GPEED_ERR_INVALID, "unknown option %d", option);
    }
}

int gpeed_ctx_profile(gpeed_ctx* c, int enable) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    int rc;
    if ((rc = set_device(c))) return rc;
    if (enable && !c->ev[0])
        for (auto& e : c->ev) GP_CUDA(cudaEventCreate(&e));
    c->prof = enable != 0;
    for (double& v : c->prof_ms) v = 0;
    c->prof_calls = 0;
    return GPEED_OK;
}

int gpeed_ctx_profile_read(gpeed_ctx* c, float* stage_ms, int* calls) {
    if (!c || !stage_ms || !calls) return fail(GPEED_ERR_INVALID, "NULL argument");
    for (int i = 0; i < 5; ++i) stage_ms[i] = c->prof_calls ? (float)(c->prof_ms[i] / c->prof_calls) : 0.f;
    *calls = (int)c->prof_calls;
    return GPEED_OK;
}

int gpeed_iq3xxs_dequantize(const void* src, float* dst, uint64_t n, void* stream) {
    if (n % 256) return fail(GPEED_ERR_INVALID, "dequantize: element count not a multiple of block size");
    if (!src || !dst) return fail(GPEED_ERR_INVALID, "NULL pointer");
    if (reinterpret_cast<uintptr_t>(dst) & 15) return fail(GPEED_ERR_INVALID, "dst must be 16-byte aligned");
    GP_CUDA(gp::launch_dequantize(static_cast<const uint8_t*>(src), dst, (int64_t)(n / 256), (cudaStream_t)stream));
    return GPEED_OK;
}

int gpeed_synth_iq3xxs(void* dst, uint64_t seed, uint64_t stream, uint64_t block0, uint64_t nblocks, void* st) {
    if (!dst) return fail(GPEED_ERR_INVALID, "NULL pointer");
    GP_CUDA(gp::launch_synth(static_cast<uint8_t*>(dst), seed, stream, block0, (int64_t)nblocks, (cudaStream_t)st));
    return GPEED_OK;
}

int gpeed_dequantize(int dtype, const void* src, float* dst, uint64_t n, void* stream) {
    const int bv = gp::codec_block_values(dtype);
    if (!bv) return fail(GPEED_ERR_UNSUPPORTED, "dequantize: type %d not implemented", dtype);
    if (n % (uint64_t)bv) return fail(GPEED_ERR_INVALID, "dequantize: element count not a multiple of block size");
    if (n == 0) return GPEED_OK;
    if (!src || !dst || (reinterpret_cast<uintptr_t>(dst) & 15) || (bv == 1 && (reinterpret_cast<uintptr_t>(src) & 3)))
        return fail(GPEED_ERR_INVALID, "dequantize: NULL or unaligned buffer (dst 16-byte, element-wise src 4-byte)");
    GP_CUDA(gp::launch_codec_dequantize(dtype, src, dst, (int64_t)n, (cudaStream_t)stream));
    return GPEED_OK;
}

int gpeed_tensor_upload(gpeed_ctx* c, const void* raw, int on_device, int dtype, uint64_t rows, int in_dim, int* handle) {
    if (!c || !raw || !handle) return fail(GPEED_ERR_INVALID, "NULL argument");
    if (dtype != GPEED_DTYPE_IQ3_XXS) return fail(GPEED_ERR_UNSUPPORTED, "dtype %d: only IQ3_XXS (18) is supported", dtype);
    if (in_dim <= 0 || in_dim % 256) return fail(GPEED_ERR_INVALID, "in_dim %d not a multiple of 256", in_dim);
    if (rows == 0) return fail(GPEED_ERR_INVALID, "rows == 0");
    int rc;
    if ((rc = set_device(c))) return rc;
    Tensor t;
    t.rows = (int64_t)rows;
    t.in_dim = in_dim;
    GP_CUDA(cudaMalloc(&t.packed, gp::repacked_bytes(padded_rows(t.rows), in_dim)));
    GP_CUDA(cudaMemset(t.packed, 0, gp::repacked_bytes(padded_rows(t.rows), in_dim)));
    if ((rc = upload_matrix(c, raw, on_device, t.rows, in_dim, t.packed, 0))) return rc;
    GP_CUDA(cudaDeviceSynchronize());
    c->tensors.push_back(t);
    *handle = (int)c->tensors.size() - 1;
    return GPEED_OK;
}

int gpeed_tensor_download(gpeed_ctx* c, int handle, void* raw_host) {
    if (!c || !raw_host || handle < 0 || handle >= (int)c->tensors.size()) return fail(GPEED_ERR_INVALID, "bad handle");
    int rc;
    if ((rc = set_device(c))) return rc;
    const Tensor& t = c->tensors[handle];
    const size_t bytes = (size_t)t.rows * (t.in_dim / 256) * 98;
    uint8_t* tmp = nullptr;
    GP_CUDA(cudaMalloc(&tmp, bytes));
    GP_CUDA(gp::launch_unpack(t.packed, tmp, t.rows, t.in_dim, 0));
    GP_CUDA(cudaMemcpy(raw_host, tmp, bytes, cudaMemcpyDeviceToHost));
    GP_CUDA(cudaFree(tmp));
    return GPEED_OK;
}

int gpeed_matmul_quant(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* X, int n_tok,
                       float* Y, void* stream) {
    MatmulPlan p;
    int rc;
    if ((rc = plan_matmul(c, handle, row0, in_dim, out_dim, X, n_tok, Y, &p)) || p.empty) return rc;
    MatmulScratch sc;
    if ((rc = c->slots.ensure(p.ns))) return rc;
    if ((rc = c->nslots.ensure(1))) return rc;
    if (!p.direct && (rc = c->mvout.ensure((size_t)n_tok * p.rows_eff))) return rc;
    sc.slots = c->slots.p;
    sc.nslots = c->nslots.p;
    sc.staged = p.direct ? nullptr : c->mvout.p;
    return run_matmul(c, p, X, Y, sc, (cudaStream_t)stream);
}

int gpeed_matvec_quant(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* x, float* dst,
                       void* stream) {
    return gpeed_matmul_quant(c, handle, row0, in_dim, out_dim, x, 1, dst, stream);
}

int gpeed_matmul_quant_host(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* X,
                            int n_tok, float* Y) {
    if (!c || handle < 0 || handle >= (int)c->tensors.size()) return fail(GPEED_ERR_INVALID, "bad handle");
    if (n_tok <= 0 || out_dim <= 0) return GPEED_OK;  // weights.cpp:88
    if (!X || !Y) return fail(GPEED_ERR_INVALID, "X and Y must be host buffers");
    int rc;
    if ((rc = set_device(c))) return rc;
    std::lock_guard<std::mutex> lock(c->host_mu);
    if (!c->host_stream) GP_CUDA(cudaStreamCreateWithFlags(&c->host_stream, cudaStreamNonBlocking));
    const size_t nx = (size_t)n_tok * in_dim, ny = (size_t)n_tok * out_dim;
    if (c->host_pin_n < nx + ny) {
        if (c->host_pin) cudaFreeHost(c->host_pin);
        c->host_pin = nullptr;
        c->host_pin_n = 0;
        GP_CUDA(cudaHostAlloc(&c->host_pin, (nx + ny) * sizeof(float), cudaHostAllocDefault));
        c->host_pin_n = nx + ny;
    }
    if ((rc = c->host_x.ensure(nx)) || (rc = c->host_y.ensure(ny))) return rc;
    cudaStream_t st = c->host_stream;
    std::memcpy(c->host_pin, X, nx * sizeof(float));
    GP_CUDA(cudaMemcpyAsync(c->host_x.p, c->host_pin, nx * sizeof(float), cudaMemcpyHostToDevice, st));
    if ((rc = gpeed_matmul_quant(c, handle, row0, in_dim, out_dim, c->host_x.p, n_tok, c->host_y.p, st))) return rc;
    GP_CUDA(cudaMemcpyAsync(c->host_pin + nx, c->host_y.p, ny * sizeof(float), cudaMemcpyDeviceToHost, st));
    GP_CUDA(cudaStreamSynchronize(st));
    std::memcpy(Y, c->host_pin + nx, ny * sizeof(float));
    uint32_t dev_status = 0;
    GP_CUDA(cudaMemcpy(&dev_status, c->status, sizeof(dev_status), cudaMemcpyDeviceToHost));
    if (dev_status) return gpeed_ctx_check(c, st);  // reports and clears it
    return GPEED_OK;
}

int gpeed_matvec_quant_host(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* x,
                            float* dst) {
    return gpeed_matmul_quant_host(c, handle, row0, in_dim, out_dim, x, 1, dst);
}

int gpeed_moe_forward_host(gpeed_ctx* c, int layer, const void* x, int x_dtype, int n, float* y) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (n == 0) return GPEED_OK;
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!x || !y) return fail(GPEED_ERR_INVALID, "x and y must be host buffers");
    const int H = it->second.shape.hidden;
    int rc;
    if ((rc = set_device(c))) return rc;
    std::lock_guard<std::mutex> lock(c->host_mu);
    if (!c->host_stream) GP_CUDA(cudaStreamCreateWithFlags(&c->host_stream, cudaStreamNonBlocking));
    // staging in floats: x (bf16 rows take half the room), then y from a
    // 16-byte boundary, then the device status word (read back with y, so
    // the call waits once)
    const size_t xbytes = (size_t)n * H * (x_dtype == GPEED_DTYPE_BF16 ? 2 : 4), ny = (size_t)n * H;
    const size_t nx = ((xbytes + 15) & ~(size_t)15) / sizeof(float);
    if (c->host_pin_n < nx + ny + 4) {
        if (c->host_pin) cudaFreeHost(c->host_pin);
        c->host_pin = nullptr;
        c->host_pin_n = 0;
        GP_CUDA(cudaHostAlloc(&c->host_pin, (nx + ny + 4) * sizeof(float), cudaHostAllocDefault));
        c->host_pin_n = nx + ny + 4;
    }
    if ((rc = c->host_x.ensure(nx)) || (rc = c->host_y.ensure(ny))) return rc;
    cudaStream_t st = c->host_stream;
    std::memcpy(c->host_pin, x, xbytes);
    GP_CUDA(cudaMemcpyAsync(c->host_x.p, c->host_pin, xbytes, cudaMemcpyHostToDevice, st));
    if ((rc = gpeed_moe_forward(c, layer, c->host_x.p, x_dtype, n, c->host_y.p, nullptr, nullptr, nullptr, st)))
        return rc;
    uint32_t* status_pin = reinterpret_cast<uint32_t*>(c->host_pin + nx + ny);
    GP_CUDA(cudaMemcpyAsync(c->host_pin + nx, c->host_y.p, ny * sizeof(float), cudaMemcpyDeviceToHost, st));
    GP_CUDA(cudaMemcpyAsync(status_pin, c->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    GP_CUDA(cudaStreamSynchronize(st));
    std::memcpy(y, c->host_pin + nx, ny * sizeof(float));
    if (*status_pin) return gpeed_ctx_check(c, st);  // reports and clears it
    return GPEED_OK;
}

int gpeed_moe_load_layer_range(gpeed_ctx* c, int layer, const gpeed_moe_shape* s, int expert_begin, int expert_count,
                               const float* router_w, const float* corr, const void* gate, const void* up,
                               const void* down, const void* gate_sh, const void* up_sh, const void* down_sh,
                               int on_device) {
    int rc;
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if ((rc = check_shape(s))) return rc;
    if (expert_begin < 0 || expert_count < 0 || expert_begin + expert_count > s->n_experts)
        return fail(GPEED_ERR_INVALID, "expert range [%d, %d) outside [0, %d)", expert_begin,
                    expert_begin + expert_count, s->n_experts);
    if (!router_w || (expert_count && (!gate || !up || !down))) return fail(GPEED_ERR_INVALID, "NULL expert tensor");
    if (s->n_shared && (!gate_sh || !up_sh || !down_sh)) return fail(GPEED_ERR_INVALID, "n_shared=1 needs the shared tensors");
    if ((rc = set_device(c))) return rc;
    Layer* L;
    if ((rc = alloc_layer(c, layer, s, expert_begin, expert_count, router_w, corr, on_device, &L))) return rc;
    const int H = s->hidden, I = s->inter, EC = expert_count;
    if (EC) {
        if ((rc = upload_matrix(c, gate, on_device, (int64_t)EC * I, H, L->gate, 0))) return rc;
        if ((rc = upload_matrix(c, up, on_device, (int64_t)EC * I, H, L->up, 0))) return rc;
        if ((rc = upload_matrix(c, down, on_device, (int64_t)EC * H, I, L->down, 0, L->down_col, EC))) return rc;
    }
    if (s->n_shared) {
        if ((rc = upload_matrix(c, gate_sh, on_device, I, H, L->gate + L->gu_stride * EC, 0))) return rc;
        if ((rc = upload_matrix(c, up_sh, on_device, I, H, L->up + L->gu_stride * EC, 0))) return rc;
        if ((rc = upload_matrix(c, down_sh, on_device, H, I, L->down + L->d_stride * EC, 0,
                                L->down_col ? L->down_col + L->dc_stride * EC : nullptr, 1)))
            return rc;
    }
    GP_CUDA(cudaDeviceSynchronize());
    return GPEED_OK;
}

int gpeed_moe_load_layer(gpeed_ctx* c, int layer, const gpeed_moe_shape* s, const float* router_w, const float* corr,
                         const void* gate, const void* up, const void* down, const void* gate_sh, const void* up_sh,
                         const void* down_sh, int on_device) {
    if (!s) return fail(GPEED_ERR_INVALID, "shape is NULL");
    return gpeed_moe_load_layer_range(c, layer, s, 0, s->n_experts, router_w, corr, gate, up, down, gate_sh, up_sh,
                                      down_sh, on_device);
}

int gpeed_moe_synth_layer_range(gpeed_ctx* c, int layer, const gpeed_moe_shape* s, int expert_begin,
                                int expert_count, const float* router_w, const float* corr, int on_device,
                                uint64_t seed, uint64_t stream0) {
    int rc;
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if ((rc = check_shape(s))) return rc;
    if (!router_w) return fail(GPEED_ERR_INVALID, "router_w is NULL");
    if (expert_begin < 0 || expert_count < 0 || expert_begin + expert_count > s->n_experts)
        return fail(GPEED_ERR_INVALID, "expert range [%d, %d) outside [0, %d)", expert_begin,
                    expert_begin + expert_count, s->n_experts);
    if ((rc = set_device(c))) return rc;
    Layer* L;
    if ((rc = alloc_layer(c, layer, s, expert_begin, expert_count, router_w, corr, on_device, &L))) return rc;
    const int H = s->hidden, I = s->inter, EC = expert_count;
    // block indices of the full layer's generator streams: a range holds the
    // same bytes as the matching slice of the whole layer
    const int64_t bgu = (int64_t)I * (H / 256), bd = (int64_t)H * (I / 256);
    const int64_t nb_gu = EC * bgu, nb_d = EC * bd;
    uint8_t* tmp = nullptr;
    GP_CUDA(cudaMalloc(&tmp, (size_t)std::max<int64_t>(std::max(nb_gu, nb_d), bgu) * 98));
    struct M { uint8_t* dst; int64_t rows; int in; int64_t block0, nb; };
    const M mats[6] = {{L->gate, (int64_t)EC * I, H, expert_begin * bgu, nb_gu},
                       {L->up, (int64_t)EC * I, H, expert_begin * bgu, nb_gu},
                       {L->down, (int64_t)EC * H, I, expert_begin * bd, nb_d},
                       {L->gate + L->gu_stride * EC, I, H, 0, bgu},
                       {L->up + L->gu_stride * EC, I, H, 0, bgu},
                       {L->down + L->d_stride * EC, H, I, 0, bd}};
    for (int m = 0; m < (s->n_shared ? 6 : 3); ++m) {
        if (!mats[m].nb) continue;
        GP_CUDA(gp::launch_synth(tmp, seed, stream0 + m, mats[m].block0, mats[m].nb, 0));
        GP_CUDA(gp::launch_repack(tmp, mats[m].dst, mats[m].rows, mats[m].in, 0));
        if (L->down_col && (m == 2 || m == 5))  // the down projections, also as column slabs
            GP_CUDA(gp::launch_repack_cols(tmp, L->down_col + (m == 5 ? L->dc_stride * EC : 0), m == 5 ? 1 : EC, H, I,
                                           0));
    }
    GP_CUDA(cudaDeviceSynchronize());
    GP_CUDA(cudaFree(tmp));
    return GPEED_OK;
}

int gpeed_moe_synth_layer(gpeed_ctx* c, int layer, const gpeed_moe_shape* s, const float* router_w, const float* corr,
                          int on_device, uint64_t seed, uint64_t stream0) {
    if (!s) return fail(GPEED_ERR_INVALID, "shape is NULL");
    return gpeed_moe_synth_layer_range(c, layer, s, 0, s->n_experts, router_w, corr, on_device, seed, stream0);
}

int gpeed_moe_slice_units(gpeed_ctx* c, int layer, int unit_begin, int unit_count) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    Layer& L = it->second;
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, NU = I / 32, E = s.n_experts;
    if (L.sliced()) return fail(GPEED_ERR_INVALID, "layer %d is already sliced", layer);
    if (L.e_cnt != E) return fail(GPEED_ERR_INVALID, "layer %d holds an expert range: slice a whole layer", layer);
    if (!L.down_col || !gp::decode_layer_slice_supported(I, unit_count))
        return fail(GPEED_ERR_UNSUPPORTED, "no persistent decode kernel for %d of the %d units of inter %d", unit_count,
                    NU, I);
    if (unit_begin < 0 || unit_begin + unit_count > NU || unit_begin % unit_count)
        return fail(GPEED_ERR_INVALID, "units [%d, %d): a whole slice of the %d, starting at a multiple of its size",
                    unit_begin, unit_begin + unit_count, NU);
    int rc;
    if ((rc = set_device(c))) return rc;
    const int NR = L.e_cnt;
    // gate/up: 4 row groups of 8 rows per unit; down: the units' column slabs,
    // then the 256-input d blocks they fall in (repacked_bytes,
    // launch_repack_cols).  The shared expert follows whole, in the same
    // layouts (it starts at NR times the sliced strides).
    const int64_t tile = gp::repacked_bytes(8, H), unit_col = (int64_t)H * 12;
    const int blk_lo = unit_begin / 8, nblk = (unit_begin + unit_count - 1) / 8 - blk_lo + 1;
    const int64_t gu_w = (int64_t)unit_count * 4 * tile;
    const int64_t dc_w = (int64_t)unit_count * unit_col, dd_w = (int64_t)nblk * H * 2;
    const int64_t sh_gu = s.n_shared ? L.gu_stride : 0, sh_dc = s.n_shared ? L.dc_stride : 0;
    uint8_t *g = nullptr, *u = nullptr, *dc = nullptr;
    auto undo = [&]() { cudaFree(g); cudaFree(u); cudaFree(dc); };
    if (cudaMalloc(&g, gu_w * NR + sh_gu + gp::repacked_bytes(32, H)) != cudaSuccess ||
        cudaMalloc(&u, gu_w * NR + sh_gu + gp::repacked_bytes(32, H)) != cudaSuccess ||
        cudaMalloc(&dc, (dc_w + dd_w) * NR + sh_dc) != cudaSuccess) {
        undo();
        cudaGetLastError();
        return fail(GPEED_ERR_CUDA, "out of device memory slicing layer %d", layer);
    }
    const cudaMemcpyKind d2d = cudaMemcpyDeviceToDevice;
    cudaError_t e = cudaMemcpy2D(g, gu_w, L.gate + unit_begin * 4 * tile, L.gu_stride, gu_w, NR, d2d);
    if (!e) e = cudaMemcpy2D(u, gu_w, L.up + unit_begin * 4 * tile, L.gu_stride, gu_w, NR, d2d);
    if (!e) e = cudaMemcpy2D(dc, dc_w + dd_w, L.down_col + unit_begin * unit_col, L.dc_stride, dc_w, NR, d2d);
    if (!e) e = cudaMemcpy2D(dc + dc_w, dc_w + dd_w, L.down_col + NU * unit_col + (int64_t)blk_lo * H * 2, L.dc_stride,
                             dd_w, NR, d2d);
    if (!e && s.n_shared) e = cudaMemcpy(g + gu_w * NR, L.gate + L.gu_stride * NR, sh_gu, d2d);
    if (!e && s.n_shared) e = cudaMemcpy(u + gu_w * NR, L.up + L.gu_stride * NR, sh_gu, d2d);
    if (!e && s.n_shared) e = cudaMemcpy(dc + (dc_w + dd_w) * NR, L.down_col + L.dc_stride * NR, sh_dc, d2d);
    if (e) {
        undo();
        return fail(GPEED_ERR_CUDA, "slicing layer %d: %s", layer, cudaGetErrorString(e));
    }
    cudaFree(L.gate); cudaFree(L.up); cudaFree(L.down); cudaFree(L.down_col);
    L.gate = g;
    L.up = u;
    L.down = nullptr;
    L.down_col = dc;
    L.gu_stride = gu_w;
    L.d_stride = 0;
    L.dc_stride = dc_w + dd_w;
    L.u_lo = unit_begin;
    L.u_cnt = unit_count;
    return GPEED_OK;
}

int gpeed_moe_forward(gpeed_ctx* c, int layer, const void* x, int x_dtype, int n, float* y, const int* forced,
                      int* topk_ids, float* topk_w, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (n == 0) return GPEED_OK;
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!x || !y || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
        return fail(GPEED_ERR_INVALID, "x and y must be 16-byte aligned device pointers");
    const Layer& L = it->second;
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, E = s.n_experts, K = s.top_k;
    if (L.e_cnt != E || L.sliced())
        return fail(GPEED_ERR_INVALID, "layer %d holds experts [%d, %d) of %d, units [%d, %d): use the "
                    "expert-parallel entry points", layer, L.e_lo, L.e_lo + L.e_cnt, E, L.u_lo, L.u_lo + L.u_cnt);
    int rc;
    if ((rc = set_device(c))) return rc;
    if ((rc = ensure_scratch(c, n, E, K, H, I))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    auto mark = [&](int i) {
        if (c->prof) cudaEventRecord(c->ev[i], st);
    };
    if (n <= c->fused_max_tokens && c->fused_decode && gp::decode_layer_supported(H, I, E, K, s.n_shared)) {
        // batch 1, and small batches one token at a time: each launch streams
        // only its token's experts, and consecutive launches overlap (PDL)
        gp::DecodeLayerArgs da{};
        if ((rc = fused_args(c, L, x, x_dtype, 1, 0, y, forced, topk_ids, topk_w, st, &da))) return rc;
        // profiling: the one kernel's time goes to the gate/up slot, the other
        // stages read 0
        mark(2);
        const size_t xrow = (size_t)H * (x_dtype == GPEED_DTYPE_BF16 ? 2 : 4);
        for (int t = 0; t < n; ++t) {
            da.x = static_cast<const uint8_t*>(x) + t * xrow;
            da.y = y + (size_t)t * H;
            da.forced = forced ? forced + (size_t)t * K : nullptr;
            da.topk_ids = topk_ids ? topk_ids + (size_t)t * K : nullptr;
            da.topk_w = topk_w ? topk_w + (size_t)t * K : nullptr;
            GP_CUDA(gp::launch_decode_layer(da, c->num_sms, st));
        }
        mark(3);
        if (c->prof) {
            GP_CUDA(cudaEventSynchronize(c->ev[3]));
            float ms = 0.f;
            GP_CUDA(cudaEventElapsedTime(&ms, c->ev[2], c->ev[3]));
            c->prof_ms[2] += ms;
            ++c->prof_calls;
        }
        return GPEED_OK;
    }
    mark(0);

    gp::RouterArgs ra{L.router, x, x_dtype == GPEED_DTYPE_BF16, n, H, E, c->partial.p,
                      c->partial.p + (size_t)n * E, c->partial.n - (size_t)n * E, L.router_split, L.router_nb, c->status};
    GP_CUDA(gp::launch_router(ra, st, false));
    mark(1);
    if (n >= c->tc_min_tokens && s.n_shared && gp::tc_moe_supported(H, I)) {
        // experts on tensor cores: slots of <= 224 rows per expert, fp16 operands
        const int npos = n * K + n;
        if ((rc = c->xp.ensure((size_t)npos * H))) return rc;
        gp::RouteArgs ro{};
        ro.logits = c->partial.p;
        ro.corr = L.corr;
        ro.forced = forced;
        ro.n = n;
        ro.E = E;
        ro.K = K;
        ro.routed_scale = s.routed_scale;
        ro.norm_topk = s.norm_topk;
        ro.nt = gp::tc_moe_slot_tokens();
        ro.with_shared = 1;
        ro.expert_lo = 0;
        ro.expert_hi = E;
        ro.topk_ids = topk_ids ? topk_ids : c->topk_ids.p;
        ro.topk_w = topk_w ? topk_w : c->topk_w.p;
        ro.perm_tok = c->perm.p;
        ro.inv_pos = c->inv_pos.p;
        ro.counts = c->counts.p;
        ro.slots = c->slots.p;
        ro.max_slots = (int)c->slots.n;
        ro.nslots = c->nslots.p;
        ro.status = c->status;
        ro.chunk_counts = c->route_chunks.p;
        ro.chunk_cap = c->route_chunks.n;
        GP_CUDA(gp::launch_route(ro, st, false));
        GP_CUDA(gp::launch_gather_cast(x, x_dtype == GPEED_DTYPE_BF16, c->perm.p, npos, H, c->xp.p, c->status, st));
        mark(2);
        uint16_t* h16 = reinterpret_cast<uint16_t*>(c->h.p);  // npos x I fp16 fits the fp32 h scratch
        gp::TcArgs ga{c->slots.p, c->nslots.p, I / 128, H, I, s.swiglu_limit, h16, c->status};
        GP_CUDA(gp::launch_tc_moe(true, L.gate, L.up, (int64_t)(E + 1) * I, c->xp.p, npos, ga, c->num_sms, st));
        mark(3);
        gp::TcArgs da{c->slots.p, c->nslots.p, H / 128, I, H, 0.f, c->D.p, c->status};
        GP_CUDA(gp::launch_tc_moe(false, L.down, nullptr, (int64_t)(E + 1) * H, h16, npos, da, c->num_sms, st));
        mark(4);
        gp::CombineArgs cb{c->D.p, c->inv_pos.p, ro.topk_w, n, K, H, 1, y, nullptr};
        GP_CUDA(gp::launch_combine(cb, st, false));
        mark(5);
        if (c->prof) {
            GP_CUDA(cudaEventSynchronize(c->ev[5]));
            for (int i = 0; i < 5; ++i) {
                float ms = 0.f;
                GP_CUDA(cudaEventElapsedTime(&ms, c->ev[i], c->ev[i + 1]));
                c->prof_ms[i] += ms;
            }
            ++c->prof_calls;
        }
        return GPEED_OK;
    }

    gp::RouteArgs ro{};
    ro.logits = c->partial.p;
    ro.corr = L.corr;
    ro.forced = forced;
    ro.n = n;
    ro.E = E;
    ro.K = K;
    ro.routed_scale = s.routed_scale;
    ro.norm_topk = s.norm_topk;
    ro.with_shared = s.n_shared;
    ro.expert_lo = 0;
    ro.expert_hi = E;
    ro.topk_ids = topk_ids ? topk_ids : c->topk_ids.p;
    ro.topk_w = topk_w ? topk_w : c->topk_w.p;
    if ((rc = expert_pass(c, L, x, x_dtype == GPEED_DTYPE_BF16, ro, s.n_shared, nullptr, y, st, mark))) return rc;
    mark(5);
    if (c->prof) {
        GP_CUDA(cudaEventSynchronize(c->ev[5]));
        for (int i = 0; i < 5; ++i) {
            float ms = 0.f;
            GP_CUDA(cudaEventElapsedTime(&ms, c->ev[i], c->ev[i + 1]));
            c->prof_ms[i] += ms;
        }
        ++c->prof_calls;
    }
    return GPEED_OK;
}

// ---- expert parallelism (no counterpart in the reference) ----------------

int gpeed_moe_decode_partial(gpeed_ctx* c, int layer, const void* x, int x_dtype, int n, int own_tok, float* y_part,
                             const int* forced, int* topk_ids, float* topk_w, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    const Layer& L = it->second;
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, E = s.n_experts, K = s.top_k;
    if (n < 1 || n > gp::kDecodeMaxTokens || n * K > gp::kDecodeMaxRouted)
        return fail(GPEED_ERR_INVALID, "n_tok %d: 1 .. %d tokens with n_tok * top_k <= %d", n, gp::kDecodeMaxTokens,
                    gp::kDecodeMaxRouted);
    if (own_tok < 0 || own_tok >= n) return fail(GPEED_ERR_INVALID, "own_tok %d not in [0, %d)", own_tok, n);
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!x || !y_part || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y_part) & 15))
        return fail(GPEED_ERR_INVALID, "x and y_part must be 16-byte aligned device pointers");
    if (!gp::decode_layer_supported(H, I, E, K, s.n_shared))
        return fail(GPEED_ERR_UNSUPPORTED, "no persistent decode kernel for hidden %d, inter %d, %d experts, top-%d, "
                    "%d shared", H, I, E, K, s.n_shared);
    if (n == 1 && L.e_cnt != E)
        return fail(GPEED_ERR_INVALID, "one token needs every expert in the layer (use gpeed_moe_forward)");
    int rc;
    if ((rc = set_device(c))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    gp::DecodeLayerArgs da{};
    if ((rc = fused_args(c, L, x, x_dtype, n, own_tok, y_part, forced, topk_ids, topk_w, st, &da))) return rc;
    GP_CUDA(gp::launch_decode_layer(da, c->num_sms, st));
    return GPEED_OK;
}


// ---- expert-parallel decode over peer memory ----
// Block of one rank: [kDecodeMaxTokens][H] tagged token words, then its two
// accumulators [2][H] fp32 (by step parity), its local partial outputs
// [kDecodeMaxTokens][H] fp32, its done counter (u64), its EP step
// generation and its tagged picks [kDecodeMaxTokens][32][2] u64.
namespace {
size_t ep_x_bytes(int H) { return (size_t)gp::kDecodeMaxTokens * H * sizeof(unsigned long long); }
size_t ep_y_off(int H) { return ep_x_bytes(H); }
size_t ep_part_off(int H) { return (ep_y_off(H) + (size_t)2 * H * 4 + 255) & ~(size_t)255; }
size_t ep_done_off(int H) { return (ep_part_off(H) + (size_t)gp::kDecodeMaxTokens * H * 4 + 255) & ~(size_t)255; }
size_t ep_sync_off(int H) { return ep_done_off(H) + 256; }
size_t ep_pk_off(int H) { return ep_sync_off(H) + 256; }
size_t ep_block_bytes(int H) { return ep_pk_off(H) + (size_t)gp::kDecodeMaxTokens * 32 * 16; }
}  // namespace

void ep_release(gpeed_ctx* c) {
    for (int r = 0; r < gp::kDecodeMaxTokens; ++r)
        if (c->ep.peer[r] && c->ep.peer[r] != c->ep.base) cudaIpcCloseMemHandle(c->ep.peer[r]);
    if (c->ep.base) cudaFree(c->ep.base);
    c->ep = gpeed_ctx::Ep{};
}

int gpeed_ep_setup(gpeed_ctx* c, int world, int rank, int hidden, void* handle_out) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if (world < 2 || world > gp::kDecodeMaxTokens || rank < 0 || rank >= world)
        return fail(GPEED_ERR_INVALID, "world %d, rank %d: 2 .. %d ranks", world, rank, gp::kDecodeMaxTokens);
    if (hidden <= 0 || hidden % 8 || !handle_out) return fail(GPEED_ERR_INVALID, "hidden %d (multiple of 8), handle_out required", hidden);
    int rc;
    if ((rc = set_device(c))) return rc;
    ep_release(c);
    void* p = nullptr;
    if (cudaMalloc(&p, ep_block_bytes(hidden)) != cudaSuccess) return fail(GPEED_ERR_CUDA, "cudaMalloc of the exchange block");
    c->ep.base = static_cast<uint8_t*>(p);
    GP_CUDA(cudaMemset(p, 0, ep_block_bytes(hidden)));  // tags, counters and generation start at 0
    GP_CUDA(cudaDeviceSynchronize());
    cudaIpcMemHandle_t h;
    GP_CUDA(cudaIpcGetMemHandle(&h, p));
    static_assert(sizeof(h) == GPEED_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    c->ep.world = world;
    c->ep.rank = rank;
    c->ep.hidden = hidden;
    return GPEED_OK;
}

int gpeed_ep_connect(gpeed_ctx* c, const void* handles) {
    if (!c || !handles) return fail(GPEED_ERR_INVALID, "ctx and handles required");
    if (!c->ep.base) return fail(GPEED_ERR_INVALID, "gpeed_ep_setup first");
    int rc;
    if ((rc = set_device(c))) return rc;
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int r = 0; r < c->ep.world; ++r) {
        if (r == c->ep.rank) {
            c->ep.peer[r] = c->ep.base;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)r * GPEED_IPC_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            ep_release(c);
            return fail(GPEED_ERR_CUDA, "cudaIpcOpenMemHandle of rank %d: %s", r, cudaGetErrorString(e));
        }
        c->ep.peer[r] = static_cast<uint8_t*>(p);
    }
    c->ep.connected = true;
    return GPEED_OK;
}

int gpeed_ep_disconnect(gpeed_ctx* c) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    int rc;
    if ((rc = set_device(c))) return rc;
    for (int r = 0; r < gp::kDecodeMaxTokens; ++r) {
        if (c->ep.peer[r] && c->ep.peer[r] != c->ep.base) GP_CUDA(cudaIpcCloseMemHandle(c->ep.peer[r]));
        c->ep.peer[r] = nullptr;
    }
    c->ep.connected = false;
    return GPEED_OK;
}

int gpeed_moe_decode_ep(gpeed_ctx* c, int layer, const void* x, int x_dtype, float* y, int* topk_ids, float* topk_w,
                        void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if (!c->ep.connected) return fail(GPEED_ERR_INVALID, "gpeed_ep_setup and gpeed_ep_connect first");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    const Layer& L = it->second;
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, E = s.n_experts, K = s.top_k, n = c->ep.world;
    if (H != c->ep.hidden) return fail(GPEED_ERR_INVALID, "hidden %d != the exchange's %d", H, c->ep.hidden);
    if (n * K > gp::kDecodeMaxRouted) return fail(GPEED_ERR_INVALID, "%d ranks x top-%d > %d picks", n, K, gp::kDecodeMaxRouted);
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!x || !y || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
        return fail(GPEED_ERR_INVALID, "x and y must be 16-byte aligned device pointers");
    if (!gp::decode_layer_supported(H, I, E, K, s.n_shared))
        return fail(GPEED_ERR_UNSUPPORTED, "no persistent decode kernel for hidden %d, inter %d, %d experts, top-%d, "
                    "%d shared", H, I, E, K, s.n_shared);
    // The ranks' shares must cover every pick exactly once: rank r holds the
    // r-th of n equal unit slices of every routed expert, or the r-th of n
    // equal expert ranges.  Any other share (a whole layer on every rank, or
    // slices of another world size) would count picks twice or not at all.
    const int NU = I / 32, r = c->ep.rank;
    const bool by_units = L.sliced() && L.e_lo == 0 && L.e_cnt == E && NU % n == 0 && L.u_cnt == NU / n &&
                          L.u_lo == r * L.u_cnt;
    const bool by_experts = !L.sliced() && E % n == 0 && L.e_cnt == E / n && L.e_lo == r * L.e_cnt;
    if (!by_units && !by_experts)
        return fail(GPEED_ERR_INVALID, "layer %d is not rank %d's share of %d (units [%d, %d) of %d, experts [%d, %d) "
                    "of %d)", layer, r, n, L.u_lo, L.u_lo + L.u_cnt, NU, L.e_lo, L.e_lo + L.e_cnt, E);
    int rc;
    if ((rc = set_device(c))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    gp::DecodeLayerArgs da{};
    float* part = reinterpret_cast<float*>(c->ep.base + ep_part_off(H));
    if ((rc = fused_args(c, L, x, x_dtype, n, c->ep.rank, part, nullptr, topk_ids, topk_w, st, &da))) return rc;
    da.ep_out = y;
    da.ep_world = n;
    da.ep_rank = c->ep.rank;
    da.ep_x = reinterpret_cast<unsigned long long*>(c->ep.base);
    for (int r = 0; r < n; ++r) {
        da.ep_x_peer[r] = reinterpret_cast<unsigned long long*>(c->ep.peer[r]);
        da.ep_y[r] = reinterpret_cast<float*>(c->ep.peer[r] + ep_y_off(H));
        da.ep_done[r] = reinterpret_cast<unsigned long long*>(c->ep.peer[r] + ep_done_off(H));
        da.ep_pk_peer[r] = reinterpret_cast<unsigned long long*>(c->ep.peer[r] + ep_pk_off(H));
    }
    da.ep_sync = reinterpret_cast<unsigned*>(c->ep.base + ep_sync_off(H));
    da.ep_pk = reinterpret_cast<unsigned long long*>(c->ep.base + ep_pk_off(H));
    GP_CUDA(gp::launch_decode_layer(da, c->num_sms, st));
    return GPEED_OK;
}

int gpeed_moe_route(gpeed_ctx* c, int layer, const void* x, int x_dtype, int n, const int* forced, int* topk_ids,
                    float* topk_w, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (n == 0) return GPEED_OK;
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!x || !topk_ids || !topk_w || (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(GPEED_ERR_INVALID, "x (16-byte aligned), topk_ids and topk_w are required");
    const Layer& L = it->second;
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, E = s.n_experts, K = s.top_k;
    int rc;
    if ((rc = set_device(c))) return rc;
    if ((rc = ensure_scratch(c, n, E, K, H, I))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    gp::RouterArgs ra{L.router, x, x_dtype == GPEED_DTYPE_BF16, n, H, E, c->partial.p,
                      c->partial.p + (size_t)n * E, c->partial.n - (size_t)n * E, L.router_split, L.router_nb, c->status};
    GP_CUDA(gp::launch_router(ra, st, false));
    gp::RouteArgs ro{};
    ro.logits = c->partial.p;
    ro.corr = L.corr;
    ro.forced = forced;
    ro.n = n;
    ro.E = E;
    ro.K = K;
    ro.routed_scale = s.routed_scale;
    ro.norm_topk = s.norm_topk;
    ro.nt = 1;
    ro.with_shared = 0;
    ro.expert_lo = ro.expert_hi = 0;  // ids and weights only: no expert slots
    ro.topk_ids = topk_ids;
    ro.topk_w = topk_w;
    ro.perm_tok = c->perm.p;
    ro.inv_pos = c->inv_pos.p;
    ro.counts = c->counts.p;
    ro.slots = c->slots.p;
    ro.max_slots = (int)c->slots.n;
    ro.nslots = c->nslots.p;
    ro.status = c->status;
    ro.chunk_counts = c->route_chunks.p;
    ro.chunk_cap = c->route_chunks.n;
    GP_CUDA(gp::launch_route(ro, st, false));
    return GPEED_OK;
}

int gpeed_ep_pack(gpeed_ctx* c, int n_experts, int world, int n, int K, const int* topk_ids, const void* x,
                  int x_dtype, int hidden, void* send_rows, int* send_ids, int* rank_counts, int* slot_of,
                  void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if (world < 1 || n_experts < world || n_experts % world)
        return fail(GPEED_ERR_INVALID, "n_experts %d must split evenly over %d ranks", n_experts, world);
    if (n < 0 || K < 1 || K > 32 || hidden % 256) return fail(GPEED_ERR_INVALID, "bad n/K/hidden");
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (!rank_counts) return fail(GPEED_ERR_INVALID, "rank_counts is NULL");
    if (n && (!topk_ids || !x || !send_rows || !send_ids || !slot_of || (reinterpret_cast<uintptr_t>(x) & 15) ||
              (reinterpret_cast<uintptr_t>(send_rows) & 15)))
        return fail(GPEED_ERR_INVALID, "NULL or unaligned buffer");
    int rc;
    if ((rc = set_device(c))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (n == 0) {
        GP_CUDA(cudaMemsetAsync(rank_counts, 0, sizeof(int) * world, st));
        return GPEED_OK;
    }
    if ((rc = ensure_scratch(c, n, n_experts, K, hidden, 256))) return rc;
    // stable bucket sort of the assignments by expert = by destination rank
    gp::RouteArgs ro{};
    ro.topk_ready = 1;
    ro.n = n;
    ro.E = n_experts;
    ro.K = K;
    ro.nt = 1;
    ro.expert_lo = ro.expert_hi = 0;
    ro.topk_ids = const_cast<int*>(topk_ids);
    ro.topk_w = c->topk_w.p;
    ro.perm_tok = c->perm.p;
    ro.inv_pos = slot_of;
    ro.counts = c->counts.p;
    ro.slots = c->slots.p;
    ro.max_slots = (int)c->slots.n;
    ro.nslots = c->nslots.p;
    ro.status = c->status;
    ro.chunk_counts = c->route_chunks.p;
    ro.chunk_cap = c->route_chunks.n;
    GP_CUDA(gp::launch_route(ro, st, false));
    GP_CUDA(gp::launch_ep_pack(x, x_dtype == GPEED_DTYPE_BF16, hidden, n, K, topk_ids, slot_of, c->counts.p,
                               n_experts, world, n_experts / world, send_rows, send_ids, rank_counts, st));
    return GPEED_OK;
}

int gpeed_moe_experts(gpeed_ctx* c, int layer, const void* rows, int rows_dtype, int m, const int* expert_ids,
                      float* out, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    auto it = c->layers.find(layer);
    if (it == c->layers.end()) return fail(GPEED_ERR_INVALID, "layer %d not loaded", layer);
    if (m < 0) return fail(GPEED_ERR_INVALID, "m < 0");
    if (m == 0) return GPEED_OK;
    if (rows_dtype != GPEED_DTYPE_BF16 && rows_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "rows_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", rows_dtype);
    if (!rows || !expert_ids || !out || (reinterpret_cast<uintptr_t>(rows) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return fail(GPEED_ERR_INVALID, "rows and out must be 16-byte aligned device pointers; expert_ids required");
    const Layer& L = it->second;
    if (L.sliced()) return fail(GPEED_ERR_INVALID, "layer %d holds a slice of each expert's units", layer);
    const gpeed_moe_shape& s = L.shape;
    const int H = s.hidden, I = s.inter, El = L.e_cnt + s.n_shared;
    int rc;
    if ((rc = set_device(c))) return rc;
    if ((rc = ensure_scratch(c, m, El, 1, H, I))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    GP_CUDA(gp::launch_local_ids(expert_ids, m, s.n_experts, L.e_lo, L.e_cnt, c->topk_ids.p, c->topk_w.p, c->status,
                                 st));
    // one assignment per row, weight 1, no shared add: out = down(SwiGLU(gate x, up x))
    gp::RouteArgs ro{};
    ro.topk_ready = 1;
    ro.n = m;
    ro.E = El;
    ro.K = 1;
    ro.with_shared = 0;
    ro.expert_lo = 0;
    ro.expert_hi = El;
    ro.topk_ids = c->topk_ids.p;
    ro.topk_w = c->topk_w.p;
    auto nomark = [](int) {};
    return expert_pass(c, L, rows, rows_dtype == GPEED_DTYPE_BF16, ro, 0, nullptr, out, st, nomark);
}

int gpeed_dense_mlp_forward(gpeed_ctx* c, int gate, int up, int down, float swiglu_limit, const void* X, int x_dtype,
                            int n, float* Y, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    const int nt = (int)c->tensors.size();
    if (gate < 0 || gate >= nt || up < 0 || up >= nt || down < 0 || down >= nt)
        return fail(GPEED_ERR_INVALID, "bad tensor handle");
    const Tensor &G = c->tensors[gate], &U = c->tensors[up], &D = c->tensors[down];
    const int H = G.in_dim;
    const int64_t I = G.rows;
    if (U.in_dim != H || U.rows != I || D.in_dim != I || D.rows != H)
        return fail(GPEED_ERR_INVALID, "gate/up must be inter x hidden and down hidden x inter (got %lld x %d, %lld x %d, "
                    "%lld x %d)", (long long)G.rows, G.in_dim, (long long)U.rows, U.in_dim, (long long)D.rows, D.in_dim);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (n && (!X || !Y || (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(Y) & 15)))
        return fail(GPEED_ERR_INVALID, "X and Y must be 16-byte aligned device pointers");
    Layer L;
    L.shape = gpeed_moe_shape{H, (int)I, 1, 1, 0, 1.f, 0, swiglu_limit};
    int rc;
    if ((rc = check_shape(&L.shape))) return rc;
    if (n == 0) return GPEED_OK;
    L.e_cnt = 1;
    L.gate = G.packed;
    L.up = U.packed;
    L.down = D.packed;
    L.gu_stride = gp::repacked_bytes(I, H);
    L.d_stride = gp::repacked_bytes(H, (int)I);
    if ((rc = set_device(c))) return rc;
    if ((rc = ensure_scratch(c, n, 1, 1, H, (int)I))) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (n < c->tc_min_tokens || !gp::tc_moe_supported(H, (int)I)) {
        // GEMV path with nothing to route: slots over the tokens in order, gate/up + SwiGLU reading x
        // rows directly, down writing Y rows directly (no permutation, no weighted combine)
        const int nt = nt_for(n);
        Geo ggu, gd;
        if ((rc = pick_geo(H, 2, nt, (int)I, &ggu))) return rc;
        if ((rc = pick_geo((int)I, 1, nt, H, &gd))) return rc;
        if (I % ggu.tile_rows || H % gd.tile_rows) return fail(GPEED_ERR_UNSUPPORTED, "row tiling of the dense MLP");
        make_slots_kernel<<<1, 256, 0, st>>>(c->slots.p, c->nslots.p, n, nt);
        GP_CUDA(cudaGetLastError());
        gp::GemvArgs g{};
        g.w0 = G.packed;
        g.w1 = U.packed;
        g.expert_stride = L.gu_stride;
        g.in_dim = H;
        g.rows = (int)I;
        g.tile_rows = ggu.tile_rows;
        g.nwarps = ggu.nwarps;
        g.stages = ggu.stages;
        g.slots = c->slots.p;
        g.nslots = c->nslots.p;
        g.perm_tok = nullptr;
        g.x = X;
        g.x_bf16 = x_dtype == GPEED_DTYPE_BF16;
        g.out = c->h.p;
        g.limit = swiglu_limit;
        g.tables = c->tables;
        g.status = c->status;
        GP_CUDA(gp::launch_gemv(g, nt, true, ggu.passes, ggu.rpw, c->num_sms, st, true));
        gp::GemvArgs d{};
        d.w0 = D.packed;
        d.expert_stride = L.d_stride;
        d.in_dim = (int)I;
        d.rows = H;
        d.tile_rows = gd.tile_rows;
        d.nwarps = gd.nwarps;
        d.stages = gd.stages;
        d.slots = c->slots.p;
        d.nslots = c->nslots.p;
        d.perm_tok = nullptr;
        d.x = c->h.p;
        d.x_bf16 = 0;
        d.out = Y;
        d.tables = c->tables;
        d.status = c->status;
        GP_CUDA(gp::launch_gemv(d, nt, false, gd.passes, gd.rpw, c->num_sms, st, true));
        return GPEED_OK;
    }
    fill_unit_kernel<<<std::min((n + 255) / 256, 148), 256, 0, st>>>(c->topk_ids.p, c->topk_w.p, n);
    GP_CUDA(cudaGetLastError());
    gp::RouteArgs ro{};
    ro.topk_ready = 1;
    ro.n = n;
    ro.E = 1;
    ro.K = 1;
    ro.with_shared = 0;
    ro.expert_lo = 0;
    ro.expert_hi = 1;
    ro.topk_ids = c->topk_ids.p;
    ro.topk_w = c->topk_w.p;
    auto nomark = [](int) {};
    return expert_pass(c, L, X, x_dtype == GPEED_DTYPE_BF16, ro, 0, nullptr, Y, st, nomark);
}

int gpeed_mhc_pre(gpeed_ctx* c, const float* streams, int n, int hidden, const gpeed_mhc_params* p, const float* fn,
                  const float* base, const float* scale, const float* norm_w, void* x_out, int x_dtype, float* post,
                  float* comb, void* stream) {
    if (!c || !p) return fail(GPEED_ERR_INVALID, "ctx or params is NULL");
    if (p->hc_mult < 1 || p->hc_mult > 4) return fail(GPEED_ERR_UNSUPPORTED, "hc_mult %d not in [1, 4]", p->hc_mult);
    if (p->sinkhorn_iters < 1) return fail(GPEED_ERR_INVALID, "sinkhorn_iters must be >= 1");
    if (hidden <= 0 || hidden % 4) return fail(GPEED_ERR_INVALID, "hidden %d must be a positive multiple of 4", hidden);
    if (x_dtype != GPEED_DTYPE_BF16 && x_dtype != GPEED_DTYPE_F32)
        return fail(GPEED_ERR_UNSUPPORTED, "x_dtype %d: use GPEED_DTYPE_BF16 or GPEED_DTYPE_F32", x_dtype);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (n == 0) return GPEED_OK;
    if (!streams || !fn || !base || !scale || !norm_w || !x_out || !post || !comb ||
        (reinterpret_cast<uintptr_t>(streams) & 15) || (reinterpret_cast<uintptr_t>(fn) & 15))
        return fail(GPEED_ERR_INVALID, "NULL buffer, or streams / fn not 16-byte aligned");
    int rc;
    if ((rc = set_device(c))) return rc;
    if ((rc = c->mhc_partial.ensure((size_t)gp::mhc_partial_floats(n, p->hc_mult, hidden)))) return rc;
    gp::MhcArgs a{p->hc_mult, hidden, p->sinkhorn_iters, p->hc_eps, p->rms_eps, fn, base, scale, norm_w, x_out,
                  x_dtype == GPEED_DTYPE_BF16, post, comb};
    GP_CUDA(gp::launch_mhc_pre(streams, n, a, c->mhc_partial.p, (cudaStream_t)stream));
    return GPEED_OK;
}

int gpeed_mhc_post(gpeed_ctx* c, const float* streams_in, const float* mlp_out, const float* post, const float* comb,
                   int n, int hidden, int hc_mult, float* streams_out, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if (hc_mult < 1 || hc_mult > 4) return fail(GPEED_ERR_UNSUPPORTED, "hc_mult %d not in [1, 4]", hc_mult);
    if (hidden <= 0 || hidden % 4) return fail(GPEED_ERR_INVALID, "hidden %d must be a positive multiple of 4", hidden);
    if (n < 0) return fail(GPEED_ERR_INVALID, "n_tok < 0");
    if (n == 0) return GPEED_OK;
    if (!streams_in || !mlp_out || !post || !comb || !streams_out ||
        ((reinterpret_cast<uintptr_t>(streams_in) | reinterpret_cast<uintptr_t>(mlp_out) |
          reinterpret_cast<uintptr_t>(streams_out)) & 15))
        return fail(GPEED_ERR_INVALID, "NULL buffer, or streams / mlp_out not 16-byte aligned");
    int rc;
    if ((rc = set_device(c))) return rc;
    GP_CUDA(gp::launch_mhc_post(streams_in, mlp_out, post, comb, n, hc_mult, hidden, streams_out, (cudaStream_t)stream));
    return GPEED_OK;
}

int gpeed_moe_combine(gpeed_ctx* c, int n, int K, int hidden, const float* d_rows, const int* slot_of,
                      const float* topk_w, const float* d_shared, float* y, void* stream) {
    if (!c) return fail(GPEED_ERR_INVALID, "ctx is NULL");
    if (n < 0 || K < 1 || K > 32 || hidden % 4) return fail(GPEED_ERR_INVALID, "bad n/K/hidden");
    if (n == 0) return GPEED_OK;
    if (!d_rows || !slot_of || !topk_w || !y || (reinterpret_cast<uintptr_t>(d_rows) & 15) ||
        (reinterpret_cast<uintptr_t>(y) & 15) || (d_shared && (reinterpret_cast<uintptr_t>(d_shared) & 15)))
        return fail(GPEED_ERR_INVALID, "NULL or unaligned buffer");
    int rc;
    if ((rc = set_device(c))) return rc;
    gp::CombineArgs cb{d_rows, slot_of, topk_w, n, K, hidden, d_shared ? 1 : 0, y, d_shared};
    GP_CUDA(gp::launch_combine(cb, (cudaStream_t)stream, false));
    return GPEED_OK;
}

}  // extern "C"

// ---- allocation-free variant of gpeed_matmul_quant -------------------------
// Some callers cannot call cudaMalloc once they are serving: an engine that
// owns the GPU's memory through its own allocator or memory pool, a process
// held to a fixed device-memory budget decided at start-up, or a host whose
// allocations must not fail or stall in the middle of a step.  For them the
// GEMV's work list and its output staging live in this file-scope device array
// instead of context scratch.  Every GPU that loads the library holds the
// array (GPEED_NOALLOC_SCRATCH_BYTES) until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GPEED_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mu;
constexpr int kMaxDevices = 64;
unsigned char* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device`, which must be current: in
// host code the array's name is only a host-side stand-in, so the address is
// looked up with cudaGetSymbolAddress, once per device, on that device's first
// call.
int noalloc_scratch(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device < 0 || device >= kMaxDevices) return fail(GPEED_ERR_INVALID, "device %d out of range", device);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(GPEED_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        g_noalloc_ptr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[device];
    return GPEED_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

extern "C" {

int gpeed_matmul_quant_noalloc(gpeed_ctx* c, int handle, uint64_t row0, int in_dim, int out_dim, const float* X,
                               int n_tok, float* Y, void* stream) {
    MatmulPlan p;
    int rc;
    if ((rc = plan_matmul(c, handle, row0, in_dim, out_dim, X, n_tok, Y, &p)) || p.empty) return rc;
    // scratch layout: [slots][nslots][staged output]; the slot kernel rewrites
    // the work list on every call, so nothing left by a previous call is read
    const size_t off_n = align256((size_t)p.ns * sizeof(gp::SlotDesc));
    const size_t off_y = off_n + 256;
    const size_t need = off_y + p.staged_floats() * sizeof(float);
    if (need > GPEED_NOALLOC_SCRATCH_BYTES)
        return fail(GPEED_ERR_INVALID, "matmul_quant_noalloc: %zu bytes of scratch needed, the static limit is %u "
                    "(n_tok * ceil(out_dim + row0 %% 8, %d) * 4 bytes of staging when row0 %% 8 != 0 or out_dim %% %d "
                    "!= 0, plus the work list)", need, GPEED_NOALLOC_SCRATCH_BYTES, p.g.tile_rows, p.g.tile_rows);
    unsigned char* scratch = nullptr;
    if ((rc = noalloc_scratch(c->device, &scratch))) return rc;
    MatmulScratch sc;
    sc.slots = reinterpret_cast<gp::SlotDesc*>(scratch);
    sc.nslots = reinterpret_cast<int*>(scratch + off_n);
    sc.staged = p.direct ? nullptr : reinterpret_cast<float*>(scratch + off_y);
    return run_matmul(c, p, X, Y, sc, (cudaStream_t)stream);
}

}  // extern "C"
