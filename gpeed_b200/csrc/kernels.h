// Host-visible kernel launch interfaces (internal to libgpeed_moe.so).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace gp {

// Raises `kern`'s opt-in dynamic shared-memory limit to `bytes` on the current
// device.  The attribute belongs to each device's context, so it is recorded
// per device (bit d of `done`, one word per kernel instantiation): a process
// that drives several GPUs sets it on each of them.  Two host threads racing
// here both set the same value, which is harmless.  Devices past 63 set it on
// every launch.
template <typename F>
inline cudaError_t raise_smem_limit(F kern, int bytes, std::atomic<unsigned long long>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// One unit of expert work: `ntok` consecutive assignments starting at `begin`
// (positions in the expert-sorted assignment list) that all use `expert`.
struct SlotDesc {
    int expert;
    int begin;
    int ntok;
    int pad;
};

// Repacked IQ3_XXS matrix layout ("row groups"): rows are grouped by 8; each
// group of 8 rows x nblk blocks (784*nblk bytes, a multiple of 16) stores
//   [qs  : 8 rows x nblk x 64 B][aux : 8 rows x nblk x 32 B][d : 8 rows x nblk x 2 B]
// i.e. the same 98 bytes per block, regrouped so every lane load is aligned and
// a warp's loads are bank-conflict free.  Lossless; see repack kernels.
inline int64_t repacked_bytes(int64_t rows, int in_dim) {
    return ((rows + 7) / 8) * 784 * (int64_t)(in_dim / 256);
}

struct GemvArgs {
    const uint8_t* w0;         // repacked matrix (gate, or the single matrix)
    const uint8_t* w1;         // repacked up matrix (gate/up mode) or nullptr
    int64_t expert_stride;     // bytes between experts in w0 / w1
    int in_dim;                // K (multiple of 256)
    int rows;                  // output rows per expert (a multiple of tile_rows)
    int tile_rows;             // rows per pipeline stage per matrix (multiple of 8)
    int nwarps;                // consumer warps; 32 * nwarps is a multiple of in_dim / 32
    int stages;
    const SlotDesc* slots;
    const int* nslots;         // device-resident slot count
    const int* perm_tok;       // assignment -> x row; nullptr: the assignment index is the x row
    const void* x;             // activations: fp32 or bf16 rows of in_dim
    int x_bf16;
    float* out;                // [assignment][rows] fp32
    float limit;               // SwiGLU clamp (gate/up mode)
    const uint8_t* tables;     // 64 KB decode-table image in global memory
    uint32_t* status;          // device status word (0 = ok)
};

// Launches the fused-decode GEMV.  nt: max tokens per slot (1, 2, 4, 8);
// gateup: w1 present, SwiGLU epilogue; passes / rows_per_warp describe the
// work mapping (see gemv.cu) and must name an instantiated variant.
bool gemv_variant_exists(int nt, bool gateup, int passes, int rows_per_warp);
int gemv_max_warps(int nt, bool gateup);
cudaError_t launch_gemv(const GemvArgs& a, int nt, bool gateup, int passes, int rows_per_warp, int grid,
                        cudaStream_t st, bool pdl);
size_t gemv_smem_bytes(const GemvArgs& a, int nt, bool gateup);

// Builds the 64 KB decode-table image (codebook + sign selectors) in global memory.
cudaError_t build_tables(uint8_t* dst, cudaStream_t st);

// Raw GGUF IQ3_XXS rows -> repacked row groups (and back, for verification).
cudaError_t launch_repack(const uint8_t* raw, uint8_t* packed, int64_t rows, int in_dim, cudaStream_t st);
cudaError_t launch_unpack(const uint8_t* packed, uint8_t* raw, int64_t rows, int in_dim, cudaStream_t st);
// Column-slab layout of a down projection (rows = H outputs, in_dim = I inputs):
// per matrix, for each 32-input unit u: [qs rows x 8 B][aux rows x 4 B], then
// for each 256-input block b: [d rows x 2 B].  The same 98 bytes per 256
// weights as GGUF; a unit's slab of every row is contiguous, so one work item
// of the persistent decode kernel streams the down columns of its 32 h values
// in whole runs.  n_mat matrices of raw row-major blocks, stacked.
cudaError_t launch_repack_cols(const uint8_t* raw, uint8_t* cols, int64_t n_mat, int rows, int in_dim,
                               cudaStream_t st);

// Bit-exact IQ3_XXS -> fp32 (raw GGUF blocks).
cudaError_t launch_dequantize(const uint8_t* raw, float* dst, int64_t nblocks, cudaStream_t st);

// Synthetic IQ3_XXS blocks (counter-based generator, synth.h).
cudaError_t launch_synth(uint8_t* dst, uint64_t seed, uint64_t stream, uint64_t block0, int64_t nblocks,
                         cudaStream_t st);

// Router: logits [n][E] = X[n][H] . W[E][H] (fp32).
struct RouterArgs {
    const float* w;       // [E][H] fp32
    const void* x;        // [n][H]
    int x_bf16;
    int n, H, E;
    float* logits;        // [n][E]
    // Large batches split K across CTAs: partial sums [split][n][E] go here and
    // are added in split order.  nullptr (or too small): no split.
    float* split_scratch;
    size_t split_floats;
    // bf16 x and these split weights (router_tc.cu): tensor-core logits.
    const uint16_t* wsplit;  // [hi; lo; lo2; 0] bf16 rows, 2 * wsplit_nb rows of H, or nullptr
    int wsplit_nb;
    uint32_t* status;        // device status word (the tensor-core kernel's wait timeouts)
};
cudaError_t launch_router(const RouterArgs& a, cudaStream_t st, bool pdl);
// Largest K split the router may use for n tokens (scratch = splits * n * E floats when > 1).
int router_splits(int n, int H, int E);
// Tensor-core router (router_tc.cu): rows per MMA half for E experts (0: unsupported),
// K splits for n tokens, the load-time weight split, and the launch.
int router_tc_nb(int E, int H);
int router_tc_splits(int n, int H);
cudaError_t launch_router_split(const float* R, int E, int H, int nb, uint16_t* out, cudaStream_t st);
cudaError_t launch_router_tc(const RouterArgs& a, int S, float* out, cudaStream_t st, bool pdl);

// Top-k, histogram, stable expert-major permutation and slot list.
struct RouteArgs {
    const float* logits;   // [n][E]
    int topk_ready;        // top-k already in topk_ids / topk_w (large batches)
    const float* corr;     // [E] or nullptr
    const int* forced;     // [n][K] or nullptr
    int n, E, K;
    float routed_scale;
    int norm_topk;
    int nt;                // tokens per slot
    int with_shared;       // append shared-expert assignments/slots (expert id E)
    int expert_lo, expert_hi;  // experts owned here (EP); others are not given slots
    int* topk_ids;         // [n][K]
    float* topk_w;         // [n][K]
    int* perm_tok;         // [n*K + n]: assignment -> token
    int* inv_pos;          // [n][K]: (t,k) -> assignment position
    int* counts;           // [E]
    SlotDesc* slots;       // capacity max_slots
    int max_slots;
    int* nslots;
    uint32_t* status;
    // large batches (see route_chunked_floats): per-chunk expert counts, or nullptr
    int* chunk_counts;
    size_t chunk_cap;
};
cudaError_t launch_route(const RouteArgs& a, cudaStream_t st, bool pdl);
// Ints of RouteArgs::chunk_counts a batch of n tokens x K picks needs (0: not chunked).
size_t route_chunk_ints(int n, int K, int E);
size_t route_smem_bytes(int n, int E, int K);

// Y[t] = sum_k w[t][k] * D[inv_pos[t][k]] (+ D[n*K + t] when with_shared).
struct CombineArgs {
    const float* D;
    const int* inv_pos;
    const float* topk_w;
    int n, K, H, with_shared;
    float* y;
    const float* D_shared;  // shared-expert rows [n][H]; nullptr: they follow the routed rows in D
};
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st, bool pdl);

// One MoE layer at batch 1 in one persistent kernel, one CTA per SM (decode_layer.cu).
constexpr int kSyncGen = 0;                     // launch generation (tags exchanged logits and picks)
constexpr int kSyncEnd = 1;                     // CTAs finished
constexpr int kDecodeMaxTokens = 8;             // tokens per launch of the persistent kernel
constexpr int kDecodeMaxRouted = 64;            // routed (token, expert) slots per launch
constexpr int kDecodeSyncWords = 64;
struct DecodeLayerArgs {
    const float* router;       // [E][H] fp32
    const float* corr;         // [E] or nullptr
    const uint8_t* gate;       // repacked row groups, routed experts held then the shared expert
    const uint8_t* up;
    const uint8_t* down_col;   // the down projections in the column-slab layout (launch_repack_cols)
    int64_t gu_stride, dc_stride;  // bytes per expert
    int H, I, E, K;
    float routed_scale;
    int norm_topk;
    float limit;
    int with_shared;
    const void* x;             // [n_tok][H] bf16 or fp32
    int x_bf16;
    float* y;                  // [n_tok][H]: the layer output (all experts held), else this range's part
    const int* forced;         // [n_tok][K] or nullptr
    int* topk_ids;             // [n_tok][K] or nullptr
    float* topk_w;             // [n_tok][K] or nullptr
    // Tokens and experts of one launch.  One token with every expert is the
    // batch-1 layer (Model::moe_forward).  Several tokens with an expert range
    // is one rank's share of an expert-parallel decode step: the (token, k)
    // picks whose expert lies in [e_lo, e_lo + e_cnt) plus the shared expert
    // of token own_tok, y[t] = that part of token t's output (zero rows for
    // tokens with nothing here); the ranks' parts sum to the layer output.
    int n_tok;                 // 1 .. kDecodeMaxTokens
    int e_lo, e_cnt;           // routed experts held (gate/up/down index e - e_lo; the shared expert at e_cnt)
    int own_tok;               // token whose shared expert runs in this launch (the whole expert)
    int u_lo, u_cnt;           // units of 32 rows of each routed expert that the layer holds and this launch
                               // runs (0, I/32: whole experts; a slice when each rank holds a slice of every
                               // routed expert: the shared expert, after them, stays whole)
    unsigned long long* logits;  // [decode_layer_logit_words(E)] router logits tagged with the launch generation
    unsigned long long* hx;      // [decode_layer_h_words(I)] h of every (slot, unit), tagged: rows of routed slot s
                                 // at s * I, the shared slot's at kDecodeMaxRouted * I
    unsigned* sync;            // [kDecodeSyncWords] launch generation and finished-CTA count
    const uint8_t* tables;
    uint32_t* status;
    int stages;
    int cooperative;           // 1: cooperative launch instead of programmatic dependent launch
    uint32_t spin_limit;       // polls before any wait gives up (sets a GP_DEV_TIMEOUT_* bit)
    int withhold_logit;        // test hook: the router logit of this expert is never published (-1: none)
    // Expert-parallel decode over peer memory (ep_world > 1; no collective
    // library): n_tok = ep_world tokens, token t owned by rank t.  Each rank
    // publishes its own token (x, [1][H]) into every rank's ep_x as words
    // tagged with the EP step generation g + 1, routes its own token and
    // publishes the picks into every rank's ep_pk the same way, reads the
    // other ranks' picks from its own ep_pk, sums its share of every token
    // into y ([n_tok][H], local), and at the end adds y[t] into owner t's
    // accumulator ep_y[t] + (g & 1) * H over NVLink, signals every owner
    // (ep_done[t]), waits for the other ranks' signals, copies its own
    // accumulator to ep_out ([1][H]) and zeroes it for step g + 2 (the next
    // signal orders that before any rank's adds there).
    int ep_world;
    int ep_rank;
    unsigned long long* ep_x;                         // this rank's [kDecodeMaxTokens][H] tagged words
    unsigned long long* ep_x_peer[kDecodeMaxTokens];  // every rank's ep_x (this rank's included)
    unsigned long long* ep_pk;                        // this rank's [kDecodeMaxTokens][32][2] tagged picks (id, weight)
    unsigned long long* ep_pk_peer[kDecodeMaxTokens];  // every rank's ep_pk
    float* ep_y[kDecodeMaxTokens];                    // every rank's accumulators [2][H] (by step parity)
    unsigned long long* ep_done[kDecodeMaxTokens];    // every rank's done counter
    unsigned* ep_sync;                                // this rank's EP step generation
    float* ep_out;                                    // this rank's token's output [1][H]
};
// Tensor-core experts for large batches (tc_moe.cu).
struct TcArgs {
    const SlotDesc* slots;  // expert slots of <= 256 rows (expert-sorted positions)
    const int* nslots;
    int mt;                 // 128-row tiles per expert matrix (nout / 128)
    int kin, nout;          // inputs per row, rows per expert
    float limit;            // SwiGLU clamp (gate/up pass)
    void* out;              // gate/up: fp16 h [position][nout]; down: fp32 D [position][nout]
    uint32_t* status;
};
// Tokens per expert slot of the tensor-core path (the MMA N bound).
int tc_moe_slot_tokens();
bool tc_moe_supported(int H, int I);
// Token rows to fp16 in expert-sorted order; a value past the fp16 range sets
// GP_DEV_FP16_RANGE in *status.
cudaError_t launch_gather_cast(const void* x, int x_bf16, const int* perm, int npos, int H, uint16_t* xp,
                               uint32_t* status, cudaStream_t st);
cudaError_t launch_tc_moe(bool gu, const uint8_t* w0, const uint8_t* w1, int64_t weight_rows, const uint16_t* b,
                          int npos, const TcArgs& args, int grid, cudaStream_t st);

// Expert parallelism helpers (ep.cu).
// global expert ids -> this layer's local expert index (routed e -> e - lo,
// the shared expert E -> cnt); ids outside [lo, lo+cnt) and != E set BAD_EXPERT.
cudaError_t launch_local_ids(const int* ids, int m, int E, int lo, int cnt, int* local, float* ones,
                             uint32_t* status, cudaStream_t st);
// send_rows[pos[i]] = x[i / K] for every assignment i, send_ids[pos[i]] = ids[i];
// rank_counts[r] = assignments whose expert lies in [r*epr, (r+1)*epr).
cudaError_t launch_ep_pack(const void* x, int x_bf16, int H, int n, int K, const int* ids, const int* pos,
                           const int* counts, int E, int world, int epr, void* send_rows, int* send_ids,
                           int* rank_counts, cudaStream_t st);

// Counter words of the persistent kernel: the generation counts launches, the
// others are zero between launches; the host clears all of them (and the
// tagged buffers) after a launch that reported an error.
// Words of DecodeLayerArgs::logits, one word per 256-byte line: per token, 8
// replicas of E tagged logits (every CTA reads every token's).
inline size_t decode_layer_logit_words(int E) { return (size_t)kDecodeMaxTokens * 8 * E * 32; }
// Words of DecodeLayerArgs::hx: one tagged h value per row of every slot's expert
// (routed slots, then the shared slot).
inline size_t decode_layer_h_words(int I) { return (size_t)(kDecodeMaxRouted + 1) * I; }
// Whether the persistent decode kernel runs a slice of u_cnt of each expert's inter / 32 units.
bool decode_layer_slice_supported(int I, int u_cnt);
bool decode_layer_supported(int H, int I, int E, int K, int with_shared);
// Dynamic shared memory of a launch: `stages` pipeline stages, n_tok tokens.
size_t decode_layer_smem(int H, int I, int stages, int n_tok);
cudaError_t launch_decode_layer(const DecodeLayerArgs& a, int grid, cudaStream_t st);

// ---- codecs.cu: the other GGUF codecs (quant.cpp:130-573), bit-exact ----
// values per block of a ggml type the reference decodes (1 for F32/F16/BF16), 0 if it decodes none
int codec_block_values(int dtype);
// dst[0, n) fp32 from src (device, GGUF bytes of `dtype`); n a whole number of blocks
cudaError_t launch_codec_dequantize(int dtype, const void* src, float* dst, int64_t n, cudaStream_t st);

// ---- mhc.cu: mHC residual mixing + RMSNorm around the MoE layer ----------
struct MhcArgs {
    int N, H;                 // hc_mult streams of H
    int iters;                // Sinkhorn iterations (hc_sinkhorn_iters)
    float hc_eps, rms_eps;
    const float* fn;          // [(2+N)N][N*H]
    const float* base;        // [(2+N)N]
    const float* scale;       // [3]
    const float* norm_w;      // [H] (ffn_norm)
    void* x_out;              // [n][H] fp32 or bf16
    int x_bf16;
    float* post_out;          // [n][N]
    float* comb_out;          // [n][N][N]
};
int mhc_partial_floats(int n, int N, int H);
cudaError_t launch_mhc_pre(const float* streams, int n, const MhcArgs& a, float* partial, cudaStream_t st);
cudaError_t launch_mhc_post(const float* in, const float* mlp, const float* post, const float* comb, int n, int N,
                            int H, float* out, cudaStream_t st);

}  // namespace gp
