/* gpeed_moe.h - C ABI of libgpeed_moe.so, the B200 (sm_100a) IQ3_XXS
 * routed-expert MoE path.
 *
 * The entry points replace, one for one, the reference engine's expert-op
 * interface (paths inside the reference project):
 *
 *   gpeed_iq3xxs_dequantize  <- glm5::dequantize / dequantize_row for IQ3_XXS
 *                               (cpp/core/include/glm5/quant.h:17-22,
 *                                cpp/core/src/quant.cpp:521-573)
 *   gpeed_tensor_upload      <- WeightStore's resident payload for one tensor
 *                               (cpp/core/include/glm5/weights.h:55-60,67-73;
 *                                weights.cpp:62-84 payload / pin_nonexpert)
 *   gpeed_matvec_quant       <- WeightStore::matvec_quant (weights.h:38-41,
 *                               weights.cpp:167-203)
 *   gpeed_matmul_quant       <- WeightStore::matmul_quant (weights.h:43-48,
 *                               weights.cpp:86-165)
 *   gpeed_moe_load_layer     <- the per-layer expert tensors Model::moe_forward
 *                               reads by name (model.cpp:700-755)
 *   gpeed_moe_forward        <- Model::moe_forward (model.cpp:692-756) for
 *                               n_tok == 1 and Model::moe_batch
 *                               (model_batch.cpp:165-281) for n_tok > 1
 *   gpeed_ep_*               <- no counterpart: the reference has no
 *                               multi-GPU path; expert parallelism over NCCL.
 *
 * Conventions: every function returns 0 (GPEED_OK) or a GPEED_ERR_* code and
 * leaves a message for gpeed_last_error() (per calling thread); the C++ shim
 * in gpeed_b200/csrc/weight_store.hpp turns non-zero codes into
 * std::runtime_error like the reference.  Pointers named *_dev are device
 * pointers; `stream` is a cudaStream_t (NULL = legacy default stream).  All
 * compute calls are asynchronous on `stream`; device-side faults that the
 * kernels detect (bounded waits that gave up, expert ids out of range) are
 * reported by gpeed_ctx_check().  Buffers must be 16-byte aligned.
 */
#ifndef GPEED_MOE_H
#define GPEED_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPEED_OK 0
#define GPEED_ERR_INVALID 1     /* bad argument (shape, alignment, handle) */
#define GPEED_ERR_CUDA 2        /* CUDA runtime error */
#define GPEED_ERR_DEVICE 3      /* a kernel reported a device-side error */
#define GPEED_ERR_UNSUPPORTED 4 /* shape or dtype this build does not handle */
#define GPEED_ERR_NCCL 5

#define GPEED_DTYPE_F32 0       /* ggml type ids (reference common.h:10-44) */
#define GPEED_DTYPE_IQ3_XXS 18
#define GPEED_DTYPE_BF16 30

#if defined(__GNUC__)
#define GPEED_API __attribute__((visibility("default")))
#else
#define GPEED_API
#endif

typedef struct gpeed_ctx gpeed_ctx;

/* MoE shape and routing constants (reference model_config.h:57-70, read from
 * GGUF metadata at model_config.cpp:406-421). */
typedef struct gpeed_moe_shape {
    int hidden;          /* H, multiple of 512 */
    int inter;           /* moe_inter I, multiple of 512 */
    int n_experts;       /* E routed experts (<= 512) */
    int top_k;           /* K (<= 32) */
    int n_shared;        /* 0 or 1 shared expert */
    float routed_scale;  /* 2.5 */
    int norm_topk;       /* 1: renormalise top-k weights */
    float swiglu_limit;  /* 10.0: silu(min(g, L)) * clamp(u, -L, L) */
} gpeed_moe_shape;

GPEED_API const char* gpeed_last_error(void);
GPEED_API int gpeed_version(void);

/* Context bound to one CUDA device; owns uploaded weights and scratch. */
GPEED_API int gpeed_ctx_create(int device, gpeed_ctx** out);
GPEED_API int gpeed_ctx_destroy(gpeed_ctx* ctx);
/* Synchronises `stream` and reports (then clears) device-side error flags. */
GPEED_API int gpeed_ctx_check(gpeed_ctx* ctx, void* stream);

/* Context options.  GPEED_OPT_FUSED_DECODE (default 1): run a batch-1
 * gpeed_moe_forward as one persistent kernel when the layer shape has a
 * compiled variant: hidden 5120 / inter 1536 with up to 256 routed experts,
 * and hidden 4096 / inter 2048 with up to 512 (the reference model's default
 * MoE shape, model_config.h:25, 59-60), one shared expert; 0 forces the
 * multi-kernel path (same results within rounding).  No counterpart in the
 * reference. */
#define GPEED_OPT_FUSED_DECODE 1
/* GPEED_OPT_FUSED_COOPERATIVE (default 0): launch that persistent kernel
 * cooperatively.  By default its CTAs start as the previous kernel's CTAs
 * leave the SMs (programmatic dependent launch), which assumes no other
 * kernel occupies SMs at the same time; a cooperative launch guarantees
 * co-residency at the cost of the launch gap.  Either way every wait inside
 * is bounded and a timeout is reported by gpeed_ctx_check. */
#define GPEED_OPT_FUSED_COOPERATIVE 2
/* GPEED_OPT_TC_MIN_TOKENS (default 8): batches of at least this many tokens
 * run the expert matrices as grouped GEMMs on the tensor cores (fp16
 * operands, fp32 accumulation; weights decoded from IQ3_XXS on the fly, each
 * touched expert once per slot of up to 224 tokens); smaller batches use the
 * quantised GEMV path (int8 x int16 dot products), and a single token the
 * fused decode kernel.  Measured per layer on B200, tensor cores vs GEMV:
 * Zipf-skewed routing 8 tokens 0.26 vs 0.34 ms, 64 tokens 0.42 vs 1.70 ms;
 * uniform routing 8 tokens 0.52 vs 0.62 ms, 32 tokens 1.11 vs 1.49 ms. */
#define GPEED_OPT_TC_MIN_TOKENS 3
/* GPEED_OPT_FUSED_MAX_TOKENS (default 12): batches of up to this many tokens
 * run the fused decode kernel once per token (each launch streams only that
 * token's nine experts; launches overlap through programmatic dependent
 * launch).  Larger batches take the tensor-core or GEMV paths above.
 * Measured with uniform routing: 8 tokens 0.30 ms per layer this way against
 * 0.52 ms on the tensor cores. */
#define GPEED_OPT_FUSED_MAX_TOKENS 4
/* GPEED_OPT_SPIN_LIMIT (default GPEED_SPIN_LIMIT_DEFAULT polls, a few seconds
 * under load): how long a wait inside the fused batch-1 kernel (on a pipeline
 * stage, or on data other CTAs publish) polls before it gives up, sets a
 * timeout bit that gpeed_ctx_check reports, and lets the kernel finish with
 * invalid results instead of hanging the GPU.  No counterpart in the
 * reference (it only throws, weights.cpp:21,25). */
#define GPEED_OPT_SPIN_LIMIT 5
#define GPEED_SPIN_LIMIT_DEFAULT (1 << 22)
/* GPEED_OPT_TEST_WITHHOLD_LOGIT (default -1): FOR TESTS ONLY.  The fused
 * kernel never publishes the router logit of this expert id, so every CTA's
 * wait for the full set of logits runs out (after GPEED_OPT_SPIN_LIMIT polls)
 * and the timeout path can be exercised without any fault; -1 turns it off. */
#define GPEED_OPT_TEST_WITHHOLD_LOGIT 6
GPEED_API int gpeed_ctx_set_option(gpeed_ctx* ctx, int option, int value);

/* Per-stage timing of gpeed_moe_forward (no counterpart in the reference;
 * its GLM5_PROFILE phase timer, model.cpp:21-38, is host wall-clock only).
 * When enabled, each forward records CUDA events between its five kernels
 * (router, route, gate/up, down, combine) on its stream and waits for them;
 * gpeed_ctx_profile_read returns the mean milliseconds per stage.  A fused
 * batch-1 forward is one kernel: its time is reported in the gate/up slot. */
GPEED_API int gpeed_ctx_profile(gpeed_ctx* ctx, int enable);
GPEED_API int gpeed_ctx_profile_read(gpeed_ctx* ctx, float* stage_ms /* [5] */, int* calls);

/* IQ3_XXS -> fp32, bit-exact with the reference codec.  n weights (multiple of
 * 256; the reference throws otherwise, quant.cpp:523-524). */
GPEED_API int gpeed_iq3xxs_dequantize(const void* src_dev, float* dst_dev, uint64_t n, void* stream);

/* Any codec the reference decodes, bit-exact (glm5::dequantize,
 * quant.cpp:521-573 with the block decoders at quant.cpp:165-503): dtype =
 * ggml id F32 0, F16 1, Q8_0 8, Q2_K 10, Q3_K 11, Q6_K 14, IQ3_XXS 18,
 * IQ3_S 21, IQ2_S 22, IQ4_XS 23, BF16 30; n a whole number of blocks (the
 * reference throws otherwise).  Device pointers; dst 16-byte aligned. */
GPEED_API int gpeed_dequantize(int dtype, const void* src_dev, float* dst_dev, uint64_t n, void* stream);

/* Uploads (or copies from device memory) an IQ3_XXS tensor of `rows` rows of
 * `in_dim` weights in GGUF row-major block order; the library keeps its own
 * device copy in a layout of its choosing.  Returns a handle (>= 0). */
GPEED_API int gpeed_tensor_upload(gpeed_ctx* ctx, const void* raw, int src_on_device, int dtype, uint64_t rows, int in_dim,
                        int* handle);
/* Reads a tensor back in GGUF byte order (verifies the lossless layout). */
GPEED_API int gpeed_tensor_download(gpeed_ctx* ctx, int handle, void* raw_host);

/* dst[j] = sum_i W[row0 + j][i] * x[i], j < out_dim; x, dst fp32 device. */
GPEED_API int gpeed_matvec_quant(gpeed_ctx* ctx, int handle, uint64_t row0, int in_dim, int out_dim, const float* x_dev,
                       float* dst_dev, void* stream);
/* Y[t][j] = sum_i W[row0 + j][i] * X[t][i], t < n_tok; row-major fp32 device. */
GPEED_API int gpeed_matmul_quant(gpeed_ctx* ctx, int handle, uint64_t row0, int in_dim, int out_dim, const float* X_dev,
                       int n_tok, float* Y_dev, void* stream);

/* The same two calls on HOST buffers, with the reference's calling convention
 * (WeightStore::matvec_quant / matmul_quant, weights.h:38-48, whose callers
 * pass std::vector data, model.cpp:733-754 and model_batch.cpp:241-279): x /
 * X are read and dst / Y written in host memory, and the call returns when
 * dst / Y hold the result.  Staged through pinned buffers on a stream of the
 * context (one host thread at a time per context); device-side errors are
 * reported here, as the reference throws inside the call. */
GPEED_API int gpeed_matvec_quant_host(gpeed_ctx* ctx, int handle, uint64_t row0, int in_dim, int out_dim,
                                      const float* x_host, float* dst_host);
GPEED_API int gpeed_matmul_quant_host(gpeed_ctx* ctx, int handle, uint64_t row0, int in_dim, int out_dim,
                                      const float* X_host, int n_tok, float* Y_host);

/* Same result as gpeed_matmul_quant (bit for bit: the same kernels on the same
 * work list), for callers that cannot call cudaMalloc once they are serving:
 * an engine whose own allocator or memory pool owns the GPU's memory, a
 * process held to a device-memory budget fixed at start-up, or a host whose
 * allocations must not fail or stall in the middle of a step.  No counterpart
 * in the reference.  It allocates nothing (no cudaMalloc, cudaFree or
 * allocating library call): its work list and output staging use one static
 * 4 MiB device array (GPEED_NOALLOC_SCRATCH_BYTES) that every GPU loading the
 * library keeps until exit.  Calls needing more scratch than that fail with
 * GPEED_ERR_INVALID: the staging is n_tok * (out_dim + row0 % 8 rounded up to
 * the row tile) * 4 bytes and is only used when row0 % 8 != 0 or out_dim is
 * not a multiple of the row tile.  The first call on a device looks the
 * array's device address up (cudaGetSymbolAddress), so make that first call
 * before any stream capture.  All calls share the array and it keeps the last
 * call's contents (each call rewrites what it reads), so calls that overlap on
 * the GPU race; serialise them. */
#define GPEED_NOALLOC_SCRATCH_BYTES (4u << 20)
GPEED_API int gpeed_matmul_quant_noalloc(gpeed_ctx* ctx, int handle, uint64_t row0, int in_dim, int out_dim,
                                         const float* X_dev, int n_tok, float* Y_dev, void* stream);

/* Registers layer `layer`: router weight fp32 [E][H], correction bias fp32 [E]
 * (may be NULL), routed expert tensors [E][rows][blocks] in raw IQ3_XXS
 * (gate/up: I rows of H; down: H rows of I) and the shared expert's three
 * matrices (NULL when n_shared == 0).  Host or device sources. */
GPEED_API int gpeed_moe_load_layer(gpeed_ctx* ctx, int layer, const gpeed_moe_shape* shape, const float* router_w,
                         const float* corr_bias, const void* gate_exps, const void* up_exps, const void* down_exps,
                         const void* gate_sh, const void* up_sh, const void* down_sh, int src_on_device);
/* Same, with every expert byte produced on the device by the counter-based
 * synthetic generator (seed, streams stream0 .. stream0+5); for benchmarks
 * and tests.  router_w / corr_bias are host or device per src_on_device. */
GPEED_API int gpeed_moe_synth_layer(gpeed_ctx* ctx, int layer, const gpeed_moe_shape* shape, const float* router_w,
                          const float* corr_bias, int src_on_device, uint64_t seed, uint64_t stream0);
/* Writes `nblocks` synthetic IQ3_XXS blocks (starting at block0 of the
 * stream) to device memory. */
GPEED_API int gpeed_synth_iq3xxs(void* dst_dev, uint64_t seed, uint64_t stream, uint64_t block0, uint64_t nblocks,
                       void* stream_);

/* y[t] = MoE(x[t]) for t < n_tok: x bf16 or fp32 [n_tok][H] (x_dtype =
 * GPEED_DTYPE_BF16 / _F32), y fp32 [n_tok][H], device pointers.  forced_topk
 * (device int [n_tok][K] or NULL) replaces the top-k choice; topk_ids /
 * topk_w (device [n_tok][K] or NULL) receive the routing. */
GPEED_API int gpeed_moe_forward(gpeed_ctx* ctx, int layer, const void* x_dev, int x_dtype, int n_tok, float* y_dev,
                      const int* forced_topk_dev, int* topk_ids_dev, float* topk_w_dev, void* stream);
/* The same layer on the caller's HOST buffers, as the reference's callers
 * hold them (Model::moe_forward / moe_batch, model.cpp:692-756 and
 * model_batch.cpp:165-281, take and fill host vectors): x_host [n_tok][H]
 * (bf16 or fp32 per x_dtype), y_host [n_tok][H] fp32.  The input goes to the
 * device through the context's pinned staging on the context's own stream,
 * and the call returns once y is on the host (synchronous, like the
 * reference call).  Calls on one context are serialised. */
GPEED_API int gpeed_moe_forward_host(gpeed_ctx* ctx, int layer, const void* x_host, int x_dtype, int n_tok,
                                     float* y_host);

/* ---- Expert parallelism (no counterpart in the reference: it runs every
 * expert on one host).  Experts split into equal contiguous ranges, one per
 * rank; tokens stay data-parallel; the router and the shared expert are
 * replicated.  The exchange between ranks (counts, token rows, expert
 * outputs) is left to the caller's collectives (NCCL all-to-all); these
 * entry points do the device work on either side of it:
 *
 *   gpeed_moe_route     -> top-k ids/weights of this rank's tokens
 *   gpeed_ep_pack       -> rows grouped by destination rank + per-rank counts
 *   (all-to-all of rows and ids)
 *   gpeed_moe_experts   -> down(SwiGLU(gate x, up x)) per received row, its expert
 *   (all-to-all of the results back)
 *   gpeed_moe_experts   -> the shared expert on this rank's own tokens (id = E)
 *   gpeed_moe_combine   -> y = sum_k w_k D_k + D_shared, in top-k order
 *
 * With the same weights every rank's y is bit-identical to gpeed_moe_forward
 * on one GPU for n_tok > 1 (the batched path). */

/* Expert-parallel decode, one rank's share in one persistent kernel (the
 * batch-1 kernel of gpeed_moe_forward generalised): x holds every rank's token
 * ([n_tok][H], n_tok <= 8 and n_tok * top_k <= 64, identical on all ranks,
 * e.g. from an all-gather), own_tok is this rank's.  The kernel routes all
 * n_tok tokens, runs gate/up -> SwiGLU -> down for the (token, k) picks whose
 * expert the layer holds (gpeed_moe_load_layer_range) plus the shared expert
 * of own_tok, and writes y_part[t] = sum of w_k D_k over those picks of token
 * t, in pick order, (+ D_shared for own_tok): zero rows for tokens with
 * nothing here.  On a layer sliced by units (gpeed_moe_slice_units) it runs
 * this slice of every pick (and own_tok's whole shared expert).  Summed over the ranks (a reduce-scatter), y_part gives
 * gpeed_moe_forward's y up to the order of that sum.  forced_topk / topk_ids /
 * topk_w are [n_tok][K] as in gpeed_moe_forward.  No counterpart in the
 * reference (Model::moe_forward, model.cpp:692-756, runs every expert on one
 * host). */
GPEED_API int gpeed_moe_decode_partial(gpeed_ctx* ctx, int layer, const void* x_dev, int x_dtype, int n_tok,
                                       int own_tok, float* y_part_dev, const int* forced_topk_dev, int* topk_ids_dev,
                                       float* topk_w_dev, void* stream);

/* Expert-parallel decode with no collective library: the step's exchanges
 * run inside the persistent kernel over NVLink peer memory.  Each rank of a
 * world of 2 .. 8 GPUs (one process per GPU) calls gpeed_ep_setup (allocates
 * this rank's exchange block and returns its CUDA IPC handle,
 * GPEED_IPC_HANDLE_BYTES bytes), hands every rank's handle to every rank (its
 * own process group does that; gpeed_b200.ep.PeerDecode uses
 * torch.distributed) and calls gpeed_ep_connect with the world's handles in
 * rank order; then, every step, every rank calls gpeed_moe_decode_ep with its
 * own token x ([1][H] bf16 or fp32) and receives that token's layer output y
 * ([1][H] fp32).  The layer is either this rank's expert range plus the
 * shared expert (gpeed_moe_load_layer_range / _gguf / _synth_layer_range),
 * E/world routed experts per rank, or a whole layer sliced by units
 * (gpeed_moe_slice_units with unit_begin = rank * unit_count): every rank then
 * runs its slice of every pick and its own token's shared expert, the same
 * work whatever the routing.  Any other share (a whole layer, or the share
 * of another rank or world size) is refused with GPEED_ERR_INVALID: the
 * ranks' shares must cover every pick exactly once.  Inside one launch: the token goes to every rank as
 * tagged words, all world tokens are routed, this rank's picks of every token
 * run, and their down sums are added straight into the owning rank's
 * accumulator; the kernel ends when every other rank has signalled that its
 * sums into this rank's accumulator are done.  Every rank must run the same
 * sequence of steps (waits are bounded: a rank that does not take part makes
 * the others' step time out, reported by gpeed_ctx_check, after which the
 * group is set up again).  Plain peer loads, stores and reductions only: no
 * TMA, multicast or switch reduction on peer memory.  topk_ids / topk_w:
 * optional [world][K] picks of every token.  No counterpart in the reference
 * (Model::moe_forward, model.cpp:692-756, runs every expert on one host). */
#define GPEED_IPC_HANDLE_BYTES 64
GPEED_API int gpeed_ep_setup(gpeed_ctx* ctx, int world, int rank, int hidden, void* handle_out);
GPEED_API int gpeed_ep_connect(gpeed_ctx* ctx, const void* handles /* world x GPEED_IPC_HANDLE_BYTES */);
GPEED_API int gpeed_moe_decode_ep(gpeed_ctx* ctx, int layer, const void* x_dev, int x_dtype, float* y_dev,
                                  int* topk_ids_dev, float* topk_w_dev, void* stream);
/* Unmaps the other ranks' blocks (after the group's last step, before any rank
 * frees its own block with gpeed_ctx_destroy: every rank disconnects, the group
 * meets at a barrier, then the contexts are destroyed). */
GPEED_API int gpeed_ep_disconnect(gpeed_ctx* ctx);

/* Loads only routed experts [expert_begin, expert_begin + expert_count) (their
 * GGUF bytes at gate/up/down) plus the shared expert; the router stays whole. */
GPEED_API int gpeed_moe_load_layer_range(gpeed_ctx* ctx, int layer, const gpeed_moe_shape* shape, int expert_begin,
                               int expert_count, const float* router_w, const float* corr_bias, const void* gate_exps,
                               const void* up_exps, const void* down_exps, const void* gate_sh, const void* up_sh,
                               const void* down_sh, int on_device);
/* As gpeed_moe_synth_layer, for an expert range: the bytes equal the matching
 * slice of the whole synthetic layer. */
GPEED_API int gpeed_moe_synth_layer_range(gpeed_ctx* ctx, int layer, const gpeed_moe_shape* shape, int expert_begin,
                                int expert_count, const float* router_w, const float* corr_bias, int on_device,
                                uint64_t seed, uint64_t stream0);
/* Keeps only units [unit_begin, unit_begin + unit_count) of a loaded whole
 * layer's routed experts, a unit being 32 intermediate rows: the gate/up rows
 * unit*32 .. +31 and the same down columns; the shared expert stays whole.
 * The tensor-parallel split of every routed expert: ranks r = 0 .. N-1
 * slicing [r*NU/N, (r+1)*NU/N) of the NU = inter/32 units each compute, for
 * every pick, a part of the down sum (SwiGLU is row-wise, so the
 * intermediate rows split exactly), and the parts add up to the layer output;
 * each rank runs its own token's shared expert.  unit_count: a divisor of NU
 * the persistent decode kernel has (NU, NU/2, NU/4, NU/8 for inter 1536 and
 * 2048);
 * unit_begin a multiple of it.  A sliced layer serves
 * gpeed_moe_decode_partial (the slice of every pick plus own_tok's shared
 * expert) and gpeed_moe_decode_ep; the other entry points refuse it.  No
 * counterpart in the reference. */
GPEED_API int gpeed_moe_slice_units(gpeed_ctx* ctx, int layer, int unit_begin, int unit_count);
/* Router + top-k only (model_batch.cpp:171-203): topk_ids/topk_w device [n_tok][K]. */
GPEED_API int gpeed_moe_route(gpeed_ctx* ctx, int layer, const void* x_dev, int x_dtype, int n_tok,
                              const int* forced_topk_dev, int* topk_ids_dev, float* topk_w_dev, void* stream);
/* Groups this rank's n_tok*K assignments by destination rank (expert /
 * (n_experts/world)), stable in token order within an expert: send_rows
 * [n_tok*K][hidden] (x's dtype), send_ids [n_tok*K] (global expert ids),
 * rank_counts [world] (device), slot_of [n_tok][K] = position of (t, k) in
 * the send buffers. */
GPEED_API int gpeed_ep_pack(gpeed_ctx* ctx, int n_experts, int world, int n_tok, int K, const int* topk_ids_dev,
                            const void* x_dev, int x_dtype, int hidden, void* send_rows_dev, int* send_ids_dev,
                            int* rank_counts_dev, int* slot_of_dev, void* stream);
/* out[i] = down_e(SwiGLU(gate_e rows[i], up_e rows[i])) for e = expert_ids[i]
 * (global id; n_experts = the shared expert), fp32 [m][hidden].  The layer
 * must hold every listed expert. */
GPEED_API int gpeed_moe_experts(gpeed_ctx* ctx, int layer, const void* rows_dev, int rows_dtype, int m,
                                const int* expert_ids_dev, float* out_dev, void* stream);
/* y[t] = sum_k w[t][k] * d_rows[slot_of[t][k]] (+ d_shared[t]), fp32, k in order
 * (model.cpp:741-755). */
GPEED_API int gpeed_moe_combine(gpeed_ctx* ctx, int n_tok, int K, int hidden, const float* d_rows_dev,
                                const int* slot_of_dev, const float* topk_w_dev, const float* d_shared_dev,
                                float* y_dev, void* stream);

/* Dense SwiGLU MLP of the leading dense layers (Model::dense_mlp,
 * model.cpp:677-690, and dense_mlp_batch, model_batch.cpp:145-163):
 *   Y[t] = down(silu(min(gate X[t], L)) * clamp(up X[t], -L, L))
 * over three IQ3_XXS tensors registered with gpeed_tensor_upload[_gguf]
 * (gate/up: inter rows of hidden weights; down: hidden rows of inter), run by
 * the expert kernels as a one-expert pass.  X bf16 or fp32 [n_tok][hidden],
 * Y fp32 [n_tok][hidden], device. */
GPEED_API int gpeed_dense_mlp_forward(gpeed_ctx* ctx, int gate, int up, int down, float swiglu_limit, const void* X_dev,
                                      int x_dtype, int n_tok, float* Y_dev, void* stream);

/* ---- mHC residual mixing + RMSNorm on either side of the MoE layer
 * (Model::hc_forward, model.cpp:205-263, the ffn norm at model.cpp:292-296 and
 * the stream update at model.cpp:309-318; run_chunk passes 4 and 6,
 * model_batch.cpp:374-410).  Per token t, hc_mult = N residual streams of H:
 *
 *   gpeed_mhc_pre:  x[t] = rmsnorm(sum_n pre[n] streams[t][n]) * norm_w, the
 *                   MoE / dense-MLP input (fp32 or bf16), with pre, post and
 *                   the Sinkhorn-normalised comb [N][N] formed from the
 *                   (2+N)N dot products of fn with rmsnorm(streams[t]);
 *   gpeed_mhc_post: streams_out[t][n] = post[t][n] mlp_out[t]
 *                   + sum_m comb[t][m][n] streams_in[t][m]  (in place allowed).
 *
 * fn [(2+N)N][N*H], base [(2+N)N], scale [3], norm_w [H], streams [n][N][H],
 * all fp32 device buffers (the reference widens these tensors to fp32 too).
 * Floating point: sums run in a different order than the reference's
 * (relative differences ~1e-6). */
typedef struct gpeed_mhc_params {
    int hc_mult;         /* N, 1..4 (model_config.h:47, default 4) */
    int sinkhorn_iters;  /* 20 */
    float hc_eps;        /* 1e-6 */
    float rms_eps;       /* 1e-5 */
} gpeed_mhc_params;
GPEED_API int gpeed_mhc_pre(gpeed_ctx* ctx, const float* streams_dev, int n_tok, int hidden,
                            const gpeed_mhc_params* params, const float* fn_dev, const float* base_dev,
                            const float* scale_dev, const float* norm_w_dev, void* x_dev, int x_dtype, float* post_dev,
                            float* comb_dev, void* stream);
GPEED_API int gpeed_mhc_post(gpeed_ctx* ctx, const float* streams_in_dev, const float* mlp_out_dev,
                             const float* post_dev, const float* comb_dev, int n_tok, int hidden, int hc_mult,
                             float* streams_out_dev, void* stream);

/* ---- GGUF model files (cpp/core/include/glm5/gguf.h; gguf.cpp).
 *
 *   gpeed_gguf_open           <- GgufModel::load(GgufModel::discover_shards(path))
 *                                (gguf.cpp:255-326, parse at gguf.cpp:133-188):
 *                                versions 2 and 3, "<stem>-NNNNN-of-MMMMM.gguf"
 *                                shards found from any one of them; a tensor
 *                                name resolves to its first shard, a metadata
 *                                key to the first shard that has it.  The
 *                                files are mapped read-only (the reference
 *                                maps them on Windows and reads them with an
 *                                ifstream elsewhere, weights.cpp:62-68).
 *   gpeed_gguf_tensor_info    <- GgufModel::find_tensor + TensorInfo
 *   gpeed_gguf_read           <- GgufFile::read_at (gguf.cpp:236-248)
 *   gpeed_gguf_meta_*         <- GgufModel::find + GgufValue::as_* (permissive
 *                                numeric coercion as gguf.cpp:85-117)
 *   gpeed_gguf_moe_shape      <- ModelConfig::from_gguf, MoE fields
 *                                (model_config.cpp:80-95) for block `blk`
 *   gpeed_tensor_upload_gguf  <- WeightStore's payload of one tensor by name
 *                                (weights.cpp:62-68)
 *   gpeed_moe_load_layer_gguf <- the tensors Model::moe_forward reads by name
 *                                (model.cpp:702-754) for block `blk`, straight
 *                                from the mapping into the library's layout;
 *                                an expert range for expert parallelism.
 * Handles are not thread-safe; the mapping lives until gpeed_gguf_close. */
typedef struct gpeed_gguf gpeed_gguf;

typedef struct gpeed_gguf_tensor {
    int dtype;           /* ggml type id (reference common.h:10-44) */
    int n_dims;          /* 1..4 */
    uint64_t dims[4];    /* ggml ne order: dims[0] is the contiguous one */
    uint64_t offset;     /* byte offset inside its shard's tensor-data section */
    uint64_t nbytes;     /* payload bytes (0 for a type without a known block size) */
    int shard;           /* index of the shard file holding it */
} gpeed_gguf_tensor;

#define GPEED_GGUF_UINT8 0      /* metadata value types (gguf.h:15-29) */
#define GPEED_GGUF_STRING 8
#define GPEED_GGUF_ARRAY 9

GPEED_API int gpeed_gguf_open(const char* path, gpeed_gguf** out);
GPEED_API int gpeed_gguf_close(gpeed_gguf* g);
GPEED_API int gpeed_gguf_counts(gpeed_gguf* g, int* n_shards, int64_t* n_tensors, int64_t* n_keys);
/* i-th tensor name in shard order (GgufModel::tensor_names); valid until close. */
GPEED_API int gpeed_gguf_tensor_name(gpeed_gguf* g, int64_t i, const char** name);
/* i-th metadata key (union over shards, first-seen order); valid until close. */
GPEED_API int gpeed_gguf_key_name(gpeed_gguf* g, int64_t i, const char** name);
GPEED_API int gpeed_gguf_tensor_info(gpeed_gguf* g, const char* name, gpeed_gguf_tensor* out);
/* Copies `bytes` bytes at `byte_off` inside tensor `name` to host memory. */
GPEED_API int gpeed_gguf_read(gpeed_gguf* g, const char* name, uint64_t byte_off, uint64_t bytes, void* dst_host);
/* Value type of `key` (GPEED_GGUF_*; for arrays also the element type and length). */
GPEED_API int gpeed_gguf_meta_type(gpeed_gguf* g, const char* key, int* type, int* elem_type, uint64_t* n);
/* Numeric scalar (index 0) or element `index` of a numeric array. */
GPEED_API int gpeed_gguf_meta_f64(gpeed_gguf* g, const char* key, uint64_t index, double* out);
GPEED_API int gpeed_gguf_meta_u64(gpeed_gguf* g, const char* key, uint64_t* out);
GPEED_API int gpeed_gguf_meta_str(gpeed_gguf* g, const char* key, const char** out);
/* MoE shape of block `blk`: H, I, E from the expert tensors' dims, the rest
 * from "<general.architecture>.<key>" metadata with the reference's defaults
 * (top_k 8, n_shared 1, scale 2.5, norm 1, swiglu limit 10); fails
 * GPEED_ERR_UNSUPPORTED unless the gating function is sigmoid (2). */
GPEED_API int gpeed_gguf_moe_shape(gpeed_gguf* g, int blk, gpeed_moe_shape* out);
/* gpeed_tensor_upload of the IQ3_XXS tensor `name` straight from the file
 * mapping (rows = product of dims[1..], in_dim = dims[0]): the payload the
 * reference's WeightStore reads by name (weights.cpp:62-68, 167-203). */
GPEED_API int gpeed_tensor_upload_gguf(gpeed_ctx* ctx, gpeed_gguf* g, const char* name, int* handle);
/* Registers block `blk`'s MoE tensors as layer `layer` of ctx: the router
 * (ffn_gate_inp, F32/F16/BF16), the bias (exp_probs_b, optional), routed
 * experts [expert_begin, expert_begin + expert_count) of ffn_{gate,up,down}_exps
 * (IQ3_XXS) and the shared expert (ffn_*_shexp).  expert_count < 0 = all. */
GPEED_API int gpeed_moe_load_layer_gguf(gpeed_ctx* ctx, gpeed_gguf* g, int blk, int layer, int expert_begin,
                                        int expert_count, gpeed_moe_shape* shape_out);

#ifdef __cplusplus
}
#endif
#endif /* GPEED_MOE_H */
