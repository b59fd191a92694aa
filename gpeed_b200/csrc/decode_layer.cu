// One MoE layer at decode batch sizes in a single persistent kernel
// (reference Model::moe_forward, cpp/core/src/model.cpp:692-756).
//
// Separate kernels for router, routing, gate/up, down and combine each pay a
// launch, a prologue (decode tables, first bytes in flight) and a tail, which
// at batch 1 costs more than streaming the 85 MB of weights.  Here one CTA per
// SM runs the whole layer.  Warp roles: 20 compute warps, one TMA producer
// warp streaming weights through a ring of shared-memory stages, and one
// epilogue warp that does the routing and turns each stage's partial sums
// into h.  Values other CTAs produced (router logits, h) are read as words
// tagged with the launch generation: the data is its own flag.
//
// Work is dealt to the CTAs one pipeline stage ("job") at a time, round-robin
// over a global job list, so every CTA gets the same number of stages within
// one: first the shared expert's gate/up tiles (they need no routing, and run
// while the routing exchange is in flight), then the routed slots' gate/up
// tiles, then every slot's down chunks.  A gate/up tile is 8 gate + 8 up rows
// of one slot's expert; the epilogue applies SwiGLU with the reference clamp
// (model.cpp:733-739) and publishes the 8 h values as tagged words.  A down
// chunk is the split-K slice of W_down that one unit of 32 h values
// multiplies, for 2560 output rows, streamed from a column-slab copy of
// W_down; the epilogue fetches and quantises the unit's h one stage ahead
// (tiles of that unit ran about eleven stages earlier, on any CTA), and the
// compute warps add w_k * D_slice into y with vector fp32 reductions.
//
//   router   CTA c owns experts c, c+G, ...; 8 warps each compute one 1/8
//            slice of an owned expert's fp32 logit for every token (weights
//            prefetched before the wait on the previous kernel); the
//            epilogue warp adds the slices in order and stores the logit
//            tagged with the launch generation, so readers poll the data itself
//   top-k    every CTA's epilogue warp polls each token's E tagged logits
//            (one of 8 replicas, spread over L2 lines), applies sigmoid + bias
//            and picks top-K by warp reductions (ties to the lower id),
//            weights score/(1e-20 + sum)*scale (model.cpp:704-725).  The picks
//            in the launch's expert range become its slots
//   y        zeroed by the CTAs before they publish their logits; every
//            reduction into y comes after its CTA has seen the routing, so
//            after every CTA's zeroing
//
// The same kernel runs one rank's share of an expert-parallel decode step:
// n_tok tokens (one per rank), the routed experts of one range, the shared
// expert of the rank's own token; y[t] is then this rank's part of token t's
// output (the ranks' parts sum to the layer).
//
// The routing exchange needs every CTA resident: one CTA per SM, launched
// either with programmatic dependent launch (default) or cooperatively.
// Every wait is bounded; a timeout sets a status bit, the CTA stops and
// finishes (results then invalid, the host reports the status and clears the
// counters and tags).  Sums into y land in a different order from launch to
// launch (fp32 reductions), so results agree to rounding, not bit for bit.
#include <cuda_fp16.h>

#include "expert_common.cuh"
#include "iq3xxs.cuh"
#include "kernels.h"

#ifndef TOPK_POLL_NS
#define TOPK_POLL_NS 32
#endif
// Optional instrumentation hook (timestamps per CTA); compiled out here.
#ifndef GP_STAMP
#define GP_STAMP(i) ((void)0)
#endif

namespace gp {
namespace {

// The CTA's shape follows the hidden size H (a multiple of 1024): H/256
// compute warps, so one gate/up pass covers 4 whole rows (H/32 lanes per row,
// a whole number of warps), and a down chunk is 4 rows per compute lane = H/2
// rows.  H = 5120: 20 compute warps; H = 4096: 16.  Then one epilogue warp
// and one TMA producer warp (warp indices NWC and NWC + 1).
__host__ __device__ constexpr int nwc_of(int H) { return H / 256; }        // compute warps
__host__ __device__ constexpr int nthreads_of(int H) { return 32 * (H / 256 + 2); }
__host__ __device__ constexpr int rc_of(int H) { return H / 2; }            // down rows per chunk
constexpr int TRG = 8;           // gate/up rows per matrix per tile
constexpr int UNIT = 32;         // rows of h per unit = input columns of its down slice
constexpr int TPU = UNIT / TRG;  // gate/up tiles per unit
constexpr int RSPLIT = 8;        // router slices per expert
constexpr int MAXK = 31;         // picks per token
constexpr int kMaxEFused = 512;  // routed experts handled by the top-k warp
constexpr int kMaxOwned = 8;     // router experts per CTA (grid >= E/8)
// Tagged logits: with one token every CTA polls all E of them, so one array
// would send every poll of every CTA to the few L2 slices holding it.  Each
// logit is then stored in kLogitCopies replicas, one word per 256-byte line;
// CTA c polls replica c % kLogitCopies.
constexpr int kLogitCopies = 8;
constexpr int kLogitStride = 32;  // words
static_assert(kLogitCopies * kLogitStride == 256, "decode_layer_logit_words (kernels.h) assumes 8 x 32");

GP_DEVINL unsigned long long ld_relaxed64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
GP_DEVINL void st_relaxed64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
GP_DEVINL unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// System-scope forms for the expert-parallel exchange over peer memory.
GP_DEVINL unsigned long long ld_relaxed_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
GP_DEVINL void st_relaxed_sys64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
GP_DEVINL unsigned long long ld_acquire_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
GP_DEVINL void red_release_sys_add64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
GP_DEVINL void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// y[0..3] += v as one fire-and-forget vector reduction: no value comes
// back, so the warp does not wait for the L2 round trip (an atomicAdd on a
// float4 returns the old values and stalls the registers that receive them).
GP_DEVINL void red_add_v4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
// The same at system scope: an owner's accumulator also takes the other
// GPUs' adds (expert-parallel).
GP_DEVINL void red_add_sys_v4(float* p, float a, float b, float c, float d) {
    asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// Warp-uniform view of the CTA's abort flag.  Lanes read the volatile word
// separately and may see it change between reads; every branch that contains
// warp-collective operations (shuffles, votes) must use one value for the
// whole warp.
GP_DEVINL bool warp_aborted(const volatile uint32_t* s_abort) { return __any_sync(0xffffffffu, *s_abort != 0u); }

// Monotonic map of a float onto u32 (for redux max); -0 is folded onto +0 first.
GP_DEVINL uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Token words of the expert-parallel exchange: token t's x as 64-bit words
// {32 bits of payload (a bf16 pair, or one fp32), the step's tag} at
// ep_x[t * H + word].  A reader loads every word it needs at once, 16 bytes
// per load (w[i] even), checks every tag, and loads again until they all
// match (each round is a round trip to memory under load, so a reader asks
// for all it needs in one round, and waits longer between rounds as it goes
// on); ok turns false when that runs out.
template <int NP>
GP_DEVINL void ep_fetch(const DecodeLayerArgs& a, const int (&w)[NP], uint32_t tag, uint32_t (&out)[2 * NP], bool& ok) {
    const unsigned long long* base = a.ep_x;  // w[i]: token * H + word
    for (uint32_t n = 0;; ++n) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            unsigned long long v0, v1;
            asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(base + w[i]) : "memory");
            all &= (uint32_t)(v0 >> 32) == tag && (uint32_t)(v1 >> 32) == tag;
            out[2 * i] = (uint32_t)v0;
            out[2 * i + 1] = (uint32_t)v1;
        }
        if (all) return;
        if (n >= a.spin_limit) {
            ok = false;
            return;
        }
        // growing pauses: many lanes poll at once, and their loads must not
        // crowd out the SM's other memory traffic (router, logits, copies)
        __nanosleep(n < 3 ? 128u << n : 1024u);
    }
}

// 32 consecutive x elements k0 .. k0+31 of token t from the exchange (k0 % 32 == 0),
// in pieces of 8 (bf16: 16) elements so that few registers are live at once.
GP_DEVINL void ep_x32(const DecodeLayerArgs& a, int t, int k0, uint32_t tag, float (&v)[32], bool& ok) {
    if (a.x_bf16) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = t * a.H + (k0 + 16 * h) / 2 + 2 * i;
            uint32_t u[8];
            ep_fetch<4>(a, w, tag, u, ok);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[16 * h + 2 * i] = __uint_as_float(u[i] << 16);
                v[16 * h + 2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
            }
        }
    } else {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            int w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = t * a.H + k0 + 8 * h + 2 * i;
            uint32_t u[8];
            ep_fetch<4>(a, w, tag, u, ok);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * h + i] = __uint_as_float(u[i]);
        }
    }
}

// x elements k .. k+3 of token t.
GP_DEVINL float4 x4_of(const DecodeLayerArgs& a, int t, int k) {
    const int64_t k0 = (int64_t)t * a.H + k;
    if (a.x_bf16) {
        const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + k0);
        return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                           __uint_as_float(r.y & 0xFFFF0000u));
    }
    return *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + k0);
}

// Per-lane view of one GEMV phase (in_dim = IN, NW warps, P passes): this
// lane's fixed sub-block, its pass-0 byte offsets inside a stage, and the
// constant offsets of the later passes.  Rows of pass p are row0 + p*ROWSTEP.
template <int IN, int NW, int P>
struct LaneMap {
    static constexpr int SB = IN / 32, NBLK = IN / 256, ROWSTEP = 32 * NW / SB;
    static constexpr uint32_t GROUP = 784u * NBLK;
    static_assert((32 * NW) % SB == 0, "lanes must tile whole rows");
    static_assert(ROWSTEP % 8 == 0 || (ROWSTEP < 8 && 8 % ROWSTEP == 0 && (8 / ROWSTEP) * ROWSTEP == 8),
                  "passes must keep a lane inside the same 8-row group pattern");
    // warps whose lanes cover row r of a pass: first_warp(r) .. first_warp(r) + span - 1
    static constexpr GP_DEVINL int first_warp(int r) { return r * SB / 32; }
    static constexpr GP_DEVINL int last_warp(int r) { return (r * SB + SB - 1) / 32; }
    static constexpr int max_span(int r = 0, int m = 0) {
        return r == ROWSTEP ? m : max_span(r + 1, last_warp(r) - first_warp(r) + 1 > m ? last_warp(r) - first_warp(r) + 1 : m);
    }
    // partial sums per row: one slot per covering warp (row * WPR + warp - first_warp)
    static constexpr int WPR = max_span();
    uint32_t q0, a0, d0;
    int sb, wrow0, wspan, jrow, row0;
    // byte offset of pass p relative to pass 0 for a stream with `stride` bytes per row in a group
    static GP_DEVINL uint32_t delta(int p, int row0, uint32_t stride) {
        const int r = row0 + p * ROWSTEP;
        return (uint32_t)((r >> 3) - (row0 >> 3)) * GROUP + (uint32_t)((r & 7) - (row0 & 7)) * stride;
    }
};

template <int IN, int NW, int P>
GP_DEVINL LaneMap<IN, NW, P> lane_map(int warp, int lane, uint32_t stage0) {
    using LM = LaneMap<IN, NW, P>;
    LM m;
    const int u0 = warp * 32 + lane;
    m.sb = u0 % LM::SB;
    m.row0 = u0 / LM::SB;
    m.wrow0 = (warp * 32) / LM::SB;
    m.wspan = (warp * 32 + 31) / LM::SB - m.wrow0 + 1;
    m.jrow = m.row0 - m.wrow0;
    const int b = m.sb >> 3, ib = m.sb & 7;
    const uint32_t gb = (m.row0 >> 3) * LM::GROUP, ri = m.row0 & 7;
    m.q0 = stage0 + gb + ri * 64u * LM::NBLK + 64u * b + 8u * ib;
    m.a0 = stage0 + gb + 512u * LM::NBLK + ri * 32u * LM::NBLK + 32u * b + 4u * ib;
    m.d0 = stage0 + gb + 768u * LM::NBLK + ri * 2u * LM::NBLK + 2u * b;
    return m;
}

// Decodes this lane's P sub-blocks of the stage at soff, dots them with the
// lane's activations and reduces over the warp; writes the per-warp row
// partials into pbuf[row * NW + warp].
template <int IN, int NW, int P, int RPW>
GP_DEVINL void consume(const LaneMap<IN, NW, P>& m, uint32_t soff, const uint32_t (&xq)[16], float sx4, float* pbuf,
                       int warp, int lane) {
    using LM = LaneMap<IN, NW, P>;
    constexpr int M = P * RPW;
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) acc[i] = 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) {
        // row0 only shifts the group boundary when ROWSTEP < 8; otherwise the
        // deltas are compile-time constants
        const uint32_t dq = LM::ROWSTEP % 8 == 0 ? p * (LM::ROWSTEP / 8) * LM::GROUP : LM::delta(p, m.row0, 64u * LM::NBLK);
        const uint32_t da = LM::ROWSTEP % 8 == 0 ? p * (LM::ROWSTEP / 8) * LM::GROUP : LM::delta(p, m.row0, 32u * LM::NBLK);
        const uint32_t dd = LM::ROWSTEP % 8 == 0 ? p * (LM::ROWSTEP / 8) * LM::GROUP : LM::delta(p, m.row0, 2u * LM::NBLK);
        const uint32_t aux = lds32(m.a0 + soff + da);
        const float d = __half2float(__ushort_as_half((unsigned short)lds16(m.d0 + soff + dd)));
        const uint2 q = lds64(m.q0 + soff + dq);
        uint32_t sw[8];
        iq3_decode_sub32(nullptr, q.x, q.y, aux, lane * 4u, sw);
        const float v = (float)(iq3_idot<8>(sw, xq) * iq3_oddscale(aux)) * (d * sx4);
        if (RPW == 1) {
            acc[p] = v;
        } else {
#pragma unroll
            for (int j = 0; j < RPW; ++j)
                if (j == m.jrow) acc[p * RPW + j] = v;
        }
    }
    const float red = warp_reduce_many<M>(acc, lane);
    constexpr int kShift = 5 - ilog2(M);
    if ((lane & ((1 << kShift) - 1)) == 0) {
        const int idx = lane >> kShift, p = idx / RPW, j = idx % RPW;
        const int r = m.wrow0 + j;  // row within the pass
        if (j < m.wspan) pbuf[(r + p * LM::ROWSTEP) * LM::WPR + warp - LM::first_warp(r)] = red;
    }
}

// Loads and quantises this lane's 32 activations (sub-block sb of row `row`).
GP_DEVINL float load_quant(const void* x, int x_bf16, int64_t row, int in_dim, int sb, uint32_t (&xq)[16]) {
    float v[32];
    load_x_unit<32>(x, x_bf16, row, in_dim, 32 * sb, v);
    return 0.25f * quant_i16<32>(v, xq);
}

// Tagged logit of token `tok`, expert e: every CTA reads every token's, so
// each is kept in kLogitCopies replicas (copy = reader's CTA % kLogitCopies).
GP_DEVINL int64_t logit_word(int copy, int tok, int e, int E) {
    return (((int64_t)tok * kLogitCopies + copy) * E + e) * kLogitStride;
}

// One token's top-K by score + bias (ties to the lower id), weights
// score/(1e-20 + sum)*scale (model.cpp:704-725), or the forced ids with their
// weights.  The E logits are polled as words tagged by their writers with this
// launch's tag: the data is its own flag, so one poll round trip suffices.
// Each lane sorts its EJ candidates (expert ids lane + 32j) by (key desc, id
// asc); a round then takes the warp maximum of the lanes' head keys (redux),
// the lowest id holding it, and that lane pops its head.  Lane k < K returns
// pick k in (my_e, my_w).  Returns false when the wait for the logits ran out.
// Loads token tok's (and tok2's, when tok2 >= 0: both in one round of loads)
// E tagged logits until every tag matches; false when the wait ran out.
template <int EJ>
GP_DEVINL bool poll_logits(const DecodeLayerArgs& a, uint32_t tag, int lane, int copy, int tok, int tok2,
                           uint32_t (&w)[EJ], uint32_t (&w2)[EJ]) {
    const int E = a.E;
    for (uint32_t n = 0; n < a.spin_limit; ++n) {
        bool ok = true;
#pragma unroll
        for (int j = 0; j < EJ; ++j) {  // (values kept as 32-bit logits, tags checked as they arrive)
            const unsigned long long v =
                lane + 32 * j < E ? ld_relaxed64(a.logits + logit_word(copy, tok, lane + 32 * j, E)) : 0ull;
            const unsigned long long v2 = tok2 >= 0 && lane + 32 * j < E
                                              ? ld_relaxed64(a.logits + logit_word(copy, tok2, lane + 32 * j, E)) : 0ull;
            ok &= lane + 32 * j >= E || (uint32_t)(v >> 32) == tag;
            ok &= tok2 < 0 || lane + 32 * j >= E || (uint32_t)(v2 >> 32) == tag;
            w[j] = (uint32_t)v;
            w2[j] = (uint32_t)v2;
        }
        if (__all_sync(0xffffffffu, ok)) return true;
        __nanosleep(TOPK_POLL_NS);
    }
    return false;
}

template <int EJ>
GP_DEVINL void select_topk(const DecodeLayerArgs& a, const float* bias, const uint32_t (&w)[EJ], int lane, int tok,
                           bool write_out, int& my_e, float& my_w);

template <int EJ>
GP_DEVINL bool topk_token(const DecodeLayerArgs& a, const float* bias, uint32_t tag, int lane, int copy, int tok,
                          bool write_out, int& my_e, float& my_w) {
    uint32_t w[EJ], w2[EJ];
    const bool got = poll_logits<EJ>(a, tag, lane, copy, tok, -1, w, w2);
    select_topk<EJ>(a, bias, w, lane, tok, write_out, my_e, my_w);
    return got;
}

// Top-K for many experts per lane (EJ > 8, up to 512 experts): the sort
// below would hold EJ keys, ids and scores per lane at once.  Here each
// round takes every lane's best remaining key (ties to the lower j, so the
// lower id), the warp maximum (redux), the lowest id holding it, and that
// lane marks the candidate taken and recomputes its score from the logit.
// Same choices, order and weights as the sorted form.
template <int EJ>
GP_DEVINL void select_topk_wide(const DecodeLayerArgs& a, const float* bias, const uint32_t (&w)[EJ], int lane,
                                int tok, bool write_out, int& my_e, float& my_w) {
    const int E = a.E, K = a.K;
    uint32_t key[EJ];
#pragma unroll
    for (int j = 0; j < EJ; ++j) {
        const int e = lane + 32 * j;
        const float sc = 1.0f / (1.0f + expf(-__uint_as_float(w[j])));
        key[j] = e < E ? order_key(sc + bias[j]) : 0u;  // 0: below every float's key (and taken)
    }
    float denom = 1e-20f, my_s = 0.f;
    my_e = 0;
    if (a.forced) {
        const int* forced = a.forced + (int64_t)tok * K;
        for (int k = 0; k < K; ++k) {
            int eb = forced[k];
            if (eb < 0 || eb >= E) {
                if (lane == 0) atomicOr(a.status, GP_DEV_BAD_EXPERT);
                eb = 0;
            }
            float lg = 0.f;
#pragma unroll
            for (int j = 0; j < EJ; ++j)
                if (lane + 32 * j == eb) lg = __uint_as_float(w[j]);
            lg = __shfl_sync(0xffffffffu, lg, eb & 31);
            const float sc = 1.0f / (1.0f + expf(-lg));
            denom += sc;  // model.cpp:718-721 order
            if (lane == k) { my_s = sc; my_e = eb; }
        }
    } else {
        for (int k = 0; k < K; ++k) {
            uint32_t bk = key[0];
            int bj = 0;
#pragma unroll
            for (int j = 1; j < EJ; ++j)
                if (key[j] > bk) { bk = key[j]; bj = j; }
            const uint32_t m = __reduce_max_sync(0xffffffffu, bk);
            const uint32_t eb = __reduce_min_sync(0xffffffffu, bk == m ? (uint32_t)(lane + 32 * bj) : 0xffffffffu);
            float lg = 0.f;
            if (lane == (int)(eb & 31u)) {
#pragma unroll
                for (int j = 0; j < EJ; ++j)
                    if (j == (int)(eb >> 5)) { lg = __uint_as_float(w[j]); key[j] = 0u; }
            }
            lg = __shfl_sync(0xffffffffu, lg, eb & 31);
            const float sc = 1.0f / (1.0f + expf(-lg));
            denom += sc;  // model.cpp:718-721 order
            if (lane == k) { my_s = sc; my_e = (int)eb; }
        }
    }
    my_w = a.norm_topk ? (my_s / denom) * a.routed_scale : my_s * a.routed_scale;
    if (write_out && a.topk_ids && lane < K) a.topk_ids[(int64_t)tok * K + lane] = my_e;
    if (write_out && a.topk_w && lane < K) a.topk_w[(int64_t)tok * K + lane] = my_w;
}

// One token's top-K from its E logits (w, one tagged word per expert lane + 32j).
template <int EJ>
GP_DEVINL void select_topk_sorted(const DecodeLayerArgs& a, const float* bias, const uint32_t (&w)[EJ], int lane,
                                  int tok, bool write_out, int& my_e, float& my_w);
template <int EJ>
GP_DEVINL void select_topk(const DecodeLayerArgs& a, const float* bias, const uint32_t (&w)[EJ], int lane, int tok,
                           bool write_out, int& my_e, float& my_w) {
    if constexpr (EJ > 8)
        select_topk_wide<EJ>(a, bias, w, lane, tok, write_out, my_e, my_w);
    else
        select_topk_sorted<EJ>(a, bias, w, lane, tok, write_out, my_e, my_w);
}

// The lane's EJ candidates sorted by (key desc, id asc), then K rounds of
// warp maxima over the lanes' heads.
template <int EJ>
GP_DEVINL void select_topk_sorted(const DecodeLayerArgs& a, const float* bias, const uint32_t (&w)[EJ], int lane,
                                  int tok, bool write_out, int& my_e, float& my_w) {
    const int E = a.E, K = a.K;
    float score[EJ];
    uint32_t key[EJ], id[EJ];
#pragma unroll
    for (int j = 0; j < EJ; ++j) {
        const int e = lane + 32 * j;
        const float lg = e < E ? __uint_as_float(w[j]) : 0.f;
        score[j] = 1.0f / (1.0f + expf(-lg));
        key[j] = e < E ? order_key(score[j] + bias[j]) : 0u;  // 0: below every float's key
        id[j] = e < E ? (uint32_t)e : 0xffffffffu;
    }
    if (lane == 0) GP_STAMP(13);
    float denom = 1e-20f, my_s = 0.f;
    my_e = 0;
    if (a.forced) {
        const int* forced = a.forced + (int64_t)tok * K;
        for (int k = 0; k < K; ++k) {
            int eb = forced[k];
            if (eb < 0 || eb >= E) {
                if (lane == 0) atomicOr(a.status, GP_DEV_BAD_EXPERT);
                eb = 0;
            }
            float sc = 0.f;
#pragma unroll
            for (int j = 0; j < EJ; ++j)
                if (lane + 32 * j == eb) sc = score[j];
            sc = __shfl_sync(0xffffffffu, sc, eb & 31);
            denom += sc;  // model.cpp:718-721 order
            if (lane == k) { my_s = sc; my_e = eb; }
        }
    } else {
        // odd-even transposition sort of the lane's candidates (EJ passes)
#pragma unroll
        for (int pass = 0; pass < EJ; ++pass) {
#pragma unroll
            for (int j = pass & 1; j + 1 < EJ; j += 2) {
                const bool sw = key[j + 1] > key[j] || (key[j + 1] == key[j] && id[j + 1] < id[j]);
                const uint32_t k0 = key[j], i0 = id[j];
                const float s0 = score[j];
                key[j] = sw ? key[j + 1] : k0;
                key[j + 1] = sw ? k0 : key[j + 1];
                id[j] = sw ? id[j + 1] : i0;
                id[j + 1] = sw ? i0 : id[j + 1];
                score[j] = sw ? score[j + 1] : s0;
                score[j + 1] = sw ? s0 : score[j + 1];
            }
        }
        for (int k = 0; k < K; ++k) {
            const uint32_t m = __reduce_max_sync(0xffffffffu, key[0]);
            const uint32_t eb = __reduce_min_sync(0xffffffffu, key[0] == m ? id[0] : 0xffffffffu);
            const float sc = __shfl_sync(0xffffffffu, score[0], eb & 31);
            if (id[0] == eb) {  // pop the head
#pragma unroll
                for (int j = 0; j + 1 < EJ; ++j) {
                    key[j] = key[j + 1];
                    id[j] = id[j + 1];
                    score[j] = score[j + 1];
                }
                key[EJ - 1] = 0u;
                id[EJ - 1] = 0xffffffffu;
            }
            denom += sc;  // model.cpp:718-721 order
            if (lane == k) { my_s = sc; my_e = (int)eb; }
        }
    }
    my_w = a.norm_topk ? (my_s / denom) * a.routed_scale : my_s * a.routed_scale;
    if (write_out && a.topk_ids && lane < K) a.topk_ids[(int64_t)tok * K + lane] = my_e;
    if (write_out && a.topk_w && lane < K) a.topk_w[(int64_t)tok * K + lane] = my_w;
}

// Slot list of a launch from the picks of its tokens: pair p = t*K + k (lane
// p, and lane p - 32 for p >= 32) holds pick (e, w) of token t.  The picks
// whose expert lies in [e_lo, e_lo + e_cnt) become routed slots in p order:
// s_se = local expert, s_st = token, s_sw = weight; s_first[t] = first slot
// of token t (s_first[n_tok] = routed slot count, also in s_nsr).
GP_DEVINL void build_slots(const DecodeLayerArgs& a, int lane, int e0, float w0, int e1, float w1, int* s_nsr,
                           int* s_first, int* s_se, int* s_st, float* s_sw) {
    const int np = a.n_tok * a.K;
    const bool in0 = lane < np && e0 >= a.e_lo && e0 < a.e_lo + a.e_cnt;
    const bool in1 = lane + 32 < np && e1 >= a.e_lo && e1 < a.e_lo + a.e_cnt;
    const uint32_t b0 = __ballot_sync(0xffffffffu, in0), b1 = __ballot_sync(0xffffffffu, in1);
    const uint32_t below = (1u << lane) - 1u;
    if (in0) {
        const int p = __popc(b0 & below);
        s_se[p] = e0 - a.e_lo;
        s_st[p] = lane / a.K;
        s_sw[p] = w0;
    }
    if (in1) {
        const int p = __popc(b0) + __popc(b1 & below);
        s_se[p] = e1 - a.e_lo;
        s_st[p] = (lane + 32) / a.K;
        s_sw[p] = w1;
    }
    if (lane <= a.n_tok) {  // slots before token `lane`: in-range pairs p < lane*K
        const int lim = lane * a.K;
        const int c0 = lim >= 32 ? __popc(b0) : __popc(b0 & ((1u << lim) - 1u));
        const int c1 = lim >= 64 ? __popc(b1) : lim > 32 ? __popc(b1 & ((1u << (lim - 32)) - 1u)) : 0;
        s_first[lane] = c0 + c1;
    }
    if (lane == 0) *s_nsr = __popc(b0) + __popc(b1);
}

// Per-stage partial sums of a gate/up tile: one per (row of the tile, covering
// warp); a row of H weights is covered by H/1024 warps.
__host__ __device__ constexpr uint32_t partial_floats_of(int H) { return 2u * TRG * (uint32_t)(H / 1024); }
static_assert(partial_floats_of(5120) == 2 * TRG * LaneMap<5120, 20, 4>::WPR &&
                  partial_floats_of(4096) == 2 * TRG * LaneMap<4096, 16, 4>::WPR,
              "partial sums per stage");

struct Smem {
    uint32_t stage_bytes, stages_off, partial_off, bar_off, misc_off, total;
};

// misc block: abort flag (16 B), routed-slot count + first slot per token (16
// ints), slot -> local expert / token / weight (3 x kDecodeMaxRouted words),
// router slices [kMaxOwned * RSPLIT][n_tok], two quantised h units (16 words +
// scale each, padded to 80 B).
__host__ __device__ inline Smem decode_smem(int H, int I, int S, int n_tok) {
    Smem L;
    const uint32_t gu = 2u * TRG * 98u * (H / 256);
    const uint32_t dn = (uint32_t)rc_of(H) * 14u;
    (void)I;
    L.stage_bytes = ((gu > dn ? gu : dn) + 15u) & ~15u;
    L.stages_off = GP_IQ3_TABLE_BYTES;
    L.partial_off = L.stages_off + S * L.stage_bytes;
    const uint32_t pb = partial_floats_of(H) * 4u;
    L.bar_off = (L.partial_off + S * pb + 15u) & ~15u;
    // 16-byte aligned: the quantised h units are read with 16-byte loads (every
    // offset inside the block below is a multiple of 16)
    L.misc_off = (L.bar_off + (3u * S + 6u) * 8u + 15u) & ~15u;
    L.total = L.misc_off + 16u + 64u + 12u * kDecodeMaxRouted + 4u * kMaxOwned * RSPLIT * n_tok + 160u;
    return L;
}

// Jobs k = c, c+G, c+2G, ... below total: count of CTA c's.
GP_DEVINL int jobs_of(int c, int G, int total) { return c < total ? (total - 1 - c) / G + 1 : 0; }

// One pipeline stage of work.  Job k of a launch, in the order: the shared
// slot's gate/up tiles (no routing needed), the routed slots' gate/up tiles,
// the shared slot's down chunks, the routed slots' down chunks.  The shared
// slot (own_tok's shared expert) covers all NU units of the expert; a routed
// slot covers the launch's UC units (all NU, or the rank's slice when every
// rank holds a slice of every routed expert).  A gate/up tile (slot, unit,
// j < TPU) gives h rows unit*32 + j*8 .. +7; a down chunk (slot, unit,
// j < NCH) adds the unit's 32 input columns into output rows j*RC .. +RC-1
// and needs the unit's 32 h rows, which tiles earlier in the order (on any
// CTA) produced.
struct Job {
    bool gu;
    int slot, unit, j;  // slot -1: the shared slot; unit: index within the slot's unit range
};
// (Every division is by a compile-time constant: the producer decodes a job
// on its critical path, sharing issue slots with the compute warps.)
template <int UC, int NU, int NCH>
GP_DEVINL Job job_of(int k, int nsr) {
    constexpr int GSS = NU * TPU, GS = UC * TPU, DSS = NU * NCH, DS = UC * NCH;  // jobs per slot, each kind
    const int cyc = GSS + GS * nsr;
    if (k < cyc) {
        if (k < GSS) return {true, -1, k / TPU, k % TPU};
        k -= GSS;
        const int si = k / GS;
        k -= si * GS;
        return {true, si, k / TPU, k % TPU};
    }
    k -= cyc;
    if (k < DSS) return {false, -1, k / NCH, k % NCH};
    k -= DSS;
    const int si = k / DS;
    k -= si * DS;
    return {false, si, k / NCH, k % NCH};
}

// Quantises the unit of h held one value per lane exactly as a lane quantises
// its activations for the GEMV (quant_i16<32>, scale * 1/4): words[w] holds
// rows 2w (low half) and 2w+1 as int16, words[16] the fp32 scale.
GP_DEVINL void quantise_unit(float v, uint32_t* words, int lane) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
    const int q = __float2int_rn(v * inv);
    const int qn = __shfl_down_sync(0xffffffffu, q, 1);
    if (!(lane & 1)) words[lane >> 1] = (static_cast<uint32_t>(q) & 0xFFFFu) | (static_cast<uint32_t>(qn) << 16);
    if (lane == 0) words[16] = __float_as_uint(0.25f * (amax * (1.0f / 32767.0f)));
}

// EP: the expert-parallel exchange over peer memory (a separate instantiation,
// so the one-GPU kernel carries none of its code).  UC: units of each routed
// slot's expert that this launch runs (NU, or NU / N when each of N ranks
// holds a slice of every routed expert).
template <int HH, int II, int PG, int RPWG, bool EP, int UC>
__global__ void __launch_bounds__(nthreads_of(HH), 1) decode_layer_kernel(const DecodeLayerArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    constexpr int H = HH, I = II;
    constexpr int NWC = nwc_of(HH), EPI = NWC, PROD = NWC + 1, RC = rc_of(HH);
    constexpr uint32_t kPartialFloats = partial_floats_of(HH);
    static_assert(HH % 1024 == 0 && LaneMap<HH, NWC, PG>::ROWSTEP == 4 && PG * 4 == 2 * TRG,
                  "4 rows of a gate/up tile per pass");
    constexpr int NU = I / UNIT, NCH = H / RC;
    constexpr uint32_t GU_BYTES = TRG * 98u * (H / 256);
    constexpr uint32_t UNIT_BYTES = (uint32_t)H * 12u;  // one column unit of W_down: qs + aux of every row
    static_assert(H % RC == 0 && GU_BYTES % 16 == 0 && (RC * 2) % 16 == 0, "bulk copies need 16-byte sizes");
    const int E = a.E, K = a.K, S = a.stages, NT = a.n_tok;
    constexpr bool ep = EP;  // expert-parallel exchange over peer memory
    const Smem L = decode_smem(H, I, S, NT);
    const uint32_t sbase = smem_u32(smem);
    // per stage: full (producer -> compute warps), pdone (compute warps ->
    // epilogue warp: partial sums written / chunk read), empty (epilogue ->
    // producer); hbar[b]: the quantised h of this CTA's down job d is in
    // s_h[b], b = d & 1
    const uint32_t full0 = sbase + L.bar_off, pdone0 = full0 + 8u * S, empty0 = pdone0 + 8u * S;
    const uint32_t tbar = empty0 + 8u * S, topk_bar = tbar + 8u, rbar = topk_bar + 8u, hbar0 = rbar + 8u;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off);
    int* s_nsr = reinterpret_cast<int*>(smem + L.misc_off + 16u);
    int* s_first = s_nsr + 1;                       // [n_tok + 1]
    int* s_se = s_nsr + 16;                         // [kDecodeMaxRouted] local expert of a slot
    int* s_st = s_se + kDecodeMaxRouted;            // token of a slot
    float* s_sw = reinterpret_cast<float*>(s_st + kDecodeMaxRouted);  // weight of a slot
    float* s_slice = s_sw + kDecodeMaxRouted;       // [task][n_tok] router slices
    uint32_t* s_h = reinterpret_cast<uint32_t*>(s_slice + kMaxOwned * RSPLIT * NT);  // [2][20]
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    constexpr uint32_t pstride = kPartialFloats;
    const uint32_t stage0 = sbase + L.stages_off;
    const int n_own = jobs_of(c, G, E);             // router experts c, c+G, ...
    const int n_tasks = n_own * RSPLIT;

    // the next kernel's CTAs may take each SM as soon as ours leaves it; they
    // wait for this grid's results before reading any of them
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(pdone0 + 8u * s, NWC);
            mbar_init(empty0 + 8u * s, 1);
        }
        mbar_init(tbar, 1);
        mbar_init(topk_bar, 1);
        mbar_init(rbar, n_tasks > 0 ? n_tasks : 1);
        mbar_init(hbar0, 1);
        mbar_init(hbar0 + 8u, 1);
        *s_abort = gp_tables_at_base(smem) ? 0u : 1u;
        if (*s_abort) atomicOr(a.status, GP_DEV_BAD_SHAPE);
        fence_mbar_init();
    }
    __syncthreads();

    // Jobs of this CTA: k = c + m*G.  Before the routing is known only the
    // shared slot's gate/up tiles (k < nsh) can be decoded; the total needs
    // the routed slot count.
    static_assert(NU % UC == 0, "a slice is a whole fraction of the units");
    constexpr int nsh = NU * TPU;
    auto routed_slots = [&]() { return min(max(*s_nsr, 0), kDecodeMaxRouted); };
    auto total_jobs = [&](int nsr) { return (NU + nsr * UC) * (TPU + NCH); };
    auto hx_row = [&](int slot) { return slot < 0 ? kDecodeMaxRouted : slot; };
    auto tok_of = [&](int slot) { return slot < 0 ? a.own_tok : s_st[slot]; };

    if (warp == PROD) {
        // ================= producer (lane 0 issues) =================
        // (Its latency per job is on the ring's critical path: it shares issue
        // slots with the compute warps, so the per-job work stays small: a
        // constant-divisor job decode, one shared-memory read, the copies.)
        if (lane == 0) {
            mbar_arrive_expect_tx(tbar, GP_IQ3_TABLE_BYTES);
            for (int k4 = 0; k4 < 4; ++k4) bulk_g2s(sbase + k4 * 16384u, a.tables + k4 * 16384, 16384u, tbar);
            int s = 0, issued = 0, n = jobs_of(c, G, nsh), nsr = 0;
            uint32_t ph = 1;
            bool have = false;  // the slot list (and so this CTA's job count) is known
            // global addresses of job m's bytes: gate/up tile, or down chunk
            // (qs, aux) of the unit's column slab and its d block
            struct Src {
                const uint8_t *p0, *p1, *p2;
            };
            auto job_src = [&](int m) -> Src {
                const Job jb = job_of<UC, NU, NCH>(c + m * G, nsr);
                const bool sh = jb.slot < 0;
                // the shared expert (whole, after the routed ones) or a routed one (a slice of UC units)
                const int e = sh ? a.e_cnt : s_se[jb.slot];
                if (jb.gu) {
                    const int64_t o = (int64_t)e * a.gu_stride + (int64_t)(jb.unit * TPU + jb.j) * GU_BYTES;
                    return {a.gate + o, a.up + o, nullptr};
                }
                // the slab holds units u_lo .. u_lo+n-1, then the d blocks from u_lo / 8 on
                const uint8_t* dc = a.down_col + (int64_t)e * a.dc_stride;
                const int ulo = sh ? 0 : a.u_lo, nun = sh ? NU : UC;
                const int dblk = ((ulo + jb.unit) >> 3) - (ulo >> 3);
                return {dc + (int64_t)jb.unit * UNIT_BYTES + (int64_t)jb.j * RC * 8,
                        dc + (int64_t)jb.unit * UNIT_BYTES + (int64_t)H * 8 + (int64_t)jb.j * RC * 4,
                        dc + (int64_t)nun * UNIT_BYTES + (int64_t)dblk * H * 2 + (int64_t)jb.j * RC * 2};
            };
            for (int m = 0;; ++m) {
                if (!have && c + m * G >= nsh) {  // routed jobs (and every down chunk) need the slot list
                    if (!mbar_wait(topk_bar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); break; }
                    GP_STAMP(10);
                    nsr = routed_slots();
                    n = jobs_of(c, G, total_jobs(nsr));
                    have = true;
                }
                if (m >= n) break;
                const Src r = job_src(m);
                if (!mbar_wait(empty0 + 8u * s, ph, a.spin_limit)) {
                    *s_abort = 1;
                    atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
                    break;
                }
                const uint32_t dst = stage0 + s * L.stage_bytes, bar = full0 + 8u * s;
                if (r.p2 == nullptr) {
                    mbar_arrive_expect_tx(bar, 2u * GU_BYTES);
                    bulk_g2s(dst, r.p0, GU_BYTES, bar);
                    bulk_g2s(dst + GU_BYTES, r.p1, GU_BYTES, bar);
                } else {
                    mbar_arrive_expect_tx(bar, (uint32_t)RC * 14u);
                    bulk_g2s(dst, r.p0, RC * 8u, bar);
                    bulk_g2s(dst + RC * 8u, r.p1, RC * 4u, bar);
                    bulk_g2s(dst + RC * 12u, r.p2, RC * 2u, bar);
                }
                ++issued;
                if (++s == S) { s = 0; ph ^= 1u; }
            }
            // no copy may still be in flight when the CTA exits (the
            // compile-time limit, whatever the run-time one)
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                mbar_wait(full0 + 8u * (i % S), (uint32_t)(i / S) & 1u);
            mbar_wait(tbar, 0);
        }
        return;
    }

    if (warp == EPI) {
        // ================= routing, then the gate/up epilogues and h fetches =================
        // top-k candidates per lane: E <= 32 * EJ (the reference model's 288 experts at H = 4096)
        constexpr int EJ = HH == 4096 ? kMaxEFused / 32 : 8;
        float bias[EJ];
#pragma unroll
        for (int j = 0; j < EJ; ++j) bias[j] = a.corr && lane + 32 * j < E ? __ldg(a.corr + lane + 32 * j) : 0.f;
        pdl_wait();
        const uint32_t tag = ld_relaxed(a.sync + kSyncGen) + 1u;
        const uint32_t ep_tag = ep ? ld_relaxed(a.ep_sync) + 1u : 0u;
        // exchange words per token, and per CTA's share (even: 16-byte pairs)
        const int ep_nw = a.x_bf16 ? H / 2 : H, ep_wpc = (((ep_nw + G - 1) / G) + 1) & ~1;
        if (ep) {
            // this CTA's share of this rank's token to every rank (no fence:
            // the words carry the step's tag)
            const uint32_t* xw = static_cast<const uint32_t*>(a.x);
            const int w_end = min(ep_nw, (c + 1) * ep_wpc);
            for (int w = c * ep_wpc + 2 * lane; w < w_end; w += 64) {  // (ep_nw and ep_wpc are even)
                const unsigned long long v0 = ((unsigned long long)ep_tag << 32) | xw[w];
                const unsigned long long v1 = ((unsigned long long)ep_tag << 32) | xw[w + 1];
                for (int r = 0; r < a.ep_world; ++r)
                    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};"
                                 ::"l"(a.ep_x_peer[r] + (int64_t)a.ep_rank * H + w), "l"(v0), "l"(v1) : "memory");
            }
        }
        {   // this CTA's share of y = 0, ordered before its logits are published
            float4* y4 = reinterpret_cast<float4*>(a.y);
            for (int i = c * 32 + lane; i < NT * H / 4; i += G * 32) y4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            fence_acq_rel_gpu();
        }
        if (n_tasks > 0) {  // this CTA's experts: slices added in order
            if (!mbar_wait(rbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            if (lane < n_own) {
                const int e = c + lane * G;
                for (int t = EP ? a.ep_rank : 0; t < (EP ? a.ep_rank + 1 : NT); ++t) {  // (EP: its own token)
                    float lg = 0.f;
#pragma unroll
                    for (int sl = 0; sl < RSPLIT; ++sl) lg += s_slice[(lane * RSPLIT + sl) * NT + t];
                    const unsigned long long v = ((unsigned long long)tag << 32) | __float_as_uint(lg);
                    if (e == a.withhold_logit) continue;  // (a test withholds one to make the top-k wait run out)
#pragma unroll
                    for (int cp = 0; cp < kLogitCopies; ++cp) st_relaxed64(a.logits + logit_word(cp, t, e, E), v);
                }
            }
        }
        int e0 = 0, e1 = 0;
        float w0 = 0.f, w1 = 0.f;
        bool ok = true;
        if constexpr (EP) {
            // this rank's token only (every CTA picks its experts itself from
            // the local logits); CTA 0 sends the picks to every rank, and
            // every CTA reads the other tokens' picks from its rank's ep_pk
            const int own = a.ep_rank;
            int me = 0;
            float mw = 0.f;
            ok = E <= 160 ? topk_token<5>(a, bias, tag, lane, c % kLogitCopies, own, c == 0, me, mw)
                          : topk_token<EJ>(a, bias, tag, lane, c % kLogitCopies, own, c == 0, me, mw);
            if (c == 0 && lane < K) {
                const unsigned long long v0 = ((unsigned long long)ep_tag << 32) | (uint32_t)me;
                const unsigned long long v1 = ((unsigned long long)ep_tag << 32) | __float_as_uint(mw);
                for (int r = 0; r < a.ep_world; ++r)
                    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};"
                                 ::"l"(a.ep_pk_peer[r] + ((int64_t)own * 32 + lane) * 2), "l"(v0), "l"(v1) : "memory");
            }
            // pair p = t*K + k on lane p (and p - 32): this token's by shuffle, the others polled
            const int np = NT * K;
            const int t0 = lane / K, k0 = lane - t0 * K, t1 = (lane + 32) / K, k1 = lane + 32 - t1 * K;
            const int oe0 = __shfl_sync(0xffffffffu, me, k0), oe1 = __shfl_sync(0xffffffffu, me, k1);
            const float ow0 = __shfl_sync(0xffffffffu, mw, k0), ow1 = __shfl_sync(0xffffffffu, mw, k1);
            const bool r0 = lane < np && t0 != own, r1 = lane + 32 < np && t1 != own;
            if (lane < np && !r0) { e0 = oe0; w0 = ow0; }
            if (lane + 32 < np && !r1) { e1 = oe1; w1 = ow1; }
            for (uint32_t n = 0;; ++n) {
                bool got = true;
                if (r0) {
                    unsigned long long v0, v1;
                    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                                 : "=l"(v0), "=l"(v1) : "l"(a.ep_pk + ((int64_t)t0 * 32 + k0) * 2) : "memory");
                    got &= (uint32_t)(v0 >> 32) == ep_tag && (uint32_t)(v1 >> 32) == ep_tag;
                    e0 = (int)(uint32_t)v0;
                    w0 = __uint_as_float((uint32_t)v1);
                }
                if (r1) {
                    unsigned long long v0, v1;
                    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                                 : "=l"(v0), "=l"(v1) : "l"(a.ep_pk + ((int64_t)t1 * 32 + k1) * 2) : "memory");
                    got &= (uint32_t)(v0 >> 32) == ep_tag && (uint32_t)(v1 >> 32) == ep_tag;
                    e1 = (int)(uint32_t)v0;
                    w1 = __uint_as_float((uint32_t)v1);
                }
                if (__all_sync(0xffffffffu, got)) break;
                if (n >= a.spin_limit) {
                    ok = false;
                    break;
                }
                __nanosleep(n < 2 ? 64u << n : 256u);
            }
            if (c == 0) {  // (ids outside [0, E) after a timeout are dropped by build_slots)
                if (r0 && a.topk_ids) a.topk_ids[lane] = e0;
                if (r0 && a.topk_w) a.topk_w[lane] = w0;
                if (r1 && a.topk_ids) a.topk_ids[lane + 32] = e1;
                if (r1 && a.topk_w) a.topk_w[lane + 32] = w1;
            }
        } else if (NT == 1) {  // every CTA picks the token's experts itself
            ok = E <= 160 ? topk_token<5>(a, bias, tag, lane, c % kLogitCopies, 0, c == 0, e0, w0)
                          : topk_token<EJ>(a, bias, tag, lane, c % kLogitCopies, 0, c == 0, e0, w0);
        } else {
            // every CTA picks every token's experts itself (no second exchange
            // of picks); lane k of token t leaves pick k in the free router
            // slice area, then pair p = t*K + k goes to lane p (p < 32) or p-32
            int* s_pe = reinterpret_cast<int*>(s_slice);
            float* s_pw = s_slice + kDecodeMaxRouted;
            for (int t = 0; t < NT; ++t) {
                uint32_t w[EJ], w2[EJ];
                ok &= poll_logits<EJ>(a, tag, lane, c % kLogitCopies, t, -1, w, w2);
                int me = 0;
                float mw = 0.f;
                select_topk<EJ>(a, bias, w, lane, t, c == 0, me, mw);
                if (lane < K) {
                    s_pe[t * K + lane] = me;
                    s_pw[t * K + lane] = mw;
                }
            }
            __syncwarp();
            const int np = NT * K;
            if (lane < np) {
                e0 = s_pe[lane];
                w0 = s_pw[lane];
            }
            if (lane + 32 < np) {
                e1 = s_pe[lane + 32];
                w1 = s_pw[lane + 32];
            }
        }
        if (!ok && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        // (after a timeout the slot list is built from whatever was read: the
        // ids stay in range, the results are invalid and the status says so)
        build_slots(a, lane, e0, w0, e1, w1, s_nsr, s_first, s_se, s_st, s_sw);
        __syncwarp();
        if (lane == 0) mbar_arrive(topk_bar);  // release: the other roles read the slot list
        GP_STAMP(2);
        // Acquire: the other CTAs zeroed their parts of y before publishing the
        // logits (or picks) read above.  Every reduction into y comes from a
        // down job, whose h this warp hands over (hbar) only after this fence;
        // the slot list above needs no such order.
        fence_acq_rel_gpu();

        const int nsr = routed_slots();
        const int n = jobs_of(c, G, total_jobs(nsr));
        int s = 0, fm = 0, d = 0;
        uint32_t ph = 0;
        constexpr int rsg = 32 * NWC / (H / 32);
        // h of down job at position fm into s_h[d & 1]: its 32 tagged rows
        // (published by the gate/up tiles of that unit), quantised as a lane
        // quantises its activations.  Fetched one stage ahead of its use.
        auto fetch_h = [&](const Job& jb) -> bool {
            const unsigned long long* src = a.hx + (int64_t)hx_row(jb.slot) * I + jb.unit * UNIT + lane;
            unsigned long long w = 0ull;
            uint32_t k = 0;
            for (; k < a.spin_limit; ++k) {
                w = ld_relaxed64(src);
                if (__all_sync(0xffffffffu, (uint32_t)(w >> 32) == tag)) break;
                __nanosleep(TOPK_POLL_NS);
            }
            quantise_unit(__uint_as_float((uint32_t)w), s_h + (d & 1) * 20, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(hbar0 + 8u * (d & 1));
            ++d;
            return k < a.spin_limit;
        };
        // A warp whose bounded wait runs out records it and leaves its loop
        // (arriving on no further barrier, so no barrier phase sees arrivals
        // from two iterations); the waits it leaves other warps in run out
        // in turn.  Decisions are warp-uniform (votes over the lanes' waits).
        for (int m = 0; m < n; ++m) {
            // the h of the down jobs at positions m and m+1, in order: the
            // buffer of down job d was last read by down job d-2, whose stage
            // (two down jobs back, so before position m) this warp has seen done
            bool fetched = true;
            const Job jb = job_of<UC, NU, NCH>(c + m * G, nsr);
            for (; fm <= m + 1 && fm < n && fetched; ++fm) {
                const Job fj = job_of<UC, NU, NCH>(c + fm * G, nsr);
                if (fj.gu) continue;
                // (not ahead of this CTA's own tile of the same unit, whose h
                // this warp publishes only below)
                if (fm == m + 1 && jb.gu && jb.slot == fj.slot && jb.unit == fj.unit) break;
                fetched = fetch_h(fj);
            }
            if (!fetched) {
                if (lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                break;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(pdone0 + 8u * s, ph, a.spin_limit))) {
                if (lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                break;
            }
            float val = 0.f;
            if (jb.gu && lane < TRG) {  // partials in warp order (LaneMap layout)
                using LG = LaneMap<HH, NWC, PG>;
                const float* pbuf = partial + (size_t)s * pstride;
                const int row = lane, ur = TRG + row;
                const int ng = LG::last_warp(row % rsg) - LG::first_warp(row % rsg);
                const int nu = LG::last_warp(ur % rsg) - LG::first_warp(ur % rsg);
                // every partial loaded at once (independent loads), then added in warp order
                float gp[LG::WPR], up[LG::WPR];
#pragma unroll
                for (int ww = 0; ww < LG::WPR; ++ww) {
                    gp[ww] = ww <= ng ? pbuf[row * LG::WPR + ww] : 0.f;
                    up[ww] = ww <= nu ? pbuf[ur * LG::WPR + ww] : 0.f;
                }
                float gs = 0.f, us = 0.f;
#pragma unroll
                for (int ww = 0; ww < LG::WPR; ++ww) {
                    gs += gp[ww];
                    us += up[ww];
                }
                val = silu_clamped(gs, us, a.limit);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8u * s);  // stage read: it may refill
            if (++s == S) { s = 0; ph ^= 1u; }
            if (jb.gu && lane < TRG) {  // h rows of the tile, tagged: the data is its own flag
                unsigned long long* dst = a.hx + (int64_t)hx_row(jb.slot) * I + jb.unit * UNIT + jb.j * TRG + lane;
                st_relaxed64(dst, ((unsigned long long)tag << 32) | __float_as_uint(val));
            }
        }
    } else {
        // ================= compute warps =================
        // router weights of this warp's first slice: independent of the
        // previous kernel, so loaded before waiting for it
        constexpr int RSL = H / RSPLIT, RV = RSL / 128;
        static_assert(H % (RSPLIT * 128) == 0 && RV <= 8, "router slices are whole float4 columns");
        float4 wv[RV];
        auto load_router = [&](int task) {
            const float* wr = a.router + (int64_t)(c + (task / RSPLIT) * G) * H + (task % RSPLIT) * RSL + lane * 4;
#pragma unroll
            for (int i = 0; i < RV; ++i) wv[i] = __ldg(reinterpret_cast<const float4*>(wr + i * 128));
        };
        if (warp < n_tasks) load_router(warp);
        pdl_wait();
        const uint32_t ep_tag = ep ? ld_relaxed(a.ep_sync) + 1u : 0u;
        bool xok = true;  // the exchange's words arrived (expert-parallel)

        // ---- router slices of this CTA's experts: warp task = (expert, slice),
        // one dot product per token ----
        for (int task = warp; task < n_tasks; task += NWC) {
            if (task != warp) load_router(task);
            const int sl = task % RSPLIT;
            if constexpr (!EP) {
                for (int t = 0; t < NT; ++t) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < RV; ++i) {
                        const float4 xv = x4_of(a, t, sl * RSL + lane * 4 + i * 128);
                        acc = fmaf(wv[i].x, xv.x, acc);
                        acc = fmaf(wv[i].y, xv.y, acc);
                        acc = fmaf(wv[i].z, xv.z, acc);
                        acc = fmaf(wv[i].w, xv.w, acc);
                    }
                    acc = warp_sum(acc);
                    if (lane == 0) s_slice[task * NT + t] = acc;
                }
            } else {  // this rank's own token (row 0 of x): the others' are routed on their ranks
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < RV; ++i) {
                    const float4 xv = x4_of(a, 0, sl * RSL + lane * 4 + i * 128);
                    acc = fmaf(wv[i].x, xv.x, acc);
                    acc = fmaf(wv[i].y, xv.y, acc);
                    acc = fmaf(wv[i].z, xv.z, acc);
                    acc = fmaf(wv[i].w, xv.w, acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) s_slice[task * NT + a.ep_rank] = acc;
            }
            if (lane == 0) mbar_arrive(rbar);
        }

        if (!mbar_wait(tbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        const auto mg = lane_map<HH, NWC, PG>(warp, lane, stage0);
        const int gl = warp * 32 + lane;  // this lane's rows of a down chunk: 4gl .. 4gl+3
        uint32_t xq[16], hq[16];
        int cur = -1;  // the token whose activations xq holds
        float sx4 = 0.f, hs = 0.f;
        int s = 0, n = jobs_of(c, G, nsh), nsr = 0, d = 0;
        uint32_t ph = 0;
        bool have = false;
        auto give_up = [&]() {
            if (lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        };
        for (int m = 0;; ++m) {
            if (!have && c + m * G >= nsh) {  // routed jobs (and every down chunk) come after the routing
                if (!__all_sync(0xffffffffu, mbar_wait(topk_bar, 0, a.spin_limit))) { give_up(); break; }
                nsr = routed_slots();
                n = jobs_of(c, G, total_jobs(nsr));
                have = true;
            }
            if (m >= n) break;
            const Job jb = job_of<UC, NU, NCH>(c + m * G, nsr);
            const int tok = tok_of(jb.slot);
            if (jb.gu) {
                if (tok != cur) {  // that token's activations
                    cur = tok;
                    if (ep && cur != a.ep_rank) {  // another rank's token: from the exchange
                        float v[32];
                        ep_x32(a, cur, 32 * mg.sb, ep_tag, v, xok);
                        sx4 = 0.25f * quant_i16<32>(v, xq);
                        if (!__all_sync(0xffffffffu, xok)) { give_up(); break; }
                    } else {  // (expert-parallel: this rank's own token is row 0 of x)
                        sx4 = load_quant(a.x, a.x_bf16, ep ? 0 : cur, H, mg.sb, xq);
                    }
                }
                if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8u * s, ph, a.spin_limit))) { give_up(); break; }
                consume<HH, NWC, PG, RPWG>(mg, s * L.stage_bytes, xq, sx4, partial + (size_t)s * pstride, warp, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(pdone0 + 8u * s);
            } else {
                // the unit's quantised h (double-buffered by down-job parity)
                if (!__all_sync(0xffffffffu, mbar_wait(hbar0 + 8u * (d & 1), (uint32_t)(d >> 1) & 1u, a.spin_limit))) {
                    give_up();
                    break;
                }
                const uint32_t hb = smem_u32(s_h + (d & 1) * 20);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = lds128(hb + 16u * i);
                    hq[4 * i] = v.x;
                    hq[4 * i + 1] = v.y;
                    hq[4 * i + 2] = v.z;
                    hq[4 * i + 3] = v.w;
                }
                hs = ldsf(hb + 64u);
                ++d;
                if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8u * s, ph, a.spin_limit))) { give_up(); break; }
                // split-K down: rows 4gl .. 4gl+3 of chunk j, this unit's 32 input columns
                const uint32_t sb = stage0 + s * L.stage_bytes;
                const uint4 q01 = lds128(sb + 32u * gl), q23 = lds128(sb + 32u * gl + 16u);
                const uint4 ax = lds128(sb + RC * 8u + 16u * gl);
                const uint2 dd = lds64(sb + RC * 12u + 8u * gl);
                float v[4];
                uint32_t sw[8];
                const uint32_t qa[4] = {q01.x, q01.z, q23.x, q23.z}, qb[4] = {q01.y, q01.w, q23.y, q23.w};
                const uint32_t aw[4] = {ax.x, ax.y, ax.z, ax.w}, dw[4] = {dd.x & 0xFFFFu, dd.x >> 16, dd.y & 0xFFFFu, dd.y >> 16};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    iq3_decode_sub32(nullptr, qa[r], qb[r], aw[r], lane * 4u, sw);
                    const float dr = __half2float(__ushort_as_half((unsigned short)dw[r]));
                    v[r] = (float)(iq3_idot<8>(sw, hq) * iq3_oddscale(aw[r])) * (dr * hs);
                }
                // the stage is read: release it first, then send the sums
                __syncwarp();
                if (lane == 0) mbar_arrive(pdone0 + 8u * s);
                const float wk = jb.slot < 0 ? 1.0f : s_sw[jb.slot];
                red_add_v4(a.y + (int64_t)tok * H + jb.j * RC + 4 * gl, wk * v[0], wk * v[1], wk * v[2], wk * v[3]);
            }
            if (++s == S) { s = 0; ph ^= 1u; }
        }
    }

    // The last CTA out advances the launch generation (the tag of the next
    // launch's exchanged words).  Expert-parallel, the last CTA first adds
    // every token's partial output into that token's owner's accumulator of
    // this step's parity over NVLink (one 16-byte add per 4 values: far less
    // traffic than sending every down job's sums), then (one system-scope
    // fence) tells every other rank that this rank's sums are in, waits for
    // every other rank's signal to this one, copies this rank's accumulator to
    // ep_out and zeroes it: no rank adds into it again before this rank's next
    // signal.
    named_bar_sync(1, (NWC + 1) * 32);
    if constexpr (!EP) {
        if (tid == 0) {
            fence_acq_rel_gpu();
            if (atomicAdd(a.sync + kSyncEnd, 1u) == (unsigned)G - 1) {
                a.sync[kSyncGen] += 1u;
                fence_acq_rel_gpu();
                a.sync[kSyncEnd] = 0;
            }
        }
        return;
    } else {
        volatile uint32_t* s_last = s_abort + 1;
        if (tid == 0) {
            fence_acq_rel_gpu();
            *s_last = atomicAdd(a.sync + kSyncEnd, 1u) == (unsigned)G - 1 ? 1u : 0u;
            if (*s_last) fence_acq_rel_gpu();  // every CTA's sums into y are in
        }
        named_bar_sync(1, (NWC + 1) * 32);
        if (*s_last) {
            const uint32_t g = ld_relaxed(a.ep_sync);
            const int64_t par = (int64_t)(g & 1u) * H;
            for (int i = tid; i < NT * (H / 4); i += (NWC + 1) * 32) {  // y[t] into owner t's accumulator
                const int t = i / (H / 4), q = i % (H / 4);
                const float4 v = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)t * H) + q);
                red_add_sys_v4(a.ep_y[t] + par + 4 * q, v.x, v.y, v.z, v.w);
            }
            named_bar_sync(1, (NWC + 1) * 32);
            if (tid == 0) {
                fence_acq_rel_sys();
                for (int r = 0; r < a.ep_world; ++r)
                    if (r != a.ep_rank) red_release_sys_add64(a.ep_done[r], 1ull);
                const unsigned long long target = (unsigned long long)(a.ep_world - 1) * (unsigned long long)(g + 1u);
                for (uint32_t n = 0; ld_acquire_sys64(a.ep_done[a.ep_rank]) < target; ++n) {
                    if (n >= a.spin_limit) {
                        atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            named_bar_sync(1, (NWC + 1) * 32);
            // this rank's token: out = its accumulator, which then starts step g + 2 at zero
            float4* ys4 = reinterpret_cast<float4*>(a.ep_y[a.ep_rank] + par);
            float4* y4 = reinterpret_cast<float4*>(a.ep_out);
            for (int i = tid; i < H / 4; i += (NWC + 1) * 32) {
                y4[i] = __ldcg(ys4 + i);
                ys4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            named_bar_sync(1, (NWC + 1) * 32);
            if (tid == 0) {
                a.ep_sync[0] = g + 1u;
                a.sync[kSyncGen] += 1u;
                fence_acq_rel_gpu();
                a.sync[kSyncEnd] = 0;
            }
        }
    }
}

}  // namespace

// Instantiated shapes: (H, I) = (5120, 1536) with up to 256 routed experts
// (the BASELINE layer) and (4096, 2048) with up to 512 (the reference
// model's default MoE shape, model_config.h:25, 59-60: 288 experts).
static int max_experts_of(int H, int I) {
    if (H == 5120 && I == 1536) return 256;
    if (H == 4096 && I == 2048) return kMaxEFused;
    return 0;
}

bool decode_layer_slice_supported(int I, int u_cnt) {
    const int nu = I / UNIT;
    return (I == 1536 || I == 2048) && (u_cnt == nu || u_cnt == nu / 2 || u_cnt == nu / 4 || u_cnt == nu / 8);
}

bool decode_layer_supported(int H, int I, int E, int K, int with_shared) {
    if (E > max_experts_of(H, I) || E < K) return false;
    // gate/up: H/256 compute warps over 4 rows of H per pass; down chunks of H/2 rows
    return K >= 1 && K <= MAXK && with_shared == 1;
}

size_t decode_layer_smem(int H, int I, int stages, int n_tok) { return decode_smem(H, I, stages, n_tok).total; }

cudaError_t launch_decode_layer(const DecodeLayerArgs& a, int grid, cudaStream_t st) {
    if (!decode_layer_supported(a.H, a.I, a.E, a.K, a.with_shared)) return cudaErrorInvalidValue;
    if (grid * kMaxOwned < a.E) return cudaErrorInvalidValue;  // router experts per CTA
    if (a.n_tok < 1 || a.n_tok > kDecodeMaxTokens || a.n_tok * a.K > kDecodeMaxRouted || a.own_tok < 0 ||
        a.own_tok >= a.n_tok || a.e_lo < 0 || a.e_cnt < 0 || a.e_lo + a.e_cnt > a.E || a.E >= 65536 ||
        !a.down_col || (reinterpret_cast<uintptr_t>(a.y) & 15))
        return cudaErrorInvalidValue;
    if (a.n_tok == 1 && (a.e_lo != 0 || a.e_cnt != a.E)) return cudaErrorInvalidValue;  // one token: every expert
    if (a.u_cnt && a.u_cnt != a.I / UNIT && (a.e_lo != 0 || a.e_cnt != a.E))
        return cudaErrorInvalidValue;  // a slice of every routed expert
    if (a.ep_world > 1) {  // the peer-memory exchange: one token per rank, every rank's block mapped
        if (a.ep_world > kDecodeMaxTokens || a.n_tok != a.ep_world || a.ep_rank < 0 || a.ep_rank >= a.ep_world ||
            a.own_tok != a.ep_rank || !a.ep_x || !a.ep_sync || !a.ep_out || !a.ep_pk || a.K > 32 ||
            ((reinterpret_cast<uintptr_t>(a.ep_out) | reinterpret_cast<uintptr_t>(a.ep_x) |
              reinterpret_cast<uintptr_t>(a.ep_pk)) & 15))
            return cudaErrorInvalidValue;
        // (16-byte pair stores and loads of tagged words, 16-byte adds)
        for (int r = 0; r < a.ep_world; ++r)
            if (!a.ep_x_peer[r] || !a.ep_y[r] || !a.ep_done[r] || !a.ep_pk_peer[r] ||
                ((reinterpret_cast<uintptr_t>(a.ep_y[r]) | reinterpret_cast<uintptr_t>(a.ep_x_peer[r]) |
                  reinterpret_cast<uintptr_t>(a.ep_pk_peer[r])) & 15) ||
                (reinterpret_cast<uintptr_t>(a.ep_done[r]) & 7))
                return cudaErrorInvalidValue;
    }
    const Smem L = decode_smem(a.H, a.I, a.stages, a.n_tok);
    if (L.total > 227u * 1024u) return cudaErrorInvalidValue;
    const bool ep = a.ep_world > 1;
    const int uc = a.u_cnt ? a.u_cnt : a.I / UNIT;
    if (a.u_lo < 0 || a.u_lo + uc > a.I / UNIT || (a.u_lo % uc)) return cudaErrorInvalidValue;
    // instantiations: (exchange, units per slot)
    using Kern = void (*)(const DecodeLayerArgs);
    Kern kern = nullptr;
    int ki = -1;
    if (a.H == 5120) {
        constexpr int kH = 5120, kI = 1536;
        if (!ep && uc == 48) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 48>; ki = 0; }
        else if (!ep && uc == 24) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 24>; ki = 1; }
        else if (!ep && uc == 12) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 12>; ki = 2; }
        else if (!ep && uc == 6) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 6>; ki = 3; }
        else if (ep && uc == 48) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 48>; ki = 4; }
        else if (ep && uc == 24) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 24>; ki = 5; }
        else if (ep && uc == 12) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 12>; ki = 6; }
        else if (ep && uc == 6) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 6>; ki = 7; }
    } else {
        constexpr int kH = 4096, kI = 2048;
        if (!ep && uc == 64) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 64>; ki = 8; }
        else if (!ep && uc == 32) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 32>; ki = 9; }
        else if (!ep && uc == 16) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 16>; ki = 10; }
        else if (!ep && uc == 8) { kern = decode_layer_kernel<kH, kI, 4, 1, false, 8>; ki = 11; }
        else if (ep && uc == 64) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 64>; ki = 12; }
        else if (ep && uc == 32) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 32>; ki = 13; }
        else if (ep && uc == 16) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 16>; ki = 14; }
        else if (ep && uc == 8) { kern = decode_layer_kernel<kH, kI, 4, 1, true, 8>; ki = 15; }
    }
    if (!kern) return cudaErrorInvalidValue;
    const int nthreads = nthreads_of(a.H);
    static std::atomic<unsigned long long> configured[16] = {};  // per device, per instantiation
    if (cudaError_t e0 = raise_smem_limit(kern, 227 * 1024, configured[ki])) return e0;
    // Co-residency: every CTA waits on data the others publish, so the grid
    // must fit the GPU at one CTA per SM.  Checked against the kernel's real
    // resource use (registers, shared memory) once per device; a grid larger
    // than the SMs that can hold a CTA is refused rather than left to time out.
    static std::atomic<unsigned long long> fits_all[16] = {};
    std::atomic<unsigned long long>& fits = fits_all[ki];
    int dev = 0;
    if (cudaError_t e1 = cudaGetDevice(&dev)) return e1;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (!bit || !(fits.load(std::memory_order_acquire) & bit)) {
        int per_sm = 0, sms = 0;
        if (cudaError_t e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, nthreads, 227 * 1024))
            return e2;
        if (cudaError_t e3 = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) return e3;
        if (per_sm < 1 || grid > sms * per_sm) return cudaErrorCooperativeLaunchTooLarge;
        if (bit) fits.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(nthreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    // One CTA per SM, all resident at once.  The default launch lets this
    // grid's CTAs take SMs as the previous kernel's leave (programmatic
    // dependent launch), which hides the launch gap between layers; it relies
    // on no other kernel holding SMs meanwhile (a concurrent kernel only
    // delays the waits, which are bounded).  A cooperative launch guarantees
    // co-residency instead, but the driver then starts the grid only after
    // the previous kernel has finished.
    cudaLaunchAttribute attr[1];
    if (a.cooperative) {
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    return e;
}

}  // namespace gp
