// One MoE layer at batch 1 in a single persistent kernel
// (reference Model::moe_forward, cpp/core/src/model.cpp:692-756).
//
// Separate kernels for router, routing, gate/up, down and combine each pay a
// launch, a prologue (decode tables, first bytes in flight) and a tail, which
// at batch 1 costs more than streaming the 85 MB of weights.  Here one CTA per
// SM runs the whole layer.  Warp roles: 24 compute warps, one TMA producer
// warp streaming weight tiles through a ring of shared-memory stages, and one
// epilogue warp that does the routing and turns each stage's partial sums
// into results.  Under full HBM load a round trip to L2 costs microseconds
// (more from the other die), so the design keeps those out of the per-tile
// path: no atomics are read back, and values other CTAs produced are read as
// words tagged with the launch generation (the data is its own flag).
//
// The same kernel runs one rank's share of an expert-parallel decode step:
// n_tok tokens (one per rank), the routed experts of one range, the shared
// expert of the rank's own token.  Its slots are then the (token, expert)
// picks that fall in the range, and it writes each token's partial output
// (the ranks' parts sum to the layer).  One token with every expert is the
// batch-1 layer, with the same arithmetic in the same order.
//
//   router   CTA c owns experts c, c+G, ...; 8 warps each compute one 1/8
//            slice of an owned expert's fp32 logit for every token (weights
//            prefetched before the wait on the previous kernel); the
//            epilogue warp adds the slices in order and stores the logit
//            tagged with the launch generation, so readers poll the data itself
//   top-k    one token: every CTA's epilogue warp polls the E tagged logits
//            (one of 8 replicas, spread over L2 lines), applies
//            sigmoid + bias and picks top-K by warp reductions (ties to the
//            lower id), weights score/(1e-20 + sum)*scale (model.cpp:704-725).
//            Several tokens: CTA t picks token t's experts and publishes the
//            picks as tagged words that every CTA then reads.  The picks in
//            the launch's expert range become its slots
//   gate/up  units of 32 rows of h, dealt round-robin in slot order (the
//            shared expert first: it needs no routing; then the routed slots
//            in pick order); a unit is 4 consecutive tiles of 8 rows of
//            gate and up.  The epilogue applies SwiGLU with the reference clamp
//            (model.cpp:733-739), quantises the finished unit to int16 (hq)
//            and counts it for its slot: no value of h leaves the CTA
//            unquantised and no counter is read back
//   down     tiles of 32 rows x all slots, a contiguous range of (tile,
//            slot) positions per CTA sized to even out the total work; the
//            producer copies each tile with its slot's hq once all units of
//            that slot are counted (model.cpp:740).  The epilogue keeps a row
//            tile's slot results in shared memory and writes y = sum_k w_k
//            D[k] + D[shared] in top-k order per token (model.cpp:741-755); for a tile
//            shared with the next CTAs it reads their slots as tagged words
//
// Waits on other CTAs need every CTA resident: one CTA per SM, launched either
// with programmatic dependent launch (default) or cooperatively.  Every wait
// is bounded; a timeout sets a status bit, the CTA stops waiting and finishes
// (results then invalid, the host reports the status and clears the
// counters and tags).
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

constexpr int NWC = 24;          // compute warps
constexpr int NWG = 20;          // of which compute gate/up (32*20 lanes = 4 rows of 5120)
constexpr int EPI = NWC;         // epilogue warp
constexpr int PROD = NWC + 1;    // TMA producer warp
constexpr int NTHREADS = 32 * (NWC + 2);
constexpr int TRG = 8;           // gate/up rows per matrix per tile
constexpr int TRD = 32;          // down rows per tile (one per epilogue lane)
constexpr int UNIT = 32;         // activation quantisation unit = rows of h per gate/up unit
constexpr int TPU = UNIT / TRG;  // gate/up tiles per unit
constexpr int RSPLIT = 8;        // router slices per expert
constexpr int MAXK = 31;         // K+1 slots fit one warp
constexpr int kMaxEFused = 256;  // routed experts handled by the top-k warp
constexpr int kMaxOwned = 8;     // router experts per CTA (grid >= E/8)
// Tagged logits: every CTA polls all E of them, so one array would send every
// poll of every CTA to the few L2 slices holding it.  Each logit is stored in
// kLogitCopies replicas, one word per 256-byte line; CTA c polls replica
// c % kLogitCopies.
constexpr int kLogitCopies = 8;
constexpr int kLogitStride = 32;  // words
static_assert(kLogitCopies * kLogitStride == 256, "decode_layer_logit_words (kernels.h) assumes 8 x 32");
static_assert(TRD == 32, "the combine maps one row of a down tile to each epilogue lane");


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

// Sentinel slot id of the shared expert in work items (its storage index is
// kSharedStore; its position among a down tile's values is the routed count).
constexpr int kShared = -1;
constexpr int kSharedStore = kDecodeMaxRouted;
GP_DEVINL int slot_store(int slot) { return slot < 0 ? kSharedStore : slot; }

// Tagged logit of token `tok`, expert e: one token is read by every CTA and
// kept in kLogitCopies replicas (copy = reader's CTA % kLogitCopies); with
// several tokens only CTA t reads token t's, one copy (copy 0).
GP_DEVINL int64_t logit_word(int copy, int tok, int e, int E) {
    return ((int64_t)(copy + tok) * E + e) * kLogitStride;
}
// Tagged top-k pick k of token t (several tokens), kLogitCopies replicas.
GP_DEVINL int64_t pick_word(int copy, int tok, int k) {
    return ((int64_t)(copy * kDecodeMaxTokens + tok) * 32 + k) * kLogitStride;
}

// One token's top-K by score + bias (ties to the lower id), weights
// score/(1e-20 + sum)*scale (model.cpp:704-725), or the forced ids with their
// weights.  The E logits are polled as words tagged by their writers with this
// launch's tag: the data is its own flag, so one poll round trip suffices.
// Each lane sorts its EJ candidates (expert ids lane + 32j) by (key desc, id
// asc); a round then takes the warp maximum of the lanes' head keys (redux),
// the lowest id holding it, and that lane pops its head.  Lane k < K returns
// pick k in (my_e, my_w).  Returns false when the wait for the logits ran out.
template <int EJ>
GP_DEVINL bool topk_token(const DecodeLayerArgs& a, const float* bias, uint32_t tag, int lane, int copy, int tok,
                          bool write_out, int& my_e, float& my_w) {
    const int E = a.E, K = a.K;
    unsigned long long w[EJ];
    uint32_t n = 0;
    for (; n < a.spin_limit; ++n) {
#pragma unroll
        for (int j = 0; j < EJ; ++j)
            w[j] = lane + 32 * j < E ? ld_relaxed64(a.logits + logit_word(copy, tok, lane + 32 * j, E)) : 0ull;
        bool ok = true;
#pragma unroll
        for (int j = 0; j < EJ; ++j) ok &= lane + 32 * j >= E || (uint32_t)(w[j] >> 32) == tag;
        if (__all_sync(0xffffffffu, ok)) break;
        __nanosleep(TOPK_POLL_NS);
    }
    if (lane == 0) GP_STAMP(11);
    float score[EJ];
    uint32_t key[EJ], id[EJ];
#pragma unroll
    for (int j = 0; j < EJ; ++j) {
        const int e = lane + 32 * j;
        const float lg = e < E ? __uint_as_float((uint32_t)w[j]) : 0.f;
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
    return n < a.spin_limit;
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

// Per-stage partial sums: one per (row of the tile, covering warp).
constexpr uint32_t kPartialFloats =
    2 * TRG * LaneMap<5120, NWG, 4>::WPR > TRD * LaneMap<1536, NWC, 2>::WPR ? 2 * TRG * LaneMap<5120, NWG, 4>::WPR
                                                                          : TRD * LaneMap<1536, NWC, 2>::WPR;

struct Smem {
    uint32_t stage_bytes, stages_off, partial_off, bar_off, misc_off, total;
};

// misc block: abort flag (16 B), routed-slot count + first slot per token (16
// ints), slot -> local expert / token / weight (3 x kDecodeMaxRouted words),
// router slices [kMaxOwned * RSPLIT][n_tok], one down row tile's values per
// slot [max_routed + 1][32].
__host__ __device__ inline Smem decode_smem(int H, int I, int S, int n_tok, int max_routed) {
    Smem L;
    const uint32_t gu = 2u * TRG * 98u * (H / 256);
    const uint32_t dn = TRD * 98u * (I / 256) + (uint32_t)I * 2u + (uint32_t)(I / UNIT) * 4u;
    L.stage_bytes = ((gu > dn ? gu : dn) + 15u) & ~15u;
    L.stages_off = GP_IQ3_TABLE_BYTES;
    L.partial_off = L.stages_off + S * L.stage_bytes;
    const uint32_t pb = kPartialFloats * 4u;
    L.bar_off = (L.partial_off + S * pb + 15u) & ~15u;
    L.misc_off = L.bar_off + (3u * S + 4u) * 8u;
    L.total = L.misc_off + 16u + 64u + 12u * kDecodeMaxRouted + 4u * kMaxOwned * RSPLIT * n_tok +
              128u * (uint32_t)(max_routed + 1);
    return L;
}

// Work item i of a phase in slot order: the shared expert first (it needs no
// routing), then routed slots 0..nsr-1; `per_slot` items each.
struct Item {
    int slot, idx;  // slot kShared: the shared expert
};
GP_DEVINL Item item_of(int i, int per_slot) {
    if (i < per_slot) return {kShared, i};
    const int r = i - per_slot, slot = r / per_slot;
    return {slot, r - slot * per_slot};
}
// Items i = c, c+G, c+2G, ... below total.
GP_DEVINL int items_of(int c, int G, int total) { return c < total ? (total - 1 - c) / G + 1 : 0; }

// Down work: positions v = tile*(nsr+1) + q over (row tile, slot position q);
// position q = nsr is the shared expert (ready first), q < nsr routed slot
// nsr-1-q (slot 0 at q = nsr-1 is ready next, slot nsr-1 at q = 0 last).  CTA
// c owns the range [v0, v1), sized so that its down work plus its routed
// gate/up units is the same for every CTA (weights: one unit ~ wu, one down
// position ~ wd).  The range is walked as: the leading partial tile, the
// first whole tile, the trailing partial tile, the other whole tiles; each
// tile in descending q.  Partial tiles thus meet the early-ready slots first,
// the tiles shared with a neighbour CTA are settled early, and the CTA ends
// on a whole tile it combines by itself.
GP_DEVINL int down_slot(int q, int nsr) { return q == nsr ? kShared : nsr - 1 - q; }
struct DownRange {
    int v0, v1, b, e, P;  // range, first / last tile boundary inside it, nsr+1
    GP_DEVINL int count() const { return v1 - v0; }
    GP_DEVINL int at(int i) const {
        const int lead_end = b < v1 ? b : v1;
        if (i < lead_end - v0) return lead_end - 1 - i;
        i -= lead_end - v0;
        const int nf = e > b ? (e - b) / P : 0;
        if (nf > 0) {
            if (i < P) return b + P - 1 - i;
            i -= P;
        }
        const int n_trail = (e >= b && e < v1) ? v1 - e : 0;
        if (i < n_trail) return v1 - 1 - i;
        i -= n_trail;
        const int f = 1 + i / P;
        return b + f * P + P - 1 - (i - (f - 1) * P);
    }
};
GP_DEVINL int prefix_rr(int c, int G, int total) {  // sum of items_of(c', G, total) over c' < c
    return (total / G) * c + (c < total % G ? c : total % G);
}
GP_DEVINL DownRange down_range(int c, int G, int n_tiles, int P, int units, int shared_units) {
    // weights set by measurement of the whole layer (not of the units alone):
    // a routed gate/up unit counts as 3 down positions, although it takes
    // about 5.7, because a CTA that finishes its units early cannot start the
    // down tiles of the slots still being computed elsewhere; a shared unit
    // mostly overlaps the routing.  32-bit arithmetic: G * W < 2^31 for the
    // supported shapes (host-checked).
    constexpr int wu = 30, ws = 17, wd = 10;
    const int routed = units - shared_units, total = n_tiles * P;
    const int W = routed * wu + shared_units * ws + total * wd;
    const int max_units = (units + G - 1) / G;
    const bool weighted = max_units * wu * G <= W;  // every CTA still gets >= 0 down positions
    auto start = [&](int cc) -> int {
        if (!weighted) return total * cc / G;
        const int sh = prefix_rr(cc, G, shared_units), all = prefix_rr(cc, G, units);
        return (cc * W - G * ((all - sh) * wu + sh * ws)) / (G * wd);
    };
    DownRange r;
    r.P = P;
    r.v0 = start(c);
    r.v1 = c + 1 == G ? (int)total : start(c + 1);
    r.b = (r.v0 + P - 1) / P * P;
    r.e = r.v1 / P * P;
    if (r.b > r.v1) r.b = r.v1;
    if (r.e < r.b) r.e = r.b;
    return r;
}

// A CTA's share of the work once the routed slot count nsr is known.
struct Work {
    int nsr, n_gu, n_items;
    DownRange R;
};
GP_DEVINL Work work_of(int c, int G, int nsr, int NU, int TD) {
    Work w;
    w.nsr = nsr < 0 ? 0 : nsr > kDecodeMaxRouted ? kDecodeMaxRouted : nsr;
    const int nsl = w.nsr + 1;
    w.n_gu = TPU * items_of(c, G, NU * nsl);
    w.R = down_range(c, G, TD, nsl, NU * nsl, NU);
    w.n_items = w.n_gu + w.R.count();
    return w;
}

// Quantises the unit of h held one value per lane exactly as a lane quantises
// its activations for the GEMV (quant_i16<32>, scale * 1/4), into hq.  hq
// layout: 4 planes of NU 16-byte chunks (plane i holds words 4i..4i+3 of every
// unit, so a warp's 16-byte loads of consecutive units are conflict-free),
// then the NU fp32 scales at 2*I.
GP_DEVINL void quantise_unit(float v, uint8_t* hq, int I, int unit, int lane) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
    const int q = __float2int_rn(v * inv);
    const int qn = __shfl_down_sync(0xffffffffu, q, 1);
    const int w = lane >> 1;  // word of the unit
    if (!(lane & 1))
        *reinterpret_cast<uint32_t*>(hq + (w >> 2) * (I / UNIT) * 16 + unit * 16 + (w & 3) * 4) =
            (static_cast<uint32_t>(q) & 0xFFFFu) | (static_cast<uint32_t>(qn) << 16);
    if (lane == 0) reinterpret_cast<float*>(hq + 2 * I)[unit] = 0.25f * (amax * (1.0f / 32767.0f));
}

template <int HH, int II, int PG, int RPWG, int PD, int RPWD>
__global__ void __launch_bounds__(NTHREADS, 1) decode_layer_kernel(const DecodeLayerArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    constexpr int H = HH, I = II;
    constexpr int TD = H / TRD, NU = I / UNIT;
    constexpr uint32_t GU_BYTES = TRG * 98u * (H / 256), DN_BYTES = TRD * 98u * (I / 256);
    constexpr uint32_t HQ_BYTES = I * 2u + NU * 4u;
    static_assert(UNIT % TRG == 0 && HQ_BYTES % 16 == 0 && DN_BYTES % 16 == 0 && GU_BYTES % 16 == 0,
                  "bulk copies need 16-byte sizes and offsets");
    const int E = a.E, K = a.K, S = a.stages, NT = a.n_tok;
    const Smem L = decode_smem(H, I, S, NT, NT * K);
    const uint32_t sbase = smem_u32(smem);
    // per stage: full (producer -> compute warps), pdone (compute warps ->
    // epilogue warp: partial sums written), empty (epilogue -> producer)
    const uint32_t full0 = sbase + L.bar_off, pdone0 = full0 + 8u * S, empty0 = pdone0 + 8u * S;
    const uint32_t tbar = empty0 + 8u * S, topk_bar = tbar + 8u, rbar = topk_bar + 8u, gbar = rbar + 8u;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off);
    int* s_nsr = reinterpret_cast<int*>(smem + L.misc_off + 16u);
    int* s_first = s_nsr + 1;                       // [n_tok + 1]
    int* s_se = s_nsr + 16;                         // [kDecodeMaxRouted] local expert of a slot
    int* s_st = s_se + kDecodeMaxRouted;            // token of a slot
    float* s_sw = reinterpret_cast<float*>(s_st + kDecodeMaxRouted);  // weight of a slot
    float* s_slice = s_sw + kDecodeMaxRouted;       // [task][n_tok] router slices
    float* s_dv = s_slice + kMaxOwned * RSPLIT * NT;  // [slot position][32] one down row tile
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    constexpr uint32_t pstride = kPartialFloats;
    const uint32_t stage0 = sbase + L.stages_off;
    const int n_shared = TPU * items_of(c, G, NU);  // leading gate/up tiles that need no routing
    const int n_own = items_of(c, G, E);            // router experts c, c+G, ...
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
        mbar_init(gbar, 1);
        *s_abort = gp_tables_at_base(smem) ? 0u : 1u;
        if (*s_abort) atomicOr(a.status, GP_DEV_BAD_SHAPE);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == PROD) {
        // ================= producer (lane 0 issues; the warp polls) =================
        if (lane == 0) {
            GP_STAMP(9);
            mbar_arrive_expect_tx(tbar, GP_IQ3_TABLE_BYTES);
            for (int k4 = 0; k4 < 4; ++k4) bulk_g2s(sbase + k4 * 16384u, a.tables + k4 * 16384, 16384u, tbar);
        }
        int s = 0, issued = 0;
        uint32_t ph = 1;
        uint32_t ready[3] = {0u, 0u, 0u};  // storage slots whose h units are all counted
        bool have = false;
        Work w{};
        for (int it = 0;; ++it) {
            if (__shfl_sync(0xffffffffu, *s_abort, 0)) break;
            if (!have && it >= n_shared) {  // routed tiles need the slot list (every lane reads it)
                const bool ok = mbar_wait(topk_bar, 0, a.spin_limit);
                if (!ok) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                if (!__all_sync(0xffffffffu, ok)) break;
                if (lane == 0) GP_STAMP(10);
                w = work_of(c, G, *s_nsr, NU, TD);
                have = true;
            }
            if (have && it >= w.n_items) break;
            int slot;
            uint32_t off, b0, b1;
            const bool gu = it < (have ? w.n_gu : n_shared);
            if (gu) {
                const Item u = item_of(c + (it / TPU) * G, NU);
                slot = u.slot;
                off = (uint32_t)(u.idx * TPU + it % TPU) * GU_BYTES;
                b0 = b1 = GU_BYTES;
            } else {
                const int v = w.R.at(it - w.n_gu), nsl = w.nsr + 1;
                slot = down_slot(v % nsl, w.nsr);
                off = (uint32_t)(v / nsl) * DN_BYTES;
                b0 = DN_BYTES;
                b1 = HQ_BYTES;
                // the tile travels with its slot's quantised h: wait (warp-wide
                // poll of the slots' counters) until all its units are counted
                const int st = slot_store(slot);
                auto is_ready = [&]() {  // bit st of the three ready words (no dynamic register index)
                    const uint32_t rw = st < 32 ? ready[0] : st < 64 ? ready[1] : ready[2];
                    return ((rw >> (st & 31)) & 1u) != 0u;
                };
                if (!is_ready()) {
                    uint32_t n = 0;
                    for (; n < a.spin_limit; ++n) {
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            const int q = lane + 32 * j;
                            const bool valid = q < w.nsr || q == kSharedStore;
                            const unsigned cnt = valid ? ld_relaxed(a.sync + kSyncSlot + q) : 0u;
                            ready[j] = __ballot_sync(0xffffffffu, valid && cnt >= (unsigned)NU);
                        }
                        if (is_ready()) break;
                        __nanosleep(64);
                    }
                    if (n == a.spin_limit) {
                        if (lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                        break;
                    }
                    // order the observed counts (and so the hq words they
                    // release) before this warp's later bulk-copy reads; a
                    // slot seen ready stays ready, so one fence per poll
                    fence_acq_rel_gpu();
                    fence_proxy_async_global();
                    if (lane == 0 && it == w.n_gu) GP_STAMP(12);
                }
            }
            if (lane == 0) {
                const int e = slot < 0 ? a.e_cnt : s_se[slot];  // local expert index
                const uint8_t *src0, *src1;
                if (gu) {
                    const int64_t eo = (int64_t)e * a.gu_stride + off;
                    src0 = a.gate + eo;
                    src1 = a.up + eo;
                } else {
                    src0 = a.down + (int64_t)e * a.d_stride + off;
                    src1 = a.hq + (int64_t)slot_store(slot) * HQ_BYTES;
                }
                if (!mbar_wait(empty0 + 8u * s, ph, a.spin_limit)) {
                    *s_abort = 1;
                    atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
                } else {
                    const uint32_t dst = stage0 + s * L.stage_bytes;
                    mbar_arrive_expect_tx(full0 + 8u * s, b0 + b1);
                    bulk_g2s(dst, src0, b0, full0 + 8u * s);
                    bulk_g2s(dst + b0, src1, b1, full0 + 8u * s);
                    ++issued;
                    if (++s == S) { s = 0; ph ^= 1u; }
                }
            }
            __syncwarp();
        }
        if (lane == 0) {
            // no copy may still be in flight when the CTA exits (the
            // compile-time limit, whatever the run-time one)
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                mbar_wait(full0 + 8u * (i % S), (uint32_t)(i / S) & 1u);
            mbar_wait(tbar, 0);
        }
        return;
    }

    if (warp == EPI) {
        // ================= routing, then the epilogues =================
        constexpr int EJ = kMaxEFused / 32;
        float bias[EJ];
#pragma unroll
        for (int j = 0; j < EJ; ++j) bias[j] = a.corr && lane + 32 * j < E ? __ldg(a.corr + lane + 32 * j) : 0.f;
        pdl_wait();
        const uint32_t tag = ld_relaxed(a.sync + kSyncGen) + 1u;
        if (n_tasks > 0) {  // this CTA's experts: slices added in order
            if (!mbar_wait(rbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            if (lane < n_own) {
                const int e = c + lane * G;
                for (int t = 0; t < NT; ++t) {
                    float lg = 0.f;
#pragma unroll
                    for (int sl = 0; sl < RSPLIT; ++sl) lg += s_slice[(lane * RSPLIT + sl) * NT + t];
                    const unsigned long long v = ((unsigned long long)tag << 32) | __float_as_uint(lg);
                    if (e == a.withhold_logit) continue;  // (a test withholds one to make the top-k wait run out)
                    if (NT == 1) {
#pragma unroll
                        for (int cp = 0; cp < kLogitCopies; ++cp) st_relaxed64(a.logits + logit_word(cp, 0, e, E), v);
                    } else {
                        st_relaxed64(a.logits + logit_word(0, t, e, E), v);
                    }
                }
            }
        }
        if (lane == 0) GP_STAMP(1);
        int e0 = 0, e1 = 0;
        float w0 = 0.f, w1 = 0.f;
        bool ok = true;
        if (NT == 1) {  // every CTA picks the token's experts itself
            ok = E <= 160 ? topk_token<5>(a, bias, tag, lane, c % kLogitCopies, 0, c == 0, e0, w0)
                          : topk_token<EJ>(a, bias, tag, lane, c % kLogitCopies, 0, c == 0, e0, w0);
        } else {
            // CTA t picks token t's experts and publishes them; every CTA
            // then reads all tokens' picks (one more exchange, no CTA sorts
            // n_tok tokens in turn)
            if (c < NT) {
                int me = 0;
                float mw = 0.f;
                ok = E <= 160 ? topk_token<5>(a, bias, tag, lane, 0, c, true, me, mw)
                              : topk_token<EJ>(a, bias, tag, lane, 0, c, true, me, mw);
                if (lane < K) {
                    const unsigned long long v = ((unsigned long long)(tag & 0xFFFFu) << 48) |
                                                 ((unsigned long long)(me & 0xFFFF) << 32) | __float_as_uint(mw);
#pragma unroll
                    for (int cp = 0; cp < kLogitCopies; ++cp) st_relaxed64(a.picks + pick_word(cp, c, lane), v);
                }
            }
            const int np = NT * K;
            unsigned long long p0 = 0ull, p1 = 0ull;
            uint32_t n = 0;
            for (; n < a.spin_limit && ok; ++n) {
                p0 = lane < np ? ld_relaxed64(a.picks + pick_word(c % kLogitCopies, lane / K, lane % K)) : 0ull;
                p1 = lane + 32 < np ? ld_relaxed64(a.picks + pick_word(c % kLogitCopies, (lane + 32) / K, (lane + 32) % K))
                                    : 0ull;
                const bool got = (lane >= np || (uint32_t)(p0 >> 48) == (tag & 0xFFFFu)) &&
                                 (lane + 32 >= np || (uint32_t)(p1 >> 48) == (tag & 0xFFFFu));
                if (__all_sync(0xffffffffu, got)) break;
                __nanosleep(TOPK_POLL_NS);
            }
            if (n == a.spin_limit) ok = false;
            e0 = (int)((p0 >> 32) & 0xFFFFu);
            w0 = __uint_as_float((uint32_t)p0);
            e1 = (int)((p1 >> 32) & 0xFFFFu);
            w1 = __uint_as_float((uint32_t)p1);
        }
        if (!ok && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        // (after a timeout the slot list is built from whatever was read: the
        // ids stay in range, the results are invalid and the status says so)
        build_slots(a, lane, e0, w0, e1, w1, s_nsr, s_first, s_se, s_st, s_sw);
        __syncwarp();
        if (lane == 0) mbar_arrive(topk_bar);  // release: the other roles read the slot list
        if (lane == 0) GP_STAMP(2);

        const Work w = work_of(c, G, *s_nsr, NU, TD);
        const int nsr = w.nsr;
        int s = 0;
        uint32_t ph = 0;
        constexpr int rsg = 32 * NWG / (H / 32), rsd = 32 * NWC / (I / 32);
        float hv = 0.f;
        // After an abort every warp leaves its loop at once (and arrives on no
        // further barrier), so no barrier phase sees arrivals from two
        // iterations; every wait left behind in another warp is bounded.
        for (int it = 0; it < w.n_items; ++it) {
            const bool gu = it < w.n_gu;
            if (warp_aborted(s_abort)) break;
            if (!mbar_wait(pdone0 + 8u * s, ph, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            if (warp_aborted(s_abort)) break;
            const float* pbuf = partial + (size_t)s * pstride;
            float val = 0.f;
            if (gu) {
                if (lane < TRG) {  // partials in warp order (LaneMap layout)
                    using LG = LaneMap<HH, NWG, PG>;
                    const int row = lane, ur = TRG + row;
                    const int ng = LG::last_warp(row % rsg) - LG::first_warp(row % rsg);
                    const int nu = LG::last_warp(ur % rsg) - LG::first_warp(ur % rsg);
                    float gs = 0.f, us = 0.f;
                    for (int ww = 0; ww <= ng; ++ww) gs += pbuf[row * LG::WPR + ww];
                    for (int ww = 0; ww <= nu; ++ww) us += pbuf[ur * LG::WPR + ww];
                    val = silu_clamped(gs, us, a.limit);
                }
            } else {
                using LD = LaneMap<II, NWC, PD>;
                const int r0 = lane % rsd;
                const int nw = LD::last_warp(r0) - LD::first_warp(r0);
                for (int ww = 0; ww <= nw; ++ww) val += pbuf[lane * LD::WPR + ww];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8u * s);  // partials read: the stage may refill
            if (++s == S) { s = 0; ph ^= 1u; }
            if (gu) {
                // rows j*8 .. j*8+7 of the unit land on lanes j*8 .. j*8+7
                const int j = it % TPU;
                const float v = __shfl_sync(0xffffffffu, val, lane & (TRG - 1));
                if ((lane / TRG) == j) hv = v;
                if (j == TPU - 1) {
                    const Item u = item_of(c + (it / TPU) * G, NU);
                    const int st = slot_store(u.slot);
                    quantise_unit(hv, a.hq + (int64_t)st * HQ_BYTES, I, u.idx, lane);
                    __syncwarp();
                    if (lane == 0) red_release_add(a.sync + kSyncSlot + st, 1);
                }
            } else {
                const int nsl = nsr + 1;
                const int v = w.R.at(it - w.n_gu), rt = v / nsl;
                const int slot = down_slot(v % nsl, nsr);
                const int j = rt * TRD + lane;
                const int tb = rt * nsl, te = tb + nsl;
                if (tb >= w.R.v0) {
                    // this CTA holds the tile's last walked position (q = 0): it
                    // writes y, with the slots other CTAs computed (positions
                    // [v1, te), walked early by them) read as tagged words
                    s_dv[(slot < 0 ? nsr : slot) * 32 + lane] = val;
                    if (v == tb) {
                        if (te > w.R.v1) {
                            uint32_t n = 0;
                            for (; n < a.spin_limit; ++n) {
                                bool got = true;
                                for (int base = w.R.v1; base < te; base += 8) {  // 8 loads in flight
                                    unsigned long long wd[8];
#pragma unroll
                                    for (int i = 0; i < 8; ++i)
                                        wd[i] = base + i < te ? ld_relaxed64(a.dx + (int64_t)slot_store(down_slot(base + i - tb, nsr)) * H + j)
                                                              : (unsigned long long)tag << 32;
#pragma unroll
                                    for (int i = 0; i < 8; ++i) {
                                        got &= (uint32_t)(wd[i] >> 32) == tag;
                                        if (base + i < te) {
                                            const int sl = down_slot(base + i - tb, nsr);
                                            s_dv[(sl < 0 ? nsr : sl) * 32 + lane] = __uint_as_float((uint32_t)wd[i]);
                                        }
                                    }
                                }
                                if (__all_sync(0xffffffffu, got)) break;
                                __nanosleep(64);
                            }
                            if (n == a.spin_limit && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                        }
                        __syncwarp();
                        // y[t] = sum over t's slots of w * D in pick order
                        // (+ the shared expert for own_tok), model.cpp:741-755
                        for (int t = 0; t < NT; ++t) {
                            float y = 0.f;
                            for (int k = s_first[t]; k < s_first[t + 1]; ++k) y = fmaf(s_sw[k], s_dv[k * 32 + lane], y);
                            if (t == a.own_tok) y += s_dv[nsr * 32 + lane];
                            a.y[(int64_t)t * H + j] = y;
                        }
                        __syncwarp();
                    }
                } else {
                    // the CTA before this one finishes the tile
                    st_relaxed64(a.dx + (int64_t)slot_store(slot) * H + j,
                                 ((unsigned long long)tag << 32) | __float_as_uint(val));
                }
            }
        }
        if (lane == 0) GP_STAMP(7);
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
        if (tid == 0) GP_STAMP(0);

        // ---- router slices of this CTA's experts: warp task = (expert, slice),
        // one dot product per token ----
        for (int task = warp; task < n_tasks; task += NWC) {
            if (task != warp) load_router(task);
            const int sl = task % RSPLIT;
            for (int t = 0; t < NT; ++t) {
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < RV; ++i) {
                    const int64_t k0 = (int64_t)t * H + sl * RSL + lane * 4 + i * 128;
                    float4 xv;
                    if (a.x_bf16) {
                        const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + k0);
                        xv = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                         __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
                    } else {
                        xv = *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + k0);
                    }
                    acc = fmaf(wv[i].x, xv.x, acc);
                    acc = fmaf(wv[i].y, xv.y, acc);
                    acc = fmaf(wv[i].z, xv.z, acc);
                    acc = fmaf(wv[i].w, xv.w, acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) s_slice[task * NT + t] = acc;
            }
            if (lane == 0) mbar_arrive(rbar);
        }

        if (!mbar_wait(tbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        int s = 0;
        uint32_t ph = 0;
        bool have = false;
        Work w{};
        // the slot list (routed slot count, slot tokens) once the top-k is in
        auto wait_slots = [&]() -> bool {
            if (!mbar_wait(topk_bar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            if (warp_aborted(s_abort)) return false;
            w = work_of(c, G, *s_nsr, NU, TD);
            have = true;
            return true;
        };
        // ---- gate/up tiles: warps 0..NWG-1; warp 0 also arrives for the
        // others, which sleep until the down phase ----
        if (warp < NWG) {
            const auto mg = lane_map<HH, NWG, PG>(warp, lane, stage0);
            uint32_t xq[16];
            int cur = a.own_tok;  // the token whose activations xq holds (the shared expert's first)
            float sx4 = load_quant(a.x, a.x_bf16, cur, H, mg.sb, xq);
            for (int it = 0;; ++it) {
                if (!have && it >= n_shared && !wait_slots()) break;
                if (have && it >= w.n_gu) break;
                if (it % TPU == 0 && NT > 1) {  // a new unit: its slot's token
                    const Item u = item_of(c + (it / TPU) * G, NU);
                    const int tk = u.slot < 0 ? a.own_tok : s_st[u.slot];
                    if (tk != cur) {
                        cur = tk;
                        sx4 = load_quant(a.x, a.x_bf16, cur, H, mg.sb, xq);
                    }
                }
                if (warp_aborted(s_abort)) break;
                if (!mbar_wait(full0 + 8u * s, ph, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                if (warp_aborted(s_abort)) break;
                if (tid == 0 && it == n_shared) GP_STAMP(3);
                consume<HH, NWG, PG, RPWG>(mg, s * L.stage_bytes, xq, sx4, partial + (size_t)s * pstride, warp, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive_cnt(pdone0 + 8u * s, warp == 0 ? 1 + NWC - NWG : 1);
                if (++s == S) { s = 0; ph ^= 1u; }
            }
            if (warp == 0 && lane == 0) mbar_arrive(gbar);
        } else {
            // once warp 0 has passed every gate/up stage, the first down
            // stage is at most one phase ahead of its parity wait
            if (!mbar_wait_sleepy(gbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            if (wait_slots()) {
                s = w.n_gu % S;
                ph = (uint32_t)(w.n_gu / S) & 1u;
            }
        }
        if (tid == 0) GP_STAMP(4);
        // ---- down tiles: the activations come with the tile ----
        if (have) {
            const auto md = lane_map<II, NWC, PD>(warp, lane, stage0);
            for (int it = w.n_gu; it < w.n_items; ++it) {
                if (warp_aborted(s_abort)) break;
                if (!mbar_wait(full0 + 8u * s, ph, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                if (warp_aborted(s_abort)) break;
                if (tid == 0 && it == w.n_gu) GP_STAMP(5);
                const uint32_t xb = stage0 + s * L.stage_bytes + DN_BYTES;
                uint32_t xq[16];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = lds128(xb + i * (NU * 16u) + md.sb * 16u);
                    xq[4 * i] = v.x;
                    xq[4 * i + 1] = v.y;
                    xq[4 * i + 2] = v.z;
                    xq[4 * i + 3] = v.w;
                }
                const float sx4 = ldsf(xb + 2u * I + md.sb * 4u);
                consume<II, NWC, PD, RPWD>(md, s * L.stage_bytes, xq, sx4, partial + (size_t)s * pstride, warp, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(pdone0 + 8u * s);
                if (++s == S) { s = 0; ph ^= 1u; }
            }
        }
        if (tid == 0) GP_STAMP(6);
    }

    // the last CTA out clears the counters that are waited on
    named_bar_sync(1, (NWC + 1) * 32);
    if (tid == 0) {
        GP_STAMP(8);
        fence_acq_rel_gpu();
        if (atomicAdd(a.sync + kSyncEnd, 1u) == (unsigned)G - 1) {
            a.sync[kSyncGen] += 1u;
            const int nsr = min(max(*s_nsr, 0), kDecodeMaxRouted);
            for (int k = 0; k < nsr; ++k) a.sync[kSyncSlot + k] = 0;
            a.sync[kSyncSlot + kSharedStore] = 0;
            fence_acq_rel_gpu();
            a.sync[kSyncEnd] = 0;
        }
    }
}

}  // namespace

bool decode_layer_supported(int H, int I, int E, int K, int with_shared) {
    if (E > kMaxEFused || E < K) return false;
    // the instantiated work mapping: gate/up 20 warps over 4 rows of H = 5120
    // (4 passes), down 24 warps over 16 rows of I = 1536 (2 passes, rows
    // straddle warps)
    return H == 5120 && I == 1536 && K >= 1 && K <= MAXK && with_shared == 1;
}

size_t decode_layer_smem(int H, int I, int stages, int n_tok, int max_routed) {
    return decode_smem(H, I, stages, n_tok, max_routed).total;
}

cudaError_t launch_decode_layer(const DecodeLayerArgs& a, int grid, cudaStream_t st) {
    if (!decode_layer_supported(a.H, a.I, a.E, a.K, a.with_shared)) return cudaErrorInvalidValue;
    if (grid * kMaxOwned < a.E) return cudaErrorInvalidValue;  // router experts per CTA
    if (a.n_tok < 1 || a.n_tok > kDecodeMaxTokens || a.n_tok * a.K > kDecodeMaxRouted || a.own_tok < 0 ||
        a.own_tok >= a.n_tok || a.e_lo < 0 || a.e_cnt < 0 || a.e_lo + a.e_cnt > a.E || a.E >= 65536 ||
        (a.n_tok > 1 && !a.picks))
        return cudaErrorInvalidValue;
    if (a.n_tok == 1 && (a.e_lo != 0 || a.e_cnt != a.E)) return cudaErrorInvalidValue;  // one token: every expert
    // down-range weights in 32-bit: grid * (units * 42 + tiles * 10) < 2^31
    const int64_t slots = (int64_t)a.n_tok * a.K + 1;
    if ((int64_t)grid * ((int64_t)(a.I / UNIT) * slots * 42 + (int64_t)(a.H / TRD) * slots * 10) >= (1ll << 31))
        return cudaErrorInvalidValue;
    const Smem L = decode_smem(a.H, a.I, a.stages, a.n_tok, a.n_tok * a.K);
    if (L.total > 227u * 1024u) return cudaErrorInvalidValue;
    auto kern = decode_layer_kernel<5120, 1536, 4, 1, 2, 2>;
    static std::atomic<unsigned long long> configured{0};  // per device
    if (cudaError_t e0 = raise_smem_limit(kern, 227 * 1024, configured)) return e0;
    // Co-residency: every CTA waits on data the others publish, so the grid
    // must fit the GPU at one CTA per SM.  Checked against the kernel's real
    // resource use (registers, shared memory) once per device; a grid larger
    // than the SMs that can hold a CTA is refused rather than left to time out.
    static std::atomic<unsigned long long> fits{0};
    int dev = 0;
    if (cudaError_t e1 = cudaGetDevice(&dev)) return e1;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (!bit || !(fits.load(std::memory_order_acquire) & bit)) {
        int per_sm = 0, sms = 0;
        if (cudaError_t e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NTHREADS, 227 * 1024))
            return e2;
        if (cudaError_t e3 = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) return e3;
        if (per_sm < 1 || grid > sms * per_sm) return cudaErrorCooperativeLaunchTooLarge;
        if (bit) fits.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHREADS);
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
