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
//   router   CTA c owns experts c, c+G, ...; 8 warps each compute one 1/8
//            slice of an owned expert's fp32 logit (weights prefetched before
//            the wait on the previous kernel); the epilogue warp adds the
//            slices in order and stores the logit tagged with the launch
//            generation, so readers poll the data itself
//   top-k    every CTA's epilogue warp polls the E tagged logits (one of 8
//            replicas, spread over L2 lines), applies
//            sigmoid + bias and picks top-K by warp reductions (ties to the
//            lower id), weights score/(1e-20 + sum)*scale (model.cpp:704-725)
//   gate/up  units of 32 rows of h, dealt round-robin in slot order (the
//            shared expert, storage slot K, first: it needs no routing; then
//            routed slots 0..K-1); a unit is 4 consecutive tiles of 8 rows of
//            gate and up.  The epilogue applies SwiGLU with the reference clamp
//            (model.cpp:733-739), quantises the finished unit to int16 (hq)
//            and counts it for its slot: no value of h leaves the CTA
//            unquantised and no counter is read back
//   down     tiles of 32 rows x (K+1) slots, a contiguous range of (tile,
//            slot) positions per CTA sized to even out the total work; the
//            producer copies each tile with its slot's hq once all units of
//            that slot are counted (model.cpp:740).  The epilogue keeps a row
//            tile's slot results in shared memory and writes y = sum_k w_k
//            D[k] + D[shared] in top-k order (model.cpp:741-755); for a tile
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
GP_DEVINL int logit_word(int copy, int e, int E) { return (copy * E + e) * kLogitStride; }
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

// Epilogue warp: sigmoid scores from the gathered logits, top-K by score +
// bias (ties to the lower id), weights score/(1e-20 + sum)*scale
// (model.cpp:704-725); publishes them to the CTA.  Each lane sorts its EJ
// candidates (expert ids lane + 32j) by (key desc, id asc); a round then takes
// the warp maximum of the lanes' head keys (redux), the lowest id holding it,
// and that lane pops its head.
template <int EJ>
GP_DEVINL void topk_warp(const DecodeLayerArgs& a, const float* bias, uint32_t tag, int lane, int c, int* s_ids,
                         float* s_w, uint32_t topk_bar, volatile uint32_t* s_abort) {
    const int E = a.E, K = a.K;
    // every CTA's logits, each word tagged by its writer with this launch's
    // tag: the data is its own flag, so one poll round trip suffices
    unsigned long long w[EJ];
    uint32_t n = 0;
    for (; n < a.spin_limit; ++n) {
#pragma unroll
        for (int j = 0; j < EJ; ++j)
            w[j] = lane + 32 * j < E ? ld_relaxed64(a.logits + logit_word(c % kLogitCopies, lane + 32 * j, E)) : 0ull;
        bool ok = true;
#pragma unroll
        for (int j = 0; j < EJ; ++j) ok &= lane + 32 * j >= E || (uint32_t)(w[j] >> 32) == tag;
        if (__all_sync(0xffffffffu, ok)) break;
        __nanosleep(TOPK_POLL_NS);
    }
    if (n == a.spin_limit && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
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
    int my_e = 0;
    if (a.forced) {
        for (int k = 0; k < K; ++k) {
            int eb = a.forced[k];
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
    if (lane < K) {
        const float w = a.norm_topk ? (my_s / denom) * a.routed_scale : my_s * a.routed_scale;
        s_ids[lane] = my_e;
        s_w[lane] = w;
        if (c == 0 && a.topk_ids) a.topk_ids[lane] = my_e;
        if (c == 0 && a.topk_w) a.topk_w[lane] = w;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(topk_bar);  // release: the producer reads s_ids
}

// Per-stage partial sums: one per (row of the tile, covering warp).
constexpr uint32_t kPartialFloats =
    2 * TRG * LaneMap<5120, NWG, 4>::WPR > TRD * LaneMap<1536, NWC, 2>::WPR ? 2 * TRG * LaneMap<5120, NWG, 4>::WPR
                                                                          : TRD * LaneMap<1536, NWC, 2>::WPR;

struct Smem {
    uint32_t stage_bytes, stages_off, partial_off, bar_off, misc_off, total;
};

__host__ __device__ inline Smem decode_smem(int H, int I, int S) {
    Smem L;
    const uint32_t gu = 2u * TRG * 98u * (H / 256);
    const uint32_t dn = TRD * 98u * (I / 256) + (uint32_t)I * 2u + (uint32_t)(I / UNIT) * 4u;
    L.stage_bytes = ((gu > dn ? gu : dn) + 15u) & ~15u;
    L.stages_off = GP_IQ3_TABLE_BYTES;
    L.partial_off = L.stages_off + S * L.stage_bytes;
    const uint32_t pb = kPartialFloats * 4u;
    L.bar_off = (L.partial_off + S * pb + 15u) & ~15u;
    L.misc_off = L.bar_off + (3u * S + 4u) * 8u;
    // abort flag, s_ids[32], s_w[32], router slices[kMaxOwned * RSPLIT],
    // one down row tile's per-slot values [MAXK + 1][32]
    L.total = L.misc_off + 16u + 8u * 32u + 4u * kMaxOwned * RSPLIT + 4u * (MAXK + 1) * 32u;
    return L;
}

// Work item i of a phase in slot order: the shared expert (storage slot K)
// first, then routed slots 0..K-1; `per_slot` items each.
struct Item {
    int slot, idx;
};
GP_DEVINL Item item_of(int i, int per_slot, int K) {
    if (i < per_slot) return {K, i};
    const int r = i - per_slot, slot = r / per_slot;
    return {slot, r - slot * per_slot};
}
// Items i = c, c+G, c+2G, ... below total.
GP_DEVINL int items_of(int c, int G, int total) { return c < total ? (total - 1 - c) / G + 1 : 0; }

// Down work: positions v = tile*(K+1) + q over (row tile, slot position q);
// position q = K is the shared expert (ready first), q < K routed slot K-1-q
// (slot 0 at q = K-1 is ready next, slot K-1 at q = 0 last).  CTA c owns the
// range [v0, v1), sized so that its down work plus its routed gate/up units
// is the same for every CTA (weights: one unit ~ wu, one down position ~ wd).
// The range is walked as: the leading partial tile, the first whole tile,
// the trailing partial tile, the other whole tiles; each tile in descending
// q.  Partial tiles thus meet the early-ready slots first, the tiles shared
// with a neighbour CTA are settled early, and the CTA ends on a whole tile
// it combines by itself.
GP_DEVINL int down_slot(int q, int K) { return q == K ? K : K - 1 - q; }
struct DownRange {
    int v0, v1, b, e, P;  // range, first / last tile boundary inside it, K+1
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
    static_assert(MAXK + 1 <= kDecodeSyncWords - kSyncSlot, "counter block too small");
    static_assert(UNIT % TRG == 0 && HQ_BYTES % 16 == 0 && DN_BYTES % 16 == 0 && GU_BYTES % 16 == 0,
                  "bulk copies need 16-byte sizes and offsets");
    const int E = a.E, K = a.K, S = a.stages;
    const Smem L = decode_smem(H, I, S);
    const uint32_t sbase = smem_u32(smem);
    // per stage: full (producer -> compute warps), pdone (compute warps ->
    // epilogue warp: partial sums written), empty (epilogue -> producer)
    const uint32_t full0 = sbase + L.bar_off, pdone0 = full0 + 8u * S, empty0 = pdone0 + 8u * S;
    const uint32_t tbar = empty0 + 8u * S, topk_bar = tbar + 8u, rbar = topk_bar + 8u, gbar = rbar + 8u;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off);
    int* s_ids = reinterpret_cast<int*>(smem + L.misc_off + 16u);
    float* s_w = reinterpret_cast<float*>(s_ids + 32);
    float* s_slice = s_w + 32;
    float* s_dv = s_slice + kMaxOwned * RSPLIT;
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    constexpr uint32_t pstride = kPartialFloats;
    const uint32_t stage0 = sbase + L.stages_off;
    const int n_gu = TPU * items_of(c, G, NU * (K + 1));
    const int n_shared = TPU * items_of(c, G, NU);  // leading gate/up tiles that need no routing
    const DownRange R = down_range(c, G, TD, K + 1, NU * (K + 1), NU);
    const int n_items = n_gu + R.count();
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
        uint32_t ph = 1, ready = 0;
        bool have_topk = false;
        for (int it = 0; it < n_items; ++it) {
            if (__shfl_sync(0xffffffffu, *s_abort, 0)) break;
            int slot;
            uint32_t off, b0, b1;
            const uint8_t *src0, *src1;
            if (it < n_gu) {
                const Item u = item_of(c + (it / TPU) * G, NU, K);
                slot = u.slot;
                off = (uint32_t)(u.idx * TPU + it % TPU) * GU_BYTES;
                b0 = b1 = GU_BYTES;
            } else {
                const int v = R.at(it - n_gu);
                slot = down_slot(v % (K + 1), K);
                off = (uint32_t)(v / (K + 1)) * DN_BYTES;
                b0 = DN_BYTES;
                b1 = HQ_BYTES;
                // the tile travels with its slot's quantised h: wait (warp-wide
                // poll of every slot's counter) until all its units are counted
                if (!((ready >> slot) & 1u)) {
                    uint32_t n = 0;
                    for (; n < a.spin_limit; ++n) {
                        const unsigned cnt = lane <= K ? ld_relaxed(a.sync + kSyncSlot + lane) : 0u;
                        ready = __ballot_sync(0xffffffffu, lane <= K && cnt >= (unsigned)NU);
                        if ((ready >> slot) & 1u) break;
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
                    if (lane == 0 && it == n_gu) GP_STAMP(12);
                }
            }
            if (lane == 0) {
                bool ok = true;
                if (it >= n_shared && !have_topk) {  // routed tiles need the top-k
                    ok = have_topk = mbar_wait(topk_bar, 0, a.spin_limit);
                    if (ok) GP_STAMP(10);
                    else { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                }
                if (ok) {
                    const int e = slot < K ? s_ids[slot] : E;
                    if (it < n_gu) {
                        const int64_t eo = (int64_t)e * a.gu_stride + off;
                        src0 = a.gate + eo;
                        src1 = a.up + eo;
                    } else {
                        src0 = a.down + (int64_t)e * a.d_stride + off;
                        src1 = a.hq + (int64_t)slot * HQ_BYTES;
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
            }
            __syncwarp();
        }
        if (lane == 0) {
            // no copy may still be in flight when the CTA exits
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                mbar_wait(full0 + 8u * (i % S), (uint32_t)(i / S) & 1u);  // the compile-time limit,
            mbar_wait(tbar, 0);                                           // whatever the run-time one
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
                float lg = 0.f;
#pragma unroll
                for (int sl = 0; sl < RSPLIT; ++sl) lg += s_slice[lane * RSPLIT + sl];
                const unsigned long long v = ((unsigned long long)tag << 32) | __float_as_uint(lg);
                if (c + lane * G != a.withhold_logit) {  // (a test withholds one to make the top-k wait run out)
#pragma unroll
                    for (int cp = 0; cp < kLogitCopies; ++cp)
                        st_relaxed64(a.logits + logit_word(cp, c + lane * G, E), v);
                }
            }
        }
        if (lane == 0) GP_STAMP(1);
        if (E <= 160) topk_warp<5>(a, bias, tag, lane, c, s_ids, s_w, topk_bar, s_abort);
        else topk_warp<kMaxEFused / 32>(a, bias, tag, lane, c, s_ids, s_w, topk_bar, s_abort);
        if (lane == 0) GP_STAMP(2);

        int s = 0;
        uint32_t ph = 0;
        constexpr int rsg = 32 * NWG / (H / 32), rsd = 32 * NWC / (I / 32);
        float hv = 0.f;
        // After an abort every warp leaves its loop at once (and arrives on no
        // further barrier), so no barrier phase sees arrivals from two
        // iterations; every wait left behind in another warp is bounded.
        for (int it = 0; it < n_items; ++it) {
            const bool gu = it < n_gu;
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
                    for (int w = 0; w <= ng; ++w) gs += pbuf[row * LG::WPR + w];
                    for (int w = 0; w <= nu; ++w) us += pbuf[ur * LG::WPR + w];
                    val = silu_clamped(gs, us, a.limit);
                }
            } else {
                using LD = LaneMap<II, NWC, PD>;
                const int r0 = lane % rsd;
                const int nw = LD::last_warp(r0) - LD::first_warp(r0);
                for (int w = 0; w <= nw; ++w) val += pbuf[lane * LD::WPR + w];
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
                    const Item u = item_of(c + (it / TPU) * G, NU, K);
                    quantise_unit(hv, a.hq + (int64_t)u.slot * HQ_BYTES, I, u.idx, lane);
                    __syncwarp();
                    if (lane == 0) red_release_add(a.sync + kSyncSlot + u.slot, 1);
                }
            } else {
                const int v = R.at(it - n_gu), t = v / (K + 1);
                const int slot = down_slot(v % (K + 1), K);
                const int j = t * TRD + lane;
                const int tb = t * (K + 1), te = tb + K + 1;
                if (tb >= R.v0) {
                    // this CTA holds the tile's last walked position (q = 0): it
                    // writes y, with the slots other CTAs computed (positions
                    // [v1, te), walked early by them) read as tagged words
                    s_dv[slot * 32 + lane] = val;
                    if (v == tb) {
                        if (te > R.v1) {
                            uint32_t n = 0;
                            for (; n < a.spin_limit; ++n) {
                                bool ok = true;
                                for (int base = R.v1; base < te; base += 8) {  // 8 loads in flight
                                    unsigned long long w[8];
#pragma unroll
                                    for (int i = 0; i < 8; ++i)
                                        w[i] = base + i < te ? ld_relaxed64(a.dx + (int64_t)down_slot(base + i - tb, K) * H + j)
                                                             : (unsigned long long)tag << 32;
#pragma unroll
                                    for (int i = 0; i < 8; ++i) {
                                        ok &= (uint32_t)(w[i] >> 32) == tag;
                                        if (base + i < te) s_dv[down_slot(base + i - tb, K) * 32 + lane] = __uint_as_float((uint32_t)w[i]);
                                    }
                                }
                                if (__all_sync(0xffffffffu, ok)) break;
                                __nanosleep(64);
                            }
                            if (n == a.spin_limit && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                        }
                        __syncwarp();
                        float y = 0.f;
                        for (int k = 0; k < K; ++k) y = fmaf(s_w[k], s_dv[k * 32 + lane], y);
                        a.y[j] = y + s_dv[K * 32 + lane];
                        __syncwarp();
                    }
                } else {
                    // the CTA before this one finishes the tile
                    st_relaxed64(a.dx + (int64_t)slot * H + j, ((unsigned long long)tag << 32) | __float_as_uint(val));
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
            const float* w = a.router + (int64_t)(c + (task / RSPLIT) * G) * H + (task % RSPLIT) * RSL + lane * 4;
#pragma unroll
            for (int i = 0; i < RV; ++i) wv[i] = __ldg(reinterpret_cast<const float4*>(w + i * 128));
        };
        if (warp < n_tasks) load_router(warp);
        pdl_wait();
        if (tid == 0) GP_STAMP(0);

        // ---- router slices of this CTA's experts: warp task = (expert, slice) ----
        for (int task = warp; task < n_tasks; task += NWC) {
            if (task != warp) load_router(task);
            const int sl = task % RSPLIT;
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < RV; ++i) {
                const int k0 = sl * RSL + lane * 4 + i * 128;
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
            if (lane == 0) {
                s_slice[task] = acc;
                mbar_arrive(rbar);
            }
        }

        if (!mbar_wait(tbar, 0, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        int s = 0;
        uint32_t ph = 0;
        // ---- gate/up tiles: warps 0..NWG-1; warp 0 also arrives for the
        // others, which sleep until the down phase ----
        if (warp < NWG) {
            const auto mg = lane_map<HH, NWG, PG>(warp, lane, stage0);
            uint32_t xq[16];
            const float sx4 = load_quant(a.x, a.x_bf16, 0, H, mg.sb, xq);
            for (int it = 0; it < n_gu; ++it) {
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
            s = n_gu % S;
            ph = (uint32_t)(n_gu / S) & 1u;
        }
        if (tid == 0) GP_STAMP(4);
        // ---- down tiles: the activations come with the tile ----
        {
            const auto md = lane_map<II, NWC, PD>(warp, lane, stage0);
            for (int it = n_gu; it < n_items; ++it) {
                if (warp_aborted(s_abort)) break;
                if (!mbar_wait(full0 + 8u * s, ph, a.spin_limit)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
                if (warp_aborted(s_abort)) break;
                if (tid == 0 && it == n_gu) GP_STAMP(5);
                {
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
                    consume<II, NWC, PD, RPWD>(md, s * L.stage_bytes, xq, sx4, partial + (size_t)s * pstride, warp,
                                               lane);
                }
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
            for (int k = 0; k <= K; ++k) a.sync[kSyncSlot + k] = 0;
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

size_t decode_layer_smem(int H, int I, int stages) { return decode_smem(H, I, stages).total; }

cudaError_t launch_decode_layer(const DecodeLayerArgs& a, int grid, cudaStream_t st) {
    if (!decode_layer_supported(a.H, a.I, a.E, a.K, a.with_shared)) return cudaErrorInvalidValue;
    if (grid * kMaxOwned < a.E) return cudaErrorInvalidValue;  // router experts per CTA
    // down-range weights in 32-bit: grid * (units * 42 + tiles * 10) < 2^31
    if ((int64_t)grid * ((int64_t)(a.I / UNIT) * (a.K + 1) * 42 + (int64_t)(a.H / TRD) * (a.K + 1) * 10) >= (1ll << 31))
        return cudaErrorInvalidValue;
    const Smem L = decode_smem(a.H, a.I, a.stages);
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
