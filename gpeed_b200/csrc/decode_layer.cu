// One MoE layer at batch 1 in a single persistent, cooperative kernel
// (reference Model::moe_forward, cpp/core/src/model.cpp:692-756).
//
// Separate kernels for router, routing, gate/up, down and combine each pay a
// launch, a prologue (decode tables, first bytes in flight) and a tail, which
// at batch 1 costs more than streaming the 85 MB of weights.  Here one CTA per
// SM runs the whole layer; the TMA producer streams weight tiles continuously
// across the phases, and the phases meet at grid-wide counters:
//
//   router   every warp computes one 1/8-row slice of the fp32 router logits
//            (fixed-order partial sums), then counter[0]
//   top-k    every CTA reads the 8 partials per expert (added in order), applies
//            sigmoid + bias, picks top-K (ties to the lower id) and the weights
//            score/(1e-20 + sum)*scale (model.cpp:704-725)
//   gate/up  the shared expert's tiles first (they need no routing, so they
//            overlap the router phase), then the routed experts'; epilogue
//            SwiGLU with the reference clamp into h[slot] (model.cpp:733-739);
//            then counter[1]
//   down     h[slot] -> D[slot] (model.cpp:740); the producer streams these
//            tiles while the consumers wait for counter[1]; then counter[2]
//   combine  y = sum_k w_k D[k] + D[shared] in top-k order (model.cpp:741-755)
//
// Grid-wide waits need every CTA resident: the kernel is launched
// cooperatively with one CTA per SM.  Every wait is bounded; a timeout sets a
// status bit, the CTA stops waiting and finishes (results then invalid, the
// host reports the status and resets the counters).
#include <cuda_fp16.h>

#include "expert_common.cuh"
#include "iq3xxs.cuh"
#include "kernels.h"

namespace gp {
namespace {

constexpr int NWC = 24;          // consumer warps
constexpr int NWG = 20;          // of which compute gate/up (32*20 lanes = 4 rows of 5120)
constexpr int NTHREADS = 32 * (NWC + 1);
constexpr int TRG = 8;           // gate/up rows per matrix per stage
constexpr int TRD = 32;          // down rows per stage
constexpr int RSPLIT = 8;        // router row slices
constexpr int MAXK = 32;
constexpr int kMaxEFused = 256;  // routed experts handled by the top-k warp

struct Smem {
    uint32_t stage_bytes, stages_off, partial_off, bar_off, misc_off, total;
};

__host__ __device__ inline Smem decode_smem(int H, int I, int S) {
    Smem L;
    const uint32_t gu = 2u * TRG * 98u * (H / 256), dn = TRD * 98u * (I / 256);
    L.stage_bytes = ((gu > dn ? gu : dn) + 15u) & ~15u;
    L.stages_off = GP_IQ3_TABLE_BYTES;
    L.partial_off = L.stages_off + S * L.stage_bytes;
    const uint32_t pb = (2 * TRG * NWG > TRD * NWC ? 2 * TRG * NWG : TRD * NWC) * 4u;
    L.bar_off = (L.partial_off + S * pb + 15u) & ~15u;
    L.misc_off = L.bar_off + (2u * S + 2u) * 8u;
    L.total = L.misc_off + 16u + 4u * S + 8u * MAXK + 8u * kMaxEFused + 16u;
    return L;
}

GP_DEVINL void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
GP_DEVINL unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded grid-wide wait for *p >= target.
GP_DEVINL bool wait_geq(const unsigned* p, unsigned target) {
    for (uint32_t i = 0; i < GP_SPIN_LIMIT; ++i) {
        if (ld_acquire(p) >= target) return true;
        __nanosleep(64);
    }
    return false;
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
        if (j < m.wspan) pbuf[(m.wrow0 + j + p * LM::ROWSTEP) * NW + warp] = red;
    }
}

// Loads and quantises this lane's 32 activations (sub-block sb of row `row`).
GP_DEVINL float load_quant(const void* x, int x_bf16, int64_t row, int in_dim, int sb, uint32_t (&xq)[16]) {
    float v[32];
    load_x_unit<32>(x, x_bf16, row, in_dim, 32 * sb, v);
    return 0.25f * quant_i16<32>(v, xq);
}

// Last of the NWC consumer warps to finish a stage?  (That warp then sums the
// stage's per-warp partials in warp order.)
GP_DEVINL bool stage_done(int* counter, int lane) {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(counter, 1) == NWC - 1;
        if (last) *counter = 0;
        __threadfence_block();
    }
    return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// One warp: top-K by choice (ties to the lower id) from the CTA's scores in
// shared memory, and the weights score/(1e-20 + sum)*scale (model.cpp:704-725);
// publishes them to the CTA.
GP_DEVINL void topk_warp(const DecodeLayerArgs& a, int lane, int c, const float* s_score, const float* s_choice,
                         int* s_ids, float* s_w, uint32_t topk_bar) {
    const int E = a.E, K = a.K;
    constexpr int EJ = kMaxEFused / 32;
    float score[EJ], choice[EJ];
#pragma unroll
    for (int j = 0; j < EJ; ++j) {
        const int e = lane + 32 * j;
        score[j] = e < E ? s_score[e] : 0.f;
        choice[j] = e < E ? s_choice[e] : -INFINITY;
    }
    float denom = 1e-20f, my_s = 0.f;
    int my_e = 0;
    for (int k = 0; k < K; ++k) {
        int eb;
        if (a.forced) {
            eb = a.forced[k];
            if (eb < 0 || eb >= E) {
                if (lane == 0) atomicOr(a.status, GP_DEV_BAD_EXPERT);
                eb = 0;
            }
        } else {
            float bv = -INFINITY;
            eb = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < EJ; ++j) {
                const int e = lane + 32 * j;
                if (e < E && (choice[j] > bv || (choice[j] == bv && e < eb))) { bv = choice[j]; eb = e; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oe = __shfl_xor_sync(0xffffffffu, eb, o);
                if (ov > bv || (ov == bv && oe < eb)) { bv = ov; eb = oe; }
            }
        }
        float sc = 0.f;
#pragma unroll
        for (int j = 0; j < EJ; ++j)
            if (lane + 32 * j == eb) { sc = score[j]; choice[j] = -INFINITY; }
        sc = __shfl_sync(0xffffffffu, sc, eb & 31);
        denom += sc;  // model.cpp:718-721 order
        if (lane == k) { my_s = sc; my_e = eb; }
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

// Shared-expert gate/up tiles of CTA cc: tiles cc, cc+G, ... below tg.
GP_DEVINL int shared_tiles(int cc, int G, int tg) { return cc < tg ? (tg - 1 - cc) / G + 1 : 0; }

template <int HH, int II, int PG, int RPWG, int PD, int RPWD>
__global__ void __launch_bounds__(NTHREADS, 1) decode_layer_kernel(const DecodeLayerArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    constexpr int H = HH, I = II;
    const int E = a.E, K = a.K, S = a.stages;
    const Smem L = decode_smem(H, I, S);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + L.bar_off, empty0 = full0 + 8u * S;
    const uint32_t tbar = empty0 + 8u * S, topk_bar = tbar + 8u;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off);
    int* s_done = reinterpret_cast<int*>(smem + L.misc_off + 16u);
    int* s_ids = reinterpret_cast<int*>(smem + L.misc_off + 16u + 4u * S);
    float* s_w = reinterpret_cast<float*>(s_ids + MAXK);
    float* s_score = s_w + MAXK;
    float* s_choice = s_score + kMaxEFused;
    const uint32_t gu_bytes = TRG * 98u * (H / 256), dn_bytes = TRD * 98u * (I / 256);
    const int TG = I / TRG, TD = H / TRD;             // tiles per expert
    // gate/up items per CTA are balanced over shared + routed tiles: CTA c
    // takes shared tiles c, c+G, ... and as many routed tiles as keeps its total
    // at floor((c+1)T/G) - floor(cT/G), T = TG * (K+1)
    const int nA = shared_tiles(c, G, TG);
    const int sharedA = (TG / G) * c + min(c, TG % G);  // shared tiles taken by CTAs before c
    const int T = TG * (K + 1), nD_total = (K + 1) * TD;
    const int rb = (int)((int64_t)T * c / G) - sharedA;
    const int re = (int)((int64_t)T * (c + 1) / G) - sharedA - nA;
    const int db = (int)((int64_t)nD_total * c / G), de = (int)((int64_t)nD_total * (c + 1) / G);
    const int n_gu = nA + (re - rb);
    const int n_items = n_gu + (de - db);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(empty0 + 8u * s, NWC);
            s_done[s] = 0;
        }
        mbar_init(tbar, 1);
        mbar_init(topk_bar, 1);
        *s_abort = gp_tables_at_base(smem) ? 0u : 1u;
        if (*s_abort) atomicOr(a.status, GP_DEV_BAD_SHAPE);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NWC) {
        // ================= producer =================
        if (lane == 0) {
            mbar_arrive_expect_tx(tbar, GP_IQ3_TABLE_BYTES);
            for (int k4 = 0; k4 < 4; ++k4) bulk_g2s(sbase + k4 * 16384u, a.tables + k4 * 16384, 16384u, tbar);
            int s = 0, issued = 0;
            uint32_t ph = 1;
            bool have_topk = false;
            for (int it = 0; it < n_items && !*s_abort; ++it, ++issued) {
                const uint8_t* src0;
                const uint8_t* src1 = nullptr;
                uint32_t bytes;
                if (it < nA) {                            // shared expert gate/up
                    const int64_t off = (int64_t)E * a.gu_stride + (int64_t)(c + it * G) * gu_bytes;
                    src0 = a.gate + off;
                    src1 = a.up + off;
                    bytes = gu_bytes;
                } else {
                    if (!have_topk) {                     // routed tiles need the top-k
                        if (!mbar_wait(topk_bar, 0)) {
                            *s_abort = 1;
                            atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
                            break;
                        }
                        have_topk = true;
                    }
                    if (it < n_gu) {                      // routed gate/up
                        const int r = rb + (it - nA), k = r / TG, t = r - k * TG;
                        const int64_t off = (int64_t)s_ids[k] * a.gu_stride + (int64_t)t * gu_bytes;
                        src0 = a.gate + off;
                        src1 = a.up + off;
                        bytes = gu_bytes;
                    } else {                              // down
                        const int r = db + (it - n_gu), slot = r / TD, t = r - slot * TD;
                        const int e = slot < K ? s_ids[slot] : E;
                        src0 = a.down + (int64_t)e * a.d_stride + (int64_t)t * dn_bytes;
                        bytes = dn_bytes;
                    }
                }
                if (!mbar_wait(empty0 + 8u * s, ph)) {
                    *s_abort = 1;
                    atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
                    break;
                }
                const uint32_t dst = sbase + L.stages_off + s * L.stage_bytes;
                mbar_arrive_expect_tx(full0 + 8u * s, src1 ? 2u * bytes : bytes);
                bulk_g2s(dst, src0, bytes, full0 + 8u * s);
                if (src1) bulk_g2s(dst + bytes, src1, bytes, full0 + 8u * s);
                if (++s == S) { s = 0; ph ^= 1u; }
            }
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                mbar_wait(full0 + 8u * (i % S), (uint32_t)(i / S) & 1u);
            mbar_wait(tbar, 0);
        }
        return;
    }

    // ================= consumers =================
    pdl_wait();
    const uint32_t stage0 = sbase + L.stages_off;
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    const uint32_t pstride = (2 * TRG * NWG > TRD * NWC ? 2 * TRG * NWG : TRD * NWC);

    // ---- router slices: warp task = (expert e, slice) ----
    {
        const int slice = H / RSPLIT;          // multiple of 128 (host-checked), <= 1024
        for (int task = c * NWC + warp; task < E * RSPLIT; task += G * NWC) {
            const int e = task % E, sl = task / E;
            const float* w = a.router + (int64_t)e * H + sl * slice + lane * 4;
            float acc = 0.f;
#pragma unroll
            for (int i0 = 0; i0 < 8; i0 += 4) {  // 4 weight + 4 activation float4s in flight
                float4 wv[4], xv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((i0 + i) * 128 < slice) wv[i] = *reinterpret_cast<const float4*>(w + (i0 + i) * 128);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((i0 + i) * 128 < slice) {
                        const int k0 = sl * slice + lane * 4 + (i0 + i) * 128;
                        if (a.x_bf16) {
                            const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + k0);
                            xv[i] = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                                __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
                        } else {
                            xv[i] = *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + k0);
                        }
                    }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((i0 + i) * 128 < slice) {
                        acc = fmaf(wv[i].x, xv[i].x, acc);
                        acc = fmaf(wv[i].y, xv[i].y, acc);
                        acc = fmaf(wv[i].z, xv[i].z, acc);
                        acc = fmaf(wv[i].w, xv[i].w, acc);
                    }
            }
            acc = warp_sum(acc);
            if (lane == 0) a.rpart[(int64_t)sl * E + e] = acc;
        }
        named_bar_sync(1, NWC * 32);
        if (tid == 0) {
            __threadfence();
            red_release_add(a.sync + 0, 1);
            if (!*s_abort && !wait_geq(a.sync + 0, (unsigned)G)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
        }
        named_bar_sync(1, NWC * 32);
        __threadfence();
    }

    // ---- logits -> scores (one thread per expert, slices added in order) ----
    for (int e = tid; e < E; e += NWC * 32) {
        float lg = 0.f;
        float v[RSPLIT];
#pragma unroll
        for (int sl = 0; sl < RSPLIT; ++sl) v[sl] = a.rpart[(int64_t)sl * E + e];
#pragma unroll
        for (int sl = 0; sl < RSPLIT; ++sl) lg += v[sl];
        const float sc = 1.0f / (1.0f + expf(-lg));
        s_score[e] = sc;
        s_choice[e] = sc + (a.corr ? a.corr[e] : 0.f);
    }
    named_bar_sync(1, NWC * 32);
    // ---- top-k (warp NWG: idle in the gate/up phase) ----
    if (warp == NWG) topk_warp(a, lane, c, s_score, s_choice, s_ids, s_w, topk_bar);

    if (!mbar_wait(tbar, 0) && lane == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
    int s = 0;
    uint32_t ph = 0;

    // ---- gate/up items: the shared expert's tiles, then the routed ones ----
    {
        const auto mg = lane_map<HH, NWG, PG>(warp < NWG ? warp : 0, lane, stage0);
        uint32_t xq[16];
        float sx4 = 0.f;
        if (warp < NWG) sx4 = load_quant(a.x, a.x_bf16, 0, H, mg.sb, xq);
        const int rs = 32 * NWG / (H / 32);
        for (int it = 0; it < n_gu; ++it) {
            int slot, tile;
            if (it < nA) { slot = K; tile = c + it * G; }
            else { const int r = rb + (it - nA); slot = r / TG; tile = r - slot * TG; }
            if (!*s_abort && !mbar_wait(full0 + 8u * s, ph)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            float* pbuf = partial + (size_t)s * pstride;
            if (!*s_abort && warp < NWG) consume<HH, NWG, PG, RPWG>(mg, s * L.stage_bytes, xq, sx4, pbuf, warp, lane);
            if (stage_done(s_done + s, lane) && !*s_abort) {
                for (int row = lane; row < TRG; row += 32) {
                    const int ur = TRG + row;
                    const int g0 = (row % rs) * (H / 32) / 32, g1 = ((row % rs + 1) * (H / 32) - 1) / 32;
                    const int u0 = (ur % rs) * (H / 32) / 32, u1 = ((ur % rs + 1) * (H / 32) - 1) / 32;
                    float gs = 0.f, us = 0.f;
                    for (int w = g0; w <= g1; ++w) gs += pbuf[row * NWG + w];
                    for (int w = u0; w <= u1; ++w) us += pbuf[ur * NWG + w];
                    a.h[(int64_t)slot * I + tile * TRG + row] = silu_clamped(gs, us, a.limit);
                }
                __syncwarp();
            }
            if (lane == 0) mbar_arrive(empty0 + 8u * s);
            if (++s == S) { s = 0; ph ^= 1u; }
        }
    }

    // every h written grid-wide before any down tile is consumed
    named_bar_sync(1, NWC * 32);
    if (tid == 0) {
        __threadfence();
        red_release_add(a.sync + 1, 1);
        if (!*s_abort && !wait_geq(a.sync + 1, (unsigned)G)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
    }
    named_bar_sync(1, NWC * 32);
    __threadfence();

    // ---- down items ----
    {
        const auto md = lane_map<II, NWC, PD>(warp, lane, stage0);
        uint32_t xq[16];
        float sx4 = 0.f;
        int cur_slot = -1;
        const int rs = 32 * NWC / (I / 32);
        for (int it = n_gu; it < n_items; ++it) {
            const int r = db + (it - n_gu), slot = r / TD, tile = r - slot * TD;
            if (slot != cur_slot) {
                cur_slot = slot;
                sx4 = load_quant(a.h, 0, slot, I, md.sb, xq);
            }
            if (!*s_abort && !mbar_wait(full0 + 8u * s, ph)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
            float* pbuf = partial + (size_t)s * pstride;
            if (!*s_abort) consume<II, NWC, PD, RPWD>(md, s * L.stage_bytes, xq, sx4, pbuf, warp, lane);
            if (stage_done(s_done + s, lane) && !*s_abort) {
                for (int row = lane; row < TRD; row += 32) {
                    const int r0 = row % rs;
                    const int w0 = r0 * (I / 32) / 32, w1 = ((r0 + 1) * (I / 32) - 1) / 32;
                    float dsum = 0.f;
                    for (int w = w0; w <= w1; ++w) dsum += pbuf[row * NWC + w];
                    a.D[(int64_t)slot * H + tile * TRD + row] = dsum;
                }
                __syncwarp();
            }
            if (lane == 0) mbar_arrive(empty0 + 8u * s);
            if (++s == S) { s = 0; ph ^= 1u; }
        }
    }

    // ---- combine: this CTA's slice of rows ----
    named_bar_sync(1, NWC * 32);
    if (tid == 0) {
        __threadfence();
        red_release_add(a.sync + 2, 1);
        if (!*s_abort && !wait_geq(a.sync + 2, (unsigned)G)) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
    }
    named_bar_sync(1, NWC * 32);
    __threadfence();
    {
        const int j0 = (int)((int64_t)H * c / G), j1 = (int)((int64_t)H * (c + 1) / G);
        for (int j = j0 + tid; j < j1; j += NWC * 32) {
            float acc = 0.f;
            for (int k = 0; k < K; ++k) acc = fmaf(s_w[k], a.D[(int64_t)k * H + j], acc);
            if (a.with_shared) acc += a.D[(int64_t)K * H + j];
            a.y[j] = acc;
        }
    }
    // the last CTA out resets the counters for the next launch
    named_bar_sync(1, NWC * 32);
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.sync + 3, 1u) == (unsigned)G - 1) {
            a.sync[0] = 0;
            a.sync[1] = 0;
            a.sync[2] = 0;
            __threadfence();
            a.sync[3] = 0;
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
    const Smem L = decode_smem(a.H, a.I, a.stages);
    if (L.total > 227u * 1024u) return cudaErrorInvalidValue;
    auto kern = decode_layer_kernel<5120, 1536, 4, 1, 2, 2>;
    static int configured = 0;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace gp
