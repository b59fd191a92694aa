// Large-batch (prefill) MoE experts on the 5th-generation tensor cores.
//
// For each expert slot (expert e, up to 256 token rows in expert-sorted
// order) and each 128-row tile of an expert matrix, one CTA computes
//   D[row][tok] = sum_k W[row][k] * X[tok][k]
// with tcgen05.mma (kind::f16, fp16 operands, fp32 accumulators in TMEM).
// The weights stay IQ3_XXS in HBM: decode warps turn each 128 x 64 slice into
// fp16 straight into the 128-byte-swizzled operand layout in shared memory:
// the reference's weight d*(0.5+s)*0.5*g*sign, computed as fp16(db)*g rounded
// to fp16 (relative error <= 2^-10 per weight; 3.6e-4 relative L2 on one
// 5120-deep GEMM with fp16 activations, against 2.9e-4 with one rounding).
//
//   gate/up pass  A = gate and up tiles (two accumulators), B = the tokens'
//                 rows (fp16); epilogue SwiGLU with the reference clamp
//                 (model_batch.cpp:249-253) -> h [position][I] fp16
//   down pass     A = down tile, B = h rows; epilogue -> D [position][H] fp32,
//                 then the batched path's combine (model_batch.cpp:257-280)
//
// Warp roles (one CTA per SM, persistent over the tile list):
//   warp 0     TMA producer of the token tiles (2-D, 128-byte swizzle), a ring
//              freed by the MMA
//   warp 1     TMEM allocation; one thread issues the MMAs and commits
//   warp 2     TMA producer of the raw IQ3_XXS bytes (3-D maps over the
//              row-group layout: index bytes, sign/scale words, per-tile fp16
//              scales), a deeper ring freed by the decoders, so that weight
//              loads run several K slices ahead of the decode
//   warps 3-6  epilogue: TMEM -> registers -> global (one lane quadrant each)
//   warps 7+   decode: one sub-block per thread per matrix per K slice
//              (8 warps per matrix); in the gate/up pass they then join the
//              epilogue, which splits each lane quadrant's columns
// 736 threads for gate/up, 480 for down.
// No cluster, no multicast.  Every wait is bounded; a timeout sets a status bit.
#include <cuda_fp16.h>

#include "expert_common.cuh"
#include "iq3xxs.cuh"
#include "kernels.h"
#include "tc_common.cuh"

// Timing hooks: no-ops here; a profiling build may define them to accumulate
// per-role wait and work cycles.
#ifndef TC_MARK
#define TC_DECL() ((void)0)
#define TC_MARK(v) ((void)0)
#define TC_ACC(i, v) ((void)0)
#define TC_DUMP(gu, role) ((void)0)
#endif

namespace gp {
namespace {

constexpr int TBM = 128;  // weight rows per tile (MMA M = TMEM lanes)
constexpr int TBN = 224;  // token rows per slot (MMA N <= 224: two accumulators + A stages fit TMEM)
constexpr int TBK = 64;   // K per slice (one 128-byte swizzled fp16 row)
constexpr int TAS = 2;    // decoded weight stages
constexpr int NEPI = 4;   // epilogue warps
// warp roles: token-tile producer, MMA issue, raw-weight producer, epilogue, decode
constexpr int WPB = 0, WMMA = 1, WPR = 2, WEPI0 = 3, WDEC0 = 7;
constexpr uint32_t B_TILE = TBN * TBK * 2;  // 28 KB
constexpr uint32_t A_TILE = TBM * TBK * 2;  // 16 KB
constexpr uint32_t RAW_QS = TBM * 16;       // 2 sub-blocks x 8 index bytes per row
constexpr uint32_t RAW_AUX = TBM * 16;      // 4 sign/scale words per row (2 used)
constexpr uint32_t TC_SMEM_MAX = 227u * 1024u;

// Per pass: the token ring is freed by the MMA, the raw-weight ring by the
// decoders as soon as they have decoded a slice, so raw loads run several
// slices ahead of the decode.  Depths and codebook copies fill shared memory.
// The down pass keeps its decoded weights in tensor memory (TA): its two
// accumulators take 2 x 224 columns and the two A stages the last 64, so the
// decoded tile never passes through shared memory.  The gate/up pass needs
// 2 x 224 columns for one gate and one up accumulator and stages A in shared
// memory.
template <bool GU>
struct TcCfg {
    static constexpr int NM = GU ? 2 : 1;   // weight matrices (gate and up, or down)
    static constexpr bool TA = !GU;         // A operand in tensor memory
    static constexpr int TSB = GU ? 3 : 5;  // token-tile stages
    static constexpr int TSR = GU ? 4 : 8;  // raw-weight stages
    static constexpr int GSH = 4;           // log2 of the interleaved codebook copies
    static constexpr int NDEC = 8 * NM;     // decode warps: one sub-block per thread per slice
    static constexpr int THREADS = 32 * (WDEC0 + NDEC);
};
constexpr uint32_t TMEM_A_COL = 2 * TBN;  // first column of the A stages (down pass)

struct TcSmem {
    uint32_t raw_stage, raw_off, a_off, d_off, dbytes, grid_off, bar_off, total;
};

template <bool GU>
__host__ __device__ inline TcSmem tc_smem(int kin) {
    using C = TcCfg<GU>;
    TcSmem L;
    L.raw_stage = C::NM * (RAW_QS + RAW_AUX);
    L.raw_off = C::TSB * B_TILE;  // token tiles first (1024-byte aligned for the swizzle)
    L.a_off = L.raw_off + C::TSR * L.raw_stage;
    L.dbytes = (uint32_t)(256 * (kin / 256) + 127) & ~127u;  // 16 groups x 16 * NBLK bytes
    L.d_off = L.a_off + (C::TA ? 0 : TAS * C::NM * A_TILE);
    L.grid_off = L.d_off + 2 * C::NM * L.dbytes;
    L.bar_off = L.grid_off + (1024u << C::GSH);
    L.total = L.bar_off + 512 + 1024;  // barriers + TMEM slot; 1 KB alignment slack
    return L;
}

struct TcMaps {
    CUtensorMap b;         // token rows, fp16 [positions][kin], box {64, TBN}, 128-byte swizzle
    CUtensorMap bh[4];     // the same rows in boxes of 16, 32, 64 and 128 rows (slots of few tokens)
    CUtensorMap qs[2];     // per matrix: index bytes {64*NBLK, 8, groups}, box {16, 8, 16}
    CUtensorMap aux[2];    // sign/scale words {32*NBLK, 8, groups}, box {16, 8, 16}
    CUtensorMap dsc[2];    // fp16 scales {16*NBLK/q, q, groups}, box {16*NBLK/q, q, 16}
};

// Sign mask of weight pair p (weights 2p, 2p+1) of a sign group: s8 = the 8
// sign bits (bit 7 = parity; bits 8-9 may hold garbage).  One multiply puts
// bit 2p on bit 15 and bit 2p+1 on bit 31 (the two shifted copies of s8 do
// not overlap, so nothing carries into them).
template <int P>
GP_DEVINL uint32_t pair_sign(uint32_t s8) {
    return s8 * ((1u << (15 - 2 * P)) | (1u << (30 - 2 * P)));
}

// Decode of one sub-block: F16 computes each pair in fp16 arithmetic, the
// other form in fp32 (for the rare scales whose fp16 intermediates would
// overflow).  Per weight pair:
//   F16   one byte permute builds the fp16 pair (1024+g0, 1024+g1); one fp16
//         FMA with db16 = fp16(db) gives (1024+g)*db16 - 1024*db16 =
//         round_fp16(g*db16) (the product is exact before the final rounding;
//         -1024*db16 is a power-of-two scaling)
//   fp32  byte permutes build floats 2^23+g; fma(db, 2^23+g, -db*2^23) is the
//         reference's fp32 product db*g, rounded once to fp16
// then one LOP3 applies the signs.
// Codebook word at shared address a (read-only after the kernel's set-up barrier).
GP_DEVINL uint32_t lds_grid(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

// TM: the 16 words (weight pairs in K order) go to o[] for a tensor-memory
// store; otherwise to the swizzled shared-memory row (row_addr, phase c0).
template <bool F16, bool TM>
GP_DEVINL void decode_sub(uint32_t row_addr, uint32_t c0, uint2 q, uint32_t w, float db, uint32_t gaddr,
                          uint32_t gstride, uint32_t (&o)[16]) {
    const __half2 dbh = __float2half2_rn(db);
    const __half2 ndbh = __float2half2_rn(-1024.0f * db);
    const float ndb = -db * 8388608.0f;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        // 8 sign bits: the 7-bit field and its parity (the reference's ksigns table)
        // w >> 7l as a high multiply (FMA pipe) rather than a shift (ALU pipe)
        const uint32_t k7 = (l == 0 ? w : __umulhi(w, 1u << ((32 - 7 * l) & 31))) & 127u;
        const uint32_t s8 = (uint32_t)__popc(k7) * 128u + k7;
        const uint32_t wd = l < 2 ? q.x : q.y;
        const uint32_t g0 = lds_grid(prmt(wd, 0u, 0x4440u | (2u * (l & 1))) * gstride + gaddr);
        const uint32_t g1 = lds_grid(prmt(wd, 0u, 0x4440u | (2u * (l & 1) + 1u)) * gstride + gaddr);
        const uint32_t m[4] = {pair_sign<0>(s8), pair_sign<1>(s8), pair_sign<2>(s8), pair_sign<3>(s8)};
        uint32_t h[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const uint32_t gw = p < 2 ? g0 : g1;
            uint32_t v;
            if (F16) {
                const uint32_t hb = prmt(gw, 0x64646464u, (p & 1) ? 0x5342u : 0x5140u);
                const __half2 r2 = __hfma2(*reinterpret_cast<const __half2*>(&hb), dbh, ndbh);
                v = *reinterpret_cast<const uint32_t*>(&r2);
            } else {
                const float fa = __uint_as_float(prmt(gw, 0x4B000000u, 0x7540u | ((2 * p) & 3)));
                const float fb = __uint_as_float(prmt(gw, 0x4B000000u, 0x7540u | ((2 * p + 1) & 3)));
                const __half2 hp = __floats2half2_rn(__fmaf_rn(db, fa, ndb), __fmaf_rn(db, fb, ndb));
                v = *reinterpret_cast<const uint32_t*>(&hp);
            }
            h[p] = v ^ (m[p] & 0x80008000u);
            if (TM) o[4 * l + p] = h[p];
        }
        if (!TM)
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr + ((c0 ^ (uint32_t)l) << 4)),
                         "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]));
    }
}

// One K slice of one weight matrix: thread (r, hf) decodes sub-block 2*(c%4)+hf
// of block c/4 in row r, into the 128-byte-swizzled fp16 tile (row_addr = the
// row in the tile, c0 = its swizzle phase) or, with TM, into o[] for tensor
// memory (qp, wp, dp = the thread's index bytes, sign/scale word and fp16
// block scale).
//
// Shared-memory bandwidth and instruction issue bound this decode: the tensor
// core reads its operands from the same shared memory, and the ALU pipe
// issues at half the rate of the FMA pipe.  So the sign masks come from
// multiplies rather than a table, and the codebook is read from one of
// several interleaved copies (gaddr = this lane's copy, gstride = bytes per
// entry across copies), so that a warp's random lookups cost few wavefronts.
template <bool TM>
GP_DEVINL void decode_slice(uint32_t row_addr, uint32_t c0, const uint8_t* qp, const uint8_t* wp, const uint8_t* dp,
                            uint32_t gaddr, uint32_t gstride, uint32_t (&o)[16]) {
    const uint2 q = *reinterpret_cast<const uint2*>(qp);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(wp);
    const float db = iq3_db(__half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(dp))), w);
    // fp16 intermediates reach 1086*|db|: below 65504 with margin
    if (__builtin_expect(fabsf(db) < 32.0f, 1))
        decode_sub<true, TM>(row_addr, c0, q, w, db, gaddr, gstride, o);
    else
        decode_sub<false, TM>(row_addr, c0, q, w, db, gaddr, gstride, o);
}

GP_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

GP_DEVINL void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(mbar)
        : "memory");
}

template <bool GU>
__global__ void __launch_bounds__(TcCfg<GU>::THREADS, 1)
    tc_moe_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    using C = TcCfg<GU>;
    constexpr int NM = C::NM, NDEC = C::NDEC, TSB = C::TSB, TSR = C::TSR;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t base = (raw0 + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw0);
    const TcSmem L = tc_smem<GU>(a.kin);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.kin / 256, nk = a.kin / TBK;
    const uint32_t bar = base + L.bar_off;
    const uint32_t sb_full = bar, sb_empty = sb_full + 8 * TSB, sr_full = sb_empty + 8 * TSB;
    const uint32_t sr_empty = sr_full + 8 * TSR, a_full = sr_empty + 8 * TSR, a_empty = a_full + 8 * TAS;
    const uint32_t d_full = a_empty + 8 * TAS, d_empty = d_full + 16, acc_full = d_empty + 16, acc_empty = acc_full + 16;
    const uint32_t tslot = acc_empty + 16;
    const int nslots = *a.nslots;
    const int ntiles = nslots * a.mt;
    TC_DECL();

    if (tid == 0) {
        for (int s = 0; s < TSB; ++s) { mbar_init(sb_full + 8 * s, 1); mbar_init(sb_empty + 8 * s, 1); }
        for (int s = 0; s < TSR; ++s) { mbar_init(sr_full + 8 * s, 1); mbar_init(sr_empty + 8 * s, NDEC); }
        for (int s = 0; s < TAS; ++s) { mbar_init(a_full + 8 * s, NDEC); mbar_init(a_empty + 8 * s, 1); }
        for (int s = 0; s < 2; ++s) {
            mbar_init(d_full + 8 * s, 1);
            mbar_init(d_empty + 8 * s, NDEC);
            mbar_init(acc_full + 8 * s, 1);
            mbar_init(acc_empty + 8 * s, GU ? NEPI + NDEC : NEPI);  // the epilogue warps
        }
        fence_mbar_init();
    }
    {
        uint32_t* s_grid = reinterpret_cast<uint32_t*>(gbase + L.grid_off);
        for (int i = tid; i < (256 << C::GSH); i += C::THREADS) s_grid[i] = gp_iq3xxs_grid_dev[i >> C::GSH];
    }
    if (warp == WMMA) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *reinterpret_cast<volatile uint32_t*>(gbase + (tslot - base));

    if (warp == WPB) {
        // ================= token-tile producer =================
        if (lane == 0) {
            TC_MARK(t_all);
            int sb = 0;
            uint32_t bph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const SlotDesc sd = a.slots[t / a.mt];
                const int row0 = sd.begin;
                // the smallest box holding the slot's rows (the MMA reads N = rows rounded up to 16):
                // a slot of a few tokens moves a few KB per slice instead of TBN rows
                const int hc = sd.ntok <= 16 ? 0 : sd.ntok <= 32 ? 1 : sd.ntok <= 64 ? 2 : sd.ntok <= 128 ? 3 : 4;
                const CUtensorMap* bm = hc < 4 ? &maps.bh[hc] : &maps.b;
                const uint32_t bbytes = (hc < 4 ? (16u << hc) : (uint32_t)TBN) * TBK * 2u;
                for (int c = 0; c < nk; ++c) {
                    TC_MARK(t_se);
                    if (!mbar_wait(sb_empty + 8 * sb, bph ^ 1u)) { ok = false; break; }
                    TC_ACC(0, t_se);
                    mbar_arrive_expect_tx(sb_full + 8 * sb, bbytes);
                    tma_load_2d(base + sb * B_TILE, bm, c * TBK, row0, sb_full + 8 * sb);
                    if (++sb == TSB) { sb = 0; bph ^= 1u; }
                }
            }
            if (!ok) atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
            TC_ACC(7, t_all);
            TC_DUMP(GU, 0);
        }
    } else if (warp == WPR) {
        // ================= raw-weight producer: per-tile scales, then per-slice bytes =================
        if (lane == 0) {
            TC_MARK(t_all);
            int sr = 0;
            uint32_t rph = 0;
            bool ok = true;
            for (int t = blockIdx.x, lt = 0; t < ntiles && ok; t += gridDim.x, ++lt) {
                const SlotDesc sd = a.slots[t / a.mt];
                const int z0 = (sd.expert * a.nout + (t % a.mt) * TBM) / 8;
                const int db = lt & 1;
                TC_MARK(t_de);
                if (!mbar_wait(d_empty + 8 * db, ((lt >> 1) & 1) ^ 1)) { ok = false; break; }
                TC_ACC(1, t_de);
                mbar_arrive_expect_tx(d_full + 8 * db, NM * 16 * 16 * nblk);
                for (int mi = 0; mi < NM; ++mi)
                    tma_load_3d(base + L.d_off + (db * NM + mi) * L.dbytes, &maps.dsc[mi], 0, 0, z0, d_full + 8 * db);
                for (int c = 0; c < nk; ++c) {
                    TC_MARK(t_re);
                    if (!mbar_wait(sr_empty + 8 * sr, rph ^ 1u)) { ok = false; break; }
                    TC_ACC(2, t_re);
                    const uint32_t rb = base + L.raw_off + sr * L.raw_stage;
                    mbar_arrive_expect_tx(sr_full + 8 * sr, L.raw_stage);
                    for (int mi = 0; mi < NM; ++mi) {
                        const uint32_t rq = rb + mi * (RAW_QS + RAW_AUX);
                        tma_load_3d(rq, &maps.qs[mi], 64 * (c >> 2) + 16 * (c & 3), 0, z0, sr_full + 8 * sr);
                        tma_load_3d(rq + RAW_QS, &maps.aux[mi], 32 * (c >> 2) + 16 * ((c & 3) >> 1), 0, z0,
                                    sr_full + 8 * sr);
                    }
                    if (++sr == TSR) { sr = 0; rph ^= 1u; }
                }
            }
            if (!ok) atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
            TC_ACC(6, t_all);
            TC_DUMP(GU, 0);
        }
    } else if (warp == WMMA) {
        // ================= MMA issue =================
        if (lane == 0) {
            TC_MARK(t_all);
            int sb = 0, as = 0;
            uint32_t bph = 0, aph = 0;
            bool ok = true;
            for (int t = blockIdx.x, lt = 0; t < ntiles && ok; t += gridDim.x, ++lt) {
                // N follows the slot's rows (multiple of 16, as M = 128 requires)
                const int ntok = a.slots[t / a.mt].ntok;
                const uint32_t idesc = umma_idesc_f16(TBM, ntok >= TBN ? TBN : (ntok + 15) & ~15, false);
                const int ab = GU ? 0 : (lt & 1);
                const uint32_t ph_e = GU ? ((lt & 1) ^ 1) : (((lt >> 1) & 1) ^ 1);
                TC_MARK(t_ae);
                if (!mbar_wait(acc_empty + 8 * ab, ph_e)) { ok = false; break; }
                TC_ACC(0, t_ae);
                tc_fence_after();
                for (int c = 0; c < nk; ++c) {
                    TC_MARK(t_af);
                    if (!mbar_wait(a_full + 8 * as, aph)) { ok = false; break; }
                    TC_ACC(1, t_af);
                    TC_MARK(t_sf);
                    if (!mbar_wait(sb_full + 8 * sb, bph)) { ok = false; break; }
                    TC_ACC(2, t_sf);
                    tc_fence_after();
                    const uint32_t bt = base + sb * B_TILE;
#pragma unroll
                    for (int kk = 0; kk < TBK / 16; ++kk) {
                        const uint64_t bdesc = umma_desc_sw128(bt + kk * 32);
#pragma unroll
                        for (int mi = 0; mi < NM; ++mi) {
                            const uint32_t dt = tbase + (GU ? mi * TBN : ab * TBN);
                            if (C::TA) {  // K = 16 per MMA: 8 columns of the A stage
                                umma_f16_ts(dt, tbase + TMEM_A_COL + 32 * as + 8 * kk, bdesc, idesc, (c | kk) != 0);
                            } else {
                                const uint32_t at = base + L.a_off + (as * NM + mi) * A_TILE;
                                umma_f16(dt, umma_desc_sw128(at + kk * 32), bdesc, idesc, (c | kk) != 0);
                            }
                        }
                    }
                    umma_commit(a_empty + 8 * as);
                    umma_commit(sb_empty + 8 * sb);
                    if (++sb == TSB) { sb = 0; bph ^= 1u; }
                    if (++as == TAS) { as = 0; aph ^= 1u; }
                }
                if (ok) umma_commit(acc_full + 8 * ab);
            }
            if (!ok) atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
            TC_ACC(7, t_all);
            TC_DUMP(GU, 1);
        }
    } else {
        // ================= workers: decode (warps >= WDEC0), then the epilogue =================
        // The epilogue of a tile is shared by every worker warp of the same TMEM
        // lane quadrant (warp % 4).  In the gate/up pass the decode warps join
        // it: that pass has a single accumulator (gate and up fill all 512
        // TMEM columns), so the MMA waits until the epilogue has read it.
        constexpr int NEP = GU ? NEPI + NDEC : NEPI;  // epilogue warps
        constexpr int PER_Q = NEP / 4;                // of them per lane quadrant
        const int wk = warp - WEPI0, q = warp & 3, kq = wk / 4;
        const bool decoder = warp >= WDEC0, epi = wk < NEP;
        // decode thread -> (matrix, row, half).  Tensor-memory A: lane = row, so a
        // warp takes the 32 rows of its TMEM lane quadrant (warp % 4) and one half.
        const int td = tid - 32 * WDEC0;
        const int mi = C::TA ? 0 : td >> 8;
        const int r = C::TA ? 32 * q + lane : (td >> 1) & 127;
        const int hf = C::TA ? (td >> 7) & 1 : td & 1;
        const uint32_t a_tm = tbase + ((uint32_t)(32 * q) << 16) + TMEM_A_COL + 16 * hf;
        // the decode thread's fixed offsets: its row in the A tile, its bytes in a raw stage
        const uint32_t gstride = 4u << C::GSH;
        const uint32_t gaddr = base + L.grid_off + 4u * ((uint32_t)lane & ((1u << C::GSH) - 1u));
        const uint32_t a_row = base + L.a_off + mi * A_TILE + (uint32_t)r * 128u;
        const uint32_t c0 = (uint32_t)(4 * hf) ^ (uint32_t)(r & 7);
        const uint8_t* raw_t = gbase + L.raw_off + mi * (RAW_QS + RAW_AUX) + r * 16;
        const uint8_t* d_t = gbase + L.d_off + mi * L.dbytes + (r >> 3) * 16 * nblk + (r & 7) * 2 * nblk;
        int sr = 0, as = 0;         // stage of the raw ring and of the A ring
        uint32_t rph = 0, aph = 0;  // their phase parities
        bool ok = true;
        bool h_over = false;  // an h value past the fp16 range (gate/up epilogue)
        TC_MARK(t_all);
        for (int t = blockIdx.x, lt = 0; t < ntiles && ok; t += gridDim.x, ++lt) {
            if (decoder) {
                const int db = lt & 1;
                TC_MARK(t_df);
                if (!mbar_wait(d_full + 8 * db, (lt >> 1) & 1)) { ok = false; break; }
                TC_ACC(0, t_df);
                const uint8_t* dsc = d_t + db * NM * L.dbytes;
                for (int c = 0; c < nk; ++c) {
                    TC_MARK(t_sf);
                    if (!mbar_wait(sr_full + 8 * sr, rph)) { ok = false; break; }
                    TC_ACC(1, t_sf);
                    TC_MARK(t_ae);
                    if (!mbar_wait(a_empty + 8 * as, aph ^ 1u)) { ok = false; break; }
                    TC_ACC(2, t_ae);
                    TC_MARK(t_dec);
                    const uint8_t* rq = raw_t + sr * L.raw_stage;
                    uint32_t o[16];
                    if (C::TA) tc_fence_after();  // the MMA that read this stage has completed
                    decode_slice<C::TA>(a_row + as * (NM * A_TILE), c0, rq + hf * 8,
                                        rq + RAW_QS + (c & 1) * 8 + hf * 4, dsc + 2 * (c >> 2), gaddr, gstride, o);
                    TC_ACC(3, t_dec);
                    TC_MARK(t_fa);
                    if (C::TA) {
                        tmem_st16(a_tm + 32 * as, o);
                        tmem_wait_st();
                        tc_fence_before();
                    } else {
                        fence_proxy_async_smem();  // the tensor core reads these writes through the async proxy
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(a_full + 8 * as);
                        mbar_arrive(sr_empty + 8 * sr);
                    }
                    if (++sr == TSR) { sr = 0; rph ^= 1u; }
                    if (++as == TAS) { as = 0; aph ^= 1u; }
                    TC_ACC(4, t_fa);
                }
                __syncwarp();
                if (!ok) break;
                if (lane == 0) mbar_arrive(d_empty + 8 * db);
            }
            if (!epi) continue;
            const SlotDesc sd = a.slots[t / a.mt];
            const int row = (t % a.mt) * TBM + 32 * q + lane;
            const int ab = GU ? 0 : (lt & 1);
            const uint32_t ph = GU ? (lt & 1) : ((lt >> 1) & 1);
            TC_MARK(t_af);
            if (!mbar_wait_sleepy(acc_full + 8 * ab, ph)) { ok = false; break; }  // a tile takes ~40 us
            TC_ACC(5, t_af);
            TC_MARK(t_ep);
            tc_fence_after();
            const uint32_t lanebase = tbase + ((uint32_t)(32 * q) << 16);
            if (GU) {
                for (int j0 = 16 * kq; j0 < TBN && j0 < sd.ntok; j0 += 16 * PER_Q) {
                    uint32_t v0[16], v1[16];
                    tmem_ld16(lanebase + j0, v0);
                    tmem_ld16(lanebase + TBN + j0, v1);
                    __half* h = static_cast<__half*>(a.out);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        if (j0 + jj < sd.ntok)
                            h[(int64_t)(sd.begin + j0 + jj) * a.nout + row] =
                                silu_clamped_h(__uint_as_float(v0[jj]), __uint_as_float(v1[jj]), a.limit, h_over);
                }
            } else {
                for (int j0 = 32 * kq; j0 < TBN && j0 < sd.ntok; j0 += 32 * PER_Q) {
                    uint32_t v0[32];
                    tmem_ld32(lanebase + ab * TBN + j0, v0);
                    float* d = static_cast<float*>(a.out);
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        if (j0 + jj < sd.ntok) d[(int64_t)(sd.begin + j0 + jj) * a.nout + row] = __uint_as_float(v0[jj]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
            TC_ACC(6, t_ep);
        }
        if (!ok && lane == 0) atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
        if (__any_sync(0xffffffffu, h_over) && lane == 0) atomicOr(a.status, GP_DEV_FP16_RANGE);
        TC_ACC(7, t_all);
        if (lane == 0 && (warp == WDEC0 || warp == WEPI0)) TC_DUMP(GU, warp == WDEC0 ? 2 : 3);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == WMMA) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// Casts token rows to fp16 in expert-sorted order: xp[p] = x[perm[p]].  One
// CTA per row at a time, 16-byte loads and stores.
__global__ void __launch_bounds__(128) gather_cast_kernel(const void* x, int x_bf16, const int* perm, int npos, int H,
                                                          __half* xp, uint32_t* status) {
    const int qpr = H / 8;  // 8 elements per thread step
    bool over = false;      // a value that rounds to an fp16 infinity (|v| >= 65520)
    for (int p = blockIdx.x; p < npos; p += gridDim.x) {
        const int64_t src = (int64_t)perm[p] * H;
        uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)p * H);
        for (int q = threadIdx.x; q < qpr; q += blockDim.x) {
            float v[8];
            if (x_bf16) {
                const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + src + q * 8);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[2 * j] = __uint_as_float(w[j] << 16);
                    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
                }
            } else {
                const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src + q * 8);
                const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src + q * 8 + 4);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) over |= fabsf(v[j]) >= 65520.0f;
            uint4 o;
            __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
            __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
            o.z = *reinterpret_cast<uint32_t*>(&h2);
            o.w = *reinterpret_cast<uint32_t*>(&h3);
            dst[q] = o;
        }
    }
    if (__any_sync(0xffffffffu, over) && (threadIdx.x & 31) == 0) atomicOr(status, GP_DEV_FP16_RANGE);
}

// Maps for one repacked IQ3_XXS matrix of `groups` 8-row groups, kin inputs.
bool encode_weight_maps(TcMaps& m, int mi, const uint8_t* w, int64_t groups, int kin) {
    const int nblk = kin / 256;
    const cuuint64_t gstride = 784ull * nblk;
    {
        const cuuint64_t dims[3] = {64ull * nblk, 8, (cuuint64_t)groups};
        const cuuint64_t str[2] = {64ull * nblk, gstride};
        const cuuint32_t box[3] = {16, 8, 16};
        if (!encode(&m.qs[mi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    {
        const cuuint64_t dims[3] = {32ull * nblk, 8, (cuuint64_t)groups};
        const cuuint64_t str[2] = {32ull * nblk, gstride};
        const cuuint32_t box[3] = {16, 8, 16};
        if (!encode(&m.aux[mi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, w + 512ull * nblk, dims, str, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    {
        // a group's 16 * NBLK scale bytes as q rows of 16 * NBLK / q (one box row at most 256 bytes,
        // a whole number of 16-byte units): q = the smallest divisor of NBLK leaving <= 16 blocks
        int q = 1;
        while (nblk / q > 16 || nblk % q) ++q;
        const cuuint64_t dims[3] = {16ull * nblk / q, (cuuint64_t)q, (cuuint64_t)groups};
        const cuuint64_t str[2] = {16ull * nblk / q, gstride};
        const cuuint32_t box[3] = {(cuuint32_t)(16 * nblk / q), (cuuint32_t)q, 16};
        if (!encode(&m.dsc[mi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, w + 768ull * nblk, dims, str, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    return true;
}

}  // namespace

int tc_moe_slot_tokens() { return TBN; }

bool tc_moe_supported(int H, int I) {
    return H % 256 == 0 && I % 256 == 0 && H % TBM == 0 && I % TBM == 0 && tc_smem<true>(H).total <= TC_SMEM_MAX &&
           tc_smem<false>(I).total <= TC_SMEM_MAX;
}

cudaError_t launch_gather_cast(const void* x, int x_bf16, const int* perm, int npos, int H, uint16_t* xp,
                               uint32_t* status, cudaStream_t st) {
    if (npos <= 0) return cudaSuccess;
    gather_cast_kernel<<<148 * 16, 128, 0, st>>>(x, x_bf16, perm, npos, H, reinterpret_cast<__half*>(xp), status);
    return cudaGetLastError();
}

// gate/up (gu = true: w0 gate, w1 up, B = xp [npos][kin]) or down (w0, B = h).
cudaError_t launch_tc_moe(bool gu, const uint8_t* w0, const uint8_t* w1, int64_t weight_rows, const uint16_t* b,
                          int npos, const TcArgs& args, int grid, cudaStream_t st) {
    TcMaps m{};
    const int kin = args.kin;
    if (kin % 256 || kin % TBM || args.nout % TBM || npos <= 0 || weight_rows % 8)
        return cudaErrorInvalidValue;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)kin, (cuuint64_t)npos};
        const cuuint64_t str[1] = {(cuuint64_t)kin * 2};
        const cuuint32_t box[2] = {TBK, TBN};
        if (!encode(&m.b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        for (int hc = 0; hc < 4; ++hc) {
            const cuuint32_t boxh[2] = {TBK, 16u << hc};
            if (!encode(&m.bh[hc], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, dims, str, boxh, CU_TENSOR_MAP_SWIZZLE_128B))
                return cudaErrorInvalidValue;
        }
    }
    if (!encode_weight_maps(m, 0, w0, weight_rows / 8, kin)) return cudaErrorInvalidValue;
    if (gu && !encode_weight_maps(m, 1, w1, weight_rows / 8, kin)) return cudaErrorInvalidValue;
    const TcSmem L = gu ? tc_smem<true>(kin) : tc_smem<false>(kin);
    if (L.total > TC_SMEM_MAX) return cudaErrorInvalidValue;
    auto kern = gu ? tc_moe_kernel<true> : tc_moe_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    kern<<<grid, gu ? TcCfg<true>::THREADS : TcCfg<false>::THREADS, L.total, st>>>(m, args);
    return cudaGetLastError();
}

}  // namespace gp
