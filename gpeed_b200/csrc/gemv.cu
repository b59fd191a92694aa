// Fused IQ3_XXS-decode GEMV for the expert path (decode and small ragged
// batches).  Replaces the reference's per-row dequantize_row + dot_f32 loop
// (cpp/core/src/weights.cpp:167-203 matvec_quant, :86-165 matmul_quant) and the
// per-expert gate/up -> SwiGLU (cpp/core/src/model.cpp:733-739,
// model_batch.cpp:241-253) that follows it.
//
// Structure (one persistent CTA per SM):
//   * a producer warp streams row tiles of the repacked weight matrices into a
//     ring of shared-memory stages with 1-D bulk copies (TMA engine), one
//     mbarrier per stage for "full" and one for "empty";
//   * consumer warps own a fixed K-slice (32 lanes x UNIT weights) and keep
//     that slice of each token's activations in registers as int16 pairs, so
//     the only shared-memory traffic per 4 weights is one conflict-free
//     codebook lookup;
//   * per row, lane sums are reduced across the warp, K-slices are summed in a
//     fixed order (deterministic), and the epilogue applies SwiGLU with the
//     reference's clamp (gate/up mode) or stores plain dot products.
// Work items are (slot, row tile); a slot is one expert applied to up to NT
// assignments.  All waits are bounded; on timeout the kernel records an error
// in *status and drains without further waiting.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "expert_common.cuh"
#include "iq3xxs.cuh"
#include "kernels.h"

namespace gp {
namespace {

// Threads per CTA (consumer warps + the producer), which fixes the register
// budget: one token per slot 24 + 1 warps (single matrix, 80 registers) or
// 20 + 1 (gate/up, 96 registers); more tokens 15 + 1 (128 registers).
constexpr int threads_cap(int nt, bool gateup) { return nt == 1 ? (gateup ? 672 : 800) : 512; }

// Instantiated (tokens per slot, passes, rows per warp per pass) variants.
#define GP_VARIANTS                                                                      \
    GP_V(1, 1, 2) GP_V(1, 2, 1) GP_V(1, 2, 2) GP_V(1, 4, 1) GP_V(1, 4, 2) GP_V(1, 8, 1)   \
    GP_V(1, 1, 4) GP_V(1, 2, 4) GP_V(2, 1, 2) GP_V(2, 2, 1) GP_V(2, 2, 2) GP_V(2, 4, 1)   \
    GP_V(2, 4, 2) GP_V(2, 8, 1) GP_V(2, 1, 4) GP_V(4, 1, 2) GP_V(4, 2, 1) GP_V(4, 2, 2)   \
    GP_V(4, 4, 1) GP_V(4, 4, 2) GP_V(4, 8, 1) GP_V(4, 1, 4)

struct SmemLayout {
    uint32_t stage_bytes, stages_off, partial_off, bar_off, total;
};

__host__ __device__ inline SmemLayout smem_layout(int in_dim, int tile_rows, int stages, int nm, int nkw, int nt) {
    SmemLayout L;
    const uint32_t nblk = in_dim / 256;
    L.stage_bytes = nm * tile_rows * 98u * nblk;  // multiple of 16 (tile_rows % 8 == 0)
    L.stages_off = GP_IQ3_TABLE_BYTES;
    L.partial_off = L.stages_off + stages * L.stage_bytes;
    const uint32_t partial_bytes = stages * nm * tile_rows * nkw * nt * 4u;
    L.bar_off = (L.partial_off + partial_bytes + 15u) & ~15u;
    L.total = L.bar_off + 2u * stages * 8u + 16u + 4u * stages + 16u;  // + table barrier, abort flag, counters
    return L;
}



// Work mapping.  A pipeline stage holds R_S = NM * TR rows (gate rows then up
// rows in gate/up mode).  Its R_S x SB sub-blocks (SB = in_dim / 32) are the
// work units; consumer warp w, lane l owns units u = 32w + l + p * 32 * NW for
// passes p < P.  Because 32 * NW is a multiple of SB, every unit of a lane
// has the same sub-block index sb = (32w + l) % SB: the lane loads that
// 32-weight slice of each token's activations once per slot and keeps it in
// registers.  In one pass a warp spans RPW consecutive rows (1 when SB is a
// multiple of 32).  Lane sums are reduced over the warp with one butterfly for
// all P * RPW * NT values, then the rows' per-warp partials are added in warp
// order by the last warp to finish the stage (deterministic).
template <int NT, bool GATEUP, int P, int RPW>
__global__ void __launch_bounds__(threads_cap(NT, GATEUP), 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int NM = GATEUP ? 2 : 1;
    constexpr int MV = P * RPW * NT;               // values reduced per lane per stage
    constexpr int M = MV <= 1 ? 1 : MV <= 2 ? 2 : MV <= 4 ? 4 : MV <= 8 ? 8 : MV <= 16 ? 16 : 32;
    static_assert(MV <= 32, "passes x rows x tokens must fit one butterfly");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NW = a.nwarps, TR = a.tile_rows, S = a.stages;
    const int RS = NM * TR;                        // rows per stage
    const int SB = a.in_dim / 32;                  // sub-blocks per row
    const int rowstep = 32 * NW / SB;              // rows covered by one pass
    const SmemLayout L = smem_layout(a.in_dim, TR, S, NM, NW, NT);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + L.bar_off, empty0 = full0 + 8u * S;
    const uint32_t tbar = full0 + 16u * S;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.bar_off + 16u * S + 8u);
    int* s_done = reinterpret_cast<int*>(smem + L.bar_off + 16u * S + 16u);  // [S] arrival counters

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(empty0 + 8u * s, NW);
            s_done[s] = 0;
        }
        mbar_init(tbar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // decode tables: one bulk copy of the 64 KB image (L2-resident after first use)
    if (tid == 0) {
        mbar_arrive_expect_tx(tbar, GP_IQ3_TABLE_BYTES);
        for (int c = 0; c < 4; ++c) bulk_g2s(sbase + c * 16384u, a.tables + c * 16384, 16384u, tbar);
    }

    pdl_wait();  // slots / activations come from the preceding kernels
    const int nblk = a.in_dim / 256;
    const uint32_t row_bytes = 98u * nblk, group_bytes = 784u * nblk;
    const int ntiles = a.rows / TR;
    const int nitems = *a.nslots * ntiles;
    const int g = gridDim.x, c = blockIdx.x;
    const int it_begin = (int)((int64_t)nitems * c / g);
    int it_end = (int)((int64_t)nitems * (c + 1) / g);
    // the table loads fold the dynamic shared memory base into an immediate:
    // if the runtime ever places it elsewhere, report it and do no work
    if (!gp_tables_at_base(smem)) {
        it_end = it_begin;
        if (tid == 0) atomicOr(a.status, GP_DEV_BAD_SHAPE);
    }

    if (warp == NW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int issued = 0, slot = it_begin / max(ntiles, 1), tile = it_begin - slot * ntiles, s = 0;
            uint32_t ph = 1;
            // the expert of the current slot is read once per slot, not per copy
            int expert = it_begin < it_end ? a.slots[slot].expert : 0;
            for (int it = it_begin; it < it_end; ++it, ++issued) {
                if (*s_abort) break;
                if (!mbar_wait(empty0 + 8u * s, ph)) {
                    *s_abort = 1;
                    atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
                    break;
                }
                const int64_t off = expert * a.expert_stride + (int64_t)tile * TR * row_bytes;
                const uint32_t dst = sbase + L.stages_off + s * L.stage_bytes;
                const uint32_t mbytes = TR * row_bytes;
                mbar_arrive_expect_tx(full0 + 8u * s, NM * mbytes);
                bulk_g2s(dst, a.w0 + off, mbytes, full0 + 8u * s);
                if (GATEUP) bulk_g2s(dst + mbytes, a.w1 + off, mbytes, full0 + 8u * s);
                if (++tile == ntiles) {
                    tile = 0;
                    ++slot;
                    if (it + 1 < it_end) expert = a.slots[slot].expert;
                }
                if (++s == S) { s = 0; ph ^= 1u; }
            }
            // never leave the CTA with copies in flight
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                mbar_wait(full0 + 8u * (i % S), (uint32_t)(i / S) & 1u);
            mbar_wait(tbar, 0);
        }
        return;
    }

    // ---------------- consumers ----------------
    const uint32_t lane4 = lane * 4u;
    const int u0 = warp * 32 + lane;
    const int sb = u0 % SB;                        // this lane's sub-block (fixed)
    const int row0 = u0 / SB;                      // its row in pass 0
    const int wrow0 = (warp * 32) / SB;            // the warp's first row in pass 0
    const int wspan = (warp * 32 + 31) / SB - wrow0 + 1;
    const int jrow = row0 - wrow0;                 // 0 .. RPW-1
    const int b = sb >> 3, ib = sb & 7;
    // per-pass byte offsets (inside a stage) of this lane's qs, aux and d
    uint32_t q_off[P], a_off[P], d_off[P];
#pragma unroll
    for (int p = 0; p < P; ++p) {
        const int row = row0 + p * rowstep;
        const uint32_t gb = (row >> 3) * group_bytes;
        const uint32_t ri = row & 7;
        q_off[p] = sbase + L.stages_off + gb + ri * 64u * nblk + 64u * b + 8u * ib;
        a_off[p] = sbase + L.stages_off + gb + 512u * nblk + ri * 32u * nblk + 32u * b + 4u * ib;
        d_off[p] = sbase + L.stages_off + gb + 768u * nblk + ri * 2u * nblk + 2u * b;
    }
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    const uint8_t* tbl = smem;
    constexpr int kShift = 5 - ilog2(M);           // lanes holding the same reduced value
    const int my_idx = lane >> kShift;             // value index this lane ends up with

    if (!mbar_wait(tbar, 0) && lane == 0) {
        *s_abort = 1;
        atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
    }

    uint32_t xq[NT][16];
    float sx4[NT];  // activation scale / 4
    int64_t xrow_cur[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) xrow_cur[t] = -2;  // nothing loaded yet
    int cur_slot = -1;
    SlotDesc sd{0, 0, 0, 0};
    int slot = it_begin / max(ntiles, 1), tile = it_begin - slot * ntiles, s = 0;
    uint32_t ph = 0, soff = 0;
    for (int it = it_begin; it < it_end; ++it) {
        if (slot != cur_slot) {
            cur_slot = slot;
            sd = a.slots[slot];
            // activation rows of this slot; reload only when they differ from the
            // previous slot's (at batch 1 every slot of the gate/up pass reads token 0)
            int64_t rows_t[NT];
            bool same = true;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int asg = sd.begin + t;
                rows_t[t] = t < sd.ntok ? (a.perm_tok ? a.perm_tok[asg] : asg) : -1;
                same = same && rows_t[t] == xrow_cur[t];
            }
            if (!same) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float v[32];
                    if (rows_t[t] >= 0) {
                        load_x_unit<32>(a.x, a.x_bf16, rows_t[t], a.in_dim, 32 * sb, v);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = 0.f;
                    }
                    sx4[t] = 0.25f * quant_i16<32>(v, xq[t]);
                    xrow_cur[t] = rows_t[t];
                }
            }
        }
        if (!*s_abort && !mbar_wait(full0 + 8u * s, ph)) {
            *s_abort = 1;
            atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
        }
        float acc[M];
#pragma unroll
        for (int i = 0; i < M; ++i) acc[i] = 0.f;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const uint32_t aux = lds32(a_off[p] + soff);
            const float d = __half2float(__ushort_as_half((unsigned short)lds16(d_off[p] + soff)));
            const uint2 q = lds64(q_off[p] + soff);
            uint32_t sw[8];
            iq3_decode_sub32(tbl, q.x, q.y, aux, lane4, sw);
            const int odd = iq3_oddscale(aux);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                // exact integer dot times the odd sub-scale, then d * sx / 4 in fp32
                const float v = (float)(iq3_idot<8>(sw, xq[t]) * odd) * (d * sx4[t]);
                if (RPW == 1) {
                    acc[p * NT + t] = v;
                } else {
#pragma unroll
                    for (int j = 0; j < RPW; ++j)
                        if (j == jrow) acc[(p * RPW + j) * NT + t] = v;
                }
            }
        }
        const float red = warp_reduce_many<M>(acc, lane);
        float* pbuf = partial + (size_t)s * RS * NW * NT;
        if (my_idx < MV && (lane & ((1 << kShift) - 1)) == 0) {
            const int t = my_idx % NT, pj = my_idx / NT;
            const int p = pj / RPW, j = pj % RPW;
            if (j < wspan) pbuf[((wrow0 + j + p * rowstep) * NW + warp) * NT + t] = red;
        }
        // last warp to finish this stage adds the per-warp partials (warp order) and stores
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&s_done[s], 1) == NW - 1;
            if (last) s_done[s] = 0;
            __threadfence_block();
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            for (int e = lane; e < TR * NT; e += 32) {
                const int row = e / NT, t = e % NT;
                if (t >= sd.ntok) continue;
                // warps whose units touch stage row r (same set for every pass)
                const int r0 = row % rowstep;
                const int wlo = (r0 * SB) / 32, whi = ((r0 + 1) * SB - 1) / 32;
                float gsum = 0.f;
                for (int ww = wlo; ww <= whi; ++ww) gsum += pbuf[(row * NW + ww) * NT + t];
                float outv = gsum;
                if (GATEUP) {
                    const int ur = TR + row, ur0 = ur % rowstep;
                    const int ulo = (ur0 * SB) / 32, uhi = ((ur0 + 1) * SB - 1) / 32;
                    float usum = 0.f;
                    for (int ww = ulo; ww <= uhi; ++ww) usum += pbuf[(ur * NW + ww) * NT + t];
                    outv = silu_clamped(gsum, usum, a.limit);
                }
                a.out[(int64_t)(sd.begin + t) * a.rows + (int64_t)tile * TR + row] = outv;
            }
            __syncwarp();
        }
        if (lane == 0) mbar_arrive(empty0 + 8u * s);
        if (++tile == ntiles) { tile = 0; ++slot; }
        if (++s == S) { s = 0; ph ^= 1u; }
        soff = s * L.stage_bytes;
    }
    pdl_launch_dependents();
}

template <int NT, bool GATEUP, int P, int RPW>
cudaError_t launch_t(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
    const int NM = GATEUP ? 2 : 1;
    const SmemLayout L = smem_layout(a.in_dim, a.tile_rows, a.stages, NM, a.nwarps, NT);
    const int nthreads = 32 * (a.nwarps + 1);
    if (nthreads > threads_cap(NT, GATEUP) || L.total > 227u * 1024u) return cudaErrorInvalidValue;
    auto kern = gemv_kernel<NT, GATEUP, P, RPW>;
    static std::atomic<unsigned long long> configured{0};  // per device, per instantiation
    cudaError_t e = raise_smem_limit(kern, 227 * 1024, configured);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(nthreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

size_t gemv_smem_bytes(const GemvArgs& a, int nt, bool gateup) {
    return smem_layout(a.in_dim, a.tile_rows, a.stages, gateup ? 2 : 1, a.nwarps, nt).total;
}

int gemv_max_warps(int nt, bool gateup) { return threads_cap(nt, gateup) / 32 - 1; }

bool gemv_variant_exists(int nt, bool gateup, int p, int rpw) {
    (void)gateup;
#define GP_V(N, PP, R) if (nt == N && p == PP && rpw == R) return true;
    GP_VARIANTS
#undef GP_V
    return false;
}

cudaError_t launch_gemv(const GemvArgs& a, int nt, bool gateup, int p, int rpw, int grid, cudaStream_t st,
                        bool pdl) {
#define GP_V(N, PP, R)                                                                         \
    if (nt == N && p == PP && rpw == R)                                                        \
        return gateup ? launch_t<N, true, PP, R>(a, grid, st, pdl) : launch_t<N, false, PP, R>(a, grid, st, pdl);
    GP_VARIANTS
#undef GP_V
    return cudaErrorInvalidValue;
}

}  // namespace gp
