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

#include "iq3xxs.cuh"
#include "kernels.h"

namespace gp {
namespace {

constexpr int kMaxThreads = 512;  // <= 15 consumer warps + 1 producer; caps registers at 128

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
    L.total = L.bar_off + 2u * stages * 8u + 32u;  // + table barrier + abort flag
    return L;
}

template <int UNIT>
GP_DEVINL void load_x_unit(const void* x, int x_bf16, int64_t row, int in_dim, int kofs, float (&v)[UNIT]) {
    if (x_bf16) {
        const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(x) + row * in_dim + kofs;
#pragma unroll
        for (int i = 0; i < UNIT; i += 8) {
            const uint4 r = *reinterpret_cast<const uint4*>(p + i);
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[i + 2 * j] = __uint_as_float(w[j] << 16);
                v[i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
            }
        }
    } else {
        const float* p = static_cast<const float*>(x) + row * in_dim + kofs;
#pragma unroll
        for (int i = 0; i < UNIT; i += 4) {
            const float4 r = *reinterpret_cast<const float4*>(p + i);
            v[i] = r.x;
            v[i + 1] = r.y;
            v[i + 2] = r.z;
            v[i + 3] = r.w;
        }
    }
}

GP_DEVINL float silu_clamped(float g, float u, float lim) {
    // model.cpp:735-739: silu(min(g, lim)) * clamp(u, -lim, lim)
    const float gi = fminf(g, lim);
    const float ui = fminf(fmaxf(u, -lim), lim);
    return gi / (1.0f + expf(-gi)) * ui;
}

template <int UNIT, int NT, bool GATEUP>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int NM = GATEUP ? 2 : 1;
    constexpr int XW = UNIT / 2;  // int16-pair words per token per lane
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nkw = a.nkw, rpm = a.rpm, TR = a.tile_rows, S = a.stages;
    const int nconsumer = NM * rpm * nkw;
    const SmemLayout L = smem_layout(a.in_dim, TR, S, NM, nkw, NT);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + L.bar_off, empty0 = full0 + 8u * S;
    const uint32_t tbar = full0 + 16u * S;
    volatile uint32_t* s_abort = reinterpret_cast<volatile uint32_t*>(smem + L.bar_off + 16u * S + 8u);

    // decode tables: one bulk copy of the 64 KB image (L2-resident after first use)
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(empty0 + 8u * s, nconsumer);
        }
        mbar_init(tbar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(tbar, GP_IQ3_TABLE_BYTES);
        for (int c = 0; c < 4; ++c)
            bulk_g2s(sbase + c * 16384u, a.tables + c * 16384, 16384u, tbar);
    }
    const bool tables_ok = mbar_wait(tbar, 0);
    if (!tables_ok && tid == 0) { *s_abort = 1; atomicOr(a.status, GP_DEV_TIMEOUT_FULL); }
    __syncthreads();

    pdl_wait();  // slots / activations come from the preceding kernels
    const int nblk = a.in_dim / 256;
    const uint32_t row_bytes = 98u * nblk, group_bytes = 784u * nblk;
    const int ntiles = a.rows / TR;
    const int nitems = *a.nslots * ntiles;
    const int g = gridDim.x, c = blockIdx.x;
    const int it_begin = (int)((int64_t)nitems * c / g), it_end = (int)((int64_t)nitems * (c + 1) / g);

    if (warp == nconsumer) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int it = it_begin; it < it_end; ++it, ++issued) {
                if (*s_abort) break;
                const int s = issued % S;
                const uint32_t round = issued / S;
                if (!mbar_wait(empty0 + 8u * s, (round & 1u) ^ 1u)) {
                    *s_abort = 1;
                    atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
                    break;
                }
                const SlotDesc sd = a.slots[it / ntiles];
                const int tile = it % ntiles;
                const int64_t off = sd.expert * a.expert_stride + (int64_t)tile * TR * row_bytes;
                const uint32_t dst = sbase + L.stages_off + s * L.stage_bytes;
                const uint32_t mbytes = TR * row_bytes;
                mbar_arrive_expect_tx(full0 + 8u * s, NM * mbytes);
                bulk_g2s(dst, a.w0 + off, mbytes, full0 + 8u * s);
                if (GATEUP) bulk_g2s(dst + mbytes, a.w1 + off, mbytes, full0 + 8u * s);
            }
            // never leave the CTA with copies in flight
            for (int i = (issued > S ? issued - S : 0); i < issued; ++i) {
                const int s = i % S;
                mbar_wait(full0 + 8u * s, (uint32_t)(i / S) & 1u);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int m = warp / (rpm * nkw);            // 0: gate (or single), 1: up
    const int rg = (warp / nkw) % rpm;
    const int k = warp % nkw;
    const int RW = TR / rpm;                     // rows per warp per stage
    const uint32_t lane4 = lane * 4u;
    // this lane's position inside a row: block b, sub-block ib, half h
    const int unit = k * 32 + lane;              // lane unit index along K
    const int kofs = unit * UNIT;                // first weight
    const int b = kofs / 256;
    const int ib = (kofs / 32) & 7;
    const int h = (UNIT == 16) ? (unit & 1) : 0;
    const uint32_t q_lane = 64u * b + 8u * ib + 4u * h;
    const uint32_t a_lane = 512u * nblk + 32u * b + 4u * ib;
    const uint32_t d_lane = 768u * nblk + 2u * b;
    float* partial = reinterpret_cast<float*>(smem + L.partial_off);
    const uint8_t* tbl = smem;

    uint32_t xq[NT][XW];
    float sx[NT];
    int cur_slot = -1;
    SlotDesc sd{0, 0, 0, 0};
    int consumed = 0;
    for (int it = it_begin; it < it_end; ++it, ++consumed) {
        const int slot = it / ntiles, tile = it % ntiles;
        if (slot != cur_slot) {
            cur_slot = slot;
            sd = a.slots[slot];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float v[UNIT];
                if (t < sd.ntok) {
                    const int asg = sd.begin + t;
                    const int64_t row = a.perm_tok ? a.perm_tok[asg] : asg;
                    load_x_unit<UNIT>(a.x, a.x_bf16, row, a.in_dim, kofs, v);
                } else {
#pragma unroll
                    for (int i = 0; i < UNIT; ++i) v[i] = 0.f;
                }
                sx[t] = quant_i16<UNIT>(v, xq[t]);
            }
        }
        const int s = consumed % S;
        const uint32_t ph = (uint32_t)(consumed / S) & 1u;
        if (!*s_abort && !mbar_wait(full0 + 8u * s, ph)) {
            *s_abort = 1;
            atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
        }
        const uint32_t st_base = L.stages_off + s * L.stage_bytes + m * TR * row_bytes;
        float* pbuf = partial + (size_t)s * NM * TR * nkw * NT;
        for (int r = 0; r < RW; ++r) {
            const int row = rg * RW + r;
            const uint32_t gbase = st_base + (row >> 3) * group_bytes;
            const int ri = row & 7;
            const uint32_t aux = lds32(sbase + gbase + a_lane + 32u * nblk * ri);
            const float d = __half2float(__ushort_as_half((unsigned short)lds16(sbase + gbase + d_lane + 2u * nblk * ri)));
            const float ds = iq3_subscale(d, aux);
            float acc[NT];
            if (UNIT == 32) {
                const uint2 q = lds64(sbase + gbase + q_lane + 64u * nblk * ri);
                uint32_t sw[8];
                iq3_decode_sub32(tbl, q.x, q.y, aux, lane4, sw);
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = (float)iq3_idot<8>(sw, xq[t]) * (ds * sx[t]);
            } else {
                const uint32_t q = lds32(sbase + gbase + q_lane + 64u * nblk * ri);
                uint32_t sw[4];
                iq3_decode_sub16(tbl, q, aux >> (14 * h), lane4, sw);
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = (float)iq3_idot<4>(sw, xq[t]) * (ds * sx[t]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[t]);
                if (lane == t) pbuf[((m * TR + row) * nkw + k) * NT + t] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8u * s);
        named_bar_sync(1, nconsumer * 32);
        // epilogue for this stage: deterministic K-slice sum, SwiGLU or plain store
        const int ctid = tid;  // consumers are warps 0..nconsumer-1
        for (int e = ctid; e < TR * NT; e += nconsumer * 32) {
            const int row = e / NT, t = e % NT;
            if (t >= sd.ntok) continue;
            float gsum = 0.f;
            for (int kk = 0; kk < nkw; ++kk) gsum += pbuf[((0 * TR + row) * nkw + kk) * NT + t];
            float outv = gsum;
            if (GATEUP) {
                float usum = 0.f;
                for (int kk = 0; kk < nkw; ++kk) usum += pbuf[((1 * TR + row) * nkw + kk) * NT + t];
                outv = silu_clamped(gsum, usum, a.limit);
            }
            a.out[(int64_t)(sd.begin + t) * a.rows + (int64_t)tile * TR + row] = outv;
        }
    }
}

template <int UNIT, int NT, bool GATEUP>
cudaError_t launch_t(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
    const int NM = GATEUP ? 2 : 1;
    const SmemLayout L = smem_layout(a.in_dim, a.tile_rows, a.stages, NM, a.nkw, NT);
    auto kern = gemv_kernel<UNIT, NT, GATEUP>;
    static int configured = 0;  // opt-in shared memory is raised once per instantiation
    if ((int)L.total > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured = 227 * 1024;
    }
    if (L.total > 227u * 1024u) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * (NM * a.rpm * a.nkw + 1));
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
    return smem_layout(a.in_dim, a.tile_rows, a.stages, gateup ? 2 : 1, a.nkw, nt).total;
}

cudaError_t launch_gemv(const GemvArgs& a, int unit, int nt, bool gateup, int grid, cudaStream_t st, bool pdl) {
#define GP_CASE(U, N)                                                             \
    if (unit == U && nt == N)                                                     \
        return gateup ? launch_t<U, N, true>(a, grid, st, pdl) : launch_t<U, N, false>(a, grid, st, pdl);
    // register budget: UNIT/2 * NT words of activations per lane (<= 64)
    GP_CASE(32, 1) GP_CASE(32, 2) GP_CASE(32, 4)
    GP_CASE(16, 1) GP_CASE(16, 2) GP_CASE(16, 4) GP_CASE(16, 8)
#undef GP_CASE
    return cudaErrorInvalidValue;
}

}  // namespace gp
