// Router logits for large batches on the 5th-generation tensor cores.
//
//   logits[t][e] = sum_k x[t][k] * R[e][k]        x bf16 [n][H], R fp32 [E][H]
//
// (the reference's router matvec, model_batch.cpp router step; fp32 weights.)
// R is split once, when the layer is loaded, into three bf16 parts with
// R = hi + lo + lo2 exactly (8 + 8 + 8 significant bits of the fp32 value),
// so every product x * part is exact in fp32.  The tensor core accumulates
// the three dot products in fp32 (TMEM); the epilogue adds them smallest
// first, (lo2 + lo) + hi.  The result differs from an fp32 dot product only
// in the order and rounding of the accumulation.
//
// Split rows are laid out [hi: E rows][lo: E rows][lo2: E rows][zero rows]
// up to 2*NB rows, NB = 16-aligned half; one CTA computes 128 tokens x 2*NB
// columns over one K range (two M=128, N=NB MMAs per K step of 16).  K is
// split over gridDim.y ranges whose partial logits the caller adds in order.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocation and
// MMA issue, warps 2-5 epilogue (one TMEM lane quadrant = 32 tokens each).
// No cluster, no multicast.  Every wait is bounded; a timeout sets a status bit.
#include <cuda_bf16.h>

#include "kernels.h"
#include "tc_common.cuh"

namespace gp {
namespace {

constexpr int RT_M = 128;   // tokens per CTA (MMA M = TMEM lanes)
constexpr int RT_K = 64;    // K per stage (one 128-byte swizzled bf16 row)
constexpr int RT_ST = 2;    // stages
constexpr int RT_THREADS = 192;
constexpr uint32_t RT_XBYTES = RT_M * 128;

struct RtMaps {
    CUtensorMap x;  // bf16 [n][H], box {64, 128}, 128-byte swizzle
    CUtensorMap w;  // bf16 [2*NB][H], box {64, NB}, 128-byte swizzle
};

struct RtArgs {
    int n, E, H, nb;
    float* out;           // logits [n][E] (one K range) or partials [gridDim.y][n][E]
    uint32_t* status;
};

__host__ __device__ inline uint32_t rt_stage_bytes(int nb) { return RT_XBYTES + 2u * nb * 128u; }
__host__ __device__ inline uint32_t rt_smem_bytes(int nb) { return RT_ST * rt_stage_bytes(nb) + 256 + 1024; }

__global__ void __launch_bounds__(RT_THREADS, 1) router_tc_kernel(const __grid_constant__ RtMaps maps, const RtArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t base = (raw0 + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t stage = rt_stage_bytes(a.nb);
    const uint32_t bar = base + RT_ST * stage;
    const uint32_t full = bar, empty = bar + 8 * RT_ST, acc_full = empty + 8 * RT_ST, tslot = acc_full + 8;
    const int t0 = blockIdx.x * RT_M;
    const int klen = a.H / (int)gridDim.y, kb = (int)blockIdx.y * klen, nk = klen / RT_K;

    if (tid == 0) {
        for (int s = 0; s < RT_ST; ++s) { mbar_init(full + 8 * s, 1); mbar_init(empty + 8 * s, 1); }
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *reinterpret_cast<volatile uint32_t*>(gbase + (tslot - base));
    pdl_wait();  // x is the previous kernel's output in a layer chain

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            for (int c = 0; c < nk; ++c) {
                const int s = c % RT_ST;
                if (!mbar_wait(empty + 8 * s, ((c / RT_ST) & 1) ^ 1)) { ok = false; break; }
                const uint32_t xs = base + s * stage, ws = xs + RT_XBYTES;
                mbar_arrive_expect_tx(full + 8 * s, stage);
                tma_load_2d(xs, &maps.x, kb + c * RT_K, t0, full + 8 * s);
                tma_load_2d(ws, &maps.w, kb + c * RT_K, 0, full + 8 * s);
                tma_load_2d(ws + a.nb * 128, &maps.w, kb + c * RT_K, a.nb, full + 8 * s);
            }
            if (!ok) atomicOr(a.status, GP_DEV_TIMEOUT_EMPTY);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(RT_M, a.nb, true);
            bool ok = true;
            for (int c = 0; c < nk; ++c) {
                const int s = c % RT_ST;
                if (!mbar_wait(full + 8 * s, (c / RT_ST) & 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t xs = base + s * stage, ws = xs + RT_XBYTES;
#pragma unroll
                for (int kk = 0; kk < RT_K / 16; ++kk) {
                    const uint64_t adesc = umma_desc_sw128(xs + kk * 32);
                    umma_f16(tbase, adesc, umma_desc_sw128(ws + kk * 32), idesc, (c | kk) != 0);
                    umma_f16(tbase + a.nb, adesc, umma_desc_sw128(ws + a.nb * 128 + kk * 32), idesc, (c | kk) != 0);
                }
                umma_commit(empty + 8 * s);
            }
            if (ok) umma_commit(acc_full);
            else atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
        }
    } else {
        const int q = warp & 3, t = t0 + 32 * q + lane;
        if (mbar_wait_sleepy(acc_full, 0)) {
            tc_fence_after();
            const uint32_t lanebase = tbase + ((uint32_t)(32 * q) << 16);
            float* out = a.out + (size_t)blockIdx.y * a.n * a.E + (size_t)t * a.E;
            for (int e0 = 0; e0 < a.E; e0 += 32) {
                uint32_t v[32], u[32];
                tmem_ld32(lanebase + 2 * a.E + e0, v);  // lo2
                tmem_ld32(lanebase + a.E + e0, u);      // lo
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
                tmem_ld32(lanebase + e0, u);  // hi
                if (t < a.n) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 o;
                        o.x = __uint_as_float(u[j]) + __uint_as_float(v[j]);
                        o.y = __uint_as_float(u[j + 1]) + __uint_as_float(v[j + 1]);
                        o.z = __uint_as_float(u[j + 2]) + __uint_as_float(v[j + 2]);
                        o.w = __uint_as_float(u[j + 3]) + __uint_as_float(v[j + 3]);
                        *reinterpret_cast<float4*>(out + e0 + j) = o;
                    }
                }
            }
        } else if (lane == 0) {
            atomicOr(a.status, GP_DEV_TIMEOUT_FULL);
        }
    }
    tc_fence_before();
    __syncthreads();
    pdl_launch_dependents();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// R -> [hi; lo; lo2; 0] bf16 rows: hi = bf16(R), lo = bf16(R - hi), lo2 = R - hi - lo
// (each difference exact in fp32; lo2 has at most 8 significant bits).
__global__ void router_split_kernel(const float* R, int E, int H, int nb, __nv_bfloat16* out) {
    const int64_t total = (int64_t)2 * nb * H;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / H), k = (int)(i % H);
        const int part = row / E, e = row % E;
        float v = 0.f;
        if (part < 3) {
            const float r = R[(int64_t)e * H + k];
            const float hi = __bfloat162float(__float2bfloat16_rn(r));
            const float r1 = r - hi;
            const float lo = __bfloat162float(__float2bfloat16_rn(r1));
            v = part == 0 ? hi : part == 1 ? lo : r1 - lo;
        }
        out[i] = __float2bfloat16_rn(v);
    }
}

}  // namespace

int router_tc_nb(int E, int H) {
    if (E % 32 || E > 160 || H % RT_K) return 0;
    const int nb = ((3 * E + 1) / 2 + 15) & ~15;
    return (nb <= 256 && rt_smem_bytes(nb) <= 227u * 1024u) ? nb : 0;
}

int router_tc_splits(int n, int H) {
    const int tiles = (n + RT_M - 1) / RT_M;
    int S = 1;  // about one CTA per SM of 148, each K range a whole number of stages
    while (S < 8 && tiles * S * 2 <= 148 + 148 / 4 && H % (2 * S * RT_K) == 0) S *= 2;
    return S;
}

cudaError_t launch_router_split(const float* R, int E, int H, int nb, uint16_t* out, cudaStream_t st) {
    router_split_kernel<<<148 * 4, 256, 0, st>>>(R, E, H, nb, reinterpret_cast<__nv_bfloat16*>(out));
    return cudaGetLastError();
}

cudaError_t launch_router_tc(const RouterArgs& ra, int S, float* out, cudaStream_t st, bool pdl) {
    const int nb = ra.wsplit_nb;
    if (!ra.x_bf16 || !ra.wsplit || nb <= 0 || ra.H % (S * RT_K)) return cudaErrorInvalidValue;
    RtMaps m{};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)ra.H, (cuuint64_t)ra.n};
        const cuuint64_t str[1] = {(cuuint64_t)ra.H * 2};
        const cuuint32_t box[2] = {RT_K, RT_M};
        if (!encode(&m.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ra.x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)ra.H, (cuuint64_t)(2 * nb)};
        const cuuint64_t str[1] = {(cuuint64_t)ra.H * 2};
        const cuuint32_t box[2] = {RT_K, (cuuint32_t)nb};
        if (!encode(&m.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ra.wsplit, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
    }
    RtArgs a{ra.n, ra.E, ra.H, nb, out, ra.status};
    const uint32_t smem = rt_smem_bytes(nb);
    cudaError_t e = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((ra.n + RT_M - 1) / RT_M, S);
    cfg.blockDim = dim3(RT_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, router_tc_kernel, m, a);
}

}  // namespace gp
