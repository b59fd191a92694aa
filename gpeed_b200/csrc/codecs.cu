// Dequantisation of every GGUF codec the reference decodes (quant.cpp:
// 130-573): F16, BF16, Q8_0, Q2_K, Q3_K, Q6_K, IQ3_XXS, IQ2_S, IQ3_S, IQ4_XS
// (F32 is a copy).  Bit-exact with the reference:
// every value is formed with the same fp32 products in the same order
// (__fmul_rn / __fsub_rn keep the compiler from contracting them), and fp16
// scales widen with the reference's integer conversion (quant.cpp:130-154),
// NaN payloads included.
//
// Layout of the work: a warp decodes 256 values per step (one K-/IQ-quant
// block, or eight Q8_0 blocks): its lanes first copy the block bytes to shared
// memory with coalesced 2-byte loads (GGUF blocks are only 2-byte aligned;
// byte loads for a source that starts at an odd address), then
// each lane forms 8 consecutive values from shared memory and writes them as
// two float4 stores, so a warp writes 1 KiB contiguously.  Codebooks (IQ2_S
// 8 KiB, IQ3_S 2 KiB, IQ4 16 B) are staged in shared memory per CTA.  The
// kernels are bound by the fp32 writes (4 bytes per value against 0.26-0.82
// bytes read).
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "iq3xxs_grid.h"
#include "quant_grids.h"

namespace gp {
namespace {

__device__ const uint64_t g_iq2s_grid[1024] = {GPEED_IQ2S_GRID_VALUES};
__device__ const uint32_t g_iq3s_grid[512] = {GPEED_IQ3S_GRID_VALUES};
__device__ const uint32_t g_iq3xxs_grid[256] = {GPEED_IQ3XXS_GRID_VALUES};
__device__ __align__(16) const int8_t g_iq4nl[16] = {GPEED_IQ4NL_VALUES};

constexpr int kCdWarps = 8;

// IEEE half -> float exactly as quant.cpp:130-154 (subnormals normalised,
// Inf/NaN keep their payload bits)
__device__ __forceinline__ float f16_ref(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            const int shift = __clz(man) - 21;  // moves the leading one to bit 10
            bits = sign | ((uint32_t)(113 - shift) << 23) | (((man << shift) & 0x3ffu) << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112) << 23) | (man << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ float ld_f16(const uint8_t* p) { return f16_ref((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

template <int T>
struct Codec;

template <>
struct Codec<8> {  // Q8_0, quant.cpp:165-184: y = d * q
    static constexpr int kBytes = 34, kVals = 32;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t*, float* y) {
        const float d = ld_f16(b);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(d, (float)(int8_t)b[2 + 8 * s + j]);
    }
};

template <>
struct Codec<14> {  // Q6_K, quant.cpp:212-307: y = (d * sc) * q
    static constexpr int kBytes = 210, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t*, float* y) {
        const int v0 = 8 * s, h = v0 >> 7, g = (v0 >> 5) & 3, l0 = v0 & 31;
        const uint8_t* ql = b + 64 * h + (g & 1) * 32;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t sc = (int8_t)b[192 + 8 * h + (l0 >> 4) + 2 * g];
        const float ds = __fmul_rn(ld_f16(b + 208), (float)sc);
        const int lshift = (g >> 1) * 4, hshift = 2 * g;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int l = l0 + j;
            const int q = (int)(((ql[l] >> lshift) & 0xF) | (((qh[l] >> hshift) & 3) << 4)) - 32;
            y[j] = __fmul_rn(ds, (float)q);
        }
    }
};

template <>
struct Codec<10> {  // Q2_K, quant.cpp:309-335: y = dl * q - ml (not contracted)
    static constexpr int kBytes = 84, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t*, float* y) {
        const int v0 = 8 * s, h = v0 >> 7, J = (v0 >> 5) & 3, half = (v0 >> 4) & 1, l0 = v0 & 15;
        const uint8_t scv = b[8 * h + 2 * J + half];
        const float dl = __fmul_rn(ld_f16(b + 80), (float)(scv & 0xF));
        const float ml = __fmul_rn(ld_f16(b + 82), (float)(scv >> 4));
        const uint8_t* q = b + 16 + 32 * h + 16 * half;
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fsub_rn(__fmul_rn(dl, (float)((q[l0 + j] >> (2 * J)) & 3)), ml);
    }
};

template <>
struct Codec<11> {  // Q3_K, quant.cpp:337-371
    static constexpr int kBytes = 110, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t*, float* y) {
        const int v0 = 8 * s, h = v0 >> 7, J = (v0 >> 5) & 3, half = (v0 >> 4) & 1;
        const int is = 8 * h + 2 * J + half;  // 6-bit scale is: low nibble from bytes 96..103, high bits from 104..107
        const int k = is & 3, grp = is >> 2;
        const uint8_t lo = b[96 + 4 * (grp & 1) + k] >> (4 * (grp >> 1));
        const uint8_t hi = b[104 + k] >> (2 * grp);
        const int sc = (int)((lo & 0xF) | ((hi & 3) << 4));
        const float dl = __fmul_rn(ld_f16(b + 108), (float)(sc - 32));
        const uint8_t m = (uint8_t)(1u << (4 * h + J));
        const int l0 = 16 * half + (v0 & 15);
        const uint8_t* q = b + 32 + 32 * h;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int l = l0 + j;
            y[j] = __fmul_rn(dl, (float)((int)((q[l] >> (2 * J)) & 3) - ((b[l] & m) ? 0 : 4)));
        }
    }
};

template <>
struct Codec<22> {  // IQ2_S, quant.cpp:373-419: y = dl * (signed grid byte), as its AVX2 branch
    static constexpr int kBytes = 82, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t* tab, float* y) {
        const int ib = s >> 2, l = s & 3;
        const uint8_t sc = b[74 + ib];
        const float d = ld_f16(b);
        const float dl = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(l < 2 ? sc & 0xf : sc >> 4))), 0.25f);
        const uint32_t idx = (uint32_t)b[2 + 4 * ib + l] | (((uint32_t)b[66 + ib] << (8 - 2 * l)) & 0x300u);
        const uint64_t g = reinterpret_cast<const uint64_t*>(tab)[idx];
        const uint8_t sg = b[34 + 4 * ib + l];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            y[j] = __fmul_rn(dl, (float)(((sg >> j) & 1) ? -(int)(uint8_t)(g >> (8 * j)) : (int)(uint8_t)(g >> (8 * j))));
    }
};

template <>
struct Codec<21> {  // IQ3_S, quant.cpp:421-483
    static constexpr int kBytes = 110, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t* tab, float* y) {
        const int k = s >> 3, pass = (s >> 2) & 1, l = s & 3;
        const uint8_t sc = b[106 + k];
        const float db = __fmul_rn(ld_f16(b), __fadd_rn(1.0f, __fmul_rn(2.0f, (float)(pass ? sc >> 4 : sc & 0xf))));
        const uint8_t* qs = b + 2 + 16 * k + 8 * pass;
        const uint32_t qh = b[66 + 2 * k + pass];
        const uint32_t i1 = (uint32_t)qs[2 * l] | ((qh << (8 - 2 * l)) & 256u);
        const uint32_t i2 = (uint32_t)qs[2 * l + 1] | ((qh << (7 - 2 * l)) & 256u);
        const uint32_t* grid = reinterpret_cast<const uint32_t*>(tab);
        const uint32_t g1 = grid[i1], g2 = grid[i2];
        const uint8_t sg = b[74 + 8 * k + 4 * pass + l];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int a1 = (uint8_t)(g1 >> (8 * j)), a2 = (uint8_t)(g2 >> (8 * j));
            y[j] = __fmul_rn(db, (float)(((sg >> j) & 1) ? -a1 : a1));
            y[j + 4] = __fmul_rn(db, (float)(((sg >> (j + 4)) & 1) ? -a2 : a2));
        }
    }
};

template <>
struct Codec<18> {  // IQ3_XXS, quant.cpp:186-210: y = (db * grid) * sign, db = d * (0.5 + aux>>28) * 0.5
    static constexpr int kBytes = 98, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t* tab, float* y) {
        const int ib = s >> 2, l = s & 3;
        const uint8_t* sa = b + 66 + 4 * ib;
        const uint32_t aux = (uint32_t)sa[0] | ((uint32_t)sa[1] << 8) | ((uint32_t)sa[2] << 16) | ((uint32_t)sa[3] << 24);
        const float db = __fmul_rn(__fmul_rn(ld_f16(b), __fadd_rn(0.5f, (float)(aux >> 28))), 0.5f);
        const uint32_t k7 = (aux >> (7 * l)) & 127u;
        const uint32_t sg = k7 | ((uint32_t)(__popc(k7) & 1) << 7);  // the sign table entry: k | parity(k) << 7
        const uint32_t* grid = reinterpret_cast<const uint32_t*>(tab);
        const uint32_t g1 = grid[b[2 + 8 * ib + 2 * l]], g2 = grid[b[2 + 8 * ib + 2 * l + 1]];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float w1 = __fmul_rn(db, (float)((g1 >> (8 * j)) & 0xFF));
            const float w2 = __fmul_rn(db, (float)((g2 >> (8 * j)) & 0xFF));
            y[j] = ((sg >> j) & 1) ? -w1 : w1;
            y[j + 4] = ((sg >> (j + 4)) & 1) ? -w2 : w2;
        }
    }
};

template <>
struct Codec<23> {  // IQ4_XS, quant.cpp:485-503: y = d * (ls - 32) * v[nibble]
    static constexpr int kBytes = 136, kVals = 256;
    __device__ static void unit(const uint8_t* b, int s, const uint8_t* tab, float* y) {
        const int ib = s >> 2, q = s & 3;
        const uint32_t sh = (uint32_t)b[2] | ((uint32_t)b[3] << 8);
        const int ls = ((b[4 + (ib >> 1)] >> (4 * (ib & 1))) & 0xf) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = __fmul_rn(ld_f16(b), (float)(ls - 32));
        const uint8_t* qs = b + 8 + 16 * ib + 8 * (q & 1);
        const int8_t* v = reinterpret_cast<const int8_t*>(tab);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(dl, (float)v[(q < 2 ? qs[j] : qs[j] >> 4) & 0xf]);
    }
};

template <int T>
__device__ __forceinline__ int table_bytes() {
    return T == 22 ? 8192 : T == 21 ? 2048 : T == 18 ? 1024 : T == 23 ? 16 : 0;
}

template <int T>
__global__ void __launch_bounds__(32 * kCdWarps) codec_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                                             int64_t nblocks, int src16) {
    using C = Codec<T>;
    constexpr int kPer = 256 / C::kVals;           // blocks per warp step
    constexpr int kStage = (kPer * C::kBytes + 15) & ~15;
    __shared__ __align__(16) uint8_t s_tab[T == 22 ? 8192 : T == 21 ? 2048 : T == 18 ? 1024 : 16];
    __shared__ __align__(16) uint8_t s_blk[kCdWarps][kStage];
    if (table_bytes<T>()) {
        const uint8_t* t = T == 22 ? reinterpret_cast<const uint8_t*>(g_iq2s_grid)
                         : T == 21 ? reinterpret_cast<const uint8_t*>(g_iq3s_grid)
                         : T == 18 ? reinterpret_cast<const uint8_t*>(g_iq3xxs_grid)
                                   : reinterpret_cast<const uint8_t*>(g_iq4nl);
        for (int i = threadIdx.x; i < table_bytes<T>() / 4; i += blockDim.x)
            reinterpret_cast<uint32_t*>(s_tab)[i] = reinterpret_cast<const uint32_t*>(t)[i];
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t steps = (nblocks + kPer - 1) / kPer;
    for (int64_t st = (int64_t)blockIdx.x * kCdWarps + warp; st < steps; st += (int64_t)gridDim.x * kCdWarps) {
        const int64_t b0 = st * kPer;
        const int nb = (int)(nblocks - b0 < kPer ? nblocks - b0 : kPer);
        const uint8_t* g = src + b0 * C::kBytes;
        __syncwarp();
        // every block size is even: 2-byte pieces when the tensor starts 2-byte aligned.  (Measured per
        // codec on B200: faster for Q8_0, Q6_K, IQ3_XXS, IQ3_S, IQ2_S; slower for Q2_K and Q3_K, which
        // keep byte pieces.)
        constexpr bool kPieces16 = T != 10 && T != 11;
        if (kPieces16 && src16) {
            const uint16_t* g2 = reinterpret_cast<const uint16_t*>(g);
            uint16_t* d2 = reinterpret_cast<uint16_t*>(s_blk[warp]);
            for (int i = lane; i < nb * C::kBytes / 2; i += 32) d2[i] = g2[i];
        } else {
            for (int i = lane; i < nb * C::kBytes; i += 32) s_blk[warp][i] = g[i];
        }
        __syncwarp();
        const int unit = lane, blk = unit / (C::kVals / 8), s = unit % (C::kVals / 8);
        if (blk < nb) {
            float y[8];
            C::unit(s_blk[warp] + blk * C::kBytes, s, s_tab, y);
            float4* o = reinterpret_cast<float4*>(dst + (b0 * C::kVals + (int64_t)unit * 8));
            o[0] = make_float4(y[0], y[1], y[2], y[3]);
            o[1] = make_float4(y[4], y[5], y[6], y[7]);
        }
    }
}

// 8 values per thread per step (one 16-byte load, two float4 stores) when the
// source is 16-byte aligned; the remainder (and unaligned sources) one by one
__global__ void f16_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, int64_t n, int bf16) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x, tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const int64_t n8 = n / 8;
        for (int64_t i = tid; i < n8; i += stride) {
            const uint4 v = reinterpret_cast<const uint4*>(src)[i];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            float y[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t lo = w[q] & 0xffffu, hi = w[q] >> 16;
                y[2 * q] = bf16 ? __uint_as_float(lo << 16) : f16_ref(lo);
                y[2 * q + 1] = bf16 ? __uint_as_float(hi << 16) : f16_ref(hi);
            }
            float4* o = reinterpret_cast<float4*>(dst + 8 * i);
            o[0] = make_float4(y[0], y[1], y[2], y[3]);
            o[1] = make_float4(y[4], y[5], y[6], y[7]);
        }
        done = n8 * 8;
    }
    for (int64_t i = done + tid; i < n; i += stride) {
        const uint32_t h = src[i];
        dst[i] = bf16 ? __uint_as_float(h << 16) : f16_ref(h);
    }
}

template <int T>
cudaError_t launch_codec(const uint8_t* src, float* dst, int64_t n, cudaStream_t st) {
    constexpr int kPer = 256 / Codec<T>::kVals;
    const int64_t nblocks = n / Codec<T>::kVals;
    const int64_t steps = (nblocks + kPer - 1) / kPer;
    int64_t grid = (steps + kCdWarps - 1) / kCdWarps;
    if (grid > 148 * 8) grid = 148 * 8;
    if (grid < 1) grid = 1;
    codec_kernel<T><<<(int)grid, 32 * kCdWarps, 0, st>>>(src, dst, nblocks,
                                                         (reinterpret_cast<uintptr_t>(src) & 1) == 0);
    return cudaGetLastError();
}

}  // namespace

int codec_block_values(int dtype) {
    switch (dtype) {
        case 0: case 1: case 30: return 1;
        case 8: return 32;
        case 10: case 11: case 14: case 18: case 21: case 22: case 23: return 256;
        default: return 0;
    }
}

cudaError_t launch_codec_dequantize(int dtype, const void* src, float* dst, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    switch (dtype) {
        case 0: return cudaMemcpyAsync(dst, src, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
        case 1:
        case 30: {
            int64_t grid = (n / 8 + 255) / 256;
            if (grid > 148 * 16) grid = 148 * 16;
            if (grid < 1) grid = 1;
            f16_kernel<<<(int)grid, 256, 0, st>>>(static_cast<const uint16_t*>(src), dst, n, dtype == 30);
            return cudaGetLastError();
        }
        case 8: return launch_codec<8>(s, dst, n, st);
        case 10: return launch_codec<10>(s, dst, n, st);
        case 11: return launch_codec<11>(s, dst, n, st);
        case 14: return launch_codec<14>(s, dst, n, st);
        case 18: return launch_codec<18>(s, dst, n, st);
        case 21: return launch_codec<21>(s, dst, n, st);
        case 22: return launch_codec<22>(s, dst, n, st);
        case 23: return launch_codec<23>(s, dst, n, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gp
