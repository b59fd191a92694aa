// mHC residual mixing and RMSNorm on either side of the MoE layer (the
// reference's Model::hc_forward, cpp/core/src/model.cpp:205-263, with the ffn
// norm of layer_forward, model.cpp:292-296, and the stream update after the
// MLP, model.cpp:309-318; batched as run_chunk passes 4 and 6,
// model_batch.cpp:374-410).  Per token, N = hc_mult residual streams of H:
//
//   pre:  r    = rsqrt(mean(streams^2) + rms_eps)              (over N*H)
//         w    = fn . (streams * r)                            (W = (2+N)N dots)
//         pre  = sigmoid(w[n] s0 + b[n]) + hc_eps
//         post = 2 sigmoid(w[N+n] s1 + b[N+n])
//         comb = softmax_j(w[2N+iN+j] s2 + b[...]) + hc_eps, then Sinkhorn
//                (columns, then iters-1 x (rows, columns); sums + hc_eps)
//         mix  = sum_n pre[n] streams[n];  x = mix * rsqrt(mean(mix^2) + eps) * norm_w
//   post: streams'[n] = post[n] mlp + sum_m comb[m][n] streams[m]
//
// Kernels: the sum of squares and the W dot products of fn with the raw
// streams per K slice (mhc_dot_vec_kernel, a CTA per token and slice, below 32
// tokens; mhc_dot_kernel, a small SGEMM over 64-token tiles that reads fn once
// per tile, above); mhc_coef_kernel (a warp per token) adds the slices,
// scales by the RMS factor (r * (fn . x) = fn . (r x)) and forms pre, post
// and comb; mhc_mix_kernel (a CTA per token) mixes the streams into shared
// memory and normalises; mhc_post_kernel updates the streams element-wise
// (one thread per (token, 4 elements) writes all N streams, so it may run in
// place).  fp32 throughout; expf / sqrtf are CUDA's.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace gp {
namespace {

constexpr int kMhcMaxW = 24;          // (2 + N) N for N <= 4
constexpr int kMhcThreads = 256;

// Dot products as a small SGEMM: a CTA of 64 threads takes a tile of 128
// tokens x all W outputs over one K slice.  Per 64-element step it copies the
// tile's 128 row pieces (256 contiguous bytes each; a warp copies one piece
// per two loads) and the W fn pieces to shared memory, natural layout.  Each
// thread accumulates 8 tokens (tm + 16 i) x W/4 outputs, reading 4 elements
// along K at a time, so a shared-memory read feeds 8 (x) or 12 (fn)
// multiply-adds per element.  The sum of squares comes from the copies,
// reduced over the 16 lanes that copied a row.
constexpr int kDotM = 128, kDotK = 64, kDotThreads = 64;

template <int N>
__global__ void __launch_bounds__(kDotThreads) mhc_dot_kernel(const float* __restrict__ streams,
                                                             const float* __restrict__ fn, int n, int HN, int klen,
                                                             float* __restrict__ partial) {
    constexpr int W = (2 + N) * N, WT = (W + 3) / 4, FR = 4 * WT;  // FR fn rows staged (zero past W)
    constexpr int XQ = kDotM * kDotK / 4 / kDotThreads;             // x float4 copied per thread (32)
    constexpr int FQ = (FR * kDotK / 4 + kDotThreads - 1) / kDotThreads;
    __shared__ __align__(16) float xs[kDotM][kDotK + 4];
    __shared__ __align__(16) float fs[FR][kDotK + 4];
    const int tid = threadIdx.x, tm = tid & 15, tn = tid >> 4;
    const int t0 = blockIdx.y * kDotM, slice = blockIdx.x;
    const int kb = slice * klen, ke = min(HN, kb + klen);
    // copy mapping: float4 i = tid + 64 q -> row i >> 4, column 4 * (i & 15)
    const int crow = tid >> 4, ccol = 4 * (tid & 15);
    float acc[8][WT], sq[XQ];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < WT; ++j) acc[i][j] = 0.f;
#pragma unroll
    for (int q = 0; q < XQ; ++q) sq[q] = 0.f;
    for (int k0 = kb; k0 < ke; k0 += kDotK) {
        const int col = k0 + ccol;
        const bool kin = col < ke;
#pragma unroll
        for (int q = 0; q < XQ; ++q) {
            const int r = crow + 4 * q;
            const float4 v = (kin && t0 + r < n)
                                 ? *reinterpret_cast<const float4*>(streams + (size_t)(t0 + r) * HN + col)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&xs[r][ccol]) = v;
            sq[q] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
#pragma unroll
        for (int q = 0; q < FQ; ++q) {
            const int row = crow + 4 * q;
            if (row < FR)
                *reinterpret_cast<float4*>(&fs[row][ccol]) =
                    (kin && row < W) ? __ldg(reinterpret_cast<const float4*>(fn + (size_t)row * HN + col))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
#pragma unroll 2
        for (int k = 0; k < kDotK; k += 4) {
            float4 f[WT];
#pragma unroll
            for (int j = 0; j < WT; ++j) f[j] = *reinterpret_cast<const float4*>(&fs[tn * WT + j][k]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 xv = *reinterpret_cast<const float4*>(&xs[tm + 16 * i][k]);
#pragma unroll
                for (int j = 0; j < WT; ++j)
                    acc[i][j] += xv.x * f[j].x + xv.y * f[j].y + xv.z * f[j].z + xv.w * f[j].w;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < XQ; ++q) {  // a copied row's 16 pieces are 16 consecutive lanes
        float v = sq[q];
#pragma unroll
        for (int o = 8; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int t = t0 + crow + 4 * q;
        if ((tid & 15) == 0 && t < n) partial[((size_t)t * gridDim.x + slice) * (W + 1)] = v;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int t = t0 + tm + 16 * i;
        if (t >= n) continue;
        float* pp = partial + ((size_t)t * gridDim.x + slice) * (W + 1);
#pragma unroll
        for (int j = 0; j < WT; ++j) {
            const int o = tn * WT + j;
            if (o < W) pp[1 + o] = acc[i][j];
        }
    }
}

// Small batches: a CTA per (token, slice of 1024 elements), a float4 per
// thread, the W + 1 sums reduced across the CTA; all fn loads of a thread are
// independent, so a slice costs about one memory latency.
template <int N>
__global__ void __launch_bounds__(kMhcThreads) mhc_dot_vec_kernel(const float* __restrict__ streams,
                                                                 const float* __restrict__ fn, int HN,
                                                                 float* __restrict__ partial) {
    constexpr int W = (2 + N) * N;
    const int slice = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = slice * 4 * kMhcThreads + 4 * tid;
    float v[W + 1];
#pragma unroll
    for (int j = 0; j <= W; ++j) v[j] = 0.f;
    if (k < HN) {
        const float4 x = *reinterpret_cast<const float4*>(streams + (size_t)t * HN + k);
        float4 f[W];
#pragma unroll
        for (int j = 0; j < W; ++j) f[j] = __ldg(reinterpret_cast<const float4*>(fn + (size_t)j * HN + k));
        v[0] = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
#pragma unroll
        for (int j = 0; j < W; ++j) v[1 + j] = f[j].x * x.x + f[j].y * x.y + f[j].z * x.z + f[j].w * x.w;
    }
    __shared__ float red[kMhcThreads / 32][W + 1];
#pragma unroll
    for (int j = 0; j <= W; ++j) {
#pragma unroll
        for (int o = 16; o; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
        if (lane == 0) red[warp][j] = v[j];
    }
    __syncthreads();
    if (tid <= W) {
        float s2 = 0.f;
#pragma unroll
        for (int w = 0; w < kMhcThreads / 32; ++w) s2 += red[w][tid];
        partial[((size_t)t * gridDim.x + slice) * (W + 1) + tid] = s2;
    }
}

// Coefficients, one warp per token: the slice partials (lanes stride, then a
// fixed tree), the RMS factor of the streams, pre / post, the row softmax and
// the Sinkhorn steps on N*N lanes (comb[i][j] on lane i*N + j).
__global__ void __launch_bounds__(kMhcThreads) mhc_coef_kernel(const float* __restrict__ partial, int S, int n,
                                                             float* __restrict__ pre_out, MhcArgs a) {
    const int lane = threadIdx.x & 31, t = blockIdx.x * (kMhcThreads / 32) + (threadIdx.x >> 5);
    if (t >= n) return;
    const int N = a.N, HN = N * a.H, W = (2 + N) * N;
    // lane i loads slice i's W + 1 sums (all loads issued together), then a fixed
    // shuffle tree per sum; lane j keeps sum j (W + 1 <= 32)
    float part[kMhcMaxW + 1];
#pragma unroll
    for (int j = 0; j <= kMhcMaxW; ++j) part[j] = 0.f;
    for (int i0 = 0; i0 < S; i0 += 32) {
        const float* pp = partial + ((size_t)t * S + i0 + lane) * (W + 1);
        const bool have = i0 + lane < S;
#pragma unroll
        for (int j = 0; j <= kMhcMaxW; ++j)
            if (j <= W && have) part[j] += pp[j];
    }
    float wv = 0.f;
#pragma unroll
    for (int j = 0; j <= kMhcMaxW; ++j) {
        float s = part[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == j) wv = s;
    }
    const float r = 1.0f / sqrtf(__shfl_sync(0xffffffffu, wv, 0) / (float)HN + a.rms_eps);
    const float w_pre = __shfl_sync(0xffffffffu, wv, (1 + lane) & 31);
    const float w_post = __shfl_sync(0xffffffffu, wv, (1 + N + lane) & 31);
    const float w_comb = __shfl_sync(0xffffffffu, wv, (1 + 2 * N + lane) & 31);
    if (lane < N) {
        pre_out[(size_t)t * N + lane] = 1.0f / (1.0f + expf(-(w_pre * r * a.scale[0] + a.base[lane]))) + a.hc_eps;
        a.post_out[(size_t)t * N + lane] = 2.0f / (1.0f + expf(-(w_post * r * a.scale[1] + a.base[N + lane])));
    }
    const int i = lane / N, j = lane % N;
    const bool on = lane < N * N;
    float c = 0.f;
    {
        const float z = on ? w_comb * r * a.scale[2] + a.base[2 * N + lane] : 0.f;
        float mx = z;
        for (int q = 0; q < N; ++q) mx = fmaxf(mx, __shfl_sync(0xffffffffu, z, (i * N + q) & 31));
        const float e = on ? expf(z - mx) : 0.f;
        float sum = 0.f;
        for (int q = 0; q < N; ++q) sum += __shfl_sync(0xffffffffu, e, (i * N + q) & 31);
        if (on) c = e * (1.0f / sum) + a.hc_eps;
    }
    // Sinkhorn: columns, then (iters - 1) x (rows, columns); sums in index order + eps
    for (int it = 0; it < a.iters; ++it) {
        if (it > 0) {
            float rs = 0.f;
            for (int q = 0; q < N; ++q) rs += __shfl_sync(0xffffffffu, c, (i * N + q) & 31);
            if (on) c = c / (rs + a.hc_eps);
        }
        float cs = 0.f;
        for (int q = 0; q < N; ++q) cs += __shfl_sync(0xffffffffu, c, (q * N + j) & 31);
        if (on) c = c / (cs + a.hc_eps);
    }
    if (on) a.comb_out[(size_t)t * N * N + lane] = c;
}

// One CTA per token: mixed = sum_n pre[n] streams[n] (kept in shared memory),
// then the weighted RMSNorm.
__global__ void __launch_bounds__(kMhcThreads) mhc_mix_kernel(const float* __restrict__ streams,
                                                            const float* __restrict__ pre, MhcArgs a) {
    extern __shared__ __align__(16) float mixed[];  // [H]
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, H = a.H;
    __shared__ float red[kMhcThreads / 32];
    const float4* S4 = reinterpret_cast<const float4*>(streams + (size_t)t * N * H);
    float p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = q < N ? pre[(size_t)t * N + q] : 0.f;
    float ss2 = 0.f;
#pragma unroll 2
    for (int d4 = tid; d4 < H / 4; d4 += kMhcThreads) {
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (q >= N) break;
            const float4 v = S4[q * (H / 4) + d4];
            m.x += p[q] * v.x;
            m.y += p[q] * v.y;
            m.z += p[q] * v.z;
            m.w += p[q] * v.w;
        }
        reinterpret_cast<float4*>(mixed)[d4] = m;
        ss2 += m.x * m.x + m.y * m.y + m.z * m.z + m.w * m.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss2 += __shfl_xor_sync(0xffffffffu, ss2, o);
    if (lane == 0) red[warp] = ss2;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kMhcThreads / 32; ++w) tot += red[w];
    const float r2 = 1.0f / sqrtf(tot / (float)H + a.rms_eps);
    const bool vec = ((reinterpret_cast<uintptr_t>(a.norm_w) | reinterpret_cast<uintptr_t>(a.x_out)) & 15) == 0;
    if (vec) {  // 4 elements per thread per step: 16-byte loads, 8-byte (bf16) or 16-byte (fp32) stores
        for (int d4 = tid; d4 < H / 4; d4 += kMhcThreads) {
            const float4 m = reinterpret_cast<const float4*>(mixed)[d4];
            const float4 w = reinterpret_cast<const float4*>(a.norm_w)[d4];
            const float4 v = make_float4(m.x * r2 * w.x, m.y * r2 * w.y, m.z * r2 * w.z, m.w * r2 * w.w);
            if (a.x_bf16) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&lo);
                u.y = *reinterpret_cast<uint32_t*>(&hi);
                reinterpret_cast<uint2*>(a.x_out)[(size_t)t * (H / 4) + d4] = u;
            } else {
                reinterpret_cast<float4*>(a.x_out)[(size_t)t * (H / 4) + d4] = v;
            }
        }
        return;
    }
#pragma unroll 4
    for (int d = tid; d < H; d += kMhcThreads) {
        const float v = mixed[d] * r2 * a.norm_w[d];
        if (a.x_bf16)
            reinterpret_cast<__nv_bfloat16*>(a.x_out)[(size_t)t * H + d] = __float2bfloat16_rn(v);
        else
            reinterpret_cast<float*>(a.x_out)[(size_t)t * H + d] = v;
    }
}

template <int N>
__global__ void mhc_post_kernel(const float* in, const float* __restrict__ mlp, const float* __restrict__ post,
                                const float* __restrict__ comb, int n, int H, float* out) {
    const int q = H / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)n * q;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / q), d4 = (int)(i % q);
        const float4 m = reinterpret_cast<const float4*>(mlp + (size_t)t * H)[d4];
        float4 s[N];
#pragma unroll
        for (int k = 0; k < N; ++k) s[k] = reinterpret_cast<const float4*>(in + ((size_t)t * N + k) * H)[d4];
        const float* c = comb + (size_t)t * N * N;
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float p = post[(size_t)t * N + k];
            float4 o = make_float4(p * m.x, p * m.y, p * m.z, p * m.w);
#pragma unroll
            for (int j = 0; j < N; ++j) {
                const float w = c[j * N + k];
                o.x += w * s[j].x;
                o.y += w * s[j].y;
                o.z += w * s[j].z;
                o.w += w * s[j].w;
            }
            reinterpret_cast<float4*>(out + ((size_t)t * N + k) * H)[d4] = o;
        }
    }
}

}  // namespace

// K slices so that tiles x slices give every SM about 8 CTAs (each slice a whole number of 32-element steps)
int mhc_slices(int n, int HN) {
    const int tiles = (n + kDotM - 1) / kDotM, steps = (HN + kDotK - 1) / kDotK;
    int S = (8 * 148 + tiles - 1) / tiles;
    if (S > 64) S = 64;  // the coefficient kernel reads a token's slices in two rounds of 32 lanes at most
    if (S > steps) S = steps;
    if (S < 1) S = 1;
    return S;
}

constexpr int kVecMaxTokens = 32;  // below this the vector kernel (one token per CTA) is used

int mhc_slices_for(int n, int HN) {
    return n < kVecMaxTokens ? (HN + 4 * kMhcThreads - 1) / (4 * kMhcThreads) : mhc_slices(n, HN);
}

// slice partials, then pre[n][N]
int mhc_partial_floats(int n, int N, int H) { return n * mhc_slices_for(n, N * H) * ((2 + N) * N + 1) + n * N; }

cudaError_t launch_mhc_pre(const float* streams, int n, const MhcArgs& a, float* partial, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int HN = a.N * a.H;
    if (a.H % 4) return cudaErrorInvalidValue;
    const int S = mhc_slices_for(n, HN);
    if (n < kVecMaxTokens) {
        const dim3 grid(S, n);
        switch (a.N) {
            case 1: mhc_dot_vec_kernel<1><<<grid, kMhcThreads, 0, st>>>(streams, a.fn, HN, partial); break;
            case 2: mhc_dot_vec_kernel<2><<<grid, kMhcThreads, 0, st>>>(streams, a.fn, HN, partial); break;
            case 3: mhc_dot_vec_kernel<3><<<grid, kMhcThreads, 0, st>>>(streams, a.fn, HN, partial); break;
            case 4: mhc_dot_vec_kernel<4><<<grid, kMhcThreads, 0, st>>>(streams, a.fn, HN, partial); break;
            default: return cudaErrorInvalidValue;
        }
    } else {
    const int steps = (HN + kDotK - 1) / kDotK, klen = (steps + S - 1) / S * kDotK;
    const dim3 grid(S, (n + kDotM - 1) / kDotM);
    switch (a.N) {
        case 1: mhc_dot_kernel<1><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 2: mhc_dot_kernel<2><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 3: mhc_dot_kernel<3><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 4: mhc_dot_kernel<4><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        default: return cudaErrorInvalidValue;
    }
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    float* pre = partial + (size_t)n * S * ((2 + a.N) * a.N + 1);
    mhc_coef_kernel<<<(n + kMhcThreads / 32 - 1) / (kMhcThreads / 32), kMhcThreads, 0, st>>>(partial, S, n, pre, a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = sizeof(float) * (size_t)a.H;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(mhc_mix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    mhc_mix_kernel<<<n, kMhcThreads, smem, st>>>(streams, pre, a);
    return cudaGetLastError();
}

cudaError_t launch_mhc_post(const float* in, const float* mlp, const float* post, const float* comb, int n, int N,
                            int H, float* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (N < 1 || N > 4 || H % 4) return cudaErrorInvalidValue;
    const int64_t items = (int64_t)n * (H / 4);
    int64_t grid = (items + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    switch (N) {
        case 1: mhc_post_kernel<1><<<(int)grid, 256, 0, st>>>(in, mlp, post, comb, n, H, out); break;
        case 2: mhc_post_kernel<2><<<(int)grid, 256, 0, st>>>(in, mlp, post, comb, n, H, out); break;
        case 3: mhc_post_kernel<3><<<(int)grid, 256, 0, st>>>(in, mlp, post, comb, n, H, out); break;
        default: mhc_post_kernel<4><<<(int)grid, 256, 0, st>>>(in, mlp, post, comb, n, H, out); break;
    }
    return cudaGetLastError();
}

}  // namespace gp
