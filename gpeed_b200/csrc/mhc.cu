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
// Kernels: mhc_dot_kernel<N> computes the W dot products of fn with the raw
// streams as a small SGEMM over token tiles and K slices (fn is read once per
// 64-token tile); mhc_finish_kernel (one CTA per token) adds the slices in
// order, scales by the RMS factor (r * (fn . x) = fn . (r x)), forms the
// coefficients with one warp, mixes the streams into shared memory and
// normalises; mhc_post_kernel updates the streams element-wise (one thread per
// (token, 4 elements) writes all N streams, so it may run in place).  fp32
// throughout; expf / sqrtf are CUDA's.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace gp {
namespace {

constexpr int kMhcMaxW = 24;          // (2 + N) N for N <= 4
constexpr int kMhcThreads = 256;

// Dot products as a small SGEMM: a CTA takes a tile of 64 tokens x all W
// outputs over one K slice, staging 64 x 32 stream values and W x 32 fn values
// per step in shared memory; 128 threads, each 4 tokens x (W / 8) outputs.
constexpr int kDotM = 64, kDotK = 32, kDotThreads = 128;

template <int N>
__global__ void __launch_bounds__(kDotThreads) mhc_dot_kernel(const float* __restrict__ streams,
                                                             const float* __restrict__ fn, int n, int HN, int klen,
                                                             float* __restrict__ partial) {
    constexpr int W = (2 + N) * N, WT = (W + 7) / 8;  // outputs per thread
    __shared__ __align__(16) float xs[kDotK][kDotM + 4];
    __shared__ __align__(16) float fs[kDotK][8 * WT + 1];
    const int tid = threadIdx.x, tm = tid & 15, tn = tid >> 4;  // 16 x 8 threads
    const int t0 = blockIdx.y * kDotM, slice = blockIdx.x;
    const int kb = slice * klen, ke = min(HN, kb + klen);
    float acc[4][WT];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < WT; ++j) acc[i][j] = 0.f;
    for (int k0 = kb; k0 < ke; k0 += kDotK) {
        // stage: 64 tokens x 32 k (512 float4, 4 per thread), W x 32 fn
        for (int i = tid; i < kDotM * kDotK / 4; i += kDotThreads) {
            const int r = i >> 3, c4 = (i & 7) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + r < n && k0 + c4 < ke) v = *reinterpret_cast<const float4*>(streams + (size_t)(t0 + r) * HN + k0 + c4);
            xs[c4][r] = v.x;
            xs[c4 + 1][r] = v.y;
            xs[c4 + 2][r] = v.z;
            xs[c4 + 3][r] = v.w;
        }
        for (int i = tid; i < 8 * WT * kDotK / 4; i += kDotThreads) {
            const int r = i >> 3, c4 = (i & 7) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < W && k0 + c4 < ke) v = __ldg(reinterpret_cast<const float4*>(fn + (size_t)r * HN + k0 + c4));
            fs[c4][r] = v.x;
            fs[c4 + 1][r] = v.y;
            fs[c4 + 2][r] = v.z;
            fs[c4 + 3][r] = v.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kDotK; ++k) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[k][4 * tm]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < WT; ++j) {
                const float f = fs[k][tn * WT + j];
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i][j] += xa[i] * f;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + 4 * tm + i;
        if (t >= n) continue;
#pragma unroll
        for (int j = 0; j < WT; ++j) {
            const int o = tn * WT + j;
            if (o < W) partial[((size_t)t * gridDim.x + slice) * W + o] = acc[i][j];
        }
    }
}

// One CTA per token: sum of squares of the streams, coefficients (one warp,
// N*N lanes for the Sinkhorn steps), mixed streams kept in shared memory, then
// the weighted RMSNorm.
__global__ void __launch_bounds__(kMhcThreads) mhc_finish_kernel(const float* __restrict__ streams,
                                                               const float* __restrict__ partial, int S,
                                                               MhcArgs a) {
    extern __shared__ __align__(16) float mixed[];  // [H]
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, H = a.H, HN = N * H, W = (2 + N) * N;
    __shared__ float wv[kMhcMaxW];
    __shared__ float coef[4];  // pre[N]
    __shared__ float red[kMhcThreads / 32];
    const float4* S4 = reinterpret_cast<const float4*>(streams + (size_t)t * HN);
    float ss = 0.f;
    for (int i = tid; i < HN / 4; i += kMhcThreads) {
        const float4 v = S4[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    for (int j = warp; j < W; j += kMhcThreads / 32) {  // slice partials: lanes stride, then a fixed tree
        float s = 0.f;
        for (int i = lane; i < S; i += 32) s += partial[((size_t)t * S + i) * W + j];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) wv[j] = s;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float tot = 0.f;
        for (int w = 0; w < kMhcThreads / 32; ++w) tot += red[w];
        const float r = 1.0f / sqrtf(tot / (float)HN + a.rms_eps);
        if (lane < N) {
            coef[lane] = 1.0f / (1.0f + expf(-(wv[lane] * r * a.scale[0] + a.base[lane]))) + a.hc_eps;
            a.post_out[(size_t)t * N + lane] = 2.0f / (1.0f + expf(-(wv[N + lane] * r * a.scale[1] + a.base[N + lane])));
        }
        // comb[i][j] on lane i * N + j; row groups of N lanes
        const int i = lane / N, j = lane % N;
        const bool on = lane < N * N;
        const unsigned grp = on ? (((1u << N) - 1u) << (i * N)) : 0u;
        float c = 0.f;
        if (on) {
            const float z = wv[2 * N + lane] * r * a.scale[2] + a.base[2 * N + lane];
            float mx = z;
            for (int q = 0; q < N; ++q) mx = fmaxf(mx, __shfl_sync(grp, z, i * N + q));
            const float e = expf(z - mx);
            float sum = 0.f;
            for (int q = 0; q < N; ++q) sum += __shfl_sync(grp, e, i * N + q);
            c = e * (1.0f / sum) + a.hc_eps;
        }
        // Sinkhorn: columns, then (iters - 1) x (rows, columns); sums in index order + eps
        const unsigned all = (N * N == 32) ? 0xffffffffu : ((1u << (N * N)) - 1u);
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
        (void)all;
        if (on) a.comb_out[(size_t)t * N * N + lane] = c;
    }
    __syncthreads();
    // mixed = sum_n pre[n] streams[n] (kept in shared memory), then the weighted RMSNorm
    float ss2 = 0.f;
    for (int d4 = tid; d4 < H / 4; d4 += kMhcThreads) {
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < N; ++q) {
            const float4 v = S4[q * (H / 4) + d4];
            const float p = coef[q];
            m.x += p * v.x;
            m.y += p * v.y;
            m.z += p * v.z;
            m.w += p * v.w;
        }
        reinterpret_cast<float4*>(mixed)[d4] = m;
        ss2 += m.x * m.x + m.y * m.y + m.z * m.z + m.w * m.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss2 += __shfl_xor_sync(0xffffffffu, ss2, o);
    __syncthreads();  // red reuse
    if (lane == 0) red[warp] = ss2;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kMhcThreads / 32; ++w) tot += red[w];
    const float r2 = 1.0f / sqrtf(tot / (float)H + a.rms_eps);
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
    if (S > steps) S = steps;
    if (S < 1) S = 1;
    return S;
}

int mhc_partial_floats(int n, int N, int H) { return n * mhc_slices(n, N * H) * (2 + N) * N; }

cudaError_t launch_mhc_pre(const float* streams, int n, const MhcArgs& a, float* partial, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int HN = a.N * a.H;
    if (a.H % 4) return cudaErrorInvalidValue;
    const int S = mhc_slices(n, HN);
    const int steps = (HN + kDotK - 1) / kDotK, klen = (steps + S - 1) / S * kDotK;
    const dim3 grid(S, (n + kDotM - 1) / kDotM);
    switch (a.N) {
        case 1: mhc_dot_kernel<1><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 2: mhc_dot_kernel<2><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 3: mhc_dot_kernel<3><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        case 4: mhc_dot_kernel<4><<<grid, kDotThreads, 0, st>>>(streams, a.fn, n, HN, klen, partial); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = sizeof(float) * (size_t)a.H;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(mhc_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    mhc_finish_kernel<<<n, kMhcThreads, smem, st>>>(streams, partial, S, a);
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
