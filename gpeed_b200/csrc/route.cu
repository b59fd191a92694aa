// Router, top-k routing and the weighted un-permute of the MoE layer.
//
//  router_kernel   fp32 router logits (reference model.cpp:41-46/702 for one
//                  token, model_batch.cpp:172 for a batch): one CTA per expert
//                  row, warps striding the row, partial sums added in a fixed
//                  order (deterministic, no atomics).
//  route_kernel    sigmoid scores, +correction bias, top-K by choice (ties to
//                  the lower expert id), weights score/(1e-20 + sum)*scale
//                  (model.cpp:704-725, model_batch.cpp:184-203), then the
//                  expert histogram, exclusive scan and stable expert-major
//                  permutation (model_batch.cpp:204-219), and the slot list
//                  (experts split into runs of <= nt assignments) consumed by
//                  the expert kernels.  One CTA.  The stable permutation is
//                  computed in parallel: each expert keeps a bitmap of the
//                  tokens that chose it, and a token's rank inside its expert
//                  is the popcount of the bitmap below it.
//  combine_kernel  y[t] = sum_k w[t][k] * D[pos(t,k)] (+ shared-expert row),
//                  in top-k order (model.cpp:741-755; the batched reference
//                  adds in expert-id order, model_batch.cpp:257-280 - a
//                  rounding-level difference).
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace gp {
namespace {

constexpr int kRouterWarps = 8;
constexpr int kRouterTok = 8;     // tokens per CTA
constexpr int kRouterMaxVec = 8;  // float4s per lane (H <= 8192)

// One CTA = one expert row e for up to 8 tokens.  The 8 warps stride the row
// in float4s; every lane issues all of its weight loads before any arithmetic,
// and the 8 warp sums are added in warp order (deterministic).
__global__ void __launch_bounds__(32 * kRouterWarps) router_kernel(const RouterArgs a) {
    __shared__ float s_part[kRouterWarps][kRouterTok];
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x;
    const int tc = blockIdx.y;
    const int nq = a.H / 4;                       // float4s per row
    const int q0 = warp * 32 + lane;              // this lane's first float4
    const float4* w = reinterpret_cast<const float4*>(a.w + (int64_t)e * a.H);
    float4 wv[kRouterMaxVec];
#pragma unroll
    for (int i = 0; i < kRouterMaxVec; ++i)
        if (q0 + 256 * i < nq) wv[i] = w[q0 + 256 * i];
    const int ntok = min(kRouterTok, a.n - tc * kRouterTok);
    for (int t = 0; t < ntok; ++t) {
        const int64_t tok = tc * kRouterTok + t;
        float acc = 0.f;
        float4 xv[kRouterMaxVec];
#pragma unroll
        for (int i = 0; i < kRouterMaxVec; ++i) {
            const int q = q0 + 256 * i;
            if (q >= nq) break;
            if (a.x_bf16) {
                const uint2 r = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + tok * a.H)[q];
                xv[i] = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                    __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
            } else {
                xv[i] = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + tok * a.H)[q];
            }
        }
#pragma unroll
        for (int i = 0; i < kRouterMaxVec; ++i) {
            if (q0 + 256 * i >= nq) break;
            acc = fmaf(wv[i].x, xv[i].x, acc);
            acc = fmaf(wv[i].y, xv[i].y, acc);
            acc = fmaf(wv[i].z, xv[i].z, acc);
            acc = fmaf(wv[i].w, xv[i].w, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) s_part[warp][t] = acc;
    }
    __syncthreads();
    if (threadIdx.x < ntok) {
        float v = 0.f;
        for (int w8 = 0; w8 < kRouterWarps; ++w8) v += s_part[w8][threadIdx.x];
        a.logits[((int64_t)tc * kRouterTok + threadIdx.x) * a.E + e] = v;
    }
    pdl_launch_dependents();
}

// Large batches: logits as a register-blocked fp32 GEMM.  CTA tile = 128
// tokens x 32 experts, K in slices of 32 staged in shared memory; each thread
// accumulates 4 tokens x 4 experts over its K range in order.  With
// gridDim.z = S > 1 CTA z covers K range z of S and writes partial sums to
// split_scratch[z]; router_split_sum_kernel adds them in order z = 0..S-1
// (deterministic).  The split gives each SM several CTAs, whose loads hide
// one another's global-memory latency.
constexpr int kRgTok = 128, kRgExp = 32, kRgK = 32;
__global__ void __launch_bounds__(256) router_gemm_kernel(const RouterArgs a) {
    __shared__ __align__(16) float xs[kRgK][kRgTok + 4];
    __shared__ __align__(16) float ws[kRgK][kRgExp + 4];
    pdl_wait();
    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const int t0 = blockIdx.y * kRgTok, e0 = blockIdx.x * kRgExp;
    const int klen = a.H / (int)gridDim.z, kbeg = (int)blockIdx.z * klen;
    float* out = gridDim.z == 1 ? a.logits : a.split_scratch + (size_t)blockIdx.z * a.n * a.E;
    float acc[4][4] = {};
    for (int k0 = kbeg; k0 < kbeg + klen; k0 += kRgK) {
        // x tile: 128 tokens x 32 k (4 consecutive k per load)
        for (int i = tid; i < kRgTok * kRgK / 4; i += 256) {
            const int t = i / (kRgK / 4), kq = (i % (kRgK / 4)) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + t < a.n) {
                const int64_t off = (int64_t)(t0 + t) * a.H + k0 + kq;
                if (a.x_bf16) {
                    const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + off);
                    v = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                    __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
                } else {
                    v = *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + off);
                }
            }
            xs[kq][t] = v.x;
            xs[kq + 1][t] = v.y;
            xs[kq + 2][t] = v.z;
            xs[kq + 3][t] = v.w;
        }
        // w tile: 32 experts x 32 k
        {
            const int e = tid / (kRgK / 4), kq = (tid % (kRgK / 4)) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 + e < a.E) v = *reinterpret_cast<const float4*>(a.w + (int64_t)(e0 + e) * a.H + k0 + kq);
            ws[kq][e] = v.x;
            ws[kq + 1][e] = v.y;
            ws[kq + 2][e] = v.z;
            ws[kq + 3][e] = v.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kRgK; ++k) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[k][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&ws[k][tx * 4]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= a.n) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < a.E) out[(int64_t)t * a.E + e] = acc[i][j];
        }
    }
    pdl_launch_dependents();
}

__global__ void router_split_sum_kernel(const RouterArgs a, int S) {
    pdl_wait();
    const size_t ne = (size_t)a.n * a.E;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ne; i += (size_t)gridDim.x * blockDim.x) {
        float v = a.split_scratch[i];
        for (int z = 1; z < S; ++z) v += a.split_scratch[z * ne + i];
        a.logits[i] = v;
    }
    pdl_launch_dependents();
}

constexpr int kRouteThreads = 1024;
constexpr int kMaxE = 512;

// Warp-level top-K of one token: lane j holds experts j, j+32, ... (<= 16 each).
GP_DEVINL void topk_token(const RouteArgs& a, int t, int lane, int* s_ids) {
    const int E = a.E, K = a.K, n = a.n;
    float lg[kMaxE / 32];
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
        const int e = lane + 32 * j;
        lg[j] = e < E ? a.logits[(int64_t)t * E + e] : 0.f;
    }
    float score[kMaxE / 32], choice[kMaxE / 32];
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
        const int e = lane + 32 * j;
        score[j] = 1.0f / (1.0f + expf(-lg[j]));
        choice[j] = e < E ? score[j] + (a.corr ? a.corr[e] : 0.f) : -INFINITY;
    }
    float denom = 1e-20f;
    float my_s = 0.f;  // lane k keeps the score of the k-th pick
    int my_e = 0;
    for (int k = 0; k < K; ++k) {
        int e_best;
        if (a.forced) {
            e_best = a.forced[(int64_t)t * K + k];
            if (e_best < 0 || e_best >= E) {
                if (lane == 0) atomicOr(a.status, GP_DEV_BAD_EXPERT);
                e_best = 0;
            }
        } else {
            float bv = -INFINITY;
            int be = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < kMaxE / 32; ++j) {
                const int e = lane + 32 * j;
                if (e < E && (choice[j] > bv || (choice[j] == bv && e < be))) { bv = choice[j]; be = e; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oe = __shfl_xor_sync(0xffffffffu, be, o);
                if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
            }
            e_best = be;
        }
        float sc = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxE / 32; ++j)
            if (lane + 32 * j == e_best) { sc = score[j]; choice[j] = -INFINITY; }
        sc = __shfl_sync(0xffffffffu, sc, e_best & 31);
        denom += sc;  // model.cpp:718-721 order
        if (lane == k) { my_s = sc; my_e = e_best; }
    }
    if (lane < K) {
        const float w = a.norm_topk ? (my_s / denom) * a.routed_scale : my_s * a.routed_scale;
        a.topk_ids[(int64_t)t * K + lane] = my_e;
        a.topk_w[(int64_t)t * K + lane] = w;
        if (s_ids) s_ids[t * K + lane] = my_e;
    }
}

// Dynamic shared memory: bitmap [E][ns] + word prefix [E][ns] (ns = ceil(n/32) rounded up to odd)
// + cached top-k ids [n*K] when n*K <= kCacheIds.
constexpr int kCacheIds = 8192;

__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteArgs a) {
    extern __shared__ __align__(16) uint32_t dsm[];
    __shared__ int s_cnt[kMaxE];
    __shared__ int s_ptr[kMaxE + 1];
    __shared__ int s_slot0[kMaxE + 1];
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = kRouteThreads / 32;
    const int E = a.E, K = a.K, n = a.n;
    if (E > kMaxE || K > 32 || K > E) {
        if (tid == 0) { atomicOr(a.status, GP_DEV_BAD_SHAPE); *a.nslots = 0; }
        return;
    }
    // per-expert token bitmaps, rows padded to an odd word count so that one
    // token word of different experts falls in different banks
    const int nw = (n + 31) / 32, ns = nw | 1;
    uint32_t* bitmap = dsm;
    uint32_t* wpref = dsm + E * ns;
    int* s_ids = (!a.topk_ready && n * K <= kCacheIds) ? reinterpret_cast<int*>(dsm + 2 * E * ns) : nullptr;
    for (int i = tid; i < E * ns; i += kRouteThreads) bitmap[i] = 0;
    for (int e = tid; e < E; e += kRouteThreads) s_cnt[e] = 0;
    __syncthreads();

    // 1. top-K per token (warp per token)
    if (!a.topk_ready)
        for (int t = warp; t < n; t += nwarp) topk_token(a, t, lane, s_ids);
    __syncthreads();

    // 2. histogram and token bitmaps (thread per assignment)
    const int nk = n * K;
    for (int i = tid; i < nk; i += kRouteThreads) {
        const int t = i / K;
        const int e = s_ids ? s_ids[i] : a.topk_ids[i];
        atomicAdd(&s_cnt[e], 1);
        atomicOr(&bitmap[e * ns + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();

    // 3. exclusive scans: counts -> bucket starts; per-expert word prefixes
    if (warp == 0) {
        int run = 0, srun = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            const int c = e < E ? s_cnt[e] : 0;
            const bool own = e >= a.expert_lo && e < a.expert_hi;
            const int ns = own ? (c + a.nt - 1) / a.nt : 0;
            int inc = c, sinc = ns;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, inc, o);
                const int sv = __shfl_up_sync(0xffffffffu, sinc, o);
                if (lane >= o) { inc += v; sinc += sv; }
            }
            if (e < E) { s_ptr[e] = run + inc - c; s_slot0[e] = srun + sinc - ns; }
            run += __shfl_sync(0xffffffffu, inc, 31);
            srun += __shfl_sync(0xffffffffu, sinc, 31);
        }
        if (lane == 0) { s_ptr[E] = run; s_slot0[E] = srun; }
    }
    for (int e = tid; e < E; e += kRouteThreads) {
        uint32_t acc = 0;
        for (int w = 0; w < nw; ++w) {
            wpref[e * ns + w] = acc;
            acc += __popc(bitmap[e * ns + w]);
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouteThreads) a.counts[e] = s_cnt[e];

    // 4. stable positions (thread per assignment)
    for (int i = tid; i < nk; i += kRouteThreads) {
        const int t = i / K;
        const int e = s_ids ? s_ids[i] : a.topk_ids[i];
        const uint32_t below = bitmap[e * ns + (t >> 5)] & ((1u << (t & 31)) - 1u);
        const int p = s_ptr[e] + (int)wpref[e * ns + (t >> 5)] + __popc(below);
        a.perm_tok[p] = t;
        a.inv_pos[i] = p;
    }
    // 5. slots: runs of <= nt assignments per owned expert, then the shared expert
    for (int e = warp; e < E; e += nwarp) {
        if (e < a.expert_lo || e >= a.expert_hi) continue;
        const int c = s_cnt[e];
        for (int i = lane; i * a.nt < c; i += 32) {
            const int sidx = s_slot0[e] + i;
            if (sidx < a.max_slots) {
                SlotDesc sd;
                sd.expert = e;
                sd.begin = s_ptr[e] + i * a.nt;
                sd.ntok = min(a.nt, c - i * a.nt);
                sd.pad = 0;
                a.slots[sidx] = sd;
            }
        }
    }
    int total = s_slot0[E];
    if (a.with_shared) {
        for (int t = tid; t < n; t += kRouteThreads) a.perm_tok[nk + t] = t;
        const int ns = (n + a.nt - 1) / a.nt;
        for (int i = tid; i < ns; i += kRouteThreads) {
            const int sidx = total + i;
            if (sidx < a.max_slots) {
                SlotDesc sd;
                sd.expert = E;  // the shared expert is stored after the routed ones
                sd.begin = nk + i * a.nt;
                sd.ntok = min(a.nt, n - i * a.nt);
                sd.pad = 0;
                a.slots[sidx] = sd;
            }
        }
        total += ns;
    }
    if (tid == 0) {
        if (total > a.max_slots) { atomicOr(a.status, GP_DEV_BAD_SHAPE); total = a.max_slots; }
        *a.nslots = total;
    }
    __syncthreads();
    pdl_launch_dependents();
}

// Multi-CTA top-K for large batches (warp per token); route_kernel then skips step 1.
__global__ void __launch_bounds__(256) topk_kernel(const RouteArgs a) {
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int t = warp; t < a.n; t += nwarps) topk_token(a, t, lane, nullptr);
    pdl_launch_dependents();
}

// ---- large batches: stable counting sort over many CTAs ---------------------
// The single-CTA route_kernel keeps per-expert token bitmaps in shared memory,
// which stops fitting (and stops being fast) past a few thousand assignments.
// For those: (1) per-chunk expert histograms, (2) one CTA scans them over
// chunks and experts into every chunk's starting position per expert and
// writes counts and the slot list, (3) one warp per chunk walks its
// assignments in order and places each one after the earlier ones of its
// expert (ranks within 32 assignments from a warp match), so the permutation
// is the same stable expert-major order as route_kernel's.
constexpr int kChunk = 256;          // assignments per chunk (one warp)
constexpr int kChunkThreshold = 8192;  // assignments from which the chunked sort runs

GP_DEVINL int assignment_expert(const RouteArgs& a, int i) { return a.topk_ids[i]; }

__global__ void __launch_bounds__(256) route_hist_kernel(const RouteArgs a, int nchunks) {
    __shared__ int hist[kMaxE];
    pdl_wait();
    const int nk = a.n * a.K;
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
        for (int e = threadIdx.x; e < a.E; e += blockDim.x) hist[e] = 0;
        __syncthreads();
        for (int i = c * kChunk + threadIdx.x; i < min(nk, (c + 1) * kChunk); i += blockDim.x) {
            const int e = assignment_expert(a, i);
            if (e >= 0 && e < a.E) atomicAdd(&hist[e], 1);
            else atomicOr(a.status, GP_DEV_BAD_EXPERT);
        }
        __syncthreads();
        for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.chunk_counts[(size_t)c * a.E + e] = hist[e];
        __syncthreads();
    }
}

// One CTA: chunk_counts[c][e] becomes the position of chunk c's first
// assignment to expert e; counts, slots and the shared-expert rows as in route_kernel.
__global__ void __launch_bounds__(kRouteThreads) route_scan_kernel(const RouteArgs a, int nchunks) {
    __shared__ int s_cnt[kMaxE];
    __shared__ int s_ptr[kMaxE + 1];
    __shared__ int s_slot0[kMaxE + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = kRouteThreads / 32;
    const int E = a.E, n = a.n, nk = n * a.K;
    for (int e = tid; e < E; e += kRouteThreads) {
        int run = 0;
        for (int c = 0; c < nchunks; ++c) {
            const int v = a.chunk_counts[(size_t)c * E + e];
            a.chunk_counts[(size_t)c * E + e] = run;
            run += v;
        }
        s_cnt[e] = run;
    }
    __syncthreads();
    if (warp == 0) {
        int run = 0, srun = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            const int c = e < E ? s_cnt[e] : 0;
            const bool own = e >= a.expert_lo && e < a.expert_hi;
            const int ns = own ? (c + a.nt - 1) / a.nt : 0;
            int inc = c, sinc = ns;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, inc, o);
                const int sv = __shfl_up_sync(0xffffffffu, sinc, o);
                if (lane >= o) { inc += v; sinc += sv; }
            }
            if (e < E) { s_ptr[e] = run + inc - c; s_slot0[e] = srun + sinc - ns; }
            run += __shfl_sync(0xffffffffu, inc, 31);
            srun += __shfl_sync(0xffffffffu, sinc, 31);
        }
        if (lane == 0) { s_ptr[E] = run; s_slot0[E] = srun; }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouteThreads) {
        a.counts[e] = s_cnt[e];
        for (int c = 0; c < nchunks; ++c) a.chunk_counts[(size_t)c * E + e] += s_ptr[e];
    }
    for (int e = warp; e < E; e += nwarp) {
        if (e < a.expert_lo || e >= a.expert_hi) continue;
        const int c = s_cnt[e];
        for (int i = lane; i * a.nt < c; i += 32) {
            const int sidx = s_slot0[e] + i;
            if (sidx < a.max_slots) {
                SlotDesc sd;
                sd.expert = e;
                sd.begin = s_ptr[e] + i * a.nt;
                sd.ntok = min(a.nt, c - i * a.nt);
                sd.pad = 0;
                a.slots[sidx] = sd;
            }
        }
    }
    int total = s_slot0[E];
    if (a.with_shared) {
        for (int t = tid; t < n; t += kRouteThreads) a.perm_tok[nk + t] = t;
        const int ns = (n + a.nt - 1) / a.nt;
        for (int i = tid; i < ns; i += kRouteThreads) {
            const int sidx = total + i;
            if (sidx < a.max_slots) {
                SlotDesc sd;
                sd.expert = E;  // the shared expert is stored after the routed ones
                sd.begin = nk + i * a.nt;
                sd.ntok = min(a.nt, n - i * a.nt);
                sd.pad = 0;
                a.slots[sidx] = sd;
            }
        }
        total += ns;
    }
    if (tid == 0) {
        if (total > a.max_slots) { atomicOr(a.status, GP_DEV_BAD_SHAPE); total = a.max_slots; }
        *a.nslots = total;
    }
}

// One warp per chunk, its assignments in order: stable positions.
__global__ void __launch_bounds__(256) route_scatter_kernel(const RouteArgs a, int nchunks) {
    __shared__ int cnt[8][kMaxE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 8 + warp;
    const int E = a.E, nk = a.n * a.K;
    if (c >= nchunks) return;
    for (int e = lane; e < E; e += 32) cnt[warp][e] = a.chunk_counts[(size_t)c * E + e];
    __syncwarp();
    for (int i0 = c * kChunk; i0 < min(nk, (c + 1) * kChunk); i0 += 32) {
        const int i = i0 + lane;
        const bool live = i < min(nk, (c + 1) * kChunk);
        int e = live ? assignment_expert(a, i) : -1;
        if (e >= E) e = -1;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int leader = __ffs(same) - 1;
        int b = (lane == leader && e >= 0) ? cnt[warp][e] : 0;
        b = __shfl_sync(0xffffffffu, b, leader);
        const int p = b + __popc(same & ((1u << lane) - 1u));
        __syncwarp();
        if (lane == leader && e >= 0) cnt[warp][e] = b + __popc(same);
        __syncwarp();
        if (live && e >= 0) {
            a.perm_tok[p] = i / a.K;
            a.inv_pos[i] = p;
        } else if (live) {
            a.inv_pos[i] = 0;  // a bad id (status already set): keep later reads in bounds
        }
    }
}

size_t route_chunk_ints_impl(int n, int K, int E) {
    const int nk = n * K;
    if (nk < kChunkThreshold) return 0;
    return (size_t)((nk + kChunk - 1) / kChunk) * E;
}

constexpr int kCombineMaxK = 32;
constexpr int kCombineThreads = 256;  // one float4 column of one token per thread
constexpr int kCombineGroup = 8;      // expert rows loaded together (16 B each per thread)

// y[t] = sum_k w[t][k] * D[pos(t,k)] (k in order, fp32 fma) + the shared-expert
// row.  The K rows are read in groups of 8 independent 16-byte loads per
// thread, so each SM keeps enough bytes in flight to stream D at HBM rate.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const CombineArgs a) {
    __shared__ int s_pos[kCombineMaxK];
    __shared__ float s_w[kCombineMaxK];
    pdl_wait();
    const int t = blockIdx.y;
    if (threadIdx.x < a.K) {
        s_pos[threadIdx.x] = a.inv_pos[(int64_t)t * a.K + threadIdx.x];
        s_w[threadIdx.x] = a.topk_w[(int64_t)t * a.K + threadIdx.x];
    }
    __syncthreads();
    const int j = (blockIdx.x * kCombineThreads + threadIdx.x) * 4;
    if (j >= a.H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < a.K; k0 += kCombineGroup) {
        float4 d[kCombineGroup];
#pragma unroll
        for (int g = 0; g < kCombineGroup; ++g)
            if (k0 + g < a.K) d[g] = __ldcs(reinterpret_cast<const float4*>(a.D + (int64_t)s_pos[k0 + g] * a.H + j));
#pragma unroll
        for (int g = 0; g < kCombineGroup; ++g)
            if (k0 + g < a.K) {
                const float w = s_w[k0 + g];
                acc.x = fmaf(w, d[g].x, acc.x);
                acc.y = fmaf(w, d[g].y, acc.y);
                acc.z = fmaf(w, d[g].z, acc.z);
                acc.w = fmaf(w, d[g].w, acc.w);
            }
    }
    if (a.with_shared) {
        const float* sh = a.D_shared ? a.D_shared + (int64_t)t * a.H : a.D + ((int64_t)a.n * a.K + t) * a.H;
        const float4 s = __ldcs(reinterpret_cast<const float4*>(sh + j));
        acc.x += s.x;
        acc.y += s.y;
        acc.z += s.z;
        acc.w += s.w;
    }
    *reinterpret_cast<float4*>(a.y + (int64_t)t * a.H + j) = acc;
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

}  // namespace

size_t route_smem_bytes(int n, int E, int K) {
    const size_t ns = ((n + 31) / 32) | 1;  // bitmap row stride (odd)
    return (2 * E * ns + ((size_t)n * K <= kCacheIds ? (size_t)n * K : 0)) * sizeof(uint32_t);
}

int router_gemm_splits(int n, int H, int E) {
    if (n < 64 || H % kRgK) return 1;
    const int tiles = ((E + kRgExp - 1) / kRgExp) * ((n + kRgTok - 1) / kRgTok);
    int S = 1;  // about four CTAs per SM of 148, each K range a whole number of slices
    while (S < 8 && tiles * S * 2 <= 148 * 5 && H % (2 * S * kRgK) == 0) S *= 2;
    return S;
}

int router_splits(int n, int H, int E) {
    const int tc = router_tc_nb(E, H) ? router_tc_splits(n, H) : 1;
    return max(router_gemm_splits(n, H, E), tc);
}

constexpr int kRouterTcMinTokens = 256;

cudaError_t launch_router(const RouterArgs& a, cudaStream_t st, bool pdl) {
    if (a.H % 4 || a.H > 4 * 256 * kRouterMaxVec) return cudaErrorInvalidValue;
    if (a.n >= kRouterTcMinTokens && a.x_bf16 && a.wsplit && a.wsplit_nb > 0 && a.status &&
        reinterpret_cast<uintptr_t>(a.x) % 16 == 0) {
        // bf16 activations: tensor cores on the exactly split weights
        int S = router_tc_splits(a.n, a.H);
        if (S > 1 && (!a.split_scratch || a.split_floats < (size_t)S * a.n * a.E)) S = 1;
        cudaError_t e = launch_router_tc(a, S, S > 1 ? a.split_scratch : a.logits, st, pdl);
        if (e != cudaSuccess || S == 1) return e;
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg2 = make_cfg(dim3(148 * 4), dim3(256), 0, st, pdl, attr);
        return cudaLaunchKernelEx(&cfg2, router_split_sum_kernel, a, S);
    }
    if (a.n >= 64 && a.H % kRgK == 0) {
        int S = router_gemm_splits(a.n, a.H, a.E);
        if (S > 1 && (!a.split_scratch || a.split_floats < (size_t)S * a.n * a.E)) S = 1;
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = make_cfg(dim3((a.E + kRgExp - 1) / kRgExp, (a.n + kRgTok - 1) / kRgTok, S),
                                          dim3(256), 0, st, pdl, attr);
        cudaError_t e = cudaLaunchKernelEx(&cfg, router_gemm_kernel, a);
        if (e != cudaSuccess || S == 1) return e;
        cudaLaunchConfig_t cfg2 = make_cfg(dim3(148 * 4), dim3(256), 0, st, pdl, attr);
        return cudaLaunchKernelEx(&cfg2, router_split_sum_kernel, a, S);
    }
    const int ntc = (a.n + kRouterTok - 1) / kRouterTok;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(a.E, ntc), dim3(32 * kRouterWarps), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, router_kernel, a);
}

size_t route_chunk_ints(int n, int K, int E) { return route_chunk_ints_impl(n, K, E); }

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st, bool pdl) {
    if (a.E > kMaxE || a.K > 32 || a.K > a.E || a.nt < 1) return cudaErrorInvalidValue;
    const size_t need = route_chunk_ints_impl(a.n, a.K, a.E);
    if (need && a.chunk_counts && a.chunk_cap >= need) {
        // large batches: top-k on many CTAs (unless given), then the chunked stable sort
        cudaLaunchAttribute attr[1];
        RouteArgs b = a;
        if (!a.topk_ready) {
            cudaLaunchConfig_t cfg = make_cfg(dim3(min(1184, (a.n + 7) / 8)), dim3(256), 0, st, pdl, attr);
            cudaError_t e = cudaLaunchKernelEx(&cfg, topk_kernel, a);
            if (e != cudaSuccess) return e;
            b.topk_ready = 1;
        }
        const int nchunks = (a.n * a.K + kChunk - 1) / kChunk;
        cudaLaunchConfig_t c1 = make_cfg(dim3(min(nchunks, 148 * 4)), dim3(256), 0, st, pdl, attr);
        cudaError_t e = cudaLaunchKernelEx(&c1, route_hist_kernel, b, nchunks);
        if (e != cudaSuccess) return e;
        route_scan_kernel<<<1, kRouteThreads, 0, st>>>(b, nchunks);
        route_scatter_kernel<<<(nchunks + 7) / 8, 256, 0, st>>>(b, nchunks);
        return cudaGetLastError();
    }
    const size_t smem = route_smem_bytes(a.n, a.E, a.K);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static std::atomic<unsigned long long> configured{0};  // per device: the limit is always 200 KB
    if (smem > 48 * 1024) {
        cudaError_t e = raise_smem_limit(route_kernel, 200 * 1024, configured);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchAttribute attr[1];
    RouteArgs b = a;
    if (a.n > 64 && !a.topk_ready) {  // large batches: top-k on many CTAs first
        cudaLaunchConfig_t cfg = make_cfg(dim3(min(1184, (a.n + 7) / 8)), dim3(256), 0, st, pdl, attr);
        cudaError_t e = cudaLaunchKernelEx(&cfg, topk_kernel, a);
        if (e != cudaSuccess) return e;
        b.topk_ready = 1;
    }
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(kRouteThreads), smem, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, route_kernel, b);
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st, bool pdl) {
    if (a.H % 4 || a.K > kCombineMaxK) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3((a.H / 4 + kCombineThreads - 1) / kCombineThreads, a.n),
                                      dim3(kCombineThreads), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, combine_kernel, a);
}

}  // namespace gp
