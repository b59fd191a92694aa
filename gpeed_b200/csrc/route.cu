// Router, top-k routing and the weighted un-permute of the MoE layer.
//
//  router_kernel   fp32 router logits (reference model.cpp:41-46/702 for one
//                  token, model_batch.cpp:172 for a batch), split along K into
//                  nsplit chunks whose partial sums are added in a fixed order
//                  by route_kernel (deterministic, no atomics).
//  route_kernel    sigmoid scores, +correction bias, top-K by choice (ties to
//                  the lower expert id), weights score/(1e-20 + sum)*scale
//                  (model.cpp:704-725, model_batch.cpp:184-203), then the
//                  expert histogram, exclusive scan and stable expert-major
//                  permutation (model_batch.cpp:204-219), and the slot list
//                  (experts split into runs of <= nt assignments) consumed by
//                  the expert kernels.  One CTA; warp-level scans and ballots.
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
constexpr int kRouterTok = 8;   // tokens per warp task

// One warp task = (expert row e, K-chunk c, token chunk); lane-strided float4s.
__global__ void __launch_bounds__(32 * kRouterWarps) router_kernel(const RouterArgs a) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int task = blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
    const int ntc = (a.n + kRouterTok - 1) / kRouterTok;
    const int ntask = a.E * a.nsplit * ntc;
    if (task >= ntask) return;
    const int e = task % a.E;
    const int c = (task / a.E) % a.nsplit;
    const int tc = task / (a.E * a.nsplit);
    const int chunk = a.H / a.nsplit;       // multiple of 128
    const int k0 = c * chunk;
    const float* w = a.w + (int64_t)e * a.H + k0;
    float acc[kRouterTok];
#pragma unroll
    for (int t = 0; t < kRouterTok; ++t) acc[t] = 0.f;
    for (int k = lane * 4; k < chunk; k += 128) {
        const float4 wv = *reinterpret_cast<const float4*>(w + k);
#pragma unroll
        for (int t = 0; t < kRouterTok; ++t) {
            const int tok = tc * kRouterTok + t;
            if (tok >= a.n) break;
            float4 xv;
            if (a.x_bf16) {
                const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) +
                                                                (int64_t)tok * a.H + k0 + k);
                xv = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                 __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
            } else {
                xv = *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (int64_t)tok * a.H + k0 + k);
            }
            acc[t] = fmaf(wv.x, xv.x, acc[t]);
            acc[t] = fmaf(wv.y, xv.y, acc[t]);
            acc[t] = fmaf(wv.z, xv.z, acc[t]);
            acc[t] = fmaf(wv.w, xv.w, acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < kRouterTok; ++t) {
        const int tok = tc * kRouterTok + t;
        const float v = warp_sum(acc[t]);
        if (lane == 0 && tok < a.n) a.partial[((int64_t)c * a.n + tok) * a.E + e] = v;
    }
    pdl_launch_dependents();
}

constexpr int kRouteThreads = 1024;
constexpr int kMaxE = 512;

__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteArgs a) {
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
    for (int e = tid; e < E; e += kRouteThreads) s_cnt[e] = 0;
    __syncthreads();

    // 1. per token: logits -> scores -> top-K (warp per token)
    for (int t = warp; t < n; t += nwarp) {
        // each lane holds experts lane, lane+32, ...
        float score[kMaxE / 32], choice[kMaxE / 32];
#pragma unroll
        for (int j = 0; j < kMaxE / 32; ++j) {
            const int e = lane + 32 * j;
            score[j] = 0.f;
            choice[j] = -INFINITY;
            if (e < E) {
                float lg = 0.f;
                for (int c = 0; c < a.nsplit; ++c) lg += a.partial[((int64_t)c * n + t) * E + e];
                score[j] = 1.0f / (1.0f + expf(-lg));
                choice[j] = score[j] + (a.corr ? a.corr[e] : 0.f);
            }
        }
        int sel_e[32];
        float sel_s[32];
        float denom = 1e-20f;
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
            // fetch the score of e_best from its owner lane, retire it
            float sc = 0.f;
#pragma unroll
            for (int j = 0; j < kMaxE / 32; ++j)
                if (lane + 32 * j == e_best) { sc = score[j]; choice[j] = -INFINITY; }
            sc = __shfl_sync(0xffffffffu, sc, e_best & 31);
            sel_e[k] = e_best;
            sel_s[k] = sc;
            denom += sc;
        }
        if (lane == 0) {
            // model.cpp:718-725: w = score / denom (if norm) * scale
            for (int k = 0; k < K; ++k) {
                const float w = a.norm_topk ? (sel_s[k] / denom) * a.routed_scale : sel_s[k] * a.routed_scale;
                a.topk_ids[(int64_t)t * K + k] = sel_e[k];
                a.topk_w[(int64_t)t * K + k] = w;
                atomicAdd(&s_cnt[sel_e[k]], 1);
            }
        }
    }
    __syncthreads();

    // 2. exclusive scan of counts (single warp), and slot offsets per owned expert
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
    for (int e = tid; e < E; e += kRouteThreads) a.counts[e] = s_cnt[e];

    // 3. stable placement: warp per expert, ballot over tokens in order
    const int nk = n * K;
    for (int e = warp; e < E; e += nwarp) {
        int pos = s_ptr[e];
        for (int t0 = 0; t0 < n; t0 += 32) {
            const int t = t0 + lane;
            int kk = -1;
            if (t < n)
                for (int k = 0; k < K; ++k)
                    if (a.topk_ids[(int64_t)t * K + k] == e) { kk = k; break; }
            const unsigned m = __ballot_sync(0xffffffffu, kk >= 0);
            if (kk >= 0) {
                const int p = pos + __popc(m & ((1u << lane) - 1u));
                a.perm_tok[p] = t;
                a.inv_pos[(int64_t)t * K + kk] = p;
            }
            pos += __popc(m);
        }
        // slots for this expert (only owned experts)
        if (e >= a.expert_lo && e < a.expert_hi) {
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
    }
    // 4. shared expert: assignments nk .. nk+n-1 are tokens 0..n-1
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

__global__ void combine_kernel(const CombineArgs a) {
    pdl_wait();
    const int t = blockIdx.y;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (j >= a.H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < a.K; ++k) {
        const float w = a.topk_w[(int64_t)t * a.K + k];
        const int p = a.inv_pos[(int64_t)t * a.K + k];
        const float4 d = *reinterpret_cast<const float4*>(a.D + (int64_t)p * a.H + j);
        acc.x = fmaf(w, d.x, acc.x);
        acc.y = fmaf(w, d.y, acc.y);
        acc.z = fmaf(w, d.z, acc.z);
        acc.w = fmaf(w, d.w, acc.w);
    }
    if (a.with_shared) {
        const float4 d = *reinterpret_cast<const float4*>(a.D + ((int64_t)a.n * a.K + t) * a.H + j);
        acc.x += d.x;
        acc.y += d.y;
        acc.z += d.z;
        acc.w += d.w;
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

cudaError_t launch_router(const RouterArgs& a, cudaStream_t st, bool pdl) {
    if (a.H % (128 * a.nsplit)) return cudaErrorInvalidValue;
    const int ntc = (a.n + kRouterTok - 1) / kRouterTok;
    const int ntask = a.E * a.nsplit * ntc;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg =
        make_cfg(dim3((ntask + kRouterWarps - 1) / kRouterWarps), dim3(32 * kRouterWarps), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, router_kernel, a);
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st, bool pdl) {
    if (a.E > kMaxE || a.K > 32 || a.K > a.E || a.nt < 1) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(kRouteThreads), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, route_kernel, a);
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st, bool pdl) {
    if (a.H % 4) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3((a.H / 4 + 127) / 128, a.n), dim3(128), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, combine_kernel, a);
}

}  // namespace gp
