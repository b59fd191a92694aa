// Device helpers shared by the expert kernels (gemv.cu, decode_layer.cu):
// activation loading, the reference's clamped SwiGLU, and a warp reduction
// that sums many per-lane values with shared shuffles.
#pragma once
#include <cuda_bf16.h>

#include "common.cuh"

namespace gp {

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

// The same, for results rounded to fp16 right after (the tensor-core path's h):
// hardware exp2 and reciprocal approximations, a few fp32 ulps, far below the
// fp16 rounding that follows.
GP_DEVINL __half silu_clamped_h(float g, float u, float lim, bool& over) {
    const float gi = fminf(g, lim);
    const float ui = fminf(fmaxf(u, -lim), lim);
    const float h = __fdividef(gi, 1.0f + __expf(-gi)) * ui;
    over |= fabsf(h) >= 65520.0f;  // rounds to an fp16 infinity
    return __float2half_rn(h);
}

// Sum of M per-lane values across the warp, sharing shuffles between values:
// each butterfly level keeps half of the remaining values (the half picked by
// the lane bit) and adds the partner's other half.  Afterwards lane l holds
// the warp total of value index (l >> (5 - log2 M)).  M <= 32, a power of 2.
template <int M>
GP_DEVINL float warp_reduce_many(float (&v)[M], int lane) {
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
        const int o = 16 >> lvl;
        const int m = (M >> lvl) > 1 ? (M >> lvl) : 1;  // values still held
        if (m > 1) {
            const bool up = lane & o;
#pragma unroll
            for (int i = 0; i < m / 2; ++i) {
                const float send = up ? v[i] : v[i + m / 2];
                const float keep = up ? v[i + m / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

}  // namespace gp
