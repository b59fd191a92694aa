// Device helpers of the expert-parallel layer: id remapping and the dispatch
// pack.  The exchange itself runs over NCCL (torch.distributed) on the host
// side; these kernels prepare and consume its buffers.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace gp {
namespace {

__global__ void local_ids_kernel(const int* ids, int m, int E, int lo, int cnt, int* local, float* ones,
                                 uint32_t* status) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) {
        const int e = ids[i];
        int l;
        if (e == E) l = cnt;                         // the shared expert
        else if (e >= lo && e < lo + cnt) l = e - lo;
        else { atomicOr(status, GP_DEV_BAD_EXPERT); l = 0; }
        local[i] = l;
        ones[i] = 1.0f;
    }
}

// One CTA per assignment: copies its token's row to the send position.
__global__ void ep_pack_kernel(const void* x, int x_bf16, int H, int K, const int* ids, const int* pos,
                               void* send_rows, int* send_ids) {
    const int i = blockIdx.x, t = i / K, p = pos[i];
    const int row_bytes = H * (x_bf16 ? 2 : 4);
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + (int64_t)t * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(send_rows) + (int64_t)p * row_bytes);
    for (int q = threadIdx.x; q < row_bytes / 16; q += blockDim.x) dst[q] = src[q];
    if (threadIdx.x == 0) send_ids[p] = ids[i];
}

__global__ void rank_counts_kernel(const int* counts, int E, int world, int epr, int* rank_counts) {
    const int r = threadIdx.x;
    if (r >= world) return;
    int c = 0;
    for (int e = r * epr; e < (r + 1) * epr && e < E; ++e) c += counts[e];
    rank_counts[r] = c;
}

}  // namespace

cudaError_t launch_local_ids(const int* ids, int m, int E, int lo, int cnt, int* local, float* ones,
                             uint32_t* status, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    local_ids_kernel<<<(m + 255) / 256, 256, 0, st>>>(ids, m, E, lo, cnt, local, ones, status);
    return cudaGetLastError();
}

cudaError_t launch_ep_pack(const void* x, int x_bf16, int H, int n, int K, const int* ids, const int* pos,
                           const int* counts, int E, int world, int epr, void* send_rows, int* send_ids,
                           int* rank_counts, cudaStream_t st) {
    if (n * K > 0) ep_pack_kernel<<<n * K, 128, 0, st>>>(x, x_bf16, H, K, ids, pos, send_rows, send_ids);
    rank_counts_kernel<<<1, 32, 0, st>>>(counts, E, world, epr, rank_counts);
    return cudaGetLastError();
}

}  // namespace gp
