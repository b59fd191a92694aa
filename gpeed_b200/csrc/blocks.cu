// Block-level IQ3_XXS kernels: the lossless raw <-> repacked layout
// conversion used for library-owned weights, the decode-table image, and the
// device side of the synthetic generator.  (The bit-exact fp32 dequantizer,
// quant.cpp:186-210 / :521-573, is the IQ3_XXS case of codecs.cu.)
#include <cuda_fp16.h>

#include "iq3xxs.cuh"
#include "kernels.h"
#include "synth.h"

namespace gp {
namespace {

// raw row-major blocks -> row groups of 8: [qs 8 x nblk x 64][aux 8 x nblk x 32][d 8 x nblk x 2]
// One thread per (row, block); rows past `rows` in the last group are zero-filled.
__global__ void repack_kernel(uint8_t* __restrict__ raw, uint8_t* __restrict__ out, int64_t rows, int nblk,
                              bool unpack) {
    const int64_t rows_pad = (rows + 7) / 8 * 8;
    const int64_t total = rows_pad * nblk;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / nblk;
        const int b = (int)(i % nblk);
        const int64_t grp = row / 8;
        const int ri = (int)(row % 8);
        uint8_t* g = out + grp * 784 * nblk;
        uint8_t* qs = g + (ri * nblk + b) * 64;
        uint8_t* ax = g + 512 * nblk + (ri * nblk + b) * 32;
        uint8_t* dd = g + 768 * nblk + (ri * nblk + b) * 2;
        if (!unpack) {
            if (row < rows) {
                const uint8_t* s = raw + (row * nblk + b) * 98;
                dd[0] = s[0];
                dd[1] = s[1];
                for (int j = 0; j < 64; ++j) qs[j] = s[2 + j];
                for (int j = 0; j < 32; ++j) ax[j] = s[66 + j];
            } else {
                dd[0] = dd[1] = 0;
                for (int j = 0; j < 64; ++j) qs[j] = 0;
                for (int j = 0; j < 32; ++j) ax[j] = 0;
            }
        } else if (row < rows) {
            uint8_t* s = raw + (row * nblk + b) * 98;  // raw is the destination when unpacking
            s[0] = dd[0];
            s[1] = dd[1];
            for (int j = 0; j < 64; ++j) s[2 + j] = qs[j];
            for (int j = 0; j < 32; ++j) s[66 + j] = ax[j];
        }
    }
}

// raw row-major blocks of n_mat matrices (rows x nblk blocks each) -> the
// column-slab layout the persistent decode kernel streams the down projection
// from (kernels.h, repacked_cols).  One thread per (matrix, row, block).
__global__ void repack_cols_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ out, int64_t n_mat,
                                   int rows, int nblk) {
    const int64_t total = n_mat * rows * nblk;
    const int64_t unit = (int64_t)rows * 12, mat = (int64_t)rows * nblk * 98;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / ((int64_t)rows * nblk);
        const int r = (int)((i / nblk) % rows);
        const int b = (int)(i % nblk);
        const uint8_t* s = raw + i * 98;
        uint8_t* base = out + m * mat;
        for (int ib = 0; ib < 8; ++ib) {
            uint8_t* u = base + (int64_t)(8 * b + ib) * unit;
            for (int j = 0; j < 8; ++j) u[(int64_t)r * 8 + j] = s[2 + 8 * ib + j];
            for (int j = 0; j < 4; ++j) u[(int64_t)rows * 8 + (int64_t)r * 4 + j] = s[66 + 4 * ib + j];
        }
        uint8_t* d = base + (int64_t)8 * nblk * unit + (int64_t)b * rows * 2 + (int64_t)r * 2;
        d[0] = s[0];
        d[1] = s[1];
    }
}

__global__ void tables_kernel(uint8_t* dst) {
    iq3_build_tables(dst, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// 128 blocks per CTA, generated into shared memory, written out with 16-byte stores
// when the destination run is 16-byte aligned (it is for block0 % 8 == 0).
__global__ void synth_kernel(uint8_t* __restrict__ dst, uint64_t seed, uint64_t stream, uint64_t block0,
                             int64_t nblocks) {
    __shared__ __align__(16) uint8_t s_buf[128 * 98];
    for (int64_t base = (int64_t)blockIdx.x * 128; base < nblocks; base += (int64_t)gridDim.x * 128) {
        const int nb = (int)gp_min64(128, nblocks - base);
        if ((int)threadIdx.x < nb) gp_synth_iq3xxs_block(seed, stream, block0 + base + threadIdx.x, s_buf + threadIdx.x * 98);
        __syncthreads();
        uint8_t* out = dst + base * 98;
        const int bytes = nb * 98;
        if ((reinterpret_cast<uintptr_t>(out) & 15) == 0 && (bytes & 15) == 0) {
            for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x)
                reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(s_buf)[i];
        } else {
            for (int i = threadIdx.x; i < bytes; i += blockDim.x) out[i] = s_buf[i];
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_dequantize(const uint8_t* raw, float* dst, int64_t nblocks, cudaStream_t st) {
    return launch_codec_dequantize(18, raw, dst, nblocks * 256, st);  // codecs.cu
}

cudaError_t launch_repack(const uint8_t* raw, uint8_t* packed, int64_t rows, int in_dim, cudaStream_t st) {
    const int nblk = in_dim / 256;
    const int64_t total = (rows + 7) / 8 * 8 * nblk;
    if (total == 0) return cudaSuccess;
    const int grid = (int)gp_min64((total + 255) / 256, 148 * 32);
    repack_kernel<<<grid, 256, 0, st>>>(const_cast<uint8_t*>(raw), packed, rows, nblk, false);
    return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t* packed, uint8_t* raw, int64_t rows, int in_dim, cudaStream_t st) {
    const int nblk = in_dim / 256;
    const int64_t total = (rows + 7) / 8 * 8 * nblk;
    if (total == 0) return cudaSuccess;
    const int grid = (int)gp_min64((total + 255) / 256, 148 * 32);
    repack_kernel<<<grid, 256, 0, st>>>(raw, const_cast<uint8_t*>(packed), rows, nblk, true);
    return cudaGetLastError();
}

cudaError_t launch_repack_cols(const uint8_t* raw, uint8_t* cols, int64_t n_mat, int rows, int in_dim,
                               cudaStream_t st) {
    const int nblk = in_dim / 256;
    const int64_t total = n_mat * rows * nblk;
    if (total == 0) return cudaSuccess;
    const int grid = (int)gp_min64((total + 255) / 256, 148 * 32);
    repack_cols_kernel<<<grid, 256, 0, st>>>(raw, cols, n_mat, rows, nblk);
    return cudaGetLastError();
}

cudaError_t build_tables(uint8_t* dst, cudaStream_t st) {
    tables_kernel<<<64, 256, 0, st>>>(dst);
    return cudaGetLastError();
}

cudaError_t launch_synth(uint8_t* dst, uint64_t seed, uint64_t stream, uint64_t block0, int64_t nblocks,
                         cudaStream_t st) {
    if (nblocks <= 0) return cudaSuccess;
    const int grid = (int)gp_min64((nblocks + 127) / 128, 148 * 64);
    synth_kernel<<<grid, 128, 0, st>>>(dst, seed, stream, block0, nblocks);
    return cudaGetLastError();
}

}  // namespace gp
