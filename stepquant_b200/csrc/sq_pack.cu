// packing.pack / packing.unpack (stepquant/packing.py:6-22) on the device:
// little-endian streams of n = 8/gcd(b,8) codes in n*b/8 bytes (also for the
// 3- and 5-bit widths of this build's extension).
#include <cuda_runtime.h>

#include "sq_common.cuh"

namespace sq {

// n = 8 / gcd(b, 8) codes in n b / 8 bytes: 4 in 1 (2 bits), 2 in 1 (4), 4 in 3
// (6), 1 in 1 (8); the width extension's 3 and 5 bits: 8 codes in 3 or 5 bytes
// (a group of up to 40 bits, accumulated in 64 bits).
__host__ __device__ inline int codes_per_group(int bits) { return bits == 6 ? 4 : (bits & 1) ? 8 : 8 / bits; }
__host__ __device__ inline int bytes_per_group(int bits) { return bits == 6 ? 3 : (bits & 1) ? bits : 1; }

__global__ void pack_kernel(const int16_t *codes, int64_t n, int bits, uint8_t *out, int64_t groups) {
    const int per = codes_per_group(bits), width = bytes_per_group(bits);
    for (int64_t g = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
        uint64_t word = 0;
        for (int i = 0; i < per; ++i) {
            const int64_t idx = g * per + i;
            const uint64_t c = idx < n ? uint64_t(uint16_t(codes[idx])) : 0u;
            word += c << (i * bits);
        }
        for (int j = 0; j < width; ++j) out[g * width + j] = uint8_t((word >> (8 * j)) & 0xffu);
    }
}

__global__ void unpack_kernel(const uint8_t *data, int64_t count, int bits, int16_t *out, int64_t groups) {
    const int per = codes_per_group(bits), width = bytes_per_group(bits);
    for (int64_t g = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
        uint64_t word = 0;
        for (int j = 0; j < width; ++j) word |= uint64_t(data[g * width + j]) << (8 * j);
        for (int i = 0; i < per; ++i) {
            const int64_t idx = g * per + i;
            if (idx < count) out[idx] = int16_t((word >> (i * bits)) & ((1u << bits) - 1u));
        }
    }
}

int64_t packed_bytes(int64_t n, int bits) {
    const int per = codes_per_group(bits);
    return (n + per - 1) / per * bytes_per_group(bits);
}

cudaError_t launch_pack(const int16_t *codes, int64_t n, int bits, uint8_t *out, cudaStream_t stream) {
    const int64_t groups = (n + codes_per_group(bits) - 1) / codes_per_group(bits);
    if (groups == 0) return cudaSuccess;
    const int blocks = int(groups < 4096 * 256 ? (groups + 255) / 256 : 4096);
    pack_kernel<<<blocks, 256, 0, stream>>>(codes, n, bits, out, groups);
    return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t *data, int64_t count, int bits, int16_t *out, cudaStream_t stream) {
    const int64_t groups = (count + codes_per_group(bits) - 1) / codes_per_group(bits);
    if (groups == 0) return cudaSuccess;
    const int blocks = int(groups < 4096 * 256 ? (groups + 255) / 256 : 4096);
    unpack_kernel<<<blocks, 256, 0, stream>>>(data, count, bits, out, groups);
    return cudaGetLastError();
}

}  // namespace sq
