// GGUF weight blocks -> float32 on the device, bit-exact with the block formats (the products d * q
// are exact in float32: an f16 scale has 11 significant bits, a q8_0 / q4_0 quant at most 8), and a
// tiled transpose used to build the backward (K = out) operand of every linear.
#include "kernels.h"
#include "common.h"

#include <cuda_fp16.h>

namespace jb {

namespace {

__device__ __forceinline__ float f16_bits_to_f32(const uint8_t * p) {
    const uint16_t h = (uint16_t) p[0] | ((uint16_t) p[1] << 8);
    return __half2float(__ushort_as_half(h));
}

// one thread per output element
__global__ void k_dequant(uint32_t type, const uint8_t * __restrict__ src, float * __restrict__ dst, int64_t n_total, int64_t ne0) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_total) return;
    const int64_t r = i / ne0, c = i % ne0;
    float v = 0.0f;
    switch (type) {
        case 0: v = ((const float *) src)[i]; break;                                  // f32
        case 1: v = f16_bits_to_f32(src + 2 * i); break;                               // f16
        case 30: v = __uint_as_float((uint32_t) (src[2 * i] | (src[2 * i + 1] << 8)) << 16); break;   // bf16
        case 8: {                                                                      // q8_0
            const uint8_t * blk = src + (r * (ne0 / 32) + c / 32) * 34;
            v = f16_bits_to_f32(blk) * (float) (int8_t) blk[2 + (c % 32)];
        } break;
        case 2: {                                                                      // q4_0
            const uint8_t * blk = src + (r * (ne0 / 32) + c / 32) * 18;
            const int j = (int) (c % 32);
            const int q = j < 16 ? (blk[2 + j] & 0x0f) : (blk[2 + j - 16] >> 4);
            v = (float) (q - 8) * f16_bits_to_f32(blk);
        } break;
        default: break;
    }
    dst[i] = v;
}

__global__ void k_transpose(const float * __restrict__ src, float * __restrict__ dst, int rows, int cols) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = src[(size_t) r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int c = bx + j, r = by + threadIdx.x;
        if (r < rows && c < cols) dst[(size_t) c * rows + r] = tile[threadIdx.x][j];
    }
}

}  // namespace

int dequant_rows(uint32_t type, const void * src, float * dst, int64_t rows, int64_t ne0, cudaStream_t st) {
    if (type != 0 && type != 1 && type != 2 && type != 8 && type != 30) {
        log("jepa: dequant: unsupported ggml type %u\n", type);
        return -1;
    }
    if ((type == 2 || type == 8) && ne0 % 32 != 0) {
        log("jepa: dequant: a block-quantised row must hold a whole number of 32-value blocks (ne0 = %lld)\n", (long long) ne0);
        return -1;
    }
    const int64_t n = rows * ne0;
    if (n <= 0) return 0;
    k_dequant<<<(unsigned) ((n + 255) / 256), 256, 0, st>>>(type, (const uint8_t *) src, dst, n, ne0);
    JB_CUDA(cudaGetLastError());
    return 0;
}

void transpose_f32(const float * src, float * dst, int rows, int cols, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return;
    const dim3 grid((unsigned) ((cols + 31) / 32), (unsigned) ((rows + 31) / 32));
    k_transpose<<<grid, dim3(32, 8), 0, st>>>(src, dst, rows, cols);
}

}  // namespace jb
