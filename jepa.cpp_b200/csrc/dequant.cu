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

// q8_0 / q4_0 rows -> the GEMM's block planes: one thread per (pair of rows, 32-value block). It reads the
// two rows' blocks and writes their scales d[b][r], their forward values (row r, columns 32 b ..) and their
// transposed values (rows 32 b .., column r: a pair of int8, or one byte of two nibbles, per column).
__global__ void k_quant_planes(uint32_t type, const uint8_t * __restrict__ src, int64_t rows, int64_t ne0,
                               uint8_t * __restrict__ q, uint8_t * __restrict__ qt, uint16_t * __restrict__ d) {
    const int64_t nb = ne0 / 32, pairs = rows / 2;
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb * pairs) return;
    const int64_t b = i / pairs, rp = i % pairs;
    const int bs = type == 8 ? 34 : 18;
    uint8_t v[2][32];   // the two rows' 32 values: int8 (q8_0) or the 4-bit value (q4_0)
    for (int h = 0; h < 2; h++) {
        const int64_t r = 2 * rp + h;
        const uint8_t * blk = src + (r * nb + b) * bs;
        d[b * rows + r] = (uint16_t) (blk[0] | (blk[1] << 8));
        for (int j = 0; j < 32; j++) {
            v[h][j] = type == 8 ? blk[2 + j] : (uint8_t) (j < 16 ? (blk[2 + j] & 0x0f) : (blk[2 + j - 16] >> 4));
        }
        if (type == 8) {
            for (int j = 0; j < 32; j++) q[r * ne0 + b * 32 + j] = v[h][j];
        } else {
            for (int m = 0; m < 16; m++) q[r * (ne0 / 2) + b * 16 + m] = (uint8_t) (v[h][2 * m] | (v[h][2 * m + 1] << 4));
        }
    }
    for (int j = 0; j < 32; j++) {
        const int64_t c = b * 32 + j;   // the transposed operand's row
        if (type == 8) {
            *(uint16_t *) (qt + c * rows + 2 * rp) = (uint16_t) (v[0][j] | (v[1][j] << 8));
        } else {
            qt[c * (rows / 2) + rp] = (uint8_t) (v[0][j] | (v[1][j] << 4));
        }
    }
}

__global__ void k_transpose_u16(const uint16_t * __restrict__ src, uint16_t * __restrict__ dst, int rows, int cols) {
    __shared__ uint16_t tile[32][34];
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

bool quant_ok(uint32_t type, int64_t rows, int64_t ne0) {
    return (type == 8 || type == 2 || type == 1) && rows >= 32 && ne0 >= 32 && rows % 32 == 0 && ne0 % 32 == 0;
}

size_t quant_plane_bytes(uint32_t type, int64_t rows, int64_t ne0) {
    const size_t n = (size_t) rows * (size_t) ne0;
    return type == 8 ? n : type == 2 ? n / 2 : type == 1 ? 2 * n : 0;
}

size_t quant_scale_count(uint32_t type, int64_t rows, int64_t ne0) {
    return type == 8 || type == 2 ? (size_t) rows * (size_t) (ne0 / 32) : 0;
}

int quant_planes(uint32_t type, const void * raw, int64_t rows, int64_t ne0, void * q, void * qt, uint16_t * d, cudaStream_t st) {
    if (!quant_ok(type, rows, ne0)) {
        log("jepa: block planes: type %u with %lld x %lld values is not supported\n", type, (long long) rows, (long long) ne0);
        return -1;
    }
    if (type == 1) {
        JB_CUDA(cudaMemcpyAsync(q, raw, quant_plane_bytes(type, rows, ne0), cudaMemcpyDeviceToDevice, st));
        const dim3 grid((unsigned) ((ne0 + 31) / 32), (unsigned) ((rows + 31) / 32));
        k_transpose_u16<<<grid, dim3(32, 8), 0, st>>>((const uint16_t *) raw, (uint16_t *) qt, (int) rows, (int) ne0);
    } else {
        const int64_t n = (ne0 / 32) * (rows / 2);
        k_quant_planes<<<(unsigned) ((n + 255) / 256), 256, 0, st>>>(type, (const uint8_t *) raw, rows, ne0, (uint8_t *) q,
                                                                        (uint8_t *) qt, d);
    }
    JB_CUDA(cudaGetLastError());
    return 0;
}

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
