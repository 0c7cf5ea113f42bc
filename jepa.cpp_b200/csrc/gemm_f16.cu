// tcgen05 / TMEM / TMA GEMM for sm_100a in f16 (kind::f16, f32 accumulate): every dense product of the
// V-JEPA 2-AC predictor -- the context embedding, the fused q/k/v projection, the attention output, the
// MLP up / down projections and the output projection, over all candidates' rows at once.
//
// Persistent, one CTA per SM, 10 warps: warp 0 issues TMA loads of 128 x 64 A and 256 x 64 B f16 tiles
// (128-byte swizzle) into a 4-stage mbarrier pipeline; one thread of warp 1 issues 4 x
// tcgen05.mma.kind::f16 (K = 16) per stage into one of two 128 x 256 f32 accumulators in TMEM; warps
// 2..9 read the other accumulator with tcgen05.ld (two warps per lane quadrant) and apply the fused
// epilogue while the next tile's products run:
//   AEPI_QKV      bias, 3-D RoPE on q and k from per-row cos / sin tables, q to its buffer, k and v into
//                 the frame's key / value cache slot (f16)
//   AEPI_ADD_F32  bias and the residual add into the f32 stream, with a row remap (the patch rows of a
//                 frame sit after its conditioning rows)
//   AEPI_GELU_F16 bias, GELU, f16
//   AEPI_F32      bias, f32 (with the remap)
// Every mbarrier wait is bounded (about two seconds): on a timeout the kernel raises an error flag,
// drains what it issued, frees its TMEM and returns.
#include "kernels.h"
#include "common.h"
#include "launch.h"
#include "tcgen05.cuh"
#include "kprof.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace jb {

namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;                 // 64 f16 = one 128-byte swizzle row
constexpr int STAGES = 4;

__device__ int g_f16_error = 0;

__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

__device__ __forceinline__ void store_h8(__half * p, const float * v) {
    __align__(16) __half h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __float2half_rn(v[i]);
    *(uint4 *) p = *(const uint4 *) h;
}

// 32 consecutive columns [col0, col0 + 32) of one output row
__device__ __forceinline__ void epilogue32(const AcGemmEpi & ep, int row, int col0, int N, float (&v)[32]) {
    if (ep.bias) {
#pragma unroll
        for (int j = 0; j < 32; j++) if (col0 + j < N) v[j] = v[j] + ep.bias[col0 + j];
    }
    const bool full = col0 + 32 <= N;
    switch (ep.mode) {
        case AEPI_F32:
        case AEPI_ADD_F32: {
            const int orow = ep.remap_g ? (row / ep.remap_g) * ep.remap_gout + ep.remap_off + row % ep.remap_g : row;
            float * o = ep.out_f32 + (size_t) orow * ep.ld_f32 + col0;
            if (full) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    if (ep.mode == AEPI_ADD_F32) {
                        const float4 r = *(const float4 *) (o + j);
                        x = make_float4(r.x + x.x, r.y + x.y, r.z + x.z, r.w + x.w);
                    }
                    *(float4 *) (o + j) = x;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    if (col0 + j < N) o[j] = ep.mode == AEPI_ADD_F32 ? o[j] + v[j] : v[j];
                }
            }
        } break;
        case AEPI_GELU_F16: {
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = gelu_f(v[j]);
            __half * o = ep.out_f16 + (size_t) row * ep.ld_f16 + col0;
            if (full) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) store_h8(o + j, v + j);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    if (col0 + j < N) o[j] = __float2half_rn(v[j]);
                }
            }
        } break;
        case AEPI_QKV: {
            const int D = ep.D;
            if (col0 < 2 * D) {
                // 3-D RoPE: out = x * C + swap(x) * S', pairs (2k, 2k+1) are adjacent columns of one head
                const int lane0 = col0 % ep.hd;
                const float * c = ep.rope_cos + (size_t) (row % ep.rope_rows) * ep.hd;
                const float * s = ep.rope_sin + (size_t) (row % ep.rope_rows) * ep.hd;
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    int l = lane0 + j;
                    while (l >= ep.hd) l -= ep.hd;        // heads narrower than 32 columns wrap inside the chunk
                    const float x0 = v[j], x1 = v[j + 1];
                    v[j] = x0 * c[l] + x1 * s[l];
                    v[j + 1] = x1 * c[l + 1] + x0 * s[l + 1];
                }
            }
            __half * o = col0 < D ? ep.out_f16 + (size_t) row * ep.ld_f16 + col0
                                  : ep.kv + (size_t) row * ep.ld_kv + (col0 - D);
#pragma unroll
            for (int j = 0; j < 32; j += 8) store_h8(o + j, v + j);
        } break;
        default: break;
    }
}

constexpr int EPI_WARPS = 8;                       // two per TMEM lane quadrant, 128 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;

// Persistent: one CTA per SM walks the tiles (n fastest, so neighbouring CTAs share the A rows). Two
// TMEM accumulators of 256 columns: the epilogue of tile i reads one while the MMA warp fills the other
// with tile i+1.
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_f16(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB, int M, int N, int K, AcGemmEpi ep) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    // instruction descriptor: D f32 (bit 4), A / B f16 (format 0), K-major both, N >> 3, M >> 4
    constexpr uint32_t IDESC = (1u << 4) | ((uint32_t) (BN >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);

    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t accf_bar[2];      // MMA -> epilogue: accumulator b holds a finished tile
    __shared__ __align__(8) uint64_t acce_bar[2];      // epilogue -> MMA: accumulator b has been read
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_k = (K + BK - 1) / BK;
    const int tiles_n = (N + BN - 1) / BN;
    const int total = ((M + BM - 1) / BM) * tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&accf_bar[b], 1); mbar_init(&acce_bar[b], EPI_WARPS); }
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base_sh)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tA) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tB) : "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_sh;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        if (lane == 0) {
            int kt = 0;
            for (int t = blockIdx.x; t < total && !*(volatile int *) &abort_sh; t += gridDim.x) {
                const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
                for (int k = 0; k < num_k; k++, kt++) {
                    const int s = kt % STAGES;
                    const uint32_t ph = (uint32_t) (kt / STAGES) & 1u;
                    if (kt >= STAGES && !mbar_wait(&empty_bar[s], ph ^ 1u, 1, &g_f16_error)) { abort_sh = 1; break; }
                    if (*(volatile int *) &abort_sh) break;
                    uint8_t * st = smem + (size_t) s * STAGE_BYTES;
                    mbar_expect_tx(&full_bar[s], STAGE_BYTES);
                    tma_load_2d(st, &tA, k * BK, m0, &full_bar[s]);
                    tma_load_2d(st + A_BYTES, &tB, k * BK, n0, &full_bar[s]);
                }
            }
            if (*(volatile int *) &abort_sh) {
                // let the copies already issued land before the CTA exits
                for (int j = kt - STAGES < 0 ? 0 : kt - STAGES; j < kt; j++) {
                    mbar_wait(&full_bar[j % STAGES], (uint32_t) (j / STAGES) & 1u, 5, &g_f16_error);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int kt = 0, i = 0;
            for (int t = blockIdx.x; t < total && !*(volatile int *) &abort_sh; t += gridDim.x, i++) {
                const int b = i & 1;
                if (i >= 2 && !mbar_wait(&acce_bar[b], (uint32_t) ((i >> 1) - 1) & 1u, 4, &g_f16_error)) { abort_sh = 1; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t) (b * BN);
                for (int k = 0; k < num_k; k++, kt++) {
                    const int s = kt % STAGES;
                    const uint32_t ph = (uint32_t) (kt / STAGES) & 1u;
                    if (!mbar_wait(&full_bar[s], ph, 2, &g_f16_error)) { abort_sh = 1; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a = smem_u32(smem + (size_t) s * STAGE_BYTES), bb = a + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint32_t off = (uint32_t) kk * 32;   // 16 f16 = 32 bytes along K
                        mma_kind_f16(d, sw128_desc(a + off), sw128_desc(bb + off), IDESC, (k | kk) != 0);
                    }
                    mma_commit(&empty_bar[s]);
                }
                if (*(volatile int *) &abort_sh) break;
                mma_commit(&accf_bar[b]);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lane quadrant this warp may read
        const int half = (warp - 2) >> 2;       // which 128 of the 256 columns
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, i++) {
            const int b = i & 1;
            const bool ok = mbar_wait(&accf_bar[b], (uint32_t) (i >> 1) & 1u, 3, &g_f16_error);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (!ok || *(volatile int *) &abort_sh) { abort_sh = 1; break; }
            const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
            const int row = m0 + q * 32 + lane;
#pragma unroll 1
            for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (b * BN + c0), r);
                if (row < M && n0 + c0 < N) {
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                    epilogue32(ep, row, n0 + c0, N, v);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce_bar[b]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

int g_num_sms = 0;

PFN_cuTensorMapEncodeTiled_v12000 g_encode16 = nullptr;
std::once_flag g_encode16_once;

bool make_map16(CUtensorMap * map, const __half * base, int rows, int cols, int ld, int box_rows) {
    std::call_once(g_encode16_once, []() {
        void * fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode16 = (PFN_cuTensorMapEncodeTiled_v12000) fn;
        }
    });
    if (!g_encode16) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t) BK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode16(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *) base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int gemm_f16(const __half * A, int lda, const __half * B, int ldb, int M, int N, int K, const AcGemmEpi & ep, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    if ((lda & 7) || (ldb & 7) || ((uintptr_t) A & 15) || ((uintptr_t) B & 15)) {
        log("jepa: gemm_f16: operands need 16-byte aligned rows (ld %d / %d)\n", lda, ldb);
        return -1;
    }
    if ((ep.mode == AEPI_QKV && (ep.D % 32 || ep.hd % 2 || ep.hd < 2 || N != 3 * ep.D || (ep.ld_f16 & 7) || (ep.ld_kv & 7))) ||
        (ep.mode == AEPI_GELU_F16 && (ep.ld_f16 & 7)) || ((ep.mode == AEPI_F32 || ep.mode == AEPI_ADD_F32) && (ep.ld_f32 & 3))) {
        log("jepa: gemm_f16: epilogue operands need vector-aligned rows\n");
        return -1;
    }
    CUtensorMap ta, tb;
    if (!make_map16(&ta, A, M, K, lda, BM) || !make_map16(&tb, B, N, K, ldb, BN)) {
        log("jepa: gemm_f16: cuTensorMapEncodeTiled refused an operand (M %d N %d K %d)\n", M, N, K);
        return -1;
    }
    constexpr size_t smem = (size_t) STAGES * (BM * BK * 2 + BN * BK * 2) + 1024;
    static bool attr_set = false;
    if (!attr_set) {
        JB_CUDA(cudaFuncSetAttribute(k_gemm_f16, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem));
        attr_set = true;
    }
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    const long long tiles = (long long) ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const dim3 grid((unsigned) (tiles < g_num_sms ? tiles : g_num_sms));
    KTimer kt("gemm_f16", st, 2.0 * M * N * K);
    JB_CUDA(launch_pdl(k_gemm_f16, grid, dim3(THREADS), smem, st, ta, tb, M, N, K, ep));
    return 0;
}

int gemm_f16_error_flag(cudaStream_t st) {
    int v = 0;
    cudaMemcpyFromSymbolAsync(&v, g_f16_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    return v;
}

}  // namespace jb
