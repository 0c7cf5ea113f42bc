// tcgen05 / TMEM / TMA GEMM for sm_100a in f16 (kind::f16, f32 accumulate): every dense product of the
// V-JEPA 2-AC predictor -- the context embedding, the fused q/k/v projection, the attention output, the
// MLP up / down projections and the output projection, over all candidates' rows at once.
//
// Persistent, one CTA per SM, 10 warps: warp 0 issues TMA loads of 128 x 64 A and 256 x 64 B f16 tiles
// (128-byte swizzle) into a 4-stage mbarrier pipeline; one thread of warp 1 issues 4 x
// tcgen05.mma.kind::f16 (K = 16) per stage into one of two 128 x 256 f32 accumulators in TMEM; warps
// 2..9 read the other accumulator with tcgen05.ld (two warps per lane quadrant, 128 columns each) and
// apply the fused epilogue while the next tile's products run:
//   AEPI_QKV      bias, 3-D RoPE on q and k from per-axis cos / sin tables, q to its buffer, k and v into
//                 the frame's key / value cache slot (f16)
//   AEPI_ADD_F32  bias, then a TMA reduce-add into the f32 residual stream (the add happens in L2)
//   AEPI_GELU_F16 bias, GELU, f16
//   AEPI_F32      bias, f32, with a row remap (the patch rows of a frame sit after its conditioning rows)
// Each warp stages a 32 x 32 block in its own 128-byte-swizzled (f32) / 64-byte-swizzled (f16) shared
// buffer and one lane issues the TMA store, so the global writes are whole coalesced lines issued by the
// copy engine. Row remaps whose groups are not 32-row aligned (small test models) fall back to direct
// per-row stores.
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
constexpr int EPI_WARPS = 8;           // two per TMEM lane quadrant, 128 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t STAGE_BYTES = (BM + BN) * BK * 2;
constexpr uint32_t EPI_BYTES = 32 * 32 * 4;                       // one warp's staging block
constexpr size_t SMEM_BYTES = (size_t) STAGES * STAGE_BYTES + (size_t) EPI_WARPS * EPI_BYTES + 1024;

__device__ int g_f16_error = 0;

__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

__device__ __forceinline__ void store_h8(__half * p, const float * v) {
    __align__(16) __half h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __float2half_rn(v[i]);
    *(uint4 *) p = *(const uint4 *) h;
}

__device__ __forceinline__ uint32_t pack2h(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t *) &h;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap * map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"((uint64_t) map), "r"(x), "r"(y), "r"(src) : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap * map, uint32_t src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"((uint64_t) map), "r"(x), "r"(y), "r"(src) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// bias, activation and RoPE on 32 consecutive columns [col0, col0 + 32) of one output row
__device__ __forceinline__ void epi_math(const AcGemmEpi & ep, int row, int col0, int N, float (&v)[32]) {
    if (ep.bias) {
#pragma unroll
        for (int j = 0; j < 32; j++) if (col0 + j < N) v[j] = v[j] + ep.bias[col0 + j];
    }
    if (ep.mode == AEPI_GELU_F16) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = gelu_f(v[j]);
    } else if (ep.mode == AEPI_QKV && col0 < 2 * ep.D && ep.rope_d > 0) {
        // 3-D RoPE: out = x * C + swap(x) * S', pairs (2k, 2k+1) are adjacent columns of one head; C and S
        // come from the per-axis tables (frame slot, grid row, grid column) of this row's position
        const int fr = row % (ep.rope_nf * ep.rope_frame_rows);
        const int slot = ep.rope_slot0 + fr / ep.rope_frame_rows;
        const int i = fr % ep.rope_frame_rows - ep.rope_cond;
        const int gh = i < 0 ? 0 : i / ep.rope_grid, gw = i < 0 ? 0 : i % ep.rope_grid;
        const int d = ep.rope_d;
        const int bt = slot * d, bh = (ep.rope_slots + gh) * d, bw = (ep.rope_slots + ep.rope_grid + gw) * d;
        int l = col0 % ep.hd;
        int ax = l / d, k = l % d;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            if (ax < 3) {
                const int o = (ax == 0 ? bt : ax == 1 ? bh : bw) + k;
                const float c0 = ep.rope_cos[o], c1 = ep.rope_cos[o + 1], s0 = ep.rope_sin[o], s1 = ep.rope_sin[o + 1];
                const float x0 = v[j], x1 = v[j + 1];
                v[j] = x0 * c0 + x1 * s0;
                v[j + 1] = x1 * c1 + x0 * s1;
            }
            // next pair: two lanes on, wrapping into the next axis and the next head
            l += 2;
            k += 2;
            if (l >= ep.hd) { l -= ep.hd; ax = 0; k = l; while (k >= d) { k -= d; ax++; } }
            else if (k >= d) { k -= d; ax++; }
        }
    }
}

__device__ __forceinline__ int remap_row(const AcGemmEpi & ep, int row) {
    return ep.remap_g ? (row / ep.remap_g) * ep.remap_gout + ep.remap_off + row % ep.remap_g : row;
}

// direct per-row stores (row remaps that are not 32-row aligned)
__device__ __forceinline__ void epi_store_direct(const AcGemmEpi & ep, int row, int col0, int N, const float (&v)[32]) {
    const bool full = col0 + 32 <= N;
    switch (ep.mode) {
        case AEPI_F32:
        case AEPI_ADD_F32: {
            float * o = ep.out_f32 + (size_t) remap_row(ep, row) * ep.ld_f32 + col0;
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
            __half * o = col0 < ep.D ? ep.out_f16 + (size_t) row * ep.ld_f16 + col0
                                     : ep.kv + (size_t) row * ep.ld_kv + (col0 - ep.D);
#pragma unroll
            for (int j = 0; j < 32; j += 8) store_h8(o + j, v + j);
        } break;
        default: break;
    }
}

// Persistent: one CTA per SM walks the tiles (n fastest, so neighbouring CTAs share the A rows). Two
// TMEM accumulators of 256 columns: the epilogue of tile i reads one while the MMA warp fills the other
// with tile i+1. tO: the f32 / f16 output (or q); tKV: the key / value cache (AEPI_QKV). tma_out = 0
// selects the direct-store epilogue.
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_f16(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
           const __grid_constant__ CUtensorMap tO, const __grid_constant__ CUtensorMap tKV,
           int M, int N, int K, AcGemmEpi ep, int tma_out) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
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
        if (tma_out) {
            asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tO) : "memory");
            if (ep.mode == AEPI_QKV) asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tKV) : "memory");
        }
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
        uint8_t * stage = smem + (size_t) STAGES * STAGE_BYTES + (size_t) (warp - 2) * EPI_BYTES;
        const uint32_t stage_u = smem_u32(stage);
        const bool f16_out = ep.mode == AEPI_GELU_F16 || ep.mode == AEPI_QKV;
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, i++) {
            const int b = i & 1;
            const bool ok = mbar_wait(&accf_bar[b], (uint32_t) (i >> 1) & 1u, 3, &g_f16_error);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (!ok || *(volatile int *) &abort_sh) { abort_sh = 1; break; }
            const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
            const int row0 = m0 + q * 32, row = row0 + lane;
#pragma unroll 1
            for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (b * BN + c0), r);
                const int col0 = n0 + c0;
                if (col0 >= N || row0 >= M) continue;          // warp-uniform
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                epi_math(ep, row, col0, N, v);
                if (!tma_out) {
                    if (row < M) epi_store_direct(ep, row, col0, N, v);
                    continue;
                }
                // f16 blocks (2 KB) alternate between the two halves of the staging buffer, so a block is
                // written while the previous one's store is still reading; an f32 block (4 KB) takes it whole
                const uint32_t half_off = f16_out ? (uint32_t) ((c0 >> 5) & 1) * 2048u : 0u;
                if (lane == 0) {
                    if (f16_out) bulk_wait_read1();   // the store that used this half (two blocks ago) has read it
                    else bulk_wait_read0();
                }
                __syncwarp();
                if (f16_out) {
                    // 32 rows x 64 B, 64-byte swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint4 u;
                        u.x = pack2h(v[8 * c + 0], v[8 * c + 1]);
                        u.y = pack2h(v[8 * c + 2], v[8 * c + 3]);
                        u.z = pack2h(v[8 * c + 4], v[8 * c + 5]);
                        u.w = pack2h(v[8 * c + 6], v[8 * c + 7]);
                        *(uint4 *) (stage + half_off + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) = u;
                    }
                } else {
                    // 32 rows x 128 B, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7)
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        *(float4 *) (stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    const uint32_t src = stage_u + half_off;
                    switch (ep.mode) {
                        case AEPI_ADD_F32: tma_reduce_add_2d(&tO, src, col0, row0); break;
                        case AEPI_F32: tma_store_2d(&tO, src, col0, remap_row(ep, row0)); break;
                        case AEPI_GELU_F16: tma_store_2d(&tO, src, col0, row0); break;
                        default:
                            if (col0 < ep.D) tma_store_2d(&tO, src, col0, row0);
                            else tma_store_2d(&tKV, src, col0 - ep.D, row0);
                            break;
                    }
                    bulk_commit();
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce_bar[b]);
        }
        if (tma_out && lane == 0) bulk_wait0();   // stores complete before the CTA exits
        __syncwarp();
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

bool encode(CUtensorMap * map, CUtensorMapDataType dt, size_t esize, const void * base, int rows, int cols, int ld,
            int box_cols, int box_rows, CUtensorMapSwizzle sw) {
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
    const cuuint64_t strides[1] = {(cuuint64_t) ld * esize};
    const cuuint32_t box[2] = {(cuuint32_t) box_cols, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode16(map, dt, 2, (void *) base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map16(CUtensorMap * map, const __half * base, int rows, int cols, int ld, int box_rows) {
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rows, cols, ld, BK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
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
    CUtensorMap ta, tb, to, tkv;
    if (!make_map16(&ta, A, M, K, lda, BM) || !make_map16(&tb, B, N, K, ldb, BN)) {
        log("jepa: gemm_f16: cuTensorMapEncodeTiled refused an operand (M %d N %d K %d)\n", M, N, K);
        return -1;
    }
    // output maps: 32 x 32 blocks at 32-aligned (column, row) coordinates; a row remap needs whole 32-row
    // groups, and rows past M must not exist in the mapped range (the copy engine clips only at its edges)
    int tma_out = 1;
    to = tkv = ta;
    bool mapped = true;
    switch (ep.mode) {
        case AEPI_F32:
        case AEPI_ADD_F32: {
            int rows_out = M;
            if (ep.remap_g) {
                if (ep.mode == AEPI_ADD_F32 || ep.remap_g % 32 || M % ep.remap_g) {
                    tma_out = 0;
                    break;
                }
                rows_out = (M / ep.remap_g - 1) * ep.remap_gout + ep.remap_off + ep.remap_g;
            }
            mapped = encode(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ep.out_f32, rows_out, N, ep.ld_f32, 32, 32,
                            CU_TENSOR_MAP_SWIZZLE_128B);
        } break;
        case AEPI_GELU_F16:
            mapped = encode(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ep.out_f16, M, N, ep.ld_f16, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
            break;
        case AEPI_QKV:
            mapped = encode(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ep.out_f16, M, ep.D, ep.ld_f16, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
                     encode(&tkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ep.kv, M, 2 * ep.D, ep.ld_kv, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
            break;
        default: tma_out = 0; break;
    }
    if (!mapped || ((uintptr_t) ep.out_f32 & 15) || ((uintptr_t) ep.out_f16 & 15) || ((uintptr_t) ep.kv & 15)) tma_out = 0;
    static bool attr_set = false;
    if (!attr_set) {
        JB_CUDA(cudaFuncSetAttribute(k_gemm_f16, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_BYTES));
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
    static const char * const kinds[] = {"gemm_f16", "gemm_f16_add", "gemm_f16_gelu", "gemm_f16_qkv"};
    KTimer kt(kinds[ep.mode >= 0 && ep.mode <= 3 ? ep.mode : 0], st, 2.0 * M * N * K);
    JB_CUDA(launch_pdl(k_gemm_f16, grid, dim3(THREADS), SMEM_BYTES, st, ta, tb, to, tkv, M, N, K, ep, tma_out));
    return 0;
}

int gemm_f16_error_flag(cudaStream_t st) {
    int v = 0;
    static const int zero = 0;
    if (!cuda_ok(cudaMemcpyFromSymbolAsync(&v, g_f16_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st), "reading the f16 GEMM error flag") ||
        !cuda_ok(cudaMemcpyToSymbolAsync(g_f16_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st), "resetting the f16 GEMM error flag") ||
        !cuda_ok(cudaStreamSynchronize(st), "reading the f16 GEMM error flag")) {
        return -1;
    }
    return v;
}

int gemm_f16_error_clear(cudaStream_t st) {
    static const int zero = 0;
    return cuda_ok(cudaMemcpyToSymbolAsync(g_f16_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                   "clearing the f16 GEMM error flag") ? 0 : -1;
}

}  // namespace jb
