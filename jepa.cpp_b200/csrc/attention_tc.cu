// Block-causal attention of the V-JEPA 2-AC predictor on the tcgen05 tensor cores (head width 64, up to
// 288 query rows per frame). Same contract as attention.cu (the frame-list keys, candidate strides, one
// query frame per grid x slot); this kernel is the one the predictor uses for its real shapes.
//
// One CTA per (query frame, head, candidate). The frame's query rows are cut into up to three 128-row
// tiles (258 = 128 + 128 + 2 for the AC predictor); the keys stream through in 64-key blocks:
//   loader        one thread issues TMA loads (3-D tensor maps: columns, rows of a frame, candidates) of
//                 the Q tiles once and of each key block's K and V boxes (64 rows x 128 B, 128-byte
//                 swizzle); a block that straddles two frames is two boxes per operand, each zero-filled
//                 outside its frame (rows past the frame end, or before its start), so their products add
//                 up to the block's; 3 stages
//   MMA warp      lane t drives query tile t: S_t = Q_t K^T (M 128, N 64, K 64) into TMEM one block ahead
//                 of the softmax; then O_t = P_t V (M 128, N 64, K 64; V read MN-major) into the tile's
//                 TMEM partial (the tiles advance independently)
//   softmax warps one thread per query row (4 warps per full tile, one per TMEM lane quadrant): reads its
//                 row of S from TMEM, keeps the running max / sum, writes P (f16) into a swizzled shared
//                 tile for the P V product, and folds each block's partial into a register accumulator
//                 with the online-softmax correction; finally divides by the sum and stores f16 rows.
// Tiles 0 and 1 double-buffer S and P (the S product of block j+1 overlaps the softmax of block j); the
// partial third tile single-buffers them. TMEM: partials at columns 0..191, S at 192..511.
// Every mbarrier wait is bounded (about two seconds): on a timeout the kernel raises the error flag and
// its warps leave their loops; the CTA drains and frees its TMEM.
#include "kernels.h"
#include "common.h"
#include "launch.h"
#include "tcgen05.cuh"
#include "kprof.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

namespace jb {

namespace {

using namespace tc;

constexpr int HD = 64;
constexpr int KBLK = 64;                        // keys per block
constexpr int KV_STAGES = 3;
constexpr int TC_FRAMES = 8;                    // key frames the tensor maps cover
constexpr int MAX_WARPS = 11;                   // 4 + 4 + 1 softmax, loader, issuer: up to 288 query rows
constexpr uint32_t TILE_BYTES = 128 * 128;      // 128 rows x 128 B (64 f16)
constexpr uint32_t KV_BYTES = KBLK * 128;       // 64 rows x 128 B
// instruction descriptors (kind::f16, f16 inputs, f32 accumulate, M 128, N 64); PV reads B MN-major (bit 16)
constexpr uint32_t IDESC_S = (1u << 4) | ((uint32_t) (64 >> 3) << 17) | ((uint32_t) (128 >> 4) << 24);
constexpr uint32_t IDESC_PV = IDESC_S | (1u << 16);

__device__ int g_attn_error = 0;

struct TcMaps {
    CUtensorMap q;                      // [cand][rows of a candidate][D], box 64 x 128 x 1
    CUtensorMap kv[TC_FRAMES];          // per key frame [cand (1 if shared)][kv_rows][2 D], box 64 x 64 x 1
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap * map, int x, int y, int z, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(dst), "l"((uint64_t) map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}

// The key block j = keys [64 j, 64 j + 64): its first frame f0 and row kr0 in it, and whether the block
// runs into the next frame (then a second box starts at row -n1 of frame f0 + 1, n1 = kv_rows - kr0).
struct KeyBlock {
    int f0, kr0, n1;
    bool split;
};
__device__ __forceinline__ KeyBlock key_block(int j, int kv_rows, int nkeys) {
    KeyBlock k;
    const int key0 = j * KBLK;
    k.f0 = key0 / kv_rows;
    k.kr0 = key0 - k.f0 * kv_rows;
    k.n1 = kv_rows - k.kr0;
    k.split = k.n1 < KBLK && key0 + k.n1 < nkeys;
    return k;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack2h(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t *) &h;
}

struct Layout {
    int n_tiles, q_last, nsw;        // query tiles, lane quadrants of the last tile, softmax warps
};

__host__ __device__ inline Layout layout_of(int nq) {
    Layout l;
    l.n_tiles = (nq + 127) / 128;
    const int rows_last = nq - 128 * (l.n_tiles - 1);
    l.q_last = (rows_last + 31) / 32;
    l.nsw = 4 * (l.n_tiles - 1) + l.q_last;
    return l;
}

// buffers of tile t: 2 for the first two tiles, 1 for a third
__device__ __forceinline__ int nbuf(int t) { return t < 2 ? 2 : 1; }
__device__ __forceinline__ uint32_t s_col(int t, int b) { return t < 2 ? 192u + 128u * t + 64u * b : 448u; }

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warps: [0, nsw) softmax (tile w / 4, lane quadrant w % 4), nsw loader, nsw + 1 the MMA issuers (lane t issues
// tile t; the lanes advance independently). Shared memory: Q tiles, then per stage K_A, K_B, V_A, V_B boxes,
// then the P tiles.
__global__ void __launch_bounds__(32 * MAX_WARPS, 1) k_attention_tc(const __grid_constant__ TcMaps maps, AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
    __shared__ __align__(8) uint64_t s_full[3][2], s_free[3][2], p_full[3][2];
    __shared__ __align__(8) uint64_t o_full[3], o_free[3];
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_sh;

    const Layout L = layout_of(a.nq);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int loader = L.nsw, mma0 = L.nsw + 1;
    const int qf = blockIdx.x, head = blockIdx.y, cand = blockIdx.z;
    const int nkeys = (a.key_frames0 + qf * a.key_step) * a.kv_rows;
    const int nblk = (nkeys + KBLK - 1) / KBLK;

    uint8_t * sQ = smem;                                             // [n_tiles][128 rows][128 B]
    uint8_t * sKV = sQ + (size_t) L.n_tiles * TILE_BYTES;            // [stage][K_A, K_B, V_A, V_B][64][128 B]
    uint8_t * sP = sKV + (size_t) KV_STAGES * 4 * KV_BYTES;          // tile t buffer b: P + (2t + b) * 16 KB

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < KV_STAGES; s++) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], L.n_tiles); }
        for (int t = 0; t < 3; t++) {
            const int w = t < L.n_tiles - 1 ? 4 : L.q_last;
            for (int b = 0; b < 2; b++) { mbar_init(&s_full[t][b], 1); mbar_init(&s_free[t][b], w); mbar_init(&p_full[t][b], w); }
            mbar_init(&o_full[t], 1);
            mbar_init(&o_free[t], w);
        }
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == mma0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(smem_u32(&tmem_sh)), "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == loader && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &maps.q) : "memory");
        const int nf = a.key_frames0 + qf * a.key_step;
        for (int f = 0; f < nf && f < TC_FRAMES; f++) asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &maps.kv[f]) : "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_sh;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == loader) {
        if (lane == 0) {
            const uint32_t q_u = smem_u32(sQ), kv_u = smem_u32(sKV);
            mbar_expect_tx(&q_full, (uint32_t) L.n_tiles * TILE_BYTES);
            for (int t = 0; t < L.n_tiles; t++) tma_load_3d(q_u + t * TILE_BYTES, &maps.q, head * HD, qf * a.q_frame + 128 * t, cand, &q_full);
            for (int j = 0; j < nblk; j++) {
                const int s = j % KV_STAGES;
                if (j >= KV_STAGES && !mbar_wait(&kv_empty[s], (uint32_t) ((j / KV_STAGES) - 1) & 1u, 21, &g_attn_error)) {
                    abort_sh = 1;
                    break;
                }
                if (*(volatile int *) &abort_sh) break;
                const KeyBlock kb = key_block(j, a.kv_rows, nkeys);
                const uint32_t st = kv_u + (uint32_t) s * 4 * KV_BYTES;
                mbar_expect_tx(&kv_full[s], (kb.split ? 4u : 2u) * KV_BYTES);
                const int z0 = a.kv_cand_stride[kb.f0] ? cand : 0;
                tma_load_3d(st, &maps.kv[kb.f0], head * HD, kb.kr0, z0, &kv_full[s]);
                tma_load_3d(st + 2 * KV_BYTES, &maps.kv[kb.f0], a.D + head * HD, kb.kr0, z0, &kv_full[s]);
                if (kb.split) {
                    const int z1 = a.kv_cand_stride[kb.f0 + 1] ? cand : 0;
                    tma_load_3d(st + KV_BYTES, &maps.kv[kb.f0 + 1], head * HD, -kb.n1, z1, &kv_full[s]);
                    tma_load_3d(st + 3 * KV_BYTES, &maps.kv[kb.f0 + 1], a.D + head * HD, -kb.n1, z1, &kv_full[s]);
                }
            }
        }
    } else if (warp == mma0) {
        // ---- MMA issue: lane t drives query tile t
        const int t = lane;
        if (t < L.n_tiles) {
            const int nb = nbuf(t);
            bool ok = mbar_wait(&q_full, 0, 22, &g_attn_error);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t qa = smem_u32(sQ) + t * TILE_BYTES, kv_u = smem_u32(sKV), p_u = smem_u32(sP);
            auto issue_s = [&](int j) -> bool {
                const int s = j % KV_STAGES, b = j % nb, u = j / nb;
                if (!mbar_wait(&kv_full[s], (uint32_t) (j / KV_STAGES) & 1u, 23, &g_attn_error)) return false;
                if (u >= 1 && !mbar_wait(&s_free[t][b], (uint32_t) (u - 1) & 1u, 24, &g_attn_error)) return false;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const bool split = key_block(j, a.kv_rows, nkeys).split;
                const uint32_t ka = kv_u + (uint32_t) s * 4 * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    mma_kind_f16(tmem + s_col(t, b), sw128_desc(qa + kk * 32), sw128_desc(ka + kk * 32), IDESC_S, kk != 0);
                }
                if (split) {
#pragma unroll
                    for (int kk = 0; kk < HD / 16; kk++) {
                        mma_kind_f16(tmem + s_col(t, b), sw128_desc(qa + kk * 32), sw128_desc(ka + KV_BYTES + kk * 32), IDESC_S, 1);
                    }
                }
                mma_commit(&s_full[t][b]);
                return true;
            };
            if (ok && nblk > 0) ok = issue_s(0);
            for (int j = 0; j < nblk && ok; j++) {
                if (j + 1 < nblk && !issue_s(j + 1)) { ok = false; break; }
                const int s = j % KV_STAGES, b = j % nb, u = j / nb;
                if (!mbar_wait(&p_full[t][b], (uint32_t) u & 1u, 25, &g_attn_error)) { ok = false; break; }
                if (j >= 1 && !mbar_wait(&o_free[t], (uint32_t) (j - 1) & 1u, 26, &g_attn_error)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const bool split = key_block(j, a.kv_rows, nkeys).split;
                const uint32_t va = kv_u + (uint32_t) s * 4 * KV_BYTES + 2 * KV_BYTES;
                const uint32_t pbuf = p_u + (uint32_t) (2 * t + b) * (128 * 128);
#pragma unroll
                for (int kk = 0; kk < KBLK / 16; kk++) {
                    // A = P (K-major, 32 B per 16 keys); B = V MN-major (16 key rows = 2048 B per step)
                    mma_kind_f16(tmem + 64u * t, sw128_desc(pbuf + kk * 32), sw128_desc(va + kk * 2048), IDESC_PV, kk != 0);
                }
                if (split) {
#pragma unroll
                    for (int kk = 0; kk < KBLK / 16; kk++) {
                        mma_kind_f16(tmem + 64u * t, sw128_desc(pbuf + kk * 32), sw128_desc(va + KV_BYTES + kk * 2048), IDESC_PV, 1);
                    }
                }
                mma_commit(&o_full[t]);
                mma_commit(&kv_empty[s]);
            }
            if (!ok) abort_sh = 1;
        }
    } else if (warp < L.nsw) {
        // ---- softmax: thread = query row 128 t + 32 q + lane
        const int t = warp >> 2, q = warp & 3;
        const int row = 128 * t + 32 * q + lane;
        const int nb = nbuf(t);
        const uint32_t lane_off = (uint32_t) (32 * q) << 16;
        const float sl2 = a.scale * 1.4426950408889634f;
        uint8_t * prow_base = sP + (size_t) (2 * t) * (128 * 128) + (size_t) (32 * q + lane) * 128;
        float acc[HD];
#pragma unroll
        for (int d = 0; d < HD; d++) acc[d] = 0.0f;
        float m = -INFINITY, l = 0.0f, c_prev = 0.0f;
        bool ok = true;
        auto fold = [&](int j) -> bool {
            // acc = acc * c_prev + partial of block j
            if (!mbar_wait(&o_full[t], (uint32_t) j & 1u, 27, &g_attn_error)) return false;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t r0[32], r1[32];
            tmem_ld32_nowait(tmem + lane_off + 64u * t, r0);
            tmem_ld32_nowait(tmem + lane_off + 64u * t + 32u, r1);
            tmem_wait_ld();
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[t]);
            if (__all_sync(0xffffffffu, c_prev == 1.0f)) {
#pragma unroll
                for (int d = 0; d < 32; d++) { acc[d] += __uint_as_float(r0[d]); acc[32 + d] += __uint_as_float(r1[d]); }
            } else {
#pragma unroll
                for (int d = 0; d < 32; d++) {
                    acc[d] = __fmaf_rn(acc[d], c_prev, __uint_as_float(r0[d]));
                    acc[32 + d] = __fmaf_rn(acc[32 + d], c_prev, __uint_as_float(r1[d]));
                }
            }
            return true;
        };
        for (int j = 0; j < nblk; j++) {
            const int b = j % nb, u = j / nb;
            // a single-buffered tile reuses its P buffer: the previous product is folded in first
            if (nb == 1 && j >= 1 && !fold(j - 1)) { ok = false; break; }
            if (!mbar_wait(&s_full[t][b], (uint32_t) u & 1u, 28, &g_attn_error)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const bool tail = j + 1 == nblk && (nkeys % KBLK) != 0;   // only the last block runs past the keys
            // one read of the row's 64 scores; the maximum and the sum in independent chains (ILP)
            uint32_t r0[32], r1[32];
            tmem_ld32_nowait(tmem + lane_off + s_col(t, b), r0);
            tmem_ld32_nowait(tmem + lane_off + s_col(t, b) + 32u, r1);
            tmem_wait_ld();
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[t][b]);
            if (tail) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    if (j * KBLK + i >= nkeys) r0[i] = __float_as_uint(-INFINITY);
                    if (j * KBLK + 32 + i >= nkeys) r1[i] = __float_as_uint(-INFINITY);
                }
            }
            float mq[8];
#pragma unroll
            for (int k = 0; k < 8; k++) mq[k] = fmaxf(__uint_as_float(r0[k]), __uint_as_float(r1[k]));
#pragma unroll
            for (int i = 8; i < 32; i += 8) {
#pragma unroll
                for (int k = 0; k < 8; k++) mq[k] = fmaxf(mq[k], fmaxf(__uint_as_float(r0[i + k]), __uint_as_float(r1[i + k])));
            }
            const float mx = fmaxf(m, fmaxf(fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])), fmaxf(fmaxf(mq[4], mq[5]), fmaxf(mq[6], mq[7]))));
            const float c = ex2((m - mx) * sl2);        // 0 on the first block (m = -inf)
            const float nm = -mx * sl2;
            m = mx;
            // P = exp2(s log2e scale - max) (masked scores are -inf -> 0), f16, into the swizzled P tile
            uint8_t * prow = prow_base + (size_t) b * (128 * 128);
            float sq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int cch = 0; cch < 8; cch++) {
                float p[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int i = (cch & 3) * 8 + e;
                    p[e] = ex2(__fmaf_rn(__uint_as_float(cch < 4 ? r0[i] : r1[i]), sl2, nm));
                }
#pragma unroll
                for (int e = 0; e < 8; e++) sq[e & 3] += p[e];
                uint4 w;
                w.x = pack2h(p[0], p[1]); w.y = pack2h(p[2], p[3]); w.z = pack2h(p[4], p[5]); w.w = pack2h(p[6], p[7]);
                *(uint4 *) (prow + ((cch ^ (lane & 7)) << 4)) = w;
            }
            const float sum = (sq[0] + sq[1]) + (sq[2] + sq[3]);
            l = __fmaf_rn(l, c, sum);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t][b]);
            if (nb == 2 && j >= 1 && !fold(j - 1)) { ok = false; break; }
            c_prev = c;
            if (*(volatile int *) &abort_sh) { ok = false; break; }
        }
        if (ok && nblk > 0) ok = fold(nblk - 1);
        if (!ok) {
            abort_sh = 1;
        } else if (row < a.nq) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            __half * dst = a.out + (size_t) cand * a.o_cand + ((size_t) qf * a.q_frame + row) * a.ldo + head * HD;
#pragma unroll
            for (int cch = 0; cch < 8; cch++) {
                uint4 w;
                w.x = pack2h(acc[8 * cch + 0] * inv, acc[8 * cch + 1] * inv);
                w.y = pack2h(acc[8 * cch + 2] * inv, acc[8 * cch + 3] * inv);
                w.z = pack2h(acc[8 * cch + 4] * inv, acc[8 * cch + 5] * inv);
                w.w = pack2h(acc[8 * cch + 6] * inv, acc[8 * cch + 7] * inv);
                *(uint4 *) (dst + 8 * cch) = w;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == mma0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(512) : "memory");
    }
}

size_t smem_bytes(const Layout & L) {
    return (size_t) L.n_tiles * TILE_BYTES + (size_t) 4 * KV_STAGES * KV_BYTES + (size_t) 5 * 128 * 128 + 1024;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode3 = nullptr;
std::once_flag g_encode3_once;

// 3-D f16 map: dims (cols, rows, planes), row stride ld elements, plane stride pstride elements, box (64, box_rows, 1)
bool encode3(CUtensorMap * map, const __half * base, long long cols, long long rows, long long planes, long long ld,
             long long pstride, int box_rows) {
    std::call_once(g_encode3_once, []() {
        void * fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode3 = (PFN_cuTensorMapEncodeTiled_v12000) fn;
        }
    });
    if (!g_encode3) return false;
    const cuuint64_t dims[3] = {(cuuint64_t) cols, (cuuint64_t) rows, (cuuint64_t) planes};
    const cuuint64_t strides[2] = {(cuuint64_t) ld * 2, (cuuint64_t) (pstride > 0 ? pstride : ld * rows) * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t) box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return g_encode3(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *) base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_tc_supported(const AttnArgs & a) {
    if (a.nq < 1 || a.nq > 384) return false;
    const Layout L = layout_of(a.nq);
    const int max_kf = a.key_frames0 + (a.n_qframes - 1) * a.key_step;
    if (a.hd != HD || L.nsw + 2 > MAX_WARPS || max_kf > TC_FRAMES || a.kv_rows < KBLK) return false;
    if ((a.ldq & 7) || (a.ld_kv & 7) || (a.ldo & 7) || (a.D & 7) || ((uintptr_t) a.q & 15) || ((uintptr_t) a.out & 15) ||
        (a.q_cand & 7) || (a.o_cand & 7) || a.q_cand < (long long) a.ldq) {
        return false;
    }
    for (int f = 0; f < max_kf; f++) {
        if (((uintptr_t) a.kv[f] & 15) || (a.kv_cand_stride[f] & 7)) return false;
    }
    return true;
}

int attention_tc(const AttnArgs & a, cudaStream_t st) {
    const Layout L = layout_of(a.nq);
    const size_t smem = smem_bytes(L);
    static bool attr_set = false;
    if (!attr_set) {
        JB_CUDA(cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem_bytes(layout_of(288))));
        attr_set = true;
    }
    // Q: planes = candidates, rows = the candidate's rows (q_cand / ldq); keys: per frame, planes = candidates
    // (1 when the frame is shared), rows = kv_rows, columns = 2 D (k then v)
    TcMaps maps;
    memset(&maps, 0, sizeof(maps));
    bool ok = encode3(&maps.q, a.q, a.D, a.q_cand / a.ldq, a.n_cand, a.ldq, a.q_cand, 128);
    const int max_kf = a.key_frames0 + (a.n_qframes - 1) * a.key_step;
    for (int f = 0; f < max_kf && ok; f++) {
        const bool shared = a.kv_cand_stride[f] == 0;
        ok = encode3(&maps.kv[f], a.kv[f], 2LL * a.D, a.kv_rows, shared ? 1 : a.n_cand, a.ld_kv, a.kv_cand_stride[f], KBLK);
    }
    if (!ok) {
        log("jepa: attention: cuTensorMapEncodeTiled refused the query / key layout\n");
        return -1;
    }
    const dim3 grid((unsigned) a.n_qframes, (unsigned) a.n_head, (unsigned) a.n_cand);
    JB_CUDA(launch_pdl(k_attention_tc, grid, dim3((unsigned) (32 * (L.nsw + 2))), smem, st, maps, a));
    return 0;
}

int attention_tc_error_flag(cudaStream_t st) {
    int v = 0;
    static const int zero = 0;
    if (!cuda_ok(cudaMemcpyFromSymbolAsync(&v, g_attn_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st), "reading the attention error flag") ||
        !cuda_ok(cudaMemcpyToSymbolAsync(g_attn_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st), "resetting the attention error flag") ||
        !cuda_ok(cudaStreamSynchronize(st), "reading the attention error flag")) {
        return -1;
    }
    return v;
}

int attention_tc_error_clear(cudaStream_t st) {
    static const int zero = 0;
    return cuda_ok(cudaMemcpyToSymbolAsync(g_attn_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                   "clearing the attention error flag") ? 0 : -1;
}

}  // namespace jb
