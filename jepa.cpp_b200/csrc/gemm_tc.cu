// tcgen05 / TMEM / TMA GEMM for sm_100a: C[M,N] = A[M,K] * B[N,K]^T in 3xTF32, fused epilogues.
//
// Every dense contraction of the planner (the predictor's V / out / up / down linears, their
// transposed backward products, the time-batched adaLN modulation and its backward) runs here.
//
// Kernel shape (one 128 x BN output tile per CTA, 6 warps):
//   warp 0      TMA producer: per K-step of 32 it loads A_hi, A_lo (128 x 32 f32 each) and B_hi, B_lo
//               (BN x 32) into one pipeline stage, 128-byte swizzled, completion on the stage's mbarrier
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues, per stage, 4 K-slices x 3
//               tcgen05.mma.kind::tf32 (hi*hi, hi*lo, lo*hi) into a 128 x BN float32 accumulator in
//               TMEM, then tcgen05.commit releases the stage to the producer
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (each warp owns the TMEM lane quadrant
//               warp % 4), bias / GELU / gated residual / split, stores to global memory
// Operand split (hi = x with the low 13 mantissa bits cleared, lo = x - hi) is done by whoever
// produces the operand, so the mainloop is pure TMA -> tensor core.
// Every mbarrier wait is bounded (about two seconds of clock64): on a timeout the kernel raises an
// error flag the host reads, drains what it issued, frees its TMEM and returns.
#include "kernels.h"
#include "common.h"
#include "launch.h"
#include "tcgen05.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace jb {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;                  // 32 f32 = one 128-byte swizzle row
// warp 0: TMA producer, warp 1: MMA issuer, warps 2-5: accumulator readers (TMEM lane quadrant = warp % 4);
// warps 6-11 join the split-K reduction and the fused epilogue, latency-bound per-thread work (a GELU per
// element) that twelve warps finish in half the time six do
constexpr int GEMM_THREADS = 384;

__device__ int g_gemm_error = 0;

using namespace tc;


__device__ __forceinline__ float split_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__device__ __forceinline__ float gelu_f(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}
__device__ __forceinline__ float gelu_grad(float v) {
    return 0.5f * (1.0f + erff(v * 0.70710678118654752f)) + v * 0.39894228040143268f * expf(-0.5f * v * v);
}
// gelu(u) and gelu'(u) from one erf: the same expressions as gelu_f and gelu_grad, so the same bits
__device__ __forceinline__ void gelu_and_grad(float u, float & g, float & d) {
    const float e = erff(u * 0.70710678118654752f);
    g = 0.5f * u * (1.0f + e);
    d = 0.5f * (1.0f + e) + u * 0.39894228040143268f * expf(-0.5f * u * u);
}
template <int MODE> __host__ __device__ constexpr bool has_bias() { return MODE != EPI_DGELU_SPLIT && MODE != EPI_MUL_SPLIT; }

// The fused epilogue of one output element (v = the accumulated product, before the bias). The mode is a
// template parameter throughout, so that a kernel holds the code of its own epilogue only: these kernels
// are latency-bound, and every instruction fetched on the way from the accumulator to the stores is time.
// The element-wise path (unaligned operands, the ragged last columns) stays out of line.
template <int MODE>
__device__ __noinline__ void apply_epi(const GemmEpi & ep, int row, int col, float v) {
    if (has_bias<MODE>() && ep.bias) v = v + ep.bias[col];
    switch (MODE) {
        case EPI_F32:
            ep.out0[(size_t) row * ep.ld0 + col] = v;
            break;
        case EPI_SPLIT: {
            const float h = split_hi(v);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = v - h;
        } break;
        case EPI_F32_SPLIT: {
            ep.out0[(size_t) row * ep.ld0 + col] = v;
            const float h = split_hi(v);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = v - h;
        } break;
        case EPI_GELU_SPLIT: {
            ep.out0[(size_t) row * ep.ld0 + col] = v;
            const float gv = gelu_f(v);
            const float h = split_hi(gv);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = gv - h;
        } break;
        case EPI_GATED: {
            ep.out0[(size_t) row * ep.ld0 + col] = v;
            const float g = ep.gate[(size_t) row * ep.ld_gate + col];
            ep.out1[(size_t) row * ep.ld1 + col] = ep.aux[(size_t) row * ep.ld_aux + col] + v * g;
        } break;
        case EPI_DGELU_SPLIT: {
            const float d = v * gelu_grad(ep.aux[(size_t) row * ep.ld_aux + col]);
            const float h = split_hi(d);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = d - h;
        } break;
        case EPI_GELU_D_SPLIT: {
            float gv, dv;
            gelu_and_grad(v, gv, dv);
            ep.out0[(size_t) row * ep.ld0 + col] = dv;
            const float h = split_hi(gv);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = gv - h;
        } break;
        case EPI_MUL_SPLIT: {
            const float d = v * ep.aux[(size_t) row * ep.ld_aux + col];
            const float h = split_hi(d);
            ep.out_hi[(size_t) row * ep.ld_split + col] = h;
            ep.out_lo[(size_t) row * ep.ld_split + col] = d - h;
        } break;
        default: break;
    }
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
__device__ __forceinline__ float4 f4_hi(float4 a) { return make_float4(split_hi(a.x), split_hi(a.y), split_hi(a.z), split_hi(a.w)); }
__device__ __forceinline__ float4 f4_sub(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
__device__ __forceinline__ float4 ld4(const float * p) { return *(const float4 *) p; }
__device__ __forceinline__ void st4(float * p, float4 v) { *(float4 *) p = v; }

// The operands a vector epilogue reads (bias, aux, gate), loaded ahead of the values they combine with.
struct Epi4In {
    float4 bias, aux, gate;
};

template <int MODE>
__device__ __forceinline__ Epi4In epi_load4(const GemmEpi & ep, int row, int col) {
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    Epi4In in{z, z, z};
    if (has_bias<MODE>() && ep.bias) in.bias = ld4(ep.bias + col);
    if (MODE == EPI_GATED || MODE == EPI_DGELU_SPLIT || MODE == EPI_MUL_SPLIT) in.aux = ld4(ep.aux + (size_t) row * ep.ld_aux + col);
    if (MODE == EPI_GATED) in.gate = ld4(ep.gate + (size_t) row * ep.ld_gate + col);
    return in;
}

// four consecutive columns of the fused epilogue, vector path (ep.vec and col + 3 < N)
template <int MODE>
__device__ __forceinline__ void epi_store4(const GemmEpi & ep, int row, int col, float4 v, const Epi4In & in) {
    if (has_bias<MODE>() && ep.bias) v = f4_add(v, in.bias);
    switch (MODE) {
        case EPI_F32: st4(ep.out0 + (size_t) row * ep.ld0 + col, v); break;
        case EPI_SPLIT: {
            const float4 h = f4_hi(v);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(v, h));
        } break;
        case EPI_F32_SPLIT: {
            st4(ep.out0 + (size_t) row * ep.ld0 + col, v);
            const float4 h = f4_hi(v);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(v, h));
        } break;
        case EPI_GELU_SPLIT: {
            st4(ep.out0 + (size_t) row * ep.ld0 + col, v);
            const float4 g = make_float4(gelu_f(v.x), gelu_f(v.y), gelu_f(v.z), gelu_f(v.w));
            const float4 h = f4_hi(g);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(g, h));
        } break;
        case EPI_GATED: {
            st4(ep.out0 + (size_t) row * ep.ld0 + col, v);
            st4(ep.out1 + (size_t) row * ep.ld1 + col, f4_add(in.aux, f4_mul(v, in.gate)));
        } break;
        case EPI_DGELU_SPLIT: {
            const float4 u = in.aux;
            const float4 d = f4_mul(v, make_float4(gelu_grad(u.x), gelu_grad(u.y), gelu_grad(u.z), gelu_grad(u.w)));
            const float4 h = f4_hi(d);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(d, h));
        } break;
        case EPI_GELU_D_SPLIT: {
            float4 g, d;
            gelu_and_grad(v.x, g.x, d.x);
            gelu_and_grad(v.y, g.y, d.y);
            gelu_and_grad(v.z, g.z, d.z);
            gelu_and_grad(v.w, g.w, d.w);
            st4(ep.out0 + (size_t) row * ep.ld0 + col, d);
            const float4 h = f4_hi(g);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(g, h));
        } break;
        case EPI_MUL_SPLIT: {
            const float4 d = f4_mul(v, in.aux);
            const float4 h = f4_hi(d);
            st4(ep.out_hi + (size_t) row * ep.ld_split + col, h);
            st4(ep.out_lo + (size_t) row * ep.ld_split + col, f4_sub(d, h));
        } break;
        default: break;
    }
}

// four consecutive columns of the fused epilogue: vector loads / stores when the operands allow it
// (ep.vec: every pointer 16-byte aligned, every leading dimension a multiple of 4), else element-wise
template <int MODE>
__device__ __forceinline__ void apply_epi4(const GemmEpi & ep, int row, int col, int N, float4 v) {
    if (!ep.vec || col + 3 >= N) {
        const float e[4] = {v.x, v.y, v.z, v.w};
        for (int j = 0; j < 4; j++) if (col + j < N) apply_epi<MODE>(ep, row, col + j, e[j]);
        return;
    }
    epi_store4<MODE>(ep, row, col, v, epi_load4<MODE>(ep, row, col));
}

__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}


__device__ __forceinline__ uint32_t peer_addr(uint32_t local_saddr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
    return remote;
}

// A bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory into a peer CTA's, completing on
// the peer's mbarrier (transaction bytes). One thread issues it; the copy engine moves the data.
__device__ __forceinline__ void bulk_to_peer(uint32_t remote_dst, uint32_t local_src, uint32_t bytes, uint32_t remote_bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(remote_dst), "r"(local_src), "r"(bytes), "r"(remote_bar) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Weight operands dequantised in the mainloop (QuantB). The producer's TMA copies a K-step's raw tile --
// BN rows of 32 block values and their f16 scales -- into the stage's B_lo area; two converter warps read it
// into registers, meet on the stage's raw barrier (after which the area may be overwritten), and write the
// split planes B_hi and B_lo in the 128-byte swizzle the TMA would have used (16-byte chunk c of row r at
// c ^ (r & 7)). The MMA warp waits on the stage's converted barrier instead of the copy barrier.
// ---------------------------------------------------------------------------------------------
struct QDesc {
    int fmt = QF_NONE;
    int orient = 0;
};
// converter warps: four in the split-K cluster kernel (its reduction warps are idle in the mainloop), PCONV_WARPS
// in the persistent kernel (added warps: its register budget caps them)
constexpr int CONV_WARPS = 4;
// (two, 384 threads, no spill; four at 448 threads measured 22.8 against 24-25 us per launch at 2048 x 768 x 768
// but cap the kernel at 128 registers, which spills its epilogue)
constexpr int PCONV_WARPS = 2;

// raw bytes of one row of a K-step (32 values) and of the K-step's scales, for BN rows
__host__ __device__ constexpr uint32_t raw_row_bytes(int fmt) { return fmt == QF_Q8 ? 32u : fmt == QF_Q4 ? 16u : fmt == QF_F16 ? 64u : 0u; }
__host__ __device__ constexpr uint32_t raw_scale_bytes(int fmt, int bn) { return fmt == QF_Q8 || fmt == QF_Q4 ? 2u * (uint32_t) bn : 0u; }

__device__ __forceinline__ float half_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short) (h & 0xFFFFu))); }

// byte k of x as the float 2^23 + byte (exact): the block values become floats by a byte permute and one
// exact subtraction instead of an integer conversion
__device__ __forceinline__ float byte_as_float(uint32_t x, int k) {
    return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650u | (uint32_t) k));
}

// value e (0..15) of a 16-value row segment: the block value times its scale, exact in float32.
// w: the segment's raw words (q8_0: int8 with the sign bit flipped; q4_0: low and high nibbles in words
// 0-1 and 2-3; f16: halves); sc: the scale(s) as f16 bits.
template <int FMT, int ORIENT>
__device__ __forceinline__ float seg_value(const uint32_t (&w)[8], const uint32_t (&sc)[8], int e) {
    if (FMT == QF_F16) return half_bits(w[e >> 1] >> ((e & 1) * 16));
    const float d = ORIENT == 0 ? half_bits(sc[0]) : half_bits(sc[e >> 1] >> ((e & 1) * 16));
    if (FMT == QF_Q8) return d * (byte_as_float(w[e >> 2], e & 3) - 8388736.0f);            // q
    return (byte_as_float(w[2 * (e & 1) + (e >> 3)], (e >> 1) & 3) - 8388616.0f) * d;      // q - 8
}

// The split planes of a converter thread's NSEG row segments (raw words w and scales sc in registers, as
// seg_value reads them) into a stage's B_hi / B_lo areas (bh, bh + BN * 128): segment g of thread ct is
// segment ct + CT g of the tile, row (ct + CT g) / 2, values 16 ((ct + CT g) % 2) ..
template <int BN, int CT, int FMT, int ORIENT, int NSEG>
__device__ __forceinline__ void write_segments(uint8_t * bh, int ct, const uint32_t (&w)[NSEG][8], const uint32_t (&sc)[NSEG][8]) {
    uint8_t * bl = bh + BN * 128;
#pragma unroll
    for (int g = 0; g < NSEG; g++) {
        const int seg = ct + CT * g, r = seg >> 1, h = seg & 1;
        float * hrow = (float *) (bh + r * 128);
        float * lrow = (float *) (bl + r * 128);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float hv[4], lv[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const float v = seg_value<FMT, ORIENT>(w[g], sc[g], 4 * c + t);
                hv[t] = split_hi(v);
                lv[t] = v - hv[t];
            }
            const int pos = ((4 * h + c) ^ (r & 7)) << 2;
            *(float4 *) (hrow + pos) = make_float4(hv[0], hv[1], hv[2], hv[3]);
            *(float4 *) (lrow + pos) = make_float4(lv[0], lv[1], lv[2], lv[3]);
        }
    }
    // the planes are read by the tensor core (async proxy) after the converted barrier
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// the raw words of a 16-value segment (q8_0: sign bit flipped; q4_0: low nibbles in words 0-1, high in 2-3)
template <int FMT>
__device__ __forceinline__ void raw_words(const uint8_t * src, uint32_t (&w)[8]) {
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = 0u;
    if (FMT == QF_Q4) {
        const uint2 x = *(const uint2 *) src;
        w[0] = x.x & 0x0F0F0F0Fu; w[1] = x.y & 0x0F0F0F0Fu;
        w[2] = (x.x >> 4) & 0x0F0F0F0Fu; w[3] = (x.y >> 4) & 0x0F0F0F0Fu;
        return;
    }
    constexpr int N4 = FMT == QF_F16 ? 2 : 1;
#pragma unroll
    for (int i = 0; i < N4; i++) {
        const uint4 x = ((const uint4 *) src)[i];
        w[4 * i] = x.x; w[4 * i + 1] = x.y; w[4 * i + 2] = x.z; w[4 * i + 3] = x.w;
    }
    if (FMT == QF_Q8) {
#pragma unroll
        for (int i = 0; i < 4; i++) w[i] ^= 0x80808080u;   // int8 -> byte + 128
    }
}

// 16 consecutive f16 scales (orient 1) into sc[0 .. 7]
__device__ __forceinline__ void scale_words(const uint16_t * src, uint32_t (&sc)[8]) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const uint4 x = ((const uint4 *) src)[i];
        sc[4 * i] = x.x; sc[4 * i + 1] = x.y; sc[4 * i + 2] = x.z; sc[4 * i + 3] = x.w;
    }
}

// Converts one stage's raw tile (in the B_lo area at bh + BN * 128) into B_hi / B_lo. The tile's rows are
// cut in 16-value segments; converter thread ct of CT owns segments ct, ct + CT, ... (segment g: row g / 2,
// values 16 (g % 2) ..). The raw area is overwritten by the planes, so the converters first read their
// segments into registers and meet on the stage's raw barrier. False = that wait gave up.
template <int BN, int CT, int FMT, int ORIENT>
__device__ __forceinline__ bool convert_rows(uint8_t * bh, int ct, int lane, uint64_t * raw_bar, uint32_t ph) {
    constexpr int NSEG = 2 * BN / CT;
    constexpr int RB = (int) raw_row_bytes(FMT), SB = RB / 2;
    static_assert(NSEG >= 1 && 2 * BN % CT == 0, "whole segments per converter thread");
    const uint8_t * bl = bh + BN * 128;
    uint32_t w[NSEG][8], sc[NSEG][8];
#pragma unroll
    for (int g = 0; g < NSEG; g++) {
        const int seg = ct + CT * g, r = seg >> 1, h = seg & 1;
        raw_words<FMT>(bl + r * RB + h * SB, w[g]);
#pragma unroll
        for (int i = 0; i < 8; i++) sc[g][i] = 0u;
        if (FMT != QF_F16) {
            const uint8_t * d = bl + BN * RB;
            if (ORIENT == 0) sc[g][0] = ((const uint16_t *) d)[r];
            else scale_words((const uint16_t *) (d + (r >> 5) * 64 + h * 32), sc[g]);
        }
    }
    // every converter thread holds its raw segments: the B_lo area may be overwritten from here on
    __syncwarp();
    if (lane == 0) mbar_arrive(raw_bar);
    if (!mbar_wait_spin(raw_bar, ph, 7, &g_gemm_error)) return false;
    write_segments<BN, CT, FMT, ORIENT, NSEG>(bh, ct, w, sc);
    return true;
}

template <int BN, int CT, bool QB>
__device__ __forceinline__ bool convert_stage(uint8_t * bh, const QDesc & qd, int ct, int lane, uint64_t * raw_bar, uint32_t ph) {
    if constexpr (!QB) return false;
    switch (qd.fmt * 2 + qd.orient) {
        case QF_Q8 * 2: return convert_rows<BN, CT, QF_Q8, 0>(bh, ct, lane, raw_bar, ph);
        case QF_Q8 * 2 + 1: return convert_rows<BN, CT, QF_Q8, 1>(bh, ct, lane, raw_bar, ph);
        case QF_Q4 * 2: return convert_rows<BN, CT, QF_Q4, 0>(bh, ct, lane, raw_bar, ph);
        case QF_Q4 * 2 + 1: return convert_rows<BN, CT, QF_Q4, 1>(bh, ct, lane, raw_bar, ph);
        default: return convert_rows<BN, CT, QF_F16, 0>(bh, ct, lane, raw_bar, ph);
    }
}

// the TMA copies of one stage's raw B tile (K-step kt of the BN rows from n0) onto `bar`
template <int BN, bool QB>
__device__ __forceinline__ void load_raw_b(uint8_t * b_lo_area, const CUtensorMap * tq, const CUtensorMap * td, const QDesc & qd,
                                           int kt, int n0, uint64_t * bar) {
    if constexpr (!QB) return;
    tma_load_2d(b_lo_area, tq, qd.fmt == QF_Q4 ? kt * 16 : kt * 32, n0, bar);
    if (qd.fmt == QF_Q8 || qd.fmt == QF_Q4) {
        uint8_t * ds = b_lo_area + BN * raw_row_bytes(qd.fmt);
        if (qd.orient == 0) tma_load_2d(ds, td, n0, kt, bar);
        else tma_load_2d(ds, td, kt * 32, n0 / 32, bar);
    }
}

// Rows of the tile each CTA of a split-K cluster reduces and stores.
__host__ __device__ constexpr int split_rows(int splits) { return (BM + splits - 1) / splits; }

// One 128 x BN tile of C per CTA, or -- split-K -- one K-slice of it per CTA of a (1, 1, splits) cluster.
//
// splits == 1: the four accumulator warps stage the tile in shared memory (a row per thread, from TMEM),
// and all twelve warps apply the fused epilogue from there row-major: coalesced loads and stores.
// splits > 1 (a reduce-scatter over distributed shared memory): CTA p of the cluster owns rows
// [p R, p R + R) of the tile (R = ceil(128 / splits)). After the mainloop the epilogue warps stage the
// partial tile in shared memory and one thread sends each peer its rows with one bulk copy into the peer's
// receive buffer (completing on the peer's mbarrier); the owner waits for its bytes, sums the splits in rank
// order (a fixed order: the bits do not depend on timing) from its own shared memory and applies the fused
// epilogue with all twelve warps, in one pass. The epilogue's operands (bias, residual, gate) are requested
// before the mainloop (before the dependency wait when they come from earlier kernels), so their latency
// hides behind it. Cluster barriers: one arrive at the start (the receive
// barriers are initialised) waited on before the first push, one after the receive completes waited on
// before exit (no CTA leaves while a push to or from it may be in flight).
template <int BN, int STAGES, int MODE, bool QB>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
k_gemm_tf32x3(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
              const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo,
              int M, int N, int K, int splits, const QDesc qd, const __grid_constant__ GemmEpi ep) {
    constexpr uint32_t A_BYTES = BM * BK * 4;
    constexpr uint32_t B_BYTES = BN * BK * 4;
    constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    // bytes a stage's copies deliver: A_hi, A_lo, B_hi, B_lo on the stage's full barrier; with a weight in block
    // planes, A alone there and the raw B tile on its own barrier (the converters need B only)
    const uint32_t raw_tx = BN * raw_row_bytes(qd.fmt) + raw_scale_bytes(qd.fmt, BN);
    // block planes: a template switch, so that the plane-operand kernels carry none of the converters' code
    // (these kernels are latency-bound, and code between the accumulator and the stores costs fetches)
    const bool qb = QB && qd.fmt != QF_NONE;
    // two accumulators: hi*hi in columns [0, BN), the small cross terms hi*lo + lo*hi in [BN, 2 BN).
    // The tensor core's float32 accumulation rounds toward zero per instruction; keeping the small terms
    // apart cuts the number of truncations the large partial sum sees by three.
    //
    // A stage holds B_hi's BN rows directly followed by B_lo's (the same 128-byte swizzle, 8-row groups
    // 1024 bytes apart), so the two read as one operand of 2 BN rows: one MMA of width 2 BN computes
    // [hi*hi | hi*lo] into both accumulators at once and a second of width BN adds lo*hi to the cross
    // terms -- two instructions per K-step instead of three, and A_hi is read from shared memory once.
    constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    // instruction descriptor: D f32 (bit 4), A/B tf32 (2 << 7, 2 << 10), K-major both, N >> 3, M >> 4
    constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t) (BN >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);
    constexpr uint32_t IDESC2 = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t) ((2 * BN) >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);
    static_assert(2 * BN <= 256 && B_BYTES % 1024 == 0, "the stacked B operand is one MMA's N (at most 256) in whole swizzle groups");
    // split-K: every thread reduces and stores PER float4 of the CTA's rows in one pass (at most 64 rows x BN at 2 splits)
    constexpr int C4 = BN / 4, NT = GEMM_THREADS, PER = (split_rows(2) * C4 + NT - 1) / NT;

    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    constexpr int PLD = BN + 4;            // padded row of the staged partial tile (conflict-free float4 row writes)
    float * tile = (float *) smem;         // the staged accumulator tile [BM][PLD], in the idle pipeline buffers
    // split-K: the peers' partials [splits - 1][R][PLD]; peer q's rows go to slot q (q < this rank) or q - 1
    float * recv = (float *) (smem + (size_t) STAGES * STAGE_BYTES);
    static_assert((size_t) BM * PLD * 4 <= (size_t) STAGES * STAGE_BYTES, "staged tile must fit in the pipeline buffers");
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t rawf_bar[STAGES];   // block planes: the raw B tile has landed
    __shared__ __align__(8) uint64_t raw_bar[STAGES];    // block planes: the converters hold the raw tile
    __shared__ __align__(8) uint64_t conv_bar[STAGES];   // block planes: B_hi / B_lo written
    __shared__ __align__(8) uint64_t acc_bar;
    __shared__ __align__(8) uint64_t recv_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int num_k = (K + BK - 1) / BK;
    const int split = splits > 1 ? (int) cluster_rank() : 0;
    const int kt_per = (num_k + splits - 1) / splits;
    const int kt0 = split * kt_per, kt1 = min(num_k, kt0 + kt_per);
    const int nkt = kt1 > kt0 ? kt1 - kt0 : 0;
    const int R = split_rows(splits);
    const int rs = split * R, re = min(BM, rs + R);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1);
            mbar_init(&rawf_bar[s], 1); mbar_init(&raw_bar[s], CONV_WARPS); mbar_init(&conv_bar[s], CONV_WARPS);
        }
        mbar_init(&acc_bar, 1);
        mbar_init(&recv_bar, 1);
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        // the partial rows the peers push here: (splits - 1) x this CTA's rows x BN floats
        if (splits > 1) mbar_expect_tx(&recv_bar, (uint32_t) ((splits - 1) * max(0, re - rs) * PLD * 4));
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base_sh)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tA_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tA_lo) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tB_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tB_lo) : "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (splits > 1) cluster_arrive_release();   // the receive barriers are initialised
    const uint32_t tmem = tmem_base_sh;
    // B operands that do not come from the preceding kernel (weights): the first stages' B tiles are
    // requested before the dependency wait, while that kernel still runs
    const int pre_stages = ep.pre_b ? min(STAGES, nkt) : 0;
    if (warp == 0 && lane == 0) {
        for (int i = 0; i < pre_stages; i++) {
            uint8_t * st = smem + (size_t) i * STAGE_BYTES;
            if (qb) {
                mbar_expect_tx(&rawf_bar[i], raw_tx);
                load_raw_b<BN, QB>(st + 2 * A_BYTES + B_BYTES, &tB_hi, &tB_lo, qd, kt0 + i, n0, &rawf_bar[i]);
            } else {
                mbar_expect_tx(&full_bar[i], STAGE_BYTES);
                tma_load_2d(st + 2 * A_BYTES, &tB_hi, (kt0 + i) * BK, n0, &full_bar[i]);
                tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tB_lo, (kt0 + i) * BK, n0, &full_bar[i]);
            }
        }
    }
    // split-K: the first round of this thread's epilogue items, and their operands
    const int n_items = splits > 1 && re > rs ? (re - rs) * C4 : 0;
    const bool items = n_items > 0;
    Epi4In in[PER];
    auto prefetch = [&]() {
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int idx = j * NT + (int) threadIdx.x;
            if (idx >= n_items) continue;
            const int row = m0 + rs + idx / C4, col = n0 + (idx % C4) * 4;
            if (row < M && ep.vec && col + 3 < N) in[j] = epi_load4<MODE>(ep, row, col);
        }
    };
    if (ep.pre_epi && items) prefetch();
    // the setup above overlapped the previous kernel (programmatic dependent launch); its outputs are
    // read from here on. The converter warps of a weight in block planes read the weight and shared memory
    // only: they convert the stages whose raw tiles were requested early while that kernel still runs, and
    // wait for it after their loop (their epilogue items' operands are read from there on). No thread lets
    // the next kernel launch before it has waited: that kernel's early reads assume this one's predecessor
    // has finished.
    const bool conv_early = qb && warp >= 6 && warp < 6 + CONV_WARPS;
    if (!conv_early) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (!ep.pre_epi && items) prefetch();
    }

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nkt; i++) {
                const int kt = kt0 + i;
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t) (i / STAGES) & 1u;
                if (i >= STAGES && !mbar_wait(&empty_bar[s], ph ^ 1u, 1, &g_gemm_error)) { abort_sh = 1; break; }
                // a stage whose B tiles are in flight always gets its A tiles (so that its barrier completes)
                if (i >= pre_stages && *(volatile int *) &abort_sh) break;
                uint8_t * st = smem + (size_t) s * STAGE_BYTES;
                if (i >= pre_stages) {
                    if (qb) {
                        mbar_expect_tx(&rawf_bar[s], raw_tx);
                        load_raw_b<BN, QB>(st + 2 * A_BYTES + B_BYTES, &tB_hi, &tB_lo, qd, kt, n0, &rawf_bar[s]);
                    } else {
                        mbar_expect_tx(&full_bar[s], STAGE_BYTES);
                        tma_load_2d(st + 2 * A_BYTES, &tB_hi, kt * BK, n0, &full_bar[s]);
                        tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tB_lo, kt * BK, n0, &full_bar[s]);
                    }
                }
                if (qb) mbar_expect_tx(&full_bar[s], 2 * A_BYTES);
                tma_load_2d(st, &tA_hi, kt * BK, m0, &full_bar[s]);
                tma_load_2d(st + A_BYTES, &tA_lo, kt * BK, m0, &full_bar[s]);
                issued = i + 1;
            }
            if (*(volatile int *) &abort_sh) {
                // drain: the copies of the last stages it armed must land before the buffers are reused
                for (int i = issued - STAGES < 0 ? 0 : issued - STAGES; i < issued; i++) {
                    mbar_wait(&full_bar[i % STAGES], (uint32_t) (i / STAGES) & 1u, 5, &g_gemm_error);
                    if (qb) mbar_wait(&rawf_bar[i % STAGES], (uint32_t) (i / STAGES) & 1u, 5, &g_gemm_error);
                }
            }
        }
        __syncwarp();
        if (splits > 1) cluster_wait();
    } else if (warp == 1) {
        if (lane == 0) {
            for (int i = 0; i < nkt; i++) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t) (i / STAGES) & 1u;
                if (!mbar_wait(&full_bar[s], ph, 2, &g_gemm_error) ||
                    (qb && !mbar_wait_spin(&conv_bar[s], ph, 2, &g_gemm_error))) { abort_sh = 1; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a_hi = smem_u32(smem + (size_t) s * STAGE_BYTES);
                const uint32_t a_lo = a_hi + A_BYTES, b_hi = a_hi + 2 * A_BYTES;   // B_lo follows B_hi
#pragma unroll
                for (int kk = 0; kk < BK / 8; kk++) {
                    const uint32_t off = (uint32_t) kk * 32;   // 8 tf32 = 32 bytes along K
                    const uint64_t dah = sw128_desc(a_hi + off), dal = sw128_desc(a_lo + off);
                    const uint64_t dbh = sw128_desc(b_hi + off);
                    mma_kind_tf32(tmem, dah, dbh, IDESC2, (i | kk) != 0);   // [hi*hi | hi*lo], 2 BN wide
                    mma_kind_tf32(tmem + BN, dal, dbh, IDESC, 1);          // + lo*hi (B_hi rows only)
                }
                mma_commit(&empty_bar[s]);
            }
            mma_commit(&acc_bar);   // also on abort / with no K-slice: completes once the issued MMAs are done
        }
        __syncwarp();
        if (splits > 1) cluster_wait();
    } else if (warp >= 6) {
        if (qb && warp < 6 + CONV_WARPS) {
            // converter warps: the raw B tile of every stage into its split planes
            const int ct = (int) threadIdx.x - 6 * 32;
            for (int i = 0; i < nkt; i++) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t) (i / STAGES) & 1u;
                if (!mbar_wait_spin(&rawf_bar[s], ph, 6, &g_gemm_error) ||
                    !convert_stage<BN, 32 * CONV_WARPS, QB>(smem + (size_t) s * STAGE_BYTES + 2 * A_BYTES, qd, ct, lane, &raw_bar[s], ph)) {
                    abort_sh = 1;
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv_bar[s]);
            }
        }
        if (conv_early) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
            if (!ep.pre_epi && items) prefetch();
        }
        if (splits > 1) cluster_wait();   // (the start's arrive; these warps join at the reduction)
    } else {
        // epilogue warps 2..5 (TMEM lane quadrant = warp % 4)
        const int q = warp & 3;
        const bool ok = mbar_wait(&acc_bar, 0, 3, &g_gemm_error);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int r = q * 32 + lane;
        const bool have = ok && nkt > 0 && !*(volatile int *) &abort_sh;
        const uint32_t trow = tmem + ((uint32_t) (q * 32) << 16);
        if constexpr (BN == 64) {
            if (splits > 1) {
                // both accumulators' 64 columns in flight at once, then this thread's row of the partial tile
                uint32_t a0[32], a1[32], b0[32], b1[32];
                tmem_ld32_async(trow, a0);
                tmem_ld32_async(trow + 32, a1);
                tmem_ld32_async(trow + BN, b0);
                tmem_ld32_async(trow + BN + 32, b1);
                tmem_ld_wait(a0);
                tmem_ld_wait(a1);
                tmem_ld_wait(b0);
                tmem_ld_wait(b1);
                auto stage = [&](const uint32_t (&x)[32], const uint32_t (&y)[32], int c0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 v = have ? make_float4(__uint_as_float(x[j]) + __uint_as_float(y[j]),
                                                            __uint_as_float(x[j + 1]) + __uint_as_float(y[j + 1]),
                                                            __uint_as_float(x[j + 2]) + __uint_as_float(y[j + 2]),
                                                            __uint_as_float(x[j + 3]) + __uint_as_float(y[j + 3]))
                                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        *(float4 *) &tile[r * PLD + c0 + j] = v;
                    }
                };
                stage(a0, b0, 0);
                stage(a1, b1, 32);
            }
        }
        if (splits == 1) {
            // one CTA per tile: the accumulator goes to shared memory a row per thread, and all twelve warps
            // apply the fused epilogue from there row-major (coalesced loads and stores, after the sync below)
            if (!have) abort_sh = 1;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t a[32], b[32];
                tmem_ld32_async(trow + (uint32_t) c0, a);
                tmem_ld32_async(trow + (uint32_t) (BN + c0), b);
                tmem_ld_wait(a);
                tmem_ld_wait(b);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    *(float4 *) &tile[r * PLD + c0 + j] = make_float4(__uint_as_float(a[j]) + __uint_as_float(b[j]),
                                                                      __uint_as_float(a[j + 1]) + __uint_as_float(b[j + 1]),
                                                                      __uint_as_float(a[j + 2]) + __uint_as_float(b[j + 2]),
                                                                      __uint_as_float(a[j + 3]) + __uint_as_float(b[j + 3]));
                }
            }
        }
        if (splits > 1) {
            // the staged rows of peer p go to it in one bulk copy: [p R, p R + R) x PLD floats, contiguous
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, 128;" ::: "memory");
            cluster_wait();   // every peer's receive barrier is initialised
            if (warp == 2 && lane < splits) {
                // one copy per lane: lane p sends peer p its rows (the copies are issued side by side)
                const int p = lane;
                const int prs = p * R, pre = min(BM, prs + R);
                if (p != split && pre > prs) {
                    const int slot = split < p ? split : split - 1;   // this CTA's slot in peer p's receive buffer
                    const uint32_t dst = peer_addr(smem_u32(recv + (size_t) slot * R * PLD), (uint32_t) p);
                    bulk_to_peer(dst, smem_u32(tile + (size_t) prs * PLD), (uint32_t) ((pre - prs) * PLD * 4),
                                 peer_addr(smem_u32(&recv_bar), (uint32_t) p));
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();   // the accumulator has been read (and this CTA's own partial rows are staged)
    if (splits == 1 && nkt > 0 && !*(volatile int *) &abort_sh) {
#pragma unroll 2
        for (int idx = (int) threadIdx.x; idx < BM * C4; idx += NT) {
            const int i = idx / C4, cc = (idx % C4) * 4;
            const int row = m0 + i;
            if (row < M) apply_epi4<MODE>(ep, row, n0 + cc, N, *(const float4 *) &tile[(size_t) i * PLD + cc]);
        }
    }
    if (splits > 1) {
        const bool got = mbar_wait(&recv_bar, 0, 4, &g_gemm_error);   // the peers' partial rows have landed
        cluster_arrive_relaxed();   // this CTA has received everything
        if (got && !*(volatile int *) &abort_sh) {
            {
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    const int idx = j * NT + (int) threadIdx.x;
                    if (idx >= n_items) continue;
                    const int i = idx / C4, cc = (idx % C4) * 4;
                    const int row = m0 + rs + i, col = n0 + cc;
                    // split p's partial: this CTA's own from the staged tile, the others from the receive buffer
                    auto part = [&](int p) -> float4 {
                        return p == split ? *(const float4 *) &tile[(size_t) (rs + i) * PLD + cc]
                                          : *(const float4 *) &recv[((size_t) (p < split ? p : p - 1) * R + i) * PLD + cc];
                    };
                    float4 v = part(0);
#pragma unroll
                    for (int p = 1; p < 8; p++) {
                        if (p < splits) {
                            const float4 w = part(p);
                            v.x = v.x + w.x; v.y = v.y + w.y; v.z = v.z + w.z; v.w = v.w + w.w;
                        }
                    }
                    if (row >= M) continue;
                    if (ep.vec && col + 3 < N) epi_store4<MODE>(ep, row, col, v, in[j]);
                    else apply_epi4<MODE>(ep, row, col, N, v);
                }
            }
        }
        cluster_wait();   // every CTA has received everything: no push to or from this CTA is in flight
    }
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}


// Wide products (N, K >= 768) and wide outputs (N >= 4096): persistent, one CTA per SM walking 128 x 128
// tiles (n fastest, so CTAs that run side by side share A rows), no K split. Warp 0 issues the TMA loads
// (A_hi, A_lo, B_hi, B_lo; 64 KB a stage, 3 stages), one thread of warp 1 the MMAs -- per K-step one of
// N = 256 over the stacked B_hi|B_lo operand and one of N = 128 (the same two as the split kernel) -- into one
// of two 256-column TMEM accumulator pairs, so that warps 2..9 drain tile i (two warps per lane quadrant,
// 64 columns each) while tile i+1's products run. A draining warp stages 32 rows x 32 columns in its own
// 4 KB shared buffer (16-byte chunk c of row r at c ^ (r & 7)) and applies the fused epilogue from there
// four rows per instruction: coalesced loads and stores. A tile's arithmetic is the split kernel's at
// one split (the same MMAs in the same order), so a row's bits do not depend on the batch.
constexpr int PBN = 128, PSTAGES = 3, PEPI_WARPS = 8, PTHREADS = 64 + 32 * PEPI_WARPS;
constexpr int PTHREADS_QB = PTHREADS + 32 * PCONV_WARPS;   // with the converter warps
constexpr int FIX_ROWS = 4;   // K-split fix-up: row groups of partial tiles loaded at once per lane
constexpr int PGROUP_M = 16;  // row tiles per group of the m-fastest tile order (2048 rows: 12.6 MB of A planes at K = 768)
constexpr uint32_t PSTAGE_BYTES = 2 * BM * BK * 4 + 2 * PBN * BK * 4;
constexpr size_t PSMEM_BYTES = (size_t) PSTAGES * PSTAGE_BYTES + (size_t) PEPI_WARPS * 32 * 32 * 4 + 1024;
static_assert(PSMEM_BYTES + 256 <= 227 * 1024, "persistent tf32x3 GEMM: stages and staging buffers fit");

// Origin (first row, first column) of output tile t in the persistent kernel's walk: n-fastest (the CTAs side
// by side share an A row tile) or, for m_fast, groups of PGROUP_M row tiles walked m-fastest, the last group
// holding the row tiles left over (the CTAs side by side share a B column tile). Host and device share it, so
// the host can check that a walk visits every output tile once.
__host__ __device__ inline void p_tile_origin(int t, int tiles_m, int tiles_n, int m_fast, int & m0, int & n0) {
    if (m_fast) {
        const int g = t / (PGROUP_M * tiles_n), r = t - g * PGROUP_M * tiles_n;
        const int left = tiles_m - g * PGROUP_M;
        const int gm = left < PGROUP_M ? left : PGROUP_M;
        m0 = (g * PGROUP_M + r % gm) * BM;
        n0 = (r / gm) * PBN;
    } else {
        m0 = (t / tiles_n) * BM;
        n0 = (t % tiles_n) * PBN;
    }
}

template <int MODE, bool QB>
__global__ void __launch_bounds__(QB ? PTHREADS_QB : PTHREADS, 1)
k_gemm_tf32x3_p(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo,
                int M, int N, int K, int splits, int m_fast, const QDesc qd, const __grid_constant__ GemmEpi ep) {
    constexpr uint32_t A_BYTES = BM * BK * 4;
    constexpr uint32_t B_BYTES = PBN * BK * 4;
    constexpr uint32_t TMEM_COLS = 4 * PBN;   // two accumulator pairs [hi*hi | cross terms], 256 columns each
    constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t) (PBN >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);
    constexpr uint32_t IDESC2 = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t) ((2 * PBN) >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);

    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    __shared__ __align__(8) uint64_t full_bar[PSTAGES];
    __shared__ __align__(8) uint64_t empty_bar[PSTAGES];
    __shared__ __align__(8) uint64_t rawf_bar[PSTAGES];   // block planes: the raw B tile has landed
    __shared__ __align__(8) uint64_t raw_bar[PSTAGES];    // block planes: the converters hold the raw tile
    __shared__ __align__(8) uint64_t conv_bar[PSTAGES];   // block planes: B_hi / B_lo written
    __shared__ __align__(8) uint64_t accf_bar[2];   // MMA -> epilogue: accumulator pair b holds a finished tile
    __shared__ __align__(8) uint64_t acce_bar[2];   // epilogue -> MMA: accumulator pair b has been read
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;
    __shared__ int epi_stop_sh, last_sh;   // K split: the epilogue warps' common abort decision; "this part sums"

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_k = (K + BK - 1) / BK;
    const int tiles_n = (N + PBN - 1) / PBN, tiles_m = (M + BM - 1) / BM;
    // work units: unit u is K-part u % splits of output tile u / splits (splits == 1: whole tiles): a tile's parts
    // run side by side, its A rows and B slice shared in L2. Tiles in n-fastest order, or, for a wide output
    // whose B operand is too large to stay in L2 (m_fast), in groups of row tiles walked m-fastest: a B column
    // tile is read from DRAM once per group rather than once per row tile, and the group's A rows stay in L2
    auto tile_origin = [&](int t, int & m0, int & n0) { p_tile_origin(t, tiles_m, tiles_n, m_fast, m0, n0); };
    const int total = ((M + BM - 1) / BM) * tiles_n * splits;
    const int kq = (num_k + splits - 1) / splits;
    const bool qb = QB && qd.fmt != QF_NONE;   // block planes (a template switch: the plane kernels carry no converter code)

    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; s++) {
            mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1);
            mbar_init(&rawf_bar[s], 1); mbar_init(&raw_bar[s], PCONV_WARPS); mbar_init(&conv_bar[s], PCONV_WARPS);
        }
        for (int b = 0; b < 2; b++) { mbar_init(&accf_bar[b], 1); mbar_init(&acce_bar[b], PEPI_WARPS); }
        abort_sh = 0;
        epi_stop_sh = 0;
        last_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base_sh)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tA_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tA_lo) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tB_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"((uint64_t) &tB_lo) : "memory");
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
            for (int u = blockIdx.x; u < total && !*(volatile int *) &abort_sh; u += gridDim.x) {
                const int t = u / splits, part = u % splits;
                int m0, n0;
                tile_origin(t, m0, n0);
                const int kb = part * kq, ke = min(num_k, kb + kq);
                for (int k = kb; k < ke; k++, kt++) {
                    const int s = kt % PSTAGES;
                    const uint32_t ph = (uint32_t) (kt / PSTAGES) & 1u;
                    if (kt >= PSTAGES && !mbar_wait(&empty_bar[s], ph ^ 1u, 1, &g_gemm_error)) { abort_sh = 1; break; }
                    if (*(volatile int *) &abort_sh) break;
                    uint8_t * st = smem + (size_t) s * PSTAGE_BYTES;
                    if (qb) {
                        // the raw B tile first, on its own barrier: the converters are on the critical path
                        mbar_expect_tx(&rawf_bar[s], PBN * raw_row_bytes(qd.fmt) + raw_scale_bytes(qd.fmt, PBN));
                        load_raw_b<PBN, QB>(st + 2 * A_BYTES + B_BYTES, &tB_hi, &tB_lo, qd, k, n0, &rawf_bar[s]);
                        mbar_expect_tx(&full_bar[s], 2 * A_BYTES);
                        tma_load_2d(st, &tA_hi, k * BK, m0, &full_bar[s]);
                        tma_load_2d(st + A_BYTES, &tA_lo, k * BK, m0, &full_bar[s]);
                    } else {
                        mbar_expect_tx(&full_bar[s], PSTAGE_BYTES);
                        tma_load_2d(st, &tA_hi, k * BK, m0, &full_bar[s]);
                        tma_load_2d(st + A_BYTES, &tA_lo, k * BK, m0, &full_bar[s]);
                        tma_load_2d(st + 2 * A_BYTES, &tB_hi, k * BK, n0, &full_bar[s]);
                        tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tB_lo, k * BK, n0, &full_bar[s]);
                    }
                }
            }
            if (*(volatile int *) &abort_sh) {
                // let the copies already issued land before the CTA exits
                for (int j = kt - PSTAGES < 0 ? 0 : kt - PSTAGES; j < kt; j++) {
                    mbar_wait(&full_bar[j % PSTAGES], (uint32_t) (j / PSTAGES) & 1u, 5, &g_gemm_error);
                    if (qb) mbar_wait(&rawf_bar[j % PSTAGES], (uint32_t) (j / PSTAGES) & 1u, 5, &g_gemm_error);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int kt = 0, i = 0;
            for (int u = blockIdx.x; u < total && !*(volatile int *) &abort_sh; u += gridDim.x, i++) {
                const int b = i & 1;
                const int kb = (u % splits) * kq, ke = min(num_k, kb + kq);
                if (i >= 2 && !mbar_wait(&acce_bar[b], (uint32_t) ((i >> 1) - 1) & 1u, 4, &g_gemm_error)) { abort_sh = 1; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t) (b * 2 * PBN);
                for (int k = kb; k < ke; k++, kt++) {
                    const int s = kt % PSTAGES;
                    const uint32_t ph = (uint32_t) (kt / PSTAGES) & 1u;
                    if (!mbar_wait(&full_bar[s], ph, 2, &g_gemm_error) ||
                        (qb && !mbar_wait_spin(&conv_bar[s], ph, 2, &g_gemm_error))) { abort_sh = 1; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a_hi = smem_u32(smem + (size_t) s * PSTAGE_BYTES);
                    const uint32_t a_lo = a_hi + A_BYTES, b_hi = a_hi + 2 * A_BYTES;   // B_lo follows B_hi
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++) {
                        const uint32_t off = (uint32_t) kk * 32;
                        const uint64_t dbh = sw128_desc(b_hi + off);
                        mma_kind_tf32(d, sw128_desc(a_hi + off), dbh, IDESC2, ((k - kb) | kk) != 0);   // [hi*hi | hi*lo]
                        mma_kind_tf32(d + PBN, sw128_desc(a_lo + off), dbh, IDESC, 1);                  // + lo*hi
                    }
                    mma_commit(&empty_bar[s]);
                }
                if (*(volatile int *) &abort_sh) break;
                mma_commit(&accf_bar[b]);
            }
        }
    } else if (warp >= 2 + PEPI_WARPS) {
        if (qb) {
            // converter warps: the raw B tile of every stage into its split planes, in the producer's order
            const int ct = (int) threadIdx.x - (2 + PEPI_WARPS) * 32;
            int kt = 0;
            for (int u = blockIdx.x; u < total && !*(volatile int *) &abort_sh; u += gridDim.x) {
                const int kb = (u % splits) * kq, ke = min(num_k, kb + kq);
                bool good = true;
                for (int k = kb; k < ke; k++, kt++) {
                    const int s = kt % PSTAGES;
                    const uint32_t ph = (uint32_t) (kt / PSTAGES) & 1u;
                    if (!mbar_wait_spin(&rawf_bar[s], ph, 6, &g_gemm_error) ||
                        !convert_stage<PBN, 32 * PCONV_WARPS, QB>(smem + (size_t) s * PSTAGE_BYTES + 2 * A_BYTES, qd, ct, lane, &raw_bar[s], ph)) {
                        good = false;
                        break;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&conv_bar[s]);
                }
                if (!good) { abort_sh = 1; break; }
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lane quadrant this warp may read
        const int half = (warp - 2) >> 2;       // which 64 of the tile's 128 columns
        float * stage = (float *) (smem + (size_t) PSTAGES * PSTAGE_BYTES + (size_t) (warp - 2) * 32 * 32 * 4);
        const uint32_t trow = tmem + ((uint32_t) (q * 32) << 16);
        int i = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x, i++) {
            const int b = i & 1;
            const int t = u / splits, part = u % splits;
            const bool ok = mbar_wait(&accf_bar[b], (uint32_t) (i >> 1) & 1u, 3, &g_gemm_error);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (splits > 1) {
                // the eight epilogue warps decide together, so that none waits at a barrier another has left
                if (!ok || *(volatile int *) &abort_sh) epi_stop_sh = 1;
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (*(volatile int *) &epi_stop_sh) { abort_sh = 1; break; }
            } else if (!ok || *(volatile int *) &abort_sh) {
                abort_sh = 1;
                break;
            }
            int m0, n0;
            tile_origin(t, m0, n0);
            const int row0 = m0 + q * 32;
            if (splits > 1) {
                // this part's partial tile (hi*hi + cross terms) into its scratch slot, row-major
                float * slot = ep.fix + ((size_t) t * splits + part) * (size_t) (BM * PBN);
#pragma unroll 1
                for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
                    uint32_t x[32], y[32];
                    tmem_ld32_async(trow + (uint32_t) (b * 2 * PBN + c0), x);
                    tmem_ld32_async(trow + (uint32_t) (b * 2 * PBN + PBN + c0), y);
                    tmem_ld_wait(x);
                    tmem_ld_wait(y);
                    if (c0 == half * 64 + 32) {
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acce_bar[b]);
                    }
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        *(float4 *) &stage[lane * 32 + ((c ^ (lane & 7)) << 2)] =
                            make_float4(__uint_as_float(x[4 * c]) + __uint_as_float(y[4 * c]),
                                        __uint_as_float(x[4 * c + 1]) + __uint_as_float(y[4 * c + 1]),
                                        __uint_as_float(x[4 * c + 2]) + __uint_as_float(y[4 * c + 2]),
                                        __uint_as_float(x[4 * c + 3]) + __uint_as_float(y[4 * c + 3]));
                    }
                    __syncwarp();
#pragma unroll 4
                    for (int j = 0; j < 8; j++) {
                        const int idx = j * 32 + lane, r = idx >> 3, c = idx & 7;
                        __stcg((float4 *) (slot + (size_t) (q * 32 + r) * PBN + c0 + 4 * c),
                               *(const float4 *) &stage[r * 32 + ((c ^ (r & 7)) << 2)]);
                    }
                }
                __threadfence();
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (warp == 2 && lane == 0) {
                    const int before = atomicAdd(&ep.fix_count[t], 1);
                    last_sh = before == splits - 1;
                    if (last_sh) ep.fix_count[t] = 0;   // every part has counted: ready for the next launch
                }
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (!last_sh) continue;
                // the last part to finish: the parts summed in order 0, 1, ..., then the fused epilogue
                __threadfence();
                const float * parts = ep.fix + (size_t) t * splits * (size_t) (BM * PBN);
                if (row0 >= M || n0 + half * 64 >= N) continue;   // warp-uniform
                // FIX_ROWS groups of every part's values are loaded before any is summed, so that a lane waits
                // out one L2 round trip per group of loads rather than one per load (every slot row exists:
                // the parts write whole tiles)
#pragma unroll 1
                for (int j0 = 0; j0 < 16; j0 += FIX_ROWS) {
                    float4 v[FIX_ROWS][GEMM_KSPLIT_MAX];
#pragma unroll
                    for (int jj = 0; jj < FIX_ROWS; jj++) {
                        const int idx = (j0 + jj) * 32 + lane, r = idx >> 4, c = idx & 15;
                        const float * p0 = parts + (size_t) (q * 32 + r) * PBN + half * 64 + 4 * c;
#pragma unroll
                        for (int p = 0; p < GEMM_KSPLIT_MAX; p++) {
                            if (p < splits) v[jj][p] = __ldcg((const float4 *) (p0 + (size_t) p * (BM * PBN)));
                        }
                    }
#pragma unroll
                    for (int jj = 0; jj < FIX_ROWS; jj++) {
                        const int idx = (j0 + jj) * 32 + lane, r = idx >> 4, c = idx & 15;
                        const int row = row0 + r, col = half * 64 + 4 * c;
                        float4 acc = v[jj][0];
#pragma unroll
                        for (int p = 1; p < GEMM_KSPLIT_MAX; p++) {
                            if (p < splits) acc = f4_add(acc, v[jj][p]);   // parts in order 0, 1, ...
                        }
                        if (row < M) apply_epi4<MODE>(ep, row, n0 + col, N, acc);
                    }
                }
                continue;
            }
#pragma unroll 1
            for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
                uint32_t x[32], y[32];
                tmem_ld32_async(trow + (uint32_t) (b * 2 * PBN + c0), x);
                tmem_ld32_async(trow + (uint32_t) (b * 2 * PBN + PBN + c0), y);
                tmem_ld_wait(x);
                tmem_ld_wait(y);
                if (c0 == half * 64 + 32) {
                    // the tile's last accumulator read by this warp: the MMA warp may refill the pair
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acce_bar[b]);
                }
                __syncwarp();   // the previous block's reads of the staging buffer are done
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    *(float4 *) &stage[lane * 32 + ((c ^ (lane & 7)) << 2)] =
                        make_float4(__uint_as_float(x[4 * c]) + __uint_as_float(y[4 * c]),
                                    __uint_as_float(x[4 * c + 1]) + __uint_as_float(y[4 * c + 1]),
                                    __uint_as_float(x[4 * c + 2]) + __uint_as_float(y[4 * c + 2]),
                                    __uint_as_float(x[4 * c + 3]) + __uint_as_float(y[4 * c + 3]));
                }
                __syncwarp();
                if (row0 >= M || n0 + c0 >= N) continue;   // warp-uniform
#pragma unroll 4
                for (int j = 0; j < 8; j++) {
                    const int idx = j * 32 + lane, r = idx >> 3, c = idx & 7;
                    const int row = row0 + r;
                    if (row < M) apply_epi4<MODE>(ep, row, n0 + c0 + 4 * c, N, *(const float4 *) &stage[r * 32 + ((c ^ (r & 7)) << 2)]);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool load_encode() {
    std::call_once(g_encode_once, []() {
        void * fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode = (PFN_cuTensorMapEncodeTiled_v12000) fn;
        }
    });
    return g_encode != nullptr;
}

bool make_map(CUtensorMap * map, const float * base, int rows, int cols, int ld, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) ld * 4};
    const cuuint32_t box[2] = {(cuuint32_t) BK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *) base, dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// a row-major 2-D map without swizzle over raw block values or scales: `inner` elements of type dt per row,
// rows `stride` bytes apart, boxes of box_inner x box_rows
bool make_raw_map(CUtensorMap * map, const void * base, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                  uint64_t stride, uint32_t box_inner, uint32_t box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t) inner, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode(map, dt, 2, (void *) base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The B operand's two maps for tiles of `bn` rows: its split planes (hi, lo), or a weight's block values
// and scales (QuantB; qd says which). False with a log line when a map cannot be made.
bool make_b_maps(const SplitMat & B, int N, int K, int bn, CUtensorMap * t0, CUtensorMap * t1, QDesc * qd) {
    *qd = QDesc{};
    if (!B.q.fmt) return make_map(t0, B.hi, N, K, B.ld, bn) && make_map(t1, B.lo, N, K, B.ld, bn);
    const QuantB & q = B.q;
    if (K % 32 || (q.orient == 1 && N % 32) || (q.orient == 0 && N % 8) || !q.q || (q.fmt != QF_F16 && !q.d)) {
        log("jepa: gemm: block-plane operand of N %d K %d (orientation %d) is not in whole blocks\n", N, K, q.orient);
        return false;
    }
    qd->fmt = q.fmt;
    qd->orient = q.orient;
    bool ok;
    if (q.fmt == QF_Q8) ok = make_raw_map(t0, q.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t) K, (uint64_t) N, (uint64_t) K, 32, (uint32_t) bn);
    else if (q.fmt == QF_Q4) ok = make_raw_map(t0, q.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t) K / 2, (uint64_t) N, (uint64_t) K / 2, 16, (uint32_t) bn);
    else ok = make_raw_map(t0, q.q, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t) K, (uint64_t) N, (uint64_t) K * 2, 32, (uint32_t) bn);
    if (ok && q.fmt != QF_F16) {
        ok = q.orient == 0 ? make_raw_map(t1, q.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t) N, (uint64_t) K / 32, (uint64_t) N * 2, (uint32_t) bn, 1)
                           : make_raw_map(t1, q.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t) K, (uint64_t) N / 32, (uint64_t) K * 2, 32, (uint32_t) bn / 32);
    } else if (ok) {
        *t1 = *t0;   // f16: no scales (the map is never used)
    }
    if (!ok) log("jepa: gemm: cuTensorMapEncodeTiled refused a block-plane operand (N %d K %d, format %d)\n", N, K, q.fmt);
    return ok;
}

// rows of the split-K receive buffer: (splits - 1) x ceil(128 / splits), at most 114 (7 splits)
constexpr int recv_rows() {
    int r = 0;
    for (int s = 2; s <= 8; s++) r = (s - 1) * split_rows(s) > r ? (s - 1) * split_rows(s) : r;
    return r;
}

template <int BN, int STAGES>
constexpr size_t smem_bytes() {
    // pipeline stages, the split-K receive buffer and alignment
    return (size_t) STAGES * (2 * BM * BK * 4 + 2 * BN * BK * 4) + (BN == 64 ? (size_t) recv_rows() * (BN + 4) * 4 : 0) + 1024;
}
static_assert(smem_bytes<64, 4>() + 256 <= 227 * 1024, "four 64-wide stages and the receive buffer fit in shared memory");

// the kernel's shared-memory and cluster attributes, once per device
template <int BN, int STAGES, int MODE, bool QB>
bool set_attrs() {
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        if (cudaFuncSetAttribute(k_gemm_tf32x3<BN, STAGES, MODE, QB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int) smem_bytes<BN, STAGES>()) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_tf32x3<BN, STAGES, MODE, QB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            return false;
        }
        done[dev] = true;
    }
    return true;
}

// How many split-K clusters of s CTAs of the 64-wide kernel the device holds at once. Clusters are
// placed inside one GPC, so this is below (SMs / s) when a GPC's SM count is not a multiple of s
// (on a 148-SM B200, 45 clusters of 3 rather than 49). Cached per device.
int resident_clusters(int s) {
    static std::mutex mu;
    static int cache[64][9] = {};
    int dev = 0;
    if (s < 1 || s > 8 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev][s]) {
        int n = 0;
        if (s == 1) {
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        } else if (set_attrs<64, 4, EPI_F32, false>()) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, 1, (unsigned) s);
            cfg.blockDim = dim3(GEMM_THREADS);
            cfg.dynamicSmemBytes = smem_bytes<64, 4>();
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 1;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = (unsigned) s;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, k_gemm_tf32x3<64, 4, EPI_F32, false>, &cfg) != cudaSuccess) n = 0;
        }
        cudaGetLastError();
        cache[dev][s] = n > 0 ? n : -1;
    }
    return cache[dev][s] > 0 ? cache[dev][s] : 0;
}

template <int BN, int STAGES, int MODE>
int launch(const SplitMat & A, const SplitMat & B, int M, int N, int K, int splits, const GemmEpi & ep, cudaStream_t st) {
    if (BN != 64 && splits > 1) { log("jepa: gemm: split-K needs the 64-wide tile\n"); return -1; }
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;
    QDesc qd;
    if (!make_map(&ta_hi, A.hi, M, K, A.ld, BM) || !make_map(&ta_lo, A.lo, M, K, A.ld, BM) ||
        !make_b_maps(B, N, K, BN, &tb_hi, &tb_lo, &qd)) {
        log("jepa: gemm: cuTensorMapEncodeTiled refused an operand (M %d N %d K %d, ld %d / %d)\n", M, N, K, A.ld, B.ld);
        return -1;
    }
    constexpr size_t smem = smem_bytes<BN, STAGES>();
    const bool qb = qd.fmt != QF_NONE;
    if (!(qb ? set_attrs<BN, STAGES, MODE, true>() : set_attrs<BN, STAGES, MODE, false>())) {
        log("jepa: gemm: cudaFuncSetAttribute failed\n");
        return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) ((M + BM - 1) / BM), (unsigned) ((N + BN - 1) / BN), (unsigned) splits);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = (unsigned) splits;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 2 : 1;
    if (qb) JB_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tf32x3<BN, STAGES, MODE, true>, ta_hi, ta_lo, tb_hi, tb_lo, M, N, K, splits, qd, ep));
    else JB_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tf32x3<BN, STAGES, MODE, false>, ta_hi, ta_lo, tb_hi, tb_lo, M, N, K, splits, qd, ep));
    return 0;
}

// The persistent kernel's tile order: grouped m-fastest for wide outputs (N >= 4096) whose B operand (N x K
// hi / lo planes) is too large to stay in L2 (above 48 MB: the adaLN modulation's 340 MB at config 5), when there
// is more than one row tile; n-fastest otherwise. Measured at N 55,296 K 768: 2048 rows 904 -> 616 us, 8192 rows
// 3577 -> 2475 us; the narrow adaLN backward (N 768) keeps n-fastest (626 against 650 us m-fastest).
int p_tile_order(int M, int N, int K) {
    return N >= 4096 && (size_t) N * (size_t) K * 8 > ((size_t) 48 << 20) && (M + BM - 1) / BM > 1 ? 1 : 0;
}

template <int MODE>
int launch_p(const SplitMat & A, const SplitMat & B, int M, int N, int K, int splits, const GemmEpi & ep, cudaStream_t st) {
    if (splits < 1 || splits > GEMM_KSPLIT_MAX) { log("jepa: gemm: %d K parts (at most %d)\n", splits, GEMM_KSPLIT_MAX); return -1; }
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;
    QDesc qd;
    if (!make_map(&ta_hi, A.hi, M, K, A.ld, BM) || !make_map(&ta_lo, A.lo, M, K, A.ld, BM) ||
        !make_b_maps(B, N, K, PBN, &tb_hi, &tb_lo, &qd)) {
        log("jepa: gemm: cuTensorMapEncodeTiled refused an operand (M %d N %d K %d, ld %d / %d)\n", M, N, K, A.ld, B.ld);
        return -1;
    }
    static std::mutex mu;
    static bool done[64] = {};
    static int sms[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!done[dev]) {
            JB_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3_p<MODE, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) PSMEM_BYTES));
            JB_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3_p<MODE, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) PSMEM_BYTES));
            JB_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
            done[dev] = true;
        }
    }
    const long units = (long) ((M + BM - 1) / BM) * ((N + PBN - 1) / PBN) * splits;
    const unsigned grid = (unsigned) std::max(1L, std::min<long>(units, sms[dev]));
    const int m_fast = p_tile_order(M, N, K);
    if (qd.fmt != QF_NONE) {
        JB_CUDA(launch_pdl(k_gemm_tf32x3_p<MODE, true>, dim3(grid), dim3(PTHREADS_QB), PSMEM_BYTES, st, ta_hi, ta_lo, tb_hi, tb_lo,
                           M, N, K, splits, m_fast, qd, ep));
    } else {
        JB_CUDA(launch_pdl(k_gemm_tf32x3_p<MODE, false>, dim3(grid), dim3(PTHREADS), PSMEM_BYTES, st, ta_hi, ta_lo, tb_hi, tb_lo,
                           M, N, K, splits, m_fast, qd, ep));
    }
    return 0;
}

int launch_p_mode(const SplitMat & A, const SplitMat & B, int M, int N, int K, int splits, const GemmEpi & ep, cudaStream_t st) {
    switch (ep.mode) {
        case EPI_F32: return launch_p<EPI_F32>(A, B, M, N, K, splits, ep, st);
        case EPI_SPLIT: return launch_p<EPI_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GELU_SPLIT: return launch_p<EPI_GELU_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GATED: return launch_p<EPI_GATED>(A, B, M, N, K, splits, ep, st);
        case EPI_DGELU_SPLIT: return launch_p<EPI_DGELU_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_F32_SPLIT: return launch_p<EPI_F32_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GELU_D_SPLIT: return launch_p<EPI_GELU_D_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_MUL_SPLIT: return launch_p<EPI_MUL_SPLIT>(A, B, M, N, K, splits, ep, st);
        default: log("jepa: gemm: unknown epilogue mode %d\n", ep.mode); return -1;
    }
}

// the persistent kernel's K split of a shape (1 = none): narrow (at most 8 column tiles), long (K >= 2048)
// products, which have too few output tiles to fill the device at planner row counts and enough K per part
// that the partial-tile round trip is small beside it. Measured on a B200 (us per launch, rows 256 / 1024 /
// 2048): N 768 K 3072 unsplit 45.8 / 46.1 / 53.7, in three parts 23.1 / 24.5 / 46.0; K 55,296 at 2048 rows
// 894 -> 629. At K = 768 the split loses at 2048 rows (15.9 -> 22.4), and the 3072-wide products (24 column
// tiles) lose from 512 rows on, so those keep whole tiles.
int p_splits(int N, int K) {
    const bool persistent = N >= 4096 || (N >= 768 && K >= 768);
    return persistent && (N + PBN - 1) / PBN <= 8 && K >= 2048 ? GEMM_KSPLIT : 1;
}

}  // namespace

// Which kernel a product takes (host arithmetic on the shape alone). Wide outputs (the adaLN modulation of
// every step at once) and wide products (output and reduction both at least 768: the widest predictors,
// which plan thousands of candidates, so there are tiles enough to fill the device) take the persistent
// kernel's 128 x 128 tiles: twice the columns per A tile read, no exchange, and each tile's epilogue
// overlapping the next tile's products. With at most two row tiles (a 4096-candidate level split over 8
// GPUs: two chains of 256 rows) a product narrower than 4096 has too few such tiles for the device and takes
// the split-K clusters instead (measured at 256 rows, us per launch: N 768 K 768 15.7 -> 7.8, N 3072 K 768
// 15.7 -> 14.0, N 768 K 3072 23.7 -> 14.1, N 768 K 55,296 317 -> 153; at 384 rows and more the persistent
// kernel wins or ties).
GemmPlan gemm_plan(int M, int N, int K) {
    GemmPlan p;
    const bool few_rows = M <= 2 * BM && N < 4096;
    p.persistent = (N >= 4096 || (N >= 768 && K >= 768)) && !few_rows;
    p.k_parts = p.persistent ? p_splits(N, K) : 0;
    p.m_fast = p.persistent ? p_tile_order(M, N, K) : 0;
    return p;
}

int gemm_tile_walk(int M, int N, int K, int * m0, int * n0, int cap) {
    const GemmPlan p = gemm_plan(M, N, K);
    if (!p.persistent) return 0;
    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + PBN - 1) / PBN;
    const long total = (long) tiles_m * tiles_n;
    if (total > cap) return -1;
    for (int t = 0; t < (int) total; t++) p_tile_origin(t, tiles_m, tiles_n, p.m_fast, m0[t], n0[t]);
    return (int) total;
}

size_t gemm_fixup_floats(int M, int N, int K) {
    const int s = p_splits(N, K);
    return s > 1 ? (size_t) ((M + BM - 1) / BM) * ((N + PBN - 1) / PBN) * s * (BM * PBN) : 0;
}

size_t gemm_fixup_counters(int M, int N, int K) {
    return p_splits(N, K) > 1 ? (size_t) ((M + BM - 1) / BM) * ((N + PBN - 1) / PBN) : 0;
}

namespace {

// one kernel per epilogue mode
template <int BN, int STAGES>
int launch_mode(const SplitMat & A, const SplitMat & B, int M, int N, int K, int splits, const GemmEpi & ep, cudaStream_t st) {
    switch (ep.mode) {
        case EPI_F32: return launch<BN, STAGES, EPI_F32>(A, B, M, N, K, splits, ep, st);
        case EPI_SPLIT: return launch<BN, STAGES, EPI_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GELU_SPLIT: return launch<BN, STAGES, EPI_GELU_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GATED: return launch<BN, STAGES, EPI_GATED>(A, B, M, N, K, splits, ep, st);
        case EPI_DGELU_SPLIT: return launch<BN, STAGES, EPI_DGELU_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_F32_SPLIT: return launch<BN, STAGES, EPI_F32_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_GELU_D_SPLIT: return launch<BN, STAGES, EPI_GELU_D_SPLIT>(A, B, M, N, K, splits, ep, st);
        case EPI_MUL_SPLIT: return launch<BN, STAGES, EPI_MUL_SPLIT>(A, B, M, N, K, splits, ep, st);
        default: log("jepa: gemm: unknown epilogue mode %d\n", ep.mode); return -1;
    }
}

bool aligned16(const void * p) { return ((uintptr_t) p & 15) == 0; }

bool vec_ok(const GemmEpi & ep, int N) {
    if (N % 4) return false;
    const void * ptrs[] = {ep.bias, ep.out0, ep.out_hi, ep.out_lo, ep.aux, ep.gate, ep.out1};
    for (const void * p : ptrs) if (p && !aligned16(p)) return false;
    const int lds[] = {ep.out0 ? ep.ld0 : 0, ep.out_hi ? ep.ld_split : 0, ep.aux ? ep.ld_aux : 0, ep.gate ? ep.ld_gate : 0,
                       ep.out1 ? ep.ld1 : 0};
    for (int l : lds) if (l % 4) return false;
    return true;
}

}  // namespace

// Tile / split choice: wide outputs and wide products take 128-wide tiles, one CTA per tile; the
// per-step products of the narrower predictors take 64-wide tiles and split K over a cluster of up to 8 CTAs, the
// largest split at which two rows of tiles (256 rows, or two candidate chains of 128 side by side) are
// resident at once: one wave, each CTA streaming a K-slice, instead of a dozen CTAs streaming everything
// or a second wave of the clusters that did not fit.
int gemm_tc(const SplitMat & A, const SplitMat & B, int M, int N, int K, const GemmEpi & ep, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    if (!load_encode()) {
        log("jepa: gemm: the CUDA driver does not provide cuTensorMapEncodeTiled\n");
        return -1;
    }
    if ((A.ld & 3) || (B.ld & 3) || ((uintptr_t) A.hi & 15) || ((uintptr_t) A.lo & 15) || ((uintptr_t) B.hi & 15) ||
        ((uintptr_t) B.lo & 15)) {
        log("jepa: gemm: operands need 16-byte aligned rows (ld %d / %d)\n", A.ld, B.ld);
        return -1;
    }
    if (B.q.fmt && (((uintptr_t) B.q.q & 15) || ((uintptr_t) B.q.d & 15))) {
        log("jepa: gemm: block planes need 16-byte aligned bases\n");
        return -1;
    }
    GemmEpi e = ep;
    e.vec = vec_ok(ep, N) ? 1 : 0;
    // The tile shape and the K split depend on (N, K), and for the wide products on one row threshold: a row's
    // arithmetic (and so its bits) is the same in every batch on the same side of it.
    const GemmPlan plan = gemm_plan(M, N, K);
    if (plan.persistent) {
        int splits = plan.k_parts;
        if (splits > 1 && (!ep.fix || !ep.fix_count || ep.fix_floats < gemm_fixup_floats(M, N, K) ||
                           ep.fix_counters < gemm_fixup_counters(M, N, K))) {
            splits = 1;   // no scratch from the caller: whole tiles
        }
        return launch_p_mode(A, B, M, N, K, splits, e, st);
    }
    const int num_k = (K + BK - 1) / BK;
    const int tiles2 = 2 * ((N + 63) / 64);
    int splits = 1;
    for (int s = std::min(8, num_k); s > 1; s--) {
        if (tiles2 <= resident_clusters(s)) { splits = s; break; }
    }
    const int kt_per = (num_k + splits - 1) / splits;
    splits = (num_k + kt_per - 1) / kt_per;   // no empty K-slices
    return launch_mode<64, 4>(A, B, M, N, K, splits, e, st);
}

int gemm_error_flag(cudaStream_t st) {
    int v = 0;
    static const int zero = 0;
    // read, then reset on the same stream: a timeout is reported once, to the call that saw it
    if (!cuda_ok(cudaMemcpyFromSymbolAsync(&v, g_gemm_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st), "reading the GEMM error flag") ||
        !cuda_ok(cudaMemcpyToSymbolAsync(g_gemm_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st), "resetting the GEMM error flag") ||
        !cuda_ok(cudaStreamSynchronize(st), "reading the GEMM error flag")) {
        return -1;
    }
    return v;
}

// The failure path of the bounded waits, exercised on purpose: one CTA takes TMEM like the GEMM does,
// initialises an mbarrier that nothing will ever arrive on, and waits on it with a short limit. The wait
// gives up, raises g_gemm_error with `code`, and the CTA releases its TMEM and returns: the same steps a
// GEMM takes when its pipeline stalls, with nothing in flight.
__global__ void k_wait_timeout_check(long long limit, int code) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base_sh;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_base_sh)), "r"(32) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_sh;
    if (threadIdx.x == 0) mbar_wait(&bar, 0, code, &g_gemm_error, limit);   // nobody arrives: runs out
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(32) : "memory");
    }
}

int wait_timeout_check(long long limit_cycles, int code, cudaStream_t st) {
    k_wait_timeout_check<<<1, 64, 0, st>>>(limit_cycles, code);
    return cuda_ok(cudaGetLastError(), "k_wait_timeout_check") ? 0 : -1;
}

int gemm_error_clear(cudaStream_t st) {
    static const int zero = 0;
    return cuda_ok(cudaMemcpyToSymbolAsync(g_gemm_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                   "clearing the GEMM error flag") ? 0 : -1;
}

}  // namespace jb
