// Block-causal attention of the V-JEPA 2-AC predictor: the rows of a frame attend to every row of that
// frame and of the frames before it (reference: the host-built frame mask of ac_predict_split,
// src/vjepa2_ac.cpp:355-366, whole N_T x N_T blocks -- so inside one frame no mask is needed).
//
// Flash-attention structure, f16 operands / f32 accumulation: a CTA owns 64 query rows of one
// (query frame, head, candidate), 16 per warp; it streams 64-key blocks of K and V through
// double-buffered shared memory (cp.async) and keeps the online softmax's running row maximum and sum in
// registers. Keys come from a list of frames, each a base pointer with a candidate stride -- 0 for
// frames every candidate shares, so the observed frames' keys and values exist once per plan, not once
// per candidate. Products use mma.sync m16n8k16 (f16 in, f32 accumulate); the projections around it run
// on tcgen05 (gemm_f16.cu).
#include "kernels.h"
#include "common.h"
#include "launch.h"
#include "kprof.h"

namespace jb {

namespace {

constexpr int QROWS = 64;       // query rows per CTA (4 warps x 16)
constexpr int KB = 64;          // keys per block

__device__ __forceinline__ uint32_t smem_addr(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void * dst, const void * src, bool valid) {
    const int n = valid ? 16 : 0;   // src-size 0 zero-fills the 16 bytes
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(smem_addr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void * p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void * p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *(uint32_t *) &h;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// HD: head width (16, 32 or 64). Query fragments: HD/16 k-chunks; output: HD/8 n-tiles of 8 columns.
// Issue-bound on the legacy tensor path, so the non-MMA work is trimmed: key rows are located per block
// with one division per block (a 64-key block spans at most two frames of kv_rows >= 64 rows; shorter
// frames take the per-row division), only the last block
// is masked, warps whose 16 rows all lie past the frame skip the products, and the softmax uses one fused
// multiply-add and ex2 per score.
template <int HD>
__global__ void __launch_bounds__(128) k_attention(AttnArgs a) {
    constexpr int PAD = HD + 8;     // padded smem row: conflict-free ldmatrix
    constexpr int KC = HD / 16;     // k-chunks of Q K^T
    constexpr int NT = HD / 8;      // n-tiles of the output
    constexpr int CH = HD / 8;      // 16-byte chunks per row
    constexpr int PER = KB * CH / 128;   // chunks of K (and of V) each thread copies per block
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ __align__(16) __half sq[QROWS][PAD];
    __shared__ __align__(16) __half sk[2][KB][PAD];
    __shared__ __align__(16) __half sv[2][KB][PAD];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qtiles = (a.nq + QROWS - 1) / QROWS;
    const int qf = blockIdx.x / qtiles;
    const int q0 = (blockIdx.x % qtiles) * QROWS, head = blockIdx.y, cand = blockIdx.z;
    const int nkf = a.key_frames0 + qf * a.key_step;
    const int nkeys = nkf * a.kv_rows;
    const int nblk = (nkeys + KB - 1) / KB;
    const bool active = q0 + warp * 16 < a.nq;     // this warp has at least one query row
    const __half * qbase = a.q + (size_t) cand * a.q_cand + (size_t) qf * a.q_frame * a.ldq + head * HD;

    for (int c = tid; c < QROWS * CH; c += 128) {
        const int r = c / CH, ch = c % CH;
        const int qr = q0 + r;
        cp_async16(&sq[r][ch * 8], qbase + (size_t) (qr < a.nq ? qr : 0) * a.ldq + ch * 8, qr < a.nq);
    }
    // this thread copies rows r0 + j * (128 / CH) of every block, chunk ch
    const int ch = tid % CH, r0 = tid / CH;
    auto load_kv = [&](int blk, int buf) {
        const int key0 = blk * KB;
        const int f0 = key0 / a.kv_rows;                 // one division per block
        const int edge = (f0 + 1) * a.kv_rows;          // first key of the next frame
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int r = r0 + j * (128 / CH);
            const int key = key0 + r;
            const bool valid = key < nkeys;
            int f = key < edge ? f0 : f0 + 1;
            if (a.kv_rows < KB) f = key / a.kv_rows;      // frames shorter than a block (small models)
            const int kr = key - f * a.kv_rows;
            const __half * base = valid ? a.kv[f] + (size_t) cand * a.kv_cand_stride[f] + (size_t) kr * a.ld_kv + head * HD + ch * 8
                                        : a.kv[0];
            cp_async16(&sk[buf][r][ch * 8], base, valid);
            cp_async16(&sv[buf][r][ch * 8], base + (valid ? a.D : 0), valid);
        }
    };
    load_kv(0, 0);
    cp_async_commit();

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
    uint32_t qa[KC][4];
    const float sl2 = a.scale * 1.4426950408889634f;   // scores in log2 units: exp(x) = 2^(x log2 e)
    const int g = lane >> 2, t = lane & 3;

    for (int blk = 0; blk < nblk; blk++) {
        const int buf = blk & 1;
        if (blk + 1 < nblk) {
            load_kv(blk + 1, buf ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (active) {
            if (blk == 0) {
#pragma unroll
                for (int kc = 0; kc < KC; kc++) {
                    const int r = warp * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
                    const int c = kc * 16 + (lane / 16) * 8;
                    ldsm_x4(qa[kc], &sq[r][c]);
                }
            }
            // S = Q K^T: 16 rows x 64 keys per warp, 8 n-tiles of 8 keys
            float s[8][4];
#pragma unroll
            for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
            for (int kc = 0; kc < KC; kc++) {
#pragma unroll
                for (int jn = 0; jn < 8; jn += 2) {
                    uint32_t kb[4];
                    const int kr = jn * 8 + (lane % 8) + (lane / 16) * 8;
                    const int kcol = kc * 16 + ((lane / 8) % 2) * 8;
                    ldsm_x4(kb, &sk[buf][kr][kcol]);
                    mma16816(s[jn], qa[kc], kb[0], kb[1]);
                    mma16816(s[jn + 1], qa[kc], kb[2], kb[3]);
                }
            }
            if (blk + 1 == nblk && nkeys % KB) {         // only the last block can run past the keys
#pragma unroll
                for (int j = 0; j < 8; j++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        if (blk * KB + j * 8 + 2 * t + (e & 1) >= nkeys) s[j][e] = -INFINITY;
                    }
                }
            }
            // online softmax over rows g and g + 8 of the warp's 16
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
                mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            }
            float nm[2], corr[2], sum[2] = {0.0f, 0.0f};
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float mnew = fmaxf(mrow[h], mx[h]);    // finite: every block has a valid key
                corr[h] = ex2((mrow[h] - mnew) * sl2);        // ex2(-inf) = 0 on the first block
                mrow[h] = mnew;
                nm[h] = -mnew * sl2;
            }
            uint32_t pa[4][4];              // P as A fragments: 4 k-chunks of 16 keys
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float p[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    p[e] = ex2(__fmaf_rn(s[j][e], sl2, nm[e >> 1]));   // -inf -> 0
                    sum[e >> 1] += p[e];
                }
                const int kc = j >> 1;
                if ((j & 1) == 0) { pa[kc][0] = pack_h2(p[0], p[1]); pa[kc][1] = pack_h2(p[2], p[3]); }
                else              { pa[kc][2] = pack_h2(p[0], p[1]); pa[kc][3] = pack_h2(p[2], p[3]); }
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
                lrow[h] = __fmaf_rn(lrow[h], corr[h], sum[h]);
            }
#pragma unroll
            for (int j = 0; j < NT; j++) {
                o[j][0] *= corr[0]; o[j][1] *= corr[0];
                o[j][2] *= corr[1]; o[j][3] *= corr[1];
            }
            // O += P V, V [key][dim] read transposed
#pragma unroll
            for (int kc = 0; kc < 4; kc++) {
#pragma unroll
                for (int jn = 0; jn < NT; jn += 2) {
                    uint32_t vb[4];
                    const int vr = kc * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
                    const int vc = jn * 8 + (lane / 16) * 8;
                    ldsm_x4_t(vb, &sv[buf][vr][vc]);
                    mma16816(o[jn], pa[kc], vb[0], vb[1]);
                    mma16816(o[jn + 1], pa[kc], vb[2], vb[3]);
                }
            }
        }
        __syncthreads();   // this buffer is refilled by the next iteration's prefetch
    }
    if (!active) return;
    __half * obase = a.out + (size_t) cand * a.o_cand + (size_t) qf * a.q_frame * a.ldo + head * HD;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int qr = q0 + warp * 16 + g + 8 * h;
        if (qr >= a.nq) continue;
        const float inv = lrow[h] > 0.0f ? 1.0f / lrow[h] : 0.0f;
        __half * dst = obase + (size_t) qr * a.ldo;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            *(__half2 *) (dst + j * 8 + 2 * t) = __floats2half2_rn(o[j][2 * h] * inv, o[j][2 * h + 1] * inv);
        }
    }
}

}  // namespace

int attention_f16(const AttnArgs & a, cudaStream_t st) {
    if (a.hd != 16 && a.hd != 32 && a.hd != 64) { log("jepa: attention: head width %d is not supported (16, 32 or 64)\n", a.hd); return -1; }
    const int max_kf = a.key_frames0 + (a.n_qframes - 1) * a.key_step;
    if (a.key_frames0 < 1 || max_kf > AC_MAX_FRAMES || a.n_qframes < 1 || a.nq < 1 || a.n_cand < 1 || a.n_cand > 65535 ||
        a.kv_rows < 1 || a.n_head * a.hd > a.D) {
        log("jepa: attention: %d..%d key frames / %d query rows / %d candidates out of range\n", a.key_frames0, max_kf, a.nq, a.n_cand);
        return -1;
    }
    for (int f = 0; f < max_kf; f++) {
        if (!a.kv[f]) { log("jepa: attention: key frame %d has no cache slot\n", f); return -1; }
    }
    if ((a.ldq & 7) || (a.ld_kv & 7) || (a.ldo & 1) || (a.D & 7) || ((uintptr_t) a.q & 15)) {
        log("jepa: attention: rows must be 16-byte aligned\n");
        return -1;
    }
    const int qtiles = (a.nq + QROWS - 1) / QROWS;
    const dim3 grid((unsigned) (qtiles * a.n_qframes), (unsigned) a.n_head, (unsigned) a.n_cand);
    double keys = 0;
    for (int k = 0; k < a.n_qframes; k++) keys += (double) (a.key_frames0 + k * a.key_step) * a.kv_rows;
    KTimer kt("attention", st, 4.0 * a.n_head * a.hd * a.nq * keys * a.n_cand,
              2.0 * a.n_cand * (2.0 * a.n_qframes * a.nq * a.n_head * a.hd + 2.0 * keys * a.n_head * a.hd));
    if (a.impl != 1 && attention_tc_supported(a)) return attention_tc(a, st);
    if (a.impl == 2) { log("jepa: attention: the tcgen05 kernel does not take this shape\n"); return -1; }
    switch (a.hd) {
        case 16: JB_CUDA(launch_pdl(k_attention<16>, grid, dim3(128), 0, st, a)); break;
        case 32: JB_CUDA(launch_pdl(k_attention<32>, grid, dim3(128), 0, st, a)); break;
        default: JB_CUDA(launch_pdl(k_attention<64>, grid, dim3(128), 0, st, a)); break;
    }
    return 0;
}

}  // namespace jb
