// Launchers of the sm_100a kernels (implemented in gemm_tc.cu, rowwise.cu, dequant.cu).
//
// Data layout everywhere: row-major [rows][cols] float32, one row per candidate (or per candidate and
// time step), leading dimension = row stride in elements. "Split" operands are the two float32 planes
// (hi, lo) of the 3xTF32 scheme: hi = x with the low 13 mantissa bits cleared (exact in TF32),
// lo = x - hi (exact in float32); a product is accumulated as hi*hi + hi*lo + lo*hi, which keeps
// about 21 bits of each operand instead of TF32's 11.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace jb {

// ------------------------------------------------------------------------------------------
// tcgen05 GEMM: C[M,N] = A[M,K] * B[N,K]^T (both operands K-contiguous), split operands, fused epilogue
// ------------------------------------------------------------------------------------------
enum EpiMode : int {
    EPI_F32 = 0,         // out0 = acc + bias
    EPI_SPLIT = 1,       // (out_hi, out_lo) = split(acc + bias)
    EPI_GELU_SPLIT = 2,  // out0 = u = acc + bias ; (out_hi, out_lo) = split(gelu(u))
    EPI_GATED = 3,       // out0 = o = acc + bias ; out1 = aux + o * gate
    EPI_DGELU_SPLIT = 4, // (out_hi, out_lo) = split(acc * gelu'(aux))
    EPI_F32_SPLIT = 5,   // out0 = acc + bias and (out_hi, out_lo) = split(acc + bias)
    EPI_GELU_D_SPLIT = 6, // u = acc + bias: out0 = gelu'(u) ; (out_hi, out_lo) = split(gelu(u)) (one erf for both)
    EPI_MUL_SPLIT = 7,   // (out_hi, out_lo) = split(acc * aux): EPI_DGELU_SPLIT with gelu' stored by EPI_GELU_D_SPLIT
};

struct GemmEpi {
    int mode = EPI_F32;
    const float * bias = nullptr;   // [N] or null
    float * out0 = nullptr; int ld0 = 0;
    float * out_hi = nullptr; float * out_lo = nullptr; int ld_split = 0;
    const float * aux = nullptr; int ld_aux = 0;
    const float * gate = nullptr; int ld_gate = 0;
    float * out1 = nullptr; int ld1 = 0;
    int vec = 0;                    // set by gemm_tc: float4 epilogue allowed
    // Operands that do not come from the kernel right before this one in the stream (they were written at
    // least two kernels earlier, or are weights): loaded before the dependency wait, while that kernel
    // still runs. pre_b: the B operand (its first pipeline stages); pre_epi: bias / aux / gate.
    int pre_b = 0, pre_epi = 0;
    // Scratch of the K-split fix-up (see gemm_fixup_floats): partial tiles and one counter per output tile,
    // the counters zero before the launch (the kernel leaves them zero). Without it the K split is off.
    float * fix = nullptr; size_t fix_floats = 0;
    int * fix_count = nullptr; size_t fix_counters = 0;
};

// A weight operand B[N][K] kept in its GGUF block values and dequantised inside the GEMM mainloop: the
// producer's TMA stages a K-step's raw tile (the block values of BN rows x 32 columns and their f16 scales)
// and converter warps write the split planes the tensor core reads. Values are exactly those of a
// load-time dequantisation (d * q is exact in float32, and so is its hi / lo split), so a product's bits do
// not depend on the layout the weight is kept in.
//   QF_Q8   q: int8 [N][K] (row stride K bytes)
//   QF_Q4   q: the 4-bit block values [N][K / 2], element 2j in the low nibble of byte j, 2j + 1 in the high
//   QF_F16  q: f16 bits [N][K]
// Scales (Q8, Q4: f16 bits): orient 0, one per row and 32-column block, stored [K / 32][N] (the forward
// operand W[out][in]); orient 1, one per 32-row group and column, stored [N / 32][K] (the transposed
// operand W^T, whose rows are the blocks' columns). Both orientations of a weight share one scale array.
enum QFmt : int { QF_NONE = 0, QF_Q8 = 1, QF_Q4 = 2, QF_F16 = 3 };
struct QuantB {
    int fmt = QF_NONE;
    int orient = 0;
    const void * q = nullptr;
    const uint16_t * d = nullptr;
};

struct SplitMat {                    // a split operand: two float32 planes with one leading dimension
    const float * hi = nullptr;
    const float * lo = nullptr;
    int ld = 0;
    QuantB q;                        // B only: when q.fmt is set, the block planes replace hi / lo
};

// The block planes of a GGUF weight [rows][ne0] (type 8 = q8_0, 2 = q4_0, 1 = f16) for both GEMM
// orientations, from its raw rows on the device: q / qt hold the forward ([rows][ne0]) and transposed
// ([ne0][rows]) values in the format's QuantB layout, d the shared scales [ne0 / 32][rows] (null for f16).
// Sizes: quant_plane_bytes each for q and qt, quant_scale_count f16 values for d.
size_t quant_plane_bytes(uint32_t type, int64_t rows, int64_t ne0);
size_t quant_scale_count(uint32_t type, int64_t rows, int64_t ne0);
int quant_planes(uint32_t type, const void * raw, int64_t rows, int64_t ne0, void * q, void * qt, uint16_t * d, cudaStream_t st);
// Whether the GEMM can read W [rows][ne0] of this type in its block planes, forward (N = rows, K = ne0)
// or transposed (N = ne0, K = rows).
bool quant_ok(uint32_t type, int64_t rows, int64_t ne0);

// Returns 0, or -1 after logging (unsupported shape / a CUDA error).
int gemm_tc(const SplitMat & A, const SplitMat & B, int M, int N, int K, const GemmEpi & ep, cudaStream_t st);
// The persistent kernel splits the K range of narrow, long products (at most 8 column tiles, K >= 2048) in
// GEMM_KSPLIT parts when the caller passes fix-up scratch: each part's partial tile goes to the scratch and
// the last part to finish sums the parts in a fixed order and applies the epilogue. The split depends on
// (N, K) only. (Which kernel a wide product takes also depends on whether it has at most 256 rows: a row's
// bits are the same in every batch on one side of that threshold.) These give the scratch a call needs:
// partial-tile floats and tile counters (0 when the shape is not split).
constexpr int GEMM_KSPLIT = 3;
constexpr int GEMM_KSPLIT_MAX = 4;   // the most parts the persistent kernel's fix-up sums
// The launch gemm_tc makes for a shape: the persistent 128 x 128 kernel or the 64-wide split-K clusters
// (whose split is chosen from the device's cluster occupancy at launch); for the persistent kernel, its K
// parts when the caller passes fix-up scratch, and its tile order (1 = grouped rows-fastest).
struct GemmPlan {
    bool persistent = false;
    int k_parts = 0;
    int m_fast = 0;
};
GemmPlan gemm_plan(int M, int N, int K);
// The persistent kernel's output tiles in walk order (the kernel's own origin function, run on the host):
// writes each tile's first row and column, returns the tile count, 0 when the shape takes the split-K
// clusters, -1 when more than `cap` tiles.
int gemm_tile_walk(int M, int N, int K, int * m0, int * n0, int cap);
size_t gemm_fixup_floats(int M, int N, int K);
size_t gemm_fixup_counters(int M, int N, int K);

// Error flag the tensor-core kernels raise when a bounded wait gives up. gemm_error_flag returns it
// (0 = fine, the waiter's code otherwise, -1 when the flag could not be read) and resets it to 0 on the
// stream; gemm_error_clear only resets it (at the start of an API call, so that a flag left by an
// earlier call that failed for another reason does not fail this one).
int gemm_error_flag(cudaStream_t st);
int gemm_error_clear(cudaStream_t st);
// Launches one CTA that takes TMEM, waits on an mbarrier nothing arrives on with a bound of limit_cycles
// (clock64), raises the GEMM error flag with `code` when the bound runs out, frees its TMEM and returns.
int wait_timeout_check(long long limit_cycles, int code, cudaStream_t st);

// ------------------------------------------------------------------------------------------
// SIMT linear for shapes the tensor-core path does not take (tiny K or N):
//   y[r][o] = sum_i x[r][i] * w[o][i] + b[o]          (w row-major [N][K])
// ------------------------------------------------------------------------------------------
void linear_simt(const float * x, int ldx, const float * w, const float * b, float * y, int ldy,
                 int M, int N, int K, cudaStream_t st);

// ------------------------------------------------------------------------------------------
// row-wise kernels (one warp per row)
// ------------------------------------------------------------------------------------------
struct LnStats { double mean; float inv; float pad; };

// adaLN block prologue: h = ln?( LN0(x) * (1 + mod[sc]) + mod[sh] ), split out; stats saved.
// mod and the ln weights are read before the dependency wait: they must have been written at least two
// kernels earlier in the stream (x may come from the kernel right before).
void block_pre(const float * x, int ldx, const float * mod, int ld_mod, int sh_off, int sc_off,
               const float * ln_w, const float * ln_b, float eps0, float eps1,
               float * h_hi, float * h_lo, int ldh, LnStats * st0, LnStats * st1, int M, int D, cudaStream_t st);

// LayerNorm with optional affine: y = LN(x) * w + b. Writes f32 y (if y) and/or split (if hi/lo).
void layer_norm(const float * x, int ldx, const float * w, const float * b, float eps,
                float * y, int ldy, float * hi, float * lo, LnStats * stats, int M, int D, cudaStream_t st);

// LayerNorm backward: gx = LN_bwd(gy) (+ residual add of `gres` when given), then optionally the
// gated-residual head of the block below it:
//   dmod[gate_col] = gx * dn ; (d_hi, d_lo) = split(gx * gate)
void layer_norm_bwd(const float * gy, int ldgy, const float * x, int ldx, const LnStats * stats, const float * w,
                    const float * gres, int ldres, float * gx, int ldgx,
                    const float * dn, int lddn, const float * gate, int ld_gate,
                    float * dmod_hi, float * dmod_lo, int ld_dmod, float * d_hi, float * d_lo, int ldd,
                    int M, int D, cudaStream_t st);

// adaLN block backward of one half (the MLP half or the attention half), fused:
//   gz  = ln?_bwd(gh)                              (ln weight optional)
//   dmod[sc] = gz * LN0(x) ; dmod[sh] = gz
//   gx  = gres + LN0_bwd(gz * (1 + mod[sc]))
//   then the gated-residual head of the next half down (optional):
//   dmod[gate2] = gx * a2 ; (d_hi, d_lo) = split(gx * mod2[gate2])
struct BlockBwdArgs {
    const float * gh; int ldgh;
    const float * gres; int ldres;
    const float * x; int ldx;                 // the half's input (recomputes LN0)
    const LnStats * st0; const LnStats * st1; // LN0 and the inner ln statistics
    const float * ln_w; const float * ln_b;   // inner ln (null = none)
    const float * mod; int ld_mod; int sh_off; int sc_off;
    float * dmod_hi; float * dmod_lo; int ld_dmod;
    float * gx; int ldgx;
    // head of the next half down (null a2 = none)
    const float * a2; int lda2; const float * mod2; int ld_mod2; int gate2_off;
    float * dmod2_hi; float * dmod2_lo; int ld_dmod2;
    float * d_hi; float * d_lo; int ldd;
    int M, D;
    float eps0, eps1;
};
// Every operand but gh is read before the dependency wait: it must have been written at least two kernels
// earlier in the stream (gh may come from the kernel right before).
void block_bwd(const BlockBwdArgs & a, cudaStream_t st);

// ------------------------------------------------------------------------------------------
// element-wise kernels
// ------------------------------------------------------------------------------------------
void split_f32(const float * x, int ldx, float * hi, float * lo, int ldo, int M, int N, cudaStream_t st);
void add_row_vec(const float * x, int ldx, const float * row, float * y, int ldy, int M, int N, cudaStream_t st);
// act: 0 gelu_erf, 2 silu, 3 relu (the reference's jepa_act_id values)
void act_fwd(const float * x, int ldx, float * y, int ldy, int M, int N, int act, cudaStream_t st);
void act_bwd(const float * gy, int ldgy, const float * x, int ldx, float * gx, int ldgx, int M, int N, int act,
             bool accumulate, cudaStream_t st);
void add_inplace(float * y, int ldy, const float * x, int ldx, int M, int N, cudaStream_t st);
void copy_rows(const float * x, int ldx, float * y, int ldy, int M, int N, cudaStream_t st);
void fill_f32(float * y, float v, size_t n, cudaStream_t st);

// actions x [S][T][A] -> a_all [(t*S + r)][A]
void gather_actions(const float * x, float * a_all, int S, int T, int A, cudaStream_t st);
// d a_all [(t*S + r)][A] -> grad [S][T][A]
void scatter_actions(const float * da, float * grad, int S, int T, int A, cudaStream_t st);

// squared-L2 cost of `W` scored state sets against their goals (double accumulation per row):
//   cost[r] += w_j * sum_i (p_j[r][i] - g_j[i])^2 ; gp_j[r][i] += 2 * w_j * diff (if want_grad)
void cost_l2(const float * const * preds, const float * goals, const float * weights, float * const * gpreds,
             int W, int M, int D, int ldp, float * cost, bool want_grad, cudaStream_t st);

// action-cost pooling (pool.cu): chunk rows of the embeddings e [Wa stride S][E] <-> the concatenated
// 'mlp' input x [Wa S][stride E]; step-linear outputs z [Wa stride S][d] <-> token groups X [Wa S][stride+1][d]
// (back = the gradient direction: writes e / z); self-attention inside groups of G rows of qkv [rows][3 d]
void pool_chunks(float * e, float * x, int Wa, int S, int stride, int E, bool back, cudaStream_t st);
void pool_tokens(float * z, const float * pos, float * X, int Wa, int S, int stride, int d, bool back, cudaStream_t st);
size_t group_mha_smem(int G, int d, int H, bool backward);
bool group_mha_prepare(int G, int d, int H);   // false: the group does not fit one CTA's shared memory
void group_mha_fwd(const float * qkv, float * o, float * probs, int n_groups, int G, int d, int H, cudaStream_t st,
                   bool causal = false);
// y = x + a * gate (the adaLN gated residual), element-wise over M rows of N
void gated_add(const float * x, int ldx, const float * a, int lda, const float * gate, int ld_gate, float * y, int ldy,
               int M, int N, cudaStream_t st);
void group_mha_bwd(const float * go, const float * qkv, const float * probs, float * gqkv, int n_groups, int G, int d, int H,
                   cudaStream_t st);

// AdamW + optional noise + clamp, then the t-major copy of the updated actions:
//   x *= 1 - lr*wd ; m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g g ; x -= step_size m / (sqrt(v)/c2s + eps)
//   x += z * noise_std ; x = min(max(x, lo[a]), hi[a])
// sched[2*k], sched[2*k+1] hold step_size and c2s of iteration k; *step_ctr is the iteration index and
// is incremented by the kernel, so one captured graph replays every iteration. The noise of iteration k
// is z + k * z_stride (z_stride 0: one slot refilled by the host every iteration).
void adam_step(float * x, float * m, float * v, const float * grad_tmajor, float * a_all,
               const float * sched, int * step_ctr, float lr_wd, const float * z, float noise_std, size_t z_stride,
               const float * lo, const float * hi, int S, int T, int A, cudaStream_t st);

// index of the first minimum of cost[0..n) (std::min_element semantics) and its value
void argmin_first(const float * cost, int n, int * idx, float * val, cudaStream_t st);

// ------------------------------------------------------------------------------------------
// V-JEPA 2-AC kernels (ac_kernels.cu, gemm_f16.cu, attention.cu): f16 operands, f32 accumulate
// ------------------------------------------------------------------------------------------
enum AcEpi : int {
    AEPI_F32 = 0,        // out_f32[remap(row)] = acc + bias
    AEPI_ADD_F32 = 1,    // out_f32[remap(row)] += acc + bias          (residual stream)
    AEPI_GELU_F16 = 2,   // out_f16[row] = gelu(acc + bias)
    AEPI_QKV = 3,        // q -> out_f16 (RoPE), k (RoPE) and v -> kv[row][0 .. 2 D)
};

struct AcGemmEpi {
    int mode = AEPI_F32;
    const float * bias = nullptr;
    float * out_f32 = nullptr; int ld_f32 = 0;
    __half * out_f16 = nullptr; int ld_f16 = 0;
    __half * kv = nullptr; int ld_kv = 0;
    // 3-D RoPE, factorised per axis: cos / sin tables [slots + 2 grid][d] (frame rows, then grid rows, then grid
    // columns; d = 2 ((hd / 3) / 2) lanes per axis, the rotation's sign folded into the even lanes of sin). Row r
    // of the GEMM is row (r mod frame_rows) of frame slot rope_slot0 + (r / frame_rows) mod rope_nf; its first
    // rope_cond rows sit at grid position (0, 0), patch p at (p / grid, p mod grid).
    const float * rope_cos = nullptr; const float * rope_sin = nullptr;
    int rope_d = 0, rope_slots = 0, rope_grid = 1, rope_slot0 = 0, rope_nf = 1, rope_frame_rows = 1, rope_cond = 2;
    int D = 0, hd = 64;
    int remap_g = 0, remap_gout = 0, remap_off = 0;   // out row = (row / g) * gout + off + row % g (g = 0: row)
};

// C[M,N] = A[M,K] * B[N,K]^T, A and B f16 row-major (K contiguous), tcgen05 kind::f16, f32 accumulate
int gemm_f16(const __half * A, int lda, const __half * B, int ldb, int M, int N, int K, const AcGemmEpi & ep, cudaStream_t st);
int gemm_f16_error_flag(cudaStream_t st);   // as gemm_error_flag, for the f16 GEMM
int gemm_f16_error_clear(cudaStream_t st);

// Attention of the rows of `n_qframes` consecutive frames over their key frames. Frames are whole blocks
// (block-causal across frames: a frame sees every row of the frames up to its own), so no mask is needed
// inside a frame: query frame k of the call sees key frames 0 .. key_frames0 + k * key_step - 1.
constexpr int AC_MAX_FRAMES = 32;
struct AttnArgs {
    const __half * q = nullptr; int ldq = 0;      // row r of query frame k of candidate c: q + c*q_cand + (k*q_frame + r)*ldq
    long long q_cand = 0;
    int nq = 0;                                   // query rows per frame
    int n_qframes = 1, q_frame = 0;               // query frames in this call, rows between them
    __half * out = nullptr; int ldo = 0;          // same row indexing as q
    long long o_cand = 0;
    int key_frames0 = 1, key_step = 1;            // key frames of query frame 0; growth per query frame (1 causal, 0 full)
    const __half * kv[AC_MAX_FRAMES] = {};        // per key frame: [cand][kv_rows][ld_kv], k at col 0, v at col D
    long long kv_cand_stride[AC_MAX_FRAMES] = {}; // elements between candidates (0: shared by all)
    int kv_rows = 0, ld_kv = 0, D = 0, n_head = 0, hd = 64;
    int n_cand = 0;
    float scale = 0.125f;
    int impl = 0;                                 // 0: the tcgen05 kernel when it takes the shape, 1: mma.sync, 2: tcgen05
};
int attention_f16(const AttnArgs & a, cudaStream_t st);
// the tcgen05 attention (attention_tc.cu): head width 64, at most 288 query rows per frame
bool attention_tc_supported(const AttnArgs & a);
int attention_tc(const AttnArgs & a, cudaStream_t st);
int attention_tc_error_flag(cudaStream_t st);   // as gemm_error_flag, for the tcgen05 attention
int attention_tc_error_clear(cudaStream_t st);
// resets all three flags on the stream (0 = done)
inline int device_flags_clear(cudaStream_t st) {
    return (gemm_error_clear(st) | gemm_f16_error_clear(st) | attention_tc_error_clear(st)) ? -1 : 0;
}

// Two-level row gather: in = (r / (g1 g2)) * s2 + ((r / g1) % g2) * s1 + off + r % g1  (g1 = 0: in = r)
struct RowMap {
    int g1 = 0, g2 = 1, s1 = 0, s2 = 0, off = 0;
};
// LayerNorm of f32 rows (optional affine) to f16 rows; input rows gathered through `map`
void ln_to_f16(const float * x, int ldx, const float * w, const float * b, float eps, __half * y, int ldy, int M, int D,
               RowMap map, cudaStream_t st);
// the reference's non-affine normalisation between rollout steps (jepa_ac_normalize) in place, plus an f16 copy
void ac_normalize_rows(float * x, int ld, __half * y16, int ldy, int M, int D, float eps, cudaStream_t st);
// f32 -> f16 rows, input rows gathered through `map`
void to_f16(const float * x, int ldx, __half * y, int ldy, int M, int N, RowMap map, cudaStream_t st);
// conditioning rows of every (candidate, frame) block of a [n_cand][n_frames][rows_per_frame] row layout:
// row 0 = action_embed(acts + c * act_cand + t * A), row 1 = state_embed(states + c * st_cand + t * S), f32
void ac_cond_rows(const float * acts, long long act_cand, const float * states, long long st_cand, int A, int S,
                  const float * wa, const float * ba, const float * ws, const float * bs, float * resid, int ld,
                  int n_cand, int n_frames, int rows_per_frame, int D, cudaStream_t st);
// copy rows [row0, row0 + rows) of candidate 0's block to the same rows of candidates 1 .. n_cand-1
void ac_broadcast_rows(float * x, int ld, long long cand_rows, int row0, int rows, int n_cand, int D, cudaStream_t st);
// CEM on the device (cem.cu). cem_sample: acts [K][H][A] from noise [H][K][4] and the distribution mean / sd
// [H][4] (translation lanes 0..2 and the gripper lane 6; rotation 0). cem_refit: the topk lowest of energy [K]
// (ties to the lower index), best[0] = the lowest, then mean / sd moved to the elites' mean and unbiased std
// with the given momenta (translation, gripper). elite: [topk] ints of device scratch.
void cem_sample(const float * noise, const float * mean, const float * sd, int K, int H, int A, float maxnorm,
                float gripper_clamp, float * acts, cudaStream_t st);
void cem_refit(const float * energy, const float * acts, float * mean, float * sd, float * best, int * elite, int K, int H,
               int A, int topk, float m_mean, float m_std, float m_mean_grip, float m_std_grip, cudaStream_t st);

// energy[c] = mean |pred[c] - goal| over n values, double accumulation (jepa_ac_energy)
void ac_energy(const float * pred, long long cand_stride, const float * goal, long long n, int n_cand, float * energy,
               cudaStream_t st);

// ------------------------------------------------------------------------------------------
// dequantisation: GGUF row bytes -> float32, bit-exact with the block formats
// ------------------------------------------------------------------------------------------
int dequant_rows(uint32_t ggml_type, const void * src, float * dst, int64_t rows, int64_t ne0, cudaStream_t st);
// dst[c][r] = src[r][c]  (rows x cols -> cols x rows)
void transpose_f32(const float * src, float * dst, int rows, int cols, cudaStream_t st);

}  // namespace jb
