// jepa-b200 extensions: entry points this engine adds next to the jepa.cpp API (include/jepa.h).
//
// None of these replaces a reference function; they expose the engine's own pieces so that its kernels
// can be checked and timed through the same C ABI (plain pointers and sizes, host memory, int 0 / -1
// returns with the reason in jepa_error_text()), and so that a multi-GPU host can shard a planner.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "jepa.h"

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)   // every declaration below is exported
#endif

// Version string of this engine ("jepa-b200 <version>").
const char * jepa_b200_version(void);

// C[M,N] = A[M,K] * B[N,K]^T on the current CUDA device through the tcgen05 3xTF32 GEMM of the planner
// (host buffers, row-major). A kernel check: the planner's linears all run through this kernel.
int jepa_b200_gemm(const float * A, const float * B, int M, int N, int K, float * C);

// The same product in the planner's configuration: narrow, long products (at most 8 output column tiles
// of 128, K >= 2048) split their K range in three parts whose partial tiles a fix-up sums in a fixed order (the
// planner passes that scratch on every such product). Agrees with jepa_b200_gemm to rounding.
int jepa_b200_gemm_ksplit(const float * A, const float * B, int M, int N, int K, float * C);

// The launch the planner's GEMM makes for a product of shape M x N x K, computed on the host (no device
// needed): out[0] = 1 for the persistent 128 x 128 kernel, 0 for the 64-wide split-K clusters; out[1] = the
// persistent kernel's K parts in the planner's configuration (1 = whole tiles; 0 for the clusters, whose split
// follows the device's cluster occupancy); out[2] = 1 when the persistent kernel walks grouped row tiles
// rows-fastest. A row's bits depend only on this plan, so rows of batches with the same plan agree bit for bit.
// Returns 0, or -1 for a null `out` or a non-positive size. No counterpart in the reference.
int jepa_b200_gemm_plan(int M, int N, int K, int * out);

// The persistent kernel's output tiles for that shape in the order its CTAs take them, computed on the host by
// the kernel's own tile-origin function: m0[t], n0[t] = first row and column of tile t. Returns the tile
// count, 0 when the shape takes the split-K clusters, -1 for null buffers, non-positive sizes or more than
// `cap` tiles. No counterpart in the reference.
int jepa_b200_gemm_tile_walk(int M, int N, int K, int * m0, int * n0, int cap);

// The planner-configuration product timed on the device: `reps` launches on device-resident operands,
// returns the mean milliseconds per launch in *ms (CUDA events around the launches).
int jepa_b200_gemm_bench(int M, int N, int K, int reps, double * ms);

// The planner's GEMM with its weight operand kept in GGUF block values and dequantised in the mainloop:
// W [rows][ne0] are the raw rows of a weight of ggml type 8 (q8_0), 2 (q4_0) or 1 (f16), rows and ne0
// multiples of 32. transposed = 0: C [M][rows] = A [M][ne0] W^T (the forward product); transposed = 1:
// C [M][ne0] = A [M][rows] W (the backward product against the same weight). ksplit = 1 passes the K-split
// scratch as the planner does. Equals jepa_b200_gemm on the dequantised weight bit for bit.
int jepa_b200_gemm_quant(uint32_t ggml_type, const void * w_raw, int rows, int ne0, int transposed, const float * A, int M,
                         float * C, int ksplit);

// jepa_b200_gemm_quant timed on the device (zero operands of shape M x N x K, `reps` launches); the mean
// milliseconds per launch in *ms.
int jepa_b200_gemm_quant_bench(uint32_t ggml_type, int M, int N, int K, int transposed, int reps, double * ms);

// jepa_b200_gemm for callers that must not allocate device memory. No counterpart in the reference.
// Some hosts cannot call cudaMalloc around a kernel call: a process whose device memory budget is fixed
// at start-up, a real-time control loop where an allocation (which can synchronise the whole device)
// would blow the cycle's deadline, or a plug-in living inside someone else's allocator. This entry point
// computes the same product as jepa_b200_gemm from the same host buffers, but keeps the device copies of
// A, B and C and the operand split planes in one fixed device array that the library reserves when it
// is loaded (JEPA_B200_NOALLOC_MAX_FLOATS floats = 16 MiB, held on every GPU that loads the library
// until the process exits), and calls no cudaMalloc / cudaFree.
//   limit  : 3 (M K + N K) + M N floats (each part rounded up to 64), at most JEPA_B200_NOALLOC_MAX_FLOATS;
//            larger sizes are refused with a message in jepa_error_text()
//   set-up : the first call on a device looks up that device's copy of the array, so make that first
//            call before any stream capture
//   sharing: every call on a device uses the same array and leaves its contents there; calls that
//            overlap on the GPU (from two host threads) race on it
// Runs on the current CUDA device and its legacy default stream; returns 0 or -1.
#define JEPA_B200_NOALLOC_MAX_FLOATS (4u * 1024u * 1024u)
int jepa_b200_gemm_noalloc(const float * A, const float * B, int M, int N, int K, float * C);

// The failure path of the engine's bounded device waits, run on purpose without a fault: one CTA takes
// tensor memory as the GEMM does, waits on an mbarrier that nothing arrives on with a bound of
// `limit_cycles` SM clock cycles (1 .. 4e9; the kernels' own bound is 4e9, about 2 s), raises the GEMM's
// error flag when the bound runs out, frees its tensor memory and returns. *code receives the flag as
// the engine reads it after a call (9 for this check, 0 if the wait did not run out); the read resets
// it. Returns 0 when the flag could be read and was reset, -1 otherwise. No counterpart in the reference
// (its planners run on the host and have no device waits).
int jepa_b200_check_wait_timeout(long long limit_cycles, int * code);

// The same rows decoded on the host by the loader's CPU decoder (no GPU needed): the decoder the engine
// uses for host-side tensors (recorded actions, the oracle's weights), checkable without a device.
int jepa_b200_host_dequant(uint32_t ggml_type, const void * src, int64_t rows, int64_t ne0, float * dst);

// Dequantise `rows` GGUF rows of `ne0` values of ggml type `ggml_type` (0 f32, 1 f16, 2 q4_0, 8 q8_0,
// 30 bf16) from the host bytes `src` into host float32 `dst` by the device kernel the weight loader uses.
int jepa_b200_dequant(uint32_t ggml_type, const void * src, int64_t rows, int64_t ne0, float * dst);

// Candidate sharding of the planners over `world` GPUs, one process (and one context) per GPU.
// Rank r plans candidates [r*S/world, (r+1)*S/world) of every level; the ranks exchange only each
// level's (min cost, index) and the winning plan, through NCCL over NVLink. `nccl_id` is the
// 128-byte ncclUniqueId from jepa_b200_nccl_unique_id() on rank 0, broadcast by the host.
// world == 1 turns sharding off. Must be called before the first planner call on `ctx`.
int jepa_b200_nccl_unique_id(void * out128);
int jepa_b200_context_set_shard(jepa_context * ctx, int rank, int world, const void * nccl_id);

// Device milliseconds of the last planner call on this context (CUDA events on its stream), and the
// number of kernels it launched.
double jepa_b200_last_plan_ms(const jepa_context * ctx);
long long jepa_b200_last_plan_launches(const jepa_context * ctx);

// Candidate streams of the H-JEPA solves on this context: a level's candidates (this GPU's share) run as
// n independent chains of consecutive rows side by side on the GPU (1..8; 0 = automatic: for predictors
// narrower than 768 one chain per 256 candidates, at most 4; for wider ones 2 from 512 candidates up, else 1).
// Results do not depend on n (rows never interact), as the reference's results do
// not depend on its thread count (its jepa_context_params.n_threads). Returns 0, or -1 for a non-H-JEPA
// context or n out of range.
int jepa_b200_hjepa_set_streams(jepa_context * ctx, int n);

// Memory mode of the H-JEPA solves on this context: 0 = automatic (the first that fits the free device memory
// of: every step's adaLN modulation and its gradient, [T S][6 P L] floats x 3; every step's modulation kept
// ([T S][6 P L] x 1) and the gradient folded step by step; one step at a time), 1 = always one step at a time
// (the modulation recomputed in the backward: more GEMM work, least memory), 2 = always the middle mode.
// Results are the same in every mode. Returns 0, or -1 for a non-H-JEPA context or a mode out of range.
int jepa_b200_hjepa_set_step_modulation(jepa_context * ctx, int mode);

// C[M,N] = f16(A)[M,K] * f16(B)[N,K]^T with f32 accumulation through the V-JEPA 2-AC predictor's
// tcgen05 kind::f16 GEMM (host f32 buffers, rounded to f16 on the device; K a multiple of 8). A kernel
// check: every linear of the AC predictor runs through this kernel.
int jepa_b200_gemm_f16(const float * A, const float * B, int M, int N, int K, float * C);
// Same product timed on device-resident operands: mean milliseconds per launch over `reps` launches.
int jepa_b200_gemm_f16_bench(int M, int N, int K, int reps, double * ms);

// The AC predictor's attention: the last of `n_frames` frames of `rows` rows attends to every row of all of
// them, for `n_cand` candidates and `heads` heads of width `hd` (16, 32 or 64). q [n_cand][rows][heads hd],
// kv [n_cand][n_frames rows][2 heads hd] (keys, then values), out like q: host f32, f16 on the device.
// impl: 0 the kernel the predictor would pick, 1 the mma.sync kernel, 2 the tcgen05 kernel (hd 64, rows <= 384).
int jepa_b200_attention(const float * q, const float * kv, int n_cand, int n_frames, int rows, int heads, int hd,
                        int impl, float * out);
// The same attention timed alone on pseudo-random device-resident f16 operands: mean milliseconds per launch.
int jepa_b200_attention_bench(int n_cand, int n_frames, int rows, int heads, int hd, int impl, int reps, double * ms);

// Per-kernel device timing for measurement runs. Between begin and end, every launch of the engine's
// instrumented kernels (the AC predictor's GEMM, attention and row kernels) in this process is bracketed
// by CUDA events on its stream. end() synchronises and writes one line per kernel kind into `out`
// ("<kind> <launches> <total ms> <algorithmic FLOPs> <algorithmic bytes>\n", at most cap bytes with the
// terminating 0) and returns the number of kinds (-1 if an event failed). The events cost a little
// overlap between neighbouring kernels, so time the headline numbers without it.
void jepa_b200_kprof_begin(void);
int jepa_b200_kprof_end(char * out, size_t cap);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
