/* C-ABI of the B200 (sm_100a) block-scaled FP8 linear path.
 *
 * Everything here takes plain device pointers, sizes and a CUDA stream passed as void*, returns
 * 0 or a positive error code, and never throws. Kernels run asynchronously on the given stream;
 * nothing allocates or synchronises except where a comment says so.
 *
 * Data formats (all row-major, all on one device):
 *   A   e4m3 activations [M, K]                    (K % 128 == 0, 16-byte aligned base)
 *   As  fp32 activation group scales [M, K/128]    (one scale per token and 128-wide K group)
 *   B   e4m3 weights, either row-major [N, K] or "tile-first" [N/128][K/128][128][128]
 *       (bs_fp8_pack_tiles makes the latter)
 *   Bs  fp32 weight block scales [N/128, K/128]    (one scale per 128x128 block)
 *   C   bf16 or fp32 output [M, ldc], columns 0..N-1 written
 *   Q   e4m3 quantised SiLU(gate)*up [M, N/2], Qs fp32 group scales [M, N/256]
 *
 * Reference interfaces are cited as path:line inside lexing-2026/ucloud-ai-infra;
 * "H" is patches/fp8_hand_sm89.py.
 */
#ifndef BS_FP8_H
#define BS_FP8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define BS_OK 0
#define BS_ERR_ARG 1          /* a shape, stride or dtype argument is outside the contract   */
#define BS_ERR_ALIGN 2        /* a pointer or row stride breaks the 16-byte alignment rule     */
#define BS_ERR_WORKSPACE 3    /* workspace missing or smaller than bs_fp8_workspace_bytes()    */
#define BS_ERR_TMAP 4         /* cuTensorMapEncodeTiled is unavailable or rejected the tensor  */
#define BS_ERR_CUDA 5         /* a CUDA runtime call failed (launch, attribute, device query)  */
#define BS_ERR_BUILD 6        /* a kernel's register count does not match its setmaxnreg split */
#define BS_ERR_SCRATCH 7      /* bs_fp8_gemm_noalloc: the shape needs more than its fixed scratch   */
#define BS_ERR_TIMEOUT_FULL 101     /* device status: bounded wait on a TMA stage ran out       */
#define BS_ERR_TIMEOUT_EMPTY 102    /* device status: bounded wait for a free stage ran out     */
#define BS_ERR_TIMEOUT_PFULL 103    /* device status: bounded wait for an MMA partial ran out   */
#define BS_ERR_TIMEOUT_PEMPTY 104   /* device status: bounded wait for a TMEM buffer ran out    */
#define BS_ERR_TIMEOUT_DRAIN 105    /* device status: teardown drain ran out                    */
#define BS_ERR_TIMEOUT_PEER 106     /* device status: a peer rank did not reach the TP reduce   */
#define BS_ERR_TIMEOUT_SELFTEST 199 /* device status: the self-test wait ran out (expected)     */

/* Block-scaled FP8 GEMM:  C[m, n] = sum_kb (A[m, kb] . B[n, kb]) * As[m, kb] * Bs[n/128, kb].
 * Replaces the launch inside H:704-719 (`matmul(A, B, C, As, Bs, M, N, K, block_size)`, kernel
 * `fp8_gemm_hand(pA, pB, pC, pAs, pBs, M, N, G)` at H:104-105) and the Triton
 * `w8a8_block_fp8_matmul_triton(A, B, As, Bs, block_size, output_dtype)` it hooks
 * (patches/apply_sglang_fp8_hand_gemm.py:26-33).
 *   b_tiled    1 if B is tile-first (H:667 layout), 0 if row-major [N, K]
 *   out_dtype  0 = bf16 (the reference's only output), 1 = fp32 (tensor-parallel partials)
 *   ldc        output row stride in elements, >= N, multiple of 8
 * M <= 128 runs the swap-AB split-K decode kernel and needs `workspace` of at least
 * bs_fp8_workspace_bytes(M, N, K, 0) bytes, zero-filled before its first use. Its first 64 KB are
 * per-tile arrival counters (at most 16384 weight tiles, N <= 2097152), which every call leaves at
 * zero, so one workspace serves any sequence of shapes on its stream. M > 128 needs no workspace; given
 * one of bs_fp8_workspace_bytes(M, N, K, 0) bytes (nonzero only for plain prefill shapes whose whole tiles
 * would fill the last wave of SMs poorly and whose K has 32+ blocks), those shapes run stream-K: every CTA
 * takes an equal range of (tile, K block) units and tiles shared by two CTAs are summed in a fixed order
 * through the workspace, under the same zeroed-counter rule.
 * M == 0 is a no-op. */
int bs_fp8_gemm(const void* A, const void* B, void* C, const float* As, const float* Bs, int M, int N, int K,
                int ldc, int b_tiled, int out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Fused MLP front half: gate_up GEMM -> SiLU(gate) * up -> per-token-group e4m3 quant.
 * B holds N2 = 2*I weight rows, gate rows first (I % 128 == 0). Writes Q [M, I] and Qs [M, I/128]
 *   y = silu(g) * u;  Qs = max(amax_128(|y|), 1e-10) / 448;  Q = sat_e4m3(y * (1 / Qs)).
 * Replaces kernel `fp8_gemm_silu_quant(pA, pB, pQ, pAs, pBs, pQs, M, N, G)` (H:341-342,
 * epilogue H:532-579) launched by `fused_gate_up(proj, x)` (H:675-701). Same workspace rule as
 * bs_fp8_gemm, with bs_fp8_workspace_bytes(M, N2, K, 1). */
int bs_fp8_gemm_silu_quant(const void* A, const void* B, void* Q, const float* As, const float* Bs, float* Qs,
                           int M, int N2, int K, int b_tiled, void* workspace, size_t workspace_bytes,
                           void* stream);

/* bs_fp8_gemm for a row-parallel layer of a tensor-parallel group, fused with the group's reduction:
 * C_mc is the multicast address (NVLink SHARP / NVLS, one buffer mapped on every rank of the group) of
 * a bf16 [M, ldc] output, and every output tile this rank computes is added, in bf16 by the switch, into
 * all ranks' copies (multimem.red.add). Replaces the NCCL all_reduce(sum) of the bf16 partials that
 * follows the row-parallel down_proj (the reference runs one GPU, scripts/run_sglang_48g.sh:117: there
 * the product is the whole sum). The caller zeroes every rank's copy and synchronises the group before
 * the call, and synchronises the group again before reading C. The order in which ranks' additions land
 * is not fixed, so the last bits of C may differ from run to run. Same arguments, workspace rule and
 * status codes as bs_fp8_gemm with out_dtype 0. */
int bs_fp8_gemm_reduce_multicast(const void* A, const void* B, void* C_mc, const float* As, const float* Bs, int M,
                                 int N, int K, int ldc, int b_tiled, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Tensor-parallel sum of the ranks' bf16 partials, in place, through the NVSwitch (no counterpart in the
 * reference, which runs TP=1: scripts/run_sglang_48g.sh:117; it replaces the all_reduce after the
 * row-parallel down_proj). Every rank calls it with the same arguments except `rank`, on its own GPU:
 *   data_mc   multicast address of a symmetric bf16 buffer of `count` elements (count % 8 == 0) that holds
 *             this rank's partial in its own copy; on return every copy holds the sum (the same bytes);
 *   flags     this rank's copy of a symmetric uint32 buffer of bs_fp8_tp_flag_words(world) words, zeroed
 *             once before the first call; flags_mc its multicast address;
 *   epoch     1 on the first call and one more on every later call with the same flags (all ranks alike);
 *   limit_ns  bound on each wait for the peers (0: 4 s); a rank that runs out records
 *             BS_ERR_TIMEOUT_PEER in the status word (bs_fp8_status) and its peers run out after it.
 * Rank r reads the r-th 1/world of the buffer reduced by the switch (fp32 accumulation, one bf16 rounding)
 * and stores the sums into every copy, so each GPU moves about (world-1)/world of the buffer each way. The
 * launch is stream-ordered after the GEMM that wrote the partial, and returns only after every rank has
 * finished writing into this rank's copy and reading from it. */
int bs_fp8_tp_reduce_switch(unsigned long long data_mc, void* flags, unsigned long long flags_mc, long long count,
                            int rank, int world, unsigned int epoch, unsigned long long limit_ns, void* stream);

/* uint32 words of the flag buffer bs_fp8_tp_reduce_switch needs for `world` ranks (0 for world < 2). */
long long bs_fp8_tp_flag_words(int world);

/* Allocation-free variant of bs_fp8_gemm, for callers that cannot call cudaMalloc (an engine that
 * reserves all device memory up front, an embedding whose only allocator is its own arena, a
 * thread that must not block on the driver's allocator). No counterpart in the reference.
 * Same arguments and results as bs_fp8_gemm without the workspace: decode shapes (M <= 128) use
 * a fixed 4 MiB scratch array inside the library (held on every GPU that loads it until exit);
 * a shape whose split-K scratch would exceed it returns BS_ERR_SCRATCH. The first call on a
 * device looks up that array's device address, so make it before any stream capture. Every call
 * shares the array: calls that overlap on the GPU (different streams, or concurrent host
 * threads) race on it. It allocates nothing (no cudaMalloc/cudaFree); it clears the array's
 * counter words with cudaMemsetAsync on `stream` before each launch. */
int bs_fp8_gemm_noalloc(const void* A, const void* B, void* C, const float* As, const float* Bs, int M, int N,
                        int K, int ldc, int b_tiled, int out_dtype, void* stream);

/* The unfused chain's activation between the gate_up GEMM and the activation quant (only when the fused
 * kernel is off: SGLANG_FP8_HAND_FUSED=0): gate_up bf16 [M, 2I] (row stride ld_in) -> out bf16 [M, I] (row
 * stride ld_out) with out = bf16(silu(g) * u) in fp32, one rounding, g = gate_up[:, :I], u = gate_up[:, I:].
 * Replaces SGLang's silu_and_mul in the chain the reference restates at
 * logs/artifacts/20261031_hand/fused_test.py:30-34 (its fallback for M < 1024, H:678-687). I % 8 == 0,
 * strides multiples of 8, pointers 16-byte aligned. */
int bs_fp8_silu_mul(const void* gate_up, int ld_in, void* out, int ld_out, int M, int I, void* stream);

/* Workspace bytes for (M, N, K): the 64 KB counter prefix plus the partial tiles. Decode shapes (M <= 128):
 * what the split-K kernel needs (0 when the shape has more than 16384 weight tiles). Prefill shapes: the
 * stream-K workspace (two 128 x 256 fp32 partial tiles per SM) when the plain GEMM runs stream-K, else 0.
 * 0 for M == 0. */
size_t bs_fp8_workspace_bytes(int M, int N, int K, int fused);

/* Per-token-group activation quant: x bf16 [M, K] (row stride ldx elements, multiple of 8) ->
 * A e4m3 [M, K], As fp32 [M, K/128] with As = max(amax_128(|x|) / 448, 1e-12), A = e4m3(x / As).
 * Replaces SGLang's `per_token_group_quant_fp8(x, 128)` called at H:690-693, with the
 * arithmetic of the reference's torch quantiser (scripts/fp8_gemm_factor_check.py:22-27). */
int bs_fp8_group_quant(const void* x, int ldx, void* A, float* As, int M, int K, void* stream);

/* RMSNorm fused with the per-token-group quant (the activation quant of the next linear), without
 * storing the bf16 norm output: h = x, or h = bf16(x + residual) written back to residual (row stride
 * ldr; residual may be NULL); y = bf16((h * (1 / sqrt(mean(h^2) + eps))) * weight[K]); then A, As as
 * bs_fp8_group_quant(y). Replaces the pair "RMSNorm -> per_token_group_quant_fp8(., 128)" ahead of
 * the hooked linears (H:690-693), in the way the reference fuses the group quant into its GDN output
 * norm (patches/apply_sglang_gdn_prefill.py:538-591). Bit-exact with that pair computed with the
 * fixed summation order stated in the kernel. K: multiple of 128, at most 16384. */
int bs_fp8_rmsnorm_group_quant(const void* x, int ldx, void* residual, int ldr, const void* weight, float eps,
                               void* A, float* As, int M, int K, void* stream);

/* Tile-first weight pre-pack: tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c] for e4m3 W [N, K].
 * Replaces the permute in `relayout(model)` (H:667). W and tiles must not overlap. */
int bs_fp8_pack_tiles(const void* W, void* tiles, int N, int K, void* stream);

/* Reads the device status word of the current device (synchronises the device). Writes the
 * code to *code and clears it when `clear` is non-zero. Counterpart of the reference's
 * RuntimeError on driver failures (H:630, :634, :649); here kernels report bounded-wait
 * timeouts through it. */
int bs_fp8_status(int* code, int clear);

/* Runs one tiny kernel whose mbarrier wait is never satisfied and must give up after
 * `limit_ns`, leaving BS_ERR_TIMEOUT_SELFTEST in the status word. Exercises the bounded-wait
 * path without any fault. No reference counterpart (the reference has no bounded waits). */
int bs_fp8_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* Launch plan of one GEMM call: what bs_fp8_gemm (fused = 0) or bs_fp8_gemm_silu_quant (fused = 1) launches
 * for an M x N x K problem on the current device (148 SMs assumed when no device is usable). Fills
 * plan[0 .. BS_PLAN_FIELDS) (n >= BS_PLAN_FIELDS) with the fields below; returns BS_ERR_ARG for a shape the
 * GEMMs refuse. Replaces the tile table behind `select(N, M)` (H:51-57, :74-87), which reported the sm_89
 * kernel variant for a product. */
#define BS_PLAN_KIND 0        /* 1 decode (swap-AB, M <= 128), 2 prefill                                   */
#define BS_PLAN_TILE_ROWS 1   /* decode: weight rows per tile (128); prefill: output rows (128, 256 pairs) */
#define BS_PLAN_TILE_COLS 2   /* decode: tokens padded to a multiple of 16; prefill: output columns (256)  */
#define BS_PLAN_STAGES 3      /* TMA pipeline stages                                                       */
#define BS_PLAN_THREADS 4     /* threads per CTA                                                           */
#define BS_PLAN_GRID 5        /* CTAs launched                                                             */
#define BS_PLAN_CLUSTER 6     /* CTAs per cluster (2: CTA pairs)                                           */
#define BS_PLAN_GROUP_M 7     /* prefill raster: M tiles per group (tiles walk down each weight column)    */
#define BS_PLAN_RESERVED 8    /* 0                                                                         */
#define BS_PLAN_TMEM_COLS 9   /* TMEM columns allocated per CTA                                            */
#define BS_PLAN_SPLIT 10      /* decode: 0 one CTA per weight tile, s > 0 equal K splits, -1 stream-K      */
#define BS_PLAN_WARPGROUPS 11 /* promotion warpgroups                                                      */
#define BS_PLAN_SMEM 12       /* dynamic shared memory bytes per CTA                                       */
#define BS_PLAN_TILES 13      /* prefill: output tiles walked by the persistent CTAs                       */
#define BS_PLAN_FIELDS 14
int bs_fp8_launch_plan(int M, int N, int K, int fused, int* plan, int n);

/* Number of SMs the kernels size their persistent grids for (current device): all of them, or
 * BS_FP8_SM_LIMIT from the environment when that is smaller (SMs left to concurrent kernels). */
int bs_fp8_num_sms(void);

/* Human-readable text for a status code. */
const char* bs_fp8_error_string(int code);

/* ABI version of this library (bumped when a signature changes). */
int bs_fp8_abi_version(void);

/* Text of the last CUDA runtime failure (BS_ERR_CUDA) seen on the calling thread: which call
 * failed and the runtime's error name. Empty when none. Counterpart of the detail the
 * reference puts in its RuntimeError messages (H:630, :634, :649). */
const char* bs_fp8_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* BS_FP8_H */
