/*
 * elastikernel B200 C-ABI.
 *
 * Plain C entry points over the sm_100a kernels and the green-context shim.
 * Pointers are device pointers unless named host_*; every compute entry point
 * is asynchronous on the CUstream / cudaStream_t passed as `stream` (NULL = the
 * legacy default stream). All functions return EK_OK (0) or an EK_ERR_* code;
 * ek_last_error() gives the message of the last failure on the calling thread.
 *
 * num_sms: size of the SM partition the launch runs in. A value <= 0 means
 * "look the stream up in the green-context registry", falling back to the
 * device's full SM count for streams the registry does not know.
 *
 * Reference interfaces (Ther-LF/elastikernel) that each group replaces are
 * cited per declaration as file:line.
 */
#ifndef ELASTIKERNEL_H_
#define ELASTIKERNEL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EK_OK 0
#define EK_ERR_INVALID 1      /* bad argument (shape, alignment, pointer)   */
#define EK_ERR_CUDA 2         /* CUDA runtime / driver call failed           */
#define EK_ERR_OVERSUB 3      /* SM request exceeds what the device has      */
#define EK_ERR_UNSUPPORTED 4  /* configuration not supported by the kernels */
#define EK_ERR_DEVICE 5       /* a kernel reported a fault in the status word */

/* Element types for the GEMM entry points. */
#define EK_DTYPE_BF16 0
#define EK_DTYPE_FP16 1
#define EK_DTYPE_E4M3 2

/* Layout of the B operand of a dense GEMM. */
#define EK_B_KN 0 /* B is [K, N] row-major (the reference's b: b.stride(0) == N) */
#define EK_B_NK 1 /* B is [N, K] row-major (weight layout, K contiguous)        */

/* ------------------------------------------------------------------ misc */

/* Version of this ABI (major * 100 + minor). */
int ek_abi_version(void);

/* Message of the last error on this thread ("" if none). */
const char* ek_last_error(void);

/* Synchronise device `dev`, read the kernels' status word into *status_out and
 * clear it when `clear` != 0. Non-zero status means a kernel hit a bounded-wait
 * timeout or an out-of-range index (see the EK_STATUS_* bits). */
int ek_device_status(int dev, int clear, int* status_out);
#define EK_STATUS_WAIT_TIMEOUT 1
#define EK_STATUS_BAD_EXPERT 2
#define EK_STATUS_BAD_INDEX 4
#define EK_STATUS_BAD_SCALE 8  /* a block-scaled (_fp8mx) GEMM got a scale that is not a power of two */
#define EK_STATUS_CAPACITY 16  /* ek_ep_capacity_layout dropped slots past a rank's capacity */

/* --------------------------------------------------- green-context partitions
 * Replaces green_ctx.py (get_sm_alignment :46, get_total_sm_count :65,
 * _split_and_create_gc :84, _remaining_to_resource :110,
 * create_sm_partition :139, create_disjoint_partitions :169).
 */

/* Device facts: total SMs, (min SMs, alignment) of a green-context split by
 * compute capability (7.x -> (2,2), 8.x -> (4,2), >= 9 -> (8,8), as
 * green_ctx.py:46-62), and the compute capability itself. */
int ek_device_sm_info(int dev, int* total_sms, int* min_sms, int* alignment, int* cc_major, int* cc_minor);

/* Create n partitions on device `dev` with (already rounded) SM counts
 * counts[0..n). disjoint != 0 chain-splits each partition off the remainder of
 * the previous split (green_ctx.py:169-235); disjoint == 0 splits every
 * partition from the full device, so partitions may overlap
 * (green_ctx.py:139-166). On success streams_out[i] receives a non-blocking
 * CUstream bound to partition i and actual_out[i] its real SM count, read from
 * the split result. Raises EK_ERR_OVERSUB when the counts do not fit. The
 * green contexts are owned by the library until ek_gctx_destroy_all(). */
int ek_gctx_create(int dev, const int* counts, int n, int disjoint, void** streams_out, int* actual_out);

/* As ek_gctx_create with disjoint = 1, plus one more partition made of the
 * SMs the n requests left over: streams_out[n] / actual_out[n] (n + 1 entries
 * each). The reference turns that remainder into a resource for its next
 * split (green_ctx.py:110-132) but never hands it out; this exposes it, e.g.
 * a 32-SM communication partition and the 116 SMs beside it, which a
 * 116-SM request could not give (it rounds up to 120). EK_ERR_OVERSUB when
 * the requests leave no SMs over. */
int ek_gctx_create_remainder(int dev, const int* counts, int n, void** streams_out, int* actual_out);

/* SM count registered for `stream` (0 if the stream is not a partition). */
int ek_gctx_stream_sm_count(void* stream, int* sm_count_out);

/* Destroy every stream and green context created so far. */
int ek_gctx_destroy_all(void);

/* Test hook: replace the CUDA driver with an in-library simulation of a device
 * with `total_sms` SMs split in units of `granularity`; the call numbered
 * `fail_call` (0-based, -1 = never) returns driver error `fail_code`.
 * enable == 0 restores the real driver. Used by host-only tests. */
int ek_gctx_fake_driver(int enable, int total_sms, int granularity, int fail_call, int fail_code);

/* -------------------------------------------------------------------- GEMM
 * Replaces the Triton matmul_vanilla / matmul_sm_aware kernels and their
 * wrappers call_vanilla / call_sm_aware (sm_aware_matmul.py:148-234;
 * duplicate in sm_aware_benchmark.py:59-137), and the GEMM operator
 * run(A, B, C, M, N, K, NUM_SMS) (sm_aware_agent/definition.py:63-65).
 */

/* Tile schedule chosen for a GEMM of this shape on a partition of num_sms SMs. */
typedef struct ek_gemm_plan {
  int bm, bn, bk;          /* tile shape (bk in elements); bm = 256 for CTA pairs */
  int cta_pair;            /* 1: 2-SM MMA, two CTAs (a cluster) per tile         */
  int tiles_m, tiles_n;    /* output tiles along M and N                         */
  int k_blocks;            /* bk-wide steps along K                              */
  int num_tiles;           /* tiles_m * tiles_n                                  */
  int num_dp_tiles;        /* tiles computed whole by one CTA                    */
  int tail_split;          /* K-split factor of the remaining tiles (1 = none)   */
  int num_units;           /* schedulable work units                             */
  int grid;                /* CTAs launched (<= num_sms)                         */
  int num_sms;             /* partition size the plan was made for              */
  int waves;               /* ceil(num_units / grid)                             */
  double wave_efficiency;  /* useful K-steps / (grid * K-steps of busiest CTA)   */
  double est_us;           /* model estimate of the kernel time                  */
  size_t workspace_bytes;  /* scratch the schedule needs (split partials)        */
  int cluster_split;       /* > 1: K split into this many slices per tile, one  */
                           /* CTA (or, with cta_pair, one CTA pair) per slice,  */
                           /* the slices of a tile forming one thread-block     */
                           /* cluster and reduced through distributed shared    */
                           /* memory (no workspace); grid = num_units * (1 or 2) */
                           /* = num_tiles * cluster_split * (1 or 2);           */
                           /* 0 = persistent schedule                           */
} ek_gemm_plan;

/* Plan a GEMM C[M,N] = A[M,K] * B on num_sms SMs (num_sms > 0 required here).
 * force_bn pins the tile: > 0 one CTA per 128 x force_bn tile (64/128/192/256),
 * < 0 a CTA pair per 256 x -force_bn tile (128/256), 0 = choose.
 * force_split > 0 pins the tail split of the persistent schedule, < 0 the
 * cluster split into -force_split K slices (2, 4 or 8 single CTAs, or with
 * force_bn < 0 2 or 4 CTA pairs; bn 128 or 256), 0 = choose. The cluster
 * split is offered on a device's full SM count only
 * (cluster placement inside a green-context partition is not known) and
 * when every cluster fits on the device at once. */
int ek_gemm_plan_make(int M, int N, int K, int num_sms, int dtype, int b_layout, int force_bn, int force_split,
                      ek_gemm_plan* out);

/* Scratch bytes ek_gemm / ek_gemm_fp8 need for this call: plan.workspace_bytes
 * (0 when the schedule does not split), plus, for a bf16 / fp16 shape with N
 * not a multiple of 8 or K not a multiple of 16, the zero-padded operand
 * copies of that shape. Returns (size_t)-1 on invalid input. */
size_t ek_gemm_workspace_bytes(int M, int N, int K, int num_sms, int dtype, int b_layout, int force_bn,
                               int force_split);

/* C[M,N] = A[M,K] @ B, fp32 accumulate, C in the input dtype (bf16 / fp16).
 * A row-major [M,K]; B per b_layout; any M, N, K >= 1 (the reference's kernel
 * masks every edge, sm_aware_matmul.py:164-172): when N is not a multiple of 8
 * or K not a multiple of 16 the operands that need it are copied on the device
 * into zero-padded buffers inside the workspace, and the product's first N
 * columns are copied back into C. All pointers 16-byte aligned. workspace:
 * ws_bytes >= ek_gemm_workspace_bytes(...) bytes of device memory, zero-filled
 * before its first use; the kernel leaves its split counters at the front
 * zero-filled again, so it can be reused by later calls on the same stream. */
int ek_gemm(const void* A, const void* B, void* C, int M, int N, int K, int dtype, int b_layout, int num_sms,
            int force_bn, int force_split, void* workspace, size_t ws_bytes, void* stream);

/* FP8 e4m3 GEMM with per-row activation scales and per-output-channel weight
 * scales: C[M,N] = (A[M,K] * a_scale[M]) @ (W[N,K] * w_scale[N])^T, bf16 C.
 * N must be a multiple of 8 and K of 16. No counterpart kernel in the
 * reference (it has no FP8 path). */
int ek_gemm_fp8(const void* A, const void* W, const float* a_scale, const float* w_scale, void* C, int M, int N,
                int K, int num_sms, int force_bn, int force_split, void* workspace, size_t ws_bytes, void* stream);

/* FP8 e4m3 quantisation with fp32 scales. x is [rows, cols] bf16 (x_dtype 0)
 * or fp32 (x_dtype 3); q is [rows, cols] e4m3 codes. Scales are
 * amax / 448 per block (1 for an all-zero block) and q = e4m3(x / scale),
 * round-to-nearest-even, saturating:
 *   block_rows = 1, block_cols <= 0 : one scale per row, scales[rows]
 *   block_rows = 1, block_cols = 128: per 1 x 128 group, scales[rows][cols/128]
 *   otherwise                       : per block_rows x block_cols block,
 *                                     scales[ceil(rows/br)][ceil(cols/bc)].
 * No counterpart in the reference (it has no FP8 path). */
/* As ek_quant_e4m3 with 1 x 128 groups, the scales written K-block-major:
 * scales_t[g][r] ([ceil(cols/128)][rows]), the layout the FP8 block-scaled
 * grouped GEMMs read token scales in. No counterpart in the reference. */
int ek_quant_e4m3_kmajor(const void* x, int x_dtype, int rows, int cols, void* q, float* scales_t, void* stream);

int ek_quant_e4m3(const void* x, int x_dtype, int rows, int cols, int block_rows, int block_cols, void* q,
                  float* scales, void* stream);

/* ek_quant_e4m3 / ek_quant_e4m3_kmajor with flags. EK_QUANT_POW2_SCALES
 * rounds every scale up to the next power of two (amax / 448 unchanged if it
 * is one), so x / scale is an exact rescaling and each scale is a UE8M0
 * exponent: the form the block-scaled _fp8mx GEMMs take. No counterpart in
 * the reference (it has no FP8 path). */
#define EK_QUANT_POW2_SCALES 1
int ek_quant_e4m3_ex(const void* x, int x_dtype, int rows, int cols, int block_rows, int block_cols, int flags,
                     void* q, float* scales, void* stream);
int ek_quant_e4m3_kmajor_ex(const void* x, int x_dtype, int rows, int cols, int flags, void* q, float* scales_t,
                            void* stream);

/* GEMM for callers that cannot allocate device memory. No counterpart in the
 * reference. Same arguments and result as ek_gemm, minus the workspace: the
 * scratch for split K-slices comes from a fixed 32 MiB device array inside
 * the library (ek_gemm_noalloc_max_scratch_bytes()), held by every GPU that
 * loads it until exit. Intended for hosts that own all device memory (a
 * serving engine with its own pool that lends plugins no allocator) and for
 * paths that must not call cudaMalloc/cudaFree because those can synchronise
 * the device. Schedules needing more scratch fail with EK_ERR_UNSUPPORTED.
 * All calls on a device share the array: calls that overlap on the GPU race
 * and must be serialised by the caller. The first call on a device looks up
 * the array's address; make it before any stream capture on that device.
 * That address is cached per device index for the life of the process and
 * does not survive cudaDeviceReset (or any teardown of the device's primary
 * context): after one, later calls would hand the kernel a stale address, so
 * do not use this entry point again in that process. */
int ek_gemm_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int dtype, int b_layout, int num_sms,
                    int force_bn, int force_split, void* stream);
size_t ek_gemm_noalloc_max_scratch_bytes(void);

/* --------------------------------------------------------------------- MoE
 * Replaces the fused-MoE operator run(hidden_states, gate_logits, w1, w2, w3,
 * out, M, K, N, NUM_EXPERTS, TOP_K, NUM_SMS) (sm_aware_agent/definition.py:
 * 149-170) as four stages, and the segment kernels fused_moe_vanilla /
 * fused_moe_sm_aware with call_moe_vanilla / call_moe_sm_aware
 * (sm_aware_benchmark.py:228-391).
 */

/* Routing (definition.py:152-153): p = softmax(logits[t, :E]) in fp32,
 * top-k by probability (ties -> lower expert id first), weights renormalised
 * to sum 1. Writes topk_ids[T, k] (int32) and topk_weights[T, k] (fp32). */
int ek_moe_route(const float* logits, int T, int E, int topk, int* topk_ids, float* topk_weights, void* stream);

/* Rows of the padded, expert-sorted layout for T tokens, top-k, E experts and
 * block_m-row blocks: T*k + E*(block_m-1), rounded up to block_m. */
int64_t ek_moe_max_padded_rows(int T, int topk, int E, int block_m);

/* moe_align_block_size-style permutation. Flattened slots s = t*k + j are
 * stably sorted by expert id; each expert's run is padded to a multiple of
 * block_m with the sentinel T*k. Outputs:
 *   sorted_slots[max_padded_rows]  slot of each padded row (sentinel = T*k)
 *   block_expert[max_padded_rows / block_m]  expert of each row block (-1 past the end)
 *   num_rows_padded[1]             padded rows in use
 *   expert_counts[E]               slots routed to each expert
 * If x != NULL (x is [T, H], element size elem_bytes) the rows are also
 * gathered: x_perm[r] = x[sorted_slots[r] / k] for every row holding a slot;
 * padding rows are left unwritten (the GEMMs' outputs for them are never
 * stored or read).
 * scratch: ek_moe_permute_scratch_bytes(T, topk, E) bytes of device memory
 * (no initial contents required). */
size_t ek_moe_permute_scratch_bytes(int T, int topk, int E);
int ek_moe_permute(const int* topk_ids, int T, int topk, int E, int block_m, int* sorted_slots,
                   int* block_expert, int* num_rows_padded, int* expert_counts, const void* x, int H,
                   int elem_bytes, void* x_perm, void* scratch, void* stream);

/* ek_moe_route followed by ek_moe_permute, with the same outputs. Small
 * batches (T*topk <= 128) run both, and the row gather while the rows are
 * few, in one single-CTA launch (decode sizes are bound by launch latency);
 * larger batches run the separate launches (scratch as for ek_moe_permute). */
int ek_moe_route_permute(const float* logits, int T, int E, int topk, int* topk_ids, float* topk_weights,
                         int block_m, int* sorted_slots, int* block_expert, int* num_rows_padded, int* expert_counts,
                         const void* x, int H, int elem_bytes, void* x_perm, void* scratch, void* stream);

/* Grouped gate/up GEMM with fused SiLU-and-multiply over the padded rows:
 *   act[r, n] = silu(x_perm[r] . w1[e, n]) * (x_perm[r] . w3[e, n]),
 * e = block_expert[r / block_m], for r < *num_rows_padded; w1, w3 are
 * [E, I, H] bf16; act is [max_rows, I] bf16. num_slots (T * topk) only
 * guides the choice of tile width. block_m is the padding the layout was
 * permuted with: 128 (one CTA per 128-row tile) or 256 (2-SM CTA pairs with
 * 256 x 256 tiles; needs 2+ SMs and force_bn 0 or 256). */
int ek_moe_gate_up(const void* x_perm, const void* w1, const void* w3, const int* block_expert,
                   const int* num_rows_padded, void* act, int max_rows, int E, int H, int I, int num_slots,
                   int num_sms, int force_bn, int block_m, void* stream);

/* Grouped down projection with the top-k weight fused into the epilogue:
 *   y[s] = topk_weight[s] * (act[r] @ w2[e]^T),  s = sorted_slots[r] < T*k,
 * w2 is [E, H, I] bf16, y is [T*k, H] bf16. block_m as for ek_moe_gate_up. */
int ek_moe_down(const void* act, const void* w2, const int* block_expert, const int* num_rows_padded,
                const int* sorted_slots, const float* topk_weights, void* y, int max_rows, int E, int H, int I,
                int T, int topk, int num_sms, int force_bn, int block_m, void* stream);

/* Packed (expert-major) variants of the two grouped GEMMs, over the layout
 * ek_moe_permute produces with block_m = 1 (rows of expert e packed at
 * [start_e, start_e + expert_counts[e]), rows = T * topk, no padding). The
 * operands are swapped on the tensor cores: expert weight rows form the
 * 128-row (or 256-row with pair = 1, a 2-SM CTA pair) side and the expert's
 * tokens the N side, in tiles of tok_tile tokens (16/32/64/128/256). Weight
 * tiles stream from HBM once per token tile, which keeps small token counts
 * HBM-efficient. tok_tile = 0 and pair = -1 choose automatically. For the
 * gate/up GEMM pair = 2 asks for wide pair tiles (256 weight rows per CTA,
 * two accumulators sharing the token rows; token tiles 128 / 256, I % 256 ==
 * 0, no K-split; bit-identical results), never chosen automatically: in bf16
 * they measured slightly slower at the Mixtral shapes.
 * Results equal the block-padded variants' (within fp32 summation order).
 * E <= 256.
 *
 * workspace (16-byte aligned, ek_moe_packed_workspace_bytes(rows, H, I)
 * bytes, or NULL) lets the kernel split K when its units would fill the SMs
 * poorly (a few experts hit at small token counts): the kernel picks the
 * split from the expert counts on the device, writes fp32 slice sums to the
 * workspace, and a second launch adds the slices in order and applies the
 * SwiGLU / writes y. With NULL (or a smaller buffer) K is never split. */
int ek_moe_gate_up_packed(const void* x_perm, const void* w1, const void* w3, const int* expert_counts, void* act,
                          int rows, int E, int H, int I, int tok_tile, int pair, int num_sms, void* workspace,
                          size_t workspace_bytes, void* stream);
int ek_moe_down_packed(const void* act, const void* w2, const int* expert_counts, const int* sorted_slots,
                       const float* topk_weights, void* y, int rows, int E, int H, int I, int T, int topk,
                       int tok_tile, int pair, int num_sms, void* workspace, size_t workspace_bytes, void* stream);
/* Workspace for the K-split of the packed GEMMs (0: no split at this size;
 * rows = T * topk up to 64). Replaces nothing in the reference (its segment
 * GEMM has no split); serves the decode-sized Mixtral layer. */
size_t ek_moe_packed_workspace_bytes(int rows, int H, int I);

/* FP8 e4m3 packed grouped GEMMs with DeepSeek-style scales: weights with
 * 128 x 128 fp32 block scales (w*_scale [E*rows/128][K/128]), tokens with
 * 1 x 128 fp32 group scales stored K-block-major (x_scale / a_scale
 * [K/128][rows], as ek_quant_e4m3_kmajor writes them); fp32
 * accumulation with the scales applied per 128-wide K block; bf16 outputs as
 * ek_moe_gate_up_packed / ek_moe_down_packed. H and I must be multiples of
 * 128; tok = token tile (16/32/64/128 on one CTA, 128/160/192/256 on a CTA pair;
 * 0 = choose), pair = 1 for the CTA-pair (2-SM MMA) kernel, 0 for one CTA,
 * -1 = choose (the down projection runs a pair only when H % 256 == 0).
 * No counterpart in the reference (it has no FP8 path). */
int ek_moe_gate_up_fp8bs(const void* xq, const float* x_scale, const void* w1q, const void* w3q,
                         const float* w1_scale, const float* w3_scale, const int* expert_counts, void* act, int rows,
                         int E, int H, int I, int tok, int pair, int num_sms, void* stream);
int ek_moe_down_fp8bs(const void* aq, const float* a_scale, const void* w2q, const float* w2_scale,
                      const int* expert_counts, const int* sorted_slots, const float* topk_weights, void* y, int rows,
                      int E, int H, int I, int T, int topk, int tok, int pair, int num_sms, void* stream);

/* The same two grouped GEMMs with the scales applied by the tensor cores
 * (tcgen05.mma kind::mxf8f6f4.block_scale): every scale must be a power of
 * two (ek_quant_e4m3_ex with EK_QUANT_POW2_SCALES), and is used as a UE8M0
 * scale factor of each 32-element K chunk. The whole K reduction then
 * accumulates in TMEM, with one epilogue per tile instead of one scaled
 * accumulation per 128-wide K block. Same arguments and outputs as the
 * _fp8bs entry points; token tiles 16/32/64/128 on one CTA, 128/160/192 on a
 * CTA pair (tok 0 = choose). pair: -1 choose, 0 one CTA, 1 a CTA pair with
 * 128 weight rows per CTA, 2 a CTA pair with 256 weight rows per CTA (two
 * accumulators share each stage's token rows, which halves the token
 * re-reads per weight byte; needs I % 256 == 0 for gate/up, H % 512 == 0 for
 * down; chosen by -1 for gate/up from ~192 routed rows per expert). A scale
 * that is not a normal power of two sets
 * EK_STATUS_BAD_SCALE in the device status word. No counterpart in the
 * reference (it has no FP8 path). */
int ek_moe_gate_up_fp8mx(const void* xq, const float* x_scale, const void* w1q, const void* w3q,
                         const float* w1_scale, const float* w3_scale, const int* expert_counts, void* act, int rows,
                         int E, int H, int I, int tok, int pair, int num_sms, void* stream);
int ek_moe_down_fp8mx(const void* aq, const float* a_scale, const void* w2q, const float* w2_scale,
                      const int* expert_counts, const int* sorted_slots, const float* topk_weights, void* y, int rows,
                      int E, int H, int I, int T, int topk, int tok, int pair, int num_sms, void* stream);

/* Row gather of the padded/packed layout: dst[r] = src[sorted_slots[r] / topk]
 * for the used rows r < *num_rows_padded with a valid slot (row_bytes a
 * multiple of 16). Used to gather rows of a second tensor (e.g. FP8 scales)
 * with a permutation ek_moe_permute already made. */
/* Transposing gather of per-row fp32 values in the same permutation:
 * dst[c][r] = src[sorted_slots[r] / topk][c] for c < cols, r < max_rows
 * (0 for unused rows); turns received [rows][K/128] group scales into the
 * K-block-major layout of the FP8 block-scaled GEMMs. No counterpart in the
 * reference. */
int ek_moe_gather_cols_f32(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int topk,
                           const float* src, int cols, float* dst, void* stream);

int ek_moe_gather_rows(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int topk,
                       const void* src, int row_bytes, void* dst, void* stream);

/* Expert-parallel helpers (no counterpart in the reference, which has no
 * multi-GPU path). After a permutation by destination rank:
 *   ek_moe_slot_rows     slot_row[sorted_slots[r]] = r for the used rows
 *                        (the row each slot occupies in send order);
 *   ek_ep_pack_meta      per send row r: local_ids[r] = topk_ids[s] % experts_per_rank,
 *                        weights_out[r] = topk_weights[s], s = sorted_slots[r];
 *   ek_moe_combine_rows  out[t] = sum_j y[slot_row[t*k + j]] (fp32, j order), bf16,
 *                        rows outside [0, n_rows) skipped. */
int ek_moe_slot_rows(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int* slot_row,
                     void* stream);
int ek_ep_pack_meta(const int* sorted_slots, int rows, const int* topk_ids, const float* topk_weights, int n_slots,
                    int experts_per_rank, int* local_ids, float* weights_out, void* stream);
int ek_moe_combine_rows(const void* y, const int* slot_row, void* out, int T, int topk, int H, int n_rows,
                        void* stream);

/* Fixed-capacity dispatch layout: after ek_moe_permute by destination rank
 * (block_m = 1; sorted_slots and the per-rank dest_counts on the device),
 * lays the n_slots = T*k slots out as world blocks of `capacity` rows, so the
 * row all-to-all has equal splits known to the host. For capacity row
 * r = g*capacity + i: cap_slots[r] = the i-th slot bound for rank g (or
 * n_slots when rank g has <= i slots), local_ids[r] = its expert id local to
 * rank g (experts_per_rank, a dummy expert, for padding rows), weights_out[r]
 * = its routing weight (0 for padding). slot_row[s] = the capacity row of
 * slot s, or -1 when s is past its rank's capacity; such slots are dropped
 * and EK_STATUS_CAPACITY is raised in the device status word. The token rows
 * then go into the capacity layout with ek_moe_gather_rows(cap_slots, ...).
 * world <= 1024. */
int ek_ep_capacity_layout(const int* sorted_slots, const int* dest_counts, int world, int capacity, int n_slots,
                          const int* topk_ids, const float* topk_weights, int experts_per_rank, int* cap_slots,
                          int* local_ids, float* weights_out, int* slot_row, void* stream);

/* Peer-to-peer exchange primitives (expert-parallel all-to-all over NVLink
 * without NCCL; no counterpart in the reference, which has no multi-GPU
 * path). ek_p2p_mem_base: the base address and size of the device allocation
 * holding ptr (cuMemGetAddressRange). ek_p2p_ipc_handle: the 64-byte CUDA IPC
 * handle of an allocation base. ek_p2p_ipc_open / _close: map / unmap another
 * process's allocation on the current device (peer access enabled on
 * demand). ek_p2p_copy: cudaMemcpyAsync device to device on `stream` (the
 * copy engines; dst may be a peer mapping). ek_p2p_signal: after the work
 * queued before it on `stream`, store `value` into each of the n int flags
 * (peer mappings allowed) with system-scope release. ek_p2p_wait: on
 * `stream`, wait until each of the n local int flags holds a value >= `value`
 * (system-scope acquire; bounded: after 2 s EK_STATUS_WAIT_TIMEOUT is raised
 * and the wait ends). n <= 64. */
int ek_p2p_mem_base(const void* ptr, unsigned long long* base, size_t* size);
int ek_p2p_ipc_handle(const void* base, void* handle_out);
int ek_p2p_ipc_open(const void* handle, void** ptr);
int ek_p2p_ipc_close(void* ptr);
int ek_p2p_copy(void* dst, const void* src, size_t bytes, void* stream);
int ek_p2p_signal(void* const* flags, int n, int value, void* stream);
int ek_p2p_wait(const int* flags, int n, int value, void* stream);
/* Device-side epochs, for exchanges replayed from a CUDA graph:
 * ek_p2p_signal_dev increments the local int *counter and stores the new
 * value into the n flags; ek_p2p_wait_dev (next on the same stream) waits
 * until each of the n local flags holds a value >= *counter (bounded as
 * ek_p2p_wait). */
int ek_p2p_signal_dev(void* const* flags, int n, int* counter, void* stream);
int ek_p2p_wait_dev(const int* flags, int n, const int* counter, void* stream);

/* Top-k combine: out[t] = sum_{j<k} y[t*k + j] (fp32 sum in j order), bf16 out. */
int ek_moe_combine(const void* y, void* out, int T, int topk, int H, void* stream);

/* Segment GEMM with the reference kernel's semantics
 * (sm_aware_benchmark.py:228-290): for each expert e with rows
 * [offsets[e], offsets[e+1]) of hs[M, K]:
 *   out[rows] = hs[rows] @ Wblk_e,   Wblk_e = weights + e*N*K viewed as [K, N],
 * i.e. the expert's [N, K] block read as a row-major [K, N] matrix.
 * fp16 / bf16 in and out (dtype), fp32 accumulate. */
int ek_moe_segment_gemm(const void* hs, const void* weights, const int* offsets, void* out, int M, int N, int K,
                        int E, int dtype, int num_sms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ELASTIKERNEL_H_ */
