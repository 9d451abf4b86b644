/*
 * tfb200.h - C ABI of the B200 (sm_100a) kernels behind
 * transformer_optimization_b200.UserOptimizedTransformer.
 *
 * The reference (namsengi11/transformer_optimization) has no native code and
 * no FFI: its hot path, UserOptimizedTransformer.forward
 * (torch_transformer_benchmark.py:3509-3611, per-layer schedule 4003-4326),
 * calls Triton kernels and ATen through Python wrappers. Each entry point
 * below replaces one of those wrappers; the comment on each names it.
 *
 * Conventions
 *   - Plain device pointers, element counts/strides in ELEMENTS, int64 sizes.
 *   - `stream` is a cudaStream_t (CUstream) passed as void*; NULL = legacy
 *     default stream. Every call only enqueues work: no host synchronisation,
 *     no device allocation (all buffers are caller-owned), safe inside CUDA
 *     graph capture once the same call has run once on the device.
 *   - Return 0 (TF_OK) or a TF_ERR_* code; tf_last_error() gives the message.
 *     Kernels never trap: a pipeline wait that exceeds its time bound writes a
 *     code into the device status word (read with tf_device_status) and the
 *     kernel returns.
 *   - fp16 = IEEE binary16 ("half"), bf16 = bfloat16, fp32 = binary32.
 *   - Two model precisions: the fp32 model (fp16 tensor-core operands, fp32
 *     residual stream and statistics: the reference's fp32-model fast path)
 *     and the half-precision models (fp16 or bf16 parameters and
 *     activations, type T below; every stored tensor is T as in the
 *     reference's eager model run in T). Flags select the second.
 */
#ifndef TFB200_H
#define TFB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define TF_OK 0
#define TF_ERR_SHAPE 1       /* unsupported or inconsistent sizes */
#define TF_ERR_ALIGN 2       /* pointer / stride alignment */
#define TF_ERR_LAUNCH 3      /* CUDA launch or attribute error */
#define TF_ERR_UNSUPPORTED 4 /* device is not sm_100 */
#define TF_ERR_DEVICE 5      /* CUDA runtime error outside a launch */
#define TF_ERR_DRIVER 6      /* driver entry point (tensor-map encode) */
#define TF_ERR_TIMEOUT 7     /* a kernel wait ran out (see tf_device_status) */

/* tf_ln_residual flags */
#define TF_LN_MASK_DELTA 1 /* zero invalid rows of delta before the add */
#define TF_LN_MASK_X 2     /* zero invalid rows of x after the add */
#define TF_LN_MASK_OUT 4   /* zero invalid rows of the normalised output */
#define TF_LN_WRITE_X 8    /* store the updated residual into x_out */
#define TF_LN_OUT_F32 16   /* normed is fp32 (default fp16) */
#define TF_LN_X_F16 32     /* x, delta, x_out and normed are fp16; x + delta is rounded to fp16 */
#define TF_LN_X_BF16 64    /* x, delta, x_out and normed are bf16; x + delta is rounded to bf16 */

/* tf_gemm epilogues (low bits) and options; T = the operand type */
#define TF_EPI_BIAS 0       /* C = T(acc + bias) */
#define TF_EPI_BIAS_GELU 1  /* C = T(gelu_erf(acc + bias)), GELU in fp32 */
#define TF_EPI_BIAS_GELU_ROUNDED 2 /* C = T(gelu_erf(T(acc + bias))): F.gelu applied to the
                                      stored T output of the Linear (half-precision models) */
#define TF_EPI_W_SPLIT 16   /* W is [N, 2K] = [W_hi | W_lo] (W_lo = fp16(W - W_hi)) */
#define TF_EPI_BF16 32      /* A, W and C are bf16 (default fp16) */

/* tf_gemm_residual mask modes (the reference's two masking points), low 2 bits */
#define TF_RES_NO_MASK 0
#define TF_RES_MASK_DELTA 1 /* invalid rows: x_out = x_in (delta zeroed) */
#define TF_RES_MASK_X 2     /* invalid rows: x_out = 0 */
/* and options, or-ed into the mask mode */
#define TF_RES_X16 4   /* x_in / x_out in the operand type T (default fp32):
                          x_out = T(mask_x(x_in + mask_delta(T(acc + bias)))) */
#define TF_RES_BF16 8  /* A and W (and x with TF_RES_X16) are bf16 (default fp16) */

/* tf_flash_fwd flags */
#define TF_ATTN_CAUSAL 1  /* mask key position > query position */
#define TF_ATTN_OUT_F32 2 /* out is fp32 (default: q's type) */
#define TF_ATTN_EXP_F16X2 4 /* packed fp16 exp2 for the probabilities (default:
                               fp32 exp2, the faster of the two on B200; P is
                               rounded to fp16 for the PV product either way);
                               fp16 operands only */
#define TF_ATTN_BF16 8      /* q, k, v and out (unless TF_ATTN_OUT_F32) are bf16;
                               P is rounded to bf16 for the PV product */
#define TF_ATTN_ROUND_SCORES 16 /* the scores of the eager model run in the operand
                               type T: T(T(q . k) * scale), then the fp32 softmax
                               (half-precision models; default: fp32 scores);
                               not with TF_ATTN_EXP_F16X2 or FMA-pipe exponentials */
/* flags bits 8..15: how many of the 64 probability pairs per row and key
 * block are exponentiated on the FMA pipes instead of the exp unit
 * (0, 8, 16 or 24; with TF_ATTN_EXP_F16X2: 0 or 16; fp16 operands only) */
#define TF_ATTN_FMA_EXP_SHIFT 8

/* ABI version, bumped on any signature change. */
int tf_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* tf_last_error(void);

/* Synchronises `stream`, then returns the device status word of the current
 * device in *code (0 = no kernel wait ran out) and clears it.
 * No reference counterpart: the reference's Triton wrappers raise
 * (torch_transformer_benchmark.py:1053-1058) and cannot time out. */
int tf_device_status(int* code, void* stream);

/* Test hook for the bounded waits every pipeline kernel uses: launches one
 * CTA that starts a 4 KiB bulk copy from `src` (16-byte aligned device
 * memory of at least 4096 bytes) into shared memory, then waits on an
 * mbarrier that nothing completes. That wait runs out after `limit_ns`
 * (1000 .. 2e9) and records device code 106 in the status word; the thread
 * then waits for its own copy (the drain every kernel does before it
 * leaves) and returns. out: int32[3] device memory; out[0] = 1 when the wait
 * ran out, out[1] = 1 when the copy drained, out[2] = the last byte copied.
 * Afterwards tf_device_status returns TF_ERR_TIMEOUT with code 106 and sets
 * tf_last_error; the device stays usable. No reference counterpart: the
 * reference's kernels cannot time out; its guard is a host-side kill switch
 * around the fast path (torch_transformer_benchmark.py:2368-2403). */
int tf_test_wait_timeout(const void* src, int64_t limit_ns, int* out, void* stream);

/* One residual-add + LayerNorm site over a contiguous [M, D] activation:
 *   x_new  = mask_x(x + mask_delta(fp32(delta)))
 *   normed = mask_out(LayerNorm(x_new) * w + b)       (fp16 or fp32 store)
 * x and x_out fp32, delta fp16 [M, D] or NULL (no add); with TF_LN_X_F16 /
 * TF_LN_X_BF16 x, delta, x_out and normed are all that 16-bit type and
 * x_new = T(x + delta) (statistics in fp32 either way). valid is uint8 [M]
 * (nonzero = valid token) or NULL when no mask flag is set; x_out may alias
 * nothing else and is written only with TF_LN_WRITE_X. w, b fp32. D must be
 * a multiple of 8, <= 4096.
 * Replaces _ln_site / _triton_add_layernorm / _add_ln_kernel
 * (torch_transformer_benchmark.py:3940-4001, 1038-1108, 884-962) and, for
 * half-precision models, `x + delta` followed by nn.LayerNorm
 * (torch_transformer_benchmark.py:218-222, 245). */
int tf_ln_residual(const void* x, const void* delta, const float* w, const float* b, float eps,
                   const uint8_t* valid, int64_t M, int64_t D, int flags, void* x_out, void* normed,
                   void* stream);

/* 16-bit GEMM, fp32 accumulation on tcgen05 tensor cores:
 *   C[M, N] = epilogue(A[M, K] * W[N, K]^T + bias[N])
 * A row-major with pitch lda, W = nn.Linear weight [N, K] (or [N, 2K] with
 * TF_EPI_W_SPLIT) with pitch ldw, C row-major with pitch ldc; A, W, C fp16
 * (bf16 with TF_EPI_BF16), bias fp32. N % 32 == 0, K and pitches % 8 == 0,
 * pointers 16-byte aligned.
 * Replaces _lin / _triton_linear / _triton_gemm_gelu / F.linear on the
 * fp16-GEMM path (torch_transformer_benchmark.py:4138-4194, 1860-1906,
 * kernel 1756-1803). */
int tf_gemm(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C, int64_t ldc,
            int64_t M, int64_t N, int64_t K, int epilogue, void* stream);

/* tf_gemm with an explicit tiling, for tuning and tests: tile_n = N tile
 * (64, 128 or 256; 0 = automatic); pair = 1 one-CTA 128-row tiles, 2 two-SM
 * 256-row tiles on a CTA pair (tile_n 128 or 256), 0 = automatic. */
int tf_gemm_tiled(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C,
                  int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int tile_n, int pair, void* stream);

/* GEMM whose epilogue closes a residual connection:
 *   x_out[M, N] = mask_x(x_in + mask_delta(A * W^T + bias))
 * x_in / x_out fp32 with pitch ldx (x_out may equal x_in: in place); valid
 * uint8 [M] for the mask modes. mask_mode may carry TF_RES_X16 (x in the
 * operand type, with the half-precision model's two roundings) and
 * TF_RES_BF16 (bf16 operands). w_split != 0: W is [N, 2K] = [W_hi | W_lo]
 * (fp16 operands only).
 * tile_n / pair: tiling as in tf_gemm_tiled (0, 0 = automatic).
 * Replaces out_proj / ffn_out (torch_transformer_benchmark.py:4163-4169,
 * 4194) together with the residual add of the following _ln_site
 * (torch_transformer_benchmark.py:3988-3995). */
int tf_gemm_residual(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                     const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                     int64_t M, int64_t N, int64_t K, int w_split, int tile_n, int pair, void* stream);

/* A residual GEMM and the LayerNorm of its output running at the same time.
 * tf_gemm_residual_ready is tf_gemm_residual (automatic tiling, x_out
 * contiguous: ldx == N) whose epilogue also adds, for every group of 8 rows,
 * the number of x_out columns it has stored to ready[group]; a group is
 * complete when its count reaches N. ready: int32[ceil(M / 8) + 2] device
 * array, all zero before the call (the last two entries are tf_ln_ready's
 * ticket counters; the GEMM does not touch them).
 * tf_ln_ready is tf_ln_residual without delta (normed = mask_out(LayerNorm(x)
 * * w + b); flags TF_LN_MASK_OUT, TF_LN_OUT_F32, TF_LN_X_F16, TF_LN_X_BF16;
 * D <= 2048) for x being written by a tf_gemm_residual_ready launched just
 * before it on the same stream with the same ready array and N == D: it waits
 * per row group for the count D instead of for the GEMM to finish, so its
 * CTAs run on the SMs the GEMM's last, partial wave leaves idle; groups are
 * handed out in ascending order from the ticket counters; each count it
 * consumes and the ticket counters are set back to 0, so the array is ready
 * for the next pair.
 * After a failed call (or a device timeout) zero the array again. A count
 * that never completes ends in device code 107 after the 2 s wait bound.
 * Replaces out_proj / ffn_out with the residual add and the LayerNorm of the
 * following _ln_site (torch_transformer_benchmark.py:4163-4169, 4194,
 * 3940-4001) or the final LayerNorm (4316-4325). */
int tf_gemm_residual_ready(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                           const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                           int64_t M, int64_t N, int64_t K, int w_split, int* ready, void* stream);
int tf_ln_ready(const void* x, const float* w, const float* b, float eps, const uint8_t* valid, int64_t M,
                int64_t D, int flags, void* normed, int* ready, void* stream);

/* Split-K forms of tf_gemm / tf_gemm_residual for few-row inputs (small
 * batch x sequence), where 128-row tiles leave most SMs idle: each tile's
 * K range is cut into `splits` parts (splits <= 0: automatic, about one work
 * unit per SM); every part writes its fp32 partial product into `workspace`,
 * and a second kernel sums the parts in a fixed order (deterministic), adds
 * the bias and applies the same epilogue as the unsplit call. `workspace`:
 * device memory of at least tf_gemm_splitk_workspace(M, N, K, splits)
 * bytes, 16-byte aligned, owned by the caller; calls on one workspace must
 * not overlap in time. No split weights (w_split). Same projections as
 * tf_gemm / tf_gemm_residual (torch_transformer_benchmark.py:4138-4194;
 * residual add 3988-3995). */
int64_t tf_gemm_splitk_workspace(int64_t M, int64_t N, int64_t K, int splits);
int tf_gemm_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C, int64_t ldc,
                   int64_t M, int64_t N, int64_t K, int epilogue, int splits, void* workspace,
                   int64_t workspace_bytes, void* stream);
int tf_gemm_residual_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                            const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                            int64_t M, int64_t N, int64_t K, int splits, void* workspace, int64_t workspace_bytes,
                            void* stream);

/* tf_gemm_residual_splitk whose reduce kernel also runs the LayerNorm of the
 * result (one warp per row):
 *   x_out  = as tf_gemm_residual_splitk
 *   normed = mask_out(LayerNorm(x_out) * ln_w + ln_b)      ([M, N] contiguous)
 * normed is fp16 (the operand type with TF_RES_X16; fp32 with TF_LN_OUT_F32);
 * ln_flags: TF_LN_MASK_OUT (rows where valid is 0 become 0), TF_LN_OUT_F32.
 * ln_w, ln_b fp32 [N]; N <= 4096. For few-row inputs, where every kernel is
 * bound by its launch and memory latency, this saves one launch per residual
 * site over tf_gemm_residual_splitk followed by tf_ln_residual. Replaces
 * out_proj / ffn_out with the residual add and the LayerNorm of the
 * reference's next _ln_site (torch_transformer_benchmark.py:4163-4169, 4194,
 * 3940-4001) or its final LayerNorm (4316-4325). */
int tf_gemm_residual_ln_splitk(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                               const void* x_in, void* x_out, int64_t ldx, const uint8_t* valid, int mask_mode,
                               int64_t M, int64_t N, int64_t K, int splits, void* workspace,
                               int64_t workspace_bytes, const float* ln_w, const float* ln_b, float eps,
                               void* normed, int ln_flags, void* stream);

/* tf_gemm_splitk without a workspace argument: the fp32 partial sums go to a
 * fixed 4 MiB device array inside this library, so the call allocates
 * nothing and needs no caller-provided memory. For callers that cannot
 * allocate device memory at the point of the call: code that must not call
 * an allocator there (cudaMalloc synchronises the device and is not
 * permitted while a stream is being captured), and foreign-language hosts
 * that have no device allocator to hand a workspace through the C
 * interface. Limit: splits * M * N * 4 bytes (tf_gemm_splitk_workspace)
 * must not exceed 4 MiB; larger calls return TF_ERR_SHAPE. Every GPU that
 * loads the library holds its copy of the array until the process exits. The
 * array is shared by all calls on a device and keeps the last call's
 * contents (a call writes every partial it reads, so nothing needs
 * clearing); calls that overlap on the GPU (on different streams or from
 * different host threads) race on it and must be serialised by the caller. The first call on each device looks up the
 * array's address (cudaGetSymbolAddress, once, with that device current);
 * make that first call before any stream capture. No reference counterpart:
 * the reference has no FFI and allocates its temporaries through PyTorch. */
int tf_gemm_splitk_static(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, void* C,
                          int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int splits, void* stream);

/* Flash attention forward (online softmax, no score matrix in HBM):
 *   out[b, i, h*hd:(h+1)*hd] = sum_j softmax_j(scale * q_i . k_j) v_j
 * q: fp16 (bf16 with TF_ATTN_BF16), token i of batch b, head h at
 * q + b*bs_q + i*ld_q + h*hd;
 * k, v: same with ld_kv / bs_kv over seq_k tokens; out: q's type (or fp32
 * with TF_ATTN_OUT_F32) with ld_o / bs_o. lse: fp32 [batch, heads, seq_q] natural
 * log-sum-exp of the scaled scores per row, or NULL. key_valid: uint8
 * [batch, seq_k] (nonzero = key may be attended) or NULL. With
 * TF_ATTN_CAUSAL key j is masked when k_pos0 + j > q_pos0 + i (positions
 * are global token indices, for context-parallel blocks). A row with no
 * admissible key gets out = 0 and lse = -inf. head_dim 64 or 128.
 * Replaces F.scaled_dot_product_attention / _triton_short_attention /
 * _flash_attn_kernel on the fp16 path (torch_transformer_benchmark.py:
 * 4146-4161, 1306-1418, 1193-1304). */
int tf_flash_fwd(const void* q, const void* k, const void* v, int64_t ld_q, int64_t ld_kv, int64_t bs_q,
                 int64_t bs_kv, void* out, int64_t ld_o, int64_t bs_o, float* lse, const uint8_t* key_valid,
                 int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k, int64_t head_dim, float scale,
                 int64_t q_pos0, int64_t k_pos0, int flags, void* stream);

/* Merge one partial attention result into a running one (log-sum-exp
 * combination, exact): with L = logaddexp(lse_acc, lse_part)
 *   o_acc   = o_acc * exp(lse_acc - L) + o_part * exp(lse_part - L)
 *   lse_acc = L
 * o_acc, o_part: fp32 [batch, seq_q, heads*head_dim] with pitch ld (tokens)
 * and bs (batches); lse_*: fp32 [batch, heads, seq_q]. If out16 is not NULL
 * the merged result is also written there as fp16 (pitch ld16, bs16).
 * No reference counterpart: the reference has no context parallelism; this
 * is the combine step of the ring attention that replaces its capacity
 * streaming (torch_transformer_benchmark.py:4686-4771, 4933-5013). */
int tf_attn_merge(float* o_acc, float* lse_acc, const float* o_part, const float* lse_part, int64_t ld,
                  int64_t bs, void* out16, int64_t ld16, int64_t bs16, int64_t batch, int64_t heads,
                  int64_t seq_q, int64_t head_dim, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TFB200_H */
