/*
 * frx.h -- C ABI of libfrx.so, the B200 (sm_100a) engine behind the drop-in
 * fast_reduction.gemm_kernel API: fused linear + cross-entropy + entropy.
 *
 * Conventions (all entry points):
 *   - Every pointer is a device pointer owned by the caller; the library allocates no device
 *     memory. Matrices are row-major with an explicit leading dimension in elements.
 *   - Every call is asynchronous on `stream` (a cudaStream_t, passed as void*; NULL = legacy
 *     default stream) and returns FRX_OK (0) or an FRX_ERR_* code. The message for the last
 *     failure on the calling thread is available from frx_last_error(). Nothing aborts.
 *   - `status` (optional, may be NULL) is a device int the kernels OR FRX_STATUS_* bits into
 *     when they detect a problem while running (a pipeline wait that timed out, a target id
 *     outside the vocabulary). The host reads it whenever it chooses to synchronise.
 *   - Vocabulary sharding: a call may cover only the slice [vocab_offset, vocab_offset +
 *     vocab_shard) of the vocabulary; `target` always holds global vocabulary ids.
 *   - 16-bit operands (bf16, or fp16 where a `dtype` argument says so) need 16-byte aligned bases
 *     and leading dimensions that are multiples of 8.
 *
 * The forward partials contract: for vocabulary tile t (columns [256 t, 256 t + 256) of the
 * shard) and row r, partials[t * tile_stride + r] holds four floats
 *     m  = max_j z_j,  s = sum_j exp(z_j - m),  u = sum_j (z_j - m) exp(z_j - m),  zt
 * where zt = z_target when the row's target falls in the tile, else 0. The reference's own
 * epilogue stores sx = sum_j z_j exp(z_j - m) in the third slot instead of u; frx_finalize
 * accepts that layout with FRX_PARTIALS_REF_LAYOUT.
 */
#ifndef FRX_H_
#define FRX_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FRX_API __attribute__((visibility("default")))
#else
#define FRX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FRX_ABI_VERSION 4

#define FRX_OK 0
#define FRX_ERR_INVALID_ARG 1
#define FRX_ERR_UNSUPPORTED 2
#define FRX_ERR_CUDA 3

#define FRX_DTYPE_BF16 0
#define FRX_DTYPE_F32 1
#define FRX_DTYPE_F16 2

/* Or-ed into the out_dtype of frx_gemm_dhidden / frx_gemm_dweight with FRX_DTYPE_F32: the product is
 * added to the fp32 values the output already holds (several launches accumulate one result). */
#define FRX_OUT_ACCUMULATE 256

/* frx_split_f32 part selectors (2 bits per part, part p at bits [2p, 2p+2)) */
#define FRX_PART_HI 0
#define FRX_PART_MID 1
#define FRX_PART_LO 2

/* Width of one vocabulary tile of the forward partials (columns per partial). */
#define FRX_VOCAB_TILE 256

/* frx_finalize flags */
#define FRX_PARTIALS_REF_LAYOUT 1 /* third slot holds sum z*exp(z-m) (reference layout) */
#define FRX_IGNORE_NEGATIVE_TARGETS 2 /* every target < 0 is ignored (ce = log_probs = 0) */

/* device status bits */
#define FRX_STATUS_TIMEOUT_PRODUCER 1
#define FRX_STATUS_TIMEOUT_MMA 2
#define FRX_STATUS_TIMEOUT_EPILOGUE 4
#define FRX_STATUS_BAD_TARGET 8
#define FRX_STATUS_DRAIN_TIMEOUT 16
#define FRX_STATUS_CHECK_FAILED 32 /* a device-side invariant check of a checked build failed */

/* ABI version of the loaded library (FRX_ABI_VERSION it was built with). */
FRX_API int frx_abi_version(void);

/* Message describing the most recent failed call on this thread ("" if none). */
FRX_API const char* frx_last_error(void);

/*
 * Forward GEMM with the CE / entropy reduction fused into its epilogue.
 * Replaces the reference's GEMM-epilogue launch `_gemm_ce_entropy_kernel`
 * (fast_reduction/gemm_kernel.py:58-165; epilogue math gemm_ce_entropy_epilogue.py:184-271)
 * and, with `logits` non-NULL, the logits-writing variant `_gemm_ce_entropy_bwd_kernel`
 * (gemm_kernel.py:168-273, gemm_ce_entropy_bwd_epilogue.py:218).
 *
 *   z[r, j]  = sum_k hidden[r, k] * weight[j, k]        (16-bit x 16-bit -> fp32, TMEM)
 *   dtype    FRX_DTYPE_BF16 or FRX_DTYPE_F16: the type of hidden, weight and bias
 *   hidden   [rows, hidden_dim], row stride ld_hidden
 *   weight   [vocab_shard, hidden_dim], row stride ld_weight (the shard's rows)
 *   bias     optional [vocab_shard] added to every logit of its column (z = x W^T + b, as the
 *            reference's fp32 baseline computes; the reference's own GEMM path ignores bias)
 *   target   [rows] int64 global ids, or NULL (then zt = 0)
 *   partials [ceil(vocab_shard / 256) * tile_stride] x float4, tile_stride >= rows
 *   logits   optional fp32 [rows, ld_logits] output of every z (NULL: logits never leave the chip);
 *            16-byte aligned, ld_logits a multiple of 4. The TMA stores write whole 16-byte chunks,
 *            so the pad columns [vocab_shard, round_up(vocab_shard, 4)) of each row may be written
 *            too: the buffer must extend to that column in its last row.
 */
FRX_API int frx_fwd_partials(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                     int dtype, const void* bias, const int64_t* target, int64_t rows, int64_t vocab_shard,
                     int64_t hidden_dim, int64_t vocab_offset, float* partials, int64_t tile_stride, float* logits,
                     int64_t ld_logits, int* status, void* stream);

/*
 * frx_fwd_partials, writing fp16 tile-relative logits instead of fp32 logits: for each row r and
 * column j of vocabulary tile t,
 *   logits_rel[r, j] = fp16(z[r, j] - m)     m = the tile maximum this launch writes to slot 0 of
 *                                             partials[t * tile_stride + r]
 * rounded to nearest (values below -65504 become -inf). Half the bytes of the fp32 logits; each
 * stored value is within 2^-11 |z - m| of z - m (2^-25 absolute near 0), so the error of a
 * probability exp(z - lse) formed from it grows with its distance below its tile's maximum, where
 * the probabilities themselves shrink as exp(-|z - m|).
 * frx_dlogits_tilerel reads them back. Replaces, like the fp32 `logits` output of
 * frx_fwd_partials, the logits store of `_gemm_ce_entropy_bwd_kernel` (fast_reduction/gemm_kernel.py:168-273,
 * gemm_ce_entropy_bwd_epilogue.py:218), which writes fp32.
 *   logits_rel  fp16 [rows, ld_logits_rel], 16-byte aligned, ld_logits_rel a multiple of 8; the pad
 *               columns [vocab_shard, round_up(vocab_shard, 8)) of each row may be written (whole
 *               16-byte chunks), so the buffer must extend to that column in its last row
 */
FRX_API int frx_fwd_partials_tilerel(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                                     int dtype, const void* bias, const int64_t* target, int64_t rows,
                                     int64_t vocab_shard, int64_t hidden_dim, int64_t vocab_offset, float* partials,
                                     int64_t tile_stride, void* logits_rel, int64_t ld_logits_rel, int* status,
                                     void* stream);

/*
 * Merges per-tile partials into per-row results.
 * Replaces the reference's `Finalize` kernel and its custom ops
 * (fast_reduction/gemm_ce_entropy_finalize.py:29-102, 123-212).
 *
 *   lse = M + log S,  entropy = log S - U / S,  ce = lse - ZT,  log_probs = -ce
 * Rows whose target equals ignore_index get ce = 0 and log_probs = 0 (torch nll_loss
 * semantics), or, with FRX_IGNORE_NEGATIVE_TARGETS, every row whose target is negative (the rule
 * of the reference's standalone reductions); other targets outside [0, vocab_size) give NaN and
 * set FRX_STATUS_BAD_TARGET.
 * target may be NULL (no CE semantics check). Any of ce/entropy/lse/log_probs may be NULL.
 * `merged` (optional, float4 per row) receives the merged (M, S, U, ZT) in the u layout, for a
 * further cross-shard merge (call frx_finalize again with n_tiles = number of shards).
 */
FRX_API int frx_finalize(const float* partials, int64_t n_tiles, int64_t rows, int64_t tile_stride, int flags,
                 const int64_t* target, int64_t vocab_size, int64_t ignore_index, float* ce,
                 float* entropy, float* lse, float* log_probs, float* merged, int* status, void* stream);

/*
 * dlogits of loss = sum_r g_ce[r] * ce[r] + g_ent[r] * entropy[r] for one vocabulary shard:
 *   p = exp(z - lse);  dz = p * (g_ce - g_ent * (log p + H)) - g_ce * [j == target]
 * Replaces `ComputeDlogits` / `compute_dlogits` (fast_reduction/cute_dlogits.py:32-100, 162-183).
 * g_ce / g_ent: per-row fp32 vectors, or NULL to use the scalars ce_weight / ent_weight.
 * Rows with target == ignore_index drop the CE term. out_dtype: FRX_DTYPE_BF16, _F16 or _F32.
 */
FRX_API int frx_dlogits(const float* logits, int64_t ld_logits, const int64_t* target, const float* lse,
                const float* entropy, const float* g_ce, const float* g_ent, float ce_weight,
                float ent_weight, void* dlogits, int64_t ld_dlogits, int out_dtype, int64_t rows,
                int64_t vocab_shard, int64_t vocab_offset, int64_t ignore_index, void* stream);

/*
 * frx_dlogits from the fp16 tile-relative logits of frx_fwd_partials_tilerel and the partials of the
 * same launch (tile maximum m_t in slot 0 of partials[t * tile_stride + r]):
 *   log p = max(logits_rel, -65504) - (lse - m_t),  dz = p * (g_ce - g_ent * (log p + H)) - g_ce * [j == target]
 * Reads 2 bytes per logit instead of 4. The values are z minus the maximum of their tile, so never
 * positive: the kernel decodes them from their magnitude bits (a positive value would be read as
 * its negation). Same arguments and rules as frx_dlogits otherwise.
 * Replaces `ComputeDlogits` / `compute_dlogits` (fast_reduction/cute_dlogits.py:32-100, 162-183)
 * in the training pass.
 */
FRX_API int frx_dlogits_tilerel(const void* logits_rel, int64_t ld_logits_rel, const float* partials,
                                int64_t tile_stride, const int64_t* target, const float* lse, const float* entropy,
                                const float* g_ce, const float* g_ent, float ce_weight, float ent_weight,
                                void* dlogits, int64_t ld_dlogits, int out_dtype, int64_t rows, int64_t vocab_shard,
                                int64_t vocab_offset, int64_t ignore_index, void* stream);

/*
 * d_hidden[rows, hidden_dim] = dlogits[rows, vocab_shard] @ weight[vocab_shard, hidden_dim]
 * (in_dtype = FRX_DTYPE_BF16 or _F16 for both inputs, fp32 accumulation, out_dtype out: BF16, F16
 * or F32, or F32 | FRX_OUT_ACCUMULATE to add into the output). Replaces the cuBLAS
 * `torch.mm(dlogits, weight)` of the reference's megakernel
 * (fast_reduction/gemm_kernel.py:859-862).
 */
FRX_API int frx_gemm_dhidden(const void* dlogits, int64_t ld_dlogits, const void* weight, int64_t ld_weight,
                     int in_dtype, void* d_hidden, int64_t ld_d_hidden, int out_dtype, int64_t rows, int64_t hidden_dim,
                     int64_t vocab_shard, int* status, void* stream);

/*
 * Vocabulary-parallel d_hidden with the cross-rank sum fused into the GEMM: this rank's
 * contribution dlogits[rows, vocab_shard] @ weight[vocab_shard, hidden_dim] is ADDED, tile by tile
 * from the epilogue, into an fp32 [rows, hidden_dim] matrix through its NVLink-SHARP multicast
 * address `d_hidden_mc` (multimem.red.add), so every rank's copy ends up holding the sum over ranks.
 * The caller zeroes every rank's copy before any rank calls this, and synchronises the ranks after
 * all of them have called it before reading. Replaces the GEMM + separate NCCL all-reduce of
 * d_hidden (no counterpart in the single-GPU reference; its d_hidden GEMM is
 * fast_reduction/gemm_kernel.py:859-862).
 */
FRX_API int frx_gemm_dhidden_multicast(const void* dlogits, int64_t ld_dlogits, const void* weight,
                                       int64_t ld_weight, int in_dtype, void* d_hidden_mc, int64_t ld_d_hidden,
                                       int64_t rows, int64_t hidden_dim, int64_t vocab_shard, int* status,
                                       void* stream);

/*
 * d_weight[vocab_shard, hidden_dim] = dlogits[rows, vocab_shard]^T @ hidden[rows, hidden_dim]
 * (in_dtype = FRX_DTYPE_BF16 or _F16 for both inputs) accumulated over all `rows` in fp32 tensor
 * memory and written once in out_dtype (BF16, F16 or F32, or F32 | FRX_OUT_ACCUMULATE). Replaces
 * the per-chunk `d_weight.add_(torch.mm(dlogits.t(), h_chunk).float())` and the final cast
 * of the reference (fast_reduction/gemm_kernel.py:864-871).
 */
FRX_API int frx_gemm_dweight(const void* dlogits, int64_t ld_dlogits, const void* hidden, int64_t ld_hidden,
                     int in_dtype, void* d_weight, int64_t ld_d_weight, int out_dtype, int64_t vocab_shard,
                     int64_t hidden_dim, int64_t rows, int* status, void* stream);

/*
 * frx_gemm_dweight on at most `max_sms` SMs (0: all of them). The GEMM is persistent and otherwise
 * holds every SM until it ends; leaving some free lets work on another stream run beside it, such as
 * the collective that sums the vocabulary-parallel d_hidden while this GEMM computes d_weight. No
 * counterpart in the single-GPU reference (its d_weight GEMM is fast_reduction/gemm_kernel.py:864-871).
 */
FRX_API int frx_gemm_dweight_sms(const void* dlogits, int64_t ld_dlogits, const void* hidden, int64_t ld_hidden,
                                 int in_dtype, void* d_weight, int64_t ld_d_weight, int out_dtype,
                                 int64_t vocab_shard, int64_t hidden_dim, int64_t rows, int max_sms, int* status,
                                 void* stream);

/*
 * Splits an fp32 matrix x [rows, cols] (row stride ld_x) into bf16 parts for the bf16x6 emulation of
 * an fp32 matrix product on the bf16 tensor cores (Henry, Tang, Heinecke, "Leveraging the bfloat16
 * Artificial Intelligence Datatype For Higher-Precision Computations", ARITH 2019):
 *   hi = bf16(x),  mid = bf16(x - hi),  lo = bf16(x - hi - mid)   (x = hi + mid + lo to ~24 bits).
 * For p < n_parts, part p (FRX_PART_HI / _MID / _LO, selected by bits [2p, 2p+2) of `parts`) is
 * written to out + p * part_stride as a [rows, cols] bf16 matrix with row stride ld_out. With the left
 * operand split as (hi, hi, mid, hi, lo, mid) and the right as (hi, mid, hi, lo, hi, mid), the six
 * products sum to x.y up to the dropped mid*lo, lo*mid and lo*lo terms (~2^-24 relative): an fp32
 * product. Replaces the fp32 matmul the reference runs for fp32 inputs (fast_reduction/kernel.py:32-45
 * `_mm_setup`; gemm_kernel.py:859-866).
 */
FRX_API int frx_split_f32(const float* x, int64_t ld_x, int64_t rows, int64_t cols, uint32_t parts, int n_parts,
                          void* out, int64_t ld_out, int64_t part_stride, void* stream);

/*
 * Column sums out[c] = sum_r x[r, c] (fp32 accumulation, fixed order, so deterministic) of a bf16 or
 * fp16 (dtype) matrix [rows, cols] with row stride ld: the bias gradient from the dlogits of one shard.
 * Replaces the reference's `d_bias.add_(dlogits.sum(dim=0))` (fast_reduction/gemm_kernel.py:867-869).
 */
FRX_API int frx_column_sums(const void* x, int dtype, int64_t ld, int64_t rows, int64_t cols, float* out,
                            void* stream);

/*
 * Softmax partials of a materialised logits matrix [rows, cols] (dtype FRX_DTYPE_BF16, _F16 or
 * _F32, row stride ld elements): for each tile of tile_cols columns and each row, the same
 * (m, s, u, zt) float4 as frx_fwd_partials writes (zt = logits[row, target] when the target lies in
 * the tile), at partials[tile * tile_stride + row]; frx_finalize then gives ce / entropy / lse.
 * Replaces the reference's standalone row reductions CrossEntropyOnly / EntropyOnly /
 * CrossEntropyEntropy and their custom ops ce_fwd / entropy_fwd / ce_entropy_fwd[_lse]
 * (fast_reduction/cute_cross_entropy.py:171-578, 583-735). target may be NULL.
 */
FRX_API int frx_logits_partials(const void* logits, int dtype, int64_t ld, int64_t rows, int64_t cols,
                                const int64_t* target, int64_t tile_cols, float* partials, int64_t tile_stride,
                                void* stream);

/*
 * Forward CE / entropy / lse / log_probs in one call that allocates no device memory: the
 * partials live in a 32 MiB scratch array that is part of the library image on each GPU.
 * No counterpart in the reference. For callers that cannot call cudaMalloc (a framework that
 * owns all device memory, a serving loop that must not synchronise on an allocation, a fixed
 * memory budget). hidden and weight must both be bf16 (there is no dtype argument; fp16 data
 * would be read as bf16). Limit: ceil(vocab_size / 256) * rows * 16 bytes <= 32 MiB, i.e. at
 * most floor(2097152 / ceil(vocab_size / 256)) rows per call (4185 at V = 128256); larger calls
 * return FRX_ERR_INVALID_ARG before any GPU work. All calls on a device share the scratch, so
 * calls that overlap on the GPU race. The first call on a device looks up the scratch address;
 * under CUDA's lazy module loading that is also when the driver reserves the 32 MiB on that
 * device, so make one small warm-up call at start-up, before handing the remaining memory to
 * another allocator and before any stream capture. The whole vocabulary is one shard (targets
 * are plain vocabulary ids).
 */
FRX_API int frx_fwd_ce_entropy_noalloc(const void* hidden, int64_t ld_hidden, const void* weight,
                                       int64_t ld_weight, const int64_t* target, int64_t rows,
                                       int64_t vocab_size, int64_t hidden_dim, int64_t ignore_index,
                                       float* ce, float* entropy, float* lse, float* log_probs, int* status,
                                       void* stream);

/*
 * loss[0] = ce_weight * sum_r ce[r] + ent_weight * sum_r entropy[r] over `rows` fp32 values (either
 * input may be NULL and then counts as zero), accumulated in fp64 in a fixed order: deterministic.
 * Replaces the reference's `ce_weight * ce.sum() + ent_weight * ent.sum()`
 * (fast_reduction/gemm_kernel.py:897).
 */
FRX_API int frx_loss_sum(const float* ce, const float* entropy, int64_t rows, float ce_weight, float ent_weight,
                         float* loss, void* stream);

/*
 * x[i] *= scale[0] for n elements of dtype FRX_DTYPE_BF16, _F16 or _F32 (16-bit values are scaled in
 * fp32 and rounded to nearest). The scale is read on the device when the kernel runs; when it is
 * exactly 1 the kernel returns without touching x, so the caller needs no host synchronisation to
 * skip the work. Replaces the reference's `d_hidden * dloss` / `d_weight * dloss` in the
 * megakernel's backward (fast_reduction/gemm_kernel.py:905-913), done in place on the stored
 * gradients.
 */
FRX_API int frx_scale_inplace(void* x, int dtype, int64_t n, const float* scale, void* stream);

/*
 * FRX_OK when the `bytes` bytes from `ptr` lie inside one device allocation (cuMemGetAddressRange),
 * else FRX_ERR_INVALID_ARG with the overrun in frx_last_error(). Checked builds (libfrx_checked.so,
 * built with FRX_CHECKED=1) run this on every buffer before each launch; it is exported by every
 * build as a debugging aid. No counterpart in the reference.
 */
FRX_API int frx_check_range(const void* ptr, int64_t bytes);

/*
 * Measurement aid: when the stream reaches it, blocks spread over the GPU write, for each SM s they
 * land on, out[2s] = that SM's cycle counter (%clock64) and out[2s + 1] = the global timer in
 * nanoseconds (%globaltimer); slots of SMs no block landed on are left as they were (zero them
 * first). Two probes around a timed region give its average SM clock per SM:
 * (c1 - c0) / (t1 - t0) GHz. `out` holds 2 * max_sms values. No counterpart in the reference.
 */
FRX_API int frx_clock_probe(uint64_t* out, int max_sms, void* stream);

/*
 * Test hook for failure detection (not part of the computation): runs the bf16 forward of
 * frx_fwd_partials with k-block `stall_kb` of each CTA pair's first tile left unfilled on purpose, so
 * the MMA warp's bounded wait on that pipeline stage runs out after `wait_limit_us` microseconds
 * (every wait of this launch uses that limit). The kernel then takes its abort path: every role
 * leaves its loop, in-flight copies and MMAs are waited for (bounded), tensor memory is freed, and
 * FRX_STATUS_TIMEOUT_* bits are set in `status`. Nothing faults and the context stays usable; the
 * partials of the affected tiles are left unwritten. No counterpart in the reference.
 */
FRX_API int frx_test_stalled_fwd(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                                 const int64_t* target, int64_t rows, int64_t vocab_shard, int64_t hidden_dim,
                                 float* partials, int64_t tile_stride, int stall_kb, int64_t wait_limit_us,
                                 int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FRX_H_ */
