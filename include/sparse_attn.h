/*
 * sparse_attn.h — C ABI of libsparse_attn.so, the B200 (sm_100a) top-k sparse
 * attention with attention sink.
 *
 * Semantics are those of track-01 of inin-zou/kernelgen-challenge:
 *   o[b,m,h,:] = sum_t softmax([s_0 .. s_{topk-1}, sink[h]])_t * kv[b, idx[b,m,t], :]
 *   s_t        = scale * <q[b,m,h,:], kv[b, idx[b,m,t], :]>     (fp32 accumulate)
 * (track-01/reference/reference.py:10-40).  A slot whose index is -1 is
 * masked (score -inf, row not read), as in the reference's NVIDIA-path kernel
 * track-01/submission.py:313-322; any other index outside [0, kv_len) is
 * masked the same way (the reference leaves it undefined).  A row with no
 * valid slot yields o = 0.
 *
 * Every entry point below replaces one piece of the reference's Python
 * boundary, the function sparse_attn(q, kv, attn_sink, topk_idxs, scale) at
 * track-01/submission.py:975-1021 (validation :989, contiguity :995-998,
 * output allocation :1000, kernel launch :1006-1021).
 *
 * Conventions
 *   - bf16 tensors are passed as untyped pointers to 16-bit words.
 *   - All device pointers live on the device that is current for the calling
 *     thread; `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - The caller owns every buffer (inputs, output, workspace).  sa_fwd never
 *     allocates device memory and never synchronises; all work is ordered on
 *     `stream`.
 *   - Reentrant: concurrent calls on different streams/devices are allowed if
 *     they use different workspaces.
 *   - Return value 0 = success, negative = error (SA_ERR_*); sa_strerror()
 *     gives a message, sa_last_cuda_error() the last cudaError_t seen by the
 *     calling thread.
 */
#ifndef SPARSE_ATTN_H_
#define SPARSE_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SA_OK 0
#define SA_ERR_INVALID_ARG (-1) /* null pointer, bad shape/stride/alignment */
#define SA_ERR_WORKSPACE (-2)   /* workspace missing or too small          */
#define SA_ERR_CUDA (-3)        /* CUDA runtime error (see last_cuda_error) */
#define SA_ERR_UNSUPPORTED (-4) /* h % 16 != 0, d != 512, or no sm_100 device */

/* Kernel variants for sa_fwd_ex (SA_VARIANT_AUTO picks the default, WS). */
#define SA_VARIANT_AUTO 0
#define SA_VARIANT_MMA 1     /* all-warp mma.sync, cp.async ring, __syncthreads     */
#define SA_VARIANT_TCGEN05 2 /* S^T by tcgen05 (TMEM), P.V warp MMAs, mbarrier pipe */
#define SA_VARIANT_WS 3      /* warp-specialized: cp.async + TMA(Q) producers,      */
                             /* mma.sync consumers with Q in registers (default)    */
#define SA_VARIANT_WT 4      /* as WS, with P.V on tcgen05.mma and O in TMEM        */

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int sa_version(void);

/* Human-readable text for an SA_* return code. */
const char* sa_strerror(int code);

/* 1 if kernel variant `variant` (SA_VARIANT_*) is built into this library and
 * can run on the current device's architecture, else 0.  No counterpart in
 * the reference (its backend probe is track-01/submission.py:927-969). */
int sa_variant_available(int variant);

/* fp8 KV cache.  kv8 is [b, kv_len, 512] e4m3 (torch.float8_e4m3fn) bytes,
 * kv_scale is [b, kv_len] fp32, and row t of batch b stands for the bf16 row
 * kv8[b,t,:] * kv_scale[b,t].  The result is sa_fwd on that dequantised cache.
 * The e4m3 values are widened to f16 in registers (exact) and both products
 * run as f16 tensor-core MMAs with fp32 accumulation; q (scaled per head by a
 * power of two) and the softmax weights are f16, so accuracy is at least the
 * bf16 path's.  kv_strides are in bytes (rows
 * 16-byte aligned); kv_scale_strides are in elements.  The workspace is sized
 * by sa_workspace_bytes.  grid_ctas = 0 picks one CTA per SM.  q must be
 * 16-byte aligned (it is loaded by TMA).  The gathered bytes per slot are 516
 * instead of 1024.  The reference has no fp8 cache; this replaces
 * track-01/submission.py:975-1021 for callers that keep one. */
int sa_fwd_fp8(const void* q, const void* kv8, const float* kv_scale, const float* sink,
               const int32_t* idx, void* o, int64_t b, int64_t m, int64_t h, int64_t d,
               int64_t kv_len, int64_t topk, const int64_t q_strides[4],
               const int64_t kv_strides[3], const int64_t kv_scale_strides[2],
               const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
               void* workspace, size_t workspace_bytes, void* stream, int grid_ctas);

/* Training forward: sa_fwd (warp-specialized kernel) that also writes
 * lse[b*m][h] (fp32): log2 of each row's full softmax denominator, the sink
 * included, in the log2 domain of the scores (weight of slot t =
 * 2^(s_t * scale * log2(e) - lse)).  sa_bwd then needs one pass instead of
 * two.  No counterpart in the reference, which has no backward. */
int sa_fwd_train(const void* q, const void* kv, const float* sink, const int32_t* idx, void* o,
                 float* lse, int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len,
                 int64_t topk, const int64_t q_strides[4], const int64_t kv_strides[3],
                 const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Backward pass: gradients of sa_fwd.  Given q, kv, sink, idx, the forward's
 * output o, its lse from sa_fwd_train (or NULL: recomputed by a first pass)
 * and the upstream gradient dout (laid out like o: o_strides), writes
 * dq (bf16, contiguous [b, m, h, 512]) and ADDS into dkv (fp32 [b, kv_len, 512],
 * element strides dkv_strides, multiples of 4, 16-byte aligned) and dsink
 * (fp32 [h]); zero those two first for a plain gradient.  Masked slots (-1 or out of range)
 * contribute nothing; duplicated indices add.  The math is the gradient of
 * the reference forward (track-01/reference/reference.py:24-40), which has no
 * backward of its own. */
int sa_bwd(const void* q, const void* kv, const float* sink, const int32_t* idx, const void* o,
           const void* dout, const float* lse, void* dq, float* dkv, float* dsink, int64_t b,
           int64_t m, int64_t h,
           int64_t d, int64_t kv_len, int64_t topk, const int64_t q_strides[4],
           const int64_t kv_strides[3], const int64_t idx_strides[3], const int64_t o_strides[4],
           const int64_t dkv_strides[3], float scale, void* stream);

/* sa_bwd with an optional fp32 scratch for dq.  dq_acc (NULL, or zero-filled
 * fp32 laid out like dq: contiguous [b, m, h, 512], 16-byte aligned) lets
 * a call with the forward's lse and fewer query rows than half the SMs
 * (decode) cut each row's slots into parts that run on separate CTAs; the
 * parts add their dq into dq_acc and the library then writes dq from it.
 * Otherwise, and with dq_acc NULL, it is sa_bwd.  No counterpart in the
 * reference, which has no backward. */
int sa_bwd_ex(const void* q, const void* kv, const float* sink, const int32_t* idx,
              const void* o, const void* dout, const float* lse, void* dq, float* dkv,
              float* dsink, int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len,
              int64_t topk, const int64_t q_strides[4], const int64_t kv_strides[3],
              const int64_t idx_strides[3], const int64_t o_strides[4],
              const int64_t dkv_strides[3], float scale, float* dq_acc, void* stream);

/* The kv rows that one call's valid slots name (idx as for sa_fwd), in a
 * dense fp32 KV gradient laid out like the dkv of sa_bwd (strides multiples
 * of 4, 16-byte aligned).  A decode-shaped backward touches only
 * b * m * topk of the b * kv_len rows, so a caller that needs the dense
 * gradient can zero just those rows of an uninitialised fp32 buffer before
 * sa_bwd (sa_dkv_zero_rows) and afterwards cast just those rows into a
 * zero-filled bf16 gradient (sa_dkv_cast_rows: out rows of 512 bf16,
 * strides out_strides, multiples of 4, 8-byte aligned).  Masked slots touch
 * nothing; duplicated indices repeat the same stores.  No counterpart in the
 * reference, which has no backward. */
int sa_dkv_zero_rows(float* dkv, const int32_t* idx, int64_t b, int64_t m, int64_t topk,
                     int64_t kv_len, const int64_t idx_strides[3], const int64_t dkv_strides[3],
                     void* stream);
int sa_dkv_cast_rows(const float* dkv, void* out, const int32_t* idx, int64_t b, int64_t m,
                     int64_t topk, int64_t kv_len, const int64_t idx_strides[3],
                     const int64_t dkv_strides[3], const int64_t out_strides[3], void* stream);

/* Top-k index producer (lightning indexer): the step that feeds topk_idxs.
 * The reference takes topk_idxs as an input and has none (track-01/
 * requirements.md:1-5); this follows the published DeepSeek-V3.2 indexer:
 *   score[b,t,s] = sum_j weights[b,t,j] * ReLU(q_idx[b,t,j,:] . k_idx[b,s,:])
 * over keys s < lengths[b,t] (a causal or cache limit), fp32 accumulation of
 * bf16 products.  topk_idxs[b,t,:] (int32, contiguous rows) receives the topk
 * keys of largest score in ascending index order, ties at the threshold to
 * the lower index, then -1 where fewer keys are valid: the layout sa_fwd
 * takes.  q_idx [b, m, 64, 128] bf16, k_idx [b, kv_len, 128] bf16, weights
 * [b, m, 64] fp32, lengths [b, m] int32; element strides, last dims
 * contiguous, q / k rows 16-byte aligned.  The workspace holds the fp32 scores
 * (sa_indexer_workspace_bytes); after the call it contains them, row b*m + t. */
size_t sa_indexer_workspace_bytes(int64_t b, int64_t m, int64_t kv_len);
int sa_indexer_topk(const void* q_idx, const void* k_idx, const float* weights,
                    const int32_t* lengths, int32_t* topk_idxs, int64_t b, int64_t m,
                    int64_t n_heads, int64_t head_dim, int64_t kv_len, int64_t topk,
                    const int64_t q_strides[4], const int64_t k_strides[3],
                    const int64_t w_strides[3], const int64_t len_strides[2],
                    const int64_t out_strides[3], void* workspace, size_t workspace_bytes,
                    void* stream);

/* Quantises a bf16 cache [b, kv_len, 512] to the layout sa_fwd_fp8 reads.  Per
 * row: amax = max |x|, kv8 = e4m3_rn_satfinite(x * (448 / amax)),
 * kv_scale = amax / 448; an all-zero row gives zeros and scale 0.  Strides are
 * in elements of each tensor.  Stream-ordered and allocation-free.  No
 * counterpart in the reference. */
int sa_quantize_kv_fp8(const void* kv, void* kv8, float* kv_scale, int64_t b, int64_t kv_len,
                       int64_t d, const int64_t kv_strides[3], const int64_t kv8_strides[3],
                       const int64_t kv_scale_strides[2], void* stream);

/* Debug/health query, synchronous: copies into *flags the error word that the
 * pipelined kernels (SA_VARIANT_TCGEN05, SA_VARIANT_WS; the latter reported
 * as 100 + code, sa_fwd_fp8 as 200 + code, the tensor-core scorer of
 * sa_indexer_topk as 300 + code, SA_VARIANT_WT as 400 + code) set on the current device when one of their
 * bounded pipeline waits gave up (0 = never).  Intended for tests and health checks,
 * not the hot path.  No counterpart in the reference. */
int sa_device_status(int* flags);

/* Debug/health query, synchronous: *count = the number of gathered slots, on
 * the current device and since the last reset, whose index was neither -1 nor
 * inside [0, kv_len).  Such slots are masked like -1 (the output never reads
 * out of bounds); this counter lets a caller detect a faulty index producer.
 * reset != 0 zeroes the counter after reading it.  Counts only kernels that
 * have completed.  The reference masks only -1 (track-01/submission.py:313-322)
 * and leaves other indices undefined. */
int sa_index_faults(uint64_t* count, int reset);

/* Zeroes the error words that sa_device_status reads, on the current device
 * (synchronous).  A caller that saw a nonzero status and dealt with it calls
 * this before its next health check.  No counterpart in the reference. */
int sa_device_status_reset(void);

/* Process-wide options for tests and comparisons; the defaults are what the
 * library is tuned for and a caller never needs to change them.
 *   SA_OPT_ROW_SCHEDULE  1 (default): prefill shapes run whole rows (row
 *                        schedule); 0: contiguous unit ranges for every shape.
 *   SA_OPT_INDEXER_TC    1 (default): sa_indexer_topk scores on tcgen05;
 *                        0: the warp-MMA scorer.
 *   SA_OPT_SPIN_LIMIT    polls before a pipeline wait of the sa_fwd and
 *                        sa_fwd_fp8 kernels gives up (0 = the default, 2^22).
 *   SA_OPT_TEST_STALL    1: the next launches of those kernels withhold one
 *                        arrival on the first ring slot, so a consumer wait
 *                        runs out (with a small SA_OPT_SPIN_LIMIT, quickly);
 *                        the kernel then records its error code, issues no
 *                        more copies, waits for those in flight and returns.
 *                        For testing the failure path; 0 (default) = off.
 *   SA_OPT_KV_POLICY     L2 policy of the KV row gathers of sa_fwd and
 *                        sa_fwd_fp8: -1 (default) by the call's reuse
 *                        (evict_first when m * topk < kv_len, else
 *                        evict_last), 0 evict_first, 1 evict_normal,
 *                        2 evict_last.
 *   SA_OPT_GATHER_ONLY   diagnostic: 1 makes the default sa_fwd kernel
 *                        gather its rows and discard them, writing no
 *                        output (the gather's share of the kernel's time);
 *                        0 (default) = off.
 *   SA_OPT_HEAD_GROUPS   h > 16 on the default sa_fwd kernel: 1 (default)
 *                        runs all groups of 16 heads in one launch, the
 *                        groups' CTAs side by side over the same rows, so
 *                        each KV row is read from HBM about once; 0 runs
 *                        the groups one after another, each gathering the
 *                        rows again.
 * Options are read when a call is made; returns SA_ERR_INVALID_ARG for an
 * unknown option or value.  No counterpart in the reference. */
#define SA_OPT_ROW_SCHEDULE 1
#define SA_OPT_INDEXER_TC 2
#define SA_OPT_SPIN_LIMIT 3
#define SA_OPT_TEST_STALL 4
#define SA_OPT_KV_POLICY 5
#define SA_OPT_GATHER_ONLY 6
#define SA_OPT_HEAD_GROUPS 7
int sa_set_option(int option, int64_t value);
int64_t sa_get_option(int option);

/* Diagnostic: the random-row gather of the forward kernels on its own, with
 * no math, to measure how fast the GPU serves scattered KV rows.  Copies
 * rows[0..n_rows) of src (row r at src + rows[r] * row_stride bytes,
 * row_bytes each: a power of two, 16..32768) into shared memory or registers
 * and discards them.  method 0 = 16-byte cp.async (the forward kernels'
 * form), 1 = one 1-D bulk copy (1-D TMA, one CTA) per row, 2 = 16-byte
 * ld.global.nc into registers; `ctas` CTAs of 256 threads; `depth` = ring
 * slots of 32 KiB (2..6, methods 0 and 1).  sink: >= ctas words (a checksum
 * keeps the loads live); *err becomes nonzero if a bounded wait gave up.
 * Stream-ordered.  No counterpart in the reference. */
int sa_probe_gather(const void* src, int64_t row_stride, const int32_t* rows, int64_t n_rows,
                    int64_t row_bytes, int method, int ctas, int depth, uint32_t* sink, int* err,
                    void* stream);

/* Last cudaError_t observed by this thread inside the library (0 if none). */
int sa_last_cuda_error(void);

/*
 * Bytes of device workspace sa_fwd needs for this problem on `device`
 * (a CUDA device ordinal).  Depends only on (b*m, topk) and the device's SM
 * count.  Replaces nothing in the reference: the reference kernel keeps all
 * state in registers (track-01/submission.py:1006-1021); the persistent
 * split kernels here spill per-CTA partial results for query rows that span
 * two CTAs, and (prefill shapes) one int per row for the row schedule.  The
 * workspace must be zero-filled before its first use; every call leaves the
 * counters it relies on zero again (one per CTA, at the start of the
 * workspace), so one memset at allocation suffices.  A workspace sized by an
 * older formula, without the per-row ints, still works (contiguous unit
 * ranges).  Returns 0 on error (e.g. bad device).
 */
size_t sa_workspace_bytes(int64_t b, int64_t m, int64_t topk, int device);

/*
 * Forward pass.  Replaces track-01/submission.py:975-1021 (the `sparse_attn`
 * wrapper and its kernel launch) — the caller has already allocated `o`
 * (submission.py:1000) and made the last dimension contiguous
 * (submission.py:995-998).
 *
 *   q     [b, m, h, d]   bf16, strides q_strides (elements), q_strides[3] == 1
 *   kv    [b, kv_len, d] bf16, strides kv_strides,           kv_strides[2] == 1
 *   sink  [h]            fp32, contiguous
 *   idx   [b, m, topk]   int32, strides idx_strides (any, elements)
 *   o     [b, m, h, d]   bf16, strides o_strides,            o_strides[3] == 1
 *   h a multiple of 16, d == 512; every row start 16-byte aligned (row
 *   strides multiples of 8 elements, base pointers 16-byte aligned).  The
 *   kernels run 16 heads; h = 16k runs as k groups of 16 heads, one after the
 *   other on `stream`, each gathering the rows again (the reference pads its
 *   head tile to max(16, next_pow2(h)), submission.py:1004; pad h up to a
 *   multiple of 16 with zero heads).
 *   workspace: device memory of at least sa_workspace_bytes(b, m, topk, dev)
 *   bytes, 256-byte aligned, zero-filled before its first use (see
 *   sa_workspace_bytes); every call leaves it zero-filled.
 */
int sa_fwd(const void* q, const void* kv, const float* sink, const int32_t* idx, void* o,
           int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len, int64_t topk,
           const int64_t q_strides[4], const int64_t kv_strides[3],
           const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
           void* workspace, size_t workspace_bytes, void* stream);

/*
 * sa_fwd with an explicit kernel variant (SA_VARIANT_*) and grid size
 * (`grid_ctas` <= 0 = one CTA per SM).  For benchmarking and tests; no
 * counterpart in the reference beyond its per-backend kernel choice at
 * track-01/submission.py:1003-1271.
 */
int sa_fwd_ex(const void* q, const void* kv, const float* sink, const int32_t* idx, void* o,
              int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len, int64_t topk,
              const int64_t q_strides[4], const int64_t kv_strides[3],
              const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
              void* workspace, size_t workspace_bytes, void* stream, int variant,
              int grid_ctas);

/* Largest persistent grid sa_fwd_noalloc serves from its built-in scratch. */
#define SA_NOALLOC_MAX_CTAS 160

/*
 * sa_fwd for callers that cannot allocate device memory (a framework that owns
 * every allocation, a pre-reserved serving loop, code that must not enter the
 * allocator).  No counterpart in the reference.  Same arguments as sa_fwd
 * without the workspace; `grid_ctas` <= 0 picks min(SM count, 160).
 *   - The scratch is one static device array of ~10.5 MB (partials of
 *     SA_NOALLOC_MAX_CTAS CTAs) that each GPU loading the library keeps until
 *     the process exits.  grid_ctas > SA_NOALLOC_MAX_CTAS returns
 *     SA_ERR_WORKSPACE.  Allocates nothing, ever.
 *   - The first call on a device looks up the array's device address (once,
 *     with that device current); make that first call before any stream
 *     capture.
 *   - All calls on a device share the array: calls that may overlap on the
 *     GPU race, so order them (one stream, or events between streams).
 */
int sa_fwd_noalloc(const void* q, const void* kv, const float* sink, const int32_t* idx, void* o,
                   int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len, int64_t topk,
                   const int64_t q_strides[4], const int64_t kv_strides[3],
                   const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
                   void* stream, int grid_ctas);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_ATTN_H_ */
