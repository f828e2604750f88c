/* hc_sinkhorn.h — C ABI of hc_split_sinkhorn (track-02 of the reference
 * project), built into libsparse_attn.so.
 *
 * Replaces track-02/submission.py:316-380 (the Triton wrapper and kernel);
 * the math is track-02/reference/reference.py:11-51.
 */
#ifndef HC_SINKHORN_H
#define HC_SINKHORN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HCS_OK 0
#define HCS_ERR_INVALID_ARG (-1)
#define HCS_ERR_CUDA (-3)
#define HCS_ERR_UNSUPPORTED (-4)

/* Per token r < n (device pointers, fp32):
 *   mixes[r * mix_stride + 0 .. 23] -> pre[r][4], post[r][4], comb[r][4][4]
 * hc_scale [3], hc_base [24].  Only hc_mult == 4 is supported: the
 * reference's own kernel asserts it (track-02/submission.py:341).
 * pre/post/comb are contiguous and 16-byte aligned.  Stream-ordered and
 * allocation-free; returns HCS_* codes. */
int hcs_split_sinkhorn(const float* mixes, const float* hc_scale, const float* hc_base,
                       float* pre, float* post, float* comb, int64_t n, int64_t mix_stride,
                       int hc_mult, int sinkhorn_iters, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HC_SINKHORN_H */
