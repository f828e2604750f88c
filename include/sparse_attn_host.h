/* sparse_attn_host.h — the CPU reference entry of sparse_attn.
 *
 * A plain C restatement of the reference algorithm (track-01/reference/
 * reference.py:10-40, plus the -1 masking of track-01/submission.py:313-322),
 * exported with the arguments of sa_fwd minus the workspace and the stream.
 * It replaces calling reference.py itself from a host that has no Python.
 * It lives in its own library (oracle/_build/libsa_host.so), which is a test
 * and baseline tool: libsparse_attn.so never calls it and has no CPU path.
 */
#ifndef SPARSE_ATTN_HOST_H
#define SPARSE_ATTN_HOST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SA_HOST_OK 0
#define SA_HOST_ERR_INVALID_ARG (-1)
#define SA_HOST_ERR_ALLOC (-5)

/* Version of the host entry (1). */
int sa_host_version(void);

/* o[b,m,h,:] = softmax-weighted sum of the gathered kv rows, computed in fp32
 * on the host and rounded to bf16.  All tensors are host memory.  Strides are
 * in elements.  q, kv and o hold bf16 bit patterns, sink is fp32 [h] and idx is
 * int32.  num_threads <= 0 uses every OpenMP thread.  Out-of-range indices are
 * masked like -1, and a row with no valid slot gives o = 0.
 * Replaces: track-01/reference/reference.py:10 (same arguments and meaning). */
int sa_fwd_host(const void* q, const void* kv, const float* sink, const int32_t* idx, void* o,
                int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len, int64_t topk,
                const int64_t q_strides[4], const int64_t kv_strides[3],
                const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
                int num_threads);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_ATTN_HOST_H */
