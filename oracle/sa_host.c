/* sa_host.c — CPU restatement of the sparse_attn reference, as a C entry.
 *
 * TEST INFRASTRUCTURE ONLY.  This builds into its own library
 * (oracle/_build/libsa_host.so), which the product library never links or
 * loads.  Its callers are the tests, which use it as a second oracle beside
 * the torch restatement in sparse_attn_oracle.py, and bench.py's CPU legs,
 * which time it as the reference's algorithm on the host cores.
 *
 * Per query row (b, m) and head h, in fp32 (bf16 inputs widened exactly):
 *   gather the top-k KV rows                        reference.py:27-30
 *   s_t = scale * <q[b,m,h,:], kv[b,idx_t,:]>       reference.py:32
 *   a slot whose index is -1 scores -inf            submission.py:313-322
 *   softmax over the topk scores plus the sink      reference.py:34-38
 *   logit, with the sink column dropped afterwards
 *   o = sum_t p_t * kv[b,idx_t,:], rounded to bf16  reference.py:39-40
 *   (round to nearest even)
 * All paths under track-01/ of the reference project.
 *
 * Two rules go beyond the reference, and the CUDA kernels follow them too:
 *   - any index outside [0, kv_len) is masked like -1;
 *   - a row with no valid slot gives o = 0, since the sink takes all the mass.
 * The softmax is taken in the reference's order: a max over all topk+1 logits,
 * then exp(x - max), the sum, and finally the division.  The fp32 summation
 * order differs from torch's einsum, so results agree with the torch oracle
 * to within one bf16 ulp, not bit for bit.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/sparse_attn_host.h"

static inline float bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))  /* NaN: keep it quiet */
    return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);  /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

int sa_host_version(void) { return 1; }

int sa_fwd_host(const void* q_, const void* kv_, const float* sink, const int32_t* idx,
                void* o_, int64_t b, int64_t m, int64_t h, int64_t d, int64_t kv_len,
                int64_t topk, const int64_t q_strides[4], const int64_t kv_strides[3],
                const int64_t idx_strides[3], const int64_t o_strides[4], float scale,
                int num_threads) {
  const uint16_t* q = (const uint16_t*)q_;
  const uint16_t* kv = (const uint16_t*)kv_;
  uint16_t* o = (uint16_t*)o_;
  if (b < 0 || m < 0 || h <= 0 || d <= 0 || kv_len < 0 || topk < 0) return SA_HOST_ERR_INVALID_ARG;
  if (b == 0 || m == 0) return SA_HOST_OK;
  if (!q || !kv || !sink || !idx || !o || !q_strides || !kv_strides || !idx_strides || !o_strides)
    return SA_HOST_ERR_INVALID_ARG;
  const int64_t rows = b * m;
  int rc = SA_HOST_OK;
#pragma omp parallel num_threads(num_threads > 0 ? num_threads : omp_get_max_threads())
  {
    float* qf = (float*)malloc(sizeof(float) * (size_t)d);
    float* acc = (float*)malloc(sizeof(float) * (size_t)d);
    float* s = (float*)malloc(sizeof(float) * (size_t)(topk > 0 ? topk : 1));
    const uint16_t** rowp = (const uint16_t**)malloc(sizeof(void*) * (size_t)(topk > 0 ? topk : 1));
    if (!qf || !acc || !s || !rowp) {
#pragma omp atomic write
      rc = SA_HOST_ERR_ALLOC;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t r = 0; r < rows; ++r) {
        const int64_t bi = r / m, mi = r - bi * m;
        const int32_t* ir = idx + bi * idx_strides[0] + mi * idx_strides[1];
        for (int64_t t = 0; t < topk; ++t) {
          const int64_t id = ir[t * idx_strides[2]];
          rowp[t] = (id >= 0 && id < kv_len) ? kv + bi * kv_strides[0] + id * kv_strides[1] : NULL;
        }
        for (int64_t hh = 0; hh < h; ++hh) {
          const uint16_t* qr = q + bi * q_strides[0] + mi * q_strides[1] + hh * q_strides[2];
          for (int64_t c = 0; c < d; ++c) qf[c] = bf16_to_f32(qr[c * q_strides[3]]);
          const float sk = sink[hh];
          float mx = sk;
          for (int64_t t = 0; t < topk; ++t) {
            if (!rowp[t]) {
              s[t] = -INFINITY;
              continue;
            }
            float dot = 0.f;
            for (int64_t c = 0; c < d; ++c) dot += qf[c] * bf16_to_f32(rowp[t][c * kv_strides[2]]);
            s[t] = dot * scale;
            if (s[t] > mx) mx = s[t];
          }
          float sum = expf(sk - mx);
          for (int64_t t = 0; t < topk; ++t) {
            s[t] = rowp[t] ? expf(s[t] - mx) : 0.f;
            sum += s[t];
          }
          for (int64_t c = 0; c < d; ++c) acc[c] = 0.f;
          for (int64_t t = 0; t < topk; ++t) {
            if (!rowp[t]) continue;
            const float p = s[t] / sum;
            for (int64_t c = 0; c < d; ++c) acc[c] += p * bf16_to_f32(rowp[t][c * kv_strides[2]]);
          }
          uint16_t* orow = o + bi * o_strides[0] + mi * o_strides[1] + hh * o_strides[2];
          for (int64_t c = 0; c < d; ++c) orow[c * o_strides[3]] = f32_to_bf16(acc[c]);
        }
      }
    }
    free(qf);
    free(acc);
    free(s);
    free(rowp);
  }
  return rc;
}
