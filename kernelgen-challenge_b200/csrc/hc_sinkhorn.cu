// hc_sinkhorn.cu — hc_split_sinkhorn (track-02 of the reference project) for
// sm_100a: per token, split the 24 mixing logits into the pre / post gates
// and a 4x4 matrix projected towards a doubly stochastic one by Sinkhorn
// iterations.
//
// Math, in fp32, as track-02/reference/reference.py:30-51:
//   pre  = sigmoid(mixes[0:4]  * hc_scale[0] + hc_base[0:4]) + eps
//   post = 2 * sigmoid(mixes[4:8] * hc_scale[1] + hc_base[4:8])
//   comb = softmax_rows(mixes[8:24] * hc_scale[2] + hc_base[8:24]) + eps
//   comb = comb / (column sums + eps)
//   (iters - 1) times: comb = comb / (row sums + eps); comb = comb / (column sums + eps)
// The reference divides each element (torch fp32 division); here each row or
// column sum is inverted once (IEEE round-to-nearest reciprocal) and the four
// elements multiplied by it: a quarter of the divisions, within one extra
// rounding per normalisation (the reference's tolerance is atol 1e-5,
// rtol 1e-4; measured against the per-element-division oracle: < 3e-7
// absolute, 1.5e-6 relative, on the 1k-1-64 prefill shape).
//
// Layout: one thread per token holds its 16 matrix entries in registers.  A
// token's 24 inputs are six 16-byte loads (rows are 96 bytes, so a warp's
// loads cover 3 KiB contiguously), and its 24 outputs are six 16-byte stores.
// The work is ~1.3k fp32 operations per 192 bytes moved, so large inputs run
// at the FP32 rate and small ones (decode: 1-64 tokens) at launch latency.
#include <cuda_runtime.h>
#include <stdint.h>

#include "hc_sinkhorn.h"

namespace hcs {

constexpr int HC = 4;
constexpr int MIX = (2 + HC) * HC;  // 24
constexpr int kThreads = 128;

struct Params {
  const float* mixes;
  const float* scale;
  const float* base;
  float* pre;
  float* post;
  float* comb;
  int64_t n;
  int64_t mix_stride;  // elements between tokens (last dim contiguous)
  int iters;
  float eps;
};

// 1 / y by the correctly rounded reciprocal: the same value as the division
__device__ __forceinline__ float sigmoidf_ref(float x) { return __frcp_rn(1.f + expf(-x)); }

__global__ void __launch_bounds__(kThreads) hc_split_sinkhorn_kernel(const Params p) {
  const int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (r >= p.n) return;
  const float* src = p.mixes + r * p.mix_stride;
  float x[MIX];
  if ((p.mix_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(p.mixes) & 15u) == 0) {
#pragma unroll
    for (int k = 0; k < MIX / 4; ++k) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src) + k);
      x[4 * k] = v.x;
      x[4 * k + 1] = v.y;
      x[4 * k + 2] = v.z;
      x[4 * k + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < MIX; ++k) x[k] = __ldg(src + k);
  }
  const float s0 = __ldg(p.scale), s1 = __ldg(p.scale + 1), s2 = __ldg(p.scale + 2);
  float pre[HC], post[HC], c[HC][HC];
#pragma unroll
  for (int j = 0; j < HC; ++j) {
    pre[j] = sigmoidf_ref(x[j] * s0 + __ldg(p.base + j)) + p.eps;
    post[j] = 2.f * sigmoidf_ref(x[HC + j] * s1 + __ldg(p.base + HC + j));
  }
  // softmax over each row of the 4x4 logits, then + eps
#pragma unroll
  for (int i = 0; i < HC; ++i) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      c[i][j] = x[2 * HC + HC * i + j] * s2 + __ldg(p.base + 2 * HC + HC * i + j);
      mx = fmaxf(mx, c[i][j]);
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      c[i][j] = expf(c[i][j] - mx);
      sum += c[i][j];
    }
    const float r = __frcp_rn(sum);
#pragma unroll
    for (int j = 0; j < HC; ++j) c[i][j] = c[i][j] * r + p.eps;
  }
  auto col_norm = [&]() {
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      const float r = __frcp_rn(((c[0][j] + c[1][j]) + c[2][j]) + c[3][j] + p.eps);
#pragma unroll
      for (int i = 0; i < HC; ++i) c[i][j] = c[i][j] * r;
    }
  };
  auto row_norm = [&]() {
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      const float r = __frcp_rn(((c[i][0] + c[i][1]) + c[i][2]) + c[i][3] + p.eps);
#pragma unroll
      for (int j = 0; j < HC; ++j) c[i][j] = c[i][j] * r;
    }
  };
  col_norm();
  for (int it = 1; it < p.iters; ++it) {
    row_norm();
    col_norm();
  }
  reinterpret_cast<float4*>(p.pre)[r] = make_float4(pre[0], pre[1], pre[2], pre[3]);
  reinterpret_cast<float4*>(p.post)[r] = make_float4(post[0], post[1], post[2], post[3]);
  float4* cd = reinterpret_cast<float4*>(p.comb) + 4 * r;
#pragma unroll
  for (int i = 0; i < HC; ++i) cd[i] = make_float4(c[i][0], c[i][1], c[i][2], c[i][3]);
}

}  // namespace hcs

extern "C" int hcs_split_sinkhorn(const float* mixes, const float* hc_scale, const float* hc_base,
                                  float* pre, float* post, float* comb, int64_t n,
                                  int64_t mix_stride, int hc_mult, int sinkhorn_iters, float eps,
                                  void* stream) {
  if (n < 0 || sinkhorn_iters < 1) return HCS_ERR_INVALID_ARG;
  if (hc_mult != hcs::HC) return HCS_ERR_UNSUPPORTED;
  if (n == 0) return HCS_OK;
  if (!mixes || !hc_scale || !hc_base || !pre || !post || !comb) return HCS_ERR_INVALID_ARG;
  if (mix_stride < hcs::MIX) return HCS_ERR_INVALID_ARG;
  for (const void* o : {(const void*)pre, (const void*)post, (const void*)comb})
    if ((reinterpret_cast<uintptr_t>(o) & 15u) != 0) return HCS_ERR_INVALID_ARG;
  hcs::Params p{mixes, hc_scale, hc_base, pre, post, comb, n, mix_stride, sinkhorn_iters, eps};
  const int64_t blocks = (n + hcs::kThreads - 1) / hcs::kThreads;
  if (blocks > INT32_MAX) return HCS_ERR_INVALID_ARG;
  hcs::hc_split_sinkhorn_kernel<<<(unsigned)blocks, hcs::kThreads, 0,
                                  static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCS_OK : HCS_ERR_CUDA;
}
